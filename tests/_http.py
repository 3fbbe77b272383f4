"""Raw HTTP/1.1 client helpers for the gateway tests (loopback sockets, no libraries)."""
import socket


class Response:
    def __init__(self, status, headers, body, chunks=None):
        self.status = status
        self.headers = headers
        self.body = body
        self.chunks = chunks

    def header(self, name):
        for k, v in self.headers:
            if k.lower() == name.lower():
                return v
        return None


def connect(port, timeout=20.0):
    s = socket.create_connection(("127.0.0.1", port), timeout=timeout)
    return s


def _read_until(sock, buf, token):
    while token not in buf:
        data = sock.recv(65536)
        if not data:
            raise ConnectionError("connection closed mid-response")
        buf += data
    return buf


def read_head(sock, buf=b""):
    buf = _read_until(sock, buf, b"\r\n\r\n")
    head, rest = buf.split(b"\r\n\r\n", 1)
    lines = head.decode().split("\r\n")
    status = int(lines[0].split(" ")[1])
    headers = []
    for line in lines[1:]:
        k, v = line.split(":", 1)
        headers.append((k.strip(), v.strip()))
    return status, headers, rest


def read_chunk(sock, buf):
    """Returns (chunk bytes or None at the terminator, remaining buffer)."""
    buf = _read_until(sock, buf, b"\r\n")
    line, rest = buf.split(b"\r\n", 1)
    n = int(line, 16)
    if n == 0:
        rest = _read_until(sock, rest, b"\r\n")
        return None, rest.split(b"\r\n", 1)[1]
    while len(rest) < n + 2:
        data = sock.recv(65536)
        if not data:
            raise ConnectionError("connection closed mid-chunk")
        rest += data
    return rest[:n], rest[n + 2:]


def read_response(sock, buf=b""):
    status, headers, rest = read_head(sock, buf)
    r = Response(status, headers, b"")
    if (r.header("transfer-encoding") or "").lower() == "chunked":
        chunks = []
        while True:
            c, rest = read_chunk(sock, rest)
            if c is None:
                break
            chunks.append(c)
        r.chunks = chunks
        r.body = b"".join(chunks)
        return r, rest
    n = int(r.header("content-length") or 0)
    while len(rest) < n:
        data = sock.recv(65536)
        if not data:
            raise ConnectionError("connection closed mid-body")
        rest += data
    r.body = rest[:n]
    return r, rest[n:]


def request(port, method, path, body=b"", headers=None):
    sock = connect(port)
    try:
        sock.sendall(build(method, path, body, headers))
        r, _ = read_response(sock)
        return r
    finally:
        sock.close()


def build(method, path, body=b"", headers=None):
    if isinstance(body, str):
        body = body.encode()
    h = {"host": "127.0.0.1"}
    if body or method == "POST":
        h["content-length"] = str(len(body))
        h["content-type"] = "application/json"
    h.update(headers or {})
    head = f"{method} {path} HTTP/1.1\r\n" + "".join(f"{k}: {v}\r\n" for k, v in h.items()) + "\r\n"
    return head.encode() + body
