#include "fabric.h"

#include <arpa/inet.h>
#include <netdb.h>
#include <netinet/in.h>
#include <netinet/tcp.h>
#include <poll.h>
#include <sys/socket.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstring>
#include <thread>

namespace spc {
namespace fabric {

void validate_lanes(uint32_t lanes) {
  if (lanes == 0 || lanes > kMaxLanes) fail(Status::InvalidArgument, "memlink: lane count must be 1..64");
}

Partition partition(uint64_t total, uint32_t lanes, uint32_t lane, uint64_t chunk) {
  validate_lanes(lanes);
  if (lane >= lanes) fail(Status::InvalidArgument, "memlink: lane index out of range");
  if (chunk == 0) fail(Status::InvalidArgument, "memlink: zero chunk size");
  const uint64_t chunks = (total + chunk - 1) / chunk;
  const uint64_t c0 = chunks * lane / lanes, c1 = chunks * (lane + 1) / lanes;
  Partition p;
  p.lane = lane;
  p.lanes = lanes;
  p.offset = std::min(total, c0 * chunk);
  p.bytes = std::min(total, c1 * chunk) - p.offset;
  return p;
}

uint32_t neighbor_rank(uint32_t rank, uint32_t ranks, Direction d) {
  if (ranks == 0 || rank >= ranks) fail(Status::InvalidArgument, "memlink: rank out of range");
  return d == Direction::Next ? (rank + 1) % ranks : (rank + ranks - 1) % ranks;
}

std::string host_from_template(const std::string& tmpl, uint32_t rank) {
  if (tmpl.empty()) fail(Status::InvalidArgument, "memlink: empty host template");
  std::string out;
  const std::string key = "{rank}";
  for (size_t i = 0; i < tmpl.size();) {
    if (tmpl.compare(i, key.size(), key) == 0) {
      out += std::to_string(rank);
      i += key.size();
    } else {
      out += tmpl[i++];
    }
  }
  if (out.size() > kMaxHostBytes) fail(Status::InvalidArgument, "memlink: host name longer than 255 bytes");
  return out;
}

Endpoint neighbor_endpoint(uint32_t rank, uint32_t ranks, Direction d, const std::string& host_template,
                           uint16_t base_port, uint32_t lanes) {
  validate_lanes(lanes);
  if (uint32_t(base_port) + lanes > 65536u) fail(Status::InvalidArgument, "memlink: lane ports beyond 65535");
  Endpoint e;
  e.host = host_from_template(host_template, neighbor_rank(rank, ranks, d));
  e.base_port = base_port;
  e.lanes = lanes;
  return e;
}

// ---------------------------------------------------------------- transfer
namespace {
constexpr uint64_t kMagic = 0x4b4e494c4d454d31ull;  // lane header tag
struct Header {
  uint64_t magic, total;
  uint32_t lane, lanes;
  uint64_t offset, bytes;
};
static_assert(sizeof(Header) == 40, "header layout");

using Clock = std::chrono::steady_clock;

bool wait_fd(int fd, short ev, Clock::time_point deadline) {
  while (true) {
    const auto left = std::chrono::duration_cast<std::chrono::milliseconds>(deadline - Clock::now()).count();
    if (left <= 0) return false;
    pollfd p{fd, ev, 0};
    const int r = ::poll(&p, 1, (int)std::min<long long>(left, 1000));
    if (r > 0) return true;
    if (r < 0 && errno != EINTR) return false;
  }
}

bool write_all(int fd, const uint8_t* p, uint64_t n, Clock::time_point deadline) {
  while (n) {
    if (!wait_fd(fd, POLLOUT, deadline)) return false;
    const ssize_t w = ::send(fd, p, (size_t)std::min<uint64_t>(n, kChunkBytes), MSG_NOSIGNAL);
    if (w < 0 && (errno == EINTR || errno == EAGAIN)) continue;
    if (w <= 0) return false;
    p += w;
    n -= (uint64_t)w;
  }
  return true;
}

bool read_all(int fd, uint8_t* p, uint64_t n, Clock::time_point deadline) {
  while (n) {
    if (!wait_fd(fd, POLLIN, deadline)) return false;
    const ssize_t r = ::recv(fd, p, (size_t)std::min<uint64_t>(n, kChunkBytes), 0);
    if (r < 0 && (errno == EINTR || errno == EAGAIN)) continue;
    if (r <= 0) return false;
    p += r;
    n -= (uint64_t)r;
  }
  return true;
}

int connect_to(const std::string& host, uint16_t port, Clock::time_point deadline) {
  addrinfo hints{};
  hints.ai_family = AF_INET;
  hints.ai_socktype = SOCK_STREAM;
  addrinfo* res = nullptr;
  if (::getaddrinfo(host.c_str(), std::to_string(port).c_str(), &hints, &res) != 0 || !res) return -1;
  int fd = -1;
  while (Clock::now() < deadline) {  // the receiver may not listen yet: retry
    fd = ::socket(res->ai_family, res->ai_socktype, 0);
    if (fd >= 0 && ::connect(fd, res->ai_addr, res->ai_addrlen) == 0) break;
    if (fd >= 0) ::close(fd);
    fd = -1;
    std::this_thread::sleep_for(std::chrono::milliseconds(5));
  }
  ::freeaddrinfo(res);
  if (fd >= 0) {
    int one = 1;
    ::setsockopt(fd, IPPROTO_TCP, TCP_NODELAY, &one, sizeof(one));
  }
  return fd;
}
}  // namespace

uint64_t Memlink::send(const std::string& host, uint16_t base_port, uint32_t lanes, const uint8_t* src,
                       uint64_t total, uint32_t timeout_ms) {
  validate_lanes(lanes);
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
  std::atomic<uint64_t> moved{0};
  std::atomic<bool> ok{true};
  std::vector<std::thread> th;
  for (uint32_t l = 0; l < lanes; ++l) {
    th.emplace_back([&, l] {
      const Partition p = partition(total, lanes, l);
      const int fd = connect_to(host, uint16_t(base_port + l), deadline);
      if (fd < 0) {
        ok = false;
        return;
      }
      const Header h{kMagic, total, l, lanes, p.offset, p.bytes};
      if (write_all(fd, reinterpret_cast<const uint8_t*>(&h), sizeof(h), deadline) &&
          write_all(fd, src + p.offset, p.bytes, deadline)) {
        uint8_t ack = 0;  // the receiver acknowledges its lane after the last byte
        if (read_all(fd, &ack, 1, deadline) && ack == 1) moved += p.bytes;
        else ok = false;
      } else {
        ok = false;
      }
      ::close(fd);
    });
  }
  for (auto& t : th) t.join();
  if (!ok) fail(Status::IoError, "memlink: send failed or timed out");
  return moved;
}

uint64_t Memlink::receive(uint16_t base_port, uint32_t lanes, uint8_t* dst, uint64_t capacity, uint32_t timeout_ms) {
  validate_lanes(lanes);
  const auto deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
  std::vector<int> listeners(lanes, -1);
  auto close_all = [&] {
    for (int fd : listeners)
      if (fd >= 0) ::close(fd);
  };
  for (uint32_t l = 0; l < lanes; ++l) {
    const int fd = ::socket(AF_INET, SOCK_STREAM, 0);
    int one = 1;
    ::setsockopt(fd, SOL_SOCKET, SO_REUSEADDR, &one, sizeof(one));
    sockaddr_in a{};
    a.sin_family = AF_INET;
    a.sin_addr.s_addr = htonl(INADDR_ANY);
    a.sin_port = htons(uint16_t(base_port + l));
    listeners[l] = fd;
    if (fd < 0 || ::bind(fd, reinterpret_cast<sockaddr*>(&a), sizeof(a)) != 0 || ::listen(fd, 1) != 0) {
      close_all();
      fail(Status::IoError, "memlink: cannot listen on port " + std::to_string(base_port + l));
    }
  }
  std::atomic<uint64_t> moved{0};
  std::atomic<bool> ok{true};
  std::vector<std::thread> th;
  for (uint32_t l = 0; l < lanes; ++l) {
    th.emplace_back([&, l] {
      if (!wait_fd(listeners[l], POLLIN, deadline)) {
        ok = false;
        return;
      }
      const int fd = ::accept(listeners[l], nullptr, nullptr);
      if (fd < 0) {
        ok = false;
        return;
      }
      Header h{};
      bool good = read_all(fd, reinterpret_cast<uint8_t*>(&h), sizeof(h), deadline) && h.magic == kMagic &&
                  h.lane == l && h.lanes == lanes && h.total <= capacity;
      if (good) {
        const Partition p = partition(h.total, lanes, l);
        good = p.offset == h.offset && p.bytes == h.bytes && read_all(fd, dst + p.offset, p.bytes, deadline);
        if (good) {
          const uint8_t ack = 1;
          good = write_all(fd, &ack, 1, deadline);
          moved += p.bytes;
        }
      }
      if (!good) ok = false;
      ::close(fd);
    });
  }
  for (auto& t : th) t.join();
  close_all();
  if (!ok) fail(Status::IoError, "memlink: receive failed, timed out or saw a bad lane header");
  return moved;
}

// ---------------------------------------------------------------- topology
const char* mode_name(Mode m) {
  switch (m) {
    case Mode::RingDebugSingleRail: return "ring-debug-single-rail";
    case Mode::SingleSwitchSingleRail: return "single-switch-single-rail";
    case Mode::DualSwitchDualRail: return "dual-switch-dual-rail";
    default: return "invalid";
  }
}

TopologyConfig default_topology(Mode mode, uint32_t nodes, uint32_t local, uint32_t mtu) {
  TopologyConfig c;
  c.mode = mode;
  c.nodes = nodes;
  c.local = local;
  c.mtu = mtu;
  switch (mode) {
    case Mode::RingDebugSingleRail: c.flags = kFlagDebugOnly; c.rails = 1; c.switches = 0; c.ports = 2; break;
    case Mode::SingleSwitchSingleRail: c.flags = kFlagSwitched; c.rails = 1; c.switches = 1; c.ports = 1; break;
    case Mode::DualSwitchDualRail:
      c.flags = kFlagSwitched | kFlagFutureOnly; c.rails = 2; c.switches = 2; c.ports = 2; break;
    default: break;
  }
  return c;
}

void validate(const TopologyConfig& c) {
  auto bad = [](const std::string& why) { fail(Status::InvalidArgument, "fabric topology: " + why); };
  if (c.nodes < 2 || c.nodes > kMaxNodes) bad("2..1024 nodes");
  if (c.local >= c.nodes) bad("local node out of range");
  if (c.link_gbps != kLinkGbps) bad("links are 100 Gb/s");
  if (c.mtu < kMinMtu || c.mtu > kMaxMtu) bad("MTU must be 1500..9600 bytes");
  if (c.flags & ~(kFlagDebugOnly | kFlagSwitched | kFlagFutureOnly)) bad("unknown flags");
  switch (c.mode) {
    case Mode::RingDebugSingleRail:
      if (c.rails != 1 || c.switches != 0 || c.ports != 2 || c.flags != kFlagDebugOnly)
        bad("a debug ring has one rail, no switch, two ports per node and the debug-only flag");
      break;
    case Mode::SingleSwitchSingleRail:
      if (c.rails != 1 || c.switches != 1 || c.ports != 1 || c.flags != kFlagSwitched)
        bad("a single-switch fabric has one rail, one switch, one port per node and the switched flag");
      break;
    case Mode::DualSwitchDualRail:
      if (c.rails != 2 || c.switches != 2 || c.ports != 2 || c.flags != (kFlagSwitched | kFlagFutureOnly))
        bad("a dual-rail fabric has two rails, two switches, two ports per node, switched and future-only flags");
      break;
    default: bad("invalid mode");
  }
}

Route resolve_route(const TopologyConfig& c, uint32_t dst) {
  validate(c);
  if (dst >= c.nodes) fail(Status::InvalidArgument, "fabric topology: destination out of range");
  if (dst == c.local) fail(Status::InvalidArgument, "fabric topology: no route to the local node");
  Route r;
  r.mode = c.mode;
  r.src = c.local;
  r.dst = dst;
  if (c.mode == Mode::DualSwitchDualRail)
    fail(Status::Unsupported, "fabric topology: the dual-rail layout is described but not routable yet");
  if (c.mode == Mode::SingleSwitchSingleRail) {
    r.first_hop = kNoNode;  // into the switch
    r.hops = 2;             // node -> switch -> node
    r.switched = true;
    return r;
  }
  // debug ring: the shorter way round, forward on a tie
  const uint32_t fwd = (dst + c.nodes - c.local) % c.nodes, back = c.nodes - fwd;
  if (fwd <= back) {
    r.port = 0;
    r.first_hop = (c.local + 1) % c.nodes;
    r.hops = fwd;
  } else {
    r.port = 1;
    r.first_hop = (c.local + c.nodes - 1) % c.nodes;
    r.hops = back;
  }
  return r;
}

}  // namespace fabric
}  // namespace spc
