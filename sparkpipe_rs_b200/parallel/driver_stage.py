"""Pipeline stages behind the model-driver ABI v6.

Each stage of the pipeline is an instance of a v6 stage driver (a shared library
exporting ``SparkModelDriverGetInterface``), loaded and validated by the C++ loader
(``core().driver_v6``). The stub CPU stage driver (``csrc/drivers/cpu_stage_driver.c``)
does no math itself: the node gives it a *stage host* as its node context, and the
driver runs every frame through the host, which computes the stage's layers of the
CPU MLA-MoE model from the frame's buffers. So the GPU-free plumbing run goes
through the same seam as a compiled stage driver: load -> validate -> create ->
admit -> submit -> completion.

Frame contract between this node and the stub driver (one sequence per frame):

=====  ========================================================================
slot   buffer
=====  ========================================================================
0      input: token ids (int32 [T]) on the first stage, hidden state (fp32 [T, H])
       on the others
1      positions (int32 [T])
2      cache rows the new tokens are written to (int32 [T])
3      decode only: cache rows of the whole context (int32 [ctx])
4      output: hidden state (fp32 [T, H]) on a stage that is not the last; logits
       of the last token (fp32 [V]) on the last stage
7      last stage: the greedy next token (uint32 [1]); the driver returns it in the
       completion
=====  ========================================================================

Programs: 2 = prefill (completes inside submit), 1 = decode (completes on the
driver's worker thread; the node polls for it).

Reference: the stage/driver ABI, crates/spark-abi/vendor/sparkpipe/include/sparkpipe/
spark_model_driver.h:12-255, and how the ring's nodes drive stage programs,
crates/spark-node/src/backend/decode.rs.
"""
from __future__ import annotations

import ctypes
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import torch

from .. import _ext

DRIVER_SOURCE = _ext.CSRC / "drivers" / "cpu_stage_driver.c"
PROGRAM_DECODE, PROGRAM_PREFILL = 1, 2
TARGET = "cpu-test"
READ, WRITE = 1, 2


# ------------------------------------------------------------------ ctypes views of the ABI
class Sp6Buffer(ctypes.Structure):
    _fields_ = [("slot", ctypes.c_uint32), ("flags", ctypes.c_uint32), ("address", ctypes.c_void_p),
                ("bytes", ctypes.c_uint64)]


class Sp6Residency(ctypes.Structure):
    _fields_ = [("word0", ctypes.c_uint64), ("word1", ctypes.c_uint64), ("generation", ctypes.c_uint64),
                ("owner", ctypes.c_uint64)]


class Sp6Frame(ctypes.Structure):
    _fields_ = [("request_id", ctypes.c_uint64), ("sequence_id", ctypes.c_uint64),
                ("sequence_position", ctypes.c_uint64), ("deadline_time_ns", ctypes.c_uint64),
                ("active_slot_count", ctypes.c_uint32), ("new_token_count", ctypes.c_uint32),
                ("priority", ctypes.c_uint32), ("flags", ctypes.c_uint32),
                ("driver_dispatch_slot", ctypes.c_uint32), ("program_id", ctypes.c_uint32),
                ("driver_dispatch_generation", ctypes.c_uint64), ("driver_dispatch_cookie0", ctypes.c_uint64),
                ("driver_dispatch_cookie1", ctypes.c_uint64), ("execution_stream", ctypes.c_void_p),
                ("buffers", ctypes.POINTER(Sp6Buffer)), ("buffer_count", ctypes.c_uint32),
                ("reserved", ctypes.c_uint32), ("scalar", ctypes.c_uint64 * 8), ("residency", Sp6Residency),
                ("user_context", ctypes.c_void_p), ("completion_function", ctypes.c_void_p),
                ("completion_context", ctypes.c_void_p)]


RUN_FN = ctypes.CFUNCTYPE(ctypes.c_int32, ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(Sp6Frame))


class StageHostStruct(ctypes.Structure):
    _fields_ = [("run", RUN_FN), ("user", ctypes.c_void_p)]


def build_stage_driver(out_dir: Path | None = None, break_variant: int = 0) -> Path:
    """Compiles the stub CPU stage driver with the system C compiler (as a driver
    vendor would) and returns the shared library's path."""
    cc = shutil.which("cc") or shutil.which("gcc")
    if cc is None:
        raise RuntimeError("no C compiler to build the stage driver")
    out_dir = Path(out_dir) if out_dir is not None else _ext.EXT_DIR / "drivers"
    out_dir.mkdir(parents=True, exist_ok=True)
    so = out_dir / (f"cpu_stage_driver_break{break_variant}.so" if break_variant else "cpu_stage_driver.so")
    src_mtime = max(DRIVER_SOURCE.stat().st_mtime, (_ext.INCLUDE / "sparkpipe_b200" / "spark_driver_abi_v6.h").stat().st_mtime)
    if so.exists() and so.stat().st_mtime >= src_mtime:
        return so
    tmp = so.with_suffix(f".{os.getpid()}.tmp")
    subprocess.run([cc, "-std=c11", "-O2", "-shared", "-fPIC", "-fvisibility=hidden", f"-I{_ext.INCLUDE}",
                    f"-DSP6_BREAK={break_variant}", str(DRIVER_SOURCE), "-o", str(tmp), "-lpthread"], check=True)
    os.replace(tmp, so)
    return so


def _view(buf: Sp6Buffer, dtype, shape):
    n = int(np.prod(shape))
    ctype = {np.float32: ctypes.c_float, np.int32: ctypes.c_int32, np.uint32: ctypes.c_uint32}[dtype]
    if buf.bytes < n * ctypes.sizeof(ctype):
        raise ValueError(f"buffer slot {buf.slot}: {buf.bytes} bytes, {n} elements needed")
    arr = np.ctypeslib.as_array((ctype * n).from_address(buf.address))
    return torch.from_numpy(arr).view(*shape)


class StageHost:
    """Runs layers [first, last] of a CPU MLA-MoE model for the frames of one stage
    driver instance (the node context handed to the driver at create)."""

    def __init__(self, model, layers, cache, is_first: bool, is_last: bool):
        self.model, self.layers, self.cache = model, list(layers), cache
        self.is_first, self.is_last = is_first, is_last
        self.errors: list[str] = []
        self._fn = RUN_FN(self._run)  # kept alive as long as the host
        self.struct = StageHostStruct(self._fn, None)

    @property
    def address(self) -> int:
        return ctypes.addressof(self.struct)

    def _run(self, _user, program_id, frame_ptr) -> int:
        try:
            self._stage(program_id, frame_ptr.contents)
            return 0
        except Exception as e:  # reported to the driver as a failed frame
            self.errors.append(repr(e))
            return 1

    def _stage(self, program_id: int, f: Sp6Frame):
        from ..models.mla_moe import ForwardBatch

        cfg = self.model.cfg
        bufs = {f.buffers[i].slot: f.buffers[i] for i in range(f.buffer_count)}
        T = int(f.new_token_count)
        pos = _view(bufs[1], np.int32, (T,)).clone()
        rows = _view(bufs[2], np.int32, (T,)).clone()
        if self.is_first:
            ids, hidden = _view(bufs[0], np.int32, (T,)).clone(), None
        else:
            ids, hidden = torch.zeros(T, dtype=torch.int32), _view(bufs[0], np.float32, (T, cfg.hidden_size)).clone()
        if program_id == PROGRAM_PREFILL:
            cu = torch.tensor([0, T], dtype=torch.int32)
            fb = ForwardBatch(mode="prefill", token_ids=ids, positions=pos, slot_mapping=rows, cu_q=cu, cu_k=cu,
                              max_q=T, logits_idx=torch.tensor([T - 1], dtype=torch.int32))
        else:
            ctx = int(f.sequence_position) + 1
            ctx_rows = _view(bufs[3], np.int32, (ctx,)).clone()
            fb = ForwardBatch(mode="decode", token_ids=ids, positions=pos, slot_mapping=rows,
                              block_table=ctx_rows.view(1, ctx), context_lens=torch.tensor([ctx], dtype=torch.int32),
                              logits_idx=torch.tensor([T - 1], dtype=torch.int32))
        out = self.model.forward(fb, self.cache, layers=self.layers, hidden_in=hidden,
                                 return_hidden=not self.is_last, layer_offset=self.layers[0])
        if self.is_last:
            logits = out.reshape(-1)
            _view(bufs[4], np.float32, (cfg.vocab_size,)).copy_(logits)
            tok = bufs[7]
            if tok.bytes < 4:
                raise ValueError("token buffer too small")
            ctypes.c_uint32.from_address(tok.address).value = int(logits.argmax())
        else:
            _view(bufs[4], np.float32, (T, cfg.hidden_size)).copy_(out.float())


class DriverPipeline:
    """Greedy generation through a chain of v6 stage-driver instances, one per
    stage, each hosting its layers of a CPU MLA-MoE model. Every sequence owns
    `max_len` cache rows (block size 1)."""

    def __init__(self, model, stages, driver_path, max_len: int = 128, max_seqs: int = 8):
        from ..core import core

        V6 = core().driver_v6
        self.model, self.cfg, self.max_len = model, model.cfg, max_len
        self.drivers, self.hosts = [], []
        for s, layers in enumerate(stages):
            cache = model.new_cache(max_seqs * max_len, 1, layers=len(layers))
            host = StageHost(model, layers, cache, s == 0, s == len(stages) - 1)
            d = V6.Driver.load(str(driver_path), TARGET)
            d.create(f"stage-{s}", TARGET, host.address)
            self.drivers.append(d)
            self.hosts.append(host)
        self._request = 0

    def close(self):
        for d in self.drivers:
            d.destroy()

    def _step(self, program, seq: int, tokens: np.ndarray, position0: int):
        """Runs one frame through every stage; returns (next token, last-token logits)."""
        cfg, T = self.cfg, len(tokens)
        pos = np.arange(position0, position0 + T, dtype=np.int32)
        rows = (seq * self.max_len + pos).astype(np.int32)
        ctx_rows = (seq * self.max_len + np.arange(position0 + T, dtype=np.int32)).astype(np.int32)
        x = np.ascontiguousarray(tokens, dtype=np.int32)
        logits = np.zeros(cfg.vocab_size, np.float32)
        token = np.zeros(1, np.uint32)
        for s, d in enumerate(self.drivers):
            last = s == len(self.drivers) - 1
            out = logits if last else np.zeros((T, cfg.hidden_size), np.float32)
            bufs = [(0, READ, x.ctypes.data, x.nbytes), (1, READ, pos.ctypes.data, pos.nbytes),
                    (2, READ, rows.ctypes.data, rows.nbytes), (4, WRITE, out.ctypes.data, out.nbytes)]
            if program == PROGRAM_DECODE:
                bufs.append((3, READ, ctx_rows.ctypes.data, ctx_rows.nbytes))
            if last:
                bufs.append((7, WRITE, token.ctypes.data, token.nbytes))
            self._request += 1
            dec = d.admit(program, request_id=self._request, sequence_id=seq, position=position0 + T - 1,
                          new_tokens=T)
            if not dec["accepted"]:
                raise RuntimeError(f"stage {s} refused the frame: reason {dec['rejection_reason']}")
            st = d.submit(program, self._request, sequence_id=seq, position=position0 + T - 1, new_tokens=T,
                          buffers=bufs, dispatch=dec)
            if st != 0:
                raise RuntimeError(f"stage {s} submit failed with status {st}")
            done = []
            while not done:  # decode completes on the driver's thread; prefill inside submit
                done = d.poll(1, 2000)
                if not done and program == PROGRAM_PREFILL:
                    raise RuntimeError("prefill did not complete inside submit")
            c = done[0]
            if c["status"] != 0 or c["request_id"] != self._request:
                raise RuntimeError(f"stage {s} completion {c} ({self.hosts[s].errors})")
            if last:
                assert c["token_ids"] == [int(token[0])], "the completion carries the stage's token"
            x = out
        return int(token[0]), torch.from_numpy(logits.copy())

    def generate(self, seq: int, prompt: list[int], new_tokens: int):
        """Greedy tokens and the logits each was chosen from (prefill, then decode)."""
        tok, lg = self._step(PROGRAM_PREFILL, seq, np.asarray(prompt), 0)
        toks, logits = [tok], [lg]
        pos = len(prompt)
        while len(toks) < new_tokens:
            tok, lg = self._step(PROGRAM_DECODE, seq, np.asarray([toks[-1]]), pos)
            toks.append(tok)
            logits.append(lg)
            pos += 1
        return toks, torch.stack(logits)
