"""Ring node context (C++): built from a rank plan and a model driver compiled from a
model description (module library + driver compiler), it runs prefill / decode work
packets on the driver, forwards them to the next rank first (to a rank daemon over a
socket pair), and on the final stage returns the program's output as a final event.

Behaviour follows crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_ring_node_context_builder.h."""
import json
import shutil
import socket
import subprocess
import time
from pathlib import Path

import pytest

from sparkpipe_rs_b200 import _ext
from sparkpipe_rs_b200.core import core

C = core()
NC, R, WC, RD, CP = C.node_context, C.ring_runtime, C.work_control, C.rank_daemon, C.control_plane
CC = shutil.which("cc") or shutil.which("gcc")
INCLUDE = str(Path(_ext.__file__).resolve().parent / "include")

MODULE_C = r"""
#include <sparkpipe_b200/model_driver.h>
#include <stdlib.h>
#include <string.h>
typedef struct { int words; } st_t;
int32_t head_init(const char* cfg, void** st) {
  st_t* s = (st_t*)malloc(sizeof(st_t));
  const char* p = strstr(cfg, "\"words\":");
  s->words = p ? atoi(p + 8) : 1;
  *st = s;
  return 0;
}
int32_t head_exec(void* st, const spb_buffer* in, spb_buffer* out) {  /* the first N u32 words of the input */
  const st_t* s = (const st_t*)st;
  uint64_t n = (uint64_t)s->words * 4;
  if (n > in->bytes || n > out->bytes) return 2;
  memcpy(out->data, in->data, n);
  out->bytes = n;
  return 0;
}
void head_destroy(void* st) { free(st); }
"""


@pytest.fixture(scope="module")
def driver(tmp_path_factory):
    if CC is None:
        pytest.skip("needs a C compiler")
    tmp = tmp_path_factory.mktemp("nc")
    (tmp / "head.c").write_text(MODULE_C)
    obj = tmp / "head.o"
    subprocess.run([CC, "-c", "-fPIC", "-O2", f"-I{INCLUDE}", "-o", str(obj), str(tmp / "head.c")], check=True)
    val = tmp / "v.sh"
    val.write_text("#!/bin/sh\ntest -s \"$1\"\n")
    val.chmod(0o755)
    CP.publish_module(library_root=str(tmp / "lib"), module_id="head", target="host.cpu", link_unit=str(obj),
                      recipe="nonempty", init_symbol="head_init", execute_symbol="head_exec",
                      destroy_symbol="head_destroy", validator=str(val))
    prog = lambda name, pid, words: {"name": name, "program_id": pid, "max_inflight": 1, "operations": [  # noqa: E731
        {"name": "out", "kind": "output_head", "module_id": "head", "configuration": {"words": words}}]}
    desc = {"schema_version": 1, "model_id": "toy", "model_revision": "r1",
            "stages": [{"name": "s0", "target": "host.cpu", "programs": [prog("prefill", 1, 2), prog("decode", 2, 1)]}]}
    (tmp / "m.json").write_text(json.dumps(desc))
    rep = CP.compile_driver(str(tmp / "m.json"), "s0", str(tmp / "lib"), str(tmp / "out"), CC, INCLUDE)
    return rep.driver_path


def ring_geometry(stages):
    g = R.Geometry()
    g.layer_count = sum(stages)
    g.first_routed_layer = 1
    g.hidden_dimension = 1024
    g.maximum_context_tokens = 8192
    g.dsa_selected_tokens = 2048
    g.max_speculative_rows_per_lane = 1
    g.max_batch_bucket = 256
    g.stage_count = len(stages)
    g.default_stage_layer_counts = list(stages)
    g.tp_geometry = C.tp.Geometry(8, 192, 256, 128)
    g.shape_inputs = C.tp.ModelInputs(sum(stages), 1024, 512, 2048, 576)
    return g


def work_config():
    w = WC.Config()
    w.output_vocab_count = 1000
    return w


def packet(tid, phase=2, seqs=(1,)):
    p = WC.Packet()
    i = WC.Identity()
    i.control_generation, i.transaction_id, i.dispatch_generation = 1, tid, 1
    i.request_generation, i.step_generation, i.step_chunk_count, i.transaction_phase = 1, 1, 1, phase
    p.identity = i
    lanes = []
    for s in seqs:
        lane = WC.Lane()
        lane.request_id = lane.sequence_id = s
        lane.sequence_position, lane.context_token_count, lane.input_token_id = 5, 6, 7
        lanes.append(lane)
    p.lanes = lanes
    p.active_sequence_count = p.execution_row_count = len(seqs)
    p.block_token_count = 64
    if phase == 1:
        p.flags = 0x1
        p.prefill_token_ids = [3, 4, 5]
        p.new_token_count = 3
    return p


def context(driver, plan, target="host.cpu"):
    c = NC.NodeContextConfig()
    c.plan, c.driver_path, c.target, c.work = plan, driver, target, work_config()
    return NC.NodeContext.build(c)


def test_final_stage_returns_final_events(driver):
    (plan,) = R.build_ring(ring_geometry([6]), 1, 16)
    ctx = context(driver, plan)
    r = ctx.decode(packet(1))
    assert r.final_stage and not r.forwarded
    assert r.final_event.token_ids == [0x35574350] and r.final_event.request_id == 1  # packet magic (1 word)
    r = ctx.prefill(packet(2, phase=1))
    assert r.final_event.token_ids == [0x35574350, 16]  # magic, ABI version (2 words)
    assert r.final_event.accepted_token_count == 2 and ctx.submitted == 2
    with pytest.raises(Exception):
        ctx.prefill(packet(3))  # a decode packet
    with pytest.raises(Exception):
        ctx.decode(packet(4, seqs=tuple(range(1, 18))))  # more rows than the rank's 16


def test_forward_then_run_to_next_rank(driver):
    plans = R.build_ring(ring_geometry([4, 4]), 1, 16)
    ctx = context(driver, plans[0])
    a, b = socket.socketpair()
    ctx.adopt_output_socket(a.detach())
    cfg = RD.DaemonConfig()
    cfg.rank, cfg.world = 1, 2
    cfg.work = work_config()
    daemon = RD.RankDaemon(cfg)
    r = ctx.decode(packet(1))
    assert r.forwarded and not r.final_stage and len(r.output) == 4 and ctx.queued_output == 1
    b.setblocking(True)
    for _ in range(200):
        st = int(ctx.pump_output())
        try:
            head = b.recv(65536, socket.MSG_DONTWAIT) if st != 0 else b""
        except BlockingIOError:
            head = b""
        if head:
            b.sendall(daemon.submit(head))
        if st == 0 and ctx.queued_output == 0:
            break
        time.sleep(0.005)
    assert ctx.queued_output == 0 and daemon.ledger.entries == 1
    b.close()


def test_build_refuses_wrong_target(driver):
    (plan,) = R.build_ring(ring_geometry([6]), 1, 16)
    with pytest.raises(Exception):
        context(driver, plan, target="sm_100a.b200")
