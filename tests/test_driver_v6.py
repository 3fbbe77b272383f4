"""Stage drivers of the reference's model-driver ABI v6, on CPU.

The stub CPU stage driver (csrc/drivers/cpu_stage_driver.c) is compiled with the
system C compiler against include/sparkpipe_b200/spark_driver_abi_v6.h and loaded
through `SparkModelDriverGetInterface` by the C++ loader (csrc/core/driver_v6.cpp).

* layout gate: sizeof / offsetof of the ABI structs agree between a C probe, the
  C++ loader and the natural C layout of the declarations (ctypes)
* fail-closed load: one broken build per rule (cases of the reference's
  crates/spark-sys/tests/driver_load.rs)
* lifecycle: create, admission decisions, submission, completions delivered on the
  driver's thread, counters
* the GPU-free plumbing run (tiny MLA-MoE, 2 layers, hidden 256, ...): a 2-stage
  pipeline whose stages are instances of the stage driver, 4 prompts of 32 uniform
  ids, 16 greedy tokens each, against a plain PyTorch CPU forward
"""
import ctypes
import shutil
import subprocess
from pathlib import Path

import pytest
import torch

from sparkpipe_rs_b200 import _ext
from sparkpipe_rs_b200.core import StatusError, core
from sparkpipe_rs_b200.parallel import driver_stage as ds

V6 = core().driver_v6
ABI_MISMATCH, VALIDATION_FAILED, TARGET_MISMATCH, DRIVER_LOAD, DUPLICATE = 10, 9, 11, 13, 16

pytestmark = pytest.mark.skipif(shutil.which("cc") is None and shutil.which("gcc") is None,
                                reason="needs a C compiler")


@pytest.fixture(scope="module")
def driver_path(tmp_path_factory):
    return ds.build_stage_driver(tmp_path_factory.mktemp("drv"))


# ------------------------------------------------------------------ layout gate
class _Profile(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in ("descriptor_bytes", "profile_flags", "max_inflight",
                                                "max_active_slots", "max_new_tokens", "max_resident_sequences")] + \
               [(n, ctypes.c_uint64) for n in ("max_sequence_tokens", "target_latency_ns", "validated_latency_ns",
                                                "resident_weight_bytes", "resident_kv_bytes", "static_workspace_bytes",
                                                "device_memcpy_ceiling", "host_staging_ceiling")] + \
               [("private_queue_count", ctypes.c_uint32), ("reserved", ctypes.c_uint32)]


class _Completion(ctypes.Structure):
    _fields_ = [("request_id", ctypes.c_uint64), ("sequence_id", ctypes.c_uint64),
                ("sequence_position", ctypes.c_uint64)] + \
               [(n, ctypes.c_uint32) for n in ("program_id", "driver_dispatch_slot", "accepted_token_count",
                                                "completion_flags", "token_count")] + \
               [("token_ids", ctypes.c_uint32 * 8), ("draft_token_count", ctypes.c_uint32),
                ("draft_token_ids", ctypes.c_uint32 * 8), ("status", ctypes.c_int32), ("residency", ds.Sp6Residency)] + \
               [(n, ctypes.c_uint64) for n in ("queue_delay_ns", "service_time_ns", "device_memcpy_bytes",
                                                "host_staging_bytes")]


class _Interface(ctypes.Structure):
    _fields_ = [("abi_version", ctypes.c_uint32), ("interface_bytes", ctypes.c_uint32)] + \
               [(n, ctypes.c_void_p) for n in ("descriptor", "create", "destroy", "admit", "snapshot")]


def _natural_layout():
    return {
        "sizeof(sp6_buffer)": ctypes.sizeof(ds.Sp6Buffer),
        "sizeof(sp6_residency)": ctypes.sizeof(ds.Sp6Residency),
        "sizeof(sp6_completion)": ctypes.sizeof(_Completion),
        "offsetof(sp6_completion,token_ids)": _Completion.token_ids.offset,
        "offsetof(sp6_completion,status)": _Completion.status.offset,
        "offsetof(sp6_completion,residency)": _Completion.residency.offset,
        "sizeof(sp6_frame)": ctypes.sizeof(ds.Sp6Frame),
        "offsetof(sp6_frame,execution_stream)": ds.Sp6Frame.execution_stream.offset,
        "offsetof(sp6_frame,scalar)": ds.Sp6Frame.scalar.offset,
        "offsetof(sp6_frame,completion_function)": ds.Sp6Frame.completion_function.offset,
        "sizeof(sp6_program_profile)": ctypes.sizeof(_Profile),
        "offsetof(sp6_program_profile,private_queue_count)": _Profile.private_queue_count.offset,
        "sizeof(sp6_interface)": ctypes.sizeof(_Interface),
        "offsetof(sp6_interface,snapshot)": _Interface.snapshot.offset,
    }


def test_abi_v6_layout_gate(tmp_path):
    cpp = dict(V6.abi_layout())
    lines = []
    for name in cpp:
        kind, rest = name.split("(", 1)
        rest = rest[:-1]
        expr = f"sizeof({rest})" if kind == "sizeof" else f"offsetof({rest.split(',')[0]}, {rest.split(',')[1]})"
        lines.append(f'  printf("%s %zu\\n", "{name}", (size_t){expr});')
    probe = tmp_path / "probe.c"
    probe.write_text("#include <stdio.h>\n#include <sparkpipe_b200/spark_driver_abi_v6.h>\nint main(void) {\n" +
                     "\n".join(lines) + "\n  return 0;\n}\n")
    cc = shutil.which("cc") or shutil.which("gcc")
    subprocess.run([cc, "-std=c11", f"-I{_ext.INCLUDE}", str(probe), "-o", str(tmp_path / "probe")], check=True)
    out = subprocess.run([str(tmp_path / "probe")], capture_output=True, text=True, check=True).stdout.split("\n")
    c_layout = {ln.split()[0]: int(ln.split()[1]) for ln in out if ln.strip()}
    assert c_layout == cpp
    for name, value in _natural_layout().items():
        assert cpp[name] == value, name


# ------------------------------------------------------------------ load
def test_load_identity_and_programs(driver_path):
    d = V6.Driver.load(str(driver_path), "cpu-test")
    assert (d.model_id, d.model_revision, d.stage_name, d.target) == ("tiny-mla-moe", "r1", "stage", "cpu-test")
    assert len(d.model_description_sha256) == 64 and d.module_instance_count == 1
    progs = {p["name"]: p for p in d.programs()}
    assert progs["decode"]["program_id"] == 1 and progs["decode"]["flags"] & V6.PROGRAM_EXTERNAL_COMPLETION
    assert progs["decode"]["validated_latency_ns"] == 1500000 and progs["prefill"]["program_id"] == 2
    with pytest.raises(StatusError) as e:
        V6.Driver.load(str(driver_path), "gb10-ring")
    assert e.value.code == TARGET_MISMATCH
    with pytest.raises(StatusError) as e:
        V6.Driver.load(str(driver_path.parent / "missing.so"), "")
    assert e.value.code == DRIVER_LOAD


@pytest.mark.parametrize("variant,code", [(1, ABI_MISMATCH), (2, ABI_MISMATCH), (3, DUPLICATE),
                                          (4, VALIDATION_FAILED), (5, ABI_MISMATCH), (6, ABI_MISMATCH),
                                          (7, ABI_MISMATCH), (8, DRIVER_LOAD)])
def test_broken_drivers_are_refused(tmp_path, variant, code):
    so = ds.build_stage_driver(tmp_path, break_variant=variant)
    with pytest.raises(StatusError) as e:
        V6.Driver.load(str(so), "")
    assert e.value.code == code


# ------------------------------------------------------------------ lifecycle
def test_admission_submission_and_completions(driver_path):
    d = V6.Driver.load(str(driver_path), "cpu-test")
    d.create("node-0", "cpu-test")
    try:
        ok = d.admit(1, request_id=7, sequence_id=3, active_slots=2, new_tokens=1)
        assert ok["accepted"] and ok["driver_dispatch_slot"] != 0xffffffff and ok["driver_dispatch_generation"] == 1
        assert d.admit(1, active_slots=65)["rejection_reason"] == 2        # beyond the KV slots
        assert d.admit(2, new_tokens=5000)["rejection_reason"] == 5        # unsupported shape
        # decode: completion arrives later, from the driver's thread
        for r in range(5):
            assert d.submit(1, 100 + r, sequence_id=3, position=10 + r, new_tokens=3, scalars=[40 + r],
                            dispatch=ok if r == 0 else None) == 0
        got = []
        while len(got) < 5:
            got += d.poll(8, 2000)
        assert [c["request_id"] for c in got] == [100, 101, 102, 103, 104]
        assert got[2]["token_ids"] == [42, 43, 44] and got[0]["driver_dispatch_slot"] == ok["driver_dispatch_slot"]
        # prefill: completed inside submit
        assert d.submit(2, 200, new_tokens=2, scalars=[9]) == 0
        assert d.poll(8, 0)[0]["token_ids"] == [9, 10]
        snap = d.snapshot(1)
        assert (snap["submitted_count"], snap["completed_count"]) == (5, 5) and d.wakes >= 1
        assert d.frames_in_flight == 0   # every frame's completion released it
        with pytest.raises(StatusError):
            d.submit(9, 1)               # no such program
    finally:
        d.destroy()
    assert not d.has_instance


# ------------------------------------------------------------------ GPU-free plumbing run
def test_two_stage_pipeline_through_the_driver_abi_matches_cpu_forward(driver_path):
    from sparkpipe_rs_b200.models import oracle
    from sparkpipe_rs_b200.models.config import tiny
    from sparkpipe_rs_b200.models.cpu_model import CpuMLAMoEModel
    from sparkpipe_rs_b200.parallel.pipeline import split_layers

    cfg = tiny()
    model = CpuMLAMoEModel(cfg, seed=0)
    pipe = ds.DriverPipeline(model, split_layers(cfg.num_layers, 2), driver_path, max_len=64, max_seqs=4)
    try:
        g = torch.Generator().manual_seed(0)
        prompts = [torch.randint(0, 1024, (32,), generator=g).tolist() for _ in range(4)]
        for s, p in enumerate(prompts):
            toks, logits = pipe.generate(s, p, 16)
            ref_toks, ref_logits = oracle.greedy_generate(cfg, model.w, torch.tensor(p), 16)
            assert toks == ref_toks.tolist()
            assert (logits - ref_logits).abs().max().item() < 1e-3
        assert all(not h.errors for h in pipe.hosts)
        assert [d.snapshot(1)["completed_count"] for d in pipe.drivers] == [60, 60]   # 4 x 15 decode frames
    finally:
        pipe.close()
