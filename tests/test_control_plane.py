"""Driver control plane end to end on the host: a C module compiled here, published
to the module library (validated once, reused after), a model description whose
stage chains two operations, a driver generated and compiled from it, loaded by the
orchestrator against the node's target, routed and submitted."""
import hashlib
import json
import shutil
import subprocess
from pathlib import Path

import pytest

from sparkpipe_rs_b200 import _ext

CC = shutil.which("cc") or shutil.which("gcc")
INCLUDE = str(Path(_ext.__file__).resolve().parent / "include")

MODULE_C = r"""
#include <sparkpipe_b200/model_driver.h>
#include <stdlib.h>
#include <string.h>
typedef struct { int add; } state_t;
int32_t addk_init(const char* cfg, void** st) {
  state_t* s = (state_t*)malloc(sizeof(state_t));
  const char* p = strstr(cfg, "\"add\":");
  s->add = p ? atoi(p + 6) : 1;
  *st = s;
  return 0;
}
int32_t addk_exec(void* st, const spb_buffer* in, spb_buffer* out) {
  const state_t* s = (const state_t*)st;
  if (out->bytes < in->bytes) return 2;
  for (uint64_t i = 0; i < in->bytes; ++i) ((unsigned char*)out->data)[i] = ((const unsigned char*)in->data)[i] + s->add;
  out->bytes = in->bytes;
  return 0;
}
void addk_destroy(void* st) { free(st); }
"""


def _cp():
    return _ext.core().control_plane


def test_sha256_known_vectors():
    cp = _cp()
    for msg in (b"", b"abc", b"a" * 1000, bytes(range(256)) * 3):
        assert cp.sha256_hex(msg) == hashlib.sha256(msg).hexdigest()


def _description(tmp, target):
    d = {"schema_version": 1, "model_id": "toy", "model_revision": "r1", "metadata": {"note": "test"},
         "stages": [{"name": "decode", "target": target, "programs": [
             {"name": "step", "program_id": 7, "max_inflight": 2,
              "scheduling": {"max_active_slots": 4, "target_latency_ns": 1000},
              "operations": [
                  {"name": "a", "kind": "dense_mlp", "module_id": "addk", "configuration": {"add": 1}},
                  {"name": "b", "kind": "output_head", "module_id": "addk", "configuration": {"add": 10}}]}]}]}
    p = tmp / "model.json"
    p.write_text(json.dumps(d))
    return p, d


def test_model_description_validation(tmp_path):
    cp = _cp()
    p, d = _description(tmp_path, "host.cpu")
    md = cp.load_model_description(str(p))
    assert md.model_id == "toy" and md.source_sha256 == hashlib.sha256(p.read_bytes()).hexdigest()
    ops = md.stages[0].programs[0].operations
    assert [o.kind for o in ops] == ["dense_mlp", "output_head"] and json.loads(ops[1].configuration_json) == {"add": 10}
    bad = json.loads(json.dumps(d))
    bad["stages"][0]["programs"][0]["operations"][0]["kind"] = "teleport"
    with pytest.raises(Exception):
        cp.parse_model_description(json.dumps(bad))
    bad = json.loads(json.dumps(d))
    bad["stages"][0]["programs"].append(dict(bad["stages"][0]["programs"][0]))
    with pytest.raises(Exception):  # duplicate program
        cp.parse_model_description(json.dumps(bad))


@pytest.mark.skipif(CC is None, reason="needs a C compiler")
def test_publish_compile_orchestrate(tmp_path):
    cp = _cp()
    src = tmp_path / "addk.c"
    src.write_text(MODULE_C)
    obj = tmp_path / "addk.o"
    subprocess.run([CC, "-c", "-fPIC", "-O2", f"-I{INCLUDE}", "-o", str(obj), str(src)], check=True)
    validator = tmp_path / "validate.sh"
    validator.write_text("#!/bin/sh\necho run >> \"$(dirname \"$0\")/validations.log\"\ntest -s \"$1\"\n")
    validator.chmod(0o755)
    lib = tmp_path / "lib"
    kw = dict(library_root=str(lib), module_id="addk", target="host.cpu", link_unit=str(obj), recipe="nonempty",
              init_symbol="addk_init", execute_symbol="addk_exec", destroy_symbol="addk_destroy",
              validator=str(validator))
    r1 = cp.publish_module(**kw)
    r2 = cp.publish_module(**kw)
    assert not r1.validation_reused and r2.validation_reused
    assert (tmp_path / "validations.log").read_text().count("run") == 1
    art = cp.resolve_module(str(lib), "addk", "host.cpu")
    assert art.validated and art.artifact_sha256 == hashlib.sha256(obj.read_bytes()).hexdigest()
    desc, _ = _description(tmp_path, "host.cpu")
    rep = cp.compile_driver(str(desc), "decode", str(lib), str(tmp_path / "out"), CC, INCLUDE)
    assert (rep.program_count, rep.operation_count, rep.link_unit_count) == (1, 2, 1)
    manifest = json.loads(Path(rep.manifest_path).read_text())
    assert manifest["driver_sha256"] == hashlib.sha256(Path(rep.driver_path).read_bytes()).hexdigest()
    orch = cp.Orchestrator()
    node = orch.add_node("n0", "host.cpu")
    drv = orch.attach_driver(node, rep.driver_path)
    route = orch.resolve_route("toy", "r1", "decode", "step")
    assert orch.submit(route, bytes([1, 2, 3]), 16) == bytes([12, 13, 14])  # +1 then +10
    assert orch.snapshot(drv) == (1, 1, 0) and orch.outstanding(drv) == 0
    with pytest.raises(Exception):
        orch.resolve_route("toy", "r2", "decode", "step")
    # a node of another target refuses the driver
    other = orch.add_node("n1", "sm_100a.b200")
    with pytest.raises(Exception):
        orch.attach_driver(other, rep.driver_path)
    # a tampered stored link unit no longer resolves
    Path(art.link_unit_path).write_bytes(b"tampered")
    with pytest.raises(Exception):
        cp.resolve_module(str(lib), "addk", "host.cpu")
