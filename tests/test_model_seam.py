"""Model seam on CPU: contract documents (envelope, geometry dialects, the K2-family
typed view, family dispatch, config mapping) and the model-driver loader (a fake
driver built with the system C compiler, fail-closed validation, the C layout gate).

Cases follow crates/spark-model/tests/contracts.rs and
crates/spark-sys/tests/driver_load.rs of the reference."""
import json
import os
import shutil
import subprocess
from pathlib import Path

import pytest

from sparkpipe_rs_b200.core import StatusError, core
from sparkpipe_rs_b200.models.config import k2, v2_lite
from sparkpipe_rs_b200.models.contract import (bundled_contract, config_from_contract, config_from_hf,
                                               k27_view, load_contract)

C = core()
INCLUDE = Path(__file__).resolve().parents[1] / "sparkpipe_rs_b200" / "include"
FIXTURE = Path(__file__).resolve().parent / "fixtures" / "fake_model_driver.c"


# ------------------------------------------------------------------ contracts
def test_envelope_validation():
    D = C.contract.ContractDocument
    d = D.parse('{"schema_version": 2, "model_id": "m", "layer_count": 4}')
    assert d.schema_version == 2 and d.model_id == "m" and d.geometry().layer_count == 4
    for bad in ['{"schema_version": 0, "layer_count": 4}', '{"schema_version": -1, "layer_count": 4}',
                '{"schema_version": "1", "layer_count": 4}', '{"model_id": "", "layer_count": 4}',
                '{"model_id": 7, "layer_count": 4}', '{"note": "no geometry"}']:
        with pytest.raises(StatusError) as e:
            D.parse(bad)
        assert e.value.code == 6  # schema_error
    with pytest.raises(StatusError) as e:
        D.parse("{not json")
    assert e.value.code == 5  # parse_error


def test_geometry_dialects():
    D = C.contract.ContractDocument
    flat = D.parse('{"hidden_dimension": 6144, "layer_count": 78, "vocab_size": 154880, "first_routed_layer": 3}')
    g = flat.geometry()
    assert (g.hidden_dimension, g.layer_count, g.vocabulary_size, g.first_routed_layer) == (6144, 78, 154880, 3)
    assert g.total_parameters == -1
    sect = D.parse('{"model": {"hidden_dimension": 7168, "layer_count": 61, "vocabulary_size": 163840}}')
    assert sect.geometry().layer_count == 61 and sect.geometry().vocabulary_size == 163840
    assert sect.section_json("model") is not None and sect.section_json("moe") is None


def test_k27_view_and_config():
    doc = load_contract(bundled_contract("kimi_k2_shape"))
    assert doc.family() == "k27"
    v = k27_view(doc)
    assert v["mla"]["kv_lora_rank"] == 512 and v["moe"]["routed_expert_count"] == 384
    assert v["sources"]["license"] == "n/a (no checkpoint)" and v["speculation"]["note"] == ""
    cfg = config_from_contract(bundled_contract("kimi_k2_shape"))
    ref = k2()
    for f in ref.__dataclass_fields__:
        if f != "name":
            assert getattr(cfg, f) == getattr(ref, f), f
    assert cfg.param_count() == v["model"]["total_parameters"]


def test_k27_view_rejects_bad_sections():
    base = json.loads(bundled_contract("kimi_k2_shape").read_text())
    for mutate, needle in [
        (lambda d: d.pop("moe"), "missing required section 'moe'"),
        (lambda d: d["mla"].pop("kv_lora_rank"), "missing field 'kv_lora_rank'"),
        (lambda d: d["model"].__setitem__("layer_count", -61), "'layer_count' has the wrong type"),
        (lambda d: d["model"].__setitem__("tie_word_embeddings", 0), "'tie_word_embeddings' has the wrong type"),
        (lambda d: d["quantization"].__setitem__("quantized_components", [1]), "'quantized_components'"),
        (lambda d: d.__setitem__("tokens", []), "section 'tokens' must be an object"),
    ]:
        d = json.loads(json.dumps(base))
        mutate(d)
        with pytest.raises(StatusError) as e:
            k27_view(load_contract(json.dumps(d)))
        assert e.value.code == 6 and needle in str(e.value), str(e.value)
    d = json.loads(json.dumps(base))
    d["rope"]["theta"] = 50000  # integers are valid where a float is expected
    assert k27_view(load_contract(json.dumps(d)))["rope"]["theta"] == 50000


def test_family_dispatch():
    D = C.contract.ContractDocument
    with pytest.raises(StatusError) as e:
        D.parse('{"layer_count": 2}').family()
    assert e.value.code == 6
    with pytest.raises(StatusError) as e:
        D.parse('{"architecture": "Glm52", "layer_count": 2}').family()
    assert e.value.code == 19  # unsupported


def test_hf_config_dialect():
    ref = v2_lite()
    hf = {"architectures": ["DeepseekV2ForCausalLM"], "vocab_size": 102400, "hidden_size": 2048,
          "num_hidden_layers": 27, "num_attention_heads": 16, "q_lora_rank": None, "kv_lora_rank": 512,
          "qk_nope_head_dim": 128, "qk_rope_head_dim": 64, "v_head_dim": 128, "intermediate_size": 10944,
          "moe_intermediate_size": 1408, "n_routed_experts": 64, "num_experts_per_tok": 6, "n_shared_experts": 2,
          "first_k_dense_replace": 1, "scoring_func": "softmax", "norm_topk_prob": False,
          "routed_scaling_factor": 1.0, "rms_norm_eps": 1e-6, "rope_theta": 10000,
          "rope_scaling": ref.rope_scaling, "max_position_embeddings": ref.max_position_embeddings}
    cfg = config_from_contract(json.dumps(hf))
    for f in ("hidden_size", "num_layers", "num_heads", "kv_lora_rank", "n_routed_experts", "num_experts_per_tok",
              "n_shared_experts", "moe_intermediate_size", "intermediate_size", "first_k_dense_replace"):
        assert getattr(cfg, f) == getattr(ref, f), f
    assert cfg.q_lora_rank is None and config_from_hf(hf).vocab_size == 102400


# ------------------------------------------------------------------ driver loader
def _cc():
    for c in ("cc", "gcc", "clang"):
        if shutil.which(c):
            return c
    pytest.skip("no C compiler")


def _build_driver(tmp_path, name, *defines):
    out = tmp_path / f"{name}.so"
    cmd = [_cc(), "-shared", "-fPIC", "-O1", f"-I{INCLUDE}", *[f"-D{d}" for d in defines], str(FIXTURE),
           "-o", str(out)]
    subprocess.run(cmd, check=True, capture_output=True)
    return str(out)


def test_loads_valid_fixture_driver(tmp_path):
    Dv = C.driver
    drv = Dv.ModelDriver.load(_build_driver(tmp_path, "ok"))
    assert (drv.model_id, drv.model_revision, drv.stage_name, drv.target) == ("fixture-model", "r1", "stage0",
                                                                             "host.cpu")
    assert drv.module_instance_count == 1
    progs = drv.programs()
    assert [p.name for p in progs] == ["fixture_program", "fixture_program_b"]
    assert progs[0].program_id == 1 and progs[0].max_inflight == 1
    assert progs[0].flags & Dv.PROGRAM_NO_DEVICE_MEMCPY
    assert drv.find_program("fixture_program_b").program_id == 2 and drv.find_program("nope") is None
    drv.create("{}")
    assert drv.admit(1, 9, 100) == 4
    assert drv.submit(1, b"abc") == b"cba" and drv.submit(2, b"xy", 2) == b"yx"
    assert drv.snapshot().submits == 2
    with pytest.raises(StatusError):
        drv.submit(7, b"a")  # unknown program
    drv.destroy()
    assert not drv.has_instance


def test_target_match_and_mismatch(tmp_path):
    path = _build_driver(tmp_path, "ok")
    assert C.driver.ModelDriver.load(path, "host.cpu").target == "host.cpu"
    with pytest.raises(StatusError) as e:
        C.driver.ModelDriver.load(path, "sm_100a.b200")
    assert e.value.code == 11 and "host.cpu" in str(e.value)  # target_mismatch


@pytest.mark.parametrize("brk,code", [(1, 10), (2, 10), (3, 9), (4, 16), (5, 13)])
def test_invalid_drivers_fail_closed(tmp_path, brk, code):
    # 1 ABI version, 2 malformed sha256, 3 latency claim without a latency, 4 duplicate program id,
    # 5 no interface symbol
    path = _build_driver(tmp_path, f"bad{brk}", f"SPB_FAKE_BREAK={brk}")
    with pytest.raises(StatusError) as e:
        C.driver.ModelDriver.load(path)
    assert e.value.code == code, str(e.value)


def test_missing_file_is_a_load_error(tmp_path):
    with pytest.raises(StatusError) as e:
        C.driver.ModelDriver.load(str(tmp_path / "absent.so"))
    assert e.value.code == 13


def test_sha256_hex():
    assert C.driver.sha256_hex_is_valid("ab" * 32) and C.driver.sha256_hex_is_valid("AB" * 32)
    assert not C.driver.sha256_hex_is_valid("ab" * 31) and not C.driver.sha256_hex_is_valid("zz" * 32)


def test_c_layout_gate(tmp_path):
    """sizeof / offsetof of every ABI struct: the C compiler's view must equal the C++ loader's."""
    layout = C.driver.abi_layout()
    probe = tmp_path / "probe.c"
    lines = ["#include <stdio.h>", "#include <stddef.h>", "#include <sparkpipe_b200/model_driver.h>",
             "int main(void) {"]
    for expr in layout:
        c_expr = expr.replace("alignof(", "_Alignof(")
        lines.append(f'  printf("%s=%llu\\n", "{expr}", (unsigned long long)({c_expr}));')
    lines.append("  return 0; }")
    probe.write_text("\n".join(lines))
    exe = tmp_path / "probe"
    subprocess.run([_cc(), "-std=c11", f"-I{INCLUDE}", str(probe), "-o", str(exe)], check=True,
                   capture_output=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    c_view = dict(line.rsplit("=", 1) for line in out.splitlines() if line)
    assert {k: int(v) for k, v in c_view.items()} == dict(layout)
    assert layout["sizeof(spb_model_driver_descriptor)"] == 72 and layout["sizeof(spb_program_profile)"] == 48
