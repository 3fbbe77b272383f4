"""Model contracts -> engine configuration.

``load_contract(text or path)`` parses and envelope-validates a contract document
(C++ ``ContractDocument``); ``config_from_contract`` dispatches on its family and
returns an ``MLAMoEConfig``. Two dialects are understood:

* the K2-family contract format (``architecture`` =
  ``KimiK25ForConditionalGeneration``; sections model / mla / rope / moe /
  quantization / speculation / cache / tokens / qualification), validated field by
  field in C++ (``ContractDocument.as_k27``);
* a Hugging Face ``config.json`` of a DeepSeek-V2 / V3 family checkpoint
  (``DeepseekV2ForCausalLM``, ``DeepseekV3ForCausalLM``).

Reference: crates/spark-model/src/{contract.rs,k27.rs,family.rs} and the
contract-to-geometry step crates/spark-node/src/backend/k27_geometry.rs:14-128.
"""
from __future__ import annotations

import json
from pathlib import Path

from ..core import core
from .config import MLAMoEConfig

HF_ARCHITECTURES = ("DeepseekV2ForCausalLM", "DeepseekV3ForCausalLM")
CONTRACT_DIR = Path(__file__).resolve().parent / "contracts"


def load_contract(text_or_path):
    """Parse a contract (JSON text, or a path to a JSON file)."""
    p = Path(text_or_path) if not str(text_or_path).lstrip().startswith("{") else None
    if p is not None:
        return core().contract.ContractDocument.parse(p.read_text(), str(p))
    return core().contract.ContractDocument.parse(str(text_or_path))


def k27_view(doc) -> dict:
    """The validated K2-family sections (defaults filled) as a dict."""
    return json.loads(doc.as_k27_json())


_TOPK_METHOD = {"greedy": "greedy", "group_limited_greedy": "group_limited_greedy", "noaux_tc": "noaux_tc"}


def config_from_k27(view: dict, name: str | None = None) -> MLAMoEConfig:
    m, a, r, e, q = view["model"], view["mla"], view["rope"], view["moe"], view["quantization"]
    if e["moe_layer_frequency"] != 1:
        raise ValueError("contract: only every-layer MoE after the dense prefix is supported")
    if a["output_gate"] or a["attention_bias"]:
        raise ValueError("contract: attention output gates / biases are not supported")
    scoring = {"sigmoid": "sigmoid", "softmax": "softmax"}.get(e["router_activation"])
    if scoring is None:
        raise ValueError(f"contract: unknown router activation {e['router_activation']!r}")
    rope_scaling = None
    if r["type"].lower() == "yarn":
        rope_scaling = {"type": "yarn", "factor": float(r["factor"]),
                        "original_max_position_embeddings": int(r["original_max_position_embeddings"]),
                        "beta_fast": float(r["beta_fast"]), "beta_slow": float(r["beta_slow"]),
                        "mscale": float(r["mscale"]), "mscale_all_dim": float(r["mscale_all_dim"])}
    fp8 = q["non_expert_weight_format"].lower().startswith("fp8") or \
        q["routed_expert_weight_format"].lower().startswith("fp8")
    return MLAMoEConfig(
        name=name or view.get("model_id", "contract-model"),
        vocab_size=m["vocabulary_size"],
        hidden_size=m["hidden_dimension"],
        num_layers=m["layer_count"],
        num_heads=a["query_head_count"],
        q_lora_rank=a["query_lora_rank"] or None,
        kv_lora_rank=a["kv_lora_rank"],
        qk_nope_head_dim=a["qk_nope_dimension"],
        qk_rope_head_dim=a["qk_unrotated_dimension"],
        v_head_dim=a["value_head_dimension"],
        intermediate_size=e["dense_intermediate_dimension"],
        moe_intermediate_size=e["expert_intermediate_dimension"],
        n_routed_experts=e["routed_expert_count"],
        num_experts_per_tok=e["experts_per_token"],
        n_shared_experts=e["shared_expert_count"],
        first_k_dense_replace=m["first_routed_layer"],
        scoring_func=scoring,
        n_group=int(e["router_group_count"]) or 1,
        topk_group=int(e.get("selected_group_count", e["router_group_count"])) or 1,
        topk_method=_TOPK_METHOD.get(e["top_k_method"], "greedy"),
        norm_topk_prob=bool(e["renormalize_selected_probabilities"]),
        routed_scaling_factor=float(e["routed_scaling_factor"]),
        rms_norm_eps=float(m["rms_norm_epsilon"]),
        rope_theta=float(r["theta"]),
        rope_scaling=rope_scaling,
        max_position_embeddings=m["maximum_context_tokens"],
        weight_dtype="fp8_block" if fp8 else "bf16",
        tie_word_embeddings=bool(m["tie_word_embeddings"]),
    )


def config_from_hf(cfg: dict, name: str | None = None) -> MLAMoEConfig:
    """DeepSeek-V2 / V3 family ``config.json`` -> MLAMoEConfig."""
    rs = cfg.get("rope_scaling")
    if rs and rs.get("type", rs.get("rope_type")) == "yarn":
        rs = {"type": "yarn", "factor": float(rs["factor"]),
              "original_max_position_embeddings": int(rs["original_max_position_embeddings"]),
              "beta_fast": float(rs.get("beta_fast", 32)), "beta_slow": float(rs.get("beta_slow", 1)),
              "mscale": float(rs.get("mscale", 1)), "mscale_all_dim": float(rs.get("mscale_all_dim", 0))}
    else:
        rs = None
    quant = cfg.get("quantization_config") or {}
    return MLAMoEConfig(
        name=name or cfg.get("_name_or_path", cfg["architectures"][0]),
        vocab_size=cfg["vocab_size"],
        hidden_size=cfg["hidden_size"],
        num_layers=cfg["num_hidden_layers"],
        num_heads=cfg["num_attention_heads"],
        q_lora_rank=cfg.get("q_lora_rank"),
        kv_lora_rank=cfg["kv_lora_rank"],
        qk_nope_head_dim=cfg["qk_nope_head_dim"],
        qk_rope_head_dim=cfg["qk_rope_head_dim"],
        v_head_dim=cfg["v_head_dim"],
        intermediate_size=cfg["intermediate_size"],
        moe_intermediate_size=cfg["moe_intermediate_size"],
        n_routed_experts=cfg["n_routed_experts"],
        num_experts_per_tok=cfg["num_experts_per_tok"],
        n_shared_experts=cfg.get("n_shared_experts", 0) or 0,
        first_k_dense_replace=cfg.get("first_k_dense_replace", 0),
        scoring_func=cfg.get("scoring_func", "softmax"),
        n_group=int(cfg.get("n_group") or 1),
        topk_group=int(cfg.get("topk_group") or 1),
        topk_method=_TOPK_METHOD.get(cfg.get("topk_method", "greedy"), "greedy"),
        norm_topk_prob=bool(cfg.get("norm_topk_prob", False)),
        routed_scaling_factor=float(cfg.get("routed_scaling_factor", 1.0)),
        rms_norm_eps=float(cfg.get("rms_norm_eps", 1e-6)),
        rope_theta=float(cfg.get("rope_theta", 10000.0)),
        rope_scaling=rs,
        max_position_embeddings=cfg.get("max_position_embeddings", 4096),
        weight_dtype="fp8_block" if quant.get("quant_method") == "fp8" else "bf16",
        tie_word_embeddings=bool(cfg.get("tie_word_embeddings", False)),
    )


def config_from_contract(doc_or_text, name: str | None = None) -> MLAMoEConfig:
    """Family dispatch: K2-family contract or HF DeepSeek config -> MLAMoEConfig."""
    if isinstance(doc_or_text, (str, Path)):
        text = Path(doc_or_text).read_text() if not str(doc_or_text).lstrip().startswith("{") else str(doc_or_text)
        raw = json.loads(text)
        if any(a in HF_ARCHITECTURES for a in raw.get("architectures", [])):
            return config_from_hf(raw, name)
        doc = core().contract.ContractDocument.parse(text)
    else:
        doc = doc_or_text
    family = doc.family()
    if family == "k27":
        return config_from_k27(k27_view(doc), name)
    raise ValueError(f"contract family {family!r} has no engine configuration")


def bundled_contract(name: str) -> Path:
    """Path of a contract shipped with the package (``contracts/<name>.json``)."""
    return CONTRACT_DIR / f"{name}.json"
