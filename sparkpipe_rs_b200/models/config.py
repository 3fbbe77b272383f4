"""MLA-MoE decoder configurations.

The field names follow the typed model-contract view of the reference
(crates/spark-model/src/k27.rs:10-162: model / MLA / RoPE-YaRN / MoE /
quantization / speculation sections) so a contract document maps onto this
dataclass field by field (see ``models.contract``).

Presets are the serving workloads this engine is measured on:
  * ``tiny``     — 2-layer CPU plumbing model (hidden 256, 8 experts top-2 + 1 shared)
  * ``v2_lite``  — DeepSeek-V2-Lite shape (27 layers, hidden 2048, 64 experts top-6 + 2 shared)
  * ``k2``       — Kimi-K2 shape 1T (61 layers, hidden 7168, 384 experts top-8 + 1 shared)
  * ``v3``       — DeepSeek-V3 shape 671B (256 experts top-8 in 8 groups, best 4 groups kept)
  * ``mtp_head`` — 1-layer MTP-style draft head for speculative decoding
"""
from __future__ import annotations

import dataclasses
import math
from dataclasses import dataclass, field


@dataclass
class MLAMoEConfig:
    name: str = "custom"
    vocab_size: int = 1024
    hidden_size: int = 256
    num_layers: int = 2
    num_heads: int = 4
    q_lora_rank: int | None = 96
    kv_lora_rank: int = 64
    qk_nope_head_dim: int = 32
    qk_rope_head_dim: int = 16
    v_head_dim: int = 32
    intermediate_size: int = 512          # dense FFN of the first_k_dense layers
    moe_intermediate_size: int = 128
    n_routed_experts: int = 8
    num_experts_per_tok: int = 2
    n_shared_experts: int = 1
    first_k_dense_replace: int = 0
    scoring_func: str = "softmax"         # "softmax" | "sigmoid"
    n_group: int = 1                      # expert groups of group-limited routing (1 = off)
    topk_group: int = 1                   # groups kept per token
    topk_method: str = "greedy"           # "greedy" | "group_limited_greedy" (group = best expert) | "noaux_tc" (best two)
    norm_topk_prob: bool = False
    routed_scaling_factor: float = 1.0
    rms_norm_eps: float = 1e-6
    rope_theta: float = 10000.0
    rope_scaling: dict | None = None      # YaRN: factor, original_max_position_embeddings, beta_fast, beta_slow, mscale, mscale_all_dim
    max_position_embeddings: int = 8192
    weight_dtype: str = "bf16"            # "bf16" | "fp8_block" (128x128 e4m3 + fp32 scales)
    init_std: float = 0.02
    tie_word_embeddings: bool = False

    @property
    def qk_head_dim(self) -> int:
        return self.qk_nope_head_dim + self.qk_rope_head_dim

    @property
    def kv_cache_dim(self) -> int:
        return self.kv_lora_rank + self.qk_rope_head_dim

    @property
    def q_out_dim(self) -> int:
        return self.num_heads * self.qk_head_dim

    def is_moe_layer(self, i: int) -> bool:
        return self.n_routed_experts > 0 and i >= self.first_k_dense_replace

    @property
    def shared_intermediate(self) -> int:
        return self.moe_intermediate_size * self.n_shared_experts

    @property
    def group_limited(self) -> bool:
        return self.n_group > 1 and self.topk_group < self.n_group

    def softmax_scale(self) -> float:
        s = 1.0 / math.sqrt(self.qk_head_dim)
        rs = self.rope_scaling
        if rs and rs.get("mscale_all_dim"):
            m = yarn_mscale(rs["factor"], rs["mscale_all_dim"])
            s = s * m * m
        return s

    def param_count(self) -> int:
        H, L = self.hidden_size, self.num_layers
        nh = self.num_heads
        att = 0
        if self.q_lora_rank:
            att += H * self.q_lora_rank + self.q_lora_rank * self.q_out_dim
        else:
            att += H * self.q_out_dim
        att += H * self.kv_cache_dim + self.kv_lora_rank * nh * (self.qk_nope_head_dim + self.v_head_dim)
        att += nh * self.v_head_dim * H
        total = 2 * self.vocab_size * H
        for i in range(L):
            total += att
            if self.is_moe_layer(i):
                total += (self.n_routed_experts + self.n_shared_experts) * 3 * H * self.moe_intermediate_size
                total += self.n_routed_experts * H
            else:
                total += 3 * H * self.intermediate_size
        return total

    def replace(self, **kw) -> "MLAMoEConfig":
        return dataclasses.replace(self, **kw)

    def to_dict(self) -> dict:
        return dataclasses.asdict(self)


def yarn_mscale(scale: float, mscale: float = 1.0) -> float:
    if scale <= 1.0:
        return 1.0
    return 0.1 * mscale * math.log(scale) + 1.0


def tiny() -> MLAMoEConfig:
    """CPU plumbing model: 2 layers, hidden 256, 4 heads, q_lora 96, kv_lora 64,
    nope 32 / rope 16 / v 32, 8 experts top-2 + 1 shared, expert FFN 128, vocab 1024."""
    return MLAMoEConfig(name="tiny-mla-moe")


def v2_lite() -> MLAMoEConfig:
    """DeepSeek-V2-Lite shape: 27 layers (first dense, FFN 10944), hidden 2048, 16 heads,
    no q LoRA, kv_lora 512, nope 128 / rope 64 / v 128, 64 experts top-6 + 2 shared (FFN 1408),
    vocab 102400, YaRN RoPE (factor 40)."""
    return MLAMoEConfig(
        name="deepseek-v2-lite-shape",
        vocab_size=102400,
        hidden_size=2048,
        num_layers=27,
        num_heads=16,
        q_lora_rank=None,
        kv_lora_rank=512,
        qk_nope_head_dim=128,
        qk_rope_head_dim=64,
        v_head_dim=128,
        intermediate_size=10944,
        moe_intermediate_size=1408,
        n_routed_experts=64,
        num_experts_per_tok=6,
        n_shared_experts=2,
        first_k_dense_replace=1,
        scoring_func="softmax",
        norm_topk_prob=False,
        routed_scaling_factor=1.0,
        rms_norm_eps=1e-6,
        rope_theta=10000.0,
        rope_scaling={"type": "yarn", "factor": 40.0, "original_max_position_embeddings": 4096,
                      "beta_fast": 32.0, "beta_slow": 1.0, "mscale": 0.707, "mscale_all_dim": 0.707},
        max_position_embeddings=163840,
    )


def k2() -> MLAMoEConfig:
    """Kimi-K2 shape (1T): 61 layers (first dense, FFN 18432), hidden 7168, 64 heads,
    q_lora 1536, kv_lora 512, 384 experts top-8 + 1 shared (FFN 2048), vocab 163840,
    block-scaled fp8 weights."""
    return MLAMoEConfig(
        name="kimi-k2-shape",
        vocab_size=163840,
        hidden_size=7168,
        num_layers=61,
        num_heads=64,
        q_lora_rank=1536,
        kv_lora_rank=512,
        qk_nope_head_dim=128,
        qk_rope_head_dim=64,
        v_head_dim=128,
        intermediate_size=18432,
        moe_intermediate_size=2048,
        n_routed_experts=384,
        num_experts_per_tok=8,
        n_shared_experts=1,
        first_k_dense_replace=1,
        scoring_func="sigmoid",
        topk_method="noaux_tc",
        norm_topk_prob=True,
        routed_scaling_factor=2.827,
        rms_norm_eps=1e-6,
        rope_theta=50000.0,
        rope_scaling={"type": "yarn", "factor": 64.0, "original_max_position_embeddings": 4096,
                      "beta_fast": 32.0, "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0},
        max_position_embeddings=262144,
        weight_dtype="fp8_block",
    )


def v3() -> MLAMoEConfig:
    """DeepSeek-V3 shape (671B): 61 layers (first 3 dense, FFN 18432), hidden 7168,
    128 heads, q_lora 1536, kv_lora 512, 256 experts top-8 + 1 shared (FFN 2048) with
    group-limited routing (8 groups, best 4 kept, group = sum of its best two),
    vocab 129280, block-scaled fp8 weights."""
    return k2().replace(
        name="deepseek-v3-shape", vocab_size=129280, num_heads=128, first_k_dense_replace=3,
        n_routed_experts=256, n_group=8, topk_group=4, routed_scaling_factor=2.5, rope_theta=10000.0,
        rope_scaling={"type": "yarn", "factor": 40.0, "original_max_position_embeddings": 4096,
                      "beta_fast": 32.0, "beta_slow": 1.0, "mscale": 1.0, "mscale_all_dim": 1.0},
        max_position_embeddings=163840)


def mtp_head(target: MLAMoEConfig) -> MLAMoEConfig:
    """1-layer MTP-style draft head: same hidden/attention as the target, 1 MLA layer
    plus one dense FFN of width 1408."""
    return target.replace(name=target.name + "-mtp", num_layers=1, first_k_dense_replace=1,
                          intermediate_size=1408)


PRESETS = {"tiny": tiny, "v2_lite": v2_lite, "k2": k2, "v3": v3}


def get_config(name: str) -> MLAMoEConfig:
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    return PRESETS[name]()
