"""Seeded random-init weights for the MLA-MoE decoder, in the engine's layout.

Every matrix is ``[out_features, in_features]`` (K-major), which is the operand
layout of the tcgen05 GEMM. Per layer ``i`` (prefix ``l{i}.``):

  in_norm [H] · w_qkv_a [Qa + kv_lora + rope, H] (q path (LoRA-A or full q) and
  kv_a fused into one GEMM) · q_a_norm [q_lora] · w_q_b [Hh*(dn+dr), q_lora] ·
  kv_a_norm [kv_lora] · w_kv_b [Hh*(dn+dv), kv_lora] · w_o [H, Hh*dv] ·
  post_norm [H] · dense: w13 [2I, H], w2 [H, I] · MoE: gate [E, H],
  gate_bias [E] (fp32), e_w13 [E + S, 2F, H], e_w2 [E + S, H, F]

plus ``embed`` [V, H], ``final_norm`` [H] and ``lm_head`` [V, H]. ``w13`` stacks
the gate projection rows on top of the up projection rows. Experts E .. E+S-1
are the S shared experts (each of width F; together they are the shared MLP of
width S*F, which decomposes exactly into per-expert SwiGLU blocks), so routed
and shared experts run in one grouped GEMM.

Values are N(0, init_std) (norm weights 1, router bias 0), drawn per tensor from
a generator seeded with (seed, tensor index), so any subset of layers or any
device produces the same numbers.

With ``weight_dtype == "fp8_block"`` (on a CUDA device) the projection and expert
matrices (``FP8_WEIGHTS``) are block-scaled e4m3 (``ops.Fp8Weight``: 128x128
blocks, fp32 scales), sampled and quantised on the device by one kernel from a
counter-based generator: element (r, c) of a 2-D view is sample r * cols + c of
the tensor's stream, so an expert-parallel rank's slice equals the same rows of
the whole tensor. Embeddings, norms, the router, ``w_kv_b`` (the absorbed-MLA
operands) and the LM head stay bf16.
"""
from __future__ import annotations

import torch

from .config import MLAMoEConfig


def weight_shapes(cfg: MLAMoEConfig) -> dict[str, tuple]:
    H, nh = cfg.hidden_size, cfg.num_heads
    dn, dr, dv = cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
    qa = cfg.q_lora_rank or cfg.q_out_dim
    shapes: dict[str, tuple] = {"embed": (cfg.vocab_size, H)}
    for i in range(cfg.num_layers):
        p = f"l{i}."
        shapes[p + "in_norm"] = (H,)
        shapes[p + "w_qkv_a"] = (qa + cfg.kv_cache_dim, H)
        if cfg.q_lora_rank:
            shapes[p + "q_a_norm"] = (cfg.q_lora_rank,)
            shapes[p + "w_q_b"] = (nh * (dn + dr), cfg.q_lora_rank)
        shapes[p + "kv_a_norm"] = (cfg.kv_lora_rank,)
        shapes[p + "w_kv_b"] = (nh * (dn + dv), cfg.kv_lora_rank)
        shapes[p + "w_o"] = (H, nh * dv)
        shapes[p + "post_norm"] = (H,)
        if cfg.is_moe_layer(i):
            E, F = cfg.n_routed_experts, cfg.moe_intermediate_size
            shapes[p + "gate"] = (E, H)
            shapes[p + "gate_bias"] = (E,)
            S = cfg.n_shared_experts
            shapes[p + "e_w13"] = (E + S, 2 * F, H)
            shapes[p + "e_w2"] = (E + S, H, F)
        else:
            shapes[p + "w13"] = (2 * cfg.intermediate_size, H)
            shapes[p + "w2"] = (H, cfg.intermediate_size)
    shapes["final_norm"] = (H,)
    shapes["lm_head"] = (cfg.vocab_size, H)
    return shapes


def _is_norm(name: str) -> bool:
    return name.endswith("norm")


FP8_WEIGHTS = ("w_qkv_a", "w_q_b", "w_o", "w13", "w2", "e_w13", "e_w2")


def is_fp8_weight(cfg: MLAMoEConfig, name: str, shape: tuple | None = None) -> bool:
    """fp8 applies to the FP8_WEIGHTS whose input dimension is whole 128-column blocks."""
    if cfg.weight_dtype != "fp8_block" or name.split(".")[-1] not in FP8_WEIGHTS:
        return False
    return shape is None or shape[-1] % 128 == 0


def _fp8_tensor(cfg: MLAMoEConfig, shape: tuple, seed: int, dev, experts):
    from .. import ops

    if len(shape) == 2:
        return ops.quant_weight_fp8(shape[0], shape[1], seed=seed, std=cfg.init_std, device=dev)
    G, R, C = shape
    parts = [(0, G)] if experts is None else [experts, (cfg.n_routed_experts, G)]
    n = sum(hi - lo for lo, hi in parts)
    q = torch.empty(n, R, C, dtype=torch.float8_e4m3fn, device=dev)
    s = torch.empty(n, R // 128, C // 128, dtype=torch.float32, device=dev)
    at = 0
    for lo, hi in parts:
        if hi > lo:
            part = ops.Fp8Weight(q[at:at + hi - lo], s[at:at + hi - lo], 128)
            ops.quant_weight_fp8((hi - lo) * R, C, seed=seed, std=cfg.init_std, flat0=lo * R * C, out=part)
            at += hi - lo
    return ops.Fp8Weight(q, s, 128)


def dequant_weights(w: dict) -> dict:
    """fp32 copy of a weight dict with every ``Fp8Weight`` dequantised (oracle use)."""
    from .. import ops

    return {k: (v.dequant() if isinstance(v, ops.Fp8Weight) else v.float()) for k, v in w.items()}


def init_weights(cfg: MLAMoEConfig, seed: int = 0, device="cpu", dtype=torch.bfloat16,
                 layers: list[int] | None = None, experts: tuple[int, int] | None = None,
                 share: dict | None = None) -> dict[str, torch.Tensor]:
    """Random-init weights. ``layers`` restricts which decoder layers are created;
    ``experts`` = (lo, hi) keeps only routed experts lo..hi-1 (plus every shared
    expert) of the expert tensors, as one expert-parallel rank holds them. The
    kept rows are bit-identical to the same rows of the full tensors. Tensors
    named in ``share`` are taken from it instead of being created (a draft head
    sharing the target's embedding and LM head)."""
    shapes = weight_shapes(cfg)
    out: dict[str, torch.Tensor] = {}
    dev = torch.device(device)
    for idx, (name, shape) in enumerate(shapes.items()):
        if share is not None and name in share:
            out[name] = share[name]
            continue
        if layers is not None and name.startswith("l"):
            li = int(name[1:name.index(".")])
            if li not in layers:
                continue
        if _is_norm(name):
            out[name] = torch.ones(shape, dtype=dtype, device=dev)
            continue
        if name.endswith("gate_bias"):
            out[name] = torch.zeros(shape, dtype=torch.float32, device=dev)
            continue
        tseed = (seed * 1_000_003 + idx) & 0x7FFFFFFFFFFFFFFF
        if dev.type == "cuda" and is_fp8_weight(cfg, name, shape):
            out[name] = _fp8_tensor(cfg, shape, tseed, dev, experts if name.endswith(("e_w13", "e_w2")) else None)
            continue
        g = torch.Generator(device=dev)
        g.manual_seed(tseed)
        t = torch.empty(shape, dtype=dtype, device=dev)
        if dtype in (torch.float32, torch.bfloat16, torch.float16):
            t.normal_(0.0, cfg.init_std, generator=g)
        else:
            t.copy_(torch.empty(shape, dtype=torch.float32, device=dev).normal_(0.0, cfg.init_std, generator=g))
        if experts is not None and (name.endswith("e_w13") or name.endswith("e_w2")):
            lo, hi = experts
            t = torch.cat([t[lo:hi], t[cfg.n_routed_experts:]]).contiguous()
        out[name] = t
    return out


def derive_decode_weights(cfg: MLAMoEConfig, w: dict[str, torch.Tensor]) -> None:
    """Adds the absorbed-attention operand ``l{i}.w_uk_t`` [Hh * kv_lora, dn]:
    per head the transpose of the k_nope rows of w_kv_b (K-major for the
    q_nope -> latent product)."""
    nh, dn, dv, kvl = cfg.num_heads, cfg.qk_nope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
    for i in range(cfg.num_layers):
        k = f"l{i}.w_kv_b"
        if k not in w:
            continue
        kvb = w[k].view(nh, dn + dv, kvl)
        w[f"l{i}.w_uk_t"] = kvb[:, :dn, :].transpose(1, 2).contiguous().view(nh * kvl, dn)


def absorb_decode_weights(cfg: MLAMoEConfig, w: dict[str, torch.Tensor]) -> bool:
    """Folds the latent up-projections into the decode projections (bf16 models
    without a q LoRA), so decode attention needs two weight GEMMs instead of four:

      l{i}.w_qkv_abs [Hh * (kv_lora + rope) + kv_lora + rope, H]: per head the
          absorbed query rows W_uk[h] . W_q_nope[h] (kv_lora x H) followed by the
          head's rope rows, then the kv_a rows: one GEMM yields q_lat directly.
      l{i}.w_ov [H, Hh * kv_lora]: per head W_o[:, head] . W_uv[h]: the output
          projection straight from the latent attention output.

    Products in fp32, stored bf16. Returns False (and adds nothing) for other models."""
    if cfg.q_lora_rank:
        return False
    nh, dn, dr, dv, kvl = cfg.num_heads, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim, cfg.kv_lora_rank
    for i in range(cfg.num_layers):
        p = f"l{i}."
        if p + "w_qkv_a" not in w or not isinstance(w[p + "w_qkv_a"], torch.Tensor) or \
                not isinstance(w.get(p + "w_o"), torch.Tensor) or w[p + "w_qkv_a"].dtype != torch.bfloat16:
            return False
    for i in range(cfg.num_layers):
        p = f"l{i}."
        wqa = w[p + "w_qkv_a"]
        H = wqa.shape[1]
        q = wqa[: nh * (dn + dr)].view(nh, dn + dr, H).float()
        uk = w[p + "w_uk_t"].view(nh, kvl, dn).float()
        q_abs = torch.bmm(uk, q[:, :dn, :])                                     # [nh, kvl, H]
        rows = torch.cat([q_abs, q[:, dn:, :]], dim=1).reshape(nh * (kvl + dr), H)
        w[p + "w_qkv_abs"] = torch.cat([rows.to(torch.bfloat16), wqa[nh * (dn + dr):]], dim=0).contiguous()
        del q, q_abs, rows
        uv = w[p + "w_kv_b"].view(nh, dn + dv, kvl)[:, dn:, :].float()           # [nh, dv, kvl]
        wo = w[p + "w_o"].view(H, nh, dv).permute(1, 0, 2).float()               # [nh, H, dv]
        w[p + "w_ov"] = torch.bmm(wo, uv).permute(1, 0, 2).reshape(H, nh * kvl).to(torch.bfloat16).contiguous()
        del uv, wo
    return True
