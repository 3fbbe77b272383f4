"""Plain PyTorch fp32 forward of the MLA-MoE decoder: the numerics oracle.

This is the reference every kernel and the engine are checked against. It uses
the expanded (non-absorbed) MLA form, dense causal attention over the whole
sequence and per-expert loops, in fp32, on whatever device its inputs live.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from .config import MLAMoEConfig
from .rope import apply_rope, cos_sin_table


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    x = x.float()
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.float()


def route(cfg: MLAMoEConfig, x: torch.Tensor, gate: torch.Tensor, bias: torch.Tensor | None):
    logits = x.float() @ gate.float().t()
    if cfg.scoring_func == "softmax":
        scores = logits.softmax(-1)
        sel = scores
    else:
        scores = logits.sigmoid()
        sel = scores + (bias.float() if bias is not None else 0.0)
    if cfg.group_limited:
        T, E = sel.shape
        g = sel.view(T, cfg.n_group, E // cfg.n_group)
        gscore = g.topk(2, -1).values.sum(-1) if cfg.topk_method == "noaux_tc" else g.max(-1).values
        keep = torch.zeros_like(gscore, dtype=torch.bool).scatter_(1, gscore.topk(cfg.topk_group, -1).indices, True)
        sel = sel.masked_fill(~keep.repeat_interleave(E // cfg.n_group, 1), float("-inf"))
    ids = sel.topk(cfg.num_experts_per_tok, dim=-1).indices
    w = scores.gather(-1, ids)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    return ids, w * cfg.routed_scaling_factor, logits


def fake_quant_e4m3(x: torch.Tensor) -> torch.Tensor:
    """Per-(row, 128-column) e4m3 quantise-dequantise (scale = block amax / 448), the
    activation rounding of the fp8 GEMM path."""
    x = x.float()
    S, K = x.shape
    b = x.view(S, K // 128, 128)
    amax = b.abs().amax(-1, keepdim=True)
    scale = torch.where(amax > 0, amax / 448.0, torch.ones_like(amax))
    q = (b * (1.0 / scale)).to(torch.float8_e4m3fn).float()
    return (q * scale).view(S, K)


def _mm(x: torch.Tensor, w: torch.Tensor, aq: bool = False) -> torch.Tensor:
    """x @ w.T in fp32; with ``aq`` the activations first take the fp8 rounding
    (where the weight is stored in fp8: input dimension in whole 128-blocks)."""
    return (fake_quant_e4m3(x) if aq and w.shape[-1] % 128 == 0 else x.float()) @ w.float().t()


def swiglu_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor, aq: bool = False) -> torch.Tensor:
    h = _mm(x, w13, aq)
    f = w13.shape[0] // 2
    return _mm(F.silu(h[..., :f]) * h[..., f:], w2, aq)


def moe(cfg: MLAMoEConfig, W: dict, p: str, x: torch.Tensor, routing=None, aq: bool = False) -> torch.Tensor:
    """Routed experts 0..E-1 (top-k) plus the shared experts E..E+S-1 on every token."""
    ids, w, _ = route(cfg, x, W[p + "gate"], W.get(p + "gate_bias")) if routing is None else routing
    out = torch.zeros_like(x, dtype=torch.float32)
    E = cfg.n_routed_experts
    for e in range(E):
        mask = ids == e
        rows = mask.any(-1).nonzero().flatten()
        if rows.numel() == 0:
            continue
        we = (w * mask).sum(-1)[rows]
        y = swiglu_mlp(x[rows].float(), W[p + "e_w13"][e], W[p + "e_w2"][e], aq)
        out[rows] += we[:, None] * y
    for s in range(cfg.n_shared_experts):
        out += swiglu_mlp(x.float(), W[p + "e_w13"][E + s], W[p + "e_w2"][E + s], aq)
    return out


def attention(cfg: MLAMoEConfig, W: dict, p: str, x: torch.Tensor, pos: torch.Tensor, table: torch.Tensor,
              aq: bool = False):
    """x [S, H] of one sequence (positions pos) -> [S, H]. ``aq``: the projections
    take fp8-rounded activations (the block-scaled fp8 weight path)."""
    S = x.shape[0]
    nh, dn, dr, dv = cfg.num_heads, cfg.qk_nope_head_dim, cfg.qk_rope_head_dim, cfg.v_head_dim
    kvl = cfg.kv_lora_rank
    qa_dim = cfg.q_lora_rank or cfg.q_out_dim
    a = _mm(x, W[p + "w_qkv_a"], aq)
    if cfg.q_lora_rank:
        q = _mm(rmsnorm(a[:, :qa_dim], W[p + "q_a_norm"], cfg.rms_norm_eps), W[p + "w_q_b"], aq)
    else:
        q = a[:, :qa_dim]
    kv_a = a[:, qa_dim:]
    latent = rmsnorm(kv_a[:, :kvl], W[p + "kv_a_norm"], cfg.rms_norm_eps)
    k_pe = apply_rope(kv_a[:, kvl:], pos, table)                     # [S, dr]
    q = q.view(S, nh, dn + dr)
    q_nope, q_pe = q[..., :dn], apply_rope(q[..., dn:], pos, table)
    kv = (latent @ W[p + "w_kv_b"].float().t()).view(S, nh, dn + dv)
    k_nope, v = kv[..., :dn], kv[..., dn:]
    qf = torch.cat([q_nope, q_pe], -1).transpose(0, 1)                # [nh, S, dn+dr]
    kf = torch.cat([k_nope, k_pe[:, None, :].expand(S, nh, dr)], -1).transpose(0, 1)
    scores = (qf @ kf.transpose(1, 2)) * cfg.softmax_scale()
    mask = torch.ones(S, S, dtype=torch.bool, device=x.device).tril()
    scores = scores.masked_fill(~mask, float("-inf"))
    o = scores.softmax(-1) @ v.transpose(0, 1)                        # [nh, S, dv]
    o = o.transpose(0, 1).reshape(S, nh * dv)
    return _mm(o, W[p + "w_o"], aq)


def forward(cfg: MLAMoEConfig, W: dict, tokens: torch.Tensor, table: torch.Tensor | None = None,
            return_hidden: bool = False, act_quant: bool = False):
    """tokens [S] (one sequence) -> logits [S, V] in fp32. ``act_quant`` rounds the
    inputs of the fp8-weight GEMMs to e4m3 per 1x128 block, as the fp8 kernels do."""
    S = tokens.shape[0]
    pos = torch.arange(S, device=tokens.device)
    if table is None:
        table = cos_sin_table(cfg, max(S, 1), device=tokens.device)
    h = W["embed"][tokens.long()].float()
    for i in range(cfg.num_layers):
        p = f"l{i}."
        h = h + attention(cfg, W, p, rmsnorm(h, W[p + "in_norm"], cfg.rms_norm_eps), pos, table, act_quant)
        x = rmsnorm(h, W[p + "post_norm"], cfg.rms_norm_eps)
        if cfg.is_moe_layer(i):
            h = h + moe(cfg, W, p, x, aq=act_quant)
        else:
            h = h + swiglu_mlp(x, W[p + "w13"], W[p + "w2"], act_quant)
    hn = rmsnorm(h, W["final_norm"], cfg.rms_norm_eps)
    logits = hn @ W["lm_head"].float().t()
    return (logits, h) if return_hidden else logits


def greedy_generate(cfg: MLAMoEConfig, W: dict, prompt: torch.Tensor, new_tokens: int):
    """Greedy decode by re-running the full forward each step (oracle for the engine).
    Returns (generated ids [new_tokens], logits of each generated position [new_tokens, V])."""
    seq = prompt.clone()
    outs, logits_all = [], []
    table = cos_sin_table(cfg, prompt.shape[0] + new_tokens + 1, device=prompt.device)
    for _ in range(new_tokens):
        logits = forward(cfg, W, seq, table)[-1]
        nxt = int(logits.argmax())
        outs.append(nxt)
        logits_all.append(logits)
        seq = torch.cat([seq, torch.tensor([nxt], dtype=seq.dtype, device=seq.device)])
    return torch.tensor(outs), torch.stack(logits_all)
