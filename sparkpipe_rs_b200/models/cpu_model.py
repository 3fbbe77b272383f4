"""CPU stage driver: the MLA-MoE forward in fp32 PyTorch over the paged latent cache.

Same call interface as ``MLAMoEModel`` (``forward(ForwardBatch, KVCache, layers,
hidden_in, return_hidden)``), so the serving engine and the pipeline runtime
drive it exactly like the GPU model. It exists for GPU-free operation: the
CPU plumbing configuration (tiny model, two pipeline stages, logits checked
against the oracle), and CPU tests of the scheduler / engine / gateway stack.

Both prefill and decode use the expanded MLA form: the context's latent rows
are gathered from the paged cache (block table or explicit slots) and
up-projected by w_kv_b, exactly as the oracle computes them.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import oracle
from .config import MLAMoEConfig
from .mla_moe import ForwardBatch, KVCache
from .rope import apply_rope, cos_sin_table
from .weights import init_weights


class CpuMLAMoEModel:
    def __init__(self, cfg: MLAMoEConfig, weights: dict | None = None, seed: int = 0, max_positions: int = 4096,
                 layers: list[int] | None = None):
        self.cfg = cfg
        self.device = torch.device("cpu")
        if weights is None:
            weights = init_weights(cfg, seed=seed, device="cpu", dtype=torch.float32, layers=layers)
        self.w = {k: v.float() for k, v in weights.items()}
        self.cos_sin = cos_sin_table(cfg, max_positions)
        self.scale = cfg.softmax_scale()

    def new_cache(self, num_blocks: int, block_size: int = 64, layers: int | None = None) -> KVCache:
        return KVCache(self.cfg, num_blocks, block_size, device="cpu", layers=layers)

    # ------------------------------------------------------------------ pieces
    def _qkv(self, p: str, x: torch.Tensor, pos: torch.Tensor):
        c, w = self.cfg, self.w
        qa = c.q_lora_rank or c.q_out_dim
        a = x @ w[p + "w_qkv_a"].t()
        if c.q_lora_rank:
            q = oracle.rmsnorm(a[:, :qa], w[p + "q_a_norm"], c.rms_norm_eps) @ w[p + "w_q_b"].t()
        else:
            q = a[:, :qa]
        kv_a = a[:, qa:]
        latent = oracle.rmsnorm(kv_a[:, : c.kv_lora_rank], w[p + "kv_a_norm"], c.rms_norm_eps)
        k_pe = apply_rope(kv_a[:, c.kv_lora_rank:], pos, self.cos_sin)
        q = q.view(-1, c.num_heads, c.qk_head_dim)
        q = torch.cat([q[..., : c.qk_nope_head_dim], apply_rope(q[..., c.qk_nope_head_dim:], pos, self.cos_sin)], -1)
        return q, torch.cat([latent, k_pe], -1)

    def _attend(self, p: str, q: torch.Tensor, ctx: torch.Tensor, q_pos: torch.Tensor) -> torch.Tensor:
        """q [Tq, H, dn+dr] at absolute positions q_pos, ctx [Tk, kvl+dr] holding positions 0..Tk-1."""
        c, w = self.cfg, self.w
        nh, dn, dv, kvl = c.num_heads, c.qk_nope_head_dim, c.v_head_dim, c.kv_lora_rank
        Tk = ctx.shape[0]
        kv = (ctx[:, :kvl] @ w[p + "w_kv_b"].t()).view(Tk, nh, dn + dv)
        k = torch.cat([kv[..., :dn], ctx[:, None, kvl:].expand(Tk, nh, c.qk_rope_head_dim)], -1)
        s = torch.einsum("qhd,khd->hqk", q, k) * self.scale
        mask = torch.arange(Tk)[None, :] <= q_pos[:, None]
        s = s.masked_fill(~mask[None], float("-inf"))
        o = torch.einsum("hqk,khd->qhd", s.softmax(-1), kv[..., dn:])
        return o.reshape(q.shape[0], nh * dv) @ w[p + "w_o"].t()

    def _mlp(self, i: int, x: torch.Tensor) -> torch.Tensor:
        c, w = self.cfg, self.w
        p = f"l{i}."
        if c.is_moe_layer(i):
            return oracle.moe(c, w, p, x)
        return oracle.swiglu_mlp(x, w[p + "w13"], w[p + "w2"])

    def write_kv(self, fb: ForwardBatch, cache: KVCache):
        """Layer 0's latent KV of the rows of ``fb`` only (see MLAMoEModel.write_kv)."""
        c = self.cfg
        h = self.w["embed"][fb.token_ids.long()].float()
        _, row = self._qkv("l0.", oracle.rmsnorm(h, self.w["l0.in_norm"], c.rms_norm_eps), fb.positions.long())
        slots = fb.slot_mapping.long()
        keep = slots >= 0
        lc = cache.layer(0)
        lc[slots[keep]] = row[keep].to(lc.dtype)

    # ------------------------------------------------------------------ forward
    def forward(self, fb: ForwardBatch, cache: KVCache, layers=None, hidden_in=None, return_hidden=False,
                layer_offset: int = 0):
        """``layer_offset`` maps model layer i to cache layer i - layer_offset (pipeline stages
        keep only their own layers' cache)."""
        c, w = self.cfg, self.w
        layers = list(layers) if layers is not None else list(range(c.num_layers))
        ids = fb.token_ids.long()
        pos = fb.positions.long()
        slots = fb.slot_mapping.long()
        h = w["embed"][ids].float() if hidden_in is None else hidden_in.float().clone()
        T = h.shape[0]
        for i in layers:
            p = f"l{i}."
            lc = cache.layer(i - layer_offset)
            q, row = self._qkv(p, oracle.rmsnorm(h, w[p + "in_norm"], c.rms_norm_eps), pos)
            keep = slots >= 0
            lc[slots[keep]] = row[keep].to(lc.dtype)
            out = torch.empty(T, c.hidden_size)
            if fb.mode == "decode":
                bs = cache.block_size
                for b in range(T):
                    L = int(fb.context_lens[b])
                    if L == 0:
                        out[b] = 0
                        continue
                    blocks = fb.block_table[b, : (L + bs - 1) // bs].long()
                    rows = (blocks[:, None] * bs + torch.arange(bs)).flatten()[:L]
                    if fb.self_slots is not None and int(fb.self_slots[b]) >= 0:
                        rows = rows.clone()
                        rows[-1] = int(fb.self_slots[b])
                    out[b] = self._attend(p, q[b:b + 1], lc[rows].float(), pos[b:b + 1])[0]
            else:
                cu_q = fb.cu_q.long().tolist()
                cu_k = fb.cu_k.long().tolist()
                for b in range(len(cu_q) - 1):
                    q0, q1, k0, k1 = cu_q[b], cu_q[b + 1], cu_k[b], cu_k[b + 1]
                    if fb.ctx_slots is not None:
                        ctx = lc[fb.ctx_slots[k0:k1].long()].float()
                    else:
                        ctx = row[q0:q1]
                    out[q0:q1] = self._attend(p, q[q0:q1], ctx, pos[q0:q1])
            h = h + out
            h = h + self._mlp(i, oracle.rmsnorm(h, w[p + "post_norm"], c.rms_norm_eps))
        if return_hidden:
            return h
        hn = oracle.rmsnorm(h, w["final_norm"], c.rms_norm_eps)
        if fb.logits_idx is not None:
            hn = hn[fb.logits_idx.long()]
        return hn @ w["lm_head"].t()


def greedy_sample(logits: torch.Tensor) -> torch.Tensor:
    return logits.float().argmax(-1).to(torch.int32)
