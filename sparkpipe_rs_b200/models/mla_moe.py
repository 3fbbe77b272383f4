"""MLA-MoE decoder running on the package's sm_100a kernels.

Decode uses the absorbed MLA form (queries projected into the 512-d latent
space, attention directly over the paged latent cache); prefill uses the
expanded form (k_nope / v re-materialised from the latent by w_kv_b) with a
flash-attention kernel, and writes the latent cache on the way.

Every GEMM-shaped op goes through the tcgen05 kernel (``ops.linear`` /
``ops.batched_gemm`` / ``ops.grouped_gemm``); the remaining ops are the
package's own kernels. The whole decode step is static-shape and stream
ordered, so ``DecodeGraph`` captures it into one CUDA graph per batch size.

The reference executes the same phases inside its (absent) resident decode
stage firmware: ATTENTION_NORM -> ATTENTION_PROJECTION -> ROPE_KV_WRITE ->
MLA_ATTENTION -> OUTPUT_PROJECTION -> POST_ATTENTION_NORM -> LOCAL_MOE ->
RESTRICTED_LOGITS (crates/spark-abi/vendor/sparkpipe/include/sparkpipe/spark_resident_decode_stage.h:445-460).
"""
from __future__ import annotations

import os

from dataclasses import dataclass

import torch

from .. import ops
from .config import MLAMoEConfig
from .rope import cos_sin_table
from .weights import absorb_decode_weights, derive_decode_weights, init_weights


@dataclass
class ForwardBatch:
    """Device-side inputs of one forward pass (all int32 tensors on the model device)."""

    mode: str                       # "prefill" | "decode"
    token_ids: torch.Tensor         # [T]
    positions: torch.Tensor         # [T]
    slot_mapping: torch.Tensor      # [T] cache row of each token (-1 = do not store)
    # decode
    block_table: torch.Tensor | None = None   # [B, max_blocks]
    context_lens: torch.Tensor | None = None  # [B] (including the current token)
    decode_splits: int = 1
    # decode: row b's own token (its last context token) is read from cache row
    # self_slots[b] rather than its block-table position; a tree verify's alternate
    # leaves write their KV to shadow rows (None: every row reads its block table)
    self_slots: torch.Tensor | None = None
    # prefill
    cu_q: torch.Tensor | None = None          # [B + 1]
    cu_k: torch.Tensor | None = None          # [B + 1]
    max_q: int = 0
    ctx_slots: torch.Tensor | None = None     # [Tk] cache rows of every context token (prefix + chunk)
    logits_idx: torch.Tensor | None = None    # rows to compute logits for (None = all)


class PhaseClock:
    """Device phase clocks of the forward pass (off unless attached to a model).

    Slots: 0 step start, 1 embedding, 2 attention (input norm, projections, KV
    write, MLA, output projection; summed over layers), 3 MLP / MoE (post-attention
    norm, router, experts, combine; summed over layers), 4 final norm + LM head.
    Each mark is one single-thread kernel reading the device global timer, so the
    totals are device time without a profiler, and they survive CUDA-graph replay.
    With ``nvtx`` the host also emits NVTX ranges per layer.
    """

    NAMES = ("start", "embedding", "attention", "mlp_moe", "lm_head")

    def __init__(self, device, nvtx: bool = False):
        self.stamps = torch.zeros(16, dtype=torch.int64, device=device)
        self.totals = torch.zeros(16, dtype=torch.int64, device=device)
        self.nvtx = nvtx

    def mark(self, slot: int, prev: int = -1):
        ops.kernels().phase_mark(self.stamps, self.totals, slot, prev)
        ops._count(1)

    def reset(self):
        self.totals.zero_()

    def report(self, steps: int = 1) -> dict:
        t = self.totals.cpu().tolist()
        return {self.NAMES[i]: t[i] / 1000.0 / max(1, steps) for i in range(1, len(self.NAMES))}  # us per step


class KVCache:
    """Paged latent KV cache: [layers, num_blocks * block_size, kv_lora + rope] bf16, or
    with ``kv_dtype="fp8"`` e4m3 rows (uint8) plus fp32 block scales [layers, slots, 5]
    (amax / 448 of each 128-element block of the row; block 4 is the 64 rope dims),
    written by the KV-write kernels and read by the fp8 decode kernel and ``kv8_gather``."""

    def __init__(self, cfg: MLAMoEConfig, num_blocks: int, block_size: int = 64, device="cuda",
                 layers: int | None = None, dtype: torch.dtype | None = None, kv_dtype: str = "bf16"):
        self.block_size = block_size
        self.num_blocks = num_blocks
        self.num_layers = layers if layers is not None else cfg.num_layers
        dev = torch.device(device)
        self.fp8 = kv_dtype == "fp8"
        slots = num_blocks * block_size
        self.scales = None
        if self.fp8:
            if dev.type != "cuda" or cfg.kv_cache_dim != 576 or block_size != 64:
                raise ValueError("the fp8 KV cache needs a CUDA device, 576-wide rows and 64-token blocks")
            self.data = torch.zeros(self.num_layers, slots, cfg.kv_cache_dim, dtype=torch.uint8, device=dev)
            self.scales = torch.zeros(self.num_layers, slots, 5, dtype=torch.float32, device=dev)
            return
        if kv_dtype not in ("bf16", "auto"):
            raise ValueError(f"kv_dtype must be bf16 or fp8, not {kv_dtype!r}")
        if dtype is None:
            dtype = torch.bfloat16 if dev.type == "cuda" else torch.float32
        self.data = torch.zeros(self.num_layers, slots, cfg.kv_cache_dim, dtype=dtype, device=dev)

    def layer(self, i: int) -> torch.Tensor:
        return self.data[i]

    def layer_scales(self, i: int) -> torch.Tensor | None:
        return None if self.scales is None else self.scales[i]

    def planes(self) -> list[torch.Tensor]:
        """The cache's arrays as [layers, slots, row] tensors of 2-byte units (bf16 views
        of the fp8 rows and their scales) for block copies; the CPU cache as it is."""
        if self.fp8:
            return [self.data.view(torch.bfloat16), self.scales.view(torch.bfloat16)]
        return [self.data]

    def dequantized(self, i: int) -> torch.Tensor:
        """Layer i's rows as fp32 (the stored values; fp8 rows times their block scales)."""
        if not self.fp8:
            return self.data[i].float()
        v = self.data[i].view(torch.float8_e4m3fn).float()
        return v * self.scales[i].repeat_interleave(128, dim=1)[:, :576]

    @property
    def bytes(self) -> int:
        b = self.data.numel() * self.data.element_size()
        return b + (self.scales.numel() * 4 if self.scales is not None else 0)


# SPARKPIPE_FUSED_ROUTER=1 computes a small router's logits inside the top-k kernel
# (each token's CTA reads the gate from L2) for decode batches. Off by default: on
# the V2-Lite shape (64 tokens, 64 x 2048 gate) it measured 7.33 ms per step against
# 7.28 ms with the split-K gate GEMM feeding the top-k kernel.
ROUTER_FUSED_MAX_TOKENS = 256 if os.environ.get("SPARKPIPE_FUSED_ROUTER", "0") == "1" else 0
# Expert groups averaging at least this many rows (prefill chunks) run the token-major
# grouped GEMM (tokens as M, row-major output, SwiGLU paired in registers);
# SPARKPIPE_MOE_TOKEN_MAJOR=0 keeps the weight-major (swap-AB) one everywhere.
MOE_TOKEN_MAJOR_MIN_ROWS = 256 if os.environ.get("SPARKPIPE_MOE_TOKEN_MAJOR", "1") != "0" else 1 << 62
# Decode-sized local MoE runs the shared experts on a forked stream, overlapping the
# routing kernels; SPARKPIPE_SHARED_SIDE_STREAM=0 keeps them as extra groups of the
# routed grouped GEMMs.
SHARED_SIDE_STREAM = os.environ.get("SPARKPIPE_SHARED_SIDE_STREAM", "1") != "0"
ROUTER_FUSED_MAX_WEIGHTS = 1 << 20


def _moe_block_n(rows: int, experts: int) -> int:
    avg = rows / max(1, experts)
    for bn in (16, 32, 64, 128):
        if avg <= bn * 0.75:
            return bn
    return 256


class MLAMoEModel:
    def __init__(self, cfg: MLAMoEConfig, weights: dict[str, torch.Tensor] | None = None, device="cuda",
                 seed: int = 0, max_positions: int | None = None, ep=None):
        """``ep``: an ``ExpertParallel`` rank; the model then holds only that
        rank's routed experts (plus the shared ones) and runs its MoE layers
        through the peer-memory expert all-to-all."""
        self.cfg = cfg
        self.device = torch.device(device)
        self.ep = ep
        if weights is None:
            weights = init_weights(cfg, seed=seed, device=self.device, dtype=torch.bfloat16,
                                   experts=ep.local_expert_range() if ep is not None else None)
        self.w = {k: (v if isinstance(v, ops.Fp8Weight) else v.to(self.device)) for k, v in weights.items()}
        del weights  # the re-laid-out expert weights below must not coexist with a second reference
        derive_decode_weights(cfg, self.w)
        # latent up-projections folded into the decode projections (SPARKPIPE_ABSORB=0: the four-GEMM form)
        self.absorbed = os.environ.get("SPARKPIPE_ABSORB", "1") != "0" and absorb_decode_weights(cfg, self.w)
        self._side = None           # forked stream of the shared experts (decode MoE)
        self._shared_tables = {}    # (T, bn) -> shared experts' row / tile prefix tables
        # routed + shared expert gate/up weights in the fused-SwiGLU tile order
        self.fused_swiglu = cfg.moe_intermediate_size % 64 == 0
        for i in range(cfg.num_layers):
            k = f"l{i}.e_w13"
            if k in self.w and self.fused_swiglu:
                v = self.w.pop(k)
                self.w[k] = ops.interleave_gate_up_fp8(v) if isinstance(v, ops.Fp8Weight) else ops.interleave_gate_up(v)
                del v
        maxp = max_positions or min(cfg.max_position_embeddings, 1 << 17)
        self.cos_sin = cos_sin_table(cfg, maxp, device=self.device)
        self.scale = cfg.softmax_scale()
        self.qa_dim = cfg.q_lora_rank or cfg.q_out_dim
        self._layer_offset = 0
        self.phase_clock: PhaseClock | None = None

    # ------------------------------------------------------------------ pieces
    def _lin(self, x: torch.Tensor, w, slab: bool = False, out_dtype=torch.bfloat16):
        """x @ w.T for a bf16 or block-scaled fp8 weight; with ``slab`` a decode-shaped
        result may stay split-K fp32 slabs (``ops.Slabs``) for a slab-aware consumer."""
        if isinstance(w, ops.Fp8Weight):
            return ops.linear_fp8(ops.quant_act_fp8(x), w, out_dtype=out_dtype, slab_out=slab)
        if slab:
            return ops.linear_slabs(x, w, out_dtype=out_dtype)
        return ops.linear(x, w, out_dtype=out_dtype)

    def _q_view(self, q2d: torch.Tensor, T: int) -> torch.Tensor:
        c = self.cfg
        return torch.as_strided(q2d, (T, c.num_heads, c.qk_head_dim), (q2d.stride(0), c.qk_head_dim, 1))

    def _project(self, i: int, xn: torch.Tensor):
        c, w = self.cfg, self.w
        p = f"l{i}."
        a = self._lin(xn, w[p + "w_qkv_a"])
        if c.q_lora_rank:
            qa = torch.empty(xn.shape[0], c.q_lora_rank, dtype=torch.bfloat16, device=self.device)
            ops.add_rmsnorm(a[:, : c.q_lora_rank], None, w[p + "q_a_norm"], qa, c.rms_norm_eps)
            q = self._lin(qa, w[p + "w_q_b"])
        else:
            q = a[:, : self.qa_dim]
        kv_a = a[:, self.qa_dim:]
        return q, kv_a

    def _attn_decode(self, i: int, xn: torch.Tensor, fb: ForwardBatch, cache: KVCache):
        """Absorbed-MLA decode attention; returns the o_proj result as ``ops.Slabs`` or a tensor."""
        c, w = self.cfg, self.w
        p = f"l{i}."
        T = xn.shape[0]
        nh, dn, dv, kvl = c.num_heads, c.qk_nope_head_dim, c.v_head_dim, c.kv_lora_rank
        layer_cache = cache.layer(i - self._layer_offset)
        kv_scales = cache.layer_scales(i - self._layer_offset)
        q_lat = torch.empty(T, nh, c.kv_cache_dim, dtype=torch.bfloat16, device=self.device)
        if c.q_lora_rank:
            q, kv_a = self._project(i, xn)
            ops.mla_kv_write(kv_a, w[p + "kv_a_norm"], fb.positions, self.cos_sin, fb.slot_mapping, layer_cache,
                             None, kvl, c.qk_rope_head_dim, c.rms_norm_eps, kv_scales)
            ops.rope_q(self._q_view(q, T), dn, q_lat, kvl, fb.positions, self.cos_sin, c.qk_rope_head_dim)
            q_src, q_batch_k = q, c.qk_head_dim
        elif self.absorbed:
            # absorbed form: the projection yields q_lat (latent + rope per head) and
            # kv_a; one kernel sums its split-K slabs, writes q_lat with query RoPE and
            # normalises / ropes / caches the latent KV
            qkv = self._lin(xn, w[p + "w_qkv_abs"], slab=True)
            ops.mla_decode_prep(qkv, w[p + "kv_a_norm"], fb.positions, self.cos_sin, fb.slot_mapping, layer_cache,
                                None, q_lat, kvl, 0, nh * c.kv_cache_dim, c.rms_norm_eps, kv_scales)
            o_lat = torch.empty(T, nh, kvl, dtype=torch.bfloat16, device=self.device)
            ops.mla_decode(q_lat, layer_cache, fb.block_table, fb.context_lens, o_lat, fb.decode_splits, self.scale,
                           last_slot=fb.self_slots, kv_scales=kv_scales)
            return self._lin(o_lat.view(T, nh * kvl), w[p + "w_ov"], slab=True)
        else:
            # one kernel: split-K reduction of the q/kv projection, latent norm + RoPE
            # + cache write, query RoPE and the compact q_nope operand
            qkv = self._lin(xn, w[p + "w_qkv_a"], slab=True)
            q_src = torch.empty(T, nh * dn, dtype=torch.bfloat16, device=self.device)
            ops.mla_decode_prep(qkv, w[p + "kv_a_norm"], fb.positions, self.cos_sin, fb.slot_mapping, layer_cache,
                                q_src, q_lat, dn, 0, self.qa_dim, c.rms_norm_eps, kv_scales)
            q_batch_k = dn
        # q_lat[t, h, :kvl] = q_nope[t, h] @ W_UK[h]
        ops.batched_gemm(w[p + "w_uk_t"], q_src, q_lat.view(T, nh * c.kv_cache_dim), M=kvl, N=T, K=dn, batch=nh,
                         a_batch_rows=kvl, b_k0=0, b_batch_k=q_batch_k, ldd=nh * c.kv_cache_dim,
                         d_batch_stride=c.kv_cache_dim)
        o_lat = torch.empty(T, nh, kvl, dtype=torch.bfloat16, device=self.device)
        ops.mla_decode(q_lat, layer_cache, fb.block_table, fb.context_lens, o_lat, fb.decode_splits, self.scale,
                       last_slot=fb.self_slots, kv_scales=kv_scales)
        attn = torch.empty(T, nh * dv, dtype=torch.bfloat16, device=self.device)
        # attn[t, h*dv + v] = o_lat[t, h] @ W_UV[h]^T
        ops.batched_gemm(w[p + "w_kv_b"], o_lat.view(T, nh * kvl), attn, M=dv, N=T, K=kvl, batch=nh, a_row0=dn,
                         a_batch_rows=dn + dv, b_batch_k=kvl, ldd=nh * dv, d_batch_stride=dv)
        return self._lin(attn, w[p + "w_o"], slab=True)

    def _attn_prefill(self, i: int, xn: torch.Tensor, fb: ForwardBatch, cache: KVCache) -> torch.Tensor:
        c, w = self.cfg, self.w
        p = f"l{i}."
        T = xn.shape[0]
        nh, dn, dv, kvl, dr = c.num_heads, c.qk_nope_head_dim, c.v_head_dim, c.kv_lora_rank, c.qk_rope_head_dim
        q, kv_a = self._project(i, xn)
        layer_cache = cache.layer(i - self._layer_offset)
        kv_scales = cache.layer_scales(i - self._layer_offset)
        lat = torch.empty(T, c.kv_cache_dim, dtype=torch.bfloat16, device=self.device)
        ops.mla_kv_write(kv_a, w[p + "kv_a_norm"], fb.positions, self.cos_sin, fb.slot_mapping, layer_cache, lat,
                         kvl, dr, c.rms_norm_eps, kv_scales)
        if fb.ctx_slots is None:
            lat_ctx = lat
        elif kv_scales is not None:  # earlier chunks / cached prefix: dequantised fp8 rows
            lat_ctx = ops.kv8_gather(layer_cache, kv_scales, fb.ctx_slots)
        else:
            lat_ctx = ops.gather_rows(layer_cache, fb.ctx_slots)
        Tk = lat_ctx.shape[0]
        kv = ops.linear(lat_ctx[:, :kvl], w[p + "w_kv_b"])              # [Tk, nh*(dn+dv)]
        q3 = self._q_view(q, T)
        ops.rope_q(q3, dn, q3, dn, fb.positions, self.cos_sin, dr)
        kv3 = kv.view(Tk, nh, dn + dv)
        o = torch.empty(T, nh, dv, dtype=torch.bfloat16, device=self.device)
        ops.prefill_attention(q3, kv3[:, :, :dn], lat_ctx[:, kvl:], kv3[:, :, dn:], o, fb.cu_q, fb.cu_k, fb.max_q,
                              self.scale, True)
        return self._lin(o.view(T, nh * dv), w[p + "w_o"])

    def _mlp(self, i: int, xn: torch.Tensor) -> torch.Tensor:
        c, w = self.cfg, self.w
        p = f"l{i}."
        if not c.is_moe_layer(i):
            return self._lin(ops.silu_mul(self._lin(xn, w[p + "w13"])), w[p + "w2"])
        T = xn.shape[0]
        E, k, F, S = c.n_routed_experts, c.num_experts_per_tok, c.moe_intermediate_size, c.n_shared_experts
        sigmoid = c.scoring_func == "sigmoid"
        route = dict(n_shared=S, n_group=c.n_group, topk_group=c.topk_group, group_top2=c.topk_method == "noaux_tc")
        bias = w[p + "gate_bias"] if sigmoid else None
        gate = w[p + "gate"]
        if T <= ROUTER_FUSED_MAX_TOKENS and gate.numel() <= ROUTER_FUSED_MAX_WEIGHTS and gate.shape[1] <= 2048:
            # small router at decode size: logits inside the top-k kernel, no gate GEMM
            ids, wts = ops.moe_route(xn, gate, bias, k, 1 if sigmoid else 0, c.norm_topk_prob,
                                     c.routed_scaling_factor, **route)
        else:
            logits = ops.linear_slabs(xn, gate, out_dtype=torch.float32)
            if (SHARED_SIDE_STREAM and S and self.ep is None and self.fused_swiglu
                    and not isinstance(w[p + "e_w13"], ops.Fp8Weight)
                    and T * (k + S) < MOE_TOKEN_MAJOR_MIN_ROWS * (E + S)):
                return self._moe_shared_apart(i, xn, logits, bias, sigmoid, route)
            ids, wts = ops.moe_topk(logits, bias, k, 1 if sigmoid else 0, c.norm_topk_prob, c.routed_scaling_factor,
                                    **route)
        kk = k + S
        if self.ep is not None:
            bn = _moe_block_n(T * kk, self.ep.n_local)
            if isinstance(w[p + "e_w13"], ops.Fp8Weight):
                bn = max(32, min(bn, 128))
            # prefill-sized groups (a rank receives ~T * k / n_local rows per local expert)
            tm = (self.fused_swiglu and not isinstance(w[p + "e_w13"], ops.Fp8Weight)
                  and T * k >= MOE_TOKEN_MAJOR_MIN_ROWS * self.ep.n_local)
            return self.ep.moe(i, xn, ids, wts, w[p + "e_w13"], w[p + "e_w2"], bn, self.fused_swiglu, token_major=tm)
        if (T * kk >= MOE_TOKEN_MAJOR_MIN_ROWS * (E + S) and self.fused_swiglu
                and not isinstance(w[p + "e_w13"], ops.Fp8Weight)):
            grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E + S, 128)
            xs = ops.gather_rows(xn, sorted_tok)
            act = torch.empty(T * kk, F, dtype=torch.bfloat16, device=self.device)
            ops.grouped_gemm_tm(w[p + "e_w13"], xs, act, grp_rows, grp_tiles, E + S, swiglu=True)
            y = torch.empty(T * kk, c.hidden_size, dtype=torch.bfloat16, device=self.device)
            ops.grouped_gemm_tm(w[p + "e_w2"], act, y, grp_rows, grp_tiles, E + S)
            return ("combine", y, inv_pos, wts, kk)
        bn = _moe_block_n(T * kk, E + S)
        if isinstance(w[p + "e_w13"], ops.Fp8Weight):
            bn = max(32, min(bn, 128))
            grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E + S, bn)
            xq = ops.quant_act_fp8(xn, sorted_tok)  # gather into the expert-sorted order while quantising
            act = torch.empty(T * kk, F, dtype=torch.bfloat16, device=self.device)
            ops.grouped_gemm_fp8(w[p + "e_w13"], xq, act, grp_rows, grp_tiles, E + S, bn, swiglu=True)
            y = torch.empty(T * kk, c.hidden_size, dtype=torch.bfloat16, device=self.device)
            ops.grouped_gemm_fp8(w[p + "e_w2"], ops.quant_act_fp8(act), y, grp_rows, grp_tiles, E + S, bn)
            return ("combine", y, inv_pos, wts, kk)
        grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E + S, bn)
        return self._moe_grouped(i, xn, wts, grp_rows, grp_tiles, sorted_tok, inv_pos)

    def _shared_layout(self, T: int, bn: int):
        """Row / tile prefix tables of the shared experts taking all T tokens each
        (cached per (T, bn); first built in a step's eager warm-up, outside capture)."""
        key = (T, bn)
        if key not in self._shared_tables:
            S = self.cfg.n_shared_experts
            nt = -(-T // bn)
            rows = torch.tensor([s * T for s in range(S + 1)], dtype=torch.int32, device=self.device)
            tiles = torch.tensor([s * nt for s in range(S + 1)], dtype=torch.int32, device=self.device)
            self._shared_tables[key] = (rows, tiles)
        return self._shared_tables[key]

    def _moe_shared_apart(self, i, xn, logits, bias, sigmoid, route):
        """Decode-sized local MoE with the shared experts on a forked stream: their two
        GEMMs (which need only xn) stream their weights while the main stream routes the
        tokens and builds the expert-sorted layout; the routed grouped GEMMs cover the E
        routed experts and the combine adds the shared rows."""
        c, w = self.cfg, self.w
        p = f"l{i}."
        T = xn.shape[0]
        E, k, F, S = c.n_routed_experts, c.num_experts_per_tok, c.moe_intermediate_size, c.n_shared_experts
        main = torch.cuda.current_stream(self.device)
        if self._side is None:
            self._side = torch.cuda.Stream(device=self.device)
        side = self._side
        fork = torch.cuda.Event()
        fork.record(main)
        side.wait_event(fork)
        bn_s = _moe_block_n(T * S, S)
        rows_s, tiles_s = self._shared_layout(T, bn_s)  # static tables, built in the eager warm-up
        # buffers come from the main stream's pool: the main stream waits for the fork's
        # end before any of them is used or freed there
        xs_s = xn if S == 1 else torch.empty(S * T, xn.shape[1], dtype=xn.dtype, device=self.device)
        act_s = torch.empty(S * T, F, dtype=torch.bfloat16, device=self.device)
        y_s = torch.empty(S * T, c.hidden_size, dtype=torch.bfloat16, device=self.device)
        w13, w2 = w[p + "e_w13"], w[p + "e_w2"]
        w13_s = w13[E:E + S] if w13.dim() == 3 else w13[E * (w13.shape[0] // (E + S)):]
        w2_s = w2[E:E + S] if w2.dim() == 3 else w2[E * (w2.shape[0] // (E + S)):]
        with torch.cuda.stream(side):
            for q in range(S if S > 1 else 0):
                xs_s[q * T:(q + 1) * T].copy_(xn)
            ops.grouped_gemm(w13_s, xs_s, act_s, rows_s, tiles_s, S, bn_s, swiglu=True, sched_early=True)
            ops.grouped_gemm(w2_s, act_s, y_s, rows_s, tiles_s, S, bn_s, sched_early=True)
            join = torch.cuda.Event()
            join.record(side)
        route = dict(route, n_shared=0)
        ids, wts = ops.moe_topk(logits, bias, k, 1 if sigmoid else 0, c.norm_topk_prob, c.routed_scaling_factor,
                                **route)
        bn = _moe_block_n(T * k, E)
        grp_rows, grp_tiles, sorted_tok, inv_pos = ops.moe_align(ids, E, bn)
        xs = ops.gather_rows(xn, sorted_tok)
        act = torch.empty(T * k, F, dtype=torch.bfloat16, device=self.device)
        ops.grouped_gemm(w[p + "e_w13"], xs, act, grp_rows, grp_tiles, E, bn, swiglu=True, sched_early=True)
        y = torch.empty(T * k, c.hidden_size, dtype=torch.bfloat16, device=self.device)
        ops.grouped_gemm(w[p + "e_w2"], act, y, grp_rows, grp_tiles, E, bn, sched_early=True)
        return ("combine", y, inv_pos, wts, k, y_s, join)

    def _moe_grouped(self, i, xn, wts, grp_rows, grp_tiles, sorted_tok, inv_pos):
        """Weight-major grouped expert GEMMs over the expert-sorted rows; returns the
        deferred weighted combine."""
        c, w = self.cfg, self.w
        p = f"l{i}."
        T = xn.shape[0]
        E, k, F, S = c.n_routed_experts, c.num_experts_per_tok, c.moe_intermediate_size, c.n_shared_experts
        kk = k + S
        bn = _moe_block_n(T * kk, E + S)
        # align -> gather -> w13 -> w2: the schedule is two or more launches old at each
        # expert GEMM, which may then stream weights before its dependency wait
        xs = ops.gather_rows(xn, sorted_tok)
        if self.fused_swiglu:
            act = torch.empty(T * kk, F, dtype=torch.bfloat16, device=self.device)
            ops.grouped_gemm(w[p + "e_w13"], xs, act, grp_rows, grp_tiles, E + S, bn, swiglu=True, sched_early=True)
        else:
            h13 = torch.empty(T * kk, 2 * F, dtype=torch.bfloat16, device=self.device)
            ops.grouped_gemm(w[p + "e_w13"], xs, h13, grp_rows, grp_tiles, E + S, bn, sched_early=True)
            act = ops.silu_mul(h13)
        y = torch.empty(T * kk, c.hidden_size, dtype=torch.bfloat16, device=self.device)
        ops.grouped_gemm(w[p + "e_w2"], act, y, grp_rows, grp_tiles, E + S, bn, sched_early=True)
        # the weighted combine is fused into the next residual add + RMSNorm
        return ("combine", y, inv_pos, wts, kk)

    def _residual_norm(self, pending, res: torch.Tensor, gamma: torch.Tensor, xn: torch.Tensor):
        """res += pending (if any); xn = rmsnorm(res) * gamma. `pending` is None, a
        bf16 tensor, split-K ``ops.Slabs`` or a deferred MoE combine."""
        eps = self.cfg.rms_norm_eps
        if pending is None:
            ops.add_rmsnorm(res, None, gamma, xn, eps)
        elif isinstance(pending, tuple) and pending[0] == "ep_combine":
            pending[1].combine_add_rmsnorm(pending[2], pending[3], res, gamma, xn, eps)
        elif isinstance(pending, tuple) and len(pending) == 7:  # shared experts from the forked stream
            _, y, inv_pos, wts, kk, y_s, join = pending
            torch.cuda.current_stream(self.device).wait_event(join)
            ops.combine_add_rmsnorm(y, inv_pos, wts, res, gamma, xn, kk, eps, shared=y_s)
        elif isinstance(pending, tuple):
            _, y, inv_pos, wts, kk = pending
            ops.combine_add_rmsnorm(y, inv_pos, wts, res, gamma, xn, kk, eps)
        else:
            ops.slab_add_rmsnorm(pending, res, gamma, xn, eps)

    def write_kv(self, fb: ForwardBatch, cache: KVCache):
        """Writes layer 0's latent KV of the rows of ``fb`` (token ids, positions, cache
        slots) and nothing else: embedding, input norm, the latent KV projection, its
        norm and RoPE. Layer 0's KV of a token depends only on the token and its
        position, so this keeps a one-layer draft model's cache current for tokens it
        did not decode itself (prompts, plainly decoded tokens, accepted tree drafts)."""
        c, w = self.cfg, self.w
        wt = w["l0.w_qkv_a"]
        if isinstance(wt, ops.Fp8Weight):
            raise ValueError("write_kv needs a bf16 latent projection")
        x = ops.embedding(w["embed"], fb.token_ids)
        xn = torch.empty_like(x)
        ops.add_rmsnorm(x, None, w["l0.in_norm"], xn, c.rms_norm_eps)
        kv_a = ops.linear(xn, wt[self.qa_dim:])
        ops.mla_kv_write(kv_a, w["l0.kv_a_norm"], fb.positions, self.cos_sin, fb.slot_mapping, cache.layer(0), None,
                         c.kv_lora_rank, c.qk_rope_head_dim, c.rms_norm_eps, cache.layer_scales(0))

    # ------------------------------------------------------------------ forward
    def forward(self, fb: ForwardBatch, cache: KVCache, layers: range | None = None,
                hidden_in: torch.Tensor | None = None, return_hidden: bool = False, layer_offset: int = 0):
        """Runs `layers` (default: all) and returns logits [n, V] (bf16) of the rows in
        fb.logits_idx, or the residual stream when return_hidden (pipeline stages).
        Model layer i uses cache layer i - layer_offset (a stage caches only its layers)."""
        self._layer_offset = layer_offset
        c, w = self.cfg, self.w
        T = fb.token_ids.shape[0]
        layers = layers if layers is not None else range(c.num_layers)
        eps = c.rms_norm_eps
        pc = self.phase_clock
        if pc is not None:
            pc.mark(0)
        if hidden_in is None:
            res = ops.embedding(w["embed"], fb.token_ids)
        else:
            res = hidden_in.clone()
        xn = torch.empty_like(res)
        pending = None
        if pc is not None:
            pc.mark(1, 0)
        prev = 1
        for i in layers:
            p = f"l{i}."
            if pc is not None and pc.nvtx:
                torch.cuda.nvtx.range_push(f"layer {i}")
            self._residual_norm(pending, res, w[p + "in_norm"], xn)
            if fb.mode == "decode":
                o = self._attn_decode(i, xn, fb, cache)
            else:
                o = self._attn_prefill(i, xn, fb, cache)
            if pc is not None:
                pc.mark(2, prev)
            self._residual_norm(o, res, w[p + "post_norm"], xn)
            pending = self._mlp(i, xn)
            if pc is not None:
                pc.mark(3, 2)
                prev = 3
                if pc.nvtx:
                    torch.cuda.nvtx.range_pop()
        if return_hidden:
            if pending is not None:
                self._residual_norm(pending, res, w["final_norm"], xn)
            if self.ep is not None:
                self.ep.end_step()
            return res
        self._residual_norm(pending, res, w["final_norm"], xn)
        if self.ep is not None:
            self.ep.end_step()
        sel = xn if fb.logits_idx is None else ops.gather_rows(xn, fb.logits_idx)
        logits = ops.linear(sel, w["lm_head"])
        if pc is not None:
            pc.mark(4, prev)
        return logits


class DecodeGraph:
    """One CUDA graph of a full decode step (forward + sampling) for a fixed batch
    size. Inputs are copied into static device buffers before replay; sampling reads
    a per-row temperature and noise key (``temps`` / ``keys``, zero = greedy), so one
    graph serves greedy and sampled requests in the same batch."""

    def __init__(self, model: MLAMoEModel, cache: KVCache, batch: int, max_blocks: int, max_context: int,
                 use_graph: bool = True, self_advance: bool = False, extra=None):
        """``extra(fb)``: more device work of the step, captured into the same graph
        (the serving engine keeps a draft model's KV current with it)."""
        self.model, self.cache, self.B = model, cache, batch
        self.extra = extra
        dev = model.device
        self.ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.slots = torch.full((batch,), -1, dtype=torch.int32, device=dev)
        self.block_table = torch.zeros(batch, max_blocks, dtype=torch.int32, device=dev)
        self.ctx = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.out_ids = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.temps = torch.zeros(batch, dtype=torch.float32, device=dev)
        self.keys = torch.zeros(batch, dtype=torch.int64, device=dev)
        self.sampling_dirty = False  # temps / keys hold a sampled batch's values
        self.self_advance = self_advance
        self.step_offset = torch.zeros(1, dtype=torch.int64)
        heads = model.cfg.num_heads
        self.fb = ForwardBatch(mode="decode", token_ids=self.ids, positions=self.pos, slot_mapping=self.slots,
                               block_table=self.block_table, context_lens=self.ctx,
                               decode_splits=ops.mla_decode_splits(batch, heads, max_context, ops.kernels().num_sms(),
                                                                   kv_fp8=cache.fp8))
        self.graph = None
        self.use_graph = use_graph
        self._run_eager()  # warm-up (also sets kernel attributes outside capture)
        torch.cuda.synchronize()
        if use_graph:
            self.graph = torch.cuda.CUDAGraph()
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                with torch.cuda.graph(self.graph, stream=s):
                    self._step()
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()

    def _step(self):
        logits = self.model.forward(self.fb, self.cache)
        ops.sample_tokens(logits, out_ids=self.out_ids, row_temp=self.temps, row_key=self.keys)
        if self.extra is not None:
            self.extra(self.fb)
        if self.self_advance:
            ops.decode_advance(self.out_ids, self.ids, self.pos, self.ctx, self.slots, self.block_table,
                               self.cache.block_size)

    def _run_eager(self):
        self._step()

    def run(self):
        if self.graph is not None:
            self.graph.replay()
        else:
            self._run_eager()
        return self.out_ids

    def release(self):
        self.graph = None
