"""Python entry points of the sm_100a kernels.

Every function here launches one of the package's own CUDA kernels on the
current stream; none falls back to a PyTorch implementation. On a machine
without the compiled extension or without a CUDA device they raise.
"""
from __future__ import annotations

import math
import os

import torch

from .. import _ext

__all__ = [
    "kernels",
    "linear",
    "gemm",
    "batched_gemm",
    "grouped_gemm",
    "interleave_gate_up",
    "add_rmsnorm",
    "mla_kv_write",
    "rope_q",
    "quant_fp8_block",
    "Fp8Weight",
    "Fp8Act",
    "quant_weight_fp8",
    "quant_act_fp8",
    "linear_fp8",
    "grouped_gemm_fp8",
    "interleave_gate_up_fp8",
    "mla_decode",
    "mla_decode_splits",
    "kv8_gather",
    "prefill_attention",
    "moe_topk",
    "moe_align",
    "gather_rows",
    "silu_mul",
    "moe_combine",
    "embedding",
    "sample_tokens",
    "spec_verify",
    "decode_advance",
    "linear_slabs",
    "Slabs",
    "slab_add_rmsnorm",
    "mla_decode_prep",
    "combine_add_rmsnorm",
    "status_word",
    "clear_status",
    "SWAP_AB_MAX_TOKENS",
    "launch_count",
]

# Up to this many tokens a linear layer runs "swap-AB": the weight fills the
# 128-row MMA tile and the tokens become the N dimension (decode shapes).
SWAP_AB_MAX_TOKENS = 256

_K = None

# Number of this package's kernels launched so far (host-side count of launches
# issued through this module; a CUDA-graph replay re-runs the captured ones).
LAUNCHES = [0]


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


def launch_count() -> int:
    return LAUNCHES[0]


def kernels():
    global _K
    if _K is None:
        _K = _ext.kernels()
    return _K


def _rows_cols_ld(t: torch.Tensor):
    assert t.dim() == 2 and t.stride(1) == 1, "operand must be a 2-D row-major view"
    return t.size(0), t.size(1), t.stride(0)


def gemm(a: torch.Tensor, b: torch.Tensor, d: torch.Tensor, *, M: int, N: int, K: int, trans_out: bool = False,
         batch: int = 1, a_row0: int = 0, a_batch_rows: int = 0, a_k0: int = 0, a_batch_k: int = 0,
         b_row0: int = 0, b_batch_rows: int = 0, b_k0: int = 0, b_batch_k: int = 0, ldd: int | None = None,
         d_batch_stride: int = 0, splits: int = 0, block_n: int = 0, grp_rows=None, grp_tiles=None,
         num_groups: int = 0, a_evict_first: bool = False, swiglu: bool = False, slab_out: bool = False,
         ep_combine=None, sched_early: bool = False):
    """Raw tcgen05 GEMM: D[m, n] = sum_k A[m, k] B[n, k] (see gemm_tcgen05.cu).
    ``ep_combine`` = (EP argument vector, comb_dst, epoch, MoE layer) sends a grouped
    GEMM's output rows straight to their source ranks' combine slots (D unused).

    Returns D, or with ``slab_out`` and a split K, ``-splits``: the result then
    is the sum of `splits` fp32 slabs in the split workspace (dense, D's
    orientation), to be consumed by a slab-aware kernel."""
    ar, ac, lda = _rows_cols_ld(a)
    br, bc, ldb = _rows_cols_ld(b)
    if ldd is None:
        ldd = d.stride(0)
    ep_args, comb_dst, epoch, ep_layer = ep_combine if ep_combine is not None else ([], None, None, 0)
    r = kernels().gemm(a, b, d, ar, ac, lda, br, bc, ldb, ldd, d_batch_stride, M, N, K, batch, a_row0,
                       a_batch_rows, a_k0, a_batch_k, b_row0, b_batch_rows, b_k0, b_batch_k, int(trans_out),
                       splits, block_n, grp_rows, grp_tiles, num_groups, int(a_evict_first), int(swiglu),
                       int(slab_out), ep_args, comb_dst, epoch, ep_layer, int(sched_early))
    if r < 0:
        _count(1)
        return r
    _count(r)
    return d


_WS = {}


def split_workspace() -> torch.Tensor:
    """The device's split-K partial workspace (fp32, owned by the kernel library)."""
    dev = torch.cuda.current_device()
    if dev not in _WS:
        _WS[dev] = kernels().split_workspace()
    return _WS[dev]


class Slabs:
    """A linear layer's result left as `splits` fp32 slabs [rows, cols] in the split workspace."""

    def __init__(self, splits: int, rows: int, cols: int):
        self.splits, self.rows, self.cols = splits, rows, cols
        self.stride = rows * cols
        self.ws = split_workspace()


def linear_slabs(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, out_dtype=torch.bfloat16):
    """Decode-shaped y = x @ w.T that may leave its split-K partial sums for the
    consumer: returns ``Slabs`` (fused consumers sum them) or the output tensor."""
    T, K = x.shape
    O = w.shape[0]
    if out is None:
        out = torch.empty(T, O, dtype=out_dtype, device=x.device)
    if T > SWAP_AB_MAX_TOKENS:
        return linear(x, w, out=out)
    r = gemm(w, x, out, M=O, N=T, K=K, trans_out=True, a_evict_first=True, slab_out=True)
    if isinstance(r, int):
        return Slabs(-r, T, O)
    return out


def linear(x: torch.Tensor, w: torch.Tensor, out: torch.Tensor | None = None, out_dtype=torch.bfloat16,
           splits: int = 0) -> torch.Tensor:
    """y = x @ w.T for x [T, K] (row-major view) and w [O, K] (bf16)."""
    T, K = x.shape
    O = w.shape[0]
    if out is None:
        out = torch.empty(T, O, dtype=out_dtype, device=x.device)
    if T == 0:
        return out
    if T <= SWAP_AB_MAX_TOKENS:
        gemm(w, x, out, M=O, N=T, K=K, trans_out=True, splits=splits, a_evict_first=True)
    else:
        gemm(x, w, out, M=T, N=O, K=K, trans_out=False, splits=1)
    return out


def batched_gemm(a, b, d, *, M, N, K, batch, a_row0=0, a_batch_rows=0, a_k0=0, a_batch_k=0, b_row0=0,
                 b_batch_rows=0, b_k0=0, b_batch_k=0, ldd=None, d_batch_stride=0, trans_out=True):
    """Strided-batched GEMM, batch index z shifts A rows / K columns, B rows / K columns and D."""
    return gemm(a, b, d, M=M, N=N, K=K, trans_out=trans_out, batch=batch, a_row0=a_row0, a_batch_rows=a_batch_rows,
                a_k0=a_k0, a_batch_k=a_batch_k, b_row0=b_row0, b_batch_rows=b_batch_rows, b_k0=b_k0,
                b_batch_k=b_batch_k, ldd=ldd, d_batch_stride=d_batch_stride, splits=1)


def grouped_gemm(w: torch.Tensor, x_sorted: torch.Tensor, out: torch.Tensor, grp_rows: torch.Tensor,
                 grp_tiles: torch.Tensor, num_groups: int, block_n: int, swiglu: bool = False,
                 ep_combine=None, sched_early: bool = False) -> torch.Tensor:
    """MoE expert GEMM: out[r] = W[g(r)] @ x_sorted[r] for rows r sorted by group.

    w is [G, M, K] (or its [G*M, K] view), x_sorted [R, K], out [R, M]. With
    swiglu, w holds per 128-row tile 64 gate rows then the 64 matching up rows
    (see ``interleave_gate_up``) and out [R, M/2] receives silu(gate) * up.
    ``sched_early``: grp_rows / grp_tiles were written at least two launches before
    this one, so the kernel streams its first weight tiles before its dependency wait.
    """
    if w.dim() == 3:
        G, M, K = w.shape
        w2 = w.view(G * M, K)
    else:
        w2 = w
        M = w.shape[0] // num_groups
        K = w.shape[1]
    gemm(w2, x_sorted, out, M=M, N=x_sorted.shape[0], K=K, trans_out=True, a_batch_rows=M, block_n=block_n,
         grp_rows=grp_rows, grp_tiles=grp_tiles, num_groups=num_groups, a_evict_first=True, swiglu=swiglu,
         ep_combine=ep_combine, sched_early=sched_early and ep_combine is None and _SCHED_EARLY)
    return out


# SPARKPIPE_GROUPED_EARLY=0: grouped GEMMs read their tile schedule after the PDL wait only.
_SCHED_EARLY = os.environ.get("SPARKPIPE_GROUPED_EARLY", "1") != "0"


def grouped_gemm_tm(w: torch.Tensor, x_sorted: torch.Tensor, out: torch.Tensor, grp_rows: torch.Tensor,
                    grp_tiles: torch.Tensor, num_groups: int, swiglu: bool = False, block_n: int = 0) -> torch.Tensor:
    """Token-major MoE expert GEMM for prefill-size groups: out[r] = W[g(r)] @ x_sorted[r]
    with the tokens as the 128-row M tiles and the expert's weight rows as N, written as
    rows (``grp_tiles`` counts 128-row token tiles: ``moe_align(ids, groups, 128)``).
    ``w`` [G, N, K] (or [G*N, K]); with ``swiglu`` the weights are interleaved as for
    ``grouped_gemm`` and out [R, N/2] receives silu(gate) * up."""
    n = w.shape[1] if w.dim() == 3 else w.shape[0] // num_groups
    w2 = w.reshape(-1, w.shape[-1])
    if not block_n:
        block_n = 256 if n % 256 == 0 or not swiglu else 128
    _count(kernels().grouped_gemm_tm(x_sorted, w2, out, grp_rows, grp_tiles, int(num_groups), int(n), int(block_n),
                                     int(swiglu)))
    return out


def interleave_gate_up(w13: torch.Tensor) -> torch.Tensor:
    """[..., 2F, K] stacked [gate; up] -> per 128-row tile [64 gate rows; 64 up rows] (F % 64 == 0)."""
    *lead, two_f, K = w13.shape
    F = two_f // 2
    assert F % 64 == 0, "fused SwiGLU needs the FFN width to be a multiple of 64"
    v = w13.reshape(*lead, 2, F // 64, 64, K).transpose(-4, -3)
    return v.reshape(*lead, two_f, K).contiguous()


def interleave_gate_up_fp8(w13: Fp8Weight) -> Fp8Weight:
    """fp8 [..., 2F, K] [gate; up] in 128x128 blocks -> the fused-SwiGLU tile layout
    (per 128 rows: 64 gate rows, 64 up rows). A tile then mixes two source blocks,
    so the result carries one scale per 64 rows (sa_rows = 64)."""
    assert w13.sa_rows == 128
    *lead, two_f, K = w13.q.shape
    F = two_f // 2
    assert F % 64 == 0, "fused SwiGLU needs the FFN width to be a multiple of 64"
    q = interleave_gate_up(w13.q.view(torch.uint8)).view(torch.float8_e4m3fn)
    s64 = w13.s.repeat_interleave(2, -2)[..., : two_f // 64, :]  # one scale per 64 source rows
    s = interleave_gate_up(s64.unsqueeze(-2).expand(*s64.shape[:-1], 64, s64.shape[-1]).reshape(
        *lead, two_f, s64.shape[-1]))[..., ::64, :].contiguous()
    return Fp8Weight(q, s, 64)


def add_rmsnorm(x, residual, w, out, eps):
    kernels().add_rmsnorm(x, residual, w, out, float(eps))
    _count(1)
    return out


def mla_kv_write(kv, norm_w, positions, cos_sin, slot_mapping, cache, latent_out, kv_lora, rope, eps, kv_scales=None):
    """Latent RMSNorm + rope-key RoPE of kv rows into the paged cache (bf16, or fp8 e4m3
    with ``kv_scales`` [slots, 5]: one amax / 448 scale per 128 elements, block 4 the
    rope dims) and optionally into ``latent_out`` (bf16)."""
    kernels().mla_kv_write(kv, norm_w, positions, cos_sin, slot_mapping, cache, latent_out, kv_lora, rope, float(eps),
                           kv_scales)
    _count(1)


def rope_q(src, src_off, dst, dst_off, positions, cos_sin, rope):
    kernels().rope_q(src, src_off, dst, dst_off, positions, cos_sin, rope)
    _count(1)


def quant_fp8_block(x):
    q = torch.empty(x.shape, dtype=torch.float8_e4m3fn, device=x.device)
    s = torch.empty(x.shape[0], x.shape[1] // 128, dtype=torch.float32, device=x.device)
    kernels().quant_fp8_block(x, q, s)
    _count(1)
    return q, s


class Fp8Weight:
    """Block-scaled fp8 weight: e4m3 values ``q`` [..., rows, K] and fp32 scales ``s``
    [..., rows / sa_rows, K / 128], one per (sa_rows x 128) block (128: the 128x128
    block format)."""

    def __init__(self, q: torch.Tensor, s: torch.Tensor, sa_rows: int = 128):
        self.q, self.s, self.sa_rows = q, s, sa_rows

    @property
    def shape(self):
        return self.q.shape

    def dequant(self) -> torch.Tensor:
        """fp32 weights (oracle / tests)."""
        rep = self.s.repeat_interleave(self.sa_rows, -2)[..., : self.q.shape[-2], :].repeat_interleave(128, -1)
        return self.q.float() * rep[..., : self.q.shape[-1]]


class Fp8Act:
    """Quantised activations: e4m3 ``q`` [rows, K] and K-block-major scales ``s`` [K / 128, rows]."""

    def __init__(self, q: torch.Tensor, s: torch.Tensor):
        self.q, self.s = q, s

    @property
    def rows(self) -> int:
        return self.q.shape[0]


def quant_weight_fp8(rows: int, cols: int, *, src: torch.Tensor | None = None, seed: int = 0, std: float = 0.02,
                     flat0: int = 0, device=None, out: Fp8Weight | None = None) -> Fp8Weight:
    """128x128-block e4m3 weight from a bf16 tensor or from seeded N(0, std) samples
    (element (r, c) is sample flat0 + r * cols + c, so shards are reproducible).
    ``out`` receives the result in place (contiguous q [rows, cols] / s views)."""
    dev = src.device if src is not None else device
    if out is None:
        q = torch.empty(rows, cols, dtype=torch.float8_e4m3fn, device=dev)
        s = torch.empty((rows + 127) // 128, cols // 128, dtype=torch.float32, device=dev)
        out = Fp8Weight(q, s, 128)
    kernels().quant_weight_fp8(src.contiguous() if src is not None else None, int(seed), int(flat0), float(std),
                               out.q.view(rows, cols), out.s.view(-1, cols // 128))
    _count(1)
    return out


def quant_act_fp8(x: torch.Tensor, src_idx: torch.Tensor | None = None, idx_div: int = 1,
                  rows: int | None = None, rows_dev: torch.Tensor | None = None, out: Fp8Act | None = None) -> Fp8Act:
    """Per-(row, 128-column) e4m3 quantisation of bf16 activations; with ``src_idx``
    row r is x[src_idx[r] // idx_div] (the MoE expert-sorted layout). ``rows_dev``
    (int32 on the device) bounds the live rows when the count is only known there."""
    R = rows if rows is not None else (src_idx.numel() if src_idx is not None else x.shape[0])
    K = x.shape[1]
    if out is None:
        q = torch.empty(R, K, dtype=torch.float8_e4m3fn, device=x.device)
        s = torch.empty(K // 128, max(R, 1), dtype=torch.float32, device=x.device)
        out = Fp8Act(q, s)
    if R > 0:
        kernels().quant_act_fp8(x, src_idx, int(idx_div), rows_dev, out.q[:R], out.s)
        _count(1)
    return out


def linear_fp8(x: Fp8Act, w: Fp8Weight, out: torch.Tensor | None = None, out_dtype=torch.bfloat16,
               slab_out: bool = False, splits: int = 0):
    """y = x @ dequant(w).T with tcgen05 fp8 MMAs (weights as the A operand, output
    written transposed). With ``slab_out`` a split-K result is returned as ``Slabs``."""
    T, K = x.q.shape
    O = w.q.shape[0]
    if out is None:
        out = torch.empty(T, O, dtype=out_dtype, device=x.q.device)
    if T == 0:
        return out
    r = kernels().gemm_fp8(w.q, w.s, w.sa_rows, x.q, x.s, out, O, T, K, 1, splits, 0, None, None, 0, 0,
                           int(slab_out), [], None, None, 0)
    if r < 0:
        _count(1)
        return Slabs(-r, T, O)
    _count(r)
    return out


def grouped_gemm_fp8(w: Fp8Weight, x_sorted: Fp8Act, out: torch.Tensor, grp_rows: torch.Tensor,
                     grp_tiles: torch.Tensor, num_groups: int, block_n: int, swiglu: bool = False,
                     ep_combine=None) -> torch.Tensor:
    """MoE expert GEMM on fp8: out[r] = dequant(W[g(r)]) @ x_sorted[r] (rows sorted by
    group; weights [G, M, K] with scales [G, M / sa_rows, K / 128])."""
    G, M, K = w.q.shape
    A = w.q.reshape(G * M, K)
    sa = w.s.reshape(-1, w.s.shape[-1])
    ep_args, comb_dst, epoch, ep_layer = ep_combine if ep_combine is not None else ([], None, None, 0)
    kernels().gemm_fp8(A, sa, w.sa_rows, x_sorted.q, x_sorted.s, out, M, x_sorted.rows, K, 1, 1, block_n, grp_rows,
                       grp_tiles, num_groups, int(swiglu), 0, ep_args, comb_dst, epoch, ep_layer)
    _count(1)
    return out


MLA_IMPL = {"auto": 0, "tc": 1, "mma": 2, "sk": 3}  # MLA decode kernels: default, tcgen05, mma.sync, stream-K

# Decode kernel: "mma" (split-KV mma.sync, default), "sk" (stream-K) or "tc" (split-KV tcgen05),
# chosen with SPARKPIPE_MLA_KERNEL.
_MLA_DEFAULT = os.environ.get("SPARKPIPE_MLA_KERNEL", "mma")
# SPARKPIPE_MLA_SK_EARLY=0: the stream-K kernel waits for its predecessor before any load,
# inside CUDA graphs too.
_MLA_SK_EARLY = os.environ.get("SPARKPIPE_MLA_SK_EARLY", "1") != "0"


def mla_decode_splits(batch: int, heads: int, max_context: int, num_sms: int = 148, impl: str = "auto",
                      kv_fp8: bool = False) -> int:
    """Split-KV factor of the split-KV kernels ("mma", "tc", the fp8-cache kernel with
    ``kv_fp8``): the most CTAs that still fit
    one wave on the SMs, without splits of under two blocks (a second partial wave costs
    more than it hides: B=64, 16 heads, ctx 1024 measured 27 us at 2 splits, 34 us at 3).
    The stream-K kernel ignores it."""
    groups = heads // (32 if heads % 32 == 0 else 16)
    ctas = max(1, batch * groups)
    k_impl = impl if impl in ("tc", "mma") else ("tc" if _MLA_DEFAULT == "tc" else "mma")
    if kv_fp8:
        slots = num_sms * int(kernels().mla_fp8_ctas_per_sm(heads))
    else:
        slots = num_sms * int(kernels().mla_ctas_per_sm(heads, MLA_IMPL[k_impl]))  # CTAs resident at once
    want = max(1, slots // ctas)
    blocks = max(1, math.ceil(max_context / 64))
    # few long sequences need many splits to use the SMs (one 131K-token sequence:
    # 128 splits of 16 blocks); the fp32 partials cost B x splits x H x 2 KB
    cap = max(1, min(128, 4096 // ctas))
    return int(max(1, min(want, blocks // 2 if blocks >= 2 else 1, cap)))


class _SkWorkspace:
    """Scratch of the stream-K decode kernel on one device: per-segment partial outputs
    and log-sum-exps, and per-row arrival counters that the kernel leaves at zero.
    Grown outside graph capture only; replaced buffers stay referenced so graphs
    captured with them remain valid."""

    def __init__(self):
        self.o = self.lse = self.cnt = None
        self.retired = []

    def get(self, device, B, H):
        K = kernels()
        hg = int(K.mla_sk_heads_per_cta(H))
        segs = int(K.mla_sk_segments(B, H, K.num_sms()))
        need = (segs * hg * 512, segs * hg, (H // hg) * B)
        if self.o is None or self.o.numel() < need[0] or self.lse.numel() < need[1] or self.cnt.numel() < need[2]:
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("mla_decode: the stream-K scratch must be sized by an eager call before capture")
            if self.o is not None:
                self.retired.append((self.o, self.lse, self.cnt))
            o = max(need[0], 0 if self.o is None else self.o.numel())
            lse = max(need[1], 0 if self.lse is None else self.lse.numel())
            cnt = max(need[2], 0 if self.cnt is None else self.cnt.numel())
            self.o = torch.empty(o, dtype=torch.float32, device=device)
            self.lse = torch.empty(lse, dtype=torch.float32, device=device)
            self.cnt = torch.zeros(cnt, dtype=torch.int32, device=device)
        return self.o, self.lse, self.cnt

    def reset_counters(self):
        if self.cnt is not None:
            self.cnt.zero_()


_SK_WS: dict = {}


def _sk_workspace(device) -> _SkWorkspace:
    key = torch.device(device).index
    ws = _SK_WS.get(key)
    if ws is None:
        ws = _SK_WS[key] = _SkWorkspace()
    return ws


def mla_decode(q, cache, block_table, context_lens, out, splits, scale, o_part=None, lse_part=None, impl="auto",
               trace=None, last_slot=None, kv_scales=None):
    """Absorbed-MLA paged decode attention. ``impl``: "mma" (split-KV mma.sync kernel,
    the default), "sk" (stream-K kernel: all SMs over the flattened 32-token KV units),
    "tc" (split-KV tcgen05 kernel) or "auto" (the default, which the
    SPARKPIPE_MLA_KERNEL environment variable can switch). With ``kv_scales`` the cache
    is fp8 e4m3 [slots, 576] with [slots, 5] block scales and the fp8 split-KV kernel
    runs (``impl`` is ignored). ``splits`` applies to the
    split-KV kernels only. ``trace`` (diagnostics, int64 CUDA tensor): for "sk", 4 x 64
    global-timer stamps (ns) of four CTAs (first, second, middle, last): start,
    schedule ready, dependency wait passed, per piece queries landed / finished, per
    stage consumed, merge start / end, end (see mla_decode_sk.cu); for "tc", 6 x 64
    pipeline event times of its first CTA. ``last_slot`` (int32 [B], mma kernel): row b
    reads its last context token from cache row last_slot[b] (-1: from its block
    table), as a tree verify's alternate leaves need."""
    B, H, _ = q.shape
    if kv_scales is not None:
        if splits > 1 and o_part is None:
            o_part = torch.empty(B, splits, H, 512, dtype=torch.float32, device=q.device)
            lse_part = torch.empty(B, splits, H, dtype=torch.float32, device=q.device)
        kernels().mla_decode(q, cache, block_table, context_lens, out, o_part, lse_part, splits, float(scale),
                             MLA_IMPL["mma"], None, last_slot, kv_scales)
        _count(1 + (1 if splits > 1 else 0))
        return out
    if impl == "auto":
        impl = _MLA_DEFAULT
    if last_slot is not None:
        impl = "mma"
    if impl == "sk" and kernels().mla_sk_supported(B, H):
        o_ws, lse_ws, cnt = _sk_workspace(q.device).get(q.device, B, H)
        kernels().mla_decode_sk(q, cache, block_table, context_lens, out, o_ws, lse_ws, cnt, float(scale),
                                _MLA_SK_EARLY and bool(torch.cuda.is_current_stream_capturing()), trace)
        _count(1)
        return out
    if impl == "sk":
        impl = "mma"
    if splits > 1 and o_part is None:
        o_part = torch.empty(B, splits, H, 512, dtype=torch.float32, device=q.device)
        lse_part = torch.empty(B, splits, H, dtype=torch.float32, device=q.device)
    kernels().mla_decode(q, cache, block_table, context_lens, out, o_part, lse_part, splits, float(scale),
                         MLA_IMPL[impl], trace, last_slot, None)
    _count(1 + (1 if splits > 1 else 0))
    return out


def kv8_gather(cache8, scales, idx, out=None):
    """Dequantised bf16 rows [n, 576] of an fp8 latent cache at row ids ``idx``."""
    if out is None:
        out = torch.empty(idx.shape[0], 576, dtype=torch.bfloat16, device=cache8.device)
    kernels().kv8_gather(cache8, scales, idx, out)
    _count(1)
    return out


ATTN_IMPL = {"auto": 0, "tc": 1, "mma": 2}  # prefill attention kernels: default, tcgen05, mma.sync


def prefill_attention(q, k, kpe, v, o, cu_q, cu_k, max_q, scale, causal=True, impl="auto"):
    """Chunked causal MLA prefill attention (expanded form). ``impl``: "tc" (tcgen05,
    the default when the tensors suit TMA), "mma" (mma.sync) or "auto"."""
    kernels().prefill_attention(q, k, kpe, v, o, cu_q, cu_k, int(max_q), float(scale), bool(causal), ATTN_IMPL[impl])
    _count(1)
    return o


def moe_route(x, gate, bias, k, scoring, renorm, scaling, n_shared=0, n_group=1, topk_group=1, group_top2=False):
    """``moe_topk`` with the router logits x @ gate.T computed inside the kernel
    (decode-sized batches of small routers: no separate gate GEMM)."""
    T = x.shape[0]
    ids = torch.empty(T, k + n_shared, dtype=torch.int32, device=x.device)
    w = torch.empty(T, k + n_shared, dtype=torch.float32, device=x.device)
    kernels().moe_route(x, gate, bias, ids, w, int(n_shared), int(scoring), bool(renorm), float(scaling),
                        int(n_group), int(topk_group), bool(group_top2))
    _count(1)
    return ids, w


def moe_topk(logits, bias, k, scoring, renorm, scaling, n_shared=0, n_group=1, topk_group=1, group_top2=False):
    """Top-k routing; the last n_shared columns are the shared experts E.. (weight 1).
    ``logits`` is a [T, E] fp32 tensor or router ``Slabs``. With n_group > 1 the
    choice is limited to the best `topk_group` expert groups, a group scored by its
    best expert or (group_top2) by the sum of its best two."""
    if isinstance(logits, Slabs):
        T, E, dev = logits.rows, logits.cols, logits.ws.device
        src, stride, splits = logits.ws, logits.stride, logits.splits
    else:
        T, E, dev = logits.shape[0], logits.shape[1], logits.device
        src, stride, splits = logits, 0, 1
    ids = torch.empty(T, k + n_shared, dtype=torch.int32, device=dev)
    w = torch.empty(T, k + n_shared, dtype=torch.float32, device=dev)
    kernels().moe_topk(src, bias, ids, w, int(n_shared), int(scoring), bool(renorm), float(scaling), T, E, stride,
                       splits, int(n_group), int(topk_group), bool(group_top2))
    _count(1)
    return ids, w


def moe_align(topk_ids, num_experts, block_n):
    dev = topk_ids.device
    n = topk_ids.numel()
    grp_rows = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    grp_tiles = torch.empty(num_experts + 1, dtype=torch.int32, device=dev)
    sorted_tok = torch.empty(n, dtype=torch.int32, device=dev)
    inv_pos = torch.empty(n, dtype=torch.int32, device=dev)
    work = torch.empty(129 * num_experts, dtype=torch.int32, device=dev)  # per-CTA counts of large layouts
    _count(kernels().moe_align(topk_ids, num_experts, block_n, grp_rows, grp_tiles, sorted_tok, inv_pos, work))
    return grp_rows, grp_tiles, sorted_tok, inv_pos


def gather_rows(x, idx, out=None):
    if out is None:
        out = torch.empty(idx.shape[0], x.shape[1], dtype=x.dtype, device=x.device)
    kernels().gather_rows(x, idx, out)
    _count(1)
    return out


def silu_mul(h, out=None):
    if out is None:
        out = torch.empty(h.shape[0], h.shape[1] // 2, dtype=h.dtype, device=h.device)
    kernels().silu_mul(h, out)
    _count(1)
    return out


def moe_combine(y, inv_pos, w, add, out, k):
    kernels().moe_combine(y, inv_pos, w, add, out, int(k))
    _count(1)
    return out


def embedding(table, ids, out=None):
    if out is None:
        out = torch.empty(ids.shape[0], table.shape[1], dtype=table.dtype, device=table.device)
    kernels().embedding(table, ids, out)
    _count(1)
    return out


def sample_tokens(logits, temperature=0.0, seed=0, offset=0, out_ids=None, out_logit=None, row_temp=None,
                  row_key=None):
    """Greedy / Gumbel-max sampling of each logits row. One temperature and seed for
    the batch, or per-row ``row_temp`` (float32) and ``row_key`` (int64 noise key) tensors."""
    if out_ids is None:
        out_ids = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    kernels().sample_tokens(logits, float(temperature), int(seed), int(offset), out_ids, out_logit, row_temp, row_key)
    _count(1)
    return out_ids


def gather_prev_tokens(ids, prev, n):
    """ids[i] = prev[ids[i]] for i < n: a decode step scheduled ahead takes its input
    tokens from the previous step's sampled tokens without a host round trip."""
    kernels().gather_prev_tokens(ids, prev, int(n))
    _count(1)


def spec_verify(draft, target, p_accept=0.0, seed=0, offset=0):
    B, L = draft.shape
    accepted = torch.empty(B, dtype=torch.int32, device=draft.device)
    committed = torch.empty(B, L + 1, dtype=torch.int32, device=draft.device)
    kernels().spec_verify(draft, target, float(p_accept), int(seed), int(offset), accepted, committed)
    _count(1)
    return accepted, committed


def spec_chain_commit(tok, tgt, ctx, pos, budget, keys, L, committed, counts, p_accept=0.0, seed=0):
    """Verify round, chain drafts: lane b (rows j * B + b) accepts its longest agreeing
    draft prefix within budget[b] (or a seeded Bernoulli(p_accept) chain keyed by
    keys[b] and its position) and commits it plus the verifier's next token:
    committed [B, L + 1] (-1 padded), counts [B] (0 for idle lanes)."""
    kernels().spec_chain_commit(tok, tgt, ctx, pos, budget, keys, int(L), float(p_accept), int(seed), committed, counts)
    _count(1)


def mtp_tree_commit(tok, tgt, ctx, slots, cache_data, committed, counts, paths, cache_scales=None):
    """Verify round, the fixed MTP tree (rows r * B + b, r = 0..5): resolved path per
    lane, committed [B, 6] / counts [B], and the KV move of an accepted alternate leaf
    from its shadow slot in ``cache_data`` [layers, slots, row] (and in its fp8 block
    scales [layers, slots, 5])."""
    kernels().mtp_tree_commit(tok, tgt, ctx, slots, cache_data, committed, counts, paths, cache_scales)
    _count(1)


def top2_rows(logits, out0, out1):
    """Ids of the two largest logits of each row (ties to the lower id)."""
    kernels().top2_rows(logits, out0, out1)
    _count(1)


def decode_advance(out_ids, ids, pos, ctx, slots, block_table, block_size=64):
    kernels().decode_advance(out_ids, ids, pos, ctx, slots, block_table, int(block_size))
    _count(1)


def slab_add_rmsnorm(x, residual, w, out, eps):
    """residual += x; out = rmsnorm(residual) * w, where x is ``Slabs`` or a bf16 tensor."""
    if isinstance(x, Slabs):
        kernels().slab_add_rmsnorm(x.ws, x.stride, x.splits, residual, w, out, float(eps))
        _count(1)
        return out
    return add_rmsnorm(x, residual, w, out, eps)


def mla_decode_prep(qkv, norm_w, positions, cos_sin, slot_mapping, cache, q_nope_out, q_lat, dn, q_off, kv_off,
                    eps, kv_scales=None):
    """Decode prologue of MLA attention from the fused q/kv projection (``Slabs`` or bf16
    [T, Qa + kv]); the latent row goes to the bf16 cache, or the fp8 one with ``kv_scales``."""
    if isinstance(qkv, Slabs):
        kernels().mla_decode_prep(qkv.ws, qkv.stride, qkv.splits, None, norm_w, positions, cos_sin, slot_mapping,
                                  cache, q_nope_out, q_lat, qkv.rows, dn, q_off, kv_off, qkv.cols, float(eps),
                                  kv_scales)
    else:
        kernels().mla_decode_prep(None, 0, 1, qkv, norm_w, positions, cos_sin, slot_mapping, cache, q_nope_out,
                                  q_lat, qkv.shape[0], dn, q_off, kv_off, qkv.shape[1], float(eps), kv_scales)
    _count(1)


def combine_add_rmsnorm(y, inv_pos, w, residual, gamma, out, k, eps, shared=None):
    """residual[t] += sum_j w[t, j] * y[inv_pos[t, j]] (+ the shared experts' rows
    shared[s * T + t], weight 1); out[t] = rmsnorm(residual[t]) * gamma."""
    kernels().combine_add_rmsnorm(y, inv_pos, w, residual, gamma, out, int(k), float(eps), shared)
    _count(1)
    return out


def status_word() -> int:
    return int(kernels().status_word())


def clear_status() -> None:
    """Clears the device status word; a launch that gave up on a bounded wait may have
    left stream-K decode counters set, so those are zeroed too."""
    kernels().clear_status()
    ws = _SK_WS.get(torch.cuda.current_device())
    if ws is not None:
        ws.reset_counters()


# ------------------------------------------------------------------ DSA sparse attention
def paged_slots(block_table, lens, rows, positions=None, block_size=64):
    """Cache slot of positions [0, lens[b]) (or of ``positions[b, :lens[b]]``) of each
    sequence through its block table, [B, rows] int32 (slot 0 past the length)."""
    B = block_table.shape[0]
    slots = torch.empty(B, rows, dtype=torch.int32, device=block_table.device)
    kernels().paged_slots(block_table, lens, positions, int(rows), int(block_size), slots)
    _count(1)
    return slots


def dsa_select(q_idx, w_idx, k_cache, block_table, context_lens, max_context, topk=2048, block_size=64):
    """DeepSeek sparse attention token selection for one decode step.

    q_idx [B, Hi, 128] bf16 index queries, w_idx [B, Hi] fp32 head weights, k_cache
    [slots, 128] bf16 paged index keys, block_table / context_lens as for decode,
    ``max_context`` an upper bound of the lengths. score[b, s] = sum_h w[b, h] *
    relu(q[b, h] . k[s]); returns (positions [B, topk] int32: the topk best positions
    of each sequence ascending, -1 padded; counts [B]). The q.k products run on the
    tcgen05 GEMM over the gathered keys; reduce, radix select and sort in one kernel."""
    B, Hi, D = q_idx.shape
    rows = -(-int(max_context) // 8) * 8  # aligned score rows; positions past a length are masked
    dev = q_idx.device
    slots = paged_slots(block_table, context_lens, rows, block_size=block_size)
    keys = gather_rows(k_cache, slots.view(-1))                       # [B * rows, 128]
    raw = torch.empty(B, Hi, rows, dtype=torch.float32, device=dev)
    batched_gemm(keys, q_idx.reshape(B * Hi, D), raw, M=rows, N=Hi, K=D, batch=B, a_batch_rows=rows,
                 b_batch_rows=Hi, ldd=rows, d_batch_stride=Hi * rows)
    scores = torch.empty(B, rows, dtype=torch.float32, device=dev)
    pos = torch.empty(B, topk, dtype=torch.int32, device=dev)
    counts = torch.empty(B, dtype=torch.int32, device=dev)
    kernels().dsa_topk(raw, w_idx.float().contiguous(), context_lens, int(topk), scores, pos, counts)
    _count(1)
    return pos, counts


def dsa_sparse_decode(q_lat, cache, block_table, positions, counts, out, scale, block_size=64):
    """MLA decode over only the selected positions: their latent KV rows are gathered
    into 64-token blocks and the paged decode kernel runs on them."""
    B, topk = positions.shape
    if topk % block_size:
        raise ValueError("topk must be a multiple of the block size")
    slots = paged_slots(block_table, counts, topk, positions=positions, block_size=block_size)
    rows = gather_rows(cache, slots.view(-1))                         # [B * topk, 576]
    nb = topk // block_size
    bt = torch.arange(B * nb, dtype=torch.int32, device=q_lat.device).view(B, nb)
    splits = mla_decode_splits(B, q_lat.shape[1], topk, kernels().num_sms())
    return mla_decode(q_lat, rows, bt, counts, out, splits, scale)
