"""Expert parallelism: routed experts split over the ranks of one box, with the
token all-to-all done by fused peer-memory kernels (``csrc/kernels/ep.cu``).

Attention stays data-parallel (every rank decodes its own requests); rank r
holds routed experts [r*El, (r+1)*El) plus all shared experts. Per MoE layer:

    dispatch -> shared experts on the local tokens (while the routed rows travel)
    -> receive/align -> gather -> grouped GEMM (gate/up + SwiGLU) -> grouped GEMM
    (down, whose epilogue stores each output row straight into its source rank's
    combine slot)

and the weighted sum of the returned rows, the residual add and the next
RMSNorm run in one kernel that reads the rows as they arrive. Every word that
crosses to a peer carries its own epoch tag, so no fences or flags are needed.
All of it is stream-ordered device work (CUDA-graph capturable): the layer
epoch lives in device memory and is advanced once per forward by ``end_step``.

Buffers: one ``cudaMalloc`` per rank, mapped by every peer through CUDA IPC.
Two parity halves (per MoE layer index) make back-to-back layers race-free.

``ExpertParallel.emulated(W, ...)`` builds W ranks inside one process on one
GPU (peer pointers are the other local buffers); driving the phases
rank-by-rank in phase order exercises every kernel without any kernel waiting
on a concurrently running one.
"""
from __future__ import annotations

import os

import torch

from .. import _ext, ops

DEFAULT_BUDGET_CYCLES = 4_000_000_000  # ~2 s at 2 GHz: far above any healthy wait


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


CHUNK_TOKENS = 8    # tokens per dispatch CTA (csrc/kernels/launch.h EP_CHUNK_TOKENS)
COMBINE_CTAS = 16   # combine-send CTAs per destination (EP_COMBINE_CTAS)


def row_words(hidden: int, fp8: bool) -> int:
    """Tagged words per dispatched row: H/2 for bf16 rows; for the fp8 transport
    H/4 words of e4m3 plus one scale word per 128 columns (rounded to even)."""
    return hidden // 4 + ((hidden // 128 + 1) & ~1) if fp8 else hidden // 2


def ep_layout(world: int, cap: int, hidden: int, kk: int, fp8: bool = False) -> dict:
    """Byte offsets of the EP regions inside one rank's buffer (cap: whole token
    chunks). Every region holds 8-byte tagged words (4 payload bytes each)."""
    off = {}
    pos = 0

    def region(name, words):
        nonlocal pos
        off[name] = pos
        pos = _align(pos + 8 * words)

    max_ranks = 8
    chunks = cap // CHUNK_TOKENS
    region("ctrl", 2 * max_ranks * chunks)             # rows per (source, chunk)
    region("nch", 2 * max_ranks)                       # chunks per source
    region("meta", 2 * world * cap * (2 + 2 * kk))     # (token, n, experts, k-slots) per row
    region("rows", 2 * world * cap * row_words(hidden, fp8))  # received hidden rows
    region("comb", 2 * cap * kk * hidden // 2)         # returned expert outputs per (token, k-slot)
    off["total"] = pos
    return off


class ExpertParallel:
    def __init__(self, cfg, rank: int, world: int, cap_tokens: int, device, group=None,
                 budget_cycles: int = DEFAULT_BUDGET_CYCLES, fp8_transport: bool | None = None,
                 shared_local: bool = False):
        """``fp8_transport`` (default: the model has block-scaled fp8 weights) sends
        dispatched rows as e4m3 with one fp32 scale per 128 columns, quantised
        once in the dispatch kernel: half the NVLink bytes, and the receiver
        gathers them straight into the fp8 expert GEMM's operand layout.

        ``shared_local``: the shared experts are not dispatched; every rank runs them
        on its own tokens while the routed rows cross NVLink, and the combine reads their
        rows locally. On the main stream this was slower (V2-Lite, 2 GPUs: the shared
        experts' own grouped GEMMs took 32.8 us against 12.7 us saved in the routed GEMM,
        5.96 -> 6.46 ms per step); on a forked stream they overlap the dispatch, receive
        and routed experts and the step is faster (5.75 -> 5.67 ms), so ranks in
        separate processes use it by default."""
        assert cfg.n_routed_experts % world == 0, "routed experts must split evenly over the ranks"
        assert 1 <= world <= 8
        cap_tokens = -(-cap_tokens // CHUNK_TOKENS) * CHUNK_TOKENS
        self.cfg, self.rank, self.world, self.cap = cfg, rank, world, cap_tokens
        self.group = group  # None: ranks emulated in one process
        self.device = torch.device(device)
        self.budget = int(budget_cycles)
        self.kk = cfg.num_experts_per_tok + cfg.n_shared_experts
        self.El = cfg.n_routed_experts // world
        self.n_local = self.El + cfg.n_shared_experts
        self.H = cfg.hidden_size
        self.moe_layers = [i for i in range(cfg.num_layers) if cfg.is_moe_layer(i)]
        self.moe_index = {layer: j for j, layer in enumerate(self.moe_layers)}
        # even layer count per step -> MoE layer j always uses buffer parity j & 1
        self.layers_per_step = len(self.moe_layers) + (len(self.moe_layers) & 1)
        self.fp8 = (cfg.weight_dtype == "fp8_block") if fp8_transport is None else bool(fp8_transport)
        self.S = cfg.n_shared_experts
        # Multi-process ranks default to local shared experts on a forked stream, which
        # measured faster than dispatching them (V2-Lite, 2 GPUs: 5.67 vs 5.75 ms per
        # step); SPARKPIPE_EP_SHARED_LOCAL=0 dispatches them, SPARKPIPE_EP_SHARED_SIDE=0
        # runs them on the main stream after the dispatch.
        # (bf16 experts: the fp8 shared-expert path is verified with dispatched shared
        # experts only, so fp8 models keep dispatching them unless asked)
        if group is not None and os.environ.get("SPARKPIPE_EP_SHARED_LOCAL", "0" if self.fp8 else "1") == "1":
            shared_local = True
        self.shared_local = bool(shared_local) and self.S > 0
        self.shared_side = os.environ.get("SPARKPIPE_EP_SHARED_SIDE", "1") == "1"
        self._side = None
        self._join = None
        self.row_words = row_words(self.H, self.fp8)
        self.layout = ep_layout(world, cap_tokens, self.H, self.kk, self.fp8)
        K = _ext.kernels()
        self.K = K
        self.buf = K.ep_alloc(self.layout["total"], self.device.index or 0)
        self._opened: list[int] = []
        self.bases = [0] * 8
        self.bases[rank] = self.buf.data_ptr()
        if group is not None:
            import torch.distributed as dist
            handles = [None] * world
            dist.all_gather_object(handles, K.ep_ipc_handle(self.buf), group=group)
            for r in range(world):
                if r != rank:
                    p = K.ep_ipc_open(handles[r], self.device.index or 0)
                    self._opened.append(p)
                    self.bases[r] = p
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        dev = self.device
        max_pairs = world * cap_tokens * min(self.kk, self.n_local)
        self.grp_rows = torch.zeros(self.n_local + 1, dtype=torch.int32, device=dev)
        self.grp_tiles = torch.zeros(self.n_local + 1, dtype=torch.int32, device=dev)
        self.src_row = torch.zeros(max_pairs, dtype=torch.int32, device=dev)
        self.comb_dst = torch.zeros(max_pairs, dtype=torch.int32, device=dev)
        F = cfg.moe_intermediate_size
        if self.fp8:
            self.xs = None
            self.xq = ops.Fp8Act(torch.zeros(max_pairs, self.H, dtype=torch.float8_e4m3fn, device=dev),
                                 torch.zeros(self.H // 128, max_pairs, dtype=torch.float32, device=dev))
            self.aq = ops.Fp8Act(torch.zeros(max_pairs, F, dtype=torch.float8_e4m3fn, device=dev),
                                 torch.zeros(F // 128, max_pairs, dtype=torch.float32, device=dev))
        else:
            self.xs = torch.zeros(max_pairs, self.H, dtype=torch.bfloat16, device=dev)
            self.xq = self.aq = None
        self.act = torch.zeros(max_pairs, F, dtype=torch.bfloat16, device=dev)
        self._sh = {}  # shared-expert buffers per power-of-two token bucket
        self._sh_tables = {}  # shared-expert row / tile / source tables per token count
        self.y = torch.zeros(max_pairs, self.H, dtype=torch.bfloat16, device=dev)

    @classmethod
    def emulated(cls, cfg, world: int, cap_tokens: int, device, budget_cycles: int = DEFAULT_BUDGET_CYCLES, **kw):
        ranks = [cls(cfg, r, world, cap_tokens, device, budget_cycles=budget_cycles, **kw) for r in range(world)]
        bases = [r.buf.data_ptr() for r in ranks] + [0] * (8 - world)
        for r in ranks:
            r.bases = list(bases)
        return ranks

    def close(self):
        for p in self._opened:
            self.K.ep_ipc_close(p)
        self._opened.clear()

    # ------------------------------------------------------------------ args
    def args(self) -> list[int]:
        L = self.layout
        c = self.cfg
        return (list(self.bases) + [L["ctrl"], L["nch"], L["meta"], L["rows"], L["comb"]] +
                [self.world, self.rank, self.cap, self.H, self.kk, c.n_routed_experts, self.El,
                 c.n_shared_experts, self.layers_per_step, self.cap // CHUNK_TOKENS, int(self.fp8), self.row_words,
                 int(self.shared_local)])

    def local_expert_range(self) -> tuple[int, int]:
        return self.rank * self.El, (self.rank + 1) * self.El

    # ------------------------------------------------------------------ phases
    def dispatch(self, layer: int, xn: torch.Tensor, ids: torch.Tensor):
        self.K.ep_dispatch(xn, ids, self.args(), self.epoch, self.moe_index[layer])
        ops._count(1)

    def receive(self, layer: int, bn: int):
        j = self.moe_index[layer]
        self.K.ep_recv_align(self.args(), self.epoch, j, bn, self.grp_rows, self.grp_tiles, self.src_row,
                             self.comb_dst, self.budget)
        if self.fp8:
            self.K.ep_gather_fp8(self.args(), self.epoch, j, self.grp_rows[self.n_local:], self.src_row, self.xq.q,
                                 self.xq.s, self.budget)
        else:
            self.K.ep_gather(self.args(), self.epoch, j, self.grp_rows[self.n_local:], self.src_row, self.xs,
                             self.budget)
        ops._count(2)

    def _comb(self, layer: int):
        """Combine epilogue arguments of the down-projection GEMM for MoE layer `layer`."""
        return (self.args(), self.comb_dst, self.epoch, self.moe_index[layer])

    def experts(self, w13, w2, bn: int, fused_swiglu: bool = True, layer: int | None = None,
                token_major: bool = False):
        """Expert GEMMs of the received rows. With `layer` the down projection's epilogue
        sends every output row straight into its source rank's combine slot (the
        combine-send kernel is not needed); without it the rows land in ``self.y``.
        ``token_major`` (prefill-sized groups, bf16, fused SwiGLU; the rows were laid out
        in 128-row tiles, bn = 128) runs the gate/up GEMM with the tokens as the M tiles."""
        comb = self._comb(layer) if layer is not None else None
        if isinstance(w13, ops.Fp8Weight):
            # block-scaled fp8 experts; the live row count stays on the device
            if not self.fp8:
                raise ValueError("expert parallel: fp8 expert weights need the fp8 transport")
            rows_dev = self.grp_rows[self.n_local:]
            ops.grouped_gemm_fp8(w13, self.xq, self.act, self.grp_rows, self.grp_tiles, self.n_local, bn, swiglu=True)
            ops.quant_act_fp8(self.act, rows_dev=rows_dev, out=self.aq)
            ops.grouped_gemm_fp8(w2, self.aq, self.y, self.grp_rows, self.grp_tiles, self.n_local, bn, ep_combine=comb)
            return
        if self.fp8:
            raise ValueError("expert parallel: the fp8 transport needs fp8 expert weights")
        if fused_swiglu and token_major:
            ops.grouped_gemm_tm(w13[:self.n_local], self.xs, self.act, self.grp_rows, self.grp_tiles, self.n_local,
                                swiglu=True)
        elif fused_swiglu:
            ops.grouped_gemm(w13, self.xs, self.act, self.grp_rows, self.grp_tiles, self.n_local, bn, swiglu=True)
        else:
            h13 = torch.empty(self.xs.shape[0], 2 * self.act.shape[1], dtype=torch.bfloat16, device=self.device)
            ops.grouped_gemm(w13, self.xs, h13, self.grp_rows, self.grp_tiles, self.n_local, bn)
            ops.silu_mul(h13, out=self.act)
        ops.grouped_gemm(w2, self.act, self.y, self.grp_rows, self.grp_tiles, self.n_local, bn, ep_combine=comb)

    def shared(self, xn: torch.Tensor, w13, w2, fused_swiglu: bool = True, token_major: bool = False):
        """The shared experts on this rank's tokens (S groups of T rows, the same grouped
        kernels as the routed experts; token-major 128-row tiles with ``token_major``);
        rows land in ``self.y_sh`` [S, T, H]."""
        T, S, F = xn.shape[0], self.S, self.act.shape[1]
        if T == 0:
            return
        # buffers per power-of-two bucket of T (bounded, and alive for any graph captured
        # with them); the small row / tile / source tables are cached per T up to 4,096
        # tokens and rebuilt per call above that
        bucket = 1 << max(0, (T - 1).bit_length())
        dev = self.device
        if bucket not in self._sh:
            self._sh[bucket] = dict(act=torch.empty(S * bucket * F, dtype=torch.bfloat16, device=dev),
                                    y=torch.empty(S * bucket * self.H, dtype=torch.bfloat16, device=dev))
        tm = token_major and fused_swiglu and not isinstance(w13, ops.Fp8Weight)
        bn = 128 if tm else max(32, min(128, bucket)) if self.fp8 else max(16, min(256, bucket))
        cb = self._sh[bucket]
        tab = self._sh_tables.get((T, bn))
        if tab is None:  # decode-sized T: built once (in the eager warm-up), replayed from then on
            tab = (torch.arange(0, (S + 1) * T, T, dtype=torch.int32, device=dev),
                   torch.arange(0, S + 1, dtype=torch.int32, device=dev) * ((T + bn - 1) // bn),
                   (torch.arange(S * T, device=dev) % T).to(torch.int32))
            if T <= 4096:
                self._sh_tables[(T, bn)] = tab
        b = dict(bn=bn, rows=tab[0], tiles=tab[1], src=tab[2],
                 act=cb["act"][:S * T * F].view(S * T, F), y=cb["y"][:S * T * self.H].view(S, T, self.H))
        El = self.El
        if isinstance(w13, ops.Fp8Weight):
            w13s = ops.Fp8Weight(w13.q[El:], w13.s[El:], w13.sa_rows)
            w2s = ops.Fp8Weight(w2.q[El:], w2.s[El:], w2.sa_rows)
            xq = ops.quant_act_fp8(xn, b["src"])  # each shared expert sees every token
            ops.grouped_gemm_fp8(w13s, xq, b["act"], b["rows"], b["tiles"], S, b["bn"], swiglu=True)
            ops.grouped_gemm_fp8(w2s, ops.quant_act_fp8(b["act"]), b["y"].view(S * T, self.H), b["rows"], b["tiles"],
                                 S, b["bn"])
        else:
            xs = ops.gather_rows(xn, b["src"])
            if tm:
                ops.grouped_gemm_tm(w13[El:], xs, b["act"], b["rows"], b["tiles"], S, swiglu=True)
                ops.grouped_gemm_tm(w2[El:], b["act"], b["y"].view(S * T, self.H), b["rows"], b["tiles"], S)
                self.y_sh = b["y"]
                return
            if fused_swiglu:
                ops.grouped_gemm(w13[El:], xs, b["act"], b["rows"], b["tiles"], S, b["bn"], swiglu=True)
            else:
                h13 = torch.empty(S * T, 2 * F, dtype=torch.bfloat16, device=self.device)
                ops.grouped_gemm(w13[El:], xs, h13, b["rows"], b["tiles"], S, b["bn"])
                ops.silu_mul(h13, out=b["act"])
            ops.grouped_gemm(w2[El:], b["act"], b["y"].view(S * T, self.H), b["rows"], b["tiles"], S, b["bn"])
        self.y_sh = b["y"]

    def combine_send(self, layer: int):
        self.K.ep_combine_send(self.y, self.grp_rows[self.n_local:], self.comb_dst, self.args(), self.epoch,
                               self.moe_index[layer])
        ops._count(1)

    def combine(self, layer: int, wts: torch.Tensor):
        """The deferred combine of this layer; ``model._residual_norm`` runs it as
        ``combine_add_rmsnorm`` (slot sum + residual add + RMSNorm in one kernel)."""
        return ("ep_combine", self, layer, wts)

    def combine_add_rmsnorm(self, layer: int, wts: torch.Tensor, res: torch.Tensor, gamma: torch.Tensor,
                            out: torch.Tensor, eps: float):
        ys = self.y_sh if self.shared_local and res.shape[0] > 0 else None
        if self.shared_local and self.shared_side and self._join is not None:
            torch.cuda.current_stream(self.device).wait_event(self._join)
            self._join = None
        self.K.ep_combine_add_rmsnorm(self.args(), self.epoch, self.moe_index[layer], wts, res, gamma, out, eps,
                                      self.budget, ys)
        ops._count(1)

    def end_step(self):
        self.K.ep_advance(self.epoch)
        ops._count(1)

    # ------------------------------------------------------------------ one layer
    def moe(self, layer: int, xn: torch.Tensor, ids: torch.Tensor, wts: torch.Tensor, w13: torch.Tensor,
            w2: torch.Tensor, bn: int, fused_swiglu: bool = True, token_major: bool = False):
        """Runs one MoE layer for this rank's tokens; returns the deferred combine.
        ``token_major`` (prefill-sized groups) lays the received rows out in 128-row
        tiles and runs the gate/up GEMMs (and the shared experts') token-major."""
        if token_major:
            bn = 128
        if xn.shape[0] > self.cap:
            raise ValueError(f"expert parallel: {xn.shape[0]} tokens exceed the buffer capacity {self.cap}")
        self.dispatch(layer, xn, ids)
        if self.shared_local and self.shared_side:
            # forked stream: the shared experts' GEMMs stream their weights while the main
            # stream waits for the routed rows, runs the routed experts and sends them back
            # (the warm-up keeps its tables built outside capture); joined before the combine
            main = torch.cuda.current_stream(self.device)
            if self._side is None:
                self._side = torch.cuda.Stream(device=self.device)
            fork = torch.cuda.Event()
            fork.record(main)
            self._side.wait_event(fork)
            with torch.cuda.stream(self._side):
                self.shared(xn, w13, w2, fused_swiglu, token_major)
                self._join = torch.cuda.Event()
                self._join.record(self._side)
        elif self.shared_local:
            self.shared(xn, w13, w2, fused_swiglu, token_major)  # runs while the routed rows cross NVLink
        self.receive(layer, bn)
        # down projection sends to the source ranks
        self.experts(w13, w2, bn, fused_swiglu, layer=layer, token_major=token_major)
        return self.combine(layer, wts)


def block_n_for(tokens_per_rank: int, kk: int, n_local: int) -> int:
    """Tile width of the expert GEMM from the expected rows per local expert."""
    from ..models.mla_moe import _moe_block_n
    return _moe_block_n(tokens_per_rank * kk, n_local)
