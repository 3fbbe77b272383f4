"""Tensor-parallel weight sharding of the MLA-MoE model.

``shard_weights(cfg, weights, tp_degree, tp_rank)`` returns this rank's slices of
the model's weights as computed by the C++ shard engine (``core().tp``): the MLA
latent projections, norms, router and embedding replicate; q_b / kv_b split their
output dimension on whole heads, o_proj its input dimension; dense and expert MLPs
split their intermediate dimension ([gate; up] stacks split each half).
``node_config(cfg, ...)`` gives the per-rank dimensions and the configuration hash
of a (TP, PP) shape.
"""
from __future__ import annotations

import torch

from ..core import core
from ..models.config import MLAMoEConfig


def geometry(cfg: MLAMoEConfig):
    T = core().tp
    return T.Geometry(cfg.num_heads, cfg.qk_nope_head_dim + cfg.qk_rope_head_dim,
                      cfg.qk_nope_head_dim + cfg.v_head_dim, cfg.v_head_dim)


def shard_tensor(name: str, t: torch.Tensor, shape, geo) -> torch.Tensor:
    T = core().tp
    view = T.compute_view(T.TensorSpec(name, list(t.shape), t.element_size()), shape, geo)
    if view.shard_class == T.ShardClass.REPLICATED:
        return t
    parts = [t.narrow(view.split_dimension, off, ext) for off, ext in view.ranges]
    out = parts[0] if len(parts) == 1 else torch.cat(parts, view.split_dimension)
    return out.contiguous()


def shard_weights(cfg: MLAMoEConfig, weights: dict, tp_degree: int, tp_rank: int, pp_stage_count: int = 1,
                  pp_stage_index: int = 0) -> dict:
    T = core().tp
    shape = T.Shape(tp_degree, tp_rank, pp_stage_count, pp_stage_index)
    geo = geometry(cfg)
    return {k: shard_tensor(k, v, shape, geo) for k, v in weights.items()}


def node_config(cfg: MLAMoEConfig, tp_degree: int, tp_rank: int, pp_stage_count: int, pp_stage_index: int,
                kv_bytes_per_element: int = 2):
    T = core().tp
    inputs = T.ModelInputs(cfg.num_layers, cfg.hidden_size, cfg.moe_intermediate_size, cfg.intermediate_size,
                           cfg.kv_cache_dim, kv_bytes_per_element)
    return T.derive_node_config(T.Shape(tp_degree, tp_rank, pp_stage_count, pp_stage_index), geometry(cfg), inputs)


# ---------------------------------------------------------------------- runtime
DEFAULT_BUDGET_CYCLES = 4_000_000_000  # ~2 s at 2 GHz


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def tp_layout(world: int, rows: int, hidden: int, max_splits: int) -> dict:
    """Byte offsets of the TP regions in one rank's buffer: rs [2][world * max_splits]
    [rows][hidden] tagged fp32 words (8 B), ag [2][world * rows][hidden] bf16, flags
    [2][world * rows] u64 (the tag of each all-gathered row)."""
    off = {"rs": 0}
    off["ag"] = _align(8 * 2 * world * max_splits * rows * hidden)
    off["flags"] = _align(off["ag"] + 2 * 2 * world * rows * hidden)
    off["total"] = _align(off["flags"] + 8 * 2 * world * rows)
    return off


class TensorParallel:
    """A sequence-parallel tensor-parallel group over NVLink peer memory.

    The T = world * rows tokens of a step are owned in blocks of ``rows``; rank r
    holds rows [r*rows, (r+1)*rows) of the residual stream. Per block of layers:

      ag_send / rs_add_rmsnorm(ag_layer=...)   normed rows -> every rank's AG region
                                               (plain stores + a released per-row flag)
      ag_gemm                                  column-parallel GEMM over all T rows: the
                                               producer acquires the row flags, then
                                               TMA-loads B from the AG region (no NCCL)
      rs_gemm                                  row-parallel GEMM whose epilogue sends
                                               fp32 partials to the token owners
      rs_add_rmsnorm                           owner: sum of partials + residual + RMSNorm

    All device work, stream-ordered and graph-capturable; the layer epoch lives in
    device memory (``end_step`` advances it). ``emulated(W, ...)`` builds W ranks in
    one process on one GPU for phase-ordered tests. ``nccl_ag_gemm`` /
    ``nccl_rs_gemm`` are the NCCL baselines of the same two operations.
    """

    def __init__(self, world: int, rank: int, rows: int, hidden: int, device, group=None, max_splits: int = 4,
                 layers_per_step: int = 2, budget_cycles: int = DEFAULT_BUDGET_CYCLES):
        from .. import _ext

        assert 1 <= world <= 8 and hidden % 8 == 0 and layers_per_step % 2 == 0
        self.world, self.rank, self.rows, self.H = world, rank, rows, hidden
        self.max_splits, self.layers_per_step = max_splits, layers_per_step
        self.device = torch.device(device)
        self.budget = int(budget_cycles)
        self.K = _ext.kernels()
        self.layout = tp_layout(world, rows, hidden, max_splits)
        self.buf = self.K.ep_alloc(self.layout["total"], self.device.index or 0)
        self.bases = [0] * 8
        self.bases[rank] = self.buf.data_ptr()
        self._opened: list[int] = []
        if group is not None:
            import torch.distributed as dist
            handles = [None] * world
            dist.all_gather_object(handles, self.K.ep_ipc_handle(self.buf), group=group)
            for r in range(world):
                if r != rank:
                    p = self.K.ep_ipc_open(handles[r], self.device.index or 0)
                    self._opened.append(p)
                    self.bases[r] = p
        self.epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
        self.group = group

    @classmethod
    def emulated(cls, world: int, rows: int, hidden: int, device, **kw):
        ranks = [cls(world, r, rows, hidden, device, **kw) for r in range(world)]
        bases = [r.buf.data_ptr() for r in ranks] + [0] * (8 - world)
        for r in ranks:
            r.bases = list(bases)
        return ranks

    def close(self):
        for p in self._opened:
            self.K.ep_ipc_close(p)
        self._opened.clear()

    def args(self) -> list[int]:
        return list(self.bases) + [self.layout["rs"], self.layout["ag"], self.layout["flags"], self.world, self.rank,
                                   self.rows, self.H, self.layers_per_step]

    # ------------------------------------------------------------------ ops
    def ag_send(self, layer: int, x: torch.Tensor):
        """All-gather this rank's rows x [<= rows, H] into every rank's AG region."""
        self.K.tp_ag_send(self.args(), self.epoch, layer, x)
        from .. import ops
        ops._count(1)

    def ag_gemm(self, layer: int, w: torch.Tensor, out: torch.Tensor | None = None, n_tokens: int | None = None,
                block_n: int = 0) -> torch.Tensor:
        """Column-parallel out [T, O] = AG(x) @ w.T for this rank's weight shard w [O, H]."""
        from .. import ops
        T = n_tokens or self.world * self.rows
        O = w.shape[0]
        if out is None:
            out = torch.empty(T, O, dtype=torch.bfloat16, device=self.device)
        self.K.gemm_tp(w, None, out, O, T, self.H, self.args(), self.epoch, layer, 0, 1, 0, 1, block_n, self.budget)
        ops._count(1)
        return out

    def rs_gemm(self, layer: int, x: torch.Tensor, w: torch.Tensor, splits: int = 1, block_n: int = 64) -> int:
        """Row-parallel: partials of x [T, Kl] @ w[H, Kl].T go to the token owners.
        Returns the number of partial slots per owner row (world x splits). Split-K
        multiplies the bytes sent (every split sends its own partial), so the
        default spreads the work over 64-token tiles instead."""
        from .. import ops
        T = x.shape[0]
        splits = max(1, splits)
        dummy = self.epoch  # D is not written
        self.K.gemm_tp(w, x, dummy, w.shape[0], T, x.shape[1], self.args(), self.epoch, layer, 1, 0, w.shape[0],
                       min(splits, self.max_splits), block_n, self.budget)
        ops._count(1)
        return self.world * min(splits, self.max_splits)

    def rs_add_rmsnorm(self, layer: int, slots: int, residual: torch.Tensor, gamma: torch.Tensor,
                       out: torch.Tensor, eps: float, ag_layer: int = -1):
        """Owner side: residual += sum of partials; out = rmsnorm(residual) * gamma
        (and, with ag_layer >= 0, all-gather of out under that layer's tag)."""
        from .. import ops
        self.K.tp_rs_add_rmsnorm(self.args(), self.epoch, layer, slots, residual, gamma, out, float(eps), ag_layer,
                                 self.budget)
        ops._count(1)

    def end_step(self):
        from .. import ops
        self.K.ep_advance(self.epoch)
        ops._count(1)

    # ------------------------------------------------------------------ NCCL baselines
    def nccl_ag_gemm(self, x_local: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        import torch.distributed as dist
        from .. import ops
        full = torch.empty(self.world * x_local.shape[0], x_local.shape[1], dtype=x_local.dtype, device=self.device)
        dist.all_gather_into_tensor(full, x_local.contiguous(), group=self.group)
        return ops.linear(full, w)

    def nccl_rs_gemm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        """fp32 partial x @ w.T, reduce-scattered over tokens (sum); returns this rank's rows."""
        import torch.distributed as dist
        from .. import ops
        part = ops.linear(x, w, out_dtype=torch.float32)
        mine = torch.empty(x.shape[0] // self.world, w.shape[0], dtype=torch.float32, device=self.device)
        dist.reduce_scatter_tensor(mine, part, group=self.group)
        return mine
