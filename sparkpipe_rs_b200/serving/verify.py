"""One speculative verify round of the serving engine: drafts from a small draft model,
one batched target forward over every lane's rows, and the commit kernel.

Rows are row-major by draft depth / tree row (row j * B + b for lane b of the B
padded lanes), so each draft step reads a contiguous slice of the same token /
position / slot arrays the target reads whole. The scheduler plans the rows
(positions, cache slots, context lengths, per-lane draft budgets); the round fills
the draft tokens on the device.

  chain (draft length L)  draft steps j = 0..L-1 decode row block j and write the
                          greedy token of row block j + 1; step L only writes the
                          draft KV of t_L. The target decodes all (L + 1) B rows,
                          then ``spec_chain_commit`` accepts per lane (agreement
                          within the lane's budget, or forced Bernoulli(p)).
  MTP tree (5 / 6)        the draft rewrites its KV of the three positions before
                          each input token (``write_kv``: accepted tree tokens may
                          not be in its cache), then decodes the input row (top-1:
                          candidate 0 in row 1), candidate 0 (top-2: candidates 1 and
                          2 in rows 2 and 3) and candidate 1 (top-2: candidates 3
                          and 4 in rows 4 and 5). The target decodes the 6 rows per
                          lane; the alternate leaves (rows 3 and 5) write their KV to
                          shadow slots and read it there (``self_slots``);
                          ``mtp_tree_commit`` resolves the path and moves an accepted
                          alternate's KV into place.

On CUDA the round is one CUDA graph per padded batch; on CPU it runs eagerly with
plain PyTorch stand-ins of the kernels (tests of the host logic).

Reference behaviour: arm / resolve of verify dispatches in
crates/spark-serve/src/request_api/speculation.rs:720-882 and the MTP tree of
crates/spark-sched/src/work_control.rs:107-253.
"""
from __future__ import annotations

import torch

from .. import ops
from ..models.mla_moe import ForwardBatch

TREE_ROWS = 6
_TREE_PARENT = (0, 0, 1, 1, 2, 2)
_TREE_DEPTH = (0, 1, 2, 2, 3, 3)
_TREE_CHILDREN = ((1,), (2, 3), (4, 5), (), (), ())


def _mix(z: int) -> int:  # SplitMix64 finaliser, the same as the kernels'
    m = (1 << 64) - 1
    z = (z + 0x9E3779B97F4A7C15) & m
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
    return z ^ (z >> 31)


def _unit(seed: int, key: int, pos: int, depth: int) -> float:
    h = _mix(seed ^ _mix((key & ((1 << 64) - 1)) ^ _mix(pos ^ _mix(depth))))
    return ((h >> 40) + 0.5) / 16777216.0


def chain_commit_reference(tok, tgt, ctx, pos, budget, keys, B, L, p_accept=0.0, seed=0):
    """Plain-Python statement of ``spec_chain_commit`` (CPU rounds and tests)."""
    committed = torch.full((B, L + 1), -1, dtype=torch.int32)
    counts = torch.zeros(B, dtype=torch.int32)
    for b in range(B):
        if int(ctx[b]) == 0:
            continue
        d = min(max(int(budget[b]), 0), L)
        a = 0
        while a < d:
            ok = (_unit(seed, int(keys[b]), int(pos[b]), a) < p_accept) if p_accept > 0 else \
                int(tok[(a + 1) * B + b]) == int(tgt[a * B + b])
            if not ok:
                break
            a += 1
        for i in range(a):
            committed[b, i] = int(tok[(i + 1) * B + b])
        committed[b, a] = int(tgt[a * B + b])
        counts[b] = a + 1
    return committed, counts


def tree_commit_reference(tok, tgt, ctx, slots, B, cache_data=None):
    """Plain-Python statement of ``mtp_tree_commit`` (CPU rounds and tests)."""
    committed = torch.full((B, TREE_ROWS), -1, dtype=torch.int32)
    counts = torch.zeros(B, dtype=torch.int32)
    paths = torch.zeros(B, dtype=torch.int32)
    for b in range(B):
        if int(ctx[b]) == 0:
            continue
        row = 0
        moved = True
        while moved:
            moved = False
            for child in _TREE_CHILDREN[row]:
                if int(tok[child * B + b]) == int(tgt[row * B + b]):
                    row, moved = child, True
                    break
        depth = _TREE_DEPTH[row]
        r = row
        for k in range(depth - 1, -1, -1):
            committed[b, k] = int(tok[r * B + b])
            r = _TREE_PARENT[r]
        committed[b, depth] = int(tgt[row * B + b])
        counts[b] = depth + 1
        paths[b] = row
        if cache_data is not None and row in (3, 5):
            src, dst = int(slots[row * B + b]), int(slots[(2 if row == 3 else 4) * B + b])
            if src >= 0 and dst >= 0:
                cache_data[:, dst] = cache_data[:, src]
    return committed, counts, paths


class VerifyRound:
    def __init__(self, target, draft, tcache, dcache, batch: int, mode: str, draft_len: int, max_blocks: int,
                 max_context: int, p_accept: float = 0.0, seed: int = 0, use_graph: bool = True):
        assert mode in ("chain", "mtp_tree")
        self.target, self.draft, self.tcache, self.dcache = target, draft, tcache, dcache
        self.B, self.mode, self.L = batch, mode, draft_len
        self.rows = TREE_ROWS if mode == "mtp_tree" else draft_len + 1
        self.p_accept, self.seed = float(p_accept), int(seed)
        dev = target.device
        self.is_cuda = dev.type == "cuda"
        B, R = batch, self.rows * batch
        i32 = dict(dtype=torch.int32, device=dev)
        self.tok = torch.zeros(R, **i32)
        self.pos = torch.zeros(R, **i32)
        self.slot = torch.full((R,), -1, **i32)
        self.ctx = torch.zeros(R, **i32)
        self.tgt = torch.zeros(R, **i32)
        self.bt = torch.zeros(B, max_blocks, **i32)
        self.bt_rows = torch.zeros(R, max_blocks, **i32)
        self.budget = torch.zeros(B, **i32)
        self.keys = torch.zeros(B, dtype=torch.int64, device=dev)
        self.sync = torch.zeros(3, 3 * B, **i32)  # token ids, positions, slots of the draft-sync rows
        self.sync[2].fill_(-1)
        self.committed = torch.full((B, self.rows), -1, **i32)
        self.counts = torch.zeros(B, **i32)
        self.paths = torch.zeros(B, **i32)
        nsm = ops.kernels().num_sms() if self.is_cuda else 1

        def splits(rows, heads, cache):
            if not self.is_cuda:
                return 1
            return ops.mla_decode_splits(rows, heads, max_context, nsm, kv_fp8=getattr(cache, "fp8", False))

        def rows_fb(j0, j1, model):
            s = slice(j0 * B, j1 * B)
            return ForwardBatch(mode="decode", token_ids=self.tok[s], positions=self.pos[s], slot_mapping=self.slot[s],
                                block_table=self.bt if j1 - j0 == 1 else self.bt_rows[s], context_lens=self.ctx[s],
                                decode_splits=splits((j1 - j0) * B, model.cfg.num_heads, self.dcache))

        steps = 3 if mode == "mtp_tree" else draft_len + 1
        self.dfb = [rows_fb(j, j + 1, draft) for j in range(steps)]
        self.sync_fb = ForwardBatch(mode="decode", token_ids=self.sync[0], positions=self.sync[1],
                                    slot_mapping=self.sync[2])
        self.vfb = ForwardBatch(mode="decode", token_ids=self.tok, positions=self.pos, slot_mapping=self.slot,
                                block_table=self.bt_rows, context_lens=self.ctx,
                                decode_splits=splits(R, target.cfg.num_heads, self.tcache),
                                self_slots=self.slot if mode == "mtp_tree" else None)
        self.use_graph = use_graph and self.is_cuda
        self.graph = None
        self.timing = None  # (start, end) CUDA events around the last replay

    # ------------------------------------------------------------------ pieces
    def _greedy(self, logits, out):
        if self.is_cuda:
            ops.sample_tokens(logits, 0.0, out_ids=out)
        else:
            out.copy_(logits.float().argmax(-1).to(torch.int32))

    def _top2(self, logits, out0, out1):
        if self.is_cuda:
            ops.top2_rows(logits, out0, out1)
        else:
            idx = logits.float().topk(2, dim=-1).indices.to(torch.int32)
            out0.copy_(idx[:, 0])
            out1.copy_(idx[:, 1])

    def _round(self):
        B, rows, mb = self.B, self.rows, self.bt.shape[1]
        self.bt_rows.view(rows, B, mb).copy_(self.bt.unsqueeze(0).expand(rows, B, mb))
        t = self.tok
        if self.mode == "chain":
            for j in range(self.L):
                self._greedy(self.draft.forward(self.dfb[j], self.dcache), t[(j + 1) * B:(j + 2) * B])
            self.draft.write_kv(self.dfb[self.L], self.dcache)
        else:
            self.draft.write_kv(self.sync_fb, self.dcache)
            self._greedy(self.draft.forward(self.dfb[0], self.dcache), t[B:2 * B])
            self._top2(self.draft.forward(self.dfb[1], self.dcache), t[2 * B:3 * B], t[3 * B:4 * B])
            self._top2(self.draft.forward(self.dfb[2], self.dcache), t[4 * B:5 * B], t[5 * B:6 * B])
        self._greedy(self.target.forward(self.vfb, self.tcache), self.tgt)
        if self.is_cuda:
            if self.mode == "chain":
                ops.spec_chain_commit(t, self.tgt, self.ctx, self.pos, self.budget, self.keys, self.L, self.committed,
                                      self.counts, self.p_accept, self.seed)
            else:
                ops.mtp_tree_commit(t, self.tgt, self.ctx, self.slot, self.tcache.data, self.committed, self.counts,
                                    self.paths, self.tcache.scales)
        elif self.mode == "chain":
            c, n = chain_commit_reference(t, self.tgt, self.ctx, self.pos, self.budget, self.keys, B, self.L,
                                          self.p_accept, self.seed)
            self.committed.copy_(c)
            self.counts.copy_(n)
        else:
            c, n, p = tree_commit_reference(t, self.tgt, self.ctx, self.slot, B, self.tcache.data)
            self.committed.copy_(c)
            self.counts.copy_(n)
            self.paths.copy_(p)

    def capture(self):
        """Warm-up round (sets kernel attributes outside capture), then the graph. Without
        a graph there is nothing to prepare, and no round runs: on a lockstep
        (expert-parallel) rank each target forward is a collective its peers must join."""
        if not self.use_graph:
            return
        self._round()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self._round()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()

    def run(self, timed: bool = False):
        """One round over the inputs already in the device arrays; returns (committed, counts, paths)."""
        if timed and self.is_cuda:
            self.timing = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self.timing[0].record()
        if self.graph is not None:
            self.graph.replay()
        else:
            self._round()
        if timed and self.is_cuda:
            self.timing[1].record()
        return self.committed, self.counts, self.paths

    def release(self):
        self.graph = None
