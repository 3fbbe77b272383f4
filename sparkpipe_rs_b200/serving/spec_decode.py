"""Speculative decoding: a small draft model proposes L tokens per sequence, the
target model verifies them in one forward pass, and one kernel commits the
accepted prefix plus the verifier's next token and prepares the next round.

One round for B sequences (all device work, one CUDA graph per round):

  draft step j = 0..L   the draft decodes row block j (token t_j at position p+j,
                        its KV written at p+j); steps 0..L-1 sample t_{j+1}
                        greedily. Step L only writes the KV of t_L, so the draft
                        cache is complete when every draft is accepted.
  verify                the target decodes all (L+1)*B rows at once: row (j, b)
                        attends to the context up to p+j, i.e. the cached
                        prefix plus t_0..t_j of this round (their KV is written
                        by the same forward before attention reads it).
  finish                ``spec_finish``: accepted prefix a (drafts that match the
                        verifier's greedy tokens, or a seeded Bernoulli(p) chain
                        for benchmarks), committed tokens t_1..t_a + verifier
                        token, and the row arrays of the next round (p += a+1).

Rows are j-major (row j*B + b), so the draft steps read contiguous slices of the
same token / position / slot arrays the verifier reads whole. KV rows of
rejected drafts are simply overwritten by later rounds.

Reference behaviour: draft/verify accept-commit of
crates/spark-serve/src/request_api/speculation.rs:211-254 and the MTP tree
resolution of crates/spark-node/src/rank_daemon/work_control.rs (a chain is the
one-branch tree); the reference's drafter itself (X16) is absent from its tree.
"""
from __future__ import annotations

import torch

from .. import ops
from ..models.config import mtp_head
from ..models.mla_moe import ForwardBatch, KVCache, MLAMoEModel
from ..models.weights import init_weights


def make_draft(target: MLAMoEModel, seed: int = 1, max_positions: int | None = None) -> MLAMoEModel:
    """The 1-layer MTP-style draft head of ``target`` (same hidden size, one MLA
    layer and one dense FFN of width 1408), sharing the target's embedding and
    LM head."""
    cfg = mtp_head(target.cfg).replace(weight_dtype="bf16")
    w = init_weights(cfg, seed=seed, device=target.device,
                     share={"embed": target.w["embed"], "lm_head": target.w["lm_head"]})
    return MLAMoEModel(cfg, weights=w, device=target.device, max_positions=max_positions)


class SpecDecoder:
    def __init__(self, target: MLAMoEModel, draft: MLAMoEModel, target_cache: KVCache, draft_cache: KVCache,
                 batch: int, draft_len: int, max_blocks: int, max_context: int, p_accept: float = 0.0,
                 seed: int = 0, use_graph: bool = True):
        assert target_cache.block_size == draft_cache.block_size
        self.target, self.draft = target, draft
        self.tcache, self.dcache = target_cache, draft_cache
        self.B, self.L = batch, draft_len
        self.p_accept, self.seed = float(p_accept), int(seed)
        self.bs = target_cache.block_size
        dev = target.device
        R = (draft_len + 1) * batch
        self.R = R
        i32 = dict(dtype=torch.int32, device=dev)
        self.tok = torch.zeros(R, **i32)
        self.pos = torch.full((R,), -1, **i32)
        self.ctx = torch.zeros(R, **i32)
        self.slot = torch.full((R,), -1, **i32)
        self.tgt = torch.zeros(R, **i32)
        self.bt = torch.zeros(batch, max_blocks, **i32)
        self.bt_rows = torch.zeros(R, max_blocks, **i32)
        self.accepted = torch.zeros(batch, **i32)
        self.committed = torch.zeros(batch, draft_len + 1, **i32)
        self.total = torch.zeros(1, dtype=torch.int64, device=dev)
        nsm = ops.kernels().num_sms()
        B = batch
        self.dfb = [ForwardBatch(mode="decode", token_ids=self.tok[j * B:(j + 1) * B],
                                 positions=self.pos[j * B:(j + 1) * B], slot_mapping=self.slot[j * B:(j + 1) * B],
                                 block_table=self.bt, context_lens=self.ctx[j * B:(j + 1) * B],
                                 decode_splits=ops.mla_decode_splits(B, draft.cfg.num_heads, max_context, nsm))
                    for j in range(draft_len + 1)]
        self.vfb = ForwardBatch(mode="decode", token_ids=self.tok, positions=self.pos, slot_mapping=self.slot,
                                block_table=self.bt_rows, context_lens=self.ctx,
                                decode_splits=ops.mla_decode_splits(R, target.cfg.num_heads, max_context, nsm))
        self.use_graph = use_graph
        self.graph = None

    # ------------------------------------------------------------------ state
    def start(self, first_tokens: torch.Tensor, positions: torch.Tensor, block_table: torch.Tensor):
        """Sequences whose prompts are in both caches: ``first_tokens`` [B] (the
        target's token after each prompt) sits at ``positions`` [B] (= prompt
        lengths); ``block_table`` [B, max_blocks] is shared by both caches."""
        B, L, bs = self.B, self.L, self.bs
        dev = self.tok.device
        self.bt.copy_(block_table)
        self.bt_rows.copy_(block_table.repeat(L + 1, 1))
        self.tok[:B].copy_(first_tokens)
        p = positions.to(device=dev, dtype=torch.int64)
        rows = p[None, :] + torch.arange(L + 1, device=dev)[:, None]        # [L+1, B]
        blk = (rows // bs).clamp(max=block_table.shape[1] - 1)
        slots = block_table.to(dev).long().gather(1, blk.t()).t() * bs + rows % bs
        slots = torch.where(rows // bs < block_table.shape[1], slots, torch.full_like(slots, -1))
        cap = block_table.shape[1] * bs
        self.pos.copy_(rows.flatten().int())
        self.ctx.copy_((rows + 1).clamp(max=cap).flatten().int())
        self.slot.copy_(slots.flatten().int())
        self.total.zero_()

    # ------------------------------------------------------------------ one round
    def _round(self):
        B, L = self.B, self.L
        for j in range(L + 1):
            logits = self.draft.forward(self.dfb[j], self.dcache)
            if j < L:
                ops.sample_tokens(logits, 0.0, out_ids=self.tok[(j + 1) * B:(j + 2) * B])
        logits = self.target.forward(self.vfb, self.tcache)
        ops.sample_tokens(logits, 0.0, out_ids=self.tgt)
        ops.kernels().spec_finish(self.tok, self.tgt, L, self.p_accept, self.seed, self.pos, self.ctx, self.slot,
                                  self.bt, self.bs, self.accepted, self.committed, self.total)
        ops._count(1)

    def round(self):
        """Runs one round; returns (accepted [B], committed [B, L+1]) device tensors
        (committed: accepted drafts, then the verifier token, then -1)."""
        if self.graph is not None:
            self.graph.replay()
            return self.accepted, self.committed
        self._round()
        if not self.use_graph:
            return self.accepted, self.committed
        # the first round ran eagerly (kernel attributes set outside capture);
        # keep its result, then capture the round for replay
        acc, com = self.accepted.clone(), self.committed.clone()
        torch.cuda.synchronize()
        self.graph = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            with torch.cuda.graph(self.graph, stream=s):
                self._round()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        return acc, com

    def committed_tokens(self) -> int:
        return int(self.total.item())

    def release(self):
        self.graph = None
