"""dSpark drafter: a block-parallel draft model fed by hidden-state taps of the
target model, with a low-rank Markov head and a confidence head, behind a
speculator that keeps per-sequence draft state and accounts verification.

Model. The target model's hidden states are captured after a few of its layers
(the "aux" layers, spread over the depth). For one sequence the taps of its last
position are concatenated and projected to the draft width: that is the draft
context. A block of ``block_size`` positions is drafted at once: position 0 holds
the last committed token, positions 1..block_size-1 a mask token. The draft layers
are pre-norm transformer blocks whose attention sees the context slot and the
whole block (bidirectional inside the block). The output head is the target's
vocabulary projection plus a Markov correction of rank ``markov_rank``, taken from
the token drafted just before each position (so a block resolves left to right in
one cheap pass after the layers). A confidence head gives each drafted token a
probability that the verifier accepts it; the speculator cuts the draft at the
first token below the minimum confidence.

Speculator. Per sequence: VALID -> TAPS_READY (taps captured for its position)
-> DRAFT_READY (tokens and confidences held) -> VERIFY_INFLIGHT -> back to VALID
once the verifier's tokens arrive; accepted = the longest prefix of the draft that
the verifier reproduces, committed = accepted + 1 (the verifier's own next token).

Reference behaviour: crates/spark-abi/vendor/sparkpipe/model-families/glm52/include/
sparkpipe/spark_glm52_dspark.h:30-311 (tap plan, model contract, sequence state
flags, speculator counters, confidence policy) and spark_glm52_model.h:55-71 (5 aux
layers, capture offset 1, 5 draft layers, block 8, at most 7 speculative tokens,
Markov rank 256). The network here is this framework's own reading of that contract.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch
import torch.nn as nn
import torch.nn.functional as F

CONFIDENCE_MILLI_ONE = 1000
FLAG_VALID, FLAG_TAPS_READY, FLAG_DRAFT_READY, FLAG_VERIFY_INFLIGHT = 0x1, 0x2, 0x4, 0x8
RESULT_CONFIDENCE_TRUNCATED = 0x1
VERIFY_ACCEPTED_ALL, VERIFY_REJECTED = 0x1, 0x2
AUX_CAPTURE_LAYER_OFFSET = 1


@dataclass
class DsparkContract:
    target_layers: int
    hidden: int
    vocab: int
    aux_layer_ids: list[int] = field(default_factory=list)  # empty: spread 5 over the depth
    draft_layers: int = 5
    block_size: int = 8
    max_speculative_tokens: int = 7
    heads: int = 8
    head_dim: int = 64
    intermediate: int = 0  # 0: 4 x hidden
    markov_rank: int = 256
    mask_token_id: int = 0
    min_confidence_milli: int = 350
    realtime_min_confidence_milli: int = 250

    def __post_init__(self):
        if not self.aux_layer_ids:
            n = 5
            self.aux_layer_ids = [round((i + 0.5) * self.target_layers / n) for i in range(n)]
        if not self.intermediate:
            self.intermediate = 4 * self.hidden
        self.validate()

    def validate(self):
        ids = self.aux_layer_ids
        if any(i < AUX_CAPTURE_LAYER_OFFSET or i > self.target_layers for i in ids) or sorted(set(ids)) != ids:
            raise ValueError("dspark: aux layer ids must be increasing and inside the target model")
        if not (1 <= self.max_speculative_tokens < self.block_size):
            raise ValueError("dspark: at most block_size - 1 speculative tokens")
        if not (0 < self.min_confidence_milli <= CONFIDENCE_MILLI_ONE):
            raise ValueError("dspark: confidence threshold in (0, 1000]")
        if self.markov_rank <= 0 or self.draft_layers <= 0 or not (0 <= self.mask_token_id < self.vocab):
            raise ValueError("dspark: bad contract")

    @property
    def capture_layers(self) -> list[int]:
        """Target layer after which each tap is captured."""
        return [i - AUX_CAPTURE_LAYER_OFFSET for i in self.aux_layer_ids]


def hidden_tap_plan(contract: DsparkContract, stage_layer_counts: list[int]) -> list[dict]:
    """Which pipeline stage captures each tap, and at which layer offset inside it."""
    if sum(stage_layer_counts) != contract.target_layers:
        raise ValueError("dspark: stages do not cover the target model")
    plan, first = [], 0
    bounds = []
    for s, n in enumerate(stage_layer_counts):
        bounds.append((s, first, n))
        first += n
    for layer in contract.capture_layers:
        s, f, n = next(b for b in bounds if b[1] <= layer < b[1] + b[2])
        plan.append(dict(target_layer_index=layer, stage_index=s, stage_first_layer_index=f,
                         stage_layer_count=n, layer_offset_in_stage=layer - f))
    return plan


class _RMSNorm(nn.Module):
    def __init__(self, d, eps=1e-6):
        super().__init__()
        self.w = nn.Parameter(torch.ones(d))
        self.eps = eps

    def forward(self, x):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps)).to(x.dtype) * self.w


class _DraftLayer(nn.Module):
    def __init__(self, c: DsparkContract):
        super().__init__()
        self.h, self.dh = c.heads, c.head_dim
        self.n1, self.n2 = _RMSNorm(c.hidden), _RMSNorm(c.hidden)
        self.qkv = nn.Linear(c.hidden, 3 * c.heads * c.head_dim, bias=False)
        self.o = nn.Linear(c.heads * c.head_dim, c.hidden, bias=False)
        self.gate_up = nn.Linear(c.hidden, 2 * c.intermediate, bias=False)
        self.down = nn.Linear(c.intermediate, c.hidden, bias=False)

    def forward(self, x):  # x: [B, 1 + block, hidden]; every slot sees every slot
        B, T, _ = x.shape
        q, k, v = self.qkv(self.n1(x)).view(B, T, 3, self.h, self.dh).permute(2, 0, 3, 1, 4)
        a = F.scaled_dot_product_attention(q, k, v)
        x = x + self.o(a.transpose(1, 2).reshape(B, T, -1))
        g, u = self.gate_up(self.n2(x)).chunk(2, -1)
        return x + self.down(F.silu(g) * u)


class DsparkDrafter(nn.Module):
    def __init__(self, c: DsparkContract, embed: torch.Tensor | None = None, lm_head: torch.Tensor | None = None):
        super().__init__()
        self.c = c
        n_taps = len(c.aux_layer_ids)
        self.embed = nn.Embedding(c.vocab, c.hidden)
        self.lm_head = nn.Linear(c.hidden, c.vocab, bias=False)
        if embed is not None:  # shared with the target model
            self.embed.weight = nn.Parameter(embed, requires_grad=False)
        if lm_head is not None:
            self.lm_head.weight = nn.Parameter(lm_head, requires_grad=False)
        self.fuse = nn.Linear(n_taps * c.hidden, c.hidden, bias=False)
        self.fuse_norm = _RMSNorm(c.hidden)
        self.pos = nn.Parameter(torch.zeros(c.block_size, c.hidden))
        self.layers = nn.ModuleList(_DraftLayer(c) for _ in range(c.draft_layers))
        self.norm = _RMSNorm(c.hidden)
        self.markov_in = nn.Embedding(c.vocab, c.markov_rank)
        self.markov_out = nn.Linear(c.markov_rank, c.vocab, bias=False)
        self.confidence = nn.Linear(c.hidden + c.markov_rank, 1)
        for p in (self.fuse.weight, self.markov_out.weight):
            nn.init.normal_(p, std=0.02 / math.sqrt(n_taps))

    @torch.no_grad()
    def forward(self, taps: torch.Tensor, last_token: torch.Tensor):
        """taps [B, n_taps, hidden] (last position of each sequence), last_token [B].
        Returns draft tokens [B, block-1] and confidences in [0, 1] [B, block-1]."""
        c = self.c
        B = taps.shape[0]
        ctx = self.fuse_norm(self.fuse(taps.reshape(B, -1).to(self.fuse.weight.dtype)))
        block = torch.full((B, c.block_size), c.mask_token_id, dtype=torch.long, device=taps.device)
        block[:, 0] = last_token
        x = torch.cat([ctx[:, None], self.embed(block) + self.pos], 1)
        for layer in self.layers:
            x = layer(x)
        h = self.norm(x[:, 2:])  # outputs for block positions 1..block-1
        base = self.lm_head(h).float()
        toks, conf = [], []
        prev = last_token
        for i in range(c.block_size - 1):  # Markov correction resolves left to right
            m = self.markov_in(prev)
            logits = base[:, i] + self.markov_out(m).float()
            t = logits.argmax(-1)
            toks.append(t)
            conf.append(torch.sigmoid(self.confidence(torch.cat([h[:, i], m.to(h.dtype)], -1)).float()).squeeze(-1))
            prev = t
        return torch.stack(toks, 1), torch.stack(conf, 1)


class DsparkSpeculator:
    """Per-sequence draft state, the confidence policy and acceptance accounting."""

    def __init__(self, drafter: DsparkDrafter, sequences: int, realtime: bool = False):
        self.d, self.c = drafter, drafter.c
        self.min_conf = self.c.realtime_min_confidence_milli if realtime else self.c.min_confidence_milli
        self.state = [dict(flags=0, request_id=0, sequence_id=0, position=0, tap_generation=0, draft_generation=0,
                           taps=None, last=0, tokens=[], conf=[]) for _ in range(sequences)]
        self.next_tap_generation = self.next_draft_generation = 1
        self.counters = dict(taps_ready=0, draft_requests=0, draft_success=0, rejected_by_confidence=0,
                             verify_dispatch=0, accepted=0, committed=0, rejected=0)

    def begin(self, slot, request_id, sequence_id, position):
        self.state[slot].update(flags=FLAG_VALID, request_id=request_id, sequence_id=sequence_id, position=position,
                                taps=None, tokens=[], conf=[])

    def taps_ready(self, slot, taps: torch.Tensor, last_token: int):
        s = self.state[slot]
        if not s["flags"] & FLAG_VALID or s["flags"] & (FLAG_DRAFT_READY | FLAG_VERIFY_INFLIGHT):
            raise RuntimeError("dspark: taps for a sequence that is not waiting for them")
        if taps.shape[-2:] != (len(self.c.aux_layer_ids), self.c.hidden):
            raise ValueError("dspark: tap shape")
        s.update(taps=taps, last=int(last_token), tap_generation=self.next_tap_generation)
        s["flags"] |= FLAG_TAPS_READY
        self.next_tap_generation += 1
        self.counters["taps_ready"] += 1

    def draft(self, slots: list[int], requested: int | None = None) -> dict[int, tuple[list[int], int]]:
        """Drafts every listed sequence in one batch: slot -> (tokens, result flags)."""
        n = min(requested or self.c.max_speculative_tokens, self.c.max_speculative_tokens)
        for sl in slots:
            if not self.state[sl]["flags"] & FLAG_TAPS_READY:
                raise RuntimeError("dspark: draft before the taps are ready")
        taps = torch.stack([self.state[sl]["taps"] for sl in slots])
        last = torch.tensor([self.state[sl]["last"] for sl in slots], device=taps.device)
        toks, conf = self.d(taps, last)
        out = {}
        for j, sl in enumerate(slots):
            s = self.state[sl]
            self.counters["draft_requests"] += 1
            milli = (conf[j, :n] * CONFIDENCE_MILLI_ONE).round().long().tolist()
            keep = next((i for i, m in enumerate(milli) if m < self.min_conf), n)
            flags = RESULT_CONFIDENCE_TRUNCATED if keep < n else 0
            s.update(tokens=toks[j, :keep].tolist(), conf=milli[:keep], draft_generation=self.next_draft_generation)
            self.next_draft_generation += 1
            s["flags"] = (s["flags"] & ~FLAG_TAPS_READY) | FLAG_DRAFT_READY
            if keep:
                self.counters["draft_success"] += 1
            else:
                self.counters["rejected_by_confidence"] += 1
            out[sl] = (s["tokens"], flags)
        return out

    def dispatch_verify(self, slot):
        s = self.state[slot]
        if not s["flags"] & FLAG_DRAFT_READY:
            raise RuntimeError("dspark: nothing drafted to verify")
        s["flags"] = (s["flags"] & ~FLAG_DRAFT_READY) | FLAG_VERIFY_INFLIGHT
        self.counters["verify_dispatch"] += 1
        return list(s["tokens"])

    def verify_result(self, slot, verifier_tokens: list[int]) -> tuple[int, int, int]:
        """verifier_tokens: the target's token at each draft position and one more.
        Returns (accepted, committed, flags)."""
        s = self.state[slot]
        if not s["flags"] & FLAG_VERIFY_INFLIGHT:
            raise RuntimeError("dspark: no verification in flight")
        d = s["tokens"]
        if len(verifier_tokens) < len(d) + 1:
            raise ValueError("dspark: the verifier returns one token per draft position and one more")
        acc = 0
        while acc < len(d) and d[acc] == verifier_tokens[acc]:
            acc += 1
        committed = acc + 1
        flags = VERIFY_ACCEPTED_ALL if acc == len(d) else VERIFY_REJECTED
        self.counters["accepted"] += acc
        self.counters["committed"] += committed
        self.counters["rejected"] += len(d) - acc
        s["position"] += committed
        s["flags"] = FLAG_VALID
        s.update(tokens=[], conf=[], taps=None)
        return acc, committed, flags
