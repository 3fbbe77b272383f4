"""DSA index-share sideband: the pipeline stage that runs the DSA indexer exports
each row's selected token positions next to its hidden state, and later stages
reuse that selection instead of running their own indexer.

Transport row layout (layer-major, one row per execution row): the row's hidden
state as bf16 (hidden x 2 bytes) followed by its selected positions as int32
(selected x 4 bytes, -1 padding past the row's count). ``pack`` writes rows into
one contiguous uint8 buffer (a single NVLink / fabric transfer per step); ``unpack``
returns strided views into it (row stride = the row size), so the receiving stage
reads hidden rows and indices without a copy; an odd hidden size (int32 columns off
their 4-byte alignment) or a non-contiguous buffer falls back to copies. The row size equals the ring geometry's ``transport_bytes_per_row`` with
``dsa_index_bytes_per_sequence = selected x 4``.

Reference behaviour: the DSA index-share sidebands of the production topology and
the layer-major transport row (hidden bf16 bytes + DSA selected index bytes) of
crates/spark-node/src/rank_daemon/ring_runtime.rs:222-300
(``layer_major_transport_bytes_per_row``).
"""
from __future__ import annotations

import torch


def row_bytes(hidden: int, selected: int) -> int:
    return hidden * 2 + selected * 4


def pack(hidden_rows: torch.Tensor, selected: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """hidden_rows [R, H] bf16, selected [R, k] int32 -> uint8 [R, row_bytes]."""
    if hidden_rows.dtype != torch.bfloat16 or selected.dtype != torch.int32:
        raise TypeError("dsa sideband: bf16 hidden rows and int32 selections")
    R, H = hidden_rows.shape
    if selected.shape[0] != R:
        raise ValueError("dsa sideband: one selection per row")
    k = selected.shape[1]
    if out is None:
        out = torch.empty(R, row_bytes(H, k), dtype=torch.uint8, device=hidden_rows.device)
    if out.shape != (R, row_bytes(H, k)):
        raise ValueError("dsa sideband: output buffer shape")
    out[:, : 2 * H].copy_(hidden_rows.contiguous().view(torch.uint8).view(R, 2 * H))
    out[:, 2 * H:].copy_(selected.contiguous().view(torch.uint8).view(R, 4 * k))
    return out


def unpack(buf: torch.Tensor, hidden: int, selected: int) -> tuple[torch.Tensor, torch.Tensor]:
    """uint8 [R, row_bytes] -> (hidden rows [R, H] bf16, selections [R, k] int32): strided
    views of ``buf`` when it is contiguous with 4-byte aligned rows and columns, else copies."""
    R = buf.shape[0]
    rb = row_bytes(hidden, selected)
    if buf.shape[1] != rb:
        raise ValueError("dsa sideband: row size")
    if buf.is_contiguous() and hidden % 2 == 0 and buf.storage_offset() % 4 == 0:
        return buf.view(torch.bfloat16)[:, :hidden], buf.view(torch.int32)[:, hidden // 2:hidden // 2 + selected]
    h = buf[:, : 2 * hidden].contiguous().view(torch.bfloat16)
    s = buf[:, 2 * hidden:].contiguous().view(torch.int32)
    return h.view(R, hidden), s.view(R, selected)


class IndexShare:
    """Per-step selection cache of a stage: the exporting stage publishes, the
    following stages reuse while the step generation matches."""

    def __init__(self):
        self.generation, self.selected, self.counts = -1, None, None

    def publish(self, generation: int, selected: torch.Tensor, counts: torch.Tensor):
        self.generation, self.selected, self.counts = generation, selected, counts

    def lookup(self, generation: int):
        if generation != self.generation or self.selected is None:
            return None
        return self.selected, self.counts
