"""DSA index-share sideband: transport row layout (matches the ring geometry's row
size), pack / unpack round trip, and the per-step selection cache."""
import pytest
import torch

from sparkpipe_rs_b200.core import core
from sparkpipe_rs_b200.parallel.dsa_sideband import IndexShare, pack, row_bytes, unpack


def test_round_trip_and_row_size():
    torch.manual_seed(0)
    R, H, k = 5, 64, 12
    h = torch.randn(R, H).bfloat16()
    sel = torch.randint(-1, 4096, (R, k), dtype=torch.int32)
    buf = pack(h, sel)
    assert buf.shape == (R, row_bytes(H, k)) and buf.dtype == torch.uint8
    h2, s2 = unpack(buf, H, k)
    assert torch.equal(h2, h) and torch.equal(s2, sel)
    # views of the transport buffer, not copies
    assert h2.data_ptr() == buf.data_ptr() and s2.data_ptr() == buf.data_ptr() + 2 * H
    assert h2.stride(0) * 2 == row_bytes(H, k) and s2.stride(0) * 4 == row_bytes(H, k)
    buf[1, 2 * H:2 * H + 4] = torch.tensor([7, 0, 0, 0], dtype=torch.uint8)
    assert s2[1, 0].item() == 7
    # an odd hidden size misaligns the int32 columns: copies, same values
    h3, s3 = unpack(pack(h[:, :63].contiguous(), sel), 63, k)
    assert torch.equal(h3, h[:, :63]) and torch.equal(s3, sel)
    g = core().ring_runtime.Geometry()
    g.hidden_dimension, g.dsa_index_bytes_per_sequence = H, 4 * k
    assert g.transport_bytes_per_row() == row_bytes(H, k)
    with pytest.raises(TypeError):
        pack(h.float(), sel)
    with pytest.raises(ValueError):
        unpack(buf[:, :-4], H, k)


def test_index_share_cache():
    c = IndexShare()
    assert c.lookup(3) is None
    sel, cnt = torch.zeros(2, 4, dtype=torch.int32), torch.tensor([4, 2])
    c.publish(3, sel, cnt)
    assert c.lookup(3)[1] is cnt and c.lookup(4) is None
