"""NVFP4 weight format: packing, the torch oracle's error bound, exact round trip of
representable values, and (GPU) the sm_100a expansion kernel against the oracle."""
import pytest
import torch

from sparkpipe_rs_b200.ops.nvfp4 import dequant_nvfp4_ref, quant_nvfp4


def test_pack_layout_and_exact_values():
    # one block holding every E2M1 code with a block scale of 1 and tensor scale chosen so
    grid = torch.tensor([0, 0.5, 1, 1.5, 2, 3, 4, 6, -0.5, -1, -1.5, -2, -3, -4, -6, 0.0])
    w = grid[None] * (448 / 448)  # amax 6 -> tensor scale 6 / (6 * 448), block scale 448
    q = quant_nvfp4(w)
    assert q.packed.shape == (1, 8) and q.scales.shape == (1, 1) and q.packed.dtype == torch.uint8
    assert int(q.packed[0, 0]) == (0x1 << 4) | 0x0  # 0 (low nibble), 0.5 (high nibble)
    assert torch.equal(dequant_nvfp4_ref(q), w)


def test_error_bound():
    torch.manual_seed(0)
    w = torch.randn(64, 256)
    q = quant_nvfp4(w)
    r = dequant_nvfp4_ref(q)
    blocks = w.reshape(-1, 16)
    s = q.scales.reshape(-1).view(torch.float8_e4m3fn).float() * q.tensor_scale
    # E2M1 spacing is at most 2 (between 4 and 6) in scaled units: error <= 1 x scale,
    # plus the clamp of values the rounded block scale left above 6
    err = (r.reshape(-1, 16) - blocks).abs()
    assert (err <= s[:, None] * 1.0 + blocks.abs().amax(-1, keepdim=True) * 0.07 + 1e-6).all()
    rel = (r - w).norm() / w.norm()
    assert rel < 0.12
    assert q.nbytes < w.numel() * 0.6  # ~4.5 bits per element


def test_zero_and_bad_shape():
    q = quant_nvfp4(torch.zeros(2, 32))
    assert torch.equal(dequant_nvfp4_ref(q), torch.zeros(2, 32))
    with pytest.raises(ValueError):
        quant_nvfp4(torch.zeros(2, 24))


@pytest.mark.gpu
def test_dequant_kernel_matches_oracle():
    from sparkpipe_rs_b200.ops.nvfp4 import dequant_nvfp4, linear_nvfp4

    torch.manual_seed(1)
    w = torch.randn(384, 2048, device="cuda")
    q = quant_nvfp4(w)
    out = dequant_nvfp4(q)
    ref = dequant_nvfp4_ref(q)
    torch.cuda.synchronize()
    assert torch.equal(out.float(), ref.bfloat16().float())
    x = torch.randn(8, 2048, device="cuda").bfloat16()
    y = linear_nvfp4(x, q)
    assert torch.allclose(y.float(), x.float() @ ref.t(), rtol=2e-2, atol=2e-1)
