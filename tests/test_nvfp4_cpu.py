"""NVFP4 format statement (ops/kernels.py): e2m1 rounding, the blocked scale layout and the
quantise / dequantise round trip, on CPU. The CUDA quantisers are checked against this statement
in tests/test_nvfp4_gpu.py."""
import torch

from appcorr_b200.ops import kernels as K


def test_e2m1_round_to_nearest_even():
    y = torch.tensor([0.0, 0.2, 0.25, 0.3, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.1, 7.0, -0.75, -6.0, -100.0])
    codes = K._e2m1_codes(y)
    table = torch.tensor(K.E2M1_VALUES + tuple(-v for v in K.E2M1_VALUES))
    got = table[codes.long()].tolist()
    assert got == [0.0, 0.0, 0.0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, -1.0, -6.0, -6.0]


def test_blocked_scale_offsets():
    idx = K.nvfp4_sf_index(300, 256)
    assert idx.shape == (300, 16)
    # row 33, block 5: tile (0, 1), row-in-32 1, 32-row group 1, block-in-tile 1
    assert idx[33, 5].item() == 512 + 1 * 16 + 1 * 4 + 1
    # row 130, block 0: tile (1, 0) with K / 64 = 4 tiles per row tile
    assert idx[130, 0].item() == 4 * 512 + 2 * 16
    # every byte of the first two row tiles is used exactly once
    flat = idx[:256].reshape(-1)
    assert flat.unique().numel() == flat.numel() and flat.max().item() < K.nvfp4_sf_bytes(256, 256)


def test_round_trip_exact_on_grid_and_error_bound():
    torch.manual_seed(0)
    # values already on the e2m1 grid with power-of-two block scales survive exactly
    g = torch.tensor(K.E2M1_VALUES)[torch.randint(0, 8, (128, 256))] * torch.where(torch.rand(128, 256) < 0.5, -1.0, 1.0)
    g[:, ::16] = 6.0  # every block reaches the e2m1 maximum, every row the same amax
    q, sf, rs = K.nvfp4_quantize_ref(g.to(torch.bfloat16))
    torch.testing.assert_close(K.nvfp4_dequantize(q, sf, rs), g, rtol=1e-6, atol=1e-6)
    x = torch.randn(200, 512) * 3
    x[7] = 0.0
    q, sf, rs = K.nvfp4_quantize_ref(x.to(torch.bfloat16))
    d = K.nvfp4_dequantize(q, sf, rs)
    assert d[7].abs().max().item() == 0.0
    err = ((d - x.bfloat16().float()).norm() / x.norm()).item()
    assert err < 0.12, err
    # per element: half the top e2m1 step (1/6 of the block amax) plus the ue4m3 rounding of the
    # block scale (at most 1/16 relative, which saturation can add on top)
    blk = x.bfloat16().float().view(200, 32, 16).abs().amax(2)
    e = (d - x.bfloat16().float()).abs().view(200, 32, 16).amax(2)
    assert (e <= blk * (1 / 6 + 1 / 16) + 1e-6).all()
