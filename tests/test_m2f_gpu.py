"""Deformable attention kernel and the Mask2Former-style head against fp32 PyTorch references."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("Dh", [8, 16, 32, 64, 128])
def test_msda_kernel_matches_grid_sample(Dh):
    from appcorr_b200.models.m2f import msda_reference
    from appcorr_b200.ops import kernels as K

    torch.manual_seed(0)
    N, M, L, P, Q = 2, 8 if Dh <= 32 else 4, 3, 4, 37
    shapes = [(16, 20), (8, 10), (4, 5)]
    S = sum(h * w for h, w in shapes)
    value = torch.randn(N, S, M, Dh, device=DEV).to(torch.bfloat16)
    ref = torch.rand(N, Q, L, 2, device=DEV)
    offs = (torch.randn(N * Q, M * L * P * 2, device=DEV) * 3).to(torch.bfloat16)
    logits = torch.randn(N * Q, M * L * P, device=DEV).to(torch.bfloat16)
    out = torch.empty(N, Q, M * Dh, device=DEV, dtype=torch.bfloat16)
    K.msda(value, ref, offs, logits, out, [v for hw in shapes for v in hw], M, L, P)
    norm = torch.tensor([[w, h] for h, w in shapes], device=DEV, dtype=torch.float32)
    off = offs.float().view(N, Q, M, L, P, 2)
    loc = ref[:, :, None, :, None, :] + off / norm[None, None, None, :, None, :]
    w = logits.float().view(N, Q, M, L * P).softmax(-1).view(N, Q, M, L, P)
    exp = msda_reference(value.float(), shapes, loc, w)
    err = (out.float() - exp).abs().max().item()
    assert err < 2e-2 * exp.abs().max().item() + 1e-2, err
