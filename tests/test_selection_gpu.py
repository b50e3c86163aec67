"""Device-side token selection against the fp32 oracle: threshold selection with and without a
cap (reference block.py:360-395, 495-560) and the token-prune select + compact kernel
(triton_kernels/token_prune.py:9-89)."""
import pytest
import torch

from appcorr_b200.models.dinov3.layers import build_update_indice, select_keep_mask

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("cap", [0, 7, 40])
def test_threshold_plan_matches_oracle(cap):
    from appcorr_b200.ops import kernels as K

    torch.manual_seed(0)
    B, N, npre = 3, 69, 5
    P = N - npre
    server = torch.rand(B, N, device=DEV)
    server[2] *= 0.01  # nothing of image 2 passes: its plan repeats the first candidate
    pre = torch.arange(npre, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    cand = torch.stack([torch.randperm(P, device=DEV) + npre for _ in range(B)]).to(torch.int32).contiguous()
    thres = 0.6
    keep = select_keep_mask(server.gather(1, cand.long()), 0.0, thres)
    ref = build_update_indice(pre.long(), cand.long(), keep, cap, True)
    k = min(cap, P) if cap > 0 else P
    T = npre + k
    upd = torch.empty(B, T, device=DEV, dtype=torch.int32)
    rows = torch.empty(B * T, device=DEV, dtype=torch.int32)
    counts = torch.empty(B, device=DEV, dtype=torch.int32)
    K.correction_plan(server, pre, cand, k, upd, rows, thres=thres, counts=counts)
    torch.cuda.synchronize()
    assert torch.equal(counts.long(), keep.sum(1))
    if cap == 0:  # the oracle pads to the longest row; the kernel's full-width plan extends it
        upd = upd[:, : ref.shape[1]]
    assert torch.equal(upd.long(), ref), (upd, ref)
    assert torch.equal(rows.view(B, T)[:, : upd.shape[1]].long(),
                       upd.long() + torch.arange(B, device=DEV)[:, None] * N)


@pytest.mark.parametrize("cap", [0, 12])
def test_engine_threshold_correction_matches_oracle(cap):
    from appcorr_b200.models.dinov3 import build_vit
    from appcorr_b200.models.dinov3.layers import PartialTokenPlan
    from appcorr_b200.models.engine import ViTEngine

    torch.manual_seed(3)
    m = build_vit("vits16", depth=2).init_weights(0).eval()
    with torch.no_grad():
        for blk in m.blocks:
            blk.ls1.gamma.fill_(0.3)
            blk.ls2.gamma.fill_(0.3)
    m = m.to(DEV)
    eng = ViTEngine.from_module(m, DEV)
    B, H, W = 2, 96, 96
    img0 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    img1 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, H, W)
    eng.prepare_tokens(sess, img0)
    eng.approx(sess, 0, 2)
    N, npre = sess.N, m.n_storage_tokens + 1
    # threshold at the median of the layer-mean score: about half of the patches pass
    score = sess.pscore[:2].mean(0)[:, npre:]
    thres = float(score.median())
    opts = dict(token_keep_thres=thres, token_keep_cap=cap, server_pscore="cls_attn_prob_layermean")
    pre = torch.arange(npre, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    cand = torch.arange(npre, N, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    eng.prepare_tokens(sess, img1)
    x = eng.correct(sess, 0, 2, pre, cand, opts)
    torch.cuda.synchronize()
    keep = select_keep_mask(sess.extra["layermean"][:, npre:], 0.0, thres)
    upd = build_update_indice(pre.long(), cand.long(), keep, cap, True)
    mean = torch.tensor([0.485, 0.456, 0.406], device=DEV).view(1, 3, 1, 1)
    std = torch.tensor([0.229, 0.224, 0.225], device=DEV).view(1, 3, 1, 1)

    def f(u8):
        return (u8.permute(0, 3, 1, 2).float() / 255 - mean) / std

    with torch.no_grad():
        x0, (gh, gw) = m.prepare_tokens_with_masks(f(img0))
        rope = m.rope_embed(H=gh, W=gw)
        cache = {}
        for i, blk in enumerate(m.blocks):
            x0, cache = blk.approx(x0, rope, cache, f"layer{i}")
        xr, _ = m.prepare_tokens_with_masks(f(img1))
        plan = PartialTokenPlan(upd, torch.zeros(1), *(torch.zeros(()) for _ in range(5)))
        dind = torch.arange(N, device=DEV).repeat(B, 1)
        for i, blk in enumerate(m.blocks):
            xr, cache = blk.correct(xr, dind, rope, cache, f"layer{i}", query_plan=plan, **opts)
    rel = ((x.view(B, -1, m.embed_dim).float() - xr).norm() / xr.norm()).item()
    assert rel < 3e-2


def _prune_ref(x, xr, N, dind, npre, thr, min_keep):
    B, M = dind.shape
    rows = (torch.arange(B, device=DEV)[:, None] * N + dind.long())
    s = (x.float()[rows] - xr.float()[rows]).abs().mean(-1)
    dsel = torch.zeros_like(dind)
    qpos = torch.zeros_like(dind)
    valid = torch.zeros(B, M, dtype=torch.bool, device=DEV)
    cnt = torch.zeros(B, dtype=torch.int32, device=DEV)
    for b in range(B):
        ps = s[b, npre:]
        keep = torch.nonzero(ps >= thr).flatten()
        if ps.numel() > 0 and keep.numel() < min_keep:
            k = min(min_keep, ps.numel())
            order = sorted(range(ps.numel()), key=lambda i: (-float(ps[i]), i))[:k]
            keep = torch.tensor(sorted(order), device=DEV, dtype=torch.long)
        sel = torch.cat([torch.arange(npre, device=DEV), keep + npre])
        dsel[b, : sel.numel()] = dind[b, sel]
        qpos[b, : sel.numel()] = sel.to(torch.int32)
        valid[b, : sel.numel()] = True
        cnt[b] = keep.numel()
    return dsel, qpos, valid, cnt


@pytest.mark.parametrize("thr,min_keep", [(0.5, 1), (5.0, 9), (0.75, 40)])
def test_token_prune_matches_reference_rule(thr, min_keep):
    from appcorr_b200.ops import kernels as K

    torch.manual_seed(4)
    B, N, D, npre = 2, 90, 384, 5
    x = torch.randn(B * N, D, device=DEV).to(torch.bfloat16)
    xr = (x.float() + torch.randn(B * N, D, device=DEV) * torch.rand(B * N, 1, device=DEV) * 1.6).to(torch.bfloat16)
    dind = torch.cat([torch.arange(npre, device=DEV).repeat(B, 1),
                      torch.stack([torch.randperm(N - npre, device=DEV)[:50] + npre for _ in range(B)])], 1)
    dind = dind.to(torch.int32).contiguous()
    got = K.token_prune(x, xr, N, dind, npre, thr, min_keep)
    torch.cuda.synchronize()
    ref = _prune_ref(x, xr, N, dind, npre, thr, min_keep)
    for g, r in zip(got, ref):
        assert torch.equal(g, r), (g, r)
