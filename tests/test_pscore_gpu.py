"""Server patch scores on the GPU path against the fp32 oracle (reference attention.py:241-274):
the tcgen05 column-sum kernel (patch_attn_prob), the pseudo-query score
(patch_pseudo_attn_prob) and the engine's approximate pass for every server_pscore kind."""
import math

import pytest
import torch

from appcorr_b200.models.dinov3.layers import server_pscore_from_qk

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("B,N,H,Dh", [(2, 300, 4, 64), (1, 1029, 2, 128), (3, 69, 3, 128), (2, 128, 2, 64)])
def test_attn_colsum_matches_fp32(B, N, H, Dh):
    from appcorr_b200.ops import kernels as K

    torch.manual_seed(0)
    q = (torch.randn(B * N, H * Dh, device=DEV) * 1.5).to(torch.bfloat16)
    k = (torch.randn(B * N, H * Dh, device=DEV) * 1.5).to(torch.bfloat16)
    v = torch.randn(B * N, H * Dh, device=DEV).to(torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, N, device=DEV)
    K.attention(q, k, v, o, B=B, Tq=N, Tk=N, H=H, Dh=Dh, lse=lse, impl="tcgen05")
    probs = torch.empty(B, H, N, device=DEV)
    out = torch.empty(B, N, device=DEV)
    K.attn_colsum_pscore(q, k, lse, B=B, N=N, H=H, Dh=Dh, probs=probs, out=out)
    torch.cuda.synchronize()
    qf = q.float().view(B, N, H, Dh)
    kf = k.float().view(B, N, H, Dh)
    p = (torch.einsum("bihd,bjhd->bhij", qf, kf) / math.sqrt(Dh)).softmax(-1)
    ref_probs = p.mean(2)
    assert _rel(probs, ref_probs) < 1e-2
    assert _rel(out, ref_probs.mean(1)) < 1e-2
    # probabilities of every query sum to 1, so each head's column means sum to 1
    torch.testing.assert_close(probs.sum(-1), torch.ones(B, H, device=DEV), rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("B,N,npre,H,Dh", [(2, 69, 5, 4, 64), (2, 261, 5, 32, 128)])
def test_pseudo_query_score_matches_fp32(B, N, npre, H, Dh):
    from appcorr_b200.ops import kernels as K

    torch.manual_seed(1)
    q = torch.randn(B * N, H * Dh, device=DEV).to(torch.bfloat16)
    k = torch.randn(B * N, H * Dh, device=DEV).to(torch.bfloat16)
    pq = torch.empty(B, H * Dh, device=DEV, dtype=torch.bfloat16)
    K.pseudo_query(q, B=B, N=N, npre=npre, H=H, Dh=Dh, out=pq)
    out = torch.empty(B, N, device=DEV)
    K.query_attn_pscore(pq, k, B=B, N=N, H=H, Dh=Dh, scratch=torch.empty(B, H, N, device=DEV), out=out)
    torch.cuda.synchronize()
    ref = server_pscore_from_qk(q.view(B, N, H, Dh), k.view(B, N, H, Dh), "patch_pseudo_attn_prob", Dh ** -0.5,
                                N - npre)
    assert _rel(out, ref) < 2e-2


KINDS = ["cls_attn_prob", "patch_attn_prob", "patch_attn_prob_layermean", "patch_pseudo_attn_prob",
         "patch_pseudo_attn_prob_layermean", "cls_attn_prob_layermean"]


@pytest.mark.parametrize("kind", KINDS)
def test_engine_scores_match_oracle_7b_shape(kind):
    """A ViT-7B-shaped stack (width 4096, 32 heads of 128, SwiGLU, 4 registers; 2 layers): the
    engine's per-layer server scores against the fp32 oracle's, and the layer-mean the correction
    pass uses."""
    from appcorr_b200.models.dinov3 import build_vit
    from appcorr_b200.models.engine import ViTEngine

    torch.manual_seed(0)
    m = build_vit("vit7b16", depth=2).init_weights(0).eval()
    with torch.no_grad():
        for blk in m.blocks:
            blk.ls1.gamma.fill_(0.3)
            blk.ls2.gamma.fill_(0.3)
    m = m.to(DEV)
    eng = ViTEngine.from_module(m, DEV)
    B, H, W = 2, 128, 160
    img = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, H, W)
    eng.prepare_tokens(sess, img)
    eng.approx(sess, 0, 2, kind)
    mean = torch.tensor([0.485, 0.456, 0.406], device=DEV).view(1, 3, 1, 1)
    std = torch.tensor([0.229, 0.224, 0.225], device=DEV).view(1, 3, 1, 1)
    with torch.no_grad():
        xr, (gh, gw) = m.prepare_tokens_with_masks((img.permute(0, 3, 1, 2).float() / 255 - mean) / std)
        rope = m.rope_embed(H=gh, W=gw)
        cache = {}
        for i, blk in enumerate(m.blocks):
            xr, cache = blk.approx(xr, rope, cache, f"layer{i}", server_pscore=kind)
    torch.cuda.synchronize()
    for i in range(2):
        assert _rel(sess.pscore[i], cache[f"layer{i}_server_pscore"]) < 3e-2, i
    if kind.endswith("layermean"):
        # the correction pass plans on the mean over the approximate layers
        pre = torch.arange(5, dtype=torch.int32, device=DEV).repeat(B, 1).contiguous()
        cand = torch.arange(5, sess.N, dtype=torch.int32, device=DEV).repeat(B, 1).contiguous()
        eng.prepare_tokens(sess, img)
        eng.correct(sess, 0, 2, pre, cand, {"token_keep_ratio": 0.5, "server_pscore": kind})
        torch.cuda.synchronize()
        ref_mean = type(m.blocks[0]).server_scores(cache, "layer0", kind)
        assert _rel(sess.extra["layermean"], ref_mean) < 3e-2


def test_engine_rejects_unknown_score():
    from appcorr_b200.models.dinov3.vit import ViTConfig
    from appcorr_b200.models.engine import ViTEngine

    cfg = ViTConfig(embed_dim=128, depth=1, num_heads=2)
    eng = ViTEngine.random(cfg, torch.device(DEV))
    sess = eng.new_session(1, 32, 32)
    eng.prepare_tokens(sess, torch.zeros(1, 32, 32, 3, dtype=torch.uint8, device=DEV))
    with pytest.raises(ValueError, match="server_pscore"):
        eng.approx(sess, 0, 1, "bogus_score")
