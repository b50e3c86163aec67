"""The sm_100a ViT engine against the fp32 PyTorch oracle of the same approx / correct passes."""
import pytest
import torch

from appcorr_b200.models.dinov3 import build_vit
from appcorr_b200.models.dinov3.layers import PartialTokenPlan

pytestmark = pytest.mark.gpu
DEV = "cuda"
MEAN = torch.tensor([0.485, 0.456, 0.406]).view(1, 3, 1, 1)
STD = torch.tensor([0.229, 0.224, 0.225]).view(1, 3, 1, 1)


def _model(name, **over):
    m = build_vit(name, **over).init_weights(0).eval()
    g = torch.Generator().manual_seed(1)
    with torch.no_grad():
        for blk in m.blocks:
            blk.ls1.gamma.copy_(0.3 + 0.1 * torch.rand(blk.ls1.gamma.shape, generator=g))
            blk.ls2.gamma.copy_(0.3 + 0.1 * torch.rand(blk.ls2.gamma.shape, generator=g))
            for ln in (blk.norm1, blk.norm2):
                ln.weight.copy_(1 + 0.1 * torch.randn(ln.weight.shape, generator=g))
                ln.bias.copy_(0.1 * torch.randn(ln.bias.shape, generator=g))
            if getattr(blk.attn.qkv, "bias", None) is not None:
                blk.attn.qkv.bias.copy_(0.1 * torch.randn(blk.attn.qkv.bias.shape, generator=g))
    return m.to(DEV)


def _float_img(u8):
    return (u8.permute(0, 3, 1, 2).float() / 255 - MEAN.to(u8.device)) / STD.to(u8.device)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


CASES = [("vits16", dict(depth=3)), ("vit7b16", dict(depth=3, embed_dim=512, num_heads=4))]


@pytest.mark.parametrize("name,over", CASES)
def test_engine_approx_matches_oracle(name, over):
    from appcorr_b200.models.engine import ViTEngine

    torch.manual_seed(0)
    m = _model(name, **over)
    eng = ViTEngine.from_module(m, DEV)
    B, H, W = 2, 96, 128
    img = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, H, W)
    eng.prepare_tokens(sess, img)
    with torch.no_grad():
        x_ref, (gh, gw) = m.prepare_tokens_with_masks(_float_img(img))
        assert _rel(sess.x_in.view(B, -1, m.embed_dim), x_ref) < 1e-2
        x = eng.approx(sess, 0, len(m.blocks))
        rope = m.rope_embed(H=gh, W=gw)
        cache = {}
        xr = x_ref
        for i, blk in enumerate(m.blocks):
            xr, cache = blk.approx(xr, rope, cache, f"layer{i}")
    torch.cuda.synchronize()
    assert _rel(x.view(B, -1, m.embed_dim), xr) < 2e-2
    for i in range(len(m.blocks)):
        assert _rel(sess.kc[i].view_as(cache[f"layer{i}_k"]), cache[f"layer{i}_k"]) < 2e-2
        assert _rel(sess.bos[i].view(B, -1, m.embed_dim), cache[f"layer{i}_bos"]) < 3e-2
        assert _rel(sess.pscore[i], cache[f"layer{i}_server_pscore"]) < 1e-2


@pytest.mark.parametrize("name,over", CASES)
def test_engine_correct_matches_oracle(name, over):
    from appcorr_b200.models.engine import ViTEngine

    torch.manual_seed(1)
    m = _model(name, **over)
    eng = ViTEngine.from_module(m, DEV)
    B, H, W = 2, 96, 128
    img0 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    img1 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, H, W)
    eng.prepare_tokens(sess, img0)
    eng.approx(sess, 0, len(m.blocks))
    eng.prepare_tokens(sess, img1)
    N, P, npre = sess.N, sess.P, m.n_storage_tokens + 1
    pre = torch.arange(npre, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    cand = torch.arange(npre, N, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    opts = dict(token_keep_ratio=0.3, server_pscore="cls_attn_prob_layermean")
    x = eng.correct(sess, 0, len(m.blocks), pre, cand, opts)
    torch.cuda.synchronize()
    k = int(P * 0.3)
    upd = sess.upd.view(-1)[: B * (npre + k)].view(B, npre + k).long()
    with torch.no_grad():
        x0, (gh, gw) = m.prepare_tokens_with_masks(_float_img(img0))
        rope = m.rope_embed(H=gh, W=gw)
        cache = {}
        for i, blk in enumerate(m.blocks):
            x0, cache = blk.approx(x0, rope, cache, f"layer{i}")
        xr, _ = m.prepare_tokens_with_masks(_float_img(img1))
        plan = PartialTokenPlan(upd, torch.zeros(1), *(torch.zeros(()) for _ in range(5)))
        dind = torch.arange(N, device=DEV).repeat(B, 1)
        for i, blk in enumerate(m.blocks):
            xr, cache = blk.correct(xr, dind, rope, cache, f"layer{i}", query_plan=plan, **opts)
    assert _rel(x.view(B, -1, m.embed_dim), xr) < 3e-2
    for i in range(len(m.blocks)):
        assert _rel(sess.bos[i].view(B, -1, m.embed_dim), cache[f"layer{i}_bos"]) < 4e-2
        assert _rel(sess.vc[i].view_as(cache[f"layer{i}_v"]), cache[f"layer{i}_v"]) < 2e-2


def test_engine_full_correction_recovers_true_forward():
    """approx(base) + correct(all tokens, true image) == approx(true image) on the engine."""
    from appcorr_b200.models.engine import ViTEngine

    m = _model("vit7b16", depth=3, embed_dim=512, num_heads=4)
    eng = ViTEngine.from_module(m, DEV)
    B, H, W = 2, 64, 64
    base = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    true = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    s1 = eng.new_session(B, H, W)
    eng.prepare_tokens(s1, base)
    eng.approx(s1, 0, 3)
    eng.prepare_tokens(s1, true)
    npre = m.n_storage_tokens + 1
    pre = torch.arange(npre, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    cand = torch.arange(npre, s1.N, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    x1 = eng.correct(s1, 0, 3, pre, cand, dict(token_keep_ratio=1.0))
    s2 = eng.new_session(B, H, W)
    eng.prepare_tokens(s2, true)
    x2 = eng.approx(s2, 0, 3)
    torch.cuda.synchronize()
    assert _rel(x1, x2) < 1e-2


def test_detr_decoder_gpu_matches_module():
    from appcorr_b200.models.detr import DetrDecoder, DetrDecoderGPU

    torch.manual_seed(0)
    dec = DetrDecoder(384, d_model=256, heads=4, layers=2, num_queries=50, num_classes=80).to(DEV).eval()
    B, hw = 2, (8, 12)
    feat = torch.randn(B * 96, 384, device=DEV)
    with torch.no_grad():
        ref = dec(feat.view(B, 96, 384), hw)
    out = DetrDecoderGPU(dec, DEV).forward(feat.to(torch.bfloat16), B, hw)
    torch.cuda.synchronize()
    assert _rel(out["pred_logits"], ref["pred_logits"]) < 3e-2
    assert _rel(out["pred_boxes"], ref["pred_boxes"]) < 2e-2


@pytest.mark.parametrize("name,over", CASES)
def test_engine_fp8_tracks_oracle(name, over):
    """e4m3 activations x e4m3 weights (fp32 accumulate): approx and correct passes stay close
    to the fp32 oracle, and the correction pass of the full token set still recovers the
    image's true forward."""
    from appcorr_b200.models.engine import ViTEngine

    torch.manual_seed(2)
    m = _model(name, **over)
    eng = ViTEngine.from_module(m, DEV, precision="fp8")
    B, H, W = 2, 96, 128
    img = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, H, W)
    eng.prepare_tokens(sess, img)
    with torch.no_grad():
        x_ref, (gh, gw) = m.prepare_tokens_with_masks(_float_img(img))
        x = eng.approx(sess, 0, len(m.blocks)).clone()
        rope = m.rope_embed(H=gh, W=gw)
        cache = {}
        xr = x_ref
        for i, blk in enumerate(m.blocks):
            xr, cache = blk.approx(xr, rope, cache, f"layer{i}")
    torch.cuda.synchronize()
    assert _rel(x.view(B, -1, m.embed_dim), xr) < 6e-2
    for i in range(len(m.blocks)):
        assert _rel(sess.pscore[i], cache[f"layer{i}_server_pscore"]) < 5e-2
    # correction with every patch token kept == full forward on the same image
    npre = m.n_storage_tokens + 1
    N = sess.N
    pre = torch.arange(npre, device=DEV, dtype=torch.int32)[None].repeat(B, 1).contiguous()
    cand = torch.arange(npre, N, device=DEV, dtype=torch.int32)[None].repeat(B, 1).contiguous()
    xc = eng.correct(sess, 0, len(m.blocks), pre, cand, {"token_keep_ratio": 1.0})
    torch.cuda.synchronize()
    assert _rel(xc.view(B, -1, m.embed_dim), xr) < 6e-2


@pytest.mark.parametrize("precision,kind", [("bf16", "cls_attn_prob_layermean"), ("nvfp4", "patch_attn_prob")])
def test_engine_graph_replay_matches_eager(precision, kind):
    """Passes run through ViTEngine.run_graphed (eager, then captured, then replayed) give the same
    bytes as eager passes over a sequence of requests with new images each time, including the
    Python-side state the replay re-applies (the layer-mean score entry that the approximate pass
    drops and the correction pass rebuilds)."""
    from appcorr_b200.models.engine import ViTEngine

    m = _model("vit7b16", depth=3, embed_dim=512, num_heads=4)
    B, H, W = 2, 64, 64
    npre = m.cfg.n_prefix
    opts = {"token_keep_ratio": 0.4, "server_pscore": kind}
    outs = {}
    for graphs in (True, False):
        eng = ViTEngine.from_module(m, DEV, precision=precision)
        eng.graphs_enabled = graphs
        sess = eng.new_session(B, H, W)
        pre = torch.arange(npre, dtype=torch.int32, device=DEV).repeat(B, 1).contiguous()
        cand = torch.arange(npre, sess.N, dtype=torch.int32, device=DEV).repeat(B, 1).contiguous()
        g = torch.Generator(device=DEV).manual_seed(0)
        res = []
        for _ in range(4):
            img0 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV, generator=g)
            img1 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV, generator=g)
            eng.prepare_tokens(sess, img0)
            x = eng.run_graphed(sess, ("approx", 0, 3, kind), lambda: eng.approx(sess, 0, 3, kind))
            res.append(x.clone())
            eng.prepare_tokens(sess, img1)
            xc = eng.run_graphed(sess, ("correct", 0, 3), lambda: eng.correct(sess, 0, 3, pre, cand, opts))
            res.append(xc.clone())
            res.append(eng.patch_features(sess).clone())
            res.append(sess.upd.clone())
        torch.cuda.synchronize()
        outs[graphs] = res
        if graphs:
            assert len(sess._graphs) == 2 and all(isinstance(v, tuple) for v in sess._graphs.values())
    for a, b in zip(outs[True], outs[False]):
        assert torch.equal(a, b)
