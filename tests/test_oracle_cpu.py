"""CPU fp32 oracle: the approximate / correct partial-token semantics of the DINOv3 block."""
import pytest
import torch

from appcorr_b200.models.dinov3 import build_vit, create_group_index
from appcorr_b200.models.dinov3.vit import ViTConfig, DinoVisionTransformer


def _model(name="vits16", seed=0, **over):
    m = build_vit(name, depth=3, **over).init_weights(seed).eval()
    with torch.no_grad():
        for blk in m.blocks:  # make the increments matter (the init LayerScale is 1e-5)
            blk.ls1.gamma.fill_(0.5)
            blk.ls2.gamma.fill_(0.5)
    return m


def _run_approx(m, img):
    x, (H, W) = m.prepare_tokens_with_masks(img)
    rope = m.rope_embed(H=H, W=W)
    cache = {}
    for i, blk in enumerate(m.blocks):
        x, cache = blk.approx(x, rope, cache, f"layer{i}")
    return x, rope, cache


@torch.no_grad()
@pytest.mark.parametrize("name,over", [("vits16", {}), ("vit7b16", dict(embed_dim=256, num_heads=2))])
def test_approx_equals_stock_forward(name, over):
    m = _model(name, **over)
    img = torch.rand(2, 3, 64, 64)
    x, _, cache = _run_approx(m, img)
    ref = m.forward_features(img)["x_prenorm"]
    assert torch.allclose(x, ref, atol=1e-5, rtol=1e-5)
    assert cache["layer0_k"].shape == (2, 21, m.num_heads, m.embed_dim // m.num_heads)


@torch.no_grad()
def test_full_correction_recovers_true_forward():
    """approx(blurred) + correct(every token of the true image) == stock(true image)."""
    m = _model()
    true = torch.rand(2, 3, 64, 64)
    blur = torch.nn.functional.avg_pool2d(true, 2).repeat_interleave(2, -1).repeat_interleave(2, -2)
    _, rope, cache = _run_approx(m, blur)
    x, _ = m.prepare_tokens_with_masks(true)
    B, N = x.shape[:2]
    dindice = torch.arange(N).repeat(B, 1)
    opts = dict(token_keep_ratio=1.0, server_pscore="cls_attn_prob")
    for i, blk in enumerate(m.blocks):
        x, cache = blk.correct(x, dindice, rope, cache, f"layer{i}", **opts)
    ref = m.forward_features(true)["x_prenorm"]
    assert torch.allclose(x, ref, atol=1e-4, rtol=1e-4)


@torch.no_grad()
def test_partial_correction_only_touches_selected_rows():
    m = _model()
    img0 = torch.rand(1, 3, 64, 64)
    _, rope, cache = _run_approx(m, img0)
    x, _ = m.prepare_tokens_with_masks(torch.rand(1, 3, 64, 64))
    N = x.shape[1]
    dindice = torch.arange(N).repeat(1, 1)
    blk = m.blocks[0]
    bos0 = cache["layer0_bos"].clone()
    out, cache = blk.correct(x, dindice, rope, cache, "layer0", token_keep_ratio=0.25, server_pscore="cls_attn_prob")
    upd = cache["layer0_plan"].update_indice[0]
    assert upd.shape[0] == 5 + 4  # prefix + int(16 * 0.25)
    assert torch.all(upd[5:].diff() > 0)
    keep = torch.zeros(N, dtype=torch.bool)
    keep[upd] = True
    # untouched rows are x + approx increment
    assert torch.allclose(out[0, ~keep], x[0, ~keep] + bos0[0, ~keep], atol=1e-6)
    # selected rows' increment was persisted
    assert torch.allclose(cache["layer0_bos"][0, keep], out[0, keep] - x[0, keep], atol=1e-5)


@torch.no_grad()
def test_topk_selects_highest_scores():
    m = _model()
    _, rope, cache = _run_approx(m, torch.rand(2, 3, 64, 64))
    x, _ = m.prepare_tokens_with_masks(torch.rand(2, 3, 64, 64))
    dindice = torch.arange(21).repeat(2, 1)
    plan = m.blocks[1].make_plan(cache, "layer1", dindice, 5, dict(token_keep_ratio=0.5, server_pscore="cls_attn_prob"))
    s = cache["layer1_server_pscore"][:, 5:]
    top = torch.topk(s, 8, dim=1).indices.sort(1).values + 5
    assert torch.equal(plan.update_indice[:, 5:], top)


def test_group_index_strategies():
    g = create_group_index(16, 4, "grid", token_hw=(4, 4))
    assert g.tolist() == [1, 2, 1, 2, 3, 4, 3, 4, 1, 2, 1, 2, 3, 4, 3, 4]
    bg = create_group_index(16, 4, "block_grid", token_hw=(4, 4))
    assert bg.tolist() == [1, 1, 2, 2, 1, 1, 2, 2, 3, 3, 4, 4, 3, 3, 4, 4]
    e = create_group_index(64, 4, "expansion", token_hw=(8, 8))
    assert sorted(torch.bincount(e)[1:].tolist()) == [16, 16, 16, 16]
    assert e.view(8, 8)[3, 3] == 1 and e.view(8, 8)[0, 0] == 4


def test_state_dict_keys_match_dinov3_layout():
    m = build_vit("vit7b16", depth=1, embed_dim=256, num_heads=2)
    keys = set(m.state_dict().keys())
    for k in ["cls_token", "storage_tokens", "mask_token", "patch_embed.proj.weight", "rope_embed.periods",
              "blocks.0.attn.qkv.weight", "blocks.0.ls1.gamma",
              "blocks.0.mlp.w1.weight", "blocks.0.mlp.w3.bias", "norm.weight", "local_cls_norm.weight"]:
        assert k in keys, k
    small = build_vit("vits16", depth=1)
    assert "blocks.0.attn.qkv.bias_mask" in small.state_dict()
    assert "blocks.0.mlp.fc1.weight" in small.state_dict()


def test_qwen_oracle_window_order_and_full_correction():
    """Window-major order is a permutation whose merge units are contiguous; correcting every
    row of the VLM LLM reproduces its approximate (full) forward exactly."""
    from appcorr_b200.models.qwen25vl import (PRESETS, Qwen25VL, merge_raster_index, mrope_positions,
                                              mrope_tables, window_order)

    order = window_order(16, 24, 8, 2)
    assert sorted(order.tolist()) == list(range(16 * 24))
    units = order.view(-1, 4)
    ys, xs = units // 24, units % 24
    assert bool(((ys // 2) == (ys[:, :1] // 2)).all()) and bool(((xs // 2) == (xs[:, :1] // 2)).all())
    inv = merge_raster_index(PRESETS["tiny"], 16, 24)
    assert sorted(inv.tolist()) == list(range(8 * 12))
    cfg = PRESETS["tiny"]
    torch.manual_seed(0)
    m = Qwen25VL(cfg).init_weights(0)
    img = torch.randint(0, 256, (224, 224, 3), dtype=torch.uint8)
    with torch.no_grad():
        emb = m.visual(img)
        s, c = mrope_tables(cfg, mrope_positions(8, 8, 8, 24))
        x0 = m.embed(torch.arange(8), emb, torch.arange(24))
        cache = {}
        x = x0
        for i, ly in enumerate(m.layers):
            x = ly.approx(x, s, c, cache, f"l{i}")
        x2 = x0
        for i, ly in enumerate(m.layers):
            x2 = ly.correct(x2, torch.arange(x0.shape[0]), s, c, cache, f"l{i}")
    assert torch.allclose(x, x2, atol=1e-5)


def test_msda_reference_matches_direct_bilinear():
    """The deformable-sampling oracle equals a direct per-point bilinear sum (zeros outside)."""
    from appcorr_b200.models.m2f import msda_reference

    torch.manual_seed(0)
    N, M, Dh, L, P, Q = 1, 2, 4, 2, 3, 5
    shapes = [(5, 6), (3, 4)]
    S = sum(h * w for h, w in shapes)
    value = torch.randn(N, S, M, Dh, dtype=torch.float64)
    loc = torch.rand(N, Q, M, L, P, 2, dtype=torch.float64) * 1.4 - 0.2
    w = torch.rand(N, Q, M, L, P, dtype=torch.float64)
    got = msda_reference(value, shapes, loc, w).view(N, Q, M, Dh)
    starts = [0, shapes[0][0] * shapes[0][1]]
    exp = torch.zeros(N, Q, M, Dh, dtype=torch.float64)
    for q in range(Q):
        for m in range(M):
            for l, (h, wd) in enumerate(shapes):
                for p in range(P):
                    x = loc[0, q, m, l, p, 0].item() * wd - 0.5
                    y = loc[0, q, m, l, p, 1].item() * h - 0.5
                    x0, y0 = int(torch.floor(torch.tensor(x))), int(torch.floor(torch.tensor(y)))
                    for cx, cy, cw in ((x0, y0, (1 - (x - x0)) * (1 - (y - y0))), (x0 + 1, y0, (x - x0) * (1 - (y - y0))),
                                       (x0, y0 + 1, (1 - (x - x0)) * (y - y0)), (x0 + 1, y0 + 1, (x - x0) * (y - y0))):
                        if 0 <= cx < wd and 0 <= cy < h:
                            exp[0, q, m] += w[0, q, m, l, p] * cw * value[0, starts[l] + cy * wd + cx, m]
    assert torch.allclose(got.double(), exp, atol=1e-5)


def test_realesrgan_key_conversion_loads_strictly():
    from appcorr_b200.models.conv import RRDBNet
    from appcorr_b200.server.sr import convert_realesrgan_state

    net = RRDBNet(nf=8, nb=2, gc=4)
    ref = {}
    for k, v in net.state_dict().items():  # rebuild the Real-ESRGAN layout from our names
        k = k.replace("conv_up.0.", "conv_up1.").replace("conv_up.1.", "conv_up2.")
        parts = k.split(".")
        if parts[0] == "body":
            k = f"body.{parts[1]}.rdb{int(parts[3]) + 1}.conv{int(parts[5]) + 1}.{parts[6]}"
        ref[k] = v
    net.load_state_dict(convert_realesrgan_state({"params_ema": ref}), strict=True)


def test_graph_replay_state_delta():
    """The Python-side effects that ViTEngine.run_graphed records around a captured pass (session
    attributes, `extra` entries set, replaced or removed, also on micro-batch sub-sessions, and the
    engine's precision flags) are re-applied exactly on replay."""
    import types

    import torch

    from appcorr_b200.models.engine import ViTEngine

    eng = types.SimpleNamespace(_GRAPH_ENGINE_ATTRS=ViTEngine._GRAPH_ENGINE_ATTRS, _fp4=False, _fp8=False)
    sub = types.SimpleNamespace(approx_done=0, extra={"k": 1})
    sess = types.SimpleNamespace(approx_done=0, extra={"layermean": torch.zeros(1), "plan_id": 3, "subs": [sub]})
    snap = ViTEngine._py_state(eng, sess)
    # the "captured" call
    new_t = torch.ones(2)
    sess.approx_done = 40
    sess.extra.pop("layermean")
    sess.extra["plan_id"] = 4
    sess.extra["tap3"] = new_t
    sub.approx_done = 40
    sub.extra["k"] = 2
    eng._fp4, eng._fp8 = True, True
    delta = ViTEngine._py_delta(eng, snap)
    # a later request: state as before the call, then the replay re-applies the recorded effects
    sess.approx_done = 0
    sess.extra["layermean"] = torch.zeros(1)
    sess.extra["plan_id"] = 9
    del sess.extra["tap3"]
    sub.approx_done, sub.extra["k"] = 0, 1
    eng._fp4 = eng._fp8 = False
    ViTEngine._py_apply(eng, delta)
    assert sess.approx_done == 40 and sub.approx_done == 40 and sub.extra["k"] == 2
    assert "layermean" not in sess.extra and sess.extra["plan_id"] == 4 and sess.extra["tap3"] is new_t
    assert eng._fp4 and eng._fp8
