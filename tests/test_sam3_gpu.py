"""Windowed-attention tower (SAM 3 geometry, small preset) on the ViT engine: approximate pass vs
the fp32 module, full correction == forward on the new image, per-query key ranges in the
attention kernel, and the executor end to end."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def _setup():
    from appcorr_b200.models.engine import ViTEngine
    from appcorr_b200.models.sam3 import SAM3_PRESETS, SAM3Tower, sam3_engine_weights

    c = SAM3_PRESETS["sam3_tiny"]
    m = SAM3Tower(c).init_weights(0).to(DEV)
    return c, m, ViTEngine(sam3_engine_weights(m, DEV), DEV)


def _float(img):
    mean = torch.tensor((0.485, 0.456, 0.406), device=DEV).view(1, 3, 1, 1)
    std = torch.tensor((0.229, 0.224, 0.225), device=DEV).view(1, 3, 1, 1)
    return (img.permute(0, 3, 1, 2).float() / 255 - mean) / std


def test_windowed_tower_approx_and_full_correction():
    c, m, eng = _setup()
    B, S = 2, 224
    img0 = torch.randint(0, 256, (B, S, S, 3), dtype=torch.uint8, device=DEV)
    img1 = torch.randint(0, 256, (B, S, S, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, S, S)
    eng.prepare_tokens(sess, img0)
    eng.approx(sess, 0, c.depth, "none")
    got = eng.normed_tokens(sess).view(B, sess.N, -1)
    with torch.no_grad():
        ref = m(_float(img0))
    assert _rel(got, ref) < 3e-2
    eng.prepare_tokens(sess, img1)
    pre = torch.zeros(B, 0, device=DEV, dtype=torch.int32)
    cand = torch.arange(sess.N, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    score = torch.rand(B, sess.N, device=DEV)
    eng.correct(sess, 0, c.depth, pre, cand, {"token_keep_ratio": 1.0}, server=score)
    got = eng.normed_tokens(sess).view(B, sess.N, -1)
    with torch.no_grad():
        ref = m(_float(img1))
    assert _rel(got, ref) < 3e-2


@pytest.mark.parametrize("impl", ["tcgen05", "tcgen05_split"])
def test_attention_per_query_key_ranges(impl):
    from appcorr_b200.ops import kernels as K

    torch.manual_seed(1)
    B, H, Dh, N, tw = 2, 4, 64, 576, 64
    k = torch.randn(B * N, H * Dh, device=DEV).to(torch.bfloat16)
    v = torch.randn(B * N, H * Dh, device=DEV).to(torch.bfloat16)
    sel = torch.sort(torch.randperm(N, device=DEV)[:150]).values
    T = sel.numel()
    q = torch.randn(B * T, H * Dh, device=DEV).to(torch.bfloat16)
    lo = (sel // tw * tw).repeat(B).to(torch.int32).contiguous()
    hi = (lo + tw - 1).contiguous()
    o = torch.empty_like(q)
    K.attention(q, k, v, o, B=B, Tq=T, Tk=N, H=H, Dh=Dh, causal=True, q_pos=hi, q_lo=lo, impl=impl)
    qq = q.float().view(B, T, H, Dh).transpose(1, 2)
    kk = k.float().view(B, N, H, Dh).transpose(1, 2)
    vv = v.float().view(B, N, H, Dh).transpose(1, 2)
    keys = torch.arange(N, device=DEV)[None]
    mask = (keys >= lo[:T, None].long()) & (keys <= hi[:T, None].long())
    ref = torch.nn.functional.scaled_dot_product_attention(qq, kk, vv, attn_mask=mask[None, None])
    ref = ref.transpose(1, 2).reshape(B * T, H * Dh)
    assert (o.float() - ref).abs().max().item() < 2e-2 * ref.abs().max().item() + 2e-2


def test_sam3_executor_end_to_end():
    from appcorr_b200.common.protocol import ExperimentConfig, Task
    from appcorr_b200.server.model import PyramidBatch, get_model_executor

    cfg = ExperimentConfig(exp_id="t", model_name="sam3", batch_size=2, image_shape=(224, 224, 3),
                           input_profile_kwargs={"sam3_arch": "sam3_tiny", "num_classes": 20},
                           transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 1},
                           appcorr_kwargs={"token_keep_ratio": 0.3})
    ex = get_model_executor("sam3", DEV)
    ex.load_model("sam3", cfg)
    base = torch.randint(0, 256, (2, 112, 112, 3), dtype=torch.uint8)
    res = torch.randint(-20, 20, (2, 224, 224, 3), dtype=torch.int16)
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])
    ctx = {}
    ex.preprocess(PyramidBatch(base, None), task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.approx_forward({}, ctx, cfg)
    ex.preprocess(PyramidBatch(base, res), task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.correct_forward({}, ctx, cfg)
    ex.head_inference(task, ctx, cfg)
    out = ex.get_final_results(task, ctx, cfg)
    assert len(out) == 2 and out[0]["mask"].shape == (224, 224)
    assert ctx["vision_embeds"].shape == (2, 16, 16, 256)


def test_vggt_executor_full_inference():
    """Multi-view tower: frame attention stays inside a frame (windows = frames), global blocks
    mix frames; per-frame depth and pose come out for every frame."""
    from appcorr_b200.common.protocol import ExperimentConfig, Task
    from appcorr_b200.server.model import get_model_executor

    cfg = ExperimentConfig(exp_id="t", model_name="vggt", batch_size=3, image_shape=(128, 128, 3),
                           input_profile_kwargs={"vggt_arch": "vggt_tiny"})
    ex = get_model_executor("vggt", DEV)
    ex.load_model("vggt", cfg)
    frames = torch.randint(0, 256, (3, 128, 128, 3), dtype=torch.uint8)
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])
    ctx = {}
    ex.preprocess(frames, task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.full_inference(task, ctx, cfg)
    out = ex.get_final_results(task, ctx, cfg)[0]
    assert out["depth"].shape == (3, 128, 128) and out["pose_enc"].shape == (3, 9) and out["num_frames"] == 3
    assert np_isfinite(out["depth"]) and np_isfinite(out["pose_enc"])


def np_isfinite(a):
    import numpy as np

    return bool(np.isfinite(a).all())


def test_vggt_interleaved_walk_recovers_full_inference():
    """The VGGTInterleaved schedule on the 48-stage axis (here the tiny tower's 6 stages): approx
    [0, 3) on the base frames, a round that corrects [0, 3) and approximates [3, 6), then a final
    correction of [0, 6). With every token kept, the corrected result equals full inference on the
    final frames; a round whose patches cover one frame corrects only that frame's tokens."""
    from appcorr_b200.common.protocol import ExperimentConfig, Patch, Task
    from appcorr_b200.server.model import get_model_executor

    cfg = ExperimentConfig(exp_id="t", model_name="vggt", batch_size=3, image_shape=(128, 128, 3),
                           input_profile_kwargs={"vggt_arch": "vggt_tiny"},
                           appcorr_kwargs={"token_keep_ratio": 1.0}, patch_size=(16, 16))
    ex = get_model_executor("vggt", DEV)
    ex.load_model("vggt", cfg)
    g = torch.Generator().manual_seed(0)
    base = torch.randint(0, 256, (3, 128, 128, 3), dtype=torch.uint8, generator=g)
    final = torch.randint(0, 256, (3, 128, 128, 3), dtype=torch.uint8, generator=g)
    t0 = Task(task_id=0, request_id=0, payload=[], instructions=[])
    ctx = {}
    ex.preprocess(base, t0, ctx, cfg)
    ex.prepare_tokens(t0, ctx, cfg)
    ex.approx_forward({"layers": (0, 3)}, ctx, cfg)
    # round 1: patches of frame 1 only
    p1 = [Patch(image_idx=1, spatial_idx=i, data=b"", res_level=0, group_id=1) for i in range(64)]
    t1 = Task(task_id=1, request_id=0, payload=p1, instructions=[])
    ex.preprocess(final, t1, ctx, cfg)
    ex.prepare_tokens(t1, ctx, cfg)
    arrived = ctx["vggt_arrived"]
    assert arrived.shape[1] == 64 and int(arrived.min()) == 64 and int(arrived.max()) == 127
    ex.correct_forward({"layers": (0, 3)}, ctx, cfg)
    ex.approx_forward({"layers": (3, 6)}, ctx, cfg)
    # final round: every token
    t2 = Task(task_id=2, request_id=0, payload=[], instructions=[])
    ex.preprocess(final, t2, ctx, cfg)
    ex.prepare_tokens(t2, ctx, cfg)
    ex.correct_forward({"layers": (0, 6)}, ctx, cfg)
    ex.head_inference(t2, ctx, cfg)
    got = ex.get_final_results(t2, ctx, cfg)[0]
    ctx2 = {}
    ex2 = get_model_executor("vggt", DEV)
    ex2.load_model("vggt", cfg)
    ex2.preprocess(final, t2, ctx2, cfg)
    ex2.prepare_tokens(t2, ctx2, cfg)
    ex2.full_inference(t2, ctx2, cfg)
    ref = ex2.get_final_results(t2, ctx2, cfg)[0]
    import numpy as np

    for key in ("depth", "pose_enc"):
        a, b = got[key].astype(np.float64), ref[key].astype(np.float64)
        assert np.linalg.norm(a - b) / np.linalg.norm(b) < 2e-2, key
