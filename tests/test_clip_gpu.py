"""CLIP tower on the ViT engine (learned position embedding, ln_pre, no RoPE, LayerScale 1)
against the fp32 module, and the zero-shot executor end to end."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.mark.parametrize("arch", ["clip_tiny", "clip_tiny_hd104"])
def test_clip_engine_matches_module(arch):
    """clip_tiny_hd104 has bigG's head width (104): heads run zero-padded to 128."""
    from appcorr_b200.models.clip import CLIP_MEAN, CLIP_PRESETS, CLIPVision, clip_engine_weights
    from appcorr_b200.models.engine import ViTEngine

    c = CLIP_PRESETS[arch]
    m = CLIPVision(c).init_weights(0).to(DEV)
    eng = ViTEngine(clip_engine_weights(m, DEV), DEV)
    B = 2
    img = torch.randint(0, 256, (B, 224, 224, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, 224, 224)
    eng.prepare_tokens(sess, img)
    x = eng.approx(sess, 0, c.layers, "none")
    mean = torch.tensor(CLIP_MEAN, device=DEV).view(1, 3, 1, 1)
    std = torch.tensor([0.26862954, 0.26130258, 0.27577711], device=DEV).view(1, 3, 1, 1)
    f = (img.permute(0, 3, 1, 2).float() / 255 - mean) / std
    with torch.no_grad():
        ref = m.tokens(f)
        assert ((sess.x_in.view(B, -1, c.width).float() - ref).norm() / ref.norm()).item() < 2e-2
        for blk in m.blocks:
            ref = blk(ref)
    rel = ((x.view(B, -1, c.width).float() - ref).norm() / ref.norm()).item()
    assert rel < 3e-2, rel


def test_openclip_executor_topk():
    from appcorr_b200.common.protocol import ExperimentConfig, Task
    from appcorr_b200.server.model import PyramidBatch, get_model_executor

    cfg = ExperimentConfig(exp_id="t", model_name="openclip", batch_size=2, image_shape=(224, 224, 3),
                           input_profile_kwargs={"clip_arch": "clip_tiny", "num_classes": 50},
                           transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 1},
                           appcorr_kwargs={"token_keep_ratio": 0.5})
    ex = get_model_executor("openclip", DEV)
    ex.load_model("openclip", cfg)
    base = torch.randint(0, 256, (2, 112, 112, 3), dtype=torch.uint8)
    res = torch.zeros(2, 224, 224, 3, dtype=torch.int16)
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])
    ctx = {}
    L = ex.cfg.depth
    ex.preprocess(PyramidBatch(base, None), task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.approx_forward({"layers": (0, L)}, ctx, cfg)
    ex.preprocess(PyramidBatch(base, res), task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.correct_forward({"layers": (0, L), "group_id": 1}, ctx, cfg)
    ex.head_inference(task, ctx, cfg)
    out = ex.get_final_results(task, ctx, cfg)
    assert len(out) == 2 and len(out[0]["topk"]) == 5
    assert abs(sum(p for _, p in out[0]["topk"]) - 1.0) < 1.0
