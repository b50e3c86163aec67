"""Detector window wrapper (reference windows.py:16-80, dinov3_detector.py:842-1000): 3 x 3
window sources + a resized global source through the backbone, [global | windows] features to
the decoder; a COCO-window correction group corrects exactly its window. Runs on the fp32 CPU
path and, when a GPU is present, on the sm_100a engine."""
import numpy as np
import pytest
import torch

from appcorr_b200.common.protocol import ExperimentConfig, Task
from appcorr_b200.server.model import get_model_executor
from appcorr_b200.server.model.dinov3_detector import window_layout


def test_window_layout_matches_reference_rule():
    # 1024 / 3 = 341 -> 352 (22 patches); the last window takes the remainder
    assert window_layout(1024, 1024, 3, 16) == ([352, 352, 320], [352, 352, 320], 352, 352)
    assert window_layout(96, 128, 3, 16) == ([32, 32, 32], [48, 48, 32], 32, 48)


def _cfg(keep=1.0):
    return ExperimentConfig(exp_id="t", model_name="dinov3_detector", batch_size=2, image_shape=(96, 128, 3),
                            input_profile_kwargs={"backbone_arch": "vits16", "decoder_layers": 2,
                                                  "num_queries": 20, "decoder_heads": 4},
                            transmission_policy_name="COCOWindowProgressiveLaplacian",
                            appcorr_kwargs={"token_keep_ratio": keep})


def _run(dev):
    cfg = _cfg()
    ex = get_model_executor("dinov3_detector", torch.device(dev))
    ex.load_model("dinov3_detector", cfg)
    if dev == "cpu":  # a shallow backbone keeps the CPU test fast
        ex.backbone.blocks = ex.backbone.blocks[:2]
        ex.cfg = ex.backbone.cfg
        ex.cfg.depth = 2
    L = ex.cfg.depth
    g = torch.Generator().manual_seed(0)
    base = torch.randint(0, 256, (2, 96, 128, 3), dtype=torch.uint8, generator=g)
    final = torch.randint(0, 256, (2, 96, 128, 3), dtype=torch.uint8, generator=g)
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])
    ctx = {}
    ex.preprocess(base, task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    assert len(ctx["det_sources"]) == 10 and ctx["det_sources"][-1]["canvas"].shape[1:3] == (32, 48)
    ex.approx_forward({"layers": (0, L), "global_only": True}, ctx, cfg)
    ex.approx_forward({"layers": (0, L), "source_kind": "local"}, ctx, cfg)
    ex.head_inference(task, ctx, cfg)
    mem0, hw = ex.memory(ctx)
    assert hw == (6, 8) and mem0.shape == (2, 48, 2 * ex.cfg.embed_dim)
    # group 5 = window (1, 1): only its features move
    ex.preprocess(final, task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.correct_forward({"layers": (0, L), "group_id": 5}, ctx, cfg)
    mem1, _ = ex.memory(ctx)
    d = (mem1.float() - mem0.float()).abs().amax(-1).view(2, 6, 8)
    moved = d > 1e-6
    win = torch.zeros(6, 8, dtype=torch.bool)
    win[2:4, 3:6] = True
    D = ex.cfg.embed_dim
    dw = (mem1[..., D:].float() - mem0[..., D:].float()).abs().amax(-1).view(2, 6, 8) > 1e-6
    assert torch.equal(dw.cpu(), win.expand(2, 6, 8)), dw
    # correcting every source with every token kept == full inference on the final image
    for gid in range(1, 10):
        ex.correct_forward({"layers": (0, L), "group_id": gid}, ctx, cfg)
    ex.approx_forward({"layers": (0, L), "global_only": True}, ctx, cfg)
    ex.head_inference(task, ctx, cfg)
    got = ex.get_final_results(task, ctx, cfg)
    ctx2 = {}
    ex.preprocess(final, task, ctx2, cfg)
    ex.full_inference(task, ctx2, cfg)
    mem2, _ = ex.memory(ctx2)
    mem3, _ = ex.memory(ctx)
    rel = ((mem3.float() - mem2.float()).norm() / mem2.float().norm()).item()
    assert rel < (1e-4 if dev == "cpu" else 2e-2), rel
    assert len(got) == 2 and got[0]["boxes"].shape[1] == 4 and np.isfinite(got[0]["scores"]).all()


def test_detector_windows_cpu():
    _run("cpu")


@pytest.mark.gpu
def test_detector_windows_gpu():
    _run("cuda")
