"""Convolution kernels (NHWC im2col + GEMM, bilinear resize) and the DPT / RRDB heads built on
them, against the fp32 PyTorch modules; the depther executor end to end on a small backbone."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("k,stride,pad,cin,cout", [(3, 1, 1, 64, 96), (3, 2, 1, 32, 32), (1, 1, 0, 48, 20)])
def test_conv_gpu_matches_conv2d(k, stride, pad, cin, cout):
    from appcorr_b200.models.conv import ConvGPU

    torch.manual_seed(0)
    conv = torch.nn.Conv2d(cin, cout, k, stride=stride, padding=pad).to(DEV)
    x = torch.randn(2, 13, 17, cin, device=DEV).to(torch.bfloat16)
    y = ConvGPU(conv, DEV)(x)
    with torch.no_grad():
        ref = conv(x.float().permute(0, 3, 1, 2)).permute(0, 2, 3, 1)
    assert y.shape == ref.shape and _rel(y, ref) < 1e-2


@pytest.mark.parametrize("align", [True, False])
def test_resize_matches_interpolate(align):
    from appcorr_b200.models.conv import resize

    x = torch.randn(2, 7, 9, 16, device=DEV).to(torch.bfloat16)
    y = resize(x, 14, 18, align)
    ref = F.interpolate(x.float().permute(0, 3, 1, 2), size=(14, 18), mode="bilinear",
                        align_corners=align).permute(0, 2, 3, 1)
    assert (y.float() - ref).abs().max().item() < 3e-2


def test_dpt_head_gpu_matches_module():
    from appcorr_b200.models.conv import DPTHead, DPTHeadGPU

    torch.manual_seed(1)
    B, gh, gw, D = 2, 8, 12, 384
    head = DPTHead(D, features=64, channels=(32, 64, 128, 128)).init_weights(0).to(DEV)
    taps = [torch.randn(B * gh * gw, D, device=DEV).to(torch.bfloat16) for _ in range(4)]
    d = DPTHeadGPU(head, DEV).forward(taps, B, gh, gw)
    with torch.no_grad():
        ref = head([t.float().view(B, gh * gw, D) for t in taps], gh, gw)[:, 0]
    assert d.shape == ref.shape and _rel(d, ref) < 5e-2


def test_rrdb_gpu_matches_module():
    from appcorr_b200.models.conv import RRDBNet, RRDBNetGPU

    torch.manual_seed(2)
    net = RRDBNet(nf=32, nb=2, gc=16).init_weights(0).to(DEV)
    img = torch.randint(0, 256, (1, 24, 20, 3), dtype=torch.uint8, device=DEV)
    out = RRDBNetGPU(net, DEV).forward(img)
    with torch.no_grad():
        ref = net(img.float().permute(0, 3, 1, 2) / 255.0).clamp(0, 1).permute(0, 2, 3, 1) * 255.0
    assert out.shape == (1, 96, 80, 3)
    assert (out.float() - ref).abs().mean().item() < 2.0


def test_depther_executor_end_to_end():
    from appcorr_b200.common.protocol import ExperimentConfig, Task
    from appcorr_b200.server.model import PyramidBatch, get_model_executor

    cfg = ExperimentConfig(exp_id="t", model_name="dinov3_depther", batch_size=2, image_shape=(128, 128, 3),
                           input_profile_name="dinov3_ade20k_linhead_official",
                           input_profile_kwargs={"backbone_arch": "vits16", "server_inference_mode": "whole",
                                                 "dpt_features": 64},
                           transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 1},
                           appcorr_kwargs={"token_keep_ratio": 0.5})
    ex = get_model_executor(cfg.model_name, DEV)
    ex.load_model(cfg.model_name, cfg)
    base = torch.randint(0, 256, (2, 64, 64, 3), dtype=torch.uint8)
    res = torch.zeros(2, 128, 128, 3, dtype=torch.int16)
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
    assert len(out) == 2 and out[0]["depth"].shape == (128, 128)
    assert bool(torch.isfinite(torch.from_numpy(out[0]["depth"])).all())


def test_lowres_sr_engine_upscales_to_target():
    from appcorr_b200.server.sr import create_lowres_sr_engine

    sr = create_lowres_sr_engine({"model": "realesrgan_x4plus", "weights_dir": "/nonexistent"}, DEV)
    base = torch.randint(0, 256, (2, 16, 24, 3), dtype=torch.uint8, device=DEV)
    assert sr.upscale(base).shape == (2, 64, 96, 3)
    out = sr.upscale(base, (32, 48))
    assert out.shape == (2, 32, 48, 3) and out.dtype == torch.uint8


def test_depther_eval_grid_and_flip_tta():
    """NYU profile: images go onto the fixed eval grid, mirrored sources are flipped back and
    averaged (so the result is mirror-symmetric for a mirror-symmetric input), and the depth map
    comes back at the image's own size."""
    from appcorr_b200.common.protocol import ExperimentConfig, Task
    from appcorr_b200.server.model import PyramidBatch, get_model_executor

    cfg = ExperimentConfig(exp_id="t", model_name="dinov3_depther", batch_size=2, image_shape=(96, 160, 3),
                           input_profile_name="dinov3_nyu_synthmix_dpt",
                           input_profile_kwargs={"backbone_arch": "vits16", "depther_eval_size": 128,
                                                 "dpt_features": 64},
                           transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 1},
                           appcorr_kwargs={"token_keep_ratio": 1.0})
    ex = get_model_executor(cfg.model_name, DEV)
    ex.load_model(cfg.model_name, cfg)
    import numpy as np

    from appcorr_b200.policies.transmission.pyramid import pyr_up

    base = torch.randint(0, 256, (2, 48, 80, 3), dtype=torch.uint8)
    half = torch.randint(0, 256, (2, 96, 80, 3), dtype=torch.int16)
    target = torch.cat([half, torch.flip(half, dims=[2])], 2)             # mirror-symmetric 96 x 160
    up = torch.from_numpy(np.stack([pyr_up(b) for b in base.numpy()]).astype(np.int16))
    res = target - up                                                      # full canvas = target
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])
    ctx = {}
    L = ex.cfg.depth
    ex.preprocess(PyramidBatch(base, None), task, ctx, cfg)
    assert ctx["canvas"].shape == (4, 128, 128, 3)  # 2 images + 2 mirrors on the 128 grid
    ex.prepare_tokens(task, ctx, cfg)
    ex.approx_forward({"layers": (0, L)}, ctx, cfg)
    ex.preprocess(PyramidBatch(base, res), task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.correct_forward({"layers": (0, L), "group_id": 1}, ctx, cfg)
    ex.head_inference(task, ctx, cfg)
    out = ex.get_final_results(task, ctx, cfg)
    d = torch.from_numpy(out[0]["depth"])
    assert d.shape == (96, 160) and bool(torch.isfinite(d).all())
    assert torch.allclose(d, torch.flip(d, dims=[1]), rtol=1e-4, atol=1e-4)
