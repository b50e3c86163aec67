"""Mask2Former segmentor on the sm_100a kernels against its fp32 oracle (small widths)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


def test_mask2former_gpu_matches_oracle():
    from appcorr_b200.models.mask2former import DINOv3M2FSegmentor, Mask2FormerGPU, semantic_map

    torch.manual_seed(0)
    D = 128
    m = DINOv3M2FSegmentor(dim=D, num_classes=9, hidden=128, heads=16, adapter_heads=4, ffn=256, enc_layers=2,
                           dec_layers=3, queries=16, inplanes=32).init_weights(1).eval().to(DEV)
    B, h, w = 2, 96, 128
    g = torch.Generator(device=DEV).manual_seed(2)
    x = torch.randn(B, 3, h, w, device=DEV, generator=g)
    taps = [torch.randn(B, (h // 16) * (w // 16), D, device=DEV, generator=g) for _ in range(4)]
    gpu = Mask2FormerGPU(m, DEV)
    xb = x.to(torch.bfloat16)
    tb = [t.to(torch.bfloat16) for t in taps]
    with torch.no_grad():
        ref_feats = m.adapter(xb.float(), [t.float() for t in tb])
        feats = gpu.adapter(xb.permute(0, 2, 3, 1).contiguous(), [t.reshape(-1, D).contiguous() for t in tb], B)
        for i, key in enumerate(("1", "2", "3", "4")):
            e = _rel(feats[i].permute(0, 3, 1, 2), ref_feats[key])
            assert e < 3e-2, (key, e)
        ref_mf, ref_lv = m.head.pixel_decoder(ref_feats)
        mf, lv = gpu.pixel_decoder(feats, B)
        assert _rel(mf.permute(0, 3, 1, 2), ref_mf) < 5e-2
        for a, r in zip(lv, ref_lv):
            assert _rel(a.permute(0, 3, 1, 2), r) < 5e-2
        out = gpu.forward(xb.permute(0, 2, 3, 1).contiguous(), [t.reshape(-1, D).contiguous() for t in tb], B)
        ref = m(xb.float(), [t.float() for t in tb])
        sem, sem_ref = semantic_map(out, (h, w)), semantic_map(ref, (h, w))
    torch.cuda.synchronize()
    from appcorr_b200.ops.native import check_errors

    check_errors(DEV)
    assert _rel(sem, sem_ref) < 0.15


def test_m2f_executor_slide_sources_end_to_end():
    """Slide mode: every image's windows become engine sources; the class maps are stitched back."""
    from appcorr_b200.common.protocol import ExperimentConfig, Task
    from appcorr_b200.server.model import PyramidBatch, get_model_executor

    cfg = ExperimentConfig(exp_id="t", model_name="dinov3_segmentor_m2f", batch_size=2, image_shape=(128, 192, 3),
                           input_profile_name="dinov3_ade20k_m2f_official",
                           input_profile_kwargs={"backbone_arch": "vits16", "server_crop_size": 128,
                                                 "server_stride": 64, "m2f_hidden_dim": 128, "m2f_adapter_heads": 12, "m2f_enc_layers": 1,
                                                 "m2f_dec_layers": 3, "m2f_queries": 16},
                           transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 1},
                           appcorr_kwargs={"token_keep_ratio": 0.5})
    ex = get_model_executor(cfg.model_name, DEV)
    ex.load_model(cfg.model_name, cfg)
    base = torch.randint(0, 256, (2, 64, 96, 3), dtype=torch.uint8)
    res = torch.zeros(2, 128, 192, 3, dtype=torch.int16)
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])
    ctx = {}
    L = ex.cfg.depth
    ex.preprocess(PyramidBatch(base, None), task, ctx, cfg)
    assert ctx["canvas"].shape == (4, 128, 128, 3)  # 2 images x 2 windows
    ex.prepare_tokens(task, ctx, cfg)
    ex.approx_forward({"layers": (0, L)}, ctx, cfg)
    ex.preprocess(PyramidBatch(base, res), task, ctx, cfg)
    ex.prepare_tokens(task, ctx, cfg)
    ex.correct_forward({"layers": (0, L), "group_id": 1}, ctx, cfg)
    ex.head_inference(task, ctx, cfg)
    out = ex.get_final_results(task, ctx, cfg)
    assert len(out) == 2 and out[0]["mask"].shape == (128, 192)
    assert int(out[0]["mask"].max()) < 150
