"""Protocol, wire format, config overrides, transmission codecs and scheduling tables (CPU)."""
import itertools
import pickle
import socket
import threading

import numpy as np
import pytest

from appcorr_b200.common.config_overrides import apply_config_overrides, parse_override_value
from appcorr_b200.common.network import recv_msg, send_msg
from appcorr_b200.common.protocol import (ExperimentConfig, InferenceResult, Instruction, OpType, Patch, Task,
                                          normalize_appcorr_kwargs)
from appcorr_b200.policies import SCHEDULER_REGISTRY, TRANSMISSION_REGISTRY, get_scheduler, get_transmission


def _img(B=2, H=64, W=64, seed=0):
    rng = np.random.default_rng(seed)
    return np.clip(rng.normal(128, 60, size=(B, H, W, 3)), 0, 255).astype(np.uint8)


def _cfg(**kw):
    base = dict(batch_size=2, image_shape=(64, 64, 3), patch_size=(16, 16))
    base.update(kw)
    return ExperimentConfig(**base)


# ------------------------------------------------------------------ protocol
def test_normalize_aliases_and_validation():
    o = normalize_appcorr_kwargs({"mobile_pscore": "residual_l2", "pscore_fusion": "mul",
                                  "server_pscore": "patch_attn_prune", "token_keep_thres": "null"})
    assert o["enabled"] and o["mobile_pscore"] == "residual_energy" and o["pscore_fusion"] == "multiply"
    assert o["server_pscore"] == "patch_attn_prob" and o["token_keep_thres"] is None
    assert normalize_appcorr_kwargs({"server_pscore_layer_fusion": "mean"})["server_pscore"] == "cls_attn_prob_layermean"
    assert not normalize_appcorr_kwargs(None)["enabled"]
    with pytest.raises(ValueError):
        normalize_appcorr_kwargs({"server_pscore": "nope"})
    with pytest.raises(ValueError):
        normalize_appcorr_kwargs({"persist_correction_residual": False})
    with pytest.raises(ValueError):
        normalize_appcorr_kwargs({"num_groups": 3}, {"num_groups": 4})
    assert normalize_appcorr_kwargs({"a": 1}, {"pyramid_levels": [2, 0]})["pyramid_levels"] == [2, 0]


def test_config_validation_and_profiles():
    with pytest.raises(ValueError):
        ExperimentConfig(precision="int8")
    c = ExperimentConfig(input_profile_name="dinov3_ade20k_linhead_official", input_profile_kwargs={"server_stride": 300})
    p = c.get_input_profile_config()
    assert p["server_crop_size"] == 512 and p["server_stride"] == 300 and p["num_classes"] == 150


def test_pickle_round_trip():
    t = Task(3, 1, [Patch(0, 5, b"xy", 1, 2, 7, 0.5, 0.25)], [Instruction(OpType.CORRECT_FORWARD, {"layers": (0, 10)})])
    t2 = pickle.loads(pickle.dumps(t))
    assert t2 == t
    r = InferenceResult(1, 2.0, {"a": 1}, partial_token_kept_patch=3.0)
    assert pickle.loads(pickle.dumps(r)) == r


def test_overrides():
    d = {"appcorr_kwargs": {"a": 1}}
    apply_config_overrides(d, ["appcorr_kwargs.token_keep_ratio=0.3", "x.y.z=true", "s=hello", "n=none", "l=[1,2]"])
    assert d["appcorr_kwargs"] == {"a": 1, "token_keep_ratio": 0.3}
    assert d["x"] == {"y": {"z": True}} and d["s"] == "hello" and d["n"] is None and d["l"] == [1, 2]
    with pytest.raises(ValueError):
        apply_config_overrides(d, ["novalue"])
    with pytest.raises(ValueError):
        apply_config_overrides(d, ["s.t=1"])
    assert parse_override_value("FALSE") is False


def test_wire_format_loopback():
    a, b = socket.socketpair()
    payload = {"big": np.arange(200000).tobytes(), "k": [1, 2, 3]}
    th = threading.Thread(target=send_msg, args=(a, payload))
    th.start()
    got = recv_msg(b)
    th.join()
    assert got == payload
    a.close()
    assert recv_msg(b) is None


# ------------------------------------------------------------------ transmission
def _collect(policy, imgs, cfg):
    return [list(g) for g in policy.encode(imgs, cfg)]


@pytest.mark.parametrize("levels", [[1, 0], [2, 1, 0], [2, 0]])
def test_laplacian_lossless(levels):
    imgs = _img()
    cfg = _cfg(transmission_policy_name="Laplacian", transmission_kwargs={"pyramid_levels": levels})
    pol = get_transmission("Laplacian")
    groups = _collect(pol, imgs, cfg)
    assert len(groups) == len(levels)
    patches = [p for g in groups for p in g]
    assert np.array_equal(pol.decode(patches, cfg), imgs)
    # GPU-reconstruction unpacking: base + residual canvases reproduce the CPU decode
    pb = pol.decode_pyramid(patches, cfg)
    from appcorr_b200.policies.transmission.pyramid import pyr_up

    cur = pb.base
    for r in pb.residual_steps():
        cur = np.stack([pyr_up(x) for x in cur]).astype(np.int32)
        if r is not None:
            cur = cur + r
        cur = np.clip(cur, 0, 255).astype(np.uint8)
    assert np.array_equal(cur, imgs)


@pytest.mark.parametrize("strategy", ["grid", "block_grid", "expansion", "sequential", "uniform_diff",
                                      "energy_asc", "energy_desc", "random", "geometric"])
def test_progressive_groups_lossless(strategy):
    imgs = _img()
    cfg = _cfg(transmission_policy_name="ProgressiveLaplacian",
               transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 4, "grouping_strategy": strategy},
               appcorr_kwargs={"mobile_pscore": "residual_energy"})
    pol = get_transmission("ProgressiveLaplacian")
    groups = _collect(pol, imgs, cfg)
    assert groups[0][0].group_id == 0 and all(p.batch_group_total == len(g) for g in groups for p in g)
    res = [p for g in groups[1:] for p in g]
    assert len(res) == 2 * 16 and all(1 <= p.group_id <= 4 for p in res)
    assert all(p.pscore_hint >= 0 for p in res)
    full = pol.decode([p for g in groups for p in g], cfg)
    assert np.array_equal(full, imgs)
    base_only = pol.decode(groups[0], cfg)
    assert base_only.shape == imgs.shape


def test_progressive_grid_matches_server_group_index():
    """The client's grid assignment must equal the server's create_group_index."""
    import torch

    from appcorr_b200.models.dinov3 import create_group_index

    imgs = _img(1, 128, 128)
    cfg = _cfg(batch_size=1, image_shape=(128, 128, 3),
               transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 4, "grouping_strategy": "expansion"})
    groups = _collect(get_transmission("ProgressiveLaplacian"), imgs, cfg)
    client = np.zeros(64, int)
    for g in groups[1:]:
        for p in g:
            client[p.spatial_idx] = p.group_id
    server = create_group_index(64, 4, "expansion", token_hw=(8, 8)).numpy()
    assert np.array_equal(client, server)


def test_top_energy_keeps_fraction():
    imgs = _img()
    cfg = _cfg(transmission_kwargs={"pyramid_levels": [1, 0], "grouping_strategy": "top_energy", "keep_rate": 0.25})
    groups = _collect(get_transmission("ProgressiveLaplacian"), imgs, cfg)
    assert len(groups) == 2 and len(groups[1]) == 2 * 4


@pytest.mark.parametrize("name", ["Raw", "Zlib"])
def test_raw_zlib_lossless(name):
    imgs = _img()
    cfg = _cfg()
    pol = get_transmission(name)
    assert np.array_equal(pol.decode([p for g in pol.encode(imgs, cfg) for p in g], cfg), imgs)


def test_full_image_png_lossless_and_jpeg_close():
    imgs = _img()
    pol = get_transmission("FullImageCompression")
    cfg = _cfg(transmission_kwargs={"format": "png"})
    ps = [p for g in pol.encode(imgs, cfg) for p in g]
    assert len(ps) == 2 * 16
    assert np.array_equal(pol.decode(ps, cfg), imgs)
    yy, xx = np.mgrid[0:64, 0:64]
    smooth = np.stack([np.stack([yy * 3, xx * 3, (yy + xx) * 2], -1)] * 2).astype(np.uint8)
    cfg = _cfg(transmission_kwargs={"format": "jpg", "quality": 95})
    out = pol.decode([p for g in pol.encode(smooth, cfg) for p in g], cfg)
    assert np.abs(out.astype(int) - smooth).mean() < 3


def test_fourier_hybrid_lossless_with_all_groups():
    imgs = _img()
    cfg = _cfg(transmission_kwargs={"pyramid_levels": [2, 0], "num_groups": 4, "grouping_strategy": "grid"})
    pol = get_transmission("FourierLaplacianProgressive")
    groups = _collect(pol, imgs, cfg)
    full = pol.decode([p for g in groups for p in g], cfg)
    assert np.array_equal(full, imgs)
    approx = pol.decode(groups[0], cfg)
    assert np.abs(approx.astype(int) - imgs).mean() > 1


def test_fourier_progressive_reconstructs():
    imgs = _img()
    cfg = _cfg(transmission_kwargs={"pyramid_levels": [2, 0], "num_groups": 4, "grouping_strategy": "grid"})
    pol = get_transmission("FourierProgressive")
    groups = _collect(pol, imgs, cfg)
    full = pol.decode([p for g in groups for p in g], cfg)
    assert np.abs(full.astype(int) - imgs).max() <= 2


def test_ade20k_crop_cover_groups():
    imgs = _img(1, 64, 96)
    cfg = _cfg(batch_size=1, image_shape=(64, 96, 3), input_profile_name="dinov3_ade20k_m2f_official",
               input_profile_kwargs={"server_crop_size": 64, "server_stride": 32},
               transmission_kwargs={"pyramid_levels": [1, 0]})
    groups = _collect(get_transmission("ADE20KWindowProgressiveLaplacian"), imgs, cfg)
    n = groups[0][0].num_correction_groups
    assert n == 2 and {p.group_id for g in groups[1:] for p in g} <= {1, 2}


def test_registries_complete():
    assert len(SCHEDULER_REGISTRY) == 11 and len(TRANSMISSION_REGISTRY) == 16


# ------------------------------------------------------------------ scheduling
def _patches(group, n, ncg=0):
    return [Patch(0, i, b"", group_id=group, batch_group_total=n, num_correction_groups=ncg) for i in range(n)]


def _ops(task):
    return [(i.op_type.name, i.params.get("layers")) for i in task.instructions]


def test_group_trigger_table():
    cfg = _cfg(transmission_kwargs={"num_groups": 4, "total_layers": 40})
    pol = get_scheduler("GroupTrigger", cfg)
    ids = itertools.count()
    assert pol.decide(_patches(0, 3)[:2], cfg, ids) is None
    t0 = pol.decide(_patches(0, 3), cfg, ids)
    assert _ops(t0) == [("LOAD_INPUT", None), ("PREPARE_TOKENS", None), ("APPROX_FORWARD", (0, 10))]
    t1 = pol.decide(_patches(1, 2), cfg, ids)
    assert t1.request_id == t0.request_id
    assert _ops(t1)[2:] == [("CORRECT_FORWARD", (0, 10)), ("APPROX_FORWARD", (10, 20))]
    t4 = pol.decide(_patches(4, 2), cfg, ids)
    assert [o for o, _ in _ops(t4)[2:]] == ["CORRECT_FORWARD", "HEAD_INFERENCE", "EXIT_ALL", "SEND_RESPONSE",
                                            "FREE_SESSION"]


def test_batch_count_waits_for_all_groups():
    cfg = _cfg(transmission_policy_name="ProgressiveLaplacian", transmission_kwargs={"num_groups": 1})
    pol = get_scheduler("BatchCountBased", cfg)
    ids = itertools.count()
    assert pol.decide(_patches(0, 4), cfg, ids) is None
    t = pol.decide(_patches(0, 4) + _patches(1, 4), cfg, ids)
    assert len(t.payload) == 8 and [o for o, _ in _ops(t)] == ["LOAD_INPUT", "FULL_INFERENCE", "SEND_RESPONSE",
                                                                 "FREE_SESSION"]
    cfg.scheduler_kwargs["approx_only"] = True
    t = pol.decide(_patches(0, 4) + _patches(1, 4), cfg, ids)
    assert ("APPROX_FORWARD", (0, 40)) in _ops(t)


def test_two_phase_and_sequential():
    cfg = _cfg(appcorr_kwargs={"token_keep_ratio": 0.5})
    pol = get_scheduler("ADE20KApproxCorrect", cfg)
    ids = itertools.count()
    t0 = pol.decide(_patches(0, 2), cfg, ids)
    t1 = pol.decide(_patches(1, 2), cfg, ids)
    assert _ops(t0)[-1] == ("APPROX_FORWARD", (0, 40)) and t1.request_id == t0.request_id
    assert [o for o, _ in _ops(t1)] == ["LOAD_INPUT", "PREPARE_TOKENS", "CORRECT_FORWARD", "HEAD_INFERENCE",
                                        "SEND_RESPONSE", "FREE_SESSION"]
    cfg2 = _cfg()
    t1b = get_scheduler("NYUApproxCorrect", cfg2).decide(_patches(1, 2), cfg2, ids)
    assert "CORRECT_FORWARD" not in [o for o, _ in _ops(t1b)]


def test_dynamic_group_trigger_feedback():
    cfg = _cfg(transmission_kwargs={"num_groups": 2, "total_layers": 6}, scheduler_kwargs={"ahead_layers": 2})
    pol = get_scheduler("DynamicGroupTrigger", cfg)
    ids = itertools.count()
    t0 = pol.decide(_patches(0, 2), cfg, ids)
    assert _ops(t0)[2:] == [("APPROX_FORWARD", (0, 1)), ("APPROX_FORWARD", (1, 2))]
    tf = pol.decide([], cfg, ids, feedback_events=[1])
    assert _ops(tf) == [("APPROX_FORWARD", (2, 3))]
    t1 = pol.decide(_patches(1, 2), cfg, ids)
    assert _ops(t1)[2] == ("CORRECT_FORWARD", (0, 3))
    t2 = pol.decide(_patches(2, 2), cfg, ids)
    assert _ops(t2)[2:4] == [("CORRECT_FORWARD", (0, 3)), ("APPROX_FORWARD", (3, 6))]


def test_ade20k_window_and_coco_static():
    cfg = _cfg(scheduler_kwargs={"total_layers": 10})
    pol = get_scheduler("ADE20KWindowInterleaved", cfg)
    ids = itertools.count()
    t0 = pol.decide(_patches(0, 1, ncg=3), cfg, ids)
    assert _ops(t0)[-1] == ("APPROX_FORWARD", (0, 4))
    t1 = pol.decide(_patches(1, 1, ncg=3), cfg, ids)
    assert _ops(t1)[2:] == [("CORRECT_FORWARD", (0, 4)), ("APPROX_FORWARD", (4, 7))]
    coco = get_scheduler("COCOWindowInterleaved", cfg)
    t0 = coco.decide(_patches(0, 1), cfg, ids)
    assert _ops(t0)[-1] == ("APPROX_FORWARD", (0, 2))
    for g in range(1, 9):
        coco.decide(_patches(g, 1), cfg, ids)
    t9 = coco.decide(_patches(9, 1), cfg, ids)
    assert _ops(t9)[2] == ("CORRECT_FORWARD", (0, 10))


def test_vggt_boundaries():
    cfg = _cfg(transmission_kwargs={"correction_groups": 3}, appcorr_kwargs={"token_keep_ratio": 0.5})
    from appcorr_b200.policies.scheduling import VGGTInterleavedPolicy

    b = VGGTInterleavedPolicy.boundaries(48, 3, cfg)
    assert b[-1] == 48 and b[0] < b[1] < b[2]
    cfg.scheduler_kwargs["layer_split"] = "uniform"
    assert VGGTInterleavedPolicy.boundaries(48, 3, cfg) == [16, 32, 48]


def test_nyu_policies_decode_on_fixed_model_grid():
    """NYU AppCorr transmission (reference nyu_appcorr_progressive.py): shape preservation is
    forced off and every decode lands on config.image_shape, whatever the input image size."""
    import numpy as np

    from appcorr_b200.common.protocol import ExperimentConfig
    from appcorr_b200.policies import get_transmission

    cfg = ExperimentConfig(exp_id="t", model_name="dinov3_depther", batch_size=2, image_shape=(64, 96, 3),
                           transmission_kwargs={"preserve_input_shape": True, "pyramid_levels": [1, 0],
                                                "num_groups": 1, "grouping_strategy": "grid"})
    rng = np.random.default_rng(0)
    imgs = rng.integers(0, 256, (2, 64, 96, 3), dtype=np.uint8)
    for name in ("NYUAppCorrLaplacian", "NYUAppCorrProgressiveLaplacian"):
        pol = get_transmission(name)
        groups = list(pol.encode(imgs, cfg))
        out = pol.decode([p for g in groups for p in g], cfg)
        out = np.stack([o["image"] if isinstance(o, dict) else o for o in out]) if isinstance(out, list) else out
        assert out.shape == (2, 64, 96, 3), name
        assert np.abs(out.astype(int) - imgs.astype(int)).max() <= 1, name   # lossless pyramid
    # raw: a differently sized image is resized onto the model grid
    big = rng.integers(0, 256, (2, 128, 192, 3), dtype=np.uint8)
    pol = get_transmission("NYUAppCorrRaw")
    (group,) = list(pol.encode(big, cfg))
    assert len(group) == 2 and group[0].target_shape == (128, 192)
    out = pol.decode(group, cfg)
    assert out.shape == (2, 64, 96, 3)


def test_check_unique_rows():
    """The debug index check (APPCORR_DEBUG_CHECKS=1) accepts distinct rows, ignores dropped (-1)
    rows and names the op when destination rows repeat."""
    import pytest
    import torch

    from appcorr_b200.ops.kernels import check_unique_rows

    check_unique_rows(torch.tensor([3, 1, -1, -1, 7], dtype=torch.int32), "x")
    with pytest.raises(RuntimeError, match="scatter_rows: 1 repeated"):
        check_unique_rows(torch.tensor([[3, 1], [3, 8]], dtype=torch.int32), "scatter_rows")
