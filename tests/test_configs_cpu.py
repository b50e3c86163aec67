"""Every shipped experiment config (offload/config/*.json) parses through ExperimentConfig and
names a registered scheduler, transmission policy, model executor and input profile; presets named
in the input profile exist; and each config's scheduler emits a first task for a base group."""
import glob
import json
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CONFIGS = sorted(glob.glob(os.path.join(ROOT, "offload", "config", "*.json")))


def test_config_corpus_is_present():
    assert len(CONFIGS) >= 25


@pytest.mark.parametrize("path", CONFIGS, ids=[os.path.basename(p) for p in CONFIGS])
def test_config_loads_and_resolves(path):
    import itertools

    from appcorr_b200.common.protocol import ExperimentConfig, Patch, normalize_appcorr_kwargs
    from appcorr_b200.policies import SCHEDULER_REGISTRY, TRANSMISSION_REGISTRY, get_scheduler
    from appcorr_b200.server import model as models

    raw = json.load(open(path))
    assert raw["exp_id"] == os.path.splitext(os.path.basename(path))[0]
    cfg = ExperimentConfig(**raw)
    assert cfg.scheduler_policy_name in SCHEDULER_REGISTRY
    assert cfg.transmission_policy_name in TRANSMISSION_REGISTRY
    prof = cfg.get_input_profile_config()
    normalize_appcorr_kwargs(cfg.appcorr_kwargs, cfg.transmission_kwargs)
    # the executor class resolves by model name (construction only; weights load at CONFIG time)
    ex = models.get_model_executor(cfg.model_name, __import__("torch").device("cpu"))
    assert ex is not None
    for key, table in (("backbone_arch", "appcorr_b200.models.dinov3.vit:PRESETS"),
                       ("clip_arch", "appcorr_b200.models.clip:CLIP_PRESETS"),
                       ("vlm_arch", "appcorr_b200.models.qwen25vl:PRESETS"),
                       ("sam3_arch", "appcorr_b200.models.sam3:SAM3_PRESETS")):
        if key in prof:
            mod, name = table.split(":")
            assert prof[key] in getattr(__import__(mod, fromlist=[name]), name), (key, prof[key])
    # a complete base group triggers the first task
    sched = get_scheduler(cfg.scheduler_policy_name, cfg)
    n = cfg.batch_size
    buf = [Patch(image_idx=i, spatial_idx=0, data=b"", res_level=1, group_id=0, batch_group_total=n,
                 num_correction_groups=1) for i in range(n)]
    task = sched.decide(buf, cfg, itertools.count())
    assert task is not None and task.instructions


def test_sweep_grid_points():
    from appcorr_b200.sweep import flatten, grid_points

    pts = grid_points(["appcorr_kwargs.token_keep_ratio=0.2,0.4", "precision=bf16"])
    assert pts == [{"appcorr_kwargs.token_keep_ratio": "0.2", "precision": "bf16"},
                   {"appcorr_kwargs.token_keep_ratio": "0.4", "precision": "bf16"}]
    assert flatten({"a": {"b": 1, "c": [1]}, "d": 2}) == {"a.b": 1, "d": 2}


@pytest.mark.timeout(600)
def test_sweep_runs_two_points_on_cpu(tmp_path):
    """Two grid points of the CPU loopback config end to end (server + client per point)."""
    import csv
    import subprocess
    import sys

    out = tmp_path / "s.csv"
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", APPCORR_RESULT_TIMEOUT="240")
    rc = subprocess.run([sys.executable, "-m", "appcorr_b200.sweep", "--config",
                         os.path.join(ROOT, "offload/config/cpu_vits16_loopback_keep05.json"),
                         "--grid", "appcorr_kwargs.token_keep_ratio=0.25,0.5", "--grid", "dataset_kwargs.num_batches=2",
                         "--num-request", "1", "--server-args", "--device cpu", "--out", str(out)],
                        cwd=ROOT, env=env, timeout=580).returncode
    rows = list(csv.DictReader(open(out)))
    assert rc == 0 and len(rows) == 2, rows
    assert {r["appcorr_kwargs.token_keep_ratio"] for r in rows} == {"0.25", "0.5"}
    assert all(float(r["latency_p50_ms"]) > 0 for r in rows)


# The reference's own experiment corpus (offload/config/**.json of the installed reference under
# baseline/_ref, when it is installed): every file must parse through this build's
# ExperimentConfig unchanged and resolve to registered policies, executors and input profiles.
REF_CONFIGS = sorted(glob.glob(os.path.join(ROOT, "baseline", "_ref", "offload", "config", "**", "*.json"),
                            recursive=True))


@pytest.mark.skipif(not REF_CONFIGS, reason="reference not installed (bash baseline/install_reference.sh)")
@pytest.mark.parametrize("path", REF_CONFIGS or ["none"],
                         ids=[os.path.relpath(p, os.path.join(ROOT, "baseline", "_ref", "offload", "config"))
                              for p in REF_CONFIGS] or ["none"])
def test_reference_config_loads(path):
    import itertools

    import torch

    from appcorr_b200.common.protocol import ExperimentConfig, Patch, normalize_appcorr_kwargs
    from appcorr_b200.policies import SCHEDULER_REGISTRY, TRANSMISSION_REGISTRY, get_scheduler
    from appcorr_b200.server import model as models

    cfg = ExperimentConfig(**json.load(open(path)))
    assert cfg.scheduler_policy_name in SCHEDULER_REGISTRY
    assert cfg.transmission_policy_name in TRANSMISSION_REGISTRY
    cfg.get_input_profile_config()
    normalize_appcorr_kwargs(cfg.appcorr_kwargs, cfg.transmission_kwargs)
    assert models.get_model_executor(cfg.model_name, torch.device("cpu")) is not None
    sched = get_scheduler(cfg.scheduler_policy_name, cfg)
    n = cfg.batch_size
    buf = [Patch(image_idx=i, spatial_idx=0, data=b"", res_level=1, group_id=0, batch_group_total=n,
                 num_correction_groups=1) for i in range(n)]
    task = sched.decide(buf, cfg, itertools.count())
    assert task is not None and task.instructions
