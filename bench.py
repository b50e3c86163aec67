#!/usr/bin/env python
"""Headline benchmark: corrected-result latency and images/s of DINOv3 ViT-7B/16 serving.

One step = one request of `--batch` synthetic 512x512 images encoded as a 2-level Laplacian
pyramid (256x256 uint8 base + 512x512 int16 residual):
    reconstruct base-only canvas -> tokens -> approximate pass over all 40 layers
    -> reconstruct full canvas -> tokens -> correction pass over all 40 layers keeping the top 30%
       of patch tokens (CLS-attention server score) with cached K/V rewrite
    -> final norm -> linear segmentation head (150 classes) -> pixel labels.

Two measurements per run:
  value  device time of K steps (CUDA events, inputs already on the device), max over ranks.
  e2e    the same request through the public executor API (`get_model_executor(...)` +
         preprocess / prepare_tokens / approx_forward / correct_forward / head_inference /
         get_final_results) including the host->device copy of the pyramid from pinned memory and
         the device->host read of the labels every step.

`--impl reference` runs the unmodified reference implementation installed under baseline/_ref
through its own executor API on the same workload.

Launch: python bench.py [--gpus 1] or, for N > 1,
  python -m torch.distributed.run --nproc-per-node N --master-addr 127.0.0.1 ... bench.py --gpus N
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))

BASELINE_METRIC = "corrected-result p50/p99 latency & images/s, ViT-7B TP at 1/2/4/8 B200"
# The reference publishes no images/s figure for this config, so vs_baseline is null.
BASELINE_VALUE = None


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="mine", choices=["mine", "reference"])
    ap.add_argument("--batch", type=int, default=None, help="images per GPU (workload default)")
    ap.add_argument("--res", type=int, default=None)
    ap.add_argument("--keep", type=float, default=None)
    ap.add_argument("--arch", default=None)
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--no-graph", action="store_true",
                    help="time the device step eagerly instead of replaying its CUDA graph")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--precision", default="nvfp4", choices=["bf16", "fp8", "nvfp4"],
                    help="GEMM operand precision of the approx and correct passes (ours; the reference arm "
                         "runs its default bf16 path: its fp8/fp4 approx controllers need torchao)")
    ap.add_argument("--workload", default="vit7b_seg", choices=["vit7b_seg", "vitl_cls", "vitl_detr", "vlm", "cpu_loopback"],
                    help="vit7b_seg: the headline ViT-7B linear-head segmentation config; vitl_cls: ViT-L/16 classifier, "
                         "224^2, 64 images per GPU, 3-level pyramid, keep 0.25 (data-parallel); vitl_detr: ViT-L/16 + "
                         "6-layer DETR decoder (300 queries, 80 classes), 1024^2, batch 4, keep 0.5, 3x3 windows + "
                         "global source; vlm: Qwen2.5-VL-7B-shaped prefill with KV rewrite (1 image 1024^2 + 128 text "
                         "tokens, keep 0.25); cpu_loopback: ViT-S/16 fp32 on the CPU over loopback TCP, 224^2, batch 4, "
                         "2-level pyramid, keep 0.5 (p50 / p99 latency)")
    ap.add_argument("--parallel", default=None, choices=["tp", "dp"],
                    help="N > 1: tensor-parallel over N GPUs (one request batch) or N data-parallel replicas")
    a = ap.parse_args()
    wl = WORKLOADS.get(a.workload, WORKLOADS["vit7b_seg"])
    for k in ("batch", "res", "keep", "arch", "parallel"):
        if getattr(a, k) is None:
            setattr(a, k, wl[k])
    return a


# ----------------------------------------------------------------------------- workloads
# the BASELINE configurations other than the headline (vit7b_seg): model, backbone, image side,
# images per GPU, pyramid levels (coarse first), keep ratio, default parallelism
WORKLOADS = {
    "vit7b_seg": dict(model="dinov3_segmentor_linhead", arch="vit7b16", res=512, batch=8, levels=[1, 0], keep=0.3,
                      parallel="tp", label="DINOv3 ViT-7B/16 + linear seg head (150 cls)",
                      profile="dinov3_ade20k_linhead_official"),
    "vitl_cls": dict(model="dinov3_classifier", arch="vitl16", res=224, batch=64, levels=[2, 1, 0], keep=0.25,
                     parallel="dp", label="DINOv3 ViT-L/16 + linear classifier (1000 cls)", profile="fixed_image_shape",
                     metric="images/s, ViT-L/16 data-parallel at 1/2/4/8 B200 (224^2, 3-level pyramid, keep 0.25)"),
    "vitl_detr": dict(model="dinov3_detector", arch="vitl16", res=1024, batch=4, levels=[1, 0], keep=0.5,
                      parallel="tp", label="DINOv3 ViT-L/16 (3x3 windows + global source) + 6-layer DETR, 300 q, 80 cls",
                      profile="fixed_image_shape",
                      metric="p50/p99 latency & images/s, ViT-L + DETR decoder, 1024^2 batch 4"),
}


# ----------------------------------------------------------------------------- data
def synthetic_pyramid_levels(batch: int, res: int, levels, seed: int):
    """Clipped N(128, 60^2) images -> (images, base uint8, [int16 residual of each finer level,
    coarse first]) for a Laplacian pyramid over `levels` (e.g. [2, 1, 0])."""
    sys.path.insert(0, ROOT)
    from appcorr_b200.policies.transmission.pyramid import pyr_down, pyr_up

    rng = np.random.default_rng(seed)
    imgs = np.clip(rng.normal(128, 60, size=(batch, res, res, 3)), 0, 255).astype(np.uint8)
    pyr = [imgs]
    for _ in range(levels[0]):
        pyr.append(np.stack([pyr_down(im) for im in pyr[-1]]))
    base = pyr[levels[0]]
    resid = []
    for lvl in levels[1:]:  # residual of level lvl against the reconstruction from level lvl + 1
        fine, coarse = pyr[lvl], pyr[lvl + 1]
        resid.append(np.stack([f.astype(np.int16) - pyr_up(c).astype(np.int16) for f, c in zip(fine, coarse)]))
    return imgs, base, resid


def synthetic_pyramid(batch: int, res: int, seed: int):
    """Clipped N(128, 60^2) RGB images -> (images, base uint8, residual int16) on the host."""
    sys.path.insert(0, ROOT)
    from appcorr_b200.policies.transmission.pyramid import pyr_down, pyr_up

    rng = np.random.default_rng(seed)
    imgs = np.clip(rng.normal(128, 60, size=(batch, res, res, 3)), 0, 255).astype(np.uint8)
    base = np.stack([pyr_down(im) for im in imgs])
    res_ = np.stack([im.astype(np.int16) - pyr_up(b).astype(np.int16) for im, b in zip(imgs, base)])
    return imgs, base, res_


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self):
        self.proc = None
        self.path = None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self, gpu_indices):
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                idx = int(parts[0])
            except ValueError:
                continue
            if gpu_indices is not None and idx not in gpu_indices:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                pass
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return None
        busy = [s for s in sm if mx is None or s > 0.5 * mx] or sm
        return {"sm_mhz": statistics.median(busy), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ----------------------------------------------------------------------------- distributed
def dist_setup(n_gpus: int):
    import torch

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(v: float, world: int) -> float:
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([v], device="cuda", dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


# ----------------------------------------------------------------------------- our implementation
def _cfg_precision(args) -> str:
    """Experiment-config spelling of --precision (the reference's config calls NVFP4 "fp4")."""
    return "fp4" if args.precision == "nvfp4" else args.precision


def make_config(args, world: int = 1):
    sys.path.insert(0, ROOT)
    from appcorr_b200.common.protocol import ExperimentConfig

    tp = world if (world > 1 and args.parallel == "tp") else 1
    wl = WORKLOADS[args.workload]
    prof = {"backbone_arch": args.arch, "server_inference_mode": "whole"}
    if args.workload == "vitl_detr":
        prof.update({"num_queries": 300, "num_classes": 80, "decoder_layers": 6, "detector_windows": 3})
    return ExperimentConfig(
        tp_size=tp, precision=_cfg_precision(args), correct_precision=_cfg_precision(args),
        exp_id="bench", model_name=wl["model"], batch_size=args.batch,
        image_shape=(args.res, args.res, 3), input_profile_name=wl["profile"],
        input_profile_kwargs=prof,
        scheduler_policy_name="GroupTrigger", transmission_policy_name="ProgressiveLaplacian",
        transmission_kwargs={"pyramid_levels": wl["levels"], "num_groups": 1, "grouping_strategy": "grid"},
        appcorr_kwargs={"token_keep_ratio": args.keep, "server_pscore": "cls_attn_prob"})


def run_mine(args, rank, world):
    import torch

    sys.path.insert(0, ROOT)
    from appcorr_b200.common.protocol import Task
    from appcorr_b200.ops import kernels as K
    from appcorr_b200.ops.native import check_errors
    from appcorr_b200.server.model import PyramidBatch, get_model_executor

    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = make_config(args, world)
    tp = cfg.tp_size > 1
    ex = get_model_executor(cfg.model_name, dev)
    ex.load_model(cfg.model_name, cfg)
    L = ex.cfg.depth
    # tensor parallel: every rank serves the same request; data parallel: independent requests
    levels = WORKLOADS[args.workload]["levels"]
    imgs, base, resid = synthetic_pyramid_levels(args.batch, args.res, levels, seed=0 if tp else rank)
    base_h = torch.from_numpy(base).pin_memory()
    res_hs = [torch.from_numpy(r).pin_memory() for r in resid]
    res_h = res_hs if len(res_hs) > 1 else res_hs[0]
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])

    # ---- device-resident variant for the kernel-time measurement
    base_d = base_h.to(dev)
    res_d = [r.to(dev) for r in res_hs] if len(res_hs) > 1 else res_hs[0].to(dev)

    def device_step(ctx):
        ex.preprocess(PyramidBatch(base_d, None, levels=levels), task, ctx, cfg)
        ex.prepare_tokens(task, ctx, cfg)
        ex.approx_forward({"layers": (0, L)}, ctx, cfg)
        ex.preprocess(PyramidBatch(base_d, res_d, levels=levels), task, ctx, cfg)
        ex.prepare_tokens(task, ctx, cfg)
        ex.correct_forward({"layers": (0, L), "group_id": 1}, ctx, cfg)
        ex.head_inference(task, ctx, cfg)

    ctx = {}
    for _ in range(args.warmup):
        device_step(ctx)
    torch.cuda.synchronize()
    check_errors(dev)
    n0 = K.LAUNCHES[0]
    device_step(ctx)
    launches_per_step = K.LAUNCHES[0] - n0
    torch.cuda.synchronize()
    step_fn = device_step
    graphed = False
    if not args.no_graph:
        # the whole step (pyramid decode, approx, plan, correct, head) has no host synchronisation,
        # so it is captured once and replayed; tensor-parallel barriers keep their epochs on the
        # device, so a replay on every rank takes fresh epochs
        graph = torch.cuda.CUDAGraph()
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            device_step(ctx)
        torch.cuda.current_stream().wait_stream(side)
        with torch.cuda.graph(graph):
            device_step(ctx)
        graph.replay()
        torch.cuda.synchronize()
        check_errors(dev)
        step_fn = lambda _ctx: graph.replay()  # noqa: E731
        graphed = True

    clocks = ClockSampler() if rank == 0 else None
    timer = getattr(ex.engine, "timer", None)
    if timer is not None and timer.enabled:
        timer.summary(reset=True)
    barrier(world)
    torch.cuda.synchronize()
    if clocks:
        clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    step_ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    t0.record()
    step_ev[0].record()
    torch.cuda.nvtx.range_push("timed")  # lets a profiler select exactly the timed steps
    for i in range(args.steps):
        step_fn(ctx)
        step_ev[i + 1].record()
    torch.cuda.nvtx.range_pop()
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop(None) if clocks else None
    check_errors(dev)
    ms = t0.elapsed_time(t1) / args.steps
    per_step = sorted(step_ev[i].elapsed_time(step_ev[i + 1]) for i in range(args.steps))
    ms_max = max_over_ranks(ms, world)
    if timer is not None and timer.enabled:  # APPCORR_PHASE_TIMING=1: per-phase device ms per step
        phases = {k: round(v / args.steps, 3) for k, v in sorted(timer.summary().items())}
        print(json.dumps({"rank": rank, "phase_ms_per_step": phases}), file=sys.stderr)

    # ---- end-to-end through the public API: pinned host inputs in, labels out, every step
    e2e = None
    if not args.no_e2e:
        n_e2e = args.e2e_steps or max(3, args.steps)
        h2d = base_h.numel() * base_h.element_size() + sum(r.numel() * r.element_size() for r in res_hs)
        d2h = {"vit7b_seg": args.batch * args.res * args.res,          # uint8 labels
               "vitl_cls": args.batch * 5 * (8 + 4),                   # top-5 (index, probability)
               "vitl_detr": args.batch * 100 * (4 + 8 + 16)}[args.workload]  # 100 x (score, label, box)
        ctx2 = {}

        def e2e_step():
            ex.preprocess(PyramidBatch(base_h, None, levels=levels), task, ctx2, cfg)
            ex.prepare_tokens(task, ctx2, cfg)
            ex.approx_forward({"layers": (0, L)}, ctx2, cfg)
            ex.preprocess(PyramidBatch(base_h, res_h, levels=levels), task, ctx2, cfg)
            ex.prepare_tokens(task, ctx2, cfg)
            ex.correct_forward({"layers": (0, L), "group_id": 1}, ctx2, cfg)
            ex.head_inference(task, ctx2, cfg)
            return ex.get_final_results(task, ctx2, cfg)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        lat = []
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n_e2e):
            s = time.perf_counter()
            out = e2e_step()
            lat.append((time.perf_counter() - s) * 1e3)
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / n_e2e, world)
        assert len(out) == args.batch
        if args.workload == "vit7b_seg":
            assert out[0]["mask"].shape == (args.res, args.res)
        lat.sort()
        e2e = {"value": round(args.batch * (1 if tp else world) * 1e3 / e2e_ms, 3), "unit": "images/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
               "p50_ms": round(lat[len(lat) // 2], 3), "p99_ms": round(lat[min(len(lat) - 1, int(0.99 * len(lat)))], 3),
               "ms_per_step": round(e2e_ms, 3)}
    return ms_max, per_step, launches_per_step, clk, e2e, graphed


# ----------------------------------------------------------------------------- VLM workload
def run_vlm(args, rank, world):
    """Qwen2.5-VL-shaped prefill: approx round on the pyramid base, correction round with the
    full image (K/V rewrite of the top 25% image tokens + the text), first token. One request
    per rank per step (data parallel)."""
    import torch

    sys.path.insert(0, ROOT)
    from appcorr_b200.common.protocol import ExperimentConfig, Task
    from appcorr_b200.ops import kernels as K
    from appcorr_b200.ops.native import check_errors
    from appcorr_b200.server.model import PyramidBatch, get_model_executor

    dev = torch.device("cuda", torch.cuda.current_device())
    res = 1024
    tp = world if (world > 1 and args.parallel == "tp") else 1
    cfg = ExperimentConfig(
        exp_id="bench_vlm", model_name="qwen25vl", batch_size=1, image_shape=(res, res, 3), tp_size=tp,
        precision=_cfg_precision(args), correct_precision=_cfg_precision(args),
        input_profile_kwargs={"vlm_arch": "qwen25vl7b", "n_text": 128, "n_text_before": 16, "seed": 0},
        scheduler_policy_name="GroupTrigger", transmission_policy_name="ProgressiveLaplacian",
        transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 1, "grouping_strategy": "grid"},
        appcorr_kwargs={"token_keep_ratio": 0.25})
    ex = get_model_executor("qwen25vl", dev)
    ex.load_model("qwen25vl", cfg)
    _, base, resid = synthetic_pyramid(1, res, seed=0 if tp > 1 else rank)
    base_h = torch.from_numpy(base).pin_memory()
    res_h = torch.from_numpy(resid).pin_memory()
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])

    def step(b, r, ctx):
        ex.preprocess(PyramidBatch(b, None), task, ctx, cfg)
        ex.prepare_tokens(task, ctx, cfg)
        ex.approx_forward({}, ctx, cfg)
        ex.preprocess(PyramidBatch(b, r), task, ctx, cfg)
        ex.prepare_tokens(task, ctx, cfg)
        ex.correct_forward({}, ctx, cfg)
        ex.head_inference(task, ctx, cfg)

    base_d, res_d = base_h.to(dev), res_h.to(dev)
    ctx = {}
    for _ in range(args.warmup):
        step(base_d, res_d, ctx)
    torch.cuda.synchronize()
    check_errors(dev)
    n0 = K.LAUNCHES[0]
    step(base_d, res_d, ctx)
    launches = K.LAUNCHES[0] - n0
    clocks = ClockSampler() if rank == 0 else None
    torch.cuda.synchronize()
    barrier(world)
    if clocks:
        clocks.start()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    ev[0].record()
    for i in range(args.steps):
        step(base_d, res_d, ctx)
        ev[i + 1].record()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop(None) if clocks else None
    check_errors(dev)
    ms = max_over_ranks(ev[0].elapsed_time(ev[-1]) / args.steps, world)
    per = sorted(ev[i].elapsed_time(ev[i + 1]) for i in range(args.steps))
    e2e = None
    if not args.no_e2e:
        ctx2 = {}

        def e2e_step():
            step(base_h, res_h, ctx2)
            return ex.get_final_results(task, ctx2, cfg)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        barrier(world)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n = max(3, args.steps)
        e0.record()
        for _ in range(n):
            out = e2e_step()
        e1.record()
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(e0.elapsed_time(e1) / n, world)
        assert "first_token" in out[0]
        e2e = {"value": round((1 if tp > 1 else world) * 1e3 / e2e_ms, 3), "unit": "requests/s",
               "h2d_bytes_per_step": int(base_h.numel() + res_h.numel() * 2), "d2h_bytes_per_step": 8,
               "ms_per_step": round(e2e_ms, 3)}
    if rank == 0:
        c = ex.cfg
        print(json.dumps({
            "metric": "VLM prefill approx+correct with KV rewrite (requests/s)",
            "value": round((1 if tp > 1 else world) * 1e3 / ms, 3),
            "unit": "requests/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(ms, 3), "p50_ms": round(per[len(per) // 2], 3), "p99_ms": round(per[-1], 3),
            "higher_is_better": True, "scaling": "strong" if tp > 1 else "weak", "vs_baseline": None,
            "dtype": "bf16" if args.precision == "bf16" else "fp8-e4m3 LLM GEMM operands, bf16 vision tower",
            "data": "synthetic 1024x1024 image + 128 random text ids, random-init weights",
            "config": {"model": "Qwen2.5-VL-7B-shaped (LLM 28x3584, GQA 28/4, FFN 18944; ViT 32x1280)",
                       "image_tokens": ex._sessions and next(iter(ex._sessions.values())).n_img,
                       "text_tokens": 128, "keep_ratio": 0.25, "kv_cache": "paged, 128-row pages",
                       "parallelism": (f"tp{world}" if tp > 1 else f"dp{world}") if world > 1 else "single",
                       "llm_layers": c.depth},
            "gpu_launches": int(launches * args.steps), "clocks": clk, "e2e": e2e}))


# ----------------------------------------------------------------------------- CPU loopback
def run_cpu_loopback(args) -> None:
    """the CPU fp32 server (ViT-S/16) and the mobile client over loopback TCP,
    224^2 batch 4, 2-level pyramid, top 50% corrected by residual energy; the client's measured
    request latencies (send of the first patch to the result) give p50 / p99."""
    import socket
    import tempfile

    def port():
        with socket.socket() as so:
            so.bind(("127.0.0.1", 0))
            return so.getsockname()[1]

    sys.path.insert(0, ROOT)
    from appcorr_b200.mobile.main import load_config, run_mobile

    rp, sp = port(), port()
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT)
    srv = subprocess.Popen([sys.executable, "-m", "offload.server.main", "--recv-port", str(rp), "--send-port", str(sp),
                            "--listen-host", "127.0.0.1", "--device", "cpu", "--group-port", str(port())],
                           cwd=ROOT, env=env, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    try:
        time.sleep(3)
        cfg = load_config(os.path.join(ROOT, "offload/config/cpu_vits16_loopback_keep05.json"),
                          [f"dataset_kwargs.num_batches={args.steps + 1}"])
        with tempfile.TemporaryDirectory() as logs:
            rc = run_mobile("127.0.0.1", rp, sp, None, None, num_request=args.steps, num_warmup=args.warmup,
                            config=cfg, log_root=logs)
            runs = os.listdir(logs)
            summ = json.load(open(os.path.join(logs, runs[0], "summary.json"))) if runs else {}
    finally:
        srv.terminate()
        try:
            srv.wait(timeout=30)
        except subprocess.TimeoutExpired:
            srv.kill()
    lat = summ.get("latency_ms", {})
    print(json.dumps({"metric": "CPU fp32 end-to-end latency over loopback TCP (p50 ms), ViT-S/16 224^2 batch 4",
                      "value": round(float(lat.get("p50", 0.0)), 3), "unit": "ms", "n_gpus": 0, "steps": args.steps,
                      "warmup": args.warmup, "p50_ms": lat.get("p50"), "p99_ms": lat.get("p99"),
                      "mean_ms": lat.get("mean"), "images_per_s": summ.get("images_per_s"),
                      "higher_is_better": False, "scaling": "none", "vs_baseline": None, "dtype": "fp32",
                      "data": "synthetic images, random-init weights", "rc": rc,
                      "config": {"model": "DINOv3 ViT-S/16 + linear classifier", "global_batch": 4, "image": "224x224",
                                 "pyramid_levels": [1, 0], "keep_ratio": 0.5, "transport": "loopback TCP"}}))


# ----------------------------------------------------------------------------- reference arm
def run_reference(args, rank, world):
    """Reference executor (baseline/_ref, unmodified) on the same synthetic workload.

    Two accommodations, neither touching the compute path: the `nvtx` Python package it imports
    is not installed here, so a no-op stand-in is registered; and there are no checkpoints, so
    its weight loader is pointed at the randomly initialised modules it just built.
    """
    import types

    import torch

    ref_root = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(ref_root, "offload")):
        return None, "baseline/_ref/offload missing (reference not installed)"
    imgs, base, resid = synthetic_pyramid(args.batch, args.res, seed=rank)
    from appcorr_b200.policies.transmission.pyramid import pyr_up  # before this repo leaves sys.path

    # This repository ships its own `offload` compatibility package; the reference's `offload`
    # must win, so the repository root leaves sys.path and any already-imported `offload` goes.
    here = {os.path.abspath(p) for p in ("", ".", ROOT)}
    sys.path[:] = [p for p in sys.path if os.path.abspath(p or ".") not in here]
    for name in [m for m in sys.modules if m == "offload" or m.startswith("offload.")]:
        del sys.modules[name]
    sys.path.insert(0, ref_root)
    if "nvtx" not in sys.modules:
        nv = types.ModuleType("nvtx")

        def annotate(*a, **k):
            if a and callable(a[0]) and not k:
                return a[0]
            return lambda f: f

        nv.annotate = annotate
        sys.modules["nvtx"] = nv
    from offload.common.protocol import ExperimentConfig, Task  # reference's own classes
    import offload.server.model.dinov3_segmentor_linhead as lh

    holder = {}
    orig_vit = None

    def fake_loader(path):
        if "head" in str(path):
            D = holder["backbone"].embed_dim
            g = torch.Generator().manual_seed(0)
            sd = {"batchnorm_layer.weight": 1 + 0.1 * torch.randn(D, generator=g),
                  "batchnorm_layer.bias": 0.1 * torch.randn(D, generator=g),
                  "batchnorm_layer.running_mean": 0.1 * torch.randn(D, generator=g),
                  "batchnorm_layer.running_var": 1 + 0.1 * torch.rand(D, generator=g),
                  "batchnorm_layer.num_batches_tracked": torch.tensor(0),
                  "conv.weight": 0.02 * torch.randn(150, D, 1, 1, generator=g), "conv.bias": torch.zeros(150)}
            return {"segmentation_model.1." + k: v for k, v in sd.items()}
        return holder["backbone"].state_dict()

    lh.load_weight_mmap = fake_loader
    lh.DINOv3SegmentorLinheadExecutor._ensure_dinov3_import_path()
    import dinov3.hub.backbones as hb

    orig_vit = hb.dinov3_vit7b16

    def capture_vit(*a, **k):
        m = orig_vit(*a, **k)
        holder["backbone"] = m
        return m

    hb.dinov3_vit7b16 = capture_vit
    dev = torch.device("cuda", torch.cuda.current_device())
    cfg = ExperimentConfig(
        exp_id="bench_ref", model_name="dinov3_segmentor_linhead", batch_size=args.batch,
        image_shape=(args.res, args.res, 3), input_profile_name="dinov3_ade20k_linhead_official",
        input_profile_kwargs={"server_inference_mode": "whole"},
        scheduler_policy_name="GroupTrigger", transmission_policy_name="ProgressiveLaplacian",
        transmission_kwargs={"pyramid_levels": [1, 0], "num_groups": 1, "grouping_strategy": "grid"},
        appcorr_kwargs={"token_keep_ratio": args.keep, "server_pscore": "cls_attn_prob"})
    ex = lh.DINOv3SegmentorLinheadExecutor(dev)
    ex.load_model("dinov3_segmentor_linhead", cfg)
    L = len(ex.vit_backbone.blocks)
    approx_imgs = [pyr_up(b) for b in base]
    task = Task(task_id=0, request_id=0, payload=[], instructions=[])

    def step():
        ctx = {}
        ex.preprocess(approx_imgs, task, ctx, cfg)
        ex.prepare_tokens(task, ctx, cfg)
        ex.approx_forward({"layers": (0, L)}, ctx, cfg)
        ex.preprocess(list(imgs), task, ctx, cfg)
        ex.prepare_tokens(task, ctx, cfg)
        ex.correct_forward({"layers": (0, L), "group_id": 1}, ctx, cfg)
        ex.head_inference(task, ctx, cfg)
        return ex.get_final_results(task, ctx, cfg)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    clocks = ClockSampler() if rank == 0 else None
    if clocks:
        clocks.start()
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    lat = []
    t0.record()
    for _ in range(args.steps):
        s = time.perf_counter()
        out = step()
        lat.append((time.perf_counter() - s) * 1e3)
    t1.record()
    torch.cuda.synchronize()
    barrier(world)
    clk = clocks.stop(None) if clocks else None
    ms = max_over_ranks(t0.elapsed_time(t1) / args.steps, world)
    assert len(out) == args.batch
    lat.sort()
    # every step uploads the approximate canvas and the full image (uint8 HWC, the reference's
    # preprocess input) and reads back one uint8 label mask per image
    h2d = int(sum(a.nbytes for a in approx_imgs) + sum(a.nbytes for a in imgs))
    d2h = int(sum(np.asarray(v["mask"]).nbytes for v in out.values()))
    return {"ms": ms, "p50": lat[len(lat) // 2], "p99": lat[min(len(lat) - 1, int(0.99 * len(lat)))],
            "clocks": clk, "h2d": h2d, "d2h": d2h}, None


def main():
    args = parse_args()
    world_env = int(os.environ.get("WORLD_SIZE", "1"))
    if args.gpus != world_env and world_env == 1 and args.gpus > 1:
        print(json.dumps({"error": "for --gpus > 1 launch with torch.distributed.run"}))
        sys.exit(2)
    if args.workload == "cpu_loopback":  # host-only: no device, no process group
        if int(os.environ.get("RANK", "0")) == 0:
            run_cpu_loopback(args)
        return
    rank, world, local = dist_setup(args.gpus)
    if args.workload == "vlm":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference's Qwen2.5-VL executor loads "
                                  "HF checkpoints (transformers from_pretrained); none exist offline"}))
        else:
            run_vlm(args, rank, world)
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    wl = WORKLOADS[args.workload]
    metric = wl.get("metric", BASELINE_METRIC)
    parallelism = (f"{args.parallel}{world}" if world > 1 else "single")
    images_per_step = args.batch * (world if (world > 1 and args.parallel == "dp") else 1)
    cfg_out = {"model": wl["label"] if args.arch == wl["arch"] else args.arch, "workload": args.workload,
               "global_batch": images_per_step, "per_gpu_batch": args.batch, "seq_len": (args.res // 16) ** 2 + 5,
               "image": f"{args.res}x{args.res}", "keep_ratio": args.keep, "pyramid_levels": wl["levels"],
               "parallelism": parallelism, "precision": args.precision if args.impl == "mine" else "bf16",
               "l2": "working set > L2 each step (13.4 GB bf16 weights + 8 GB K/V/increment caches)"}
    if args.impl == "reference" and args.workload != "vit7b_seg":
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the reference arm runs the headline workload "
                              "(vit7b_seg); this workload has no reference run"}))
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    if args.impl == "reference":
        try:
            res, why = run_reference(args, rank, world)
        except Exception as exc:  # report, do not crash the driver
            res, why = None, f"{type(exc).__name__}: {exc}"[:300]
        if rank == 0:
            if res is None:
                print(json.dumps({"impl": "reference", "unavailable": why}))
            else:
                v = args.batch * world * 1e3 / res["ms"]
                print(json.dumps({"impl": "reference", "metric": BASELINE_METRIC, "value": round(v, 3),
                                  "unit": "images/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                                  "ms_per_step": round(res["ms"], 3), "p50_ms": round(res["p50"], 3),
                                  "p99_ms": round(res["p99"], 3), "higher_is_better": True,
                                  "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
                                  "data": "synthetic images, random-init weights", "config": cfg_out,
                                  "clocks": res["clocks"],
                                  # the reference's timed loop is already end to end: host images in
                                  # through its executor API, host masks out
                                  "e2e": {"value": round(v, 3), "unit": "images/s",
                                          "h2d_bytes_per_step": res["h2d"], "d2h_bytes_per_step": res["d2h"],
                                          "ms_per_step": round(res["ms"], 3),
                                          "note": "same loop as value: host uint8 images in, host masks out"}}))
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return
    ms, per_step, launches, clk, e2e, graphed = run_mine(args, rank, world)
    cfg_out["cuda_graph"] = graphed
    if rank == 0:
        value = images_per_step * 1e3 / ms
        line = {"metric": metric, "value": round(value, 3), "unit": "images/s", "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 3),
                "p50_ms": round(per_step[len(per_step) // 2], 3),
                "p99_ms": round(per_step[min(len(per_step) - 1, int(0.99 * len(per_step)))], 3),
                "higher_is_better": True, "scaling": "strong" if parallelism.startswith("tp") else "weak",
                "vs_baseline": (round(value / BASELINE_VALUE, 4) if BASELINE_VALUE else None),
                "dtype": ("bf16" if args.precision == "bf16" else
                          "fp8-e4m3 GEMM operands (per-row activation / per-channel weight scales, fp32 "
                          "accumulate), bf16 attention and residual stream" if args.precision == "fp8" else
                          "nvfp4 qkv / fc1 / fc2 GEMM operands (e2m1 + ue4m3 per 16 + fp32 per row / channel), "
                          "e4m3 attn.proj, fp32 accumulate, bf16 attention and residual stream"),
                "data": "synthetic images (clipped N(128,60^2)), random-init weights",
                "config": cfg_out, "gpu_launches": int(launches * args.steps), "clocks": clk, "e2e": e2e}
        if args.workload != "vit7b_seg":
            line["scaling"] = "weak" if args.parallel == "dp" or world == 1 else "strong"
            line["dtype"] = args.precision
        print(json.dumps(line))
    if world > 1:
        import torch.distributed as dist

        dist.destroy_process_group()


if __name__ == "__main__":
    main()
