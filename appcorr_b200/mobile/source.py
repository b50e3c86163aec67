"""Mobile request loop (reference offload/mobile/source.py:28-743).

CONFIG handshake -> time-sync ping-pong -> warm-up requests -> measured requests. Each request is
encoded group by group and streamed as soon as each group is ready; the result wait is bounded
(APPCORR_RESULT_TIMEOUT seconds, default 900). Server events are shifted onto the mobile clock
with the measured offset. Logs: logs/offload/<exp_id>_<timestamp>/{events.jsonl, summary.json}.
"""
from __future__ import annotations

import datetime
import json
import multiprocessing
import os
import queue
import re
import time
from typing import Any, Dict, List

import numpy as np

from ..common.protocol import ExperimentConfig
from ..policies import get_transmission
from .dataset import get_dataset_loader, topk_correct

_GROUP_SUFFIX = re.compile(r"_G\d+$")


def perform_time_sync(out_q, in_q, rounds: int = 10, timeout: float = 120.0) -> float:
    """Mean clock offset (server - mobile) from `rounds` ping-pongs after one warm-up ping."""
    out_q.put(("TIME_SYNC", None))
    in_q.get(timeout=timeout)
    offsets = []
    for _ in range(rounds):
        t1 = time.time()
        out_q.put(("TIME_SYNC", None))
        ts = in_q.get(timeout=timeout)
        t2 = time.time()
        offsets.append(ts - (t2 - t1) / 2 - t1)
    return sum(offsets) / len(offsets)


class SourceModule(multiprocessing.Process):
    def __init__(self, output_queue, feedback_queue, config: ExperimentConfig, data_root, loader_batch_size: int,
                 num_requests=None, num_warmup: int = 1, log_root: str = os.path.join("logs", "offload")):
        super().__init__()
        self.output_queue, self.feedback_queue = output_queue, feedback_queue
        self.config, self.data_root = config, data_root
        self.loader_batch_size = loader_batch_size
        self.num_requests, self.num_warmup = num_requests, max(int(num_warmup), 0)
        self.log_root = log_root

    # ------------------------------------------------------------------ one request
    def execute_request(self, policy, images: np.ndarray, labels, offset: float) -> Dict[str, Any]:
        cfg = self.config
        B = cfg.batch_size
        if images.shape[0] < B:  # pad a partial final batch
            pad = np.zeros((B - images.shape[0],) + images.shape[1:], images.dtype)
            images = np.concatenate([images, pad])
        events: List[Dict[str, Any]] = []
        patches = []
        t_send_start = t_stage = time.time()
        for g, group in enumerate(policy.encode(images, cfg)):
            t_enc = time.time()
            events.append({"type": f"MOBILE_ENCODE_G{g}", "timestamp": t_stage, "duration": t_enc - t_stage})
            for p in group:
                self.output_queue.put(p)
            t_tx = time.time()
            events.append({"type": f"MOBILE_SEND_G{g}", "timestamp": t_enc, "duration": t_tx - t_enc})
            patches.extend(group)
            t_stage = time.time()
        limit = float(os.environ.get("APPCORR_RESULT_TIMEOUT", 900))
        try:
            result = self.feedback_queue.get(timeout=limit)
        except queue.Empty:
            raise RuntimeError(f"no result from the server within {limit:.0f}s ({len(patches)} patches sent); "
                               "see the server log for a pipeline error or a group that never completed") from None
        t_recv = time.time()
        events.append({"type": "MOBILE_RECEIVE", "timestamp": t_recv, "duration": 0.0})
        for e in result.server_events:
            e = dict(e)
            start, end = e.pop("start"), e.pop("end")
            e["timestamp"], e["duration"] = start - offset, end - start
            events.append(e)
        events.sort(key=lambda e: e.get("timestamp", 0.0))
        return {"result": result, "events": events, "bytes": sum(len(p.data) for p in patches),
                "latency": t_recv - t_send_start, "patches": len(patches)}

    # ------------------------------------------------------------------ loop
    def run(self):
        cfg = self.config
        try:
            loader = get_dataset_loader(cfg.dataset_name, self.data_root, self.loader_batch_size, cfg.image_shape,
                                        **(cfg.dataset_kwargs or {}))
        except Exception as exc:
            self.output_queue.put(("ERROR", f"failed to load dataset {cfg.dataset_name}: {exc}"))
            self.output_queue.put("STOP")
            return
        stamp = datetime.datetime.now().strftime("%Y%m%d_%H%M%S")
        log_dir = os.path.join(self.log_root, f"{cfg.exp_id or 'exp'}_{stamp}")
        os.makedirs(log_dir, exist_ok=True)
        self.output_queue.put(("CONFIG", cfg))
        offset = perform_time_sync(self.output_queue, self.feedback_queue, timeout=float(
            os.environ.get("APPCORR_RESULT_TIMEOUT", 900)))
        policy = get_transmission(cfg.transmission_policy_name)
        batches = iter(loader)
        for _ in range(self.num_warmup):
            try:
                imgs, labels = next(batches)
            except StopIteration:
                batches = iter(loader)
                imgs, labels = next(batches)
            self.execute_request(policy, imgs, labels, offset)
        lat, per_type, correct1, correct5, seen = [], {}, 0, 0, 0
        total_bytes, cache_max = 0, 0
        with open(os.path.join(log_dir, "events.jsonl"), "w") as ef:
            for i, (imgs, labels) in enumerate(loader):
                if self.num_requests is not None and i >= self.num_requests:
                    break
                r = self.execute_request(policy, imgs, labels, offset)
                n = len(labels)
                preds = r["result"].output[:n]
                if hasattr(loader, "evaluate_batch"):  # dataset loaders with task metrics
                    try:
                        loader.evaluate_batch(preds, labels)
                    except Exception as exc:  # a malformed prediction must not end the run
                        print(f"!!! [Source] evaluate_batch: {exc}", flush=True)
                elif preds and isinstance(preds[0], dict) and "topk" in preds[0]:
                    correct1 += topk_correct(preds, labels, 1)
                    correct5 += topk_correct(preds, labels, 5)
                seen += n
                lat.append(r["latency"] * 1e3)
                total_bytes += r["bytes"]
                cache_max = max(cache_max, r["result"].cache_size_bytes)
                totals: Dict[str, float] = {}
                for e in r["events"]:
                    if e.get("include_in_latency_stats") is False or e.get("detail"):
                        continue
                    t = _GROUP_SUFFIX.sub("", e["type"])
                    totals[t] = totals.get(t, 0.0) + e.get("duration", 0.0) * 1e3
                for t, v in totals.items():
                    s = per_type.setdefault(t, {"count": 0, "sum": 0.0, "min": float("inf"), "max": float("-inf")})
                    s["count"] += 1
                    s["sum"] += v
                    s["min"] = min(s["min"], v)
                    s["max"] = max(s["max"], v)
                ef.write(json.dumps({"request": i, "latency_ms": lat[-1], "bytes": r["bytes"],
                                     "events": r["events"]}, default=float) + "\n")
        lat_sorted = sorted(lat)
        summary = {
            "exp_id": cfg.exp_id, "requests": len(lat), "images": seen,
            "latency_ms": {"mean": float(np.mean(lat)) if lat else 0.0,
                           "p50": lat_sorted[len(lat) // 2] if lat else 0.0,
                           "p99": lat_sorted[min(len(lat) - 1, int(0.99 * len(lat)))] if lat else 0.0},
            "images_per_s": (seen / (sum(lat) / 1e3)) if lat else 0.0,
            "kb_per_request": total_bytes / 1024.0 / max(len(lat), 1),
            "cache_mb_max": cache_max / 2 ** 20,
            "events": {t: {**s, "avg": s["sum"] / s["count"]} for t, s in per_type.items()},
        }
        if correct1 or correct5:
            summary["top1"] = correct1 / max(seen, 1)
            summary["top5"] = correct5 / max(seen, 1)
        if hasattr(loader, "get_summary"):
            summary["metrics"] = loader.get_summary()
        with open(os.path.join(log_dir, "summary.json"), "w") as f:
            json.dump(summary, f, indent=2, default=float)
        print(f"[Source] done: {json.dumps(summary['latency_ms'])} ms, logs in {log_dir}", flush=True)
        self.output_queue.put("STOP")
