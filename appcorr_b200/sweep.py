"""Local sweep driver: one server + mobile client per point of an override grid
(the reference's offload/run_local.sh and scripts/*.sh sweeps, in Python).

    python -m appcorr_b200.sweep --config offload/config/imagenet_vit7b_interleaved_g4.json \\
        --grid appcorr_kwargs.token_keep_ratio=0.2,0.4,0.6 --grid precision=bf16,fp8 \\
        --num-request 20 --out sweep.csv [--server-args "--tp 2"] [--data /path/to/dataset]

Each point starts `offload.server.main` on free loopback ports, runs the mobile client with the
point's `--set` overrides, stops the server and appends one CSV row: the overrides, latency
mean / p50 / p99, images/s, KB per request, cache size and the task metrics of summary.json.
"""
from __future__ import annotations

import argparse
import csv
import itertools
import json
import os
import shlex
import socket
import subprocess
import sys
import tempfile
import time
from typing import Dict, List

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def grid_points(grid: List[str]) -> List[Dict[str, str]]:
    """["a=1,2", "b=x"] -> [{"a": "1", "b": "x"}, {"a": "2", "b": "x"}]."""
    keys, values = [], []
    for g in grid:
        k, v = g.split("=", 1)
        keys.append(k)
        values.append(v.split(","))
    return [dict(zip(keys, combo)) for combo in itertools.product(*values)] if keys else [{}]


def flatten(d, prefix="") -> Dict[str, object]:
    out = {}
    for k, v in (d or {}).items():
        if isinstance(v, dict):
            out.update(flatten(v, f"{prefix}{k}."))
        elif not isinstance(v, (list, tuple)):
            out[f"{prefix}{k}"] = v
    return out


def run_point(config: str, point: Dict[str, str], num_request: int, num_warmup: int, data: str, server_args: str,
              timeout: float) -> Dict[str, object]:
    rp, sp = free_port(), free_port()
    env = dict(os.environ, PYTHONPATH=ROOT + os.pathsep + os.environ.get("PYTHONPATH", ""))
    srv = subprocess.Popen([sys.executable, "-m", "offload.server.main", "--recv-port", str(rp), "--send-port", str(sp),
                            "--listen-host", "127.0.0.1", "--group-port", str(free_port()), *shlex.split(server_args)],
                           cwd=ROOT, env=env, stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
    row: Dict[str, object] = dict(point)
    with tempfile.TemporaryDirectory() as logs:
        try:
            time.sleep(3)
            cmd = [sys.executable, "-m", "offload.mobile.main", "--ip", "127.0.0.1", "--recv-port", str(rp),
                   "--send-port", str(sp), "--config", config, "-nr", str(num_request), "-nw", str(num_warmup),
                   "--log-root", logs]
            if data:
                cmd += ["--data", data]
            for k, v in point.items():
                cmd += ["--set", f"{k}={v}"]
            rc = subprocess.run(cmd, cwd=ROOT, env=env, timeout=timeout).returncode
            row["rc"] = rc
            runs = sorted(os.listdir(logs))
            if runs:
                s = json.load(open(os.path.join(logs, runs[-1], "summary.json")))
                row.update({"latency_mean_ms": s["latency_ms"]["mean"], "latency_p50_ms": s["latency_ms"]["p50"],
                            "latency_p99_ms": s["latency_ms"]["p99"], "images_per_s": s["images_per_s"],
                            "kb_per_request": s["kb_per_request"], "cache_mb_max": s["cache_mb_max"]})
                row.update({f"metric.{k}": v for k, v in flatten(s.get("metrics")).items()})
                for k in ("top1", "top5"):
                    if k in s:
                        row[k] = s[k]
        except subprocess.TimeoutExpired:
            row["rc"] = "timeout"
        finally:
            srv.terminate()
            try:
                srv.wait(timeout=30)
            except subprocess.TimeoutExpired:
                srv.kill()
    return row


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description="appcorr_b200 local sweep")
    ap.add_argument("--config", required=True)
    ap.add_argument("--grid", action="append", default=[], metavar="KEY=V1,V2,...")
    ap.add_argument("--num-request", type=int, default=10)
    ap.add_argument("--num-warmup", type=int, default=1)
    ap.add_argument("--data", default=None)
    ap.add_argument("--server-args", default="")
    ap.add_argument("--timeout", type=float, default=3600.0)
    ap.add_argument("--out", default="sweep.csv")
    a = ap.parse_args(argv)
    rows = []
    for point in grid_points(a.grid):
        print(f"[sweep] {point}", flush=True)
        rows.append(run_point(a.config, point, a.num_request, a.num_warmup, a.data, a.server_args, a.timeout))
        print(f"[sweep]   -> {rows[-1]}", flush=True)
    cols = sorted({k for r in rows for k in r})
    with open(a.out, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=cols)
        w.writeheader()
        w.writerows(rows)
    print(f"[sweep] {len(rows)} point(s) -> {a.out}")
    return 0 if all(r.get("rc") == 0 for r in rows) else 1


if __name__ == "__main__":
    sys.exit(main())
