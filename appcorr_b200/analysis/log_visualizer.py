"""Timeline report of a serving run: per-request event timelines (as SVG files, no plotting
library needed) and per-event-type statistics, from the mobile client's log directory.

Reference: analysis/log_tools/log_visualizer.py (per-request timeline of the logged events,
latest log directory by default). Input: `<log_dir>/events.jsonl` written by
appcorr_b200/mobile/source.py (one JSON record per request: latency_ms, bytes, events with type,
start, end / duration).

    python -m appcorr_b200.analysis.log_visualizer [--log-dir DIR] [--requests 0,1] [--out DIR]
"""
from __future__ import annotations

import argparse
import glob
import json
import os
from collections import defaultdict
from typing import Dict, List, Optional

DEFAULT_LOG_ROOT = os.path.join("logs", "offload")
_PALETTE = ["#4e79a7", "#f28e2b", "#e15759", "#76b7b2", "#59a14f", "#edc948", "#b07aa1", "#ff9da7", "#9c755f"]


def latest_log_dir(root: str = DEFAULT_LOG_ROOT) -> Optional[str]:
    dirs = [d for d in glob.glob(os.path.join(root, "*")) if os.path.isfile(os.path.join(d, "events.jsonl"))]
    return max(dirs, key=os.path.getmtime) if dirs else None


def read_requests(log_dir: str) -> List[Dict]:
    out = []
    with open(os.path.join(log_dir, "events.jsonl")) as f:
        for line in f:
            line = line.strip()
            if line:
                out.append(json.loads(line))
    return out


def normalize(record: Dict) -> List[Dict]:
    """Events with start / end in ms relative to the request's first event, sorted by start."""
    evs = []
    for e in record.get("events", []):
        s = e.get("start", e.get("timestamp"))
        if s is None:
            continue
        t = e.get("end")
        if t is None:
            t = s + float(e.get("duration", 0.0))
        evs.append({"type": str(e.get("type", "?")), "start": float(s), "end": float(t)})
    if not evs:
        return []
    t0 = min(e["start"] for e in evs)
    for e in evs:
        e["start_ms"], e["end_ms"] = (e["start"] - t0) * 1e3, (e["end"] - t0) * 1e3
    return sorted(evs, key=lambda e: e["start_ms"])


def type_stats(records: List[Dict]) -> Dict[str, Dict[str, float]]:
    acc: Dict[str, List[float]] = defaultdict(list)
    for r in records:
        for e in normalize(r):
            acc[e["type"]].append(e["end_ms"] - e["start_ms"])
    return {t: {"count": len(v), "mean_ms": sum(v) / len(v), "min_ms": min(v), "max_ms": max(v)}
            for t, v in sorted(acc.items())}


def timeline_svg(events: List[Dict], title: str = "", width: int = 1000, row_h: int = 18) -> str:
    """One row per event type, one bar per event, time axis in ms."""
    if not events:
        return "<svg xmlns='http://www.w3.org/2000/svg' width='200' height='40'><text x='5' y='20'>no events</text></svg>"
    types = list(dict.fromkeys(e["type"] for e in events))
    span = max(e["end_ms"] for e in events) or 1.0
    left = 180
    scale = (width - left - 20) / span
    h = 40 + row_h * len(types)
    parts = [f"<svg xmlns='http://www.w3.org/2000/svg' width='{width}' height='{h}' font-family='monospace' font-size='11'>",
             f"<text x='5' y='14'>{title} ({span:.2f} ms)</text>"]
    for i, t in enumerate(types):
        y = 24 + i * row_h
        parts.append(f"<text x='5' y='{y + 12}'>{t[:24]}</text>")
        for e in events:
            if e["type"] != t:
                continue
            x = left + e["start_ms"] * scale
            w = max((e["end_ms"] - e["start_ms"]) * scale, 1.0)
            parts.append(f"<rect x='{x:.1f}' y='{y}' width='{w:.1f}' height='{row_h - 4}' "
                         f"fill='{_PALETTE[i % len(_PALETTE)]}'><title>{t}: {e['end_ms'] - e['start_ms']:.3f} ms"
                         f"</title></rect>")
    parts.append("</svg>")
    return "\n".join(parts)


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--log-dir", default=None, help="log directory (default: latest under logs/offload)")
    ap.add_argument("--requests", default="0", help="comma-separated request indices to draw, or 'all'")
    ap.add_argument("--out", default=None, help="output directory for the SVG files (default: the log dir)")
    a = ap.parse_args(argv)
    log_dir = a.log_dir or latest_log_dir()
    if log_dir is None:
        print("no log directory found")
        return 1
    recs = read_requests(log_dir)
    out = a.out or log_dir
    os.makedirs(out, exist_ok=True)
    idx = range(len(recs)) if a.requests == "all" else [int(i) for i in a.requests.split(",") if i != ""]
    for i in idx:
        if i < len(recs):
            with open(os.path.join(out, f"timeline_{i}.svg"), "w") as f:
                f.write(timeline_svg(normalize(recs[i]), f"request {i}"))
    stats = type_stats(recs)
    print(f"{'event':28s} {'count':>6s} {'mean ms':>10s} {'min':>10s} {'max':>10s}")
    for t, s in stats.items():
        print(f"{t:28s} {s['count']:6d} {s['mean_ms']:10.3f} {s['min_ms']:10.3f} {s['max_ms']:10.3f}")
    lat = sorted(r.get("latency_ms", 0.0) for r in recs)
    if lat:
        print(f"latency ms: p50 {lat[len(lat) // 2]:.3f}  p99 {lat[min(len(lat) - 1, int(0.99 * len(lat)))]:.3f}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
