"""Offline early-exit simulation: given, per request, the class probabilities produced after each
stage (correction group) and the time each stage finished, pick for every image the first stage
whose confidence passes a threshold and report accuracy, mean exit stage and mean latency.

Reference: analysis/log_tools/simulate_exit.py (metrics max_prob, entropy, top2_margin over logged
per-stage outputs). Input: JSONL records {"labels": [...], "stages": [{"t_ms": float,
"probs": [[p_0 .. p_C-1] per image]}, ...]} (or "topk": [[[cls, p], ...] per image] instead of
full "probs").

    python -m appcorr_b200.analysis.simulate_exit stages.jsonl --metric max_prob --thresholds 0.5,0.7,0.9
"""
from __future__ import annotations

import argparse
import json
import math
from typing import Dict, List, Sequence


def _conf(probs: Sequence[float], metric: str) -> float:
    p = sorted(probs, reverse=True)
    if metric == "max_prob":
        return p[0]
    if metric == "top2_margin":
        return p[0] - (p[1] if len(p) > 1 else 0.0)
    if metric == "entropy":  # lower is more confident: negate so that ">= threshold" means exit
        return sum(q * math.log(q) for q in p if q > 0)
    raise ValueError(f"unknown metric {metric!r}")


def _image_view(stage: Dict, j: int):
    """(pred, probs) of image j in one stage record."""
    if "probs" in stage:
        pr = stage["probs"][j]
        return max(range(len(pr)), key=pr.__getitem__), pr
    tk = stage["topk"][j]
    return int(tk[0][0]), [float(p) for _, p in tk]


def simulate(records: List[Dict], metric: str, threshold: float) -> Dict[str, float]:
    """Exit at the first stage with confidence >= threshold (entropy: <= threshold)."""
    thr = -threshold if metric == "entropy" else threshold
    n = correct = 0
    stage_sum = lat_sum = 0.0
    hist: Dict[int, int] = {}
    for r in records:
        stages = r["stages"]
        for j, label in enumerate(r["labels"]):
            exit_at = len(stages) - 1
            for s, st in enumerate(stages):
                _, pr = _image_view(st, j)
                if _conf(pr, metric) >= thr:
                    exit_at = s
                    break
            pred, _ = _image_view(stages[exit_at], j)
            n += 1
            correct += int(pred == int(label))
            stage_sum += exit_at
            lat_sum += float(stages[exit_at].get("t_ms", 0.0))
            hist[exit_at] = hist.get(exit_at, 0) + 1
    return {"accuracy": correct / max(n, 1), "mean_exit_stage": stage_sum / max(n, 1),
            "mean_latency_ms": lat_sum / max(n, 1), "images": n, "exit_hist": hist}


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("path")
    ap.add_argument("--metric", default="max_prob", choices=["max_prob", "top2_margin", "entropy"])
    ap.add_argument("--thresholds", default="0.5,0.7,0.9")
    a = ap.parse_args(argv)
    with open(a.path) as f:
        recs = [json.loads(line) for line in f if line.strip()]
    for t in [float(x) for x in a.thresholds.split(",")]:
        r = simulate(recs, a.metric, t)
        print(f"{a.metric} >= {t}: acc {r['accuracy']:.4f}  exit stage {r['mean_exit_stage']:.2f}  "
              f"latency {r['mean_latency_ms']:.2f} ms  hist {r['exit_hist']}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
