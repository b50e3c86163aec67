"""Re-time serving events from an Nsight Systems export: the worker wraps every instruction in an
NVTX range `APPCORR_INSTR|req=<r>|task=<t>|seq=<s>|op=<OP>` (appcorr_b200/server/worker.py); this
tool reads those ranges from the exported SQLite database (`nsys export --type sqlite`) and
writes one JSONL record per request with the ranges as events (start / end in seconds).

Reference: analysis/log_tools/nsys_events.py (rebuilds events.jsonl from an nsys sqlite by
matching APPCORR_INSTR ranges). Schema used: NVTX_EVENTS(start, end, text, textId) with
StringIds(id, value) for registered strings.

    python -m appcorr_b200.analysis.nsys_events profile.sqlite -o events_nsys.jsonl
"""
from __future__ import annotations

import argparse
import json
import re
import sqlite3
from collections import defaultdict
from typing import Dict, List

_INSTR = re.compile(r"APPCORR_INSTR\|req=(\d+)\|task=(\d+)\|seq=(\d+)\|op=(\w+)")


def read_ranges(db_path: str) -> List[Dict]:
    con = sqlite3.connect(db_path)
    try:
        tables = {r[0] for r in con.execute("SELECT name FROM sqlite_master WHERE type='table'")}
        if "NVTX_EVENTS" not in tables:
            return []
        strings = {}
        if "StringIds" in tables:
            strings = dict(con.execute("SELECT id, value FROM StringIds"))
        cols = {r[1] for r in con.execute("PRAGMA table_info(NVTX_EVENTS)")}
        sel = "SELECT start, end, " + ("text" if "text" in cols else "NULL") + ", " + \
              ("textId" if "textId" in cols else "NULL") + " FROM NVTX_EVENTS WHERE end IS NOT NULL"
        out = []
        for start, end, text, tid in con.execute(sel):
            name = text if text is not None else strings.get(tid)
            m = _INSTR.match(name or "")
            if m:
                out.append({"request": int(m[1]), "task": int(m[2]), "seq": int(m[3]), "type": m[4],
                            "start": start * 1e-9, "end": end * 1e-9})
        return out
    finally:
        con.close()


def to_requests(ranges: List[Dict]) -> List[Dict]:
    by_req: Dict[int, List[Dict]] = defaultdict(list)
    for r in ranges:
        by_req[r["request"]].append(r)
    recs = []
    for req in sorted(by_req):
        evs = sorted(by_req[req], key=lambda e: (e["start"], e["seq"]))
        recs.append({"request": req, "latency_ms": (evs[-1]["end"] - evs[0]["start"]) * 1e3,
                     "events": [{"type": e["type"], "start": e["start"], "end": e["end"], "task": e["task"],
                                 "seq": e["seq"]} for e in evs]})
    return recs


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("sqlite")
    ap.add_argument("-o", "--out", default="events_nsys.jsonl")
    a = ap.parse_args(argv)
    recs = to_requests(read_ranges(a.sqlite))
    with open(a.out, "w") as f:
        for r in recs:
            f.write(json.dumps(r) + "\n")
    print(f"{len(recs)} requests -> {a.out}")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
