"""Offline analysis tools: timeline report, early-exit simulation, nsys SQLite re-timing."""
import json
import sqlite3

from appcorr_b200.analysis import log_visualizer as lv
from appcorr_b200.analysis import nsys_events as ne
from appcorr_b200.analysis import simulate_exit as se


def test_log_visualizer_report_and_svg(tmp_path, capsys):
    recs = [{"request": i, "latency_ms": 10.0 + i, "bytes": 100,
             "events": [{"type": "APPROX_FORWARD", "start": 1.0, "end": 1.004},
                        {"type": "CORRECT_FORWARD", "start": 1.004, "end": 1.010},
                        {"type": "MOBILE_SEND", "timestamp": 0.999, "duration": 0.0005}]} for i in range(3)]
    (tmp_path / "events.jsonl").write_text("\n".join(json.dumps(r) for r in recs))
    assert lv.main(["--log-dir", str(tmp_path), "--requests", "all"]) == 0
    svg = (tmp_path / "timeline_1.svg").read_text()
    assert svg.startswith("<svg") and "CORRECT_FORWARD" in svg
    st = lv.type_stats(recs)
    assert st["APPROX_FORWARD"]["count"] == 3 and abs(st["CORRECT_FORWARD"]["mean_ms"] - 6.0) < 1e-6
    assert "p50" in capsys.readouterr().out


def test_simulate_exit_metrics():
    recs = [{"labels": [0, 1], "stages": [
        {"t_ms": 10.0, "probs": [[0.9, 0.1], [0.6, 0.4]]},
        {"t_ms": 20.0, "probs": [[0.8, 0.2], [0.05, 0.95]]}]}]
    r = se.simulate(recs, "max_prob", 0.85)
    assert r["exit_hist"] == {0: 1, 1: 1} and r["accuracy"] == 1.0 and r["mean_latency_ms"] == 15.0
    r = se.simulate(recs, "max_prob", 0.5)   # both exit at stage 0; image 1 is then wrong
    assert r["exit_hist"] == {0: 2} and r["accuracy"] == 0.5
    r = se.simulate(recs, "top2_margin", 0.7)
    assert r["exit_hist"] == {0: 1, 1: 1}
    r = se.simulate(recs, "entropy", 0.4)    # entropy of [.9,.1] = 0.325 <= 0.4 exits at 0
    assert r["exit_hist"][0] == 1


def test_nsys_events_from_sqlite(tmp_path):
    db = tmp_path / "p.sqlite"
    con = sqlite3.connect(db)
    con.execute("CREATE TABLE StringIds (id INTEGER, value TEXT)")
    con.execute("CREATE TABLE NVTX_EVENTS (start INTEGER, end INTEGER, text TEXT, textId INTEGER)")
    con.execute("INSERT INTO StringIds VALUES (7, 'APPCORR_INSTR|req=3|task=1|seq=1|op=CORRECT_FORWARD')")
    con.executemany("INSERT INTO NVTX_EVENTS VALUES (?, ?, ?, ?)", [
        (1_000_000, 3_000_000, "APPCORR_INSTR|req=3|task=0|seq=0|op=APPROX_FORWARD", None),
        (3_500_000, 9_000_000, None, 7),
        (0, 100, "unrelated", None)])
    con.commit()
    con.close()
    recs = ne.to_requests(ne.read_ranges(str(db)))
    assert len(recs) == 1 and [e["type"] for e in recs[0]["events"]] == ["APPROX_FORWARD", "CORRECT_FORWARD"]
    assert abs(recs[0]["latency_ms"] - 8.0) < 1e-9
