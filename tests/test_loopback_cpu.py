"""End-to-end over loopback TCP on the CPU: server processes + mobile client, ViT-S classifier,
2-level progressive Laplacian, GroupTrigger, top-50% correction by residual energy."""
import json
import os
import socket
import subprocess
import sys
import time

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(300)
def test_loopback_classifier_cpu(tmp_path):
    from appcorr_b200.mobile.main import load_config, run_mobile

    rp, sp = _free_port(), _free_port()
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT, APPCORR_RESULT_TIMEOUT="240")
    srv = subprocess.Popen([sys.executable, "-m", "offload.server.main", "--recv-port", str(rp), "--send-port", str(sp),
                            "--listen-host", "127.0.0.1", "--device", "cpu"], cwd=ROOT, env=env,
                           stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    try:
        time.sleep(3)
        cfg = load_config(os.path.join(ROOT, "offload/config/cpu_vits16_loopback_keep05.json"),
                          ["dataset_kwargs.num_batches=3"])
        os.environ["APPCORR_RESULT_TIMEOUT"] = "240"
        rc = run_mobile("127.0.0.1", rp, sp, None, None, num_request=2, num_warmup=1, config=cfg,
                        log_root=str(tmp_path))
        assert rc == 0
        runs = os.listdir(tmp_path)
        assert len(runs) == 1
        summary = json.load(open(tmp_path / runs[0] / "summary.json"))
        assert summary["requests"] == 2 and summary["images"] == 8
        assert summary["latency_ms"]["p50"] > 0
        ev = summary["events"]
        for t in ("APPROX_FORWARD", "CORRECT_FORWARD", "HEAD_INFERENCE", "Decode", "MOBILE_ENCODE"):
            assert t in ev, (t, list(ev))
        lines = open(tmp_path / runs[0] / "events.jsonl").read().splitlines()
        assert len(lines) == 2
    finally:
        srv.terminate()
        try:
            out, _ = srv.communicate(timeout=20)
        except subprocess.TimeoutExpired:
            srv.kill()
            out, _ = srv.communicate()
        print(out[-3000:])
