"""End-to-end over loopback TCP with the worker on the GPU: the server's decoder / launcher /
reaper threads serve enough requests that every approximate and correction pass runs eagerly,
is captured as a CUDA graph by the launcher thread while the other threads keep working, and is
then replayed; every request still returns its results."""
import json
import os
import socket
import subprocess
import sys
import time

import pytest

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.timeout(400)
def test_loopback_classifier_gpu_graph_replay(tmp_path):
    from appcorr_b200.mobile.main import load_config, run_mobile

    rp, sp = _free_port(), _free_port()
    env = dict(os.environ, PYTHONPATH=ROOT, APPCORR_RESULT_TIMEOUT="240")
    srv = subprocess.Popen([sys.executable, "-m", "offload.server.main", "--recv-port", str(rp), "--send-port", str(sp),
                            "--listen-host", "127.0.0.1", "--device", "cuda:0"], cwd=ROOT, env=env,
                           stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    try:
        time.sleep(5)
        cfg = load_config(os.path.join(ROOT, "offload/config/cpu_vits16_loopback_keep05.json"),
                          # server-side scores only, so the correction passes have static inputs
                          ["dataset_kwargs.num_batches=6", "appcorr_kwargs.mobile_pscore_weight=0.0",
                           "appcorr_kwargs.server_pscore_weight=1.0"])
        os.environ["APPCORR_RESULT_TIMEOUT"] = "240"
        rc = run_mobile("127.0.0.1", rp, sp, None, None, num_request=5, num_warmup=1, config=cfg,
                        log_root=str(tmp_path))
        assert rc == 0
        runs = os.listdir(tmp_path)
        summary = json.load(open(tmp_path / runs[0] / "summary.json"))
        assert summary["requests"] == 5 and summary["images"] == 20
        for t in ("APPROX_FORWARD", "CORRECT_FORWARD", "HEAD_INFERENCE"):
            assert t in summary["events"], (t, list(summary["events"]))
    finally:
        srv.terminate()
        try:
            out, _ = srv.communicate(timeout=20)
        except subprocess.TimeoutExpired:
            srv.kill()
            out, _ = srv.communicate()
        print(out[-3000:])
    assert "Traceback" not in out, out[-3000:]
