"""Multi-rank serving over loopback TCP on the CPU (gloo): `offload.server.main --tp 3` with the
leader publishing tasks to two followers through the shared-memory ring; one follower leaves the
group between requests and the survivors re-form and keep serving. Also `--dp 2`: requests are
sharded over two replicas."""
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


def _serve(tmp_path, extra, num_request):
    from appcorr_b200.mobile.main import load_config, run_mobile

    rp, sp, gp = _free_port(), _free_port(), _free_port()
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="", PYTHONPATH=ROOT, APPCORR_RESULT_TIMEOUT="240")
    srv = subprocess.Popen([sys.executable, "-m", "offload.server.main", "--recv-port", str(rp), "--send-port", str(sp),
                            "--listen-host", "127.0.0.1", "--device", "cpu", "--group-port", str(gp), *extra],
                           cwd=ROOT, env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    try:
        time.sleep(4)
        cfg = load_config(os.path.join(ROOT, "offload/config/cpu_vits16_loopback_keep05.json"),
                          [f"dataset_kwargs.num_batches={num_request + 1}"])
        os.environ["APPCORR_RESULT_TIMEOUT"] = "240"
        rc = run_mobile("127.0.0.1", rp, sp, None, None, num_request=num_request, num_warmup=1, config=cfg,
                        log_root=str(tmp_path))
        runs = os.listdir(tmp_path)
        summary = json.load(open(tmp_path / runs[0] / "summary.json")) if runs else {}
    finally:
        srv.terminate()
        try:
            out, _ = srv.communicate(timeout=30)
        except subprocess.TimeoutExpired:
            srv.kill()
            out, _ = srv.communicate()
    return rc, summary, out


@pytest.mark.timeout(600)
def test_tp_group_keeps_serving_after_a_rank_leaves(tmp_path):
    # follower rank 2 leaves after its 2nd answered request (the warm-up request is the 1st)
    rc, summary, out = _serve(tmp_path, ["--tp", "3", "--leave", "2:2"], num_request=3)
    print(out[-4000:])
    assert rc == 0, out[-3000:]
    assert summary["requests"] == 3 and summary["images"] == 12
    assert "leaving after 2 requests" in out
    assert "re-forming over [0, 1]" in out
    assert "disagree" not in out


@pytest.mark.timeout(600)
def test_dp_replicas_share_the_requests(tmp_path):
    rc, summary, out = _serve(tmp_path, ["--dp", "2"], num_request=3)
    print(out[-4000:])
    assert rc == 0, out[-3000:]
    assert summary["requests"] == 3
    assert out.count("[Group 0] configured") >= 1 and out.count("[Group 1] configured") >= 1
