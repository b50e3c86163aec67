"""Mobile client entry point: `python -m appcorr_b200.mobile.main` (or `python -m offload.mobile.main`).
Flags as the reference (offload/mobile/main.py:108-155)."""
from __future__ import annotations

import argparse
import json
import multiprocessing

from ..common.config_overrides import apply_config_overrides
from ..common.protocol import ExperimentConfig


def load_config(path: str, overrides=None) -> ExperimentConfig:
    with open(path) as f:
        data = json.load(f)
    apply_config_overrides(data, overrides)
    for key in ("image_shape", "patch_size"):
        if key in data:
            data[key] = tuple(data[key])
    return ExperimentConfig(**data)


def run_mobile(server_ip, recv_port, send_port, data_root, config_path, num_request=None, num_warmup=1,
               reverse_connect=False, listen_host="0.0.0.0", config_overrides=None, config=None, log_root=None):
    from .modules import MobileReceiver, MobileSender
    from .source import SourceModule

    ctx = multiprocessing.get_context("spawn")
    cfg = config if config is not None else load_config(config_path, config_overrides)
    send_q, fb_q = ctx.Queue(), ctx.Queue()
    procs = [MobileSender(server_ip, recv_port, send_q, listen=reverse_connect, listen_host=listen_host),
             MobileReceiver(server_ip, send_port, fb_q, listen=reverse_connect, listen_host=listen_host)]
    kw = {"log_root": log_root} if log_root else {}
    source = SourceModule(send_q, fb_q, cfg, data_root, cfg.batch_size, num_request, num_warmup, **kw)
    try:
        for p in procs:
            p.start()
        source.start()
        source.join()
        procs[0].join(timeout=5)
    finally:
        for p in procs + [source]:
            if p.is_alive():
                p.terminate()
                p.join()
    return source.exitcode


def main(argv=None):
    ap = argparse.ArgumentParser(description="appcorr_b200 mobile client")
    ap.add_argument("--ip", type=str, default="127.0.0.1")
    ap.add_argument("--recv-port", type=int, default=39990)
    ap.add_argument("--send-port", type=int, default=39991)
    ap.add_argument("--listen-host", type=str, default="0.0.0.0")
    ap.add_argument("-rc", "--reverse-connect", action="store_true")
    ap.add_argument("--data", type=str, default=None)
    ap.add_argument("--config", type=str, required=True)
    ap.add_argument("-nr", "--num-request", type=int, default=None)
    ap.add_argument("-nw", "--num-warmup", type=int, default=1)
    ap.add_argument("--set", dest="config_overrides", action="append", default=[], metavar="KEY=VALUE")
    ap.add_argument("--log-root", type=str, default=None, help="directory for summary.json / events.jsonl runs")
    a = ap.parse_args(argv)
    if a.num_request is not None and a.num_request <= 0:
        ap.error("--num-request must be a positive integer")
    if a.num_warmup < 0:
        ap.error("--num-warmup must be zero or a positive integer")
    data = a.data
    if data is None:
        with open(a.config) as f:
            raw = json.load(f)
        apply_config_overrides(raw, a.config_overrides)
        data = raw.get("dataset_kwargs", {}).get("data_root")
    rc = run_mobile(a.ip, a.recv_port, a.send_port, data, a.config, a.num_request, a.num_warmup,
                    reverse_connect=a.reverse_connect, listen_host=a.listen_host, config_overrides=a.config_overrides,
                    log_root=a.log_root)
    raise SystemExit(rc or 0)


if __name__ == "__main__":
    main()
