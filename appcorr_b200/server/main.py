"""Server entry point: `python -m appcorr_b200.server.main` (or `python -m offload.server.main`).

Starts four processes connected by queues (reference offload/server/main.py:13-119):
receiver -> scheduler -> worker -> sender, with a feedback queue from the worker's reaper to the
scheduler. `--device cuda:N` pins the worker to one GPU. `--tp N --dp M` serves with M
data-parallel replicas of N tensor-parallel ranks, one process per GPU (appcorr_b200/server/group.py):
requests are sharded over the replicas by request id; in a replica the leader rank decodes,
publishes each task through a shared-memory ring to its follower ranks and answers the client.
"""
from __future__ import annotations

import argparse
import multiprocessing
import time


def run_server(recv_port: int, send_port: int, reverse_connect: bool = False, mobile_ip: str = "127.0.0.1",
               listen_host: str = "0.0.0.0", device: str | None = None, stop_event=None, tp: int = 1, dp: int = 1,
               group_port: int = 29700, leave: dict | None = None) -> None:
    from .modules import ServerReceiver, ServerSender
    from .scheduler import SchedulerModule
    from .worker import WorkerModule

    ctx = multiprocessing.get_context("spawn")
    print("=== appcorr_b200 server ===", flush=True)
    sched_q, worker_q, result_q, control_q, feedback_q = (ctx.Queue() for _ in range(5))
    shutdown = ctx.Event()
    host = mobile_ip if reverse_connect else None
    if tp * dp > 1:
        from .group import launch_group

        router, workers = launch_group(tp, dp, worker_q, result_q, feedback_q, device, ctx, group_port, leave)
        print(f"[Main] {dp} replica(s) x {tp} tensor-parallel rank(s)", flush=True)
    else:
        router, workers = worker_q, [WorkerModule(worker_q, result_q, feedback_q, device=device)]
    procs = [ServerReceiver(recv_port, sched_q, control_q, shutdown, listen_host=listen_host, connect_host=host),
             SchedulerModule(sched_q, router, control_q, feedback_q),
             *workers,
             ServerSender(send_port, result_q, listen_host=listen_host, connect_host=host)]
    import signal

    def _term(signum, frame):  # SIGTERM: run the orderly shutdown below so no child is orphaned
        raise KeyboardInterrupt

    try:
        signal.signal(signal.SIGTERM, _term)
    except ValueError:  # not the main thread
        pass
    try:
        for p in procs:
            p.start()
        while not shutdown.is_set() and not (stop_event is not None and stop_event.is_set()):
            time.sleep(0.2)
    except KeyboardInterrupt:
        print("[Main] interrupted", flush=True)
    finally:
        for q, item in ((control_q, ("STOP", None)), (router, "STOP"), (result_q, "STOP")):
            try:
                q.put(item)
            except Exception:
                pass
        for p in procs:
            p.join(timeout=10)
        for p in procs:
            if p.is_alive():
                p.terminate()
                p.join()
        print("server stopped", flush=True)


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description="appcorr_b200 server")
    ap.add_argument("--recv-port", type=int, default=39990)
    ap.add_argument("--send-port", type=int, default=39991)
    ap.add_argument("--listen-host", type=str, default="0.0.0.0")
    ap.add_argument("-rc", "--reverse-connect", action="store_true")
    ap.add_argument("--mobile-ip", type=str, default="127.0.0.1")
    ap.add_argument("--device", type=str, default=None)
    ap.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks per replica (one GPU each)")
    ap.add_argument("--dp", type=int, default=1, help="data-parallel replicas (requests sharded by id)")
    ap.add_argument("--group-port", type=int, default=29700, help="first store port of the replica groups")
    ap.add_argument("--leave", type=str, default="",
                    help="testing: 'rank:n,...' makes follower `rank` leave its group after n requests")
    a = ap.parse_args(argv)
    leave = {int(k): int(v) for k, v in (x.split(":") for x in a.leave.split(",") if x)} if a.leave else None
    run_server(a.recv_port, a.send_port, reverse_connect=a.reverse_connect, mobile_ip=a.mobile_ip,
               listen_host=a.listen_host, device=a.device, tp=a.tp, dp=a.dp, group_port=a.group_port, leave=leave)


if __name__ == "__main__":
    main()
