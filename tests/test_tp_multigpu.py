"""Tensor-parallel engine on 2 GPUs (one process per GPU, peer-memory collectives) against the
single-GPU engine with the same weights."""
import os
import socket

import pytest
import torch

pytestmark = [pytest.mark.gpu, pytest.mark.multigpu]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    import torch.distributed as dist

    from appcorr_b200.models.dinov3.vit import ViTConfig
    from appcorr_b200.models.engine import ViTEngine, random_weights
    from appcorr_b200.parallel.comm import TPComm
    from appcorr_b200.parallel.tp import ViTEngineTP

    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    dev = torch.device("cuda", rank)
    cfg = ViTConfig(embed_dim=512, depth=3, num_heads=4, ffn_ratio=3, qkv_bias=False, ffn_layer="swiglu64",
                    layerscale_init=0.3)
    full = random_weights(cfg, dev, seed=3, std=0.05)
    comm = TPComm(device=dev)
    tp = ViTEngineTP.from_full(full, comm)
    ref = ViTEngine(full, dev)
    B, H, W = 2, 64, 96
    g = torch.Generator(device=dev).manual_seed(0)
    img0 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=dev, generator=g)
    img1 = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=dev, generator=g)
    outs = []
    for eng in (ref, tp):
        s = eng.new_session(B, H, W)
        eng.prepare_tokens(s, img0)
        eng.approx(s, 0, cfg.depth)
        xa = s.x.clone()
        eng.prepare_tokens(s, img1)
        pre = torch.arange(cfg.n_prefix, dtype=torch.int32, device=dev).repeat(B, 1).contiguous()
        cand = torch.arange(cfg.n_prefix, s.N, dtype=torch.int32, device=dev).repeat(B, 1).contiguous()
        xc = eng.correct(s, 0, cfg.depth, pre, cand, {"token_keep_ratio": 0.5, "server_pscore": "cls_attn_prob_layermean"})
        torch.cuda.synchronize()
        outs.append((xa, xc.clone(), s.pscore.clone()))
    comm.check()
    (ra, rc, rp), (ta, tc, tpp) = outs
    rel = lambda a, b: ((a.float() - b.float()).norm() / b.float().norm()).item()  # noqa: E731
    q.put((rank, rel(ta, ra), rel(tc, rc), rel(tpp, rp)))
    dist.barrier()
    comm.close()
    dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_single_gpu():
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, a, c, ps in res:
        assert a < 2e-2 and c < 3e-2 and ps < 1e-2, (rank, a, c, ps)
