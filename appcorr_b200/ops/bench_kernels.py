"""Kernel micro-benchmarks (CUDA-event timing after warm-up) and single-launch drivers for ncu.

    python -m appcorr_b200.ops.bench_kernels gemm --M 8232 --N 12288 --K 4096 [--bn 256] [--epi bf16]
    python -m appcorr_b200.ops.bench_kernels attention --B 8 --H 32 --Dh 128 --Tq 1029 --Tk 1029
    python -m appcorr_b200.ops.bench_kernels layernorm --M 8232 --D 4096
    python -m appcorr_b200.ops.bench_kernels sp_row --M 8232 --D 4096 --world 2   (tensor-parallel
        owner row kernel, every "peer" emulated by a local buffer on this GPU)
    ... --once    launch the kernel exactly once (for `ncu -k ... -c 1`)

Prints one JSON line: time per launch (ms), achieved TFLOP/s or GB/s, and the library
reference (cuBLAS / cuDNN through PyTorch) for the same shape when --ref is given.
"""
from __future__ import annotations

import argparse
import json

import torch

from . import kernels as K


def _time(fn, iters: int, warmup: int = 3) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("op", choices=["gemm", "attention", "layernorm", "sp_row", "msda"])
    ap.add_argument("--world", type=int, default=2)
    ap.add_argument("--M", type=int, default=8232)
    ap.add_argument("--N", type=int, default=12288)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--D", type=int, default=4096)
    ap.add_argument("--bn", type=int, default=None)
    ap.add_argument("--epi", default="bf16", choices=["bf16", "f32", "gelu"])
    ap.add_argument("--fp8", action="store_true", help="e4m3 operands (kind::f8f6f4); --ref times torch._scaled_mm")
    ap.add_argument("--fp4", action="store_true",
                    help="NVFP4 operands (kind::mxf4nvf4 block16); --ref times torch._scaled_mm on the same bytes")
    ap.add_argument("--B", type=int, default=8)
    ap.add_argument("--H", type=int, default=32)
    ap.add_argument("--Dh", type=int, default=128)
    ap.add_argument("--Tq", type=int, default=1029)
    ap.add_argument("--Tk", type=int, default=1029)
    ap.add_argument("--impl", default="tcgen05")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--once", action="store_true")
    ap.add_argument("--ref", action="store_true")
    ap.add_argument("--prof", action="store_true",
                    help="gemm: one extra launch with the kernel's wait-cycle counters on; prints each wait "
                         "as a share of the MMA warp's loop time")
    a = ap.parse_args(argv)
    torch.manual_seed(0)
    dev = "cuda"
    res = {"op": a.op}
    if a.op == "gemm":
        x = torch.randn(a.M, a.K, device=dev).to(torch.bfloat16)
        w = (torch.randn(a.N, a.K, device=dev) * a.K ** -0.5).to(torch.bfloat16)
        epi = {"bf16": K.EPI_BF16, "f32": K.EPI_F32, "gelu": K.EPI_GELU}[a.epi]
        out = torch.empty(a.M, a.N, device=dev, dtype=torch.float32 if a.epi == "f32" else torch.bfloat16)
        flops = 2.0 * a.M * a.N * a.K
        if a.fp4:
            x4 = torch.empty(a.M, a.K // 2, device=dev, dtype=torch.uint8)
            xsf = torch.zeros(K.nvfp4_sf_bytes(a.M, a.K), device=dev, dtype=torch.uint8)
            xs = torch.empty(a.M, device=dev)
            K.quant_rows_nvfp4(x, x4, xsf, xs)
            w4, (ws, wsf) = K.quantize_weight_nvfp4(w)
            fn = lambda: K.gemm(x4, w4, out, epi=epi, bn=a.bn, a_scale=(xs, xsf), b_scale=(ws, wsf))  # noqa: E731
            ref = None
            if a.ref:
                fa, fb = x4.view(torch.float4_e2m1fn_x2), w4.view(torch.float4_e2m1fn_x2)
                sa, sb = xsf.view(torch.float8_e4m3fn), wsf.view(torch.float8_e4m3fn)
                ref = lambda: torch._scaled_mm(fa, fb.T, sa, sb, out_dtype=torch.bfloat16)  # noqa: E731
        elif a.fp8:
            x8 = torch.empty(a.M, a.K, device=dev, dtype=torch.float8_e4m3fn)
            sx = torch.empty(a.M, device=dev)
            K.quant_rows_e4m3(x, x8, sx)
            w8, sw = K.quantize_weight_e4m3(w)
            fn = lambda: K.gemm(x8, w8, out, epi=epi, bn=a.bn, a_scale=sx, b_scale=sw)  # noqa: E731
            one = torch.ones((), device=dev)
            ref = (lambda: torch._scaled_mm(x8, w8.T, one, one, out_dtype=torch.bfloat16)) if a.ref else None  # noqa: E731
        else:
            fn = lambda: K.gemm(x, w, out, epi=epi, bn=a.bn)  # noqa: E731
            ref = (lambda: torch.matmul(x, w.T)) if a.ref else None  # noqa: E731
        res.update(M=a.M, N=a.N, K=a.K, bn=a.bn, fp8=a.fp8, fp4=a.fp4)
    elif a.op == "attention":
        q = torch.randn(a.B * a.Tq, a.H * a.Dh, device=dev).to(torch.bfloat16)
        k = torch.randn(a.B * a.Tk, a.H * a.Dh, device=dev).to(torch.bfloat16)
        v = torch.randn(a.B * a.Tk, a.H * a.Dh, device=dev).to(torch.bfloat16)
        o = torch.empty_like(q)
        fn = lambda: K.attention(q, k, v, o, B=a.B, Tq=a.Tq, Tk=a.Tk, H=a.H, Dh=a.Dh, impl=a.impl)  # noqa: E731
        flops = 4.0 * a.B * a.H * a.Tq * a.Tk * a.Dh
        if a.ref:
            qq = q.view(a.B, a.Tq, a.H, a.Dh).transpose(1, 2)
            kk = k.view(a.B, a.Tk, a.H, a.Dh).transpose(1, 2)
            vv = v.view(a.B, a.Tk, a.H, a.Dh).transpose(1, 2)
            ref = lambda: torch.nn.functional.scaled_dot_product_attention(qq, kk, vv)  # noqa: E731
        else:
            ref = None
        res.update(B=a.B, H=a.H, Dh=a.Dh, Tq=a.Tq, Tk=a.Tk, impl=a.impl)
    elif a.op == "msda":  # Mask2Former pixel decoder shape: 3 levels of a 64x64 grid, 8 heads x 32, 4 points
        N, M, Dh, L, P = a.B, 8, 32, 3, 4
        shapes = [(64, 64), (32, 32), (16, 16)]
        S = sum(h * w for h, w in shapes)
        value = torch.randn(N, S, M, Dh, device=dev).to(torch.bfloat16)
        refp = torch.rand(N, S, L, 2, device=dev)
        offs = torch.randn(N * S, M * L * P * 3, device=dev).to(torch.bfloat16)
        out = torch.empty(N, S, M * Dh, device=dev, dtype=torch.bfloat16)
        sh = [v for hw in shapes for v in hw]
        fn = lambda: K.msda(value, refp, offs, offs[:, M * L * P * 2:], out, sh, M, L, P)  # noqa: E731
        flops = 0.0
        # bytes: the value rows each sample touches (4 corners x Dh bf16, mostly L2 hits) are not
        # counted; count the per-query inputs and outputs (offsets, logits, reference, output)
        res.update(N=N, S=S, bytes=N * S * (M * L * P * 3 * 2 + L * 2 * 4 + M * Dh * 2) + value.numel() * 2)
        ref = None
    elif a.op == "sp_row":
        from .native import lib

        W, M, D = a.world, a.M, a.D
        R = (M + W - 1) // W
        parts = [torch.randn(M, D, device=dev).to(torch.bfloat16) for _ in range(W)]
        x = torch.randn(M, D, device=dev).to(torch.bfloat16)
        aux = torch.zeros(M, D, device=dev, dtype=torch.bfloat16)
        vec = torch.ones(D, device=dev, dtype=torch.bfloat16)
        ag = [torch.empty(M, D, device=dev, dtype=torch.float8_e4m3fn) for _ in range(W)]
        ags = [torch.empty(M, device=dev) for _ in range(W)]
        fn = lambda: lib().sp_row(M, None, R, 0, W, D, [p.data_ptr() for p in parts], [0] * W, vec, vec, x, True,  # noqa: E731
                                  None, x, True, aux, K.AUX_ADD, None, None, vec, vec, 1e-6, False, 1,
                                  [t.data_ptr() for t in ag], D, [t.data_ptr() for t in ags])
        flops = 0.0
        rows = R
        res.update(M=M, D=D, world=W, rows=rows,
                   bytes=rows * D * (2 * W + 2 + 4 + 2) + rows * D * W)  # partials, resid, aux rw, out, e4m3 gather
        ref = None
    else:
        x = torch.randn(a.M, a.D, device=dev).to(torch.bfloat16)
        wt = torch.ones(a.D, device=dev, dtype=torch.bfloat16)
        bt = torch.zeros(a.D, device=dev, dtype=torch.bfloat16)
        flops = 0.0
        if a.fp4:  # NVFP4 output: packed rows + blocked block scales + row scales
            out = torch.empty(a.M, a.D // 2, device=dev, dtype=torch.uint8)
            sf = torch.zeros(K.nvfp4_sf_bytes(a.M, a.D), device=dev, dtype=torch.uint8)
            sc = torch.empty(a.M, device=dev)
            fn = lambda: K.layernorm(x, wt, bt, 1e-5, out, scale8=sc, sf=sf)  # noqa: E731
            res.update(M=a.M, D=a.D, fp4=True, bytes=x.numel() * 2 + out.numel() + sf.numel() + sc.numel() * 4)
        else:
            out = torch.empty_like(x)
            fn = lambda: K.layernorm(x, wt, bt, 1e-5, out)  # noqa: E731
            res.update(M=a.M, D=a.D, bytes=2 * x.numel() * 2)
        ref = (lambda: torch.nn.functional.layer_norm(x, (a.D,), wt, bt, 1e-5)) if a.ref else None  # noqa: E731
    if a.once:
        fn()
        torch.cuda.synchronize()
        from .native import check_errors

        check_errors(torch.device(dev))
        print(json.dumps({**res, "launched": 1}))
        return
    if a.prof and a.op == "gemm":
        from .native import lib

        fn()
        cnt = torch.zeros(16, dtype=torch.int64, device=dev)
        lib().gemm_set_profile(cnt)
        fn()
        torch.cuda.synchronize()
        lib().gemm_set_profile(None)
        c = cnt.tolist()
        loop = max(c[4], 1)
        res["prof"] = {"ctas": c[7], "mma_loop_cycles_per_cta": c[4] // max(c[7], 1),
                       "share_of_mma_loop": {"mma_wait_acc_free": round(c[1] / loop, 3),
                                             "mma_wait_stage_full": round(c[2] / loop, 3),
                                             "mma_wait_scales": round(c[3] / loop, 3),
                                             "producer_wait_stage_free": round(c[0] / loop, 3),
                                             "epilogue_wait_acc_full": round(c[5] / loop, 3),
                                             "epilogue_body": round(c[6] / loop, 3),
                                             "epilogue_release": round(c[10] / loop, 3),
                                             "scale_warp_wait_bytes": round(c[8] / loop, 3),
                                             "scale_warp_store": round(c[9] / loop, 3)}}
    ms = _time(fn, a.iters)
    res["ms"] = round(ms, 4)
    if flops:
        res["tflops"] = round(flops / ms / 1e9, 1)
    else:
        res["gbps"] = round(res["bytes"] / ms / 1e6, 1)
    if ref is not None:
        rms = _time(ref, a.iters)
        res["ref_ms"] = round(rms, 4)
        if flops:
            res["ref_tflops"] = round(flops / rms / 1e9, 1)
    print(json.dumps(res))


if __name__ == "__main__":
    main()
