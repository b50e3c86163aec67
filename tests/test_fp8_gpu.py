"""e4m3 path: LayerNorm / row quantisers and the kind::f8f6f4 tcgen05 GEMM with scale-folding
epilogues, each against a plain PyTorch fp32 computation on the dequantised operands."""
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _k():
    from appcorr_b200.ops import kernels as K

    return K


def _rand(*shape, scale=1.0):
    return (torch.randn(*shape, device=DEV) * scale).to(torch.bfloat16)


def _close(a, b, rtol=2e-2, atol=2e-2):
    a, b = a.float(), b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= atol + rtol * ref, f"max err {err} (ref max {ref})"


def _deq(q8, s):
    return q8.float() * s.float()[:, None]


def _quant(x):
    K = _k()
    q = torch.empty(x.shape, device=DEV, dtype=torch.float8_e4m3fn)
    s = torch.empty(x.shape[0], device=DEV, dtype=torch.float32)
    K.quant_rows_e4m3(x, q, s)
    return q, s


@pytest.mark.parametrize("K", [1024, 18944])
def test_quant_rows_e4m3_matches_torch_cast(K):
    torch.manual_seed(0)
    x = _rand(333, K, scale=3.0)
    q, s = _quant(x)
    ref_s = x.float().abs().amax(1) / 448.0
    torch.testing.assert_close(s, ref_s, rtol=1e-6, atol=0)
    ref_q = (x.float() / ref_s[:, None]).to(torch.float8_e4m3fn)
    # identical bytes except for the odd last-ulp tie (reciprocal-multiply vs divide)
    mism = (q.view(torch.uint8) != ref_q.view(torch.uint8)).float().mean().item()
    assert mism < 5e-3
    _close(_deq(q, s), x, rtol=7e-2, atol=0)


@pytest.mark.parametrize("D", [384, 1024, 4096])
def test_layernorm_e4m3(D):
    K = _k()
    torch.manual_seed(1)
    x = _rand(257, D, scale=2.0)
    w, b = _rand(D), _rand(D, scale=0.1)
    q = torch.empty(257, D, device=DEV, dtype=torch.float8_e4m3fn)
    s = torch.empty(257, device=DEV, dtype=torch.float32)
    K.layernorm(x, w, b, 1e-6, q, scale8=s)
    ref = torch.nn.functional.layer_norm(x.float(), (D,), w.float(), b.float(), 1e-6)
    _close(_deq(q, s), ref, rtol=7e-2, atol=0)
    torch.testing.assert_close(s, ref.abs().amax(1) / 448.0, rtol=1e-2, atol=0)


@pytest.mark.parametrize("D", [384, 1024, 4096])
def test_layernorm_e4m3_gather_copy_out(D):
    """The shared-memory LayerNorm with a row gather and the raw-row copy, e4m3 output."""
    K = _k()
    torch.manual_seed(11)
    x = _rand(60, D, scale=2.0)
    w, b = _rand(D), _rand(D, scale=0.1)
    rows = torch.tensor([5, 0, 59, 5, 31, 2, 44], device=DEV, dtype=torch.int32)
    q = torch.empty(7, D, device=DEV, dtype=torch.float8_e4m3fn)
    s = torch.empty(7, device=DEV, dtype=torch.float32)
    cp = torch.empty(7, D, device=DEV, dtype=torch.bfloat16)
    K.layernorm(x, w, b, 1e-6, q, rows=rows, copy_out=cp, scale8=s)
    ref = torch.nn.functional.layer_norm(x.float()[rows.long()], (D,), w.float(), b.float(), 1e-6)
    _close(_deq(q, s), ref, rtol=7e-2, atol=0)
    assert torch.equal(cp, x[rows.long()])


@pytest.mark.parametrize("M,N,K", [(1, 256, 128), (300, 512, 1024), (1029, 1024, 4096), (255, 384, 256),
                                   (2500, 256, 768)])
def test_gemm_e4m3_bias(M, N, K):
    K_ = _k()
    torch.manual_seed(2)
    a8, sa = _quant(_rand(M, K))
    w8, sw = K_.quantize_weight_e4m3(_rand(N, K, scale=K ** -0.5))
    bias = _rand(N, scale=0.1)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a8, w8, out, bias=bias, a_scale=sa, b_scale=sw)
    ref = _deq(a8, sa) @ _deq(w8, sw).T + bias.float()
    _close(out, ref)


def test_gemm_e4m3_swiglu_and_resid():
    K_ = _k()
    torch.manual_seed(3)
    from appcorr_b200.models.weights import pack_swiglu

    M, Hd, D = 300, 512, 256
    a8, sa = _quant(_rand(M, D))
    w1, w2 = _rand(Hd, D, scale=D ** -0.5), _rand(Hd, D, scale=D ** -0.5)
    b1, b2 = _rand(Hd, scale=0.1), _rand(Hd, scale=0.1)
    wp, bp = pack_swiglu(w1, w2, b1, b2)
    wp8, swp = K_.quantize_weight_e4m3(wp)
    h = torch.empty(M, Hd, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a8, wp8, h, epi=K_.EPI_SWIGLU, bias=bp, a_scale=sa, b_scale=swp)
    wd = _deq(wp8, swp)
    from appcorr_b200.models.weights import unpack_swiglu

    w1d, w2d = unpack_swiglu(wd)
    x1 = _deq(a8, sa) @ w1d.T + b1.float()
    x2 = _deq(a8, sa) @ w2d.T + b2.float()
    _close(h, torch.nn.functional.silu(x1) * x2, rtol=3e-2, atol=3e-2)
    # fc2 with the LayerScale residual epilogue on a re-quantised h
    h8, sh = _quant(h)
    w3 = _rand(D, Hd, scale=Hd ** -0.5)
    w38, sw3 = K_.quantize_weight_e4m3(w3)
    gamma, resid = _rand(D, scale=0.5), _rand(M, D)
    out = torch.empty(M, D, device=DEV, dtype=torch.bfloat16)
    K_.gemm(h8, w38, out, epi=K_.EPI_RESID, gamma=gamma, resid=resid, a_scale=sh, b_scale=sw3)
    ref = resid.float() + (_deq(h8, sh) @ _deq(w38, sw3).T) * gamma.float()
    _close(out, ref)


def test_qkv_e4m3_grouped_query():
    """q / k / v widths differ (grouped-query attention): 4 q heads, 2 kv heads of 128."""
    K_ = _k()
    torch.manual_seed(4)
    Dh, Hq, Hkv, K = 128, 4, 2, 256
    B, N = 2, 17
    M = B * N
    a8, sa = _quant(_rand(M, K))
    w = _rand((Hq + 2 * Hkv) * Dh, K, scale=K ** -0.5)
    w8, sw = K_.quantize_weight_e4m3(w)
    q = torch.zeros(M, Hq * Dh, device=DEV, dtype=torch.bfloat16)
    k = torch.zeros(M, Hkv * Dh, device=DEV, dtype=torch.bfloat16)
    v = torch.zeros(M, Hkv * Dh, device=DEV, dtype=torch.bfloat16)
    K_.qkv_gemm(a8, w8, None, q, k, v, head_dim=Dh, seq_len=N, n_prefix=N, a_scale=sa, b_scale=sw,
                kv_dim=Hkv * Dh, bn=128)
    ref = _deq(a8, sa) @ _deq(w8, sw).T
    _close(q, ref[:, : Hq * Dh])
    _close(k, ref[:, Hq * Dh:(Hq + Hkv) * Dh])
    _close(v, ref[:, (Hq + Hkv) * Dh:])


def test_auto_precision_picks_by_rows():
    """precision "auto" (reference dinov3_precision.py:479-488): e4m3 operands for a pass with at
    least fp8_auto_min_rows GEMM rows, bf16 below; results stay close to the bf16 engine."""
    from appcorr_b200.models.dinov3.vit import ViTConfig
    from appcorr_b200.models.engine import ViTEngine, random_weights

    cfg = ViTConfig(embed_dim=256, depth=2, num_heads=4, layerscale_init=0.3)
    dev = torch.device(DEV)
    eng = ViTEngine(random_weights(cfg, dev, seed=1, std=0.05), dev, "auto")
    ref = ViTEngine(random_weights(cfg, dev, seed=1, std=0.05), dev, "bf16")
    B, H, W = 4, 128, 128                      # 4 x (64 + 5) = 276 approx rows
    eng.auto_min_rows = 200                    # approx (276 rows) -> fp8; correction (4 x 21) -> bf16
    img = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    outs = []
    for e in (eng, ref):
        s = e.new_session(B, H, W)
        e.prepare_tokens(s, img)
        xa = e.approx(s, 0, 2).clone()
        if e is eng:
            assert s.extra["pass_precision"] == ("approx", "fp8")
        pre = torch.arange(5, dtype=torch.int32, device=DEV).repeat(B, 1).contiguous()
        cand = torch.arange(5, s.N, dtype=torch.int32, device=DEV).repeat(B, 1).contiguous()
        xc = e.correct(s, 0, 2, pre, cand, {"token_keep_ratio": 0.25}).clone()
        if e is eng:
            assert s.extra["pass_precision"] == ("correct", "bf16")
        outs.append((xa, xc))
    torch.cuda.synchronize()
    rel = ((outs[0][0].float() - outs[1][0].float()).norm() / outs[1][0].float().norm()).item()
    assert 1e-4 < rel < 6e-2   # e4m3 noise on the approximate pass, not bit-identical to bf16
