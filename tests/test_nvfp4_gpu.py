"""NVFP4 path on sm_100a: the row quantiser and the NVFP4 LayerNorm against the PyTorch statement
of the format (ops/kernels.py nvfp4_quantize_ref), the tcgen05 kind::mxf4nvf4 block-scaled GEMM
(plain, SwiGLU, residual and qkv epilogues) against an fp32 GEMM of the dequantised operands, the
TP row kernel's NVFP4 all-gather (one rank) and the engine's nvfp4 precision against bf16."""
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


def _quant(x):
    K = _k()
    M, Kd = x.shape
    q = torch.empty(M, Kd // 2, device=DEV, dtype=torch.uint8)
    sf = torch.zeros(K.nvfp4_sf_bytes(M, Kd), device=DEV, dtype=torch.uint8)
    s = torch.empty(M, device=DEV, dtype=torch.float32)
    K.quant_rows_nvfp4(x, q, sf, s)
    return q, sf, s


def _bytes_match(q, sf, s, ref):
    rq, rsf, rs = ref
    torch.testing.assert_close(s, rs, rtol=1e-6, atol=0)
    # identical bytes except for rare last-ulp ties (the LayerNorm rows reach more of them)
    assert (sf != rsf).float().mean().item() < 4e-3
    assert (q != rq).float().mean().item() < 4e-3


@pytest.mark.parametrize("M,Kd", [(1, 64), (333, 1024), (130, 4096), (7, 18944)])
def test_quant_rows_nvfp4_matches_reference(M, Kd):
    K = _k()
    torch.manual_seed(0)
    x = _rand(M, Kd, scale=3.0)
    q, sf, s = _quant(x)
    _bytes_match(q, sf, s, K.nvfp4_quantize_ref(x))


@pytest.mark.parametrize("D,rms", [(1024, False), (4096, False), (3584, True)])
def test_layernorm_nvfp4(D, rms):
    K = _k()
    torch.manual_seed(1)
    n = 257
    x = _rand(n, D, scale=2.0)
    w, b = _rand(D), (None if rms else _rand(D, scale=0.1))
    q = torch.empty(n, D // 2, device=DEV, dtype=torch.uint8)
    sf = torch.zeros(K.nvfp4_sf_bytes(n, D), device=DEV, dtype=torch.uint8)
    s = torch.empty(n, device=DEV, dtype=torch.float32)
    K.layernorm(x, w, b, 1e-6, q, scale8=s, sf=sf, rms=rms)
    # the bf16 LayerNorm kernel's output is the value the NVFP4 LayerNorm quantises
    ln = torch.empty(n, D, device=DEV, dtype=torch.bfloat16)
    K.layernorm(x, w, b, 1e-6, ln, rms=rms)
    _bytes_match(q, sf, s, K.nvfp4_quantize_ref(ln))


@pytest.mark.parametrize("M,N,Kd,bn", [(1, 128, 256, None), (300, 512, 1024, None), (1029, 1024, 4096, None),
                                       (1029, 1024, 4096, 256), (2500, 256, 768, 256), (200, 384, 18944, None)])
def test_gemm_nvfp4_bias(M, N, Kd, bn):
    K = _k()
    torch.manual_seed(2)
    a4, a_sf, a_s = _quant(_rand(M, Kd))
    w4, (w_s, w_sf) = K.quantize_weight_nvfp4(_rand(N, Kd, scale=Kd ** -0.5))
    bias = _rand(N, scale=0.1)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K.gemm(a4, w4, out, bias=bias, a_scale=(a_s, a_sf), b_scale=(w_s, w_sf), bn=bn)
    ref = K.nvfp4_dequantize(a4, a_sf, a_s) @ K.nvfp4_dequantize(w4, w_sf, w_s).T + bias.float()
    _close(out, ref)


@pytest.mark.parametrize("bn", [512, 513])
@pytest.mark.parametrize("M,N,Kd", [(300, 512, 512), (1029, 1536, 1024)])
def test_gemm_nvfp4_2cta_matches_one_cta(M, N, Kd, bn):
    """The CTA-pair kernels (256 x 256 and 256 x 128 tiles, cta_group::2) produce the same bytes as
    the one-CTA 128 x 128 kernel: identical fp32 accumulation order per output."""
    K = _k()
    torch.manual_seed(5)
    a4, a_sf, a_s = _quant(_rand(M, Kd))
    w4, (w_s, w_sf) = K.quantize_weight_nvfp4(_rand(N, Kd, scale=Kd ** -0.5))
    bias = _rand(N, scale=0.1)
    ref = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    out = torch.full((M, N), float("nan"), device=DEV, dtype=torch.bfloat16)
    K.gemm(a4, w4, ref, bias=bias, a_scale=(a_s, a_sf), b_scale=(w_s, w_sf), bn=128)
    K.gemm(a4, w4, out, bias=bias, a_scale=(a_s, a_sf), b_scale=(w_s, w_sf), bn=bn)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("block,bn", [(64, None), (128, 256)])
def test_gemm_nvfp4_swiglu_resid_qkv(block, bn):
    K = _k()
    from appcorr_b200.models.weights import pack_swiglu, unpack_swiglu

    torch.manual_seed(3)
    M, Hd, D = 300, 512, 256
    a4, a_sf, a_s = _quant(_rand(M, D))
    ad = K.nvfp4_dequantize(a4, a_sf, a_s)
    w1, w2 = _rand(Hd, D, scale=D ** -0.5), _rand(Hd, D, scale=D ** -0.5)
    b1, b2 = _rand(Hd, scale=0.1), _rand(Hd, scale=0.1)
    wp, bp = pack_swiglu(w1, w2, b1, b2, block)
    w4, (ws, wsf) = K.quantize_weight_nvfp4(wp)
    h = torch.empty(M, Hd, device=DEV, dtype=torch.bfloat16)
    K.gemm(a4, w4, h, epi=K.EPI_SWIGLU, bias=bp, a_scale=(a_s, a_sf), b_scale=(ws, wsf), bn=bn)
    w1d, w2d = unpack_swiglu(K.nvfp4_dequantize(w4, wsf, ws), block)
    x1 = ad @ w1d.T + b1.float()
    x2 = ad @ w2d.T + b2.float()
    _close(h, torch.nn.functional.silu(x1) * x2, rtol=3e-2, atol=3e-2)
    # residual + LayerScale epilogue on a re-quantised h
    h4, h_sf, h_s = _quant(h)
    w3 = _rand(D, Hd, scale=Hd ** -0.5)
    w34, (w3s, w3sf) = K.quantize_weight_nvfp4(w3)
    gamma, resid = _rand(D, scale=0.5), _rand(M, D)
    out = torch.empty(M, D, device=DEV, dtype=torch.bfloat16)
    K.gemm(h4, w34, out, epi=K.EPI_RESID, gamma=gamma, resid=resid, a_scale=(h_s, h_sf), b_scale=(w3s, w3sf),
           bn=bn)
    ref = resid.float() + (K.nvfp4_dequantize(h4, h_sf, h_s) @ K.nvfp4_dequantize(w34, w3sf, w3s).T) * gamma.float()
    _close(out, ref)
    # qkv split (no RoPE), 128-wide tiles
    Dh, H = 128, 2
    wq = _rand(3 * H * Dh, D, scale=D ** -0.5)
    wq4, (wqs, wqsf) = K.quantize_weight_nvfp4(wq)
    q = torch.zeros(M, H * Dh, device=DEV, dtype=torch.bfloat16)
    k = torch.zeros_like(q)
    v = torch.zeros_like(q)
    K.qkv_gemm(a4, wq4, None, q, k, v, head_dim=Dh, seq_len=M, n_prefix=M, a_scale=(a_s, a_sf),
               b_scale=(wqs, wqsf), bn=bn if bn else 128)
    ref = ad @ K.nvfp4_dequantize(wq4, wqsf, wqs).T
    _close(q, ref[:, : H * Dh])
    _close(k, ref[:, H * Dh: 2 * H * Dh])
    _close(v, ref[:, 2 * H * Dh:])


def test_sp_row_nvfp4_gather_one_rank():
    """Row kernel in load mode with an NVFP4 all-gather into this rank's own buffers."""
    K = _k()
    from appcorr_b200.ops.native import lib

    torch.manual_seed(4)
    M, D = 300, 1024
    x = _rand(M, D, scale=2.0)
    w, b = _rand(D), _rand(D, scale=0.1)
    ag = torch.zeros(M, D // 2, device=DEV, dtype=torch.uint8)
    sc = torch.zeros(M, device=DEV, dtype=torch.float32)
    sf = torch.zeros(K.nvfp4_sf_bytes(M, D), device=DEV, dtype=torch.uint8)
    lib().sp_row(M, None, M, 0, 1, D, [], [], None, None, None, True, None, None, True, None, 0, x, None, w, b,
                 1e-6, False, 2, [ag.data_ptr()], ag.stride(0), [sc.data_ptr()], [sf.data_ptr()])
    ln = torch.empty(M, D, device=DEV, dtype=torch.bfloat16)
    K.layernorm(x, w, b, 1e-6, ln)
    _bytes_match(ag, sf, sc, K.nvfp4_quantize_ref(ln))


def test_engine_nvfp4_tracks_oracle():
    """nvfp4 precision (NVFP4 qkv / fc1 / fc2, e4m3 proj): the approximate pass and the full-set
    correction stay close to the fp32 oracle of a ViT-7B-shaped (SwiGLU, 128-dim heads) stack."""
    from appcorr_b200.models.engine import ViTEngine
    from test_engine_gpu import _float_img, _model, _rel

    torch.manual_seed(2)
    m = _model("vit7b16", depth=3, embed_dim=512, num_heads=4)
    eng = ViTEngine.from_module(m, DEV, precision="nvfp4")
    B, H, W = 2, 96, 128
    img = torch.randint(0, 256, (B, H, W, 3), dtype=torch.uint8, device=DEV)
    sess = eng.new_session(B, H, W)
    eng.prepare_tokens(sess, img)
    with torch.no_grad():
        x_ref, (gh, gw) = m.prepare_tokens_with_masks(_float_img(img))
        x = eng.approx(sess, 0, len(m.blocks)).clone()
        rope = m.rope_embed(H=gh, W=gw)
        xr = x_ref
        for i, blk in enumerate(m.blocks):
            xr, _ = blk.approx(xr, rope, {}, f"layer{i}")
    torch.cuda.synchronize()
    assert _rel(x.view(B, -1, m.embed_dim), xr) < 0.15
    npre = m.n_storage_tokens + 1
    N = sess.N
    pre = torch.arange(npre, device=DEV, dtype=torch.int32)[None].repeat(B, 1).contiguous()
    cand = torch.arange(npre, N, device=DEV, dtype=torch.int32)[None].repeat(B, 1).contiguous()
    xc = eng.correct(sess, 0, len(m.blocks), pre, cand, {"token_keep_ratio": 1.0})
    torch.cuda.synchronize()
    assert _rel(xc.view(B, -1, m.embed_dim), xr) < 0.15


@pytest.mark.parametrize("M", [1029, 77])
def test_gemm_nvfp4_wide_tiles_match_narrow(M):
    """128 x 256 tiles (one accumulator, released to the MMA warp before the epilogue's stores and
    fused work) give the same bytes as 128 x 128 tiles (two accumulators, classic epilogue) for
    every bf16 epilogue: plain + row map, GELU, SwiGLU, residual with each increment mode, and
    qkv with RoPE, a k/v row scatter and dropped rows. Both accumulate each output in the same
    K order, so the results are identical."""
    K = _k()
    from appcorr_b200.models.weights import pack_swiglu

    torch.manual_seed(11)
    D, N = 512, 768
    a4, a_sf, a_s = _quant(_rand(M, D))
    A = (a_s, a_sf)

    def both(fn):
        outs = []
        for bn in (128, 256):
            outs.append(fn(bn))
        torch.cuda.synchronize()
        for x, y in zip(*outs):
            assert torch.equal(x, y), f"max diff {(x.float() - y.float()).abs().max().item()}"

    w4, (ws, wsf) = K.quantize_weight_nvfp4(_rand(N, D, scale=D ** -0.5))
    W = (ws, wsf)
    bias = _rand(N, scale=0.1)
    perm = torch.randperm(M, device=DEV).to(torch.int32)
    perm[::7] = -1  # dropped rows

    def plain(bn, epi):
        out = torch.full((M, N), 7.0, device=DEV, dtype=torch.bfloat16)
        K.gemm(a4, w4, out, epi=epi, bias=bias, out_rows=perm, a_scale=A, b_scale=W, bn=bn)
        return [out]

    both(lambda bn: plain(bn, K.EPI_BF16))
    both(lambda bn: plain(bn, K.EPI_GELU))

    Hd = 512
    w1, w2 = _rand(Hd, D, scale=D ** -0.5), _rand(Hd, D, scale=D ** -0.5)
    b1, b2 = _rand(Hd, scale=0.1), _rand(Hd, scale=0.1)

    def swiglu(bn):
        wp, bp = pack_swiglu(w1, w2, b1, b2, bn // 2)
        wq, (s, sf) = K.quantize_weight_nvfp4(wp)
        h = torch.empty(M, Hd, device=DEV, dtype=torch.bfloat16)
        K.gemm(a4, wq, h, epi=K.EPI_SWIGLU, bias=bp, a_scale=A, b_scale=(s, sf), bn=bn)
        return [h]

    both(swiglu)

    gamma, resid, resid2 = _rand(N, scale=0.5), _rand(M, N), _rand(M, N)
    rows = torch.randperm(M, device=DEV).to(torch.int32)
    aux0 = _rand(M, N)
    for mode in (K.AUX_SET, K.AUX_ADD, K.AUX_OUT_MINUS):
        def resid_fn(bn, mode=mode):
            out = resid.clone()
            aux = aux0.clone()
            K.gemm(a4, w4, out, epi=K.EPI_RESID, bias=bias, gamma=gamma, resid=resid, out_rows=rows, aux=aux,
                   aux_mode=mode, resid2=resid2 if mode == K.AUX_OUT_MINUS else None, a_scale=A, b_scale=W, bn=bn)
            return [out, aux]

        both(resid_fn)

    Dh, H, npre = 128, 2, 5
    wq4, (wqs, wqsf) = K.quantize_weight_nvfp4(_rand(3 * H * Dh, D, scale=D ** -0.5))
    bq = _rand(3 * H * Dh, scale=0.1)
    sin = torch.randn(M, Dh // 2, device=DEV).repeat(1, 2).contiguous()
    cos = torch.randn(M, Dh // 2, device=DEV).repeat(1, 2).contiguous()
    tok = torch.randint(0, M, (M,), device=DEV, dtype=torch.int32)
    kvr = torch.randperm(M, device=DEV).to(torch.int32)
    kvr[::5] = -1

    def qkv(bn):
        q = torch.zeros(M, H * Dh, device=DEV, dtype=torch.bfloat16)
        k = torch.zeros_like(q)
        v = torch.zeros_like(q)
        K.qkv_gemm(a4, wq4, bq, q, k, v, head_dim=Dh, tok_idx=tok, kv_rows=kvr, rope=(sin, cos), n_prefix=npre,
                   a_scale=A, b_scale=(wqs, wqsf), bn=bn)
        return [q, k, v]

    both(qkv)
