"""Numerics of the sm_100a kernels against plain PyTorch fp32 references of the same op."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _k():
    from appcorr_b200.ops import kernels as K

    return K


def _rand(*shape, scale=1.0, dtype=torch.bfloat16):
    return (torch.randn(*shape, device=DEV) * scale).to(dtype)


def _close(a, b, rtol=2e-2, atol=2e-2):
    a = a.float()
    b = b.float()
    err = (a - b).abs().max().item()
    ref = b.abs().max().item() + 1e-6
    assert err <= atol + rtol * ref, f"max err {err} (ref max {ref})"


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (127, 256, 256), (300, 512, 1024), (1029, 1024, 4096),
                                   (2500, 160, 768), (128, 128, 64), (513, 384, 192)])
def test_gemm_bf16_bias(M, N, K):
    K_ = _k()
    torch.manual_seed(0)
    a = _rand(M, K)
    w = _rand(N, K, scale=K ** -0.5)
    bias = _rand(N, scale=0.1)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a, w, out, bias=bias)
    ref = a.float() @ w.float().T + bias.float()
    torch.cuda.synchronize()
    _close(out, ref)


@pytest.mark.parametrize("bn", [64, 128, 256])
def test_gemm_tile_widths_f32(bn):
    K_ = _k()
    torch.manual_seed(1)
    M, N, K = 700, 512, 512
    a = _rand(M, K)
    w = _rand(N, K, scale=K ** -0.5)
    out = torch.empty(M, N, device=DEV, dtype=torch.float32)
    K_.gemm(a, w, out, epi=K_.EPI_F32, bn=bn)
    ref = a.float() @ w.float().T
    _close(out, ref, rtol=1e-3, atol=1e-3)


def test_gemm_row_map_and_gelu():
    K_ = _k()
    torch.manual_seed(2)
    M, N, K = 200, 256, 128
    a = _rand(M, K)
    w = _rand(N, K, scale=K ** -0.5)
    bias = _rand(N, scale=0.1)
    rows = torch.randperm(400, device=DEV)[:M].to(torch.int32)
    out = torch.zeros(400, N, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a, w, out, epi=K_.EPI_GELU, bias=bias, out_rows=rows)
    ref = torch.nn.functional.gelu(a.float() @ w.float().T + bias.float())
    _close(out[rows.long()], ref)
    mask = torch.ones(400, dtype=torch.bool, device=DEV)
    mask[rows.long()] = False
    assert out[mask].abs().max().item() == 0


def test_gemm_swiglu():
    K_ = _k()
    torch.manual_seed(3)
    M, Hd, K = 333, 512, 256
    a = _rand(M, K)
    w1 = _rand(Hd, K, scale=K ** -0.5)
    w2 = _rand(Hd, K, scale=K ** -0.5)
    b1 = _rand(Hd, scale=0.1)
    b2 = _rand(Hd, scale=0.1)
    from appcorr_b200.models.weights import pack_swiglu

    wp, bp = pack_swiglu(w1, w2, b1, b2)
    out = torch.empty(M, Hd, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a, wp, out, epi=K_.EPI_SWIGLU, bias=bp)
    x1 = a.float() @ w1.float().T + b1.float()
    x2 = a.float() @ w2.float().T + b2.float()
    ref = torch.nn.functional.silu(x1) * x2
    _close(out, ref, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("mode", ["set", "add", "out_minus"])
def test_gemm_resid_layerscale(mode):
    K_ = _k()
    torch.manual_seed(4)
    M, N, K = 300, 512, 256
    a = _rand(M, K)
    w = _rand(N, K, scale=K ** -0.5)
    bias = _rand(N, scale=0.1)
    gamma = _rand(N, scale=0.5)
    resid = _rand(M, N)
    resid2 = _rand(M, N)
    rows = torch.randperm(600, device=DEV)[:M].to(torch.int32)
    out = torch.zeros(600, N, device=DEV, dtype=torch.bfloat16)
    aux0 = _rand(600, N)
    aux = aux0.clone()
    am = {"set": K_.AUX_SET, "add": K_.AUX_ADD, "out_minus": K_.AUX_OUT_MINUS}[mode]
    K_.gemm(a, w, out, epi=K_.EPI_RESID, bias=bias, gamma=gamma, resid=resid, out_rows=rows, aux=aux,
            aux_mode=am, resid2=resid2 if mode == "out_minus" else None)
    delta = (a.float() @ w.float().T + bias.float()) * gamma.float()
    _close(out[rows.long()], resid.float() + delta)
    if mode == "set":
        ref_aux = delta
    elif mode == "add":
        ref_aux = aux0[rows.long()].float() + delta
    else:
        ref_aux = resid.float() - resid2.float() + delta
    _close(aux[rows.long()], ref_aux)


def _rope_ref(x, sin, cos):
    h = x.shape[-1] // 2
    rot = torch.cat([-x[..., h:], x[..., :h]], dim=-1)
    return x * cos + rot * sin


@pytest.mark.parametrize("Dh,H", [(128, 4), (64, 8)])
def test_qkv_rope_scatter(Dh, H):
    K_ = _k()
    torch.manual_seed(5)
    D = H * Dh
    B, N, npre = 2, 21, 5
    K = 256
    M = B * N
    a = _rand(M, K)
    w = _rand(3 * D, K, scale=K ** -0.5)
    bias = _rand(3 * D, scale=0.1)
    # RoPE tables repeat their first half (angles tiled twice), as RopePositionEmbedding builds them
    sin = torch.randn(N - npre, Dh // 2, device=DEV).repeat(1, 2).contiguous()
    cos = torch.randn(N - npre, Dh // 2, device=DEV).repeat(1, 2).contiguous()
    q = torch.zeros(M, D, device=DEV, dtype=torch.bfloat16)
    k = torch.zeros(M, D, device=DEV, dtype=torch.bfloat16)
    v = torch.zeros(M, D, device=DEV, dtype=torch.bfloat16)
    K_.qkv_gemm(a, w, bias, q, k, v, head_dim=Dh, seq_len=N, rope=(sin, cos), n_prefix=npre)
    qkv = (a.float() @ w.float().T + bias.float()).view(B, N, 3, H, Dh)
    qr = qkv[:, :, 0].clone()
    kr = qkv[:, :, 1].clone()
    qr[:, npre:] = _rope_ref(qr[:, npre:], sin[None, :, None], cos[None, :, None])
    kr[:, npre:] = _rope_ref(kr[:, npre:], sin[None, :, None], cos[None, :, None])
    _close(q.view(B, N, H, Dh), qr)
    _close(k.view(B, N, H, Dh), kr)
    _close(v.view(B, N, H, Dh), qkv[:, :, 2])
    # scatter form: 7 selected rows, k/v written into cache rows, q packed
    sel_tok = torch.tensor([0, 3, 6, 9, 12, 15, 20], device=DEV, dtype=torch.int32)
    sel_rows = sel_tok + N  # batch 1
    a_sel = a[sel_rows.long()].contiguous()
    q2 = torch.zeros(7, D, device=DEV, dtype=torch.bfloat16)
    k2 = k.clone()
    v2 = v.clone()
    k2[sel_rows.long()] = 0
    K_.qkv_gemm(a_sel, w, bias, q2, k2, v2, head_dim=Dh, tok_idx=sel_tok, kv_rows=sel_rows, rope=(sin, cos),
                n_prefix=npre)
    _close(q2, q[sel_rows.long()], rtol=1e-2, atol=1e-2)
    _close(k2, k, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("impl", ["tcgen05", "tcgen05_split", "tcgen05_2q", "mma"])
@pytest.mark.parametrize("Dh,H,Tq,Tk", [(128, 4, 1029, 1029), (64, 6, 197, 197), (128, 2, 312, 1029), (64, 3, 5, 70),
                                        (128, 2, 130, 260)])
def test_attention(Dh, H, Tq, Tk, impl):
    K_ = _k()
    torch.manual_seed(6)
    B = 2
    q = _rand(B * Tq, H * Dh)
    k = _rand(B * Tk, H * Dh)
    v = _rand(B * Tk, H * Dh)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, Tq, device=DEV)
    K_.attention(q, k, v, o, B=B, Tq=Tq, Tk=Tk, H=H, Dh=Dh, lse=lse, impl=impl)
    torch.cuda.synchronize()
    from appcorr_b200.ops.native import check_errors

    check_errors(q.device)
    qf = q.float().view(B, Tq, H, Dh).transpose(1, 2)
    kf = k.float().view(B, Tk, H, Dh).transpose(1, 2)
    vf = v.float().view(B, Tk, H, Dh).transpose(1, 2)
    s = qf @ kf.transpose(-1, -2) / math.sqrt(Dh)
    ref = (s.softmax(-1) @ vf).transpose(1, 2).reshape(B * Tq, H * Dh)
    _close(o, ref, rtol=2e-2, atol=2e-2)
    _close(lse, torch.logsumexp(s, -1), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("D", [384, 1024, 4096])
def test_layernorm_gather(D):
    K_ = _k()
    torch.manual_seed(7)
    x = _rand(50, D, scale=3.0)
    w = _rand(D)
    b = _rand(D)
    rows = torch.tensor([3, 7, 7, 49, 0], device=DEV, dtype=torch.int32)
    out = torch.empty(5, D, device=DEV, dtype=torch.bfloat16)
    cp = torch.empty(5, D, device=DEV, dtype=torch.bfloat16)
    K_.layernorm(x, w, b, 1e-5, out, rows=rows, copy_out=cp)
    ref = torch.nn.functional.layer_norm(x.float()[rows.long()], (D,), w.float(), b.float(), 1e-5)
    _close(out, ref)
    assert torch.equal(cp, x[rows.long()])


def test_cls_pscore_and_plan():
    K_ = _k()
    torch.manual_seed(8)
    B, N, H, Dh, npre = 3, 69, 4, 64, 5
    q = _rand(B * N, H * Dh)
    k = _rand(B * N, H * Dh)
    scratch = torch.empty(B, H, N, device=DEV)
    ps = torch.empty(B, N, device=DEV)
    K_.cls_attn_pscore(q, k, B=B, N=N, H=H, Dh=Dh, scratch=scratch, out=ps)
    qf = q.float().view(B, N, H, Dh)[:, 0]  # [B,H,Dh]
    kf = k.float().view(B, N, H, Dh)
    s = torch.einsum("bhd,bnhd->bhn", qf, kf) / math.sqrt(Dh)
    ref = s.softmax(-1).mean(1)
    _close(ps, ref, rtol=1e-3, atol=1e-4)
    cand = torch.arange(npre, N, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    pre = torch.arange(npre, device=DEV, dtype=torch.int32).repeat(B, 1).contiguous()
    kk = int((N - npre) * 0.3)
    upd = torch.empty(B, npre + kk, device=DEV, dtype=torch.int32)
    rows = torch.empty(B * (npre + kk), device=DEV, dtype=torch.int32)
    stats = torch.empty(B, 2, device=DEV)
    K_.correction_plan(ps, pre, cand, kk, upd, rows, stats=stats)
    top = torch.topk(ps[:, npre:], kk, dim=1).indices.sort(1).values + npre
    assert torch.equal(upd[:, npre:].long(), top)
    assert torch.equal(upd[:, :npre], pre)
    assert torch.equal(rows.view(B, -1).long(), upd.long() + torch.arange(B, device=DEV)[:, None] * N)


def test_pyrup_matches_numpy_cv2_rule():
    K_ = _k()
    from appcorr_b200.policies.transmission.pyramid import pyr_up

    rng = np.random.default_rng(0)
    base = rng.integers(0, 256, (2, 37, 50, 3), dtype=np.uint8)
    res = rng.integers(-60, 60, (2, 74, 100, 3)).astype(np.int16)
    ref = np.stack([np.clip(pyr_up(base[i]).astype(np.int32) + res[i], 0, 255).astype(np.uint8) for i in range(2)])
    out = torch.empty(2, 74, 100, 3, dtype=torch.uint8, device=DEV)
    K_.pyrup_add(torch.from_numpy(base).to(DEV), torch.from_numpy(res).to(DEV), out)
    assert np.array_equal(out.cpu().numpy(), ref)


def test_upsample_argmax():
    K_ = _k()
    torch.manual_seed(9)
    B, h, w, C = 2, 8, 8, 150
    logits = torch.randn(B, h, w, 160, device=DEV)
    out = torch.empty(B, 64, 64, dtype=torch.uint8, device=DEV)
    K_.upsample_argmax(logits, C, 64, 64, out)
    ref = torch.nn.functional.interpolate(logits[..., :C].permute(0, 3, 1, 2), size=(64, 64), mode="bilinear",
                                          align_corners=False).argmax(1)
    agree = (out.long() == ref).float().mean().item()
    assert agree > 0.999


def test_patch_im2col():
    K_ = _k()
    img = torch.randint(0, 256, (2, 32, 48, 3), dtype=torch.uint8, device=DEV)
    out = torch.empty(2 * 2 * 3, 768, device=DEV, dtype=torch.bfloat16)
    K_.patch_im2col(img, 16, out)
    mean = torch.tensor(K_.IMAGENET_MEAN, device=DEV)
    std = torch.tensor(K_.IMAGENET_STD, device=DEV)
    x = (img.float() / 255 - mean) / std  # B H W C
    x = x.permute(0, 3, 1, 2)  # B C H W
    cols = torch.nn.functional.unfold(x, 16, stride=16)  # B, C*256, L
    ref = cols.transpose(1, 2).reshape(-1, 768)
    _close(out, ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (300, 512, 1024), (1029, 1024, 4096), (2496, 768, 256), (255, 256, 128)])
def test_gemm_2cta_bias(M, N, K):
    """bn=512 selects the cluster-of-two (cta_group::2, 256x256 tile) kernel."""
    K_ = _k()
    torch.manual_seed(10)
    a = _rand(M, K)
    w = _rand(N, K, scale=K ** -0.5)
    bias = _rand(N, scale=0.1)
    out = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a, w, out, bias=bias, bn=512)
    _close(out, a.float() @ w.float().T + bias.float())


def test_gemm_2cta_epilogues():
    K_ = _k()
    from appcorr_b200.models.weights import pack_swiglu

    torch.manual_seed(11)
    M, Hd, K = 333, 512, 256
    a = _rand(M, K)
    w1, w2 = _rand(Hd, K, scale=K ** -0.5), _rand(Hd, K, scale=K ** -0.5)
    b1, b2 = _rand(Hd, scale=0.1), _rand(Hd, scale=0.1)
    wp, bp = pack_swiglu(w1, w2, b1, b2)
    out = torch.empty(M, Hd, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a, wp, out, epi=K_.EPI_SWIGLU, bias=bp, bn=512)
    ref = torch.nn.functional.silu(a.float() @ w1.float().T + b1.float()) * (a.float() @ w2.float().T + b2.float())
    _close(out, ref, rtol=3e-2, atol=3e-2)
    N = 512
    w = _rand(N, K, scale=K ** -0.5)
    gamma, resid = _rand(N, scale=0.5), _rand(M, N)
    aux = _rand(M, N)
    aux0 = aux.clone()
    out2 = torch.empty(M, N, device=DEV, dtype=torch.bfloat16)
    K_.gemm(a, w, out2, epi=K_.EPI_RESID, gamma=gamma, resid=resid, aux=aux, aux_mode=K_.AUX_ADD, bn=512)
    delta = (a.float() @ w.float().T) * gamma.float()
    _close(out2, resid.float() + delta)
    _close(aux, aux0.float() + delta)
    # qkv with RoPE on the 2-CTA path equals the 1-CTA path
    H, Dh, B, Nt, npre = 4, 128, 2, 37, 5
    D = H * Dh
    a3 = _rand(B * Nt, K)
    w3 = _rand(3 * D, K, scale=K ** -0.5)
    sin = torch.randn(Nt - npre, Dh // 2, device=DEV).repeat(1, 2).contiguous()
    cos = torch.randn(Nt - npre, Dh // 2, device=DEV).repeat(1, 2).contiguous()
    bufs = [[torch.zeros(B * Nt, D, device=DEV, dtype=torch.bfloat16) for _ in range(3)] for _ in range(2)]
    for bn, (q, k, v) in zip((256, 512), bufs):
        K_.qkv_gemm(a3, w3, None, q, k, v, head_dim=Dh, seq_len=Nt, rope=(sin, cos), n_prefix=npre, bn=bn)
    for x, y in zip(*bufs):
        _close(x, y, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("impl", ["tcgen05", "tcgen05_split"])
def test_attention_fused_cls_score(impl):
    """The tcgen05 attention's CLS softmax row equals the standalone CLS score kernel."""
    K_ = _k()
    torch.manual_seed(12)
    B, N, H, Dh = 2, 300, 4, 128
    q = _rand(B * N, H * Dh)
    k = _rand(B * N, H * Dh)
    v = _rand(B * N, H * Dh)
    o = torch.empty_like(q)
    probs = torch.empty(B, H, N, device=DEV)
    K_.attention(q, k, v, o, B=B, Tq=N, Tk=N, H=H, Dh=Dh, impl=impl, cls_probs=probs)
    fused = torch.empty(B, N, device=DEV)
    K_.head_mean(probs, B, H, N, fused)
    ref = torch.empty(B, N, device=DEV)
    K_.cls_attn_pscore(q, k, B=B, N=N, H=H, Dh=Dh, scratch=torch.empty(B, H, N, device=DEV), out=ref)
    _close(fused, ref, rtol=1e-3, atol=1e-5)


def test_exp2_poly_error_bound():
    """The FMA-pipe exp2 that the attention softmax uses for part of its probabilities stays within
    its fitted relative-error bound (7.5e-5, plus fp32 rounding) of exp2 on the softmax's input
    range x <= 0, and gives tiny non-negative values (no sign or exponent wrap) far below it."""
    from appcorr_b200.ops.native import lib

    x = torch.cat([torch.linspace(-124.0, 0.0, 1 << 20, device=DEV),
                   -torch.rand(1 << 16, device=DEV) * 8, torch.tensor([0.0, -0.5, -1e-7], device=DEV)])
    y = torch.empty_like(x)
    lib().exp2_poly(x, y)
    ref = torch.exp2(x.double())
    rel = ((y.double() - ref).abs() / ref).max().item()
    assert rel < 8e-5, rel
    far = torch.tensor([-125.0, -200.0, -1e30, -3.0e38], device=DEV)
    yf = torch.empty_like(far)
    lib().exp2_poly(far, yf)
    assert bool((yf >= 0).all()) and bool((yf < 1e-37).all()), yf.tolist()
