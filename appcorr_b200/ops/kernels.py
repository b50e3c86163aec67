"""Functional wrappers around the sm_100a kernels (one call = one or two kernel launches).

All tensors are CUDA tensors in the layouts the kernels expect (bf16 row-major activations, BTHD
attention tensors, int32 row maps). Shapes are validated in the C++ bindings.
"""
from __future__ import annotations

import os
from typing import Optional, Sequence, Tuple

import torch

from .native import err_word, lib

EPI_BF16, EPI_F32, EPI_GELU, EPI_SWIGLU, EPI_RESID, EPI_QKV = range(6)
AUX_NONE, AUX_SET, AUX_ADD, AUX_OUT_MINUS = range(4)

# Number of native kernel launches issued through this module (read by the benchmark).
LAUNCHES = [0]
# NVFP4 tile width of the qkv GEMM: 0 = 256 when the widths allow (one accumulator; measured
# 18.7 ms per ViT-7B step against 20.2 ms at 128), 128 = always 128 (two accumulators). The other
# NVFP4 GEMMs run 128-wide tiles (SwiGLU 20.4 vs 24.0 ms, residual fc2 12.6 vs 13.3 ms).
FP4_BN = [int(os.environ.get("APPCORR_FP4_BN", "0"))]
# NVFP4 GEMMs that run 128 x 256 tiles (one accumulator, early-release epilogue); the others run
# 128 x 128 tiles with two accumulators. A SwiGLU weight is packed in BN / 2-row blocks to match.
FP4_WIDE = set(filter(None, os.environ.get("APPCORR_FP4_WIDE", "qkv,fc1").split(",")))


def fp4_tile(name: str) -> int:
    """Tile width of the NVFP4 GEMM `name` ("qkv", "fc1", "fc2")."""
    return 256 if name in FP4_WIDE and FP4_BN[0] != 128 else 128


def _count(n: int = 1) -> None:
    LAUNCHES[0] += n


IMAGENET_MEAN = (0.485, 0.456, 0.406)
IMAGENET_STD = (0.229, 0.224, 0.225)


def _pick_bn(n: int, m: int) -> int:
    if n >= 1024 and n % 256 == 0:
        return 256
    if n % 128 == 0 and n >= 128:
        return 128
    return 64


def gemm(a: torch.Tensor, w: torch.Tensor, out: torch.Tensor, *, epi: int = EPI_BF16,
         bias: Optional[torch.Tensor] = None, out_rows: Optional[torch.Tensor] = None,
         gamma: Optional[torch.Tensor] = None, resid: Optional[torch.Tensor] = None,
         resid_rows: Optional[torch.Tensor] = None, aux: Optional[torch.Tensor] = None,
         aux_rows: Optional[torch.Tensor] = None, aux_mode: int = AUX_NONE,
         resid2: Optional[torch.Tensor] = None, bn: Optional[int] = None,
         max_ctas: int = 0, a_scale: Optional[torch.Tensor] = None,
         b_scale=None, rs: Optional[tuple] = None) -> torch.Tensor:
    """out = epilogue(a @ w^T). `a` [M, K], `w` [N, K] (nn.Linear layout), both bf16, both e4m3
    or both NVFP4. e4m3 operands carry fp32 scales a_scale [M] (per row) and b_scale [N] (per
    output channel) that the epilogue applies to the fp32 accumulator before bias / activation.
    NVFP4 operands are uint8 [rows, K/2] (packed e2m1) and pass (row scale [rows] fp32, block
    scales uint8) pairs as a_scale / b_scale (see quant_rows_nvfp4); their default tile width is
    128, so a SwiGLU weight is packed in 64-row blocks (bn=256 takes the usual 128-row packing).
    rs = (slot_ptrs, rows_per_rank, rank, slot_rows, ld): reduce-scatter epilogue; row m goes to
    rank (out_rows[m] or m) // rows_per_rank, slot row rank * slot_rows + m (`out` unused)."""
    fp8 = a.dtype == torch.float8_e4m3fn
    a_sf = b_sf = None
    if isinstance(a_scale, tuple):
        a_scale, a_sf = a_scale
        b_scale, b_sf = b_scale
        if bn is None:
            bn = 128
    if bn is None:
        bn = 256 if epi == EPI_SWIGLU else _pick_bn(w.shape[0], a.shape[0])
        if fp8 and bn == 64:
            bn = 128
    _count()
    lib().gemm(a, w, epi, bn, err_word(a.device), out=out, out_rows=out_rows, bias=bias, gamma=gamma,
               resid=resid, resid_rows=resid_rows, aux=aux, aux_rows=aux_rows, aux_mode=aux_mode,
               resid2=resid2, max_ctas=max_ctas, a_scale=a_scale, b_scale=b_scale, a_sf=a_sf, b_sf=b_sf,
               **({} if rs is None else dict(rs_out=list(rs[0]), rs_rows_per_rank=int(rs[1]), rs_rank=int(rs[2]),
                                             rs_slot_rows=int(rs[3]), rs_ld=int(rs[4]))))
    return out


def qkv_gemm(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], q_out: torch.Tensor,
             k_out: torch.Tensor, v_out: torch.Tensor, *, head_dim: int, seq_len: int = 0,
             tok_idx: Optional[torch.Tensor] = None, kv_rows: Optional[torch.Tensor] = None,
             rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, n_prefix: int = 0,
             bn: Optional[int] = None, a_scale=None, b_scale=None, kv_dim: int = 0) -> None:
    """qkv projection with RoPE on q/k (tokens >= n_prefix) split into three BTHD buffers.

    q row m is written at q_out[m]; k/v rows at kv_rows[m] (or m). `rope` = (sin, cos) fp32
    tables [n_patch_tokens, head_dim] whose second half repeats the first (the DINOv3 angle
    layout); the kernel reads only the first half. kv_dim > 0: grouped-query weight rows
    [q (N - 2 kv_dim) | k (kv_dim) | v (kv_dim)].
    """
    dim = w.shape[0] - 2 * kv_dim if kv_dim else w.shape[0] // 3
    a_sf = b_sf = None
    if isinstance(a_scale, tuple):  # NVFP4 operands: (row scale, block scales); 256- or 128-wide tiles
        a_scale, a_sf = a_scale
        b_scale, b_sf = b_scale
        if bn is None:
            bn = 256 if dim % 256 == 0 and (kv_dim or dim) % 256 == 0 and fp4_tile("qkv") == 256 else 128
    if bn is None:  # widest tile that divides the q and the k / v widths (tiles never straddle)
        bn = next((t for t in (256, 128, 64) if dim % t == 0 and (kv_dim or dim) % t == 0), 128)
    sin, cos = rope if rope is not None else (None, None)
    _count()
    lib().gemm(a, w, EPI_QKV, bn, err_word(a.device), bias=bias, q_out=q_out, k_out=k_out, v_out=v_out,
               kv_rows=kv_rows, tok_idx=tok_idx, seq_len=seq_len, rope_sin=sin, rope_cos=cos,
               n_prefix=n_prefix, head_dim=head_dim, a_scale=a_scale, b_scale=b_scale, kv_dim=kv_dim,
               a_sf=a_sf, b_sf=b_sf)


def layernorm(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], eps: float, out: torch.Tensor,
              rows: Optional[torch.Tensor] = None, copy_out: Optional[torch.Tensor] = None,
              scale8: Optional[torch.Tensor] = None, rms: bool = False,
              sf: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out[i] = LN(x[rows[i]]) (rows=None: every row). copy_out[i] receives the raw gathered row.
    An e4m3 `out` receives the bf16-rounded LN row divided by scale8[i] = amax_i / 448; a uint8
    `out` [n, D/2] receives it as NVFP4 (block scales into `sf`, row scale scale8[i]).
    rms=True: RMSNorm x * rsqrt(mean(x^2) + eps) * w (b must be None)."""
    _count()
    lib().layernorm(x, rows, w, b, float(eps), out, copy_out, scale8, rms, sf)
    return out


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, out: torch.Tensor, **kw) -> torch.Tensor:
    return layernorm(x, w, None, eps, out, rms=True, **kw)


def quant_rows_e4m3(x: torch.Tensor, out: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """out = x / scale[:, None] in e4m3 with scale = row amax / 448 (fp32)."""
    _count()
    lib().quant_rows_e4m3(x, out, scale)
    return out


def quantize_weight_e4m3(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Per-output-channel e4m3 weight: (w8 [N, K], scale [N] fp32) with w ~= w8 * scale[:, None].
    One-time weight preparation (any device)."""
    wf = w.float()
    sc = (wf.abs().amax(dim=1).clamp_min(1e-12) / 448.0).contiguous()
    w8 = (wf / sc[:, None]).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).contiguous()
    return w8, sc


# ---------------------------------------------------------------------------------------- NVFP4
# Format: e2m1 values packed two per byte (element 2i in the low nibble), one ue4m3 scale per 16
# elements of a row, and an fp32 row scale = row amax / (6 * 448) so every block scale fits ue4m3:
# x ~= e2m1 * block_scale * row_scale. Block scales are stored in 128-row x 64-element tiles of
# 512 bytes (tile (row // 128, k // 64) at ((row // 128) * (K // 64) + k // 64) * 512; inside a
# tile row r, 16-element block j sits at (r % 32) * 16 + ((r % 128) // 32) * 4 + j % 4) -- the
# blocked scale layout of CUTLASS / torch._scaled_mm, which is also the tcgen05.cp source pattern.
# Reference: the Triton quantiser appcorr/models/dinov3/layers/triton_kernels/nvfp4_fused.py:54-145
# (per-tensor second-level scale there; per-row here, which the GEMM epilogue folds per row).
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
# round-to-nearest-even boundaries between consecutive magnitudes: (threshold, upper code even)
_E2M1_BOUNDS = ((0.25, False), (0.75, True), (1.25, False), (1.75, True), (2.5, False), (3.5, True), (5.0, False))


def nvfp4_sf_bytes(rows: int, k: int) -> int:
    """Bytes of the blocked scale tensor of a [rows, k] NVFP4 matrix."""
    return ((rows + 127) // 128) * (k // 64) * 512


def nvfp4_sf_index(rows: int, k: int, device=None) -> torch.Tensor:
    """int64 [rows, k // 16]: byte offset of each block scale in the blocked layout."""
    r = torch.arange(rows, device=device)[:, None]
    j = torch.arange(k // 16, device=device)[None, :]
    return (((r // 128) * (k // 64) + j // 4) * 512 + (r % 32) * 16 + ((r % 128) // 32) * 4 + j % 4)


def _e2m1_codes(y: torch.Tensor) -> torch.Tensor:
    a = y.abs()
    code = torch.zeros(y.shape, dtype=torch.uint8, device=y.device)
    for t, incl in _E2M1_BOUNDS:
        code += (a >= t if incl else a > t).to(torch.uint8)
    return code | (torch.signbit(y).to(torch.uint8) << 3)


def nvfp4_quantize_ref(x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """PyTorch statement of the NVFP4 quantiser (same fp32 operation order as the CUDA kernels):
    x [M, K] -> (packed uint8 [M, K/2], block scales uint8 [nvfp4_sf_bytes], row scale fp32 [M])."""
    xf = x.float()
    M, Kd = xf.shape
    assert Kd % 64 == 0, "NVFP4 rows need K % 64 == 0"
    rs = xf.abs().amax(1).clamp_min(1e-12) / (6.0 * 448.0)
    inv_rs = 1.0 / rs
    blk = xf.view(M, Kd // 16, 16)
    bm = blk.abs().amax(2)
    s = (bm * torch.tensor(1.0 / 6.0, dtype=torch.float32) * inv_rs[:, None]).clamp(max=448.0)
    s8 = s.to(torch.float8_e4m3fn)
    sd = s8.float()
    mul = torch.where(sd > 0, 1.0 / (sd * rs[:, None]), torch.zeros_like(sd))
    codes = _e2m1_codes((blk * mul[..., None]).view(M, Kd))
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    sf = torch.zeros(nvfp4_sf_bytes(M, Kd), dtype=torch.uint8, device=x.device)
    sf[nvfp4_sf_index(M, Kd, x.device).reshape(-1)] = s8.view(torch.uint8).reshape(-1)
    return packed, sf, rs.contiguous()


def nvfp4_dequantize(q: torch.Tensor, sf: torch.Tensor, rs: torch.Tensor) -> torch.Tensor:
    """fp32 [M, K] values of an NVFP4 matrix (oracle for tests)."""
    M, half = q.shape
    Kd = 2 * half
    table = torch.tensor(E2M1_VALUES + tuple(-v for v in E2M1_VALUES), dtype=torch.float32, device=q.device)
    codes = torch.stack([q & 0xF, q >> 4], dim=2).view(M, Kd).long()
    vals = table[codes]
    s8 = sf[nvfp4_sf_index(M, Kd, q.device)].view(torch.float8_e4m3fn).float()
    return (vals.view(M, Kd // 16, 16) * s8[..., None]).view(M, Kd) * rs[:M, None].float()


def quant_rows_nvfp4(x: torch.Tensor, out: torch.Tensor, sf: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """NVFP4 rows of bf16 x [M, K]: out uint8 [M, K/2], sf (blocked block scales), scale fp32 [M]."""
    _count()
    lib().quant_rows_nvfp4(x, out, sf, scale)
    return out


def quantize_weight_nvfp4(w: torch.Tensor) -> Tuple[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """One-time NVFP4 weight preparation: (w4 [N, K/2] uint8, (channel scale [N] fp32, block scales))
    -- the (operand, scales) pair the GEMM wrappers take."""
    q, sf, rs = nvfp4_quantize_ref(w)
    return q, (rs, sf)


def add_(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    _count()
    lib().add_(x, y)
    return x


# "tcgen05_split" (default: measured fastest): one 128-row query tile per CTA, two softmax threads
# per row (64 key columns each), P in TMEM, 3-stage K/V ring;
# "tcgen05": the same tile with one softmax thread per row, P in shared memory;
# "tcgen05_2q": two query tiles per CTA sharing K/V, P kept in TMEM; "mma": the mma.sync kernel
ATTENTION_IMPL = ["tcgen05_split"]
_ATTN_VARIANT = {"tcgen05_2q": 0, "tcgen05": 1, "tcgen05_split": 2}


def attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, o: torch.Tensor, *, B: int, Tq: int,
              Tk: int, H: int, Dh: int, scale: Optional[float] = None,
              lse: Optional[torch.Tensor] = None, impl: Optional[str] = None,
              cls_probs: Optional[torch.Tensor] = None, Hkv: int = 0, causal: bool = False,
              q_pos: Optional[torch.Tensor] = None, block_table: Optional[torch.Tensor] = None,
              q_lo: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Attention on BTHD tensors: q/o [B*Tq, H*Dh], k/v [B*Tk, Hkv*Dh].

    cls_probs (tcgen05 path): fp32 [B, H, Tk] receives the softmax row of query 0 (the CLS
    token) of every (batch, head), computed in the same pass.
    Hkv: key/value heads (grouped-query attention; 0 = H). causal: query row i sees keys up to
    q_pos[i] (int32 [B*Tq]; default i + Tk - Tq), so a packed, non-contiguous query set attends
    with its own causal frontier. block_table: int32 [B, blocks] of 128-row pages in a paged
    K/V pool (k/v are then the pools). q_lo: int32 [B*Tq] first key of each query row; with
    causal=True and q_pos as the last key, each query attends the key range [q_lo, q_pos]
    (windowed attention of packed queries).
    """
    if scale is None:
        scale = Dh ** -0.5
    impl = impl or ATTENTION_IMPL[0]
    if impl == "mma" and (Hkv or causal or q_pos is not None or block_table is not None):
        impl = "tcgen05"
    if q_lo is not None and impl not in ("tcgen05", "tcgen05_split"):
        impl = "tcgen05"
    _count()
    if impl in _ATTN_VARIANT:
        lib().attention_sm100(q, k, v, o, B, Tq, Tk, H, Dh, float(scale), lse, err_word(q.device), cls_probs,
                              Hkv, causal, q_pos, block_table, _ATTN_VARIANT[impl], q_lo)
    else:
        lib().attention(q, k, v, o, B, Tq, Tk, H, Dh, float(scale), lse)
    return o


def patch_im2col(img: torch.Tensor, patch: int, out: torch.Tensor,
                 mean: Sequence[float] = IMAGENET_MEAN, std: Sequence[float] = IMAGENET_STD,
                 perm: Optional[torch.Tensor] = None) -> torch.Tensor:
    """uint8 [B,H,W,3] -> normalised patch rows [B*P, >= 3*p*p] (pad columns untouched); row r of
    an image holds patch perm[r] (row-major patch index) when perm is given."""
    _count()
    lib().patch_im2col(img, patch, list(mean), list(std), out, perm)
    return out


def set_prefix(x: torch.Tensor, prefix: torch.Tensor, B: int, N: int) -> None:
    _count()
    lib().set_prefix(x, prefix, B, N)


def msda(value: torch.Tensor, ref: torch.Tensor, offs: torch.Tensor, logits: torch.Tensor, out: torch.Tensor,
         shapes, M: int, L: int, P: int) -> torch.Tensor:
    """Multi-scale deformable attention: value [N, S, M, Dh] bf16, ref [N, Q, L, 2] fp32,
    offs / logits bf16 rows per query (offsets [M, L, P, 2], logits [M, L*P]) -> out [N, Q, M*Dh]."""
    _count()
    lib().msda(value, ref, offs, logits, out, [int(v) for v in shapes], int(M), int(L), int(P))
    return out


def im2col_nhwc(x: torch.Tensor, kh: int, kw: int, stride: int, pad: int, out: torch.Tensor) -> torch.Tensor:
    """NHWC patches for a kh x kw convolution: out [B*Ho*Wo, >= kh*kw*C], column (ky*kw+kx)*C + c."""
    _count()
    lib().im2col_nhwc(x, kh, kw, stride, pad, out)
    return out


def resize_nhwc(x: torch.Tensor, out: torch.Tensor, align_corners: bool = False,
                add: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Bilinear resize of [B, H, W, C] bf16 into out [B, Ho, Wo, C] (+ add)."""
    _count()
    lib().resize_nhwc(x, out, bool(align_corners), add)
    return out


def row_sqdist(a: torch.Tensor, b: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out[r] = ||a[r] - b[r]||^2 (fp32)."""
    _count()
    lib().row_sqdist(a, b, out)
    return out


def gather_rows(src: torch.Tensor, rows: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    _count()
    lib().gather_rows(src, rows, out)
    return out


# APPCORR_DEBUG_CHECKS=1: host-side index checks after the kernels that assume them (each one
# synchronises with the device; skipped while a CUDA graph is being captured)
DEBUG_CHECKS = os.environ.get("APPCORR_DEBUG_CHECKS", "0") == "1"


def check_unique_rows(rows: torch.Tensor, what: str) -> None:
    """Raise if the non-negative entries of `rows` repeat: a scatter to repeated destination rows
    races (which writer wins is undefined)."""
    r = rows.reshape(-1)
    r = r[r >= 0]
    n_unique = torch.unique(r).numel()
    if n_unique != r.numel():
        raise RuntimeError(f"{what}: {r.numel() - n_unique} repeated destination rows")


def _debug_checks_on() -> bool:
    return DEBUG_CHECKS and not torch.cuda.is_current_stream_capturing()


def scatter_rows(src: torch.Tensor, rows: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
    if _debug_checks_on():
        check_unique_rows(rows, "scatter_rows")
    _count()
    lib().scatter_rows(src, rows, dst)
    return dst


def cls_attn_pscore(q: torch.Tensor, k: torch.Tensor, *, B: int, N: int, H: int, Dh: int,
                    scratch: torch.Tensor, out: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
    if scale is None:
        scale = Dh ** -0.5
    _count(2)
    lib().cls_attn_pscore(q, k, B, N, H, Dh, float(scale), scratch, out)
    return out


def query_attn_pscore(qb: torch.Tensor, k: torch.Tensor, *, B: int, N: int, H: int, Dh: int,
                      scratch: torch.Tensor, out: torch.Tensor, scale: Optional[float] = None) -> torch.Tensor:
    """Softmax over keys of ONE query per image, averaged over heads: qb bf16 [B, H*Dh]
    (e.g. the pseudo queries), k [B*N, H*Dh] rows -> out fp32 [B, N]."""
    if scale is None:
        scale = Dh ** -0.5
    _count(2)
    lib().cls_attn_pscore(qb, k, B, N, H, Dh, float(scale), scratch, out, qb.stride(0))
    return out


def pseudo_query(q: torch.Tensor, *, B: int, N: int, npre: int, H: int, Dh: int, out: torch.Tensor) -> torch.Tensor:
    """Pseudo query per (image, head) (reference attention.py:261-268): the mean of the patch
    queries q[b*N + npre : (b+1)*N] rescaled to their mean norm -> out bf16 [B, H*Dh]."""
    _count()
    lib().pseudo_query(q, B, N, npre, H, Dh, out)
    return out


def attn_colsum_pscore(q: torch.Tensor, k: torch.Tensor, lse: torch.Tensor, *, B: int, N: int, H: int, Dh: int,
                       probs: torch.Tensor, out: Optional[torch.Tensor], scale: Optional[float] = None) -> torch.Tensor:
    """Column means of the attention probabilities (tcgen05): probs[b, h, j] = mean_i
    exp(q_i . k_j * scale - lse[b, h, i]); out[b, j] = mean_h probs[b, h, j] (patch_attn_prob,
    reference attention.py:258-260). lse: fp32 [B, H, N] from `attention(..., lse=...)`."""
    if scale is None:
        scale = Dh ** -0.5
    _count(1 if out is None else 2)
    lib().attn_colsum_pscore(q, k, lse, B, N, H, Dh, float(scale), probs, out, err_word(q.device))
    return probs


def head_mean(probs: torch.Tensor, B: int, H: int, N: int, out: torch.Tensor) -> torch.Tensor:
    """out[b, j] = mean over heads of probs[b, h, j]."""
    _count()
    lib().head_mean(probs, B, H, N, out)
    return out


FUSION = {"add": 0, "multiply": 1, "geo_mean": 2}


def correction_plan(server: torch.Tensor, pre: torch.Tensor, cand: torch.Tensor, k: int, upd: torch.Tensor,
                    rows: torch.Tensor, *, mobile: Optional[torch.Tensor] = None, ws: float = 1.0,
                    wm: float = 0.0, fusion: str = "add", valid: Optional[torch.Tensor] = None,
                    stats: Optional[torch.Tensor] = None, thres: Optional[float] = None,
                    counts: Optional[torch.Tensor] = None) -> None:
    """Packed correction plan per image, on the device with no host synchronisation.

    Top-k (thres None): the k highest combined scores, in ascending candidate order after the
    prefix tokens. Threshold: candidates scoring >= thres; the first k of them (k is the cap) in
    candidate order, short rows padded with their last kept candidate; counts[b] (int32)
    receives the number of candidates that passed the threshold."""
    _count()
    lib().correction_plan(server, pre, cand, mobile, float(ws), float(wm), FUSION.get(fusion, 0), valid, int(k),
                          upd, rows, stats, None if thres is None else float(thres), counts)
    if thres is None and valid is None and _debug_checks_on():  # top-k rows feed row scatters
        check_unique_rows(rows, "correction_plan")


def token_prune(x: torch.Tensor, x_ref: torch.Tensor, N: int, dindice: torch.Tensor, npre: int, threshold: float,
                min_keep: int):
    """Token-prune select + compact (reference triton_kernels/token_prune.py:9-89): per image,
    score = mean |x - x_ref| over channels of the tokens dindice[b] (rows b*N + dindice); keep
    the prefix, the patches scoring >= threshold, or the min_keep best patches when fewer pass.
    Returns (dindice_sel [B, M], query_pos [B, M], valid [B, M] bool, kept_count [B])."""
    B, M = dindice.shape
    dsel = torch.empty(B, M, device=x.device, dtype=torch.int32)
    qpos = torch.empty_like(dsel)
    valid = torch.empty(B, M, device=x.device, dtype=torch.bool)
    count = torch.empty(B, device=x.device, dtype=torch.int32)
    _count()
    lib().token_prune(x, x_ref, N, dindice, npre, float(threshold), int(min_keep), dsel, qpos, valid, count)
    return dsel, qpos, valid, count


def pyrup_add(src: torch.Tensor, res: Optional[torch.Tensor], out: torch.Tensor) -> torch.Tensor:
    _count()
    lib().pyrup_add(src, res, out)
    return out


def upsample_argmax(logits: torch.Tensor, C: int, H: int, W: int, out: torch.Tensor) -> torch.Tensor:
    _count()
    lib().upsample_argmax(logits, C, H, W, out)
    return out


def mean_rows(x: torch.Tensor, B: int, N: int, start: int, out: torch.Tensor) -> torch.Tensor:
    _count()
    lib().mean_rows(x, B, N, start, out)
    return out
