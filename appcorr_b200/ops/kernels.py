"""Functional wrappers around the sm_100a kernels (one call = one or two kernel launches).

All tensors are CUDA tensors in the layouts the kernels expect (bf16 row-major activations, BTHD
attention tensors, int32 row maps). Shapes are validated in the C++ bindings.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from .native import err_word, lib

EPI_BF16, EPI_F32, EPI_GELU, EPI_SWIGLU, EPI_RESID, EPI_QKV = range(6)
AUX_NONE, AUX_SET, AUX_ADD, AUX_OUT_MINUS = range(4)

# Number of native kernel launches issued through this module (read by the benchmark).
LAUNCHES = [0]


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
         b_scale: Optional[torch.Tensor] = None, rs: Optional[tuple] = None) -> torch.Tensor:
    """out = epilogue(a @ w^T). `a` [M, K], `w` [N, K] (nn.Linear layout), both bf16 or both
    e4m3; e4m3 operands carry fp32 scales a_scale [M] (per row) and b_scale [N] (per output
    channel) that the epilogue applies to the fp32 accumulator before bias / activation.
    rs = (slot_ptrs, rows_per_rank, rank, slot_rows, ld): reduce-scatter epilogue; row m goes to
    rank (out_rows[m] or m) // rows_per_rank, slot row rank * slot_rows + m (`out` unused)."""
    fp8 = a.dtype == torch.float8_e4m3fn
    if bn is None:
        bn = 256 if epi == EPI_SWIGLU else _pick_bn(w.shape[0], a.shape[0])
        if fp8 and bn == 64:
            bn = 128
    _count()
    lib().gemm(a, w, epi, bn, err_word(a.device), out=out, out_rows=out_rows, bias=bias, gamma=gamma,
               resid=resid, resid_rows=resid_rows, aux=aux, aux_rows=aux_rows, aux_mode=aux_mode,
               resid2=resid2, max_ctas=max_ctas, a_scale=a_scale, b_scale=b_scale,
               **({} if rs is None else dict(rs_out=list(rs[0]), rs_rows_per_rank=int(rs[1]), rs_rank=int(rs[2]),
                                             rs_slot_rows=int(rs[3]), rs_ld=int(rs[4]))))
    return out


def qkv_gemm(a: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], q_out: torch.Tensor,
             k_out: torch.Tensor, v_out: torch.Tensor, *, head_dim: int, seq_len: int = 0,
             tok_idx: Optional[torch.Tensor] = None, kv_rows: Optional[torch.Tensor] = None,
             rope: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, n_prefix: int = 0,
             bn: Optional[int] = None, a_scale: Optional[torch.Tensor] = None,
             b_scale: Optional[torch.Tensor] = None, kv_dim: int = 0) -> None:
    """qkv projection with RoPE on q/k (tokens >= n_prefix) split into three BTHD buffers.

    q row m is written at q_out[m]; k/v rows at kv_rows[m] (or m). `rope` = (sin, cos) fp32
    tables [n_patch_tokens, head_dim] whose second half repeats the first (the DINOv3 angle
    layout); the kernel reads only the first half. kv_dim > 0: grouped-query weight rows
    [q (N - 2 kv_dim) | k (kv_dim) | v (kv_dim)].
    """
    dim = w.shape[0] - 2 * kv_dim if kv_dim else w.shape[0] // 3
    if bn is None:  # widest tile that divides the q and the k / v widths (tiles never straddle)
        bn = next((t for t in (256, 128, 64) if dim % t == 0 and (kv_dim or dim) % t == 0), 128)
    sin, cos = rope if rope is not None else (None, None)
    _count()
    lib().gemm(a, w, EPI_QKV, bn, err_word(a.device), bias=bias, q_out=q_out, k_out=k_out, v_out=v_out,
               kv_rows=kv_rows, tok_idx=tok_idx, seq_len=seq_len, rope_sin=sin, rope_cos=cos,
               n_prefix=n_prefix, head_dim=head_dim, a_scale=a_scale, b_scale=b_scale, kv_dim=kv_dim)


def layernorm(x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], eps: float, out: torch.Tensor,
              rows: Optional[torch.Tensor] = None, copy_out: Optional[torch.Tensor] = None,
              scale8: Optional[torch.Tensor] = None, rms: bool = False) -> torch.Tensor:
    """out[i] = LN(x[rows[i]]) (rows=None: every row). copy_out[i] receives the raw gathered row.
    An e4m3 `out` receives the bf16-rounded LN row divided by scale8[i] = amax_i / 448.
    rms=True: RMSNorm x * rsqrt(mean(x^2) + eps) * w (b must be None)."""
    _count()
    lib().layernorm(x, rows, w, b, float(eps), out, copy_out, scale8, rms)
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


def add_(x: torch.Tensor, y: torch.Tensor) -> torch.Tensor:
    _count()
    lib().add_(x, y)
    return x


# "tcgen05": one 128-row query tile per CTA, P in shared memory (default: measured faster);
# "tcgen05_2q": two query tiles per CTA sharing K/V, P kept in TMEM; "mma": the mma.sync kernel
ATTENTION_IMPL = ["tcgen05"]


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
    if q_lo is not None:
        impl = "tcgen05"
    _count()
    if impl in ("tcgen05", "tcgen05_2q"):
        lib().attention_sm100(q, k, v, o, B, Tq, Tk, H, Dh, float(scale), lse, err_word(q.device), cls_probs,
                              Hkv, causal, q_pos, block_table, 0 if impl == "tcgen05_2q" else 1, q_lo)
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


def scatter_rows(src: torch.Tensor, rows: torch.Tensor, dst: torch.Tensor) -> torch.Tensor:
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


def head_mean(probs: torch.Tensor, B: int, H: int, N: int, out: torch.Tensor) -> torch.Tensor:
    """out[b, j] = mean over heads of probs[b, h, j]."""
    _count()
    lib().head_mean(probs, B, H, N, out)
    return out


FUSION = {"add": 0, "multiply": 1, "geo_mean": 2}


def correction_plan(server: torch.Tensor, pre: torch.Tensor, cand: torch.Tensor, k: int, upd: torch.Tensor,
                    rows: torch.Tensor, *, mobile: Optional[torch.Tensor] = None, ws: float = 1.0,
                    wm: float = 0.0, fusion: str = "add", valid: Optional[torch.Tensor] = None,
                    stats: Optional[torch.Tensor] = None) -> None:
    _count()
    lib().correction_plan(server, pre, cand, mobile, float(ws), float(wm), FUSION.get(fusion, 0), valid, int(k),
                          upd, rows, stats)


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
