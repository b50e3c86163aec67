"""Integer Gaussian-pyramid primitives, bit-exact with OpenCV's pyrDown / pyrUp on uint8.

The Laplacian codecs (reference offload/policies/transmission/laplacian.py:89-120,234-262) use a
closed loop: each residual is taken against the *decoder's own* upsample of the reconstructed
coarser level, so encode -> decode is lossless only if both ends compute pyrUp identically. The
server decodes with the CUDA kernel `pyrup_add` (csrc/elementwise.cu); this module is the numpy
statement of the same integer rule, used by the CPU decoder and as the kernel's test oracle, and is
checked against cv2 in the CPU tests.

pyrUp, per axis on source samples s[0..n): even output 2i = s[i-1] + 6 s[i] + s[i+1]; odd output
2i+1 = 4 s[i] + 4 s[i+1]; s[-1] mirrors to s[1]; the last sample gives s[n-2] + 7 s[n-1] (even)
and 8 s[n-1] (odd). The two passes' product is divided by 64 with rounding: (sum + 32) >> 6.
"""
from __future__ import annotations

import numpy as np

try:  # cv2 is the fast path where installed; the integer rule below is the definition.
    import cv2  # type: ignore
except Exception:  # pragma: no cover
    cv2 = None


def _up_axis(a: np.ndarray, axis: int) -> np.ndarray:
    n = a.shape[axis]
    idx = np.arange(n)
    prev = np.where(idx - 1 < 0, min(1, n - 1), idx - 1)
    nxt = np.where(idx + 1 >= n, max(n - 2, 0), idx + 1)
    A = np.take(a, idx, axis)
    P = np.take(a, prev, axis)
    Nx = np.take(a, nxt, axis)
    even = P + 6 * A + Nx
    odd = 4 * A + 4 * Nx
    last = [slice(None)] * a.ndim
    last[axis] = n - 1
    last = tuple(last)
    even[last] = P[last] + 7 * A[last]
    odd[last] = 8 * A[last]
    out = np.stack([even, odd], axis=axis + 1)
    shape = list(a.shape)
    shape[axis] = 2 * n
    return out.reshape(shape)


def pyr_up_int(src: np.ndarray) -> np.ndarray:
    s = src.astype(np.int64)
    r = _up_axis(_up_axis(s, 0), 1)
    return ((r + 32) >> 6).clip(0, 255).astype(np.uint8)


def pyr_up(src: np.ndarray, use_cv2: bool = True) -> np.ndarray:
    """uint8 HxW(xC) -> 2Hx2W(xC), identical to cv2.pyrUp."""
    if use_cv2 and cv2 is not None:
        out = cv2.pyrUp(src)
        if out.ndim == 2 and src.ndim == 3:
            out = out[..., None]
        return out
    return pyr_up_int(src)


def _down_axis(a: np.ndarray, axis: int, out_n: int) -> np.ndarray:
    # 5-tap [1 4 6 4 1] at even positions with reflect-101 borders.
    n = a.shape[axis]

    def refl(i):
        i = np.where(i < 0, -i, i)
        return np.where(i >= n, 2 * (n - 1) - i, i)

    c = 2 * np.arange(out_n)
    taps = [refl(c - 2), refl(c - 1), c.clip(0, n - 1), refl(c + 1), refl(c + 2)]
    w = [1, 4, 6, 4, 1]
    acc = sum(wk * np.take(a, t, axis) for wk, t in zip(w, taps))
    return acc


def pyr_down_int(src: np.ndarray) -> np.ndarray:
    h, w = src.shape[:2]
    oh, ow = (h + 1) // 2, (w + 1) // 2
    s = src.astype(np.int64)
    r = _down_axis(_down_axis(s, 0, oh), 1, ow)
    return ((r + 128) >> 8).clip(0, 255).astype(np.uint8)


def pyr_down(src: np.ndarray, use_cv2: bool = True) -> np.ndarray:
    if use_cv2 and cv2 is not None:
        out = cv2.pyrDown(src)
        if out.ndim == 2 and src.ndim == 3:
            out = out[..., None]
        return out
    return pyr_down_int(src)
