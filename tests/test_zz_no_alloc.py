"""The allocation-free C entry point, called through its exported symbol.

`appcorr_cls_attn_pscore_noalloc` is for callers that cannot allocate device memory themselves
(code inside a custom allocator or memory-pool callback, runtimes that reserve all device memory
up front, plain-C hosts without PyTorch's allocator). It keeps its scratch in a fixed array inside
the library. This checks it against the regular `cls_attn_pscore` op on two consecutive calls and
checks that an oversized problem is refused. The file name makes pytest collect it last.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _entry():
    from appcorr_b200.ops.native import lib

    so = ctypes.CDLL(lib().__file__)
    fn = so.appcorr_cls_attn_pscore_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_long, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                   ctypes.c_int, ctypes.c_float, ctypes.c_void_p, ctypes.c_void_p]
    err = so.appcorr_noalloc_last_error
    err.restype = ctypes.c_char_p
    return fn, err


@pytest.mark.parametrize("B,N,H,Dh", [(3, 69, 4, 64), (8, 1029, 32, 128)])
def test_noalloc_matches_regular_op_twice(B, N, H, Dh):
    from appcorr_b200.ops import kernels as K

    fn, err = _entry()
    torch.manual_seed(0)
    stream = torch.cuda.current_stream()
    for call in range(2):
        q = torch.randn(B * N, H * Dh, device="cuda").to(torch.bfloat16)
        k = torch.randn(B * N, H * Dh, device="cuda").to(torch.bfloat16)
        scale = Dh ** -0.5
        ref = torch.empty(B, N, device="cuda")
        scratch = torch.empty(B, H, N, device="cuda")
        K.cls_attn_pscore(q, k, B=B, N=N, H=H, Dh=Dh, scratch=scratch, out=ref, scale=scale)
        out = torch.full((B, N), float("nan"), device="cuda")
        rc = fn(q.data_ptr(), k.data_ptr(), q.stride(0), B, N, H, Dh, scale, out.data_ptr(), stream.cuda_stream)
        assert rc == 0, err()
        torch.cuda.synchronize()
        assert torch.allclose(out, ref, rtol=1e-3, atol=1e-4), f"call {call}: max err {(out - ref).abs().max()}"


def test_noalloc_rejects_oversized_problem():
    fn, err = _entry()
    q = torch.zeros(16, 64, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(16, device="cuda")
    # B*H*N = 64 * 64 * 512 > 1 << 20 (row stride H*head_dim = 4096): refused before any launch
    rc = fn(q.data_ptr(), q.data_ptr(), 64 * 64, 64, 512, 64, 64, 0.125, out.data_ptr(), None)
    assert rc == 1
    assert b"exceeds" in err()


def test_noalloc_large_smem_after_regular_op():
    """A regular call that sets the kernel's shared-memory limit to ~60 KB, then an entry-point call
    that needs ~160 KB: the entry point raises the limit itself on every call that needs it."""
    from appcorr_b200.ops import kernels as K

    fn, err = _entry()
    torch.manual_seed(1)
    H, Dh = 8, 64
    q = torch.randn(15000, H * Dh, device="cuda").to(torch.bfloat16)
    ref = torch.empty(1, 15000, device="cuda")
    K.cls_attn_pscore(q, q, B=1, N=15000, H=H, Dh=Dh, scratch=torch.empty(1, H, 15000, device="cuda"), out=ref)
    N = 40000
    q = torch.randn(N, H * Dh, device="cuda").to(torch.bfloat16)
    k = torch.randn(N, H * Dh, device="cuda").to(torch.bfloat16)
    ref = torch.empty(1, N, device="cuda")
    K.cls_attn_pscore(q, k, B=1, N=N, H=H, Dh=Dh, scratch=torch.empty(1, H, N, device="cuda"), out=ref,
                      scale=Dh ** -0.5)
    for _ in range(2):
        out = torch.full((1, N), float("nan"), device="cuda")
        rc = fn(q.data_ptr(), k.data_ptr(), q.stride(0), 1, N, H, Dh, Dh ** -0.5, out.data_ptr(),
                torch.cuda.current_stream().cuda_stream)
        assert rc == 0, err()
        torch.cuda.synchronize()
        assert torch.allclose(out, ref, rtol=1e-3, atol=1e-6)


def test_noalloc_rejects_misaligned_operands():
    """Checked on the host: nothing is launched for a refused call."""
    fn, err = _entry()
    q = torch.zeros(8, 128, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(8, device="cuda")
    base = q.data_ptr()
    assert fn(base + 2, base, 128, 1, 8, 2, 64, 0.125, out.data_ptr(), None) == 2   # q 2-byte aligned
    assert b"aligned" in err()
    assert fn(base, base + 2, 128, 1, 8, 2, 64, 0.125, out.data_ptr(), None) == 2   # k 2-byte aligned
    assert fn(base, base, 129, 1, 8, 2, 64, 0.125, out.data_ptr(), None) == 2       # odd row stride
