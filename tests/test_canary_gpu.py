"""Out-of-bounds write detection: every output below is a view into the middle of a larger buffer
whose guard regions (before and after, and the padding columns of strided rows) are filled with a
sentinel byte pattern; after the kernel ran on a ragged shape (rows, columns and key counts that
are not multiples of the tiles), the guards must be untouched. This is the canary half of the
race / bounds checking in this repository; the other half is the bounded-wait error word every
kernel reports through `check_errors`."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
SENTINEL = 0xA5
GUARD = 4096  # bytes before and after each output


class Guarded:
    """A [rows, cols] output of `dtype` with row stride `ld` >= cols inside a sentinel-filled buffer."""

    def __init__(self, rows: int, cols: int, dtype, ld: int = 0):
        self.rows, self.cols = rows, cols
        self.ld = ld or cols
        esz = torch.empty((), dtype=dtype).element_size()
        pad = GUARD // esz
        self.raw = torch.full((2 * GUARD + rows * self.ld * esz,), SENTINEL, device=DEV, dtype=torch.uint8)
        flat = self.raw.view(dtype)
        self.t = flat[pad:pad + rows * self.ld].view(rows, self.ld)[:, :cols]
        self.esz = esz

    def check(self, what: str):
        torch.cuda.synchronize()
        raw = self.raw
        assert bool((raw[:GUARD] == SENTINEL).all()), f"{what}: write before the output"
        assert bool((raw[-GUARD:] == SENTINEL).all()), f"{what}: write after the output"
        if self.ld > self.cols:
            body = raw[GUARD:-GUARD].view(self.rows, self.ld * self.esz)[:, self.cols * self.esz:]
            assert bool((body == SENTINEL).all()), f"{what}: write into the row padding"


def _check_errors():
    from appcorr_b200.ops.native import check_errors

    torch.cuda.synchronize()
    check_errors(torch.device(DEV))


@pytest.mark.parametrize("M,N,K,ld", [(333, 224, 256, 256), (1, 96, 64, 96), (515, 384, 320, 400)])
def test_gemm_guards(M, N, K, ld):
    from appcorr_b200.ops import kernels as K_

    torch.manual_seed(0)
    a = torch.randn(M, K, device=DEV).to(torch.bfloat16)
    w = torch.randn(N, K, device=DEV).to(torch.bfloat16)
    out = Guarded(M, N, torch.bfloat16, ld)
    K_.gemm(a, w, out.t)
    _check_errors()
    out.check("gemm bf16")
    assert torch.allclose(out.t.float(), a.float() @ w.float().t(), rtol=3e-2, atol=3e-1)
    res = torch.randn(M, N, device=DEV).to(torch.bfloat16)
    out2 = Guarded(M, N, torch.bfloat16, ld)
    K_.gemm(a, w, out2.t, epi=K_.EPI_RESID, gamma=torch.ones(N, device=DEV, dtype=torch.bfloat16), resid=res)
    out2.check("gemm residual epilogue")


def test_nvfp4_gemm_and_quant_guards():
    from appcorr_b200.ops import kernels as K_

    torch.manual_seed(1)
    M, N, Kd = 300, 256, 512
    x = torch.randn(M, Kd, device=DEV).to(torch.bfloat16)
    w = torch.randn(N, Kd, device=DEV).to(torch.bfloat16)
    q = Guarded(M, Kd // 2, torch.uint8)
    sf = Guarded(1, K_.nvfp4_sf_bytes(M, Kd), torch.uint8)
    sf.t.zero_()
    rs = Guarded(1, M, torch.float32)
    K_.quant_rows_nvfp4(x, q.t, sf.t.view(-1), rs.t.view(-1))
    _check_errors()
    for g, n in ((q, "nvfp4 rows"), (sf, "nvfp4 block scales"), (rs, "nvfp4 row scales")):
        g.check(n)
    w4, ws = K_.quantize_weight_nvfp4(w)
    out = Guarded(M, N, torch.bfloat16)
    K_.gemm(q.t.contiguous(), w4, out.t, a_scale=(rs.t.view(-1).contiguous(), sf.t.view(-1).contiguous()), b_scale=ws)
    _check_errors()
    out.check("nvfp4 gemm")


@pytest.mark.parametrize("impl", ["tcgen05", "tcgen05_split"])
def test_attention_guards(impl):
    from appcorr_b200.ops import kernels as K_

    torch.manual_seed(2)
    B, H, Dh, Tq, Tk = 2, 3, 128, 130, 261
    q = torch.randn(B * Tq, H * Dh, device=DEV).to(torch.bfloat16)
    k = torch.randn(B * Tk, H * Dh, device=DEV).to(torch.bfloat16)
    v = torch.randn(B * Tk, H * Dh, device=DEV).to(torch.bfloat16)
    # Tq != Tk is the packed-query correction shape: queries are the first Tq rows of each image
    o = Guarded(B * Tq, H * Dh, torch.bfloat16, H * Dh + 64)
    lse = Guarded(1, B * H * Tq, torch.float32)
    cls = Guarded(1, B * H * Tk, torch.float32)
    K_.attention(q, k, v, o.t, B=B, Tq=Tq, Tk=Tk, H=H, Dh=Dh, lse=lse.t.view(B, H, Tq), impl=impl,
                 cls_probs=cls.t.view(B, H, Tk))
    _check_errors()
    o.check("attention output")
    lse.check("attention lse")
    cls.check("attention CLS row")


def test_layernorm_rows_guards():
    from appcorr_b200.ops import kernels as K_

    torch.manual_seed(3)
    R, D = 77, 1024
    x = torch.randn(200, D, device=DEV).to(torch.bfloat16)
    rows = torch.randperm(200, device=DEV)[:R].to(torch.int32)
    w = torch.ones(D, device=DEV, dtype=torch.bfloat16)
    b = torch.zeros(D, device=DEV, dtype=torch.bfloat16)
    out = Guarded(R, D, torch.bfloat16)
    cp = Guarded(R, D, torch.bfloat16)
    K_.layernorm(x, w, b, 1e-6, out.t, rows=rows, copy_out=cp.t)
    _check_errors()
    out.check("layernorm")
    cp.check("layernorm copy_out")
    assert torch.equal(cp.t, x[rows.long()])


def test_msda_and_im2col_guards():
    from appcorr_b200.ops import kernels as K_

    torch.manual_seed(4)
    N, M, Dh, L, P, Q = 2, 4, 32, 2, 4, 45
    shapes = [(7, 9), (4, 5)]
    S = sum(h * w for h, w in shapes)
    value = torch.randn(N, S, M, Dh, device=DEV).to(torch.bfloat16)
    ref = torch.rand(N, Q, L, 2, device=DEV)
    offs = torch.randn(N * Q, M * L * P * 3, device=DEV).to(torch.bfloat16)
    out = Guarded(N * Q, M * Dh, torch.bfloat16)
    K_.msda(value, ref, offs, offs[:, M * L * P * 2:], out.t.view(N, Q, M * Dh), [v for hw in shapes for v in hw],
            M, L, P)
    _check_errors()
    out.check("msda")
    x = torch.randn(2, 11, 13, 16, device=DEV).to(torch.bfloat16)
    cols = Guarded(2 * 6 * 7, 9 * 16, torch.bfloat16, 160)
    K_.im2col_nhwc(x, 3, 3, 2, 1, cols.t)
    _check_errors()
    cols.check("im2col")
