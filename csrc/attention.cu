// Flash-attention forward for the approx and correction passes (bf16, head dim 64 or 128).
//
// Replaces cuDNN SDPA in the reference (attention.py:242,276 approx over all tokens; :502 the
// correction pass, packed queries of the selected rows against the full cached K/V whose selected
// rows were just rewritten). Layout is BTHD throughout: row (b, t) of Q / K / V / O holds all
// heads contiguously, so the QKV GEMM epilogue writes straight into it and the output feeds the
// proj GEMM without a transpose.
//
// One CTA = 64 query rows of one (batch, head), 4 warps x 16 rows. K/V tiles of 64 keys are
// double-buffered in XOR-swizzled shared memory with cp.async; S = QK^T and O += PV use
// mma.sync m16n8k16 (bf16 in, fp32 accumulate), softmax is the online (running max / sum) form
// in base 2. Optionally writes the natural-log LSE per (b, h, query) for score passes.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cfloat>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;

constexpr int kAttnBM = 64;
constexpr int kAttnBN = 64;
constexpr int kAttnThreads = 128;

__device__ __forceinline__ uint32_t swz(int row, int chunk, int row_bytes) {
  return row * row_bytes + ((chunk ^ (row & 7)) << 4);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

struct AttnParams {
  const bf16* q; const bf16* k; const bf16* v; bf16* o;
  long ldq, ldk, ldv, ldo;     // row strides (elements)
  int Tq, Tk, H;
  float scale_log2;            // softmax scale * log2(e)
  float* lse;                  // [B, H, Tq] natural-log LSE or nullptr
};

template <int DH>
__global__ void __launch_bounds__(kAttnThreads) attn_fwd_kernel(AttnParams p) {
  constexpr int RB = DH * 2;          // bytes per smem row
  constexpr int CH = DH / 8;          // 16-byte chunks per row
  constexpr int KT = DH / 16;         // k-chunks of the QK^T product
  constexpr int NT = kAttnBN / 8;     // n-tiles of S per warp
  constexpr int DT = DH / 8;          // n-tiles of O per warp
  extern __shared__ __align__(128) uint8_t sm[];
  uint8_t* sQ = sm;
  uint8_t* sK = sQ + kAttnBM * RB;
  uint8_t* sV = sK + 2 * kAttnBN * RB;

  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int q0 = qb * kAttnBM;
  const bf16* qbase = p.q + (long)b * p.Tq * p.ldq + (long)h * DH;
  const bf16* kbase = p.k + (long)b * p.Tk * p.ldk + (long)h * DH;
  const bf16* vbase = p.v + (long)b * p.Tk * p.ldv + (long)h * DH;

  // Q tile -> smem
  for (int i = tid; i < kAttnBM * CH; i += kAttnThreads) {
    const int r = i / CH, c = i - (i / CH) * CH;
    const int qr = min(q0 + r, p.Tq - 1);
    cp_async16(smem_addr(sQ) + swz(r, c, RB), qbase + (long)qr * p.ldq + c * 8, q0 + r < p.Tq);
  }
  auto load_kv = [&](int kb, int buf) {
    const int k0 = kb * kAttnBN;
    for (int i = tid; i < kAttnBN * CH; i += kAttnThreads) {
      const int r = i / CH, c = i - (i / CH) * CH;
      const int kr = min(k0 + r, p.Tk - 1);
      const bool ok = k0 + r < p.Tk;
      cp_async16(smem_addr(sK + buf * kAttnBN * RB) + swz(r, c, RB), kbase + (long)kr * p.ldk + c * 8, ok);
      cp_async16(smem_addr(sV + buf * kAttnBN * RB) + swz(r, c, RB), vbase + (long)kr * p.ldv + c * 8, ok);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  const int nkb = (p.Tk + kAttnBN - 1) / kAttnBN;
  uint32_t qf[KT][4];
  float o[DT][4];
#pragma unroll
  for (int i = 0; i < DT; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_run[2] = {-FLT_MAX, -FLT_MAX}, l_run[2] = {0.f, 0.f};
  const int g = lane >> 2, t4 = lane & 3;

  for (int kb = 0; kb < nkb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < nkb) load_kv(kb + 1, buf ^ 1);
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int kk = 0; kk < KT; ++kk) {
        const int mi = lane >> 3;
        const int r = warp * 16 + (lane & 7) + (mi & 1) * 8;
        const int c = kk * 2 + (mi >> 1);
        ldsm_x4(smem_addr(sQ) + swz(r, c, RB), qf[kk][0], qf[kk][1], qf[kk][2], qf[kk][3]);
      }
    }
    // S = Q K^T for this warp's 16 rows x 64 keys
    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const uint32_t kaddr = smem_addr(sK + buf * kAttnBN * RB);
#pragma unroll
    for (int kk = 0; kk < KT; ++kk) {
#pragma unroll
      for (int j = 0; j < NT; j += 2) {
        const int mi = lane >> 3;
        const int r = j * 8 + (mi >> 1) * 8 + (lane & 7);
        const int c = kk * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(kaddr + swz(r, c, RB), b0, b1, b2, b3);
        mma_bf16(s[j], qf[kk], b0, b1);
        mma_bf16(s[j + 1], qf[kk], b2, b3);
      }
    }
    // mask out-of-range keys, online softmax (base 2)
    const int k0 = kb * kAttnBN;
    float mx[2] = {-FLT_MAX, -FLT_MAX};
#pragma unroll
    for (int j = 0; j < NT; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + j * 8 + 2 * t4 + (e & 1);
        float val = s[j][e] * p.scale_log2;
        if (key >= p.Tk) val = -FLT_MAX;
        s[j][e] = val;
        mx[e >> 1] = fmaxf(mx[e >> 1], val);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
      const float mnew = fmaxf(m_run[r], mx[r]);
      corr[r] = exp2f(m_run[r] - mnew);
      m_run[r] = mnew;
      l_run[r] *= corr[r];
    }
#pragma unroll
    for (int i = 0; i < DT; ++i) {
      o[i][0] *= corr[0]; o[i][1] *= corr[0];
      o[i][2] *= corr[1]; o[i][3] *= corr[1];
    }
    uint32_t pf[NT / 2][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      const float p0 = exp2f(s[j][0] - m_run[0]), p1 = exp2f(s[j][1] - m_run[0]);
      const float p2 = exp2f(s[j][2] - m_run[1]), p3 = exp2f(s[j][3] - m_run[1]);
      l_run[0] += p0 + p1;
      l_run[1] += p2 + p3;
      pf[j >> 1][(j & 1) * 2 + 0] = pack_bf16x2(p0, p1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_bf16x2(p2, p3);
    }
    // O += P V
    const uint32_t vaddr = smem_addr(sV + buf * kAttnBN * RB);
#pragma unroll
    for (int kc = 0; kc < NT / 2; ++kc) {
#pragma unroll
      for (int n = 0; n < DT; n += 2) {
        const int mi = lane >> 3;
        const int r = kc * 16 + (mi & 1) * 8 + (lane & 7);
        const int c = n + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(vaddr + swz(r, c, RB), b0, b1, b2, b3);
        mma_bf16(o[n], pf[kc], b0, b1);
        mma_bf16(o[n + 1], pf[kc], b2, b3);
      }
    }
    __syncthreads();
  }
  // finalize
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 1);
    l_run[r] += __shfl_xor_sync(0xffffffffu, l_run[r], 2);
  }
  const float inv0 = 1.f / l_run[0], inv1 = 1.f / l_run[1];
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
  bf16* obase = p.o + (long)b * p.Tq * p.ldo + (long)h * DH;
#pragma unroll
  for (int n = 0; n < DT; ++n) {
    const int col = n * 8 + 2 * t4;
    if (row0 < p.Tq)
      *reinterpret_cast<uint32_t*>(obase + (long)row0 * p.ldo + col) = pack_bf16x2(o[n][0] * inv0, o[n][1] * inv0);
    if (row1 < p.Tq)
      *reinterpret_cast<uint32_t*>(obase + (long)row1 * p.ldo + col) = pack_bf16x2(o[n][2] * inv1, o[n][3] * inv1);
  }
  if (p.lse != nullptr && t4 == 0) {
    const float ln2 = 0.69314718055994531f;
    float* lb = p.lse + ((long)b * p.H + h) * p.Tq;
    if (row0 < p.Tq) lb[row0] = (m_run[0] + log2f(l_run[0])) * ln2;
    if (row1 < p.Tq) lb[row1] = (m_run[1] + log2f(l_run[1])) * ln2;
  }
}

void attention_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, int64_t B, int64_t Tq,
                  int64_t Tk, int64_t H, int64_t Dh, double scale, c10::optional<at::Tensor> lse) {
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&q, &k, &v, &o}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->stride(-1) == 1, "attention: bf16 CUDA tensors");
    TORCH_CHECK(t->stride(-2) % 8 == 0 && (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0, "attention: 16B-aligned rows");
  }
  TORCH_CHECK(Dh == 64 || Dh == 128, "attention: head_dim 64 or 128");
  TORCH_CHECK(q.numel() >= B * Tq * H * Dh && k.numel() >= B * Tk * H * Dh && v.numel() >= B * Tk * H * Dh, "attention: sizes");
  AttnParams p;
  p.q = reinterpret_cast<const bf16*>(q.data_ptr());
  p.k = reinterpret_cast<const bf16*>(k.data_ptr());
  p.v = reinterpret_cast<const bf16*>(v.data_ptr());
  p.o = reinterpret_cast<bf16*>(o.data_ptr());
  p.ldq = q.stride(-2); p.ldk = k.stride(-2); p.ldv = v.stride(-2); p.ldo = o.stride(-2);
  p.Tq = static_cast<int>(Tq); p.Tk = static_cast<int>(Tk); p.H = static_cast<int>(H);
  p.scale_log2 = static_cast<float>(scale * 1.4426950408889634);
  p.lse = nullptr;
  if (lse.has_value()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() >= B * H * Tq, "attention: lse fp32 [B,H,Tq]");
    p.lse = lse->data_ptr<float>();
  }
  if (B * Tq * H == 0) return;
  TORCH_CHECK(Tk > 0, "attention: empty key set");
  c10::cuda::CUDAGuard g(q.device());
  dim3 grid((Tq + kAttnBM - 1) / kAttnBM, H, B);
  auto st = at::cuda::getCurrentCUDAStream();
  if (Dh == 128) {
    const int smem = (kAttnBM + 4 * kAttnBN) * 128 * 2;
    cudaFuncSetAttribute(attn_fwd_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_fwd_kernel<128><<<grid, kAttnThreads, smem, st>>>(p);
  } else {
    const int smem = (kAttnBM + 4 * kAttnBN) * 64 * 2;
    cudaFuncSetAttribute(attn_fwd_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_fwd_kernel<64><<<grid, kAttnThreads, smem, st>>>(p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_attention_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("attention", &attention_op, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("B"), py::arg("Tq"),
        py::arg("Tk"), py::arg("H"), py::arg("Dh"), py::arg("scale"), py::arg("lse") = py::none());
}

}  // namespace appcorr
