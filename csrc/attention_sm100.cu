// Flash-attention forward on the 5th-generation tensor cores (tcgen05 + TMEM + TMA), bf16,
// head dim 64 or 128, non-causal, BTHD layout (see attention.cu for the layout contract).
//
// One CTA = 128 query rows of one (batch, head); 6 warps:
//   warp 0      TMA: Q once; K and V tiles of 128 keys into a 2-stage ring (128-byte swizzle)
//   warp 1      MMA (one thread): S_j = Q K_j^T into one of two TMEM S buffers, and
//               O += P_j V_j into a TMEM O accumulator. S_{j+1} is issued before PV_j so the
//               tensor core works on the next scores while the softmax warps handle the current
//               ones. V is consumed as an MN-major operand straight from its TMA tile.
//   warps 2..5  softmax, one query row per thread: tcgen05.ld of the S row, running max / sum in
//               base 2, P (bf16) written to shared memory in the K-major swizzled layout the MMA
//               reads. O is rescaled in TMEM only when a row's running max grows by more than
//               2^8 (otherwise the stale max is kept; the final 1/l normalisation is exact either
//               way). Finally O is read from TMEM, divided by l and stored.
// All waits are bounded (error word, no hang).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cfloat>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;

constexpr int kFaBM = 128;   // query rows per CTA
constexpr int kFaBN = 128;   // keys per block
constexpr int kFaThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

// Shared-memory descriptor for an MN-major operand tile with the 128-byte swizzle: 8 K-rows of
// 128 B (64 MN elements) per atom, atoms along K `sbo` bytes apart, along MN `lbo` bytes apart.
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_byte_addr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_byte_addr >> 4) & 0x3FFF);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// kind::f16 instruction descriptor, bf16 inputs, fp32 accumulate, A K-major, B MN-major if b_mn.
__host__ __device__ constexpr uint32_t idesc_bf16_f32_b(int M, int N, bool b_mn) {
  return idesc_bf16_f32(M, N) | (b_mn ? (1u << 16) : 0u);
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

struct FaParams {
  int B, Tq, Tk, H;
  float scale_log2;
  bf16* o;
  long ldo;
  float* lse;      // [B, H, Tq] natural-log LSE or nullptr
  float* cls;      // [B, H, Tk] softmax probabilities of query row 0 (CLS) or nullptr
  int* err;
};

template <int DH>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, FaParams p) {
  constexpr int NCH = DH / 64;                          // 64-column chunks per row
  constexpr uint32_t CHUNK_BYTES = 128 * 128;           // one [128 rows x 64 cols] bf16 box
  constexpr uint32_t Q_BYTES = NCH * CHUNK_BYTES;
  constexpr uint32_t KV_BYTES = NCH * CHUNK_BYTES;      // per K (or V) stage
  constexpr uint32_t P_BYTES = 2 * CHUNK_BYTES;         // [128 q x 128 keys]
  constexpr uint32_t IDESC_S = idesc_bf16_f32(kFaBM, kFaBN);
  constexpr uint32_t IDESC_O = idesc_bf16_f32_b(kFaBM, DH, true);
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t O_COL = 2 * kFaBN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Q_BYTES;          // 2 stages
  uint8_t* sV = sK + 2 * KV_BYTES;     // 2 stages
  uint8_t* sP = sV + 2 * KV_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + P_BYTES);
  uint64_t* q_full = bars;           // 1
  uint64_t* kv_full = bars + 1;      // 2
  uint64_t* kv_empty = bars + 3;     // 2
  uint64_t* s_full = bars + 5;       // 2
  uint64_t* s_free = bars + 7;       // 2
  uint64_t* p_full = bars + 9;       // 1
  uint64_t* p_empty = bars + 10;     // 1
  uint64_t* o_full = bars + 11;      // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 12);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kFaBM;
  const int nkb = (p.Tk + kFaBN - 1) / kFaBN;

  if (warp == 0 && lane == 0) {
    mbar_init(smem_addr(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&kv_full[i]), 1);
      mbar_init(smem_addr(&kv_empty[i]), 1);
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&s_free[i]), 128);
    }
    mbar_init(smem_addr(p_full), 128);
    mbar_init(smem_addr(p_empty), 1);
    mbar_init(smem_addr(o_full), 1);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t qb = smem_addr(q_full);
      mbar_arrive_expect_tx(qb, Q_BYTES);
      for (int c = 0; c < NCH; ++c)
        tma_load_2d(smem_addr(sQ + c * CHUNK_BYTES), &tmQ, qb, h * DH + c * 64, b * p.Tq + q0);
      for (int j = 0; j < nkb; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(smem_addr(&kv_empty[s]), ph ^ 1, p.err, kErrTimeoutProducer)) break;
        const uint32_t fb = smem_addr(&kv_full[s]);
        mbar_arrive_expect_tx(fb, 2 * KV_BYTES);
        const int row = b * p.Tk + j * kFaBN;
        for (int c = 0; c < NCH; ++c) {
          tma_load_2d(smem_addr(sK + s * KV_BYTES + c * CHUNK_BYTES), &tmK, fb, h * DH + c * 64, row);
          tma_load_2d(smem_addr(sV + s * KV_BYTES + c * CHUNK_BYTES), &tmV, fb, h * DH + c * 64, row);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(smem_addr(q_full), 0, p.err, kErrTimeoutMma);
      const uint32_t qa = smem_addr(sQ);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!mbar_wait(smem_addr(&kv_full[s]), (j >> 1) & 1, p.err, kErrTimeoutMma)) return false;
        if (!mbar_wait(smem_addr(&s_free[s]), ((j >> 1) & 1) ^ 1, p.err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t ka = smem_addr(sK + s * KV_BYTES);
#pragma unroll
        for (int k = 0; k < DH / 16; ++k) {
          const uint32_t off = (k >> 2) * CHUNK_BYTES + (k & 3) * 32;
          umma_f16(tmem + s * kFaBN, sw128_kmajor_desc(qa + off), sw128_kmajor_desc(ka + off), IDESC_S, k > 0);
        }
        umma_commit(smem_addr(&s_full[s]));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkb; ++j) {
        if (j + 1 < nkb && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(smem_addr(p_full), j & 1, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const int s = j & 1;
        const uint32_t pa = smem_addr(sP), va = smem_addr(sV + s * KV_BYTES);
#pragma unroll
        for (int k = 0; k < kFaBN / 16; ++k) {
          const uint32_t aoff = (k >> 2) * CHUNK_BYTES + (k & 3) * 32;
          umma_f16(tmem + O_COL, sw128_kmajor_desc(pa + aoff), sw128_mnmajor_desc(va + k * 2048, CHUNK_BYTES, 1024),
                   IDESC_O, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(smem_addr(p_empty));
        umma_commit(smem_addr(&kv_empty[s]));
      }
      if (ok) umma_commit(smem_addr(o_full));
    }
  } else {
    const int qd = warp & 3;                      // TMEM lane quadrant
    const int row = qd * 32 + lane;               // query row inside the tile
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    float m_run = -FLT_MAX, l_run = 0.f;
    bool ok = true;
    const bool cls_row = p.cls != nullptr && qt == 0 && row == 0;
    uint8_t* prow = sP + row * 128;
    const int rsw = row & 7;
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1;
      if (!mbar_wait(smem_addr(&s_full[s]), (j >> 1) & 1, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      float sv[kFaBN];
#pragma unroll
      for (int c = 0; c < kFaBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + s * kFaBN + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) sv[c * 32 + t] = __uint_as_float(r[t]) * p.scale_log2;
      }
      tc_fence_before();
      mbar_arrive(smem_addr(&s_free[s]));
      const int kbase = j * kFaBN;
      float mx = -FLT_MAX;
#pragma unroll
      for (int t = 0; t < kFaBN; ++t) {
        if (kbase + t >= p.Tk) sv[t] = -FLT_MAX;
        mx = fmaxf(mx, sv[t]);
      }
      if (cls_row) {  // keep the CLS row's scaled logits; normalised once the row's max / sum are final
        float* dst = p.cls + ((long)b * p.H + h) * p.Tk + kbase;
        const int n = min(kFaBN, p.Tk - kbase);
#pragma unroll
        for (int t = 0; t < kFaBN; ++t)
          if (t < n) dst[t] = sv[t];
      }
      // rescale decision (warp-uniform because tcgen05.ld/st are warp-collective)
      const bool grow = mx > m_run + kRescaleThreshold;
      const bool any_grow = __any_sync(0xffffffffu, grow) && j > 0;
      float corr = 1.f;
      if (grow || j == 0) {
        const float mnew = fmaxf(m_run, mx);
        corr = (j == 0) ? 0.f : exp2f(m_run - mnew);
        m_run = mnew;
      }
      if (j > 0) {  // P buffer and O are busy until PV_{j-1} completes
        if (!mbar_wait(smem_addr(p_empty), (j - 1) & 1, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
        tc_fence_after();
      }
      if (any_grow) {
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + O_COL + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * corr);
          tmem_st32(tmem + lane_base + O_COL + c * 32, r);
        }
        tmem_wait_st();
      }
      l_run *= (j == 0) ? 0.f : corr;
      float lsum = 0.f;
#pragma unroll
      for (int c = 0; c < kFaBN / 64; ++c) {
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          float e[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            e[t] = exp2f(sv[c * 64 + v * 8 + t] - m_run);
            lsum += e[t];
          }
          const uint4 pk = make_uint4(pack_bf16x2(e[0], e[1]), pack_bf16x2(e[2], e[3]), pack_bf16x2(e[4], e[5]),
                                      pack_bf16x2(e[6], e[7]));
          *reinterpret_cast<uint4*>(prow + c * CHUNK_BYTES + ((v ^ rsw) << 4)) = pk;
        }
      }
      l_run += lsum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_addr(p_full));
    }
    if (ok && mbar_wait(smem_addr(o_full), 0, p.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const int qrow = q0 + row;
      const float inv = 1.f / l_run;
      bf16* orow = p.o + ((long)b * p.Tq + qrow) * p.ldo + (long)h * DH;
#pragma unroll 1
      for (int c = 0; c < DH / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + O_COL + c * 32, r);
        tmem_wait_ld();
        if (qrow < p.Tq) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int v = 0; v < 4; ++v)
            dst[v] = make_uint4(pack_bf16x2(__uint_as_float(r[8 * v]) * inv, __uint_as_float(r[8 * v + 1]) * inv),
                                pack_bf16x2(__uint_as_float(r[8 * v + 2]) * inv, __uint_as_float(r[8 * v + 3]) * inv),
                                pack_bf16x2(__uint_as_float(r[8 * v + 4]) * inv, __uint_as_float(r[8 * v + 5]) * inv),
                                pack_bf16x2(__uint_as_float(r[8 * v + 6]) * inv, __uint_as_float(r[8 * v + 7]) * inv));
        }
      }
      if (p.lse != nullptr && qrow < p.Tq)
        p.lse[((long)b * p.H + h) * p.Tq + qrow] = (m_run + log2f(l_run)) * 0.69314718055994531f;
    }
    if (p.cls != nullptr && qt == 0 && qd == 0) {  // the warp holding row 0 normalises the CLS row
      __syncwarp();
      const float m0 = __shfl_sync(0xffffffffu, m_run, 0);
      const float inv0 = 1.f / __shfl_sync(0xffffffffu, l_run, 0);
      float* src = p.cls + ((long)b * p.H + h) * p.Tk;
      for (int t = lane; t < p.Tk; t += 32) src[t] = exp2f(src[t] - m0) * inv0;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

void attention_sm100_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, int64_t B,
                        int64_t Tq, int64_t Tk, int64_t H, int64_t Dh, double scale, c10::optional<at::Tensor> lse,
                        const at::Tensor& err, c10::optional<at::Tensor> cls) {
  for (const at::Tensor* t : std::initializer_list<const at::Tensor*>{&q, &k, &v, &o}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->stride(-1) == 1, "attention: bf16 CUDA tensors");
    TORCH_CHECK(t->stride(-2) % 8 == 0 && (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0, "attention: 16B-aligned rows");
  }
  TORCH_CHECK(Dh == 64 || Dh == 128, "attention: head_dim 64 or 128");
  TORCH_CHECK(Tk > 0, "attention: empty key set");
  if (B * Tq * H == 0) return;
  c10::cuda::CUDAGuard g(q.device());
  // 2-D views [rows, H*Dh] with 128-row x 64-column boxes.
  CUtensorMap tq = make_tmap_bf16_2d(q.data_ptr(), B * Tq, H * Dh, q.stride(-2), kFaBM, 64);
  CUtensorMap tk = make_tmap_bf16_2d(k.data_ptr(), B * Tk, H * Dh, k.stride(-2), kFaBN, 64);
  CUtensorMap tv = make_tmap_bf16_2d(v.data_ptr(), B * Tk, H * Dh, v.stride(-2), kFaBN, 64);
  FaParams p{static_cast<int>(B), static_cast<int>(Tq), static_cast<int>(Tk), static_cast<int>(H),
             static_cast<float>(scale * 1.4426950408889634), reinterpret_cast<bf16*>(o.data_ptr()), o.stride(-2),
             nullptr, nullptr, err.data_ptr<int>()};
  if (cls.has_value()) {
    TORCH_CHECK(cls->scalar_type() == at::kFloat && cls->is_contiguous() && cls->numel() >= B * H * Tk,
                "attention: cls fp32 [B,H,Tk]");
    p.cls = cls->data_ptr<float>();
  }
  if (lse.has_value()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() >= B * H * Tq, "attention: lse fp32 [B,H,Tq]");
    p.lse = lse->data_ptr<float>();
  }
  dim3 grid((Tq + kFaBM - 1) / kFaBM, H, B);
  auto st = at::cuda::getCurrentCUDAStream();
  const int nch = static_cast<int>(Dh / 64);
  const int smem = nch * 16384 * 5 + 2 * 16384 + 1024 + 256;
  if (Dh == 128) {
    cudaFuncSetAttribute(fa_fwd_sm100_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    fa_fwd_sm100_kernel<128><<<grid, kFaThreads, smem, st>>>(tq, tk, tv, p);
  } else {
    cudaFuncSetAttribute(fa_fwd_sm100_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    fa_fwd_sm100_kernel<64><<<grid, kFaThreads, smem, st>>>(tq, tk, tv, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_attention_sm100_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("attention_sm100", &attention_sm100_op, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("B"),
        py::arg("Tq"), py::arg("Tk"), py::arg("H"), py::arg("Dh"), py::arg("scale"), py::arg("lse"), py::arg("err"),
        py::arg("cls") = py::none());
}

}  // namespace appcorr
