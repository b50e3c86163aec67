// Server patch scores that need more than the CLS row, on the 5th-generation tensor cores.
//
//   patch_attn_prob      score[b, j] = mean_h mean_i softmax_j(q_i . k_j * scale)
//                        (reference appcorr/models/dinov3/layers/attention.py:258-260 and its
//                        fused kernel triton_kernels/attention_pscore.py:21-98: the column sums
//                        of the normalised attention probabilities)
//   patch_pseudo_attn_prob
//                        one pseudo query per (image, head): the mean of the patch queries,
//                        rescaled to the mean patch-query norm, then a softmax over keys
//                        (attention.py:261-269)
//
// Column sums. The row log-sum-exp of every query comes from the attention pass that runs anyway
// (attention_sm100 writes `lse`), so one more Q K^T pass gives normalised probabilities without
// a second softmax. The kernel computes S^T = K Q^T with the KEYS on the 128 TMEM lanes:
//   one CTA = 128 keys of one (image, head); 6 warps
//   warp 0      TMA: the K tile once, Q tiles of 128 queries into a 2-stage ring
//   warp 1      MMA (one thread): S^T_j = K Q_j^T into one of two TMEM buffers (128 columns each)
//   warps 2..5  one key per thread: tcgen05.ld of its row of S^T_j (128 queries), stage the 128
//               queries' log2-LSE in shared memory, accumulate exp2(s * scale*log2e - lse2) in
//               registers. A thread owns a whole column of P, so the column sum needs no
//               cross-thread reduction; it writes colsum / N to probs[b, h, key].
// A head-mean pass turns probs [B, H, N] into the score [B, N]. All waits are bounded.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cfloat>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;

constexpr int kCsBM = 128;       // keys per CTA (TMEM lanes)
constexpr int kCsBN = 128;       // queries per block (TMEM columns)
constexpr int kCsThreads = 192;

__global__ void head_mean_kernel(const float* probs, int B, int H, int N, float* out);

template <int DH>
__global__ void __launch_bounds__(kCsThreads, 1)
    attn_colsum_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                             const float* __restrict__ lse, int N, int H, float scale_log2, float* __restrict__ probs,
                             int* err) {
  constexpr int NCH = DH / 64;
  constexpr uint32_t CHUNK_BYTES = 128 * 128;          // [128 rows x 64 cols] bf16 box
  constexpr uint32_t TILE_BYTES = NCH * CHUNK_BYTES;
  constexpr uint32_t IDESC = idesc_bf16_f32(kCsBM, kCsBN);
  constexpr uint32_t TMEM_COLS = 2 * kCsBN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sQ = sK + TILE_BYTES;                                  // 2 stages
  float* sL = reinterpret_cast<float*>(sQ + 2 * TILE_BYTES);      // 2 x 128 log2-LSE
  uint64_t* bars = reinterpret_cast<uint64_t*>(sL + 2 * kCsBN);
  uint64_t* k_full = bars;         // 1
  uint64_t* q_full = bars + 1;     // 2
  uint64_t* q_empty = bars + 3;    // 2
  uint64_t* s_full = bars + 5;     // 2
  uint64_t* s_free = bars + 7;     // 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 9);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int k0 = kt * kCsBM;
  const int nqb = (N + kCsBN - 1) / kCsBN;

  if (warp == 0 && lane == 0) {
    mbar_init(smem_addr(k_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&q_full[i]), 1);
      mbar_init(smem_addr(&q_empty[i]), 1);
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&s_free[i]), 128);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
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
      const uint32_t kb = smem_addr(k_full);
      mbar_arrive_expect_tx(kb, TILE_BYTES);
      for (int c = 0; c < NCH; ++c) tma_load_2d(smem_addr(sK + c * CHUNK_BYTES), &tmK, kb, h * DH + c * 64, b * N + k0);
      for (int j = 0; j < nqb; ++j) {
        const int s = j & 1;
        if (!mbar_wait(smem_addr(&q_empty[s]), ((j >> 1) & 1) ^ 1, err, kErrTimeoutProducer)) break;
        const uint32_t fb = smem_addr(&q_full[s]);
        mbar_arrive_expect_tx(fb, TILE_BYTES);
        for (int c = 0; c < NCH; ++c)
          tma_load_2d(smem_addr(sQ + s * TILE_BYTES + c * CHUNK_BYTES), &tmQ, fb, h * DH + c * 64, b * N + j * kCsBN);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(smem_addr(k_full), 0, err, kErrTimeoutMma);
      const uint32_t ka = smem_addr(sK);
      for (int j = 0; ok && j < nqb; ++j) {
        const int s = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(smem_addr(&q_full[s]), ph, err, kErrTimeoutMma)) break;
        if (!mbar_wait(smem_addr(&s_free[s]), ph ^ 1, err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t qa = smem_addr(sQ + s * TILE_BYTES);
#pragma unroll
        for (int k = 0; k < DH / 16; ++k) {
          const uint32_t off = (k >> 2) * CHUNK_BYTES + (k & 3) * 32;
          umma_f16(tmem + s * kCsBN, sw128_kmajor_desc(ka + off), sw128_kmajor_desc(qa + off), IDESC, k > 0);
        }
        umma_commit(smem_addr(&s_full[s]));
        umma_commit(smem_addr(&q_empty[s]));
      }
    }
  } else {
    const int et = threadIdx.x - 64;              // 0..127 among the four epilogue warps
    const int qd = warp & 3;                      // TMEM lane quadrant of this warp
    const int row = qd * 32 + lane;               // key row inside the tile
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const float* lse_bh = lse + ((long)b * H + h) * N;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    bool ok = true;
    // Every epilogue thread runs all nqb iterations (the named barrier counts on it); after a
    // timed-out wait a thread only keeps meeting the barrier.
    for (int j = 0; j < nqb; ++j) {
      const int s = j & 1;
      // stage this query block's log2-LSE (queries past N get +inf: probability 0)
      const int qi = j * kCsBN + et;
      sL[s * kCsBN + et] = qi < N ? lse_bh[qi] * 1.4426950408889634f : INFINITY;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (ok) ok = mbar_wait(smem_addr(&s_full[s]), (j >> 1) & 1, err, kErrTimeoutEpilogue);
      if (!__all_sync(0xffffffffu, ok)) ok = false;  // tcgen05.ld is warp-collective
      if (!ok) continue;
      tc_fence_after();
      const float* L = sL + s * kCsBN;
#pragma unroll
      for (int c = 0; c < kCsBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + s * kCsBN + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          float y;
          asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(fmaf(__uint_as_float(r[t]), scale_log2, -L[c * 32 + t])));
          acc[t & 3] += y;
        }
      }
      tc_fence_before();
      mbar_arrive(smem_addr(&s_free[s]));
    }
    const int key = k0 + row;
    if (ok && key < N) probs[((long)b * H + h) * N + key] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) / N;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// q, k: [B*N, >= H*Dh] bf16 rows (same layout as the attention inputs); lse: fp32 [B, H, N]
// natural-log row LSE of softmax(q k^T * scale) (attention_sm100's `lse`). probs: fp32 [B, H, N]
// receives the per-head column means; out: fp32 [B, N] their head mean (nullptr: skipped).
void attn_colsum_pscore_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& lse, int64_t B, int64_t N,
                           int64_t H, int64_t Dh, double scale, at::Tensor& probs, c10::optional<at::Tensor> out,
                           const at::Tensor& err) {
  for (const at::Tensor* t : {&q, &k}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kBFloat16 && t->stride(-1) == 1, "attn_colsum: bf16 CUDA q/k");
    TORCH_CHECK(t->stride(-2) % 8 == 0 && (reinterpret_cast<uintptr_t>(t->data_ptr()) & 15) == 0,
                "attn_colsum: 16B-aligned rows");
    TORCH_CHECK(t->dim() == 2 && t->size(0) >= B * N && t->size(1) >= H * Dh, "attn_colsum: q/k [>= B*N, >= H*Dh]");
  }
  TORCH_CHECK(Dh == 64 || Dh == 128, "attn_colsum: head_dim 64 or 128");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.numel() >= B * H * N,
              "attn_colsum: lse fp32 [B,H,N]");
  TORCH_CHECK(probs.scalar_type() == at::kFloat && probs.is_contiguous() && probs.numel() >= B * H * N,
              "attn_colsum: probs fp32 [B,H,N]");
  if (B * N * H == 0) return;
  c10::cuda::CUDAGuard g(q.device());
  CUtensorMap tq = make_tmap_bf16_2d(q.data_ptr(), B * N, H * Dh, q.stride(-2), kCsBN, 64);
  CUtensorMap tk = make_tmap_bf16_2d(k.data_ptr(), B * N, H * Dh, k.stride(-2), kCsBM, 64);
  const float sl2 = static_cast<float>(scale * 1.4426950408889634);
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 grid((N + kCsBM - 1) / kCsBM, H, B);
  const int nch = static_cast<int>(Dh / 64);
  const int smem = nch * 16384 * 3 + 2 * kCsBN * 4 + 1024 + 256;
  if (Dh == 128) {
    cudaFuncSetAttribute(attn_colsum_sm100_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_colsum_sm100_kernel<128><<<grid, kCsThreads, smem, st>>>(tq, tk, lse.data_ptr<float>(), (int)N, (int)H, sl2,
                                                                  probs.data_ptr<float>(), err.data_ptr<int>());
  } else {
    cudaFuncSetAttribute(attn_colsum_sm100_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    attn_colsum_sm100_kernel<64><<<grid, kCsThreads, smem, st>>>(tq, tk, lse.data_ptr<float>(), (int)N, (int)H, sl2,
                                                                 probs.data_ptr<float>(), err.data_ptr<int>());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  if (out.has_value()) {
    TORCH_CHECK(out->scalar_type() == at::kFloat && out->is_contiguous() && out->numel() == B * N,
                "attn_colsum: out fp32 [B,N]");
    head_mean_kernel<<<static_cast<int>(std::max<long>(1, (B * N + 255) / 256)), 256, 0, st>>>(
        probs.data_ptr<float>(), (int)B, (int)H, (int)N, out->data_ptr<float>());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// ------------------------------------------------------------------------------ pseudo query
// grid (B, H), 128 threads. q_pseudo[b, h*Dh + d] = qm[d] * (mean_i |q_i| / max(|qm|, eps)),
// qm = mean over the patch queries i in [npre, N) of q_i (head h). Rounded to bf16 (the query
// operand of the probability pass).
constexpr int kPqThreads = 128;

__global__ void __launch_bounds__(kPqThreads) pseudo_query_kernel(const bf16* __restrict__ q, long ld, int N, int npre,
                                                                  int H, int Dh, bf16* __restrict__ out) {
  extern __shared__ float s_pq[];  // [Dh] column sums, then reductions
  __shared__ float red[kPqThreads / 32];
  const int b = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int d = threadIdx.x; d < Dh; d += kPqThreads) s_pq[d] = 0.f;
  __syncthreads();
  // one warp per query row; lanes hold 4 consecutive dims each (Dh <= 128)
  float colsum[4] = {0.f, 0.f, 0.f, 0.f};
  float norm_sum = 0.f;
  const int d0 = lane * 4;
  for (int i = npre + warp; i < N; i += kPqThreads / 32) {
    const bf16* row = q + ((long)b * N + i) * ld + (long)h * Dh;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    if (d0 < Dh) {
      const uint2 u = *reinterpret_cast<const uint2*>(row + d0);
      const float2 a = unpack_bf16x2(u.x), c = unpack_bf16x2(u.y);
      v[0] = a.x; v[1] = a.y; v[2] = c.x; v[3] = c.y;
    }
    float ss = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    norm_sum += sqrtf(ss);
#pragma unroll
    for (int t = 0; t < 4; ++t) colsum[t] += v[t];
  }
  if (d0 < Dh) {
#pragma unroll
    for (int t = 0; t < 4; ++t) atomicAdd(&s_pq[d0 + t], colsum[t]);
  }
  if (lane == 0) red[warp] = norm_sum;
  __syncthreads();
  const int P = N - npre;
  __shared__ float s_ratio;
  if (threadIdx.x < 32) {
    float qq = 0.f;
    for (int d = lane; d < Dh; d += 32) {
      const float m = s_pq[d] / P;
      qq += m * m;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qq += __shfl_xor_sync(0xffffffffu, qq, o);
    if (lane == 0) {
      float ns = 0.f;
      for (int w = 0; w < kPqThreads / 32; ++w) ns += red[w];
      const float target = ns / P;
      s_ratio = target / fmaxf(sqrtf(qq), FLT_EPSILON);
    }
  }
  __syncthreads();
  for (int d = threadIdx.x; d < Dh; d += kPqThreads)
    out[(long)b * H * Dh + (long)h * Dh + d] = __float2bfloat16(s_pq[d] / P * s_ratio);
}

void pseudo_query_op(const at::Tensor& q, int64_t B, int64_t N, int64_t npre, int64_t H, int64_t Dh, at::Tensor& out) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == at::kBFloat16 && q.stride(-1) == 1 && q.stride(-2) % 4 == 0 &&
                  (reinterpret_cast<uintptr_t>(q.data_ptr()) & 7) == 0,
              "pseudo_query: bf16 q rows, 8-byte aligned, row stride a multiple of 4");
  TORCH_CHECK(Dh <= 128 && Dh % 4 == 0, "pseudo_query: head_dim <= 128, multiple of 4");
  TORCH_CHECK(N > npre, "pseudo_query: no patch queries");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() >= B * H * Dh,
              "pseudo_query: out bf16 [B, H*Dh]");
  c10::cuda::CUDAGuard g(q.device());
  pseudo_query_kernel<<<dim3(B, H), kPqThreads, Dh * sizeof(float), at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(q.data_ptr()), q.stride(-2), (int)N, (int)npre, (int)H, (int)Dh,
      reinterpret_cast<bf16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_pscore_sm100_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("attn_colsum_pscore", &attn_colsum_pscore_op, py::arg("q"), py::arg("k"), py::arg("lse"), py::arg("B"),
        py::arg("N"), py::arg("H"), py::arg("Dh"), py::arg("scale"), py::arg("probs"), py::arg("out"), py::arg("err"));
  m.def("pseudo_query", &pseudo_query_op);
}

}  // namespace appcorr
