// Token-prune select + compact (reference appcorr/models/dinov3/layers/triton_kernels/token_prune.py:9-89,
// called from models/vision_transformer.py:453-489 before a correction segment).
//
// Per image b, over the M selected tokens dindice[b, 0..M) (prefix tokens first):
//   score_i   = mean_c |x[b*N + dindice_i, c] - x_ref[b*N + dindice_i, c]|
//   patch i (i >= npre) is kept if score_i >= threshold; if fewer than min_keep patches pass, the
//   min(min_keep, #patches) highest-scoring patches are kept instead (ties: lower position first).
//   Prefix tokens are always kept. Kept tokens are compacted in position order:
//     dindice_sel[b, j] = dindice[b, i], query_pos[b, j] = i, valid[b, j] = 1 for the j-th kept i;
//     the tail is zero; kept_count[b] = number of kept patches.
// One CTA per image: a warp per token computes its score (16-byte loads), the top-k fallback
// ranks candidates by counting (exact, deterministic), a block scan compacts.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cfloat>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;
constexpr int kTpThreads = 512;

__global__ void __launch_bounds__(kTpThreads) token_prune_kernel(
    const bf16* __restrict__ x, const bf16* __restrict__ xr, long ldx, int N, int D, const int* __restrict__ dindice,
    int M, int npre, float threshold, int min_keep, int* __restrict__ dsel, int* __restrict__ qpos,
    uint8_t* __restrict__ valid, int* __restrict__ count) {
  extern __shared__ float s_tp[];            // [M] scores, then [M] flags (int)
  float* score = s_tp;
  int* flag = reinterpret_cast<int*>(s_tp + M);
  __shared__ int s_cnt, warp_tot[kTpThreads / 32];
  const int b = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) s_cnt = 0;
  // scores: one warp per token, 8 bf16 per lane per step
  for (int i = warp; i < M; i += kTpThreads / 32) {
    const long row = (long)b * N + dindice[(long)b * M + i];
    const uint4* a = reinterpret_cast<const uint4*>(x + row * ldx);
    const uint4* r = reinterpret_cast<const uint4*>(xr + row * ldx);
    float acc = 0.f;
    for (int c = lane; c < D / 8; c += 32) {
      const uint4 u = a[c], v = r[c];
      const uint32_t* pu = &u.x;
      const uint32_t* pv = &v.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 fa = unpack_bf16x2(pu[j]), fb = unpack_bf16x2(pv[j]);
        acc += fabsf(fa.x - fb.x) + fabsf(fa.y - fb.y);
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) score[i] = acc / D;
  }
  __syncthreads();
  int local = 0;
  for (int i = npre + threadIdx.x; i < M; i += kTpThreads) local += score[i] >= threshold ? 1 : 0;
  atomicAdd(&s_cnt, local);
  __syncthreads();
  const int P = max(M - npre, 0);
  const bool use_topk = P > 0 && s_cnt < min_keep;
  const int k = min(min_keep, P);
  for (int i = threadIdx.x; i < M; i += kTpThreads) {
    int f;
    if (i < npre) {
      f = 1;
    } else if (!use_topk) {
      f = score[i] >= threshold ? 1 : 0;
    } else {  // rank among the patches: strictly better scores, or equal scores at lower positions
      const float si = score[i];
      int rank = 0;
      for (int j = npre; j < M && rank < k; ++j) {
        const float sj = score[j];
        rank += (sj > si || (sj == si && j < i)) ? 1 : 0;
      }
      f = rank < k ? 1 : 0;
    }
    flag[i] = f;
  }
  __syncthreads();
  // compact in position order (chunked block scan)
  int base = 0;
  for (int c0 = 0; c0 < M; c0 += kTpThreads) {
    const int i = c0 + threadIdx.x;
    const int f = i < M ? flag[i] : 0;
    int incl = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int woff = 0, tot = 0;
    for (int w = 0; w < kTpThreads / 32; ++w) {
      if (w < warp) woff += warp_tot[w];
      tot += warp_tot[w];
    }
    if (f) {
      const int pos = base + woff + incl - 1;
      dsel[(long)b * M + pos] = dindice[(long)b * M + i];
      qpos[(long)b * M + pos] = i;
      valid[(long)b * M + pos] = 1;
    }
    base += tot;
    __syncthreads();
  }
  for (int j = base + threadIdx.x; j < M; j += kTpThreads) {
    dsel[(long)b * M + j] = 0;
    qpos[(long)b * M + j] = 0;
    valid[(long)b * M + j] = 0;
  }
  if (threadIdx.x == 0) count[b] = base - min(npre, M);
}

// x, x_ref: bf16 [B*N, D] rows (same row stride); dindice: int32 [B, M]. Outputs int32 [B, M]
// dindice_sel / query_pos, bool [B, M] valid, int32 [B] kept patch counts.
void token_prune_op(const at::Tensor& x, const at::Tensor& x_ref, int64_t N, const at::Tensor& dindice, int64_t npre,
                    double threshold, int64_t min_keep, at::Tensor& dsel, at::Tensor& qpos, at::Tensor& valid,
                    at::Tensor& count) {
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && x_ref.scalar_type() == at::kBFloat16 && x.dim() == 2 &&
                  x.stride(1) == 1 && x_ref.stride(0) == x.stride(0) && x_ref.stride(1) == 1,
              "token_prune: bf16 [B*N, D] rows with a shared row stride");
  const int D = static_cast<int>(x.size(1));
  TORCH_CHECK(D % 8 == 0 && x.stride(0) % 8 == 0 && (reinterpret_cast<uintptr_t>(x.data_ptr()) & 15) == 0 &&
                  (reinterpret_cast<uintptr_t>(x_ref.data_ptr()) & 15) == 0,
              "token_prune: 16-byte aligned rows, D a multiple of 8");
  TORCH_CHECK(dindice.scalar_type() == at::kInt && dindice.dim() == 2 && dindice.is_contiguous(), "token_prune: dindice int32 [B, M]");
  const int B = static_cast<int>(dindice.size(0)), M = static_cast<int>(dindice.size(1));
  TORCH_CHECK(x.size(0) >= (long)B * N && x_ref.size(0) >= (long)B * N, "token_prune: x rows < B*N");
  for (const at::Tensor* t : {&dsel, &qpos})
    TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous() && t->numel() == (long)B * M, "token_prune: int32 [B, M] outputs");
  TORCH_CHECK(valid.scalar_type() == at::kBool && valid.is_contiguous() && valid.numel() == (long)B * M, "token_prune: valid bool [B, M]");
  TORCH_CHECK(count.scalar_type() == at::kInt && count.numel() == B, "token_prune: count int32 [B]");
  TORCH_CHECK(min_keep >= 1, "token_prune: min_keep >= 1");
  if (B == 0 || M == 0) return;
  const size_t smem = 2 * sizeof(float) * M;
  TORCH_CHECK(smem <= 190 * 1024, "token_prune: too many tokens");
  c10::cuda::CUDAGuard g(x.device());
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(token_prune_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  token_prune_kernel<<<B, kTpThreads, smem, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(x_ref.data_ptr()), x.stride(0),
      static_cast<int>(N), D, dindice.data_ptr<int>(), M, static_cast<int>(npre), static_cast<float>(threshold),
      static_cast<int>(min_keep), dsel.data_ptr<int>(), qpos.data_ptr<int>(),
      reinterpret_cast<uint8_t*>(valid.data_ptr()), count.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_token_prune_ops(pybind11::module_& m) { m.def("token_prune", &token_prune_op); }

}  // namespace appcorr
