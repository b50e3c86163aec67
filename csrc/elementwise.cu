// Memory-bound sm_100a kernels of appcorr_b200: normalisation, row movement, token preparation,
// attention-derived patch scores, the sync-free correction plan builder, pyramid decode and heads.
//
// Each replaces one reference op (file:line within the reference project):
//   layernorm_rows      norm1/norm2/final norm, optionally fused with the active-row gather
//                       (block.py:1111 gather + norm1; triton token_update.py:352-473)
//   add_rows            x + blocks_out_sum for every token (block.py:1146-1149)
//   patch_im2col        uint8 HWC pixels -> normalised bf16 16x16 patches feeding the patch-embed
//                       GEMM (layers/patch_embed.py:61-76 Conv2d k=s=16)
//   set_prefix_rows     CLS + storage tokens in front of the patch tokens
//                       (models/vision_transformer.py:308-340)
//   cls_attn_pscore     softmax(q_cls k^T / sqrt(d)) averaged over heads (attention.py:266-268)
//   correction_plan     server pscore (+ mobile hint) -> top-k over candidates -> ascending packed
//                       plan with gather/scatter row maps (block.py:360-443, 1017-1078)
//   pyrup_add           cv2.pyrUp of the coarser level + int16 residual, clipped to uint8
//                       (policies/transmission/laplacian.py:122-162, closed loop :234-262)
//   upsample_argmax     bilinear upsample of head logits + argmax (dinov3_segmentor_linhead.py:
//                       749-851 interpolate/softmax/argmax)
//   mean_rows           mean over patch tokens for the classifier head (dinov3_classifier.py:665)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cfloat>
#include <cuda_fp8.h>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < NT / 32) ? red[l] : 0.f;
  return warp_sum(t);
}

template <int NT>
__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  float t = (l < NT / 32) ? red[l] : -FLT_MAX;
  return warp_max(t);
}

// ------------------------------------------------------------------------------ LayerNorm
// One CTA (128 threads) per row; the row stays in registers (D <= 8192, D % 8 == 0).
constexpr int kLnThreads = 128;
constexpr int kLnMaxVec = 8;

__device__ __forceinline__ uint32_t pack_e4m3x4(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

// e4m3 row quantisation of 8 values per vector slot: q = y / scale, scale = amax / 448.
constexpr float kE4m3Max = 448.f;

// FP8 = true: the normalised row is emitted as e4m3 (out8, stride ldo bytes) with one fp32
// scale per row (scale8[r]) instead of bf16, ready for the e4m3 GEMM.
// OUTK = 2: NVFP4 row (packed e2m1, out8 row stride ldo bytes) + ue4m3 block scales (sf, blocked
// layout) + fp32 row scale (scale8[r] = amax / (6 * 448)).
template <int OUTK>
__global__ void __launch_bounds__(kLnThreads) layernorm_kernel(
    const bf16* __restrict__ x, long ldx, const int* __restrict__ rows, const bf16* __restrict__ w,
    const bf16* __restrict__ b, float eps, bf16* __restrict__ out, long ldo, bf16* __restrict__ copy_out,
    long ldc, int D, int nrows, uint8_t* __restrict__ out8, float* __restrict__ scale8, int rms,
    uint8_t* __restrict__ sf = nullptr) {
  __shared__ float red[kLnThreads / 32];
  const int r = blockIdx.x;
  if (r >= nrows) return;
  const long src = rows ? rows[r] : r;
  const uint4* xr = reinterpret_cast<const uint4*>(x + src * ldx);
  const int nvec = D >> 3;
  float v[kLnMaxVec][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    if (c < nvec) {
      uint4 u = xr[c];
      if (copy_out) reinterpret_cast<uint4*>(copy_out + (long)r * ldc)[c] = u;
      float2 p0 = unpack_bf16x2(u.x), p1 = unpack_bf16x2(u.y), p2 = unpack_bf16x2(u.z), p3 = unpack_bf16x2(u.w);
      v[i][0] = p0.x; v[i][1] = p0.y; v[i][2] = p1.x; v[i][3] = p1.y;
      v[i][4] = p2.x; v[i][5] = p2.y; v[i][6] = p3.x; v[i][7] = p3.y;
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[i][j];
    }
  }
  // rms: RMSNorm (no centring, no bias)
  const float mean = rms ? 0.f : block_sum<kLnThreads>(s, red) / D;
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    if (c < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[i][j] - mean;
        q += d * d;
      }
    }
  }
  const float rstd = rsqrtf(block_sum<kLnThreads>(q, red) / D + eps);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
  const uint4 zero4 = make_uint4(0u, 0u, 0u, 0u);
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    if (c < nvec) {
      uint4 wu = __ldg(wv + c), bu = b ? __ldg(bv + c) : zero4;
      const uint32_t* wp = &wu.x;
      const uint32_t* bp = &bu.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 ww = unpack_bf16x2(wp[j]), bb = unpack_bf16x2(bp[j]);
        // the bf16 rounding matches the bf16 path, so both precisions quantise the same values
        v[i][2 * j] = bf16_round((v[i][2 * j] - mean) * rstd * ww.x + bb.x);
        v[i][2 * j + 1] = bf16_round((v[i][2 * j + 1] - mean) * rstd * ww.y + bb.y);
        amax = fmaxf(amax, fmaxf(fabsf(v[i][2 * j]), fabsf(v[i][2 * j + 1])));
      }
    }
  }
  if constexpr (OUTK == 2) {
    // vector c covers elements 8c..8c+7; 16-element block c/2 = this lane and its xor-1 partner
    amax = block_max<kLnThreads>(amax, red);
    const float rs = fmaxf(amax, 1e-12f) / kNvfp4RowDiv;
    const float inv_rs = 1.f / rs;
    if (threadIdx.x == 0) scale8[r] = rs;
    uint32_t* orow = reinterpret_cast<uint32_t*>(out8 + (long)r * ldo);
#pragma unroll
    for (int i = 0; i < kLnMaxVec; ++i) {
      const int c = threadIdx.x + i * kLnThreads;
      float bm = 0.f;
      if (c < nvec) {
#pragma unroll
        for (int j = 0; j < 8; ++j) bm = fmaxf(bm, fabsf(v[i][j]));
      }
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));  // nvec is even: partners are both live
      if (c < nvec) {
        float mul;
        const uint32_t sb = nvfp4_block_scale(bm, inv_rs, rs, mul);
        orow[c] = pack_e2m1x8(v[i], mul);
        if ((c & 1) == 0) sf[nvfp4_sf_offset(r, c >> 1, D >> 6)] = static_cast<uint8_t>(sb);
      }
    }
  } else if constexpr (OUTK == 1) {
    amax = block_max<kLnThreads>(amax, red);
    const float sc = fmaxf(amax, 1e-12f) / kE4m3Max;
    const float inv = 1.f / sc;
    if (threadIdx.x == 0) scale8[r] = sc;
    uint2* orow = reinterpret_cast<uint2*>(out8 + (long)r * ldo);
#pragma unroll
    for (int i = 0; i < kLnMaxVec; ++i) {
      const int c = threadIdx.x + i * kLnThreads;
      if (c < nvec)
        orow[c] = make_uint2(pack_e4m3x4(v[i][0] * inv, v[i][1] * inv, v[i][2] * inv, v[i][3] * inv),
                             pack_e4m3x4(v[i][4] * inv, v[i][5] * inv, v[i][6] * inv, v[i][7] * inv));
    }
  } else {
    uint4* orow = reinterpret_cast<uint4*>(out + (long)r * ldo);
#pragma unroll
    for (int i = 0; i < kLnMaxVec; ++i) {
      const int c = threadIdx.x + i * kLnThreads;
      if (c < nvec)
        orow[c] = make_uint4(pack_bf16x2(v[i][0], v[i][1]), pack_bf16x2(v[i][2], v[i][3]),
                             pack_bf16x2(v[i][4], v[i][5]), pack_bf16x2(v[i][6], v[i][7]));
    }
  }
}

// Warp-per-row LayerNorm for D % 256 == 0, D <= 4096, the row staged in shared memory: each warp
// copies its row (D * 2 bytes) with 16-byte cp.async, then runs the statistics, normalisation and
// output passes from shared memory. Registers stay low, so ~28 rows per SM are in flight (a
// register-resident version held 254 registers and 8 rows per SM, latency-bound at 14 % DRAM
// throughput). Same arithmetic and outputs as layernorm_kernel (one CTA per row, block reductions),
// which stays for other widths.
constexpr int kLnsRows = 4;  // rows (warps) per CTA

__device__ __forceinline__ void ln_cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <int OUTK>
__global__ void __launch_bounds__(kLnsRows * 32) layernorm_smem_kernel(
    const bf16* __restrict__ x, long ldx, const int* __restrict__ rows, const bf16* __restrict__ w,
    const bf16* __restrict__ b, float eps, bf16* __restrict__ out, long ldo, bf16* __restrict__ copy_out,
    long ldc, int D, int nrows, uint8_t* __restrict__ out8, float* __restrict__ scale8, int rms,
    uint8_t* __restrict__ sf) {
  extern __shared__ uint4 lns_smem[];
  const int lane = threadIdx.x & 31;
  const int wid = threadIdx.x >> 5;
  const int r = blockIdx.x * kLnsRows + wid;
  if (r >= nrows) return;
  const int nvec = D >> 3;  // a multiple of 32
  uint4* row = lns_smem + wid * nvec;
  const long src = rows ? rows[r] : r;
  const uint4* xr = reinterpret_cast<const uint4*>(x + src * ldx);
  for (int c = lane; c < nvec; c += 32) ln_cp_async16(smem_addr(row + c), xr + c);
  asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
  __syncwarp();
  float s = 0.f;
#pragma unroll 4
  for (int c = lane; c < nvec; c += 32) {
    const uint4 u = row[c];
    if (copy_out) reinterpret_cast<uint4*>(copy_out + (long)r * ldc)[c] = u;
    const uint32_t* p = &u.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(p[j]);
      s += f.x + f.y;
    }
  }
  const float mean = rms ? 0.f : warp_sum(s) / D;
  float q = 0.f;
#pragma unroll 4
  for (int c = lane; c < nvec; c += 32) {
    const uint4 u = row[c];
    const uint32_t* p = &u.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(p[j]);
      q += (f.x - mean) * (f.x - mean) + (f.y - mean) * (f.y - mean);
    }
  }
  const float rstd = rsqrtf(warp_sum(q) / D + eps);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
  float amax = 0.f;
#pragma unroll 4
  for (int c = lane; c < nvec; c += 32) {
    uint4 u = row[c];
    const uint4 wu = __ldg(wv + c);
    const uint4 bu = b ? __ldg(bv + c) : make_uint4(0u, 0u, 0u, 0u);
    uint32_t* p = &u.x;
    const uint32_t* wp = &wu.x;
    const uint32_t* bp = &bu.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(p[j]), ww = unpack_bf16x2(wp[j]), bb = unpack_bf16x2(bp[j]);
      const float y0 = bf16_round((f.x - mean) * rstd * ww.x + bb.x);
      const float y1 = bf16_round((f.y - mean) * rstd * ww.y + bb.y);
      amax = fmaxf(amax, fmaxf(fabsf(y0), fabsf(y1)));
      p[j] = pack_bf16x2(y0, y1);
    }
    if constexpr (OUTK == 0) reinterpret_cast<uint4*>(out + (long)r * ldo)[c] = u;
    else row[c] = u;  // normalised row back in place (this lane reads it again below)
  }
  if constexpr (OUTK == 1) {
    amax = warp_max(amax);
    const float sc = fmaxf(amax, 1e-12f) / kE4m3Max;
    const float inv = 1.f / sc;
    if (lane == 0) scale8[r] = sc;
#pragma unroll 4
    for (int c = lane; c < nvec; c += 32) {
      const uint4 u = row[c];
      const float2 a0 = unpack_bf16x2(u.x), a1 = unpack_bf16x2(u.y), a2 = unpack_bf16x2(u.z), a3 = unpack_bf16x2(u.w);
      reinterpret_cast<uint2*>(out8 + (long)r * ldo)[c] =
          make_uint2(pack_e4m3x4(a0.x * inv, a0.y * inv, a1.x * inv, a1.y * inv),
                     pack_e4m3x4(a2.x * inv, a2.y * inv, a3.x * inv, a3.y * inv));
    }
  } else if constexpr (OUTK == 2) {
    amax = warp_max(amax);
    const float rs = fmaxf(amax, 1e-12f) / kNvfp4RowDiv;
    const float inv_rs = 1.f / rs;
    if (lane == 0) scale8[r] = rs;
    // vector c = lane + 32 i: 16-element blocks pair lanes (l, l ^ 1); the four block scales of a
    // 64-element tile (lanes c..c+7) go out as one 4-byte store
#pragma unroll 2
    for (int c = lane; c < nvec; c += 32) {
      const uint4 u = row[c];
      float v[8];
      const uint32_t* p = &u.x;
      float bm = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(p[j]);
        v[2 * j] = f.x;
        v[2 * j + 1] = f.y;
        bm = fmaxf(bm, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
      float mul;
      const uint32_t sb = nvfp4_block_scale(bm, inv_rs, rs, mul);
      reinterpret_cast<uint32_t*>(out8 + (long)r * ldo)[c] = pack_e2m1x8(v, mul);
      const uint32_t s1 = __shfl_down_sync(0xffffffffu, sb, 2);
      const uint32_t s2 = __shfl_down_sync(0xffffffffu, sb, 4);
      const uint32_t s3 = __shfl_down_sync(0xffffffffu, sb, 6);
      if ((c & 7) == 0)
        *reinterpret_cast<uint32_t*>(sf + nvfp4_sf_offset(r, c >> 1, D >> 6)) = sb | (s1 << 8) | (s2 << 16) | (s3 << 24);
    }
  }
}

template <int OUTK>
static bool launch_layernorm_warp(int D, int nrows, cudaStream_t st, const bf16* x, long ldx, const int* rp,
                                  const bf16* w, const bf16* b, float eps, bf16* out, long ldo, bf16* cp, long ldc,
                                  uint8_t* out8, float* scale8, int rms, uint8_t* sf) {
  if (D % 256 != 0 || D > 4096) return false;
  const int grid = (nrows + kLnsRows - 1) / kLnsRows;
  const size_t smem = static_cast<size_t>(kLnsRows) * D * 2;  // <= 32 KB: no opt-in needed
  layernorm_smem_kernel<OUTK><<<grid, kLnsRows * 32, smem, st>>>(x, ldx, rp, w, b, eps, out, ldo, cp, ldc, D, nrows,
                                                                  out8, scale8, rms, sf);
  return true;
}

// bf16 rows -> e4m3 rows + one fp32 scale per row (amax / 448). One CTA per row, K <= 8192.
__global__ void __launch_bounds__(kLnThreads) quant_rows_e4m3_kernel(const bf16* __restrict__ x, long ldx,
                                                                     uint8_t* __restrict__ out, long ldo,
                                                                     float* __restrict__ scale, int K) {
  __shared__ float red[kLnThreads / 32];
  const int r = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (long)r * ldx);
  const int nvec = K >> 3;
  uint4 u[kLnMaxVec];
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    if (c < nvec) {
      u[i] = xr[c];
      const uint32_t* p = &u[i].x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(p[j]);
        amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
  }
  amax = block_max<kLnThreads>(amax, red);
  const float sc = fmaxf(amax, 1e-12f) / kE4m3Max;
  const float inv = 1.f / sc;
  if (threadIdx.x == 0) scale[r] = sc;
  uint2* orow = reinterpret_cast<uint2*>(out + (long)r * ldo);
#pragma unroll
  for (int i = 0; i < kLnMaxVec; ++i) {
    const int c = threadIdx.x + i * kLnThreads;
    if (c < nvec) {
      const uint32_t* p = &u[i].x;
      const float2 a = unpack_bf16x2(p[0]), b = unpack_bf16x2(p[1]), cc = unpack_bf16x2(p[2]), d = unpack_bf16x2(p[3]);
      orow[c] = make_uint2(pack_e4m3x4(a.x * inv, a.y * inv, b.x * inv, b.y * inv),
                           pack_e4m3x4(cc.x * inv, cc.y * inv, d.x * inv, d.y * inv));
    }
  }
}

// Rows longer than the register-resident kernel holds (K > 8192, e.g. a 18944-wide MLP hidden):
// pass 1 finds the amax, pass 2 re-reads the row (L1/L2 hits) and quantises.
__global__ void __launch_bounds__(kLnThreads) quant_rows_e4m3_long_kernel(const bf16* __restrict__ x, long ldx,
                                                                          uint8_t* __restrict__ out, long ldo,
                                                                          float* __restrict__ scale, int K) {
  __shared__ float red[kLnThreads / 32];
  const int r = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (long)r * ldx);
  float amax = 0.f;
  for (int c = threadIdx.x; c < (K >> 3); c += kLnThreads) {
    const uint4 u = xr[c];
    const uint32_t* p = &u.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(p[j]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  amax = block_max<kLnThreads>(amax, red);
  const float sc = fmaxf(amax, 1e-12f) / kE4m3Max;
  const float inv = 1.f / sc;
  if (threadIdx.x == 0) scale[r] = sc;
  uint2* orow = reinterpret_cast<uint2*>(out + (long)r * ldo);
  for (int c = threadIdx.x; c < (K >> 3); c += kLnThreads) {
    const uint4 u = xr[c];
    const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), cc = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
    orow[c] = make_uint2(pack_e4m3x4(a.x * inv, a.y * inv, b.x * inv, b.y * inv),
                         pack_e4m3x4(cc.x * inv, cc.y * inv, d.x * inv, d.y * inv));
  }
}

void quant_rows_e4m3_op(const at::Tensor& x, at::Tensor& out, at::Tensor& scale) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1,
              "quant_rows_e4m3: bf16 [M,K] CUDA x");
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1));
  TORCH_CHECK(K % 16 == 0, "quant_rows_e4m3: K % 16 == 0");
  TORCH_CHECK(out.scalar_type() == at::kFloat8_e4m3fn && out.size(0) >= M && out.size(1) == K && out.stride(1) == 1,
              "quant_rows_e4m3: out e4m3 [M,K]");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.numel() >= M, "quant_rows_e4m3: scale fp32 [M]");
  TORCH_CHECK(x.stride(0) % 8 == 0 && out.stride(0) % 16 == 0, "quant_rows_e4m3: 16-byte aligned rows");
  if (M == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  auto kern = K <= kLnThreads * kLnMaxVec * 8 ? quant_rows_e4m3_kernel : quant_rows_e4m3_long_kernel;
  kern<<<M, kLnThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0), reinterpret_cast<uint8_t*>(out.data_ptr()),
      out.stride(0), scale.data_ptr<float>(), K);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// bf16 rows -> NVFP4 rows (any K % 64 == 0): pass 1 finds the row amax, pass 2 quantises one
// 16-element block per thread step (re-reading the row from L1/L2).
__global__ void __launch_bounds__(kLnThreads) quant_rows_nvfp4_kernel(const bf16* __restrict__ x, long ldx,
                                                                      uint8_t* __restrict__ out, long ldo,
                                                                      uint8_t* __restrict__ sf,
                                                                      float* __restrict__ scale, int K) {
  __shared__ float red[kLnThreads / 32];
  const int r = blockIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (long)r * ldx);
  float amax = 0.f;
  for (int c = threadIdx.x; c < (K >> 3); c += kLnThreads) {
    const uint4 u = xr[c];
    const uint32_t* p = &u.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = unpack_bf16x2(p[j]);
      amax = fmaxf(amax, fmaxf(fabsf(f.x), fabsf(f.y)));
    }
  }
  amax = block_max<kLnThreads>(amax, red);
  const float rs = fmaxf(amax, 1e-12f) / kNvfp4RowDiv;
  const float inv_rs = 1.f / rs;
  if (threadIdx.x == 0) scale[r] = rs;
  uint2* orow = reinterpret_cast<uint2*>(out + (long)r * ldo);
  for (int blk = threadIdx.x; blk < (K >> 4); blk += kLnThreads) {
    float v[16];
    float bm = 0.f;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4 u = xr[2 * blk + h];
      const uint32_t* p = &u.x;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = unpack_bf16x2(p[j]);
        v[8 * h + 2 * j] = f.x;
        v[8 * h + 2 * j + 1] = f.y;
        bm = fmaxf(bm, fmaxf(fabsf(f.x), fabsf(f.y)));
      }
    }
    float mul;
    const uint32_t sb = nvfp4_block_scale(bm, inv_rs, rs, mul);
    orow[blk] = make_uint2(pack_e2m1x8(v, mul), pack_e2m1x8(v + 8, mul));
    sf[nvfp4_sf_offset(r, blk, K >> 6)] = static_cast<uint8_t>(sb);
  }
}

static void check_nvfp4_out(const at::Tensor& out, const at::Tensor& sf, int M, int K, const char* who) {
  TORCH_CHECK(out.scalar_type() == at::kByte && out.dim() == 2 && out.size(0) >= M && out.size(1) == K / 2 &&
                  out.stride(1) == 1 && out.stride(0) % 16 == 0,
              who, ": out uint8 [M, K/2] with 16-byte aligned rows");
  TORCH_CHECK(K % 64 == 0, who, ": K % 64 == 0");
  TORCH_CHECK(sf.scalar_type() == at::kByte && sf.is_contiguous() &&
                  sf.numel() >= (long)((M + 127) / 128) * (K / 64) * 512,
              who, ": sf uint8 of ceil(M/128) * K/64 * 512 bytes");
}

void quant_rows_nvfp4_op(const at::Tensor& x, at::Tensor& out, at::Tensor& sf, at::Tensor& scale) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.stride(1) == 1 &&
                  x.stride(0) % 8 == 0,
              "quant_rows_nvfp4: bf16 [M,K] CUDA x with 16-byte aligned rows");
  const int M = static_cast<int>(x.size(0)), K = static_cast<int>(x.size(1));
  check_nvfp4_out(out, sf, M, K, "quant_rows_nvfp4");
  TORCH_CHECK(scale.scalar_type() == at::kFloat && scale.numel() >= M, "quant_rows_nvfp4: scale fp32 [M]");
  if (M == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  quant_rows_nvfp4_kernel<<<M, kLnThreads, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(0), out.data_ptr<uint8_t>(), out.stride(0),
      sf.data_ptr<uint8_t>(), scale.data_ptr<float>(), K);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void layernorm_op(const at::Tensor& x, c10::optional<at::Tensor> rows, const at::Tensor& w,
                  c10::optional<at::Tensor> b_opt, double eps, at::Tensor& out, c10::optional<at::Tensor> copy_out, c10::optional<at::Tensor> scale8,
                  bool rms, c10::optional<at::Tensor> sf) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.stride(-1) == 1, "layernorm: bf16 CUDA x");
  const int D = static_cast<int>(x.size(-1));
  TORCH_CHECK(D % 8 == 0 && D <= kLnThreads * kLnMaxVec * 8, "layernorm: D % 8 == 0 and D <= 8192");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && w.numel() == D, "layernorm: bf16 weight [D]");
  const at::Tensor b = b_opt.has_value() ? *b_opt : at::Tensor();
  TORCH_CHECK(!b.defined() || (b.scalar_type() == at::kBFloat16 && b.numel() == D), "layernorm: bf16 bias [D]");
  const bf16* bptr = b.defined() ? reinterpret_cast<const bf16*>(b.data_ptr()) : nullptr;
  const long ldx = x.stride(-2);
  const int nrows = static_cast<int>(out.size(0));
  const int* rp = nullptr;
  if (rows.has_value()) {
    TORCH_CHECK(rows->scalar_type() == at::kInt && rows->numel() == nrows, "layernorm: rows int32 [nrows]");
    rp = rows->data_ptr<int>();
  } else {
    TORCH_CHECK(x.numel() / D == nrows, "layernorm: row count mismatch");
  }
  bf16* cp = nullptr;
  long ldc = 0;
  if (copy_out.has_value()) {
    cp = reinterpret_cast<bf16*>(copy_out->data_ptr());
    ldc = copy_out->stride(0);
  }
  const bool fp4 = out.scalar_type() == at::kByte;
  const bool fp8 = out.scalar_type() == at::kFloat8_e4m3fn || fp4;
  TORCH_CHECK(fp8 || out.scalar_type() == at::kBFloat16, "layernorm: out bf16, e4m3 or nvfp4 (uint8)");
  TORCH_CHECK(fp8 == scale8.has_value(), "layernorm: e4m3 / nvfp4 output needs scale8 [nrows]");
  TORCH_CHECK(fp4 == sf.has_value(), "layernorm: nvfp4 output needs sf (block scales)");
  if (fp4) {
    check_nvfp4_out(out, *sf, nrows, D, "layernorm");
    TORCH_CHECK(D <= kLnThreads * kLnMaxVec * 8, "layernorm: D <= 8192");
  }
  if (fp8) {
    TORCH_CHECK(scale8->scalar_type() == at::kFloat && scale8->numel() >= nrows, "layernorm: scale8 fp32 [nrows]");
    TORCH_CHECK(out.stride(0) % 8 == 0, "layernorm: e4m3 rows must be 8-byte aligned");
  }
  if (nrows == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  auto st = at::cuda::getCurrentCUDAStream();
  {
    const bf16* xp = reinterpret_cast<const bf16*>(x.data_ptr());
    const bf16* wp = reinterpret_cast<const bf16*>(w.data_ptr());
    const float e = static_cast<float>(eps);
    bool done;
    if (fp4)
      done = launch_layernorm_warp<2>(D, nrows, st, xp, ldx, rp, wp, bptr, e, nullptr, out.stride(0), cp, ldc,
                                      out.data_ptr<uint8_t>(), scale8->data_ptr<float>(), rms ? 1 : 0,
                                      sf->data_ptr<uint8_t>());
    else if (fp8)
      done = launch_layernorm_warp<1>(D, nrows, st, xp, ldx, rp, wp, bptr, e, nullptr, out.stride(0), cp, ldc,
                                      reinterpret_cast<uint8_t*>(out.data_ptr()), scale8->data_ptr<float>(),
                                      rms ? 1 : 0, nullptr);
    else
      done = launch_layernorm_warp<0>(D, nrows, st, xp, ldx, rp, wp, bptr, e, reinterpret_cast<bf16*>(out.data_ptr()),
                                      out.stride(0), cp, ldc, nullptr, nullptr, rms ? 1 : 0, nullptr);
    if (done) {
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      return;
    }
  }
  if (fp4)
    layernorm_kernel<2><<<nrows, kLnThreads, 0, st>>>(
        reinterpret_cast<const bf16*>(x.data_ptr()), ldx, rp, reinterpret_cast<const bf16*>(w.data_ptr()),
        bptr, static_cast<float>(eps), nullptr, out.stride(0), cp, ldc, D,
        nrows, out.data_ptr<uint8_t>(), scale8->data_ptr<float>(), rms ? 1 : 0, sf->data_ptr<uint8_t>());
  else if (fp8)
    layernorm_kernel<1><<<nrows, kLnThreads, 0, st>>>(
        reinterpret_cast<const bf16*>(x.data_ptr()), ldx, rp, reinterpret_cast<const bf16*>(w.data_ptr()),
        bptr, static_cast<float>(eps), nullptr, out.stride(0), cp, ldc, D,
        nrows, reinterpret_cast<uint8_t*>(out.data_ptr()), scale8->data_ptr<float>(), rms ? 1 : 0);
  else
    layernorm_kernel<0><<<nrows, kLnThreads, 0, st>>>(
        reinterpret_cast<const bf16*>(x.data_ptr()), ldx, rp, reinterpret_cast<const bf16*>(w.data_ptr()),
        bptr, static_cast<float>(eps), reinterpret_cast<bf16*>(out.data_ptr()),
        out.stride(0), cp, ldc, D, nrows, nullptr, nullptr, rms ? 1 : 0);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ x += y
__global__ void add_bf16_kernel(bf16* __restrict__ x, const bf16* __restrict__ y, long n8) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n8; i += (long)gridDim.x * blockDim.x) {
    uint4 a = reinterpret_cast<uint4*>(x)[i];
    uint4 c = reinterpret_cast<const uint4*>(y)[i];
    uint32_t* ap = &a.x;
    const uint32_t* cp = &c.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float2 p = unpack_bf16x2(ap[j]), q = unpack_bf16x2(cp[j]);
      ap[j] = pack_bf16x2(p.x + q.x, p.y + q.y);
    }
    reinterpret_cast<uint4*>(x)[i] = a;
  }
}

void add_inplace_op(at::Tensor& x, const at::Tensor& y) {
  TORCH_CHECK(x.is_contiguous() && y.is_contiguous() && x.numel() == y.numel() && x.numel() % 8 == 0, "add_: contiguous, numel % 8");
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && y.scalar_type() == at::kBFloat16, "add_: bf16");
  const long n8 = x.numel() / 8;
  if (n8 == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  const int grid = static_cast<int>(std::min<long>((n8 + 255) / 256, num_sms() * 8L));
  add_bf16_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<bf16*>(x.data_ptr()), reinterpret_cast<const bf16*>(y.data_ptr()), n8);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ patch im2col
// img: uint8 [B, H, W, 3] (HWC as decoded). out: bf16 [B * (H/p) * (W/p), 3*p*p], column index
// c*p*p + ky*p + kx (the Conv2d weight flattening order). Pixels are normalised as
// (v / 255 - mean[c]) / std[c].
// Output row r of image b holds patch perm[r] (row-major patch index; perm == nullptr: r), in a
// buffer of row stride ldo >= 3*p*p (columns past 3*p*p are left untouched).
__global__ void patch_im2col_kernel(const uint8_t* __restrict__ img, int H, int W, int p, float3 mean,
                                    float3 inv_std, bf16* __restrict__ out, long total, long ldo,
                                    const int* __restrict__ perm) {
  const int gw = W / p, gh = H / p;
  const int K = 3 * p * p;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / K;
    const int col = static_cast<int>(i - row * K);
    const int c = col / (p * p);
    const int rem = col - c * p * p;
    const int ky = rem / p, kx = rem - (rem / p) * p;
    const long b = row / (gh * gw);
    const int r = static_cast<int>(row - b * gh * gw);
    const int t = perm ? perm[r] : r;
    const int py = t / gw, px = t - (t / gw) * gw;
    const int y = py * p + ky, x = px * p + kx;
    const float v = img[((b * H + y) * W + x) * 3 + c] * (1.0f / 255.0f);
    const float m = c == 0 ? mean.x : (c == 1 ? mean.y : mean.z);
    const float s = c == 0 ? inv_std.x : (c == 1 ? inv_std.y : inv_std.z);
    out[row * ldo + col] = __float2bfloat16_rn((v - m) * s);
  }
}

void patch_im2col_op(const at::Tensor& img, int64_t patch, std::vector<double> mean, std::vector<double> std_,
                     at::Tensor& out, c10::optional<at::Tensor> perm) {
  TORCH_CHECK(img.is_cuda() && img.scalar_type() == at::kByte && img.dim() == 4 && img.size(3) == 3 && img.is_contiguous(),
              "patch_im2col: uint8 [B,H,W,3] contiguous");
  const int H = static_cast<int>(img.size(1)), W = static_cast<int>(img.size(2)), p = static_cast<int>(patch);
  TORCH_CHECK(H % p == 0 && W % p == 0, "patch_im2col: H, W multiples of patch");
  const long total = img.size(0) * (long)(H / p) * (W / p) * 3 * p * p;
  const long rows = img.size(0) * (long)(H / p) * (W / p);
  TORCH_CHECK(out.dim() == 2 && out.size(0) == rows && out.size(1) >= 3 * p * p && out.stride(1) == 1 &&
                  out.scalar_type() == at::kBFloat16,
              "patch_im2col: out bf16 [B*patches, >= 3*p*p]");
  const int* pp = nullptr;
  if (perm.has_value()) {
    TORCH_CHECK(perm->scalar_type() == at::kInt && perm->numel() == (H / p) * (W / p) && perm->is_cuda(),
                "patch_im2col: perm int32 [patches]");
    pp = perm->data_ptr<int>();
  }
  c10::cuda::CUDAGuard g(img.device());
  const int grid = static_cast<int>(std::min<long>((total + 255) / 256, num_sms() * 16L));
  patch_im2col_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      img.data_ptr<uint8_t>(), H, W, p, make_float3(mean[0], mean[1], mean[2]),
      make_float3(1.0 / std_[0], 1.0 / std_[1], 1.0 / std_[2]), reinterpret_cast<bf16*>(out.data_ptr()), total,
      out.stride(0), pp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ row distance
// out[r] = sum_c (a[r,c] - b[r,c])^2 in fp32; one warp per row (D % 8 == 0). The VLM correction
// ranks image tokens by how much their embedding moved between the approximate and the current
// canvas.
__global__ void row_sqdist_kernel(const bf16* __restrict__ a, long lda, const bf16* __restrict__ b, long ldb,
                                  float* __restrict__ out, int M, int D) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= M) return;
  const uint4* pa = reinterpret_cast<const uint4*>(a + (long)row * lda);
  const uint4* pb = reinterpret_cast<const uint4*>(b + (long)row * ldb);
  float acc = 0.f;
  for (int c = lane; c < (D >> 3); c += 32) {
    const uint4 ua = pa[c], ub = pb[c];
    const uint32_t* xa = &ua.x;
    const uint32_t* xb = &ub.x;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 fa = unpack_bf16x2(xa[j]), fb = unpack_bf16x2(xb[j]);
      const float d0 = fa.x - fb.x, d1 = fa.y - fb.y;
      acc = fmaf(d0, d0, fmaf(d1, d1, acc));
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) out[row] = acc;
}

void row_sqdist_op(const at::Tensor& a, const at::Tensor& b, at::Tensor& out) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && a.dim() == 2 &&
                  b.sizes() == a.sizes() && a.stride(1) == 1 && b.stride(1) == 1,
              "row_sqdist: bf16 [M, D] a, b");
  const int M = static_cast<int>(a.size(0)), D = static_cast<int>(a.size(1));
  TORCH_CHECK(D % 8 == 0 && a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "row_sqdist: 16-byte rows");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() == M && out.is_contiguous(), "row_sqdist: out fp32 [M]");
  if (M == 0) return;
  c10::cuda::CUDAGuard g(a.device());
  row_sqdist_kernel<<<(M + 7) / 8, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(a.data_ptr()), a.stride(0), reinterpret_cast<const bf16*>(b.data_ptr()),
      b.stride(0), out.data_ptr<float>(), M, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ prefix rows
// x: [B, N, D]; rows 0..npre-1 of each image <- prefix [npre, D].
__global__ void set_prefix_kernel(bf16* __restrict__ x, long ldx, int N, const bf16* __restrict__ prefix, int npre,
                                  int D, int B) {
  const int n8 = D >> 3;
  const long total = (long)B * npre * n8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long row = i / n8;
    const int c = static_cast<int>(i - row * n8);
    const int b = static_cast<int>(row / npre);
    const int t = static_cast<int>(row - (long)b * npre);
    reinterpret_cast<uint4*>(x + ((long)b * N + t) * ldx)[c] = reinterpret_cast<const uint4*>(prefix + (long)t * D)[c];
  }
}

void set_prefix_op(at::Tensor& x, const at::Tensor& prefix, int64_t B, int64_t N) {
  const int D = static_cast<int>(x.size(-1));
  const int npre = static_cast<int>(prefix.size(0));
  TORCH_CHECK(prefix.is_contiguous() && prefix.size(1) == D && D % 8 == 0, "set_prefix: prefix [npre, D]");
  if (B * npre == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  set_prefix_kernel<<<std::max<long>(1, (B * npre * (D / 8) + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<bf16*>(x.data_ptr()), x.stride(-2), static_cast<int>(N),
      reinterpret_cast<const bf16*>(prefix.data_ptr()), npre, D, static_cast<int>(B));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ row gather
__global__ void gather_rows_kernel(const bf16* __restrict__ src, long lds, const int* __restrict__ rows,
                                   bf16* __restrict__ dst, long ldd, int n8, int nrows) {
  const long total = (long)nrows * n8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / n8);
    const int c = static_cast<int>(i - (long)r * n8);
    reinterpret_cast<uint4*>(dst + (long)r * ldd)[c] = reinterpret_cast<const uint4*>(src + (long)rows[r] * lds)[c];
  }
}

__global__ void scatter_rows_kernel(const bf16* __restrict__ src, long lds, const int* __restrict__ rows,
                                    bf16* __restrict__ dst, long ldd, int n8, int nrows) {
  const long total = (long)nrows * n8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / n8);
    const int c = static_cast<int>(i - (long)r * n8);
    reinterpret_cast<uint4*>(dst + (long)rows[r] * ldd)[c] = reinterpret_cast<const uint4*>(src + (long)r * lds)[c];
  }
}

void gather_rows_op(const at::Tensor& src, const at::Tensor& rows, at::Tensor& dst) {
  const int D = static_cast<int>(src.size(-1));
  TORCH_CHECK(D % 8 == 0 && src.scalar_type() == at::kBFloat16 && dst.scalar_type() == at::kBFloat16, "gather_rows: bf16, D%8");
  TORCH_CHECK(rows.scalar_type() == at::kInt, "gather_rows: int32 rows");
  const int nrows = static_cast<int>(rows.numel());
  if (nrows == 0) return;
  c10::cuda::CUDAGuard g(src.device());
  const long total = (long)nrows * (D / 8);
  gather_rows_kernel<<<static_cast<int>(std::min<long>((total + 255) / 256, num_sms() * 16L)), 256, 0,
                       at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const bf16*>(src.data_ptr()), src.stride(-2),
                                                           rows.data_ptr<int>(), reinterpret_cast<bf16*>(dst.data_ptr()),
                                                           dst.stride(-2), D / 8, nrows);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void scatter_rows_op(const at::Tensor& src, const at::Tensor& rows, at::Tensor& dst) {
  const int D = static_cast<int>(src.size(-1));
  TORCH_CHECK(D % 8 == 0 && src.scalar_type() == at::kBFloat16 && dst.scalar_type() == at::kBFloat16, "scatter_rows: bf16, D%8");
  TORCH_CHECK(rows.scalar_type() == at::kInt, "scatter_rows: int32 rows");
  const int nrows = static_cast<int>(rows.numel());
  if (nrows == 0) return;
  c10::cuda::CUDAGuard g(src.device());
  const long total = (long)nrows * (D / 8);
  scatter_rows_kernel<<<static_cast<int>(std::min<long>((total + 255) / 256, num_sms() * 16L)), 256, 0,
                        at::cuda::getCurrentCUDAStream()>>>(reinterpret_cast<const bf16*>(src.data_ptr()), src.stride(-2),
                                                            rows.data_ptr<int>(), reinterpret_cast<bf16*>(dst.data_ptr()),
                                                            dst.stride(-2), D / 8, nrows);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ CLS attention pscore
// grid (B, H). q: image b's query row at q + b * q_bstride (row b*N of [B*N, H*Dh] rows for the
// CLS query: q_bstride = N * ld; a [B, H*Dh] pseudo-query buffer: q_bstride = H*Dh), k: [B*N, H*Dh].
// probs: fp32 [B, H, N] = softmax over keys of that query. A second pass averages over heads.
constexpr int kPsThreads = 256;

__global__ void __launch_bounds__(kPsThreads) cls_attn_probs_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                                    long ld, long q_bstride, int N, int H, int Dh,
                                                                    float scale, float* __restrict__ probs) {
  extern __shared__ float s_buf[];  // [N] logits, then [Dh] query
  __shared__ float red[kPsThreads / 32];
  const int b = blockIdx.x, h = blockIdx.y;
  float* qs = s_buf + N;
  const bf16* qrow = q + (long)b * q_bstride + (long)h * Dh;
  for (int d = threadIdx.x; d < Dh; d += kPsThreads) qs[d] = __bfloat162float(qrow[d]);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // One warp per key; lanes split the head dim.
  for (int j = warp; j < N; j += kPsThreads / 32) {
    const bf16* krow = k + ((long)b * N + j) * ld + (long)h * Dh;
    float acc = 0.f;
    for (int d = lane * 2; d < Dh; d += 64) {
      float2 kk = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(krow + d));
      acc += kk.x * qs[d] + kk.y * qs[d + 1];
    }
    acc = warp_sum(acc);
    if (lane == 0) s_buf[j] = acc * scale;
  }
  __syncthreads();
  float mx = -FLT_MAX;
  for (int j = threadIdx.x; j < N; j += kPsThreads) mx = fmaxf(mx, s_buf[j]);
  mx = block_max<kPsThreads>(mx, red);
  float sum = 0.f;
  for (int j = threadIdx.x; j < N; j += kPsThreads) {
    const float e = __expf(s_buf[j] - mx);
    s_buf[j] = e;
    sum += e;
  }
  sum = block_sum<kPsThreads>(sum, red);
  const float inv = 1.0f / sum;
  float* out = probs + ((long)b * H + h) * N;
  for (int j = threadIdx.x; j < N; j += kPsThreads) out[j] = s_buf[j] * inv;
}

// out[b, j] = mean_h probs[b, h, j]
__global__ void head_mean_kernel(const float* __restrict__ probs, int B, int H, int N, float* __restrict__ out) {
  const long total = (long)B * N;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long b = i / N;
    const int j = static_cast<int>(i - b * N);
    float s = 0.f;
    for (int h = 0; h < H; ++h) s += probs[(b * H + h) * N + j];
    out[i] = s / H;
  }
}

void cls_attn_pscore_op(const at::Tensor& q, const at::Tensor& k, int64_t B, int64_t N, int64_t H, int64_t Dh,
                        double scale, at::Tensor& scratch, at::Tensor& out, int64_t q_bstride) {
  TORCH_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16, "cls_attn_pscore: bf16");
  // q_bstride < 0: the CLS row of [B*N, H*Dh] q rows sharing k's row stride
  if (q_bstride < 0) {
    TORCH_CHECK(q.stride(0) == k.stride(0), "cls_attn_pscore: q and k share a row stride");
    q_bstride = N * q.stride(0);
  } else {
    TORCH_CHECK(q.is_contiguous() && q.numel() >= (B - 1) * q_bstride + H * Dh, "cls_attn_pscore: query buffer too small");
  }
  TORCH_CHECK(k.stride(0) % 2 == 0 && q_bstride % 2 == 0, "cls_attn_pscore: even row strides");
  TORCH_CHECK(scratch.scalar_type() == at::kFloat && scratch.numel() >= B * H * N, "cls_attn_pscore: scratch fp32 [B,H,N]");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.numel() == B * N && out.is_contiguous(), "cls_attn_pscore: out fp32 [B,N]");
  TORCH_CHECK(Dh % 64 == 0, "cls_attn_pscore: Dh multiple of 64");
  c10::cuda::CUDAGuard g(q.device());
  auto st = at::cuda::getCurrentCUDAStream();
  const size_t smem = (N + Dh) * sizeof(float);
  TORCH_CHECK(smem <= 200 * 1024, "cls_attn_pscore: sequence too long");
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(cls_attn_probs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  cls_attn_probs_kernel<<<dim3(B, H), kPsThreads, smem, st>>>(
      reinterpret_cast<const bf16*>(q.data_ptr()), reinterpret_cast<const bf16*>(k.data_ptr()), k.stride(0), q_bstride,
      static_cast<int>(N), static_cast<int>(H), static_cast<int>(Dh), static_cast<float>(scale), scratch.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  head_mean_kernel<<<static_cast<int>(std::max<long>(1, (B * N + 255) / 256)), 256, 0, st>>>(
      scratch.data_ptr<float>(), static_cast<int>(B), static_cast<int>(H), static_cast<int>(N), out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ correction plan
// One CTA per image. Candidates are the patch tokens cand[b, 0..P). The combined score is
//   s = ws * server[b, cand] (+|*|geo) wm * mobile[b, i]
// and the plan keeps the k highest-scoring candidates (radix select on the fp32 order key; ties
// resolved towards lower candidate position), emitted in ascending candidate order after the
// npre prefix tokens, exactly the layout of the fixed-k builder (block.py:398-443).
// Outputs (T = npre + k):
//   upd  [B, T]      token indices (update_indice)
//   rows [B*T]       b*N + token: gather rows of x, scatter rows of the KV cache / stream
//   stats [B, 2]     kept / full score mass (block.py:763-791)
constexpr int kPlanThreads = 512;

__device__ __forceinline__ uint32_t f32_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__global__ void __launch_bounds__(kPlanThreads) correction_plan_kernel(
    const float* __restrict__ server, int N, const int* __restrict__ pre, int npre, const int* __restrict__ cand, int P,
    const float* __restrict__ mobile, float ws, float wm, int fusion, const uint8_t* __restrict__ valid, int k,
    int* __restrict__ upd, int* __restrict__ rows, float* __restrict__ stats, int use_thres, float thres,
    int* __restrict__ counts) {
  extern __shared__ uint32_t sm[];
  uint32_t* keys = sm;                                  // [P]
  float* sc = reinterpret_cast<float*>(sm + P);         // [P]
  int* flag = reinterpret_cast<int*>(sm + 2 * P);       // [P]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t s_prefix, s_remaining;
  __shared__ float red[kPlanThreads / 32];
  __shared__ int warp_tot[kPlanThreads / 32];
  const int b = blockIdx.x;
  const int T = npre + k;
  float full = 0.f;
  for (int i = threadIdx.x; i < P; i += kPlanThreads) {
    const int tok = cand[(long)b * P + i];
    float s = ws * server[(long)b * N + tok];
    if (mobile != nullptr && wm != 0.f) {
      const float mt = wm * mobile[(long)b * P + i];
      if (fusion == 1) s = s * mt;
      else if (fusion == 2) s = sqrtf(fmaxf(s * mt, 0.f));
      else s = s + mt;
    }
    if (valid != nullptr && !valid[(long)b * P + i]) s = -INFINITY;
    sc[i] = s;
    keys[i] = f32_order_key(s);
    if (isfinite(s)) full += s;
  }
  full = block_sum<kPlanThreads>(full, red);
  if (use_thres) {
    // Threshold selection (block.py:373-375): keep every candidate scoring >= thres; the plan
    // holds the first k of them in candidate order (k = the cap) and is padded below.
    for (int i = threadIdx.x; i < P; i += kPlanThreads) flag[i] = sc[i] >= thres ? 1 : 0;
    __syncthreads();
  } else {
  // Radix select the k-th largest key, 8 bits per pass, most significant first.
  if (threadIdx.x == 0) { s_prefix = 0; s_remaining = k; }
  __syncthreads();
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    const uint32_t hi_mask = pass == 0 ? 0u : (0xFFFFFFFFu << (shift + 8));
    for (int i = threadIdx.x; i < 256; i += kPlanThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t pref = s_prefix;
    for (int i = threadIdx.x; i < P; i += kPlanThreads) {
      const uint32_t kk = keys[i];
      if ((kk & hi_mask) == (pref & hi_mask)) atomicAdd(&hist[(kk >> shift) & 0xFF], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t rem = s_remaining;
      int digit = 255;
      for (; digit > 0; --digit) {
        if (hist[digit] >= rem) break;
        rem -= hist[digit];
      }
      s_prefix = pref | (static_cast<uint32_t>(digit) << shift);
      s_remaining = rem;
    }
    __syncthreads();
  }
  const uint32_t kth = s_prefix;
  const uint32_t ties_needed = s_remaining;  // how many keys equal to kth are kept
  // Flag: 1 if kept. Keys > kth are kept; keys == kth kept in ascending position until filled.
  for (int i = threadIdx.x; i < P; i += kPlanThreads) flag[i] = keys[i] > kth ? 1 : (keys[i] == kth ? 2 : 0);
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t left = ties_needed;
    for (int i = 0; i < P; ++i) {
      if (flag[i] == 2) {
        flag[i] = left > 0 ? 1 : 0;
        if (left > 0) --left;
      }
    }
  }
  __syncthreads();
  }
  // Block-wide exclusive scan over flags in chunks of kPlanThreads, emitting kept candidates in order.
  float kept = 0.f;
  int base = 0;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int c0 = 0; c0 < P; c0 += kPlanThreads) {
    const int i = c0 + threadIdx.x;
    const int f = (i < P && k > 0) ? flag[i] : 0;
    int incl = f;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += t;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int woff = 0, tot = 0;
    for (int w = 0; w < kPlanThreads / 32; ++w) {
      if (w < warp) woff += warp_tot[w];
      tot += warp_tot[w];
    }
    if (f) {
      const int pos = base + woff + incl - 1;
      const int tok = cand[(long)b * P + i];
      if (pos < k) {  // top-k: always; threshold: the first k (the cap) kept candidates
        upd[(long)b * T + npre + pos] = tok;
        rows[(long)b * T + npre + pos] = b * N + tok;
      }
      if (isfinite(sc[i])) kept += sc[i];
    }
    base += tot;
    __syncthreads();
  }
  if (use_thres) {
    // Pad the unused tail with the row's last kept candidate (the first candidate if none was
    // kept), as the sync-free threshold builder does (block.py:495-560): a duplicated row is
    // corrected twice with identical results, so the padding changes nothing.
    const int nk = min(base, k);
    const int fill = nk > 0 ? upd[(long)b * T + npre + nk - 1] : (P > 0 ? cand[(long)b * P] : 0);
    for (int pos = nk + threadIdx.x; pos < k; pos += kPlanThreads) {
      upd[(long)b * T + npre + pos] = fill;
      rows[(long)b * T + npre + pos] = b * N + fill;
    }
    if (threadIdx.x == 0 && counts != nullptr) counts[b] = base;
  }
  for (int i = threadIdx.x; i < npre; i += kPlanThreads) {
    const int tok = pre[(long)b * npre + i];
    upd[(long)b * T + i] = tok;
    rows[(long)b * T + i] = b * N + tok;
  }
  kept = block_sum<kPlanThreads>(kept, red);
  if (threadIdx.x == 0 && stats != nullptr) {
    stats[2 * b] = kept;
    stats[2 * b + 1] = full;
  }
}

void correction_plan_op(const at::Tensor& server, const at::Tensor& pre, const at::Tensor& cand,
                        c10::optional<at::Tensor> mobile, double ws, double wm, int64_t fusion,
                        c10::optional<at::Tensor> valid, int64_t k, at::Tensor& upd, at::Tensor& rows,
                        c10::optional<at::Tensor> stats, c10::optional<double> thres,
                        c10::optional<at::Tensor> counts) {
  TORCH_CHECK(server.scalar_type() == at::kFloat && server.dim() == 2 && server.is_contiguous(), "plan: server fp32 [B,N]");
  const int B = static_cast<int>(server.size(0)), N = static_cast<int>(server.size(1));
  TORCH_CHECK(cand.scalar_type() == at::kInt && cand.dim() == 2 && cand.size(0) == B && cand.is_contiguous(), "plan: cand int32 [B,P]");
  TORCH_CHECK(pre.scalar_type() == at::kInt && pre.dim() == 2 && pre.size(0) == B && pre.is_contiguous(), "plan: pre int32 [B,npre]");
  const int P = static_cast<int>(cand.size(1)), npre = static_cast<int>(pre.size(1));
  TORCH_CHECK(k >= 0 && k <= P, "plan: 0 <= k <= P");
  TORCH_CHECK(upd.scalar_type() == at::kInt && upd.numel() == (long)B * (npre + k), "plan: upd int32 [B, npre+k]");
  TORCH_CHECK(rows.scalar_type() == at::kInt && rows.numel() == (long)B * (npre + k), "plan: rows int32 [B*(npre+k)]");
  const float* mp = nullptr;
  if (mobile.has_value()) {
    TORCH_CHECK(mobile->scalar_type() == at::kFloat && mobile->numel() == (long)B * P, "plan: mobile fp32 [B,P]");
    mp = mobile->data_ptr<float>();
  }
  const uint8_t* vp = nullptr;
  if (valid.has_value()) {
    TORCH_CHECK(valid->scalar_type() == at::kBool && valid->numel() == (long)B * P, "plan: valid bool [B,P]");
    vp = reinterpret_cast<const uint8_t*>(valid->data_ptr());
  }
  float* sp = nullptr;
  if (stats.has_value()) {
    TORCH_CHECK(stats->scalar_type() == at::kFloat && stats->numel() >= 2L * B, "plan: stats fp32 [B,2]");
    sp = stats->data_ptr<float>();
  }
  int* cp = nullptr;
  if (counts.has_value()) {
    TORCH_CHECK(counts->scalar_type() == at::kInt && counts->numel() >= B, "plan: counts int32 [B]");
    cp = counts->data_ptr<int>();
  }
  const size_t smem = 3 * sizeof(uint32_t) * P;
  TORCH_CHECK(smem <= 190 * 1024, "plan: too many candidates");
  c10::cuda::CUDAGuard g(server.device());
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(correction_plan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  correction_plan_kernel<<<B, kPlanThreads, smem, at::cuda::getCurrentCUDAStream()>>>(
      server.data_ptr<float>(), N, pre.data_ptr<int>(), npre, cand.data_ptr<int>(), P, mp, static_cast<float>(ws),
      static_cast<float>(wm), static_cast<int>(fusion), vp, static_cast<int>(k), upd.data_ptr<int>(), rows.data_ptr<int>(), sp,
      thres.has_value() ? 1 : 0, thres.has_value() ? static_cast<float>(*thres) : 0.f, cp);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ pyramid decode
// Integer pyrUp matching OpenCV (5-tap [1 4 6 4 1] kernel on the zero-upsampled image, x4 gain):
// per axis, even output 2i = s[i-1] + 6 s[i] + s[i+1], odd 2i+1 = 4 s[i] + 4 s[i+1], with the
// left border mirrored (s[-1] = s[1]) and the last source sample giving s[n-2] + 7 s[n-1] and
// 8 s[n-1]; result = (sum + 32) >> 6. Optionally adds an int16 residual and clips to [0, 255].
__device__ __forceinline__ void pyr_taps(int o, int n, int (&idx)[3], int (&wt)[3]) {
  const int i = o >> 1;
  if ((o & 1) == 0) {
    if (i == n - 1) {
      idx[0] = n > 1 ? n - 2 : 0; wt[0] = 1; idx[1] = n - 1; wt[1] = 7; idx[2] = n - 1; wt[2] = 0;
    } else {
      idx[0] = i == 0 ? (n > 1 ? 1 : 0) : i - 1; wt[0] = 1;
      idx[1] = i; wt[1] = 6;
      idx[2] = i + 1; wt[2] = 1;
    }
  } else {
    if (i == n - 1) {
      idx[0] = i; wt[0] = 8; idx[1] = i; wt[1] = 0; idx[2] = i; wt[2] = 0;
    } else {
      idx[0] = i; wt[0] = 4; idx[1] = i + 1; wt[1] = 4; idx[2] = i + 1; wt[2] = 0;
    }
  }
}

__global__ void pyrup_add_kernel(const uint8_t* __restrict__ src, int h, int w, const int16_t* __restrict__ res,
                                 uint8_t* __restrict__ dst, int B, int C) {
  const int H = 2 * h, W = 2 * w;
  const long total = (long)B * H * W;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long b = i / ((long)H * W);
    const int rem = static_cast<int>(i - b * H * W);
    const int y = rem / W, x = rem - (rem / W) * W;
    int yi[3], yw[3], xi[3], xw[3];
    pyr_taps(y, h, yi, yw);
    pyr_taps(x, w, xi, xw);
    const uint8_t* sb = src + b * h * w * C;
    for (int c = 0; c < C; ++c) {
      int acc = 0;
#pragma unroll
      for (int a = 0; a < 3; ++a) {
        int rs = 0;
#pragma unroll
        for (int e = 0; e < 3; ++e) rs += xw[e] * sb[((long)yi[a] * w + xi[e]) * C + c];
        acc += yw[a] * rs;
      }
      int v = (acc + 32) >> 6;
      if (res != nullptr) v += res[i * C + c];
      dst[i * C + c] = static_cast<uint8_t>(min(255, max(0, v)));
    }
  }
}

void pyrup_add_op(const at::Tensor& src, c10::optional<at::Tensor> res, at::Tensor& dst) {
  TORCH_CHECK(src.scalar_type() == at::kByte && src.dim() == 4 && src.is_contiguous(), "pyrup: uint8 [B,h,w,C]");
  const int B = static_cast<int>(src.size(0)), h = static_cast<int>(src.size(1)), w = static_cast<int>(src.size(2)),
            C = static_cast<int>(src.size(3));
  TORCH_CHECK(dst.scalar_type() == at::kByte && dst.is_contiguous() && dst.size(1) == 2 * h && dst.size(2) == 2 * w &&
                  dst.size(3) == C, "pyrup: dst uint8 [B,2h,2w,C]");
  const int16_t* rp = nullptr;
  if (res.has_value()) {
    TORCH_CHECK(res->scalar_type() == at::kShort && res->is_contiguous() && res->numel() == dst.numel(), "pyrup: residual int16 like dst");
    rp = reinterpret_cast<const int16_t*>(res->data_ptr());
  }
  const long total = (long)B * 4 * h * w;
  if (total == 0) return;
  c10::cuda::CUDAGuard g(src.device());
  pyrup_add_kernel<<<static_cast<int>(std::min<long>((total + 255) / 256, num_sms() * 16L)), 256, 0,
                     at::cuda::getCurrentCUDAStream()>>>(src.data_ptr<uint8_t>(), h, w, rp, dst.data_ptr<uint8_t>(), B, C);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ segmentation head tail
// logits: fp32 [B, h, w, ldl] (first C channels valid). Bilinear upsample (align_corners=False,
// PyTorch's source-index rule) to [H, W] and argmax over channels -> uint8 labels.
__global__ void upsample_argmax_kernel(const float* __restrict__ logits, int h, int w, int ldl, int C, int H, int W,
                                       uint8_t* __restrict__ out, long total) {
  const float sy = static_cast<float>(h) / H, sx = static_cast<float>(w) / W;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const long b = i / ((long)H * W);
    const int rem = static_cast<int>(i - b * H * W);
    const int y = rem / W, x = rem - (rem / W) * W;
    float fy = fmaxf((y + 0.5f) * sy - 0.5f, 0.f);
    float fx = fmaxf((x + 0.5f) * sx - 0.5f, 0.f);
    int y0 = min(static_cast<int>(fy), h - 1), x0 = min(static_cast<int>(fx), w - 1);
    const int y1 = min(y0 + 1, h - 1), x1 = min(x0 + 1, w - 1);
    const float ly = fy - y0, lx = fx - x0;
    const float w00 = (1.f - ly) * (1.f - lx), w01 = (1.f - ly) * lx, w10 = ly * (1.f - lx), w11 = ly * lx;
    const float* p00 = logits + ((b * h + y0) * (long)w + x0) * ldl;
    const float* p01 = logits + ((b * h + y0) * (long)w + x1) * ldl;
    const float* p10 = logits + ((b * h + y1) * (long)w + x0) * ldl;
    const float* p11 = logits + ((b * h + y1) * (long)w + x1) * ldl;
    float best = -FLT_MAX;
    int arg = 0;
    for (int c = 0; c < C; ++c) {
      const float v = w00 * __ldg(p00 + c) + w01 * __ldg(p01 + c) + w10 * __ldg(p10 + c) + w11 * __ldg(p11 + c);
      if (v > best) { best = v; arg = c; }
    }
    out[i] = static_cast<uint8_t>(arg);
  }
}

void upsample_argmax_op(const at::Tensor& logits, int64_t C, int64_t H, int64_t W, at::Tensor& out) {
  TORCH_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 4 && logits.stride(3) == 1 && logits.is_contiguous(),
              "upsample_argmax: fp32 [B,h,w,ldl] contiguous");
  TORCH_CHECK(out.scalar_type() == at::kByte && out.is_contiguous(), "upsample_argmax: uint8 out");
  const int B = static_cast<int>(logits.size(0)), h = static_cast<int>(logits.size(1)), w = static_cast<int>(logits.size(2));
  const long total = (long)B * H * W;
  TORCH_CHECK(out.numel() == total && C <= 256 && C <= logits.size(3), "upsample_argmax: shapes");
  c10::cuda::CUDAGuard g(logits.device());
  upsample_argmax_kernel<<<static_cast<int>(std::min<long>((total + 255) / 256, num_sms() * 16L)), 256, 0,
                           at::cuda::getCurrentCUDAStream()>>>(logits.data_ptr<float>(), h, w, static_cast<int>(logits.size(3)),
                                                               static_cast<int>(C), static_cast<int>(H), static_cast<int>(W),
                                                               out.data_ptr<uint8_t>(), total);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ mean over rows
// x: [B, N, D] bf16 rows [start, N) averaged -> out bf16 [B, D] (written at out + b*ldo).
__global__ void mean_rows_kernel(const bf16* __restrict__ x, long ldx, int N, int start, int D, bf16* __restrict__ out,
                                 long ldo) {
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= D) return;
  float s = 0.f;
  for (int t = start; t < N; ++t) s += __bfloat162float(x[((long)b * N + t) * ldx + c]);
  out[(long)b * ldo + c] = __float2bfloat16_rn(s / (N - start));
}

void mean_rows_op(const at::Tensor& x, int64_t B, int64_t N, int64_t start, at::Tensor& out) {
  const int D = static_cast<int>(x.size(-1));
  TORCH_CHECK(x.scalar_type() == at::kBFloat16 && out.scalar_type() == at::kBFloat16, "mean_rows: bf16");
  c10::cuda::CUDAGuard g(x.device());
  mean_rows_kernel<<<dim3((D + 255) / 256, B), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), x.stride(-2), static_cast<int>(N), static_cast<int>(start), D,
      reinterpret_cast<bf16*>(out.data_ptr()), out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void head_mean_op(const at::Tensor& probs, int64_t B, int64_t H, int64_t N, at::Tensor& out) {
  TORCH_CHECK(probs.scalar_type() == at::kFloat && probs.numel() >= B * H * N, "head_mean: fp32 [B,H,N]");
  TORCH_CHECK(out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() == B * N, "head_mean: out fp32 [B,N]");
  c10::cuda::CUDAGuard g(probs.device());
  head_mean_kernel<<<static_cast<int>(std::max<long>(1, (B * N + 255) / 256)), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      probs.data_ptr<float>(), static_cast<int>(B), static_cast<int>(H), static_cast<int>(N), out.data_ptr<float>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// The FMA-pipe exp2 of the attention softmax, exposed for its accuracy test.
__global__ void exp2_poly_kernel(const float* __restrict__ x, float* __restrict__ y, long n) {
  const long i = blockIdx.x * static_cast<long>(blockDim.x) + threadIdx.x;
  if (i < n) y[i] = exp2_poly(x[i]);
}

void exp2_poly_op(const at::Tensor& x, at::Tensor& y) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kFloat && x.is_contiguous() && y.sizes() == x.sizes() &&
                  y.scalar_type() == at::kFloat && y.is_contiguous(), "exp2_poly: contiguous fp32 x, y");
  c10::cuda::CUDAGuard g(x.device());
  const long n = x.numel();
  if (n == 0) return;
  exp2_poly_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      x.data_ptr<float>(), y.data_ptr<float>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_elementwise_ops(pybind11::module_& m) {
  m.def("exp2_poly", &exp2_poly_op);
  m.def("head_mean", &head_mean_op);
  namespace py = pybind11;
  m.def("layernorm", &layernorm_op, py::arg("x"), py::arg("rows"), py::arg("w"), py::arg("b"), py::arg("eps"),
        py::arg("out"), py::arg("copy_out") = py::none(), py::arg("scale8") = py::none(), py::arg("rms") = false,
        py::arg("sf") = py::none());
  m.def("quant_rows_e4m3", &quant_rows_e4m3_op, py::arg("x"), py::arg("out"), py::arg("scale"));
  m.def("quant_rows_nvfp4", &quant_rows_nvfp4_op, py::arg("x"), py::arg("out"), py::arg("sf"), py::arg("scale"));
  m.def("add_", &add_inplace_op);
  m.def("row_sqdist", &row_sqdist_op, py::arg("a"), py::arg("b"), py::arg("out"));
  m.def("patch_im2col", &patch_im2col_op, py::arg("img"), py::arg("patch"), py::arg("mean"), py::arg("std"),
        py::arg("out"), py::arg("perm") = py::none());
  m.def("set_prefix", &set_prefix_op);
  m.def("gather_rows", &gather_rows_op);
  m.def("scatter_rows", &scatter_rows_op);
  m.def("cls_attn_pscore", &cls_attn_pscore_op, py::arg("q"), py::arg("k"), py::arg("B"), py::arg("N"), py::arg("H"),
        py::arg("Dh"), py::arg("scale"), py::arg("scratch"), py::arg("out"), py::arg("q_bstride") = -1);
  m.def("correction_plan", &correction_plan_op, py::arg("server"), py::arg("pre"), py::arg("cand"), py::arg("mobile"),
        py::arg("ws"), py::arg("wm"), py::arg("fusion"), py::arg("valid"), py::arg("k"), py::arg("upd"), py::arg("rows"),
        py::arg("stats") = py::none(), py::arg("thres") = py::none(), py::arg("counts") = py::none());
  m.def("pyrup_add", &pyrup_add_op);
  m.def("upsample_argmax", &upsample_argmax_op);
  m.def("mean_rows", &mean_rows_op);
}

}  // namespace appcorr
