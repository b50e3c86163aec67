// Sequence-parallel tensor-parallel row kernel: the owner-side half of the fused
// GEMM -> reduce-scatter and the producer side of the all-gather -> GEMM, over NVLink peer memory.
//
// Layout (appcorr_b200/parallel/tp.py): the residual stream is split by rows; rank r owns token
// rows [r*R, (r+1)*R). The row-parallel GEMMs (attention proj, MLP fc2) produce bf16 partial
// products; the reduce-scatter is finished here by the owner of each row, either
//   pull: every rank's GEMM writes its partial locally; the owner loads row i of every peer's
//         partial over NVLink (16-byte coalesced peer loads), or
//   push: the GEMM epilogue (csrc/gemm_sm100.cu, GemmEpilogue::rs_out) stores each partial row
//         into the owner's slot buffer over NVLink while the GEMM runs; the owner loads locally.
// After a barrier the owner runs this kernel, one CTA per (packed) row i:
//
//   reduce   acc = sum_src partial[src][i] + bias;  d = gamma * acc;  o = resid + d
//            out := o; increment bookkeeping on the owner's rows (aux := d | aux += d |
//            aux := (resid - resid2) + d)
//   or load  o = x[tok(i)]  (copy_out[i] := o)
//   then     optional LayerNorm / RMSNorm of o, quantised to e4m3 with one scale per row (or
//            kept bf16), stored into row i of EVERY rank's gather buffer (peer stores): the
//            all-gather that feeds the next column-parallel GEMM, fused into its producer.
//
// Rows whose token is owned by another rank return immediately, so the same launch serves the
// contiguous approximate pass (tok(i) = i) and the packed correction rows (tok(i) = rows[i]).
// Reference: none (the reference is single-GPU); the per-row math is that of the block epilogue
// (block.py:1146-1191) and LayerNorm.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <algorithm>
#include <cfloat>
#include <cstdlib>
#include <cuda_fp8.h>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;
constexpr int kSpThreads = 128;
constexpr int kSpMaxVec = 8;  // D <= 128 * 8 * 8 = 8192
constexpr int kSpMaxRanks = 8;

struct SpArgs {
  // rows
  int M;                    // packed rows
  const int* tok;           // packed row -> token row (nullptr: identity)
  int rows_per_rank, rank, world;
  int D;
  // reduce
  int reduce;               // 1: sum the partial rows; 0: load x[tok]
  const bf16* src[kSpMaxRanks];  // partial row i of source s at src[s] + (src_off[s] + i) * D:
  long src_off[kSpMaxRanks];     // local slots (push) or the peers' own partial buffers (pull)
  const bf16* bias;
  const bf16* gamma;        // nullptr: d = acc
  const bf16* resid;        // resid row = tok (resid_tok) or i
  long ldr;
  int resid_tok;
  const bf16* resid2;       // packed i (AUX_OUT_MINUS)
  long ldr2;
  bf16* out;                // out row = tok (out_tok) or i
  long ldo;
  int out_tok;
  bf16* aux;                // row tok
  long ldaux;
  int aux_mode;
  // load mode
  const bf16* x;            // row tok
  long ldx;
  bf16* copy_out;           // row i
  long ldc;
  // norm + all-gather
  const bf16* ln_w;         // nullptr: no norm / gather
  const bf16* ln_b;
  float eps;
  int rms;
  int fp8;                  // gather format: 0 bf16, 1 e4m3 + row scale, 2 NVFP4 (+ block scales)
  void* ag[kSpMaxRanks];    // gather buffers (row i), bf16, e4m3 or packed e2m1
  long ld_ag;               // elements (bf16 / e4m3) or bytes (NVFP4)
  float* ag_scale[kSpMaxRanks];
  uint8_t* ag_sf[kSpMaxRanks];  // NVFP4 block scales (blocked layout, K = D)
  int ag_self;              // 1: write only this rank's gather buffers (a bulk push follows)
};

__device__ __forceinline__ void sp_unpack8(const uint4& u, float (&v)[8]) {
  const uint32_t* w = &u.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = unpack_bf16x2(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 sp_pack8(const float (&v)[8]) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}
__device__ __forceinline__ uint32_t sp_e4m3x4(float a, float b, float c, float d) {
  const uint32_t lo = __nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
  const uint32_t hi = __nv_cvt_float2_to_fp8x2(make_float2(c, d), __NV_SATFINITE, __NV_E4M3);
  return lo | (hi << 16);
}

template <bool MAX>
__device__ __forceinline__ float sp_block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = MAX ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < kSpThreads / 32 ? red[lane] : (MAX ? 0.f : 0.f);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, t, o);
    t = MAX ? fmaxf(t, w) : t + w;
  }
  return t;
}

// NV: 16-byte vectors per thread (D <= 1024 * NV); W: ranks (partial sources). The finished row is
// held as packed bf16 (it is bf16-rounded anyway) to keep registers low.
template <int NV, int W>
__device__ __forceinline__ void sp_row_one(const SpArgs& a, int i, float* red) {
  const int tok = a.tok ? a.tok[i] : i;
  if (tok < 0 || tok / a.rows_per_rank != a.rank) return;  // another rank owns this row
  const int nvec = a.D >> 3;
  uint4 vb[NV];
  if (a.reduce) {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = threadIdx.x + k * kSpThreads;
      if (c >= nvec) continue;
      // issue the partial-row loads of every source before summing (peer loads in flight together)
      uint4 u[W];
#pragma unroll
      for (int s = 0; s < W; ++s) u[s] = reinterpret_cast<const uint4*>(a.src[s] + (a.src_off[s] + i) * a.D)[c];
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int s = 0; s < W; ++s) {
        float p[8];
        sp_unpack8(u[s], p);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += p[j];
      }
      if (a.bias) {
        float b[8];
        sp_unpack8(__ldg(reinterpret_cast<const uint4*>(a.bias) + c), b);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] += b[j];
      }
      float d[8], o[8];
      const long rr = a.resid_tok ? tok : i;
      float rs[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (a.resid) sp_unpack8(reinterpret_cast<const uint4*>(a.resid + rr * a.ldr)[c], rs);
      if (a.gamma) {
        float g[8];
        sp_unpack8(__ldg(reinterpret_cast<const uint4*>(a.gamma) + c), g);
#pragma unroll
        for (int j = 0; j < 8; ++j) d[j] = bf16_round(bf16_round(acc[j]) * g[j]);
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) d[j] = bf16_round(acc[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = bf16_round(rs[j] + d[j]);
      if (a.aux_mode != AUX_NONE) {
        uint4* ap = reinterpret_cast<uint4*>(a.aux + (long)tok * a.ldaux) + c;
        float x[8];
        if (a.aux_mode == AUX_SET) {
#pragma unroll
          for (int j = 0; j < 8; ++j) x[j] = d[j];
        } else if (a.aux_mode == AUX_ADD) {
          sp_unpack8(*ap, x);
#pragma unroll
          for (int j = 0; j < 8; ++j) x[j] += d[j];
        } else {
          float r2[8];
          sp_unpack8(reinterpret_cast<const uint4*>(a.resid2 + (long)i * a.ldr2)[c], r2);
#pragma unroll
          for (int j = 0; j < 8; ++j) x[j] = bf16_round(rs[j] - r2[j]) + d[j];
        }
        *ap = sp_pack8(x);
      }
      const long orow = a.out_tok ? tok : i;
      vb[k] = sp_pack8(o);
      reinterpret_cast<uint4*>(a.out + orow * a.ldo)[c] = vb[k];
    }
  } else {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = threadIdx.x + k * kSpThreads;
      if (c >= nvec) continue;
      vb[k] = reinterpret_cast<const uint4*>(a.x + (long)tok * a.ldx)[c];
      if (a.copy_out) reinterpret_cast<uint4*>(a.copy_out + (long)i * a.ldc)[c] = vb[k];
    }
  }
  if (a.ln_w == nullptr) return;
  // ---- LayerNorm / RMSNorm of the finished row, then the all-gather stores
  float s = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (threadIdx.x + k * kSpThreads < nvec) {
      float v[8];
      sp_unpack8(vb[k], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[j];
    }
  const float mean = a.rms ? 0.f : sp_block_reduce<false>(s, red) / a.D;
  float q = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k)
    if (threadIdx.x + k * kSpThreads < nvec) {
      float v[8];
      sp_unpack8(vb[k], v);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float dd = v[j] - mean;
        q += dd * dd;
      }
    }
  const float rstd = rsqrtf(sp_block_reduce<false>(q, red) / a.D + a.eps);
  float amax = 0.f;
#pragma unroll
  for (int k = 0; k < NV; ++k) {
    const int c = threadIdx.x + k * kSpThreads;
    if (c >= nvec) continue;
    float v[8], w[8], b[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    sp_unpack8(vb[k], v);
    sp_unpack8(__ldg(reinterpret_cast<const uint4*>(a.ln_w) + c), w);
    if (a.ln_b) sp_unpack8(__ldg(reinterpret_cast<const uint4*>(a.ln_b) + c), b);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[j] = (v[j] - mean) * rstd * w[j] + b[j];
      amax = fmaxf(amax, fabsf(bf16_round(v[j])));
    }
    vb[k] = sp_pack8(v);  // the normalised row, bf16-rounded (the bf16 path's GEMM operand)
  }
  if (a.fp8 == 2) {
    // NVFP4: 16-element blocks = vector pairs (c, c ^ 1) of neighbouring lanes; the four block
    // scales of a 64-element tile (lanes c..c+7) go out as one 4-byte store per rank
    amax = sp_block_reduce<true>(amax, red);
    const float rs = fmaxf(amax, 1e-12f) / kNvfp4RowDiv;
    const float inv_rs = 1.f / rs;
    if (threadIdx.x < W && (!a.ag_self || threadIdx.x == a.rank)) a.ag_scale[threadIdx.x][i] = rs;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = threadIdx.x + k * kSpThreads;
      const bool live = c < nvec;  // D % 64 == 0: a lane octet is live or dead as a whole
      float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (live) sp_unpack8(vb[k], v);
      float bm = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) bm = fmaxf(bm, fabsf(v[j]));
      bm = fmaxf(bm, __shfl_xor_sync(0xffffffffu, bm, 1));
      float mul;
      const uint32_t sb = nvfp4_block_scale(bm, inv_rs, rs, mul);
      const uint32_t pk = pack_e2m1x8(v, mul);
      const uint32_t s1 = __shfl_down_sync(0xffffffffu, sb, 2);
      const uint32_t s2 = __shfl_down_sync(0xffffffffu, sb, 4);
      const uint32_t s3 = __shfl_down_sync(0xffffffffu, sb, 6);
      if (!live) continue;
      const uint32_t sw = sb | (s1 << 8) | (s2 << 16) | (s3 << 24);
      const long so = nvfp4_sf_offset(i, c >> 1, a.D >> 6);
#pragma unroll
      for (int r = 0; r < W; ++r) {
        if (a.ag_self && r != a.rank) continue;
        reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(a.ag[r]) + (long)i * a.ld_ag)[c] = pk;
        if ((c & 7) == 0) *reinterpret_cast<uint32_t*>(a.ag_sf[r] + so) = sw;
      }
    }
  } else if (a.fp8) {
    amax = sp_block_reduce<true>(amax, red);
    const float sc = fmaxf(amax, 1e-12f) / 448.f;
    const float inv = 1.f / sc;
    if (threadIdx.x < W && (!a.ag_self || threadIdx.x == a.rank)) a.ag_scale[threadIdx.x][i] = sc;
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = threadIdx.x + k * kSpThreads;
      if (c >= nvec) continue;
      float v[8];
      sp_unpack8(vb[k], v);
      const uint2 pk = make_uint2(sp_e4m3x4(v[0] * inv, v[1] * inv, v[2] * inv, v[3] * inv),
                                  sp_e4m3x4(v[4] * inv, v[5] * inv, v[6] * inv, v[7] * inv));
#pragma unroll
      for (int r = 0; r < W; ++r)
        if (!a.ag_self || r == a.rank)
          reinterpret_cast<uint2*>(reinterpret_cast<uint8_t*>(a.ag[r]) + (long)i * a.ld_ag)[c] = pk;
    }
  } else {
#pragma unroll
    for (int k = 0; k < NV; ++k) {
      const int c = threadIdx.x + k * kSpThreads;
      if (c >= nvec) continue;
#pragma unroll
      for (int r = 0; r < W; ++r)
        if (!a.ag_self || r == a.rank)
          reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(a.ag[r]) + (long)i * a.ld_ag)[c] = vb[k];
    }
  }
}

// Persistent over rows: a bounded grid (about two CTAs per SM) walks the rows, so the kernel leaves
// SM room for the GEMM of the other micro-batch instead of flooding every SM with row CTAs.
template <int NV, int W>
__global__ void __launch_bounds__(kSpThreads) sp_row_kernel(SpArgs a, int row0, int row_end) {
  __shared__ float red[kSpThreads / 32];
  for (int i = row0 + blockIdx.x; i < row_end; i += gridDim.x) sp_row_one<NV, W>(a, i, red);
}

template <typename T = void>
static T* sp_opt(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

void sp_row_op(int64_t M, c10::optional<at::Tensor> tok, int64_t rows_per_rank, int64_t rank, int64_t world, int64_t D,
               std::vector<int64_t> src, std::vector<int64_t> src_off, c10::optional<at::Tensor> bias,
               c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> resid, bool resid_tok,
               c10::optional<at::Tensor> resid2, c10::optional<at::Tensor> out, bool out_tok,
               c10::optional<at::Tensor> aux, int64_t aux_mode, c10::optional<at::Tensor> x,
               c10::optional<at::Tensor> copy_out, c10::optional<at::Tensor> ln_w, c10::optional<at::Tensor> ln_b,
               double eps, bool rms, int64_t fp8, std::vector<int64_t> ag, int64_t ld_ag, std::vector<int64_t> ag_scale,
               std::vector<int64_t> ag_sf, bool ag_self) {
  TORCH_CHECK(D % 8 == 0 && D <= kSpThreads * kSpMaxVec * 8, "sp_row: D % 8 == 0 and D <= 8192");
  TORCH_CHECK(world >= 1 && world <= kSpMaxRanks, "sp_row: 1..8 ranks");
  SpArgs a{};
  a.M = static_cast<int>(M);
  a.tok = sp_opt<const int>(tok);
  a.rows_per_rank = static_cast<int>(rows_per_rank);
  a.rank = static_cast<int>(rank);
  a.world = static_cast<int>(world);
  a.D = static_cast<int>(D);
  a.reduce = src.empty() ? 0 : 1;
  if (a.reduce) {
    TORCH_CHECK(out.has_value(), "sp_row: reduce needs out");
    TORCH_CHECK(static_cast<int64_t>(src.size()) == world && src_off.size() == src.size(),
                "sp_row: one partial source (and row offset) per rank");
    for (int r = 0; r < world; ++r) {
      a.src[r] = reinterpret_cast<const bf16*>(src[r]);
      a.src_off[r] = src_off[r];
    }
    a.bias = sp_opt<const bf16>(bias);
    a.gamma = sp_opt<const bf16>(gamma);
    a.resid = sp_opt<const bf16>(resid);
    a.ldr = resid.has_value() ? resid->stride(0) : 0;
    a.resid_tok = resid_tok ? 1 : 0;
    a.resid2 = sp_opt<const bf16>(resid2);
    a.ldr2 = resid2.has_value() ? resid2->stride(0) : 0;
    a.out = sp_opt<bf16>(out);
    a.ldo = out->stride(0);
    a.out_tok = out_tok ? 1 : 0;
    a.aux = sp_opt<bf16>(aux);
    a.ldaux = aux.has_value() ? aux->stride(0) : 0;
    a.aux_mode = aux.has_value() ? static_cast<int>(aux_mode) : AUX_NONE;
    if (a.aux_mode == AUX_OUT_MINUS) TORCH_CHECK(a.resid2 && a.resid, "sp_row: AUX_OUT_MINUS needs resid, resid2");
  } else {
    TORCH_CHECK(x.has_value(), "sp_row: load mode needs x");
    a.x = sp_opt<const bf16>(x);
    a.ldx = x->stride(0);
    a.copy_out = sp_opt<bf16>(copy_out);
    a.ldc = copy_out.has_value() ? copy_out->stride(0) : 0;
  }
  a.ln_w = sp_opt<const bf16>(ln_w);
  a.ln_b = sp_opt<const bf16>(ln_b);
  a.eps = static_cast<float>(eps);
  a.rms = rms ? 1 : 0;
  TORCH_CHECK(fp8 >= 0 && fp8 <= 2, "sp_row: gather format 0 (bf16), 1 (e4m3) or 2 (nvfp4)");
  a.fp8 = static_cast<int>(fp8);
  a.ag_self = ag_self ? 1 : 0;
  if (a.ln_w) {
    TORCH_CHECK(static_cast<int64_t>(ag.size()) == world, "sp_row: one gather buffer per rank");
    for (int r = 0; r < world; ++r) a.ag[r] = reinterpret_cast<void*>(ag[r]);
    a.ld_ag = ld_ag;
    if (fp8) {
      TORCH_CHECK(static_cast<int64_t>(ag_scale.size()) == world, "sp_row: one scale buffer per rank");
      for (int r = 0; r < world; ++r) a.ag_scale[r] = reinterpret_cast<float*>(ag_scale[r]);
    }
    if (fp8 == 2) {
      TORCH_CHECK(D % 64 == 0 && static_cast<int64_t>(ag_sf.size()) == world && ld_ag % 16 == 0,
                  "sp_row: nvfp4 gather needs D % 64 == 0, one block-scale buffer per rank, 16-byte rows");
      for (int r = 0; r < world; ++r) a.ag_sf[r] = reinterpret_cast<uint8_t*>(ag_sf[r]);
    }
  }
  if (M == 0) return;
  // contiguous rows (no token map): only this rank's block [rank*R, (rank+1)*R) is visited
  int row0 = 0, nrows = static_cast<int>(M);
  if (a.tok == nullptr) {
    row0 = static_cast<int>(std::min<int64_t>(M, rank * rows_per_rank));
    nrows = static_cast<int>(std::min<int64_t>(M, (rank + 1) * rows_per_rank)) - row0;
    if (nrows <= 0) return;
  }
  const int nv = (static_cast<int>(D) / 8 + kSpThreads - 1) / kSpThreads;
  auto st = at::cuda::getCurrentCUDAStream();
  const int row_end = row0 + nrows;
  static const int ctas_per_sm = [] {
    const char* e = std::getenv("APPCORR_SP_CTAS_PER_SM");
    return e ? std::max(1, std::atoi(e)) : 2;
  }();
  nrows = std::min(nrows, ctas_per_sm * num_sms());
#define APPCORR_SP_LAUNCH_W(NV)                                                             \
  switch (world) {                                                                          \
    case 1: sp_row_kernel<NV, 1><<<nrows, kSpThreads, 0, st>>>(a, row0, row_end); break;             \
    case 2: sp_row_kernel<NV, 2><<<nrows, kSpThreads, 0, st>>>(a, row0, row_end); break;             \
    case 4: sp_row_kernel<NV, 4><<<nrows, kSpThreads, 0, st>>>(a, row0, row_end); break;             \
    case 8: sp_row_kernel<NV, 8><<<nrows, kSpThreads, 0, st>>>(a, row0, row_end); break;             \
    default: TORCH_CHECK(false, "sp_row: world must be 1, 2, 4 or 8");                      \
  }
  if (nv <= 1) { APPCORR_SP_LAUNCH_W(1) }
  else if (nv <= 2) { APPCORR_SP_LAUNCH_W(2) }
  else if (nv <= 4) { APPCORR_SP_LAUNCH_W(4) }
  else { APPCORR_SP_LAUNCH_W(8) }
#undef APPCORR_SP_LAUNCH_W
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ row push
// Reduce-scatter, sending half: after a row-parallel GEMM wrote this rank's partial rows into its
// own slot `rank` of the symmetric slot buffer [world, M, D], every row owned by another rank is
// copied into slot `rank` of the owner's buffer (fully coalesced 16-byte peer stores, one row per
// CTA; remote stores are posted writes, so NVLink carries them without a read round trip). Rows
// are visited in an order rotated by the rank so that all peers' links are loaded at once. After
// a barrier each owner reduces its rows from local memory (sp_row with the slot sources).
struct PushArgs {
  const uint4* src;         // this rank's slot (packed rows, D/8 vectors each)
  uint4* dst[kSpMaxRanks];  // every rank's slot `rank` (same packed row index)
  const int* tok;           // packed row -> token row (nullptr: identity)
  int M, nvec, rows_per_rank, rank, world;
};

__global__ void __launch_bounds__(kSpThreads) sp_push_rows_kernel(PushArgs a) {
  for (int j = blockIdx.x; j < a.M; j += gridDim.x) {
    const int i = (j + a.rank * (a.M / max(a.world, 1))) % a.M;  // rotated start per rank
    const int tok = a.tok ? a.tok[i] : i;
    if (tok < 0) continue;
    const int owner = tok / a.rows_per_rank;
    if (owner == a.rank || owner >= a.world) continue;
    const uint4* s = a.src + (long)i * a.nvec;
    uint4* d = a.dst[owner] + (long)i * a.nvec;
    for (int c = threadIdx.x; c < a.nvec; c += kSpThreads) d[c] = s[c];
  }
}

void sp_push_rows_op(int64_t src, std::vector<int64_t> dst, c10::optional<at::Tensor> tok, int64_t M, int64_t D,
                     int64_t rows_per_rank, int64_t rank) {
  const int world = static_cast<int>(dst.size());
  TORCH_CHECK(world >= 1 && world <= kSpMaxRanks && D % 8 == 0, "sp_push_rows: 1..8 ranks, D % 8 == 0");
  TORCH_CHECK((src & 15) == 0, "sp_push_rows: 16-byte aligned source");
  PushArgs a{};
  a.src = reinterpret_cast<const uint4*>(src);
  for (int r = 0; r < world; ++r) {
    TORCH_CHECK((dst[r] & 15) == 0, "sp_push_rows: 16-byte aligned destinations");
    a.dst[r] = reinterpret_cast<uint4*>(dst[r]);
  }
  a.tok = sp_opt<const int>(tok);
  a.M = static_cast<int>(M);
  a.nvec = static_cast<int>(D / 8);
  a.rows_per_rank = static_cast<int>(rows_per_rank);
  a.rank = static_cast<int>(rank);
  a.world = world;
  if (M == 0 || world == 1) return;
  const int grid = static_cast<int>(std::min<int64_t>(M, 4 * num_sms()));
  sp_push_rows_kernel<<<grid, kSpThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ all-gather push
// All-gather, sending half, for the contiguous row block [r0, r1) of this rank: the row kernel
// wrote the gathered operand of these rows into this rank's own gather buffers only (local
// stores); this kernel copies them into every peer's buffers at the same offsets with 16-byte
// peer stores: the packed rows (one contiguous byte range), the fp32 row scales, and for NVFP4
// the block scales. In the blocked scale layout a 16-byte chunk holds one k-group of rows
// {c, c+32, c+64, c+96} of a 128-row tile; chunks whose four rows are all this rank's go out
// whole, chunks shared with a neighbour's rows word by word.
struct AgPushArgs {
  const uint8_t* rows_src;   // local gather buffer
  uint8_t* rows_dst[kSpMaxRanks];
  long rows_lo, rows_bytes;  // byte range of the rows (16-byte aligned)
  const float* rs_src;       // local row scales (nullptr: none)
  float* rs_dst[kSpMaxRanks];
  int r0, r1;
  const uint8_t* sf_src;     // local block scales (nullptr: none)
  uint8_t* sf_dst[kSpMaxRanks];
  int sf_kt;                 // 64-element groups per row (D / 64)
  int t0, t1;                // 128-row tiles touched by [r0, r1)
  int rank, world;
};

__global__ void __launch_bounds__(kSpThreads) sp_push_ag_kernel(AgPushArgs a) {
  const long nrow16 = a.rows_bytes >> 4;
  const long nsf16 = a.sf_src ? (long)(a.t1 - a.t0 + 1) * a.sf_kt * 32 : 0;  // 16-byte chunks
  const long nrs = a.rs_src ? (a.r1 - a.r0) : 0;
  const long per_peer = nrow16 + nsf16 + nrs;
  const long total = per_peer * (a.world - 1);
  for (long w = blockIdx.x * (long)blockDim.x + threadIdx.x; w < total; w += (long)gridDim.x * blockDim.x) {
    const int pk = static_cast<int>(w / per_peer);
    const int peer = (a.rank + 1 + pk) % a.world;  // rotated so every link is busy
    long j = w - (long)pk * per_peer;
    if (j < nrow16) {
      const long off = a.rows_lo + (j << 4);
      *reinterpret_cast<uint4*>(a.rows_dst[peer] + off) = *reinterpret_cast<const uint4*>(a.rows_src + off);
      continue;
    }
    j -= nrow16;
    if (j < nsf16) {
      const long base = (long)a.t0 * a.sf_kt * 512;
      const long off = base + (j << 4);
      const int tile = a.t0 + static_cast<int>(j / ((long)a.sf_kt * 32));
      const int c = static_cast<int>(j & 31);
      const int row0 = tile * 128 + c;
      if (row0 >= a.r0 && row0 + 96 < a.r1) {
        *reinterpret_cast<uint4*>(a.sf_dst[peer] + off) = *reinterpret_cast<const uint4*>(a.sf_src + off);
      } else {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int row = row0 + 32 * q;
          if (row >= a.r0 && row < a.r1)
            *reinterpret_cast<uint32_t*>(a.sf_dst[peer] + off + 4 * q) =
                *reinterpret_cast<const uint32_t*>(a.sf_src + off + 4 * q);
        }
      }
      continue;
    }
    j -= nsf16;
    a.rs_dst[peer][a.r0 + j] = a.rs_src[a.r0 + j];
  }
}

void sp_push_ag_op(std::vector<int64_t> rows, int64_t row_bytes, int64_t r0, int64_t r1, std::vector<int64_t> rs,
                   std::vector<int64_t> sf, int64_t sf_kt, int64_t rank) {
  const int world = static_cast<int>(rows.size());
  TORCH_CHECK(world >= 1 && world <= kSpMaxRanks, "sp_push_ag: 1..8 ranks");
  TORCH_CHECK(row_bytes % 16 == 0, "sp_push_ag: row bytes a multiple of 16");
  if (world == 1 || r1 <= r0) return;
  AgPushArgs a{};
  a.rows_src = reinterpret_cast<const uint8_t*>(rows[rank]);
  for (int r = 0; r < world; ++r) a.rows_dst[r] = reinterpret_cast<uint8_t*>(rows[r]);
  a.rows_lo = r0 * row_bytes;
  a.rows_bytes = (r1 - r0) * row_bytes;
  a.r0 = static_cast<int>(r0);
  a.r1 = static_cast<int>(r1);
  if (!rs.empty()) {
    TORCH_CHECK(static_cast<int>(rs.size()) == world, "sp_push_ag: one row-scale buffer per rank");
    a.rs_src = reinterpret_cast<const float*>(rs[rank]);
    for (int r = 0; r < world; ++r) a.rs_dst[r] = reinterpret_cast<float*>(rs[r]);
  }
  if (!sf.empty()) {
    TORCH_CHECK(static_cast<int>(sf.size()) == world && sf_kt > 0, "sp_push_ag: one block-scale buffer per rank");
    a.sf_src = reinterpret_cast<const uint8_t*>(sf[rank]);
    for (int r = 0; r < world; ++r) a.sf_dst[r] = reinterpret_cast<uint8_t*>(sf[r]);
    a.sf_kt = static_cast<int>(sf_kt);
    a.t0 = static_cast<int>(r0 / 128);
    a.t1 = static_cast<int>((r1 - 1) / 128);
  }
  a.rank = static_cast<int>(rank);
  a.world = world;
  const long per_peer = (a.rows_bytes >> 4) + (a.sf_src ? (long)(a.t1 - a.t0 + 1) * a.sf_kt * 32 : 0) + (a.rs_src ? r1 - r0 : 0);
  const long total = per_peer * (world - 1);
  const int grid = static_cast<int>(std::min<long>((total + kSpThreads - 1) / kSpThreads, 4L * num_sms()));
  sp_push_ag_kernel<<<grid, kSpThreads, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_sp_ops(pybind11::module_& m) {
  m.def("sp_push_rows", &sp_push_rows_op);
  m.def("sp_push_ag", &sp_push_ag_op);
  namespace py = pybind11;
  m.def("sp_row", &sp_row_op, py::arg("M"), py::arg("tok"), py::arg("rows_per_rank"), py::arg("rank"),
        py::arg("world"), py::arg("D"), py::arg("src"), py::arg("src_off"), py::arg("bias"), py::arg("gamma"),
        py::arg("resid"), py::arg("resid_tok"), py::arg("resid2"), py::arg("out"), py::arg("out_tok"),
        py::arg("aux"), py::arg("aux_mode"), py::arg("x"), py::arg("copy_out"), py::arg("ln_w"), py::arg("ln_b"),
        py::arg("eps"), py::arg("rms"), py::arg("fp8"), py::arg("ag"), py::arg("ld_ag"), py::arg("ag_scale"),
        py::arg("ag_sf") = std::vector<int64_t>{}, py::arg("ag_self") = false);
}

}  // namespace appcorr
