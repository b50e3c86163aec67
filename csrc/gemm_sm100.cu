// Persistent tcgen05 GEMM for sm_100a with fused epilogues.
//
// C[M, N] = A[M, K] * B[N, K]^T with bf16 operands and fp32 accumulation in TMEM. A is the
// activation matrix (row-major, K contiguous) and B an nn.Linear weight (row-major [out, in]),
// so both operands are K-major.
//
// Structure (one CTA per SM, 10 warps; 14 for NVFP4):
//   warp 0      TMA producer: streams 128xBK A tiles and BNxBK B tiles into a STAGES-deep ring
//               of 128-byte-swizzled shared-memory buffers, signalling `full[s]` by tx-count.
//   warp 1      MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16) into one of two
//               TMEM accumulators, commits `empty[s]` per stage and `tfull[acc]` per tile.
//   warps 2..9  epilogue: tcgen05.ld of the accumulator (one TMEM lane = one output row per
//               thread, two warps per lane quarter splitting the columns), fused elementwise
//               work, direct global stores; then `tempty[acc]`.
// Two accumulators let the epilogue of tile t overlap the main loop of tile t+1.
//
// The fused epilogues replace the separate elementwise launches of the reference block
// (appcorr/models/dinov3/layers/block.py:312-349 approx, :943-1191 correct):
//   EPI_BF16 / EPI_F32  bias add (+ optional output row map, e.g. patch-embed into token rows)
//   EPI_GELU            fc1 + exact GELU (Mlp, layers/ffn_layers.py:24-49)
//   EPI_SWIGLU          w1||w2 interleaved in 128-row blocks -> silu(x1) * x2 (ffn_layers.py:60-104,
//                       the Triton SwiGLU epilogue token_update.py:620-669)
//   EPI_RESID           out = resid + gamma * (acc + bias) with an optional increment side output
//                       (LayerScale + residual, token_update.py:11-60; blocks_out_sum bookkeeping
//                       block.py:333,342,1177-1179; active-row scatter token_update.py:257-347)
//   EPI_QKV             qkv + bias, RoPE on q/k of patch tokens, split into q / k-cache / v-cache
//                       with a scatter row map (attention.py:215-240,393-454; rope.py:121-184)
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cudaTypedefs.h>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kThreads = 192;

template <int BN>
struct TmemCols {
  static constexpr uint32_t value = (2 * BN <= 32) ? 32 : (2 * BN <= 64) ? 64 : (2 * BN <= 128) ? 128
                                    : (2 * BN <= 256) ? 256 : 512;
};

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb) {
  // Grouped raster: walk 16 M-tiles for every N-tile so a weight tile is reused from L2.
  constexpr int G = 16;
  const int per_group = G * num_n;
  const int group = tile / per_group;
  const int first_m = group * G;
  const int gsz = min(G, num_m - first_m);
  const int r = tile - group * per_group;
  mb = first_m + r % gsz;
  nb = r / gsz;
}

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = __ldg(q + i);
    float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
    v[8 * i + 0] = a.x; v[8 * i + 1] = a.y; v[8 * i + 2] = b.x; v[8 * i + 3] = b.y;
    v[8 * i + 4] = c.x; v[8 * i + 5] = c.y; v[8 * i + 6] = d.x; v[8 * i + 7] = d.y;
  }
}

__device__ __forceinline__ void load_bf16x32_plain(const __nv_bfloat16* p, float (&v)[32]) {
  const uint4* q = reinterpret_cast<const uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u = q[i];
    float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
    v[8 * i + 0] = a.x; v[8 * i + 1] = a.y; v[8 * i + 2] = b.x; v[8 * i + 3] = b.y;
    v[8 * i + 4] = c.x; v[8 * i + 5] = c.y; v[8 * i + 6] = d.x; v[8 * i + 7] = d.y;
  }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* p, const float (&v)[32]) {
  uint4* q = reinterpret_cast<uint4*>(p);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u;
    u.x = pack_bf16x2(v[8 * i + 0], v[8 * i + 1]);
    u.y = pack_bf16x2(v[8 * i + 2], v[8 * i + 3]);
    u.z = pack_bf16x2(v[8 * i + 4], v[8 * i + 5]);
    u.w = pack_bf16x2(v[8 * i + 6], v[8 * i + 7]);
    q[i] = u;
  }
}

__device__ __forceinline__ void store_f32x32(float* p, const float (&v)[32]) {
  float4* q = reinterpret_cast<float4*>(p);
#pragma unroll
  for (int i = 0; i < 8; ++i) q[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
}

__device__ __forceinline__ void acc_to_float(const uint32_t (&r)[32], float (&v)[32]) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ void add_bias(float (&v)[32], const __nv_bfloat16* bias, int n) {
  if (bias == nullptr) return;
  float b[32];
  load_bf16x32(bias + n, b);
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] += b[j];
}

// FP8 operands: fold the per-row activation scale and per-column weight scale into the accumulator.
__device__ __forceinline__ void scale_acc(float (&v)[32], const GemmEpilogue& ep, float row_scale, int n) {
  if (ep.a_scale == nullptr) return;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(ep.b_scale + n) + i);
    v[4 * i + 0] *= row_scale * w.x;
    v[4 * i + 1] *= row_scale * w.y;
    v[4 * i + 2] *= row_scale * w.z;
    v[4 * i + 3] *= row_scale * w.w;
  }
}

// Epilogue for one 128 x BN accumulator; each thread owns one row (`m`, possibly >= M).
// part / nparts: this warp takes every nparts-th 32-column chunk (several warps share a lane quarter).
template <int BN, int EPI>
__device__ __forceinline__ void run_epilogue(uint32_t taddr, int m, int n0, const GemmShape& shp,
                                             const GemmEpilogue& ep, int part = 0, int nparts = 1) {
  const bool row_ok = m < shp.M;
  const float rs = (ep.a_scale != nullptr && row_ok) ? ep.a_scale[m] : 1.f;
  if constexpr (EPI == EPI_SWIGLU) {
    // Tile columns [0,BN/2) hold w1 rows, [BN/2,BN) the matching w2 rows.
    constexpr int H = BN / 2;
    const int nout0 = n0 / 2;
    const int orow = row_ok ? (ep.out_rows ? ep.out_rows[m] : m) : -1;
#pragma unroll 1
    for (int c = part; c < H / 32; c += nparts) {
      uint32_t r1[32], r2[32];
      tmem_ld32(taddr + c * 32, r1);
      tmem_ld32(taddr + H + c * 32, r2);
      tmem_wait_ld();
      if (orow < 0) continue;
      float a[32], g[32];
      acc_to_float(r1, a);
      acc_to_float(r2, g);
      scale_acc(a, ep, rs, n0 + c * 32);
      scale_acc(g, ep, rs, n0 + H + c * 32);
      add_bias(a, ep.bias, n0 + c * 32);
      add_bias(g, ep.bias, n0 + H + c * 32);
      float h[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float x1 = bf16_round(a[j]);
        const float x2 = bf16_round(g[j]);
        h[j] = bf16_round(silu(x1)) * x2;
      }
      store_bf16x32(reinterpret_cast<__nv_bfloat16*>(ep.out) + (long)orow * ep.ldo + nout0 + c * 32, h);
    }
  } else if constexpr (EPI == EPI_QKV) {
    const int kvd = ep.kv_dim > 0 ? ep.kv_dim : ep.dim;
    const int which = n0 < ep.dim ? 0 : (n0 < ep.dim + kvd ? 1 : 2);  // q / k / v (tiles never straddle)
    const int c0 = which == 0 ? n0 : (which == 1 ? n0 - ep.dim : n0 - ep.dim - kvd);
    const long ldkv = ep.ld_kv > 0 ? ep.ld_kv : ep.ld_qkv;
    int tok = 0, kvrow = 0;
    if (row_ok) {
      tok = ep.tok_idx ? ep.tok_idx[m] : (m % ep.seq_len);
      kvrow = ep.kv_rows ? ep.kv_rows[m] : m;
    }
    __nv_bfloat16* dst = nullptr;
    if (row_ok) {
      if (which == 0) dst = ep.q_out + (long)m * ep.ld_qkv;
      else if (which == 1) dst = ep.k_out + (long)kvrow * ldkv;
      else dst = ep.v_out + (long)kvrow * ldkv;
      if (kvrow < 0 && which != 0) dst = nullptr;
    }
    if (which == 2) {
#pragma unroll 1
      for (int c = part; c < BN / 32; c += nparts) {
        uint32_t r[32];
        tmem_ld32(taddr + c * 32, r);
        tmem_wait_ld();
        if (dst == nullptr) continue;
        float v[32];
        acc_to_float(r, v);
        scale_acc(v, ep, rs, n0 + c * 32);
        add_bias(v, ep.bias, n0 + c * 32);
        store_bf16x32(dst + c0 + c * 32, v);
      }
    } else {
      const int Dh = ep.head_dim;
      const int half = Dh >> 1;
      const bool rope = row_ok && ep.rope_sin != nullptr && tok >= ep.n_prefix;
      const int rrow = tok - ep.n_prefix;
      int it = 0;
#pragma unroll 1
      for (int hb = 0; hb < BN; hb += Dh) {
#pragma unroll 1
        for (int c = 0; c < half; c += 32) {
          if (it++ % nparts != part) continue;
          uint32_t rl[32], rh[32];
          tmem_ld32(taddr + hb + c, rl);
          tmem_ld32(taddr + hb + half + c, rh);
          tmem_wait_ld();
          if (dst == nullptr) continue;
          float lo[32], hi[32];
          acc_to_float(rl, lo);
          acc_to_float(rh, hi);
          scale_acc(lo, ep, rs, n0 + hb + c);
          scale_acc(hi, ep, rs, n0 + hb + half + c);
          add_bias(lo, ep.bias, n0 + hb + c);
          add_bias(hi, ep.bias, n0 + hb + half + c);
          if (rope) {
            // DINOv3 RoPE tables repeat their first half (angles tiled twice), so the pair
            // (d, d + half) shares one sin / cos value; read them as float4 vectors.
            const float4* sn = reinterpret_cast<const float4*>(ep.rope_sin + (long)rrow * Dh + c);
            const float4* cs = reinterpret_cast<const float4*>(ep.rope_cos + (long)rrow * Dh + c);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 s4 = __ldg(sn + j4), c4 = __ldg(cs + j4);
              const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
              const float cv[4] = {c4.x, c4.y, c4.z, c4.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int j = 4 * j4 + e;
                const float xl = bf16_round(lo[j]);
                const float xh = bf16_round(hi[j]);
                lo[j] = xl * cv[e] - xh * sv[e];
                hi[j] = xh * cv[e] + xl * sv[e];
              }
            }
          }
          store_bf16x32(dst + c0 + hb + c, lo);
          store_bf16x32(dst + c0 + hb + half + c, hi);
        }
      }
    }
  } else {
    int orow = -1, rrow = -1, arow = -1;
    if (row_ok) {
      orow = ep.out_rows ? ep.out_rows[m] : m;
      if constexpr (EPI == EPI_RESID) {
        rrow = ep.resid_rows ? ep.resid_rows[m] : m;
        arow = ep.aux_rows ? ep.aux_rows[m] : orow;
      }
    }
#pragma unroll 1
    for (int c = part; c < BN / 32; c += nparts) {
      uint32_t r[32];
      tmem_ld32(taddr + c * 32, r);
      tmem_wait_ld();
      const int n = n0 + c * 32;
      if (orow < 0 || n >= shp.N) continue;
      float v[32];
      acc_to_float(r, v);
      scale_acc(v, ep, rs, n);
      add_bias(v, ep.bias, n);
      if constexpr (EPI == EPI_F32) {
        store_f32x32(reinterpret_cast<float*>(ep.out) + (long)orow * ep.ldo + n, v);
      } else if constexpr (EPI == EPI_BF16) {
        if (ep.rs_out[0] != nullptr) {  // fused reduce-scatter: partial row to its owner's slot
          const int owner = orow / ep.rs_rows_per_rank;
          store_bf16x32(ep.rs_out[owner] + ((long)ep.rs_rank * ep.rs_slot_rows + m) * ep.ldo + n, v);
        } else {
          store_bf16x32(reinterpret_cast<__nv_bfloat16*>(ep.out) + (long)orow * ep.ldo + n, v);
        }
      } else if constexpr (EPI == EPI_GELU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_erf(bf16_round(v[j]));
        store_bf16x32(reinterpret_cast<__nv_bfloat16*>(ep.out) + (long)orow * ep.ldo + n, v);
      } else if constexpr (EPI == EPI_RESID) {
        float gm[32], rs[32];
        load_bf16x32(ep.gamma + n, gm);
        load_bf16x32_plain(ep.resid + (long)rrow * ep.ldr + n, rs);
        float d[32], o[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          d[j] = bf16_round(bf16_round(v[j]) * gm[j]);
          o[j] = rs[j] + d[j];
        }
        if (ep.aux_mode != AUX_NONE && arow >= 0) {
          __nv_bfloat16* ap = ep.aux + (long)arow * ep.ldaux + n;
          float a[32];
          if (ep.aux_mode == AUX_SET) {
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = d[j];
          } else if (ep.aux_mode == AUX_ADD) {
            load_bf16x32_plain(ap, a);
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = a[j] + d[j];
          } else {
            float r2[32];
            load_bf16x32_plain(ep.resid2 + (long)m * ep.ldr2 + n, r2);
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = bf16_round(rs[j] - r2[j]) + d[j];
          }
          store_bf16x32(ap, a);
        }
        store_bf16x32(reinterpret_cast<__nv_bfloat16*>(ep.out) + (long)orow * ep.ldo + n, o);
      }
    }
  }
}

// ------------------------------------------------------------ early-release epilogue
// With one accumulator (NVFP4, 128 x 256 tiles: the scale slots leave no room for a second) the
// MMA warp idles while the epilogue runs, and an NVFP4 tile's main loop (16 stages at K = 4096)
// is only a few microseconds long. So every thread first drains its BN / 64 chunks of 32
// columns into registers -- scaled, biased and rounded to bf16, which every bf16 epilogue does
// first anyway -- and releases the accumulator; the stores and the fused elementwise work then
// overlap the next tile's main loop. Each warp of a lane-quarter pair takes every other chunk
// (SwiGLU: matching w1 / w2 chunks; QKV: matching rotate-half chunks of a head).
__device__ __forceinline__ uint4 ldg_u4(const __nv_bfloat16* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
__device__ __forceinline__ uint4 ld_u4(const __nv_bfloat16* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ void st_u4(__nv_bfloat16* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }
__device__ __forceinline__ void unpack8(uint4 u, float (&f)[8]) {
  const float2 a = unpack_bf16x2(u.x), b = unpack_bf16x2(u.y), c = unpack_bf16x2(u.z), d = unpack_bf16x2(u.w);
  f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y; f[4] = c.x; f[5] = c.y; f[6] = d.x; f[7] = d.y;
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}

template <int BN, int EPI>
__device__ __forceinline__ bool early_epilogue_ok(const GemmEpilogue& ep) {
  if constexpr (EPI == EPI_F32) return false;
  if constexpr (EPI == EPI_QKV) return ep.head_dim % 64 == 0 && ep.head_dim <= BN;
  return true;
}

// Columns of the tile this thread drains, per epilogue (see run_epilogue_early).
template <int BN, int EPI>
struct EarlyCols {
  static constexpr int NCH = BN / 64;  // 32-column chunks per thread (two warps per lane quarter)
  int col[NCH];
  int which = 0, half = 0, c0 = 0;
  __device__ __forceinline__ EarlyCols(const GemmEpilogue& ep, int n0, int part) {
    if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
      for (int j = 0; j < NCH / 2; ++j) {
        col[2 * j] = (part + 2 * j) * 32;
        col[2 * j + 1] = BN / 2 + (part + 2 * j) * 32;
      }
    } else if constexpr (EPI == EPI_QKV) {
      const int kvd = ep.kv_dim > 0 ? ep.kv_dim : ep.dim;
      which = n0 < ep.dim ? 0 : (n0 < ep.dim + kvd ? 1 : 2);
      c0 = which == 0 ? n0 : (which == 1 ? n0 - ep.dim : n0 - ep.dim - kvd);
      half = ep.head_dim >> 1;
      const int per = half / 32;
#pragma unroll
      for (int j = 0; j < NCH / 2; ++j) {
        if (which == 2) {
          col[2 * j] = (part + 4 * j) * 32;
          col[2 * j + 1] = (part + 4 * j + 2) * 32;
        } else {
          const int i = part + 2 * j;
          col[2 * j] = (i / per) * ep.head_dim + (i % per) * 32;
          col[2 * j + 1] = col[2 * j] + half;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < NCH; ++j) col[j] = (part + 2 * j) * 32;
    }
  }
};

// Before the accumulator is ready: the warp copies the column scales and the bias of its
// chunks into its own shared-memory slice cs ([NCH * 32] scales, then [NCH * 32] biases), so
// draining the accumulator waits on no global load.
template <int BN, int EPI>
__device__ __forceinline__ void early_stage_columns(float* cs, const EarlyCols<BN, EPI>& cc, int n0,
                                                   const GemmShape& shp, const GemmEpilogue& ep, int lane) {
  constexpr int NCH = EarlyCols<BN, EPI>::NCH;
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    const int n = n0 + cc.col[j] + lane;
    const bool ok = n < shp.N;
    cs[j * 32 + lane] = (ep.a_scale != nullptr && ok) ? __ldg(ep.b_scale + n) : 1.f;
    cs[(NCH + j) * 32 + lane] = (ep.bias != nullptr && ok) ? __bfloat162float(ep.bias[n]) : 0.f;
  }
  __syncwarp();
}

template <int BN, int EPI>
__device__ __forceinline__ void run_epilogue_early(uint32_t taddr, int m, int n0, const GemmShape& shp,
                                                   const GemmEpilogue& ep, const EarlyCols<BN, EPI>& cc,
                                                   const float* cs, float rs, uint32_t tempty_bar,
                                                   long long* phase1_cycles = nullptr) {
  const long long tp_ = phase1_cycles ? clock64() : 0;
  constexpr int NCH = EarlyCols<BN, EPI>::NCH;
  const bool row_ok = m < shp.M;
  const int* col = cc.col;
  const int which = cc.which, half = cc.half, c0 = cc.c0;
  (void)which; (void)half; (void)c0;
  // phase 1: accumulator -> registers (bf16 pairs), then release it
  uint32_t pk[NCH][16];
#pragma unroll
  for (int j = 0; j < NCH; ++j) {
    uint32_t r[32];
    tmem_ld32(taddr + col[j], r);
    tmem_wait_ld();
    // the same arithmetic as scale_acc + add_bias: acc * (row scale * column scale) + bias
    const float4* sc4 = reinterpret_cast<const float4*>(cs + j * 32);
    const float4* bi4 = reinterpret_cast<const float4*>(cs + (NCH + j) * 32);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 w = sc4[i], bb = bi4[i];
      float v0 = __uint_as_float(r[4 * i]), v1 = __uint_as_float(r[4 * i + 1]);
      float v2 = __uint_as_float(r[4 * i + 2]), v3 = __uint_as_float(r[4 * i + 3]);
      if (ep.a_scale != nullptr) {
        v0 *= rs * w.x;
        v1 *= rs * w.y;
        v2 *= rs * w.z;
        v3 *= rs * w.w;
      }
      if (ep.bias != nullptr) {
        v0 += bb.x;
        v1 += bb.y;
        v2 += bb.z;
        v3 += bb.w;
      }
      pk[j][2 * i] = pack_bf16x2(v0, v1);
      pk[j][2 * i + 1] = pack_bf16x2(v2, v3);
    }
  }
  tc_fence_before();
  mbar_arrive(tempty_bar);
  if (phase1_cycles) *phase1_cycles += clock64() - tp_;
  if (!row_ok) return;
  // phase 2: fused elementwise work and stores, 8 columns (16 bytes) at a time
  if constexpr (EPI == EPI_SWIGLU) {
    const int orow = ep.out_rows ? ep.out_rows[m] : m;
    if (orow < 0) return;
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(ep.out) + (long)orow * ep.ldo + n0 / 2;
#pragma unroll
    for (int j = 0; j < NCH / 2; ++j) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        float a[8], b[8];
        unpack8(make_uint4(pk[2 * j][4 * g], pk[2 * j][4 * g + 1], pk[2 * j][4 * g + 2], pk[2 * j][4 * g + 3]), a);
        unpack8(make_uint4(pk[2 * j + 1][4 * g], pk[2 * j + 1][4 * g + 1], pk[2 * j + 1][4 * g + 2],
                           pk[2 * j + 1][4 * g + 3]), b);
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = bf16_round(silu(a[e])) * b[e];
        st_u4(dst + col[2 * j] + 8 * g, pack8(a));
      }
    }
  } else if constexpr (EPI == EPI_QKV) {
    const int tok = ep.tok_idx ? ep.tok_idx[m] : (m % ep.seq_len);
    const int kvrow = ep.kv_rows ? ep.kv_rows[m] : m;
    const long ldkv = ep.ld_kv > 0 ? ep.ld_kv : ep.ld_qkv;
    __nv_bfloat16* dst;
    if (which == 0) dst = ep.q_out + (long)m * ep.ld_qkv;
    else if (kvrow < 0) return;
    else dst = (which == 1 ? ep.k_out : ep.v_out) + (long)kvrow * ldkv;
    dst += c0;
    const bool rope = which != 2 && ep.rope_sin != nullptr && tok >= ep.n_prefix;
    const int rrow = tok - ep.n_prefix;
#pragma unroll
    for (int j = 0; j < NCH / 2; ++j) {
      const int cl = col[2 * j];
      const int ch = col[2 * j + 1];
      const int cin = cl % ep.head_dim;  // offset inside the first half of the head
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 ul = make_uint4(pk[2 * j][4 * g], pk[2 * j][4 * g + 1], pk[2 * j][4 * g + 2], pk[2 * j][4 * g + 3]);
        uint4 uh = make_uint4(pk[2 * j + 1][4 * g], pk[2 * j + 1][4 * g + 1], pk[2 * j + 1][4 * g + 2],
                              pk[2 * j + 1][4 * g + 3]);
        if (rope) {
          // DINOv3 RoPE tables repeat their first half, so the pair (d, d + half) shares one angle
          const float4* sn = reinterpret_cast<const float4*>(ep.rope_sin + (long)rrow * ep.head_dim + cin + 8 * g);
          const float4* cs = reinterpret_cast<const float4*>(ep.rope_cos + (long)rrow * ep.head_dim + cin + 8 * g);
          const float4 s0 = __ldg(sn), s1 = __ldg(sn + 1), k0 = __ldg(cs), k1 = __ldg(cs + 1);
          const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
          const float cv[8] = {k0.x, k0.y, k0.z, k0.w, k1.x, k1.y, k1.z, k1.w};
          float lo[8], hi[8];
          unpack8(ul, lo);
          unpack8(uh, hi);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const float xl = lo[e], xh = hi[e];
            lo[e] = xl * cv[e] - xh * sv[e];
            hi[e] = xh * cv[e] + xl * sv[e];
          }
          ul = pack8(lo);
          uh = pack8(hi);
        }
        st_u4(dst + cl + 8 * g, ul);
        st_u4(dst + ch + 8 * g, uh);
      }
    }
  } else {
    const int orow = ep.out_rows ? ep.out_rows[m] : m;
    if (orow < 0) return;
    int rrow = -1, arow = -1;
    if constexpr (EPI == EPI_RESID) {
      rrow = ep.resid_rows ? ep.resid_rows[m] : m;
      arow = ep.aux_rows ? ep.aux_rows[m] : orow;
    }
#pragma unroll
    for (int j = 0; j < NCH; ++j) {
      const int n = n0 + col[j];
      if (n >= shp.N) continue;
      __nv_bfloat16* dst;
      if constexpr (EPI == EPI_BF16) {
        if (ep.rs_out[0] != nullptr) {
          const int owner = orow / ep.rs_rows_per_rank;
          dst = ep.rs_out[owner] + ((long)ep.rs_rank * ep.rs_slot_rows + m) * ep.ldo + n;
        } else {
          dst = reinterpret_cast<__nv_bfloat16*>(ep.out) + (long)orow * ep.ldo + n;
        }
      } else {
        dst = reinterpret_cast<__nv_bfloat16*>(ep.out) + (long)orow * ep.ldo + n;
      }
      uint4 gmv[4], rsv[4], axv[4];  // RESID: every load of the chunk before its stores
      if constexpr (EPI == EPI_RESID) {
        __nv_bfloat16* ap = ep.aux + (long)arow * ep.ldaux + n;
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          gmv[g] = ldg_u4(ep.gamma + n + 8 * g);
          rsv[g] = ld_u4(ep.resid + (long)rrow * ep.ldr + n + 8 * g);
          if (ep.aux_mode == AUX_ADD && arow >= 0) axv[g] = ld_u4(ap + 8 * g);
          else if (ep.aux_mode == AUX_OUT_MINUS && arow >= 0) axv[g] = ld_u4(ep.resid2 + (long)m * ep.ldr2 + n + 8 * g);
        }
      }
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint4 u = make_uint4(pk[j][4 * g], pk[j][4 * g + 1], pk[j][4 * g + 2], pk[j][4 * g + 3]);
        if constexpr (EPI == EPI_GELU) {
          float f[8];
          unpack8(u, f);
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = gelu_erf(f[e]);
          u = pack8(f);
        } else if constexpr (EPI == EPI_RESID) {
          float v[8], gm[8], rv[8], d[8];
          unpack8(u, v);
          unpack8(gmv[g], gm);
          unpack8(rsv[g], rv);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            d[e] = bf16_round(v[e] * gm[e]);
            v[e] = rv[e] + d[e];
          }
          if (ep.aux_mode != AUX_NONE && arow >= 0) {
            __nv_bfloat16* ap = ep.aux + (long)arow * ep.ldaux + n + 8 * g;
            float a[8];
            if (ep.aux_mode == AUX_SET) {
#pragma unroll
              for (int e = 0; e < 8; ++e) a[e] = d[e];
            } else if (ep.aux_mode == AUX_ADD) {
              unpack8(axv[g], a);
#pragma unroll
              for (int e = 0; e < 8; ++e) a[e] += d[e];
            } else {
              float r2[8];
              unpack8(axv[g], r2);
#pragma unroll
              for (int e = 0; e < 8; ++e) a[e] = bf16_round(rv[e] - r2[e]) + d[e];
            }
            st_u4(ap, pack8(a));
          }
          u = pack8(v);
        }
        st_u4(dst + 8 * g, u);
      }
    }
  }
}

// KIND 0: bf16 x bf16 (kind::f16, 64-element K blocks); KIND 1: e4m3 x e4m3 (kind::f8f6f4,
// 128-element K blocks). Both stage 128-byte rows, so the shared-memory layout is identical.
__device__ __forceinline__ void umma_f8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// KIND 2: NVFP4 x NVFP4 (kind::mxf4nvf4, block16): e2m1 pairs packed two per byte (element 2i in
// the low nibble), 256-element K blocks (again 128-byte rows), one ue4m3 scale per 16 elements
// of each row. The scales live in TMEM: per 64-element MMA step, row r's four scales sit in
// column r / 32, lane r % 32 of every 32-lane quarter (byte s = the s-th 16-element block).
// In the blocked global layout (128-row x 64-element tiles of 512 bytes, row r at byte
// (r % 32) * 16 + ((r % 128) / 32) * 4) lane a's 16 bytes of a tile are exactly its four columns.
__device__ __forceinline__ void umma_f4(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t tmem_sfa, uint32_t tmem_sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tmem_sfa), "r"(tmem_sfb)
      : "memory");
}

// Instruction descriptor for kind::mxf4nvf4: A / B format E2M1 (1), scale format UE4M3 (bit 23 = 0),
// dense K = 64, both operands K-major, scale-factor ids 0. The accumulator is always fp32.
__host__ __device__ constexpr uint32_t idesc_nvf4_f32(int M, int N) {
  return (1u << 7) | (1u << 10) | (static_cast<uint32_t>(N >> 3) << 17) | (static_cast<uint32_t>(M >> 4) << 24);
}

// Plain (non-tensor, non-multicast) bulk copy global -> this CTA's shared memory, completing on `bar`.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

// NVFP4 adds four scale warps (10..13): they move each stage's block scales from shared memory into
// the stage's TMEM scale slot with tcgen05.st (one warp per 32-lane quarter; the MMA reads every
// row's scales replicated in all four quarters) and release the stage to the MMA warp through
// `sfull[s]`. (Staging them with tcgen05.cp from the MMA thread put eight copies per stage in
// the MMA issue stream and cost about a quarter of the GEMM's time.)
// Eight epilogue warps (2..9): two per TMEM lane quarter, each draining half of the columns, so a
// heavy epilogue (residual + increment, SwiGLU, RoPE) stays shorter than the next tile's main loop.
constexpr int kEpiWarps = 8;
constexpr uint32_t kBarRegion = 256;     // mbarriers + TMEM slot after the stage ring
constexpr int kEarlyColFloats = 256;     // early-release epilogue: per-warp column scales + biases
// shared memory beyond the stage ring: alignment slack, barrier region, early-epilogue slices
template <int BN, int KIND>
constexpr size_t gemm_smem_extra() {
  return 1024 + kBarRegion + ((KIND == 2 && BN == 256) ? kEpiWarps * kEarlyColFloats * 4 : 0);
}
template <int KIND>
constexpr int gemm_threads() { return 64 + kEpiWarps * 32 + (KIND == 2 ? 128 : 0); }

template <int BN, int STAGES, int EPI, int KIND = 0>
__global__ void __launch_bounds__(gemm_threads<KIND>(), 1)
    gemm_bf16_tn_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GemmShape shp, GemmEpilogue ep) {
  constexpr bool F4 = KIND == 2;
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t B_BYTES = BN * kBK * 2;
  constexpr uint32_t SFA_BYTES = F4 ? kBM * 16 : 0;  // 4 x 512-byte scale tiles per stage
  constexpr uint32_t SFB_BYTES = F4 ? BN * 16 : 0;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  // F4: two accumulators, then one 16 + BN/8 column scale slot per stage
  constexpr uint32_t SF_COLS = 16 + BN / 8;
  // accumulators: two (the epilogue of tile t overlaps the main loop of t+1), except NVFP4 with
  // BN = 256, whose 256-column accumulator leaves room for one only beside the scale slots (the
  // producer keeps prefetching the next tile's stages while the epilogue drains it)
  constexpr int NACC = (F4 && BN == 256) ? 1 : 2;
  static_assert(!F4 || NACC * BN + STAGES * SF_COLS <= 512, "NVFP4 TMEM budget");
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep the 1024-byte swizzle alignment");
  constexpr uint32_t TMEM_COLS = F4 ? 512 : TmemCols<BN>::value;
  constexpr uint32_t IDESC = KIND == 2 ? idesc_nvf4_f32(kBM, BN)
                                       : (KIND == 1 ? idesc_e4m3_f32(kBM, BN) : idesc_bf16_f32(kBM, BN));
  constexpr int BKE = KIND == 2 ? 256 : (KIND == 1 ? 128 : kBK);  // K elements per stage (128-byte rows)
  constexpr int BKX = KIND == 0 ? kBK : 128;                       // the same in tensor-map columns

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* sfull = tempty + 2;  // F4: scales of stage s are in TMEM (4 scale warps)
  uint64_t* sf_full = sfull + (F4 ? STAGES : 0);  // F4: scale bytes of stage s landed in shared memory
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sf_full + (F4 ? STAGES : 0));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // GemmProf counters (ep.prof): clock64 spent in each wait, summed over CTAs
  long long pw0 = 0, pw1 = 0, pw2 = 0, pw3 = 0;
  const bool prof = ep.prof != nullptr;
#define GEMM_TIMED(acc_, expr_)                      \
  ([&]() {                                            \
    const long long t0_ = prof ? clock64() : 0;       \
    const bool r_ = (expr_);                          \
    if (prof) acc_ += clock64() - t0_;                \
    return r_;                                        \
  }())

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
      if constexpr (F4) {
        mbar_init(smem_addr(&sfull[s]), 4);
        mbar_init(smem_addr(&sf_full[s]), 1);
      }
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      mbar_init(smem_addr(&tempty[a]), kEpiWarps * 32);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (shp.M + kBM - 1) / kBM;
  const int num_n = (shp.N + BN - 1) / BN;
  const int KB = (shp.K + BKE - 1) / BKE;
  const int total = num_m * num_n;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < KB; ++kb) {
          if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&empty[s]), ph ^ 1, shp.err, kErrTimeoutProducer))) goto producer_done;
          const uint32_t fb = smem_addr(&full[s]);
          const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
          if constexpr (F4) {  // scales first, on their own barrier: the scale warps move them to
                               // TMEM while A / B are still in flight
            const uint32_t sfb = smem_addr(&sf_full[s]);
            mbar_arrive_expect_tx(sfb, SFA_BYTES + SFB_BYTES);
            const uint32_t sf = sa + A_BYTES + B_BYTES;
            bulk_g2s(sf, ep.sfa + ((long)mb * ep.sf_kt + kb * 4) * 512, SFA_BYTES, sfb);
#pragma unroll
            for (int j = 0; j < BN / 128; ++j)
              bulk_g2s(sf + SFA_BYTES + j * 2048, ep.sfb + ((long)(nb * (BN / 128) + j) * ep.sf_kt + kb * 4) * 512,
                       2048, sfb);
          }
          mbar_arrive_expect_tx(fb, A_BYTES + B_BYTES);
          tma_load_2d(sa, &tmA, fb, kb * BKX, mb * kBM);
          tma_load_2d(sa + A_BYTES, &tmB, fb, kb * BKX, nb * BN);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      // Drain: wait until the consumer has released every stage we filled.
      for (int i = 0; i < STAGES; ++i) {
        if (!mbar_wait(smem_addr(&empty[s]), ph ^ 1, shp.err, kErrTimeoutProducer)) break;
        if (++s == STAGES) { s = 0; ph ^= 1; }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int t_local = 0;
      bool issued = false;
      const long long tstart = prof ? clock64() : 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++t_local) {
        const int acc = NACC == 2 ? (t_local & 1) : 0;
        const uint32_t acc_ph = NACC == 2 ? ((t_local >> 1) & 1) : (t_local & 1);
        if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&tempty[acc]), acc_ph ^ 1, shp.err, kErrTimeoutMma))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!GEMM_TIMED(pw1, mbar_wait(smem_addr(&full[s]), ph, shp.err, kErrTimeoutMma))) { ok = false; break; }
          if constexpr (F4)
            if (!GEMM_TIMED(pw2, mbar_wait(smem_addr(&sfull[s]), ph, shp.err, kErrTimeoutMma))) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          const uint32_t sf_col = tmem_base + NACC * BN + s * SF_COLS;  // F4: this stage's scale slot
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 4 MMAs of 32 bytes of K per 128-byte stage row
            if constexpr (KIND == 2)
              umma_f4(d_tmem, sw128_kmajor_desc(sa + k * 32), sw128_kmajor_desc(sb + k * 32), IDESC, sf_col + k * 4,
                      sf_col + 16 + k * (BN / 32), (kb | k) != 0 ? 1u : 0u);
            else if constexpr (KIND == 1)
              umma_f8(d_tmem, sw128_kmajor_desc(sa + k * 32), sw128_kmajor_desc(sb + k * 32), IDESC,
                      (kb | k) != 0 ? 1u : 0u);
            else
              umma_f16(d_tmem, sw128_kmajor_desc(sa + k * 32), sw128_kmajor_desc(sb + k * 32), IDESC,
                       (kb | k) != 0 ? 1u : 0u);
          }
          issued = true;
          umma_commit(smem_addr(&empty[s]));
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit(smem_addr(&tfull[acc]));
      }
      (void)issued;
      if (prof) pw3 = clock64() - tstart;
    }
  } else if (F4 && warp >= 2 + kEpiWarps) {
    // scale warps: lane a of quarter q writes, for every 64-element step k, the words of rows
    // 32b + a (b = 0..3) -- bytes k*512 + a*16 .. +15 of the blocked tile -- into columns
    // k*4 + b of the slot (A), then the same for B's rows after 16 columns
    if constexpr (F4) {
      // slot columns in groups of four: group g < 4 is A's 64-element step g; group 4 + g' is B's
      // step g' / (BN / 128), 128-row tile g' % (BN / 128) -- one 16-byte load per group per lane
      constexpr int NG = SF_COLS / 4;
      static_assert(NG == 8 || NG == 12, "scale slot of 32 (BN 128) or 48 (BN 256) columns");
      const int q = warp & 3;
      int s = 0;
      uint32_t ph = 0;
      for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&sf_full[s]), ph, shp.err, kErrTimeoutEpilogue))) { ok = false; break; }
          const long long ts_ = prof ? clock64() : 0;
          const uint8_t* sfs = smem + s * STAGE_BYTES + A_BYTES + B_BYTES;
          uint32_t r[32], r2[16];
#pragma unroll
          for (int g = 0; g < NG; ++g) {
            const int gb = g - 4;
            const int off = g < 4 ? g * 512 : SFA_BYTES + (gb % (BN / 128)) * 2048 + (gb / (BN / 128)) * 512;
            const uint4 u = *reinterpret_cast<const uint4*>(sfs + off + lane * 16);
            uint32_t* dst = g < 8 ? &r[4 * g] : &r2[4 * (g - 8)];
            dst[0] = u.x;
            dst[1] = u.y;
            dst[2] = u.z;
            dst[3] = u.w;
          }
          const uint32_t ta = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + NACC * BN + s * SF_COLS;
          tmem_st32(ta, r);
          if constexpr (NG == 12) tmem_st16(ta + 32, r2);
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(&sfull[s]));
          if (prof) pw1 += clock64() - ts_;
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
      }
    }
  } else {
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    int t_local = 0;
    for (int tile = blockIdx.x; tile < total; tile += gridDim.x, ++t_local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int acc = NACC == 2 ? (t_local & 1) : 0;
      const uint32_t acc_ph = NACC == 2 ? ((t_local >> 1) & 1) : (t_local & 1);
      // All lanes wait (tcgen05.ld below is warp-collective).
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      bool early = false;
      if constexpr (NACC == 1) {
        static_assert(kEpiWarps == 8 && BN == 256, "early-release epilogue: two warps per lane quarter");
        early = early_epilogue_ok<BN, EPI>(ep);
        if (early) {
          const int m = mb * kBM + row_in_tile;
          const EarlyCols<BN, EPI> cc(ep, nb * BN, (warp - 2) / 4);
          float* cs = reinterpret_cast<float*>(smem + STAGES * STAGE_BYTES + kBarRegion) + (warp - 2) * kEarlyColFloats;
          early_stage_columns<BN, EPI>(cs, cc, nb * BN, shp, ep, lane);
          const float rs = (ep.a_scale != nullptr && m < shp.M) ? ep.a_scale[m] : 1.f;
          if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&tfull[acc]), acc_ph, shp.err, kErrTimeoutEpilogue))) break;
          tc_fence_after();
          GEMM_TIMED(pw1, (run_epilogue_early<BN, EPI>(taddr, m, nb * BN, shp, ep, cc, cs, rs, smem_addr(&tempty[acc]), prof ? &pw2 : nullptr), true));
        }
      }
      if (!early) {
        if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&tfull[acc]), acc_ph, shp.err, kErrTimeoutEpilogue))) break;
        tc_fence_after();
        GEMM_TIMED(pw1, (run_epilogue<BN, EPI>(taddr, mb * kBM + row_in_tile, nb * BN, shp, ep, (warp - 2) / 4, kEpiWarps / 4), true));
        tc_fence_before();
        mbar_arrive(smem_addr(&tempty[acc]));
      }
    }
  }
#undef GEMM_TIMED
  if (prof && lane == 0) {  // 0 producer empty; 1-3 MMA tempty / full / sfull; 4 MMA loop; 5-6 epilogue tfull / body
    if (warp == 0) atomicAdd(ep.prof + 0, (unsigned long long)pw0);
    if (warp == 1) {
      atomicAdd(ep.prof + 1, (unsigned long long)pw0);
      atomicAdd(ep.prof + 2, (unsigned long long)pw1);
      atomicAdd(ep.prof + 3, (unsigned long long)pw2);
      atomicAdd(ep.prof + 4, (unsigned long long)pw3);
    }
    if (warp == 2) {
      atomicAdd(ep.prof + 5, (unsigned long long)pw0);
      atomicAdd(ep.prof + 6, (unsigned long long)pw1);
    }
    if (threadIdx.x == 0) atomicAdd(ep.prof + 7, 1ull);
    if (F4 && warp == 2 + kEpiWarps) {  // 8-9 scale warp: bytes wait / TMEM store + wait
      atomicAdd(ep.prof + 8, (unsigned long long)pw0);
      atomicAdd(ep.prof + 9, (unsigned long long)pw1);
    }
    if (warp == 2) atomicAdd(ep.prof + 10, (unsigned long long)pw2);  // 10 epilogue phase 1
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------ 2-CTA variant
// Same structure, but a cluster of two CTAs computes a 256 x 256 output tile with
// tcgen05.mma.cta_group::2 (M = 256): each CTA stages its own 128 rows of A and 128 of the 256 B
// rows, so per-SM shared-memory traffic per MMA is halved. The even CTA issues all MMAs; both CTAs
// hold 128 accumulator rows in their TMEM and run their own epilogue. The odd CTA's TMA loads
// complete on the even CTA's `full` barrier; MMA completion is committed separately to each CTA's
// `empty` / `tfull` barrier; epilogue threads of both CTAs arrive on the even CTA's `tempty`.
template <int STAGES, int EPI>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tn_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                            GemmShape shp, GemmEpilogue ep) {
  constexpr int BN = 256;                       // output tile width (both CTAs)
  constexpr int BH = BN / 2;                    // B rows staged per CTA
  constexpr uint32_t A_BYTES = kBM * kBK * 2;
  constexpr uint32_t B_BYTES = BH * kBK * 2;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t IDESC = idesc_bf16_f32(2 * kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      mbar_init(smem_addr(&tempty[a]), 256);
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised before anyone signals them
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (shp.M + 2 * kBM - 1) / (2 * kBM);
  const int num_n = (shp.N + BN - 1) / BN;
  const int KB = (shp.K + kBK - 1) / kBK;
  const int total = num_m * num_n;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int tile = cluster_id; tile < total; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(smem_addr(&empty[s]), ph ^ 1, shp.err, kErrTimeoutProducer)) goto producer_done;
          const uint32_t fb = mapa_shared(smem_addr(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx_cluster(fb, 2 * STAGE_BYTES);
          const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
          tma_load_2d_pair(sa, &tmA, fb, kb * kBK, mb * 2 * kBM + rank * kBM);
          tma_load_2d_pair(sa + A_BYTES, &tmB, fb, kb * kBK, nb * BN + rank * BH);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      for (int i = 0; i < STAGES; ++i) {
        if (!mbar_wait(smem_addr(&empty[s]), ph ^ 1, shp.err, kErrTimeoutProducer)) break;
        if (++s == STAGES) { s = 0; ph ^= 1; }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int t_local = 0;
      for (int tile = cluster_id; tile < total; tile += num_clusters, ++t_local) {
        const int acc = t_local & 1;
        const uint32_t acc_ph = (t_local >> 1) & 1;
        if (!mbar_wait(smem_addr(&tempty[acc]), acc_ph ^ 1, shp.err, kErrTimeoutMma)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!mbar_wait(smem_addr(&full[s]), ph, shp.err, kErrTimeoutMma)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < kBK / 16; ++k)
            umma_f16_pair(d_tmem, sw128_kmajor_desc(sa + k * 32), sw128_kmajor_desc(sb + k * 32), IDESC,
                          (kb | k) != 0 ? 1u : 0u);
#ifdef APPCORR_PAIR_COMMIT_SPLIT
          umma_commit_pair(mapa_shared(smem_addr(&empty[s]), 0));
          umma_commit_pair(mapa_shared(smem_addr(&empty[s]), 1));
#else
          umma_commit_pair_mask(smem_addr(&empty[s]), 0x3);
#endif
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
#ifdef APPCORR_PAIR_COMMIT_SPLIT
        umma_commit_pair(mapa_shared(smem_addr(&tfull[acc]), 0));
        umma_commit_pair(mapa_shared(smem_addr(&tfull[acc]), 1));
#else
        umma_commit_pair_mask(smem_addr(&tfull[acc]), 0x3);
#endif
      }
    }
  } else {
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    int t_local = 0;
    for (int tile = cluster_id; tile < total; tile += num_clusters, ++t_local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int acc = t_local & 1;
      const uint32_t acc_ph = (t_local >> 1) & 1;
      if (!mbar_wait(smem_addr(&tfull[acc]), acc_ph, shp.err, kErrTimeoutEpilogue)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      run_epilogue<BN, EPI>(taddr, mb * 2 * kBM + rank * kBM + row_in_tile, nb * BN, shp, ep);
      tc_fence_before();
      mbar_arrive_cluster(mapa_shared(smem_addr(&tempty[acc]), 0));
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal it
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------- 2-CTA NVFP4 variant
// NVFP4 x NVFP4 on a CTA pair: one 256 x BN output tile per cluster with
// tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 (M = 256, N = BN, K = 64 per MMA),
// four MMAs per 256-element K stage. Per CTA and stage: its 128 A rows (16 KB), its half of the
// BN B rows and block scales (SFA of its own rows; SFB of all BN B rows: the pair's MMA reads the
// B scales from each CTA's own TMEM). Both CTAs stage their scales into their own TMEM (four scale
// warps each, tcgen05.st); the follower's scale warps arrive on the leader's `sfull`. The leader
// issues the MMAs once both CTAs' tiles landed (`full`, tx-counted across the pair) and both CTAs'
// scales are in TMEM, then commits `empty` to both CTAs. TMEM per CTA: BN = 128 keeps two
// 128-column accumulators (the epilogue of tile t overlaps the main loop of tile t + 1), BN = 256
// one. Cross-CTA arrivals that only publish tensor-memory state (scales written, accumulator
// drained, both complete by tcgen05.wait) are relaxed: a release at cluster scope would make every
// epilogue thread wait for its global stores. Loads are plain per-CTA TMA (no multicast).
__device__ __forceinline__ void umma_f4_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t tmem_sfa, uint32_t tmem_sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(
          tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate), "r"(tmem_sfa), "r"(tmem_sfb)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_cluster_relaxed(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(gemm_threads<2>(), 1)
    gemm_f4_2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                       GemmShape shp, GemmEpilogue ep) {
  constexpr int BH = BN / 2;                       // B rows staged per CTA
  constexpr int NACC = BN == 128 ? 2 : 1;
  constexpr uint32_t A_BYTES = kBM * 128;          // 128 rows x 256 e2m1
  constexpr uint32_t B_BYTES = BH * 128;
  constexpr uint32_t SFA_BYTES = kBM * 16;         // four 512-byte groups
  constexpr uint32_t SFB_BYTES = BN * 16;
  constexpr uint32_t STAGE_BYTES = A_BYTES + B_BYTES + SFA_BYTES + SFB_BYTES;
  constexpr uint32_t SFB_COLS = BN / 8;            // 4 per 64-element step per 128 B rows
  constexpr uint32_t SF_COLS = 16 + SFB_COLS;
  constexpr uint32_t TMEM_COLS = 512;
  static_assert(NACC * BN + STAGES * SF_COLS <= TMEM_COLS, "2-CTA NVFP4 TMEM budget");
  static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
  constexpr uint32_t IDESC = idesc_nvf4_f32(2 * kBM, BN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);  // leader: A/B of both CTAs
  uint64_t* empty = full + STAGES;
  uint64_t* sf_full = empty + STAGES;   // local: this CTA's scale bytes landed
  uint64_t* sfull = sf_full + STAGES;   // leader: both CTAs' scales are in TMEM
  uint64_t* tfull = sfull + STAGES;     // 2
  uint64_t* tempty = tfull + 2;         // 2 (leader)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  long long pw0 = 0, pw1 = 0, pw2 = 0, pw3 = 0;
  const bool prof = ep.prof != nullptr;
#define GEMM_TIMED(acc_, expr_)                      \
  ([&]() {                                            \
    const long long t0_ = prof ? clock64() : 0;       \
    const bool r_ = (expr_);                          \
    if (prof) acc_ += clock64() - t0_;                \
    return r_;                                        \
  }())

  if (warp == 0 && lane == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_addr(&full[s]), 1);
      mbar_init(smem_addr(&empty[s]), 1);
      mbar_init(smem_addr(&sf_full[s]), 1);
      mbar_init(smem_addr(&sfull[s]), 8);   // 4 scale warps x 2 CTAs
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_addr(&tfull[a]), 1);
      mbar_init(smem_addr(&tempty[a]), 2 * kEpiWarps);   // one arrival per epilogue warp of each CTA
    }
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int num_m = (shp.M + 2 * kBM - 1) / (2 * kBM);
  const int num_n = (shp.N + BN - 1) / BN;
  const int KB = (shp.K + 255) / 256;
  const int total = num_m * num_n;
  const int cluster_id = blockIdx.x >> 1;
  const int num_clusters = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int tile = cluster_id; tile < total; tile += num_clusters) {
        int mb, nb;
        tile_coords(tile, num_m, num_n, mb, nb);
        for (int kb = 0; kb < KB; ++kb) {
          if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&empty[s]), ph ^ 1, shp.err, kErrTimeoutProducer))) goto producer_done;
          const uint32_t fb = mapa_shared(smem_addr(&full[s]), 0);
          if (leader) mbar_arrive_expect_tx_cluster(fb, 2 * (A_BYTES + B_BYTES));
          const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
          tma_load_2d_pair(sa, &tmA, fb, kb * 128, mb * 2 * kBM + rank * kBM);
          tma_load_2d_pair(sa + A_BYTES, &tmB, fb, kb * 128, nb * BN + rank * BH);
          const uint32_t sfb = smem_addr(&sf_full[s]);
          mbar_arrive_expect_tx(sfb, SFA_BYTES + SFB_BYTES);
          const uint32_t sf = sa + A_BYTES + B_BYTES;
          bulk_g2s(sf, ep.sfa + ((long)(mb * 2 + rank) * ep.sf_kt + kb * 4) * 512, SFA_BYTES, sfb);
#pragma unroll
          for (int j = 0; j < BN / 128; ++j)
            bulk_g2s(sf + SFA_BYTES + j * 2048, ep.sfb + ((long)(nb * (BN / 128) + j) * ep.sf_kt + kb * 4) * 512,
                     2048, sfb);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
      }
      for (int i = 0; i < STAGES; ++i) {
        if (!mbar_wait(smem_addr(&empty[s]), ph ^ 1, shp.err, kErrTimeoutProducer)) break;
        if (++s == STAGES) { s = 0; ph ^= 1; }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (leader && lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      int t_local = 0;
      const long long tstart = prof ? clock64() : 0;
      for (int tile = cluster_id; tile < total; tile += num_clusters, ++t_local) {
        const int acc = NACC == 2 ? (t_local & 1) : 0;
        const uint32_t acc_ph = NACC == 2 ? ((t_local >> 1) & 1) : (t_local & 1);
        if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&tempty[acc]), acc_ph ^ 1, shp.err, kErrTimeoutMma))) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < KB; ++kb) {
          if (!GEMM_TIMED(pw1, mbar_wait(smem_addr(&full[s]), ph, shp.err, kErrTimeoutMma))) { ok = false; break; }
          if (!GEMM_TIMED(pw2, mbar_wait(smem_addr(&sfull[s]), ph, shp.err, kErrTimeoutMma))) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_addr(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
          const uint32_t sf_col = tmem_base + NACC * BN + s * SF_COLS;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f4_pair(d_tmem, sw128_kmajor_desc(sa + k * 32), sw128_kmajor_desc(sb + k * 32), IDESC,
                         sf_col + k * 4, sf_col + 16 + k * (SFB_COLS / 4), (kb | k) != 0 ? 1u : 0u);
          umma_commit_pair_mask(smem_addr(&empty[s]), 0x3);
          if (++s == STAGES) { s = 0; ph ^= 1; }
        }
        if (!ok) break;
        umma_commit_pair_mask(smem_addr(&tfull[acc]), 0x3);
      }
      if (prof) pw3 = clock64() - tstart;
    }
  } else if (warp >= 2 + kEpiWarps) {
    // scale warps: stage s's A scales (4 groups of 4 columns) and B scales (SFB_COLS columns)
    constexpr int NG = SF_COLS / 4;
    const int q = warp & 3;
    const uint32_t sfull_leader = mapa_shared(smem_addr(&sfull[0]), 0);
    int s = 0;
    uint32_t ph = 0;
    for (int tile = cluster_id; tile < total; tile += num_clusters) {
      bool ok = true;
      for (int kb = 0; kb < KB; ++kb) {
        if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&sf_full[s]), ph, shp.err, kErrTimeoutEpilogue))) { ok = false; break; }
        const long long ts_ = prof ? clock64() : 0;
        const uint8_t* sfs = smem + s * STAGE_BYTES + A_BYTES + B_BYTES;
        uint32_t r[32], r2[16];
#pragma unroll
        for (int g = 0; g < NG; ++g) {
          const int gb = g - 4;   // B: step gb / (BN / 128), 128-row B tile gb % (BN / 128)
          const int off = g < 4 ? g * 512 : SFA_BYTES + (gb % (BN / 128)) * 2048 + (gb / (BN / 128)) * 512;
          const uint4 u = *reinterpret_cast<const uint4*>(sfs + off + lane * 16);
          uint32_t* dst = g < 8 ? &r[4 * g] : &r2[4 * (g - 8)];
          dst[0] = u.x;
          dst[1] = u.y;
          dst[2] = u.z;
          dst[3] = u.w;
        }
        const uint32_t ta = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + NACC * BN + s * SF_COLS;
        tmem_st32(ta, r);
        if constexpr (NG == 12) tmem_st16(ta + 32, r2);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster_relaxed(sfull_leader + s * 8);
        if (prof) pw1 += clock64() - ts_;
        if (++s == STAGES) { s = 0; ph ^= 1; }
      }
      if (!ok) break;
    }
  } else {
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    int t_local = 0;
    const uint32_t tempty_leader = mapa_shared(smem_addr(&tempty[0]), 0);
    for (int tile = cluster_id; tile < total; tile += num_clusters, ++t_local) {
      int mb, nb;
      tile_coords(tile, num_m, num_n, mb, nb);
      const int acc = NACC == 2 ? (t_local & 1) : 0;
      const uint32_t acc_ph = NACC == 2 ? ((t_local >> 1) & 1) : (t_local & 1);
      if (!GEMM_TIMED(pw0, mbar_wait(smem_addr(&tfull[acc]), acc_ph, shp.err, kErrTimeoutEpilogue))) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * BN;
      GEMM_TIMED(pw1, (run_epilogue<BN, EPI>(taddr, mb * 2 * kBM + rank * kBM + row_in_tile, nb * BN, shp, ep,
                                             (warp - 2) / 4, kEpiWarps / 4), true));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster_relaxed(tempty_leader + acc * 8);
    }
  }
#undef GEMM_TIMED
  if (prof && lane == 0 && leader) {  // the leader CTA's warps, same slots as the one-CTA kernel
    if (warp == 0) atomicAdd(ep.prof + 0, (unsigned long long)pw0);
    if (warp == 1) {
      atomicAdd(ep.prof + 1, (unsigned long long)pw0);
      atomicAdd(ep.prof + 2, (unsigned long long)pw1);
      atomicAdd(ep.prof + 3, (unsigned long long)pw2);
      atomicAdd(ep.prof + 4, (unsigned long long)pw3);
    }
    if (warp == 2) {
      atomicAdd(ep.prof + 5, (unsigned long long)pw0);
      atomicAdd(ep.prof + 6, (unsigned long long)pw1);
    }
    if (warp == 0) atomicAdd(ep.prof + 7, 1ull);
    if (warp == 2 + kEpiWarps) {
      atomicAdd(ep.prof + 8, (unsigned long long)pw0);
      atomicAdd(ep.prof + 9, (unsigned long long)pw1);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------------ host side
namespace {

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult qres;
    void* p = nullptr;
    auto st = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &qres);
    TORCH_CHECK(st == cudaSuccess && qres == cudaDriverEntryPointSuccess && p != nullptr,
                "appcorr_b200: cuTensorMapEncodeTiled is unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

// Row-major bf16 matrix [rows, cols] with row stride `ld` elements, box = box_rows x 64 columns,
// 128-byte swizzle. Exposed for the attention kernels as well.
CUtensorMap make_tmap_bf16_2d(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                              int box_cols) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld * 2)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides,
                               box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(r));
  return m;
}

CUtensorMap make_tmap_u8_2d(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols) {
  CUtensorMap m;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  TORCH_CHECK((reinterpret_cast<uintptr_t>(ptr) & 15) == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK(ld % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (u8) failed: ", static_cast<int>(r));
  return m;
}

int num_sms() {
  static int n = 0;
  if (n == 0) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  }
  return n;
}

template <int BN, int STAGES, int EPI, int KIND = 0>
void launch_gemm(const at::Tensor& A, const at::Tensor& B, int M, int N, int K, const GemmEpilogue& ep,
                 int* err, int max_ctas, cudaStream_t stream) {
  constexpr uint32_t STAGE_BYTES = (kBM + BN) * kBK * 2 + (KIND == 2 ? (kBM + BN) * 16 : 0);
  constexpr size_t SMEM = STAGES * STAGE_BYTES + gemm_smem_extra<BN, KIND>();
  static_assert(SMEM <= 232448, "shared memory per CTA");
  auto kern = gemm_bf16_tn_kernel<BN, STAGES, EPI, KIND>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM));
    configured = true;
  }
  CUtensorMap ta, tb;
  if constexpr (KIND == 1) {
    ta = make_tmap_u8_2d(A.data_ptr(), M, K, A.stride(0), kBM, 128);
    tb = make_tmap_u8_2d(B.data_ptr(), B.size(0), K, B.stride(0), BN, 128);
  } else if constexpr (KIND == 2) {  // packed e2m1: K / 2 bytes per row
    ta = make_tmap_u8_2d(A.data_ptr(), M, K / 2, A.stride(0), kBM, 128);
    tb = make_tmap_u8_2d(B.data_ptr(), B.size(0), K / 2, B.stride(0), BN, 128);
  } else {
    ta = make_tmap_bf16_2d(A.data_ptr(), M, K, A.stride(0), kBM, kBK);
    tb = make_tmap_bf16_2d(B.data_ptr(), B.size(0), K, B.stride(0), BN, kBK);
  }
  GemmShape shp{M, N, K, err};
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  int grid = std::min(tiles, max_ctas > 0 ? max_ctas : num_sms());
  if (grid <= 0) return;
  kern<<<grid, gemm_threads<KIND>(), SMEM, stream>>>(ta, tb, shp, ep);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int STAGES, int EPI>
void launch_gemm_2sm(const at::Tensor& A, const at::Tensor& B, int M, int N, int K, const GemmEpilogue& ep,
                     int* err, int max_ctas, cudaStream_t stream) {
  constexpr uint32_t STAGE_BYTES = (kBM + 128) * kBK * 2;
  constexpr size_t SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  auto kern = gemm_bf16_tn_2sm_kernel<STAGES, EPI>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM));
    configured = true;
  }
  CUtensorMap ta = make_tmap_bf16_2d(A.data_ptr(), M, K, A.stride(0), kBM, kBK);
  CUtensorMap tb = make_tmap_bf16_2d(B.data_ptr(), B.size(0), K, B.stride(0), 128, kBK);
  GemmShape shp{M, N, K, err};
  const int tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + 255) / 256);
  int clusters = std::min(tiles, (max_ctas > 0 ? max_ctas : num_sms()) / 2);
  if (clusters <= 0) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, shp, ep));
}

template <int BN, int STAGES, int EPI>
void launch_gemm_f4_2sm(const at::Tensor& A, const at::Tensor& B, int M, int N, int K, const GemmEpilogue& ep,
                        int* err, int max_ctas, cudaStream_t stream) {
  constexpr uint32_t STAGE_BYTES = kBM * 128 + (BN / 2) * 128 + kBM * 16 + BN * 16;
  constexpr size_t SMEM = STAGES * STAGE_BYTES + 1024 + 256;
  auto kern = gemm_f4_2sm_kernel<BN, STAGES, EPI>;
  static bool configured = false;
  if (!configured) {
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(SMEM));
    configured = true;
  }
  TORCH_CHECK(K % 256 == 0, "nvfp4 2-CTA gemm: K % 256 == 0");
  CUtensorMap ta = make_tmap_u8_2d(A.data_ptr(), M, K / 2, A.stride(0), kBM, 128);
  CUtensorMap tb = make_tmap_u8_2d(B.data_ptr(), B.size(0), K / 2, B.stride(0), BN / 2, 128);
  GemmShape shp{M, N, K, err};
  const int tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + BN - 1) / BN);
  int clusters = std::min(tiles, (max_ctas > 0 ? max_ctas : num_sms()) / 2);
  if (clusters <= 0) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * clusters);
  cfg.blockDim = dim3(gemm_threads<2>());
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  C10_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ta, tb, shp, ep));
}

// Dispatch on (epilogue, BN). STAGES chosen to fill ~192 KB of shared memory.
void gemm_dispatch_fp8(int epi, int bn, const at::Tensor& A, const at::Tensor& B, int M, int N, int K,
                       const GemmEpilogue& ep, int* err, int max_ctas) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(bn == 256 || bn == 128, "fp8 gemm: BN 128 or 256");
  switch (epi) {
#define APPCORR_GEMM8_CASE(E)                                                                     \
  case E:                                                                                         \
    if (bn == 256) launch_gemm<256, 4, E, 1>(A, B, M, N, K, ep, err, max_ctas, st);               \
    else launch_gemm<128, 6, E, 1>(A, B, M, N, K, ep, err, max_ctas, st);                         \
    break;
    APPCORR_GEMM8_CASE(EPI_BF16)
    APPCORR_GEMM8_CASE(EPI_F32)
    APPCORR_GEMM8_CASE(EPI_GELU)
    APPCORR_GEMM8_CASE(EPI_RESID)
    APPCORR_GEMM8_CASE(EPI_QKV)
#undef APPCORR_GEMM8_CASE
    case EPI_SWIGLU:
      TORCH_CHECK(bn == 256, "swiglu epilogue uses BN=256");
      launch_gemm<256, 4, EPI_SWIGLU, 1>(A, B, M, N, K, ep, err, max_ctas, st);
      break;
    default:
      TORCH_CHECK(false, "unknown epilogue ", epi);
  }
}

// NVFP4 tiles: 128 x 256 (one accumulator + four stage scale slots, the default) or 128 x 128 (two
// accumulators + six slots) in the 512 TMEM columns. The SwiGLU epilogue's w1 || w2 interleave
// block is BN / 2 rows (128 for the 256-wide tile).
void gemm_dispatch_fp4(int epi, int bn, const at::Tensor& A, const at::Tensor& B, int M, int N, int K,
                       const GemmEpilogue& ep, int* err, int max_ctas) {
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  TORCH_CHECK(bn == 128 || bn == 256 || bn == 512 || bn == 513,
              "nvfp4 gemm: BN 128, 256, 512 (2-CTA 256 x 256) or 513 (2-CTA 256 x 128)");
  switch (epi) {
#define APPCORR_GEMM4_CASE(E)                                                                  \
  case E:                                                                                      \
    if (bn == 512) launch_gemm_f4_2sm<256, 5, E>(A, B, M, N, K, ep, err, max_ctas, st);       \
    else if (bn == 513) launch_gemm_f4_2sm<128, 6, E>(A, B, M, N, K, ep, err, max_ctas, st);  \
    else if (bn == 256) launch_gemm<256, 4, E, 2>(A, B, M, N, K, ep, err, max_ctas, st);       \
    else launch_gemm<128, 6, E, 2>(A, B, M, N, K, ep, err, max_ctas, st);                     \
    break;
    APPCORR_GEMM4_CASE(EPI_BF16)
    APPCORR_GEMM4_CASE(EPI_F32)
    APPCORR_GEMM4_CASE(EPI_GELU)
    APPCORR_GEMM4_CASE(EPI_RESID)
    APPCORR_GEMM4_CASE(EPI_QKV)
    APPCORR_GEMM4_CASE(EPI_SWIGLU)
#undef APPCORR_GEMM4_CASE
    default:
      TORCH_CHECK(false, "unknown epilogue ", epi);
  }
}

void gemm_dispatch(int epi, int bn, const at::Tensor& A, const at::Tensor& B, int M, int N, int K,
                   const GemmEpilogue& ep, int* err, int max_ctas, int kind) {
  if (kind == 1) {
    gemm_dispatch_fp8(epi, bn, A, B, M, N, K, ep, err, max_ctas);
    return;
  }
  if (kind == 2) {
    gemm_dispatch_fp4(epi, bn, A, B, M, N, K, ep, err, max_ctas);
    return;
  }
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
#define APPCORR_GEMM_CASE(E)                                                              \
  case E:                                                                                 \
    if (bn == 512) launch_gemm_2sm<6, E>(A, B, M, N, K, ep, err, max_ctas, st);           \
    else if (bn == 256) launch_gemm<256, 4, E>(A, B, M, N, K, ep, err, max_ctas, st);     \
    else if (bn == 128) launch_gemm<128, 6, E>(A, B, M, N, K, ep, err, max_ctas, st);     \
    else if (bn == 64) launch_gemm<64, 8, E>(A, B, M, N, K, ep, err, max_ctas, st);       \
    else TORCH_CHECK(false, "unsupported BN ", bn);                                       \
    break;
  switch (epi) {
    APPCORR_GEMM_CASE(EPI_BF16)
    APPCORR_GEMM_CASE(EPI_F32)
    APPCORR_GEMM_CASE(EPI_GELU)
    APPCORR_GEMM_CASE(EPI_RESID)
    case EPI_SWIGLU:
      TORCH_CHECK(bn == 256 || bn == 512, "swiglu epilogue uses BN=256 (512: 2-CTA)");
      if (bn == 512) launch_gemm_2sm<6, EPI_SWIGLU>(A, B, M, N, K, ep, err, max_ctas, st);
      else launch_gemm<256, 4, EPI_SWIGLU>(A, B, M, N, K, ep, err, max_ctas, st);
      break;
    case EPI_QKV:
      if (bn == 512) launch_gemm_2sm<6, EPI_QKV>(A, B, M, N, K, ep, err, max_ctas, st);
      else if (bn == 256) launch_gemm<256, 4, EPI_QKV>(A, B, M, N, K, ep, err, max_ctas, st);
      else if (bn == 128) launch_gemm<128, 6, EPI_QKV>(A, B, M, N, K, ep, err, max_ctas, st);
      else if (bn == 64) launch_gemm<64, 8, EPI_QKV>(A, B, M, N, K, ep, err, max_ctas, st);
      else TORCH_CHECK(false, "qkv epilogue uses BN=64, 128 or 256");
      break;
    default:
      TORCH_CHECK(false, "unknown epilogue ", epi);
  }
#undef APPCORR_GEMM_CASE
}

}  // namespace appcorr
