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
//               base 2 (scale folded into one FFMA before ex2.approx), P (bf16) written to one of
//               two shared-memory buffers in the K-major swizzled layout the MMA reads, so the
//               exponentials of block j+1 overlap PV_j. Max and sum use 8 independent partial
//               chains. O is rescaled in TMEM only when a row's running max grows by more than
//               2^8 (otherwise the stale max is kept; the final 1/l normalisation is exact either
//               way); only then does the softmax wait for PV_{j-1}. Finally O is read from TMEM,
//               divided by l and stored.
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
  int Hkv;                  // key/value heads (grouped-query attention: head h reads kv head h / (H / Hkv))
  int causal;               // 1: query row i sees keys 0..qpos(i) only
  const int* q_pos;         // [B * Tq] key-axis position of each query row (causal; nullptr: i + Tk - Tq)
  const int* block_table;   // [B, max_blocks] physical 128-row page of each key block (nullptr: b * Tk + j * 128)
  int max_blocks;
  const int* q_lo;          // [B * Tq] first key each query row may see (nullptr: 0); with causal / q_pos
                            // as the last one this gives per-query key ranges (windowed attention)
};

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int DH>
__global__ void __launch_bounds__(kFaThreads, 1)
    fa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, FaParams p) {
  constexpr int NCH = DH / 64;                          // 64-column chunks per row
  constexpr uint32_t CHUNK_BYTES = 128 * 128;           // one [128 rows x 64 cols] bf16 box
  constexpr uint32_t Q_BYTES = NCH * CHUNK_BYTES;
  constexpr uint32_t KV_BYTES = NCH * CHUNK_BYTES;      // per K (or V) stage
  constexpr uint32_t P_BYTES = 2 * CHUNK_BYTES;         // [128 q x 128 keys], two buffers
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
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * P_BYTES);
  uint64_t* q_full = bars;           // 1
  uint64_t* kv_full = bars + 1;      // 2
  uint64_t* kv_empty = bars + 3;     // 2
  uint64_t* s_full = bars + 5;       // 2
  uint64_t* s_free = bars + 7;       // 2
  uint64_t* p_full = bars + 9;       // 2
  uint64_t* p_empty = bars + 11;     // 2 (completes when PV of that buffer is done)
  uint64_t* o_full = bars + 13;      // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 14);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kFaBM;
  const int kvh = h / (p.H / p.Hkv);
  __shared__ int s_nkb, s_kb0;

  if (warp == 0 && lane == 0) {
    mbar_init(smem_addr(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&kv_full[i]), 1);
      mbar_init(smem_addr(&kv_empty[i]), 1);
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&s_free[i]), 128);
      mbar_init(smem_addr(&p_full[i]), 128);
      mbar_init(smem_addr(&p_empty[i]), 1);
    }
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
  if (warp == 2) {  // key blocks this tile needs: all of them, or (causal) up to its last query's position
    int nk = (p.Tk + kFaBN - 1) / kFaBN;
    if (p.causal) {
      int mq = 0;
      for (int r = lane; r < kFaBM; r += 32) {
        const int qi = min(q0 + r, p.Tq - 1);
        mq = max(mq, p.q_pos ? p.q_pos[(long)b * p.Tq + qi] : qi + p.Tk - p.Tq);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mq = max(mq, __shfl_xor_sync(0xffffffffu, mq, o));
      nk = max(1, min(nk, mq / kFaBN + 1));
    }
    int kb0 = 0;  // first key block (per-query lower bounds: the tile's smallest)
    if (p.q_lo) {
      int lo = 0x7FFFFFFF;
      for (int r = lane; r < kFaBM; r += 32) lo = min(lo, p.q_lo[(long)b * p.Tq + min(q0 + r, p.Tq - 1)]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      kb0 = min(max(lo, 0) / kFaBN, nk - 1);
    }
    if (lane == 0) {
      s_nkb = nk - kb0;
      s_kb0 = kb0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkb = s_nkb;   // key blocks visited: kb0 .. kb0 + nkb - 1
  const int kb0 = s_kb0;

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
        const int jb = kb0 + j;
        const int row = p.block_table ? p.block_table[(long)b * p.max_blocks + jb] * kFaBN : b * p.Tk + jb * kFaBN;
        for (int c = 0; c < NCH; ++c) {
          tma_load_2d(smem_addr(sK + s * KV_BYTES + c * CHUNK_BYTES), &tmK, fb, kvh * DH + c * 64, row);
          tma_load_2d(smem_addr(sV + s * KV_BYTES + c * CHUNK_BYTES), &tmV, fb, kvh * DH + c * 64, row);
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
        const int s = j & 1;
        if (!mbar_wait(smem_addr(&p_full[s]), (j >> 1) & 1, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t pa = smem_addr(sP + s * P_BYTES), va = smem_addr(sV + s * KV_BYTES);
#pragma unroll
        for (int k = 0; k < kFaBN / 16; ++k) {
          const uint32_t aoff = (k >> 2) * CHUNK_BYTES + (k & 3) * 32;
          umma_f16(tmem + O_COL, sw128_kmajor_desc(pa + aoff), sw128_mnmajor_desc(va + k * 2048, CHUNK_BYTES, 1024),
                   IDESC_O, (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(smem_addr(&p_empty[s]));
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
    const int rsw = row & 7;
    const float sl2 = p.scale_log2;
    int qpos = 0x7FFFFFFF;  // last key this row may see
    if (p.causal) {
      const int qi = min(q0 + row, p.Tq - 1);
      qpos = p.q_pos ? p.q_pos[(long)b * p.Tq + qi] : qi + p.Tk - p.Tq;
    }
    const int qlo = p.q_lo ? p.q_lo[(long)b * p.Tq + min(q0 + row, p.Tq - 1)] : 0;  // first key it may see
    // m_run: running max of the raw scores; exponent = S * sl2 - m_run * sl2 (one FFMA)
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
        for (int t = 0; t < 32; ++t) sv[c * 32 + t] = __uint_as_float(r[t]);
      }
      tc_fence_before();
      mbar_arrive(smem_addr(&s_free[s]));
      const int kbase = (kb0 + j) * kFaBN;
      const int klim = min(p.Tk - 1, qpos);  // keys past Tk do not exist; causal rows stop at qpos
      if (kbase + kFaBN - 1 > klim || kbase < qlo) {
#pragma unroll
        for (int t = 0; t < kFaBN; ++t)
          if (kbase + t > klim || kbase + t < qlo) sv[t] = -FLT_MAX;
      }
      float mx8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx8[u] = sv[u];
#pragma unroll
      for (int t = 8; t < kFaBN; ++t) mx8[t & 7] = fmaxf(mx8[t & 7], sv[t]);
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      if (cls_row) {  // keep the CLS row's scaled logits; normalised once the row's max / sum are final
        float* dst = p.cls + ((long)b * p.H + h) * p.Tk + kbase;
        const int n = min(kFaBN, p.Tk - kbase);
#pragma unroll
        for (int t = 0; t < kFaBN; ++t)
          if (t < n) dst[t] = sv[t] * sl2;
      }
      // rescale decision (warp-uniform because tcgen05.ld/st are warp-collective)
      const bool grow = (mx - m_run) * sl2 > kRescaleThreshold;
      const bool any_grow = __any_sync(0xffffffffu, grow) && j > 0;
      float corr = 1.f;
      if (grow || j == 0) {
        const float mnew = fmaxf(m_run, mx);
        corr = (j == 0) ? 0.f : ex2_approx((m_run - mnew) * sl2);
        m_run = mnew;
      }
      if (any_grow) {  // O is being accumulated by PV_{j-1}: wait for it, then rescale in TMEM
        if (!mbar_wait(smem_addr(&p_empty[(j - 1) & 1]), ((j - 1) >> 1) & 1, p.err, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
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
      if (j >= 2) {  // P buffer s is free once PV_{j-2} completed
        if (!mbar_wait(smem_addr(&p_empty[s]), ((j >> 1) & 1) ^ 1, p.err, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      l_run *= (j == 0) ? 0.f : corr;
      const float moff = m_run * sl2;
      uint8_t* prow = sP + s * P_BYTES + row * 128;
      float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < kFaBN / 64; ++c) {
#pragma unroll
        for (int v = 0; v < 8; ++v) {
          float e[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) {
            e[t] = ex2_approx(fmaf(sv[c * 64 + v * 8 + t], sl2, -moff));
            ls8[t] += e[t];
          }
          const uint4 pk = make_uint4(pack_bf16x2(e[0], e[1]), pack_bf16x2(e[2], e[3]), pack_bf16x2(e[4], e[5]),
                                      pack_bf16x2(e[6], e[7]));
          *reinterpret_cast<uint4*>(prow + c * CHUNK_BYTES + ((v ^ rsw) << 4)) = pk;
        }
      }
      l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(smem_addr(&p_full[s]));
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
        p.lse[((long)b * p.H + h) * p.Tq + qrow] = (m_run * sl2 + log2f(l_run)) * 0.69314718055994531f;
    }
    if (p.cls != nullptr && qt == 0 && qd == 0) {  // the warp holding row 0 normalises the CLS row
      __syncwarp();
      const float m0 = __shfl_sync(0xffffffffu, m_run, 0) * sl2;
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

// tcgen05.mma with the A operand in TMEM (P) and B from shared memory.
__device__ __forceinline__ void umma_f16_tmem_a(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// ------------------------------------------------------------------------------ split-row variant
// One 128-row query tile per CTA like fa_fwd_sm100_kernel, with three changes:
//  * P (bf16) is written back into the TMEM columns of its own S block and read from there as
//    the A operand of PV, so shared memory holds Q and a 3-stage K/V ring (the load of block
//    j + 3 is in flight while blocks j + 1 and j + 2 are computed);
//  * tcgen05 MMAs of one thread complete in issue order (issue order S_{j+1}, PV_j), so the
//    completion of S_j implies that of PV_{j-2}, the last reader of that TMEM buffer;
//  * every query row is handled by two softmax threads, each owning 64 of the block's 128 keys: warps 2..5 take columns 0..63 and
// warps 6..9 columns 64..127 (warps w and w + 4 share a TMEM lane quadrant). Per key block the
// two threads of a row swap their partial maxima through shared memory under a 64-thread
// mbarrier (bounded wait, unlike bar.sync), then use the same running max, so the two partial
// row sums add up exactly at the end. Against the one-thread-per-row kernel this halves the
// exponentials and the dependent chains per thread and puts two softmax warps on every
// scheduler to hide the ex2 / tcgen05.ld latencies. Warps whose 32 rows lie past Tq and
// column halves that lie wholly past the last key skip their exponentials.
constexpr int kFaSThreads = 320;
constexpr int kFaPoly8Default = 0;

// POLY8: of every 8 consecutive probabilities a thread computes, the first POLY8 use exp2_poly
// (FMA pipe) and the rest ex2.approx (MUFU), so both pipes share the softmax's exponentials.
template <int DH, int POLY8 = 0>
__global__ void __launch_bounds__(kFaSThreads, 1)
    fa_fwd_split_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, FaParams p) {
  constexpr int NCH = DH / 64;
  constexpr uint32_t CHUNK_BYTES = 128 * 128;
  constexpr uint32_t Q_BYTES = NCH * CHUNK_BYTES;
  constexpr uint32_t KV_BYTES = NCH * CHUNK_BYTES;
  constexpr int NST = 3;  // K/V stages
  constexpr uint32_t IDESC_S = idesc_bf16_f32(kFaBM, kFaBN);
  constexpr uint32_t IDESC_O = idesc_bf16_f32_b(kFaBM, DH, true);
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t O_COL = 2 * kFaBN;
  constexpr int HALF = kFaBN / 2;  // key columns per softmax thread

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Q_BYTES;           // NST stages
  uint8_t* sV = sK + NST * KV_BYTES;    // NST stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + NST * KV_BYTES);
  uint64_t* q_full = bars;           // 1
  uint64_t* kv_full = bars + 1;      // NST
  uint64_t* kv_empty = bars + 4;     // NST
  uint64_t* s_full = bars + 7;       // 2
  uint64_t* p_full = bars + 9;       // 2
  uint64_t* p_empty = bars + 11;     // 2 (PV of that S / P buffer completed)
  uint64_t* o_full = bars + 13;      // 1
  uint64_t* x_bar = bars + 14;       // [quadrant][2] partial-max exchange, + [quadrant] final sum exchange
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 26);
  // [block parity][half][row] partial maxima, rounded up to bf16 so that both halves derive the
  // same (never smaller) running max from the pair (the final 1/l normalisation is exact either way)
  __shared__ bf16 xm[2][2][kFaBM];
  __shared__ int s_nkb, s_kb0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * kFaBM;
  const int kvh = h / (p.H / p.Hkv);

  if (warp == 0 && lane == 0) {
    mbar_init(smem_addr(q_full), 1);
    for (int i = 0; i < NST; ++i) {
      mbar_init(smem_addr(&kv_full[i]), 1);
      mbar_init(smem_addr(&kv_empty[i]), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&p_full[i]), 2 * kFaBM);
      mbar_init(smem_addr(&p_empty[i]), 1);
    }
    mbar_init(smem_addr(o_full), 1);
    for (int i = 0; i < 12; ++i) mbar_init(smem_addr(&x_bar[i]), 64);
    fence_barrier_init();
    tma_prefetch_desc(&tmQ);
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  if (warp == 1) {
    tmem_alloc(smem_addr(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == 2) {
    int nk = (p.Tk + kFaBN - 1) / kFaBN;
    if (p.causal) {
      int mq = 0;
      for (int r = lane; r < kFaBM; r += 32) {
        const int qi = min(q0 + r, p.Tq - 1);
        mq = max(mq, p.q_pos ? p.q_pos[(long)b * p.Tq + qi] : qi + p.Tk - p.Tq);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mq = max(mq, __shfl_xor_sync(0xffffffffu, mq, o));
      nk = max(1, min(nk, mq / kFaBN + 1));
    }
    int kb0 = 0;
    if (p.q_lo) {
      int lo = 0x7FFFFFFF;
      for (int r = lane; r < kFaBM; r += 32) lo = min(lo, p.q_lo[(long)b * p.Tq + min(q0 + r, p.Tq - 1)]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lo = min(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      kb0 = min(max(lo, 0) / kFaBN, nk - 1);
    }
    if (lane == 0) {
      s_nkb = nk - kb0;
      s_kb0 = kb0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkb = s_nkb;
  const int kb0 = s_kb0;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t qb = smem_addr(q_full);
      mbar_arrive_expect_tx(qb, Q_BYTES);
      for (int c = 0; c < NCH; ++c)
        tma_load_2d(smem_addr(sQ + c * CHUNK_BYTES), &tmQ, qb, h * DH + c * 64, b * p.Tq + q0);
      for (int j = 0; j < nkb; ++j) {
        const int s = j % NST;
        const uint32_t ph = (j / NST) & 1;
        if (!mbar_wait(smem_addr(&kv_empty[s]), ph ^ 1, p.err, kErrTimeoutProducer)) break;
        const uint32_t fb = smem_addr(&kv_full[s]);
        mbar_arrive_expect_tx(fb, 2 * KV_BYTES);
        const int jb = kb0 + j;
        const int row = p.block_table ? p.block_table[(long)b * p.max_blocks + jb] * kFaBN : b * p.Tk + jb * kFaBN;
        for (int c = 0; c < NCH; ++c) {
          tma_load_2d(smem_addr(sK + s * KV_BYTES + c * CHUNK_BYTES), &tmK, fb, kvh * DH + c * 64, row);
          tma_load_2d(smem_addr(sV + s * KV_BYTES + c * CHUNK_BYTES), &tmV, fb, kvh * DH + c * 64, row);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(smem_addr(q_full), 0, p.err, kErrTimeoutMma);
      const uint32_t qa = smem_addr(sQ);
      // S_j goes into TMEM buffer j & 1; it is issued after PV_{j-2}, the last reader of P_{j-2}
      // in that buffer, and the softmax threads finished reading S_{j-2} before P_{j-2} was
      // released, so no further wait is needed before overwriting it
      auto issue_s = [&](int j) -> bool {
        const int st = j % NST;
        if (!mbar_wait(smem_addr(&kv_full[st]), (j / NST) & 1, p.err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t ka = smem_addr(sK + st * KV_BYTES);
#pragma unroll
        for (int k = 0; k < DH / 16; ++k) {
          const uint32_t off = (k >> 2) * CHUNK_BYTES + (k & 3) * 32;
          umma_f16(tmem + (j & 1) * kFaBN, sw128_kmajor_desc(qa + off), sw128_kmajor_desc(ka + off), IDESC_S, k > 0);
        }
        umma_commit(smem_addr(&s_full[j & 1]));
        return true;
      };
      if (ok) ok = issue_s(0);
      for (int j = 0; ok && j < nkb; ++j) {
        if (j + 1 < nkb && !issue_s(j + 1)) { ok = false; break; }
        const int s = j & 1;
        if (!mbar_wait(smem_addr(&p_full[s]), (j >> 1) & 1, p.err, kErrTimeoutMma)) { ok = false; break; }
        tc_fence_after();
        const uint32_t va = smem_addr(sV + (j % NST) * KV_BYTES);
#pragma unroll
        for (int k = 0; k < kFaBN / 16; ++k)  // P_j: bf16 pairs in columns 0..63 of S_j's buffer
          umma_f16_tmem_a(tmem + O_COL, tmem + s * kFaBN + k * 8, sw128_mnmajor_desc(va + k * 2048, CHUNK_BYTES, 1024),
                          IDESC_O, (j > 0 || k > 0) ? 1u : 0u);
        umma_commit(smem_addr(&p_empty[s]));
        umma_commit(smem_addr(&kv_empty[j % NST]));
      }
      if (ok) umma_commit(smem_addr(o_full));
    }
  } else {
    const int qd = warp & 3;                 // TMEM lane quadrant
    const int hf = (warp - 2) >> 2;          // key-column half
    const int row = qd * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const int c0 = hf * HALF;
    const bool dead = q0 + qd * 32 >= p.Tq;  // all 32 rows of this warp lie past Tq (warp-uniform)
    float m_run = -FLT_MAX, l_run = 0.f;
    bool ok = true;
    const bool cls_row = p.cls != nullptr && qt == 0 && row == 0;
    const float sl2 = p.scale_log2;
    int qpos = 0x7FFFFFFF;
    if (p.causal) {
      const int qi = min(q0 + row, p.Tq - 1);
      qpos = p.q_pos ? p.q_pos[(long)b * p.Tq + qi] : qi + p.Tk - p.Tq;
    }
    const int qlo = p.q_lo ? p.q_lo[(long)b * p.Tq + min(q0 + row, p.Tq - 1)] : 0;
    for (int j = 0; j < nkb; ++j) {
      const int s = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      if (!mbar_wait(smem_addr(&s_full[s]), ph, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      if (dead) {  // nothing of this warp's rows is ever stored: release P untouched
        tc_fence_before();
        mbar_arrive(smem_addr(&p_full[s]));
        continue;
      }
      float sv[HALF];
      {
        uint32_t r0[32], r1[32];
        tmem_ld32(tmem + lane_base + s * kFaBN + c0, r0);
        tmem_ld32(tmem + lane_base + s * kFaBN + c0 + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          sv[t] = __uint_as_float(r0[t]);
          sv[32 + t] = __uint_as_float(r1[t]);
        }
      }
      const int kbase = (kb0 + j) * kFaBN + c0;
      const int klim = min(p.Tk - 1, qpos);
      const bool cdead = kbase > klim || kbase + HALF - 1 < qlo;  // no key of this half is visible
      if (!cdead && (kbase + HALF - 1 > klim || kbase < qlo)) {
#pragma unroll
        for (int t = 0; t < HALF; ++t)
          if (kbase + t > klim || kbase + t < qlo) sv[t] = -FLT_MAX;
      }
      float mx = -FLT_MAX;
      if (!cdead) {
        float mx8[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mx8[u] = sv[u];
#pragma unroll
        for (int t = 8; t < HALF; ++t) mx8[t & 7] = fmaxf(mx8[t & 7], sv[t]);
        mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                   fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
        if (cls_row) {
          float* dst = p.cls + ((long)b * p.H + h) * p.Tk + kbase;
          const int n = min(HALF, p.Tk - kbase);
#pragma unroll
          for (int t = 0; t < HALF; ++t)
            if (t < n) dst[t] = sv[t] * sl2;
        }
      }
      // swap partial maxima with the other half of the row
      const bf16 mxr = __float2bfloat16_ru(mx);
      xm[s][hf][row] = mxr;
      const uint32_t xb = smem_addr(&x_bar[qd * 2 + s]);
      mbar_arrive(xb);
      if (!mbar_wait(xb, ph, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      mx = fmaxf(__bfloat162float(mxr), __bfloat162float(xm[s][hf ^ 1][row]));
      const bool grow = (mx - m_run) * sl2 > kRescaleThreshold;
      const bool any_grow = __any_sync(0xffffffffu, grow) && j > 0;
      float corr = 1.f;
      if (grow || j == 0) {
        const float mnew = fmaxf(m_run, mx);
        corr = (j == 0) ? 0.f : ex2_approx((m_run - mnew) * sl2);
        m_run = mnew;
      }
      if (any_grow) {  // rescale this half's O columns once PV_{j-1} has completed
        if (!mbar_wait(smem_addr(&p_empty[(j - 1) & 1]), ((j - 1) >> 1) & 1, p.err, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < DH / 64; ++c) {
          uint32_t r[32];
          const uint32_t oa = tmem + lane_base + O_COL + hf * (DH / 2) + c * 32;
          tmem_ld32(oa, r);
          tmem_wait_ld();
#pragma unroll
          for (int t = 0; t < 32; ++t) r[t] = __float_as_uint(__uint_as_float(r[t]) * corr);
          tmem_st32(oa, r);
        }
        tmem_wait_st();
      }
      l_run *= (j == 0) ? 0.f : corr;
      // P of this half: 64 bf16 = 32 columns at S column hf * 32 (the partner's S columns there
      // were read before the max exchange above)
      uint32_t pk[32];
      if (cdead) {
#pragma unroll
        for (int t = 0; t < 32; ++t) pk[t] = 0u;
      } else {
        const float moff = m_run * sl2;
        float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const float x0 = fmaf(sv[2 * t], sl2, -moff), x1 = fmaf(sv[2 * t + 1], sl2, -moff);
          const float e0 = ((2 * t) & 7) < POLY8 ? exp2_poly(x0) : ex2_approx(x0);
          const float e1 = ((2 * t + 1) & 7) < POLY8 ? exp2_poly(x1) : ex2_approx(x1);
          ls8[(2 * t) & 7] += e0;
          ls8[(2 * t + 1) & 7] += e1;
          pk[t] = pack_bf16x2(e0, e1);
        }
        l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      }
      tmem_st32(tmem + lane_base + s * kFaBN + hf * 32, pk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_addr(&p_full[s]));
    }
    if (ok && !dead) ok = mbar_wait(smem_addr(o_full), 0, p.err, kErrTimeoutEpilogue);
    if (ok && !dead) {  // add the two partial row sums (every PV is done, so P's buffer is free)
      float* xl = reinterpret_cast<float*>(sQ);  // [half][row] (Q is no longer read)
      xl[hf * kFaBM + row] = l_run;
      const uint32_t xb = smem_addr(&x_bar[8 + qd]);
      mbar_arrive(xb);
      if (!mbar_wait(xb, 0, p.err, kErrTimeoutEpilogue)) ok = false;
      else l_run += xl[(hf ^ 1) * kFaBM + row];
    }
    if (ok && !dead) {
      tc_fence_after();
      const int qrow = q0 + row;
      const float inv = 1.f / l_run;
      bf16* orow = p.o + ((long)b * p.Tq + qrow) * p.ldo + (long)h * DH + hf * (DH / 2);
#pragma unroll 1
      for (int c = 0; c < DH / 64; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + O_COL + hf * (DH / 2) + c * 32, r);
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
      if (hf == 0 && p.lse != nullptr && qrow < p.Tq)
        p.lse[((long)b * p.H + h) * p.Tq + qrow] = (m_run * sl2 + log2f(l_run)) * 0.69314718055994531f;
      if (p.cls != nullptr && qt == 0 && qd == 0 && hf == 0) {  // both halves' CLS logits are written
        __syncwarp();
        const float m0 = __shfl_sync(0xffffffffu, m_run, 0) * sl2;
        const float inv0 = 1.f / __shfl_sync(0xffffffffu, l_run, 0);
        float* src = p.cls + ((long)b * p.H + h) * p.Tk;
        for (int t = lane; t < p.Tk; t += 32) src[t] = exp2f(src[t] - m0) * inv0;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------ two-tile variant
// One CTA = two 128-row query tiles of one (batch, head) sharing every K / V tile; 10 warps:
//   warp 0      TMA: both Q tiles once; K and V tiles of 128 keys into a 2-stage ring
//   warp 1      MMA (one thread), issue order per key block j:
//                 PV0_j, S0_{j+1}, PV1_j, [release K/V stage j], S1_{j+1}
//               so each tile's softmax of block j+1 overlaps the other tile's PV_j and S_{j+1}.
//               P is written by the softmax warps into the tile's S columns of TMEM (bf16, two per
//               32-bit column) and read from there as the A operand of PV (no shared-memory P);
//               tcgen05 MMAs of one thread complete in issue order, so S_{j+1} overwriting P_j
//               after PV_j was issued is safe, and the completion of S_{j+1} (its commit) also
//               means PV_j has completed, which is when a softmax warp may rescale O in TMEM.
//   warps 2..5  softmax of tile 0, warps 6..9 softmax of tile 1 (one query row per thread).
// TMEM (512 columns): S0 / P0 at 0, S1 / P1 at 128, O0 at 256, O1 at 256 + DH.
constexpr int kFa2Threads = 320;


template <int DH>
__global__ void __launch_bounds__(kFa2Threads, 1)
    fa2_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                         const __grid_constant__ CUtensorMap tmV, FaParams p) {
  constexpr int NCH = DH / 64;
  constexpr uint32_t CHUNK_BYTES = 128 * 128;
  constexpr uint32_t QT_BYTES = NCH * CHUNK_BYTES;   // one 128-row Q tile
  constexpr uint32_t KV_BYTES = NCH * CHUNK_BYTES;   // one K (or V) stage
  constexpr uint32_t IDESC_S = idesc_bf16_f32(kFaBM, kFaBN);
  constexpr uint32_t IDESC_O = idesc_bf16_f32_b(kFaBM, DH, true);
  constexpr uint32_t TMEM_COLS = 512;
  constexpr uint32_t O_COL = 2 * kFaBN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                   // 2 tiles
  uint8_t* sK = sQ + 2 * QT_BYTES;      // 2 stages
  uint8_t* sV = sK + 2 * KV_BYTES;      // 2 stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + 2 * KV_BYTES);
  uint64_t* q_full = bars;              // 1
  uint64_t* kv_full = bars + 1;         // 2
  uint64_t* kv_empty = bars + 3;        // 2
  uint64_t* s_full = bars + 5;          // 2 (per tile)
  uint64_t* p_full = bars + 7;          // 2 (per tile)
  uint64_t* o_full = bars + 9;          // 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  __shared__ int s_nkb;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int q0 = qt * 2 * kFaBM;
  const bool has1 = q0 + kFaBM < p.Tq;  // the second tile holds at least one query row
  const int kvh = h / (p.H / p.Hkv);

  if (warp == 0 && lane == 0) {
    mbar_init(smem_addr(q_full), 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(smem_addr(&kv_full[i]), 1);
      mbar_init(smem_addr(&kv_empty[i]), 1);
      mbar_init(smem_addr(&s_full[i]), 1);
      mbar_init(smem_addr(&p_full[i]), 128);
    }
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
  if (warp == 2) {  // key blocks this CTA needs (causal: up to its last query's position)
    int nk = (p.Tk + kFaBN - 1) / kFaBN;
    if (p.causal) {
      int mq = 0;
      for (int r = lane; r < 2 * kFaBM; r += 32) {
        const int qi = min(q0 + r, p.Tq - 1);
        mq = max(mq, p.q_pos ? p.q_pos[(long)b * p.Tq + qi] : qi + p.Tk - p.Tq);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) mq = max(mq, __shfl_xor_sync(0xffffffffu, mq, o));
      nk = max(1, min(nk, mq / kFaBN + 1));
    }
    if (lane == 0) s_nkb = nk;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nkb = s_nkb;

  if (warp == 0) {
    if (lane == 0) {
      const uint32_t qb = smem_addr(q_full);
      mbar_arrive_expect_tx(qb, 2 * QT_BYTES);
      for (int t = 0; t < 2; ++t)
        for (int c = 0; c < NCH; ++c)
          tma_load_2d(smem_addr(sQ + t * QT_BYTES + c * CHUNK_BYTES), &tmQ, qb, h * DH + c * 64,
                      b * p.Tq + q0 + t * kFaBM);
      for (int j = 0; j < nkb; ++j) {
        const int s = j & 1;
        if (!mbar_wait(smem_addr(&kv_empty[s]), ((j >> 1) & 1) ^ 1, p.err, kErrTimeoutProducer)) break;
        const uint32_t fb = smem_addr(&kv_full[s]);
        mbar_arrive_expect_tx(fb, 2 * KV_BYTES);
        const int row = p.block_table ? p.block_table[(long)b * p.max_blocks + j] * kFaBN : b * p.Tk + j * kFaBN;
        for (int c = 0; c < NCH; ++c) {
          tma_load_2d(smem_addr(sK + s * KV_BYTES + c * CHUNK_BYTES), &tmK, fb, kvh * DH + c * 64, row);
          tma_load_2d(smem_addr(sV + s * KV_BYTES + c * CHUNK_BYTES), &tmV, fb, kvh * DH + c * 64, row);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      bool ok = mbar_wait(smem_addr(q_full), 0, p.err, kErrTimeoutMma);
      auto issue_s = [&](int t, int j) -> bool {
        const int s = j & 1;
        if (t == 0 && !mbar_wait(smem_addr(&kv_full[s]), (j >> 1) & 1, p.err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t qa = smem_addr(sQ + t * QT_BYTES), ka = smem_addr(sK + s * KV_BYTES);
#pragma unroll
        for (int k = 0; k < DH / 16; ++k) {
          const uint32_t off = (k >> 2) * CHUNK_BYTES + (k & 3) * 32;
          umma_f16(tmem + t * kFaBN, sw128_kmajor_desc(qa + off), sw128_kmajor_desc(ka + off), IDESC_S, k > 0);
        }
        umma_commit(smem_addr(&s_full[t]));
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {
        if (!mbar_wait(smem_addr(&p_full[t]), j & 1, p.err, kErrTimeoutMma)) return false;
        tc_fence_after();
        const uint32_t va = smem_addr(sV + (j & 1) * KV_BYTES);
#pragma unroll
        for (int k = 0; k < kFaBN / 16; ++k)
          umma_f16_tmem_a(tmem + O_COL + t * DH, tmem + t * kFaBN + k * 8,
                          sw128_mnmajor_desc(va + k * 2048, CHUNK_BYTES, 1024), IDESC_O, (j > 0 || k > 0) ? 1u : 0u);
        return true;
      };
      if (ok) ok = issue_s(0, 0);
      if (ok && has1) ok = issue_s(1, 0);
      for (int j = 0; ok && j < nkb; ++j) {
        if (!issue_pv(0, j)) { ok = false; break; }
        if (j + 1 < nkb && !issue_s(0, j + 1)) { ok = false; break; }
        if (has1 && !issue_pv(1, j)) { ok = false; break; }
        umma_commit(smem_addr(&kv_empty[j & 1]));
        if (has1 && j + 1 < nkb && !issue_s(1, j + 1)) { ok = false; break; }
      }
      if (ok) umma_commit(smem_addr(o_full));
    }
  } else {
    const int t = (warp - 2) >> 2;                // query tile of this softmax warpgroup
    const int qd = warp & 3;                      // TMEM lane quadrant
    const int row = qd * 32 + lane;               // query row inside the tile
    const uint32_t lane_base = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t s_col = t * kFaBN;
    const int qrow = q0 + t * kFaBM + row;
    float m_run = -FLT_MAX, l_run = 0.f;
    bool ok = t == 0 || has1;
    const bool cls_row = p.cls != nullptr && qt == 0 && t == 0 && row == 0;
    const float sl2 = p.scale_log2;
    int qpos = 0x7FFFFFFF;
    if (p.causal) {
      const int qi = min(qrow, p.Tq - 1);
      qpos = p.q_pos ? p.q_pos[(long)b * p.Tq + qi] : qi + p.Tk - p.Tq;
    }
    for (int j = 0; ok && j < nkb; ++j) {
      if (!mbar_wait(smem_addr(&s_full[t]), j & 1, p.err, kErrTimeoutEpilogue)) { ok = false; break; }
      tc_fence_after();
      const int kbase = j * kFaBN;
      const int klim = min(p.Tk - 1, qpos);
      const bool ragged = kbase + kFaBN - 1 > klim;
      // pass 1: row max (S is read again in pass 2, so only 32 scores are live at a time)
      float mx8[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mx8[u] = -FLT_MAX;
#pragma unroll
      for (int c = 0; c < kFaBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + s_col + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          float x = __uint_as_float(r[u]);
          if (ragged && kbase + c * 32 + u > klim) x = -FLT_MAX;
          mx8[u & 7] = fmaxf(mx8[u & 7], x);
          if (cls_row && kbase + c * 32 + u < p.Tk) p.cls[((long)b * p.H + h) * p.Tk + kbase + c * 32 + u] = x * sl2;
        }
      }
      const float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                             fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      const bool grow = (mx - m_run) * sl2 > kRescaleThreshold;
      const bool any_grow = __any_sync(0xffffffffu, grow) && j > 0;
      float corr = 1.f;
      if (grow || j == 0) {
        const float mnew = fmaxf(m_run, mx);
        corr = (j == 0) ? 0.f : ex2_approx((m_run - mnew) * sl2);
        m_run = mnew;
      }
      if (any_grow) {  // PV_{j-1} of this tile completed before S_j did: O may be rescaled now
#pragma unroll 1
        for (int c = 0; c < DH / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tmem + lane_base + O_COL + t * DH + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int u = 0; u < 32; ++u) r[u] = __float_as_uint(__uint_as_float(r[u]) * corr);
          tmem_st32(tmem + lane_base + O_COL + t * DH + c * 32, r);
        }
      }
      l_run *= (j == 0) ? 0.f : corr;
      const float moff = m_run * sl2;
      float ls8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      // pass 2: P = exp2(S * scale - m) for 64 keys at a time, packed two per 32-bit TMEM column
      // into the tile's S columns [32c, 32c + 32): those scores were consumed by an earlier chunk
#pragma unroll
      for (int c = 0; c < kFaBN / 64; ++c) {
        uint32_t r0[32], r1[32], pk[32];
        tmem_ld32(tmem + lane_base + s_col + c * 64, r0);
        tmem_ld32(tmem + lane_base + s_col + c * 64 + 32, r1);
        tmem_wait_ld();
#pragma unroll
        for (int u = 0; u < 32; ++u) {
          const int k0 = kbase + c * 64 + 2 * u;
          const uint32_t a0 = u < 16 ? r0[2 * u] : r1[2 * u - 32];
          const uint32_t a1 = u < 16 ? r0[2 * u + 1] : r1[2 * u - 31];
          float e0 = ex2_approx(fmaf(__uint_as_float(a0), sl2, -moff));
          float e1 = ex2_approx(fmaf(__uint_as_float(a1), sl2, -moff));
          if (ragged) {
            if (k0 > klim) e0 = 0.f;
            if (k0 + 1 > klim) e1 = 0.f;
          }
          ls8[(2 * u) & 7] += e0;
          ls8[(2 * u + 1) & 7] += e1;
          pk[u] = pack_bf16x2(e0, e1);
        }
        tmem_st32(tmem + lane_base + s_col + c * 32, pk);
      }
      tmem_wait_st();
      l_run += ((ls8[0] + ls8[1]) + (ls8[2] + ls8[3])) + ((ls8[4] + ls8[5]) + (ls8[6] + ls8[7]));
      tc_fence_before();
      mbar_arrive(smem_addr(&p_full[t]));
    }
    if (ok && (t == 0 || has1) && mbar_wait(smem_addr(o_full), 0, p.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      bf16* orow = p.o + ((long)b * p.Tq + qrow) * p.ldo + (long)h * DH;
#pragma unroll 1
      for (int c = 0; c < DH / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tmem + lane_base + O_COL + t * DH + c * 32, r);
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
        p.lse[((long)b * p.H + h) * p.Tq + qrow] = (m_run * sl2 + log2f(l_run)) * 0.69314718055994531f;
    }
    if (p.cls != nullptr && qt == 0 && t == 0 && qd == 0) {  // the warp holding row 0 normalises the CLS row
      __syncwarp();
      const float m0 = __shfl_sync(0xffffffffu, m_run, 0) * sl2;
      const float inv0 = 1.f / __shfl_sync(0xffffffffu, l_run, 0);
      float* src = p.cls + ((long)b * p.H + h) * p.Tk;
      for (int u = lane; u < p.Tk; u += 32) src[u] = exp2f(src[u] - m0) * inv0;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Dynamic shared memory above the per-block opt-in limit is refused here, not at launch.
#define FA_CHECK_ATTR(call)                                                                          \
  do {                                                                                               \
    const cudaError_t e_ = (call);                                                                   \
    TORCH_CHECK(e_ == cudaSuccess, "attention: shared-memory attribute refused: ", cudaGetErrorString(e_)); \
  } while (0)

void attention_sm100_op(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, int64_t B,
                        int64_t Tq, int64_t Tk, int64_t H, int64_t Dh, double scale, c10::optional<at::Tensor> lse,
                        const at::Tensor& err, c10::optional<at::Tensor> cls, int64_t Hkv, bool causal,
                        c10::optional<at::Tensor> q_pos, c10::optional<at::Tensor> block_table, int64_t variant,
                        c10::optional<at::Tensor> q_lo) {
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
  if (Hkv <= 0) Hkv = H;
  TORCH_CHECK(H % Hkv == 0, "attention: H must be a multiple of Hkv");
  int64_t kv_rows = B * Tk;
  int max_blocks = 0;
  if (block_table.has_value()) {
    TORCH_CHECK(block_table->scalar_type() == at::kInt && block_table->dim() == 2 && block_table->size(0) == B &&
                    block_table->is_contiguous(),
                "attention: block_table int32 [B, max_blocks]");
    max_blocks = static_cast<int>(block_table->size(1));
    TORCH_CHECK(max_blocks * 128 >= Tk, "attention: block_table too short for Tk");
    kv_rows = k.size(0);  // the page pool
    TORCH_CHECK(kv_rows % 128 == 0, "attention: paged K/V pool rows must be a multiple of 128");
  }
  if (q_pos.has_value())
    TORCH_CHECK(q_pos->scalar_type() == at::kInt && q_pos->numel() == B * Tq && q_pos->is_contiguous(),
                "attention: q_pos int32 [B*Tq]");
  CUtensorMap tk = make_tmap_bf16_2d(k.data_ptr(), kv_rows, Hkv * Dh, k.stride(-2), kFaBN, 64);
  CUtensorMap tv = make_tmap_bf16_2d(v.data_ptr(), kv_rows, Hkv * Dh, v.stride(-2), kFaBN, 64);
  FaParams p{static_cast<int>(B), static_cast<int>(Tq), static_cast<int>(Tk), static_cast<int>(H),
             static_cast<float>(scale * 1.4426950408889634), reinterpret_cast<bf16*>(o.data_ptr()), o.stride(-2),
             nullptr, nullptr, err.data_ptr<int>(), static_cast<int>(Hkv), causal ? 1 : 0,
             q_pos.has_value() ? q_pos->data_ptr<int>() : nullptr,
             block_table.has_value() ? block_table->data_ptr<int>() : nullptr, max_blocks, nullptr};
  if (q_lo.has_value()) {
    TORCH_CHECK(q_lo->scalar_type() == at::kInt && q_lo->numel() == B * Tq && q_lo->is_contiguous(),
                "attention: q_lo int32 [B*Tq]");
    TORCH_CHECK(variant != 0, "attention: per-query lower key bounds run on the one-tile kernel");
    p.q_lo = q_lo->data_ptr<int>();
  }
  if (cls.has_value()) {
    TORCH_CHECK(cls->scalar_type() == at::kFloat && cls->is_contiguous() && cls->numel() >= B * H * Tk,
                "attention: cls fp32 [B,H,Tk]");
    p.cls = cls->data_ptr<float>();
  }
  if (lse.has_value()) {
    TORCH_CHECK(lse->scalar_type() == at::kFloat && lse->numel() >= B * H * Tq, "attention: lse fp32 [B,H,Tq]");
    p.lse = lse->data_ptr<float>();
  }
  auto st = at::cuda::getCurrentCUDAStream();
  if (variant == 2) {  // one query tile per CTA, two softmax threads per row
    dim3 grid((Tq + kFaBM - 1) / kFaBM, H, B);
    const int smem = static_cast<int>(Dh / 64) * 16384 * 7 + 1024 + 256;  // Q + 3 K/V stages
    if (Dh == 128) {
      // share of exponentials on the FMA pipe (APPCORR_ATTN_POLY8: 0..4 of every 8)
      static const int poly8 = [] {
        const char* e = std::getenv("APPCORR_ATTN_POLY8");
        return e ? std::atoi(e) : kFaPoly8Default;
      }();
      auto launch = [&](auto kern) {
        FA_CHECK_ATTR(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        kern<<<grid, kFaSThreads, smem, st>>>(tq, tk, tv, p);
      };
      if (poly8 == 1) launch(fa_fwd_split_kernel<128, 1>);
      else if (poly8 == 2) launch(fa_fwd_split_kernel<128, 2>);
      else if (poly8 == 3) launch(fa_fwd_split_kernel<128, 3>);
      else if (poly8 == 4) launch(fa_fwd_split_kernel<128, 4>);
      else launch(fa_fwd_split_kernel<128, 0>);
    } else {
      FA_CHECK_ATTR(cudaFuncSetAttribute(fa_fwd_split_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      fa_fwd_split_kernel<64><<<grid, kFaSThreads, smem, st>>>(tq, tk, tv, p);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  if (variant == 0) {  // two query tiles per CTA
    dim3 grid2((Tq + 2 * kFaBM - 1) / (2 * kFaBM), H, B);
    const int nch2 = static_cast<int>(Dh / 64);
    const int smem2 = nch2 * 16384 * 6 + 1024 + 256;
    if (Dh == 128) {
      FA_CHECK_ATTR(cudaFuncSetAttribute(fa2_fwd_sm100_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2));
      fa2_fwd_sm100_kernel<128><<<grid2, kFa2Threads, smem2, st>>>(tq, tk, tv, p);
    } else {
      FA_CHECK_ATTR(cudaFuncSetAttribute(fa2_fwd_sm100_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem2));
      fa2_fwd_sm100_kernel<64><<<grid2, kFa2Threads, smem2, st>>>(tq, tk, tv, p);
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return;
  }
  dim3 grid((Tq + kFaBM - 1) / kFaBM, H, B);
  const int nch = static_cast<int>(Dh / 64);
  const int smem = nch * 16384 * 5 + 4 * 16384 + 1024 + 256;
  if (Dh == 128) {
    FA_CHECK_ATTR(cudaFuncSetAttribute(fa_fwd_sm100_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    fa_fwd_sm100_kernel<128><<<grid, kFaThreads, smem, st>>>(tq, tk, tv, p);
  } else {
    FA_CHECK_ATTR(cudaFuncSetAttribute(fa_fwd_sm100_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    fa_fwd_sm100_kernel<64><<<grid, kFaThreads, smem, st>>>(tq, tk, tv, p);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_attention_sm100_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("attention_sm100", &attention_sm100_op, py::arg("q"), py::arg("k"), py::arg("v"), py::arg("o"), py::arg("B"),
        py::arg("Tq"), py::arg("Tk"), py::arg("H"), py::arg("Dh"), py::arg("scale"), py::arg("lse"), py::arg("err"),
        py::arg("cls") = py::none(), py::arg("Hkv") = 0, py::arg("causal") = false, py::arg("q_pos") = py::none(),
        py::arg("block_table") = py::none(), py::arg("variant") = 0, py::arg("q_lo") = py::none());
}

}  // namespace appcorr
