// Host-visible declarations shared by the CUDA sources and the pybind11 bindings.
#pragma once
#include <torch/extension.h>
#include <cuda.h>
#include <cuda_bf16.h>

namespace appcorr {

enum EpiKind : int { EPI_BF16 = 0, EPI_F32 = 1, EPI_GELU = 2, EPI_SWIGLU = 3, EPI_RESID = 4, EPI_QKV = 5 };
enum AuxMode : int { AUX_NONE = 0, AUX_SET = 1, AUX_ADD = 2, AUX_OUT_MINUS = 3 };

struct GemmEpilogue {
  void* out;
  long ldo;
  const int* out_rows;          // output row map (row m -> out_rows[m]; <0 drops the row)
  const __nv_bfloat16* bias;    // [N] or nullptr
  const __nv_bfloat16* gamma;   // [N] LayerScale (EPI_RESID)
  const __nv_bfloat16* resid;   // EPI_RESID residual rows
  long ldr;
  const int* resid_rows;        // residual row map (nullptr: row m)
  __nv_bfloat16* aux;           // EPI_RESID side output (per-layer increment cache)
  long ldaux;
  const int* aux_rows;
  int aux_mode;
  const __nv_bfloat16* resid2;  // AUX_OUT_MINUS: aux = (resid - resid2) + delta
  long ldr2;
  // EPI_QKV
  __nv_bfloat16* q_out;
  __nv_bfloat16* k_out;
  __nv_bfloat16* v_out;
  long ld_qkv;
  const int* kv_rows;           // k/v destination rows (nullptr: row m)
  const int* tok_idx;           // token index of row m inside its image (nullptr: m % seq_len)
  int seq_len;
  const float* rope_sin;        // [n_rope_rows, head_dim]
  const float* rope_cos;
  int n_prefix;
  int head_dim;
  int dim;             // q width (= k/v width unless kv_dim is set)
  int kv_dim;          // k / v width (grouped-query attention); 0: same as dim
  long ld_kv;          // row stride of k_out / v_out (0: ld_qkv)
  // FP8 operands: acc * a_scale[m] * b_scale[n] before the epilogue (nullptr: no scaling)
  const float* a_scale;
  const float* b_scale;
  // reduce-scatter epilogue (EPI_BF16): row m is stored to rank owner = (out_rows ? out_rows[m] : m)
  // / rs_rows_per_rank, into its slot buffer rs_out[owner] at row rs_rank * rs_slot_rows + m
  // (a peer store over NVLink unless owner == rs_rank). rs_out[0] == nullptr: off.
  __nv_bfloat16* rs_out[8];
  int rs_rows_per_rank;
  int rs_rank;
  long rs_slot_rows;
  // NVFP4 operands (e2m1 pairs + ue4m3 scales per 16 elements): scale bytes of A and B in the
  // 128-row x 64-element blocked layout, sf_kt = K / 64 blocks per 128-row tile
  const uint8_t* sfa;
  const uint8_t* sfb;
  int sf_kt;
  // optional wait-cycle counters (gemm_set_profile); nullptr: off
  unsigned long long* prof;
};

struct GemmShape {
  int M, N, K;
  int* err;
};


void gemm_dispatch(int epi, int bn, const at::Tensor& A, const at::Tensor& B, int M, int N, int K,
                   const GemmEpilogue& ep, int* err, int max_ctas, int kind);
CUtensorMap make_tmap_bf16_2d(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                              int box_cols);
CUtensorMap make_tmap_u8_2d(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, int box_cols);
int num_sms();

}  // namespace appcorr
