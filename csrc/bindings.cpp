#include <cstdlib>
// Python bindings of the appcorr_b200 native extension (`appcorr_b200._C`).
//
// Every op here launches hand-written sm_100a kernels on the current CUDA stream. Tensor
// arguments are validated on the host (device, dtype, contiguity, alignment) before launch so a
// bad call raises a Python exception instead of faulting the GPU.
#include <torch/extension.h>
#include <c10/cuda/CUDAGuard.h>

#include "ops.h"
#include "registry.h"

namespace py = pybind11;
using at::Tensor;
using c10::optional;

namespace appcorr {

template <typename T = void>
static T* opt_ptr(const optional<Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<T*>(t->data_ptr()) : nullptr;
}

static void check_cuda(const Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
}

static void check_rows_i32(const optional<Tensor>& t, const char* name) {
  if (t.has_value() && t->defined()) {
    check_cuda(*t, name);
    TORCH_CHECK(t->scalar_type() == at::kInt && t->is_contiguous(), name, " must be contiguous int32");
  }
}

// Wait-cycle counters of the persistent GEMM (clock64 sums over CTAs: 0 producer waits for free
// stages; 1-3 MMA waits for a free accumulator / a landed stage / the scales; 4 MMA loop; 5-6
// epilogue waits / body; 7 CTAs; 8-9 scale warps waiting for bytes / storing; 10 epilogue release):
// a CUDA int64 tensor of at least 16 entries, or None to switch them off.
// The counters live on one device; GEMMs launched on any other device run without them.
static unsigned long long* g_gemm_prof = nullptr;
static int g_gemm_prof_device = -1;
void gemm_set_profile(optional<Tensor> counters) {
  if (!counters.has_value()) {
    g_gemm_prof = nullptr;
    g_gemm_prof_device = -1;
    return;
  }
  TORCH_CHECK(counters->is_cuda() && counters->scalar_type() == at::kLong && counters->numel() >= 16 &&
                  counters->is_contiguous(), "gemm profile counters: contiguous CUDA int64 [>= 16]");
  g_gemm_prof = reinterpret_cast<unsigned long long*>(counters->data_ptr());
  g_gemm_prof_device = counters->device().index();
}

void gemm_op(const Tensor& A, const Tensor& B, int64_t epi, int64_t bn, const Tensor& err,
             optional<Tensor> out, optional<Tensor> out_rows, optional<Tensor> bias, optional<Tensor> gamma,
             optional<Tensor> resid, optional<Tensor> resid_rows, optional<Tensor> aux,
             optional<Tensor> aux_rows, int64_t aux_mode, optional<Tensor> resid2, optional<Tensor> q_out,
             optional<Tensor> k_out, optional<Tensor> v_out, optional<Tensor> kv_rows,
             optional<Tensor> tok_idx, int64_t seq_len, optional<Tensor> rope_sin, optional<Tensor> rope_cos,
             int64_t n_prefix, int64_t head_dim, int64_t max_ctas, optional<Tensor> a_scale,
             optional<Tensor> b_scale, int64_t kv_dim, std::vector<int64_t> rs_out, int64_t rs_rows_per_rank,
             int64_t rs_rank, int64_t rs_slot_rows, int64_t rs_ld, optional<Tensor> a_sf, optional<Tensor> b_sf) {
  check_cuda(A, "A");
  check_cuda(B, "B");
  // kind 0: bf16; 1: e4m3; 2: NVFP4 (uint8 rows of packed e2m1 pairs + ue4m3 block scales a_sf / b_sf)
  const int kind = A.scalar_type() == at::kFloat8_e4m3fn ? 1 : (A.scalar_type() == at::kByte ? 2 : 0);
  const bool fp8 = kind != 0;  // both low-precision kinds carry a_scale / b_scale
  TORCH_CHECK((kind == 0 && A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16) ||
                  (kind == 1 && B.scalar_type() == at::kFloat8_e4m3fn) || (kind == 2 && B.scalar_type() == at::kByte),
              "gemm expects bf16 x bf16, e4m3 x e4m3 or nvfp4 (uint8) x nvfp4 operands");
  TORCH_CHECK(fp8 == (a_scale.has_value() && b_scale.has_value()),
              "e4m3 / nvfp4 operands need a_scale [M] and b_scale [N]");
  TORCH_CHECK((kind == 2) == (a_sf.has_value() && b_sf.has_value()), "nvfp4 operands need a_sf and b_sf");
  TORCH_CHECK(A.dim() == 2 && B.dim() == 2 && A.size(1) == B.size(1), "gemm: A [M,K], B [N,K]");
  TORCH_CHECK(A.stride(1) == 1 && B.stride(1) == 1, "gemm operands must have unit inner stride");
  TORCH_CHECK(err.scalar_type() == at::kInt && err.is_cuda(), "err must be a CUDA int32 tensor");
  c10::cuda::CUDAGuard guard(A.device());
  const int M = static_cast<int>(A.size(0));
  const int K = static_cast<int>(A.size(1)) * (kind == 2 ? 2 : 1);
  int N = static_cast<int>(B.size(0));
  TORCH_CHECK(K % (kind == 1 ? 16 : 8) == 0, "gemm: K rows must be a multiple of 16 bytes");
  const uint8_t* sfa = nullptr;
  const uint8_t* sfb = nullptr;
  if (kind == 2) {
    TORCH_CHECK(K % 256 == 0, "nvfp4 gemm: K must be a multiple of 256");
    const long tile_bytes = static_cast<long>(K / 64) * 512;
    for (auto* t : {&a_sf, &b_sf}) {
      TORCH_CHECK((*t)->is_cuda() && (*t)->scalar_type() == at::kByte && (*t)->is_contiguous() &&
                      (reinterpret_cast<uintptr_t>((*t)->data_ptr()) & 15) == 0,
                  "nvfp4 scales: contiguous uint8, 16-byte aligned");
    }
    TORCH_CHECK(a_sf->numel() >= ((M + 127) / 128) * tile_bytes, "a_sf: ceil(M/128) x K/64 x 512 bytes");
    TORCH_CHECK(b_sf->numel() >= ((N + 127) / 128) * tile_bytes, "b_sf: ceil(N/128) x K/64 x 512 bytes");
    sfa = a_sf->data_ptr<uint8_t>();
    sfb = b_sf->data_ptr<uint8_t>();
  }
  if (fp8) {
    TORCH_CHECK(a_scale->scalar_type() == at::kFloat && a_scale->is_contiguous() && a_scale->numel() >= M,
                "a_scale: fp32 [M]");
    TORCH_CHECK(b_scale->scalar_type() == at::kFloat && b_scale->is_contiguous() && b_scale->numel() >= N &&
                    (reinterpret_cast<uintptr_t>(b_scale->data_ptr()) & 15) == 0,
                "b_scale: fp32 [N], 16-byte aligned");
  }
  for (auto* t : {&out_rows, &resid_rows, &aux_rows, &kv_rows, &tok_idx}) check_rows_i32(*t, "row map");
  GemmEpilogue ep{};
  ep.out = opt_ptr(out);
  ep.ldo = out.has_value() ? out->stride(0) : 0;
  ep.out_rows = opt_ptr<const int>(out_rows);
  ep.bias = opt_ptr<const __nv_bfloat16>(bias);
  ep.gamma = opt_ptr<const __nv_bfloat16>(gamma);
  ep.resid = opt_ptr<const __nv_bfloat16>(resid);
  ep.ldr = resid.has_value() ? resid->stride(0) : 0;
  ep.resid_rows = opt_ptr<const int>(resid_rows);
  ep.aux = opt_ptr<__nv_bfloat16>(aux);
  ep.ldaux = aux.has_value() ? aux->stride(0) : 0;
  ep.aux_rows = opt_ptr<const int>(aux_rows);
  ep.aux_mode = static_cast<int>(aux_mode);
  ep.resid2 = opt_ptr<const __nv_bfloat16>(resid2);
  ep.ldr2 = resid2.has_value() ? resid2->stride(0) : 0;
  ep.q_out = opt_ptr<__nv_bfloat16>(q_out);
  ep.k_out = opt_ptr<__nv_bfloat16>(k_out);
  ep.v_out = opt_ptr<__nv_bfloat16>(v_out);
  ep.ld_qkv = q_out.has_value() ? q_out->stride(0) : 0;
  ep.kv_rows = opt_ptr<const int>(kv_rows);
  ep.tok_idx = opt_ptr<const int>(tok_idx);
  ep.seq_len = static_cast<int>(seq_len);
  ep.rope_sin = opt_ptr<const float>(rope_sin);
  ep.rope_cos = opt_ptr<const float>(rope_cos);
  ep.n_prefix = static_cast<int>(n_prefix);
  ep.head_dim = static_cast<int>(head_dim);
  ep.a_scale = fp8 ? a_scale->data_ptr<float>() : nullptr;
  ep.b_scale = fp8 ? b_scale->data_ptr<float>() : nullptr;
  ep.sfa = sfa;
  ep.sfb = sfb;
  ep.sf_kt = K / 64;
  ep.prof = A.device().index() == g_gemm_prof_device ? g_gemm_prof : nullptr;
  if (!rs_out.empty()) {
    TORCH_CHECK(epi == EPI_BF16 && rs_out.size() <= 8 && rs_rows_per_rank > 0 && rs_ld % 8 == 0,
                "gemm: the reduce-scatter epilogue is EPI_BF16 with 1..8 slot buffers");
    for (size_t r = 0; r < rs_out.size(); ++r) ep.rs_out[r] = reinterpret_cast<__nv_bfloat16*>(rs_out[r]);
    ep.rs_rows_per_rank = static_cast<int>(rs_rows_per_rank);
    ep.rs_rank = static_cast<int>(rs_rank);
    ep.rs_slot_rows = rs_slot_rows;
    ep.ldo = rs_ld;
  }
  if (epi == EPI_QKV) {
    TORCH_CHECK(q_out && k_out && v_out, "qkv epilogue needs q_out, k_out, v_out");
    if (kv_dim > 0) {  // grouped-query: rows are [q (dim) | k (kv_dim) | v (kv_dim)]
      ep.dim = N - 2 * static_cast<int>(kv_dim);
      ep.kv_dim = static_cast<int>(kv_dim);
      TORCH_CHECK(ep.dim > 0, "qkv: kv_dim too large");
      TORCH_CHECK(k_out->stride(0) == v_out->stride(0), "qkv: k_out and v_out need one row stride");
      ep.ld_kv = k_out->stride(0);
    } else {
      TORCH_CHECK(N % 3 == 0, "qkv weight rows must be 3*dim");
      ep.dim = N / 3;
    }
    const int tile_n = bn == 512 ? 256 : (bn == 513 ? 128 : static_cast<int>(bn));  // 512 / 513: 2-CTA tiles
    TORCH_CHECK(ep.dim % tile_n == 0 && (ep.kv_dim == 0 || ep.kv_dim % tile_n == 0),
                "qkv: q and kv widths must be multiples of the tile width");
    TORCH_CHECK(head_dim == 64 || head_dim == 128, "qkv: head_dim must be 64 or 128");
    TORCH_CHECK(tile_n % head_dim == 0, "qkv: tile width must be a multiple of head_dim");
    TORCH_CHECK(tok_idx.has_value() || seq_len > 0, "qkv: need tok_idx or seq_len");
  } else if (rs_out.empty()) {
    TORCH_CHECK(out.has_value(), "gemm: out is required");
    check_cuda(*out, "out");
    TORCH_CHECK(out->stride(1) == 1, "out must have unit inner stride");
    if (epi == EPI_SWIGLU) {
      TORCH_CHECK(N % 256 == 0, "swiglu: packed w1||w2 rows must be a multiple of 256");
    } else {
      TORCH_CHECK(N % 32 == 0, "gemm: N must be a multiple of 32 (pad the weight)");
    }
    if (epi == EPI_RESID) TORCH_CHECK(resid.has_value() && gamma.has_value(), "resid epilogue needs resid, gamma");
    if (aux_mode == AUX_OUT_MINUS) TORCH_CHECK(resid2.has_value(), "AUX_OUT_MINUS needs resid2");
  }
  if (M == 0) return;
  gemm_dispatch(static_cast<int>(epi), static_cast<int>(bn), A, B, M, N, K, ep, err.data_ptr<int>(),
                static_cast<int>(max_ctas), kind);
}

}  // namespace appcorr

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  using namespace appcorr;
  m.doc() = "appcorr_b200 native sm_100a kernels";
  m.def("gemm_set_profile", &gemm_set_profile, py::arg("counters") = py::none());
  m.def("gemm", &gemm_op, py::arg("A"), py::arg("B"), py::arg("epi"), py::arg("bn"), py::arg("err"),
        py::arg("out") = py::none(), py::arg("out_rows") = py::none(), py::arg("bias") = py::none(),
        py::arg("gamma") = py::none(), py::arg("resid") = py::none(), py::arg("resid_rows") = py::none(),
        py::arg("aux") = py::none(), py::arg("aux_rows") = py::none(), py::arg("aux_mode") = 0,
        py::arg("resid2") = py::none(), py::arg("q_out") = py::none(), py::arg("k_out") = py::none(),
        py::arg("v_out") = py::none(), py::arg("kv_rows") = py::none(), py::arg("tok_idx") = py::none(),
        py::arg("seq_len") = 0, py::arg("rope_sin") = py::none(), py::arg("rope_cos") = py::none(),
        py::arg("n_prefix") = 0, py::arg("head_dim") = 128, py::arg("max_ctas") = 0,
        py::arg("a_scale") = py::none(), py::arg("b_scale") = py::none(), py::arg("kv_dim") = 0,
        py::arg("rs_out") = std::vector<int64_t>{}, py::arg("rs_rows_per_rank") = 0, py::arg("rs_rank") = 0,
        py::arg("rs_slot_rows") = 0, py::arg("rs_ld") = 0, py::arg("a_sf") = py::none(), py::arg("b_sf") = py::none());
  m.attr("EPI_BF16") = static_cast<int>(EPI_BF16);
  m.attr("EPI_F32") = static_cast<int>(EPI_F32);
  m.attr("EPI_GELU") = static_cast<int>(EPI_GELU);
  m.attr("EPI_SWIGLU") = static_cast<int>(EPI_SWIGLU);
  m.attr("EPI_RESID") = static_cast<int>(EPI_RESID);
  m.attr("EPI_QKV") = static_cast<int>(EPI_QKV);
  m.attr("AUX_NONE") = static_cast<int>(AUX_NONE);
  m.attr("AUX_SET") = static_cast<int>(AUX_SET);
  m.attr("AUX_ADD") = static_cast<int>(AUX_ADD);
  m.attr("AUX_OUT_MINUS") = static_cast<int>(AUX_OUT_MINUS);
  register_elementwise_ops(m);
  register_attention_ops(m);
  register_comm_ops(m);
  register_sp_ops(m);
  register_msda_ops(m);
  register_conv_ops(m);
  register_attention_sm100_ops(m);
  register_pscore_sm100_ops(m);
  register_token_prune_ops(m);
}
