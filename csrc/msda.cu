// Multi-scale deformable attention (inference forward) for the Mask2Former pixel decoder.
//
// Reference: appcorr/models/dinov3/eval/segmentation/models/utils/ms_deform_attn.py:159-222
// (MSDeformAttn.forward: softmax of the attention logits over levels x points, sampling
// locations = reference point + offset / (W_l, H_l)) and the bilinear gather-and-sum of
// ops/src/cuda/ms_deform_im2col_cuda.cuh (zero padding outside the map, sample at
// (x * W_l - 0.5, y * H_l - 0.5), i.e. grid_sample with align_corners=False).
//
// One warp per (image, query, head): the L*P attention logits are softmaxed across the warp's
// lanes, each lane owns Dh/32 channels of the head, and every bilinear corner is one contiguous
// 64-byte (Dh = 32) row segment of the value map, so a sample costs four coalesced loads. The
// softmax, the location arithmetic and the weighted sum are fused; nothing is materialised.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cfloat>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;
constexpr int kMsdaMaxLevels = 8;

struct MsdaArgs {
  const bf16* value;        // [N, S, M, Dh]
  const float* ref;         // [N, Q, L, 2] (x, y) in [0, 1]
  const bf16* offs;         // [N, Q, M, L, P, 2] (row stride ld_offs per query)
  long ld_offs;
  const bf16* logits;       // [N, Q, M, L*P]   (row stride ld_logits per query)
  long ld_logits;
  bf16* out;                // [N, Q, M * Dh]
  int N, Q, S, M, L, P;
  int H[kMsdaMaxLevels], W[kMsdaMaxLevels], start[kMsdaMaxLevels];
};

template <int DH>
__global__ void __launch_bounds__(256) msda_fwd_kernel(MsdaArgs a) {
  constexpr int CPL = DH / 32;  // channels per lane
  const int warp = (blockIdx.x * (blockDim.x >> 5)) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long total = (long)a.N * a.Q * a.M;
  if (warp >= total) return;
  const int m = warp % a.M;
  const long nq = warp / a.M;
  const int n = static_cast<int>(nq / a.Q);
  const int LP = a.L * a.P;
  // softmax of the L*P logits (LP <= 32 handled one per lane)
  const bf16* lg = a.logits + nq * a.ld_logits + (long)m * LP;
  float z = lane < LP ? __bfloat162float(lg[lane]) : -FLT_MAX;
  float mx = z;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float e = lane < LP ? __expf(z - mx) : 0.f;
  float sum = e;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float wgt = e / sum;
  // sampling location of sample `lane` (lane < LP)
  float sx = 0.f, sy = 0.f;
  if (lane < LP) {
    const int l = lane / a.P;
    const bf16* of = a.offs + nq * a.ld_offs + ((long)m * LP + lane) * 2;
    const float* rp = a.ref + (nq * a.L + l) * 2;
    // location in [0,1] -> pixel coordinate of the sample (align_corners = False)
    sx = (rp[0] + __bfloat162float(of[0]) / a.W[l]) * a.W[l] - 0.5f;
    sy = (rp[1] + __bfloat162float(of[1]) / a.H[l]) * a.H[l] - 0.5f;
  }
  float acc[CPL];
#pragma unroll
  for (int c = 0; c < CPL; ++c) acc[c] = 0.f;
  const long vstride = (long)a.M * DH;  // between value rows
  const bf16* vbase = a.value + (long)n * a.S * vstride + (long)m * DH + lane * CPL;
  for (int s = 0; s < LP; ++s) {
    const int l = s / a.P;
    const float x = __shfl_sync(0xffffffffu, sx, s);
    const float y = __shfl_sync(0xffffffffu, sy, s);
    const float w = __shfl_sync(0xffffffffu, wgt, s);
    const int Hl = a.H[l], Wl = a.W[l];
    if (!(x > -1.f && y > -1.f && x < Wl && y < Hl)) continue;  // entirely outside: zero padding
    const int x0 = static_cast<int>(floorf(x)), y0 = static_cast<int>(floorf(y));
    const float fx = x - x0, fy = y - y0;
    const float cw[4] = {(1.f - fx) * (1.f - fy), fx * (1.f - fy), (1.f - fx) * fy, fx * fy};
    const int cx[4] = {x0, x0 + 1, x0, x0 + 1};
    const int cy[4] = {y0, y0, y0 + 1, y0 + 1};
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (cx[k] < 0 || cy[k] < 0 || cx[k] >= Wl || cy[k] >= Hl) continue;
      const bf16* vp = vbase + (long)(a.start[l] + cy[k] * Wl + cx[k]) * vstride;
      const float ww = w * cw[k];
      if constexpr (CPL == 1) {
        acc[0] += ww * __bfloat162float(vp[0]);
      } else {
#pragma unroll
        for (int c = 0; c < CPL; c += 2) {
          const float2 f = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(vp + c));
          acc[c] += ww * f.x;
          acc[c + 1] += ww * f.y;
        }
      }
    }
  }
  bf16* op = a.out + nq * ((long)a.M * DH) + (long)m * DH + lane * CPL;
#pragma unroll
  for (int c = 0; c < CPL; ++c) op[c] = __float2bfloat16_rn(acc[c]);
}

void msda_op(const at::Tensor& value, const at::Tensor& ref, const at::Tensor& offs, const at::Tensor& logits,
             at::Tensor& out, std::vector<int64_t> shapes, int64_t M, int64_t L, int64_t P) {
  TORCH_CHECK(value.is_cuda() && value.scalar_type() == at::kBFloat16 && value.dim() == 4 && value.is_contiguous(),
              "msda: value bf16 [N, S, M, Dh] contiguous");
  const int N = static_cast<int>(value.size(0)), S = static_cast<int>(value.size(1));
  const int Dh = static_cast<int>(value.size(3));
  TORCH_CHECK(value.size(2) == M && (Dh == 32 || Dh == 64), "msda: head dim 32 or 64");
  TORCH_CHECK(L >= 1 && L <= kMsdaMaxLevels && L * P <= 32, "msda: L <= 8 and L * P <= 32");
  TORCH_CHECK(static_cast<int64_t>(shapes.size()) == 2 * L, "msda: shapes = [H0, W0, H1, W1, ...]");
  const int Q = static_cast<int>(out.size(1));
  TORCH_CHECK(ref.scalar_type() == at::kFloat && ref.is_contiguous() && ref.numel() == (long)N * Q * L * 2,
              "msda: ref fp32 [N, Q, L, 2]");
  TORCH_CHECK(offs.scalar_type() == at::kBFloat16 && offs.stride(-1) == 1 && offs.size(-1) >= M * L * P * 2,
              "msda: offsets bf16 [N*Q, >= M*L*P*2]");
  TORCH_CHECK(logits.scalar_type() == at::kBFloat16 && logits.stride(-1) == 1 && logits.size(-1) >= M * L * P,
              "msda: logits bf16 [N*Q, >= M*L*P]");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.is_contiguous() && out.numel() == (long)N * Q * M * Dh,
              "msda: out bf16 [N, Q, M*Dh]");
  MsdaArgs a{};
  a.value = reinterpret_cast<const bf16*>(value.data_ptr());
  a.ref = ref.data_ptr<float>();
  a.offs = reinterpret_cast<const bf16*>(offs.data_ptr());
  a.ld_offs = offs.stride(-2);
  a.logits = reinterpret_cast<const bf16*>(logits.data_ptr());
  a.ld_logits = logits.stride(-2);
  a.out = reinterpret_cast<bf16*>(out.data_ptr());
  a.N = N;
  a.Q = Q;
  a.S = S;
  a.M = static_cast<int>(M);
  a.L = static_cast<int>(L);
  a.P = static_cast<int>(P);
  int acc = 0;
  for (int l = 0; l < L; ++l) {
    a.H[l] = static_cast<int>(shapes[2 * l]);
    a.W[l] = static_cast<int>(shapes[2 * l + 1]);
    a.start[l] = acc;
    acc += a.H[l] * a.W[l];
  }
  TORCH_CHECK(acc == S, "msda: level shapes must cover the value rows");
  const long warps = (long)N * Q * M;
  if (warps == 0) return;
  c10::cuda::CUDAGuard g(value.device());
  const int grid = static_cast<int>((warps + 7) / 8);
  auto st = at::cuda::getCurrentCUDAStream();
  if (Dh == 32) msda_fwd_kernel<32><<<grid, 256, 0, st>>>(a);
  else msda_fwd_kernel<64><<<grid, 256, 0, st>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_msda_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("msda", &msda_op, py::arg("value"), py::arg("ref"), py::arg("offs"), py::arg("logits"), py::arg("out"),
        py::arg("shapes"), py::arg("M"), py::arg("L"), py::arg("P"));
}

}  // namespace appcorr
