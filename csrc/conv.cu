// Convolution building blocks for the dense-prediction heads (DPT depth head, super-resolution
// network): NHWC im2col feeding the tcgen05 GEMM, and bilinear resampling of NHWC maps.
//
//   im2col_nhwc     x [B, H, W, C] bf16 -> rows [B*Ho*Wo, ldo] with column (ky*kw + kx)*C + c
//                   (zero padding outside the map; columns past kh*kw*C are left untouched, so
//                   a padded K stays zero). A KxK convolution is then one GEMM against the weight
//                   reshaped to [Cout, ky, kx, Cin] (see appcorr_b200/models/conv.py).
//   resize_nhwc     bilinear resize of [B, H, W, C] bf16 (align_corners true or false), optionally
//                   adding a second map of the output size (the fusion blocks' skip connection).
// Reference: the DPT head and the Real-ESRGAN network are nn.Conv2d / F.interpolate stacks in the
// reference (appcorr/models/dinov3/eval/depth/..., offload/server/sr/realesrgan.py:102-304).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "sm100_common.cuh"
#include "ops.h"

namespace appcorr {

using bf16 = __nv_bfloat16;

// One thread per 8 channels of one (output pixel, kernel tap).
__global__ void im2col_nhwc_kernel(const bf16* __restrict__ x, int B, int H, int W, int C, int kh, int kw, int stride,
                                   int pad, int Ho, int Wo, bf16* __restrict__ out, long ldo) {
  const int c8 = C >> 3;
  const long total = (long)B * Ho * Wo * kh * kw * c8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int cv = static_cast<int>(i % c8);
    long r = i / c8;
    const int tap = static_cast<int>(r % (kh * kw));
    r /= (kh * kw);
    const int ox = static_cast<int>(r % Wo);
    r /= Wo;
    const int oy = static_cast<int>(r % Ho);
    const int b = static_cast<int>(r / Ho);
    const int ky = tap / kw, kx = tap % kw;
    const int iy = oy * stride - pad + ky, ix = ox * stride - pad + kx;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (iy >= 0 && iy < H && ix >= 0 && ix < W)
      v = reinterpret_cast<const uint4*>(x + (((long)b * H + iy) * W + ix) * C)[cv];
    const long orow = ((long)b * Ho + oy) * Wo + ox;
    reinterpret_cast<uint4*>(out + orow * ldo + (long)tap * C)[cv] = v;
  }
}

void im2col_nhwc_op(const at::Tensor& x, int64_t kh, int64_t kw, int64_t stride, int64_t pad, at::Tensor& out) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 4 && x.is_contiguous(),
              "im2col_nhwc: bf16 [B, H, W, C] contiguous");
  const int B = x.size(0), H = x.size(1), W = x.size(2), C = x.size(3);
  TORCH_CHECK(C % 8 == 0, "im2col_nhwc: C % 8 == 0");
  const int Ho = (H + 2 * pad - kh) / stride + 1, Wo = (W + 2 * pad - kw) / stride + 1;
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 2 && out.size(0) == (long)B * Ho * Wo &&
                  out.size(1) >= kh * kw * C && out.stride(1) == 1 && out.stride(0) % 8 == 0,
              "im2col_nhwc: out bf16 [B*Ho*Wo, >= kh*kw*C]");
  const long total = (long)B * Ho * Wo * kh * kw * (C / 8);
  if (total == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  const int grid = static_cast<int>(std::min<long>((total + 255) / 256, num_sms() * 16L));
  im2col_nhwc_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), B, H, W, C, static_cast<int>(kh), static_cast<int>(kw),
      static_cast<int>(stride), static_cast<int>(pad), Ho, Wo, reinterpret_cast<bf16*>(out.data_ptr()), out.stride(0));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// One thread per 8 channels of one output pixel.
__global__ void resize_nhwc_kernel(const bf16* __restrict__ x, int B, int H, int W, int C, int Ho, int Wo,
                                   int align, const bf16* __restrict__ add, bf16* __restrict__ out) {
  const int c8 = C >> 3;
  const long total = (long)B * Ho * Wo * c8;
  const float sy = align ? (Ho > 1 ? float(H - 1) / (Ho - 1) : 0.f) : float(H) / Ho;
  const float sx = align ? (Wo > 1 ? float(W - 1) / (Wo - 1) : 0.f) : float(W) / Wo;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int cv = static_cast<int>(i % c8);
    long r = i / c8;
    const int ox = static_cast<int>(r % Wo);
    r /= Wo;
    const int oy = static_cast<int>(r % Ho);
    const int b = static_cast<int>(r / Ho);
    float fy = align ? oy * sy : fmaxf((oy + 0.5f) * sy - 0.5f, 0.f);
    float fx = align ? ox * sx : fmaxf((ox + 0.5f) * sx - 0.5f, 0.f);
    const int y0 = min(static_cast<int>(fy), H - 1), x0 = min(static_cast<int>(fx), W - 1);
    const int y1 = min(y0 + 1, H - 1), x1 = min(x0 + 1, W - 1);
    const float wy = fy - y0, wx = fx - x0;
    const uint4* base = reinterpret_cast<const uint4*>(x + (long)b * H * W * C);
    float a[8], bb[8], c[8], d[8], o[8];
    auto ld = [&](int yy, int xx, float (&v)[8]) {
      const uint4 u = base[((long)yy * W + xx) * c8 + cv];
      const uint32_t* w = &u.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(w[k]);
        v[2 * k] = f.x;
        v[2 * k + 1] = f.y;
      }
    };
    ld(y0, x0, a);
    ld(y0, x1, bb);
    ld(y1, x0, c);
    ld(y1, x1, d);
#pragma unroll
    for (int k = 0; k < 8; ++k)
      o[k] = (1.f - wy) * ((1.f - wx) * a[k] + wx * bb[k]) + wy * ((1.f - wx) * c[k] + wx * d[k]);
    const long orow = ((long)b * Ho + oy) * Wo + ox;
    if (add) {
      const uint4 u = reinterpret_cast<const uint4*>(add + orow * C)[cv];
      const uint32_t* w = &u.x;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = unpack_bf16x2(w[k]);
        o[2 * k] += f.x;
        o[2 * k + 1] += f.y;
      }
    }
    reinterpret_cast<uint4*>(out + orow * C)[cv] =
        make_uint4(pack_bf16x2(o[0], o[1]), pack_bf16x2(o[2], o[3]), pack_bf16x2(o[4], o[5]), pack_bf16x2(o[6], o[7]));
  }
}

void resize_nhwc_op(const at::Tensor& x, at::Tensor& out, bool align_corners, c10::optional<at::Tensor> add) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 4 && x.is_contiguous(),
              "resize_nhwc: bf16 [B, H, W, C] contiguous");
  TORCH_CHECK(out.scalar_type() == at::kBFloat16 && out.dim() == 4 && out.is_contiguous() && out.size(0) == x.size(0) &&
                  out.size(3) == x.size(3),
              "resize_nhwc: out bf16 [B, Ho, Wo, C]");
  const int C = x.size(3);
  TORCH_CHECK(C % 8 == 0, "resize_nhwc: C % 8 == 0");
  const bf16* ap = nullptr;
  if (add.has_value()) {
    TORCH_CHECK(add->sizes() == out.sizes() && add->is_contiguous() && add->scalar_type() == at::kBFloat16,
                "resize_nhwc: add must match out");
    ap = reinterpret_cast<const bf16*>(add->data_ptr());
  }
  const long total = out.numel() / 8;
  if (total == 0) return;
  c10::cuda::CUDAGuard g(x.device());
  const int grid = static_cast<int>(std::min<long>((total + 255) / 256, num_sms() * 16L));
  resize_nhwc_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<const bf16*>(x.data_ptr()), x.size(0), x.size(1), x.size(2), C, out.size(1), out.size(2),
      align_corners ? 1 : 0, ap, reinterpret_cast<bf16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_conv_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("im2col_nhwc", &im2col_nhwc_op, py::arg("x"), py::arg("kh"), py::arg("kw"), py::arg("stride"), py::arg("pad"),
        py::arg("out"));
  m.def("resize_nhwc", &resize_nhwc_op, py::arg("x"), py::arg("out"), py::arg("align_corners"),
        py::arg("add") = py::none());
}

}  // namespace appcorr
