// Allocation-free variant of the CLS-attention patch score. See noalloc.h for who needs it, its
// limits and its rules; the interface has no counterpart in the reference project.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "noalloc.h"

namespace appcorr {
// The two kernels of the regular `cls_attn_pscore` op (csrc/elementwise.cu); this entry point
// launches them unchanged and only supplies a different probability buffer.
__global__ void cls_attn_probs_kernel(const __nv_bfloat16* q, const __nv_bfloat16* k, long ld, long q_bstride, int N,
                                      int H, int Dh, float scale, float* probs);
__global__ void head_mean_kernel(const float* probs, int B, int H, int N, float* out);
}  // namespace appcorr

namespace {

// The [B, H, N] softmax probabilities of the last call. In host code this name is only a
// stand-in; its device address comes from cudaGetSymbolAddress, once per device.
static __device__ __align__(256) float g_pscore_scratch[APPCORR_NOALLOC_PSCORE_MAX_ELEMS];

constexpr int kMaxDevices = 64;
constexpr int kProbThreads = 256;   // matches the kernel's launch bounds
constexpr int kMaxSmem = 200 * 1024;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {nullptr};
thread_local char g_err[256] = "";

int fail(int code, const char* msg) {
  std::snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}

}  // namespace

extern "C" __attribute__((visibility("default"))) const char* appcorr_noalloc_last_error(void) { return g_err; }

extern "C" __attribute__((visibility("default"))) int appcorr_cls_attn_pscore_noalloc(
    const void* q, const void* k, long ld, int B, int N, int H, int head_dim, float scale, float* out,
    cudaStream_t stream) {
  if (q == nullptr || k == nullptr || out == nullptr || B <= 0 || N <= 0 || H <= 0 || head_dim <= 0 ||
      head_dim % 64 != 0 || ld < (long)H * head_dim)
    return fail(APPCORR_NOALLOC_ERR_BAD_ARG, "appcorr_cls_attn_pscore_noalloc: invalid argument");
  // The kernel reads q and k two bf16 values at a time: both pointers 4-byte aligned and an even
  // row stride, or the loads would be misaligned on the device.
  if ((reinterpret_cast<uintptr_t>(q) & 3) != 0 || (reinterpret_cast<uintptr_t>(k) & 3) != 0 || (ld & 1) != 0 ||
      (reinterpret_cast<uintptr_t>(out) & 3) != 0)
    return fail(APPCORR_NOALLOC_ERR_BAD_ARG,
                "appcorr_cls_attn_pscore_noalloc: q/k/out must be 4-byte aligned and ld even");
  if ((long)B * H * N > APPCORR_NOALLOC_PSCORE_MAX_ELEMS)
    return fail(APPCORR_NOALLOC_ERR_TOO_LARGE,
                "appcorr_cls_attn_pscore_noalloc: B*H*N exceeds the scratch array of 1<<20 fp32 values");
  const size_t smem = (size_t)(N + head_dim) * sizeof(float);
  if (smem > (size_t)kMaxSmem)
    return fail(APPCORR_NOALLOC_ERR_TOO_LARGE, "appcorr_cls_attn_pscore_noalloc: sequence too long for shared memory");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices)
    return fail(APPCORR_NOALLOC_ERR_CUDA, "appcorr_cls_attn_pscore_noalloc: no usable current CUDA device");
  float* scratch = nullptr;
  {
    // Set-up on the first call per device (device `dev` is current here).
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_pscore_scratch) != cudaSuccess || p == nullptr)
        return fail(APPCORR_NOALLOC_ERR_CUDA, "appcorr_cls_attn_pscore_noalloc: cudaGetSymbolAddress failed");
      g_scratch_ptr[dev] = static_cast<float*>(p);
    }
    scratch = g_scratch_ptr[dev];
  }
  // The regular op sets this kernel's shared-memory limit to its own size, so the limit is set on
  // every call that needs more than the default 48 KB (no allocation involved).
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(appcorr::cls_attn_probs_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           (int)smem) != cudaSuccess)
    return fail(APPCORR_NOALLOC_ERR_CUDA, "appcorr_cls_attn_pscore_noalloc: cudaFuncSetAttribute failed");
  // Launch errors are read with cudaPeekAtLastError: an error left by earlier, unrelated work is
  // not cleared here, and it is reported as such rather than as this call's launch failure.
  if (cudaPeekAtLastError() != cudaSuccess)
    return fail(APPCORR_NOALLOC_ERR_CUDA, "appcorr_cls_attn_pscore_noalloc: a CUDA error was pending before this call");
  appcorr::cls_attn_probs_kernel<<<dim3(B, H), kProbThreads, smem, stream>>>(
      static_cast<const __nv_bfloat16*>(q), static_cast<const __nv_bfloat16*>(k), ld, (long)N * ld, N, H, head_dim, scale, scratch);
  if (cudaPeekAtLastError() != cudaSuccess)
    return fail(APPCORR_NOALLOC_ERR_CUDA, "appcorr_cls_attn_pscore_noalloc: probability kernel launch failed");
  const long total = (long)B * N;
  appcorr::head_mean_kernel<<<(int)((total + 255) / 256), 256, 0, stream>>>(scratch, B, H, N, out);
  if (cudaPeekAtLastError() != cudaSuccess)
    return fail(APPCORR_NOALLOC_ERR_CUDA, "appcorr_cls_attn_pscore_noalloc: head-mean kernel launch failed");
  g_err[0] = '\0';
  return APPCORR_NOALLOC_OK;
}
