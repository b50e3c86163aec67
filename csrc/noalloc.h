// Allocation-free C entry point of appcorr_b200.
//
// This interface has no counterpart in the reference project. It is for callers that cannot
// allocate device memory themselves: code that runs inside a custom CUDA allocator or a
// memory-pool callback (allocating there would re-enter the allocator), runtimes that reserve all
// device memory at start-up and forbid later cudaMalloc calls, and plain-C hosts that link this
// library without PyTorch and so have no caching allocator to borrow a scratch buffer from.
//
// appcorr_cls_attn_pscore_noalloc computes what the `cls_attn_pscore` op of the Python extension
// computes: for each image b, the softmax over keys of the CLS query's attention logits, averaged
// over heads, written to out[b * N + j] (fp32). The per-head probabilities, which the regular op
// keeps in a caller-provided [B, H, N] buffer, live in a fixed device array inside the library.
//
// Limits and rules:
//  * B * H * N must not exceed APPCORR_NOALLOC_PSCORE_MAX_ELEMS (1 << 20 fp32 values, 4 MiB);
//    larger problems are refused with APPCORR_NOALLOC_ERR_TOO_LARGE and nothing is launched.
//    Every GPU that loads the library keeps this 4 MiB array until the process exits.
//  * (N + head_dim) fp32 values must fit the kernel's shared memory (N up to about 50k tokens).
//  * q and k must be 4-byte aligned with an even row stride `ld`, and out 4-byte aligned; other
//    pointers are refused with APPCORR_NOALLOC_ERR_BAD_ARG before anything is launched.
//  * The first call on a device looks up the array's device address with that device current.
//    With lazy module loading the driver also loads the library's device code, the 4 MiB array
//    included, on that first call. So make the first call per device at start-up: outside any
//    allocator or memory-pool callback and before any stream capture. Later calls allocate nothing.
//  * A CUDA error already pending on the calling thread when the function is entered is not
//    cleared; the call returns APPCORR_NOALLOC_ERR_CUDA without launching.
//  * All calls share the one array, which keeps the last call's contents (every element a call
//    reads is first written by the same call, so nothing needs clearing). Calls that overlap on
//    the GPU (different streams, or different host threads on one device) race on the array;
//    serialise them on one stream.
//  * Neither this function nor anything it calls allocates or frees device memory.
#pragma once
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

#define APPCORR_NOALLOC_PSCORE_MAX_ELEMS (1 << 20)

enum {
  APPCORR_NOALLOC_OK = 0,
  APPCORR_NOALLOC_ERR_TOO_LARGE = 1,
  APPCORR_NOALLOC_ERR_BAD_ARG = 2,
  APPCORR_NOALLOC_ERR_CUDA = 3,
};

// q, k: bf16 row-major [B*N, H*head_dim] with the same row stride `ld` (elements); row b*N of q is
// image b's CLS query. out: fp32 [B*N]. Returns APPCORR_NOALLOC_OK or an error code; the message
// of the last failure on the calling thread is available from appcorr_noalloc_last_error().
int appcorr_cls_attn_pscore_noalloc(const void* q, const void* k, long ld, int B, int N, int H, int head_dim,
                                    float scale, float* out, cudaStream_t stream);

const char* appcorr_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
