// Intra-node tensor-parallel communication over NVLink / NVSwitch peer memory.
//
// The reference has no multi-GPU path; this is the communication layer of the tensor-parallel
// ViT engine (appcorr_b200/parallel/tp.py). One process per GPU. Symmetric buffers are plain
// cudaMalloc allocations exported with CUDA IPC handles and mapped into every peer process, so a
// kernel can load and store another GPU's buffer directly; no library collective is involved.
//
//   ipc_alloc / ipc_open / ipc_close / ipc_free   symmetric buffer management
//   tp_barrier          every rank advances its device-side epoch counter, stores the epoch into
//                       slot [my_rank] of every peer's flag array, then waits (bounded, ~1 s)
//                       until its own slots reach it; release / acquire at system scope make the
//                       preceding writes visible. Graph-capturable: no host-side state.
//   tp_mean_f32         small fp32 all-reduce (mean) of per-rank vectors (patch scores)
// The reduce-scatter and all-gather of the layer activations are fused into the GEMM epilogue
// (csrc/gemm_sm100.cu, rs_out) and into the owner-side row kernel (csrc/tp_sp.cu).
//
// Every wait is bounded: on expiry the kernel records kErrTimeoutPeer in the caller's error word
// and returns, so a missing peer surfaces as a host-side error instead of a hung GPU.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "sm100_common.cuh"
#include "ops.h"

namespace py = pybind11;

namespace appcorr {

using bf16 = __nv_bfloat16;
constexpr int kMaxRanks = 8;

struct PeerPtrs {
  void* p[kMaxRanks];
};

// ------------------------------------------------------------------------------ memory
std::tuple<int64_t, py::bytes> ipc_alloc(int64_t bytes) {
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&ptr, bytes));
  C10_CUDA_CHECK(cudaMemset(ptr, 0, bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, ptr));
  return {reinterpret_cast<int64_t>(ptr), py::bytes(reinterpret_cast<const char*>(&h), sizeof(h))};
}

int64_t ipc_open(py::bytes handle) {
  std::string s = handle;
  TORCH_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* ptr = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(ptr);
}

void ipc_close(int64_t ptr) { C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }
void ipc_free(int64_t ptr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

at::Tensor tensor_from_ptr(int64_t ptr, std::vector<int64_t> shape, at::ScalarType dtype, int64_t device) {
  auto opts = at::TensorOptions().dtype(dtype).device(at::kCUDA, device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), shape, [](void*) {}, opts);
}

// ------------------------------------------------------------------------------ barrier
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// flags: per rank an array of kFlagWords uint32: slots [0, kMaxRanks) are written by the ranks
// (slot s by rank s); slot kMaxRanks is this rank's own epoch counter. The epoch lives in device
// memory, so a captured barrier (CUDA graph) takes a fresh epoch on every replay. Barriers of one
// channel run in stream order on every rank, so the counters of all ranks stay equal.
constexpr int kFlagWords = 16;
__global__ void tp_barrier_kernel(PeerPtrs flags, int rank, int world, int* err) {
  const int t = threadIdx.x;
  __shared__ uint32_t s_epoch;
  uint32_t* counter = reinterpret_cast<uint32_t*>(flags.p[rank]) + kMaxRanks;
  if (t == 0) s_epoch = (*counter + 1u) & 0x7FFFFFFFu;
  __syncthreads();
  const uint32_t epoch = s_epoch;
  __threadfence_system();
  if (t < world) st_release_sys(reinterpret_cast<uint32_t*>(flags.p[t]) + rank, epoch);
  if (t < world) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(flags.p[rank]) + t;
    const uint64_t t0 = global_timer_ns();
    while (static_cast<int32_t>((ld_acquire_sys(mine) - epoch) << 1) < 0) {
      if (global_timer_ns() - t0 > kWaitBudgetNs) {
        record_error(err, kErrTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
  if (t == 0) *counter = epoch;
}

void tp_barrier_op(std::vector<int64_t> flag_ptrs, int64_t rank, const at::Tensor& err) {
  const int world = static_cast<int>(flag_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "tp_barrier: 1..8 ranks");
  PeerPtrs f{};
  for (int i = 0; i < world; ++i) f.p[i] = reinterpret_cast<void*>(flag_ptrs[i]);
  tp_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(f, static_cast<int>(rank), world,
                                                                    err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

static PeerPtrs to_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() <= kMaxRanks, "at most 8 ranks");
  PeerPtrs p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = reinterpret_cast<void*>(v[i]);
  return p;
}

// ------------------------------------------------------------------------------ small fp32 mean
__global__ void tp_mean_f32_kernel(PeerPtrs src, int world, float* dst, long n) {
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < world; ++r) s += reinterpret_cast<const float*>(src.p[r])[i];
    dst[i] = s / world;
  }
}

void tp_mean_f32_op(std::vector<int64_t> src, at::Tensor& dst) {
  TORCH_CHECK(dst.scalar_type() == at::kFloat && dst.is_contiguous(), "tp_mean_f32: fp32 dst");
  const long n = dst.numel();
  if (n == 0) return;
  tp_mean_f32_kernel<<<static_cast<int>(std::min<long>((n + 255) / 256, 1024)), 256, 0,
                       at::cuda::getCurrentCUDAStream()>>>(to_peers(src), static_cast<int>(src.size()),
                                                           dst.data_ptr<float>(), n);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_comm_ops(pybind11::module_& m) {
  namespace py = pybind11;
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
  m.def("ipc_free", &ipc_free);
  m.def("tensor_from_ptr", &tensor_from_ptr);
  m.def("tp_barrier", &tp_barrier_op);
  m.def("tp_mean_f32", &tp_mean_f32_op);
}

}  // namespace appcorr
