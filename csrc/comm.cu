// Intra-node tensor-parallel communication over NVLink / NVSwitch peer memory.
//
// The reference has no multi-GPU path; this is the communication layer of the tensor-parallel
// ViT engine (appcorr_b200/parallel/tp.py). One process per GPU. Symmetric buffers are plain
// cudaMalloc allocations exported with CUDA IPC handles and mapped into every peer process, so a
// kernel can load and store another GPU's buffer directly; no library collective is involved.
//
//   ipc_alloc / ipc_open / ipc_close / ipc_free   symmetric buffer management
//   tp_barrier          every rank stores `epoch` into slot [my_rank] of every peer's flag array,
//                       then waits (bounded, ~1 s) until its own slots reach `epoch`; release /
//                       acquire at system scope make the preceding writes visible
//   tp_allreduce_epi    one-shot all-reduce fused with the block epilogue: rank r owns rows
//                       [r*M/T, (r+1)*M/T); it sums the T peers' bf16 partial products of those
//                       rows (peer loads), applies  delta = gamma * (sum + bias),
//                       out = resid + delta, and the increment bookkeeping (aux := delta,
//                       aux += delta, or aux := (resid - resid2) + delta), and stores out / aux
//                       rows into every rank's replica (peer stores). Equivalent bytes to a
//                       reduce-scatter + all-gather, in one kernel, with the epilogue fused.
//   tp_allreduce_f32    small fp32 all-reduce (mean) of per-rank vectors (patch scores)
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

// flags: per rank an array of kMaxRanks uint32 slots (slot s written by rank s).
__global__ void tp_barrier_kernel(PeerPtrs flags, int rank, int world, uint32_t epoch, int* err) {
  const int t = threadIdx.x;
  __threadfence_system();
  if (t < world) st_release_sys(reinterpret_cast<uint32_t*>(flags.p[t]) + rank, epoch);
  if (t < world) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(flags.p[rank]) + t;
    const uint64_t t0 = global_timer_ns();
    while (static_cast<int32_t>(ld_acquire_sys(mine) - epoch) < 0) {
      if (global_timer_ns() - t0 > kWaitBudgetNs) {
        record_error(err, kErrTimeoutPeer);
        break;
      }
    }
  }
  __syncthreads();
}

void tp_barrier_op(std::vector<int64_t> flag_ptrs, int64_t rank, int64_t epoch, const at::Tensor& err) {
  const int world = static_cast<int>(flag_ptrs.size());
  TORCH_CHECK(world >= 1 && world <= kMaxRanks, "tp_barrier: 1..8 ranks");
  PeerPtrs f{};
  for (int i = 0; i < world; ++i) f.p[i] = reinterpret_cast<void*>(flag_ptrs[i]);
  tp_barrier_kernel<<<1, 32, 0, at::cuda::getCurrentCUDAStream()>>>(f, static_cast<int>(rank), world,
                                                                    static_cast<uint32_t>(epoch), err.data_ptr<int>());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

// ------------------------------------------------------------------------------ fused all-reduce
struct ArEpi {
  PeerPtrs part;        // bf16 [M, N] partial products, one per rank
  long ldp;
  PeerPtrs out;         // bf16 output replicas (row stride ldo), rows via out_rows
  long ldo;
  const int* out_rows;
  PeerPtrs aux;         // bf16 increment replicas (row stride ldaux), rows via aux_rows
  long ldaux;
  const int* aux_rows;
  int aux_mode;
  const bf16* bias;
  const bf16* gamma;    // nullptr: plain sum (+bias)
  const bf16* resid;    // local, row m (or resid_rows[m])
  long ldr;
  const int* resid_rows;
  const bf16* resid2;   // local, row m (AUX_OUT_MINUS)
  long ldr2;
  int M, N, world, rank;
};

__device__ __forceinline__ void unpack8(const uint4& u, float (&v)[8]) {
  const uint32_t* w = &u.x;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 f = unpack_bf16x2(w[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ uint4 pack8(const float (&v)[8]) {
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}

__global__ void tp_allreduce_epi_kernel(ArEpi e) {
  const int rows_per = (e.M + e.world - 1) / e.world;
  const int lo = e.rank * rows_per, hi = min(e.M, lo + rows_per);
  const int n8 = e.N >> 3;
  const long total = (long)max(hi - lo, 0) * n8;
  for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
    const int m = lo + static_cast<int>(i / n8);
    const int c = static_cast<int>(i - (long)(m - lo) * n8);
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int r = 0; r < e.world; ++r) {
      const uint4 u = reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(e.part.p[r]) + (long)m * e.ldp)[c];
      float v[8];
      unpack8(u, v);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += v[j];
    }
    if (e.bias) {
      float b[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(e.bias) + c), b);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += b[j];
    }
    float o[8], d[8];
    if (e.gamma) {
      float g[8], rs[8];
      unpack8(__ldg(reinterpret_cast<const uint4*>(e.gamma) + c), g);
      const long rr = e.resid_rows ? e.resid_rows[m] : m;
      unpack8(reinterpret_cast<const uint4*>(e.resid + rr * e.ldr)[c], rs);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        d[j] = bf16_round(bf16_round(acc[j]) * g[j]);
        o[j] = rs[j] + d[j];
      }
      if (e.aux_mode != AUX_NONE) {
        const long ar = e.aux_rows ? e.aux_rows[m] : (e.out_rows ? e.out_rows[m] : m);
        float a[8];
        if (e.aux_mode == AUX_SET) {
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] = d[j];
        } else if (e.aux_mode == AUX_ADD) {
          unpack8(reinterpret_cast<const uint4*>(reinterpret_cast<const bf16*>(e.aux.p[e.rank]) + ar * e.ldaux)[c], a);
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] += d[j];
        } else {
          float r2[8];
          unpack8(reinterpret_cast<const uint4*>(e.resid2 + (long)m * e.ldr2)[c], r2);
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] = bf16_round(rs[j] - r2[j]) + d[j];
        }
        const uint4 pa = pack8(a);
        for (int r = 0; r < e.world; ++r)
          reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(e.aux.p[r]) + ar * e.ldaux)[c] = pa;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = acc[j];
    }
    const long orow = e.out_rows ? e.out_rows[m] : m;
    const uint4 po = pack8(o);
    for (int r = 0; r < e.world; ++r)
      reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(e.out.p[r]) + orow * e.ldo)[c] = po;
  }
}

static PeerPtrs to_peers(const std::vector<int64_t>& v) {
  TORCH_CHECK(v.size() <= kMaxRanks, "at most 8 ranks");
  PeerPtrs p{};
  for (size_t i = 0; i < v.size(); ++i) p.p[i] = reinterpret_cast<void*>(v[i]);
  return p;
}

template <typename T = void>
static const T* optp(const c10::optional<at::Tensor>& t) {
  return (t.has_value() && t->defined()) ? reinterpret_cast<const T*>(t->data_ptr()) : nullptr;
}

void tp_allreduce_epi_op(std::vector<int64_t> part, int64_t ldp, std::vector<int64_t> out, int64_t ldo,
                         c10::optional<at::Tensor> out_rows, std::vector<int64_t> aux, int64_t ldaux,
                         c10::optional<at::Tensor> aux_rows, int64_t aux_mode, c10::optional<at::Tensor> bias,
                         c10::optional<at::Tensor> gamma, c10::optional<at::Tensor> resid,
                         c10::optional<at::Tensor> resid_rows, c10::optional<at::Tensor> resid2, int64_t M, int64_t N,
                         int64_t rank) {
  const int world = static_cast<int>(part.size());
  TORCH_CHECK(out.size() == part.size() && (aux.empty() || aux.size() == part.size()), "peer lists must match");
  TORCH_CHECK(N % 8 == 0 && ldp % 8 == 0 && ldo % 8 == 0, "allreduce_epi: N and strides multiples of 8");
  if (gamma.has_value()) TORCH_CHECK(resid.has_value(), "allreduce_epi: gamma needs resid");
  if (aux_mode == AUX_OUT_MINUS) TORCH_CHECK(resid2.has_value(), "allreduce_epi: AUX_OUT_MINUS needs resid2");
  ArEpi e{};
  e.part = to_peers(part);
  e.ldp = ldp;
  e.out = to_peers(out);
  e.ldo = ldo;
  e.out_rows = optp<int>(out_rows);
  if (!aux.empty()) e.aux = to_peers(aux);
  e.ldaux = ldaux;
  e.aux_rows = optp<int>(aux_rows);
  e.aux_mode = aux.empty() ? AUX_NONE : static_cast<int>(aux_mode);
  e.bias = optp<bf16>(bias);
  e.gamma = optp<bf16>(gamma);
  e.resid = optp<bf16>(resid);
  e.ldr = resid.has_value() ? resid->stride(0) : 0;
  e.resid_rows = optp<int>(resid_rows);
  e.resid2 = optp<bf16>(resid2);
  e.ldr2 = resid2.has_value() ? resid2->stride(0) : 0;
  e.M = static_cast<int>(M);
  e.N = static_cast<int>(N);
  e.world = world;
  e.rank = static_cast<int>(rank);
  if (M == 0) return;
  const long work = ((M + world - 1) / world) * (N / 8);
  const int grid = static_cast<int>(std::min<long>((work + 255) / 256, num_sms() * 4L));
  tp_allreduce_epi_kernel<<<std::max(grid, 1), 256, 0, at::cuda::getCurrentCUDAStream()>>>(e);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
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
  m.def("tp_allreduce_epi", &tp_allreduce_epi_op, py::arg("part"), py::arg("ldp"), py::arg("out"), py::arg("ldo"),
        py::arg("out_rows"), py::arg("aux"), py::arg("ldaux"), py::arg("aux_rows"), py::arg("aux_mode"),
        py::arg("bias"), py::arg("gamma"), py::arg("resid"), py::arg("resid_rows"), py::arg("resid2"), py::arg("M"),
        py::arg("N"), py::arg("rank"));
  m.def("tp_mean_f32", &tp_mean_f32_op);
}

}  // namespace appcorr
