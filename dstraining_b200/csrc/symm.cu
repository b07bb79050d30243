// Peer ("symmetric") memory over NVLink and the fused data-parallel kernel.
//
// Runtime: every rank of a group allocates an equal-sized device buffer,
// exports a CUDA IPC handle, the handles are exchanged over the process
// group (Python side) and each rank maps its peers' buffers, so kernels can
// load from and store to any peer's buffer directly (NVLink 5 through
// NVSwitch). Synchronisation between ranks uses 32-bit flags in a peer buffer:
// a rank publishes progress by storing a launch epoch into slot [kind][rank]
// of every peer's flag array (release, system scope) and waits, bounded by
// %globaltimer, until every peer has published at least that epoch into its
// own array (acquire, system scope). An expired wait records an error code in
// the status word and the kernel returns; nothing traps or spins forever.
//
// Fused DP step (one launch per gradient bucket, on a side stream so it
// overlaps the rest of backward):
//   1. publish "my bucket gradients are complete"; wait for every peer's;
//   2. rank r owns elements [r*S, (r+1)*S) of the bucket: sum the bf16
//      gradients of all ranks in rank order 0..N-1 (fp32), scale by 1/N;
//   3. Adam on the owned fp32 master slice (the moments are sharded: ZeRO-1);
//   4. round to bf16 and store into EVERY rank's parameter buffer (the
//      all-gather, as peer stores);
//   5. the last CTA publishes "my slice is written" and waits for all peers'
//      slices, so when the kernel completes this rank's parameters are whole.
// No TMA: plain 16-byte peer loads/stores.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>

#include "common.h"
#include "ptx.cuh"

namespace dst {
namespace symm {

constexpr int kMaxRanks = 8;

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Wait until flags[kind * kMaxRanks + p] >= epoch for all p < n (wrap-safe).
__device__ bool wait_all(const uint32_t* flags, int kind, int n, uint32_t epoch, int* status) {
  const unsigned long long t0 = globaltimer_ns();
  for (int p = 0; p < n; ++p) {
    const uint32_t* f = flags + kind * kMaxRanks + p;
    while (static_cast<int32_t>(ld_acquire_sys(f) - epoch) < 0) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) {
        record_status(status, kTimeoutPeer);
        return false;
      }
    }
  }
  return true;
}

// Publish `epoch` into slot [kind][rank] of every peer's flag array.
__device__ void publish(uint32_t* const* peer_flags, int kind, int rank, int n, uint32_t epoch) {
  __threadfence_system();
  for (int p = 0; p < n; ++p) st_release_sys(peer_flags[p] + kind * kMaxRanks + rank, epoch);
}

struct DpArgs {
  __nv_bfloat16* grad[kMaxRanks];   // each rank's bucket gradient buffer
  __nv_bfloat16* param[kMaxRanks];  // each rank's bucket parameter buffer
  uint32_t* flags[kMaxRanks];       // each rank's flag array
  float* master;                    // owned slice, fp32
  float* m;
  float* v;
  unsigned int* done_ctas;          // local counter (reset by the last CTA)
  int64_t slice;                    // elements per rank (multiple of 8)
  int64_t valid;                    // bucket elements that are real (rest is padding)
  int rank, n;
  uint32_t epoch;
  float beta1, beta2, eps, step_size, inv_sqrt_bc2, inv_n;
  float decay;  // decoupled weight decay factor 1 - lr * wd (1: plain Adam)
  int* status;
};

constexpr int kReady = 0;
constexpr int kWritten = 1;

__global__ void __launch_bounds__(256) fused_dp_adam_kernel(const __grid_constant__ DpArgs a) {
  __shared__ bool go;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) publish(a.flags, kReady, a.rank, a.n, a.epoch);
    go = wait_all(a.flags[a.rank], kReady, a.n, a.epoch, a.status);
  }
  __syncthreads();
  if (go) {
    const int64_t base = static_cast<int64_t>(a.rank) * a.slice;
    const int64_t nvec = a.slice / 8;
    for (int64_t vi = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; vi < nvec;
         vi += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int64_t e = vi * 8;  // offset inside the owned slice
      float g[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      for (int p = 0; p < a.n; ++p) {  // fixed rank order: identical sums on every rank
        const uint4 u = *reinterpret_cast<const uint4*>(a.grad[p] + base + e);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __bfloat1622float2(h[j]);
          g[2 * j] += f.x;
          g[2 * j + 1] += f.y;
        }
      }
      float4* M4 = reinterpret_cast<float4*>(a.master + e);
      float4* A4 = reinterpret_cast<float4*>(a.m + e);
      float4* V4 = reinterpret_cast<float4*>(a.v + e);
      float w[8], mm[8], vv[8];
      *reinterpret_cast<float4*>(w) = M4[0];
      *reinterpret_cast<float4*>(w + 4) = M4[1];
      *reinterpret_cast<float4*>(mm) = A4[0];
      *reinterpret_cast<float4*>(mm + 4) = A4[1];
      *reinterpret_cast<float4*>(vv) = V4[0];
      *reinterpret_cast<float4*>(vv + 4) = V4[1];
      uint4 out;
      __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&out);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (base + e + j < a.valid) {
          const float gj = g[j] * a.inv_n;
          mm[j] = mm[j] + (gj - mm[j]) * (1.f - a.beta1);
          vv[j] = vv[j] * a.beta2 + (1.f - a.beta2) * gj * gj;
          w[j] = w[j] * a.decay - a.step_size * (mm[j] / (sqrtf(vv[j]) * a.inv_sqrt_bc2 + a.eps));
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(w[2 * j], w[2 * j + 1]);
      M4[0] = *reinterpret_cast<float4*>(w);
      M4[1] = *reinterpret_cast<float4*>(w + 4);
      A4[0] = *reinterpret_cast<float4*>(mm);
      A4[1] = *reinterpret_cast<float4*>(mm + 4);
      V4[0] = *reinterpret_cast<float4*>(vv);
      V4[1] = *reinterpret_cast<float4*>(vv + 4);
      for (int p = 0; p < a.n; ++p) *reinterpret_cast<uint4*>(a.param[p] + base + e) = out;
    }
  }
  // The last CTA to finish publishes "written" and waits for every peer.
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(a.done_ctas, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(a.done_ctas, 0u);
      publish(a.flags, kWritten, a.rank, a.n, a.epoch);
      wait_all(a.flags[a.rank], kWritten, a.n, a.epoch, a.status);
    }
  }
}

}  // namespace symm
}  // namespace dst

using namespace dst;

// ---------------------------------------------------------------- runtime
// Allocate `bytes` of device memory (zeroed) and return (tensor, IPC handle).
std::vector<at::Tensor> symm_alloc(int64_t bytes, int64_t device) {
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, bytes));
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto opts = at::TensorOptions().dtype(at::kByte).device(at::kCUDA, device);
  at::Tensor t = at::from_blob(
      p, {bytes}, [](void* q) { cudaFree(q); }, opts);
  at::Tensor handle = at::empty({static_cast<int64_t>(sizeof(h))}, at::TensorOptions().dtype(at::kByte));
  std::memcpy(handle.data_ptr(), &h, sizeof(h));
  return {t, handle};
}

int64_t symm_open(const at::Tensor& handle, int64_t device) {
  TORCH_CHECK(handle.numel() == sizeof(cudaIpcMemHandle_t), "symm_open: bad handle");
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void symm_close(int64_t ptr, int64_t device) {
  c10::cuda::CUDAGuard g(static_cast<c10::DeviceIndex>(device));
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

void fused_dp_adam(const std::vector<int64_t>& grad_ptrs, const std::vector<int64_t>& param_ptrs,
                   const std::vector<int64_t>& flag_ptrs, at::Tensor& master, at::Tensor& m, at::Tensor& v,
                   at::Tensor& done_ctas, int64_t slice, int64_t valid, int64_t rank, int64_t epoch, double lr,
                   double beta1, double beta2, double eps, double step, double weight_decay) {
  const int n = static_cast<int>(grad_ptrs.size());
  TORCH_CHECK(n >= 1 && n <= symm::kMaxRanks && param_ptrs.size() == static_cast<size_t>(n) &&
                  flag_ptrs.size() == static_cast<size_t>(n),
              "fused_dp_adam: 1..8 ranks");
  TORCH_CHECK(slice % 8 == 0 && master.numel() == slice && m.numel() == slice && v.numel() == slice,
              "fused_dp_adam: slice");
  symm::DpArgs a{};
  for (int p = 0; p < n; ++p) {
    a.grad[p] = reinterpret_cast<__nv_bfloat16*>(grad_ptrs[p]);
    a.param[p] = reinterpret_cast<__nv_bfloat16*>(param_ptrs[p]);
    a.flags[p] = reinterpret_cast<uint32_t*>(flag_ptrs[p]);
  }
  a.master = master.data_ptr<float>();
  a.m = m.data_ptr<float>();
  a.v = v.data_ptr<float>();
  a.done_ctas = reinterpret_cast<unsigned int*>(done_ctas.data_ptr<int32_t>());
  a.slice = slice;
  a.valid = valid;
  a.rank = static_cast<int>(rank);
  a.n = n;
  a.epoch = static_cast<uint32_t>(epoch);
  const double bc1 = 1.0 - std::pow(beta1, step), bc2 = 1.0 - std::pow(beta2, step);
  a.beta1 = static_cast<float>(beta1);
  a.beta2 = static_cast<float>(beta2);
  a.eps = static_cast<float>(eps);
  a.step_size = static_cast<float>(lr / bc1);
  a.inv_sqrt_bc2 = static_cast<float>(1.0 / std::sqrt(bc2));
  a.inv_n = 1.f / n;
  a.decay = static_cast<float>(1.0 - lr * weight_decay);
  a.status = status_ptr();
  c10::cuda::CUDAGuard g(master.device());
  const int64_t nvec = slice / 8;
  const int blocks = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((nvec + 255) / 256, 4 * num_sms())));
  symm::fused_dp_adam_kernel<<<blocks, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_symm(pybind11::module& m) {
  m.def("symm_alloc", &symm_alloc, "allocate an IPC-exportable zeroed device buffer: (tensor, handle)");
  m.def("symm_open", &symm_open, "map a peer's buffer from its IPC handle; returns the device pointer");
  m.def("symm_close", &symm_close, "unmap a peer buffer");
  namespace py = pybind11;
  m.def("fused_dp_adam", &fused_dp_adam,
        "fused DP bucket reduce + sharded Adam (decoupled weight decay optional) + parameter all-gather over NVLink",
        py::arg("grad_ptrs"), py::arg("param_ptrs"), py::arg("flag_ptrs"), py::arg("master"), py::arg("exp_avg"),
        py::arg("exp_avg_sq"), py::arg("done_ctas"), py::arg("slice"), py::arg("valid"), py::arg("rank"),
        py::arg("epoch"), py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("step"),
        py::arg("weight_decay") = 0.0);
}
