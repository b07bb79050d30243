// Tensor-parallel companions of the peer GEMM modes (gemm.cuh):
//
// tp_reduce: after every rank's scatter-mode GEMM has stored its partial
//   output rows for this rank's sequence shard into this rank's receive
//   slots [tp][rows_local][N], sum the slots in rank order (fp32), add the
//   bias and the residual, and write the bf16 result. Waits (bounded) for
//   every peer's "written" flag first and, once all CTAs are done reading,
//   tells every peer the slots are drained. Completes a GEMM + reduce-scatter.
//
// tp_allgather: each rank holds its sequence shard [rows_local, N] in a peer
//   buffer; copy all shards into a full [B*T, N] tensor with 16-byte peer
//   loads. Used to finish an all-reduce (reduce-scatter + all-gather) when the
//   layer's output is replicated rather than sequence-sharded.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.h"
#include "gemm.cuh"

namespace dst {
namespace tp {

struct ReduceArgs {
  const __nv_bfloat16* recv;  // [tp][rows][N]
  __nv_bfloat16* out;         // [rows][N]
  const __nv_bfloat16* bias;  // [N] or null
  const __nv_bfloat16* resid; // [rows][N] or null
  uint32_t* flags[kMaxPeers];
  unsigned int* done_ctas;
  int tp, rank, rows, N;
  uint32_t epoch;
  int* status;
};

__global__ void __launch_bounds__(256) reduce_kernel(const __grid_constant__ ReduceArgs a) {
  __shared__ bool go;
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int p = 0; p < a.tp && ok; ++p)
      ok = flag_wait_geq(a.flags[a.rank] + kSWritten * kMaxPeers + p, a.epoch, a.status, kTimeoutPeer);
    go = ok;
  }
  __syncthreads();
  if (go) {
    const int vpr = a.N / 8;
    const int64_t total = static_cast<int64_t>(a.rows) * vpr;
    const size_t slot = static_cast<size_t>(a.rows) * a.N;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    // two 8-element vectors per thread and iteration, every slot's loads of
    // both issued before any is summed
    for (int64_t i0 = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i0 < total; i0 += 2 * stride) {
      constexpr int V = 2;
      int64_t iv[V];
      bool in[V];
      uint4 u[V][kMaxPeers];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        iv[v] = i0 + v * stride;
        in[v] = iv[v] < total;
        const int row = static_cast<int>(iv[v] / vpr), c8 = static_cast<int>(iv[v] % vpr) * 8;
        const size_t off = static_cast<size_t>(row) * a.N + c8;
#pragma unroll
        for (int s = 0; s < kMaxPeers; ++s)
          if (in[v] && s < a.tp) u[v][s] = *reinterpret_cast<const uint4*>(a.recv + s * slot + off);
      }
#pragma unroll
      for (int v = 0; v < V; ++v) {
        if (!in[v]) continue;
        const int row = static_cast<int>(iv[v] / vpr), c8 = static_cast<int>(iv[v] % vpr) * 8;
        const size_t off = static_cast<size_t>(row) * a.N + c8;
        float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int s = 0; s < kMaxPeers; ++s) {  // summed in fixed rank order
          if (s < a.tp) {
            const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u[v][s]);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float2 f = __bfloat1622float2(h[j]);
              acc[2 * j] += f.x;
              acc[2 * j + 1] += f.y;
            }
          }
        }
        if (a.bias) {
          const uint4 bu = *reinterpret_cast<const uint4*>(a.bias + c8);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&bu);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            acc[2 * j] += f.x;
            acc[2 * j + 1] += f.y;
          }
        }
        if (a.resid) {
          const uint4 ru = *reinterpret_cast<const uint4*>(a.resid + off);
          const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&ru);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float2 f = __bfloat1622float2(h[j]);
            acc[2 * j] += f.x;
            acc[2 * j + 1] += f.y;
          }
        }
        uint4 o;
        __nv_bfloat162* oh = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) oh[j] = __floats2bfloat162_rn(acc[2 * j], acc[2 * j + 1]);
        *reinterpret_cast<uint4*>(a.out + off) = o;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned int prev = atomicAdd(a.done_ctas, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(a.done_ctas, 0u);
      __threadfence_system();
      for (int p = 0; p < a.tp; ++p) flag_store_release(a.flags[p] + kSConsumed * kMaxPeers + a.rank, a.epoch);
    }
  }
}

struct GatherArgs {
  const __nv_bfloat16* shard[kMaxPeers];  // each rank's [rows_local][N]
  __nv_bfloat16* out;                     // [B*T][N]
  uint32_t* flags[kMaxPeers];
  unsigned int* done_ctas;
  int tp, rank, seq, seq_local, tokens, N;
  uint32_t epoch;
  int* status;
};

__global__ void __launch_bounds__(256) allgather_kernel(const __grid_constant__ GatherArgs a) {
  __shared__ bool go;
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) {
      __threadfence_system();
      for (int p = 0; p < a.tp; ++p) flag_store_release(a.flags[p] + kGReady * kMaxPeers + a.rank, a.epoch);
    }
    bool ok = true;
    for (int p = 0; p < a.tp && ok; ++p)
      ok = flag_wait_geq(a.flags[a.rank] + kGReady * kMaxPeers + p, a.epoch, a.status, kTimeoutPeer);
    go = ok;
  }
  __syncthreads();
  if (go) {
    const int vpr = a.N / 8;
    const int64_t total = static_cast<int64_t>(a.tokens) * vpr;
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
      const int tok = static_cast<int>(i / vpr), c8 = static_cast<int>(i % vpr) * 8;
      const int b = tok / a.seq, t = tok - b * a.seq;
      const int src = t / a.seq_local;
      const int local = b * a.seq_local + (t - src * a.seq_local);
      *reinterpret_cast<uint4*>(a.out + static_cast<size_t>(tok) * a.N + c8) =
          *reinterpret_cast<const uint4*>(a.shard[src] + static_cast<size_t>(local) * a.N + c8);
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    const unsigned int prev = atomicAdd(a.done_ctas, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(a.done_ctas, 0u);
      for (int p = 0; p < a.tp; ++p) flag_store_release(a.flags[p] + kGConsumed * kMaxPeers + a.rank, a.epoch);
      for (int p = 0; p < a.tp; ++p)
        flag_wait_geq(a.flags[a.rank] + kGConsumed * kMaxPeers + p, a.epoch, a.status, kTimeoutPeer);
    }
  }
}

}  // namespace tp
}  // namespace dst

using namespace dst;

static int grid_for(int64_t vectors) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((vectors + 255) / 256, 4 * num_sms())));
}

at::Tensor tp_reduce(const at::Tensor& recv, int64_t tp_size, const c10::optional<at::Tensor>& bias,
                     const c10::optional<at::Tensor>& resid, const std::vector<int64_t>& flags, const at::Tensor& done,
                     int64_t rank, int64_t epoch) {
  TORCH_CHECK(recv.is_cuda() && recv.scalar_type() == at::kBFloat16 && recv.dim() == 3 && recv.is_contiguous() &&
                  recv.size(0) == tp_size,
              "tp_reduce: recv must be a contiguous bf16 [tp, rows, N] tensor");
  c10::cuda::CUDAGuard g(recv.device());
  const int rows = recv.size(1), N = recv.size(2);
  TORCH_CHECK(N % 8 == 0, "tp_reduce: N must be a multiple of 8");
  at::Tensor out = at::empty({rows, N}, recv.options());
  tp::ReduceArgs a{};
  a.recv = reinterpret_cast<const __nv_bfloat16*>(recv.data_ptr());
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (bias.has_value()) a.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  if (resid.has_value()) {
    TORCH_CHECK(resid->is_contiguous() && resid->numel() == static_cast<int64_t>(rows) * N, "tp_reduce: residual");
    a.resid = reinterpret_cast<const __nv_bfloat16*>(resid->data_ptr());
  }
  for (size_t p = 0; p < flags.size(); ++p) a.flags[p] = reinterpret_cast<uint32_t*>(flags[p]);
  a.done_ctas = reinterpret_cast<unsigned int*>(done.data_ptr<int32_t>());
  a.tp = static_cast<int>(tp_size);
  a.rank = static_cast<int>(rank);
  a.rows = rows;
  a.N = N;
  a.epoch = static_cast<uint32_t>(epoch);
  a.status = status_ptr();
  // about two CTAs per SM: enough loads in flight (2 vectors x tp slots per thread) without a long
  // tail of CTAs with almost no work behind the launch-wide completion counter
  const int64_t vecs = static_cast<int64_t>(rows) * N / 8;
  const int grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((vecs + 511) / 512, 2 * num_sms())));
  tp::reduce_kernel<<<grid, 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

at::Tensor tp_allgather(const std::vector<int64_t>& shards, int64_t rows_local, int64_t N, int64_t seq,
                        const std::vector<int64_t>& flags, const at::Tensor& done, int64_t rank, int64_t epoch,
                        const at::Tensor& like) {
  const int tp_size = static_cast<int>(shards.size());
  TORCH_CHECK(tp_size >= 2 && tp_size <= kMaxPeers && N % 8 == 0 && seq % tp_size == 0, "tp_allgather: shapes");
  c10::cuda::CUDAGuard g(like.device());
  const int64_t tokens = rows_local * tp_size;
  at::Tensor out = at::empty({tokens, N}, like.options());
  tp::GatherArgs a{};
  for (int p = 0; p < tp_size; ++p) {
    a.shard[p] = reinterpret_cast<const __nv_bfloat16*>(shards[p]);
    a.flags[p] = reinterpret_cast<uint32_t*>(flags[p]);
  }
  a.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  a.done_ctas = reinterpret_cast<unsigned int*>(done.data_ptr<int32_t>());
  a.tp = tp_size;
  a.rank = static_cast<int>(rank);
  a.seq = static_cast<int>(seq);
  a.seq_local = static_cast<int>(seq / tp_size);
  a.tokens = static_cast<int>(tokens);
  a.N = static_cast<int>(N);
  a.epoch = static_cast<uint32_t>(epoch);
  a.status = status_ptr();
  tp::allgather_kernel<<<grid_for(tokens * N / 8), 256, 0, at::cuda::getCurrentCUDAStream()>>>(a);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

void register_tp(pybind11::module& m) {
  m.def("tp_reduce", &tp_reduce, "sum the receive slots of a scatter-mode GEMM (+bias, +residual)", py::arg("recv"),
        py::arg("tp"), py::arg("bias"), py::arg("resid"), py::arg("flags"), py::arg("done"), py::arg("rank"),
        py::arg("epoch"));
  m.def("tp_allgather", &tp_allgather, "gather sequence shards from peer memory into a full tensor");
}
