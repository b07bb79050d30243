// Memory-bound kernels: token+position embedding (forward / deterministic
// backward), the fp32-master multi-tensor Adam step, and the softmax
// statistics merge / in-place gradient of the fused LM-head cross-entropy.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <cmath>

#include "common.h"
#include "ptx.cuh"

namespace dst {

__device__ __forceinline__ void unpack8f(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8f(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  return u;
}

// ---------------------------------------------------------------- embedding
// out[b, t, :] = wte[idx[b, t0 + t]] + wpe[t0 + t] for t in [0, tl)
__global__ void embed_fwd_kernel(const int64_t* __restrict__ idx, const __nv_bfloat16* __restrict__ wte,
                                 const __nv_bfloat16* __restrict__ wpe, __nv_bfloat16* __restrict__ out, int B, int T,
                                 int t0, int tl, int C, int V, int* status) {
  const int warps = blockDim.x >> 5;
  const int r = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= B * tl) return;
  const int b = r / tl, t = t0 + r % tl;
  int64_t tok = idx[static_cast<size_t>(b) * T + t];
  if (tok < 0 || tok >= V) {
    if (lane == 0) record_status(status, kIndexOutOfRange);
    tok = 0;
  }
  const uint4* e = reinterpret_cast<const uint4*>(wte + static_cast<size_t>(tok) * C);
  const uint4* p = reinterpret_cast<const uint4*>(wpe + static_cast<size_t>(t) * C);
  uint4* o = reinterpret_cast<uint4*>(out + static_cast<size_t>(r) * C);
  for (int v = lane; v < C / 8; v += 32) {
    float a[8], c[8];
    unpack8f(e[v], a);
    unpack8f(p[v], c);
#pragma unroll
    for (int j = 0; j < 8; ++j) a[j] += c[j];
    o[v] = pack8f(a);
  }
}

// dwpe[t] = sum_b dy[b, t] (b in order)
__global__ void embed_bwd_pos_kernel(const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dwpe, int B,
                                     int T, int C) {
  const int t = blockIdx.x;
  for (int v = threadIdx.x; v < C / 8; v += blockDim.x) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int b = 0; b < B; ++b) {
      float f[8];
      unpack8f(reinterpret_cast<const uint4*>(dy + (static_cast<size_t>(b) * T + t) * C)[v], f);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += f[j];
    }
    reinterpret_cast<uint4*>(dwpe + static_cast<size_t>(t) * C)[v] = pack8f(acc);
  }
}

// One warp per run of equal ids in the stably sorted token list: sums those
// gradient rows in token order into wte's row. An id outside [0, V) is
// recorded in the status word and its rows are dropped (never written).
__global__ void embed_bwd_tok_kernel(const int64_t* __restrict__ sorted, const int64_t* __restrict__ perm,
                                     const __nv_bfloat16* __restrict__ dy, __nv_bfloat16* __restrict__ dwte, int N,
                                     int C, int64_t V, int* status) {
  const int warps = blockDim.x >> 5;
  const int i = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (i >= N) return;
  const int64_t tok = sorted[i];
  if (i > 0 && sorted[i - 1] == tok) return;  // not the start of a run
  if (tok < 0 || tok >= V) {
    if (lane == 0) record_status(status, kIndexOutOfRange);
    return;
  }
  int end = i + 1;
  while (end < N && sorted[end] == tok) ++end;
  for (int v = lane; v < C / 8; v += 32) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = i; j < end; ++j) {
      float f[8];
      unpack8f(reinterpret_cast<const uint4*>(dy + static_cast<size_t>(perm[j]) * C)[v], f);
#pragma unroll
      for (int q = 0; q < 8; ++q) acc[q] += f[q];
    }
    reinterpret_cast<uint4*>(dwte + static_cast<size_t>(tok) * C)[v] = pack8f(acc);
  }
}

// ---------------------------------------------------------------- Adam
constexpr int kAdamMaxTensors = 96;

struct AdamTable {
  __nv_bfloat16* param[kAdamMaxTensors];
  const __nv_bfloat16* grad[kAdamMaxTensors];
  float* master[kAdamMaxTensors];
  float* m[kAdamMaxTensors];
  float* v[kAdamMaxTensors];
  int64_t n[kAdamMaxTensors];
  int64_t chunk_start[kAdamMaxTensors + 1];  // prefix sum of chunk counts
  int count;
};

constexpr int kAdamChunk = 4096;

// Adam (Kingma & Ba) on fp32 masters with bf16 params/grads, with decoupled
// weight decay (Loshchilov & Hutter, AdamW) as the factor `decay` = 1 - lr*wd:
//   m = b1 m + (1-b1) g;  v = b2 v + (1-b2) g^2
//   master = master * decay - (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps);  param = bf16(master)
// decay == 1 is plain Adam.
__global__ void adam_kernel(const __grid_constant__ AdamTable tab, float lr, float beta1, float beta2, float eps,
                            float step_size, float inv_sqrt_bc2, float decay) {
  const int64_t chunk = blockIdx.x;
  int lo = 0, hi = tab.count - 1;
  while (lo < hi) {  // last tensor whose chunk_start <= chunk
    int mid = (lo + hi + 1) >> 1;
    if (tab.chunk_start[mid] <= chunk)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int t = lo;
  const int64_t base = (chunk - tab.chunk_start[t]) * kAdamChunk;
  const int64_t n = tab.n[t];
  const int64_t end = min(n, base + kAdamChunk);
  __nv_bfloat16* P = tab.param[t];
  const __nv_bfloat16* G = tab.grad[t];
  float* W = tab.master[t];
  float* M = tab.m[t];
  float* Vv = tab.v[t];
  for (int64_t i = base + threadIdx.x; i < end; i += blockDim.x) {
    const float g = __bfloat162float(G[i]);
    float m = M[i], v = Vv[i];
    m = m + (g - m) * (1.f - beta1);
    v = v * beta2 + (1.f - beta2) * g * g;
    const float denom = sqrtf(v) * inv_sqrt_bc2 + eps;
    const float w = W[i] * decay - step_size * (m / denom);
    M[i] = m;
    Vv[i] = v;
    W[i] = w;
    P[i] = __float2bfloat16_rn(w);
  }
}

// ---------------------------------------------------------------- fused CE
// Merge per-(row, tile) softmax statistics in tile order -> per-row (max,
// sum exp relative to max). A target id outside [0, vocab) (which no tile
// can match) is recorded in the status word.
__global__ void ce_merge_tiles_kernel(const float* __restrict__ tmax, const float* __restrict__ tsum, int M, int tiles,
                                      float* __restrict__ row_max, float* __restrict__ row_sum,
                                      const int64_t* __restrict__ targets, int64_t vocab, int* status) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M) return;
  const int64_t tgt = targets[r];
  if (tgt < 0 || tgt >= vocab) record_status(status, kIndexOutOfRange);
  float m = -INFINITY, s = 0.f;
  for (int t = 0; t < tiles; ++t) {
    const float tm = tmax[static_cast<size_t>(r) * tiles + t];
    const float ts = tsum[static_cast<size_t>(r) * tiles + t];
    if (tm == -INFINITY) continue;
    const float nm = fmaxf(m, tm);
    s = s * __expf(m - nm) + ts * __expf(tm - nm);
    m = nm;
  }
  row_max[r] = m;
  row_sum[r] = s;
}

// In place: logits -> (softmax - onehot) * scale on the real columns, 0 on
// padded ones.
__global__ void ce_grad_inplace_kernel(__nv_bfloat16* __restrict__ logits, const float* __restrict__ lse,
                                       const int64_t* __restrict__ targets, int M, int N, int col0, int valid_cols,
                                       const float* __restrict__ grad, float inv_n) {
  const int r = blockIdx.y;
  const int v8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= M || v8 * 8 >= N) return;
  const float scale = grad[0] * inv_n;
  const float l = lse[r];
  const int64_t tgt = targets[r] - col0;
  uint4* row = reinterpret_cast<uint4*>(logits + static_cast<size_t>(r) * N);
  float f[8];
  unpack8f(row[v8], f);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int c = v8 * 8 + j;
    float g = 0.f;
    if (c < valid_cols) g = (__expf(f[j] - l) - (c == tgt ? 1.f : 0.f)) * scale;
    f[j] = g;
  }
  row[v8] = pack8f(f);
}

}  // namespace dst

using namespace dst;

at::Tensor embedding_fwd(const at::Tensor& idx, const at::Tensor& wte, const at::Tensor& wpe, int64_t t0, int64_t tl) {
  TORCH_CHECK(idx.is_cuda() && idx.scalar_type() == at::kLong && idx.dim() == 2 && idx.is_contiguous(), "embedding: idx");
  TORCH_CHECK(wte.scalar_type() == at::kBFloat16 && wpe.scalar_type() == at::kBFloat16 && wte.is_contiguous() &&
                  wpe.is_contiguous(),
              "embedding: bf16 tables");
  c10::cuda::CUDAGuard g(idx.device());
  const int B = idx.size(0), T = idx.size(1), C = wte.size(1);
  TORCH_CHECK(C % 8 == 0 && wpe.size(1) == C && t0 + tl <= T && T <= wpe.size(0), "embedding: shapes");
  at::Tensor out = at::empty({B, tl, C}, wte.options());
  const int rows = B * tl, threads = 256, per = threads / 32;
  embed_fwd_kernel<<<(rows + per - 1) / per, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      idx.data_ptr<int64_t>(), reinterpret_cast<const __nv_bfloat16*>(wte.data_ptr()),
      reinterpret_cast<const __nv_bfloat16*>(wpe.data_ptr()), reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), B, T,
      static_cast<int>(t0), static_cast<int>(tl), C, wte.size(0), status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> embedding_bwd(const at::Tensor& dy, const at::Tensor& idx, int64_t vocab, int64_t block) {
  TORCH_CHECK(dy.is_contiguous() && dy.dim() == 3 && dy.scalar_type() == at::kBFloat16, "embedding_bwd: dy");
  c10::cuda::CUDAGuard g(dy.device());
  const int B = dy.size(0), T = dy.size(1), C = dy.size(2);
  TORCH_CHECK(idx.dim() == 2 && idx.size(0) == B && idx.size(1) == T, "embedding_bwd: idx shape");
  TORCH_CHECK(C % 8 == 0 && block >= T && vocab > 0, "embedding_bwd: C % 8 == 0 and block >= T required");
  auto st = at::cuda::getCurrentCUDAStream();
  at::Tensor dwte = at::zeros({vocab, C}, dy.options());
  at::Tensor dwpe = at::zeros({block, C}, dy.options());
  embed_bwd_pos_kernel<<<T, 128, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                                          reinterpret_cast<__nv_bfloat16*>(dwpe.data_ptr()), B, T, C);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  at::Tensor flat = idx.reshape({-1});
  auto sorted = flat.sort(/*stable=*/true, /*dim=*/0, /*descending=*/false);
  at::Tensor keys = std::get<0>(sorted).contiguous();
  at::Tensor perm = std::get<1>(sorted).contiguous();
  const int N = B * T, threads = 256, per = threads / 32;
  embed_bwd_tok_kernel<<<(N + per - 1) / per, threads, 0, st>>>(keys.data_ptr<int64_t>(), perm.data_ptr<int64_t>(),
                                                                reinterpret_cast<const __nv_bfloat16*>(dy.data_ptr()),
                                                                reinterpret_cast<__nv_bfloat16*>(dwte.data_ptr()), N, C,
                                                                vocab, status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dwte, dwpe};
}

void adam_master_step(const std::vector<at::Tensor>& params, const std::vector<at::Tensor>& grads,
                      const std::vector<at::Tensor>& masters, const std::vector<at::Tensor>& m1,
                      const std::vector<at::Tensor>& m2, double lr, double beta1, double beta2, double eps,
                      double step, double weight_decay) {
  const size_t n = params.size();
  const float decay = static_cast<float>(1.0 - lr * weight_decay);
  TORCH_CHECK(grads.size() == n && masters.size() == n && m1.size() == n && m2.size() == n, "adam: list sizes");
  if (n == 0) return;
  c10::cuda::CUDAGuard g(params[0].device());
  const double bc1 = 1.0 - std::pow(beta1, step);
  const double bc2 = 1.0 - std::pow(beta2, step);
  const float step_size = static_cast<float>(lr / bc1);
  const float inv_sqrt_bc2 = static_cast<float>(1.0 / std::sqrt(bc2));
  auto st = at::cuda::getCurrentCUDAStream();
  for (size_t off = 0; off < n; off += kAdamMaxTensors) {
    AdamTable tab{};
    const int cnt = static_cast<int>(std::min<size_t>(kAdamMaxTensors, n - off));
    int64_t chunks = 0;
    for (int i = 0; i < cnt; ++i) {
      const auto& p = params[off + i];
      const auto& gr = grads[off + i];
      TORCH_CHECK(p.scalar_type() == at::kBFloat16 && gr.scalar_type() == at::kBFloat16 && p.is_contiguous() &&
                      gr.is_contiguous() && gr.numel() == p.numel(),
                  "adam: bf16 contiguous params/grads");
      TORCH_CHECK(masters[off + i].scalar_type() == at::kFloat && masters[off + i].is_contiguous() &&
                      m1[off + i].is_contiguous() && m2[off + i].is_contiguous(),
                  "adam: fp32 contiguous state");
      tab.param[i] = reinterpret_cast<__nv_bfloat16*>(p.data_ptr());
      tab.grad[i] = reinterpret_cast<const __nv_bfloat16*>(gr.data_ptr());
      tab.master[i] = masters[off + i].data_ptr<float>();
      tab.m[i] = m1[off + i].data_ptr<float>();
      tab.v[i] = m2[off + i].data_ptr<float>();
      tab.n[i] = p.numel();
      tab.chunk_start[i] = chunks;
      chunks += (p.numel() + kAdamChunk - 1) / kAdamChunk;
    }
    tab.chunk_start[cnt] = chunks;
    tab.count = cnt;
    if (chunks == 0) continue;
    adam_kernel<<<static_cast<unsigned>(chunks), 256, 0, st>>>(tab, static_cast<float>(lr), static_cast<float>(beta1),
                                                               static_cast<float>(beta2), static_cast<float>(eps),
                                                               step_size, inv_sqrt_bc2, decay);
    C10_CUDA_KERNEL_LAUNCH_CHECK();
  }
}

// targets: the [rows] int64 target ids (checked against the real vocabulary
// size, not used otherwise).
std::vector<at::Tensor> ce_merge_tiles(const at::Tensor& tmax, const at::Tensor& tsum, const at::Tensor& targets,
                                       int64_t vocab) {
  TORCH_CHECK(tmax.scalar_type() == at::kFloat && tmax.is_contiguous() && tsum.sizes() == tmax.sizes(), "ce_merge");
  TORCH_CHECK(tmax.is_cuda() && tmax.dim() == 2 && tsum.is_contiguous(), "ce_merge: [rows, tiles] fp32 statistics");
  const int M = tmax.size(0), tiles = tmax.size(1);
  TORCH_CHECK(targets.is_cuda() && targets.scalar_type() == at::kLong && targets.is_contiguous() &&
                  targets.numel() == M && vocab > 0,
              "ce_merge: one contiguous int64 target per row and vocab > 0");
  c10::cuda::CUDAGuard g(tmax.device());
  at::Tensor m = at::empty({M}, tmax.options());
  at::Tensor s = at::empty({M}, tmax.options());
  ce_merge_tiles_kernel<<<(M + 255) / 256, 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      tmax.data_ptr<float>(), tsum.data_ptr<float>(), M, tiles, m.data_ptr<float>(), s.data_ptr<float>(),
      targets.data_ptr<int64_t>(), vocab, status_ptr());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {m, s};
}

// grad: fp32 scalar on the device (the loss gradient); each element is
// scaled by grad * inv_n without a host synchronisation.
void ce_grad_inplace(at::Tensor& logits, const at::Tensor& lse, const at::Tensor& targets, int64_t col0,
                     int64_t valid_cols, const at::Tensor& grad, double inv_n) {
  TORCH_CHECK(logits.is_contiguous() && logits.scalar_type() == at::kBFloat16 && logits.dim() == 2, "ce_grad: logits");
  TORCH_CHECK(grad.is_cuda() && grad.scalar_type() == at::kFloat && grad.numel() == 1, "ce_grad: fp32 scalar grad");
  c10::cuda::CUDAGuard g(logits.device());
  const int M = logits.size(0), N = logits.size(1);
  TORCH_CHECK(N % 8 == 0, "ce_grad: N must be a multiple of 8");
  TORCH_CHECK(lse.is_contiguous() && lse.numel() == M && targets.is_contiguous() && targets.numel() == M,
              "ce_grad: lse and targets must hold one contiguous value per logits row");
  dim3 grid((N / 8 + 127) / 128, M);
  ce_grad_inplace_kernel<<<grid, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      reinterpret_cast<__nv_bfloat16*>(logits.data_ptr()), lse.data_ptr<float>(), targets.data_ptr<int64_t>(), M, N,
      static_cast<int>(col0), static_cast<int>(valid_cols), grad.data_ptr<float>(), static_cast<float>(inv_n));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

void register_embed(pybind11::module& m) {
  m.def("embedding_fwd", &embedding_fwd, "token + position embedding (local sequence slice)");
  m.def("embedding_bwd", &embedding_bwd, "deterministic embedding backward");
}

void register_adam(pybind11::module& m) {
  namespace py = pybind11;
  m.def("adam_master_step", &adam_master_step,
        "multi-tensor Adam (decoupled weight decay optional) on fp32 masters with bf16 write-back",
        py::arg("params"), py::arg("grads"), py::arg("masters"), py::arg("exp_avg"), py::arg("exp_avg_sq"),
        py::arg("lr"), py::arg("beta1"), py::arg("beta2"), py::arg("eps"), py::arg("step"),
        py::arg("weight_decay") = 0.0);
}

void register_ce(pybind11::module& m) {
  m.def("ce_merge_tiles", &ce_merge_tiles, "merge per-tile softmax statistics");
  m.def("ce_grad_inplace", &ce_grad_inplace, "logits -> dlogits in place");
}
