// LayerNorm forward/backward over the last dimension, bf16 in/out, fp32 math.
//
// Forward: one warp per row; the row is held in registers as 16-byte bf16
// vectors, mean and variance are two-pass (sum, then sum of squared
// deviations) and the fp32 mean / rstd are saved for backward.
//
// Backward: one warp per row computes
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = w * dy;
// dγ = Σ dy·xhat and dβ = Σ dy are deterministic two-pass column reductions
// (reduce.cuh). No atomics anywhere.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.h"
#include "ptx.cuh"
#include "reduce.cuh"

namespace dst {

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  return u;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

// MAXV: max 8-element vectors per lane (C <= 256 * MAXV).
template <int MAXV>
__global__ void ln_fwd_kernel(const __nv_bfloat16* __restrict__ x, const __nv_bfloat16* __restrict__ w,
                              const __nv_bfloat16* __restrict__ b, __nv_bfloat16* __restrict__ y,
                              float* __restrict__ mean_out, float* __restrict__ rstd_out, int rows, int C, float eps) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = C >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * C);
  float v[MAXV][8];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      unpack8(xr[vi], v[i]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s += v[i][j];
    }
  }
  const float mean = warp_sum(s) / C;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    if (lane + 32 * i < nvec) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = v[i][j] - mean;
        ss += d * d;
      }
    }
  }
  const float rstd = rsqrtf(warp_sum(ss) / C + eps);
  uint4* yr = reinterpret_cast<uint4*>(y + static_cast<size_t>(row) * C);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  const uint4* bv = reinterpret_cast<const uint4*>(b);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      float wf[8], bf[8], o[8];
      unpack8(wv[vi], wf);
      unpack8(bv[vi], bf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = (v[i][j] - mean) * rstd * wf[j] + bf[j];
      yr[vi] = pack8(o);
    }
  }
  if (lane == 0) {
    mean_out[row] = mean;
    rstd_out[row] = rstd;
  }
}

// dx only: one warp per row, x and dy kept packed (bf16) in registers, the
// weight re-read through L1. dγ/dβ come from the column reduction in
// reduce.cuh, which re-reads x and dy; splitting the two keeps this kernel's
// register footprint small enough for full occupancy.
template <int MAXV>
__global__ void __launch_bounds__(256) ln_bwd_dx_kernel(const __nv_bfloat16* __restrict__ dy,
                                                        const __nv_bfloat16* __restrict__ x,
                                                        const __nv_bfloat16* __restrict__ w,
                                                        const float* __restrict__ mean, const float* __restrict__ rstd,
                                                        __nv_bfloat16* __restrict__ dx, int rows, int C) {
  const int warps = blockDim.x >> 5;
  const int row = blockIdx.x * warps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = C >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * C);
  const uint4* gr = reinterpret_cast<const uint4*>(dy + static_cast<size_t>(row) * C);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4 xp[MAXV], gp[MAXV];
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      xp[i] = xr[vi];
      gp[i] = gr[vi];
    }
  }
  const float mu = mean[row], rs = rstd[row];
  float s1 = 0.f, s2 = 0.f;
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      float xf[8], df[8], wf[8];
      unpack8(xp[i], xf);
      unpack8(gp[i], df);
      unpack8(__ldg(wv + vi), wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g = df[j] * wf[j];
        s1 += g;
        s2 += g * (xf[j] - mu) * rs;
      }
    }
  }
  s1 = warp_sum(s1) / C;
  s2 = warp_sum(s2) / C;
  uint4* dxr = reinterpret_cast<uint4*>(dx + static_cast<size_t>(row) * C);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
    const int vi = lane + 32 * i;
    if (vi < nvec) {
      float xf[8], df[8], wf[8], o[8];
      unpack8(xp[i], xf);
      unpack8(gp[i], df);
      unpack8(__ldg(wv + vi), wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j] = rs * (df[j] * wf[j] - s1 - (xf[j] - mu) * rs * s2);
      dxr[vi] = pack8(o);
    }
  }
}

}  // namespace dst

using namespace dst;

#define LN_DISPATCH(C, KERNEL, ...)                                  \
  do {                                                               \
    const int nv = (C) / 8;                                          \
    if (nv <= 32) { KERNEL<1> __VA_ARGS__; }                         \
    else if (nv <= 64) { KERNEL<2> __VA_ARGS__; }                    \
    else if (nv <= 128) { KERNEL<4> __VA_ARGS__; }                   \
    else if (nv <= 256) { KERNEL<8> __VA_ARGS__; }                   \
    else if (nv <= 512) { KERNEL<16> __VA_ARGS__; }                  \
    else { TORCH_CHECK(false, "layernorm: hidden size too large"); } \
  } while (0)

static const __nv_bfloat16* cbf(const at::Tensor& t) { return reinterpret_cast<const __nv_bfloat16*>(t.data_ptr()); }
static __nv_bfloat16* bf(at::Tensor& t) { return reinterpret_cast<__nv_bfloat16*>(t.data_ptr()); }

std::vector<at::Tensor> layernorm_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& b, double eps) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == at::kBFloat16 && x.dim() == 2 && x.is_contiguous(), "layernorm_fwd: x");
  TORCH_CHECK(w.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16 && w.is_contiguous() && b.is_contiguous(),
              "layernorm_fwd: bf16 contiguous weight/bias");
  c10::cuda::CUDAGuard g(x.device());
  const int rows = x.size(0), C = x.size(1);
  TORCH_CHECK(C % 8 == 0 && w.numel() == C && b.numel() == C, "layernorm_fwd: C must be a multiple of 8");
  at::Tensor y = at::empty_like(x);
  at::Tensor mean = at::empty({rows}, x.options().dtype(at::kFloat));
  at::Tensor rstd = at::empty({rows}, x.options().dtype(at::kFloat));
  const int threads = 256, per = threads / 32;
  const int blocks = (rows + per - 1) / per;
  auto st = at::cuda::getCurrentCUDAStream();
  LN_DISPATCH(C, ln_fwd_kernel, <<<blocks, threads, 0, st>>>(cbf(x), cbf(w), cbf(b), bf(y), mean.data_ptr<float>(),
                                                             rstd.data_ptr<float>(), rows, C, static_cast<float>(eps)));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {y, mean, rstd};
}

std::vector<at::Tensor> layernorm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                      const at::Tensor& mean, const at::Tensor& rstd) {
  TORCH_CHECK(dy.is_contiguous() && x.is_contiguous() && dy.sizes() == x.sizes(), "layernorm_bwd: shapes");
  TORCH_CHECK(x.is_cuda() && x.dim() == 2 && x.scalar_type() == at::kBFloat16 && dy.scalar_type() == at::kBFloat16 &&
                  w.scalar_type() == at::kBFloat16 && w.is_contiguous(),
              "layernorm_bwd: bf16 dy / x [rows, C] and weight required");
  TORCH_CHECK(w.numel() == x.size(1) && mean.numel() == x.size(0) && rstd.numel() == x.size(0) &&
                  mean.is_contiguous() && rstd.is_contiguous(),
              "layernorm_bwd: weight [C], mean and rstd [rows] required");
  c10::cuda::CUDAGuard g(x.device());
  const int rows = x.size(0), C = x.size(1);
  at::Tensor dx = at::empty_like(x);
  auto st = at::cuda::getCurrentCUDAStream();
  const int threads = 256, per = threads / 32;
  LN_DISPATCH(C, ln_bwd_dx_kernel, <<<(rows + per - 1) / per, threads, 0, st>>>(
                                       cbf(dy), cbf(x), cbf(w), mean.data_ptr<float>(), rstd.data_ptr<float>(), bf(dx),
                                       rows, C));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const int R = (rows + kColredRows - 1) / kColredRows;
  at::Tensor part = at::empty({2, R, C}, x.options().dtype(at::kFloat));
  at::Tensor dwb = at::empty({2, C}, x.options());
  dim3 g1((C + 255) / 256, R);
  colred_stage1<true><<<g1, 256, 0, st>>>(cbf(dy), cbf(x), mean.data_ptr<float>(), rstd.data_ptr<float>(), rows, C,
                                          part.data_ptr<float>(), part.data_ptr<float>() + static_cast<size_t>(R) * C);
  dim3 g2((C + 31) / 32, 2);
  colred_stage2<<<g2, 256, 0, st>>>(part.data_ptr<float>(), R, C, bf(dwb));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dx, dwb[0], dwb[1]};
}

void register_norm(pybind11::module& m) {
  m.def("layernorm_fwd", &layernorm_fwd, "LayerNorm forward (bf16)");
  m.def("layernorm_bwd", &layernorm_bwd, "LayerNorm backward (bf16), deterministic dγ/dβ");
}
