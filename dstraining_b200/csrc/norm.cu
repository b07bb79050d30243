// LayerNorm forward/backward over the last dimension, bf16 in/out, fp32 math.
//
// Forward: one warp per row; the row is held in registers as 16-byte bf16
// vectors, mean and variance are two-pass (sum, then sum of squared
// deviations) and the fp32 mean / rstd are saved for backward.
//
// Backward: one warp per row computes
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = w * dy
// and accumulates dγ = Σ dy·xhat, dβ = Σ dy for its columns in registers
// across the rows its CTA owns; the CTA's warps are combined in shared memory
// in warp order and written as one fp32 partial row per CTA, which a second
// kernel sums in CTA order. Deterministic: no atomics anywhere.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.h"
#include "ptx.cuh"

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

template <int MAXV>
__global__ void ln_bwd_kernel(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                              const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean,
                              const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx,
                              float* __restrict__ part_dw, float* __restrict__ part_db, int rows, int C,
                              int rows_per_block) {
  extern __shared__ float red[];  // [2][C]
  const int warps = blockDim.x >> 5;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nvec = C >> 3;
  float adw[MAXV][8], adb[MAXV][8];
  float wf[MAXV][8];
  const uint4* wv = reinterpret_cast<const uint4*>(w);
#pragma unroll
  for (int i = 0; i < MAXV; ++i) {
#pragma unroll
    for (int j = 0; j < 8; ++j) adw[i][j] = adb[i][j] = 0.f;
    if (lane + 32 * i < nvec) unpack8(wv[lane + 32 * i], wf[i]);
  }
  const int r0 = blockIdx.x * rows_per_block;
  const int r1 = min(rows, r0 + rows_per_block);
  for (int row = r0 + warp; row < r1; row += warps) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * C);
    const uint4* gr = reinterpret_cast<const uint4*>(dy + static_cast<size_t>(row) * C);
    const float mu = mean[row], rs = rstd[row];
    float xh[MAXV][8], g[MAXV][8];
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
      const int vi = lane + 32 * i;
      if (vi < nvec) {
        float xf[8], df[8];
        unpack8(xr[vi], xf);
        unpack8(gr[vi], df);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] = (xf[j] - mu) * rs;
          g[i][j] = df[j] * wf[i][j];
          s1 += g[i][j];
          s2 += g[i][j] * xh[i][j];
          adw[i][j] += df[j] * xh[i][j];
          adb[i][j] += df[j];
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
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = rs * (g[i][j] - s1 - xh[i][j] * s2);
        dxr[vi] = pack8(o);
      }
    }
  }
  // Combine the warps of this CTA in warp order (sequential adds into one
  // shared row pair keep the order fixed without per-warp copies).
  float* acc_w = red;
  float* acc_b = red + C;
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) red[c] = 0.f;
  __syncthreads();
  for (int k = 0; k < warps; ++k) {
    if (warp == k) {
#pragma unroll
      for (int i = 0; i < MAXV; ++i) {
        const int vi = lane + 32 * i;
        if (vi < nvec) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc_w[vi * 8 + j] += adw[i][j];
            acc_b[vi * 8 + j] += adb[i][j];
          }
        }
      }
    }
    __syncthreads();
  }
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    part_dw[static_cast<size_t>(blockIdx.x) * C + c] = acc_w[c];
    part_db[static_cast<size_t>(blockIdx.x) * C + c] = acc_b[c];
  }
}

__global__ void sum_partials_kernel(const float* __restrict__ pw, const float* __restrict__ pb, int R, int C,
                                    __nv_bfloat16* __restrict__ dw, __nv_bfloat16* __restrict__ db) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float a = 0.f, b = 0.f;
  for (int r = 0; r < R; ++r) {
    a += pw[static_cast<size_t>(r) * C + c];
    b += pb[static_cast<size_t>(r) * C + c];
  }
  dw[c] = __float2bfloat16_rn(a);
  db[c] = __float2bfloat16_rn(b);
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
  c10::cuda::CUDAGuard g(x.device());
  const int rows = x.size(0), C = x.size(1);
  at::Tensor dx = at::empty_like(x);
  const int threads = 256, warps = threads / 32;
  const int sms = num_sms();
  // Enough CTAs to fill the GPU a few times over, each owning a row range.
  int rows_per_block = std::max(warps, (rows + 4 * sms - 1) / (4 * sms));
  const int R = (rows + rows_per_block - 1) / rows_per_block;
  at::Tensor pw = at::empty({R, C}, x.options().dtype(at::kFloat));
  at::Tensor pb = at::empty({R, C}, x.options().dtype(at::kFloat));
  at::Tensor dw = at::empty({C}, x.options());
  at::Tensor db = at::empty({C}, x.options());
  const size_t smem = 2 * static_cast<size_t>(C) * sizeof(float);
  TORCH_CHECK(smem <= 48 * 1024, "layernorm_bwd: hidden size too large");
  auto st = at::cuda::getCurrentCUDAStream();
  LN_DISPATCH(C, ln_bwd_kernel, <<<R, threads, smem, st>>>(cbf(dy), cbf(x), cbf(w), mean.data_ptr<float>(),
                                                           rstd.data_ptr<float>(), bf(dx), pw.data_ptr<float>(),
                                                           pb.data_ptr<float>(), rows, C, rows_per_block));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  sum_partials_kernel<<<(C + 255) / 256, 256, 0, st>>>(pw.data_ptr<float>(), pb.data_ptr<float>(), R, C, bf(dw), bf(db));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {dx, dw, db};
}

void register_norm(pybind11::module& m) {
  m.def("layernorm_fwd", &layernorm_fwd, "LayerNorm forward (bf16)");
  m.def("layernorm_bwd", &layernorm_bwd, "LayerNorm backward (bf16), deterministic dγ/dβ");
}
