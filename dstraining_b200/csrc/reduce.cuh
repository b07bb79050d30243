// Deterministic column reductions of row-major matrices.
//
// Pass 1 (colred_stage1): CTA (x, y) owns 256 columns and a block of 64
// rows; each of its 8 warps walks every 8th row of the block with one
// 16-byte load (8 columns) per lane, four rows' loads issued before any is
// used (enough bytes in flight to keep HBM busy), accumulating in fp32
// registers in row order; the warps are then combined through shared memory
// in warp order and the CTA writes one fp32 partial row. Optional per-row
// transform for LayerNorm's dγ: the value summed is dy * (x - mean) * rstd,
// and a second output receives Σ dy.
//
// Pass 2 (colred_stage2): each CTA owns 32 columns of the [R, C] partials;
// warp w sums rows w, w+8, ... in order, then warp 0 adds the 8 warp sums in
// order. No atomics anywhere, so results are bitwise reproducible.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace dst {

constexpr int kColredRows = 64;  // rows per pass-1 CTA

__device__ __forceinline__ void colred_unpack(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

// LN = false: part0[y][c] = Σ_rows a[r][c]
// LN = true : part0[y][c] = Σ_rows a[r][c] * (x[r][c] - mean[r]) * rstd[r],
//             part1[y][c] = Σ_rows a[r][c]            (a = dy)
template <bool LN>
static __global__ void __launch_bounds__(256) colred_stage1(const __nv_bfloat16* __restrict__ a, const __nv_bfloat16* __restrict__ x,
                                                     const float* __restrict__ mean, const float* __restrict__ rstd,
                                                     int rows, int C, float* __restrict__ part0,
                                                     float* __restrict__ part1) {
  __shared__ float red[2][8][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = blockIdx.x * 256 + lane * 8;
  const int r0 = blockIdx.y * kColredRows;
  const int r1 = min(rows, r0 + kColredRows);
  float s0[8] = {0, 0, 0, 0, 0, 0, 0, 0}, s1[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (col < C) {
    constexpr int U = 4;  // rows in flight per warp
    for (int rb = r0 + warp; rb < r1; rb += 8 * U) {
      uint4 ap[U], xp[U];
      float mu[U], rs[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int r = rb + 8 * u;
        if (r < r1) {
          ap[u] = __ldg(reinterpret_cast<const uint4*>(a + static_cast<size_t>(r) * C + col));
          if (LN) {
            xp[u] = __ldg(reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * C + col));
            mu[u] = mean[r];
            rs[u] = rstd[r];
          }
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (rb + 8 * u < r1) {
          float av[8];
          colred_unpack(ap[u], av);
          if (LN) {
            float xv[8];
            colred_unpack(xp[u], xv);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              s0[j] += av[j] * (xv[j] - mu[u]) * rs[u];
              s1[j] += av[j];
            }
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) s0[j] += av[j];
          }
        }
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    red[0][warp][lane * 8 + j] = s0[j];
    red[1][warp][lane * 8 + j] = s1[j];
  }
  __syncthreads();
  const int c = blockIdx.x * 256 + threadIdx.x;
  if (c < C) {
    float t0 = 0.f, t1 = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      t0 += red[0][w][threadIdx.x];
      t1 += red[1][w][threadIdx.x];
    }
    part0[static_cast<size_t>(blockIdx.y) * C + c] = t0;
    if (LN) part1[static_cast<size_t>(blockIdx.y) * C + c] = t1;
  }
}

// out[m][c] = bf16(Σ_r part[m][r][c]), m = blockIdx.y (matrices back to back).
static __global__ void __launch_bounds__(256) colred_stage2(const float* __restrict__ part, int R, int C,
                                                     __nv_bfloat16* __restrict__ out) {
  __shared__ float red[8][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = blockIdx.x * 32 + lane;
  const float* p = part + static_cast<size_t>(blockIdx.y) * R * C;
  float s = 0.f;
  if (c < C)
    for (int r = warp; r < R; r += 8) s += p[static_cast<size_t>(r) * C + c];
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < C) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += red[w][lane];
    out[static_cast<size_t>(blockIdx.y) * C + c] = __float2bfloat16_rn(t);
  }
}

}  // namespace dst
