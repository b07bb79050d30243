// dst_layernorm_bwd_noalloc: LayerNorm backward whose scratch space (the
// per-CTA partial dgamma/dbeta rows) is a fixed array compiled into the
// library instead of memory allocated per call. See dst_noalloc.h for the
// contract. This entry point has no counterpart in the reference.
//
// Same algorithm as the allocating LayerNorm backward in norm.cu: pass one
// (one warp per row) writes dx and one fp32 partial row of dgamma and of
// dbeta per CTA, combining the CTA's warps in warp order; pass two sums the
// partial rows in CTA order. Hidden sizes above 1024 take three kernels
// instead (dx; per-row-block column partials of dgamma and dbeta into the
// same scratch rows; their ordered sum), because the per-lane accumulators of
// pass one would spill out of registers there. No atomics, so results are
// deterministic.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "dst_noalloc.h"

namespace {

constexpr int kMaxHidden = DST_NOALLOC_MAX_HIDDEN;
constexpr int kMaxCtas = DST_NOALLOC_MAX_CTAS;
constexpr int kMaxDevices = 64;

// The scratch array: [2][kMaxCtas][kMaxHidden] fp32 (dgamma rows, then dbeta
// rows). In host code this name is only a stand-in for the symbol, never a
// device address; kernels receive the address from cudaGetSymbolAddress.
static __device__ __align__(256) float g_ln_scratch[2 * kMaxCtas * kMaxHidden];

std::mutex g_setup_mu;
float* g_scratch_addr[kMaxDevices] = {nullptr};

// Once per device, with that device current: resolve the array's address.
cudaError_t scratch_for_current_device(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_setup_mu);
  if (g_scratch_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_ln_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return cudaSuccess;
}

__device__ __forceinline__ void bf8_to_f(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 t = __bfloat1622float2(h[j]);
    f[2 * j] = t.x;
    f[2 * j + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 f_to_bf8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
  return u;
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffff, v, o);
  return v;
}

// Pass one. VPL: 8-element vectors per lane (hidden <= 256 * VPL).
template <int VPL>
__global__ void ln_bwd_rows(const __nv_bfloat16* __restrict__ dy, const __nv_bfloat16* __restrict__ x,
                            const __nv_bfloat16* __restrict__ w, const float* __restrict__ mean,
                            const float* __restrict__ rstd, __nv_bfloat16* __restrict__ dx, float* __restrict__ scratch,
                            int rows, int C, int rows_per_cta) {
  __shared__ float acc[2 * kMaxHidden];
  const int nwarp = blockDim.x >> 5, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nvec = C >> 3;
  float gw[VPL][8], gb[VPL][8], wf[VPL][8];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
#pragma unroll
    for (int j = 0; j < 8; ++j) gw[i][j] = gb[i][j] = 0.f;
    if (lane + 32 * i < nvec) bf8_to_f(reinterpret_cast<const uint4*>(w)[lane + 32 * i], wf[i]);
  }
  const int r0 = blockIdx.x * rows_per_cta, r1 = min(rows, r0 + rows_per_cta);
  for (int r = r0 + warp; r < r1; r += nwarp) {
    const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(r) * C);
    const uint4* dr = reinterpret_cast<const uint4*>(dy + static_cast<size_t>(r) * C);
    const float mu = mean[r], rs = rstd[r];
    float xh[VPL][8], g[VPL][8], a = 0.f, bsum = 0.f;
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (lane + 32 * i < nvec) {
        float xf[8], df[8];
        bf8_to_f(xr[lane + 32 * i], xf);
        bf8_to_f(dr[lane + 32 * i], df);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          xh[i][j] = (xf[j] - mu) * rs;
          g[i][j] = df[j] * wf[i][j];
          a += g[i][j];
          bsum += g[i][j] * xh[i][j];
          gw[i][j] += df[j] * xh[i][j];
          gb[i][j] += df[j];
        }
      }
    }
    a = warp_allsum(a) / C;
    bsum = warp_allsum(bsum) / C;
    uint4* o = reinterpret_cast<uint4*>(dx + static_cast<size_t>(r) * C);
#pragma unroll
    for (int i = 0; i < VPL; ++i) {
      if (lane + 32 * i < nvec) {
        float v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = rs * (g[i][j] - a - xh[i][j] * bsum);
        o[lane + 32 * i] = f_to_bf8(v);
      }
    }
  }
  for (int c = threadIdx.x; c < 2 * C; c += blockDim.x) acc[c] = 0.f;
  __syncthreads();
  for (int k = 0; k < nwarp; ++k) {  // warp order
    if (warp == k) {
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int v = lane + 32 * i;
        if (v < nvec) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            acc[v * 8 + j] += gw[i][j];
            acc[C + v * 8 + j] += gb[i][j];
          }
        }
      }
    }
    __syncthreads();
  }
  float* pw = scratch + static_cast<size_t>(blockIdx.x) * kMaxHidden;
  float* pb = scratch + static_cast<size_t>(kMaxCtas + blockIdx.x) * kMaxHidden;
  for (int c = threadIdx.x; c < C; c += blockDim.x) {
    pw[c] = acc[c];
    pb[c] = acc[C + c];
  }
}

// Hidden sizes above 1024 (more than 4 vectors per lane): the per-lane
// dgamma/dbeta accumulators of ln_bwd_rows would spill out of registers,
// so dx and the parameter gradients are computed by separate kernels. First
// dx alone, one warp per row, with x and dy held packed (bf16) in registers.
template <int VPL>
__global__ void __launch_bounds__(256) ln_bwd_dx_only(const __nv_bfloat16* __restrict__ dy,
                                                      const __nv_bfloat16* __restrict__ x,
                                                      const __nv_bfloat16* __restrict__ w,
                                                      const float* __restrict__ mean, const float* __restrict__ rstd,
                                                      __nv_bfloat16* __restrict__ dx, int rows, int C) {
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int nvec = C >> 3;
  const uint4* xr = reinterpret_cast<const uint4*>(x + static_cast<size_t>(row) * C);
  const uint4* dr = reinterpret_cast<const uint4*>(dy + static_cast<size_t>(row) * C);
  const uint4* wv = reinterpret_cast<const uint4*>(w);
  uint4 xp[VPL], dp[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (lane + 32 * i < nvec) {
      xp[i] = xr[lane + 32 * i];
      dp[i] = dr[lane + 32 * i];
    }
  }
  const float mu = mean[row], rs = rstd[row];
  float a = 0.f, bsum = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (lane + 32 * i < nvec) {
      float xf[8], df[8], wf[8];
      bf8_to_f(xp[i], xf);
      bf8_to_f(dp[i], df);
      bf8_to_f(__ldg(wv + lane + 32 * i), wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float g = df[j] * wf[j];
        a += g;
        bsum += g * (xf[j] - mu) * rs;
      }
    }
  }
  a = warp_allsum(a) / C;
  bsum = warp_allsum(bsum) / C;
  uint4* o = reinterpret_cast<uint4*>(dx + static_cast<size_t>(row) * C);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    if (lane + 32 * i < nvec) {
      float xf[8], df[8], wf[8], v[8];
      bf8_to_f(xp[i], xf);
      bf8_to_f(dp[i], df);
      bf8_to_f(__ldg(wv + lane + 32 * i), wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = rs * (df[j] * wf[j] - a - (xf[j] - mu) * rs * bsum);
      o[lane + 32 * i] = f_to_bf8(v);
    }
  }
}

// Then one partial row of dgamma and of dbeta per block of rows: block
// (blockIdx.x, blockIdx.y) sums 256 columns over rows [y * rows_per_blk,
// (y + 1) * rows_per_blk) in row order into scratch rows y and kMaxCtas + y.
__global__ void __launch_bounds__(256) ln_bwd_col_partials(const __nv_bfloat16* __restrict__ dy,
                                                           const __nv_bfloat16* __restrict__ x,
                                                           const float* __restrict__ mean,
                                                           const float* __restrict__ rstd, float* __restrict__ scratch,
                                                           int rows, int C, int rows_per_blk) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int r0 = blockIdx.y * rows_per_blk, r1 = min(rows, r0 + rows_per_blk);
  float gw = 0.f, gb = 0.f;
  for (int r = r0; r < r1; ++r) {
    const size_t off = static_cast<size_t>(r) * C + c;
    const float d = __bfloat162float(dy[off]);
    gw += d * (__bfloat162float(x[off]) - mean[r]) * rstd[r];
    gb += d;
  }
  scratch[static_cast<size_t>(blockIdx.y) * kMaxHidden + c] = gw;
  scratch[static_cast<size_t>(kMaxCtas + blockIdx.y) * kMaxHidden + c] = gb;
}

// Pass two: sum the partial rows in CTA order.
__global__ void ln_bwd_sum(const float* __restrict__ scratch, int ctas, int C, __nv_bfloat16* __restrict__ dw,
                           __nv_bfloat16* __restrict__ db) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float a = 0.f, b = 0.f;
  for (int k = 0; k < ctas; ++k) {
    a += scratch[static_cast<size_t>(k) * kMaxHidden + c];
    b += scratch[static_cast<size_t>(kMaxCtas + k) * kMaxHidden + c];
  }
  dw[c] = __float2bfloat16_rn(a);
  db[c] = __float2bfloat16_rn(b);
}

template <int VPL>
cudaError_t launch_rows(const void* dy, const void* x, const void* w, const float* mean, const float* rstd, void* dx,
                        float* scratch, int rows, int C, int ctas, int rows_per_cta, cudaStream_t st) {
  ln_bwd_rows<VPL><<<ctas, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
                                         static_cast<const __nv_bfloat16*>(w), mean, rstd,
                                         static_cast<__nv_bfloat16*>(dx), scratch, rows, C, rows_per_cta);
  return cudaGetLastError();
}

bool misaligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; }

}  // namespace

extern "C" __attribute__((visibility("default"))) int dst_layernorm_bwd_noalloc(
    const void* dy, const void* x, const void* w, const float* mean, const float* rstd, void* dx, void* dw, void* db,
    int rows, int hidden, cudaStream_t stream) {
  if (!dy || !x || !w || !mean || !rstd || !dx || !dw || !db || rows < 1 || hidden < 8 || hidden % 8 != 0)
    return DST_NOALLOC_ERR_BAD_ARG;
  // The row kernels move dy, x, w and dx in 16-byte vectors.
  if (misaligned(dy, 16) || misaligned(x, 16) || misaligned(w, 16) || misaligned(dx, 16) || misaligned(mean, 4) ||
      misaligned(rstd, 4) || misaligned(dw, 2) || misaligned(db, 2))
    return DST_NOALLOC_ERR_BAD_ARG;
  if (hidden > kMaxHidden) return DST_NOALLOC_ERR_TOO_LARGE;
  float* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != cudaSuccess) return DST_NOALLOC_ERR_CUDA;
  if (hidden > 1024) {
    // dx, then per-block column partials, then their ordered sum.
    const int dx_blocks = (rows + 7) / 8;
    if (hidden <= 2048)
      ln_bwd_dx_only<8><<<dx_blocks, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
          static_cast<const __nv_bfloat16*>(w), mean, rstd, static_cast<__nv_bfloat16*>(dx), rows, hidden);
    else
      ln_bwd_dx_only<16><<<dx_blocks, 256, 0, stream>>>(
          static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
          static_cast<const __nv_bfloat16*>(w), mean, rstd, static_cast<__nv_bfloat16*>(dx), rows, hidden);
    if (cudaGetLastError() != cudaSuccess) return DST_NOALLOC_ERR_CUDA;
    const int rows_per_blk = (rows + kMaxCtas - 1) / kMaxCtas;
    const int blks = (rows + rows_per_blk - 1) / rows_per_blk;
    ln_bwd_col_partials<<<dim3((hidden + 255) / 256, blks), 256, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x), mean, rstd, scratch, rows,
        hidden, rows_per_blk);
    if (cudaGetLastError() != cudaSuccess) return DST_NOALLOC_ERR_CUDA;
    ln_bwd_sum<<<(hidden + 255) / 256, 256, 0, stream>>>(scratch, blks, hidden, static_cast<__nv_bfloat16*>(dw),
                                                         static_cast<__nv_bfloat16*>(db));
    return cudaGetLastError() == cudaSuccess ? DST_NOALLOC_OK : DST_NOALLOC_ERR_CUDA;
  }
  // At least 8 rows (one per warp) per CTA, and no more CTAs than partial
  // rows in the scratch array.
  int rows_per_cta = (rows + kMaxCtas - 1) / kMaxCtas;
  if (rows_per_cta < 8) rows_per_cta = 8;
  const int ctas = (rows + rows_per_cta - 1) / rows_per_cta;
  cudaError_t e;
  const int nvec = hidden / 8;
  if (nvec <= 32)
    e = launch_rows<1>(dy, x, w, mean, rstd, dx, scratch, rows, hidden, ctas, rows_per_cta, stream);
  else if (nvec <= 64)
    e = launch_rows<2>(dy, x, w, mean, rstd, dx, scratch, rows, hidden, ctas, rows_per_cta, stream);
  else  // nvec <= 128: hidden <= 1024
    e = launch_rows<4>(dy, x, w, mean, rstd, dx, scratch, rows, hidden, ctas, rows_per_cta, stream);
  if (e != cudaSuccess) return DST_NOALLOC_ERR_CUDA;
  ln_bwd_sum<<<(hidden + 255) / 256, 256, 0, stream>>>(scratch, ctas, hidden, static_cast<__nv_bfloat16*>(dw),
                                                       static_cast<__nv_bfloat16*>(db));
  return cudaGetLastError() == cudaSuccess ? DST_NOALLOC_OK : DST_NOALLOC_ERR_CUDA;
}
