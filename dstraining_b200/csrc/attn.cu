// Causal flash attention forward / backward, bf16 in, fp32 softmax state.
//
// Q, K and V are read in place from the fused QKV projection output
// [B, T, H, 3, D] (head-major: per head q|k|v), so no split or transpose
// copies exist; the output is written as [B, T, H, D] (the layout the output
// projection consumes) and the per-row log-sum-exp (base 2, pre-scaled) is
// saved for backward.
//
// Forward: one CTA of 4 warps per (64-query block, head, batch); each warp
// owns 16 query rows. K/V tiles stream through double-buffered, XOR-swizzled
// shared memory (cp.async), S = Q K^T and O += P V run on m16n8k16 bf16 MMAs
// with the online-softmax rescale in registers (the S accumulator fragment is
// re-used directly as the A fragment of P V).
//
// Backward is deterministic (no atomics, fixed loop orders), in three
// kernels: Di = rowsum(dO * O); a dK/dV kernel per 64-key block that walks
// the query blocks at or after it; a dQ kernel per 64-query block that walks
// the key blocks up to its diagonal. Both recompute P from Q, K and the
// saved log-sum-exp.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.h"
#include "ptx.cuh"

namespace dst {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void cp_async16(uint32_t saddr, const void* g, bool pred) {
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(saddr), "l"(g), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Element offset of (row, col) in a [rows][D] bf16 tile whose 16-byte chunks
// are XOR-swizzled by (row % 8) (bank-conflict-free ldmatrix).
template <int D>
__device__ __forceinline__ int swz(int row, int col) {
  return row * D + ((((col >> 3) ^ (row & 7))) << 3) + (col & 7);
}

// Copy ROWS rows x D of a strided bf16 matrix into a swizzled tile; rows
// beyond `valid` are zero-filled.
template <int ROWS, int D, int THREADS>
__device__ __forceinline__ void load_tile(__nv_bfloat16* s, const __nv_bfloat16* g, int ld, int valid) {
  constexpr int CH = D / 8;
  for (int i = threadIdx.x; i < ROWS * CH; i += THREADS) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < valid;
    cp_async16(smem_u32(s + swz<D>(r, c * 8)), g + static_cast<size_t>(ok ? r : 0) * ld + c * 8, ok);
  }
}

// A fragment (16 rows x 16 k) of a swizzled [rows][D] tile at (row0, k0).
template <int D>
__device__ __forceinline__ void frag_a(uint32_t (&a)[4], const __nv_bfloat16* s, int row0, int k0, int lane) {
  const int r = row0 + (lane & 7) + 8 * ((lane >> 3) & 1);
  const int c = k0 + 8 * (lane >> 4);
  ldsm_x4(a, smem_u32(s + swz<D>(r, c)));
}

// Two B fragments (k 16 x n 8, n-blocks n0 and n0+8) where the tile stores
// [n][k] (k contiguous): non-transposed ldmatrix.
template <int D>
__device__ __forceinline__ void frag_b_nk(uint32_t (&b)[4], const __nv_bfloat16* s, int n0, int k0, int lane) {
  const int r = n0 + (lane & 7) + 8 * (lane >> 4);
  const int c = k0 + 8 * ((lane >> 3) & 1);
  ldsm_x4(b, smem_u32(s + swz<D>(r, c)));
  // b[0], b[1]: n-block n0; b[2], b[3]: n-block n0 + 8
}

// Two B fragments where the tile stores [k][n] (n contiguous): transposed
// ldmatrix. Returns b[0], b[1] for n-block n0 and b[2], b[3] for n0 + 8.
template <int D>
__device__ __forceinline__ void frag_b_kn(uint32_t (&b)[4], const __nv_bfloat16* s, int k0, int n0, int lane) {
  const int r = k0 + (lane & 7) + 8 * ((lane >> 3) & 1);
  const int c = n0 + 8 * (lane >> 4);
  ldsm_x4_t(b, smem_u32(s + swz<D>(r, c)));
}

// ------------------------------------------------------------------ forward
template <int D>
__global__ void __launch_bounds__(128) fwd_kernel(const __nv_bfloat16* __restrict__ qkv, __nv_bfloat16* __restrict__ out,
                                                  float* __restrict__ lse2, int T, int H, float scale_log2) {
  constexpr int BM = 64, BN = 64;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);
  __nv_bfloat16* sK = sQ + BM * D;      // [2][BN][D]
  __nv_bfloat16* sV = sK + 2 * BN * D;  // [2][BN][D]
  const int qb = gridDim.x - 1 - blockIdx.x;  // heaviest blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = 3 * H * D;
  const __nv_bfloat16* base = qkv + static_cast<size_t>(b) * T * ld + h * 3 * D;
  const int q0 = qb * BM;

  load_tile<BM, D, 128>(sQ, base + static_cast<size_t>(q0) * ld, ld, T - q0);
  load_tile<BN, D, 128>(sK, base + D, ld, T);
  load_tile<BN, D, 128>(sV, base + 2 * D, ld, T);
  cp_commit();

  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];
  const int nkb = qb + 1;
  for (int kb = 0; kb < nkb; ++kb) {
    const int cur = kb & 1;
    if (kb + 1 < nkb) {
      const int k0 = (kb + 1) * BN;
      load_tile<BN, D, 128>(sK + (cur ^ 1) * BN * D, base + static_cast<size_t>(k0) * ld + D, ld, T - k0);
      load_tile<BN, D, 128>(sV + (cur ^ 1) * BN * D, base + static_cast<size_t>(k0) * ld + 2 * D, ld, T - k0);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) frag_a<D>(qf[ks], sQ, warp * 16, ks * 16, lane);
    }
    const __nv_bfloat16* k_s = sK + cur * BN * D;
    const __nv_bfloat16* v_s = sV + cur * BN * D;
    float s[BN / 8][4];
#pragma unroll
    for (int i = 0; i < BN / 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int p = 0; p < BN / 16; ++p) {
        uint32_t bf[4];
        frag_b_nk<D>(bf, k_s, p * 16, ks * 16, lane);
        mma16816(s[2 * p], qf[ks], bf[0], bf[1]);
        mma16816(s[2 * p + 1], qf[ks], bf[2], bf[3]);
      }
    }
    // scale, causal mask, online softmax
    const int row_a = q0 + warp * 16 + (lane >> 2);
    const int kbase = kb * BN + 2 * (lane & 3);
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = row_a + (e >> 1) * 8;
        const int key = kbase + nb * 8 + (e & 1);
        float v = s[nb][e] * scale_log2;
        if (kb == qb && key > row) v = -INFINITY;
        s[nb][e] = v;
        mx[e >> 1] = fmaxf(mx[e >> 1], v);
      }
    }
    float corr[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffff, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffff, mx[r], 2));
      const float nm = fmaxf(m_r[r], mx[r]);
      corr[r] = exp2f(m_r[r] - nm);
      m_r[r] = nm;
      l_r[r] *= corr[r];
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      o[i][0] *= corr[0];
      o[i][1] *= corr[0];
      o[i][2] *= corr[1];
      o[i][3] *= corr[1];
    }
#pragma unroll
    for (int nb = 0; nb < BN / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float pv = exp2f(s[nb][e] - m_r[e >> 1]);
        s[nb][e] = pv;
        l_r[e >> 1] += pv;
      }
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bf[4];
        frag_b_kn<D>(bf, v_s, kk * 16, dp * 16, lane);
        mma16816(o[2 * dp], pa, bf[0], bf[1]);
        mma16816(o[2 * dp + 1], pa, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffff, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffff, l_r[r], 2);
  }
  const int ldo = H * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = q0 + warp * 16 + (lane >> 2) + r * 8;
    if (row < T) {
      const float inv = 1.f / l_r[r];
      __nv_bfloat16* orow = out + (static_cast<size_t>(b) * T + row) * ldo + h * D + 2 * (lane & 3);
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<uint32_t*>(orow + i * 8) = pack_bf16(o[i][2 * r] * inv, o[i][2 * r + 1] * inv);
      if ((lane & 3) == 0) lse2[(static_cast<size_t>(b) * H + h) * T + row] = m_r[r] + log2f(l_r[r]);
    }
  }
}

// ------------------------------------------------------------------ Di
// Di[b, h, t] = sum_d dO[b, t, h, d] * O[b, t, h, d]
__global__ void dot_do_o_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                float* __restrict__ di, int B, int T, int H, int D) {
  const int warps = blockDim.x >> 5;
  const int idx = blockIdx.x * warps + (threadIdx.x >> 5);  // (b, t, h)
  const int lane = threadIdx.x & 31;
  if (idx >= B * T * H) return;
  const int h = idx % H, bt = idx / H, t = bt % T, b = bt / T;
  const __nv_bfloat16* a = dout + static_cast<size_t>(idx) * D;
  const __nv_bfloat16* c = out + static_cast<size_t>(idx) * D;
  float s = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a + d));
    float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(c + d));
    s += x.x * y.x + x.y * y.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffff, s, o);
  if (lane == 0) di[(static_cast<size_t>(b) * H + h) * T + t] = s;
}

// ------------------------------------------------------------------ dK, dV
// One CTA per (64-key block, head, batch); each warp owns 16 keys. Walks
// query blocks of BQ rows from the diagonal to the end.
template <int D, int BQ>
__global__ void __launch_bounds__(128) dkdv_kernel(const __nv_bfloat16* __restrict__ qkv,
                                                   const __nv_bfloat16* __restrict__ dout,
                                                   const float* __restrict__ lse2, const float* __restrict__ di,
                                                   __nv_bfloat16* __restrict__ dqkv, int T, int H, float scale_log2,
                                                   float scale) {
  constexpr int BK = 64;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sK = reinterpret_cast<__nv_bfloat16*>(smem);  // [BK][D]
  __nv_bfloat16* sV = sK + BK * D;                              // [BK][D]
  __nv_bfloat16* sQ = sV + BK * D;                              // [2][BQ][D]
  __nv_bfloat16* sO = sQ + 2 * BQ * D;                          // [2][BQ][D] (dO)
  float* sL = reinterpret_cast<float*>(sO + 2 * BQ * D);       // [2][BQ]
  float* sD = sL + 2 * BQ;                                      // [2][BQ]
  const int kb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = 3 * H * D, ldo = H * D;
  const __nv_bfloat16* base = qkv + static_cast<size_t>(b) * T * ld + h * 3 * D;
  const __nv_bfloat16* obase = dout + static_cast<size_t>(b) * T * ldo + h * D;
  const float* lrow = lse2 + (static_cast<size_t>(b) * H + h) * T;
  const float* drow = di + (static_cast<size_t>(b) * H + h) * T;
  const int k0 = kb * BK;

  load_tile<BK, D, 128>(sK, base + static_cast<size_t>(k0) * ld + D, ld, T - k0);
  load_tile<BK, D, 128>(sV, base + static_cast<size_t>(k0) * ld + 2 * D, ld, T - k0);
  const int qb0 = k0 / BQ;
  const int nqb = (T + BQ - 1) / BQ;
  auto load_q = [&](int qb, int buf) {
    const int q0 = qb * BQ;
    load_tile<BQ, D, 128>(sQ + buf * BQ * D, base + static_cast<size_t>(q0) * ld, ld, T - q0);
    load_tile<BQ, D, 128>(sO + buf * BQ * D, obase + static_cast<size_t>(q0) * ldo, ldo, T - q0);
    for (int i = threadIdx.x; i < BQ; i += 128) {
      sL[buf * BQ + i] = (q0 + i < T) ? lrow[q0 + i] : 0.f;
      sD[buf * BQ + i] = (q0 + i < T) ? drow[q0 + i] : 0.f;
    }
  };
  load_q(qb0, 0);
  cp_commit();

  float dk[D / 8][4], dv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) dk[i][e] = dv[i][e] = 0.f;

  for (int qb = qb0; qb < nqb; ++qb) {
    const int cur = (qb - qb0) & 1;
    __syncthreads();  // previous readers of buffer cur^1 are done
    if (qb + 1 < nqb) load_q(qb + 1, cur ^ 1);
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    const __nv_bfloat16* q_s = sQ + cur * BQ * D;
    const __nv_bfloat16* o_s = sO + cur * BQ * D;
    const float* l_s = sL + cur * BQ;
    const float* d_s = sD + cur * BQ;
    // S^T = K Q^T : [16 keys x BQ]
    float st[BQ / 8][4], dpt[BQ / 8][4];
#pragma unroll
    for (int i = 0; i < BQ / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) st[i][e] = dpt[i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      uint32_t ka[4], va[4];
      frag_a<D>(ka, sK, warp * 16, ks * 16, lane);
      frag_a<D>(va, sV, warp * 16, ks * 16, lane);
#pragma unroll
      for (int p = 0; p < BQ / 16; ++p) {
        uint32_t bq[4], bo[4];
        frag_b_nk<D>(bq, q_s, p * 16, ks * 16, lane);
        mma16816(st[2 * p], ka, bq[0], bq[1]);
        mma16816(st[2 * p + 1], ka, bq[2], bq[3]);
        frag_b_nk<D>(bo, o_s, p * 16, ks * 16, lane);
        mma16816(dpt[2 * p], va, bo[0], bo[1]);
        mma16816(dpt[2 * p + 1], va, bo[2], bo[3]);
      }
    }
    // P^T and dS^T
    const int key_a = k0 + warp * 16 + (lane >> 2);
#pragma unroll
    for (int nb = 0; nb < BQ / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key_a + (e >> 1) * 8;
        const int ql = nb * 8 + 2 * (lane & 3) + (e & 1);
        const int q = qb * BQ + ql;
        float p = 0.f;
        if (key <= q && q < T && key < T) p = exp2f(st[nb][e] * scale_log2 - l_s[ql]);
        st[nb][e] = p;
        dpt[nb][e] = p * (dpt[nb][e] - d_s[ql]);
      }
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
      uint32_t pa[4], sa[4];
      pa[0] = pack_bf16(st[2 * kk][0], st[2 * kk][1]);
      pa[1] = pack_bf16(st[2 * kk][2], st[2 * kk][3]);
      pa[2] = pack_bf16(st[2 * kk + 1][0], st[2 * kk + 1][1]);
      pa[3] = pack_bf16(st[2 * kk + 1][2], st[2 * kk + 1][3]);
      sa[0] = pack_bf16(dpt[2 * kk][0], dpt[2 * kk][1]);
      sa[1] = pack_bf16(dpt[2 * kk][2], dpt[2 * kk][3]);
      sa[2] = pack_bf16(dpt[2 * kk + 1][0], dpt[2 * kk + 1][1]);
      sa[3] = pack_bf16(dpt[2 * kk + 1][2], dpt[2 * kk + 1][3]);
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bo[4], bq[4];
        frag_b_kn<D>(bo, o_s, kk * 16, dp * 16, lane);
        mma16816(dv[2 * dp], pa, bo[0], bo[1]);
        mma16816(dv[2 * dp + 1], pa, bo[2], bo[3]);
        frag_b_kn<D>(bq, q_s, kk * 16, dp * 16, lane);
        mma16816(dk[2 * dp], sa, bq[0], bq[1]);
        mma16816(dk[2 * dp + 1], sa, bq[2], bq[3]);
      }
    }
  }
  __nv_bfloat16* gbase = dqkv + static_cast<size_t>(b) * T * ld + h * 3 * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = k0 + warp * 16 + (lane >> 2) + r * 8;
    if (key < T) {
      __nv_bfloat16* krow = gbase + static_cast<size_t>(key) * ld + D + 2 * (lane & 3);
      __nv_bfloat16* vrow = krow + D;
#pragma unroll
      for (int i = 0; i < D / 8; ++i) {
        *reinterpret_cast<uint32_t*>(krow + i * 8) = pack_bf16(dk[i][2 * r] * scale, dk[i][2 * r + 1] * scale);
        *reinterpret_cast<uint32_t*>(vrow + i * 8) = pack_bf16(dv[i][2 * r], dv[i][2 * r + 1]);
      }
    }
  }
}

// ------------------------------------------------------------------ dQ
template <int D, int BKV>
__global__ void __launch_bounds__(128) dq_kernel(const __nv_bfloat16* __restrict__ qkv, const __nv_bfloat16* __restrict__ dout,
                                                 const float* __restrict__ lse2, const float* __restrict__ di,
                                                 __nv_bfloat16* __restrict__ dqkv, int T, int H, float scale_log2,
                                                 float scale) {
  constexpr int BM = 64;
  extern __shared__ __align__(128) uint8_t smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(smem);  // [BM][D]
  __nv_bfloat16* sO = sQ + BM * D;                             // [BM][D]
  __nv_bfloat16* sK = sO + BM * D;                             // [2][BKV][D]
  __nv_bfloat16* sV = sK + 2 * BKV * D;                        // [2][BKV][D]
  const int qb = gridDim.x - 1 - blockIdx.x;
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ld = 3 * H * D, ldo = H * D;
  const __nv_bfloat16* base = qkv + static_cast<size_t>(b) * T * ld + h * 3 * D;
  const __nv_bfloat16* obase = dout + static_cast<size_t>(b) * T * ldo + h * D;
  const int q0 = qb * BM;
  load_tile<BM, D, 128>(sQ, base + static_cast<size_t>(q0) * ld, ld, T - q0);
  load_tile<BM, D, 128>(sO, obase + static_cast<size_t>(q0) * ldo, ldo, T - q0);
  load_tile<BKV, D, 128>(sK, base + D, ld, T);
  load_tile<BKV, D, 128>(sV, base + 2 * D, ld, T);
  cp_commit();
  const int row_a = q0 + warp * 16 + (lane >> 2);
  float lrow[2], drow[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = min(row_a + r * 8, T - 1);
    lrow[r] = lse2[(static_cast<size_t>(b) * H + h) * T + row];
    drow[r] = di[(static_cast<size_t>(b) * H + h) * T + row];
  }
  float dq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) dq[i][0] = dq[i][1] = dq[i][2] = dq[i][3] = 0.f;
  uint32_t qf[D / 16][4], of[D / 16][4];
  const int last_key = min(T, q0 + BM) - 1;
  const int nkb = last_key / BKV + 1;
  for (int kb = 0; kb < nkb; ++kb) {
    const int cur = kb & 1;
    if (kb + 1 < nkb) {
      const int k0 = (kb + 1) * BKV;
      load_tile<BKV, D, 128>(sK + (cur ^ 1) * BKV * D, base + static_cast<size_t>(k0) * ld + D, ld, T - k0);
      load_tile<BKV, D, 128>(sV + (cur ^ 1) * BKV * D, base + static_cast<size_t>(k0) * ld + 2 * D, ld, T - k0);
    }
    cp_commit();
    cp_wait<1>();
    __syncthreads();
    if (kb == 0) {
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        frag_a<D>(qf[ks], sQ, warp * 16, ks * 16, lane);
        frag_a<D>(of[ks], sO, warp * 16, ks * 16, lane);
      }
    }
    const __nv_bfloat16* k_s = sK + cur * BKV * D;
    const __nv_bfloat16* v_s = sV + cur * BKV * D;
    float s[BKV / 8][4], dp[BKV / 8][4];
#pragma unroll
    for (int i = 0; i < BKV / 8; ++i)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[i][e] = dp[i][e] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int p = 0; p < BKV / 16; ++p) {
        uint32_t bk[4], bv[4];
        frag_b_nk<D>(bk, k_s, p * 16, ks * 16, lane);
        mma16816(s[2 * p], qf[ks], bk[0], bk[1]);
        mma16816(s[2 * p + 1], qf[ks], bk[2], bk[3]);
        frag_b_nk<D>(bv, v_s, p * 16, ks * 16, lane);
        mma16816(dp[2 * p], of[ks], bv[0], bv[1]);
        mma16816(dp[2 * p + 1], of[ks], bv[2], bv[3]);
      }
    }
#pragma unroll
    for (int nb = 0; nb < BKV / 8; ++nb) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = row_a + (e >> 1) * 8;
        const int key = kb * BKV + nb * 8 + 2 * (lane & 3) + (e & 1);
        float p = 0.f;
        if (key <= row && row < T) p = exp2f(s[nb][e] * scale_log2 - lrow[e >> 1]);
        s[nb][e] = p * (dp[nb][e] - drow[e >> 1]);  // dS
      }
    }
#pragma unroll
    for (int kk = 0; kk < BKV / 16; ++kk) {
      uint32_t sa[4];
      sa[0] = pack_bf16(s[2 * kk][0], s[2 * kk][1]);
      sa[1] = pack_bf16(s[2 * kk][2], s[2 * kk][3]);
      sa[2] = pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      sa[3] = pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int dpi = 0; dpi < D / 16; ++dpi) {
        uint32_t bk[4];
        frag_b_kn<D>(bk, k_s, kk * 16, dpi * 16, lane);
        mma16816(dq[2 * dpi], sa, bk[0], bk[1]);
        mma16816(dq[2 * dpi + 1], sa, bk[2], bk[3]);
      }
    }
    __syncthreads();
  }
  __nv_bfloat16* gbase = dqkv + static_cast<size_t>(b) * T * ld + h * 3 * D;
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int row = row_a + r * 8;
    if (row < T) {
      __nv_bfloat16* qrow = gbase + static_cast<size_t>(row) * ld + 2 * (lane & 3);
#pragma unroll
      for (int i = 0; i < D / 8; ++i)
        *reinterpret_cast<uint32_t*>(qrow + i * 8) = pack_bf16(dq[i][2 * r] * scale, dq[i][2 * r + 1] * scale);
    }
  }
}

template <typename K>
static void set_smem(K kern, int bytes) {
  if (bytes > 48 * 1024) C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
}

}  // namespace attn
}  // namespace dst

using namespace dst;
using namespace dst::attn;

static void check_qkv(const at::Tensor& qkv, int64_t H, int64_t D) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3 && qkv.is_contiguous(),
              "attention: contiguous bf16 [B, T, 3 H D] qkv required");
  TORCH_CHECK(qkv.size(2) == 3 * H * D, "attention: qkv width must be 3 * heads * head_dim");
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(qkv.size(1) % 64 == 0, "attention: sequence length must be a multiple of 64");
}

std::vector<at::Tensor> flash_attn_fwd(const at::Tensor& qkv, int64_t H, int64_t D) {
  check_qkv(qkv, H, D);
  c10::cuda::CUDAGuard g(qkv.device());
  const int B = qkv.size(0), T = qkv.size(1);
  at::Tensor out = at::empty({B, T, H * D}, qkv.options());
  at::Tensor lse = at::empty({B, H, T}, qkv.options().dtype(at::kFloat));
  const float scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D))) * kLog2e;
  dim3 grid(T / 64, H, B);
  auto st = at::cuda::getCurrentCUDAStream();
  auto* q = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (D == 64) {
    const int smem = (64 + 4 * 64) * 64 * 2;
    set_smem(fwd_kernel<64>, smem);
    fwd_kernel<64><<<grid, 128, smem, st>>>(q, o, lse.data_ptr<float>(), T, H, scale_log2);
  } else {
    const int smem = (64 + 4 * 64) * 128 * 2;
    set_smem(fwd_kernel<128>, smem);
    fwd_kernel<128><<<grid, 128, smem, st>>>(q, o, lse.data_ptr<float>(), T, H, scale_log2);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, lse};
}

at::Tensor flash_attn_bwd(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out, const at::Tensor& lse,
                          int64_t H, int64_t D) {
  check_qkv(qkv, H, D);
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous() && dout.sizes() == out.sizes(), "attention bwd: dout/out");
  TORCH_CHECK(out.dim() == 3 && out.size(0) == qkv.size(0) && out.size(1) == qkv.size(1) && out.size(2) == H * D &&
                  out.scalar_type() == at::kBFloat16 && dout.scalar_type() == at::kBFloat16,
              "attention bwd: bf16 out / dout [B, T, H * D] required");
  TORCH_CHECK(lse.numel() == qkv.size(0) * H * qkv.size(1), "attention bwd: lse [B, H, T] required");
  c10::cuda::CUDAGuard g(qkv.device());
  const int B = qkv.size(0), T = qkv.size(1);
  at::Tensor dqkv = at::empty_like(qkv);
  at::Tensor di = at::empty({B, H, T}, qkv.options().dtype(at::kFloat));
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(D)));
  const float scale_log2 = scale * kLog2e;
  auto st = at::cuda::getCurrentCUDAStream();
  auto* q = reinterpret_cast<const __nv_bfloat16*>(qkv.data_ptr());
  auto* dO = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
  auto* dq = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  const int rows = B * T * H;
  dot_do_o_kernel<<<(rows + 7) / 8, 256, 0, st>>>(dO, reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
                                                  di.data_ptr<float>(), B, T, H, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  dim3 grid(T / 64, H, B);
  if (D == 64) {
    constexpr int BQ = 64, BKV = 64;
    const int s1 = (2 * 64 + 4 * BQ) * 64 * 2 + 4 * BQ * 4;
    set_smem(dkdv_kernel<64, BQ>, s1);
    dkdv_kernel<64, BQ><<<grid, 128, s1, st>>>(q, dO, lse.data_ptr<float>(), di.data_ptr<float>(), dq, T, H, scale_log2, scale);
    const int s2 = (2 * 64 + 4 * BKV) * 64 * 2;
    set_smem(dq_kernel<64, BKV>, s2);
    dq_kernel<64, BKV><<<grid, 128, s2, st>>>(q, dO, lse.data_ptr<float>(), di.data_ptr<float>(), dq, T, H, scale_log2, scale);
  } else {
    constexpr int BQ = 32, BKV = 32;
    const int s1 = (2 * 64 + 4 * BQ) * 128 * 2 + 4 * BQ * 4;
    set_smem(dkdv_kernel<128, BQ>, s1);
    dkdv_kernel<128, BQ><<<grid, 128, s1, st>>>(q, dO, lse.data_ptr<float>(), di.data_ptr<float>(), dq, T, H, scale_log2, scale);
    const int s2 = (2 * 64 + 4 * BKV) * 128 * 2;
    set_smem(dq_kernel<128, BKV>, s2);
    dq_kernel<128, BKV><<<grid, 128, s2, st>>>(q, dO, lse.data_ptr<float>(), di.data_ptr<float>(), dq, T, H, scale_log2, scale);
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

void register_attn(pybind11::module& m) {
  m.def("flash_attn_fwd", &flash_attn_fwd, "causal flash attention forward on a fused QKV buffer");
  m.def("flash_attn_bwd", &flash_attn_bwd, "causal flash attention backward (deterministic)");
}
