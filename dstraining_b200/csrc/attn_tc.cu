// Causal flash attention forward on the sm_100a tensor cores (tcgen05).
//
// One CTA per (128-query block, head, batch), 10 warps:
//   warp 0     TMA producer: the Q tile once, then K_j / V_j tiles into a
//              two-stage ring, straight out of the fused QKV buffer
//              [B*T, H*3*D] (head-major q|k|v, 128B-swizzled boxes).
//   warp 1     MMA issuer (one elected thread):
//                S_j = Q K_j^T     (M=128 queries, N=128 keys, K=D) -> TMEM
//                O_j = P_j V_j     (M=128, N=D, K=128 keys)         -> TMEM
//              each into one of two TMEM buffers, so S_{j+1} and O_j run
//              while the softmax works on S_j.
//   warps 2-9  softmax, two warps per TMEM lane quadrant (a warp may only
//              read its own quadrant): each thread owns half of one query
//              row - 64 of the 128 key columns of S_j and half of the output
//              columns. The two halves exchange their row maxima through
//              shared memory (a named barrier per quadrant), exp2 the scores
//              straight from TMEM, write P_j as bf16 into a 128B-swizzled
//              shared tile (the A operand of the next MMA), and keep the
//              running output in registers: O = O * exp2(m_prev - m_new) + O_j.
//              Keeping O in registers means the MMAs never accumulate across
//              key blocks, so no rescaling of TMEM state is ever needed.
// Output rows are normalised by the running sum and written as bf16
// [B, T, H, D]; the base-2 log-sum-exp (pre-scaled) goes to lse2[B, H, T]
// for the backward kernels. All waits are bounded (status word on expiry).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "common.h"
#include "ptx.cuh"

namespace dst {
namespace attn_tc {

constexpr int BM = 128;  // queries per CTA
constexpr int BN = 128;  // keys per block
constexpr int kThreads = 320;  // producer, MMA, 8 softmax warps
constexpr int kAtom = 128 * 128;  // one 128-row x 128-byte swizzled atom column

template <int D>
struct Cfg {
  static constexpr int kDAtoms = D / 64;
  static constexpr int kQBytes = kDAtoms * kAtom;
  static constexpr int kKBytes = kDAtoms * kAtom;
  static constexpr int kVBytes = kDAtoms * kAtom;
  static constexpr int kPBytes = 2 * kAtom;  // 128 keys = 2 atoms (one P buffer)
  // half-row exchange: max [2 parity][2 half][128]; status [2][2][128] in the
  // loop plus [2][128] for the final exchange; row sum [2][128]
  static constexpr int kRedBytes = (512 + 768 + 256) * 4;
  static constexpr int kSmem = kQBytes + 2 * (kKBytes + kVBytes) + kPBytes + kRedBytes + 1024 + 256;
  static constexpr uint32_t kTmemCols = 512;  // S[2] (2 x 128) + O[2] (2 x D)
};

// keys [32*qtr, 32*qtr + 32) of `row`: swizzle atom qtr/2, 16-byte chunks
// (qtr%2)*4 .. +3 of the P tile (K-major, 128B-swizzled A operand)
__device__ __forceinline__ void store_p_quarter(uint8_t* pbuf, int row, int qtr, const float (&p)[32]) {
  uint8_t* atom = pbuf + (qtr >> 1) * kAtom + row * 128;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 pk;
    uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(p[c * 8 + 2 * j], p[c * 8 + 2 * j + 1]);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    const int c16 = (qtr & 1) * 4 + c;
    *reinterpret_cast<uint4*>(atom + ((c16 ^ (row & 7)) << 4)) = pk;
  }
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQKV, __nv_bfloat16* __restrict__ out, float* __restrict__ lse2,
                  int T, int H, float scale_log2, int* status) {
  using C = Cfg<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + C::kQBytes;      // [2][kKBytes]
  uint8_t* sV = sK + 2 * C::kKBytes;  // [2][kVBytes]
  uint8_t* sP = sV + 2 * C::kVBytes;  // [kPBytes]
  float* red_max = reinterpret_cast<float*>(sP + C::kPBytes);
  int* red_ok = reinterpret_cast<int*>(red_max + 512);
  float* red_sum = red_max + 512 + 768;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + C::kPBytes + C::kRedBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;    // [2]
  uint64_t* s_empty = bars + 7;   // [2]
  uint64_t* p_full = bars + 9;    // [2]
  uint64_t* o_full = bars + 11;   // [2]
  uint64_t* o_empty = bars + 13;  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 15);

  const int qb = gridDim.x - 1 - blockIdx.x;  // heaviest blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = qb + 1;  // causal: key blocks 0..qb
  const int row0 = b * T;
  const int q0 = qb * BM;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], 256);
    }
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;             // S buffers at columns 0, 128
  const uint32_t tO = tmem + 2 * BN;    // O buffers at columns 256, 256 + D

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmQKV);
      mbar_arrive_expect_tx(q_full, C::kQBytes);
#pragma unroll
      for (int a = 0; a < C::kDAtoms; ++a) tma_load_2d(sQ + a * kAtom, &tmQKV, q_full, h * 3 * D + a * 64, row0 + q0);
      for (int j = 0; j < nkb; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, status, kTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&kv_full[st], C::kKBytes + C::kVBytes);
        const int k0 = j * BN;
#pragma unroll
        for (int a = 0; a < C::kDAtoms; ++a) {
          tma_load_2d(sK + st * C::kKBytes + a * kAtom, &tmQKV, &kv_full[st], h * 3 * D + D + a * 64, row0 + k0);
          tma_load_2d(sV + st * C::kVBytes + a * kAtom, &tmQKV, &kv_full[st], h * 3 * D + 2 * D + a * 64, row0 + k0);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BN, false, false);
      constexpr uint32_t idPV = idesc_bf16_f32(BM, D, false, true);
      bool ok = mbar_wait(q_full, 0, status, kTimeoutTmaFull);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&kv_full[st], ph, status, kTimeoutTmaFull)) return false;
        if (!mbar_wait(&s_empty[st], ph ^ 1, status, kTimeoutTmemEmpty)) return false;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK + st * C::kKBytes);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          umma_f16_ss(tS + st * BN, smem_desc_sw128(q_addr + off, 16, 1024), smem_desc_sw128(k_addr + off, 16, 1024), idS,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[st]);
        return true;
      };
      auto issue_pv = [&](int j) -> bool {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&p_full[st], ph, status, kTimeoutTmaFull)) return false;
        if (!mbar_wait(&o_empty[st], ph ^ 1, status, kTimeoutTmemEmpty)) return false;
        tc_fence_after();
        const uint32_t p_addr = smem_u32(sP), v_addr = smem_u32(sV + st * C::kVBytes);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint32_t poff = (kk >> 2) * kAtom + (kk & 3) * 32;
          umma_f16_ss(tO + st * D, smem_desc_sw128(p_addr + poff, 16, 1024),
                      smem_desc_sw128(v_addr + kk * 2048, kAtom, 1024), idPV, kk > 0 ? 1u : 0u);
        }
        umma_commit(&o_full[st]);
        umma_commit(&kv_empty[st]);  // K_j and V_j have now been consumed
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkb > 1) ok = issue_s(1);
      for (int j = 0; j < nkb && ok; ++j) {
        ok = issue_pv(j);
        if (ok && j + 2 < nkb) ok = issue_s(j + 2);
      }
    }
    __syncwarp();
  } else {
    // Two softmax warps per TMEM lane quadrant: `half` selects key columns
    // [64*half, 64*half + 64) of S and output columns [half*D/2, (half+1)*D/2).
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;  // row within the query block
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    constexpr int DH = D / 2;
    float o_acc[DH];
#pragma unroll
    for (int i = 0; i < DH; ++i) o_acc[i] = 0.f;
    float m = -INFINITY, l = 0.f, c_prev = 0.f;
    // `alive` is kept identical in both warps of a quadrant pair (exchanged at
    // every named barrier), so a bounded wait that expires in one of them can
    // never leave the other waiting on the pair's barrier.
    bool alive = true;
    for (int j = 0; j < nkb; ++j) {
      const int st = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      bool good = alive && mbar_wait(&s_full[st], ph, status, kTimeoutTmemFull);
      const bool diag = (j == qb);
      const int kbase = j * BN + half * 64;
      const uint32_t s_addr = tS + st * BN + half * 64 + lane_off;
      float mx = -INFINITY;
      if (good) {
        // pass 1: masked row max of this half (32 columns at a time)
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float v[32];
          tmem_ld32(s_addr + c * 32, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const bool masked = diag && (kbase + c * 32 + i > q);
            mx = fmaxf(mx, masked ? -INFINITY : v[i]);
          }
        }
        mx *= scale_log2;
      }
      // exchange half-row maxima and liveness with the partner warp
      red_max[st * 256 + half * 128 + r] = mx;
      red_ok[st * 256 + half * 128 + r] = good ? 1 : 0;
      named_bar_sync(1 + quad, 64);
      alive = good && red_ok[st * 256 + (half ^ 1) * 128 + r] != 0;
      if (!alive) break;
      mx = fmaxf(mx, red_max[st * 256 + (half ^ 1) * 128 + r]);
      const float m_new = fmaxf(m, mx);
      const float c_j = exp2f(m - m_new);
      // Fold O_{j-1} = P_{j-1} V_{j-1}; its completion also means P_{j-1} has
      // been read, so the single P tile can take P_j.
      if (j > 0) {
        const int ps = (j - 1) & 1;
        if (mbar_wait(&o_full[ps], ((j - 1) >> 1) & 1, status, kTimeoutTmemFull)) {
          tc_fence_after();
#pragma unroll
          for (int dch = 0; dch < DH / 32; ++dch) {
            float t[32];
            tmem_ld32(tO + ps * D + half * DH + dch * 32 + lane_off, t);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 32; ++i) o_acc[dch * 32 + i] = o_acc[dch * 32 + i] * c_prev + t[i];
          }
          tc_fence_before();
          mbar_arrive(&o_empty[ps]);
        } else {
          alive = false;  // reported to the partner at the next barrier
          continue;
        }
      }
      // pass 2: P = exp2(s * scale - m_new), 32 columns at a time, into the P tile
      float rowsum = 0.f;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        float v[32];
        tmem_ld32(s_addr + c * 32, v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const bool masked = diag && (kbase + c * 32 + i > q);
          v[i] = masked ? 0.f : exp2f(v[i] * scale_log2 - m_new);
          rowsum += v[i];
        }
        store_p_quarter(sP, r, half * 2 + c, v);
      }
      tc_fence_before();
      mbar_arrive(&s_empty[st]);  // S_j fully read; the buffer may be reused
      fence_proxy_async_smem();
      mbar_arrive(&p_full[st]);
      l = l * c_j + rowsum;
      m = m_new;
      c_prev = c_j;
    }
    bool ok = alive;
    if (ok) {
      const int ps = (nkb - 1) & 1;
      ok = mbar_wait(&o_full[ps], ((nkb - 1) >> 1) & 1, status, kTimeoutTmemFull);
      if (ok) {
        tc_fence_after();
#pragma unroll
        for (int dch = 0; dch < DH / 32; ++dch) {
          float t[32];
          tmem_ld32(tO + ps * D + half * DH + dch * 32 + lane_off, t);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o_acc[dch * 32 + i] = o_acc[dch * 32 + i] * c_prev + t[i];
        }
      }
    }
    // full row sum = both halves (same running max and corrections)
    red_sum[half * 128 + r] = l;
    red_ok[512 + half * 128 + r] = ok ? 1 : 0;  // slots of their own: no reuse race
    named_bar_sync(1 + quad, 64);
    l += red_sum[(half ^ 1) * 128 + r];
    ok = ok && red_ok[512 + (half ^ 1) * 128 + r] != 0;
    if (ok) {
      const float inv = 1.f / l;
      __nv_bfloat16* orow = out + (static_cast<size_t>(row0 + q) * H + h) * D + half * DH;
#pragma unroll
      for (int i = 0; i < DH; i += 8) {
        uint4 pk;
        uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          __nv_bfloat162 hv = __floats2bfloat162_rn(o_acc[i + 2 * t] * inv, o_acc[i + 2 * t + 1] * inv);
          w[t] = *reinterpret_cast<uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(orow + i) = pk;
      }
      if (half == 0) lse2[(static_cast<size_t>(b) * H + h) * T + q] = m + log2f(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}


// ------------------------------------------------------------------ backward
// Di[b, h, t] = sum_d dO[b, t, h, d] * O[b, t, h, d]; one warp per (b, t, h).
__global__ void bwd_rowdot_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                  float* __restrict__ di, int rows, int T, int H, int D) {
  const int w = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  const __nv_bfloat16* a = dout + static_cast<size_t>(w) * D;
  const __nv_bfloat16* c = out + static_cast<size_t>(w) * D;
  float acc = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    const float2 x = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(a + d));
    const float2 y = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(c + d));
    acc += x.x * y.x + x.y * y.y;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  if (lane == 0) {
    const int hh = w % H, bt = w / H;
    di[(static_cast<size_t>(bt / T) * H + hh) * T + bt % T] = acc;
  }
}

__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const float (&v)[32], float scale) {
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    uint4 pk;
    uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      __nv_bfloat162 hv = __floats2bfloat162_rn(v[i + 2 * t] * scale, v[i + 2 * t + 1] * scale);
      w[t] = *reinterpret_cast<uint32_t*>(&hv);
    }
    *reinterpret_cast<uint4*>(dst + i) = pk;
  }
}

// dK / dV: one CTA per (128-key block, head, batch), walking the query blocks
// (BQ rows) at or after the key block. Per query block:
//   S^T = K Q^T, dP^T = V dO^T            (tcgen05, M=128 keys, N=BQ)
//   P^T = exp2(S^T * scale - lse2[q]), dS^T = P^T * (dP^T - Di[q])   (8 warps)
//   dV += P^T dO, dK += dS^T Q            (tcgen05, M=128, N=D, TMEM-resident)
template <int D, int BQ>
struct DkdvCfg {
  static constexpr int kDAtoms = D / 64;
  static constexpr int kKVTile = kDAtoms * kAtom;  // 128 rows x D
  static constexpr int kQAtom = BQ * 128;          // BQ rows x 64 columns
  static constexpr int kQTile = kDAtoms * kQAtom;
  static constexpr int kPTile = (BQ / 64) * kAtom;  // 128 rows x BQ
  static constexpr int kSmem = 2 * kKVTile + 4 * kQTile + 2 * kPTile + 4 * BQ * 4 + 1024 + 256;
};

template <int D, int BQ>
__global__ void __launch_bounds__(kThreads, 1)
    dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmKV, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmDO, const float* __restrict__ lse2,
                   const float* __restrict__ di, __nv_bfloat16* __restrict__ dqkv, int T, int H, float scale_log2,
                   float scale, int* status) {
  using C = DkdvCfg<D, BQ>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::kKVTile;
  uint8_t* sQ = sV + C::kKVTile;     // [2][kQTile]
  uint8_t* sDO = sQ + 2 * C::kQTile; // [2][kQTile]
  uint8_t* sP = sDO + 2 * C::kQTile;
  uint8_t* sDS = sP + C::kPTile;
  float* sL = reinterpret_cast<float*>(sDS + C::kPTile);  // [2][BQ]
  float* sDi = sL + 2 * BQ;                               // [2][BQ]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDi + 2 * BQ);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;   // [2]
  uint64_t* q_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* pd_free = bars + 8;
  uint64_t* fin = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int kb = blockIdx.x;  // key block 0 has the most query blocks: first
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = b * T, k0 = kb * BM;
  const int qb0 = k0 / BQ;
  const int nq = T / BQ - qb0;
  const float* lrow = lse2 + (static_cast<size_t>(b) * H + h) * T;
  const float* drow = di + (static_cast<size_t>(b) * H + h) * T;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(p_full, 256);
    mbar_init(pd_free, 1);
    mbar_init(fin, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + BQ, tDV = tmem + 2 * BQ, tDK = tmem + 2 * BQ + D;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * C::kKVTile);
#pragma unroll
      for (int a = 0; a < C::kDAtoms; ++a) {
        tma_load_2d(sK + a * kAtom, &tmKV, kv_full, h * 3 * D + D + a * 64, row0 + k0);
        tma_load_2d(sV + a * kAtom, &tmKV, kv_full, h * 3 * D + 2 * D + a * 64, row0 + k0);
      }
      for (int i = 0; i < nq; ++i) {
        const int st = i & 1;
        if (!mbar_wait(&q_empty[st], ((i >> 1) & 1) ^ 1, status, kTimeoutSmemEmpty)) break;
        const int q0 = (qb0 + i) * BQ;
        mbar_arrive_expect_tx(&q_full[st], 2 * C::kQTile + 2 * BQ * 4);
#pragma unroll
        for (int a = 0; a < C::kDAtoms; ++a) {
          tma_load_2d(sQ + st * C::kQTile + a * C::kQAtom, &tmQ, &q_full[st], h * 3 * D + a * 64, row0 + q0);
          tma_load_2d(sDO + st * C::kQTile + a * C::kQAtom, &tmDO, &q_full[st], h * D + a * 64, row0 + q0);
        }
        bulk_load(sL + st * BQ, lrow + q0, BQ * 4, &q_full[st]);
        bulk_load(sDi + st * BQ, drow + q0, BQ * 4, &q_full[st]);
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BQ, false, false);
      constexpr uint32_t idG = idesc_bf16_f32(BM, D, false, true);
      bool ok = mbar_wait(kv_full, 0, status, kTimeoutTmaFull);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV), p_addr = smem_u32(sP), ds_addr = smem_u32(sDS);
      for (int i = 0; i < nq && ok; ++i) {
        const int st = i & 1;
        const uint32_t ph = (i >> 1) & 1, pi = i & 1;
        ok = mbar_wait(&q_full[st], ph, status, kTimeoutTmaFull) && mbar_wait(s_free, pi ^ 1, status, kTimeoutTmemEmpty);
        if (!ok) break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + st * C::kQTile), do_addr = smem_u32(sDO + st * C::kQTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * kAtom + (kk & 3) * 32;
          const uint32_t b_off = (kk >> 2) * C::kQAtom + (kk & 3) * 32;
          umma_f16_ss(tS, smem_desc_sw128(k_addr + a_off, 16, 1024), smem_desc_sw128(q_addr + b_off, 16, 1024), idS,
                      kk > 0 ? 1u : 0u);
          umma_f16_ss(tDP, smem_desc_sw128(v_addr + a_off, 16, 1024), smem_desc_sw128(do_addr + b_off, 16, 1024), idS,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (!(ok = mbar_wait(p_full, pi, status, kTimeoutTmaFull))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BQ / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * kAtom + (kk & 3) * 32;
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          umma_f16_ss(tDV, smem_desc_sw128(p_addr + a_off, 16, 1024), smem_desc_sw128(do_addr + kk * 2048, C::kQAtom, 1024),
                      idG, acc);
          umma_f16_ss(tDK, smem_desc_sw128(ds_addr + a_off, 16, 1024), smem_desc_sw128(q_addr + kk * 2048, C::kQAtom, 1024),
                      idG, acc);
        }
        umma_commit(&q_empty[st]);
        umma_commit(pd_free);
      }
      umma_commit(fin);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int key = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    constexpr int HB = BQ / 2;  // query columns per thread
    bool ok = true;
    for (int i = 0; i < nq && ok; ++i) {
      const int st = i & 1;
      const uint32_t ph = (i >> 1) & 1, pi = i & 1;
      ok = mbar_wait(&q_full[st], ph, status, kTimeoutTmaFull) && mbar_wait(s_full, pi, status, kTimeoutTmemFull) &&
           mbar_wait(pd_free, pi ^ 1, status, kTimeoutTmemFull);
      if (!ok) break;
      tc_fence_after();
      const int q0 = (qb0 + i) * BQ;
#pragma unroll
      for (int c = 0; c < HB / 32; ++c) {
        const int col = half * HB + c * 32;
        float sv[32], dp[32];
        tmem_ld32(tS + col + lane_off, sv);
        tmem_ld32(tDP + col + lane_off, dp);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int qc = col + t;
          const float p = (key > q0 + qc) ? 0.f : exp2f(sv[t] * scale_log2 - sL[st * BQ + qc]);
          sv[t] = p;
          dp[t] = p * (dp[t] - sDi[st * BQ + qc]);
        }
        store_p_quarter(sP, r, col / 32, sv);
        store_p_quarter(sDS, r, col / 32, dp);
      }
      tc_fence_before();
      mbar_arrive(s_free);
      fence_proxy_async_smem();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(fin, 0, status, kTimeoutTmemFull)) {
      tc_fence_after();
      __nv_bfloat16* krow = dqkv + (static_cast<size_t>(row0 + key) * H + h) * 3 * D + D + half * (D / 2);
      __nv_bfloat16* vrow = krow + D;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        float v[32];
        tmem_ld32(tDK + half * (D / 2) + c * 32 + lane_off, v);
        tmem_wait_ld();
        store_row_bf16(krow + c * 32, v, scale);
        tmem_ld32(tDV + half * (D / 2) + c * 32 + lane_off, v);
        tmem_wait_ld();
        store_row_bf16(vrow + c * 32, v, 1.f);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// dQ: one CTA per (128-query block, head, batch), walking key blocks (BK
// wide) up to the diagonal:
//   S = Q K^T, dP = dO V^T                 (tcgen05, M=128 queries, N=BK)
//   dS = exp2(S * scale - lse2) * (dP - Di)   (8 warps, into shared memory)
//   dQ += dS K                             (tcgen05, M=128, N=D, TMEM-resident)
template <int D, int BK>
struct DqCfg {
  static constexpr int kDAtoms = D / 64;
  static constexpr int kQTile = kDAtoms * kAtom;  // 128 rows x D
  static constexpr int kKAtom = BK * 128;
  static constexpr int kKTile = kDAtoms * kKAtom;  // BK rows x D
  static constexpr int kSTile = (BK / 64) * kAtom;  // 128 rows x BK
  static constexpr int kSmem = 2 * kQTile + 4 * kKTile + kSTile + 1024 + 256;
};

template <int D, int BK>
__global__ void __launch_bounds__(kThreads, 1)
    dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                 const __grid_constant__ CUtensorMap tmKV, const float* __restrict__ lse2, const float* __restrict__ di,
                 __nv_bfloat16* __restrict__ dqkv, int T, int H, float scale_log2, float scale, int* status) {
  using C = DqCfg<D, BK>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + C::kQTile;
  uint8_t* sK = sDO + C::kQTile;     // [2][kKTile]
  uint8_t* sV = sK + 2 * C::kKTile;  // [2][kKTile]
  uint8_t* sDS = sV + 2 * C::kKTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + C::kSTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;   // [2]
  uint64_t* kv_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;
  uint64_t* s_free = bars + 6;
  uint64_t* p_full = bars + 7;
  uint64_t* pd_free = bars + 8;
  uint64_t* fin = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);

  const int qb = gridDim.x - 1 - blockIdx.x;  // heaviest (most key blocks) first
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = b * T, q0 = qb * BM;
  const int nkb = (q0 + BM - 1) / BK + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, 256);
    mbar_init(p_full, 256);
    mbar_init(pd_free, 1);
    mbar_init(fin, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem, tDP = tmem + BK, tDQ = tmem + 2 * BK;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, 2 * C::kQTile);
#pragma unroll
      for (int a = 0; a < C::kDAtoms; ++a) {
        tma_load_2d(sQ + a * kAtom, &tmQ, q_full, h * 3 * D + a * 64, row0 + q0);
        tma_load_2d(sDO + a * kAtom, &tmDO, q_full, h * D + a * 64, row0 + q0);
      }
      for (int j = 0; j < nkb; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&kv_empty[st], ((j >> 1) & 1) ^ 1, status, kTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::kKTile);
#pragma unroll
        for (int a = 0; a < C::kDAtoms; ++a) {
          tma_load_2d(sK + st * C::kKTile + a * C::kKAtom, &tmKV, &kv_full[st], h * 3 * D + D + a * 64, row0 + j * BK);
          tma_load_2d(sV + st * C::kKTile + a * C::kKAtom, &tmKV, &kv_full[st], h * 3 * D + 2 * D + a * 64, row0 + j * BK);
        }
      }
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BK, false, false);
      constexpr uint32_t idG = idesc_bf16_f32(BM, D, false, true);
      bool ok = mbar_wait(q_full, 0, status, kTimeoutTmaFull);
      const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sDO), ds_addr = smem_u32(sDS);
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1, pj = j & 1;
        ok = mbar_wait(&kv_full[st], ph, status, kTimeoutTmaFull) && mbar_wait(s_free, pj ^ 1, status, kTimeoutTmemEmpty);
        if (!ok) break;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sK + st * C::kKTile), v_addr = smem_u32(sV + st * C::kKTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * kAtom + (kk & 3) * 32;
          const uint32_t b_off = (kk >> 2) * C::kKAtom + (kk & 3) * 32;
          umma_f16_ss(tS, smem_desc_sw128(q_addr + a_off, 16, 1024), smem_desc_sw128(k_addr + b_off, 16, 1024), idS,
                      kk > 0 ? 1u : 0u);
          umma_f16_ss(tDP, smem_desc_sw128(do_addr + a_off, 16, 1024), smem_desc_sw128(v_addr + b_off, 16, 1024), idS,
                      kk > 0 ? 1u : 0u);
        }
        umma_commit(s_full);
        if (!(ok = mbar_wait(p_full, pj, status, kTimeoutTmaFull))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk) {
          const uint32_t a_off = (kk >> 2) * kAtom + (kk & 3) * 32;
          umma_f16_ss(tDQ, smem_desc_sw128(ds_addr + a_off, 16, 1024), smem_desc_sw128(k_addr + kk * 2048, C::kKAtom, 1024),
                      idG, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&kv_empty[st]);
        umma_commit(pd_free);
      }
      umma_commit(fin);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quad * 32 + lane;
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float lq = lse2[(static_cast<size_t>(b) * H + h) * T + q];
    const float dq_i = di[(static_cast<size_t>(b) * H + h) * T + q];
    constexpr int HB = BK / 2;
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const uint32_t pj = j & 1;
      ok = mbar_wait(s_full, pj, status, kTimeoutTmemFull) && mbar_wait(pd_free, pj ^ 1, status, kTimeoutTmemFull);
      if (!ok) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HB / 32; ++c) {
        const int col = half * HB + c * 32;
        float sv[32], dp[32];
        tmem_ld32(tS + col + lane_off, sv);
        tmem_ld32(tDP + col + lane_off, dp);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) {
          const int kk = j * BK + col + t;
          const float p = (kk > q) ? 0.f : exp2f(sv[t] * scale_log2 - lq);
          dp[t] = p * (dp[t] - dq_i);
        }
        store_p_quarter(sDS, r, col / 32, dp);
      }
      tc_fence_before();
      mbar_arrive(s_free);
      fence_proxy_async_smem();
      mbar_arrive(p_full);
    }
    if (ok && mbar_wait(fin, 0, status, kTimeoutTmemFull)) {
      tc_fence_after();
      __nv_bfloat16* qrow = dqkv + (static_cast<size_t>(row0 + q) * H + h) * 3 * D + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        float v[32];
        tmem_ld32(tDQ + half * (D / 2) + c * 32 + lane_off, v);
        tmem_wait_ld();
        store_row_bf16(qrow + c * 32, v, scale);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn_tc
}  // namespace dst

using namespace dst;

// Forward on the tensor-core path; T must be a multiple of 128.
std::vector<at::Tensor> flash_attn_fwd_tc(const at::Tensor& qkv, int64_t H, int64_t D) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3 && qkv.is_contiguous(),
              "attention: contiguous bf16 [B, T, 3 H D] qkv required");
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(qkv.size(2) == 3 * H * D && qkv.size(1) % 128 == 0, "attention (tc): shapes");
  c10::cuda::CUDAGuard g(qkv.device());
  const int B = qkv.size(0), T = qkv.size(1);
  at::Tensor out = at::empty({B, T, H * D}, qkv.options());
  at::Tensor lse = at::empty({B, H, T}, qkv.options().dtype(at::kFloat));
  const float scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(D)));
  CUtensorMap tm = make_tmap_bf16(qkv.data_ptr(), 3 * H * D, static_cast<uint64_t>(B) * T, 3 * H * D, 64, 128);
  dim3 grid(T / 128, H, B);
  auto st = at::cuda::getCurrentCUDAStream();
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  if (D == 64) {
    auto k = attn_tc::fwd_tc_kernel<64>;
    constexpr int smem = attn_tc::Cfg<64>::kSmem;
    C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    k<<<grid, attn_tc::kThreads, smem, st>>>(tm, o, lse.data_ptr<float>(), T, H, scale_log2, status_ptr());
  } else {
    auto k = attn_tc::fwd_tc_kernel<128>;
    constexpr int smem = attn_tc::Cfg<128>::kSmem;
    C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    k<<<grid, attn_tc::kThreads, smem, st>>>(tm, o, lse.data_ptr<float>(), T, H, scale_log2, status_ptr());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return {out, lse};
}


// Backward on the tensor-core path; T must be a multiple of 128.
at::Tensor flash_attn_bwd_tc(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out,
                             const at::Tensor& lse, int64_t H, int64_t D) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3 && qkv.is_contiguous(),
              "attention bwd: contiguous bf16 qkv required");
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(qkv.size(2) == 3 * H * D && qkv.size(1) % 128 == 0, "attention bwd (tc): shapes");
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous() && dout.sizes() == out.sizes(), "attention bwd: dout/out");
  TORCH_CHECK(lse.is_contiguous() && lse.scalar_type() == at::kFloat, "attention bwd: lse");
  c10::cuda::CUDAGuard g(qkv.device());
  const int B = qkv.size(0), T = qkv.size(1);
  at::Tensor dqkv = at::empty_like(qkv);
  at::Tensor di = at::empty({B, H, T}, qkv.options().dtype(at::kFloat));
  const double sc = 1.0 / std::sqrt(static_cast<double>(D));
  const float scale = static_cast<float>(sc), scale_log2 = static_cast<float>(sc * 1.4426950408889634);
  auto st = at::cuda::getCurrentCUDAStream();
  const int rows = B * T * static_cast<int>(H);
  attn_tc::bwd_rowdot_kernel<<<(rows + 7) / 8, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr()),
                                                             reinterpret_cast<const __nv_bfloat16*>(out.data_ptr()),
                                                             di.data_ptr<float>(), rows, T, H, D);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  const uint64_t nrows = static_cast<uint64_t>(B) * T;
  const int blk = (D == 64) ? 128 : 64;  // inner block: BQ of dK/dV, BK of dQ
  CUtensorMap tmQKV128 = make_tmap_bf16(qkv.data_ptr(), 3 * H * D, nrows, 3 * H * D, 64, 128);
  CUtensorMap tmQKVb = make_tmap_bf16(qkv.data_ptr(), 3 * H * D, nrows, 3 * H * D, 64, blk);
  CUtensorMap tmDO128 = make_tmap_bf16(dout.data_ptr(), H * D, nrows, H * D, 64, 128);
  CUtensorMap tmDOb = make_tmap_bf16(dout.data_ptr(), H * D, nrows, H * D, 64, blk);
  auto* dq = reinterpret_cast<__nv_bfloat16*>(dqkv.data_ptr());
  const float* l = lse.data_ptr<float>();
  const float* d = di.data_ptr<float>();
  dim3 grid(T / 128, H, B);
  if (D == 64) {
    auto k1 = attn_tc::dkdv_tc_kernel<64, 128>;
    constexpr int s1 = attn_tc::DkdvCfg<64, 128>::kSmem;
    C10_CUDA_CHECK(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
    k1<<<grid, attn_tc::kThreads, s1, st>>>(tmQKV128, tmQKVb, tmDOb, l, d, dq, T, H, scale_log2, scale, status_ptr());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    auto k2 = attn_tc::dq_tc_kernel<64, 128>;
    constexpr int s2 = attn_tc::DqCfg<64, 128>::kSmem;
    C10_CUDA_CHECK(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, s2));
    k2<<<grid, attn_tc::kThreads, s2, st>>>(tmQKV128, tmDO128, tmQKVb, l, d, dq, T, H, scale_log2, scale, status_ptr());
  } else {
    auto k1 = attn_tc::dkdv_tc_kernel<128, 64>;
    constexpr int s1 = attn_tc::DkdvCfg<128, 64>::kSmem;
    C10_CUDA_CHECK(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
    k1<<<grid, attn_tc::kThreads, s1, st>>>(tmQKV128, tmQKVb, tmDOb, l, d, dq, T, H, scale_log2, scale, status_ptr());
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    auto k2 = attn_tc::dq_tc_kernel<128, 64>;
    constexpr int s2 = attn_tc::DqCfg<128, 64>::kSmem;
    C10_CUDA_CHECK(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, s2));
    k2<<<grid, attn_tc::kThreads, s2, st>>>(tmQKV128, tmDO128, tmQKVb, l, d, dq, T, H, scale_log2, scale, status_ptr());
  }
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return dqkv;
}

void register_attn_tc(pybind11::module& m) {
  m.def("flash_attn_fwd_tc", &flash_attn_fwd_tc, "causal flash attention forward on tcgen05 (T % 128 == 0)");
  m.def("flash_attn_bwd_tc", &flash_attn_bwd_tc, "causal flash attention backward on tcgen05 (T % 128 == 0)");
}
