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

// The whole 128-key row `row` of P into the P tile (four quarters of 32 keys).
__device__ __forceinline__ void store_p_row(uint8_t* pbuf, int row, const float (&p)[128]) {
#pragma unroll
  for (int qtr = 0; qtr < 4; ++qtr) {
    uint8_t* atom = pbuf + (qtr >> 1) * kAtom + row * 128;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 pk;
      uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 h = __floats2bfloat162_rn(p[qtr * 32 + c * 8 + 2 * j], p[qtr * 32 + c * 8 + 2 * j + 1]);
        w[j] = *reinterpret_cast<uint32_t*>(&h);
      }
      const int c16 = (qtr & 1) * 4 + c;
      *reinterpret_cast<uint4*>(atom + ((c16 ^ (row & 7)) << 4)) = pk;
    }
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

// ------------------------------------------------------- ping-pong forward
// Two 128-query tiles per CTA (256 queries of one (batch, head)), 10 warps:
//   warp 0     TMA: Q0 and Q1 once, then K_0, V_0, K_1, V_1, ... through one
//              ring of kSlots tiles (released strictly in load order).
//   warp 1     MMA issuer. Steady-state order
//                PV0_j, S0_{j+1}, PV1_j, S1_{j+1}
//              so the tensor core works on one tile while the other tile's
//              softmax runs; S_g,j and O_g live in TMEM (columns S0 0-127,
//              S1 128-255, O0 256.., O1 256+D..), O accumulating across key
//              blocks.
//   warps 2-5  softmax of tile 0, warps 6-9 softmax of tile 1: one thread per
//              query row, all 128 key columns of S (no cross-warp exchange).
// Rescaling of O is conditional: a row keeps its reference maximum until a
// block's maximum exceeds it by more than 8 (log2 units), so probabilities
// stay below 2^8 and the TMEM read-modify-write of the row's O is rare
// after the first blocks. A commit on S_g,{j+1} also covers PV_g,j, so a
// softmax thread that holds S_g,j may rewrite its O row and the P_g tile
// without further waits. The last key block of tile 1 has no tile-0 work
// (tile 0 ends one block earlier on the causal diagonal).
template <int D>
struct PPCfg {
  static constexpr int kDAtoms = D / 64;
  static constexpr int kTile = kDAtoms * kAtom;      // 128 rows x D
  static constexpr int kSlots = (D == 64) ? 4 : 3;   // K/V ring
  static constexpr int kPTile = 2 * kAtom;           // 128 rows x 128 keys
  static constexpr int kBars = 1 + 2 * 4 + 2 + 2 + 2 + 1;
  static constexpr int kSmem = 2 * kTile + kSlots * kTile + 2 * kPTile + kBars * 8 + 16 + 1024;
  static_assert(kSmem <= 232448, "ping-pong forward: shared memory");
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    fwd_pp_kernel(const __grid_constant__ CUtensorMap tmQKV, __nv_bfloat16* __restrict__ out,
                  float* __restrict__ lse2, int T, int H, float scale_log2, int* status) {
  using C = PPCfg<D>;
  constexpr int S = C::kSlots;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                       // [2][kTile]
  uint8_t* sRing = sQ + 2 * C::kTile;       // [S][kTile]
  uint8_t* sP = sRing + S * C::kTile;       // [2][kPTile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * C::kPTile);
  uint64_t* q_full = bars;
  uint64_t* ring_full = bars + 1;           // [S] (S <= 4)
  uint64_t* ring_empty = bars + 5;          // [S]
  uint64_t* s_full = bars + 9;              // [2]
  uint64_t* p_full = bars + 11;             // [2]
  uint64_t* o_final = bars + 13;            // [2]
  uint64_t* drained = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kBars);

  const int cb = gridDim.x - 1 - blockIdx.x;  // heaviest blocks first
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb0 = 2 * cb + 1, nkb1 = 2 * cb + 2;  // key blocks of tile 0 / tile 1
  const int row0 = b * T;
  const int q0 = cb * 256;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < S; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], 1);
    }
    for (int g = 0; g < 2; ++g) {
      mbar_init(&s_full[g], 1);
      mbar_init(&p_full[g], 128);
      mbar_init(&o_final[g], 1);
    }
    mbar_init(drained, 1);
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

  if (warp == 0) {
    if (elect_one()) {
      tma_prefetch_desc(&tmQKV);
      mbar_arrive_expect_tx(q_full, 2 * C::kTile);
#pragma unroll
      for (int g = 0; g < 2; ++g)
#pragma unroll
        for (int a = 0; a < C::kDAtoms; ++a)
          tma_load_2d(sQ + g * C::kTile + a * kAtom, &tmQKV, q_full, h * 3 * D + a * 64, row0 + q0 + g * 128);
      int last = -1;
      for (int t = 0; t < 2 * nkb1; ++t) {
        const int slot = t % S, n = t / S;
        if (!mbar_wait(&ring_empty[slot], (n & 1) ^ 1, status, kTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&ring_full[slot], C::kTile);
        const int col = h * 3 * D + ((t & 1) ? 2 * D : D);
#pragma unroll
        for (int a = 0; a < C::kDAtoms; ++a)
          tma_load_2d(sRing + slot * C::kTile + a * kAtom, &tmQKV, &ring_full[slot], col + a * 64,
                      row0 + (t >> 1) * 128);
        last = t;
      }
      // no copy may still be landing when the CTA exits
      mbar_wait(q_full, 0, status, kTimeoutTmaFull);
      if (last >= 0) mbar_wait(&ring_full[last % S], (last / S) & 1, status, kTimeoutTmaFull);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idPV = idesc_bf16_f32(128, D, false, true);
      auto wait_tile = [&](int t) -> bool {
        return mbar_wait(&ring_full[t % S], (t / S) & 1, status, kTimeoutTmaFull);
      };
      auto issue_s = [&](int g, int t) {  // S_g = Q_g K^T, K in ring tile t
        const uint32_t q_addr = smem_u32(sQ + g * C::kTile), k_addr = smem_u32(sRing + (t % S) * C::kTile);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * kAtom + (kk & 3) * 32;
          umma_f16_ss(tmem + g * 128, smem_desc_sw128(q_addr + off, 16, 1024),
                      smem_desc_sw128(k_addr + off, 16, 1024), idS, kk > 0 ? 1u : 0u);
        }
        umma_commit(&s_full[g]);
      };
      auto issue_pv = [&](int g, int t, bool acc) {  // O_g (+)= P_g V, V in ring tile t
        const uint32_t p_addr = smem_u32(sP + g * C::kPTile), v_addr = smem_u32(sRing + (t % S) * C::kTile);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t poff = (kk >> 2) * kAtom + (kk & 3) * 32;
          umma_f16_ss(tmem + 256 + g * D, smem_desc_sw128(p_addr + poff, 16, 1024),
                      smem_desc_sw128(v_addr + kk * 2048, kAtom, 1024), idPV, (acc || kk > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(q_full, 0, status, kTimeoutTmaFull) && wait_tile(0);
      if (ok) {
        tc_fence_after();
        issue_s(0, 0);
        issue_s(1, 0);
        umma_commit(&ring_empty[0]);  // K_0 consumed by both tiles
      }
      for (int j = 0; j < nkb1 && ok; ++j) {
        const int tv = 2 * j + 1, tk = 2 * j + 2;  // V_j, K_{j+1}
        bool k_ready = false;
        ok = wait_tile(tv);
        if (ok && j < nkb0) {
          ok = mbar_wait(&p_full[0], j & 1, status, kTimeoutTmemFull);
          if (!ok) break;
          tc_fence_after();
          issue_pv(0, tv, j > 0);
          if (j == nkb0 - 1) umma_commit(&o_final[0]);
          if (j + 1 < nkb0) {
            ok = wait_tile(tk);
            if (!ok) break;
            k_ready = true;
            issue_s(0, tk);
          }
        }
        if (!ok) break;
        ok = mbar_wait(&p_full[1], j & 1, status, kTimeoutTmemFull);
        if (!ok) break;
        tc_fence_after();
        issue_pv(1, tv, j > 0);
        umma_commit(&ring_empty[tv % S]);  // V_j consumed by both tiles
        if (j == nkb1 - 1) umma_commit(&o_final[1]);
        if (j + 1 < nkb1) {
          if (!k_ready) ok = wait_tile(tk);
          if (!ok) break;
          issue_s(1, tk);
          umma_commit(&ring_empty[tk % S]);  // K_{j+1} consumed by both tiles
        }
      }
      umma_commit(drained);  // every MMA issued above has completed
      mbar_wait(drained, 0, status, kTimeoutTmemFull);
    }
    __syncwarp();
  } else {
    const int grp = (warp - 2) >> 2;  // the query tile of this warp
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access
    const int r = quad * 32 + lane;
    const int q = q0 + grp * 128 + r;
    const int nkb = nkb0 + grp;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t tS = tmem + grp * 128 + lane_off;
    const uint32_t tO = tmem + 256 + grp * D + lane_off;
    uint8_t* pbuf = sP + grp * C::kPTile;
    float m_ref = -INFINITY, l = 0.f;
    bool alive = true;
    for (int j = 0; j < nkb; ++j) {
      // tcgen05.ld / st are warp-collective (.sync.aligned): every branch
      // around them is decided by the whole warp
      if (!__all_sync(0xffffffff, mbar_wait(&s_full[grp], j & 1, status, kTimeoutTmemFull))) {
        alive = false;
        break;
      }
      tc_fence_after();
      // The whole 128-key row of S_j in registers: one TMEM read per block.
      float v[128];
      tmem_ld128_sync(tS, v);
      if (j == nkb - 1) {  // diagonal block (warp-uniform): keys after the query are masked
        const int kbase = j * 128;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (kbase + i > q) v[i] = -INFINITY;
      }
      float mx4[4] = {v[0], v[1], v[2], v[3]};
#pragma unroll
      for (int i = 4; i < 128; ++i) mx4[i & 3] = fmaxf(mx4[i & 3], v[i]);
      const float m_blk = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * scale_log2;
      const bool need = m_blk > m_ref + 8.f;  // this row's reference maximum moves
      const float c = need ? exp2f(m_ref - m_blk) : 1.f;
      if (need) {
        l *= c;
        m_ref = m_blk;
      }
      // P = exp2(s * scale - m_ref), packed to bf16 pairs as it is made (the
      // fp32 scores die as the packed row grows), then into the P tile.
      uint32_t pk[64];
      float rs4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 64; ++i) {
        const float p0 = exp2f(fmaf(v[2 * i], scale_log2, -m_ref));
        const float p1 = exp2f(fmaf(v[2 * i + 1], scale_log2, -m_ref));
        rs4[i & 3] += p0 + p1;
        __nv_bfloat162 h2 = __floats2bfloat162_rn(p0, p1);
        pk[i] = *reinterpret_cast<uint32_t*>(&h2);
      }
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {  // 16-byte chunk c16 of the row: keys 8*c16 .. +7
        uint8_t* atom = pbuf + (c16 >> 3) * kAtom + r * 128;
        *reinterpret_cast<uint4*>(atom + (((c16 & 7) ^ (r & 7)) << 4)) =
            make_uint4(pk[4 * c16], pk[4 * c16 + 1], pk[4 * c16 + 2], pk[4 * c16 + 3]);
      }
      const float rowsum = (rs4[0] + rs4[1]) + (rs4[2] + rs4[3]);
      // O rescale (rare once the reference maxima settle); PV_{j-1} has
      // completed (covered by the commit of S_j), PV_j is issued only after
      // this thread arrives on p_full below.
      if (j > 0 && __any_sync(0xffffffff, need)) {  // whole warp; other rows scale by 1
#pragma unroll 1
        for (int ch = 0; ch < D / 32; ++ch) {
          float o[32];
          tmem_ld32_sync(tO + ch * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= c;
          tmem_st32_sync(tO + ch * 32, o);
        }
      }
      l += rowsum;
      tc_fence_before();
      fence_proxy_async_smem();
      mbar_arrive(&p_full[grp]);
    }
    if (__all_sync(0xffffffff, alive && mbar_wait(&o_final[grp], 0, status, kTimeoutTmemFull))) {
      tc_fence_after();
      const float inv = 1.f / l;
      __nv_bfloat16* orow = out + (static_cast<size_t>(row0 + q) * H + h) * D;
#pragma unroll
      for (int ch = 0; ch < D / 32; ++ch) {
        float o[32];
        tmem_ld32_sync(tO + ch * 32, o);
        store_row_bf16(orow + ch * 32, o, inv);
      }
      lse2[(static_cast<size_t>(b) * H + h) * T + q] = m_ref + log2f(l);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ backward
// Di[b, h, t] = sum_d dO[b, t, h, d] * O[b, t, h, d]. D/8 threads per
// (b, t, h) row, one 16-byte load of each operand per thread, so a warp reads
// 32 * 16 contiguous bytes of each tensor; the partial sums meet by shuffles.
template <int D>
__global__ void bwd_rowdot_kernel(const __nv_bfloat16* __restrict__ dout, const __nv_bfloat16* __restrict__ out,
                                  float* __restrict__ di, int rows, int T, int H) {
  constexpr int kPer = D / 8;  // threads per row
  const int64_t gt = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t w = gt / kPer;
  const int part = static_cast<int>(gt % kPer);
  float acc = 0.f;
  if (w < rows) {
    const uint4 a = *reinterpret_cast<const uint4*>(dout + w * D + part * 8);
    const uint4 c = *reinterpret_cast<const uint4*>(out + w * D + part * 8);
    const __nv_bfloat162* ah = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* ch = reinterpret_cast<const __nv_bfloat162*>(&c);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 x = __bfloat1622float2(ah[j]), y = __bfloat1622float2(ch[j]);
      acc += x.x * y.x + x.y * y.y;
    }
  }
#pragma unroll
  for (int o = kPer / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffff, acc, o);
  if (w < rows && part == 0) {
    const int64_t hh = w % H, bt = w / H;
    di[(bt / T * H + hh) * T + bt % T] = acc;
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
    if (__all_sync(0xffffffff, ok && mbar_wait(fin, 0, status, kTimeoutTmemFull))) {
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
    if (__all_sync(0xffffffff, ok && mbar_wait(fin, 0, status, kTimeoutTmemFull))) {
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

// ------------------------------------------------ double-buffered backward
// The same two deterministic kernels as above, restructured so that the
// tensor core and the softmax warps overlap: S and dP of block i+1 are
// computed into the second pair of TMEM buffers while the softmax warps turn
// block i into P and dS, and the dV/dK (or dQ) MMAs of block i run one step
// later. Blocks are 64 wide (BQ / BK = 64) so that two S/dP pairs plus the
// accumulators fit in TMEM (4 x 64 + 2 x D <= 512 columns); operands stream
// through a 3-stage ring so a TMA load has a full iteration of slack.
//
// dK/dV, one CTA per (128-key block, head, batch), per 64-query block i:
//   MMA:     S^T_i = K Q_i^T, dP^T_i = V dO_i^T -> TMEM pair i % 2
//            then dV += P^T_{i-1} dO_{i-1}, dK += dS^T_{i-1} Q_{i-1}
//   softmax: P^T = exp2(S^T * scale - lse2[q]) (0 above the diagonal),
//            dS^T = P^T * (dP^T - Di[q]) -> shared tiles i % 2
template <int D>
struct DkdvDbCfg {
  static constexpr int kDAtoms = D / 64;
  static constexpr int kNS = 3;                    // Q / dO / lse / Di stages
  static constexpr int kKVTile = kDAtoms * kAtom;  // 128 keys x D
  static constexpr int kQAtom = 64 * 128;          // 64 rows x 64 columns
  static constexpr int kQTile = kDAtoms * kQAtom;  // 64 queries x D
  static constexpr int kPTile = kAtom;             // 128 keys x 64 queries
  static constexpr int kBars = 1 + 2 * kNS + 2 * 4 + 1;
  static constexpr int kSmem = 2 * kKVTile + 2 * kNS * kQTile + 4 * kPTile + 2 * kNS * 64 * 4 + kBars * 8 + 16 + 1024;
  static_assert(kSmem <= 232448, "dK/dV: shared memory");
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    dkdv_db_kernel(const __grid_constant__ CUtensorMap tmKV, const __grid_constant__ CUtensorMap tmQ,
                   const __grid_constant__ CUtensorMap tmDO, const float* __restrict__ lse2,
                   const float* __restrict__ di, __nv_bfloat16* __restrict__ dqkv, int T, int H, float scale_log2,
                   float scale, int* status) {
  using C = DkdvDbCfg<D>;
  constexpr int NS = C::kNS;
  constexpr int BQ = 64;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::kKVTile;
  uint8_t* sQ = sV + C::kKVTile;          // [NS][kQTile]
  uint8_t* sDO = sQ + NS * C::kQTile;     // [NS][kQTile]
  uint8_t* sP = sDO + NS * C::kQTile;     // [2][kPTile]
  uint8_t* sDS = sP + 2 * C::kPTile;      // [2][kPTile]
  float* sL = reinterpret_cast<float*>(sDS + 2 * C::kPTile);  // [NS][64]
  float* sDi = sL + NS * BQ;                                  // [NS][64]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDi + NS * BQ);
  uint64_t* kv_full = bars;
  uint64_t* q_full = bars + 1;          // [NS]
  uint64_t* q_empty = q_full + NS;      // [NS]
  uint64_t* s_full = q_empty + NS;      // [2]
  uint64_t* s_free = s_full + 2;        // [2]
  uint64_t* p_full = s_free + 2;        // [2]
  uint64_t* pds_free = p_full + 2;      // [2]
  uint64_t* fin = pds_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kBars);

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
    for (int i = 0; i < NS; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&pds_free[i], 1);
    }
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
  const uint32_t tS = tmem, tDP = tmem + 128, tDV = tmem + 256, tDK = tmem + 256 + D;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(kv_full, 2 * C::kKVTile);
#pragma unroll
      for (int a = 0; a < C::kDAtoms; ++a) {
        tma_load_2d(sK + a * kAtom, &tmKV, kv_full, h * 3 * D + D + a * 64, row0 + k0);
        tma_load_2d(sV + a * kAtom, &tmKV, kv_full, h * 3 * D + 2 * D + a * 64, row0 + k0);
      }
      int last = -1;
      for (int i = 0; i < nq; ++i) {
        const int st = i % NS;
        if (!mbar_wait(&q_empty[st], ((i / NS) & 1) ^ 1, status, kTimeoutSmemEmpty)) break;
        const int q0 = (qb0 + i) * BQ;
        mbar_arrive_expect_tx(&q_full[st], 2 * C::kQTile + 2 * BQ * 4);
#pragma unroll
        for (int a = 0; a < C::kDAtoms; ++a) {
          tma_load_2d(sQ + st * C::kQTile + a * C::kQAtom, &tmQ, &q_full[st], h * 3 * D + a * 64, row0 + q0);
          tma_load_2d(sDO + st * C::kQTile + a * C::kQAtom, &tmDO, &q_full[st], h * D + a * 64, row0 + q0);
        }
        bulk_load(sL + st * BQ, lrow + q0, BQ * 4, &q_full[st]);
        bulk_load(sDi + st * BQ, drow + q0, BQ * 4, &q_full[st]);
        last = i;
      }
      mbar_wait(kv_full, 0, status, kTimeoutTmaFull);
      if (last >= 0) mbar_wait(&q_full[last % NS], (last / NS) & 1, status, kTimeoutTmaFull);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BQ, false, false);
      constexpr uint32_t idG = idesc_bf16_f32(BM, D, false, true);
      bool ok = mbar_wait(kv_full, 0, status, kTimeoutTmaFull);
      const uint32_t k_addr = smem_u32(sK), v_addr = smem_u32(sV);
      for (int i = 0; i <= nq && ok; ++i) {
        if (i < nq) {
          const int st = i % NS, pb = i & 1;
          ok = mbar_wait(&q_full[st], (i / NS) & 1, status, kTimeoutTmaFull) &&
               mbar_wait(&s_free[pb], ((i >> 1) & 1) ^ 1, status, kTimeoutTmemEmpty);
          if (!ok) break;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQ + st * C::kQTile), do_addr = smem_u32(sDO + st * C::kQTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t a_off = (kk >> 2) * kAtom + (kk & 3) * 32;
            const uint32_t b_off = (kk >> 2) * C::kQAtom + (kk & 3) * 32;
            umma_f16_ss(tS + pb * 64, smem_desc_sw128(k_addr + a_off, 16, 1024),
                        smem_desc_sw128(q_addr + b_off, 16, 1024), idS, kk > 0 ? 1u : 0u);
            umma_f16_ss(tDP + pb * 64, smem_desc_sw128(v_addr + a_off, 16, 1024),
                        smem_desc_sw128(do_addr + b_off, 16, 1024), idS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[pb]);
        }
        if (i >= 1) {
          const int j = i - 1, sj = j % NS, pb = j & 1;
          ok = mbar_wait(&p_full[pb], (j >> 1) & 1, status, kTimeoutTmaFull);
          if (!ok) break;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(sQ + sj * C::kQTile), do_addr = smem_u32(sDO + sj * C::kQTile);
          const uint32_t p_addr = smem_u32(sP + pb * C::kPTile), ds_addr = smem_u32(sDS + pb * C::kPTile);
#pragma unroll
          for (int kk = 0; kk < BQ / 16; ++kk) {
            const uint32_t a_off = (kk & 3) * 32;
            const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
            umma_f16_ss(tDV, smem_desc_sw128(p_addr + a_off, 16, 1024),
                        smem_desc_sw128(do_addr + kk * 2048, C::kQAtom, 1024), idG, acc);
            umma_f16_ss(tDK, smem_desc_sw128(ds_addr + a_off, 16, 1024),
                        smem_desc_sw128(q_addr + kk * 2048, C::kQAtom, 1024), idG, acc);
          }
          umma_commit(&q_empty[sj]);
          umma_commit(&pds_free[pb]);
        }
      }
      umma_commit(fin);
      mbar_wait(fin, 0, status, kTimeoutTmemFull);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // query columns [32 half, 32 half + 32)
    const int r = quad * 32 + lane;
    const int key = k0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const int col = half * 32;
    bool ok = true;
    for (int i = 0; i < nq && ok; ++i) {
      const int st = i % NS, pb = i & 1;
      const uint32_t ph = (i >> 1) & 1;
      ok = __all_sync(0xffffffff, mbar_wait(&q_full[st], (i / NS) & 1, status, kTimeoutTmaFull) &&
                                      mbar_wait(&s_full[pb], ph, status, kTimeoutTmemFull) &&
                                      mbar_wait(&pds_free[pb], ph ^ 1, status, kTimeoutTmemFull));
      if (!ok) break;
      tc_fence_after();
      float sv[32], dp[32];
      tmem_ld32x2_sync(tS + pb * 64 + col + lane_off, tDP + pb * 64 + col + lane_off, sv, dp);
      tc_fence_before();
      mbar_arrive(&s_free[pb]);  // the TMEM pair may take block i + 2
      const int q0 = (qb0 + i) * BQ;
      const float* lq = sL + st * BQ + col;
      const float* dq = sDi + st * BQ + col;
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const float p = (key > q0 + col + t) ? 0.f : exp2f(sv[t] * scale_log2 - lq[t]);
        sv[t] = p;
        dp[t] = p * (dp[t] - dq[t]);
      }
      store_p_quarter(sP + pb * C::kPTile, r, half, sv);
      store_p_quarter(sDS + pb * C::kPTile, r, half, dp);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[pb]);
    }
    if (__all_sync(0xffffffff, ok && mbar_wait(fin, 0, status, kTimeoutTmemFull))) {
      tc_fence_after();
      __nv_bfloat16* krow = dqkv + (static_cast<size_t>(row0 + key) * H + h) * 3 * D + D + half * (D / 2);
      __nv_bfloat16* vrow = krow + D;
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        float v[32];
        tmem_ld32_sync(tDK + half * (D / 2) + c * 32 + lane_off, v);
        store_row_bf16(krow + c * 32, v, scale);
        tmem_ld32_sync(tDV + half * (D / 2) + c * 32 + lane_off, v);
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

// dQ, one CTA per (128-query block, head, batch), per 64-key block j up to the
// diagonal:
//   MMA:     S_j = Q K_j^T, dP_j = dO V_j^T -> TMEM pair j % 2
//            then dQ += dS_{j-1} K_{j-1}
//   softmax: dS = exp2(S * scale - lse2) * (dP - Di) -> shared tile j % 2
template <int D>
struct DqDbCfg {
  static constexpr int kDAtoms = D / 64;
  static constexpr int kNS = 3;                    // K / V stages
  static constexpr int kQTile = kDAtoms * kAtom;   // 128 queries x D
  static constexpr int kKAtom = 64 * 128;
  static constexpr int kKTile = kDAtoms * kKAtom;  // 64 keys x D
  static constexpr int kSTile = kAtom;             // 128 queries x 64 keys
  static constexpr int kBars = 1 + 2 * kNS + 2 * 4 + 1;
  static constexpr int kSmem = 2 * kQTile + 2 * kNS * kKTile + 2 * kSTile + kBars * 8 + 16 + 1024;
  static_assert(kSmem <= 232448, "dQ: shared memory");
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    dq_db_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmDO,
                 const __grid_constant__ CUtensorMap tmKV, const float* __restrict__ lse2, const float* __restrict__ di,
                 __nv_bfloat16* __restrict__ dqkv, int T, int H, float scale_log2, float scale, int* status) {
  using C = DqDbCfg<D>;
  constexpr int NS = C::kNS;
  constexpr int BK = 64;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sDO = sQ + C::kQTile;
  uint8_t* sK = sDO + C::kQTile;       // [NS][kKTile]
  uint8_t* sV = sK + NS * C::kKTile;   // [NS][kKTile]
  uint8_t* sDS = sV + NS * C::kKTile;  // [2][kSTile]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sDS + 2 * C::kSTile);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;         // [NS]
  uint64_t* kv_empty = kv_full + NS;    // [NS]
  uint64_t* s_full = kv_empty + NS;     // [2]
  uint64_t* s_free = s_full + 2;        // [2]
  uint64_t* p_full = s_free + 2;        // [2]
  uint64_t* ds_free = p_full + 2;       // [2]
  uint64_t* fin = ds_free + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kBars);

  const int qb = gridDim.x - 1 - blockIdx.x;  // heaviest (most key blocks) first
  const int h = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = b * T, q0 = qb * BM;
  const int nkb = (q0 + BM - 1) / BK + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < NS; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 256);
      mbar_init(&p_full[i], 256);
      mbar_init(&ds_free[i], 1);
    }
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
  const uint32_t tS = tmem, tDP = tmem + 128, tDQ = tmem + 256;

  if (warp == 0) {
    if (elect_one()) {
      mbar_arrive_expect_tx(q_full, 2 * C::kQTile);
#pragma unroll
      for (int a = 0; a < C::kDAtoms; ++a) {
        tma_load_2d(sQ + a * kAtom, &tmQ, q_full, h * 3 * D + a * 64, row0 + q0);
        tma_load_2d(sDO + a * kAtom, &tmDO, q_full, h * D + a * 64, row0 + q0);
      }
      int last = -1;
      for (int j = 0; j < nkb; ++j) {
        const int st = j % NS;
        if (!mbar_wait(&kv_empty[st], ((j / NS) & 1) ^ 1, status, kTimeoutSmemEmpty)) break;
        mbar_arrive_expect_tx(&kv_full[st], 2 * C::kKTile);
#pragma unroll
        for (int a = 0; a < C::kDAtoms; ++a) {
          tma_load_2d(sK + st * C::kKTile + a * C::kKAtom, &tmKV, &kv_full[st], h * 3 * D + D + a * 64, row0 + j * BK);
          tma_load_2d(sV + st * C::kKTile + a * C::kKAtom, &tmKV, &kv_full[st], h * 3 * D + 2 * D + a * 64,
                      row0 + j * BK);
        }
        last = j;
      }
      mbar_wait(q_full, 0, status, kTimeoutTmaFull);
      if (last >= 0) mbar_wait(&kv_full[last % NS], (last / NS) & 1, status, kTimeoutTmaFull);
    }
  } else if (warp == 1) {
    if (elect_one()) {
      constexpr uint32_t idS = idesc_bf16_f32(BM, BK, false, false);
      constexpr uint32_t idG = idesc_bf16_f32(BM, D, false, true);
      bool ok = mbar_wait(q_full, 0, status, kTimeoutTmaFull);
      const uint32_t q_addr = smem_u32(sQ), do_addr = smem_u32(sDO);
      for (int j = 0; j <= nkb && ok; ++j) {
        if (j < nkb) {
          const int st = j % NS, pb = j & 1;
          ok = mbar_wait(&kv_full[st], (j / NS) & 1, status, kTimeoutTmaFull) &&
               mbar_wait(&s_free[pb], ((j >> 1) & 1) ^ 1, status, kTimeoutTmemEmpty);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + st * C::kKTile), v_addr = smem_u32(sV + st * C::kKTile);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t a_off = (kk >> 2) * kAtom + (kk & 3) * 32;
            const uint32_t b_off = (kk >> 2) * C::kKAtom + (kk & 3) * 32;
            umma_f16_ss(tS + pb * 64, smem_desc_sw128(q_addr + a_off, 16, 1024),
                        smem_desc_sw128(k_addr + b_off, 16, 1024), idS, kk > 0 ? 1u : 0u);
            umma_f16_ss(tDP + pb * 64, smem_desc_sw128(do_addr + a_off, 16, 1024),
                        smem_desc_sw128(v_addr + b_off, 16, 1024), idS, kk > 0 ? 1u : 0u);
          }
          umma_commit(&s_full[pb]);
        }
        if (j >= 1) {
          const int jj = j - 1, sj = jj % NS, pb = jj & 1;
          ok = mbar_wait(&p_full[pb], (jj >> 1) & 1, status, kTimeoutTmaFull);
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + sj * C::kKTile), ds_addr = smem_u32(sDS + pb * C::kSTile);
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            umma_f16_ss(tDQ, smem_desc_sw128(ds_addr + (kk & 3) * 32, 16, 1024),
                        smem_desc_sw128(k_addr + kk * 2048, C::kKAtom, 1024), idG, (jj > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&kv_empty[sj]);
          umma_commit(&ds_free[pb]);
        }
      }
      umma_commit(fin);
      mbar_wait(fin, 0, status, kTimeoutTmemFull);
    }
    __syncwarp();
  } else {
    const int quad = warp & 3;
    const int half = (warp - 2) >> 2;  // key columns [32 half, 32 half + 32)
    const int r = quad * 32 + lane;
    const int q = q0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(quad * 32) << 16;
    const float lq = lse2[(static_cast<size_t>(b) * H + h) * T + q];
    const float dq_i = di[(static_cast<size_t>(b) * H + h) * T + q];
    const int col = half * 32;
    bool ok = true;
    for (int j = 0; j < nkb && ok; ++j) {
      const int pb = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      ok = __all_sync(0xffffffff, mbar_wait(&s_full[pb], ph, status, kTimeoutTmemFull) &&
                                      mbar_wait(&ds_free[pb], ph ^ 1, status, kTimeoutTmemFull));
      if (!ok) break;
      tc_fence_after();
      float sv[32], dp[32];
      tmem_ld32x2_sync(tS + pb * 64 + col + lane_off, tDP + pb * 64 + col + lane_off, sv, dp);
      tc_fence_before();
      mbar_arrive(&s_free[pb]);
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const int kk = j * BK + col + t;
        const float p = (kk > q) ? 0.f : exp2f(sv[t] * scale_log2 - lq);
        dp[t] = p * (dp[t] - dq_i);
      }
      store_p_quarter(sDS + pb * C::kSTile, r, half, dp);
      fence_proxy_async_smem();
      mbar_arrive(&p_full[pb]);
    }
    if (__all_sync(0xffffffff, ok && mbar_wait(fin, 0, status, kTimeoutTmemFull))) {
      tc_fence_after();
      __nv_bfloat16* qrow = dqkv + (static_cast<size_t>(row0 + q) * H + h) * 3 * D + half * (D / 2);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        float v[32];
        tmem_ld32_sync(tDQ + half * (D / 2) + c * 32 + lane_off, v);
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
// mode: 0 = choose, 1 = ping-pong kernel (two query tiles per CTA), 2 = one tile per CTA.
std::vector<at::Tensor> flash_attn_fwd_tc(const at::Tensor& qkv, int64_t H, int64_t D, int64_t mode) {
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
  auto st = at::cuda::getCurrentCUDAStream();
  auto* o = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  // Two query tiles per CTA when that still gives at least two CTAs per SM
  // to schedule; otherwise one tile per CTA keeps more SMs busy.
  const long pp_ctas = static_cast<long>(T / 256) * H * B;
  const bool pingpong = (mode == 1) || (mode == 0 && T % 256 == 0 && pp_ctas >= 2L * num_sms());
  if (pingpong) {
    TORCH_CHECK(T % 256 == 0, "attention (ping-pong): T must be a multiple of 256");
    dim3 grid2(T / 256, H, B);
    if (D == 64) {
      auto k = attn_tc::fwd_pp_kernel<64>;
      constexpr int smem = attn_tc::PPCfg<64>::kSmem;
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      k<<<grid2, attn_tc::kThreads, smem, st>>>(tm, o, lse.data_ptr<float>(), T, H, scale_log2, status_ptr());
    } else {
      auto k = attn_tc::fwd_pp_kernel<128>;
      constexpr int smem = attn_tc::PPCfg<128>::kSmem;
      C10_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
      k<<<grid2, attn_tc::kThreads, smem, st>>>(tm, o, lse.data_ptr<float>(), T, H, scale_log2, status_ptr());
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return {out, lse};
  }
  dim3 grid(T / 128, H, B);
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
// mode: 0 = double-buffered kernels (64-wide inner blocks), 2 = the single-buffered kernels.
at::Tensor flash_attn_bwd_tc(const at::Tensor& dout, const at::Tensor& qkv, const at::Tensor& out,
                             const at::Tensor& lse, int64_t H, int64_t D, int64_t mode) {
  TORCH_CHECK(qkv.is_cuda() && qkv.scalar_type() == at::kBFloat16 && qkv.dim() == 3 && qkv.is_contiguous(),
              "attention bwd: contiguous bf16 qkv required");
  TORCH_CHECK(D == 64 || D == 128, "attention: head_dim must be 64 or 128");
  TORCH_CHECK(qkv.size(2) == 3 * H * D && qkv.size(1) % 128 == 0, "attention bwd (tc): shapes");
  TORCH_CHECK(dout.is_contiguous() && out.is_contiguous() && dout.sizes() == out.sizes(), "attention bwd: dout/out");
  TORCH_CHECK(lse.is_contiguous() && lse.scalar_type() == at::kFloat, "attention bwd: lse");
  TORCH_CHECK(out.dim() == 3 && out.size(0) == qkv.size(0) && out.size(1) == qkv.size(1) && out.size(2) == H * D &&
                  out.scalar_type() == at::kBFloat16 && dout.scalar_type() == at::kBFloat16,
              "attention bwd: bf16 out / dout [B, T, H * D] required");
  TORCH_CHECK(lse.numel() == qkv.size(0) * H * qkv.size(1), "attention bwd: lse [B, H, T] required");
  c10::cuda::CUDAGuard g(qkv.device());
  const int B = qkv.size(0), T = qkv.size(1);
  at::Tensor dqkv = at::empty_like(qkv);
  at::Tensor di = at::empty({B, H, T}, qkv.options().dtype(at::kFloat));
  const double sc = 1.0 / std::sqrt(static_cast<double>(D));
  const float scale = static_cast<float>(sc), scale_log2 = static_cast<float>(sc * 1.4426950408889634);
  auto st = at::cuda::getCurrentCUDAStream();
  const int rows = B * T * static_cast<int>(H);
  {
    const auto* dop = reinterpret_cast<const __nv_bfloat16*>(dout.data_ptr());
    const auto* op = reinterpret_cast<const __nv_bfloat16*>(out.data_ptr());
    const int64_t threads = static_cast<int64_t>(rows) * (D / 8);
    const int blocks = static_cast<int>((threads + 255) / 256);
    if (D == 64)
      attn_tc::bwd_rowdot_kernel<64><<<blocks, 256, 0, st>>>(dop, op, di.data_ptr<float>(), rows, T, H);
    else
      attn_tc::bwd_rowdot_kernel<128><<<blocks, 256, 0, st>>>(dop, op, di.data_ptr<float>(), rows, T, H);
  }
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
  if (mode != 2) {  // double-buffered kernels (64-wide inner blocks)
    CUtensorMap tmQKV64 = make_tmap_bf16(qkv.data_ptr(), 3 * H * D, nrows, 3 * H * D, 64, 64);
    CUtensorMap tmDO64 = make_tmap_bf16(dout.data_ptr(), H * D, nrows, H * D, 64, 64);
    if (D == 64) {
      auto k1 = attn_tc::dkdv_db_kernel<64>;
      constexpr int s1 = attn_tc::DkdvDbCfg<64>::kSmem;
      C10_CUDA_CHECK(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
      k1<<<grid, attn_tc::kThreads, s1, st>>>(tmQKV128, tmQKV64, tmDO64, l, d, dq, T, H, scale_log2, scale, status_ptr());
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      auto k2 = attn_tc::dq_db_kernel<64>;
      constexpr int s2 = attn_tc::DqDbCfg<64>::kSmem;
      C10_CUDA_CHECK(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, s2));
      k2<<<grid, attn_tc::kThreads, s2, st>>>(tmQKV128, tmDO128, tmQKV64, l, d, dq, T, H, scale_log2, scale, status_ptr());
    } else {
      auto k1 = attn_tc::dkdv_db_kernel<128>;
      constexpr int s1 = attn_tc::DkdvDbCfg<128>::kSmem;
      C10_CUDA_CHECK(cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, s1));
      k1<<<grid, attn_tc::kThreads, s1, st>>>(tmQKV128, tmQKV64, tmDO64, l, d, dq, T, H, scale_log2, scale, status_ptr());
      C10_CUDA_KERNEL_LAUNCH_CHECK();
      auto k2 = attn_tc::dq_db_kernel<128>;
      constexpr int s2 = attn_tc::DqDbCfg<128>::kSmem;
      C10_CUDA_CHECK(cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, s2));
      k2<<<grid, attn_tc::kThreads, s2, st>>>(tmQKV128, tmDO128, tmQKV64, l, d, dq, T, H, scale_log2, scale, status_ptr());
    }
    C10_CUDA_KERNEL_LAUNCH_CHECK();
    return dqkv;
  }
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
  m.def("flash_attn_fwd_tc", &flash_attn_fwd_tc, "causal flash attention forward on tcgen05 (T % 128 == 0)",
        pybind11::arg("qkv"), pybind11::arg("H"), pybind11::arg("D"), pybind11::arg("mode") = 0);
  m.def("flash_attn_bwd_tc", &flash_attn_bwd_tc, "causal flash attention backward on tcgen05 (T % 128 == 0)",
        pybind11::arg("dout"), pybind11::arg("qkv"), pybind11::arg("out"), pybind11::arg("lse"), pybind11::arg("H"),
        pybind11::arg("D"), pybind11::arg("mode") = 0);
}
