// Persistent warp-specialised bf16 GEMM on the sm_100a tensor cores.
//
//   C[M, N] = A[M, K] . B[N, K]^T   (fp32 accumulate in TMEM, fused epilogue)
//
// A and B are each either K-major ("row-major [rows][K]") or MN-major
// ("[K][rows]"), which covers every product a linear layer needs:
//   forward  y  = x W^T : A = x  (K-major), B = W  (K-major)
//   backward dx = dy W  : A = dy (K-major), B = W  (MN-major)
//   backward dW = dy^T x: A = dy (MN-major), B = x (MN-major)
//
// Structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128B-swizzled tiles of A and B into a ring of
//               smem stages, completion on per-stage "full" mbarriers.
//   warp 1      TMEM allocator + MMA issuer: one elected thread issues
//               tcgen05.mma (M=128, N=BN, K=16) x 4 per 64-wide K stage and
//               tcgen05.commit's the stage back to the producer; after a
//               tile's last stage it commits the accumulator to the epilogue.
//   warps 2..5  epilogue: each warp owns 32 TMEM lanes (= 32 output rows).
//               Per 64-column chunk it reads the accumulator with
//               tcgen05.ld, applies the fused epilogue, writes the bf16
//               chunk into a 128B-swizzled 32x64 staging tile in shared
//               memory and one lane issues a TMA bulk-tensor store (two
//               staging tiles per warp, so a store drains while the next
//               chunk is computed). fp32 epilogues (split-K partials,
//               accumulation) store straight from registers.
// The accumulator is double-buffered in TMEM (2 x BN fp32 columns), so the
// epilogue of tile i overlaps the MMAs of tile i+1.
//
// Split-K: a work unit is (tile, k-split). With splits > 1 the epilogue
// writes fp32 partial tiles to a workspace and a separate kernel sums them in
// split order (deterministic, no atomics).
#pragma once

#include "ptx.cuh"

namespace dst {

enum Epilogue : int {
  kEpiStore = 0,      // C = acc
  kEpiBias = 1,       // C = acc + bias[n]
  kEpiBiasGelu = 2,   // aux_out = acc + bias (pre-activation), C = gelu(aux_out)
  kEpiBiasResid = 3,  // C = acc + bias[n] + aux[m, n]
  kEpiDGelu = 4,      // C = acc * gelu'(aux[m, n])
  kEpiPartialF32 = 5, // ws[split][m][n] = acc (fp32)
  kEpiCEStats = 6,    // C = bf16(acc); per (row, tile): max / sum exp; target logit
  kEpiAccumF32 = 7,   // accf32[m, n] += acc  (fp32 output, e.g. grad accumulation)
};

struct GemmParams {
  int M, N, K;
  int splits;             // K splits (>= 1)
  int k_blocks_per_split; // in units of 64
  __nv_bfloat16* out;     // [M, ldo]
  int ldo;
  const __nv_bfloat16* bias;  // [N] or null
  const __nv_bfloat16* aux;   // [M, ld_aux] (residual / pre-activation)
  int ld_aux;
  __nv_bfloat16* aux_out;     // [M, ldo] (pre-activation output)
  float* ws;                  // split-K workspace [splits, M, N] / fp32 accumulation target [M, N]
  // CE statistics epilogue
  float* ce_max;        // [M, n_tiles]
  float* ce_sum;        // [M, n_tiles]
  float* ce_tgt;        // [M]
  const int64_t* ce_targets;  // [M]
  int ce_col0;          // global vocab id of local column 0
  int ce_valid_cols;    // local columns < this are real vocab entries
  int* status;
};

// ---------------------------------------------------------------- TP peers
// Tensor parallelism with sequence sharding: the token dimension (rows of
// [B*T, C] activations) is split so that rank r holds, for every batch row b,
// tokens [r*Tl, (r+1)*Tl) with Tl = T / tp, stored as local rows b*Tl + t.
//
// Gather mode (AG + GEMM): the operand whose token dimension is sharded is
// TMA-loaded tile by tile directly from the owning rank's buffer (a plain,
// single-CTA TMA load from peer memory over NVLink). For a K-major operand
// the tokens are its rows; for an MN-major operand they are the K dimension.
// Scatter mode (GEMM + reduce-scatter): each 32-row chunk of the output is
// TMA-stored straight into the owning rank's receive slot [src rank][local
// row][N] over NVLink while later tiles are still being computed; a separate
// reduction sums the slots (tp_reduce in tp.cu).
//
// Flags (per channel, kinds x 8 ranks, epochs identical on every rank):
enum PeerFlag : int {
  kGReady = 0,     // my gathered-operand shard is complete
  kGConsumed = 1,  // I have finished reading every peer's shard
  kSWritten = 2,   // all my scatter stores into your receive slots are complete
  kSConsumed = 3,  // I have finished reading my receive slots
  kAGWritten = 4,  // (all-reduce form) my reduced rows are in every rank's output
};
constexpr int kMaxPeers = 8;

struct PeerArgs {
  CUtensorMap gather[kMaxPeers];   // each rank's gathered operand (same shape as the local one)
  CUtensorMap scatter[kMaxPeers];  // each rank's receive buffer [tp * rows_local, N]
  uint32_t* flags[kMaxPeers];      // each rank's flag words for this channel [kinds][8]
  unsigned int* done_ctas;         // this rank's CTA completion counter (self-resetting)
  unsigned int* claim;             // gather mode: next copy chunk to claim (reset by the last CTA)
  int tp, rank;
  int seq;         // T (tokens per batch row of the gathered / scattered tensor)
  int seq_local;   // T / tp
  int rows_local;  // B * T / tp (rows of one receive slot)
  uint32_t epoch;
  // Gather mode with a K-major operand (rows gathered): remote shards are
  // copied ONCE into a local gather buffer by a copier warp in every CTA, so
  // each remote byte crosses NVLink a single time; tiles of this rank's own
  // shard are computed first while the copies are in flight.
  const __nv_bfloat16* shard[kMaxPeers];  // each rank's shard (rows_local x K)
  int shard_ld;                            // row stride (elements) of shards and gather buffer
  __nv_bfloat16* gath;                     // local gather buffer [tokens, K]
  unsigned int* arrive;                    // per 128-row block: copied 64-column chunks (monotonic)
  int kchunks;                             // 64-column chunks per row block
  CUtensorMap gath_map;                    // TMA map over gath (box 64 x 128)
};

// Row-block processing order of the gathered GEMM: this rank's own shard
// first, then the shards of rank+1, rank+2, ... (the order their copies are
// issued in). Logical index i -> global 128-row block.
__device__ __forceinline__ int gather_mblock(const PeerArgs& pa, int i, int num_m) {
  const int per_seg = pa.seq_local / 128;     // row blocks per (batch row, rank)
  const int seg_blocks = pa.seq / 128;        // row blocks per batch row
  const int per_src = (num_m / seg_blocks) * per_seg;
  const int s = i / per_src, j = i - s * per_src;
  const int src = (pa.rank + s) % pa.tp;
  const int b = j / per_seg, tb = j - b * per_seg;
  return b * seg_blocks + src * per_seg + tb;
}

// Output tile index -> (row block, column block). Plain GEMMs walk rows
// fastest. The row-gathered GEMM goes source by source (all of this rank's
// own tiles, over every column block, before any tile that needs a copied
// block), rows fastest inside a source.
template <bool ROW_GATHER>
__device__ __forceinline__ void tile_coords(const PeerArgs& pa, int t, int num_m, int num_n, int& m_blk, int& n_blk) {
  if (ROW_GATHER) {
    const int per_src = num_m / pa.tp;
    const int s = t / (per_src * num_n), r = t - s * per_src * num_n;
    n_blk = r / per_src;
    m_blk = gather_mblock(pa, s * per_src + (r - n_blk * per_src), num_m);
  } else {
    m_blk = t % num_m;
    n_blk = t / num_m;
  }
}

// Global token index -> (owning rank, row in the owner's local shard).
__device__ __forceinline__ void token_owner(const PeerArgs& pa, int tok, int& src, int& local) {
  const int b = tok / pa.seq, t = tok - b * pa.seq;
  src = t / pa.seq_local;
  local = b * pa.seq_local + (t - src * pa.seq_local);
}

__device__ __forceinline__ void peer_publish(const PeerArgs& pa, int kind, uint32_t epoch) {
  __threadfence_system();
  for (int p = 0; p < pa.tp; ++p) flag_store_release(pa.flags[p] + kind * kMaxPeers + pa.rank, epoch);
}

__device__ __forceinline__ bool peer_wait_all(const PeerArgs& pa, int kind, uint32_t epoch, int* status) {
  for (int p = 0; p < pa.tp; ++p)
    if (!flag_wait_geq(pa.flags[pa.rank] + kind * kMaxPeers + p, epoch, status, kTimeoutPeer)) return false;
  return true;
}

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kGemmThreads = 224;  // producer, MMA, 4 epilogue warps, copier (gather mode)
constexpr int kEpiChunk = 64;                        // columns per epilogue chunk
constexpr int kStageTileBytes = 32 * kEpiChunk * 2;  // one 32x64 bf16 staging tile

// RG: the row-gather (AG + GEMM) form, whose copier warp stages remote row
// blocks through two 128 x 64 shared-memory tiles (one ring stage fewer).
template <int BN, bool RG = false>
struct GemmCfg {
  static constexpr int kStageA = kBM * kBK * 2;
  static constexpr int kStageB = BN * kBK * 2;
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kStages = (BN == 256) ? (RG ? 3 : 4) : (RG ? 4 : 6);
  static constexpr int kTmemCols = 2 * BN;  // power of two: 256 or 512
  static constexpr int kOutStaging = 4 * 2 * kStageTileBytes;  // 4 warps x 2 tiles
  static constexpr int kBiasStaging = 4 * kEpiChunk * 4;       // 4 warps x 64 fp32
  static constexpr int kCopyTile = kBM * 64 * 2;               // one 128-row x 64-column chunk
  static constexpr int kCopyBytes = RG ? 1024 + 2 * kCopyTile : 0;  // aligned, double-buffered
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kOutStaging + kBiasStaging + kCopyBytes + 1024 /*align*/ + 256 /*barriers*/;
  static_assert(kSmemBytes <= 232448, "GEMM: shared memory");
};

__device__ __forceinline__ void load_bf16x32(const __nv_bfloat16* src, float (&v)[32], int valid) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    if (q * 8 < valid) {
      uint4 pk = *reinterpret_cast<const uint4*>(src + q * 8);
      const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&pk);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float2 f = __bfloat1622float2(h[j]);
        v[q * 8 + 2 * j] = f.x;
        v[q * 8 + 2 * j + 1] = f.y;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[q * 8 + j] = 0.f;
    }
  }
}

// Write 32 fp32 values (columns [half*32, half*32+32) of this lane's row) as
// bf16 into a 128B-swizzled 32x64 staging tile (row = lane).
__device__ __forceinline__ void stage_bf16x32(uint8_t* tile, int lane, int half, const float (&v)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 pk;
    uint32_t* w = reinterpret_cast<uint32_t*>(&pk);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 h = __floats2bfloat162_rn(v[q * 8 + 2 * j], v[q * 8 + 2 * j + 1]);
      w[j] = *reinterpret_cast<uint32_t*>(&h);
    }
    const int chunk16 = half * 4 + q;  // 16-byte chunk within the 128-byte row
    *reinterpret_cast<uint4*>(tile + lane * 128 + ((chunk16 ^ (lane & 7)) << 4)) = pk;
  }
}

// GATHER: 0 none, 1 operand A gathered over TP, 2 operand B gathered.
// SCATTER: bf16 output chunks go to the owning rank's receive slot.
template <int BN, bool A_MN, bool B_MN, int EPI, int GATHER = 0, bool SCATTER = false>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmOut, const __grid_constant__ CUtensorMap tmAux,
                     GemmParams p, const __grid_constant__ PeerArgs pa) {
  constexpr bool kRowGather = (GATHER == 1 && !A_MN);  // rows of A gathered via the copier
  using Cfg = GemmCfg<BN, kRowGather>;
  constexpr int S = Cfg::kStages;
  static_assert(!(SCATTER && (EPI == kEpiPartialF32 || EPI == kEpiAccumF32 || EPI == kEpiBiasGelu ||
                              EPI == kEpiCEStats)),
                "scatter mode takes a plain bf16 output");
  constexpr bool kF32Out = (EPI == kEpiPartialF32 || EPI == kEpiAccumF32);
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte alignment for the 128B swizzle atoms.
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stage_base = smem;
  uint8_t* out_stage = smem + S * Cfg::kStageBytes;  // [4 warps][2][32x64 bf16], 1024-aligned
  float* bias_stage = reinterpret_cast<float*>(out_stage + Cfg::kOutStaging);  // [4 warps][64]
  // row gather: two 1024-aligned copy tiles after the bias staging
  uint8_t* copy_base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(out_stage + Cfg::kOutStaging + Cfg::kBiasStaging) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(out_stage + Cfg::kOutStaging + Cfg::kBiasStaging + Cfg::kCopyBytes);
  uint64_t* full_bar = bars;               // [S]
  uint64_t* empty_bar = bars + S;          // [S]
  uint64_t* tfull_bar = bars + 2 * S;      // [2]
  uint64_t* tempty_bar = bars + 2 * S + 2; // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * S + 4);
  uint64_t* copy_bar = bars + 2 * S + 5;   // [2] (row gather)

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int num_m = (p.M + kBM - 1) / kBM;
  const int num_n = (p.N + BN - 1) / BN;
  const int num_tiles = num_m * num_n;
  const int num_units = num_tiles * p.splits;
  const int k_blocks_total = (p.K + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full_bar[i], 1);
      mbar_init(&empty_bar[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&tfull_bar[i], 1);
      mbar_init(&tempty_bar[i], 128);
      if (kRowGather) mbar_init(&copy_bar[i], 1);
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Gather mode: this rank's shard was completed by earlier kernels on the
  // stream; announce it before anyone waits for a peer's.
  if (GATHER != 0 && blockIdx.x == 0 && threadIdx.x == 0) peer_publish(pa, kGReady, pa.epoch);

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t ready_mask = 0;  // gather sources whose shard is known ready
      auto source = [&](int tok, int& local) -> const CUtensorMap* {
        int src;
        token_owner(pa, tok, src, local);
        if (!(ready_mask & (1u << src))) {
          if (!flag_wait_geq(pa.flags[pa.rank] + kGReady * kMaxPeers + src, pa.epoch, p.status, kTimeoutPeer))
            return nullptr;
          ready_mask |= 1u << src;
        }
        return &pa.gather[src];
      };
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
        const int tile = u % num_tiles;
        const int split = u / num_tiles;
        int mb_, nb_;
        tile_coords<kRowGather>(pa, tile, num_m, num_n, mb_, nb_);
        const int m0 = mb_ * kBM;
        const int n0 = nb_ * BN;
        const int kb0 = split * p.k_blocks_per_split;
        const int kb1 = min(kb0 + p.k_blocks_per_split, k_blocks_total);
        if (EPI == kEpiBiasResid || EPI == kEpiDGelu) {
          // The epilogue reads this tile's auxiliary operand (residual /
          // pre-activation) a mainloop later: bring it into L2 now.
#pragma unroll 1
          for (int r = 0; r < kBM; r += 32)
#pragma unroll 1
            for (int c = 0; c < BN; c += kEpiChunk) tma_prefetch_l2_2d(&tmAux, n0 + c, m0 + r);
        }
        const CUtensorMap* rowA = &tmA;
        int row_a = m0;
        if (kRowGather) {
          // Own rows straight from the local shard; remote rows from the
          // gather buffer once the copier warps have landed all of them.
          int src, local;
          token_owner(pa, m0, src, local);
          if (src == pa.rank) {
            rowA = &pa.gather[pa.rank];
            row_a = local;
          } else {
            const unsigned int need = pa.epoch * static_cast<unsigned int>(pa.kchunks);
            if (!flag_wait_geq(pa.arrive + m0 / kBM, need, p.status, kTimeoutPeer)) {
              ok = false;
              break;
            }
            fence_proxy_async_global();
            rowA = &pa.gath_map;
          }
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, p.status, kTimeoutSmemEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = stage_base + stage * Cfg::kStageBytes;
          uint8_t* sb = sa + Cfg::kStageA;
          const int k0 = kb * kBK;
          // Operand sources: local tensor maps, or (gather mode) the owning
          // rank's shard for the token coordinate of the gathered operand.
          const CUtensorMap* mapA = &tmA;
          const CUtensorMap* mapB = &tmB;
          int a_m = m0, a_k = k0, b_n = n0, b_k = k0;
          if (kRowGather) {
            mapA = rowA;
            a_m = row_a;
          } else if (GATHER == 1) {
            mapA = A_MN ? source(k0, a_k) : source(m0, a_m);
            if (mapA == nullptr) {
              ok = false;
              break;
            }
          } else if (GATHER == 2) {
            mapB = B_MN ? source(k0, b_k) : source(n0, b_n);
            if (mapB == nullptr) {
              ok = false;
              break;
            }
          }
          mbar_arrive_expect_tx(&full_bar[stage], Cfg::kStageBytes);
          if (!A_MN) {
            tma_load_2d(sa, mapA, &full_bar[stage], a_k, a_m);
          } else {
#pragma unroll
            for (int j = 0; j < kBM / 64; ++j) tma_load_2d(sa + j * 64 * kBK * 2, mapA, &full_bar[stage], a_m + 64 * j, a_k);
          }
          if (!B_MN) {
            tma_load_2d(sb, mapB, &full_bar[stage], b_k, b_n);
          } else {
#pragma unroll
            for (int j = 0; j < BN / 64; ++j) tma_load_2d(sb + j * 64 * kBK * 2, mapB, &full_bar[stage], b_n + 64 * j, b_k);
          }
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN, A_MN, B_MN);
    if (elect_one()) {
      int stage = 0;
      uint32_t phase = 0;
      int iter = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++iter) {
        const int split = u / num_tiles;
        const int kb0 = split * p.k_blocks_per_split;
        const int kb1 = min(kb0 + p.k_blocks_per_split, k_blocks_total);
        const int acc = iter & 1;
        const uint32_t acc_phase = (iter >> 1) & 1;
        if (!mbar_wait(&tempty_bar[acc], acc_phase ^ 1, p.status, kTimeoutTmemEmpty)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, p.status, kTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(stage_base + stage * Cfg::kStageBytes);
          const uint32_t sb = sa + Cfg::kStageA;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            uint64_t da, db;
            if (!A_MN)
              da = smem_desc_sw128(sa + kk * 32, 16, 1024);
            else
              da = smem_desc_sw128(sa + kk * 2048, 64 * kBK * 2, 1024);
            if (!B_MN)
              db = smem_desc_sw128(sb + kk * 32, 16, 1024);
            else
              db = smem_desc_sw128(sb + kk * 2048, 64 * kBK * 2, 1024);
            umma_f16_ss(d_tmem, da, db, idesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&empty_bar[stage]);
          if (++stage == S) {
            stage = 0;
            phase ^= 1;
          }
        }
        umma_commit(&tfull_bar[acc]);
      }
    }
    __syncwarp();
  } else if (warp >= 6) {
    // ------------------------------------------------------------ copier
    // Gather mode: pull every remote row block of A into the local gather
    // buffer once, in processing order (the copier threads of all CTAs claim
    // the next 128-row x 64-column chunk from a launch-wide counter, so the
    // copies progress with whichever CTAs are resident: the kernel never
    // needs all of its CTAs on the GPU at once, e.g. next to NCCL kernels
    // that occupy some SMs). Each landed chunk bumps its block's counter.
    if (kRowGather && elect_one()) {
      // One thread drives bulk tensor copies through two shared-memory tiles:
      // while chunk i is loaded (a plain TMA load from the owner's shard, no
      // multicast), chunk i-1 is stored into the local gather buffer; a
      // chunk's arrival is counted once its store has completed.
      const int per_src = num_m / pa.tp;
      const int total = (pa.tp - 1) * per_src * pa.kchunks;
      uint32_t ready = 0;
      uint32_t phase[2] = {0u, 0u};
      int ld_mb = -1, ld_kc = 0;  // chunk whose load was issued last iteration (tile (i-1) & 1)
      int st_mb = -1;             // chunk whose store was committed last iteration
      bool ok = true, claiming = true;
      for (int i = 0;; ++i) {
        const int buf = i & 1;
        // A: claim the next chunk and load it into tile `buf`
        int new_mb = -1, new_kc = 0;
        if (claiming && ok) {
          const int c = static_cast<int>(atomicAdd(pa.claim, 1u));
          if (c < total) {
            new_mb = gather_mblock(pa, per_src + c / pa.kchunks, num_m);  // skip own blocks
            new_kc = c % pa.kchunks;
            int src, local;
            token_owner(pa, new_mb * kBM, src, local);
            if (!(ready & (1u << src))) {
              if (flag_wait_geq(pa.flags[pa.rank] + kGReady * kMaxPeers + src, pa.epoch, p.status, kTimeoutPeer))
                ready |= 1u << src;
              else
                ok = false;
            }
            if (ok) {
              bulk_wait_read<0>();  // the store that last used this tile (committed last iteration) has read it
              mbar_arrive_expect_tx(&copy_bar[buf], Cfg::kCopyTile);
              tma_load_2d(copy_base + buf * Cfg::kCopyTile, &pa.gather[src], &copy_bar[buf], new_kc * 64, local);
            } else {
              new_mb = -1;
            }
          } else {
            claiming = false;
          }
        }
        // B: the previous chunk's load has landed: store it into the gather buffer
        bool committed = false;
        if (ld_mb >= 0) {
          const int pb = buf ^ 1;
          if (mbar_wait(&copy_bar[pb], phase[pb], p.status, kTimeoutTmaFull)) {
            phase[pb] ^= 1u;
            tma_store_2d(&pa.gath_map, copy_base + pb * Cfg::kCopyTile, ld_kc * 64, ld_mb * kBM);
            bulk_commit();
            committed = true;
          } else {
            ok = false;
          }
        }
        // C: the store committed last iteration has completed: count its chunk
        if (st_mb >= 0) {
          if (committed)
            bulk_wait_group<1>();
          else
            bulk_wait_group<0>();
          fence_proxy_async_global();
          __threadfence();
          atomicAdd(pa.arrive + st_mb, 1u);
        }
        st_mb = committed ? ld_mb : -1;
        ld_mb = new_mb;
        ld_kc = new_kc;
        if (ld_mb < 0 && st_mb < 0) break;  // nothing claimed, loading or storing
      }
      bulk_wait_group<0>();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = quad * 32 + lane;
    uint8_t* my_stage = out_stage + (warp - 2) * 2 * kStageTileBytes;
    float* my_bias = bias_stage + (warp - 2) * kEpiChunk;
    int iter = 0;
    int chunk_count = 0;
    uint32_t scatter_ok = 0;  // owners whose receive slot is known drained (lane 0)
    for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++iter) {
      const int tile = u % num_tiles;
      const int split = u / num_tiles;
      int m_blk, n_blk;
      tile_coords<kRowGather>(pa, tile, num_m, num_n, m_blk, n_blk);
      const int m0 = m_blk * kBM;
      const int n0 = n_blk * BN;
      const int acc = iter & 1;
      const uint32_t acc_phase = (iter >> 1) & 1;
      if (!mbar_wait(&tfull_bar[acc], acc_phase, p.status, kTimeoutTmemFull)) break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const bool row_ok = row < p.M;
      float ce_m = -INFINITY, ce_s = 0.f;
      int64_t tgt = -1;
      if (EPI == kEpiCEStats && row_ok) tgt = p.ce_targets[row] - p.ce_col0;
#pragma unroll 1
      for (int c = 0; c < BN / kEpiChunk; ++c) {
        const int col0 = n0 + c * kEpiChunk;
        if (col0 >= p.N) break;  // uniform across the CTA
        if ((EPI == kEpiBias || EPI == kEpiBiasGelu || EPI == kEpiBiasResid) && p.bias != nullptr) {
          const int bc = col0 + 2 * lane;
          float2 bv = make_float2(0.f, 0.f);
          if (bc < p.N) bv = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p.bias + bc));
          __syncwarp();
          my_bias[2 * lane] = bv.x;
          my_bias[2 * lane + 1] = bv.y;
          __syncwarp();
        }
        // Auxiliary operand (residual / pre-activation) of this 64-column
        // chunk: issue the row's loads now so they overlap the TMEM reads.
        uint4 auxv[8];
        if (EPI == kEpiBiasResid || EPI == kEpiDGelu) {
          const int nvalid = max(0, min(kEpiChunk, p.N - col0));
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            auxv[q] = make_uint4(0u, 0u, 0u, 0u);
            if (row_ok && q * 8 < nvalid)
              auxv[q] = *reinterpret_cast<const uint4*>(p.aux + static_cast<size_t>(row) * p.ld_aux + col0 + q * 8);
          }
        }
        uint8_t* tile_a = my_stage + (chunk_count & 1) * kStageTileBytes;
        uint8_t* tile_b = my_stage + ((chunk_count & 1) ^ 1) * kStageTileBytes;
        if (!kF32Out) {
          // The staging tile(s) about to be written must have been read by
          // the TMA stores issued for earlier chunks.
          if (lane == 0) {
            if (EPI == kEpiBiasGelu)
              bulk_wait_read<0>();
            else
              bulk_wait_read<1>();
          }
          __syncwarp();
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          const int col = col0 + half * 32;
          float v[32];
          tmem_ld32(tmem_base + (static_cast<uint32_t>(quad * 32) << 16) + acc * BN + c * kEpiChunk + half * 32, v);
          tmem_wait_ld();
          const int valid = max(0, min(32, p.N - col));
          if (EPI == kEpiPartialF32 || EPI == kEpiAccumF32) {
            if (!row_ok || valid == 0) continue;
            float* dst = (EPI == kEpiPartialF32 ? p.ws + (static_cast<size_t>(split) * p.M + row) * p.N
                                                : p.ws + static_cast<size_t>(row) * p.N) +
                         col;
#pragma unroll
            for (int q = 0; q < 8; ++q)
              if (q * 4 < valid) {
                float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
                if (EPI == kEpiAccumF32) {
                  const float4 old = *reinterpret_cast<float4*>(dst + q * 4);
                  o.x += old.x;
                  o.y += old.y;
                  o.z += old.z;
                  o.w += old.w;
                }
                *reinterpret_cast<float4*>(dst + q * 4) = o;
              }
            continue;
          }
          if (EPI == kEpiBias || EPI == kEpiBiasGelu || EPI == kEpiBiasResid) {
            if (p.bias != nullptr) {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] += my_bias[half * 32 + i];
            }
          }
          if (EPI == kEpiBiasGelu) {
            stage_bf16x32(tile_b, lane, half, v);  // pre-activation
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              // gelu of the bf16-rounded pre-activation, so forward and the
              // dGELU backward see the same input.
              const float x = __bfloat162float(__float2bfloat16_rn(v[i]));
              v[i] = gelu_tanh(x);
            }
          } else if (EPI == kEpiBiasResid || EPI == kEpiDGelu) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&auxv[half * 4 + q]);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float2 f = __bfloat1622float2(h2[j]);
                if (EPI == kEpiBiasResid) {
                  v[q * 8 + 2 * j] += f.x;
                  v[q * 8 + 2 * j + 1] += f.y;
                } else {
                  v[q * 8 + 2 * j] *= gelu_tanh_grad(f.x);
                  v[q * 8 + 2 * j + 1] *= gelu_tanh_grad(f.y);
                }
              }
            }
          } else if (EPI == kEpiCEStats) {
            float cm = -INFINITY;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              v[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
              const int lc = col + i;  // local column
              if (lc < p.ce_valid_cols) cm = fmaxf(cm, v[i]);
              if (row_ok && lc == tgt) p.ce_tgt[row] = v[i];
            }
            if (cm > -INFINITY) {
              const float nm = fmaxf(ce_m, cm);
              float s = 0.f;
#pragma unroll
              for (int i = 0; i < 32; ++i)
                if (col + i < p.ce_valid_cols) s += __expf(v[i] - nm);
              ce_s = ce_s * __expf(ce_m - nm) + s;
              ce_m = nm;
            }
          }
          stage_bf16x32(tile_a, lane, half, v);
        }
        if (!kF32Out) {
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) {
            if (SCATTER) {
              // This 32-row chunk belongs to one rank's sequence shard: store it
              // into that rank's receive slot for this source rank, once the
              // owner has drained the slot's previous contents.
              int owner, local;
              token_owner(pa, m0 + quad * 32, owner, local);
              if (!(scatter_ok & (1u << owner))) {
                if (flag_wait_geq(pa.flags[pa.rank] + kSConsumed * kMaxPeers + owner, pa.epoch - 1, p.status,
                                  kTimeoutPeer))
                  scatter_ok |= 1u << owner;
              }
              if (scatter_ok & (1u << owner))
                tma_store_2d(&pa.scatter[owner], tile_a, col0, pa.rank * pa.rows_local + local);
            } else {
              tma_store_2d(&tmOut, tile_a, col0, m0 + quad * 32);
              if (EPI == kEpiBiasGelu) tma_store_2d(&tmAux, tile_b, col0, m0 + quad * 32);
            }
            bulk_commit();
          }
        }
        ++chunk_count;
      }
      if (EPI == kEpiCEStats && row_ok) {
        const int n_tiles = num_n;
        p.ce_max[static_cast<size_t>(row) * n_tiles + n_blk] = ce_m;
        p.ce_sum[static_cast<size_t>(row) * n_tiles + n_blk] = ce_s;
      }
      tc_fence_before();
      mbar_arrive(&tempty_bar[acc]);
    }
    if (!kF32Out && lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
  if ((GATHER != 0 || SCATTER) && threadIdx.x == 0) {
    // Every CTA's loads have been consumed by its MMAs and its stores have
    // completed; the last CTA to get here speaks for the whole launch.
    __threadfence_system();
    const unsigned int prev = atomicAdd(pa.done_ctas, 1u);
    if (prev == gridDim.x - 1) {
      atomicExch(pa.done_ctas, 0u);
      if (kRowGather) atomicExch(pa.claim, 0u);  // every copier warp has left its loop
      if (SCATTER) peer_publish(pa, kSWritten, pa.epoch);
      if (GATHER != 0) {
        // Peers may overwrite their shards only after everyone has read them.
        peer_publish(pa, kGConsumed, pa.epoch);
        peer_wait_all(pa, kGConsumed, pa.epoch, p.status);
      }
    }
  }
}

}  // namespace dst
