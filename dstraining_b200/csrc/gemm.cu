// Host side of the tcgen05 GEMM: TMA descriptor encoding, tile-shape and
// split-K selection, launch; plus the deterministic split-K reduction and
// the column-sum (bias gradient) entry.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <mutex>

#include "common.h"
#include "gemm.cuh"
#include "reduce.cuh"

namespace dst {

// ---------------------------------------------------------------- tensor maps
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    TORCH_CHECK(e == cudaSuccess && q == cudaDriverEntryPointSuccess && p != nullptr,
                "cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D bf16 tensor [outer][inner] with row stride `ld` elements; 128B-swizzled
// box of box_inner (<= 64) x box_outer.
CUtensorMap make_tmap_bf16(const void* base, uint64_t inner, uint64_t outer, uint64_t ld, uint32_t box_inner,
                           uint32_t box_outer) {
  CUtensorMap m;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  TORCH_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TORCH_CHECK((ld * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUresult r = encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", static_cast<int>(r));
  return m;
}

int num_sms() {
  static int n[64] = {0};
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (n[dev] == 0) C10_CUDA_CHECK(cudaDeviceGetAttribute(&n[dev], cudaDevAttrMultiProcessorCount, dev));
  return n[dev];
}

template <int BN, bool A_MN, bool B_MN, int EPI, int GATHER = 0, bool SCATTER = false>
static void launch_one(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const CUtensorMap& tx,
                       const GemmParams& p, int grid, cudaStream_t st, const PeerArgs* pa = nullptr) {
  auto kern = gemm_bf16_kernel<BN, A_MN, B_MN, EPI, GATHER, SCATTER>;
  constexpr int smem = GemmCfg<BN, GATHER == 1 && !A_MN>::kSmemBytes;
  static bool configured[64] = {false};
  int dev;
  C10_CUDA_CHECK(cudaGetDevice(&dev));
  if (!configured[dev]) {
    C10_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    configured[dev] = true;
  }
  static const PeerArgs none{};
  kern<<<grid, kGemmThreads, smem, st>>>(ta, tb, to, tx, p, pa ? *pa : none);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

template <int BN, bool A_MN, bool B_MN>
static void dispatch_epi(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                         const CUtensorMap& tx, const GemmParams& p, int grid, cudaStream_t st) {
  switch (epi) {
    case kEpiStore: return launch_one<BN, A_MN, B_MN, kEpiStore>(ta, tb, to, tx, p, grid, st);
    case kEpiBias: return launch_one<BN, A_MN, B_MN, kEpiBias>(ta, tb, to, tx, p, grid, st);
    case kEpiBiasGelu: return launch_one<BN, A_MN, B_MN, kEpiBiasGelu>(ta, tb, to, tx, p, grid, st);
    case kEpiBiasResid: return launch_one<BN, A_MN, B_MN, kEpiBiasResid>(ta, tb, to, tx, p, grid, st);
    case kEpiDGelu: return launch_one<BN, A_MN, B_MN, kEpiDGelu>(ta, tb, to, tx, p, grid, st);
    case kEpiPartialF32: return launch_one<BN, A_MN, B_MN, kEpiPartialF32>(ta, tb, to, tx, p, grid, st);
    case kEpiCEStats: return launch_one<BN, A_MN, B_MN, kEpiCEStats>(ta, tb, to, tx, p, grid, st);
    case kEpiAccumF32: return launch_one<BN, A_MN, B_MN, kEpiAccumF32>(ta, tb, to, tx, p, grid, st);
    default: TORCH_CHECK(false, "unknown epilogue ", epi);
  }
}

template <int BN>
static void dispatch_layout(bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                            const CUtensorMap& to, const CUtensorMap& tx, const GemmParams& p, int grid,
                            cudaStream_t st) {
  if (!a_mn && !b_mn) return dispatch_epi<BN, false, false>(epi, ta, tb, to, tx, p, grid, st);
  if (!a_mn && b_mn) return dispatch_epi<BN, false, true>(epi, ta, tb, to, tx, p, grid, st);
  if (a_mn && b_mn) return dispatch_epi<BN, true, true>(epi, ta, tb, to, tx, p, grid, st);
  return dispatch_epi<BN, true, false>(epi, ta, tb, to, tx, p, grid, st);
}

// Pick the number of K splits: minimise waves / splits (time per unit of K)
// for small tile counts; prefer fewer splits on ties.
static int choose_splits(int tiles, int k_blocks, int sms) {
  if (tiles >= sms || k_blocks < 8) return 1;
  int best = 1;
  double best_cost = 1e30;
  for (int s = 1; s <= 8 && k_blocks / s >= 4; ++s) {
    int waves = (tiles * s + sms - 1) / sms;
    double cost = static_cast<double>(waves) / s + 0.02 * s;  // small penalty for the reduce pass
    if (cost < best_cost - 1e-9) {
      best_cost = cost;
      best = s;
    }
  }
  return best;
}

void gemm_run(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int M, int N, int K, int epi,
              GemmParams p, int splits_hint) {
  TORCH_CHECK(A.scalar_type() == at::kBFloat16 && B.scalar_type() == at::kBFloat16, "gemm: bf16 operands required");
  TORCH_CHECK(A.is_cuda() && B.is_cuda(), "gemm: CUDA tensors required");
  TORCH_CHECK(A.stride(-1) == 1 && B.stride(-1) == 1, "gemm: operands must have unit inner stride");
  TORCH_CHECK(M > 0 && N > 0 && K > 0, "gemm: empty problem");
  TORCH_CHECK(N % 8 == 0, "gemm: N must be a multiple of 8");
  const int64_t lda = A.stride(0), ldb = B.stride(0);
  const int BN = (N >= 256) ? 256 : 128;
  CUtensorMap ta = a_mn ? make_tmap_bf16(A.data_ptr(), M, K, lda, 64, 64) : make_tmap_bf16(A.data_ptr(), K, M, lda, 64, kBM);
  CUtensorMap tb = b_mn ? make_tmap_bf16(B.data_ptr(), N, K, ldb, 64, 64) : make_tmap_bf16(B.data_ptr(), K, N, ldb, 64, BN);
  const int sms = num_sms();
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  const int k_blocks = (K + kBK - 1) / kBK;
  int splits = 1;
  if (epi == kEpiPartialF32) splits = splits_hint > 0 ? splits_hint : choose_splits(tiles, k_blocks, sms);
  splits = std::max(1, std::min(splits, k_blocks));
  p.M = M;
  p.N = N;
  p.K = K;
  p.splits = splits;
  p.k_blocks_per_split = (k_blocks + splits - 1) / splits;
  p.status = status_ptr();
  const int units = tiles * splits;
  const int grid = std::min(units, sms);
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
  // bf16 outputs are written by TMA stores of 32x64 boxes.
  CUtensorMap to = ta, tx = ta;
  if (epi != kEpiPartialF32 && epi != kEpiAccumF32) {
    TORCH_CHECK(p.out != nullptr, "gemm: missing output");
    to = make_tmap_bf16(p.out, N, M, p.ldo, kEpiChunk, 32);
    if (epi == kEpiBiasGelu) tx = make_tmap_bf16(p.aux_out, N, M, p.ldo, kEpiChunk, 32);
    // residual / pre-activation operand: prefetched into L2 by the producer
    if ((epi == kEpiBiasResid || epi == kEpiDGelu) && p.aux != nullptr)
      tx = make_tmap_bf16(p.aux, N, M, p.ld_aux, kEpiChunk, 32);
  }
  if (BN == 256)
    dispatch_layout<256>(a_mn, b_mn, epi, ta, tb, to, tx, p, grid, st);
  else
    dispatch_layout<128>(a_mn, b_mn, epi, ta, tb, to, tx, p, grid, st);
}

int gemm_splits_for(int M, int N, int K) {
  const int BN = (N >= 256) ? 256 : 128;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
  return choose_splits(tiles, (K + kBK - 1) / kBK, num_sms());
}

// ---------------------------------------------------------------- reductions
// out[m, n] = bf16(sum_s ws[s, m, n]) (+ the old out when accumulate), summed
// in split order.
__global__ void splitk_reduce_kernel(const float* __restrict__ ws, int splits, size_t mn, __nv_bfloat16* __restrict__ out,
                                     float* __restrict__ out_f32) {
  size_t i = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) * 4;
  if (i >= mn) return;
  float4 acc = *reinterpret_cast<const float4*>(ws + i);
  for (int s = 1; s < splits; ++s) {
    float4 v = *reinterpret_cast<const float4*>(ws + s * mn + i);
    acc.x += v.x;
    acc.y += v.y;
    acc.z += v.z;
    acc.w += v.w;
  }
  if (out_f32) {
    float4 o = *reinterpret_cast<float4*>(out_f32 + i);
    o.x += acc.x;
    o.y += acc.y;
    o.z += acc.z;
    o.w += acc.w;
    *reinterpret_cast<float4*>(out_f32 + i) = o;
  } else {
    __nv_bfloat162 a = __floats2bfloat162_rn(acc.x, acc.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(acc.z, acc.w);
    reinterpret_cast<__nv_bfloat162*>(out + i)[0] = a;
    reinterpret_cast<__nv_bfloat162*>(out + i)[1] = b;
  }
}

}  // namespace dst

// ---------------------------------------------------------------- bindings
using namespace dst;

static void check_bf16_2d(const at::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.scalar_type() == at::kBFloat16 && t.dim() == 2, name, ": CUDA bf16 2-D tensor required");
  TORCH_CHECK(t.stride(1) == 1, name, ": inner dimension must be contiguous");
}

// Generic entry: C = op(A) . op(B)^T with the requested epilogue.
// a_mn: A is [K, M] (else [M, K]); b_mn: B is [K, N] (else [N, K]).
at::Tensor gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t epi,
                const c10::optional<at::Tensor>& bias, const c10::optional<at::Tensor>& aux,
                const c10::optional<at::Tensor>& aux_out, const c10::optional<at::Tensor>& out_opt) {
  check_bf16_2d(A, "A");
  check_bf16_2d(B, "B");
  c10::cuda::CUDAGuard g(A.device());
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const int N = b_mn ? B.size(1) : B.size(0);
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "gemm: K mismatch");
  at::Tensor out = out_opt.has_value() ? *out_opt : at::empty({M, N}, A.options());
  check_bf16_2d(out, "out");
  TORCH_CHECK(out.size(0) == M && out.size(1) == N, "gemm: out shape");
  GemmParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
  p.ldo = out.stride(0);
  if (bias.has_value()) {
    TORCH_CHECK(bias->numel() == N && bias->is_contiguous(), "gemm: bias shape");
    p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (aux.has_value()) {
    check_bf16_2d(*aux, "aux");
    TORCH_CHECK(aux->size(0) == M && aux->size(1) == N, "gemm: aux shape");
    p.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
    p.ld_aux = aux->stride(0);
  }
  if (aux_out.has_value()) {
    check_bf16_2d(*aux_out, "aux_out");
    TORCH_CHECK(aux_out->stride(0) == out.stride(0), "gemm: aux_out stride must match out");
    p.aux_out = reinterpret_cast<__nv_bfloat16*>(aux_out->data_ptr());
  }
  TORCH_CHECK(epi != kEpiPartialF32 && epi != kEpiCEStats && epi != kEpiAccumF32, "gemm: use the dedicated entry");
  TORCH_CHECK(!(epi == kEpiBiasResid || epi == kEpiDGelu) || aux.has_value(), "gemm: epilogue needs aux");
  TORCH_CHECK(epi != kEpiBiasGelu || aux_out.has_value(), "gemm: gelu epilogue needs aux_out");
  gemm_run(A, a_mn, B, b_mn, M, N, K, static_cast<int>(epi), p, 0);
  return out;
}

// Weight gradient dW[M, N] = A^T-style product with K = tokens, split-K with a
// deterministic fp32 reduction. If accum_f32 is given, the result is added
// into it (fp32) instead of being returned as bf16.
at::Tensor gemm_splitk(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t splits,
                       const c10::optional<at::Tensor>& accum_f32) {
  check_bf16_2d(A, "A");
  check_bf16_2d(B, "B");
  c10::cuda::CUDAGuard g(A.device());
  const int M = a_mn ? A.size(1) : A.size(0);
  const int K = a_mn ? A.size(0) : A.size(1);
  const int N = b_mn ? B.size(1) : B.size(0);
  TORCH_CHECK((b_mn ? B.size(0) : B.size(1)) == K, "gemm_splitk: K mismatch");
  TORCH_CHECK(N % 4 == 0, "gemm_splitk: N must be a multiple of 4");
  int s = splits > 0 ? static_cast<int>(splits) : gemm_splits_for(M, N, K);
  const int k_blocks = (K + kBK - 1) / kBK;
  s = std::max(1, std::min(s, k_blocks));
  // Clamp so that every split gets at least one K block.
  const int per = (k_blocks + s - 1) / s;
  s = (k_blocks + per - 1) / per;
  at::Tensor ws = at::empty({s, M, N}, A.options().dtype(at::kFloat));
  GemmParams p{};
  p.ws = ws.data_ptr<float>();
  gemm_run(A, a_mn, B, b_mn, M, N, K, kEpiPartialF32, p, s);
  const size_t mn = static_cast<size_t>(M) * N;
  at::Tensor out;
  float* acc = nullptr;
  if (accum_f32.has_value()) {
    TORCH_CHECK(accum_f32->scalar_type() == at::kFloat && accum_f32->is_contiguous() &&
                    accum_f32->numel() == static_cast<int64_t>(mn),
                "gemm_splitk: accum_f32 must be a contiguous fp32 [M, N] tensor");
    acc = accum_f32->data_ptr<float>();
    out = *accum_f32;
  } else {
    out = at::empty({M, N}, A.options());
  }
  const int threads = 256;
  const int blocks = static_cast<int>((mn / 4 + threads - 1) / threads);
  splitk_reduce_kernel<<<blocks, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      ws.data_ptr<float>(), s, mn, acc ? nullptr : reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), acc);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Column sums (bias gradient) via the deterministic two-pass reduction.
at::Tensor colsum_bf16(const at::Tensor& x) {
  check_bf16_2d(x, "x");
  TORCH_CHECK(x.is_contiguous(), "colsum: contiguous input required");
  c10::cuda::CUDAGuard g(x.device());
  const int M = x.size(0), N = x.size(1);
  TORCH_CHECK(N % 8 == 0, "colsum: N must be a multiple of 8");
  const int R = (M + kColredRows - 1) / kColredRows;
  at::Tensor partial = at::empty({R, N}, x.options().dtype(at::kFloat));
  at::Tensor out = at::empty({N}, x.options());
  auto st = at::cuda::getCurrentCUDAStream();
  dim3 g1((N + 255) / 256, R);
  colred_stage1<false><<<g1, 256, 0, st>>>(reinterpret_cast<const __nv_bfloat16*>(x.data_ptr()), nullptr, nullptr,
                                           nullptr, M, N, partial.data_ptr<float>(), nullptr);
  dim3 g2((N + 31) / 32, 1);
  colred_stage2<<<g2, 256, 0, st>>>(partial.data_ptr<float>(), R, N, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Sum a split-K fp32 workspace [splits, M, N] in split order -> bf16 [M, N].
at::Tensor splitk_reduce(const at::Tensor& ws) {
  TORCH_CHECK(ws.is_cuda() && ws.scalar_type() == at::kFloat && ws.dim() == 3 && ws.is_contiguous(), "splitk_reduce: ws");
  c10::cuda::CUDAGuard g(ws.device());
  const int s = ws.size(0), M = ws.size(1), N = ws.size(2);
  TORCH_CHECK(N % 4 == 0, "splitk_reduce: N must be a multiple of 4");
  at::Tensor out = at::empty({M, N}, ws.options().dtype(at::kBFloat16));
  const size_t mn = static_cast<size_t>(M) * N;
  splitk_reduce_kernel<<<static_cast<int>((mn / 4 + 255) / 256), 256, 0, at::cuda::getCurrentCUDAStream()>>>(
      ws.data_ptr<float>(), s, mn, reinterpret_cast<__nv_bfloat16*>(out.data_ptr()), nullptr);
  C10_CUDA_KERNEL_LAUNCH_CHECK();
  return out;
}

// Fused LM-head forward: logits (bf16, optional) and per-(row, tile) softmax
// statistics from the fp32 accumulator, target logits for targets inside
// this shard. Returns (logits, tile_max, tile_sum, tgt_logit).
std::vector<at::Tensor> gemm_ce_stats(const at::Tensor& X, const at::Tensor& W, const at::Tensor& targets,
                                      int64_t col0, int64_t valid_cols) {
  check_bf16_2d(X, "X");
  check_bf16_2d(W, "W");
  TORCH_CHECK(targets.scalar_type() == at::kLong && targets.is_contiguous() && targets.numel() == X.size(0),
              "gemm_ce_stats: int64 targets [M] required");
  c10::cuda::CUDAGuard g(X.device());
  const int M = X.size(0), K = X.size(1), N = W.size(0);
  TORCH_CHECK(W.size(1) == K, "gemm_ce_stats: K mismatch");
  const int BN = (N >= 256) ? 256 : 128;
  const int n_tiles = (N + BN - 1) / BN;
  at::Tensor logits = at::empty({M, N}, X.options());
  at::Tensor tmax = at::empty({M, n_tiles}, X.options().dtype(at::kFloat));
  at::Tensor tsum = at::empty({M, n_tiles}, X.options().dtype(at::kFloat));
  at::Tensor tgt = at::zeros({M}, X.options().dtype(at::kFloat));
  GemmParams p{};
  p.out = reinterpret_cast<__nv_bfloat16*>(logits.data_ptr());
  p.ldo = N;
  p.ce_max = tmax.data_ptr<float>();
  p.ce_sum = tsum.data_ptr<float>();
  p.ce_tgt = tgt.data_ptr<float>();
  p.ce_targets = targets.data_ptr<int64_t>();
  p.ce_col0 = static_cast<int>(col0);
  p.ce_valid_cols = static_cast<int>(valid_cols);
  gemm_run(X, false, W, false, M, N, K, kEpiCEStats, p, 0);
  return {logits, tmax, tsum, tgt};
}

// ---------------------------------------------------------------- tensor parallel
// Peer-aware GEMM (gemm.cuh): mode 1 gathers operand A over the TP group,
// mode 2 gathers operand B, mode 3 scatters the output into the owning
// ranks' receive slots. `peers` holds each rank's base pointer of the
// gathered shard (modes 1, 2) or of the receive buffer (mode 3); `flags`
// each rank's flag words of this channel; `epoch` the channel's launch count.
template <int BN, bool A_MN, bool B_MN, int MODE>
static void peer_dispatch(int epi, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to,
                          const CUtensorMap& tx, const GemmParams& p, int grid, cudaStream_t st, const PeerArgs& pa) {
  constexpr int G = MODE == 3 ? 0 : MODE;
  constexpr bool SC = MODE == 3;
  if constexpr (MODE == 1 && !A_MN && !B_MN) {
    switch (epi) {
      case kEpiStore: return launch_one<BN, A_MN, B_MN, kEpiStore, G, SC>(ta, tb, to, ta, p, grid, st, &pa);
      case kEpiBias: return launch_one<BN, A_MN, B_MN, kEpiBias, G, SC>(ta, tb, to, ta, p, grid, st, &pa);
      case kEpiBiasGelu: return launch_one<BN, A_MN, B_MN, kEpiBiasGelu, G, SC>(ta, tb, to, tx, p, grid, st, &pa);
      case kEpiCEStats: return launch_one<BN, A_MN, B_MN, kEpiCEStats, G, SC>(ta, tb, to, ta, p, grid, st, &pa);
      default: break;
    }
  } else if constexpr (MODE == 1 && !A_MN && B_MN) {
    switch (epi) {
      case kEpiStore: return launch_one<BN, A_MN, B_MN, kEpiStore, G, SC>(ta, tb, to, ta, p, grid, st, &pa);
      case kEpiDGelu: return launch_one<BN, A_MN, B_MN, kEpiDGelu, G, SC>(ta, tb, to, tx, p, grid, st, &pa);
      default: break;
    }
  } else if constexpr ((MODE == 1 || MODE == 2) && A_MN && B_MN) {
    switch (epi) {
      case kEpiPartialF32: return launch_one<BN, A_MN, B_MN, kEpiPartialF32, G, SC>(ta, tb, to, ta, p, grid, st, &pa);
      case kEpiStore: return launch_one<BN, A_MN, B_MN, kEpiStore, G, SC>(ta, tb, to, ta, p, grid, st, &pa);
      default: break;
    }
  } else if constexpr (MODE == 3 && !A_MN) {
    if (epi == kEpiStore) return launch_one<BN, A_MN, B_MN, kEpiStore, G, SC>(ta, tb, to, ta, p, grid, st, &pa);
  }
  TORCH_CHECK(false, "tp_gemm: unsupported mode/layout/epilogue combination");
}

template <int BN, int MODE>
static void peer_layout(bool a_mn, bool b_mn, int epi, const CUtensorMap& ta, const CUtensorMap& tb,
                        const CUtensorMap& to, const CUtensorMap& tx, const GemmParams& p, int grid, cudaStream_t st,
                        const PeerArgs& pa) {
  if (!a_mn && !b_mn) return peer_dispatch<BN, false, false, MODE>(epi, ta, tb, to, tx, p, grid, st, pa);
  if (!a_mn && b_mn) return peer_dispatch<BN, false, true, MODE>(epi, ta, tb, to, tx, p, grid, st, pa);
  if (a_mn && b_mn) return peer_dispatch<BN, true, true, MODE>(epi, ta, tb, to, tx, p, grid, st, pa);
  TORCH_CHECK(false, "tp_gemm: unsupported layout");
}

// Returns the bf16 output (modes 1, 2 with a bf16 epilogue), the fp32 split-K
// workspace (PartialF32), or an empty tensor (mode 3: the data went to the
// peers). The gathered dimension of size `tokens` is split evenly over the
// group; `seq` is the per-batch sequence length of that dimension.
std::vector<at::Tensor> tp_gemm(const at::Tensor& A, bool a_mn, const at::Tensor& B, bool b_mn, int64_t M, int64_t N,
                                int64_t K, int64_t epi, int64_t mode, const std::vector<int64_t>& peers,
                                const std::vector<int64_t>& flags, const at::Tensor& done, int64_t rank, int64_t seq,
                                int64_t epoch, int64_t splits, const c10::optional<at::Tensor>& bias,
                                const c10::optional<at::Tensor>& aux, const c10::optional<at::Tensor>& aux_out,
                                const c10::optional<at::Tensor>& targets, int64_t ce_col0, int64_t ce_valid,
                                const c10::optional<at::Tensor>& gath, const c10::optional<at::Tensor>& arrive) {
  check_bf16_2d(A, "A");
  check_bf16_2d(B, "B");
  c10::cuda::CUDAGuard g(A.device());
  const int tp = static_cast<int>(peers.size());
  TORCH_CHECK(tp >= 2 && tp <= kMaxPeers && flags.size() == peers.size(), "tp_gemm: 2..8 ranks");
  TORCH_CHECK(mode >= 1 && mode <= 3, "tp_gemm: mode");
  const int64_t tokens = (mode == 3 || (mode == 1 && !a_mn)) ? M : K;
  TORCH_CHECK(tokens % seq == 0 && seq % tp == 0, "tp_gemm: token dimension must split evenly");
  const int seq_local = static_cast<int>(seq / tp);
  const int rows_local = static_cast<int>(tokens / tp);
  const int BN = (N >= 256) ? 256 : 128;
  if (mode == 1 && !a_mn) TORCH_CHECK(seq_local % kBM == 0, "tp_gemm: T/tp must be a multiple of 128");
  if (mode == 3) TORCH_CHECK(seq_local % 32 == 0, "tp_gemm: T/tp must be a multiple of 32");
  if ((mode == 1 && a_mn) || mode == 2) TORCH_CHECK(seq_local % kBK == 0, "tp_gemm: T/tp must be a multiple of 64");

  PeerArgs pa{};
  pa.tp = tp;
  pa.rank = static_cast<int>(rank);
  pa.seq = static_cast<int>(seq);
  pa.seq_local = seq_local;
  pa.rows_local = rows_local;
  pa.epoch = static_cast<uint32_t>(epoch);
  TORCH_CHECK(done.scalar_type() == at::kInt && done.numel() >= 2, "tp_gemm: done must hold 2 int32 counters");
  pa.done_ctas = reinterpret_cast<unsigned int*>(done.data_ptr<int32_t>());
  pa.claim = pa.done_ctas + 1;
  for (int r = 0; r < tp; ++r) pa.flags[r] = reinterpret_cast<uint32_t*>(flags[r]);

  // Local operand maps (the gathered one is only a shape template).
  CUtensorMap ta = a_mn ? make_tmap_bf16(A.data_ptr(), A.size(1), A.size(0), A.stride(0), 64, 64)
                        : make_tmap_bf16(A.data_ptr(), A.size(1), A.size(0), A.stride(0), 64, kBM);
  CUtensorMap tb = b_mn ? make_tmap_bf16(B.data_ptr(), B.size(1), B.size(0), B.stride(0), 64, 64)
                        : make_tmap_bf16(B.data_ptr(), B.size(1), B.size(0), B.stride(0), 64, BN);
  const at::Tensor& G = (mode == 2) ? B : A;
  const bool g_mn = (mode == 2) ? b_mn : a_mn;
  if (mode == 1 || mode == 2) {
    for (int r = 0; r < tp; ++r)
      pa.gather[r] = make_tmap_bf16(reinterpret_cast<void*>(peers[r]), G.size(1), G.size(0), G.stride(0), 64,
                                    g_mn ? 64 : kBM);
    if (mode == 1 && !a_mn) {
      // rows gathered through the local gather buffer (one NVLink crossing per byte)
      TORCH_CHECK(gath.has_value() && arrive.has_value(), "tp_gemm: row gather needs gath and arrive buffers");
      TORCH_CHECK(gath->is_contiguous() && gath->size(0) == M && gath->size(1) == K && gath->scalar_type() == at::kBFloat16,
                  "tp_gemm: gath must be a contiguous bf16 [M, K] tensor");
      TORCH_CHECK(A.is_contiguous() && K % 64 == 0, "tp_gemm: row gather needs a contiguous shard and K % 64 == 0");
      TORCH_CHECK(arrive->scalar_type() == at::kInt && arrive->numel() >= (M + kBM - 1) / kBM, "tp_gemm: arrive");
      for (int r = 0; r < tp; ++r) pa.shard[r] = reinterpret_cast<const __nv_bfloat16*>(peers[r]);
      pa.shard_ld = static_cast<int>(K);
      pa.gath = reinterpret_cast<__nv_bfloat16*>(gath->data_ptr());
      pa.arrive = reinterpret_cast<unsigned int*>(arrive->data_ptr<int32_t>());
      pa.kchunks = static_cast<int>(K / 64);
      pa.gath_map = make_tmap_bf16(gath->data_ptr(), K, M, K, 64, kBM);
    }
  } else {
    for (int r = 0; r < tp; ++r)
      pa.scatter[r] = make_tmap_bf16(reinterpret_cast<void*>(peers[r]), N, static_cast<uint64_t>(tp) * rows_local, N,
                                     kEpiChunk, 32);
  }

  GemmParams p{};
  std::vector<at::Tensor> result;
  at::Tensor out, ws;
  int s = 1;
  const int k_blocks = static_cast<int>((K + kBK - 1) / kBK);
  if (epi == kEpiPartialF32) {
    s = splits > 0 ? static_cast<int>(splits) : gemm_splits_for(M, N, K);
    s = std::max(1, std::min(s, k_blocks));
    const int per = (k_blocks + s - 1) / s;
    s = (k_blocks + per - 1) / per;
    ws = at::empty({s, M, N}, A.options().dtype(at::kFloat));
    p.ws = ws.data_ptr<float>();
    result.push_back(ws);
  } else if (mode != 3) {
    out = at::empty({M, N}, A.options());
    p.out = reinterpret_cast<__nv_bfloat16*>(out.data_ptr());
    p.ldo = N;
    result.push_back(out);
  } else {
    result.push_back(at::Tensor());
  }
  if (bias.has_value()) p.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  if (aux.has_value()) {
    check_bf16_2d(*aux, "aux");
    p.aux = reinterpret_cast<const __nv_bfloat16*>(aux->data_ptr());
    p.ld_aux = aux->stride(0);
  }
  at::Tensor pre;
  if (epi == kEpiBiasGelu) {
    TORCH_CHECK(mode == 1, "tp_gemm: the GELU epilogue is offered in gather mode only");
    pre = at::empty({M, N}, A.options());  // pre-activation, returned after the output
  }
  at::Tensor tmax, tsum, tgt;
  if (epi == kEpiCEStats) {
    TORCH_CHECK(targets.has_value(), "tp_gemm: CE statistics need targets");
    const int n_tiles = static_cast<int>((N + BN - 1) / BN);
    tmax = at::empty({M, n_tiles}, A.options().dtype(at::kFloat));
    tsum = at::empty({M, n_tiles}, A.options().dtype(at::kFloat));
    tgt = at::zeros({M}, A.options().dtype(at::kFloat));
    p.ce_max = tmax.data_ptr<float>();
    p.ce_sum = tsum.data_ptr<float>();
    p.ce_tgt = tgt.data_ptr<float>();
    p.ce_targets = targets->data_ptr<int64_t>();
    p.ce_col0 = static_cast<int>(ce_col0);
    p.ce_valid_cols = static_cast<int>(ce_valid);
    result.push_back(tmax);
    result.push_back(tsum);
    result.push_back(tgt);
  }
  p.M = static_cast<int>(M);
  p.N = static_cast<int>(N);
  p.K = static_cast<int>(K);
  p.splits = s;
  p.k_blocks_per_split = (k_blocks + s - 1) / s;
  p.status = status_ptr();
  CUtensorMap to = ta, tx = ta;
  if (mode != 3 && epi != kEpiPartialF32) to = make_tmap_bf16(p.out, N, M, N, kEpiChunk, 32);
  if ((epi == kEpiBiasResid || epi == kEpiDGelu) && p.aux != nullptr)
    tx = make_tmap_bf16(p.aux, N, M, p.ld_aux, kEpiChunk, 32);
  if (epi == kEpiBiasGelu) {
    p.aux_out = reinterpret_cast<__nv_bfloat16*>(pre.data_ptr());
    tx = make_tmap_bf16(pre.data_ptr(), N, M, N, kEpiChunk, 32);
    result.push_back(pre);
  }
  const int tiles = static_cast<int>(((M + kBM - 1) / kBM) * ((N + BN - 1) / BN));
  const int grid = std::min(tiles * s, num_sms());
  cudaStream_t st = at::cuda::getCurrentCUDAStream();
#define PEER_MODE(BNV, MV) peer_layout<BNV, MV>(a_mn, b_mn, static_cast<int>(epi), ta, tb, to, tx, p, grid, st, pa)
  if (BN == 256) {
    if (mode == 1) PEER_MODE(256, 1); else if (mode == 2) PEER_MODE(256, 2); else PEER_MODE(256, 3);
  } else {
    if (mode == 1) PEER_MODE(128, 1); else if (mode == 2) PEER_MODE(128, 2); else PEER_MODE(128, 3);
  }
#undef PEER_MODE
  return result;
}

void register_gemm(pybind11::module& m) {
  m.def("gemm", &gemm, "bf16 tcgen05 GEMM with fused epilogue", py::arg("A"), py::arg("a_mn"), py::arg("B"),
        py::arg("b_mn"), py::arg("epi"), py::arg("bias") = py::none(), py::arg("aux") = py::none(),
        py::arg("aux_out") = py::none(), py::arg("out") = py::none());
  m.def("gemm_splitk", &gemm_splitk, "split-K bf16 GEMM with deterministic fp32 reduction", py::arg("A"),
        py::arg("a_mn"), py::arg("B"), py::arg("b_mn"), py::arg("splits") = 0, py::arg("accum_f32") = py::none());
  m.def("colsum_bf16", &colsum_bf16, "column sums of a bf16 matrix (bias gradient)");
  m.def("splitk_reduce", &splitk_reduce, "sum a split-K fp32 workspace in split order to bf16");
  m.def("gemm_ce_stats", &gemm_ce_stats, "LM-head GEMM with fused softmax statistics");
  m.def("tp_gemm", &tp_gemm, "tensor-parallel GEMM fused with an NVLink all-gather (modes 1, 2) or reduce-scatter (mode 3)",
        py::arg("A"), py::arg("a_mn"), py::arg("B"), py::arg("b_mn"), py::arg("M"), py::arg("N"), py::arg("K"),
        py::arg("epi"), py::arg("mode"), py::arg("peers"), py::arg("flags"), py::arg("done"), py::arg("rank"),
        py::arg("seq"), py::arg("epoch"), py::arg("splits") = 0, py::arg("bias") = py::none(),
        py::arg("aux") = py::none(), py::arg("aux_out") = py::none(), py::arg("targets") = py::none(),
        py::arg("ce_col0") = 0, py::arg("ce_valid") = 0, py::arg("gath") = py::none(), py::arg("arrive") = py::none());
}
