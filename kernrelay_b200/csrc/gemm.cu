// tcgen05 GEMM kernels (plain store / bias / SiLU-mul epilogues) and launchers.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "common.h"
#include "gemm.cuh"

namespace krb {

// configuration variant of a plain GEMM: fp32 outputs stage in fp32, the rest in 2 bytes;
// one-CTA tiles: eight epilogue warps for the QKV and fp32-output epilogues, four for the
// others; CTA pairs (PAIR): 256-row tiles, eight epilogue warps
template <int MODE, bool PAIR>
constexpr int plain_cfg() {
  if (PAIR) return MODE == kEpiStoreF32 ? kCfgPairF32 : kCfgPair;
  return MODE == kEpiStoreF32 ? kCfgPlainF32 : MODE == kEpiQkvRope ? kCfgPlain : kCfgPlain4;
}

// F16: fp16 operands and 2-byte outputs (bf16 otherwise); fp32 accumulation either way.
// Warps: TMA producer, MMA issuer, 4 or 8 epilogue warps.  PAIR: launched in clusters of
// two CTAs (cta_group::2 MMAs on 256-row tiles).
template <int BN, int MODE, bool F16, bool PAIR>
__global__ void __launch_bounds__(GemmCfg<BN, plain_cfg<MODE, PAIR>()>::kThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                const __grid_constant__ CUtensorMap tb2, TileSched ts, int M, int K, EpiArgs ea,
                uint32_t *status) {
  constexpr int V = plain_cfg<MODE, PAIR>();
  using C = GemmCfg<BN, V>;
  extern __shared__ uint8_t smem_raw[];
  const GemmSmemView<BN, V> s = GemmSmemView<BN, V>::carve(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
    tma_prefetch_desc(&tb2);
  }
  gemm_setup<BN, V>(s, C::kEpiWarps * 32);
  if (warp == 0) {
    if (lane == 0) gemm_producer<BN, V>(s, &ta, &tb, &tb2, ts, K, status);
  } else if (warp == 1) {
    if (lane == 0) gemm_mma<BN, V, F16>(s, ts, K, status);
  } else {
    gemm_epilogue<BN, V, MODE, F16>(s, ts, M, ea, status);
  }
  gemm_teardown<BN, V>(s);
}

// ------------------------------------------------------------------ host side
int sm_count(int device) {
  static int cached[64] = {0};
  if (device >= 0 && device < 64 && cached[device]) return cached[device];
  int n = 0;
  KRB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device));
  if (device >= 0 && device < 64) cached[device] = n;
  return n;
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    KRB_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    if (q != cudaDriverEntryPointSuccess || !p) throw CudaError("cuTensorMapEncodeTiled missing");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMap make_tmap_2d_bf16(const void *base, uint64_t rows, uint64_t cols, uint64_t ld,
                              uint32_t box_rows, uint32_t box_cols) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw CudaError("tensor map base not 16B aligned");
  if ((ld * 2) % 16 != 0) throw CudaError("tensor map row pitch not a multiple of 16 bytes");
  CUtensorMap m;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * 2};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapSwizzle sw =
      (box_cols * 2 == 128) ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = get_encode_fn()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base),
                               dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw CudaError("cuTensorMapEncodeTiled failed: " + std::to_string(int(r)));
  return m;
}

static double wave_eff(long tiles, int sms) {
  const long waves = (tiles + sms - 1) / sms;
  return double(tiles) / double(waves * sms);
}

int pick_bn_store(int M, int N, int sms) {
  const int cands[3] = {256, 224, 128};
  // relative throughput of one tile: a 128-wide tile moves 1.33x the operand bytes per
  // FLOP of a 256-wide one and measured ~0.65 of its rate on B200 (fp16 M=8192 N=2048
  // row chunks: ~775 against ~1300 TFLOP/s)
  const double tile_eff[3] = {1.0, 0.97, 0.65};
  const long mblk = (M + kBM - 1) / kBM;
  int best = 256;
  double best_score = -1;
  for (int i = 0; i < 3; ++i) {
    const int bn = cands[i];
    const long tiles = mblk * ((N + bn - 1) / bn);
    // efficiency of waves, times column utilisation of the last N block
    const double col_util = double(N) / double(((N + bn - 1) / bn) * bn);
    const double score = wave_eff(tiles, sms) * col_util * tile_eff[i];
    if (score > best_score + 1e-9) {
      best_score = score;
      best = bn;
    }
  }
  return best;
}

int pick_bn_silu(int M, int n_out, int sms) {
  const long mblk = (M + kBM - 1) / kBM;
  const int cands[3] = {256, 192, 128};
  // relative throughput of one tile (CTA pairs): per 64-deep k-block a pair's SM moves
  // A 16 KB + its half of B in through TMA and out to the MMA; 256-wide tiles stay within
  // the SM's shared-memory bandwidth, 192-wide ones exceed it by ~15 %, 128-wide ones by
  // ~50 % (measured ~0.65 of the 256-wide rate)
  const double tile_eff[3] = {1.0, 0.87, 0.65};
  int best = 256;
  double best_score = -1;
  for (int i = 0; i < 3; ++i) {
    const int bn = cands[i];
    const int half = bn / 2;
    const long nblk = (n_out + half - 1) / half;
    const double col_util = double(n_out) / double(nblk * half);
    const double score = wave_eff(mblk * nblk, sms) * col_util * tile_eff[i];
    if (score > best_score + 1e-9) {
      best_score = score;
      best = bn;
    }
  }
  return best;
}

// Tile raster of a plain GEMM.  Row blocks fastest (one band over all rows) keeps a B
// column block hot while a wave sweeps the rows and re-reads A once per column block;
// that is right while A stays in L2.  When A is too large for that (tall activations, a
// small weight) column blocks go fastest instead (band = 1), so each A row block is read
// once and the small B stays resident.  KRB_GEMM_RASTER=row|col forces one order.
static int pick_band(long M, long N, long K, int num_m) {
  static const char *force = std::getenv("KRB_GEMM_RASTER");
  if (force && std::strcmp(force, "row") == 0) return num_m;
  if (force && std::strcmp(force, "col") == 0) return 1;
  const double a_bytes = double(M) * double(K) * 2.0, b_bytes = double(N) * double(K) * 2.0;
  return (a_bytes > 48e6 && b_bytes < 24e6) ? 1 : num_m;
}

// CTA pairs (cta_group::2) for every plain GEMM whose 128-row blocks pair up (an even
// count); KRB_GEMM_PAIR=0 keeps one-CTA tiles.
static bool pairs_enabled() {
  static const bool on = [] {
    const char *e = std::getenv("KRB_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on;
}

// The plain GEMMs with a per-tile column layout (store / fp32 store) take the two-phase
// tail re-cut (TileSched); the SiLU-gated (B interleaved per BN block) and QKV (heads
// per tile) epilogues keep one tile width.
template <int BN, int MODE, bool F16, bool PAIR>
static void launch_gemm_cfg(const CUtensorMap &ta, const void *B, long ldb, int M, int n_b_rows,
                            int K, const EpiArgs &ea, int grid_limit, uint32_t *status,
                            cudaStream_t stream) {
  using C = GemmCfg<BN, plain_cfg<MODE, PAIR>()>;
  constexpr int CG = C::kCG;
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  static bool configured[64] = {false};
  auto kern = gemm_kernel<BN, MODE, F16, PAIR>;
  if (!configured[dev & 63]) {
    KRB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(C::kSmemBytes)));
    configured[dev & 63] = true;
  }
  const int num_m = (M + kBM - 1) / kBM;
  const int band = pick_band(M, n_b_rows, K, num_m);
  // tile rows of CG 128-row blocks; one wave = the CTA groups that fit on the SMs
  const int rows = num_m / CG, band_rows = std::max(1, band / CG);
  int groups = std::min(rows * ((n_b_rows + BN - 1) / BN), sm_count(dev) / CG);
  if (grid_limit > 0) groups = std::min(groups, std::max(1, grid_limit / CG));
  constexpr bool two_phase = MODE == kEpiStore || MODE == kEpiStoreF32;
  const TileSched ts = TileSched::make(rows, n_b_rows, BN, band_rows, groups, two_phase, 16 * CG);
  // B boxes: the tile's rows of B, split between the pair's CTAs
  const CUtensorMap tb = make_tmap_2d_bf16(B, n_b_rows, K, ldb, BN / CG, kBK);
  const CUtensorMap tb2 =
      ts.bn2 != BN ? make_tmap_2d_bf16(B, n_b_rows, K, ldb, ts.bn2 / CG, kBK) : tb;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(groups * CG);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = CG;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  KRB_CUDA(cudaLaunchKernelEx(&cfg, kern, ta, tb, tb2, ts, M, K, ea, status));
}

template <int BN, int MODE, bool F16>
static void launch_gemm(const CUtensorMap &ta, const void *B, long ldb, int M, int n_b_rows,
                        int K, const EpiArgs &ea, int grid_limit, uint32_t *status,
                        cudaStream_t stream) {
  const int num_m = (M + kBM - 1) / kBM;
  // the QKV epilogue (RoPE) spills at the pair kernel's register budget and ran 2-5 %
  // slower on pairs; every other GEMM ran 1-5 % faster
  if (MODE != kEpiQkvRope && pairs_enabled() && num_m % 2 == 0 && num_m >= 2)
    launch_gemm_cfg<BN, MODE, F16, true>(ta, B, ldb, M, n_b_rows, K, ea, grid_limit, status,
                                         stream);
  else
    launch_gemm_cfg<BN, MODE, F16, false>(ta, B, ldb, M, n_b_rows, K, ea, grid_limit, status,
                                          stream);
}

// The launch of MODE for element type T at tile width bn
template <int MODE, typename T>
static void dispatch_bn(int bn, const CUtensorMap &ta, const T *B, long ldb, int M, int n_b_rows,
                        int K, const EpiArgs &ea, int grid_limit, uint32_t *status,
                        cudaStream_t stream, const char *what) {
  constexpr bool F16 = ActFmt<T>::f16;
  switch (bn) {
    case 256:
      launch_gemm<256, MODE, F16>(ta, B, ldb, M, n_b_rows, K, ea, grid_limit, status, stream);
      break;
    case 224:
      if constexpr (MODE != kEpiSiluMul && MODE != kEpiQkvRope) {
        launch_gemm<224, MODE, F16>(ta, B, ldb, M, n_b_rows, K, ea, grid_limit, status, stream);
        break;
      }
      [[fallthrough]];
    case 192:
      if constexpr (MODE == kEpiSiluMul) {
        if (bn == 192) {
          launch_gemm<192, MODE, F16>(ta, B, ldb, M, n_b_rows, K, ea, grid_limit, status, stream);
          break;
        }
      }
      [[fallthrough]];
    case 128:
      if (bn == 128) {
        launch_gemm<128, MODE, F16>(ta, B, ldb, M, n_b_rows, K, ea, grid_limit, status, stream);
        break;
      }
      [[fallthrough]];
    default:
      throw CudaError(std::string(what) + ": unsupported bn " + std::to_string(bn));
  }
}

template <typename T>
void gemm_store(const T *A, long lda, const T *B, long ldb, T *C, long ldc,
                const __nv_bfloat16 *bias, int M, int N, int K, int bn, int grid_limit,
                uint32_t *status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) throw CudaError("gemm: empty shape");
  if (N % 8 != 0 || ldc % 8 != 0) throw CudaError("gemm: N and ldc must be multiples of 8");
  if (reinterpret_cast<uintptr_t>(C) % 16 || (bias && reinterpret_cast<uintptr_t>(bias) % 16))
    throw CudaError("gemm: C/bias must be 16-byte aligned");
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  if (bn <= 0) bn = pick_bn_store(M, N, sm_count(dev));
  EpiArgs ea{};
  ea.c = reinterpret_cast<__nv_bfloat16 *>(C);  // 2-byte rows; the epilogue packs T
  ea.ldc = ldc;
  ea.bias = bias;
  ea.n_out = N;
  const CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, kBM, kBK);
  dispatch_bn<kEpiStore>(bn, ta, B, ldb, M, N, K, ea, grid_limit, status, stream, "gemm");
}

void gemm_bf16(const __nv_bfloat16 *A, long lda, const __nv_bfloat16 *B, long ldb,
               __nv_bfloat16 *C, long ldc, const __nv_bfloat16 *bias, int M, int N, int K,
               int bn, int grid_limit, uint32_t *status, cudaStream_t stream) {
  gemm_store<__nv_bfloat16>(A, lda, B, ldb, C, ldc, bias, M, N, K, bn, grid_limit, status, stream);
}

void gemm_f16(const __half *A, long lda, const __half *B, long ldb, __half *C, long ldc, int M,
              int N, int K, int bn, uint32_t *status, cudaStream_t stream) {
  gemm_store<__half>(A, lda, B, ldb, C, ldc, nullptr, M, N, K, bn, 0, status, stream);
}

template <typename T>
void gemm_f32out(const T *A, long lda, const T *B, long ldb, float *out, long ld, int M, int N,
                 int K, int bn, uint32_t *status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) throw CudaError("gemm_f32out: empty shape");
  if (N % 4 != 0 || ld % 4 != 0) throw CudaError("gemm_f32out: N and ld must be multiples of 4");
  if (reinterpret_cast<uintptr_t>(out) % 16) throw CudaError("gemm_f32out: out must be 16B aligned");
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  if (bn <= 0) bn = pick_bn_store(M, N, sm_count(dev));
  EpiArgs ea{};
  ea.ldc = ld;
  ea.n_out = N;
  ea.out_f32 = out;
  const CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, kBM, kBK);
  dispatch_bn<kEpiStoreF32>(bn, ta, B, ldb, M, N, K, ea, 0, status, stream, "gemm_f32out");
}

template <typename T>
void gemm_qkv_rope(const T *A, long lda, const T *B, long ldb, T *C, long ldc,
                   const __nv_bfloat16 *bias, int M, int K, int HQ, int HKV, int D,
                   const __nv_bfloat16 *cos_tab, const __nv_bfloat16 *sin_tab,
                   const __nv_bfloat16 *qn, const __nv_bfloat16 *kn, float eps, uint32_t *status,
                   cudaStream_t stream, __half *vt, long ldvt) {
  const int N = (HQ + 2 * HKV) * D;
  if (M <= 0 || K <= 0 || HQ <= 0 || HKV <= 0) throw CudaError("gemm_qkv_rope: empty shape");
  if (D != 64 && D != 128) throw CudaError("gemm_qkv_rope: head_dim must be 64 or 128");
  if (ldc % 8 != 0 || reinterpret_cast<uintptr_t>(C) % 16 ||
      (bias && reinterpret_cast<uintptr_t>(bias) % 16))
    throw CudaError("gemm_qkv_rope: C/bias must be 16-byte aligned, ldc % 8 == 0");
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  // heads must not straddle tiles: 256 or 128 (multiples of D), fewer waves wins
  const int sms = sm_count(dev);
  const long mblk = (M + kBM - 1) / kBM;
  auto cost = [&](int bn) {
    const long tiles = mblk * ((N + bn - 1) / bn);
    return double((tiles + sms - 1) / sms) * double(bn + 16);
  };
  const int bn = cost(256) <= cost(128) ? 256 : 128;
  EpiArgs ea{};
  ea.c = reinterpret_cast<__nv_bfloat16 *>(C);
  ea.ldc = ldc;
  ea.bias = bias;
  ea.n_out = N;
  ea.cos_tab = cos_tab;
  ea.sin_tab = sin_tab;
  ea.qn = qn;
  ea.kn = kn;
  ea.q_cols = HQ * D;
  ea.rope_cols = (HQ + HKV) * D;
  ea.D = D;
  ea.eps = eps;
  ea.vt = vt;
  ea.ldvt = ldvt;
  if (vt && ldvt < M) throw CudaError("gemm_qkv_rope: V^T pitch below the row count");
  const CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, kBM, kBK);
  dispatch_bn<kEpiQkvRope>(bn, ta, B, ldb, M, N, K, ea, 0, status, stream, "gemm_qkv_rope");
}

void gemm_qkv_rope_bf16(const __nv_bfloat16 *A, long lda, const __nv_bfloat16 *B, long ldb,
                        __nv_bfloat16 *C, long ldc, const __nv_bfloat16 *bias, int M, int K,
                        int HQ, int HKV, int D, const __nv_bfloat16 *cos_tab,
                        const __nv_bfloat16 *sin_tab, const __nv_bfloat16 *qn,
                        const __nv_bfloat16 *kn, float eps, uint32_t *status,
                        cudaStream_t stream, __half *vt, long ldvt) {
  gemm_qkv_rope<__nv_bfloat16>(A, lda, B, ldb, C, ldc, bias, M, K, HQ, HKV, D, cos_tab, sin_tab,
                               qn, kn, eps, status, stream, vt, ldvt);
}

template <typename T>
void gemm_silu(const T *A, long lda, const T *Bgu, long ldb, T *act, long ldact, int M,
               int n_out, int K, int bn, int grid_limit, uint32_t *status, cudaStream_t stream) {
  if (M <= 0 || n_out <= 0 || K <= 0) throw CudaError("gemm_silu: empty shape");
  if (n_out % 8 != 0 || ldact % 8 != 0) throw CudaError("gemm_silu: n_out % 8 != 0");
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  if (bn <= 0) bn = pick_bn_silu(M, n_out, sm_count(dev));
  if (bn != 256 && bn != 192 && bn != 128)
    throw CudaError("gemm_silu: unsupported bn " + std::to_string(bn));
  const int half = bn / 2;
  const int nblk = (n_out + half - 1) / half;
  const int n_b_rows = nblk * bn;
  EpiArgs ea{};
  ea.c = reinterpret_cast<__nv_bfloat16 *>(act);
  ea.ldc = ldact;
  ea.n_out = n_out;
  const CUtensorMap ta = make_tmap_2d_bf16(A, M, K, lda, kBM, kBK);
  dispatch_bn<kEpiSiluMul>(bn, ta, Bgu, ldb, M, n_b_rows, K, ea, grid_limit, status, stream,
                           "gemm_silu");
}

void gemm_silu_bf16(const __nv_bfloat16 *A, long lda, const __nv_bfloat16 *Bgu, long ldb,
                    __nv_bfloat16 *act, long ldact, int M, int n_out, int K, int bn,
                    int grid_limit, uint32_t *status, cudaStream_t stream) {
  gemm_silu<__nv_bfloat16>(A, lda, Bgu, ldb, act, ldact, M, n_out, K, bn, grid_limit, status,
                           stream);
}

template void gemm_store<__half>(const __half *, long, const __half *, long, __half *, long,
                                 const __nv_bfloat16 *, int, int, int, int, int, uint32_t *,
                                 cudaStream_t);
template void gemm_f32out<__nv_bfloat16>(const __nv_bfloat16 *, long, const __nv_bfloat16 *, long,
                                         float *, long, int, int, int, int, uint32_t *,
                                         cudaStream_t);
template void gemm_f32out<__half>(const __half *, long, const __half *, long, float *, long, int,
                                  int, int, int, uint32_t *, cudaStream_t);
template void gemm_qkv_rope<__half>(const __half *, long, const __half *, long, __half *, long,
                                    const __nv_bfloat16 *, int, int, int, int, int,
                                    const __nv_bfloat16 *, const __nv_bfloat16 *,
                                    const __nv_bfloat16 *, const __nv_bfloat16 *, float,
                                    uint32_t *, cudaStream_t, __half *, long);
template void gemm_silu<__half>(const __half *, long, const __half *, long, __half *, long, int,
                                int, int, int, int, uint32_t *, cudaStream_t);

}  // namespace krb
