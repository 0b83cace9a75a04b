// Persistent warp-specialised tcgen05 GEMM for sm_100a.
//
//   C[M, N] = A[M, K] . B[N, K]^T        (A, B bf16 K-major; fp32 accumulate in TMEM)
//
// Roles inside one CTA (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: streams 128x64 A tiles and BNx64 B tiles into a
//               STAGES-deep shared-memory ring (128-byte swizzle).
//   warp 1      MMA issuer: one elected thread issues tcgen05.mma (M=128, N=BN,
//               K=16) into one of two TMEM accumulators and commits to mbarriers.
//               Warp 1 also owns the TMEM allocation.
//   warps 2..    epilogue (8 warps in plain GEMMs, 4 in the relay kernel):
//               tcgen05.ld the accumulator (warp w reads TMEM lanes 32*(w%4)..+31 =
//               tile rows; two warps per quadrant split the columns), apply the
//               epilogue, store to HBM, and hand the accumulator back so the next
//               tile's MMAs overlap.
//
// Tiles are visited in "band" order: the output rows are cut into bands of
// `band` 128-row blocks; all tiles of band 0 come first (row blocks fastest),
// then band 1, ...  A plain GEMM uses one band covering all rows.  The relay
// kernel uses one band per row tile of the tp_split schedule so that row tile t
// completes before row tile t+1 starts.
#pragma once

#include "ptx.cuh"
#include "tile_sched.h"

namespace krb {

constexpr int kBM = 128;        // UMMA M (cta_group::1)
constexpr int kBK = 64;         // K per stage: one 128-byte swizzle row of bf16
constexpr int kUmmaK = 16;      // K per tcgen05.mma kind::f16

enum EpiMode : int {
  kEpiStore = 0,    // C = bf16(acc [+ bias])
  kEpiSiluMul = 1,  // C[:, j] = bf16(silu(acc[:, g(j)]) * acc[:, u(j)]), interleaved blocks
  kEpiStoreF32 = 2, // out_f32 = acc (fp32, unrounded; consumed by the residual Add+RMSNorm)
  kEpiQkvRope = 3,  // fused QKV: (+bias), per-head QK-RMSNorm (optional) and RoPE on q, k
};
// Every mode runs with bf16 or fp16 operands (the kernels' F16 parameter); 2-byte
// outputs take the operands' format.

// Configuration variants (second template parameter of every helper below):
//   kCfgPlain    plain GEMM, 8 epilogue warps, 2-byte output staging (bf16 / fp16 outputs)
//   kCfgRelay    the fused relay kernel: 4 epilogue warps, fp32 staging (its own
//                budget: relay row buffers sit behind this layout)
//   kCfgPlainF32 plain GEMM, 8 epilogue warps, fp32 output staging (kEpiStoreF32)
//   kCfgPlain4   plain GEMM, 4 epilogue warps, 2-byte output staging
// Eight epilogue warps (two per TMEM lane quadrant, splitting the tile's columns) cut
// the exposed epilogue of the last tile of GEMMs with two tiles per SM (QKV with its
// RoPE epilogue, o_proj's fp32 output: 3-5 % faster on B200); the SiLU-gated and plain
// stores, with many tiles per SM, ran 1-2 % faster with four.
//   kCfgPair / kCfgPairF32 / kCfgPairRelay: the same three roles on CTA PAIRS (clusters of
//                2, cta_group::2): 256-row tiles, each CTA holding 128 rows of A and BN/2
//                rows of B in its stages, the even CTA issuing the M=256 MMA for both.  Per
//                SM a k-block then moves A 16 KB + B BN*64 B through shared memory (TMA
//                write + MMA read) for the same MMA time as a one-CTA 128 x BN tile, which
//                moves A 16 KB + B BN*128 B: the one-CTA 128x256 tile needs ~190 B/clk of
//                shared-memory traffic at the full MMA rate, the pair ~125 B/clk.
constexpr int kCfgPlain = 0, kCfgRelay = 1, kCfgPlainF32 = 2, kCfgPlain4 = 3, kCfgPair = 4,
              kCfgPairF32 = 5, kCfgPairRelay = 6;

template <int BN, int V = kCfgPlain>
struct GemmCfg {
  static_assert(BN % 16 == 0 && BN >= 32 && BN <= 256, "UMMA N for M=128");
  static constexpr int kCG = V >= kCfgPair ? 2 : 1;  // CTAs per MMA
  static constexpr bool kRelay = V == kCfgRelay || V == kCfgPairRelay;
  static_assert(kCG == 1 || (BN / 2) % 16 == 0, "pair: B halves of whole swizzle atoms");
  static constexpr int kEpiWarps = (kRelay || V == kCfgPlain4) ? 4 : 8;
  static constexpr int kThreads = 64 + 32 * kEpiWarps;
  static constexpr uint32_t kABytes = kBM * kBK * 2;
  static constexpr uint32_t kBBytes = (BN / kCG) * kBK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  // epilogue staging per warp: 32 rows of 32 fp32 padded to 36 (conflict-free
  // row-wise writes and column-block reads), or 32 rows of 32 2-byte values padded to
  // 80 bytes (kCfgPlain)
  static constexpr uint32_t kStageRow = 36;
  static constexpr uint32_t kStage2Pitch = 80;
  static constexpr bool kStage2 = V == kCfgPlain || V == kCfgPlain4 || V == kCfgPair;
  static constexpr uint32_t kWarpEpiBytes = kStage2 ? 32 * kStage2Pitch : 32 * kStageRow * 4;
  static constexpr uint32_t kEpiBytes = kEpiWarps * kWarpEpiBytes;
  // barriers: full[S], empty[S], tfull[2], tempty[2]; then tmem slot + abort flag
  // ... + 16 bytes (tmem slot, abort, flag, relay GEMM-done) + 64 bytes of relay scratch (pair sums)
  static constexpr uint32_t kMaxStages = (kCG == 2 || BN < 224) ? 6 : 4;
  static constexpr uint32_t kBarBytesMax = (2 * 6 + 4) * 8 + 16 + 64;
  // the relay's pair row buffers (up to H = 4096) and their barriers sit behind this layout
  static constexpr uint32_t kReserve = V == kCfgPairRelay ? 4u * 4096u * 2u + 256u : 0u;
  static constexpr uint32_t kFit =
      (232448u - kReserve - kEpiBytes - kBarBytesMax - 1024u) / kStageBytes;
  static constexpr uint32_t kStages = V == kCfgRelay ? kMaxStages
                                                     : (kFit < kMaxStages ? kFit : kMaxStages);
  static constexpr uint32_t kTileBytes = kStages * kStageBytes;
  // TMEM accumulator spacing (power of two) and total allocation.
  static constexpr uint32_t kAccStride = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr uint32_t kTmemCols = 2 * kAccStride;
  static constexpr uint32_t kBarBytes = (2 * kStages + 4) * 8 + 16 + 64;
  static constexpr uint32_t kSmemBytes =
      kTileBytes + kEpiBytes + kBarBytes + 1024;  // +1024 alignment slack
  static_assert(kStages >= 3, "pipeline depth");
  static_assert(kABytes % 1024 == 0 && kBBytes % 1024 == 0, "swizzle atoms");
  static_assert(kSmemBytes <= 232448, "shared memory budget");
};

template <int BN, int RELAY = 0>
struct GemmSmemView {
  uint8_t *tiles;
  uint64_t *full;
  uint64_t *empty;
  uint64_t *tfull;
  uint64_t *tempty;
  uint32_t *tmem_slot;
  volatile int *abort;
  float *epi;  // kEpiWarps staging chunks of kWarpEpiBytes (epilogue warps)
  float *scratch;  // 16 floats for the relay warps
  __device__ __forceinline__ static GemmSmemView carve(uint8_t *raw) {
    using C = GemmCfg<BN, RELAY>;
    GemmSmemView v;
    uint8_t *base = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) &
                                                ~uintptr_t(1023));
    v.tiles = base;
    v.epi = reinterpret_cast<float *>(base + C::kTileBytes);
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + C::kTileBytes + C::kEpiBytes);
    v.full = bars;
    v.empty = bars + C::kStages;
    v.tfull = bars + 2 * C::kStages;
    v.tempty = bars + 2 * C::kStages + 2;
    v.tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * C::kStages + 4);
    v.abort = reinterpret_cast<volatile int *>(v.tmem_slot + 1);
    v.scratch = reinterpret_cast<float *>(v.tmem_slot + 4);
    return v;
  }
};

// One-time CTA setup: barriers by thread 0, TMEM by warp 1.  Ends with
// __syncthreads so every role sees the TMEM base address.
// Pairs: the leader's tempty counts the epilogue threads of BOTH CTAs, and a cluster
// barrier makes every barrier initialisation visible to the peer before any remote arrive
// or TMA completion; warp 1 of both CTAs allocates the pair's TMEM together.
template <int BN, int RELAY = 0>
__device__ __forceinline__ void gemm_setup(const GemmSmemView<BN, RELAY> &s, int epi_threads) {
  using C = GemmCfg<BN, RELAY>;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kStages; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.tfull[i], 1);
      mbar_init(&s.tempty[i], C::kCG * epi_threads);
    }
    s.abort[0] = 0;
    s.abort[2] = 0;  // relay kernel: "this CTA's GEMM is done" (the pipeline buffers are free)
    fence_mbar_init();
  }
  if (warp == 1) {
    if constexpr (C::kCG == 2) {
      tmem_alloc_pair(s.tmem_slot, C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(s.tmem_slot, C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  if constexpr (C::kCG == 2) cluster_sync();
  tc_fence_after();
}

template <int BN, int RELAY = 0>
__device__ __forceinline__ void gemm_teardown(const GemmSmemView<BN, RELAY> &s) {
  using C = GemmCfg<BN, RELAY>;
  tc_fence_before();
  __syncthreads();
  // pairs: neither CTA leaves (or frees TMEM) while the other may still signal its
  // barriers or the leader's MMAs may still touch its shared memory or TMEM
  if constexpr (C::kCG == 2) cluster_sync();
  tc_fence_after();
  if ((threadIdx.x >> 5) == 1) {
    if constexpr (C::kCG == 2)
      tmem_dealloc_pair(*s.tmem_slot, C::kTmemCols);
    else
      tmem_dealloc(*s.tmem_slot, C::kTmemCols);
  }
}

// Tile loop of this CTA: one-CTA kernels step over CTAs, pairs over clusters (both CTAs
// of a cluster take the same tiles).  row_block(mb) = this CTA's 128-row block of tile row
// mb (tile rows are 256 rows for pairs).
template <int CG>
struct TileWalk {
  int first, step, rank;
  __device__ __forceinline__ static TileWalk make() {
    TileWalk w;
    if constexpr (CG == 2) {
      w.first = int(cluster_id_x());
      w.step = int(nclusters_x());
      w.rank = int(cluster_ctarank());
    } else {
      w.first = blockIdx.x;
      w.step = gridDim.x;
      w.rank = 0;
    }
    return w;
  }
  __device__ __forceinline__ int row_block(int mb) const { return CG == 2 ? 2 * mb + rank : mb; }
};

// ---- warp 0, one thread: TMA producer
template <int BN, int RELAY = 0>
__device__ __forceinline__ void gemm_producer(const GemmSmemView<BN, RELAY> &s, const CUtensorMap *ta,
                                              const CUtensorMap *tb, const CUtensorMap *tb2,
                                              const TileSched &ts, int K, uint32_t *status) {
  using C = GemmCfg<BN, RELAY>;
  const int nkb = (K + kBK - 1) / kBK;
  int stage = 0;
  uint32_t phase = 0;
  long issued = 0;
  const uint64_t pol_a = l2_policy_evict_last();
  const TileWalk<C::kCG> w = TileWalk<C::kCG>::make();
  // pairs: every load of both CTAs completes on the leader's full[stage]
  const uint32_t leader_full = C::kCG == 2 ? mapa_shared(&s.full[0], 0) : 0u;
  for (int t = w.first; t < ts.total() && !*s.abort; t += w.step) {
    int mb, n0, bn;
    ts.tile(t, mb, n0, bn);
    const bool narrow = bn != BN;  // phase-2 tile: B rows through the bn2-row tensor map
    // bytes of one stage: this CTA's A rows and B rows (pairs: both CTAs' on the leader)
    const uint32_t stage_tx = C::kCG * (C::kABytes + uint32_t(bn / C::kCG) * kBK * 2);
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(&s.empty[stage], phase ^ 1, kMbarLimitNs) || *s.abort) {
        report_status(status, kStatusTmaWait);
        *s.abort = 1;
        goto drain;
      }
      {
        uint8_t *a = s.tiles + stage * C::kStageBytes;
        uint8_t *b = a + C::kABytes;
        if constexpr (C::kCG == 2) {
          if (w.rank == 0) mbar_arrive_expect_tx(&s.full[stage], stage_tx);
          const uint32_t bar = leader_full + 8u * uint32_t(stage);
          tma_load_2d_pair(a, ta, bar, kb * kBK, w.row_block(mb) * kBM, pol_a);
          tma_load_2d_pair(b, narrow ? tb2 : tb, bar, kb * kBK, n0 + w.rank * (bn / 2),
                           l2_policy_evict_first());
        } else {
          mbar_arrive_expect_tx(&s.full[stage], stage_tx);
          tma_load_2d_hint(a, ta, &s.full[stage], kb * kBK, mb * kBM, pol_a);
          tma_load_2d(b, narrow ? tb2 : tb, &s.full[stage], kb * kBK, n0);
        }
      }
      ++issued;
      if (++stage == C::kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
  }
drain:
  // Make sure no TMA write is still in flight into this CTA's shared memory
  // before the CTA can exit: wait on the last phase armed for each stage.  (Pairs: the
  // leader's full barriers count both CTAs' bytes, so the leader waits for both; the
  // peer is held at the teardown's cluster barrier until then.)
  if (C::kCG == 2 && w.rank != 0) return;
  {
    const long n = issued < C::kStages ? issued : C::kStages;
    int st = stage;
    uint32_t ph = phase;
    for (long i = 0; i < n; ++i) {
      if (st == 0) {
        st = C::kStages - 1;
        ph ^= 1;
      } else {
        --st;
      }
      mbar_wait(&s.full[st], ph, kMbarLimitNs / 4);
    }
  }
}

// ---- warp 1, one thread: tcgen05.mma issuer
// F16 selects fp16 operands (both A and B) instead of bf16.
template <int BN, int RELAY = 0, bool F16 = false>
__device__ __forceinline__ void gemm_mma(const GemmSmemView<BN, RELAY> &s, const TileSched &ts,
                                         int K, uint32_t *status) {
  using C = GemmCfg<BN, RELAY>;
  constexpr int kM = kBM * C::kCG;  // pairs: one M = 256 MMA for both CTAs
  constexpr uint32_t idesc1 = F16 ? idesc_f16_f32(kM, BN) : idesc_bf16_f32(kM, BN);
  const uint32_t idesc2 = F16 ? idesc_f16_f32(kM, ts.bn2) : idesc_bf16_f32(kM, ts.bn2);
  const uint32_t tmem = *s.tmem_slot;
  const int nkb = (K + kBK - 1) / kBK;
  int stage = 0;
  uint32_t phase = 0;
  int it = 0;
  const TileWalk<C::kCG> w = TileWalk<C::kCG>::make();
  if (w.rank != 0) return;  // pairs: the leader issues every MMA
  for (int t = w.first; t < ts.total(); t += w.step, ++it) {
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    const uint32_t idesc = t < ts.p1 ? idesc1 : idesc2;
    if (!mbar_wait(&s.tempty[acc], acc_phase ^ 1, kMbarLimitNs) || *s.abort) {
      report_status(status, kStatusMmaWait);
      *s.abort = 1;
      break;
    }
    tc_fence_after();
    const uint32_t d = tmem + acc * C::kAccStride;
    bool ok = true;
    for (int kb = 0; kb < nkb; ++kb) {
      if (!mbar_wait(&s.full[stage], phase, kMbarLimitNs) || *s.abort) {
        report_status(status, kStatusMmaWait);
        *s.abort = 1;
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t a = smem_u32(s.tiles + stage * C::kStageBytes);
      const uint32_t b = a + C::kABytes;
#pragma unroll
      for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
        if constexpr (C::kCG == 2)
          umma_pair(d, sdesc_kmajor_sw128(a + kk * kUmmaK * 2),
                    sdesc_kmajor_sw128(b + kk * kUmmaK * 2), idesc, (kb | kk) != 0);
        else
          umma_bf16(d, sdesc_kmajor_sw128(a + kk * kUmmaK * 2),
                    sdesc_kmajor_sw128(b + kk * kUmmaK * 2), idesc, (kb | kk) != 0);
      }
      // pairs: the stage is free in both CTAs once these MMAs completed
      if constexpr (C::kCG == 2)
        umma_commit_pair(&s.empty[stage], 0x3);
      else
        umma_commit(&s.empty[stage]);
      if (++stage == C::kStages) {
        stage = 0;
        phase ^= 1;
      }
    }
    if constexpr (C::kCG == 2)
      umma_commit_pair(&s.tfull[acc], 0x3);  // both CTAs' epilogues
    else
      umma_commit(&s.tfull[acc]);
    if (!ok) break;
  }
}

// Epilogue helpers -----------------------------------------------------------
__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// Store 32 fp32 values as bf16 at dst (16-byte aligned when full).
__device__ __forceinline__ void store_row32_bf16(__nv_bfloat16 *dst, const float *v, int valid) {
  if (valid >= 32) {
    uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      uint4 w;
      w.x = pack_bf16x2(v[q * 8 + 0], v[q * 8 + 1]);
      w.y = pack_bf16x2(v[q * 8 + 2], v[q * 8 + 3]);
      w.z = pack_bf16x2(v[q * 8 + 4], v[q * 8 + 5]);
      w.w = pack_bf16x2(v[q * 8 + 6], v[q * 8 + 7]);
      d4[q] = w;
    }
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (j < valid) dst[j] = __float2bfloat16_rn(v[j]);
  }
}

struct EpiArgs {
  __nv_bfloat16 *c;           // output
  long ldc;                   // output row pitch (elements)
  const __nv_bfloat16 *bias;  // [N] or null (kEpiStore, kEpiQkvRope)
  int n_out;                  // valid output columns
  float *out_f32;             // kEpiStoreF32: output [M, ldc] fp32
  // kEpiQkvRope: heads of D columns; columns [0, q_cols) are q heads, [q_cols,
  // rope_cols) k heads (normalised with qn / kn when non-null, then rotated), the
  // rest v heads (bias only).  cos / sin: bf16 [max_pos, D], position = row.
  const __nv_bfloat16 *cos_tab, *sin_tab, *qn, *kn;
  int q_cols, rope_cols, D;
  float eps;
  // kEpiQkvRope, optional: the v heads also go out transposed in fp16 for the attention,
  // vt[(col - rope_cols) * ldvt + row] = fp16(bf16(v)) (null: not written)
  __half *vt;
  long ldvt;
};

// The accumulator chunk a warp holds is row-per-thread (thread = TMEM lane = row,
// 32 consecutive columns).  Writing that straight to HBM gives 32 scattered
// 16-byte pieces per instruction.  Instead each warp stages the 32 x 32 fp32
// chunk in its own padded shared-memory block and writes it back row-contiguous:
// 64 bytes per row for bf16 outputs (4 lanes per row), 128 bytes per row for fp32
// outputs (8 lanes per row).  Padding rows to 36 floats keeps both the row-wise
// writes and the column-block reads free of bank conflicts.
__device__ __forceinline__ void epi_stage_put(float *stage, const float *v) {
  const int lane = threadIdx.x & 31;
  float4 *row = reinterpret_cast<float4 *>(stage + lane * 36);
#pragma unroll
  for (int q = 0; q < 8; ++q) row[q] = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __syncwarp();
}

// bf16 write-back: lane l covers row (l/4 + 8*it) columns [8*(l%4), +8).  F16 rounds to
// fp16 instead (same 2-byte layout; the row pointers then address an fp16 matrix).
template <bool F16 = false, typename RowPtr>
__device__ __forceinline__ void epi_stage_store_bf16(const float *stage, RowPtr row_ptr,
                                                     const __nv_bfloat16 *bias, int col0,
                                                     int valid_cols) {
  const int lane = threadIdx.x & 31;
  const int piece = lane & 3;
  const int c = piece * 8;
  float b[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (bias && c < valid_cols) {
    const uint4 w = __ldg(reinterpret_cast<const uint4 *>(bias + col0 + c));
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 f = unpack_bf16x2(ws[e]);
      b[2 * e] = f.x;
      b[2 * e + 1] = f.y;
    }
  }
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane >> 2);
    const float4 x = *reinterpret_cast<const float4 *>(stage + r * 36 + c);
    const float4 y = *reinterpret_cast<const float4 *>(stage + r * 36 + c + 4);
    __nv_bfloat16 *dst = row_ptr(r);
    if (dst && c < valid_cols) {
      uint4 w;
      if constexpr (F16) {
        w.x = pack_f16x2(x.x + b[0], x.y + b[1]);
        w.y = pack_f16x2(x.z + b[2], x.w + b[3]);
        w.z = pack_f16x2(y.x + b[4], y.y + b[5]);
        w.w = pack_f16x2(y.z + b[6], y.w + b[7]);
      } else {
        w.x = pack_bf16x2(x.x + b[0], x.y + b[1]);
        w.y = pack_bf16x2(x.z + b[2], x.w + b[3]);
        w.z = pack_bf16x2(y.x + b[4], y.y + b[5]);
        w.w = pack_bf16x2(y.z + b[6], y.w + b[7]);
      }
      *reinterpret_cast<uint4 *>(dst + col0 + c) = w;
    }
  }
  __syncwarp();
}

// fp32 write-back: lane l covers row (l/8 + 4*it) columns [4*(l%8), +4), i.e. 128
// contiguous bytes per row and instruction group.  Store-only: an epilogue that
// also reads HBM (e.g. a residual) holds the TMEM accumulator for a full memory
// latency per chunk and throttles the MMA.
__device__ __forceinline__ void epi_stage_store_f32(const float *stage, float *out, long ld,
                                                    int row0, int M, int col0, int valid_cols) {
  const int lane = threadIdx.x & 31;
  const int c = (lane & 7) * 4;
#pragma unroll
  for (int it = 0; it < 8; ++it) {
    const int r = it * 4 + (lane >> 3);
    const int grow = row0 + r;
    if (grow < M && c < valid_cols) {
      const float4 a = *reinterpret_cast<const float4 *>(stage + r * 36 + c);
      *reinterpret_cast<float4 *>(out + static_cast<size_t>(grow) * ld + col0 + c) = a;
    }
  }
  __syncwarp();
}

// ---- kEpiQkvRope: fused QKV epilogue (one thread = one output row = one position)
// For every q / k head of the tile: v = acc + bias; with QK-norm, the head's
// RMSNorm over D (sum of squares from a first pass over TMEM; the normalised value
// times the weight is rounded to bf16 as HF's Qwen3 RMSNorm returns bf16); then
// rotate-half RoPE with the bf16 cos / sin tables of this row's position:
//   out[d] = v[d] cos[d] - v[d + D/2] sin[d],  out[d + D/2] = v[d + D/2] cos[d + D/2] + v[d] sin[d + D/2]
// (same math as qk_norm_rope_kernel, without rounding q / k to bf16 before it).
// v heads only get the bias.  Needs BN % D == 0 (heads never straddle tiles).
__device__ __forceinline__ void epi_load32(uint32_t taddr, const __nv_bfloat16 *bias, int col,
                                           float *v) {
  uint32_t r[32];
  tmem_ld_32x32(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
  if (bias) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 w = __ldg(reinterpret_cast<const uint4 *>(bias + col) + q);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = unpack_bf16x2(ws[e]);
        v[q * 8 + 2 * e] += f.x;
        v[q * 8 + 2 * e + 1] += f.y;
      }
    }
  }
}

__device__ __forceinline__ void unpack8_f(const uint4 &w, float *f) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 t = unpack_bf16x2(ws[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

// 2-byte write-back through the warp's staging block (kCfgPlain): each thread packs
// its row's 32 values (this 32-column chunk, + bias) into 64 bytes at row pitch 80 B;
// then lane l stores rows (l % 8) + 8 * it, 16-byte piece l / 8 (a quarter-warp reads
// 8 rows of one piece: conflict-free, as are the row-wise writes).  row_ptr(r) gives
// the output row (or null past M); valid = output columns left in this chunk (a
// multiple of 8 by the callers' checks).
template <bool F16, typename RowPtr>
__device__ __forceinline__ void epi2_store(uint8_t *stage2, float *v, const __nv_bfloat16 *bias,
                                           RowPtr row_ptr, int col0, int valid) {
  const int lane = threadIdx.x & 31;
  if (bias) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      if (q * 8 < valid) {
        const uint4 w = __ldg(reinterpret_cast<const uint4 *>(bias + col0) + q);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = unpack_bf16x2(ws[e]);
          v[q * 8 + 2 * e] += f.x;
          v[q * 8 + 2 * e + 1] += f.y;
        }
      }
    }
  }
  uint4 *srow = reinterpret_cast<uint4 *>(stage2 + lane * 80);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = pack2<F16>(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = pack2<F16>(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = pack2<F16>(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = pack2<F16>(v[q * 8 + 6], v[q * 8 + 7]);
    srow[q] = w;
  }
  __syncwarp();
  const int piece = lane >> 3;
#pragma unroll
  for (int it = 0; it < 4; ++it) {
    const int r = it * 8 + (lane & 7);
    const uint4 w = *reinterpret_cast<const uint4 *>(stage2 + r * 80 + piece * 16);
    __nv_bfloat16 *dst = row_ptr(r);
    if (dst && piece * 8 < valid) *reinterpret_cast<uint4 *>(dst + col0 + piece * 8) = w;
  }
  __syncwarp();
}

// ---- kEpiQkvRope: fused QKV epilogue (one thread = one output row = one position)
// For every q / k head of the tile: v = acc + bias; with QK-norm, the head's
// RMSNorm over D (sum of squares from a first pass over TMEM; the normalised value
// times the weight is rounded to bf16 as HF's Qwen3 RMSNorm returns bf16, for bf16
// outputs); then rotate-half RoPE with the bf16 cos / sin tables of this row's position:
//   out[d] = v[d] cos[d] - v[d + D/2] sin[d],  out[d + D/2] = v[d + D/2] cos[d + D/2] + v[d] sin[d + D/2]
// (same math as qk_norm_rope_kernel, without rounding q / k before it).
// v heads only get the bias.  Needs BN % D == 0 (heads never straddle tiles).  The
// tile's heads are shared between the NG column groups of epilogue warps: group grp
// takes heads grp, grp + NG, ...
template <int BN, bool F16, typename RowPtr>
__device__ __forceinline__ void epi_qkv_rope(uint32_t tbase, uint8_t *stage2, RowPtr out_row,
                                             const EpiArgs &ea, int row, bool row_ok, int n0,
                                             int grp, int NG) {
  const int D = ea.D, half = D / 2, nch = D / 32;
#pragma unroll 1
  for (int h0 = grp * D; h0 < BN; h0 += NG * D) {
    const int hcol = n0 + h0;  // first column of this head
    if (hcol >= ea.n_out) break;    // warp-uniform
    if (hcol >= ea.rope_cols) {
      // v head: bias only; with ea.vt also transposed (lanes = 32 consecutive rows, so
      // each store instruction writes 64 contiguous bytes of one V^T row)
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        float v[32];
        epi_load32(tbase + h0 + c * 32, ea.bias, hcol + c * 32, v);
        if (ea.vt && row_ok) {
          __half *dst = ea.vt + static_cast<long>(hcol - ea.rope_cols + c * 32) * ea.ldvt + row;
#pragma unroll
          for (int j = 0; j < 32; ++j) dst[static_cast<long>(j) * ea.ldvt] = __float2half_rn(round2<F16>(v[j]));
        }
        epi2_store<F16>(stage2, v, nullptr, out_row, hcol + c * 32, ea.n_out - hcol - c * 32);
      }
      continue;
    }
    const __nv_bfloat16 *nw = hcol < ea.q_cols ? ea.qn : ea.kn;
    float rn = 1.f;
    if (nw) {
      float ss = 0.f;
#pragma unroll 1
      for (int c = 0; c < nch; ++c) {
        float v[32];
        epi_load32(tbase + h0 + c * 32, ea.bias, hcol + c * 32, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) ss += v[j] * v[j];
      }
      rn = rsqrtf(ss / float(D) + ea.eps);
    }
    const __nv_bfloat16 *ct = ea.cos_tab + size_t(row) * D;
    const __nv_bfloat16 *st = ea.sin_tab + size_t(row) * D;
#pragma unroll 1
    for (int c = 0; c < nch / 2; ++c) {
      const int dlo = c * 32, dhi = half + c * 32;
      float lo[32], hi[32];
      epi_load32(tbase + h0 + dlo, ea.bias, hcol + dlo, lo);
      epi_load32(tbase + h0 + dhi, ea.bias, hcol + dhi, hi);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float wl[8], wh[8], cl[8], sl[8], ch[8], sh[8];
        unpack8_f(__ldg(reinterpret_cast<const uint4 *>(ct + dlo) + q), cl);
        unpack8_f(__ldg(reinterpret_cast<const uint4 *>(st + dlo) + q), sl);
        unpack8_f(__ldg(reinterpret_cast<const uint4 *>(ct + dhi) + q), ch);
        unpack8_f(__ldg(reinterpret_cast<const uint4 *>(st + dhi) + q), sh);
        if (nw) {
          unpack8_f(__ldg(reinterpret_cast<const uint4 *>(nw + dlo) + q), wl);
          unpack8_f(__ldg(reinterpret_cast<const uint4 *>(nw + dhi) + q), wh);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float a = lo[q * 8 + e], b = hi[q * 8 + e];
          if (nw) {
            // bf16 outputs keep HF Qwen3's bf16 rounding of the normed head; fp16 ones
            // round once, at the store
            a = a * rn * wl[e];
            b = b * rn * wh[e];
            if constexpr (!F16) {
              a = bf16_round(a);
              b = bf16_round(b);
            }
          }
          lo[q * 8 + e] = a * cl[e] - b * sl[e];
          hi[q * 8 + e] = b * ch[e] + a * sh[e];
        }
      }
      epi2_store<F16>(stage2, lo, nullptr, out_row, hcol + dlo, 32);
      epi2_store<F16>(stage2, hi, nullptr, out_row, hcol + dhi, 32);
    }
  }
}

// ---- warps 2..: the plain GEMM's epilogue (kEpiStore / kEpiSiluMul / kEpiStoreF32 /
// kEpiQkvRope).  Warp w reads TMEM lane quadrant w % 4 (rows); with 8 warps the two
// warps of a quadrant split the tile's 32-column chunks (or heads) between them: group
// (w - 2) / 4 takes chunks grp, grp + 2, ...  F16: fp16 operands and 2-byte outputs in
// fp16 instead of bf16.
template <int BN, int V, int MODE, bool F16 = false>
__device__ __forceinline__ void gemm_epilogue(const GemmSmemView<BN, V> &s, const TileSched &ts,
                                              int M, const EpiArgs &ea, uint32_t *status) {
  using C = GemmCfg<BN, V>;
  constexpr int NG = C::kEpiWarps / 4;  // column groups
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quad = warp & 3;
  const int grp = (warp - 2) / 4;
  const uint32_t tmem = *s.tmem_slot;
  uint8_t *stage_raw = reinterpret_cast<uint8_t *>(s.epi) + (warp - 2) * C::kWarpEpiBytes;
  float *stage = reinterpret_cast<float *>(stage_raw);
  int it = 0;
  const TileWalk<C::kCG> w = TileWalk<C::kCG>::make();
  // the accumulator is handed back to the MMA issuer: the leader's tempty (pairs: both
  // CTAs' epilogue threads arrive there)
  const uint32_t leader_tempty = C::kCG == 2 ? mapa_shared(&s.tempty[0], 0) : 0u;
  for (int t = w.first; t < ts.total(); t += w.step, ++it) {
    int mb, n0, bn;
    ts.tile(t, mb, n0, bn);
    mb = w.row_block(mb);
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    if (!mbar_wait(&s.tfull[acc], acc_phase, kMbarLimitNs) || *s.abort) {
      report_status(status, kStatusEpiWait);
      *s.abort = 1;
      break;
    }
    tc_fence_after();
    const int row0 = mb * kBM + quad * 32;
    const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + acc * C::kAccStride;
    auto out_row = [&](int r) -> __nv_bfloat16 * {
      return (row0 + r < M) ? ea.c + static_cast<long>(row0 + r) * ea.ldc : nullptr;
    };
    if constexpr (MODE == kEpiQkvRope) {
      static_assert(C::kStage2, "2-byte staging");
      // rows past M are not stored; clamp their table position
      const int erow = mb * kBM + quad * 32 + lane;
      epi_qkv_rope<BN, F16>(tbase, stage_raw, out_row, ea, min(erow, M - 1), erow < M, n0, grp, NG);
    } else if constexpr (MODE == kEpiStore || MODE == kEpiStoreF32) {
#pragma unroll 1
      for (int c = grp; c * 32 < bn; c += NG) {
        const int col0 = n0 + c * 32;
        if (col0 >= ea.n_out) break;  // warp-uniform
        const int valid = min(bn - c * 32, ea.n_out - col0);
        uint32_t r[32];
        tmem_ld_32x32(tbase + c * 32, r);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
        if constexpr (MODE == kEpiStore) {
          static_assert(C::kStage2, "2-byte staging");
          epi2_store<F16>(stage_raw, v, ea.bias, out_row, col0, valid);
        } else {
          static_assert(!C::kStage2, "fp32 staging");
          epi_stage_put(stage, v);
          epi_stage_store_f32(stage, ea.out_f32, ea.ldc, row0, M, col0, valid);
        }
      }
    } else {
      static_assert(C::kStage2, "2-byte staging");
      constexpr int HALF = BN / 2;
      static_assert(HALF % 32 == 0, "silu epilogue needs BN/2 % 32 == 0");
#pragma unroll 1
      for (int c = grp; c < HALF / 32; c += NG) {
        const int col0 = n0 / 2 + c * 32;
        if (col0 >= ea.n_out) break;
        uint32_t g[32], u[32];
        tmem_ld_32x32(tbase + c * 32, g);
        tmem_ld_32x32(tbase + HALF + c * 32, u);
        tmem_wait_ld();
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j)
          v[j] = silu_f(__uint_as_float(g[j])) * __uint_as_float(u[j]);
        epi2_store<F16>(stage_raw, v, nullptr, out_row, col0, ea.n_out - col0);
      }
    }
    tc_fence_before();
    if constexpr (C::kCG == 2)
      mbar_arrive_cluster(leader_tempty + 8u * uint32_t(acc));
    else
      mbar_arrive(&s.tempty[acc]);
  }
}

}  // namespace krb
