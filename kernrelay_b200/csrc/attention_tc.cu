// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Replaces aclnnFlashAttentionScore (BSND, sparse_mode 3, scale 1/sqrt(D);
// qwen_main.cpp:591-614) for head_dim 128.  One CTA = one query head x 128
// query rows; it walks the 128-key blocks 0..diagonal:
//
//   warp 0      TMA: Q once (2 x 64-column chunks, 128-byte swizzle); K blocks
//               from the fused qkv buffer and V^T blocks from a transposed copy
//               of V ([kv_head * D + d][key]), double-buffered.
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T into TMEM (two S buffers),
//               then O += P_{j-1} V_{j-1} with P read from TMEM (the "TS" form).
//               QK^T of block j is issued before PV of block j-1 so the tensor
//               pipe has work while the softmax of j-1 finishes.
//   warps 2..5  softmax: thread = query row = TMEM lane.  Loads the 128 scores of
//               its row, applies the causal mask, keeps the running max and sum
//               in fp32 (log2 domain), writes P (bf16, rounded; the row sum uses
//               the rounded values) into TMEM, rescales the O row in TMEM when
//               the running max grew, and finally normalises O and stores bf16.
//
// Every operand is K-major with the same 128-byte-swizzle descriptor: Q [row][d],
// K [key][d], V^T [d][key] and P [row][key] (TMEM: lane = row, 2 keys per column).
// All waits are bounded (status bits as in the GEMM).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <string>

#include "common.h"
#include "ptx.cuh"

namespace krb {

namespace {

constexpr int kAttnThreads = 192;
constexpr int kTileRows = 128;       // query rows per CTA = keys per block
constexpr uint32_t kChunkBytes = 128 * 128;  // 128 rows x 64 bf16 (one swizzle width)
constexpr uint32_t kTileBytes = 2 * kChunkBytes;  // 128 rows x 128 bf16
// TMEM columns
constexpr uint32_t kColS0 = 0, kColS1 = 128, kColO = 256, kColP = 384, kTmemCols = 512;

struct AttnSmem {
  uint8_t *q;  // K stage s at q + (1 + s) * kTileBytes, V^T stage s at q + (3 + s) * kTileBytes
  uint64_t *q_full, *kv_full, *kv_empty, *s_full, *s_free, *p_ready, *o_done;
  uint32_t *tmem_slot;
};

__device__ __forceinline__ AttnSmem carve(uint8_t *raw) {
  AttnSmem a;
  uint8_t *base =
      reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  a.q = base;
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + 5 * kTileBytes);
  a.q_full = bars;
  a.kv_full = bars + 1;   // [2]
  a.kv_empty = bars + 3;  // [2]
  a.s_full = bars + 5;    // [2]
  a.s_free = bars + 7;    // [2]
  a.p_ready = bars + 9;
  a.o_done = bars + 10;
  a.tmem_slot = reinterpret_cast<uint32_t *>(bars + 11);
  return a;
}

__device__ __forceinline__ uint8_t *k_stage(const AttnSmem &a, int st) {
  return a.q + (1 + st) * kTileBytes;
}
__device__ __forceinline__ uint8_t *v_stage(const AttnSmem &a, int st) {
  return a.q + (3 + st) * kTileBytes;
}

constexpr uint32_t kAttnSmemBytes = 5 * kTileBytes + 11 * 8 + 16 + 1024;

// descriptor of k-step kk (16 elements) of a 128 x 128 K-major tile stored as two
// 64-element chunks of 128 rows (128-byte swizzle)
__device__ __forceinline__ uint64_t tile_desc(const uint8_t *tile, int kk) {
  return sdesc_kmajor_sw128(smem_u32(tile) + (kk >> 2) * kChunkBytes + (kk & 3) * 32);
}

__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st_32x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16,"
      " %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
      "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
      "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2^x with the MUFU.EX2 instruction (flush-to-zero; the probabilities are rounded
// to bf16 right after, so its ~2 ulp fp32 error is far below that rounding)
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA pipe, to share the softmax's exponentials with the MUFU unit:
// Cody-Waite style range reduction x = n + f, n = round(x) (by the 1.5*2^23
// shift), f in [-1/2, 1/2], and a cubic for 2^f fitted here by weighted least
// squares for relative error on Chebyshev nodes (max relative error 2.2e-4,
// a tenth of the bf16 rounding the probabilities get next); n is added to the
// exponent field.  x < -125 gives exactly 0 (masked scores are -inf).
__device__ __forceinline__ float exp2_poly(float x) {
  const float xc = fmaxf(x, -125.0f);
  const float t = xc + 12582912.0f;  // 1.5 * 2^23: round(xc) in the low mantissa bits
  const float n = t - 12582912.0f;
  const float f = xc - n;
  const float p = fmaf(fmaf(fmaf(0.05286743491888046f, f, 0.2421518862247467f), f,
                            0.6935867667198181f),
                       f, 0.9999627470970154f);
  const int e = (__float_as_int(t) - __float_as_int(12582912.0f)) << 23;
  const float r = __int_as_float(__float_as_int(p) + e);
  return x < -125.0f ? 0.0f : r;
}

// the running max is only moved (and O rescaled) when a row's max grew by more
// than 2^8: until then P = 2^(s - m_stale) <= 256 stays exact enough in bf16 and
// O and the row sum carry the same stale max, so O / l is unchanged
constexpr float kRescaleLog2 = 8.0f;

__device__ __forceinline__ void tmem_st_32x32_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0],"
      " {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// ---------------------------------------------------------------- two-tile kernel
// One CTA = one query head x two consecutive 128-row query tiles (A = q-block 2i,
// B = 2i+1), 10 warps:
//   warp 0      TMA: Q_A, Q_B once; K_j / V^T_j double-buffered (shared by both tiles)
//   warp 1      MMA issuer: per key block j: QK(A,j), QK(B,j), PV(A,j), PV(B,j).  QK(X,j)
//               waits for PV(X,j-1) (S and P of a tile share TMEM columns), so while
//               one tile's softmax runs, the tensor pipe works on the other tile.
//   warps 2..5  softmax of tile A, warps 6..9 softmax of tile B (thread = row).
// TMEM (512 columns): tile X's S at 256X (P written over its first 64 columns as
// packed bf16 pairs once read), O at 256X + 128.  The softmax reads S twice
// (row max, then exp and P) so a thread holds 32 scores at a time.
constexpr int kAttn2Threads = 320;
constexpr uint32_t kAttn2SmemBytes = 6 * kTileBytes + 12 * 8 + 16 + 1024;

struct Attn2Smem {
  uint8_t *q;  // Q_A, Q_B; K stage s at q + (2 + s) * kTileBytes; V^T stage s at q + (4 + s) * kTileBytes
  uint64_t *q_full, *kv_full, *kv_empty, *s_full, *p_ready, *o_done;  // [1], [2], [2], [2], [2], [2]
  uint32_t *tmem_slot;
};

__device__ __forceinline__ Attn2Smem carve2(uint8_t *raw) {
  Attn2Smem a;
  uint8_t *base =
      reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  a.q = base;
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + 6 * kTileBytes);
  a.q_full = bars;
  a.kv_full = bars + 1;
  a.kv_empty = bars + 3;
  a.s_full = bars + 5;
  a.p_ready = bars + 7;
  a.o_done = bars + 9;
  a.tmem_slot = reinterpret_cast<uint32_t *>(bars + 11);
  return a;
}

// One key block of the two-tile kernel's softmax for one row (thread): row max
// (pass 1), lazy O rescale, P = 2^(s*scale - m) rounded to bf16 written over S's
// first 64 columns (pass 2; chunk c's P lands on columns already read), and the
// running max / sum update.  The chunk loops stay rolled (code size).
template <bool kMask>
__device__ __forceinline__ void attn2_softmax_block(uint32_t s_col, uint32_t o_col, int key0,
                                                    int row, int S, float scale_log2, bool has_o,
                                                    float &m_run, float &l_run) {
  float m8[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) m8[e] = -INFINITY;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld_32x32(s_col + c * 32, r);
    tmem_wait_ld();
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      float v = __uint_as_float(r[e]);
      if constexpr (kMask) {
        const int key = key0 + c * 32 + e;
        v = ((key > row) | (key >= S)) ? -INFINITY : v;
      }
      m8[e & 7] = fmaxf(m8[e & 7], v);
    }
  }
  const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                         fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * scale_log2;
  const bool grow = mx - m_run > kRescaleLog2;  // true on the first block (m_run = -inf)
  const float m_use = grow ? mx : m_run;
  const float alpha = grow ? ex2_approx(m_run - mx) : 1.f;
  // PV of the previous block is complete (the commit that released this S covers it)
  if (has_o && __any_sync(0xffffffffu, grow)) {
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t r[32];
      tmem_ld_32x32(o_col + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
      tmem_st_32x32(o_col + c * 32, r);
    }
  }
  float r8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint32_t r[32];
    tmem_ld_32x32(s_col + c * 32, r);
    tmem_wait_ld();
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      float s0 = __uint_as_float(r[2 * e]);
      float s1 = __uint_as_float(r[2 * e + 1]);
      if constexpr (kMask) {
        const int key = key0 + c * 32 + 2 * e;
        s0 = ((key > row) | (key >= S)) ? -INFINITY : s0;
        s1 = ((key + 1 > row) | (key + 1 >= S)) ? -INFINITY : s1;
      }
      // half of the pairs on MUFU.EX2, half on the FMA pipe (balances the two units)
      const float a0 = fmaf(s0, scale_log2, -m_use), a1 = fmaf(s1, scale_log2, -m_use);
      const float p0 = (e & 1) ? exp2_poly(a0) : ex2_approx(a0);
      const float p1 = (e & 1) ? exp2_poly(a1) : ex2_approx(a1);
      pk[e] = pack_bf16x2(p0, p1);
      // the row sum uses the rounded probabilities that the PV product sees
      r8[e & 7] += __uint_as_float(pk[e] << 16) + __uint_as_float(pk[e] & 0xffff0000u);
    }
    tmem_st_32x32_x16(s_col + c * 16, pk);
  }
  tmem_wait_st();
  const float rs = ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
  l_run = l_run * alpha + rs;
  m_run = m_use;
}

}  // namespace

__global__ void __launch_bounds__(kAttn2Threads, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_vt,
                    __nv_bfloat16 *__restrict__ out, long ldo, int S, int HQ, int group,
                    float scale_log2, uint32_t *status) {
  extern __shared__ uint8_t smem_raw[];
  const Attn2Smem sm = carve2(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // grid (HQ, tile pairs), longest pair first over all heads (see attn_tc_kernel)
  const int npairs = gridDim.y;
  const int pr = npairs - 1 - blockIdx.y;
  const int h = blockIdx.x;
  const int kvh = h / group;
  const int nqb = (S + kTileRows - 1) / kTileRows;
  const int qa = 2 * pr, qb = 2 * pr + 1;
  const bool has_b = qb < nqb;
  const int nA = qa + 1;              // key blocks of tile A (causal)
  const int nB = has_b ? qb + 1 : 0;  // key blocks of tile B
  const int nkb = has_b ? nB : nA;
  constexpr int D = 128;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_qk);
    tma_prefetch_desc(&tm_vt);
    mbar_init(sm.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.p_ready[i], 128);
      mbar_init(&sm.o_done[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      bool ok = true;
      mbar_arrive_expect_tx(sm.q_full, (has_b ? 2 : 1) * kTileBytes);
      tma_load_2d(sm.q, &tm_qk, sm.q_full, h * D, qa * kTileRows);
      tma_load_2d(sm.q + kChunkBytes, &tm_qk, sm.q_full, h * D + 64, qa * kTileRows);
      if (has_b) {
        tma_load_2d(sm.q + kTileBytes, &tm_qk, sm.q_full, h * D, qb * kTileRows);
        tma_load_2d(sm.q + kTileBytes + kChunkBytes, &tm_qk, sm.q_full, h * D + 64, qb * kTileRows);
      }
      int issued = 0;
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&sm.kv_empty[st], ((j >> 1) & 1) ^ 1, kMbarLimitNs)) {
          report_status(status, kStatusTmaWait);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kTileBytes);
        uint8_t *kst = sm.q + (2 + st) * kTileBytes;
        uint8_t *vst = sm.q + (4 + st) * kTileBytes;
        const int kc = (HQ + kvh) * D;
        tma_load_2d(kst, &tm_qk, &sm.kv_full[st], kc, j * kTileRows);
        tma_load_2d(kst + kChunkBytes, &tm_qk, &sm.kv_full[st], kc + 64, j * kTileRows);
        tma_load_2d(vst, &tm_vt, &sm.kv_full[st], j * kTileRows, kvh * D);
        tma_load_2d(vst + kChunkBytes, &tm_vt, &sm.kv_full[st], j * kTileRows + 64, kvh * D);
        ++issued;
      }
      // no TMA write may still be in flight when the CTA exits
      mbar_wait(sm.q_full, 0, kMbarLimitNs / 4);
      for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
        mbar_wait(&sm.kv_full[j & 1], (j >> 1) & 1, kMbarLimitNs / 4);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D);
      // descriptors of every smem tile, computed once; k-step kk of a tile is the
      // base descriptor plus the step's byte offset >> 4 in the start-address field
      // (all offsets stay inside the 14-bit field: shared memory < 256 KB)
      const uint64_t dq0 = tile_desc(sm.q, 0), dq1 = tile_desc(sm.q + kTileBytes, 0);
      const uint64_t dk0 = tile_desc(sm.q + 2 * kTileBytes, 0), dk1 = tile_desc(sm.q + 3 * kTileBytes, 0);
      const uint64_t dv0 = tile_desc(sm.q + 4 * kTileBytes, 0), dv1 = tile_desc(sm.q + 5 * kTileBytes, 0);
      auto kstep = [](int kk) -> uint64_t {
        return static_cast<uint64_t>(((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4);
      };
      // issue order per key block j: PV(A,j), QK(A,j+1), PV(B,j), QK(B,j+1) -- tile
      // A's next scores are computed while tile B's softmax runs and vice versa
      // (ping-pong).  QK(x,j+1) overwrites the TMEM columns that hold P_x(j), so it
      // waits until PV(x,j) has completed.
      auto issue_qk = [&](int x, int jj) {
        tc_fence_after();
        const uint32_t sacc = tmem + 256 * x;
        const uint64_t qd = x ? dq1 : dq0, kd = (jj & 1) ? dk1 : dk0;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_bf16(sacc, qd + kstep(kk), kd + kstep(kk), idesc_s, kk > 0);
        umma_commit(&sm.s_full[x]);
      };
      bool ok = mbar_wait(sm.q_full, 0, kMbarLimitNs) &&
                mbar_wait(&sm.kv_full[0], 0, kMbarLimitNs);
      if (ok) {
        issue_qk(0, 0);
        if (nB > 0) issue_qk(1, 0);
      }
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        if (j + 1 < nkb) ok = mbar_wait(&sm.kv_full[(j + 1) & 1], ((j + 1) >> 1) & 1, kMbarLimitNs);
        for (int x = 0; x < 2 && ok; ++x) {
          const int nx = x ? nB : nA;
          if (j >= nx) continue;
          ok = mbar_wait(&sm.p_ready[x], j & 1, kMbarLimitNs);
          if (!ok) break;
          tc_fence_after();
          const uint64_t vd = st ? dv1 : dv0;
#pragma unroll
          for (int kk = 0; kk < kTileRows / 16; ++kk)
            umma_bf16_ts(tmem + 256 * x + 128, tmem + 256 * x + kk * 8, vd + kstep(kk), idesc_o,
                         (j > 0 || kk > 0));
          umma_commit(&sm.o_done[x]);
          if (j + 1 < nx) {
            ok = mbar_wait(&sm.o_done[x], j & 1, kMbarLimitNs);
            if (!ok) break;
            issue_qk(x, j + 1);
          }
        }
        if (ok) umma_commit(&sm.kv_empty[st]);
      }
      if (!ok) report_status(status, kStatusMmaWait);
    }
  } else {
    // ---------------- softmax / correction / epilogue: 128 threads per tile
    const int x = (warp - 2) >> 2;          // 0: tile A (warps 2..5), 1: tile B (6..9)
    const int quad = warp & 3;              // TMEM lane quadrant of this warp
    const int qx = x ? qb : qa;
    const int nx = x ? nB : nA;
    const int q0 = qx * kTileRows;
    const int row = q0 + quad * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t s_col = tmem + lane_addr + 256 * x;
    const uint32_t o_col = s_col + 128;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nx; ++j) {
      ok = mbar_wait(&sm.s_full[x], j & 1, kMbarLimitNs);
      if (!ok) break;
      tc_fence_after();
      const int key0 = j * kTileRows;
      // the causal / sequence-end mask applies only on the diagonal and last key
      // blocks: a uniform branch picks the masked or the plain instantiation (a
      // per-element short-circuit test cost ~10x the max loop itself)
      if (key0 + kTileRows - 1 > q0 || key0 + kTileRows > S)
        attn2_softmax_block<true>(s_col, o_col, key0, row, S, scale_log2, j > 0, m_run, l_run);
      else
        attn2_softmax_block<false>(s_col, o_col, key0, row, S, scale_log2, j > 0, m_run, l_run);
      tc_fence_before();
      mbar_arrive(&sm.p_ready[x]);
    }
    if (ok && nx > 0) ok = mbar_wait(&sm.o_done[x], (nx - 1) & 1, kMbarLimitNs);
    if (!ok) {
      report_status(status, kStatusEpiWait);
    } else if (nx > 0) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      __nv_bfloat16 *orow = out + static_cast<long>(row) * ldo + static_cast<long>(h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32(o_col + c * 32, r);
        tmem_wait_ld();
        if (row < S) {
          uint4 *o4 = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[q * 8 + 0]) * inv, __uint_as_float(r[q * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r[q * 8 + 2]) * inv, __uint_as_float(r[q * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r[q * 8 + 4]) * inv, __uint_as_float(r[q * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r[q * 8 + 6]) * inv, __uint_as_float(r[q * 8 + 7]) * inv);
            o4[q] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_vt,
                   __nv_bfloat16 *__restrict__ out, long ldo, int S, int HQ, int group,
                   float scale_log2, uint32_t *status) {
  extern __shared__ uint8_t smem_raw[];
  const AttnSmem sm = carve(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // grid (HQ, q tiles): blocks are dispatched x-fastest, so every head's longest
  // causal row tile goes first and the shortest last (longest-processing-time
  // order over the whole grid, not per head)
  const int nqb = gridDim.y;
  const int qb = nqb - 1 - blockIdx.y;
  const int h = blockIdx.x;
  const int kvh = h / group;
  const int q0 = qb * kTileRows;
  const int nkb = min(qb + 1, (S + kTileRows - 1) / kTileRows);
  constexpr int D = 128;

  if (threadIdx.x == 0) {
    tma_prefetch_desc(&tm_qk);
    tma_prefetch_desc(&tm_vt);
    mbar_init(sm.q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&sm.kv_full[i], 1);
      mbar_init(&sm.kv_empty[i], 1);
      mbar_init(&sm.s_full[i], 1);
      mbar_init(&sm.s_free[i], 128);
    }
    mbar_init(sm.p_ready, 128);
    mbar_init(sm.o_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(sm.tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sm.tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------- TMA producer
      bool ok = true;
      mbar_arrive_expect_tx(sm.q_full, kTileBytes);
      tma_load_2d(sm.q, &tm_qk, sm.q_full, h * D, q0);
      tma_load_2d(sm.q + kChunkBytes, &tm_qk, sm.q_full, h * D + 64, q0);
      int issued = 0;
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&sm.kv_empty[st], ((j >> 1) & 1) ^ 1, kMbarLimitNs)) {
          report_status(status, kStatusTmaWait);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * kTileBytes);
        const int kc = (HQ + kvh) * D;
        tma_load_2d(k_stage(sm, st), &tm_qk, &sm.kv_full[st], kc, j * kTileRows);
        tma_load_2d(k_stage(sm, st) + kChunkBytes, &tm_qk, &sm.kv_full[st], kc + 64, j * kTileRows);
        tma_load_2d(v_stage(sm, st), &tm_vt, &sm.kv_full[st], j * kTileRows, kvh * D);
        tma_load_2d(v_stage(sm, st) + kChunkBytes, &tm_vt, &sm.kv_full[st], j * kTileRows + 64, kvh * D);
        ++issued;
      }
      // no TMA write may still be in flight when the CTA exits
      mbar_wait(sm.q_full, 0, kMbarLimitNs / 4);
      for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j)
        mbar_wait(&sm.kv_full[j & 1], (j >> 1) & 1, kMbarLimitNs / 4);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, D);
      bool ok = mbar_wait(sm.q_full, 0, kMbarLimitNs);
      for (int j = 0; j <= nkb && ok; ++j) {
        if (j < nkb) {
          const int st = j & 1;
          ok = mbar_wait(&sm.kv_full[st], (j >> 1) & 1, kMbarLimitNs);
          if (ok && j >= 2) ok = mbar_wait(&sm.s_free[st], ((j >> 1) - 1) & 1, kMbarLimitNs);
          if (!ok) break;
          tc_fence_after();
          const uint32_t sacc = tmem + (st ? kColS1 : kColS0);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk)
            umma_bf16(sacc, tile_desc(sm.q, kk), tile_desc(k_stage(sm, st), kk), idesc_s, kk > 0);
          umma_commit(&sm.s_full[st]);
        }
        if (j >= 1) {
          const int i = j - 1;
          ok = mbar_wait(sm.p_ready, i & 1, kMbarLimitNs);
          if (!ok) break;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kTileRows / 16; ++kk)
            umma_bf16_ts(tmem + kColO, tmem + kColP + kk * 8, tile_desc(v_stage(sm, i & 1), kk), idesc_o,
                         (i > 0 || kk > 0));
          umma_commit(sm.o_done);
          umma_commit(&sm.kv_empty[i & 1]);
        }
      }
      if (!ok) report_status(status, kStatusMmaWait);
    }
  } else {
    // ---------------- softmax / correction / epilogue (128 threads)
    const int quad = warp & 3;
    const int rloc = quad * 32 + lane;
    const int row = q0 + rloc;
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkb; ++j) {
      const int sb = j & 1;
      ok = mbar_wait(&sm.s_full[sb], (j >> 1) & 1, kMbarLimitNs);
      if (!ok) break;
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld_32x32(tmem + lane_addr + (sb ? kColS1 : kColS0) + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) s[c * 32 + e] = __uint_as_float(r[e]);
      }
      tc_fence_before();
      mbar_arrive(&sm.s_free[sb]);
      const int key0 = j * kTileRows;
      if (key0 + kTileRows - 1 > q0 || key0 + kTileRows > S) {
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (key0 + c > row || key0 + c >= S) s[c] = -INFINITY;
      }
      // row max with eight independent chains (scale_log2 > 0 commutes with max)
      float m8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) m8[e] = s[e];
#pragma unroll
      for (int c = 8; c < 128; ++c) m8[c & 7] = fmaxf(m8[c & 7], s[c]);
      const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * scale_log2;
      const bool grow = mx - m_run > kRescaleLog2;  // true on the first block (m_run = -inf)
      const float m_use = grow ? mx : m_run;
      const float alpha = grow ? ex2_approx(m_run - mx) : 1.f;  // 0 on the first block
      uint32_t p[64];
      float r8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 64; ++c) {
        const float p0 = ex2_approx(fmaf(s[2 * c], scale_log2, -m_use));
        const float p1 = ex2_approx(fmaf(s[2 * c + 1], scale_log2, -m_use));
        p[c] = pack_bf16x2(p0, p1);
        // the row sum uses the rounded probabilities that the PV product sees
        r8[c & 7] += __uint_as_float(p[c] << 16) + __uint_as_float(p[c] & 0xffff0000u);
      }
      const float rs = ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
      l_run = l_run * alpha + rs;
      if (j > 0) {
        // PV_{j-1} must be complete before O is rescaled and P is overwritten
        ok = mbar_wait(sm.o_done, (j - 1) & 1, kMbarLimitNs);
        if (!ok) break;
        tc_fence_after();
        if (__any_sync(0xffffffffu, grow)) {
#pragma unroll 1
          for (int c = 0; c < D / 32; ++c) {
            uint32_t r[32];
            tmem_ld_32x32(tmem + lane_addr + kColO + c * 32, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st_32x32(tmem + lane_addr + kColO + c * 32, r);
          }
        }
      }
      m_run = m_use;
      {
        uint32_t lo[32], hi[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          lo[e] = p[e];
          hi[e] = p[32 + e];
        }
        tmem_st_32x32(tmem + lane_addr + kColP, lo);
        tmem_st_32x32(tmem + lane_addr + kColP + 32, hi);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(sm.p_ready);
    }
    if (ok) ok = mbar_wait(sm.o_done, (nkb - 1) & 1, kMbarLimitNs);
    if (!ok) {
      report_status(status, kStatusEpiWait);
    } else {
      tc_fence_after();
      const float inv = 1.f / l_run;
      __nv_bfloat16 *orow = out + static_cast<long>(row) * ldo + static_cast<long>(h) * D;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld_32x32(tmem + lane_addr + kColO + c * 32, r);
        tmem_wait_ld();
        if (row < S) {
          uint4 *o4 = reinterpret_cast<uint4 *>(orow + c * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(r[q * 8 + 0]) * inv, __uint_as_float(r[q * 8 + 1]) * inv);
            w.y = pack_bf16x2(__uint_as_float(r[q * 8 + 2]) * inv, __uint_as_float(r[q * 8 + 3]) * inv);
            w.z = pack_bf16x2(__uint_as_float(r[q * 8 + 4]) * inv, __uint_as_float(r[q * 8 + 5]) * inv);
            w.w = pack_bf16x2(__uint_as_float(r[q * 8 + 6]) * inv, __uint_as_float(r[q * 8 + 7]) * inv);
            o4[q] = w;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, kTmemCols);
}

// ------------------------------------------------------------------ host side
// V^T [HKV*D rows][ldv >= S] from the fused qkv buffer (one transpose launch).
void attention_vt_bf16(const __nv_bfloat16 *qkv, __nv_bfloat16 *vt, long ldv, int S, int HQ,
                       int HKV, int D, cudaStream_t stream) {
  const long ld = static_cast<long>(HQ + 2 * HKV) * D;
  transpose_bf16(qkv + static_cast<long>(HQ + HKV) * D, ld, vt, ldv, S, HKV * D, stream);
}

void attention_tc_bf16(const __nv_bfloat16 *qkv, const __nv_bfloat16 *vt, long ldv,
                       __nv_bfloat16 *out, int S, int HQ, int HKV, int D, float scale,
                       uint32_t *status, cudaStream_t stream) {
  if (D != 128) throw CudaError("attention_tc: head_dim must be 128");
  if (HKV <= 0 || HQ % HKV) throw CudaError("attention_tc: HQ % HKV != 0");
  if (ldv % 8) throw CudaError("attention_tc: V^T pitch must be a multiple of 8");
  const long ld = static_cast<long>(HQ + 2 * HKV) * D;
  const CUtensorMap tm_qk = make_tmap_2d_bf16(qkv, S, ld, ld, kTileRows, 64);
  // V^T map: only the first S key columns are valid; TMA zero-fills beyond them
  const CUtensorMap tm_vt = make_tmap_2d_bf16(vt, static_cast<uint64_t>(HKV) * D, S, ldv, kTileRows, 64);
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  static bool configured[64] = {false};
  if (!configured[dev & 63]) {
    KRB_CUDA(cudaFuncSetAttribute(attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(kAttnSmemBytes)));
    KRB_CUDA(cudaFuncSetAttribute(attn_tc2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(kAttn2SmemBytes)));
    configured[dev & 63] = true;
  }
  // KRB_ATTN=tc1: the one-tile kernel (kept for comparison)
  static const bool one_tile = [] {
    const char *e = std::getenv("KRB_ATTN");
    return e && std::string(e) == "tc1";
  }();
  const int nqb = (S + kTileRows - 1) / kTileRows;
  const float sl2 = scale * 1.4426950408889634f;
  if (one_tile) {
    dim3 grid(HQ, nqb);
    attn_tc_kernel<<<grid, kAttnThreads, kAttnSmemBytes, stream>>>(
        tm_qk, tm_vt, out, static_cast<long>(HQ) * D, S, HQ, HQ / HKV, sl2, status);
  } else {
    dim3 grid(HQ, (nqb + 1) / 2);
    attn_tc2_kernel<<<grid, kAttn2Threads, kAttn2SmemBytes, stream>>>(
        tm_qk, tm_vt, out, static_cast<long>(HQ) * D, S, HQ, HQ / HKV, sl2, status);
  }
  KRB_CUDA(cudaGetLastError());
}

}  // namespace krb
