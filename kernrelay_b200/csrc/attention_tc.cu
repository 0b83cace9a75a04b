// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM).
// Q, K and the output are bf16 or fp16 (the engine runs fp16); V^T and P are fp16.
//
// Replaces aclnnFlashAttentionScore (BSND, sparse_mode 3, scale 1/sqrt(D);
// qwen_main.cpp:591-614) for head_dim 64 and 128.  One CTA = one query head x two
// consecutive 128-row query tiles; it walks the 128-key blocks up to the diagonal.
// Q and K tiles come from the fused qkv buffer, V from a transposed copy
// ([kv_head * D + d][key]) so that every operand is K-major with the same
// 128-byte-swizzle descriptor: Q [row][d], K [key][d], V^T [d][key] and P [row][key]
// (TMEM: lane = row, 2 keys per column).  All waits are bounded (status bits as in
// the GEMM).
#include <cudaTypedefs.h>

#include <cstdlib>
#include <string>

#include "common.h"
#include "ptx.cuh"

namespace krb {

namespace {

constexpr int kTileRows = 128;               // query rows per tile = keys per block
constexpr uint32_t kChunkBytes = 128 * 128;  // 128 rows x 64 bf16 (one swizzle width)
constexpr uint32_t kTmemCols = 512;

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
// squares for relative error on Chebyshev nodes (max relative error 2.2e-4, below
// the fp16 rounding the probabilities get next, 4.9e-4); n is added to the
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
// packed fp16 pairs once read), O at 256X + 128 (D columns).  PV multiplies fp16 P by
// fp16 V^T (the transposed copy of V is written in fp16).  The softmax reads S
// twice (row max, then exp and P) so a thread holds 32 scores at a time.
// Shared memory: six tiles of 256*D bytes (Q_A, Q_B, K x2, V^T x2): a Q or K tile is
// D/64 chunks of 128 rows x 64 elements, a V^T tile two chunks of D rows x 64 keys.
constexpr int kAttn2Threads = 320;

template <int D>
struct Attn2Cfg {
  static_assert(D == 64 || D == 128, "head_dim 64 or 128");
  static constexpr uint32_t kTile = 256u * D;     // bytes of one Q, K or V^T tile
  static constexpr uint32_t kVChunk = 128u * D;   // D rows x 64 keys
  static constexpr uint32_t kSmem = 6 * kTile + 12 * 8 + 16 + 1024;
};

struct Attn2Smem {
  uint8_t *q;  // Q_A, Q_B; K stage s at q + (2 + s) * tile; V^T stage s at q + (4 + s) * tile
  uint64_t *q_full, *kv_full, *kv_empty, *s_full, *p_ready, *o_done;  // [1], [2], [2], [2], [2], [2]
  uint32_t *tmem_slot;
};

__device__ __forceinline__ Attn2Smem carve2(uint8_t *raw, uint32_t tile_bytes) {
  Attn2Smem a;
  uint8_t *base =
      reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~uintptr_t(1023));
  a.q = base;
  uint64_t *bars = reinterpret_cast<uint64_t *>(base + 6 * tile_bytes);
  a.q_full = bars;
  a.kv_full = bars + 1;
  a.kv_empty = bars + 3;
  a.s_full = bars + 5;
  a.p_ready = bars + 7;
  a.o_done = bars + 9;
  a.tmem_slot = reinterpret_cast<uint32_t *>(bars + 11);
  return a;
}

__device__ __forceinline__ void tmem_ld_32x32_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32"
      " {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// One key block of the two-tile kernel's softmax for one row (thread), in ONE pass over
// the 128 scores: chunk c (32 scores) is processed while chunk c + 1's TMEM load is in
// flight.  P = 2^(s*scale - m) with the row's current offset m, rounded to fp16 and
// written over S's first 64 columns as fp16 pairs (chunk c's P lands on columns already
// read).  The offset moves only when a chunk's max exceeds it by more than 2^8 (then
// the P chunks this row already wrote are rescaled in TMEM -- warp-uniformly, rare
// after the first chunk), so every P stays <= 2^8 in fp16.  Afterwards O (if the offset
// moved since the previous block: the PV of that block is complete, the commit that
// released this S covers it) and the running sum follow the offset.
template <bool kMask, int D>
__device__ __forceinline__ void attn2_softmax_block(uint32_t s_col, uint32_t o_col, int key0,
                                                    int row, int S, float scale_log2, bool has_o,
                                                    float &m_run, float &l_run) {
  float m_cur = m_run;  // offset of the P values written so far in this block
  float r8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  uint32_t ra[32], rb[32];
  tmem_ld_32x32(s_col, ra);
  tmem_wait_ld();
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t(&r)[32] = (c & 1) ? rb : ra;
    if (c + 1 < 4) tmem_ld_32x32(s_col + (c + 1) * 32, (c & 1) ? ra : rb);
    float m8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) m8[e] = -INFINITY;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      float v = __uint_as_float(r[e]);
      if constexpr (kMask) {
        const int key = key0 + c * 32 + e;
        v = ((key > row) | (key >= S)) ? -INFINITY : v;
        r[e] = __float_as_uint(v);
      }
      m8[e & 7] = fmaxf(m8[e & 7], v);
    }
    const float cmax = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                             fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * scale_log2;
    const bool grow = cmax - m_cur > kRescaleLog2;  // first chunk of a row: m_cur = -inf
    if (c > 0 && __any_sync(0xffffffffu, grow)) {
      // rebase the P chunks 0..c-1 of this row (f = 1 for rows that keep their offset)
      const float f = grow ? ex2_approx(m_cur - cmax) : 1.f;
      tmem_wait_st();
#pragma unroll 1
      for (int pc = 0; pc < c; ++pc) {
        uint32_t q[16];
        tmem_ld_32x32_x16(s_col + pc * 16, q);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          const float2 pr = unpack_f16x2(q[e]);
          q[e] = pack_f16x2(pr.x * f, pr.y * f);
        }
        tmem_st_32x32_x16(s_col + pc * 16, q);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) r8[e] *= f;
    }
    if (grow) m_cur = cmax;
    uint32_t pk[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float s0 = __uint_as_float(r[2 * e]);
      const float s1 = __uint_as_float(r[2 * e + 1]);
      // 13 of 16 pairs on MUFU.EX2 (one issue slot, 8 cycles of its pipe per warp), 3 on the
      // FMA-pipe cubic (~11 issue slots): with two softmax warps per SM sub-partition this
      // balances the MUFU pipe against instruction issue (a 50/50 split is issue-bound)
      const float a0 = fmaf(s0, scale_log2, -m_cur), a1 = fmaf(s1, scale_log2, -m_cur);
      const bool poly = (e % 5) == 4;
      const float p0 = poly ? exp2_poly(a0) : ex2_approx(a0);
      const float p1 = poly ? exp2_poly(a1) : ex2_approx(a1);
      // P in fp16 (P <= 2^kRescaleLog2 = 256: far inside its range; 8x finer than bf16);
      // the row sum takes the fp32 values (one rounding of 2^-11 per term, unbiased)
      pk[e] = pack_f16x2(p0, p1);
      r8[e & 7] += p0 + p1;
    }
    tmem_st_32x32_x16(s_col + c * 16, pk);
    if (c + 1 < 4) tmem_wait_ld();
  }
  tmem_wait_st();
  const float rs = ((r8[0] + r8[1]) + (r8[2] + r8[3])) + ((r8[4] + r8[5]) + (r8[6] + r8[7]));
  // O and l still carry the previous block's offset m_run (-inf before the first block:
  // alpha = 0, l_run = 0, no O yet)
  const bool moved = m_cur != m_run;
  const float alpha = moved ? ex2_approx(m_run - m_cur) : 1.f;
  if (has_o && __any_sync(0xffffffffu, moved)) {
#pragma unroll 1
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      tmem_ld_32x32(o_col + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int e = 0; e < 32; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
      tmem_st_32x32(o_col + c * 32, r);
    }
    tmem_wait_st();
  }
  l_run = l_run * alpha + rs;
  m_run = m_cur;
}

}  // namespace

// Grid (heads of this launch, tile pairs); query head h = h0 + blockIdx.x reads KV head
// kv0 + blockIdx.x / group.  HQ is the head count of the qkv layout (K columns start at
// HQ * D).  Pairs are dispatched longest first over all heads (blocks go x-fastest).
// F16: q / k (and so the QK^T operands) and the output are fp16, else bf16.
template <int D, bool F16>
__global__ void __launch_bounds__(kAttn2Threads, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tm_qk, const __grid_constant__ CUtensorMap tm_vt,
                    uint16_t *__restrict__ out, long ldo, int S, int HQ, int h0, int kv0,
                    int group, float scale_log2, uint32_t *status) {
  using C = Attn2Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  const Attn2Smem sm = carve2(smem_raw, C::kTile);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int npairs = gridDim.y;
  const int pr = npairs - 1 - blockIdx.y;
  const int h = h0 + blockIdx.x;
  const int kvh = kv0 + blockIdx.x / group;
  const int nqb = (S + kTileRows - 1) / kTileRows;
  const int qa = 2 * pr, qb = 2 * pr + 1;
  const bool has_b = qb < nqb;
  const int nA = qa + 1;              // key blocks of tile A (causal)
  const int nB = has_b ? qb + 1 : 0;  // key blocks of tile B
  const int nkb = has_b ? nB : nA;

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
      mbar_arrive_expect_tx(sm.q_full, (has_b ? 2 : 1) * C::kTile);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_2d(sm.q + c * kChunkBytes, &tm_qk, sm.q_full, h * D + 64 * c, qa * kTileRows);
        if (has_b)
          tma_load_2d(sm.q + C::kTile + c * kChunkBytes, &tm_qk, sm.q_full, h * D + 64 * c,
                      qb * kTileRows);
      }
      int issued = 0;
      for (int j = 0; j < nkb && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&sm.kv_empty[st], ((j >> 1) & 1) ^ 1, kMbarLimitNs)) {
          report_status(status, kStatusTmaWait);
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&sm.kv_full[st], 2 * C::kTile);
        uint8_t *kst = sm.q + (2 + st) * C::kTile;
        uint8_t *vst = sm.q + (4 + st) * C::kTile;
        const int kc = (HQ + kvh) * D;
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_2d(kst + c * kChunkBytes, &tm_qk, &sm.kv_full[st], kc + 64 * c, j * kTileRows);
        tma_load_2d(vst, &tm_vt, &sm.kv_full[st], j * kTileRows, kvh * D);
        tma_load_2d(vst + C::kVChunk, &tm_vt, &sm.kv_full[st], j * kTileRows + 64, kvh * D);
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
      constexpr uint32_t idesc_s = F16 ? idesc_f16_f32(128, 128) : idesc_bf16_f32(128, 128);
      constexpr uint32_t idesc_o = idesc_f16_f32(128, D);  // P and V^T both fp16
      // descriptors of every smem tile, computed once; k-step kk of a tile is the
      // base descriptor plus the step's byte offset >> 4 in the start-address field
      // (all offsets stay inside the 14-bit field: shared memory < 256 KB)
      const uint64_t dq0 = tile_desc(sm.q, 0), dq1 = tile_desc(sm.q + C::kTile, 0);
      const uint64_t dk0 = tile_desc(sm.q + 2 * C::kTile, 0), dk1 = tile_desc(sm.q + 3 * C::kTile, 0);
      const uint64_t dv0 = tile_desc(sm.q + 4 * C::kTile, 0), dv1 = tile_desc(sm.q + 5 * C::kTile, 0);
      // Q / K: 16 head dims per step, 64 per chunk of 128 rows; V^T: 16 keys per step,
      // 64 per chunk of D rows
      auto kstep = [](int kk) -> uint64_t {
        return static_cast<uint64_t>(((kk >> 2) * kChunkBytes + (kk & 3) * 32) >> 4);
      };
      auto vstep = [](int kk) -> uint64_t {
        return static_cast<uint64_t>(((kk >> 2) * C::kVChunk + (kk & 3) * 32) >> 4);
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
            umma_bf16_ts(tmem + 256 * x + 128, tmem + 256 * x + kk * 8, vd + vstep(kk), idesc_o,
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
        attn2_softmax_block<true, D>(s_col, o_col, key0, row, S, scale_log2, j > 0, m_run, l_run);
      else
        attn2_softmax_block<false, D>(s_col, o_col, key0, row, S, scale_log2, j > 0, m_run, l_run);
      tc_fence_before();
      mbar_arrive(&sm.p_ready[x]);
    }
    if (ok && nx > 0) ok = mbar_wait(&sm.o_done[x], (nx - 1) & 1, kMbarLimitNs);
    if (!ok) {
      report_status(status, kStatusEpiWait);
    } else if (nx > 0) {
      tc_fence_after();
      const float inv = 1.f / l_run;
      uint16_t *orow = out + static_cast<long>(row) * ldo + static_cast<long>(h) * D;
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
            w.x = pack2<F16>(__uint_as_float(r[q * 8 + 0]) * inv, __uint_as_float(r[q * 8 + 1]) * inv);
            w.y = pack2<F16>(__uint_as_float(r[q * 8 + 2]) * inv, __uint_as_float(r[q * 8 + 3]) * inv);
            w.z = pack2<F16>(__uint_as_float(r[q * 8 + 4]) * inv, __uint_as_float(r[q * 8 + 5]) * inv);
            w.w = pack2<F16>(__uint_as_float(r[q * 8 + 6]) * inv, __uint_as_float(r[q * 8 + 7]) * inv);
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
// fp16 V^T [HKV*D rows][ldv >= S] of KV heads [kv0, kv0 + nkv) from the fused qkv buffer
template <typename T>
void attention_vt(const T *qkv, __half *vt, long ldv, int S, int HQ, int HKV, int D,
                  cudaStream_t stream, int kv0, int nkv) {
  if (nkv < 0) nkv = HKV - kv0;
  if (kv0 < 0 || nkv <= 0 || kv0 + nkv > HKV) throw CudaError("attention_vt: KV head range");
  const long ld = static_cast<long>(HQ + 2 * HKV) * D;
  if constexpr (ActFmt<T>::f16)
    transpose_f16(qkv + static_cast<long>(HQ + HKV + kv0) * D, ld,
                  vt + static_cast<long>(kv0) * D * ldv, ldv, S, nkv * D, stream);
  else
    transpose_bf16_to_f16(qkv + static_cast<long>(HQ + HKV + kv0) * D, ld,
                          vt + static_cast<long>(kv0) * D * ldv, ldv, S, nkv * D, stream);
}

template <int D, bool F16>
static void launch_attn_tc2(const void *qkv, const __half *vt, long ldv, void *out, int S, int HQ,
                            int HKV, int h0, int nh, int kv0, int group, float scale,
                            uint32_t *status, cudaStream_t stream) {
  using C = Attn2Cfg<D>;
  const long ld = static_cast<long>(HQ + 2 * HKV) * D;
  const CUtensorMap tm_qk = make_tmap_2d_bf16(qkv, S, ld, ld, kTileRows, 64);
  // V^T map: only the first S key columns are valid; TMA zero-fills beyond them
  const CUtensorMap tm_vt = make_tmap_2d_bf16(vt, static_cast<uint64_t>(HKV) * D, S, ldv, D, 64);
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  static bool configured[64] = {false};
  if (!configured[dev & 63]) {
    KRB_CUDA(cudaFuncSetAttribute(attn_tc2_kernel<D, F16>,
                                  cudaFuncAttributeMaxDynamicSharedMemorySize, int(C::kSmem)));
    configured[dev & 63] = true;
  }
  const int nqb = (S + kTileRows - 1) / kTileRows;
  dim3 grid(nh, (nqb + 1) / 2);
  attn_tc2_kernel<D, F16><<<grid, kAttn2Threads, C::kSmem, stream>>>(
      tm_qk, tm_vt, static_cast<uint16_t *>(out), static_cast<long>(HQ) * D, S, HQ, h0, kv0,
      group, scale * 1.4426950408889634f, status);
  KRB_CUDA(cudaGetLastError());
}

template <typename T>
void attention_tc(const T *qkv, const __half *vt, long ldv, T *out, int S, int HQ, int HKV, int D,
                  float scale, uint32_t *status, cudaStream_t stream, int h0, int nh, int kv0,
                  int group) {
  constexpr bool F16 = ActFmt<T>::f16;
  if (D != 64 && D != 128) throw CudaError("attention_tc: head_dim must be 64 or 128");
  if (HKV <= 0 || HQ % HKV) throw CudaError("attention_tc: HQ % HKV != 0");
  if (ldv % 8) throw CudaError("attention_tc: V^T pitch must be a multiple of 8");
  if (S <= 0) throw CudaError("attention_tc: empty sequence");
  if (nh < 0) nh = HQ;
  if (group <= 0) group = HQ / HKV;
  if (h0 < 0 || nh <= 0 || h0 + nh > HQ || kv0 < 0 || kv0 + (nh - 1) / group >= HKV)
    throw CudaError("attention_tc: head range outside the qkv layout");
  if (D == 128)
    launch_attn_tc2<128, F16>(qkv, vt, ldv, out, S, HQ, HKV, h0, nh, kv0, group, scale, status,
                              stream);
  else
    launch_attn_tc2<64, F16>(qkv, vt, ldv, out, S, HQ, HKV, h0, nh, kv0, group, scale, status,
                             stream);
}

template void attention_vt<__nv_bfloat16>(const __nv_bfloat16 *, __half *, long, int, int, int,
                                          int, cudaStream_t, int, int);
template void attention_vt<__half>(const __half *, __half *, long, int, int, int, int,
                                   cudaStream_t, int, int);
template void attention_tc<__nv_bfloat16>(const __nv_bfloat16 *, const __half *, long,
                                          __nv_bfloat16 *, int, int, int, int, float, uint32_t *,
                                          cudaStream_t, int, int, int, int);
template void attention_tc<__half>(const __half *, const __half *, long, __half *, int, int, int,
                                   int, float, uint32_t *, cudaStream_t, int, int, int, int);

}  // namespace krb
