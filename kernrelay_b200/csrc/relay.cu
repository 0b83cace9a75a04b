// tp_split: the fused down_proj producer + relay consumer for one layer.
//
// Reference path (qwen_main.cpp:1274-1302): for each of T row tiles,
//   down_t = act_t . W_down_r            (aclnnMatmul on the AIC stream)
//   publish/wait GM flag                 (kr_publish_aic / kr_wait_aiv)
//   red_t = AllReduce_sum(down_t)        (HcclAllReduce on the comm stream)
//   h0_t, x_t = AddRmsNorm(h1_t, red_t)  (aclnnAddRmsNorm)
//
// B200 design: ONE persistent cooperative kernel per layer and rank, 15 warps:
//   warps 0..5   tcgen05 GEMM (TMA producer, MMA issuer, 4 epilogue warps) over the
//                output tiles in row-tile order (CTA pairs where the rows allow).  The
//                epilogue writes the 2-byte partial tile into this rank's `part` buffer
//                (local, coalesced; k = 1: the fp32 tile straight into sum_out) and,
//                after a barrier of the epilogue warps, one thread adds 1 to the local
//                completion counter of its row tile at GPU scope.
//   warps 6..13  relay, per row tile t (or run of tiles), one of two forms:
//                direct (default for k <= 2): acquire rs_cnt[t][*] (the bounded
//                GM-flag wait), then h0 = h1 + sum_src part_src (the k partial rows
//                pulled from every rank's `part`, local or over NVLink, summed in
//                fp32), x = RMSNorm(h0) * gamma, two warps per row, the half row
//                held in registers.  One synchronisation per tile.
//                rsag (k >= 4; fixed order rs(t+1) before ag(t) by default): acquire
//                rs_cnt[t][*]; PULL the k partial slices of the rows this rank owns,
//                sum in fp32, round once, store into the local `red` buffer and add
//                to the local ag_done[t]; acquire ag_cnt[t][*] and apply the
//                Add+RMSNorm with the reduced rows pulled from each row's owner.
//                NVLink bytes per rank and tile: direct (k-1)/k * k = k-1 tiles,
//                rsag 2(k-1)/k tiles; equal at k = 2, where direct saves the second
//                system-scope synchronisation (~17 us per tile measured).
//   warp 14      signal: one thread per (row tile, counter) and GPU waits for the local
//                completion counter, fences at system scope and forwards the tile to
//                rs_cnt / ag_cnt on every rank (the GM-flag publish).
// Every region is written only by its own rank, so every system-scope fence
// covers local stores only; all NVLink traffic is loads.  Releases are two-level:
// GPU-scope adds into local completion counters (~1 us), and one signal thread
// per (row tile, counter) and GPU that fences at system scope and forwards the
// tile to every rank.  Measured on B200 under NVLink load: a system-scope fence
// costs 12 us (k = 2) to 40 us (k = 4) when every CTA issues one, 2.5-4.5 us
// when only the 2T signal threads do.
// No kernel waits on another kernel of the same GPU: the waits target other CTAs
// of this co-resident cooperative grid and the same kernel on the peer GPUs.
// Counters are monotone; targets derive from the run epoch and the layer, so
// CUDA-graph replays need no reset.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>
#include <string>
#include <type_traits>

#include "common.h"
#include "gemm.cuh"
#include "relay.cuh"

namespace krb {

TileSched relay_tile_sched(int S, int H, int T, int bn, int grid,
                           int cta_group);  // bottom of this file

constexpr int kRelayWarp0 = 6;                      // warps 0..5: GEMM roles
constexpr int kRelayWarps = 8;                      // consumer warps per CTA
constexpr int kRelaySlots = 8;                      // staging slots (mbarriers) per warp pair
constexpr int kSignalWarp = kRelayWarp0 + kRelayWarps;  // warp 14: system-scope signals
constexpr int kRelayThreads = (kSignalWarp + 1) * 32;

__device__ __forceinline__ uint32_t *flag_ptr(uint8_t *base, size_t off) {
  return reinterpret_cast<uint32_t *>(base + off);
}

__device__ __forceinline__ void trace_mark(const RelayArgs &ra, int slot) {
  if (ra.trace) ra.trace[size_t(blockIdx.x) * kTraceSlots + slot] = globaltimer_ns();
}

// fp32 accumulate of 8 bf16 from a 16-byte vector (L2-coherent load)
__device__ __forceinline__ void acc8_cg(float *acc, const __nv_bfloat16 *p) {
  const uint4 w = __ldcg(reinterpret_cast<const uint4 *>(p));
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack_bf16x2(ws[e]);
    acc[2 * e] += f.x;
    acc[2 * e + 1] += f.y;
  }
}

// fp32 accumulate of 8 activations (bf16 or fp16) held in a 16-byte register vector
template <bool F16>
__device__ __forceinline__ void acc8_act(float *acc, const uint4 &w) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack2<F16>(ws[e]);
    acc[2 * e] += f.x;
    acc[2 * e + 1] += f.y;
  }
}

// fp32 accumulate of 8 bf16 held in a 16-byte register vector (weights: gamma)
__device__ __forceinline__ void acc8_bits(float *acc, const uint4 &w) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = unpack_bf16x2(ws[e]);
    acc[2 * e] += f.x;
    acc[2 * e + 1] += f.y;
  }
}

template <bool F16>
__device__ __forceinline__ uint4 pack8f(const float *f) {
  uint4 w;
  w.x = pack2<F16>(f[0], f[1]);
  w.y = pack2<F16>(f[2], f[3]);
  w.z = pack2<F16>(f[4], f[5]);
  w.w = pack2<F16>(f[6], f[7]);
  return w;
}

// ---------------------------------------------------------------- push epilogue
// Peer region bases, copied from the kernel parameters into shared memory so the
// epilogue can index them by owner rank without a local-memory copy.
__shared__ uint8_t *g_peer_base[kMaxRanks];

template <int BN, int V, bool F16>
__device__ __forceinline__ void relay_push_epilogue(const GemmSmemView<BN, V> &s,
                                                    const TileSched &ts, const RelayArgs &ra) {
  using C = GemmCfg<BN, V>;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quad = warp & 3;
  const uint32_t tmem = *s.tmem_slot;
  __nv_bfloat16 *part = reinterpret_cast<__nv_bfloat16 *>(ra.local_base + ra.part_off);
  float *stage = s.epi + (warp - 2) * 32 * C::kStageRow;
  uint64_t fence_ns = 0, fence_cnt = 0, fence_max = 0;  // trace only
  int it = 0;
  const TileWalk<C::kCG> w = TileWalk<C::kCG>::make();
  const uint32_t leader_tempty = C::kCG == 2 ? mapa_shared(&s.tempty[0], 0) : 0u;
  bool clean = true;
  for (int t = w.first; t < ts.total(); t += w.step, ++it) {
    int mb, n0, bn;
    ts.tile(t, mb, n0, bn);
    mb = w.row_block(mb);  // this CTA's 128 rows of the tile
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    // collective decision: the four epilogue warps meet at named barrier 1 below,
    // so either all of them continue with this tile or all of them stop
    bool ok = mbar_wait(&s.tfull[acc], acc_phase, kMbarLimitNs) && !*s.abort;
    ok = named_bar_and(1, 128, ok);
    if (!ok) {
      report_status(ra.status, kStatusEpiWait);
      *s.abort = 1;
      clean = false;
      break;
    }
    tc_fence_after();
    const int row0 = mb * kBM + quad * 32;  // first row of this warp (< S)
    const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + acc * C::kAccStride;
    auto part_row = [&](int r) -> __nv_bfloat16 * {
      return part + static_cast<size_t>(row0 + r) * ra.H;
    };
#pragma unroll 1
    for (int c = 0; c * 32 < bn; ++c) {
      const int col0 = n0 + c * 32;
      if (col0 >= ra.H) break;
      const int valid = min(bn - c * 32, ra.H - col0);
      uint32_t r[32];
      tmem_ld_32x32(tbase + c * 32, r);
      tmem_wait_ld();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      epi_stage_put(stage, v);
      if (ra.k == 1)
        // one rank: nothing to reduce; the fp32 partial goes straight into sum_out
        // and the relay warps add the residual in place
        epi_stage_store_f32(stage, ra.sum_out, ra.H, row0, ra.S, col0, valid);
      else
        epi_stage_store_bf16<F16>(stage, part_row, nullptr, col0, valid);
    }
    tc_fence_before();
    // accumulator free for the next tile (pairs: on the leader, for both CTAs)
    if constexpr (C::kCG == 2)
      mbar_arrive_cluster(leader_tempty + 8u * uint32_t(acc));
    else
      mbar_arrive(&s.tempty[acc]);
    named_bar_sync(1, 128);       // all four epilogue warps' stores are issued
    if (warp == 2 && lane == 0) {
      const uint64_t f0 = ra.trace ? globaltimer_ns() : 0;
      // GPU-scope release, cumulative over the four warps' stores that the named
      // barrier ordered before it.  k = 1: straight to the consumer's counter;
      // k > 1: into the local completion counter that the signal warp forwards.
      const int t_row = (mb * kBM) / ra.R;
      const size_t line = ra.k == 1
                              ? ra.flag_off + size_t(t_row) * 128
                              : ra.flag_off + (2 * size_t(ra.T) * ra.k + 2 + t_row) * 128;
      red_add_release_gpu(flag_ptr(ra.local_base, line), 1u);
      if (ra.trace) {
        const uint64_t df = globaltimer_ns() - f0;
        fence_ns += df;
        fence_max = df > fence_max ? df : fence_max;
        ++fence_cnt;
      }
    }
  }
  if (warp == 2 && lane == 0) {
    // Every accumulator of this CTA has been drained, so every MMA (and, before it,
    // every TMA load) that used the pipeline buffers is complete: the relay warps may
    // stage copies there from now on.
    if (clean) {
      __threadfence_block();
      s.abort[2] = 1;
    }
    trace_mark(ra, 1);
    if (ra.trace) {
      unsigned long long *tr = ra.trace + size_t(blockIdx.x) * kTraceSlots;
      tr[43] = fence_ns;
      tr[44] = fence_cnt;
      tr[45] = fence_max;
    }
  }
}

// ---------------------------------------------------------------- relay warps
// The first relay warp polls the k counters of tile t, lane s the counter of source s
// (bounded, all k round trips in flight at once); the relay warps then meet at named
// barrier 2, which orders every lane's acquire before the other relay threads' loads.
// Returns 0 (all threads) if the wait expired, else 1, plus 2 when `gemm_done` (this
// CTA's GEMM has finished, read once by the poller so every thread sees the same) is set,
// plus e << 8: once the GEMM is done, tiles t+1 .. e-1 (e <= extend_limit) were found
// complete too (non-blocking checks), so the caller may take [t, e) as one run.
__device__ __forceinline__ bool sources_ready(const RelayArgs &ra, size_t cnt_base, int t,
                                              uint32_t target);
__device__ __forceinline__ int wait_all_sources(const RelayArgs &ra, size_t cnt_base, int t,
                                                uint32_t target, uint32_t code,
                                                uint64_t timeout_ns, volatile int *flag_smem,
                                                const volatile int *gemm_done = nullptr,
                                                int extend_limit = 0) {
  if ((threadIdx.x >> 5) == kRelayWarp0) {
    const int src = threadIdx.x & 31;
    bool ok = true;
    if (src < ra.k)
      ok = wait_counter_geq(flag_ptr(ra.local_base, cnt_base + (size_t(t) * ra.k + src) * 128),
                            target, timeout_ns);
    ok = __all_sync(0xffffffffu, ok);
    // one read, broadcast from lane 0: the epilogue may set the flag while the lanes read
    // it, and every lane must take the same branch into sources_ready's __all_sync
    const bool done =
        __shfl_sync(0xffffffffu, (gemm_done && *gemm_done) ? 1 : 0, 0) != 0;
    int e = t + 1;
    if (ok && done)
      while (e < extend_limit && sources_ready(ra, cnt_base, e, target)) ++e;
    if (src == 0) {
      if (!ok) report_status(ra.status, code);
      *flag_smem = ok ? 1 | (done ? 2 : 0) | (e << 8) : 0;
    }
  }
  // Cumulativity through the barrier (the same pattern as a cooperative grid sync)
  // makes every source's release visible to all relay threads.  Payload loads go to
  // L2 (ld.global.cg), so no stale L1 line can be hit.
  named_bar_sync(2, kRelayWarps * 32);
  const int w = *flag_smem;
  named_bar_sync(2, kRelayWarps * 32);  // flag_smem may be rewritten by the next wait
  return w;
}

// Non-blocking, called by the whole first relay warp: true in every lane when each
// source's counter of tile t has reached target (lane s loads source s's counter).
__device__ __forceinline__ bool sources_ready(const RelayArgs &ra, size_t cnt_base, int t,
                                              uint32_t target) {
  const int src = threadIdx.x & 31;
  bool r = true;
  if (src < ra.k)
    r = static_cast<int32_t>(
            ld_acquire_sys(flag_ptr(ra.local_base, cnt_base + (size_t(t) * ra.k + src) * 128)) -
            target) >= 0;
  return __all_sync(0xffffffffu, r);
}

__device__ __forceinline__ float warp_allsum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Residual update + RMSNorm of one row by a PAIR of relay warps (half a row each).
// The half row stays in registers between the sum and the normalisation, so HBM is
// read once and every load of the half row is in flight at the same time:
//   h[c] = resid[c] + delta[c]  (delta: bf16 reduced rows, or fp32 partial in place)
//   sum_out[c] = h[c];  x[c] = h[c] * rsqrt(mean(h^2) + eps) * gamma[c]
// The two halves exchange their sums of squares through shared memory at the
// pair's own named barrier (ids 3..6, 64 threads).
constexpr int kHalfVec = 8;  // 16-byte vectors per lane per half row: H <= 2*8*256 = 4096

//   kSrc = 0: delta is one fp32 row; kSrc = 1: delta is one bf16 row;
//   kSrc >= 2: delta is the sum of the kSrc ranks' bf16 partial rows, rank s's at
//   g_peer_base[s] + part_off, element offset part_elem (pulled over NVLink)
template <int kSrc, bool F16>
__device__ __forceinline__ void pair_addnorm_row(const float *resid, const void *delta,
                                                 size_t part_off, size_t part_elem, float *sum_out,
                                                 const __nv_bfloat16 *gamma, __nv_bfloat16 *x_out,
                                                 int hv, float inv_h, float eps, bool do_norm,
                                                 int pair, int half, float *pair_ss) {
  const int lane = threadIdx.x & 31;
  const int hv0 = (hv + 1) / 2;                  // vectors of half 0
  const int vbeg = half ? hv0 : 0;
  const int vend = half ? hv : hv0;
  float h[kHalfVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kHalfVec; ++i) {
    const int v = vbeg + lane + 32 * i;
    if (v < vend) {
      const float4 r0 = __ldcg(reinterpret_cast<const float4 *>(resid) + 2 * v);
      const float4 r1 = __ldcg(reinterpret_cast<const float4 *>(resid) + 2 * v + 1);
      h[i][0] = r0.x; h[i][1] = r0.y; h[i][2] = r0.z; h[i][3] = r0.w;
      h[i][4] = r1.x; h[i][5] = r1.y; h[i][6] = r1.z; h[i][7] = r1.w;
      if constexpr (kSrc == 0) {
        const float4 d0 = __ldcg(reinterpret_cast<const float4 *>(delta) + 2 * v);
        const float4 d1 = __ldcg(reinterpret_cast<const float4 *>(delta) + 2 * v + 1);
        h[i][0] += d0.x; h[i][1] += d0.y; h[i][2] += d0.z; h[i][3] += d0.w;
        h[i][4] += d1.x; h[i][5] += d1.y; h[i][6] += d1.z; h[i][7] += d1.w;
      } else if constexpr (kSrc == 1) {
        acc8_act<F16>(h[i], __ldcg(reinterpret_cast<const uint4 *>(delta) + v));
      } else {
        // the partials are summed in fp32 first (same association as the
        // reduce-scatter path), then added to the residual
        float d[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int src = 0; src < kSrc; ++src)
          acc8_act<F16>(d, __ldcg(reinterpret_cast<const uint4 *>(
                              reinterpret_cast<const __nv_bfloat16 *>(g_peer_base[src] + part_off) +
                              part_elem) + v));
#pragma unroll
        for (int e = 0; e < 8; ++e) h[i][e] += d[e];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kHalfVec; ++i) {
    const int v = vbeg + lane + 32 * i;
    if (v < vend) {
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += h[i][e] * h[i][e];
      reinterpret_cast<float4 *>(sum_out)[2 * v] = make_float4(h[i][0], h[i][1], h[i][2], h[i][3]);
      reinterpret_cast<float4 *>(sum_out)[2 * v + 1] = make_float4(h[i][4], h[i][5], h[i][6], h[i][7]);
    }
  }
  ss = warp_allsum(ss);
  if (lane == 0) pair_ss[pair * 2 + half] = ss;
  named_bar_sync(3 + pair, 64);
  const float tot = pair_ss[pair * 2] + pair_ss[pair * 2 + 1];
  named_bar_sync(3 + pair, 64);  // both halves read before the slots are reused
  if (!do_norm) return;
  const float r = rsqrtf(tot * inv_h + eps);
#pragma unroll
  for (int i = 0; i < kHalfVec; ++i) {
    const int v = vbeg + lane + 32 * i;
    if (v < vend) {
      float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      acc8_bits(g, __ldg(reinterpret_cast<const uint4 *>(gamma) + v));
#pragma unroll
      for (int e = 0; e < 8; ++e) h[i][e] = h[i][e] * r * g[e];
      reinterpret_cast<uint4 *>(x_out)[v] = pack8f<F16>(h[i]);
    }
  }
}


// Bulk-staged form of pair_addnorm_row: the pair's leader has issued one bulk
// copy of the row's bf16 delta into shared memory (`stage`, completing on `bar`
// with parity `phase`); meanwhile the 64 threads load the residual (and, for the
// direct relay, this rank's own partial row) with ordinary loads.
//   kLocalPart = false: delta = stage                      (reduced row of the owner)
//   kLocalPart = true:  delta = local_part + stage          (k = 2: both partials,
//                       summed first, so every rank forms the same fp32 value)
// Returns false if the copy did not complete within limit_ns (the row is then
// left unwritten; the pair still meets at its barriers).
template <bool kLocalPart, bool F16>
__device__ __forceinline__ bool pair_addnorm_row_staged(
    const float *resid, const __nv_bfloat16 *local_part, const uint4 *stage, uint64_t *bar,
    uint32_t phase, uint64_t limit_ns, float *sum_out, const __nv_bfloat16 *gamma,
    __nv_bfloat16 *x_out, int hv, float inv_h, float eps, bool do_norm, int pair, int half,
    float *pair_ss) {
  const int lane = threadIdx.x & 31;
  const int hv0 = (hv + 1) / 2;
  const int vbeg = half ? hv0 : 0;
  const int vend = half ? hv : hv0;
  float h[kHalfVec][8];
  uint4 lp[kLocalPart ? kHalfVec : 1];
#pragma unroll
  for (int i = 0; i < kHalfVec; ++i) {
    const int v = vbeg + lane + 32 * i;
    if (v < vend) {
      const float4 r0 = __ldcg(reinterpret_cast<const float4 *>(resid) + 2 * v);
      const float4 r1 = __ldcg(reinterpret_cast<const float4 *>(resid) + 2 * v + 1);
      h[i][0] = r0.x; h[i][1] = r0.y; h[i][2] = r0.z; h[i][3] = r0.w;
      h[i][4] = r1.x; h[i][5] = r1.y; h[i][6] = r1.z; h[i][7] = r1.w;
      if constexpr (kLocalPart) lp[i] = __ldcg(reinterpret_cast<const uint4 *>(local_part) + v);
    }
  }
  const bool ok = mbar_wait(bar, phase, limit_ns);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kHalfVec; ++i) {
    const int v = vbeg + lane + 32 * i;
    if (v < vend) {
      float d[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if constexpr (kLocalPart) acc8_act<F16>(d, lp[i]);
      if (ok) acc8_act<F16>(d, stage[v]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        h[i][e] += d[e];
        ss += h[i][e] * h[i][e];
      }
      if (ok) {
        reinterpret_cast<float4 *>(sum_out)[2 * v] = make_float4(h[i][0], h[i][1], h[i][2], h[i][3]);
        reinterpret_cast<float4 *>(sum_out)[2 * v + 1] =
            make_float4(h[i][4], h[i][5], h[i][6], h[i][7]);
      }
    }
  }
  ss = warp_allsum(ss);
  if (lane == 0) pair_ss[pair * 2 + half] = ss;
  // pair-uniform outcome; also: every thread is done reading `stage`
  const bool pair_ok = named_bar_and(3 + pair, 64, ok);
  const float tot = pair_ss[pair * 2] + pair_ss[pair * 2 + 1];
  named_bar_sync(3 + pair, 64);
  if (!do_norm || !pair_ok) return pair_ok;
  const float r = rsqrtf(tot * inv_h + eps);
#pragma unroll
  for (int i = 0; i < kHalfVec; ++i) {
    const int v = vbeg + lane + 32 * i;
    if (v < vend) {
      float g[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      acc8_bits(g, __ldg(reinterpret_cast<const uint4 *>(gamma) + v));
#pragma unroll
      for (int e = 0; e < 8; ++e) h[i][e] = h[i][e] * r * g[e];
      reinterpret_cast<uint4 *>(x_out)[v] = pack8f<F16>(h[i]);
    }
  }
  return pair_ok;
}

// KR: ranks (compile-time so the partial registers fit); F16: fp16 data; BULK: staged bulk
// copies (each form is its own kernel, so the register-heavy forms do not share one
// register allocation)
template <int KR, bool F16, bool BULK>
__device__ __forceinline__ void relay_consumer(const RelayArgs &ra, const TileSched &ts,
                                               volatile int *flag_smem, float *pair_ss,
                                               uint8_t *stage_base, uint8_t *big_base,
                                               int big_slots, const volatile int *gemm_done) {
  // reduce-scatter units in flight per warp: KR partial vectors each
  constexpr int kRsBatch = KR <= 2 ? 4 : (KR == 4 ? 2 : 1);
  const int lane = threadIdx.x & 31;
  const int wl = (threadIdx.x >> 5) - kRelayWarp0;
  const int gw = blockIdx.x * kRelayWarps + wl;
  const int GW = gridDim.x * kRelayWarps;
  const int pair = wl >> 1, half = wl & 1;
  const int gp = blockIdx.x * (kRelayWarps / 2) + pair;
  const int GP = gridDim.x * (kRelayWarps / 2);
  // Exchange pairs (bulk forms): with quiet_signals the CTAs that run signal jobs (the
  // first T, or 2T for rsag) take no rows, so the system-scope fence of a signal job
  // does not wait behind its own CTA's NVLink loads; xgp < 0: no exchange rows here.
  const int nsig0 = (KR > 1 && ra.quiet_signals) ? (ra.direct ? ra.T : 2 * ra.T) : 0;
  const int nsig = (GP - nsig0 * (kRelayWarps / 2) >= GP / 2) ? nsig0 : 0;
  const int xgp = gp - nsig * (kRelayWarps / 2);
  const int XGP = GP - nsig * (kRelayWarps / 2);
  const uint32_t seq = (*ra.epoch - 1u) * uint32_t(ra.L) + uint32_t(ra.layer) + 1u;
  // k > 1: one forwarded signal per (row tile, source) and per (row tile, owner) each run
  const uint32_t rs_target = seq;
  const uint32_t ag_target = seq;
  const size_t rs_cnt_base = ra.flag_off;
  const size_t ag_cnt_base = ra.flag_off + size_t(ra.T) * ra.k * 128;
  const int units = ra.Rk * ra.nseg;
  const int hv = ra.H / 8;
  const float inv_h = 1.0f / float(ra.H);
  // after any earlier failure (status word set) do not wait again: give up fast
  uint64_t timeout = ra.timeout_ns;
  if (ra.status && *reinterpret_cast<volatile uint32_t *>(ra.status) != 0) timeout = 0;
  // bulk staging (BULK): one H-element row buffer and kRelaySlots mbarriers per pair (one
  // per staging slot); the pair's leader issues the copies, all 64 threads wait on them
  const bool leader = half == 0 && lane == 0;
  uint8_t *pbuf = BULK ? stage_base + size_t(pair) * ra.H * 2 : nullptr;
  uint64_t *pbar = BULK ? reinterpret_cast<uint64_t *>(stage_base + size_t(kRelayWarps / 2) *
                                                                          ra.H * 2) +
                                 pair * kRelaySlots
                           : nullptr;
  bool stuck = false;  // a copy did not complete in time: no new copies, drain at exit
  auto stage_fail = [&]() {
    if (!stuck) report_status(ra.status, kStatusRsWait);
    stuck = true;
    timeout = 0;
  };
  // Staging slots (bulk): while this CTA's GEMM runs, one H-element slot per pair (the
  // reserve behind the GEMM layout); once the GEMM is done here (the epilogue drained the
  // last accumulator, so no TMA load or MMA touches the pipeline buffers again),
  // `big_slots` slots per pair in the pipeline buffers, one copy in flight per slot.
  uint32_t parity = 0;    // bit i: the parity slot i's barrier completes next
  uint32_t inflight = 0;  // bit i: slot i holds a copy not yet waited for
  auto slot_ptr = [&](bool big, int i) -> uint8_t * {
    return big ? big_base + (size_t(pair) * big_slots + i) * ra.H * 2 : pbuf;
  };
  auto drain_slots = [&]() {
    // no bulk copy may still be writing this CTA's shared memory when it exits; a copy
    // that does not land within another timeout is reported and the CTA leaves anyway
    for (int i = 0; i < kRelaySlots; ++i)
      if (((inflight >> i) & 1u) && !mbar_wait(&pbar[i], (parity >> i) & 1u, ra.timeout_ns)) {
        if (leader) report_status(ra.status, kStatusCopyDrain);
      }
  };

  if constexpr (KR == 1) {
    // single rank: the fp32 partial rows of tile t sit in sum_out once the tile's
    // GEMM tiles are released; sum_out = resid + partial in place, then RMSNorm
    for (int t = 0; t < ra.T; ++t) {
      const bool ok =
          wait_all_sources(ra, rs_cnt_base, t, seq * uint32_t(ra.cta_group * ts.band_tiles(t)),
                           kStatusLocalWait,
                           timeout, flag_smem);
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 3 + 4 * t);
      if (!ok) {
        timeout = 0;
        continue;
      }
      for (int q = gp; q < ra.R; q += GP) {
        const size_t g = size_t(t) * ra.R + q;
        pair_addnorm_row<0, F16>(ra.resid + g * ra.H, ra.sum_out + g * ra.H, 0, 0, ra.sum_out + g * ra.H,
                            ra.gamma, ra.x_out + g * ra.H, hv, inv_h, ra.eps, ra.do_norm != 0, pair,
                            half, pair_ss);
      }
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 6 + 4 * t);
    }
    if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 2);
    return;
  }

  if constexpr (KR == 2 && BULK) {
    if (ra.direct) {
      // direct all-pull with bulk staging, over runs of row tiles found complete
      // together: each slot receives the peer's partial row by one bulk copy while the
      // pair loads the residual and this rank's own partial
      const int peer = 1 - ra.rank;
      const __nv_bfloat16 *mine = reinterpret_cast<const __nv_bfloat16 *>(ra.local_base + ra.part_off);
      const uint8_t *theirs = g_peer_base[peer] + ra.part_off;
      const int per = (xgp >= 0 && ra.R > xgp) ? (ra.R - xgp + XGP - 1) / XGP : 0;  // rows per tile
      int t0 = 0;
      while (t0 < ra.T) {
        const int w = wait_all_sources(ra, rs_cnt_base, t0, rs_target, kStatusRsWait, timeout,
                                       flag_smem, gemm_done, ra.T);
        const int t1 = w ? (w >> 8) : t0 + 1;
        for (int t = t0; t < t1; ++t)
          if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 3 + 4 * t);
        if (w == 0) {
          stuck = true;
          timeout = 0;
        }
        if (!stuck) {
          const bool big = (w & 2) && big_slots > 1;
          const int n = per * (t1 - t0);
          const int ns = big ? big_slots : 1;
          auto row_of = [&](int i) -> size_t {
            const int t = t0 + i / per;
            return size_t(t) * ra.R + xgp + size_t(i - (t - t0) * per) * XGP;
          };
          auto issue = [&](int i) {
            const int sl = i % ns;
            inflight |= 1u << sl;
            if (!leader) return;
            mbar_arrive_expect_tx(&pbar[sl], uint32_t(ra.H) * 2);
            bulk_load(slot_ptr(big, sl), theirs + row_of(i) * ra.H * 2, uint32_t(ra.H) * 2,
                      &pbar[sl]);
          };
          if (leader && n > 0) {
            fence_proxy_async_global();
            if (big) fence_proxy_async_shared();
          }
          for (int i = 0; i < n && i < ns; ++i) issue(i);
          for (int i = 0; i < n; ++i) {
            const int sl = i % ns;
            const size_t g = row_of(i);
            const bool rok = pair_addnorm_row_staged<true, F16>(
                ra.resid + g * ra.H, mine + g * ra.H,
                reinterpret_cast<const uint4 *>(slot_ptr(big, sl)), &pbar[sl], (parity >> sl) & 1u,
                ra.timeout_ns, ra.sum_out + g * ra.H, ra.gamma, ra.x_out + g * ra.H, hv, inv_h,
                ra.eps, ra.do_norm != 0, pair, half, pair_ss);
            if (!rok) {
              stage_fail();
              break;
            }
            parity ^= 1u << sl;
            inflight &= ~(1u << sl);
            if (i + ns < n) issue(i + ns);
          }
        }
        for (int t = t0; t < t1; ++t)
          if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 6 + 4 * t);
        t0 = t1;
      }
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 2);
      drain_slots();
      return;
    }
  }

  if constexpr (KR <= 4 && !BULK) {  // direct all-pull is offered up to 4 ranks
    if (ra.direct) {
      // direct all-pull: once every rank released tile t, each pair of warps sums
      // the k partial rows (local + NVLink loads) inside its Add+RMSNorm
      for (int t = 0; t < ra.T; ++t) {
        const bool ok =
            wait_all_sources(ra, rs_cnt_base, t, rs_target, kStatusRsWait, timeout, flag_smem);
        if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 3 + 4 * t);
        if (!ok) {
          timeout = 0;
          continue;
        }
        for (int q = gp; q < ra.R; q += GP) {
          const size_t g = size_t(t) * ra.R + q;
          pair_addnorm_row<KR, F16>(ra.resid + g * ra.H, nullptr, ra.part_off, g * ra.H,
                               ra.sum_out + g * ra.H, ra.gamma, ra.x_out + g * ra.H, hv, inv_h,
                               ra.eps, ra.do_norm != 0, pair, half, pair_ss);
        }
        if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 6 + 4 * t);
      }
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 2);
      return;
    }
  }

  // ---- rsag: reduce-scatter, then all-gather, over runs of row tiles [t0, t1).
  // Row tiles that become ready together (the GEMM completes them in the same wave) are
  // exchanged as ONE phase: one wait and one CTA barrier per phase instead of per tile,
  // and more copies in flight per pair.
  // one wait on slot i: every thread of the pair tracks the same parity / inflight bits
  auto slot_wait = [&](int i) -> bool {
    const bool ok = mbar_wait(&pbar[i], (parity >> i) & 1u, ra.timeout_ns);
    if (ok) {
      parity ^= 1u << i;
      inflight &= ~(1u << i);
    }
    return ok;
  };
  __nv_bfloat16 *red = reinterpret_cast<__nv_bfloat16 *>(ra.local_base + ra.red_off);

  // reduce-scatter of tiles [t0, t1): sum the k sources' partials of the rows this rank
  // owns in fp32 (source order), round once, store into the local `red` buffer, then
  // release ag_done[t] for each tile (the signal warp forwards it to every rank)
  auto rs_phase = [&](int t0, int t1, bool big) {
    for (int t = t0; t < t1; ++t)
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 3 + 4 * t);
    if (BULK && !stuck) {
      // unit = (owned row i, column segment seg of W = H/k columns): the leader stages
      // the k sources' segments (k bulk copies, source order) in one slot; the pair
      // sums them in fp32 in that order and stores the row segment
      const int W = ra.H / KR;
      const uint32_t seg_bytes = uint32_t(W) * 2;
      const int wv = W / 8;
      const int tid = half * 32 + lane;
      const int upt = ra.Rk * KR;                                  // units per tile
      const int mine = (xgp >= 0 && upt > xgp) ? (upt - xgp + XGP - 1) / XGP : 0;  // per tile
      const int n = mine * (t1 - t0);
      const int ns = big ? big_slots : 1;
      auto unit_at = [&](int i, size_t &g, int &seg) {
        const int t = t0 + i / mine;
        const int u = xgp + (i - (t - t0) * mine) * XGP;
        const int row = u / KR;
        seg = u - row * KR;
        g = size_t(t) * ra.R + size_t(ra.rank) * ra.Rk + row;
      };
      auto issue = [&](int i) {
        const int sl = i % ns;
        inflight |= 1u << sl;
        if (!leader) return;
        size_t g;
        int seg;
        unit_at(i, g, seg);
        const size_t off = (g * ra.H + size_t(seg) * W) * 2;
        uint8_t *dst = slot_ptr(big, sl);
        mbar_arrive_expect_tx(&pbar[sl], seg_bytes * KR);
#pragma unroll
        for (int src = 0; src < KR; ++src)
          bulk_load(dst + src * seg_bytes, g_peer_base[src] + ra.part_off + off, seg_bytes,
                    &pbar[sl]);
      };
      if (leader && n > 0) {
        fence_proxy_async_global();
        if (big) fence_proxy_async_shared();
      }
      for (int i = 0; i < n && i < ns; ++i) issue(i);
      for (int i = 0; i < n; ++i) {
        const int sl = i % ns;
        const bool uok = slot_wait(sl);
        if (uok) {
          size_t g;
          int seg;
          unit_at(i, g, seg);
          const uint4 *sv = reinterpret_cast<const uint4 *>(slot_ptr(big, sl));
          for (int v = tid; v < wv; v += 64) {
            float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int src = 0; src < KR; ++src) acc8_act<F16>(acc, sv[src * wv + v]);
            reinterpret_cast<uint4 *>(red + g * ra.H + size_t(seg) * W)[v] = pack8f<F16>(acc);
          }
        }
        // pair-uniform outcome, and every thread is done reading the slot
        if (!named_bar_and(3 + pair, 64, uok)) {
          stage_fail();
          break;
        }
        if (i + ns < n) issue(i + ns);
      }
    } else if (!BULK && !stuck) {
      for (int t = t0; t < t1; ++t)
        for (int u0 = gw * kRsBatch; u0 < units; u0 += GW * kRsBatch) {
          uint4 part[kRsBatch][KR];
#pragma unroll
          for (int b = 0; b < kRsBatch; ++b) {
            const int u = u0 + b;
            const int i = u / ra.nseg;
            const int col = (u - i * ra.nseg) * 256 + lane * 8;
            const size_t g = size_t(t) * ra.R + size_t(ra.rank) * ra.Rk + i;
            if (u < units && col < ra.H) {
              // pull: every source's partial row g (remote for src != rank)
#pragma unroll
              for (int src = 0; src < KR; ++src)
                part[b][src] = __ldcg(reinterpret_cast<const uint4 *>(
                    reinterpret_cast<const __nv_bfloat16 *>(g_peer_base[src] + ra.part_off) +
                    g * ra.H + col));
            }
          }
#pragma unroll
          for (int b = 0; b < kRsBatch; ++b) {
            const int u = u0 + b;
            const int i = u / ra.nseg;
            const int col = (u - i * ra.nseg) * 256 + lane * 8;
            if (u < units && col < ra.H) {
              float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
              for (int src = 0; src < KR; ++src) acc8_act<F16>(acc, part[b][src]);
              const size_t g = size_t(t) * ra.R + size_t(ra.rank) * ra.Rk + i;
              *reinterpret_cast<uint4 *>(red + g * ra.H + col) = pack8f<F16>(acc);
            }
          }
        }
    }
    // release of my reduced rows: one GPU-scope add per CTA and tile to the local
    // ag_done[t] by one thread after the CTA barrier (cumulative over the relay
    // threads' stores); the signal warp forwards each completed tile to every rank
    named_bar_sync(2, kRelayWarps * 32);
    for (int t = t0; t < t1; ++t) {
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 4 + 4 * t);
      if (threadIdx.x == kRelayWarp0 * 32 && !stuck) {
        red_add_release_gpu(
            flag_ptr(ra.local_base, ra.flag_off + (2 * size_t(ra.T) * KR + 2 + ra.T + t) * 128), 1u);
        if (t < 8) trace_mark(ra, 35 + t);
      }
    }
  };

  // all-gather of tiles [t0, t1): the reduced rows pulled from each row's owner, then
  // Add+RMSNorm
  auto ag_phase = [&](int t0, int t1, bool big) {
    for (int t = t0; t < t1; ++t)
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 5 + 4 * t);
    if (BULK && !stuck) {
      const int mine = (xgp >= 0 && ra.R > xgp) ? (ra.R - xgp + XGP - 1) / XGP : 0;  // rows per tile
      const int n = mine * (t1 - t0);
      const int ns = big ? big_slots : 1;
      auto row_at = [&](int i, size_t &g, int &q) {
        const int t = t0 + i / mine;
        q = xgp + (i - (t - t0) * mine) * XGP;
        g = size_t(t) * ra.R + q;
      };
      auto issue = [&](int i) {
        const int sl = i % ns;
        inflight |= 1u << sl;
        if (!leader) return;
        size_t g;
        int q;
        row_at(i, g, q);
        mbar_arrive_expect_tx(&pbar[sl], uint32_t(ra.H) * 2);
        bulk_load(slot_ptr(big, sl), g_peer_base[q / ra.Rk] + ra.red_off + g * ra.H * 2,
                  uint32_t(ra.H) * 2, &pbar[sl]);
      };
      if (leader && n > 0) {
        fence_proxy_async_global();
        if (big) fence_proxy_async_shared();
      }
      for (int i = 0; i < n && i < ns; ++i) issue(i);
      for (int i = 0; i < n; ++i) {
        const int sl = i % ns;
        size_t g;
        int q;
        row_at(i, g, q);
        const bool rok = pair_addnorm_row_staged<false, F16>(
            ra.resid + g * ra.H, nullptr, reinterpret_cast<const uint4 *>(slot_ptr(big, sl)),
            &pbar[sl], (parity >> sl) & 1u, ra.timeout_ns, ra.sum_out + g * ra.H, ra.gamma,
            ra.x_out + g * ra.H, hv, inv_h, ra.eps, ra.do_norm != 0, pair, half, pair_ss);
        if (!rok) {
          stage_fail();
          break;
        }
        parity ^= 1u << sl;
        inflight &= ~(1u << sl);
        if (i + ns < n) issue(i + ns);
      }
    } else if (!BULK && !stuck) {
      for (int t = t0; t < t1; ++t)
        for (int q = gp; q < ra.R; q += GP) {
          const size_t g = size_t(t) * ra.R + q;
          // reduced row g lives in its owner's `red` buffer (pulled over NVLink)
          const __nv_bfloat16 *red_row =
              reinterpret_cast<const __nv_bfloat16 *>(g_peer_base[q / ra.Rk] + ra.red_off) + g * ra.H;
          pair_addnorm_row<1, F16>(ra.resid + g * ra.H, red_row, 0, 0, ra.sum_out + g * ra.H,
                                   ra.gamma, ra.x_out + g * ra.H, hv, inv_h, ra.eps,
                                   ra.do_norm != 0, pair, half, pair_ss);
        }
    }
    for (int t = t0; t < t1; ++t)
      if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 6 + 4 * t);
  };

  // Phase order.  ra.ready_order (default): the first relay warp polls both counter sets
  // and takes whichever is ready -- the reduce-scatter when both are (the peers'
  // all-gathers wait on it) -- extended over every following tile that is ready too,
  // and publishes the choice; an all-gather never runs before its own reduce-scatter.
  // Otherwise the fixed software pipeline rs(0), rs(1), ag(0), rs(2), ag(1), ..., one
  // tile per phase, each behind a blocking wait.
  int next_rs = 0, next_ag = 0;
  while (next_ag < ra.T) {
    int choice = 0, t1 = 0;
    bool big = false;
    if (ra.ready_order) {
      // every decision below is the poller's, published through shared memory: the
      // relay threads' own `timeout` / `stuck` may differ by pair after a failure
      const uint64_t t0 = globaltimer_ns();
      while (choice == 0) {
        if ((threadIdx.x >> 5) == kRelayWarp0) {
          // runs only once the GEMM is done here: before that a pair has one slot and a
          // run would only delay the first tile's all-gather (one read, broadcast from lane
          // 0, so every lane takes the same branch into sources_ready's __all_sync)
          const bool done = __shfl_sync(0xffffffffu, *gemm_done != 0 ? 1 : 0, 0) != 0;
          int c = 0, e = 0;
          if (next_rs < ra.T && sources_ready(ra, rs_cnt_base, next_rs, rs_target)) {
            c = 1;
            e = next_rs + 1;
            while (done && e < ra.T && sources_ready(ra, rs_cnt_base, e, rs_target)) ++e;
          } else if (next_ag < next_rs && sources_ready(ra, ag_cnt_base, next_ag, ag_target)) {
            c = 2;
            e = next_ag + 1;
            while (done && e < next_rs && sources_ready(ra, ag_cnt_base, e, ag_target)) ++e;
          } else if (timeout == 0 || globaltimer_ns() - t0 > timeout) {
            c = 3;
          }
          if (lane == 0) flag_smem[0] = c | (e << 8) | (int(done) << 16);
        }
        // the lanes' acquire loads are ordered before every relay thread's later loads
        named_bar_sync(2, kRelayWarps * 32);
        const int w = flag_smem[0];
        named_bar_sync(2, kRelayWarps * 32);
        choice = w & 0xff;
        t1 = (w >> 8) & 0xff;
        big = ((w >> 16) & 1) && big_slots > 1;
        if (choice == 0) __nanosleep(64);
      }
    } else {
      choice = 3;
    }
    if (choice == 3) {
      // fixed order, or a poll that ran out of time: one tile behind a blocking wait
      // (which reports an expiry).  Fixed order: rs(t+1) goes before ag(t).
      const bool rs_now = ra.ready_order ? next_rs == next_ag
                                         : next_rs < ra.T && next_rs <= next_ag + 1;
      const int t = rs_now ? next_rs : next_ag;
      const int w = wait_all_sources(ra, rs_now ? rs_cnt_base : ag_cnt_base, t,
                                     rs_now ? rs_target : ag_target,
                                     rs_now ? kStatusRsWait : kStatusAgWait, timeout, flag_smem,
                                     gemm_done);
      if (w == 0) {
        stuck = true;
        timeout = 0;
      }
      choice = rs_now ? 1 : 2;
      t1 = t + 1;
      big = (w & 2) && big_slots > 1;
    }
    if (choice == 1) {
      rs_phase(next_rs, t1, big);
      next_rs = t1;
    } else {
      ag_phase(next_ag, t1, big);
      next_ag = t1;
    }
  }
  if (threadIdx.x == kRelayWarp0 * 32) trace_mark(ra, 2);
  drain_slots();
}

// ---------------------------------------------------------------- signal warp
// k > 1: the system-scope half of the two-level release.  Job j of this GPU (one
// per CTA j < njobs) waits until the local completion counter of its row tile is
// complete (acquire), then fences at system scope -- cumulative over every store
// those GPU-scope releases covered -- and adds 1 to the tile's counter on every
// rank.  Jobs 0..T-1 forward rs_done[t] to rs_cnt[t][rank]; jobs T..2T-1 (rsag)
// forward ag_done[t] to ag_cnt[t][rank].  Only 2T threads per GPU pay for a
// system-scope fence, off the GEMM epilogue and the relay warps.
__device__ __forceinline__ void relay_signal(const RelayArgs &ra, const TileSched &ts) {
  const int j = blockIdx.x;
  const int njobs = ra.direct ? ra.T : 2 * ra.T;
  if (ra.k == 1 || j >= njobs) return;
  uint64_t timeout = ra.timeout_ns;
  if (ra.status && *reinterpret_cast<volatile uint32_t *>(ra.status) != 0) timeout = 0;
  const uint32_t seq = (*ra.epoch - 1u) * uint32_t(ra.L) + uint32_t(ra.layer) + 1u;
  const bool ag = j >= ra.T;
  const int t = ag ? j - ra.T : j;
  const size_t tk = 2 * size_t(ra.T) * ra.k;
  const size_t done_line = ra.flag_off + (tk + 2 + (ag ? ra.T : 0) + t) * 128;
  const uint32_t target =
      seq * (ag ? uint32_t(gridDim.x) : uint32_t(ra.cta_group * ts.band_tiles(t)));
  if (!wait_counter_geq(flag_ptr(ra.local_base, done_line), target, timeout)) {
    report_status(ra.status, kStatusLocalWait);
    return;
  }
  const uint64_t f0 = ra.trace ? globaltimer_ns() : 0;
  fence_sys();
  const size_t cnt = ra.flag_off + ((ag ? size_t(ra.T) * ra.k : 0) + size_t(t) * ra.k + ra.rank) * 128;
  for (int p = 0; p < ra.k; ++p) red_add_relaxed_sys(flag_ptr(g_peer_base[p], cnt), 1u);
  if (ra.trace) {
    unsigned long long *tr = ra.trace + size_t(blockIdx.x) * kTraceSlots;
    const uint64_t now = globaltimer_ns();
    tr[46] = now;
    tr[47] = now - f0;
  }
}

template <int BN, int KR, bool F16, int V, bool BULK>
__global__ void __launch_bounds__(kRelayThreads, 1)
    relay_down_kernel(const __grid_constant__ CUtensorMap ta,
                      const __grid_constant__ CUtensorMap tb,
                      const __grid_constant__ CUtensorMap tb2, TileSched ts,
                      const __grid_constant__ RelayArgs ra) {
  extern __shared__ uint8_t smem_raw[];
  const GemmSmemView<BN, V> s = GemmSmemView<BN, V>::carve(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
    tma_prefetch_desc(&tb2);
  }
  // relay staging: kRelayWarps/2 pair buffers of H bf16, then their mbarriers
  using C = GemmCfg<BN, V>;
  uint8_t *stage_base = s.tiles + ((C::kTileBytes + C::kEpiBytes + C::kBarBytes + 127) & ~127u);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int i = 0; i < kMaxRanks; ++i) g_peer_base[i] = ra.peer_base[i];
    trace_mark(ra, 0);
    if (BULK) {
      uint64_t *bars = reinterpret_cast<uint64_t *>(stage_base + size_t(kRelayWarps / 2) * ra.H * 2);
      for (int i = 0; i < (kRelayWarps / 2) * kRelaySlots; ++i) mbar_init(&bars[i], 1);
    }
  }
  gemm_setup<BN, V>(s, 128);  // its barrier-init fence and __syncthreads cover the above
  if (warp == 0) {
    if (lane == 0) gemm_producer<BN, V>(s, &ta, &tb, &tb2, ts, ra.K, ra.status);
  } else if (warp == 1) {
    if (lane == 0) gemm_mma<BN, V, F16>(s, ts, ra.K, ra.status);
  } else if (warp < kRelayWarp0) {
    relay_push_epilogue<BN, V, F16>(s, ts, ra);
  } else if (warp < kSignalWarp) {
    // once this CTA's GEMM is done, its pipeline buffers hold big_slots row slots per pair
    const int big_slots =
        min(kRelaySlots, int(C::kTileBytes / (uint32_t(kRelayWarps / 2) * uint32_t(ra.H) * 2u)));
    relay_consumer<KR, F16, BULK>(ra, ts, reinterpret_cast<volatile int *>(s.abort) + 1, s.scratch,
                            stage_base, s.tiles, big_slots,
                            reinterpret_cast<volatile int *>(s.abort) + 2);
  } else if (lane == 0) {
    relay_signal(ra, ts);
  }
  gemm_teardown<BN, V>(s);
}

// ------------------------------------------------------------------ host side

// dynamic shared memory of the relay kernel: the GEMM pipeline, plus (bulk) the
// pair row buffers and their mbarriers behind it
template <int BN, int V>
static size_t relay_smem_bytes(int H, bool bulk) {
  using C = GemmCfg<BN, V>;
  if (!bulk) return C::kSmemBytes;
  return C::kSmemBytes + 128 + size_t(kRelayWarps / 2) * H * 2 + (kRelayWarps / 2) * kRelaySlots * 8;
}

// Bulk staging needs the row buffers to fit next to the GEMM pipeline (within the
// opt-in dynamic shared memory left beside the kernel's static shared memory) and
// every copy to be 16-byte aligned: rows (H bf16) and, for the reduce-scatter
// units, segments of H/k columns.
template <int BN, int V>
static bool relay_bulk_fits(int H, int k, size_t dyn_limit) {
  if (relay_smem_bytes<BN, V>(H, true) > dyn_limit) return false;
  if ((H * 2) % 16) return false;
  if (k > 1 && (H % k || (H / k) % 8)) return false;
  return true;
}

// The down GEMM runs on CTA pairs (256-row tiles, cta_group::2) when every row tile is a
// whole number of 256-row blocks and the tile width splits into two B halves of whole
// 16-row UMMA blocks; KRB_GEMM_PAIR=0 keeps one-CTA tiles.
bool relay_uses_pairs(int S, int T, int bn) {
  static const bool on = [] {
    const char *e = std::getenv("KRB_GEMM_PAIR");
    return !(e && e[0] == '0');
  }();
  return on && (bn == 256 || bn == 224) && (S / T) % 256 == 0;
}

// the opt-in dynamic shared memory left beside a relay kernel's static shared memory
// (set once per kernel and device)
template <int BN, int KR, bool F16, int V, bool BULK>
static size_t relay_dyn_limit(int dev) {
  static size_t lim[64] = {0};
  if (!lim[dev & 63]) {
    auto kern = relay_down_kernel<BN, KR, F16, V, BULK>;
    int optin = 0;
    KRB_CUDA(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
    cudaFuncAttributes fa{};
    KRB_CUDA(cudaFuncGetAttributes(&fa, kern));
    const size_t l = size_t(optin) - fa.sharedSizeBytes;
    KRB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(l)));
    lim[dev & 63] = l;
  }
  return lim[dev & 63];
}

template <int BN, int KR, bool F16, int V>
static void launch_relay(const CUtensorMap &tma, const void *w_down, long ldb,
                         const RelayArgs &ra_in, bool want_bulk, int grid, cudaStream_t stream) {
  using C = GemmCfg<BN, V>;
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  // k = 1 has no exchange; the direct form stages in bulk only at k = 2
  constexpr bool kBulkForm = KR > 1;
  static const bool quiet_env = [] {
    const char *e = std::getenv("KRB_RELAY_QUIET_SIGNALS");
    return !(e && e[0] == '0');
  }();
  RelayArgs ra = ra_in;
  ra.cta_group = C::kCG;
  ra.quiet_signals = quiet_env ? 1 : 0;
  ra.bulk = (kBulkForm && want_bulk && (!ra.direct || ra.k == 2) &&
             relay_bulk_fits<BN, V>(ra.H, ra.k, relay_dyn_limit<BN, KR, F16, V, kBulkForm>(dev)))
                ? 1
                : 0;
  auto kern = ra.bulk ? relay_down_kernel<BN, KR, F16, V, kBulkForm>
                      : relay_down_kernel<BN, KR, F16, V, false>;
  const size_t lim = ra.bulk ? relay_dyn_limit<BN, KR, F16, V, kBulkForm>(dev)
                             : relay_dyn_limit<BN, KR, F16, V, false>(dev);
  const size_t smem = relay_smem_bytes<BN, V>(ra.H, ra.bulk != 0);
  if (smem > lim) throw CudaError("relay: shared memory budget exceeded");
  const TileSched ts = relay_tile_sched(ra.S, ra.H, ra.T, BN, grid, C::kCG);
  // B boxes: the tile's rows of W_down, split between the pair's CTAs
  const CUtensorMap tmb = make_tmap_2d_bf16(w_down, ra.H, ra.K, ldb, BN / C::kCG, kBK);
  const CUtensorMap tmb2 = make_tmap_2d_bf16(w_down, ra.H, ra.K, ldb, ts.bn2 / C::kCG, kBK);
  // cooperative: every CTA must be co-resident, because the relay warps wait
  // for tiles produced by other CTAs of the same grid; pairs: clusters of two
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRelayThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = C::kCG;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = C::kCG == 2 ? 2 : 1;
  KRB_CUDA(cudaLaunchKernelEx(&cfg, kern, tma, tmb, tmb2, ts, ra));
}

template <typename T>
void relay_down_layer(const T *act, long lda, const T *w_down, long ldb, int bn,
                      const RelayArgs &ra, cudaStream_t stream) {
  constexpr bool F16 = ActFmt<T>::f16;
  if (ra.S % kBM) throw CudaError("relay: seq must be a multiple of 128");
  if (ra.R % kBM) throw CudaError("relay: rows per tile must be a multiple of 128");
  if (ra.H % 8) throw CudaError("relay: hidden must be a multiple of 8");
  if (ra.H > 4096) throw CudaError("relay: hidden must be at most 4096");
  if (ra.k < 1 || ra.k > kMaxRanks || ra.R % ra.k) throw CudaError("relay: bad rank count");
  // bf16 serves the one-device entry points; the exchange paths are built for fp16
  if (!F16 && ra.k != 1) throw CudaError("relay: bf16 operands only with one rank");
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  const CUtensorMap tma = make_tmap_2d_bf16(act, ra.S, ra.K, lda, kBM, kBK);
  const int grid = sm_count(dev);
  if (ra.k > 1 && 2 * ra.T > grid) throw CudaError("relay: more row tiles than signal jobs");
  // the consumer publishes its choice of a run of row tiles with tile indexes in 8-bit
  // fields; 32 row tiles stay well inside them
  if (ra.k > 1 && ra.T > 32) throw CudaError("relay: at most 32 row tiles with more than one rank");
  auto by_ranks = [&](auto bn_tag) {
    constexpr int B = decltype(bn_tag)::value;
    // bulk staging serves the exchange paths: reduce-scatter + all-gather, and the
    // direct relay at k = 2 (one remote row per row); KRB_RELAY_BULK=0 turns it off
    static const bool bulk_env = [] {
      const char *e = std::getenv("KRB_RELAY_BULK");
      return !(e && e[0] == '0');
    }();
    auto with_cfg = [&](auto v_tag) {
      constexpr int V = decltype(v_tag)::value;
      if constexpr (!F16) {
        launch_relay<B, 1, false, V>(tma, w_down, ldb, ra, false, grid, stream);
      } else {
        const bool want = bulk_env && ra.k > 1 && (!ra.direct || ra.k == 2);
        switch (ra.k) {
          case 1: launch_relay<B, 1, true, V>(tma, w_down, ldb, ra, false, grid, stream); break;
          case 2: launch_relay<B, 2, true, V>(tma, w_down, ldb, ra, want, grid, stream); break;
          case 4: launch_relay<B, 4, true, V>(tma, w_down, ldb, ra, want, grid, stream); break;
          case 8: launch_relay<B, 8, true, V>(tma, w_down, ldb, ra, want, grid, stream); break;
          default: throw CudaError("relay: rank count must be 1, 2, 4 or 8");
        }
      }
    };
    if constexpr (B == 256 || B == 224) {
      if (relay_uses_pairs(ra.S, ra.T, B)) {
        with_cfg(std::integral_constant<int, kCfgPairRelay>{});
        return;
      }
    }
    with_cfg(std::integral_constant<int, kCfgRelay>{});
  };
  switch (bn) {
    case 256: by_ranks(std::integral_constant<int, 256>{}); break;
    case 224: by_ranks(std::integral_constant<int, 224>{}); break;
    case 128: by_ranks(std::integral_constant<int, 128>{}); break;
    default: throw CudaError("relay: unsupported bn");
  }
}

template void relay_down_layer<__nv_bfloat16>(const __nv_bfloat16 *, long, const __nv_bfloat16 *,
                                              long, int, const RelayArgs &, cudaStream_t);
template void relay_down_layer<__half>(const __half *, long, const __half *, long, int,
                                       const RelayArgs &, cudaStream_t);

// ------------------------------------------------- allocation-free relay scratch
// Scratch of krb_relay_down_single_noalloc: the flag counters and the run epoch
// of a one-device relay (k = 1 needs no partial or reduced-row buffers: the fp32
// partial tile goes straight into sum_out).  A module-scope device array exists
// once per device, so concurrent calls on one device share it.
static __device__ __align__(256) uint8_t g_relay_noalloc_scratch[kRelayNoAllocScratchBytes];

uint8_t *relay_noalloc_scratch() {
  static std::mutex mu;
  static uint8_t *addr[64] = {};
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) throw CudaError("relay scratch: device index out of range");
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    // once per device, with that device current: look up this device's copy
    void *p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_relay_noalloc_scratch);
    if (rc != cudaSuccess || !p)
      throw CudaError(std::string("cudaGetSymbolAddress(relay scratch) failed: ") +
                      cudaGetErrorString(rc));
    addr[dev] = static_cast<uint8_t *>(p);
  }
  return addr[dev];
}

// The relay GEMM's tile schedule: one band per row tile (row tile t completes before t+1),
// the two-phase tail re-cut when the tiles need between one and two waves of `grid` CTAs.
// cta_group 2: tile rows of 256 over grid / 2 CTA pairs.
TileSched relay_tile_sched(int S, int H, int T, int bn, int grid, int cta_group) {
  const int rows = kBM * cta_group;
  return TileSched::make(S / rows, H, bn, (S / T) / rows, grid / cta_group, true, 16 * cta_group);
}

}  // namespace krb
