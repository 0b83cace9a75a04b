// Shared definitions of the tp_split relay: row ownership, the symmetric buffer
// layout and the argument block of the fused down-GEMM + reduce + Add+RMSNorm kernel.
#pragma once

#include <stdint.h>

#include <cuda_bf16.h>

namespace krb {

constexpr int kMaxRanks = 8;

#ifdef __CUDACC__
#define KRB_RELAY_HD __host__ __device__ __forceinline__
#else
#define KRB_RELAY_HD inline
#endif

// Row ownership of the tp_split relay: global row g of the S rows lies in row
// tile rt = g / R; within the tile the rows are cut into k contiguous owner
// slices of Rk = R / k rows.  Used by the host (the relay plan's per-block owners).
struct RowRoute {
  int tile, owner, local;
};
KRB_RELAY_HD RowRoute relay_route(int g, int R, int Rk) {
  RowRoute r;
  r.tile = g / R;
  const int within = g - r.tile * R;
  r.owner = within / Rk;
  r.local = within - r.owner * Rk;
  return r;
}

// Per-rank symmetric region (one allocation, mapped by every peer).  All writes
// into a region are made by its own rank; peers only READ it (pull protocol), so
// every system-scope release covers local stores only.
//   part   [S][H] 2-byte this rank's partial down_proj output (GEMM epilogue; fp16 in
//                        the engine)
//   red    [S][H] 2-byte reduced rows (sum over ranks) of the rows this rank owns
//   flags  rs_cnt[T][k]: "source src released tile t" (incremented by the sources),
//          ag_cnt[T][k]: "owner j released its reduced rows of tile t" (incremented
//          by the owners), the local run epoch (+1 spare line), then the local
//          completion counters rs_done[T] (GEMM tiles of row tile t stored) and
//          ag_done[T] (CTAs that stored their reduced rows of tile t); one
//          128-byte line each.
struct SymLayout {
  size_t part_off, red_off, flag_off, bytes;
  static constexpr size_t kLine = 128;
  int T, k;
  static SymLayout make(int S, int H, int T, int k) {
    SymLayout L;
    L.T = T;
    L.k = k;
    const size_t rows_bytes = (size_t(S) * size_t(H) * 2 + 4095) & ~size_t(4095);
    L.part_off = 0;
    L.red_off = rows_bytes;
    L.flag_off = 2 * rows_bytes;
    L.bytes = L.flag_off + (2 * size_t(T) * size_t(k) + 2 + 2 * size_t(T)) * kLine;
    return L;
  }
  // counters and epoch only, at offset 0 (one-device relay: k = 1, where the
  // partial rows go straight to sum_out and no reduced rows exist)
  static SymLayout flags_only(int T) {
    SymLayout L;
    L.T = T;
    L.k = 1;
    L.part_off = 0;
    L.red_off = 0;
    L.flag_off = 0;
    L.bytes = (2 * size_t(T) + 2) * kLine;
    return L;
  }
  size_t rs_cnt(int t, int src) const { return flag_off + (size_t(t) * k + src) * kLine; }
  size_t ag_cnt(int t, int src) const {
    return flag_off + (size_t(T) * k + size_t(t) * k + src) * kLine;
  }
  size_t epoch() const { return flag_off + 2 * size_t(T) * k * kLine; }
  size_t rs_done(int t) const { return flag_off + (2 * size_t(T) * k + 2 + t) * kLine; }
  size_t ag_done(int t) const { return flag_off + (2 * size_t(T) * k + 2 + T + t) * kLine; }
};

// Size of the static device scratch behind krb_relay_down_single_noalloc: one
// 128-byte counter line per row tile plus the epoch lines of the flags-only
// layout, (2 * tiles + 2) * 128 bytes, so at most 127 row tiles.
constexpr size_t kRelayNoAllocScratchBytes = 32768;

struct RelayArgs {
  int S, H, K;          // down GEMM: M = S rows, N = H, K = I/k
  int T, k, rank;       // row tiles, ranks, this rank
  int R, Rk;            // rows per tile, rows per owner slice (R = k * Rk)
  int nseg;             // 256-column segments per row (H / 256, rounded up)
  // peers' symmetric regions as seen from this GPU (index = peer rank)
  uint8_t *peer_base[kMaxRanks];
  uint8_t *local_base;
  size_t part_off, red_off, flag_off;
  // Releases, per layer.  k = 1: every GEMM tile's epilogue adds 1 to rs_cnt[t][0]
  // (target: the GEMM tiles of row tile t, TileSched::band_tiles(t)).  k > 1, two
  // levels: each GEMM tile's epilogue adds 1 to the local rs_done[t] at GPU scope
  // (target band_tiles(t)); once it is complete, one signal thread per GPU fences at
  // system scope and adds 1 to rs_cnt[t][rank] on every rank (target 1); likewise
  // every CTA adds 1 to ag_done[t] after storing its reduced rows (target: the grid)
  // and one signal thread forwards 1 to ag_cnt[t][rank] (target 1).  Targets scale
  // with the run epoch and layer (monotone counters).
  // CTAs per GEMM tile (2: the down GEMM runs on CTA pairs with 256-row tiles; every CTA
  // releases its 128 rows, so a row tile's target is cta_group x its GEMM tiles)
  int cta_group;
  // 1: direct all-pull (every rank sums all k partials of every row inside its
  // Add+RMSNorm; one synchronisation per tile, (k-1) tiles over NVLink per rank);
  // 0: reduce-scatter + all-gather (2(k-1)/k tiles over NVLink, two synchronisations)
  int direct;
  // 1: the relay warps stage remote rows in shared memory with bulk copies (set
  // by the launcher when the shared-memory budget and the alignment allow it)
  int bulk;
  // reduce-scatter + all-gather form only: 0 = reduce-scatter of tile t+1 before the
  // all-gather of t (default), 1 = take whichever phase is ready first, in runs of ready
  // tiles once the GEMM is done (KRB_RELAY_ORDER=ready)
  int ready_order;
  // 1 (default): the CTAs that run signal jobs take no exchange rows, so their
  // system-scope fences do not wait behind their own NVLink loads (set by the launcher;
  // KRB_RELAY_QUIET_SIGNALS=0 spreads the rows over every CTA)
  int quiet_signals;
  const uint32_t *epoch;  // local run counter (bumped once per prefill)
  int layer, L;
  const float *resid;          // h1 [S, H] fp32 residual stream
  const __nv_bfloat16 *gamma;  // [H]
  float *sum_out;              // h0 (or hf) [S, H] fp32
  __nv_bfloat16 *x_out;        // x (or xf) [S, H]
  float eps;
  int do_norm;
  uint64_t timeout_ns;
  uint32_t *status;
  // optional phase trace (globaltimer ns), kTraceSlots per CTA; null = off
  unsigned long long *trace;
};

// trace slots per CTA: 0 start, 1 GEMM epilogue done, 2 relay end,
// then per row tile t < 8: 3+4t partials arrived, 4+4t reduced rows stored,
// 5+4t reduced rows of all owners arrived, 6+4t add+norm done;
// 35+t: reduced rows released (local GPU-scope release);
// 43/44/45: the epilogue's releases: total ns, count, longest ns;
// 46: this CTA's signal job forwarded (k > 1), 47: its system-scope fence in ns
constexpr int kTraceSlots = 48;

}  // namespace krb
