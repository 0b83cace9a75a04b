// Shared definitions of the tp_split relay: symmetric buffer layout and the
// argument block of the fused down-GEMM + reduce + all-gather + Add+RMSNorm kernel.
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
// slices of Rk = R / k rows.  Used by the device epilogue (where to push a
// partial row) and by the host (expected counter increments).
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

// Per-rank symmetric region (one allocation, mapped by every peer):
//   rs_buf  [T][k][Rk][H] bf16   partial rows pushed by each source rank for the
//                                 rows this rank owns (owner slice of each tile)
//   ag_buf  [S][H] bf16           reduced rows pushed by every owner (all-gather)
//   flags   rs_cnt[T][k], ag_cnt[T][k] u32 monotone counters, then the local
//           run epoch counter; each counter on its own 128-byte line.
struct SymLayout {
  size_t rs_off, ag_off, flag_off, bytes;
  static constexpr size_t kLine = 128;
  int T, k;
  static SymLayout make(int S, int H, int T, int k) {
    SymLayout L;
    L.T = T;
    L.k = k;
    const size_t rows_bytes = size_t(S) * size_t(H) * 2;
    L.rs_off = 0;
    L.ag_off = (rows_bytes + 4095) & ~size_t(4095);
    L.flag_off = L.ag_off + ((rows_bytes + 4095) & ~size_t(4095));
    L.bytes = L.flag_off + (2 * size_t(T) * size_t(k) + 2) * kLine;
    return L;
  }
  size_t rs_cnt(int t, int src) const { return flag_off + (size_t(t) * k + src) * kLine; }
  size_t ag_cnt(int t, int src) const {
    return flag_off + (size_t(T) * k + size_t(t) * k + src) * kLine;
  }
  size_t epoch() const { return flag_off + 2 * size_t(T) * k * kLine; }
};

struct RelayArgs {
  int S, H, K;          // down GEMM: M = S rows, N = H, K = I/k
  int T, k, rank;       // row tiles, ranks, this rank
  int R, Rk;            // rows per tile, rows per owner slice (R = k * Rk)
  int nseg;             // 256-column segments per row (H / 256, rounded up)
  // peers' symmetric regions as seen from this GPU (index = peer rank)
  uint8_t *peer_base[kMaxRanks];
  uint8_t *local_base;
  size_t rs_off, ag_off, flag_off;
  uint32_t rs_expect;   // increments per (tile, source) per layer on the owner
  uint32_t ag_expect;   // increments per (tile, owner) per layer on every rank
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
};

}  // namespace krb
