// Output tile schedule of the persistent tcgen05 GEMMs (host and device).
#pragma once

#ifdef __CUDACC__
#define KRB_TS_HD __host__ __device__
#else
#define KRB_TS_HD
#endif

namespace krb {

// Output tile schedule of a persistent GEMM over `grid` CTAs.
//
// Phase 1: tiles of width BN in band order -- the output rows are cut into bands of
// `band` 128-row blocks; all tiles of band 0 come first (row blocks fastest), then band
// 1, ...  A plain GEMM uses one band covering all rows; the relay kernel uses one band
// per row tile of the tp_split schedule, so row tile t completes before row tile t+1.
//
// Phase 2 (two_phase): when the BN tiles need more than one wave but less than two,
// phase 1 stops after the largest whole number of band columns that fits in one wave
// (p1 <= grid tiles), and the columns left over -- the rest of band b1 from column c1,
// then every later band -- are re-cut into the narrowest tiles (width bn2, a multiple of
// 16) that still fit in one more wave.  The GEMM then ends after 1 + bn2/BN tile times
// instead of 2 (Qwen 7B down_proj / o_proj, N = 3584 at BN = 224 on 148 SMs: 256 tiles
// become 148 + 140 tiles of width 176, 1.79 instead of 2 tile times).
struct TileSched {
  int num_m;   // 128-row blocks
  int num_n;   // BN-column blocks (phase 1)
  int band;    // row blocks per band (num_m % band == 0)
  int BN;      // phase-1 tile width
  int N;       // output columns
  int p1;      // phase-1 tiles (all tiles when there is no phase 2)
  int bn2;     // phase-2 tile width
  int b1, c1;  // band where phase 2 starts, and its first column there
  int t2a;     // phase-2 tiles of band b1
  int t2b;     // phase-2 tiles of each later band
  int total_;

  static int cdiv(int a, int b) { return (a + b - 1) / b; }

  // host: one phase, or two when that shortens the GEMM
  // step: granularity of the phase-2 width (16; 32 for CTA pairs, whose B halves are
  // whole 16-row UMMA blocks)
  static TileSched make(int num_m, int N, int BN, int band, int grid, bool two_phase,
                        int step = 16) {
    TileSched t{};
    t.num_m = num_m;
    t.N = N;
    t.BN = BN;
    t.num_n = cdiv(N, BN);
    t.band = band;
    t.bn2 = BN;
    const int total1 = num_m * t.num_n;
    t.p1 = total1;
    t.total_ = total1;
    t.b1 = num_m / band;
    t.c1 = 0;
    t.t2a = t.t2b = 0;
    if (!two_phase || total1 <= grid || total1 > 2 * grid) return t;
    const int per_band = band * t.num_n;
    const int p1 = (grid / band) * band;
    if (p1 <= 0 || p1 >= total1) return t;
    const int b1 = p1 / per_band;
    const int c1 = ((p1 - b1 * per_band) / band) * BN;
    const int later = num_m / band - b1 - 1;
    for (int w = 64; w < BN; w += step) {
      const int a = (b1 < num_m / band) ? cdiv(N - c1, w) * band : 0;
      const int b = cdiv(N, w) * band;
      if (a + later * b <= grid) {
        t.p1 = p1;
        t.bn2 = w;
        t.b1 = b1;
        t.c1 = c1;
        t.t2a = a;
        t.t2b = b;
        t.total_ = p1 + a + later * b;
        return t;
      }
    }
    return t;
  }

  KRB_TS_HD int total() const { return total_; }

  // tile idx -> first row block mb, first column n0, width bn (columns past N are
  // computed on zero-filled operands and not stored)
  KRB_TS_HD void tile(int idx, int &mb, int &n0, int &bn) const {
    if (idx < p1) {
      const int per_band = band * num_n;
      const int b = idx / per_band;
      const int r = idx - b * per_band;
      const int nb = r / band;
      mb = b * band + (r - nb * band);
      n0 = nb * BN;
      bn = BN;
      return;
    }
    int j = idx - p1;
    int b, c0;
    if (j < t2a) {
      b = b1;
      c0 = c1;
    } else {
      j -= t2a;
      const int q = j / t2b;
      b = b1 + 1 + q;
      j -= q * t2b;
      c0 = 0;
    }
    const int nb = j / band;
    mb = b * band + (j - nb * band);
    n0 = c0 + nb * bn2;
    bn = bn2;
  }

  // tiles of row band b (every width): the releases that complete the band
  KRB_TS_HD int band_tiles(int b) const {
    if (b < b1) return band * num_n;
    const int two = p1 < total_;
    if (b == b1) return two ? c1 / BN * band + t2a : band * num_n;
    return two ? t2b : band * num_n;
  }
};

}  // namespace krb
