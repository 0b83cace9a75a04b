// tp_split: the fused down_proj producer + relay consumer for one layer.
//
// Reference path (qwen_main.cpp:1274-1302): for each of T row tiles,
//   down_t = act_t . W_down_r            (aclnnMatmul on the AIC stream)
//   publish/wait GM flag                 (kr_publish_aic / kr_wait_aiv)
//   red_t = AllReduce_sum(down_t)        (HcclAllReduce on the comm stream)
//   h0_t, x_t = AddRmsNorm(h1_t, red_t)  (aclnnAddRmsNorm)
//
// B200 design: ONE persistent cooperative kernel per layer and rank, 320 threads:
//   warps 0..5  tcgen05 GEMM (producer, MMA, 4 push-epilogue warps) over the
//               output tiles in row-tile order.  The epilogue stores each row of
//               its partial tile directly into the OWNER rank's rs_buf (owner =
//               row slice of the row tile; remote rows go over NVLink through the
//               peer mapping), fences at system scope and releases the owner's
//               rs_cnt[t][rank] counter (the GM-flag publish).
//   warps 6..9  relay: for t = 0..T-1, acquire rs_cnt[t][*] (the GM-flag wait,
//               bounded), sum the k partial slices of this rank's owned rows in
//               fp32, round once to bf16 and push the reduced rows to every
//               rank's ag_buf (all-gather), release ag_cnt[t][rank] on each
//               rank; then acquire ag_cnt[t][*] and apply h0 = h1 + red,
//               x = RMSNorm(h0) * gamma to the tile's rows.
// The reduction of tile t and its Add+RMSNorm overlap the GEMM of later tiles.
// No kernel ever waits on another kernel of the same GPU: the waits inside
// this kernel target (a) other CTAs of this co-resident cooperative grid and
// (b) the same kernel on peer GPUs.  Counters are monotone; targets are derived
// from the run epoch and layer index, so CUDA-graph replays need no reset.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.h"
#include "gemm.cuh"
#include "relay.cuh"

namespace krb {

constexpr int kRelayThreads = 320;
constexpr int kRelayWarp0 = 6;

__device__ __forceinline__ uint32_t *flag_ptr(uint8_t *base, size_t off) {
  return reinterpret_cast<uint32_t *>(base + off);
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

__device__ __forceinline__ uint4 pack8f(const float *f) {
  uint4 w;
  w.x = pack_bf16x2(f[0], f[1]);
  w.y = pack_bf16x2(f[2], f[3]);
  w.z = pack_bf16x2(f[4], f[5]);
  w.w = pack_bf16x2(f[6], f[7]);
  return w;
}

// ---------------------------------------------------------------- push epilogue
template <int BN>
__device__ __forceinline__ void relay_push_epilogue(const GemmSmemView<BN> &s, const TileSched &ts,
                                                    const RelayArgs &ra) {
  using C = GemmCfg<BN>;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int quad = warp & 3;
  const uint32_t tmem = *s.tmem_slot;
  int it = 0;
  for (int t = blockIdx.x; t < ts.total(); t += gridDim.x, ++it) {
    int mb, nb;
    ts.tile(t, mb, nb);
    const int acc = it & 1;
    const uint32_t acc_phase = (it >> 1) & 1;
    // collective decision: the four epilogue warps meet at named barrier 1 below,
    // so either all of them continue with this tile or all of them stop
    bool ok = mbar_wait(&s.tfull[acc], acc_phase, kMbarLimitNs) && !*s.abort;
    ok = named_bar_and(1, 128, ok);
    if (!ok) {
      report_status(ra.status, kStatusEpiWait);
      *s.abort = 1;
      break;
    }
    tc_fence_after();
    const int g = mb * kBM + quad * 32 + lane;      // global row (< S: S % 128 == 0)
    const RowRoute rr = relay_route(g, ra.R, ra.Rk);
    __nv_bfloat16 *dst = reinterpret_cast<__nv_bfloat16 *>(ra.peer_base[rr.owner] + ra.rs_off) +
                         ((static_cast<size_t>(rr.tile) * ra.k + ra.rank) * ra.Rk + rr.local) *
                             static_cast<size_t>(ra.H);
    const uint32_t tbase = tmem + (static_cast<uint32_t>(quad * 32) << 16) + acc * C::kAccStride;
#pragma unroll 1
    for (int c = 0; c < BN / 32; ++c) {
      const int col0 = nb * BN + c * 32;
      if (col0 >= ra.H) break;
      uint32_t r[32];
      tmem_ld_32x32(tbase + c * 32, r);
      tmem_wait_ld();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      store_row32_bf16(dst + col0, v, min(32, ra.H - col0));
    }
    tc_fence_before();
    mbar_arrive(&s.tempty[acc]);  // accumulator free for the next tile
    fence_sys();                  // this thread's pushes visible system-wide
    named_bar_sync(1, 128);
    if (warp == 2 && lane == 0) {
      // one release per owner whose slice this 128-row block touches
      const RowRoute first = relay_route(mb * kBM, ra.R, ra.Rk);
      const RowRoute last = relay_route(mb * kBM + kBM - 1, ra.R, ra.Rk);
      for (int j = first.owner; j <= last.owner; ++j)
        red_add_release_sys(
            flag_ptr(ra.peer_base[j], ra.flag_off + (size_t(first.tile) * ra.k + ra.rank) * 128),
            1u);
    }
  }
}

// ---------------------------------------------------------------- relay warps
__device__ __forceinline__ bool wait_all_sources(const RelayArgs &ra, size_t cnt_base, int t,
                                                 uint32_t target, uint32_t code) {
  const int lane = threadIdx.x & 31;
  int ok = 1;
  if (lane == 0) {
    for (int src = 0; src < ra.k; ++src) {
      const uint32_t *p = flag_ptr(ra.local_base, cnt_base + (size_t(t) * ra.k + src) * 128);
      if (!wait_counter_geq(p, target, ra.timeout_ns)) {
        report_status(ra.status, code);
        ok = 0;
        break;
      }
    }
  }
  ok = __shfl_sync(0xffffffffu, ok, 0);
  if (ok) {
    // every lane performs its own acquire so its later loads are ordered
    for (int src = 0; src < ra.k; ++src)
      (void)ld_acquire_sys(flag_ptr(ra.local_base, cnt_base + (size_t(t) * ra.k + src) * 128));
  }
  return ok != 0;
}

__device__ void relay_consumer(const RelayArgs &ra) {
  const int lane = threadIdx.x & 31;
  const int wl = (threadIdx.x >> 5) - kRelayWarp0;   // 0..3
  const int gw = blockIdx.x * 4 + wl;
  const int GW = gridDim.x * 4;
  const uint32_t seq = (*ra.epoch - 1u) * uint32_t(ra.L) + uint32_t(ra.layer) + 1u;
  const uint32_t rs_target = seq * ra.rs_expect;
  const uint32_t ag_target = seq * ra.ag_expect;
  const size_t rs_cnt_base = ra.flag_off;
  const size_t ag_cnt_base = ra.flag_off + size_t(ra.T) * ra.k * 128;
  const int units = ra.Rk * ra.nseg;
  const __nv_bfloat16 *rs_local =
      reinterpret_cast<const __nv_bfloat16 *>(ra.local_base + ra.rs_off);
  const __nv_bfloat16 *ag_local =
      reinterpret_cast<const __nv_bfloat16 *>(ra.local_base + ra.ag_off);
  const float inv_h = 1.0f / float(ra.H);
  // after any earlier failure (status word set) do not wait again: give up fast
  RelayArgs rq = ra;
  if (ra.status && *reinterpret_cast<volatile uint32_t *>(ra.status) != 0) rq.timeout_ns = 0;

  for (int t = 0; t < ra.T; ++t) {
    // ---- reduce-scatter half: wait for every source's partial of my slice
    const bool rs_ok = wait_all_sources(rq, rs_cnt_base, t, rs_target, kStatusRsWait);
    int done = 0;
    if (rs_ok) {
      for (int u = gw; u < units; u += GW) {
        const int i = u / ra.nseg;
        const int sg = u - i * ra.nseg;
        const int col = sg * 256 + lane * 8;
        if (col < ra.H) {
          float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
          for (int src = 0; src < ra.k; ++src)
            acc8_cg(acc, rs_local + ((size_t(t) * ra.k + src) * ra.Rk + i) * size_t(ra.H) + col);
          const uint4 w = pack8f(acc);
          const size_t g = size_t(t) * ra.R + size_t(ra.rank) * ra.Rk + i;
          for (int p = 0; p < ra.k; ++p) {
            uint4 *dst = reinterpret_cast<uint4 *>(
                reinterpret_cast<__nv_bfloat16 *>(ra.peer_base[p] + ra.ag_off) + g * ra.H + col);
            *dst = w;
          }
        }
        ++done;
      }
    }
    // ---- all-gather release: one signal per CTA and destination rank
    fence_sys();
    named_bar_sync(2, 128);
    if (wl == 0 && lane == 0 && rs_ok) {
      uint32_t cta_units = 0;
      for (int w = 0; w < 4; ++w) {
        const int g0 = blockIdx.x * 4 + w;
        if (g0 < units) cta_units += uint32_t((units - 1 - g0) / GW + 1);
      }
      if (cta_units)
        for (int p = 0; p < ra.k; ++p)
          red_add_release_sys(
              flag_ptr(ra.peer_base[p], ag_cnt_base + (size_t(t) * ra.k + ra.rank) * 128),
              cta_units);
    }
    (void)done;
    // ---- wait for every owner's reduced slice of tile t, then Add+RMSNorm
    const bool ag_ok = wait_all_sources(rq, ag_cnt_base, t, ag_target, kStatusAgWait);
    if (!rs_ok || !ag_ok) rq.timeout_ns = 0;
    if (!ag_ok || !ra.do_norm) continue;
    for (int q = gw; q < ra.R; q += GW) {
      const size_t g = size_t(t) * ra.R + q;
      const float4 *hr = reinterpret_cast<const float4 *>(ra.resid + g * ra.H);
      const __nv_bfloat16 *ar = ag_local + g * ra.H;
      float4 *so = reinterpret_cast<float4 *>(ra.sum_out + g * ra.H);
      float ss = 0.f;
      for (int col = lane * 8; col < ra.H; col += 256) {
        float a[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        acc8_cg(a, ar + col);
        const float4 r0 = __ldcg(hr + col / 4), r1 = __ldcg(hr + col / 4 + 1);
        a[0] += r0.x; a[1] += r0.y; a[2] += r0.z; a[3] += r0.w;
        a[4] += r1.x; a[5] += r1.y; a[6] += r1.z; a[7] += r1.w;
#pragma unroll
        for (int e = 0; e < 8; ++e) ss += a[e] * a[e];
        so[col / 4] = make_float4(a[0], a[1], a[2], a[3]);
        so[col / 4 + 1] = make_float4(a[4], a[5], a[6], a[7]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float r = rsqrtf(ss * inv_h + ra.eps);
      __nv_bfloat16 *xo = ra.x_out + g * ra.H;
      for (int col = lane * 8; col < ra.H; col += 256) {
        float gm[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        acc8_cg(gm, ra.gamma + col);
        const float4 s0 = so[col / 4], s1 = so[col / 4 + 1];
        float a[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
        for (int e = 0; e < 8; ++e) a[e] = a[e] * r * gm[e];
        *reinterpret_cast<uint4 *>(xo + col) = pack8f(a);
      }
    }
  }
}

template <int BN>
__global__ void __launch_bounds__(kRelayThreads, 1)
    relay_down_kernel(const __grid_constant__ CUtensorMap ta,
                      const __grid_constant__ CUtensorMap tb, TileSched ts, RelayArgs ra) {
  extern __shared__ uint8_t smem_raw[];
  const GemmSmemView<BN> s = GemmSmemView<BN>::carve(smem_raw);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
  }
  gemm_setup<BN>(s, 128);
  if (warp == 0) {
    if (lane == 0) gemm_producer<BN>(s, &ta, &tb, ts, ra.K, ra.status);
  } else if (warp == 1) {
    if (lane == 0) gemm_mma<BN>(s, ts, ra.K, ra.status);
  } else if (warp < kRelayWarp0) {
    relay_push_epilogue<BN>(s, ts, ra);
  } else {
    relay_consumer(ra);
  }
  gemm_teardown<BN>(s);
}

// ------------------------------------------------------------------ host side
template <int BN>
static void launch_relay(const CUtensorMap &tma, const __nv_bfloat16 *w_down, long ldb,
                         TileSched ts, const RelayArgs &ra, int grid, cudaStream_t stream) {
  using C = GemmCfg<BN>;
  auto kern = relay_down_kernel<BN>;
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  static bool configured[64] = {false};
  if (!configured[dev & 63]) {
    KRB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  int(C::kSmemBytes)));
    configured[dev & 63] = true;
  }
  const CUtensorMap tmb = make_tmap_2d_bf16(w_down, ra.H, ra.K, ldb, BN, kBK);
  ts.num_n = (ra.H + BN - 1) / BN;
  // cooperative: every CTA must be co-resident, because the relay warps wait
  // for tiles produced by other CTAs of the same grid
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kRelayThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  KRB_CUDA(cudaLaunchKernelEx(&cfg, kern, tma, tmb, ts, ra));
}

void relay_down_layer(const __nv_bfloat16 *act, long lda, const __nv_bfloat16 *w_down, long ldb,
                      int bn, const RelayArgs &ra, cudaStream_t stream) {
  if (ra.S % kBM) throw CudaError("relay: seq must be a multiple of 128");
  if (ra.R % kBM) throw CudaError("relay: rows per tile must be a multiple of 128");
  if (ra.H % 8) throw CudaError("relay: hidden must be a multiple of 8");
  if (ra.k < 1 || ra.k > kMaxRanks || ra.R % ra.k) throw CudaError("relay: bad rank count");
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  TileSched ts;
  ts.num_m = ra.S / kBM;
  ts.band = ra.R / kBM;
  ts.num_n = 0;
  const CUtensorMap tma = make_tmap_2d_bf16(act, ra.S, ra.K, lda, kBM, kBK);
  const int grid = sm_count(dev);
  switch (bn) {
    case 256: launch_relay<256>(tma, w_down, ldb, ts, ra, grid, stream); break;
    case 224: launch_relay<224>(tma, w_down, ldb, ts, ra, grid, stream); break;
    case 128: launch_relay<128>(tma, w_down, ldb, ts, ra, grid, stream); break;
    default: throw CudaError("relay: unsupported bn");
  }
}

// Expected counter increments for the relay (host helper): owner `rank`
// receives one rs increment per (n block, 128-row block touching its slice)
// from every source, and one ag increment per reduced 256-column unit of each
// owner's slice.
void relay_expectations(int S, int H, int T, int k, int rank, int bn, uint32_t *rs_expect,
                        uint32_t *ag_expect, int *nseg) {
  const int R = S / T, Rk = R / k;
  const int num_n = (H + bn - 1) / bn;
  int touching = 0;
  for (int b = 0; b < R / kBM; ++b) {
    const RowRoute first = relay_route(b * kBM, R, Rk);
    const RowRoute last = relay_route(b * kBM + kBM - 1, R, Rk);
    if (first.owner <= rank && rank <= last.owner) ++touching;
  }
  *rs_expect = uint32_t(num_n * touching);
  *nseg = (H + 255) / 256;
  *ag_expect = uint32_t(Rk * *nseg);
}

}  // namespace krb
