// Memory-bound kernels of the prefill: embedding gather, RMSNorm, Add+RMSNorm,
// per-head QK-RMSNorm + rotate-half RoPE, and a tiled transpose used at load time.
//
// Activations are bf16 (the stand-alone op entry points) or fp16 (the engine), read and
// written with 16-byte vector accesses where the layout allows; reductions run in fp32
// with warp shuffles and round once on output.  Weights (gamma, norm weights, rope
// tables) stay bf16.
#include <algorithm>

#include "common.h"
#include "ptx.cuh"

namespace krb {

// ------------------------------------------------------------------ embedding
// out[s, :] = table[ids[s], :]   (aclnnEmbedding in qwen_main.cpp:646-659)
__global__ void embed_kernel(const int64_t *__restrict__ ids, const uint4 *__restrict__ table,
                             uint4 *__restrict__ out, int S, int hv, int V, uint32_t *status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= S) return;
  const int64_t id = ids[warp];
  uint4 *dst = out + static_cast<long>(warp) * hv;
  if (id < 0 || id >= V) {
    if (lane == 0) report_status(status, kStatusBadArgs);
    for (int i = lane; i < hv; i += 32) dst[i] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4 *src = table + id * hv;
  for (int i = lane; i < hv; i += 32) dst[i] = __ldg(src + i);
}

// fp32 residual variant: out[s, :] = float(table[ids[s], :])
__global__ void embed_f32_kernel(const int64_t *__restrict__ ids, const uint4 *__restrict__ table,
                                 float4 *__restrict__ out, int S, int hv, int V, uint32_t *status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= S) return;
  const int64_t id = ids[warp];
  float4 *dst = out + static_cast<long>(warp) * hv * 2;
  const bool ok = id >= 0 && id < V;
  if (!ok && lane == 0) report_status(status, kStatusBadArgs);
  for (int i = lane; i < hv; i += 32) {
    float f[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (ok) {
      const uint4 w = __ldg(table + id * hv + i);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 t = unpack_bf16x2(ws[e]);
        f[2 * e] = t.x;
        f[2 * e + 1] = t.y;
      }
    }
    dst[2 * i] = make_float4(f[0], f[1], f[2], f[3]);
    dst[2 * i + 1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

void embed_f32(const int64_t *ids, const __nv_bfloat16 *table, float *out, int S, int H, int V,
               uint32_t *status, cudaStream_t stream) {
  if (H % 8) throw CudaError("embed: H % 8 != 0");
  const int threads = 256;
  const int blocks = (S * 32 + threads - 1) / threads;
  embed_f32_kernel<<<blocks, threads, 0, stream>>>(ids, reinterpret_cast<const uint4 *>(table),
                                                   reinterpret_cast<float4 *>(out), S, H / 8, V,
                                                   status);
  KRB_CUDA(cudaGetLastError());
}

void embed_bf16(const int64_t *ids, const __nv_bfloat16 *table, __nv_bfloat16 *out, int S, int H,
                int V, uint32_t *status, cudaStream_t stream) {
  if (H % 8) throw CudaError("embed: H % 8 != 0");
  const int threads = 256;
  const int blocks = (S * 32 + threads - 1) / threads;
  embed_kernel<<<blocks, threads, 0, stream>>>(ids, reinterpret_cast<const uint4 *>(table),
                                               reinterpret_cast<uint4 *>(out), S, H / 8, V,
                                               status);
  KRB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------ RMSNorm family
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void unpack8(const uint4 &w, float *f) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 t = unpack_bf16x2(ws[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float *f) {
  uint4 w;
  w.x = pack_bf16x2(f[0], f[1]);
  w.y = pack_bf16x2(f[2], f[3]);
  w.z = pack_bf16x2(f[4], f[5]);
  w.w = pack_bf16x2(f[6], f[7]);
  return w;
}

// 8 activations in either 2-byte format
template <bool F16>
__device__ __forceinline__ void unpack8a(const uint4 &w, float *f) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    float2 t = unpack2<F16>(ws[e]);
    f[2 * e] = t.x;
    f[2 * e + 1] = t.y;
  }
}

template <bool F16>
__device__ __forceinline__ uint4 pack8a(const float *f) {
  uint4 w;
  w.x = pack2<F16>(f[0], f[1]);
  w.y = pack2<F16>(f[2], f[3]);
  w.z = pack2<F16>(f[4], f[5]);
  w.w = pack2<F16>(f[6], f[7]);
  return w;
}

// 8 elements of a residual row as fp32 (from fp32 or bf16 storage)
__device__ __forceinline__ void load8(const float *p, long v, float *f) {
  const float4 *q = reinterpret_cast<const float4 *>(p) + v * 2;
  const float4 x = __ldg(q), y = __ldg(q + 1);
  f[0] = x.x; f[1] = x.y; f[2] = x.z; f[3] = x.w;
  f[4] = y.x; f[5] = y.y; f[6] = y.z; f[7] = y.w;
}
__device__ __forceinline__ void load8(const __nv_bfloat16 *p, long v, float *f) {
  unpack8(__ldg(reinterpret_cast<const uint4 *>(p) + v), f);
}
__device__ __forceinline__ void load8(const __half *p, long v, float *f) {
  unpack8a<true>(__ldg(reinterpret_cast<const uint4 *>(p) + v), f);
}
__device__ __forceinline__ void store8(float *p, long v, const float *f) {
  float4 *q = reinterpret_cast<float4 *>(p) + v * 2;
  q[0] = make_float4(f[0], f[1], f[2], f[3]);
  q[1] = make_float4(f[4], f[5], f[6], f[7]);
}

// One CTA per row, blockDim = 32 * ceil(hv / 128): every lane owns at most kNormVec
// 8-element vectors, so all of a row's loads are in flight at once (HBM-bound).
//   s = a (+ b)            a: residual (fp32 or bf16), b: bf16/fp32 delta or null
//   sum_f <- s (fp32, unrounded)   or   sum_b <- bf16(s) and the norm uses bf16(s)
//   y = s * rsqrt(mean(s^2) + eps) * gamma  (2-byte TY: bf16 or fp16)
// With a bf16 sum the norm is taken over the rounded value, as the stored
// bf16 residual is what later layers see (aclnnAddRmsNorm semantics).
constexpr int kNormVec = 4;

template <typename TA, typename TB, typename TY>
__global__ void add_rmsnorm_kernel(const TA *__restrict__ a, const TB *__restrict__ b,
                                   const uint4 *__restrict__ gamma, uint4 *__restrict__ y,
                                   float *__restrict__ rstd, float *__restrict__ sum_f,
                                   uint4 *__restrict__ sum_b, int hv, float inv_h, float eps) {
  __shared__ float part[32];
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const long base = static_cast<long>(row) * hv;
  float x[kNormVec][8];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < kNormVec; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < hv) {
      load8(a, base + v, x[i]);
      if (b) {
        float t[8];
        load8(b, base + v, t);
#pragma unroll
        for (int e = 0; e < 8; ++e) x[i][e] += t[e];
      }
    }
  }
#pragma unroll
  for (int i = 0; i < kNormVec; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < hv) {
      if (sum_b) {
#pragma unroll
        for (int e = 0; e < 8; ++e) x[i][e] = bf16_round(x[i][e]);
        sum_b[base + v] = pack8(x[i]);
      }
      if (sum_f) store8(sum_f, base + v, x[i]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += x[i][e] * x[i][e];
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) part[warp] = ss;
  __syncthreads();
  float tot = 0.f;
  const int nw = blockDim.x >> 5;
  for (int w = 0; w < nw; ++w) tot += part[w];
  const float r = rsqrtf(tot * inv_h + eps);
  if (rstd && threadIdx.x == 0) rstd[row] = r;
#pragma unroll
  for (int i = 0; i < kNormVec; ++i) {
    const int v = threadIdx.x + i * blockDim.x;
    if (v < hv) {
      float g[8];
      unpack8(__ldg(gamma + v), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[i][e] = x[i][e] * r * g[e];
      y[base + v] = pack8a<ActFmt<TY>::f16>(x[i]);
    }
  }
}

template <typename TA, typename TB, typename TY = __nv_bfloat16>
static void launch_add_rmsnorm(const TA *a, const TB *b, const __nv_bfloat16 *gamma,
                               TY *y, float *rstd, float *sum_f, __nv_bfloat16 *sum_b,
                               int rows, int H, float eps, cudaStream_t stream) {
  if (H % 8) throw CudaError("rmsnorm: H % 8 != 0");
  if (rows <= 0) throw CudaError("rmsnorm: no rows");
  const int hv = H / 8;
  const int warps = (hv + 32 * kNormVec - 1) / (32 * kNormVec);
  if (warps > 32) throw CudaError("rmsnorm: H too large");
  const auto *g4 = reinterpret_cast<const uint4 *>(gamma);
  auto *y4 = reinterpret_cast<uint4 *>(y);
  auto *s4 = reinterpret_cast<uint4 *>(sum_b);
  const float inv_h = 1.0f / float(H);
  add_rmsnorm_kernel<TA, TB, TY><<<rows, warps * 32, 0, stream>>>(a, b, g4, y4, rstd, sum_f, s4,
                                                                  hv, inv_h, eps);
  KRB_CUDA(cudaGetLastError());
}

void rmsnorm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *gamma, __nv_bfloat16 *y,
                  float *rstd, int rows, int H, float eps, cudaStream_t stream) {
  launch_add_rmsnorm<__nv_bfloat16, __nv_bfloat16>(x, nullptr, gamma, y, rstd, nullptr, nullptr,
                                                   rows, H, eps, stream);
}

void add_rmsnorm_bf16(const __nv_bfloat16 *a, const __nv_bfloat16 *b, const __nv_bfloat16 *gamma,
                      __nv_bfloat16 *y, float *rstd, __nv_bfloat16 *sum, int rows, int H,
                      float eps, cudaStream_t stream) {
  launch_add_rmsnorm<__nv_bfloat16, __nv_bfloat16>(a, b, gamma, y, rstd, nullptr, sum, rows, H,
                                                   eps, stream);
}

template <typename T>
void rmsnorm_act(const T *x, const __nv_bfloat16 *gamma, T *y, int rows, int H, float eps,
                 cudaStream_t stream) {
  launch_add_rmsnorm<T, T, T>(x, static_cast<const T *>(nullptr), gamma, y, nullptr, nullptr,
                              nullptr, rows, H, eps, stream);
}
template void rmsnorm_act<__half>(const __half *, const __nv_bfloat16 *, __half *, int, int, float,
                                  cudaStream_t);

template <typename TD, typename TY>
void add_rmsnorm_res_f32(const float *res, const TD *delta, const __nv_bfloat16 *gamma, TY *y,
                         float *sum, int rows, int H, float eps, cudaStream_t stream) {
  launch_add_rmsnorm<float, TD, TY>(res, delta, gamma, y, nullptr, sum, nullptr, rows, H, eps,
                                    stream);
}
template void add_rmsnorm_res_f32<__nv_bfloat16, __nv_bfloat16>(const float *,
                                                                const __nv_bfloat16 *,
                                                                const __nv_bfloat16 *,
                                                                __nv_bfloat16 *, float *, int, int,
                                                                float, cudaStream_t);
template void add_rmsnorm_res_f32<float, __nv_bfloat16>(const float *, const float *,
                                                        const __nv_bfloat16 *, __nv_bfloat16 *,
                                                        float *, int, int, float, cudaStream_t);
template void add_rmsnorm_res_f32<__half, __half>(const float *, const __half *,
                                                  const __nv_bfloat16 *, __half *, float *, int,
                                                  int, float, cudaStream_t);
template void add_rmsnorm_res_f32<float, __half>(const float *, const float *,
                                                 const __nv_bfloat16 *, __half *, float *, int,
                                                 int, float, cudaStream_t);

// ------------------------------------------------------------------ QK-norm + RoPE
// One warp per (position, head) for the HQ query heads and HKV key heads of the
// fused qkv row.  Optional per-head RMSNorm over D (Qwen3 q_norm/k_norm, applied
// before RoPE as in HF Qwen3Attention), then rotate-half RoPE with the bf16
// cos/sin tables of the model directory (export_model.py:70-77 layout [max_pos, D]).
template <int D, bool F16>
__global__ void qk_norm_rope_kernel(uint16_t *__restrict__ qkv, int S, int HQ, int HKV,
                                    const __nv_bfloat16 *__restrict__ cos_tab,
                                    const __nv_bfloat16 *__restrict__ sin_tab,
                                    const __nv_bfloat16 *__restrict__ q_norm,
                                    const __nv_bfloat16 *__restrict__ k_norm, float eps) {
  // one thread per 8 rotation pairs: elements j..j+7 of the first half and
  // HALF+j..HALF+j+7 of the second, 16-byte loads and stores; the head's
  // kLanes = HALF/8 threads are consecutive lanes of one warp
  constexpr int HALF = D / 2;
  constexpr int kLanes = HALF / 8;
  const long gt = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nh = HQ + HKV;
  const long head = gt / kLanes;
  const int j = static_cast<int>(gt % kLanes) * 8;
  if (head >= static_cast<long>(S) * nh) return;  // whole heads only: warp-uniform per head
  const int s = static_cast<int>(head / nh);
  const int h = static_cast<int>(head - static_cast<long>(s) * nh);
  uint16_t *p = qkv + (static_cast<long>(s) * (HQ + 2 * HKV) + h) * D;
  const __nv_bfloat16 *nw = (h < HQ) ? q_norm : k_norm;
  float lo[8], hi[8];
  unpack8a<F16>(*reinterpret_cast<const uint4 *>(p + j), lo);
  unpack8a<F16>(*reinterpret_cast<const uint4 *>(p + HALF + j), hi);
  const long trow = static_cast<long>(s) * D;
  float c0[8], s0[8], c1[8], s1[8];
  unpack8(__ldg(reinterpret_cast<const uint4 *>(cos_tab + trow + j)), c0);
  unpack8(__ldg(reinterpret_cast<const uint4 *>(sin_tab + trow + j)), s0);
  unpack8(__ldg(reinterpret_cast<const uint4 *>(cos_tab + trow + HALF + j)), c1);
  unpack8(__ldg(reinterpret_cast<const uint4 *>(sin_tab + trow + HALF + j)), s1);
  if (nw) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += lo[e] * lo[e] + hi[e] * hi[e];
    // the head's kLanes lanes (all active or all returned together)
    const unsigned lane = threadIdx.x & 31;
    const unsigned mask = ((1u << kLanes) - 1u) << (lane & ~unsigned(kLanes - 1));
#pragma unroll
    for (int o = kLanes / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(mask, ss, o);
    const float r = rsqrtf(ss / float(D) + eps);
    float wl[8], wh[8];
    unpack8(__ldg(reinterpret_cast<const uint4 *>(nw + j)), wl);
    unpack8(__ldg(reinterpret_cast<const uint4 *>(nw + HALF + j)), wh);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      // bf16 data: HF RMSNorm returns bf16 before RoPE, keep that rounding point;
      // fp16 data rounds once, at the store
      lo[e] = lo[e] * r * wl[e];
      hi[e] = hi[e] * r * wh[e];
      if constexpr (!F16) {
        lo[e] = bf16_round(lo[e]);
        hi[e] = bf16_round(hi[e]);
      }
    }
  }
  float olo[8], ohi[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    olo[e] = lo[e] * c0[e] - hi[e] * s0[e];
    ohi[e] = hi[e] * c1[e] + lo[e] * s1[e];
  }
  *reinterpret_cast<uint4 *>(p + j) = pack8a<F16>(olo);
  *reinterpret_cast<uint4 *>(p + HALF + j) = pack8a<F16>(ohi);
}

template <typename T>
void qk_norm_rope(T *qkv_t, int S, int HQ, int HKV, int D, const __nv_bfloat16 *cos_tab,
                  const __nv_bfloat16 *sin_tab, const __nv_bfloat16 *q_norm,
                  const __nv_bfloat16 *k_norm, float eps, cudaStream_t stream) {
  constexpr bool F16 = ActFmt<T>::f16;
  uint16_t *qkv = reinterpret_cast<uint16_t *>(qkv_t);
  const long threads_total = static_cast<long>(S) * (HQ + HKV) * (D / 16);
  const int threads = 256;
  const long blocks = (threads_total + threads - 1) / threads;
  switch (D) {
    case 64:
      qk_norm_rope_kernel<64, F16><<<blocks, threads, 0, stream>>>(qkv, S, HQ, HKV, cos_tab,
                                                                   sin_tab, q_norm, k_norm, eps);
      break;
    case 128:
      qk_norm_rope_kernel<128, F16><<<blocks, threads, 0, stream>>>(qkv, S, HQ, HKV, cos_tab,
                                                                    sin_tab, q_norm, k_norm, eps);
      break;
    default:
      throw CudaError("qk_norm_rope: head_dim must be 64 or 128");
  }
  KRB_CUDA(cudaGetLastError());
}

template void qk_norm_rope<__nv_bfloat16>(__nv_bfloat16 *, int, int, int, int,
                                          const __nv_bfloat16 *, const __nv_bfloat16 *,
                                          const __nv_bfloat16 *, const __nv_bfloat16 *, float,
                                          cudaStream_t);
template void qk_norm_rope<__half>(__half *, int, int, int, int, const __nv_bfloat16 *,
                                   const __nv_bfloat16 *, const __nv_bfloat16 *,
                                   const __nv_bfloat16 *, float, cudaStream_t);

// ------------------------------------------------------------------ transpose
__device__ __forceinline__ void store_as(__nv_bfloat16 *p, __nv_bfloat16 v) { *p = v; }
__device__ __forceinline__ void store_as(__half *p, __nv_bfloat16 v) {
  *p = __float2half_rn(__bfloat162float(v));
}
__device__ __forceinline__ void store_as(__half *p, __half v) { *p = v; }

// 32 x 32 tiles through padded shared memory; TS -> TD: bf16 -> bf16 (copy), bf16 -> fp16
// (converted), fp16 -> fp16 (copy)
template <typename TS, typename TD>
__global__ void transpose_kernel(const TS *__restrict__ src, long ld_src,
                                 TD *__restrict__ dst, long ld_dst, int rows, int cols) {
  __shared__ TS tile[32][33];
  const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int r = r0 + i, c = c0 + threadIdx.x;
    if (r < rows && c < cols) tile[i][threadIdx.x] = src[r * ld_src + c];
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += blockDim.y) {
    const int c = c0 + i, r = r0 + threadIdx.x;
    if (r < rows && c < cols) store_as(dst + c * ld_dst + r, tile[threadIdx.x][i]);
  }
}

void transpose_bf16(const __nv_bfloat16 *src, long ld_src, __nv_bfloat16 *dst, long ld_dst,
                    int rows, int cols, cudaStream_t stream) {
  dim3 block(32, 8);
  dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  transpose_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, block, 0, stream>>>(src, ld_src, dst,
                                                                             ld_dst, rows, cols);
  KRB_CUDA(cudaGetLastError());
}

void transpose_bf16_to_f16(const __nv_bfloat16 *src, long ld_src, __half *dst, long ld_dst,
                           int rows, int cols, cudaStream_t stream) {
  dim3 block(32, 8);
  dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  transpose_kernel<__nv_bfloat16, __half><<<grid, block, 0, stream>>>(src, ld_src, dst, ld_dst,
                                                                      rows, cols);
  KRB_CUDA(cudaGetLastError());
}

void transpose_f16(const __half *src, long ld_src, __half *dst, long ld_dst, int rows, int cols,
                   cudaStream_t stream) {
  dim3 block(32, 8);
  dim3 grid((cols + 31) / 32, (rows + 31) / 32);
  transpose_kernel<__half, __half><<<grid, block, 0, stream>>>(src, ld_src, dst, ld_dst, rows,
                                                               cols);
  KRB_CUDA(cudaGetLastError());
}

// ------------------------------------------------------------------ format conversions
__global__ void bf16_to_f16_kernel(uint4 *__restrict__ data, size_t nvec) {
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < nvec;
       i += size_t(gridDim.x) * blockDim.x) {
    float f[8];
    unpack8(data[i], f);
    data[i] = pack8a<true>(f);
  }
}

__global__ void bf16_to_f16_tail_kernel(uint16_t *__restrict__ data, size_t from, size_t n) {
  const size_t i = from + size_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) {
    const float f = __bfloat162float(*reinterpret_cast<const __nv_bfloat16 *>(data + i));
    const __half h = __float2half_rn(f);
    data[i] = *reinterpret_cast<const uint16_t *>(&h);
  }
}

void bf16_to_f16_inplace(void *data, size_t n, cudaStream_t stream) {
  if (reinterpret_cast<uintptr_t>(data) % 16) throw CudaError("bf16_to_f16: unaligned buffer");
  const size_t nvec = n / 8;
  if (nvec) {
    const size_t blocks = std::min<size_t>((nvec + 255) / 256, 148 * 16);
    bf16_to_f16_kernel<<<unsigned(blocks), 256, 0, stream>>>(static_cast<uint4 *>(data), nvec);
    KRB_CUDA(cudaGetLastError());
  }
  if (n % 8) {
    bf16_to_f16_tail_kernel<<<1, 8, 0, stream>>>(static_cast<uint16_t *>(data), nvec * 8, n);
    KRB_CUDA(cudaGetLastError());
  }
}

__global__ void f16_to_f32_kernel(const __half *__restrict__ src, float *__restrict__ dst, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[i] = __half2float(src[i]);
}

void f16_to_f32(const __half *src, float *dst, int n, cudaStream_t stream) {
  const int blocks = std::min((n + 255) / 256, 1024);
  f16_to_f32_kernel<<<blocks > 0 ? blocks : 1, 256, 0, stream>>>(src, dst, n);
  KRB_CUDA(cudaGetLastError());
}

}  // namespace krb
