// Causal GQA prefill attention (flash-attention style, online softmax).
//
// Replaces aclnnFlashAttentionScore(BSND, sparse_mode 3, scale 1/sqrt(D))
// (qwen_main.cpp:591-614).  Q, K, V are read in place from the fused
// [S, (HQ + 2*HKV) * D] projection buffer after QK-norm/RoPE; the output is
// [S, HQ*D] bf16.  Query head h reads KV head h / (HQ/HKV).
//
// One CTA = 4 warps = 64 query rows of one head; 64-key K/V blocks are
// double-buffered in shared memory with cp.async (XOR-swizzled 16-byte chunks
// so ldmatrix is conflict-free).  QK^T and PV use mma.sync m16n8k16 bf16 with
// fp32 accumulation; P is rounded to bf16 before PV (as every bf16 flash kernel
// does); the softmax statistics stay fp32.  Causal blocks above the diagonal are
// skipped entirely; query blocks are scheduled heaviest first.
#include "common.h"
#include "ptx.cuh"

namespace krb {

namespace {

__device__ __forceinline__ void cp_async16(void *smem, const void *gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                          uint32_t &r2, uint32_t &r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                               uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7},"
      " {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

}  // namespace

template <int D>
struct AttnCfg {
  static constexpr int BM = 64;
  static constexpr int BN = 64;
  static constexpr int CH = D / 8;  // 16-byte chunks per row
  static constexpr int TILE = 64 * D;  // elements per 64-row tile
  static constexpr int SMEM = (TILE + 4 * TILE) * 2;  // Q + 2x(K,V)
};

// element offset of (row, chunk) inside a swizzled tile
template <int D>
__device__ __forceinline__ int swz(int row, int chunk) {
  return row * D + ((chunk ^ (row & 7)) << 3);
}

template <int D>
__global__ void __launch_bounds__(128)
    attn_prefill_kernel(const __nv_bfloat16 *__restrict__ qp, const __nv_bfloat16 *__restrict__ kp,
                        const __nv_bfloat16 *__restrict__ vp, long ld, __nv_bfloat16 *__restrict__ out,
                        long ldo, int S, int group, float scale_log2) {
  using C = AttnCfg<D>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __nv_bfloat16 *sQ = reinterpret_cast<__nv_bfloat16 *>(smem_raw);
  __nv_bfloat16 *sK = sQ + C::TILE;       // [2][TILE]
  __nv_bfloat16 *sV = sK + 2 * C::TILE;   // [2][TILE]

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int qb = gridDim.x - 1 - blockIdx.x;  // heaviest query blocks first
  const int h = blockIdx.y;
  const int kvh = h / group;
  const __nv_bfloat16 *Qg = qp + static_cast<long>(h) * D;
  const __nv_bfloat16 *Kg = kp + static_cast<long>(kvh) * D;
  const __nv_bfloat16 *Vg = vp + static_cast<long>(kvh) * D;
  const int q0 = qb * C::BM;

  auto load_tile = [&](__nv_bfloat16 *dst, const __nv_bfloat16 *src, int row0) {
    for (int i = tid; i < 64 * C::CH; i += 128) {
      const int r = i / C::CH, c = i - (i / C::CH) * C::CH;
      const bool ok = (row0 + r) < S;
      const __nv_bfloat16 *g = ok ? src + static_cast<long>(row0 + r) * ld + c * 8 : src;
      cp_async16(dst + swz<D>(r, c), g, ok ? 16 : 0);
    }
  };

  const int n_kb = min(qb + 1, (S + C::BN - 1) / C::BN);
  load_tile(sQ, Qg, q0);
  load_tile(sK, Kg, 0);
  load_tile(sV, Vg, 0);
  cp_async_commit();

  // per-warp state: 16 query rows; thread holds rows g and g+8
  const int g = lane >> 2, t4 = lane & 3;
  uint32_t qf[D / 16][4];
  float o[D / 8][4];
#pragma unroll
  for (int j = 0; j < D / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.f, 0.f};
  const int row_a = q0 + warp * 16 + g;  // global query row of c0/c1
  const int row_b = row_a + 8;           // of c2/c3

  for (int kb = 0; kb < n_kb; ++kb) {
    const int buf = kb & 1;
    if (kb + 1 < n_kb) {
      load_tile(sK + (buf ^ 1) * C::TILE, Kg, (kb + 1) * C::BN);
      load_tile(sV + (buf ^ 1) * C::TILE, Vg, (kb + 1) * C::BN);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kb == 0) {
      // Q fragments: rows warp*16 + {0..15}, k-steps of 16 dims
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        const int r = warp * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
        const int c = ks * 2 + (lane >> 4);
        ldsm_x4(smem_u32(sQ + swz<D>(r, c)), qf[ks][0], qf[ks][1], qf[ks][2], qf[ks][3]);
      }
    }
    const __nv_bfloat16 *k_s = sK + buf * C::TILE;
    const __nv_bfloat16 *v_s = sV + buf * C::TILE;

    // S = Q K^T : 16 x 64 per warp = 8 n-tiles of 8 keys
    float sc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
      for (int jp = 0; jp < 4; ++jp) {  // pairs of n-tiles
        const int mi = lane >> 3;
        const int r = jp * 16 + (lane & 7) + (mi >> 1) * 8;
        const int c = ks * 2 + (mi & 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(k_s + swz<D>(r, c)), b0, b1, b2, b3);
        mma_bf16_16816(sc[2 * jp], qf[ks], b0, b1);
        mma_bf16_16816(sc[2 * jp + 1], qf[ks], b2, b3);
      }
    }
    // mask (diagonal block and keys beyond S)
    const int k0 = kb * C::BN;
    const bool need_mask = (kb == qb) || (k0 + C::BN > S);
    if (need_mask) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int key = k0 + j * 8 + t4 * 2;
        if (key > row_a || key >= S) sc[j][0] = -INFINITY;
        if (key + 1 > row_a || key + 1 >= S) sc[j][1] = -INFINITY;
        if (key > row_b || key >= S) sc[j][2] = -INFINITY;
        if (key + 1 > row_b || key + 1 >= S) sc[j][3] = -INFINITY;
      }
    }
    // online softmax (log2 domain)
    float mx[2] = {m_run[0], m_run[1]};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx[0] = fmaxf(mx[0], fmaxf(sc[j][0], sc[j][1]) * scale_log2);
      mx[1] = fmaxf(mx[1], fmaxf(sc[j][2], sc[j][3]) * scale_log2);
    }
#pragma unroll
    for (int o2 = 1; o2 <= 2; o2 <<= 1) {
      mx[0] = fmaxf(mx[0], __shfl_xor_sync(0xffffffffu, mx[0], o2));
      mx[1] = fmaxf(mx[1], __shfl_xor_sync(0xffffffffu, mx[1], o2));
    }
    const float corr0 = exp2f(m_run[0] - mx[0]);
    const float corr1 = exp2f(m_run[1] - mx[1]);
    m_run[0] = mx[0];
    m_run[1] = mx[1];
    float rs[2] = {0.f, 0.f};
    uint32_t pf[4][4];  // P as A fragments for 4 k-steps of 16 keys
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(sc[j][0] * scale_log2 - mx[0]);
      const float p1 = exp2f(sc[j][1] * scale_log2 - mx[0]);
      const float p2 = exp2f(sc[j][2] * scale_log2 - mx[1]);
      const float p3 = exp2f(sc[j][3] * scale_log2 - mx[1]);
      // sum the bf16-rounded probabilities so numerator and denominator agree
      const uint32_t u01 = pack_bf16x2(p0, p1);
      const uint32_t u23 = pack_bf16x2(p2, p3);
      const float2 f01 = unpack_bf16x2(u01), f23 = unpack_bf16x2(u23);
      rs[0] += f01.x + f01.y;
      rs[1] += f23.x + f23.y;
      const int ks = j >> 1;
      if ((j & 1) == 0) {
        pf[ks][0] = u01;
        pf[ks][1] = u23;
      } else {
        pf[ks][2] = u01;
        pf[ks][3] = u23;
      }
    }
    l_run[0] = l_run[0] * corr0 + rs[0];
    l_run[1] = l_run[1] * corr1 + rs[1];
#pragma unroll
    for (int j = 0; j < D / 8; ++j) {
      o[j][0] *= corr0;
      o[j][1] *= corr0;
      o[j][2] *= corr1;
      o[j][3] *= corr1;
    }
    // O += P V : V tile [64 keys][D]; B fragments via ldmatrix.trans
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int jp = 0; jp < D / 16; ++jp) {  // pairs of 8-wide d tiles
        const int mi = lane >> 3;
        const int r = ks * 16 + (lane & 7) + (mi & 1) * 8;
        const int c = jp * 2 + (mi >> 1);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(v_s + swz<D>(r, c)), b0, b1, b2, b3);
        mma_bf16_16816(o[2 * jp], pf[ks], b0, b1);
        mma_bf16_16816(o[2 * jp + 1], pf[ks], b2, b3);
      }
    }
    __syncthreads();  // buffer `buf` is reloaded two iterations later
  }

  // finalize: quad-reduce the row sums, normalise, store bf16
#pragma unroll
  for (int o2 = 1; o2 <= 2; o2 <<= 1) {
    l_run[0] += __shfl_xor_sync(0xffffffffu, l_run[0], o2);
    l_run[1] += __shfl_xor_sync(0xffffffffu, l_run[1], o2);
  }
  const float inv0 = 1.f / l_run[0];
  const float inv1 = 1.f / l_run[1];
  __nv_bfloat16 *Oa = out + static_cast<long>(row_a) * ldo + static_cast<long>(h) * D;
  __nv_bfloat16 *Ob = Oa + 8 * ldo;
#pragma unroll
  for (int j = 0; j < D / 8; ++j) {
    const int col = j * 8 + t4 * 2;
    if (row_a < S)
      *reinterpret_cast<uint32_t *>(Oa + col) = pack_bf16x2(o[j][0] * inv0, o[j][1] * inv0);
    if (row_b < S)
      *reinterpret_cast<uint32_t *>(Ob + col) = pack_bf16x2(o[j][2] * inv1, o[j][3] * inv1);
  }
}

void attention_heads_bf16(const __nv_bfloat16 *q, const __nv_bfloat16 *k, const __nv_bfloat16 *v,
                          long ld, __nv_bfloat16 *out, long ldo, int S, int nq, int group, int D,
                          float scale, cudaStream_t stream) {
  if (group <= 0 || nq <= 0) throw CudaError("attention: bad head grouping");
  if ((ld * 2) % 16 || (ldo * 2) % 4) throw CudaError("attention: bad leading dimension");
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid((S + 63) / 64, nq);
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  static bool configured[2][64] = {{false}};
  switch (D) {
    case 64: {
      auto kern = attn_prefill_kernel<64>;
      if (!configured[0][dev & 63]) {
        KRB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      AttnCfg<64>::SMEM));
        configured[0][dev & 63] = true;
      }
      kern<<<grid, 128, AttnCfg<64>::SMEM, stream>>>(q, k, v, ld, out, ldo, S, group, scale_log2);
      break;
    }
    case 128: {
      auto kern = attn_prefill_kernel<128>;
      if (!configured[1][dev & 63]) {
        KRB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      AttnCfg<128>::SMEM));
        configured[1][dev & 63] = true;
      }
      kern<<<grid, 128, AttnCfg<128>::SMEM, stream>>>(q, k, v, ld, out, ldo, S, group, scale_log2);
      break;
    }
    default:
      throw CudaError("attention: head_dim must be 64 or 128");
  }
  KRB_CUDA(cudaGetLastError());
}

void attention_prefill_bf16(const __nv_bfloat16 *qkv, __nv_bfloat16 *out, int S, int HQ, int HKV,
                            int D, float scale, cudaStream_t stream) {
  if (HKV <= 0 || HQ % HKV) throw CudaError("attention: HQ % HKV != 0");
  const long ld = static_cast<long>(HQ + 2 * HKV) * D;
  attention_heads_bf16(qkv, qkv + static_cast<long>(HQ) * D, qkv + static_cast<long>(HQ + HKV) * D,
                       ld, out, static_cast<long>(HQ) * D, S, HQ, HQ / HKV, D, scale, stream);
}

}  // namespace krb
