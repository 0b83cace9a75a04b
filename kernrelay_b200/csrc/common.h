// Host-side helpers shared by every translation unit of libkernrelay.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace krb {

struct CudaError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

inline void check_cuda(cudaError_t e, const char *what) {
  if (e != cudaSuccess) {
    throw CudaError(std::string(what) + ": " + cudaGetErrorName(e) + " (" +
                    cudaGetErrorString(e) + ")");
  }
}

#define KRB_CUDA(call) ::krb::check_cuda((call), #call)

int sm_count(int device);

// 2D bf16 tensor map for a row-major [rows, cols] matrix with row pitch `ld`
// elements, box [box_rows, box_cols], 128-byte swizzle when box_cols*2 == 128.
CUtensorMap make_tmap_2d_bf16(const void *base, uint64_t rows, uint64_t cols, uint64_t ld,
                              uint32_t box_rows, uint32_t box_cols);

// ---- op launchers (all asynchronous on `stream`; shapes validated, throw on misuse)
// C[M,N] = A[M,K] . B[N,K]^T (+bias[N]); lda/ldb/ldc in elements.
void gemm_bf16(const __nv_bfloat16 *A, long lda, const __nv_bfloat16 *B, long ldb,
               __nv_bfloat16 *C, long ldc, const __nv_bfloat16 *bias, int M, int N, int K,
               int bn, int grid_limit, uint32_t *status, cudaStream_t stream);

// fp16 variant of gemm_bf16 (no bias): C[M,N] = f16(A[M,K] . B[N,K]^T), fp32 accumulate.
void gemm_f16(const __half *A, long lda, const __half *B, long ldb, __half *C, long ldc, int M,
              int N, int K, int bn, uint32_t *status, cudaStream_t stream);
// Either 2-byte format T (__nv_bfloat16 or __half) for A, B and C; bias stays bf16.
template <typename T>
void gemm_store(const T *A, long lda, const T *B, long ldb, T *C, long ldc,
                const __nv_bfloat16 *bias, int M, int N, int K, int bn, int grid_limit,
                uint32_t *status, cudaStream_t stream);

// fp32 output: out[M,N] = A . B^T unrounded (row pitch ld), for residual updates
// (T = __nv_bfloat16 or __half operands).
template <typename T>
void gemm_f32out(const T *A, long lda, const T *B, long ldb, float *out, long ld, int M, int N,
                 int K, int bn, uint32_t *status, cudaStream_t stream);

// Fused QKV projection: C[M, (HQ+2HKV)D] = A . B^T + bias, then per q / k head an
// optional RMSNorm over D (qn / kn, Qwen3) and rotate-half RoPE with the bf16 cos /
// sin tables [max_pos, D] at position = row; v heads get the bias only.
void gemm_qkv_rope_bf16(const __nv_bfloat16 *A, long lda, const __nv_bfloat16 *B, long ldb,
                        __nv_bfloat16 *C, long ldc, const __nv_bfloat16 *bias, int M, int K,
                        int HQ, int HKV, int D, const __nv_bfloat16 *cos_tab,
                        const __nv_bfloat16 *sin_tab, const __nv_bfloat16 *qn,
                        const __nv_bfloat16 *kn, float eps, uint32_t *status,
                        cudaStream_t stream, __half *vt = nullptr,
                        long ldvt = 0);
// Same for either operand format T (q / k / v written in T; V^T always fp16).
template <typename T>
void gemm_qkv_rope(const T *A, long lda, const T *B, long ldb, T *C, long ldc,
                   const __nv_bfloat16 *bias, int M, int K, int HQ, int HKV, int D,
                   const __nv_bfloat16 *cos_tab, const __nv_bfloat16 *sin_tab,
                   const __nv_bfloat16 *qn, const __nv_bfloat16 *kn, float eps, uint32_t *status,
                   cudaStream_t stream, __half *vt, long ldvt);

// act[M, n_out] = silu(gate) * up, with B rows interleaved in blocks of bn:
// rows [b*bn, b*bn+bn/2) gate, [b*bn+bn/2, (b+1)*bn) up for outputs [b*bn/2, (b+1)*bn/2).
void gemm_silu_bf16(const __nv_bfloat16 *A, long lda, const __nv_bfloat16 *Bgu, long ldb,
                    __nv_bfloat16 *act, long ldact, int M, int n_out, int K, int bn,
                    int grid_limit, uint32_t *status, cudaStream_t stream);
template <typename T>
void gemm_silu(const T *A, long lda, const T *Bgu, long ldb, T *act, long ldact, int M,
               int n_out, int K, int bn, int grid_limit, uint32_t *status, cudaStream_t stream);

// Choose the UMMA N tile that minimises wave-quantisation loss for a plain GEMM.
int pick_bn_store(int M, int N, int sms);
int pick_bn_silu(int M, int n_out, int sms);

// ---- elementwise / normalisation kernels (norm.cu)
void embed_bf16(const int64_t *ids, const __nv_bfloat16 *table, __nv_bfloat16 *out, int S,
                int H, int V, uint32_t *status, cudaStream_t stream);
void rmsnorm_bf16(const __nv_bfloat16 *x, const __nv_bfloat16 *gamma, __nv_bfloat16 *y,
                  float *rstd, int rows, int H, float eps, cudaStream_t stream);
// sum = a + b (bf16-rounded, written when sum != null); y = rmsnorm(sum) * gamma
void add_rmsnorm_bf16(const __nv_bfloat16 *a, const __nv_bfloat16 *b,
                      const __nv_bfloat16 *gamma, __nv_bfloat16 *y, float *rstd,
                      __nv_bfloat16 *sum, int rows, int H, float eps, cudaStream_t stream);
// y = rmsnorm(x) * gamma for 2-byte activations T (input and output in T)
template <typename T>
void rmsnorm_act(const T *x, const __nv_bfloat16 *gamma, T *y, int rows, int H, float eps,
                 cudaStream_t stream);
// fp32 residual stream: sum = res + delta (fp32, unrounded); y = rmsnorm(sum) * gamma
// (delta 2-byte TD or fp32, or null; y in the 2-byte format TY)
template <typename TD, typename TY>
void add_rmsnorm_res_f32(const float *res, const TD *delta, const __nv_bfloat16 *gamma, TY *y,
                         float *sum, int rows, int H, float eps, cudaStream_t stream);
// embedding gather into an fp32 residual row
void embed_f32(const int64_t *ids, const __nv_bfloat16 *table, float *out, int S, int H, int V,
               uint32_t *status, cudaStream_t stream);
// In-place per-head RMSNorm over D (optional) + rotate-half RoPE on the q and k
// heads of a fused [S, (HQ+2*HKV)*D] qkv buffer; positions 0..S-1.
template <typename T>
void qk_norm_rope(T *qkv, int S, int HQ, int HKV, int D, const __nv_bfloat16 *cos_tab,
                  const __nv_bfloat16 *sin_tab, const __nv_bfloat16 *q_norm,
                  const __nv_bfloat16 *k_norm, float eps, cudaStream_t stream);
inline void qk_norm_rope_bf16(__nv_bfloat16 *qkv, int S, int HQ, int HKV, int D,
                              const __nv_bfloat16 *cos_tab, const __nv_bfloat16 *sin_tab,
                              const __nv_bfloat16 *q_norm, const __nv_bfloat16 *k_norm, float eps,
                              cudaStream_t stream) {
  qk_norm_rope<__nv_bfloat16>(qkv, S, HQ, HKV, D, cos_tab, sin_tab, q_norm, k_norm, eps, stream);
}
// tcgen05 causal GQA prefill attention (head_dim 64 or 128).  attention_vt writes
// V^T in fp16 ([kv head * D + d][key], pitch ldv >= S) for KV heads [kv0, kv0 + nkv)
// (nkv < 0: all); attention_tc_bf16 reads Q/K from qkv and V from V^T, out [S, HQ*D].
// A launch may cover query heads [h0, h0 + nh) reading KV heads kv0 + (h - h0) / group
// (nh < 0: all HQ heads, group <= 0: HQ / HKV).  The probabilities enter the PV
// product in fp16 (both operands fp16), a finer rounding than bf16.
// T = __nv_bfloat16 or __half: the format of qkv (and so of the QK^T operands) and out.
template <typename T>
void attention_vt(const T *qkv, __half *vt, long ldv, int S, int HQ, int HKV, int D,
                  cudaStream_t stream, int kv0 = 0, int nkv = -1);
template <typename T>
void attention_tc(const T *qkv, const __half *vt, long ldv, T *out, int S, int HQ, int HKV, int D,
                  float scale, uint32_t *status, cudaStream_t stream, int h0 = 0, int nh = -1,
                  int kv0 = 0, int group = -1);
inline void attention_tc_bf16(const __nv_bfloat16 *qkv, const __half *vt, long ldv,
                              __nv_bfloat16 *out, int S, int HQ, int HKV, int D, float scale,
                              uint32_t *status, cudaStream_t stream, int h0 = 0, int nh = -1,
                              int kv0 = 0, int group = -1) {
  attention_tc<__nv_bfloat16>(qkv, vt, ldv, out, S, HQ, HKV, D, scale, status, stream, h0, nh,
                              kv0, group);
}
// Transpose a row-major [rows, cols] bf16 matrix into [cols, rows] (dst pitch ld_dst).
void transpose_bf16(const __nv_bfloat16 *src, long ld_src, __nv_bfloat16 *dst, long ld_dst,
                    int rows, int cols, cudaStream_t stream);
// Same, converting to fp16 on the way (source bf16 or fp16).
void transpose_bf16_to_f16(const __nv_bfloat16 *src, long ld_src, __half *dst, long ld_dst,
                           int rows, int cols, cudaStream_t stream);
void transpose_f16(const __half *src, long ld_src, __half *dst, long ld_dst, int rows, int cols,
                   cudaStream_t stream);
// In place: n bf16 values -> the same values in fp16 (exact for bf16 weights of normal
// magnitude; values beyond the fp16 range or below its subnormals are not expected in
// weights and saturate / lose low bits).
void bf16_to_f16_inplace(void *data, size_t n, cudaStream_t stream);
// n fp16 values -> fp32
void f16_to_f32(const __half *src, float *dst, int n, cudaStream_t stream);

}  // namespace krb
