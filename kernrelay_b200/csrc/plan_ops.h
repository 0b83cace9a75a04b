// fp16 operator launchers of the schedule executor (plan.cu).  Shapes are row-major
// [rows, cols]; every launcher is asynchronous on `stream`.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace krb {
namespace plan {

constexpr int64_t kMaxSortCols = 16384;  // one row's 64-bit keys fit in shared memory

// deterministic inputs (exec/exec_main.cpp:74-88), generated on the device
void det_fill_f16(__half *dst, uint64_t n, uint32_t seed, cudaStream_t stream);
// K-major copy of a logical row-major [K, N] matrix: dst[n * K + k] = value(k * N + n)
void det_fill_f16_t(__half *dst, int64_t K, int64_t N, uint32_t seed, cudaStream_t stream);
void embedding_indices(int64_t *idx, int64_t rows, int64_t dim0, uint32_t seed,
                       cudaStream_t stream);

void add_f16(const __half *a, const __half *b, __half *out, uint64_t n, cudaStream_t stream);
void gelu_f16(const __half *in, __half *out, uint64_t n, cudaStream_t stream);
void scale_f16(const __half *in, __half *out, uint64_t n, float k, uint32_t iters,
               cudaStream_t stream);
void cast_f16_f32(const __half *in, float *out, uint64_t n, cudaStream_t stream);
void softmax_rows_f16(const __half *in, __half *out, int64_t rows, int64_t cols,
                      cudaStream_t stream);
void layernorm_rows_f16(const __half *in, const __half *w, const __half *b, __half *out,
                        int64_t rows, int64_t cols, float eps, cudaStream_t stream);
void topk_rows_f16(const __half *in, int64_t rows, int64_t cols, int64_t k, __half *vals,
                   int64_t *idx, cudaStream_t stream);
void sort_rows_f16(const __half *in, int64_t rows, int64_t cols, __half *vals, int64_t *idx,
                   cudaStream_t stream);
void embedding_f16(const __half *weight, const int64_t *idx, __half *out, int64_t rows,
                   int64_t cols, int64_t V, uint32_t *status, cudaStream_t stream);
void mac_f16(const __half *in, __half *out, uint32_t elems, uint32_t iters, uint32_t blocks,
             float acc0, cudaStream_t stream);

}  // namespace plan
}  // namespace krb
