// Device-side weight synthesis and small utility kernels.
#include "common.h"
#include "model.h"
#include "synth.cuh"

namespace krb {

__global__ void synth_normal_kernel(uint16_t *dst, size_t n, uint64_t key, double scale,
                                    double mean) {
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
    dst[i] = synth_normal_bf16(key, i, scale, mean);
}

void synth_normal_device(__nv_bfloat16 *dst, size_t n, uint64_t key, double std_, double mean,
                         cudaStream_t stream) {
  if (!n) return;
  int dev = 0;
  KRB_CUDA(cudaGetDevice(&dev));
  const int blocks = sm_count(dev) * 8;
  synth_normal_kernel<<<blocks, 256, 0, stream>>>(reinterpret_cast<uint16_t *>(dst), n, key,
                                                  synth_scale(std_), mean);
  KRB_CUDA(cudaGetLastError());
}

__global__ void fill_kernel(__nv_bfloat16 *dst, size_t n, float v) {
  const size_t stride = size_t(gridDim.x) * blockDim.x;
  const __nv_bfloat16 b = __float2bfloat16_rn(v);
  for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) dst[i] = b;
}

void fill_const_device(__nv_bfloat16 *dst, size_t n, float value, cudaStream_t stream) {
  if (!n) return;
  fill_kernel<<<512, 256, 0, stream>>>(dst, n, value);
  KRB_CUDA(cudaGetLastError());
}

__global__ void bump_kernel(uint32_t *epoch) { *epoch += 1u; }

void bump_epoch(uint32_t *epoch, cudaStream_t stream) {
  bump_kernel<<<1, 1, 0, stream>>>(epoch);
  KRB_CUDA(cudaGetLastError());
}

__global__ void bf16_to_f32_kernel(const __nv_bfloat16 *src, float *dst, int n) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
    dst[i] = __bfloat162float(src[i]);
}

void bf16_row_to_f32(const __nv_bfloat16 *src, float *dst, int n, cudaStream_t stream) {
  bf16_to_f32_kernel<<<(n + 255) / 256 < 1024 ? (n + 255) / 256 : 1024, 256, 0, stream>>>(src, dst,
                                                                                           n);
  KRB_CUDA(cudaGetLastError());
}

}  // namespace krb
