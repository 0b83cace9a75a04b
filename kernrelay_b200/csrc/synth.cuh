// Deterministic, order-independent weight synthesis shared by the host (model
// generator, oracle fixtures) and the device (loading models whose manifest
// marks large tensors as synthetic instead of storing them in weights.bin).
//
// Element i of tensor `name` with seed `seed`:
//   key  = mix64(fnv1a64(name) ^ mix64(seed))
//   h_j  = mix64(key + (12*i/2 + j + 1) * GAMMA), j = 0..5   (SplitMix64 stream)
//   u    = the low and high 24-bit fields of each h_j -> 12 integers in [0, 2^24)
//   c    = sum(u) - 6*(2^24 - 1)                        (exact in int64)
//   x    = mean + double(c) * (std * 2^-24)               (Irwin-Hall(12) ~ N(mean, std^2))
//   bf16 = round-to-nearest-even(float(x))
// Every step is exact integer work or a single correctly rounded IEEE operation,
// so host and device produce bit-identical values.
#pragma once

#include <stdint.h>

#ifndef __CUDACC__
#define KRB_HD
#else
#define KRB_HD __host__ __device__
#endif

namespace krb {

constexpr uint64_t kSynthGamma = 0x9E3779B97F4A7C15ull;

KRB_HD inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

inline uint64_t fnv1a64(const char *s) {
  uint64_t h = 0xCBF29CE484222325ull;
  for (; *s; ++s) {
    h ^= static_cast<unsigned char>(*s);
    h *= 0x100000001B3ull;
  }
  return h;
}

inline uint64_t synth_key(const char *name, uint64_t seed) {
  return mix64(fnv1a64(name) ^ mix64(seed));
}

KRB_HD inline uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
#ifdef __CUDA_ARCH__
  u = __float_as_uint(f);
#else
  __builtin_memcpy(&u, &f, 4);
#endif
  if ((u & 0x7F800000u) == 0x7F800000u) return static_cast<uint16_t>((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

KRB_HD inline uint16_t synth_normal_bf16(uint64_t key, uint64_t i, double scale /* std*2^-24 */,
                                         double mean = 0.0) {
  int64_t s = 0;
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    const uint64_t h = mix64(key + (i * 6ull + uint64_t(j) + 1ull) * kSynthGamma);
    s += static_cast<int64_t>(h & 0xFFFFFFull) + static_cast<int64_t>((h >> 32) & 0xFFFFFFull);
  }
  const int64_t c = s - 6ll * ((1ll << 24) - 1ll);
  const double x = mean + static_cast<double>(c) * scale;
#ifdef __CUDA_ARCH__
  const float f = __double2float_rn(x);
#else
  const float f = static_cast<float>(x);
#endif
  return f32_to_bf16_bits(f);
}

inline double synth_scale(double std_) { return std_ * (1.0 / 16777216.0); }

}  // namespace krb
