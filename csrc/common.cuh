// Shared device helpers for the thundersync_b200 native kernels (sm_100a).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define TS_HOST_DEVICE __host__ __device__ __forceinline__
#define TS_DEVICE __device__ __forceinline__

namespace ts {

TS_DEVICE float to_f(float x) { return x; }
TS_DEVICE float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
TS_DEVICE float to_f(__half x) { return __half2float(x); }

template <typename T> TS_DEVICE T from_f(float x);
template <> TS_DEVICE float from_f<float>(float x) { return x; }
template <> TS_DEVICE __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> TS_DEVICE __half from_f<__half>(float x) { return __float2half_rn(x); }

// Round-trip through T (the rounding a tensor of dtype T would apply).
template <typename T> TS_DEVICE float round_to(float x) { return to_f(from_f<T>(x)); }

TS_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
TS_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 16-byte vector of T elements.
template <typename T> struct Vec {
  static constexpr int N = 16 / sizeof(T);
  union {
    uint4 raw;
    T e[N];
  };
};

template <typename T> TS_DEVICE Vec<T> load_vec(const T* p) {
  Vec<T> v;
  v.raw = *reinterpret_cast<const uint4*>(p);
  return v;
}
template <typename T> TS_DEVICE void store_vec(T* p, const Vec<T>& v) { *reinterpret_cast<uint4*>(p) = v.raw; }

// Online-softmax merge of (max, sum) pairs, sum expressed relative to its max.
TS_DEVICE void lse_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) { m = m2; s = s2; return; }
  float mx = fmaxf(m, m2);
  s = s * expf(m - mx) + s2 * expf(m2 - mx);
  m = mx;
}

}  // namespace ts
