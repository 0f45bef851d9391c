// Host-side helpers shared by the native sources.
#pragma once

#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <map>
#include <mutex>
#include <utility>

#define TS_CHECK(cond, ...) TORCH_CHECK(cond, "thundersync_b200: ", __VA_ARGS__)
#define TS_CUDA_CHECK(expr)                                                                 \
  do {                                                                                      \
    cudaError_t _e = (expr);                                                                \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error ", cudaGetErrorString(_e), " at ", __FILE__, \
                ":", __LINE__);                                                             \
  } while (0)
#define TS_LAUNCH_CHECK() TS_CUDA_CHECK(cudaGetLastError())

namespace ts {

inline int sm_count(int device) {
  static int cached[64] = {0};
  if (device < 64 && cached[device]) return cached[device];
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
  if (device < 64) cached[device] = n;
  return n;
}

inline cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device): the attribute persists, and
// setting it on every launch cost host time on the layer loop's critical path
inline void ensure_smem(const void* fn, int bytes) {
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> done;
  int dev = 0;
  TS_CUDA_CHECK(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  int& have = done[{fn, dev}];
  if (have >= bytes) return;
  TS_CUDA_CHECK(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  have = bytes;
}

inline void check_cuda(const at::Tensor& t, const char* name) {
  TS_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TS_CHECK(t.is_contiguous(), name, " must be contiguous");
}

}  // namespace ts
