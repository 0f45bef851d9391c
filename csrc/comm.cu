// NVLink / NVSwitch collectives over symmetric (peer-mapped) memory (N1-N3).
//
// Every rank holds the same-sized buffers; `PeerPtrs` carries each rank's
// device address of a buffer (peer pointers, readable and writable over
// NVLink). All waits spin on a flag with a bounded clock64 budget and, on
// expiry, record which rank they waited for in a device status word and
// return; nothing traps.
//
// symm_barrier       : rank r stores epoch into flags[peer][r] of every peer
//                      (release, system scope) and waits until its own
//                      flags[r][p] >= epoch for every peer p (acquire).
// symm_reduce        : two-shot, in place: rank r owns chunk r of the flat
//                      fp32 buffer; it sums chunk r over all ranks in fixed
//                      rank order (bitwise identical on every rank), scales,
//                      and writes the result to its own chunk (reduce-scatter)
//                      and, for an all-reduce, to every peer's chunk r. A
//                      per-CTA partial of the squared norm of the reduced
//                      chunk is written for the clip.
// symm_reduce_oneshot: one-shot all-reduce for short buffers: every rank reads
//                      the whole buffer of every rank (fixed rank order, so
//                      bitwise identical everywhere) and writes the scaled sum
//                      to a local output; one NVLink read phase, no second
//                      write phase (latency-bound sizes; the two-shot moves
//                      fewer bytes per rank at large sizes).
// symm_norm_put      : sum of the partials (fixed order) stored into every
//                      peer's norm slot r.
// symm_adamw_gather  : fused AdamW on this rank's shard (fp32 master and
//                      moments, clip coefficient from the W norm slots) that
//                      writes the rounded bf16 parameters into every rank's
//                      parameter buffer (all-gather fused with the cast).
#include "common.cuh"
#include "common.h"

namespace ts {
namespace {

constexpr int kMaxRanks = 8;

struct PeerPtrs {
  unsigned long long p[kMaxRanks];
};

TS_DEVICE void st_release_sys(uint32_t* addr, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(addr), "r"(v) : "memory");
}
TS_DEVICE uint32_t ld_acquire_sys(const uint32_t* addr) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(addr) : "memory");
  return v;
}

// flags layout in each rank's flag buffer: [slot][rank] u32
__global__ void symm_barrier_kernel(PeerPtrs flags, int rank, int world, int slot, uint32_t epoch,
                                    int* __restrict__ status, long long budget) {
  const int p = threadIdx.x;
  if (p < world) {
    uint32_t* remote = reinterpret_cast<uint32_t*>(flags.p[p]) + slot * kMaxRanks + rank;
    __threadfence_system();
    st_release_sys(remote, epoch);
  }
  __syncthreads();
  if (p < world) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(flags.p[rank]) + slot * kMaxRanks + p;
    const long long t0 = clock64();
    while (ld_acquire_sys(mine) < epoch) {
      if (clock64() - t0 > budget) {
        atomicCAS(status, 0, 1000 + p);  // first timeout wins: which peer never arrived
        break;
      }
    }
  }
}

__global__ void symm_reduce_kernel(PeerPtrs bufs, int rank, int world, long long lo, long long hi, float scale,
                                   int write_all, float* __restrict__ partial) {
  __shared__ float red[32];
  float sq = 0.f;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long nv = (hi - lo) / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv; i += stride) {
    const long long e = lo + i * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < world) {
        const float4 v = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(bufs.p[r]) + e);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
    }
    acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
    sq += acc.x * acc.x + acc.y * acc.y + acc.z * acc.z + acc.w * acc.w;
    if (write_all) {
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r)
        if (r < world) *reinterpret_cast<float4*>(reinterpret_cast<float*>(bufs.p[r]) + e) = acc;
    } else {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(bufs.p[rank]) + e) = acc;
    }
  }
  // scalar tail
  for (long long e = lo + nv * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; e < hi; e += stride) {
    float acc = 0.f;
    for (int r = 0; r < world; ++r) acc += reinterpret_cast<const float*>(bufs.p[r])[e];
    acc *= scale;
    sq += acc * acc;
    if (write_all) {
      for (int r = 0; r < world; ++r) reinterpret_cast<float*>(bufs.p[r])[e] = acc;
    } else {
      reinterpret_cast<float*>(bufs.p[rank])[e] = acc;
    }
  }
  __threadfence_system();
  sq = warp_sum(sq);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
  __syncthreads();
  if (threadIdx.x < 32) {
    sq = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    sq = warp_sum(sq);
    if (threadIdx.x == 0) partial[blockIdx.x] = sq;
  }
}

__global__ void symm_reduce_oneshot_kernel(PeerPtrs bufs, int world, long long n, float scale,
                                           float* __restrict__ out) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long nv = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv; i += stride) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r) {
      if (r < world) {
        const float4 v = reinterpret_cast<const float4*>(bufs.p[r])[i];
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
      }
    }
    acc.x *= scale; acc.y *= scale; acc.z *= scale; acc.w *= scale;
    reinterpret_cast<float4*>(out)[i] = acc;
  }
  for (long long e = nv * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; e < n; e += stride) {
    float acc = 0.f;
    for (int r = 0; r < world; ++r) acc += reinterpret_cast<const float*>(bufs.p[r])[e];
    out[e] = acc * scale;
  }
}

// norm slots live in each rank's flag buffer after the barrier slots, as floats
__global__ void symm_norm_put_kernel(const float* __restrict__ partial, int n, PeerPtrs flags, int rank, int world,
                                     int norm_offset) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    float s = 0.f;
    for (int i = 0; i < n; ++i) s += partial[i];
    for (int r = 0; r < world; ++r) {
      float* slot = reinterpret_cast<float*>(reinterpret_cast<uint32_t*>(flags.p[r]) + norm_offset) + rank;
      *slot = s;
    }
    __threadfence_system();
  }
}

__global__ void symm_adamw_gather_kernel(float* __restrict__ master, float* __restrict__ m, float* __restrict__ v,
                                         const float* __restrict__ grad, PeerPtrs params, int world, long long lo,
                                         long long n, float lr, float b1, float b2, float eps, float wd, float bc1,
                                         float bc2, int maximize, const float* __restrict__ norm_slots,
                                         float max_norm, float* __restrict__ norm_out) {
  float sq = 0.f;
  for (int r = 0; r < world; ++r) sq += norm_slots[r];
  const float nrm = sqrtf(sq);
  float coef = 1.f;
  if (max_norm > 0.f) {
    coef = max_norm / (nrm + 1e-6f);
    coef = coef < 1.f ? coef : 1.f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && norm_out != nullptr) norm_out[0] = nrm;
  const float decay = 1.f - lr * wd;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    float g = grad[i] * coef;
    if (maximize) g = -g;
    const float mi = b1 * m[i] + (1.f - b1) * g;
    const float vi = b2 * v[i] + (1.f - b2) * g * g;
    m[i] = mi;
    v[i] = vi;
    const float w = master[i] * decay - lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    master[i] = w;
    const __nv_bfloat16 wb = __float2bfloat16_rn(w);
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) reinterpret_cast<__nv_bfloat16*>(params.p[r])[lo + i] = wb;
  }
  __threadfence_system();
}

// symm_adamw_gather_kernel with four elements per 16-byte access and 8-byte bf16 stores to each peer
// (2-byte stores would cross NVLink as one small packet per element). Needs n4 = n / 4 groups,
// 16-byte aligned fp32 shards and lo % 4 == 0 (8-byte aligned bf16 destinations).
__global__ void symm_adamw_gather_vec_kernel(float4* __restrict__ master, float4* __restrict__ m,
                                             float4* __restrict__ v, const float4* __restrict__ grad, PeerPtrs params,
                                             int world, long long lo, long long n4, float lr, float b1, float b2,
                                             float eps, float wd, float bc1, float bc2, int maximize,
                                             const float* __restrict__ norm_slots, float max_norm,
                                             float* __restrict__ norm_out) {
  float sq = 0.f;
  for (int r = 0; r < world; ++r) sq += norm_slots[r];
  const float nrm = sqrtf(sq);
  float coef = 1.f;
  if (max_norm > 0.f) {
    coef = max_norm / (nrm + 1e-6f);
    coef = coef < 1.f ? coef : 1.f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0 && norm_out != nullptr) norm_out[0] = nrm;
  const float decay = 1.f - lr * wd;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 gv = grad[i];
    float4 mv = m[i], vv = v[i], wv = master[i];
    float* gp = const_cast<float*>(&gv.x);
    float* mp = &mv.x;
    float* vp = &vv.x;
    float* wp = &wv.x;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float g = gp[e] * coef;
      if (maximize) g = -g;
      const float mi = b1 * mp[e] + (1.f - b1) * g;
      const float vi = b2 * vp[e] + (1.f - b2) * g * g;
      mp[e] = mi;
      vp[e] = vi;
      wp[e] = wp[e] * decay - lr * (mi / bc1) / (sqrtf(vi / bc2) + eps);
    }
    m[i] = mv;
    v[i] = vv;
    master[i] = wv;
    __nv_bfloat162 lo2 = __floats2bfloat162_rn(wv.x, wv.y), hi2 = __floats2bfloat162_rn(wv.z, wv.w);
    const uint2 packed = make_uint2(*reinterpret_cast<unsigned*>(&lo2), *reinterpret_cast<unsigned*>(&hi2));
#pragma unroll
    for (int r = 0; r < kMaxRanks; ++r)
      if (r < world) reinterpret_cast<uint2*>(reinterpret_cast<__nv_bfloat16*>(params.p[r]) + lo)[i] = packed;
  }
  __threadfence_system();
}

PeerPtrs to_peers(const std::vector<int64_t>& ptrs) {
  TS_CHECK(!ptrs.empty() && ptrs.size() <= (size_t)kMaxRanks, "1..8 ranks supported, got ", ptrs.size());
  PeerPtrs pp{};
  for (size_t i = 0; i < ptrs.size(); ++i) pp.p[i] = (unsigned long long)ptrs[i];
  return pp;
}

}  // namespace

void symm_barrier(const std::vector<int64_t>& flag_ptrs, int64_t rank, int64_t slot, int64_t epoch,
                  at::Tensor& status, double timeout_s) {
  TS_CHECK(status.is_cuda() && status.scalar_type() == at::kInt, "status must be a CUDA int32 tensor");
  TS_CHECK(slot >= 0 && slot < 64, "barrier slot out of range");
  const c10::cuda::CUDAGuard guard(status.device());
  const int world = (int)flag_ptrs.size();
  const long long budget = (long long)(timeout_s * 2.0e9);
  symm_barrier_kernel<<<1, 32, 0, stream()>>>(to_peers(flag_ptrs), (int)rank, world, (int)slot, (uint32_t)epoch,
                                              status.data_ptr<int>(), budget);
  TS_LAUNCH_CHECK();
}

at::Tensor symm_reduce(const std::vector<int64_t>& buf_ptrs, int64_t rank, int64_t lo, int64_t hi, double scale,
                       bool write_all, const at::Tensor& like) {
  const c10::cuda::CUDAGuard guard(like.device());
  TS_CHECK(lo % 4 == 0 && lo <= hi, "chunk must start on a 16-byte boundary");
  const int blocks = 2 * sm_count(like.get_device());
  auto partial = at::zeros({blocks}, like.options().dtype(at::kFloat));
  symm_reduce_kernel<<<blocks, 512, 0, stream()>>>(to_peers(buf_ptrs), (int)rank, (int)buf_ptrs.size(), lo, hi,
                                                   (float)scale, write_all ? 1 : 0, partial.data_ptr<float>());
  TS_LAUNCH_CHECK();
  return partial;
}

void symm_reduce_oneshot(const std::vector<int64_t>& buf_ptrs, int64_t n, double scale, at::Tensor& out) {
  TS_CHECK(out.is_cuda() && out.scalar_type() == at::kFloat && out.is_contiguous() && out.numel() >= n,
           "one-shot all-reduce: out must be a contiguous fp32 CUDA tensor of at least n elements");
  TS_CHECK((reinterpret_cast<uintptr_t>(out.data_ptr()) & 15) == 0, "one-shot all-reduce: out must be 16-byte aligned");
  const c10::cuda::CUDAGuard guard(out.device());
  if (n == 0) return;
  const int blocks = (int)std::min<long long>((n / 4 + 511) / 512 + 1, 2LL * sm_count(out.get_device()));
  symm_reduce_oneshot_kernel<<<blocks, 512, 0, stream()>>>(to_peers(buf_ptrs), (int)buf_ptrs.size(), n,
                                                           (float)scale, out.data_ptr<float>());
  TS_LAUNCH_CHECK();
}

void symm_norm_put(const at::Tensor& partial, const std::vector<int64_t>& flag_ptrs, int64_t rank,
                   int64_t norm_offset) {
  const c10::cuda::CUDAGuard guard(partial.device());
  symm_norm_put_kernel<<<1, 32, 0, stream()>>>(partial.data_ptr<float>(), (int)partial.numel(),
                                               to_peers(flag_ptrs), (int)rank, (int)flag_ptrs.size(),
                                               (int)norm_offset);
  TS_LAUNCH_CHECK();
}

void symm_adamw_gather(at::Tensor& master, at::Tensor& m, at::Tensor& v, const at::Tensor& grad,
                       const std::vector<int64_t>& param_ptrs, int64_t lo, double lr, double b1, double b2,
                       double eps, double wd, int64_t step, bool maximize, const at::Tensor& norm_slots,
                       double max_norm, at::Tensor& norm_out) {
  check_cuda(master, "master");
  check_cuda(grad, "grad");
  TS_CHECK(grad.numel() == master.numel(), "grad shard size differs from the master shard");
  const c10::cuda::CUDAGuard guard(master.device());
  const long long n = master.numel();
  if (n == 0) return;
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2 = 1.f - (float)std::pow(b2, (double)step);
  const int blocks = 4 * sm_count(master.get_device());
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  bool vec = n % 4 == 0 && lo % 4 == 0 && al(master.data_ptr()) && al(m.data_ptr()) && al(v.data_ptr()) &&
             al(grad.data_ptr());
  for (int64_t p : param_ptrs) vec = vec && (p % 8 == 0);
  if (vec) {
    symm_adamw_gather_vec_kernel<<<blocks, 256, 0, stream()>>>(
        (float4*)master.data_ptr<float>(), (float4*)m.data_ptr<float>(), (float4*)v.data_ptr<float>(),
        (const float4*)grad.data_ptr<float>(), to_peers(param_ptrs), (int)param_ptrs.size(), lo, n / 4, (float)lr,
        (float)b1, (float)b2, (float)eps, (float)wd, bc1, bc2, maximize ? 1 : 0, norm_slots.data_ptr<float>(),
        (float)max_norm, norm_out.data_ptr<float>());
  } else {
    symm_adamw_gather_kernel<<<blocks, 256, 0, stream()>>>(
        master.data_ptr<float>(), m.data_ptr<float>(), v.data_ptr<float>(), grad.data_ptr<float>(),
        to_peers(param_ptrs), (int)param_ptrs.size(), lo, n, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd,
        bc1, bc2, maximize ? 1 : 0, norm_slots.data_ptr<float>(), (float)max_norm, norm_out.data_ptr<float>());
  }
  TS_LAUNCH_CHECK();
}

}  // namespace ts
