// Flat-buffer optimizer kernels: deterministic squared-norm reduction and the
// fused AdamW update over an fp32 master copy.
//
// adamw_flat updates, for every element i of one contiguous parameter range:
//   g   = grad[i] * grad_scale            (global-norm clip folded in)
//   g   = maximize ? -g : g
//   m   = b1 m + (1 - b1) g ;  v = b2 v + (1 - b2) g^2
//   w   = w * (1 - lr wd) - lr * (m / bc1) / (sqrt(v / bc2) + eps)
//   param[i] = round(w)                   (bf16 or fp32 model copy)
// matching torch.optim.AdamW's decoupled weight decay and bias correction.
#include "common.cuh"
#include "common.h"

namespace ts {
namespace {

__global__ void sq_partial_kernel(const float* __restrict__ x, long long n, float* __restrict__ partial) {
  __shared__ float red[32];
  float s = 0.f;
  const long long stride = (long long)gridDim.x * blockDim.x;
  const long long nv = n / 4;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    s += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  for (long long i = nv * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) s += x[i] * x[i];
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    s = warp_sum(s);
    if (threadIdx.x == 0) partial[blockIdx.x] = s;
  }
}

__global__ void sum_small_kernel(const float* __restrict__ partial, int n, float* __restrict__ out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    double s = 0.0;
    for (int i = 0; i < n; ++i) s += (double)partial[i];
    out[0] = (float)s;
  }
}

struct AdamArgs {
  float lr, b1, b2, eps, decay, bc1, bc2, gs;
  int maximize;
};

__device__ __forceinline__ float adam_one(float& w, float& mi, float& vi, float g, const AdamArgs& a) {
  g = g * a.gs;
  if (a.maximize) g = -g;
  mi = a.b1 * mi + (1.f - a.b1) * g;
  vi = a.b2 * vi + (1.f - a.b2) * g * g;
  const float denom = sqrtf(vi / a.bc2) + a.eps;
  w = w * a.decay - a.lr * (mi / a.bc1) / denom;
  return w;
}

__device__ __forceinline__ AdamArgs adam_args(float lr, float b1, float b2, float eps, float wd, float bc1,
                                              float bc2, const float* scale_ptr, float scale, int maximize) {
  AdamArgs a;
  a.lr = lr; a.b1 = b1; a.b2 = b2; a.eps = eps; a.decay = 1.f - lr * wd; a.bc1 = bc1; a.bc2 = bc2;
  a.gs = scale_ptr != nullptr ? scale * scale_ptr[0] : scale;
  a.maximize = maximize;
  return a;
}

template <typename P>
__global__ void adamw_kernel(float* __restrict__ master, P* __restrict__ param, const float* __restrict__ grad,
                             float* __restrict__ m, float* __restrict__ v, long long n, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, const float* __restrict__ scale_ptr,
                             float scale, int maximize) {
  const AdamArgs a = adam_args(lr, b1, b2, eps, wd, bc1, bc2, scale_ptr, scale, maximize);
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    float w = master[i], mi = m[i], vi = v[i];
    adam_one(w, mi, vi, grad[i], a);
    m[i] = mi;
    v[i] = vi;
    master[i] = w;
    param[i] = from_f<P>(w);
  }
}

template <typename P> struct Pack4;
template <> struct Pack4<float> {
  using T = float4;
  static __device__ __forceinline__ T make(const float4& w) { return w; }
};
template <> struct Pack4<__nv_bfloat16> {
  using T = uint2;
  static __device__ __forceinline__ T make(const float4& w) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(w.x, w.y), hi = __floats2bfloat162_rn(w.z, w.w);
    return make_uint2(*reinterpret_cast<unsigned*>(&lo), *reinterpret_cast<unsigned*>(&hi));
  }
};

// Same per-element arithmetic as adamw_kernel, four elements per 16-byte access and two such groups in
// flight per thread (five streams of fp32 traffic need many bytes in flight to reach HBM bandwidth).
// Every pointer is 16-byte aligned (8-byte for a bf16 model copy); n4 = n / 4 groups.
template <typename P>
__global__ void __launch_bounds__(256) adamw_vec_kernel(float4* __restrict__ master, typename Pack4<P>::T* __restrict__ param,
                                 const float4* __restrict__ grad, float4* __restrict__ m, float4* __restrict__ v,
                                 long long n4, float lr, float b1, float b2, float eps, float wd, float bc1,
                                 float bc2, const float* __restrict__ scale_ptr, float scale, int maximize) {
  const AdamArgs a = adam_args(lr, b1, b2, eps, wd, bc1, bc2, scale_ptr, scale, maximize);
  const long long stride = (long long)gridDim.x * blockDim.x;
  long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x;
  for (; i + stride < n4; i += 2 * stride) {
    float4 w[2], mi[2], vi[2], g[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const long long k = i + u * stride;
      w[u] = master[k]; mi[u] = m[k]; vi[u] = v[k]; g[u] = grad[k];
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const long long k = i + u * stride;
      adam_one(w[u].x, mi[u].x, vi[u].x, g[u].x, a);
      adam_one(w[u].y, mi[u].y, vi[u].y, g[u].y, a);
      adam_one(w[u].z, mi[u].z, vi[u].z, g[u].z, a);
      adam_one(w[u].w, mi[u].w, vi[u].w, g[u].w, a);
      m[k] = mi[u]; v[k] = vi[u]; master[k] = w[u];
      param[k] = Pack4<P>::make(w[u]);
    }
  }
  if (i < n4) {
    float4 w = master[i], mi = m[i], vi = v[i];
    const float4 g = grad[i];
    adam_one(w.x, mi.x, vi.x, g.x, a);
    adam_one(w.y, mi.y, vi.y, g.y, a);
    adam_one(w.z, mi.z, vi.z, g.z, a);
    adam_one(w.w, mi.w, vi.w, g.w, a);
    m[i] = mi; v[i] = vi; master[i] = w;
    param[i] = Pack4<P>::make(w);
  }
}

// clip coefficient min(1, max_norm / (norm + 1e-6)) computed on the device from
// the squared norm, so no host round trip is needed before the update.
__global__ void clip_coef_kernel(const float* __restrict__ sq, float max_norm, float* __restrict__ coef,
                                 float* __restrict__ norm_out) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    const float nrm = sqrtf(sq[0]);
    norm_out[0] = nrm;
    const float c = max_norm / (nrm + 1e-6f);
    coef[0] = c < 1.f ? c : 1.f;
  }
}

}  // namespace

at::Tensor sq_norm(const at::Tensor& x) {
  check_cuda(x, "x");
  TS_CHECK(x.scalar_type() == at::kFloat, "sq_norm expects fp32");
  const c10::cuda::CUDAGuard guard(x.device());
  const int blocks = 2 * sm_count(x.get_device());
  auto partial = at::empty({blocks}, x.options());
  auto out = at::empty({1}, x.options());
  sq_partial_kernel<<<blocks, 512, 0, stream()>>>(x.data_ptr<float>(), x.numel(), partial.data_ptr<float>());
  sum_small_kernel<<<1, 32, 0, stream()>>>(partial.data_ptr<float>(), blocks, out.data_ptr<float>());
  TS_LAUNCH_CHECK();
  return out;
}

std::vector<at::Tensor> clip_coef(const at::Tensor& sq, double max_norm) {
  const c10::cuda::CUDAGuard guard(sq.device());
  auto coef = at::empty({1}, sq.options());
  auto nrm = at::empty({1}, sq.options());
  clip_coef_kernel<<<1, 32, 0, stream()>>>(sq.data_ptr<float>(), (float)max_norm, coef.data_ptr<float>(),
                                           nrm.data_ptr<float>());
  TS_LAUNCH_CHECK();
  return {coef, nrm};
}

void adamw_flat(at::Tensor& master, at::Tensor& param, const at::Tensor& grad, at::Tensor& m, at::Tensor& v,
                double lr, double b1, double b2, double eps, double wd, int64_t step,
                const c10::optional<at::Tensor>& scale_t, double scale, bool maximize) {
  check_cuda(master, "master");
  check_cuda(param, "param");
  check_cuda(grad, "grad");
  check_cuda(m, "m");
  check_cuda(v, "v");
  const long long n = master.numel();
  TS_CHECK(param.numel() == n && grad.numel() == n && m.numel() == n && v.numel() == n, "adamw size mismatch");
  TS_CHECK(step >= 1, "adamw step counts from 1");
  const c10::cuda::CUDAGuard guard(master.device());
  if (n == 0) return;
  const float bc1 = 1.f - (float)std::pow(b1, (double)step);
  const float bc2 = 1.f - (float)std::pow(b2, (double)step);
  const float* sp = scale_t ? scale_t->data_ptr<float>() : nullptr;
  const bool bf16 = param.scalar_type() == at::kBFloat16;
  TS_CHECK(bf16 || param.scalar_type() == at::kFloat, "adamw: unsupported parameter dtype");
  auto al = [](const void* p, uintptr_t b) { return (reinterpret_cast<uintptr_t>(p) % b) == 0; };
  const bool vec = al(master.data_ptr(), 16) && al(grad.data_ptr(), 16) && al(m.data_ptr(), 16) &&
                   al(v.data_ptr(), 16) && al(param.data_ptr(), bf16 ? 8 : 16);
  const long long n4 = vec ? n / 4 : 0;
  const long long head = n4 * 4;  // elements done by the vector kernel; the rest by the scalar one
  const int sms = sm_count(master.get_device());
  if (n4 > 0) {
    const long long want = (n4 + 511) / 512;  // two groups per thread per pass
    const int blocks = (int)std::min<long long>(want, 8LL * sms);
    if (bf16)
      adamw_vec_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>(
          (float4*)master.data_ptr<float>(), (uint2*)param.data_ptr(), (const float4*)grad.data_ptr<float>(),
          (float4*)m.data_ptr<float>(), (float4*)v.data_ptr<float>(), n4, (float)lr, (float)b1, (float)b2,
          (float)eps, (float)wd, bc1, bc2, sp, (float)scale, maximize ? 1 : 0);
    else
      adamw_vec_kernel<float><<<blocks, 256, 0, stream()>>>(
          (float4*)master.data_ptr<float>(), (float4*)param.data_ptr<float>(), (const float4*)grad.data_ptr<float>(),
          (float4*)m.data_ptr<float>(), (float4*)v.data_ptr<float>(), n4, (float)lr, (float)b1, (float)b2,
          (float)eps, (float)wd, bc1, bc2, sp, (float)scale, maximize ? 1 : 0);
  }
  if (head < n) {
    const long long rest = n - head;
    const int blocks = (int)std::min<long long>((rest + 255) / 256, 4LL * sms);
    float* mp = master.data_ptr<float>() + head;
    if (bf16)
      adamw_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>(
          mp, (__nv_bfloat16*)param.data_ptr() + head, grad.data_ptr<float>() + head, m.data_ptr<float>() + head,
          v.data_ptr<float>() + head, rest, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, bc1, bc2, sp,
          (float)scale, maximize ? 1 : 0);
    else
      adamw_kernel<float><<<blocks, 256, 0, stream()>>>(
          mp, param.data_ptr<float>() + head, grad.data_ptr<float>() + head, m.data_ptr<float>() + head,
          v.data_ptr<float>() + head, rest, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, bc1, bc2, sp,
          (float)scale, maximize ? 1 : 0);
  }
  TS_LAUNCH_CHECK();
}

}  // namespace ts
