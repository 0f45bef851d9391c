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

template <typename P>
__global__ void adamw_kernel(float* __restrict__ master, P* __restrict__ param, const float* __restrict__ grad,
                             float* __restrict__ m, float* __restrict__ v, long long n, float lr, float b1, float b2,
                             float eps, float wd, float bc1, float bc2, const float* __restrict__ scale_ptr,
                             float scale, int maximize) {
  const float gs = scale_ptr != nullptr ? scale * scale_ptr[0] : scale;
  const float decay = 1.f - lr * wd;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    float g = grad[i] * gs;
    if (maximize) g = -g;
    const float mi = b1 * m[i] + (1.f - b1) * g;
    const float vi = b2 * v[i] + (1.f - b2) * g * g;
    m[i] = mi;
    v[i] = vi;
    const float denom = sqrtf(vi / bc2) + eps;
    const float w = master[i] * decay - lr * (mi / bc1) / denom;
    master[i] = w;
    param[i] = from_f<P>(w);
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
  const int blocks = 4 * sm_count(master.get_device());
  const float* sp = scale_t ? scale_t->data_ptr<float>() : nullptr;
  if (param.scalar_type() == at::kBFloat16) {
    adamw_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>(
        master.data_ptr<float>(), (__nv_bfloat16*)param.data_ptr(), grad.data_ptr<float>(), m.data_ptr<float>(),
        v.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2, (float)eps, (float)wd, bc1, bc2, sp, (float)scale,
        maximize ? 1 : 0);
  } else if (param.scalar_type() == at::kFloat) {
    adamw_kernel<float><<<blocks, 256, 0, stream()>>>(master.data_ptr<float>(), param.data_ptr<float>(),
                                                      grad.data_ptr<float>(), m.data_ptr<float>(),
                                                      v.data_ptr<float>(), n, (float)lr, (float)b1, (float)b2,
                                                      (float)eps, (float)wd, bc1, bc2, sp, (float)scale,
                                                      maximize ? 1 : 0);
  } else {
    TS_CHECK(false, "adamw: unsupported parameter dtype");
  }
  TS_LAUNCH_CHECK();
}

}  // namespace ts
