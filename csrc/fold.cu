// Flat-buffer statistic kernels (K15', K10') and the LM-head softmax passes.
//
// fold_stats : g2 += src; g1 += r * src          (GRPO reward-linear statistics)
// axpby      : out += a * x + b * y               (group-close combine)
// scale      : x *= s
// reduce_into: out += sum_i part_i, fixed order   (boundary-adjoint reduction, <=16 parts)
// lse_gather : per row of fp32 logits, online max/sum -> log-prob of the target,
//              log-sum-exp and (optionally) entropy, one pass over the row
// dlogits    : g * (onehot - softmax) (+ entropy terms), written as bf16 or fp32
//
// Flat kernels are grid-stride loops over 16-byte vectors sized to 4 CTAs per
// SM; they are HBM-bound and issue one load per operand per element.
#include "common.cuh"
#include "common.h"
#include "bounds.cuh"

namespace ts {
namespace {

constexpr int kSiteGatherTarget = 2;  // bounds site: log-prob gather target id
constexpr int kSiteFlatVector = 3;   // bounds site (debug build): a flat kernel's float4 index past the end

template <typename S>
__global__ void fold_kernel(float* __restrict__ g1, float* __restrict__ g2, const S* __restrict__ src, long long n,
                            float r) {
  const long long nv = n / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv; i += stride) {
    TS_BOUND_DEBUG(4 * i + 3 < n, kSiteFlatVector, i);
    float s[4];
    if constexpr (std::is_same<S, float>::value) {
      float4 v = reinterpret_cast<const float4*>(src)[i];
      s[0] = v.x; s[1] = v.y; s[2] = v.z; s[3] = v.w;
    } else {
      const S* p = src + i * 4;
#pragma unroll
      for (int e = 0; e < 4; ++e) s[e] = to_f(p[e]);
    }
    float4 b = reinterpret_cast<float4*>(g2)[i];
    b.x += s[0]; b.y += s[1]; b.z += s[2]; b.w += s[3];
    reinterpret_cast<float4*>(g2)[i] = b;
    if (g1 != nullptr) {
      float4 a = reinterpret_cast<float4*>(g1)[i];
      a.x = fmaf(r, s[0], a.x); a.y = fmaf(r, s[1], a.y); a.z = fmaf(r, s[2], a.z); a.w = fmaf(r, s[3], a.w);
      reinterpret_cast<float4*>(g1)[i] = a;
    }
  }
  // tail
  for (long long i = nv * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float s = to_f(src[i]);
    g2[i] += s;
    if (g1 != nullptr) g1[i] = fmaf(r, s, g1[i]);
  }
}

__global__ void axpby_kernel(float* __restrict__ out, const float* __restrict__ x, const float* __restrict__ y,
                             long long n, float a, float b) {
  const long long nv = n / 4;
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < nv; i += stride) {
    TS_BOUND_DEBUG(4 * i + 3 < n, kSiteFlatVector, i);
    float4 o = reinterpret_cast<float4*>(out)[i];
    const float4 xv = reinterpret_cast<const float4*>(x)[i];
    if (y != nullptr) {
      const float4 yv = reinterpret_cast<const float4*>(y)[i];
      o.x += fmaf(a, xv.x, b * yv.x); o.y += fmaf(a, xv.y, b * yv.y);
      o.z += fmaf(a, xv.z, b * yv.z); o.w += fmaf(a, xv.w, b * yv.w);
    } else {
      o.x = fmaf(a, xv.x, o.x); o.y = fmaf(a, xv.y, o.y); o.z = fmaf(a, xv.z, o.z); o.w = fmaf(a, xv.w, o.w);
    }
    reinterpret_cast<float4*>(out)[i] = o;
  }
  for (long long i = nv * 4 + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    out[i] += y != nullptr ? fmaf(a, x[i], b * y[i]) : a * x[i];
  }
}

__global__ void scale_kernel(float* __restrict__ x, long long n, float s) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) x[i] *= s;
}

struct PartList {
  const void* p[16];
  int n;
  int is_bf16;
};

__global__ void reduce_into_kernel(float* __restrict__ out, PartList parts, long long n) {
  const long long stride = (long long)gridDim.x * blockDim.x;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += stride) {
    float acc = out[i];
    for (int k = 0; k < parts.n; ++k) {
      acc += parts.is_bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(parts.p[k])[i])
                           : reinterpret_cast<const float*>(parts.p[k])[i];
    }
    out[i] = acc;
  }
}

// One CTA per row of fp32 logits [R, V].
__global__ void __launch_bounds__(512) lse_gather_kernel(const float* __restrict__ logits,
                                                         const int64_t* __restrict__ tgt, float* __restrict__ lp,
                                                         float* __restrict__ lse, float* __restrict__ ent, int V) {
  const int row = blockIdx.x;
  const float* l = logits + (size_t)row * V;
  float m = -INFINITY, s = 0.f, t = 0.f;  // t = sum exp(l - m) * l (entropy)
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float x = l[j];
    if (x > m) {
      const float c = expf(m - x);
      s *= c;
      t *= c;
      m = x;
    }
    const float e = expf(x - m);
    s += e;
    t += e * x;
  }
  __shared__ float sm[32], ss[32], st[32];
  // warp merge
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const float t2 = __shfl_xor_sync(0xffffffffu, t, o);
    const float mx = fmaxf(m, m2);
    const float c1 = m == -INFINITY ? 0.f : expf(m - mx);
    const float c2 = m2 == -INFINITY ? 0.f : expf(m2 - mx);
    s = s * c1 + s2 * c2;
    t = t * c1 + t2 * c2;
    m = mx;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) { sm[warp] = m; ss[warp] = s; st[warp] = t; }
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    m = lane < nw ? sm[lane] : -INFINITY;
    s = lane < nw ? ss[lane] : 0.f;
    t = lane < nw ? st[lane] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
      const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
      const float t2 = __shfl_xor_sync(0xffffffffu, t, o);
      const float mx = fmaxf(m, m2);
      const float c1 = m == -INFINITY ? 0.f : expf(m - mx);
      const float c2 = m2 == -INFINITY ? 0.f : expf(m2 - mx);
      s = s * c1 + s2 * c2;
      t = t * c1 + t2 * c2;
      m = mx;
    }
    if (lane == 0) {
      const float L = m + logf(s);
      lse[row] = L;
      const int64_t target = tgt[row];
      if (target < 0 || target >= V) {  // a target id outside the vocabulary: recorded, log-prob NaN, no read
        TS_BOUND_RECORD(kSiteGatherTarget, target);
        lp[row] = __int_as_float(0x7fc00000);
      } else {
        lp[row] = l[target] - L;
      }
      if (ent != nullptr) ent[row] = L - t / s;
    }
  }
}

template <typename O>
__global__ void __launch_bounds__(512) dlogits_kernel(const float* __restrict__ logits, const int64_t* __restrict__ tgt,
                                                      const float* __restrict__ lse, const float* __restrict__ g_lp,
                                                      const float* __restrict__ g_ent, const float* __restrict__ ent,
                                                      O* __restrict__ out, int V) {
  const int row = blockIdx.x;
  const float* l = logits + (size_t)row * V;
  O* o = out + (size_t)row * V;
  const float L = lse[row];
  const float gl = g_lp[row];
  const float ge = g_ent != nullptr ? g_ent[row] : 0.f;
  const float H = ent != nullptr ? ent[row] : 0.f;
  const int64_t t = tgt[row];
  for (int j = threadIdx.x; j < V; j += blockDim.x) {
    const float lg = l[j] - L;
    const float p = expf(lg);
    float d = g_ent != nullptr ? -p * (gl + ge * (lg + H)) : -p * gl;
    if (j == t) d += gl;
    o[j] = from_f<O>(d);
  }
}

inline int flat_blocks(int device) { return 4 * sm_count(device); }

}  // namespace

void fold_stats(const c10::optional<at::Tensor>& g1, at::Tensor& g2, const at::Tensor& src, double r) {
  check_cuda(g2, "g2");
  check_cuda(src, "src");
  TS_CHECK(g2.scalar_type() == at::kFloat, "statistics must be fp32");
  TS_CHECK(src.numel() == g2.numel(), "fold size mismatch");
  const c10::cuda::CUDAGuard guard(g2.device());
  float* p1 = nullptr;
  if (g1 && r != 0.0) {
    check_cuda(*g1, "g1");
    p1 = g1->data_ptr<float>();
  }
  const long long n = g2.numel();
  if (n == 0) return;
  const int blocks = flat_blocks(g2.get_device());
  if (src.scalar_type() == at::kFloat) {
    fold_kernel<float><<<blocks, 256, 0, stream()>>>(p1, g2.data_ptr<float>(), src.data_ptr<float>(), n, (float)r);
  } else if (src.scalar_type() == at::kBFloat16) {
    fold_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>(p1, g2.data_ptr<float>(),
                                                             (const __nv_bfloat16*)src.data_ptr(), n, (float)r);
  } else {
    TS_CHECK(false, "fold: unsupported source dtype");
  }
  TS_LAUNCH_CHECK();
}

void axpby(at::Tensor& out, const at::Tensor& x, const c10::optional<at::Tensor>& y, double a, double b) {
  check_cuda(out, "out");
  check_cuda(x, "x");
  TS_CHECK(out.scalar_type() == at::kFloat && x.scalar_type() == at::kFloat, "axpby operands must be fp32");
  TS_CHECK(out.numel() == x.numel(), "axpby size mismatch");
  const c10::cuda::CUDAGuard guard(out.device());
  const float* py = nullptr;
  if (y) {
    check_cuda(*y, "y");
    TS_CHECK(y->numel() == x.numel() && y->scalar_type() == at::kFloat, "axpby y mismatch");
    py = y->data_ptr<float>();
  }
  if (out.numel() == 0) return;
  axpby_kernel<<<flat_blocks(out.get_device()), 256, 0, stream()>>>(out.data_ptr<float>(), x.data_ptr<float>(), py,
                                                                      out.numel(), (float)a, (float)b);
  TS_LAUNCH_CHECK();
}

void scale(at::Tensor& x, double s) {
  check_cuda(x, "x");
  TS_CHECK(x.scalar_type() == at::kFloat, "scale operand must be fp32");
  const c10::cuda::CUDAGuard guard(x.device());
  if (x.numel() == 0) return;
  scale_kernel<<<flat_blocks(x.get_device()), 256, 0, stream()>>>(x.data_ptr<float>(), x.numel(), (float)s);
  TS_LAUNCH_CHECK();
}

void reduce_into(at::Tensor& out, const std::vector<at::Tensor>& parts) {
  check_cuda(out, "out");
  TS_CHECK(out.scalar_type() == at::kFloat, "reduce target must be fp32");
  TS_CHECK(parts.size() <= 16, "at most 16 parts per reduction");
  if (parts.empty() || out.numel() == 0) return;
  const c10::cuda::CUDAGuard guard(out.device());
  PartList pl{};
  pl.n = (int)parts.size();
  pl.is_bf16 = parts[0].scalar_type() == at::kBFloat16;
  for (size_t i = 0; i < parts.size(); ++i) {
    check_cuda(parts[i], "part");
    TS_CHECK(parts[i].numel() == out.numel(), "part size mismatch");
    TS_CHECK(parts[i].scalar_type() == parts[0].scalar_type(), "parts must share a dtype");
    TS_CHECK(pl.is_bf16 || parts[i].scalar_type() == at::kFloat, "parts must be fp32 or bf16");
    pl.p[i] = parts[i].data_ptr();
  }
  reduce_into_kernel<<<flat_blocks(out.get_device()), 256, 0, stream()>>>(out.data_ptr<float>(), pl, out.numel());
  TS_LAUNCH_CHECK();
}

std::vector<c10::optional<at::Tensor>> lse_gather(const at::Tensor& logits, const at::Tensor& tgt, bool with_entropy) {
  check_cuda(logits, "logits");
  check_cuda(tgt, "target");
  TS_CHECK(logits.scalar_type() == at::kFloat && logits.dim() == 2, "logits must be fp32 [R, V]");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int R = logits.size(0), V = logits.size(1);
  auto lp = at::empty({R}, logits.options());
  auto lse = at::empty({R}, logits.options());
  c10::optional<at::Tensor> ent;
  if (with_entropy) ent = at::empty({R}, logits.options());
  if (R > 0) {
    lse_gather_kernel<<<R, 512, 0, stream()>>>(logits.data_ptr<float>(), tgt.data_ptr<int64_t>(), lp.data_ptr<float>(),
                                               lse.data_ptr<float>(), with_entropy ? ent->data_ptr<float>() : nullptr,
                                               V);
    TS_LAUNCH_CHECK();
  }
  return {lp, lse, ent};
}

at::Tensor logprob_dlogits(const at::Tensor& logits, const at::Tensor& tgt, const at::Tensor& lse,
                           const at::Tensor& g_lp, const c10::optional<at::Tensor>& g_ent,
                           const c10::optional<at::Tensor>& ent, bool out_bf16) {
  check_cuda(logits, "logits");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int R = logits.size(0), V = logits.size(1);
  auto out = at::empty({R, V}, logits.options().dtype(out_bf16 ? at::kBFloat16 : at::kFloat));
  if (R == 0) return out;
  const float* pge = g_ent ? g_ent->data_ptr<float>() : nullptr;
  const float* pent = ent ? ent->data_ptr<float>() : nullptr;
  if (out_bf16) {
    dlogits_kernel<__nv_bfloat16><<<R, 512, 0, stream()>>>(logits.data_ptr<float>(), tgt.data_ptr<int64_t>(),
                                                           lse.data_ptr<float>(), g_lp.data_ptr<float>(), pge, pent,
                                                           (__nv_bfloat16*)out.data_ptr(), V);
  } else {
    dlogits_kernel<float><<<R, 512, 0, stream()>>>(logits.data_ptr<float>(), tgt.data_ptr<int64_t>(),
                                                   lse.data_ptr<float>(), g_lp.data_ptr<float>(), pge, pent,
                                                   out.data_ptr<float>(), V);
  }
  TS_LAUNCH_CHECK();
  return out;
}

}  // namespace ts

TS_BOUNDS_ACCESSOR(bounds_word_fold)
