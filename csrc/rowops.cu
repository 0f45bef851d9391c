// Row-wise memory-bound kernels: RMSNorm (K12'), fused QK-norm + RoPE,
// SwiGLU and the deterministic embedding backward.
//
// All math is fp32; every output is rounded once to the storage dtype. Weight
// gradients are reduced without atomics: each CTA writes a partial row and a
// second kernel sums the partials in CTA order, so results are bitwise
// reproducible run to run.
#include "common.cuh"
#include "common.h"
#include "noalloc.h"
#include "bounds.cuh"

#include <atomic>
#include <cstdint>

namespace ts {
namespace {

constexpr int kSiteEmbeddingId = 1;  // bounds site: embedding backward token id

constexpr int kWarps = 8;

// ----------------------------------------------------------------- RMSNorm fwd
// One warp per row; the row stays in registers (V 16-byte vectors per lane).
template <typename T, int V>
__global__ void __launch_bounds__(kWarps * 32) rms_fwd_kernel(const T* __restrict__ x, const T* __restrict__ w,
                                                              T* __restrict__ y, float* __restrict__ rstd,
                                                              int rows, int H, float eps, int unit) {
  constexpr int E = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const T* xr = x + (size_t)row * H;
  Vec<T> buf[V];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * 32 + lane) * E;
    if (c < H) {
      buf[v] = load_vec(xr + c);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float f = to_f(buf[v].e[e]);
        ss += f * f;
      }
    }
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)H + eps);
  T* yr = y + (size_t)row * H;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * 32 + lane) * E;
    if (c < H) {
      Vec<T> wv = load_vec(w + c);
      Vec<T> o;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if (unit) {  // (1 + w) * x * rstd, one rounding
          o.e[e] = from_f<T>(to_f(buf[v].e[e]) * r * (1.f + to_f(wv.e[e])));
        } else {     // w * round(x * rstd)
          float n = round_to<T>(to_f(buf[v].e[e]) * r);
          o.e[e] = from_f<T>(to_f(wv.e[e]) * n);
        }
      }
      store_vec(yr + c, o);
    }
  }
  if (lane == 0) rstd[row] = r;
}

// ----------------------------------------------------------------- RMSNorm bwd (dx)
template <typename T, int V>
__global__ void __launch_bounds__(kWarps * 32) rms_bwd_dx_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                                 const T* __restrict__ w,
                                                                 const float* __restrict__ rstd,
                                                                 T* __restrict__ dx, int rows, int H, float woff) {
  constexpr int E = Vec<T>::N;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const float r = rstd[row];
  const T* xr = x + (size_t)row * H;
  const T* dyr = dy + (size_t)row * H;
  Vec<T> xb[V], db[V];
  float dot = 0.f;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * 32 + lane) * E;
    if (c < H) {
      xb[v] = load_vec(xr + c);
      db[v] = load_vec(dyr + c);
      Vec<T> wv = load_vec(w + c);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float n = to_f(xb[v].e[e]) * r;
        float dn = to_f(db[v].e[e]) * (to_f(wv.e[e]) + woff);
        dot += dn * n;
      }
    }
  }
  dot = warp_sum(dot) / (float)H;
  T* dxr = dx + (size_t)row * H;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int c = (v * 32 + lane) * E;
    if (c < H) {
      Vec<T> wv = load_vec(w + c);
      Vec<T> o;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        float n = to_f(xb[v].e[e]) * r;
        float dn = to_f(db[v].e[e]) * (to_f(wv.e[e]) + woff);
        o.e[e] = from_f<T>(r * (dn - n * dot));
      }
      store_vec(dxr + c, o);
    }
  }
}

// ----------------------------------------------------------------- RMSNorm bwd (dx + dw partials)
// One pass over dy and x, one row per warp: the warp writes dx (+ dres, the
// residual branch's gradient, added before the single rounding) and stores
// its row's weight-gradient terms dy·x·rstd in its own shared-memory row;
// after one barrier the block's threads add the kWarps rows in warp order and
// the block writes one partial row, which sum_partials_kernel adds up in
// block order. Shared and partial rows use the lane-major order
// p = (v*E + e)*32 + lane for column (v*32 + lane)*E + e, so consecutive
// lanes touch consecutive words. The grid size depends only on the row count,
// so the sums are reproducible run to run. No per-lane accumulators stay live
// across the row, which keeps the kernel near 100 registers (two or more
// blocks per SM; an accumulating form at 163 registers ran one).
template <typename T, int V>
__global__ void __launch_bounds__(kWarps * 32) rms_bwd_fused_kernel(
    const T* __restrict__ dy, const T* __restrict__ x, const T* __restrict__ w, const float* __restrict__ rstd,
    const T* __restrict__ dres, T* __restrict__ dx, float* __restrict__ partial, int rows, int H, float woff) {
  extern __shared__ float red[];  // [kWarps][P]
  constexpr int E = Vec<T>::N;
  constexpr int P = V * 32 * E;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row = blockIdx.x * kWarps + warp;
  float* mine = red + warp * P;
  if (row < rows) {
    const float r = rstd[row];
    const T* xr = x + (size_t)row * H;
    const T* dyr = dy + (size_t)row * H;
    Vec<T> xb[V], db[V];
    float dot = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * 32 + lane) * E;
      if (c < H) {
        xb[v] = load_vec(xr + c);
        db[v] = load_vec(dyr + c);
        Vec<T> wv = load_vec(w + c);
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float n = to_f(xb[v].e[e]) * r;
          const float d = to_f(db[v].e[e]);
          dot += d * (to_f(wv.e[e]) + woff) * n;
          mine[(v * E + e) * 32 + lane] = d * n;
        }
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) mine[(v * E + e) * 32 + lane] = 0.f;
      }
    }
    dot = warp_sum(dot) / (float)H;
    T* dxr = dx + (size_t)row * H;
    const T* rr = dres == nullptr ? nullptr : dres + (size_t)row * H;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c = (v * 32 + lane) * E;
      if (c < H) {
        Vec<T> wv = load_vec(w + c);
        Vec<T> res;
        if (rr != nullptr) res = load_vec(rr + c);
        Vec<T> o;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const float n = to_f(xb[v].e[e]) * r;
          const float dn = to_f(db[v].e[e]) * (to_f(wv.e[e]) + woff);
          float g = r * (dn - n * dot);
          if (rr != nullptr) g += to_f(res.e[e]);
          o.e[e] = from_f<T>(g);
        }
        store_vec(dxr + c, o);
      }
    }
  } else {
    for (int q = lane; q < P; q += 32) mine[q] = 0.f;
  }
  __syncthreads();
  for (int q = threadIdx.x; q < P; q += blockDim.x) {
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < kWarps; ++k) acc += red[k * P + q];
    partial[(size_t)blockIdx.x * P + q] = acc;
  }
}

// ----------------------------------------------------------------- column partial sums
// partial[chunk, c] = sum over the chunk's rows of dy[r, c] * x[r, c] * rstd[r].
// Block = 32 x 8 threads: x-dim walks 16-byte column vectors, y-dim rows.
template <typename T>
__global__ void __launch_bounds__(256) rms_dw_partial_kernel(const T* __restrict__ dy, const T* __restrict__ x,
                                                             const float* __restrict__ rstd,
                                                             float* __restrict__ partial, int rows, int H,
                                                             int rows_per_chunk) {
  constexpr int E = Vec<T>::N;
  __shared__ float red[8][32 * E + 1];
  const int c = (blockIdx.x * 32 + threadIdx.x) * E;
  const int r0 = blockIdx.y * rows_per_chunk;
  const int r1 = min(rows, r0 + rows_per_chunk);
  float acc[E];
#pragma unroll
  for (int e = 0; e < E; ++e) acc[e] = 0.f;
  if (c < H) {
    for (int r = r0 + threadIdx.y; r < r1; r += 8) {
      Vec<T> xv = load_vec(x + (size_t)r * H + c);
      Vec<T> dv = load_vec(dy + (size_t)r * H + c);
      const float rs = rstd[r];
#pragma unroll
      for (int e = 0; e < E; ++e) acc[e] += to_f(dv.e[e]) * (to_f(xv.e[e]) * rs);
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) red[threadIdx.y][threadIdx.x * E + e] = acc[e];
  __syncthreads();
  if (threadIdx.y == 0 && c < H) {
#pragma unroll
    for (int e = 0; e < E; ++e) {
      float s = 0.f;
      for (int k = 0; k < 8; ++k) s += red[k][threadIdx.x * E + e];
      partial[(size_t)blockIdx.y * H + c + e] = s;
    }
  }
}

// out[c] = sum_k partial[k, c]: block (32 x kSumRows) covers 32 columns; warp row y
// sums chunks y, y + kSumRows, ... and the kSumRows row sums are added in y
// order, so the result is the same every run. (32 warps per block: these
// grids have only H / 32 blocks, so the loads in flight per block set the pace.)
// lane_e > 0: partial rows are in the lane-major order of rms_bwd_fused_kernel (row length H, an index
// p there is column ((p / 32) / lane_e * 32 + p % 32) * lane_e + (p / 32) % lane_e; out has `cols` entries).
constexpr int kSumRows = 32;
__global__ void __launch_bounds__(32 * kSumRows) sum_partials_kernel(const float* __restrict__ partial,
                                                                    float* __restrict__ out, int chunks, int H,
                                                                    float scale = 1.f, int accumulate = 0,
                                                                    int lane_e = 0, int cols = 0) {
  __shared__ float red[kSumRows][33];
  const int p = blockIdx.x * 32 + threadIdx.x;
  int c = p;
  if (lane_e > 0) {
    const int ve = p >> 5;
    c = ((ve / lane_e) * 32 + (p & 31)) * lane_e + ve % lane_e;
  }
  float s = 0.f;
  if (p < H)
    for (int k = threadIdx.y; k < chunks; k += kSumRows) s += partial[(size_t)k * H + p];
  red[threadIdx.y][threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.y == 0 && p < H && (lane_e == 0 || c < cols)) {
    float t = 0.f;
#pragma unroll
    for (int y = 0; y < kSumRows; ++y) t += red[y][threadIdx.x];
    out[c] = accumulate ? out[c] + scale * t : t;  // accumulate: into a gradient sink, scaled
  }
}

template <typename T, int V>
void launch_rms_fwd(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, float eps, int unit) {
  const int rows = x.size(0), H = x.size(1);
  dim3 grid((rows + kWarps - 1) / kWarps);
  rms_fwd_kernel<T, V><<<grid, kWarps * 32, 0, stream()>>>(
      (const T*)x.data_ptr(), (const T*)w.data_ptr(), (T*)y.data_ptr(), rstd.data_ptr<float>(), rows, H, eps, unit);
}

template <typename T, int V>
void launch_rms_dx(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                   at::Tensor& dx, float woff) {
  const int rows = x.size(0), H = x.size(1);
  dim3 grid((rows + kWarps - 1) / kWarps);
  rms_bwd_dx_kernel<T, V><<<grid, kWarps * 32, 0, stream()>>>(
      (const T*)dy.data_ptr(), (const T*)x.data_ptr(), (const T*)w.data_ptr(), rstd.data_ptr<float>(),
      (T*)dx.data_ptr(), rows, H, woff);
}

template <typename T>
at::Tensor column_weight_grad(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& rstd) {
  // dw[c] = sum_r dy[r,c] * x[r,c] * rstd[r], deterministic two-level sum.
  constexpr int E = Vec<T>::N;
  const int rows = x.size(0), H = x.size(1);
  const int col_blocks = (H + 32 * E - 1) / (32 * E);
  const int target = 2 * sm_count(x.get_device());
  int chunks = std::max(1, std::min((rows + 7) / 8, target / std::max(col_blocks, 1)));
  const int rows_per_chunk = (rows + chunks - 1) / chunks;
  chunks = (rows + rows_per_chunk - 1) / rows_per_chunk;
  auto partial = at::empty({std::max(chunks, 1), H}, x.options().dtype(at::kFloat));
  auto dw = at::empty({H}, x.options().dtype(at::kFloat));
  if (rows == 0) return dw.zero_();
  rms_dw_partial_kernel<T><<<dim3(col_blocks, chunks), dim3(32, 8), 0, stream()>>>(
      (const T*)dy.data_ptr(), (const T*)x.data_ptr(), rstd.data_ptr<float>(), partial.data_ptr<float>(), rows, H,
      rows_per_chunk);
  sum_partials_kernel<<<(H + 31) / 32, dim3(32, kSumRows), 0, stream()>>>(partial.data_ptr<float>(), dw.data_ptr<float>(),
                                                                     chunks, H);
  return dw;
}

template <typename T>
void rms_fwd_dispatch(const at::Tensor& x, const at::Tensor& w, at::Tensor& y, at::Tensor& rstd, float eps, int unit) {
  constexpr int E = Vec<T>::N;
  const int H = x.size(1);
  const int nv = (H + 32 * E - 1) / (32 * E);
  if (nv <= 1) launch_rms_fwd<T, 1>(x, w, y, rstd, eps, unit);
  else if (nv <= 2) launch_rms_fwd<T, 2>(x, w, y, rstd, eps, unit);
  else if (nv <= 4) launch_rms_fwd<T, 4>(x, w, y, rstd, eps, unit);
  else if (nv <= 8) launch_rms_fwd<T, 8>(x, w, y, rstd, eps, unit);
  else if (nv <= 12) launch_rms_fwd<T, 12>(x, w, y, rstd, eps, unit);
  else if (nv <= 16) launch_rms_fwd<T, 16>(x, w, y, rstd, eps, unit);
  else TS_CHECK(false, "RMSNorm row width ", H, " is too large");
}

template <typename T, int V>
at::Tensor launch_rms_bwd_fused(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                const at::Tensor& rstd, const T* dres, at::Tensor& dx, float woff,
                                const c10::optional<at::Tensor>& dw_acc, float dw_scale) {
  const int rows = x.size(0), H = x.size(1);
  // one row per warp: enough warps in flight to cover memory latency (a grid capped at one block per SM,
  // with each warp walking many rows, ran twice as long)
  const int grid = std::max(1, (rows + kWarps - 1) / kWarps);
  constexpr int E = Vec<T>::N;
  constexpr int P = V * 32 * E;  // lane-major partial row length
  auto partial = at::empty({grid, P}, x.options().dtype(at::kFloat));
  auto dw = dw_acc ? *dw_acc : at::empty({H}, x.options().dtype(at::kFloat));
  const int smem = kWarps * P * (int)sizeof(float);
  static bool configured[16] = {false};
  bool& done = configured[x.get_device() & 15];
  if (!done) {
    TS_CUDA_CHECK(cudaFuncSetAttribute(rms_bwd_fused_kernel<T, V>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    TS_CUDA_CHECK(cudaFuncSetAttribute(rms_bwd_fused_kernel<T, V>, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       100));
    done = true;
  }
  rms_bwd_fused_kernel<T, V><<<grid, kWarps * 32, smem, stream()>>>(
      (const T*)dy.data_ptr(), (const T*)x.data_ptr(), (const T*)w.data_ptr(), rstd.data_ptr<float>(), dres,
      (T*)dx.data_ptr(), partial.data_ptr<float>(), rows, H, woff);
  sum_partials_kernel<<<(P + 31) / 32, dim3(32, kSumRows), 0, stream()>>>(partial.data_ptr<float>(), dw.data_ptr<float>(),
                                                                     grid, P, dw_scale, dw_acc ? 1 : 0, E, H);
  return dw;
}

// dx (+ dres) and dw in two launches for rows up to 8 vectors per lane; empty tensor otherwise.
template <typename T>
at::Tensor rms_bwd_fused_dispatch(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                  const at::Tensor& rstd, const T* dres, at::Tensor& dx, float woff,
                                  const c10::optional<at::Tensor>& acc, float sc) {
  constexpr int E = Vec<T>::N;
  const int H = x.size(1);
  const int nv = (H + 32 * E - 1) / (32 * E);
  if (nv <= 1) return launch_rms_bwd_fused<T, 1>(dy, x, w, rstd, dres, dx, woff, acc, sc);
  if (nv <= 2) return launch_rms_bwd_fused<T, 2>(dy, x, w, rstd, dres, dx, woff, acc, sc);
  if (nv <= 4) return launch_rms_bwd_fused<T, 4>(dy, x, w, rstd, dres, dx, woff, acc, sc);
  if (nv <= 8) return launch_rms_bwd_fused<T, 8>(dy, x, w, rstd, dres, dx, woff, acc, sc);
  return at::Tensor();
}

template <typename T>
void rms_dx_dispatch(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w, const at::Tensor& rstd,
                     at::Tensor& dx, float woff) {
  constexpr int E = Vec<T>::N;
  const int H = x.size(1);
  const int nv = (H + 32 * E - 1) / (32 * E);
  if (nv <= 1) launch_rms_dx<T, 1>(dy, x, w, rstd, dx, woff);
  else if (nv <= 2) launch_rms_dx<T, 2>(dy, x, w, rstd, dx, woff);
  else if (nv <= 4) launch_rms_dx<T, 4>(dy, x, w, rstd, dx, woff);
  else if (nv <= 8) launch_rms_dx<T, 8>(dy, x, w, rstd, dx, woff);
  else if (nv <= 12) launch_rms_dx<T, 12>(dy, x, w, rstd, dx, woff);
  else if (nv <= 16) launch_rms_dx<T, 16>(dy, x, w, rstd, dx, woff);
  else TS_CHECK(false, "RMSNorm row width ", H, " is too large");
}

// ----------------------------------------------------------------- QK-norm + RoPE
// One warp per (token, head) row of q or k; lane owns EPL = D/32 consecutive
// elements, so the rotate-half partner (element i +- D/2) lives on lane ^ 16.
// EPL consecutive elements of one lane as one vector access (8 bytes for 4 bf16 at head_dim 128)
template <typename T, int EPL>
TS_DEVICE void load_lane(const T* __restrict__ p, float (&out)[EPL]) {
  if constexpr (sizeof(T) * EPL == 8) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = to_f(e[i]);
  } else if constexpr (sizeof(T) * EPL == 16) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = to_f(e[i]);
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = to_f(p[i]);
  }
}
template <typename T, int EPL>
TS_DEVICE void store_lane(T* __restrict__ p, const float (&in)[EPL]) {
  if constexpr (sizeof(T) * EPL == 8) {
    uint2 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < EPL; ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint2*>(p) = u;
  } else if constexpr (sizeof(T) * EPL == 16) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < EPL; ++i) e[i] = from_f<T>(in[i]);
    *reinterpret_cast<uint4*>(p) = u;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) p[i] = from_f<T>(in[i]);
  }
}
template <int EPL>
TS_DEVICE void load_f32_lane(const float* __restrict__ p, float (&out)[EPL]) {
  if constexpr (EPL == 4) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    out[0] = u.x; out[1] = u.y; out[2] = u.z; out[3] = u.w;
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) out[i] = p[i];
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_fwd_kernel(
    const T* __restrict__ qkv, const T* __restrict__ qw, const T* __restrict__ kw, const int64_t* __restrict__ pos,
    const float* __restrict__ inv_freq, const float* __restrict__ cos_tab, const float* __restrict__ sin_tab,
    int tab_len, T* __restrict__ q, T* __restrict__ k, T* __restrict__ v, int tokens, int hq,
    int hkv, float eps, int unit, int rot_lanes) {
  constexpr int EPL = D / 32;
  const int lane = threadIdx.x & 31;
  const int heads = hq + 2 * hkv;
  const long long item = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (item >= (long long)tokens * heads) return;
  const int t = (int)(item / heads);
  const int h = (int)(item % heads);
  const T* src = qkv + (size_t)t * heads * D + (size_t)h * D + lane * EPL;
  float xv[EPL];
  load_lane<T, EPL>(src, xv);
  if (h >= hq + hkv) {  // value head: plain copy
    store_lane<T, EPL>(v + ((size_t)t * hkv + (h - hq - hkv)) * D + lane * EPL, xv);
    return;
  }
  const bool is_q = h < hq;
  const T* wt = is_q ? qw : kw;
  float y[EPL];
  if (wt != nullptr) {
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) ss += xv[e] * xv[e];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + eps);
    float wv[EPL];
    load_lane<T, EPL>(wt + lane * EPL, wv);
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      y[e] = unit ? round_to<T>(xv[e] * r * (1.f + wv[e])) : round_to<T>(wv[e] * round_to<T>(xv[e] * r));
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) y[e] = xv[e];
  }
  const int64_t pi = pos[t];
  const float p = (float)pi;
  const int nfreq = rot_lanes * EPL / 2;
  const bool tab = pi >= 0 && pi < tab_len;
  T* dst = is_q ? q + ((size_t)t * hq + h) * D + lane * EPL : k + ((size_t)t * hkv + (h - hq)) * D + lane * EPL;
  // rotary over the first rot_lanes * EPL dims; the rotate-half partner of an
  // element sits half_mask lanes away; the remaining dims pass through
  const int half_mask = rot_lanes >> 1;
  const bool rotary = lane < rot_lanes;
  const bool low = (lane & half_mask) == 0;
  const int f0 = (lane & (half_mask - 1)) * EPL;  // first frequency index of this lane
  float cs[EPL], sn[EPL];
  if (rotary && tab) {  // cos/sin of the fp32 angle, precomputed per (position, frequency)
    load_f32_lane<EPL>(cos_tab + pi * nfreq + f0, cs);
    load_f32_lane<EPL>(sin_tab + pi * nfreq + f0, sn);
  } else if (rotary) {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      float s_, c_;
      sincosf(p * inv_freq[f0 + e], &s_, &c_);
      sn[e] = s_;
      cs[e] = c_;
    }
  }
  float out[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[e], half_mask);
    out[e] = rotary ? y[e] * cs[e] + (low ? -partner : partner) * sn[e] : y[e];
  }
  store_lane<T, EPL>(dst, out);
}

template <typename T, int D>
__global__ void __launch_bounds__(kWarps * 32) qk_norm_rope_bwd_kernel(
    const T* __restrict__ dq, const T* __restrict__ dk, const T* __restrict__ dv, const T* __restrict__ qkv,
    const T* __restrict__ qw, const T* __restrict__ kw, const int64_t* __restrict__ pos,
    const float* __restrict__ inv_freq, const float* __restrict__ cos_tab, const float* __restrict__ sin_tab,
    int tab_len, T* __restrict__ dqkv, float* __restrict__ dqw_part,
    float* __restrict__ dkw_part, int tokens, int hq, int hkv, float eps, int items_per_block, int unit, int rot_lanes,
    int part_stride) {
  constexpr int EPL = D / 32;
  __shared__ float red_q[kWarps][D];
  __shared__ float red_k[kWarps][D];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int heads = hq + 2 * hkv;
  float aq[EPL], ak[EPL];
#pragma unroll
  for (int e = 0; e < EPL; ++e) aq[e] = ak[e] = 0.f;
  const long long total = (long long)tokens * heads;
  const long long i0 = (long long)blockIdx.x * items_per_block;
  const long long i1 = i0 + items_per_block < total ? i0 + items_per_block : total;
  for (long long item = i0 + warp; item < i1; item += kWarps) {
    const int t = (int)(item / heads);
    const int h = (int)(item % heads);
    T* out = dqkv + (size_t)t * heads * D + (size_t)h * D + lane * EPL;
    if (h >= hq + hkv) {
      float gv[EPL];
      load_lane<T, EPL>(dv + ((size_t)t * hkv + (h - hq - hkv)) * D + lane * EPL, gv);
      store_lane<T, EPL>(out, gv);
      continue;
    }
    const bool is_q = h < hq;
    const T* g = is_q ? dq + ((size_t)t * hq + h) * D + lane * EPL : dk + ((size_t)t * hkv + (h - hq)) * D + lane * EPL;
    const T* src = qkv + (size_t)t * heads * D + (size_t)h * D + lane * EPL;
    const int64_t pi = pos[t];
    const float p = (float)pi;
    const int nfreq = rot_lanes * EPL / 2;
    const bool tab = pi >= 0 && pi < tab_len;
    const int half_mask = rot_lanes >> 1;
    const bool rotary = lane < rot_lanes;
    const bool low = (lane & half_mask) == 0;
    const T* wt = is_q ? qw : kw;
    // all of this row's loads issue together: the gradient, the input row, the norm weight, cos/sin
    float go[EPL], xv[EPL], wv[EPL], cs[EPL], sn[EPL];
    load_lane<T, EPL>(g, go);
    if (wt != nullptr) {
      load_lane<T, EPL>(src, xv);
      load_lane<T, EPL>(wt + lane * EPL, wv);
    }
    const int f0 = (lane & (half_mask - 1)) * EPL;
    if (rotary && tab) {
      load_f32_lane<EPL>(cos_tab + pi * nfreq + f0, cs);
      load_f32_lane<EPL>(sin_tab + pi * nfreq + f0, sn);
    } else if (rotary) {
#pragma unroll
      for (int e = 0; e < EPL; ++e) {
        float s_, c_;
        sincosf(p * inv_freq[f0 + e], &s_, &c_);
        sn[e] = s_;
        cs[e] = c_;
      }
    }
    float dy[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, go[e], half_mask);
      // d/dy_i of sum_j go_j * (y_j c_j + rot(y)_j s_j)
      dy[e] = rotary ? go[e] * cs[e] + (low ? partner : -partner) * sn[e] : go[e];
    }
    if (wt == nullptr) {
      store_lane<T, EPL>(out, dy);
      continue;
    }
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) ss += xv[e] * xv[e];
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + eps);
    float dot = 0.f;
    float dn[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float n = xv[e] * r;
      dn[e] = dy[e] * (wv[e] + (unit ? 1.f : 0.f));
      dot += dn[e] * n;
      if (is_q) aq[e] += dy[e] * n; else ak[e] += dy[e] * n;
    }
    dot = warp_sum(dot) / (float)D;
    float res[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) res[e] = r * (dn[e] - xv[e] * r * dot);
    store_lane<T, EPL>(out, res);
  }
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    red_q[warp][lane * EPL + e] = aq[e];
    red_k[warp][lane * EPL + e] = ak[e];
  }
  __syncthreads();
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float sq = 0.f, sk = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      sq += red_q[w][c];
      sk += red_k[w][c];
    }
    dqw_part[(size_t)blockIdx.x * part_stride + c] = sq;
    dkw_part[(size_t)blockIdx.x * part_stride + c] = sk;
  }
}

// ----------------------------------------------------------------- SwiGLU
template <typename T>
__global__ void swiglu_fwd_kernel(const T* __restrict__ gu, T* __restrict__ a, long long rows, int F) {
  constexpr int E = Vec<T>::N;
  const long long n_vec = rows * (F / E);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_vec; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (F / E);
    const int c = (int)(i % (F / E)) * E;
    Vec<T> g = load_vec(gu + r * 2 * F + c);
    Vec<T> u = load_vec(gu + r * 2 * F + F + c);
    Vec<T> o;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float gf = to_f(g.e[e]);
      const float sg = 1.f / (1.f + expf(-gf));
      o.e[e] = from_f<T>(gf * sg * to_f(u.e[e]));
    }
    store_vec(a + r * F + c, o);
  }
}

template <typename T>
__global__ void swiglu_bwd_kernel(const T* __restrict__ da, const T* __restrict__ gu, T* __restrict__ dgu,
                                  long long rows, int F) {
  constexpr int E = Vec<T>::N;
  const long long n_vec = rows * (F / E);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n_vec; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / (F / E);
    const int c = (int)(i % (F / E)) * E;
    Vec<T> g = load_vec(gu + r * 2 * F + c);
    Vec<T> u = load_vec(gu + r * 2 * F + F + c);
    Vec<T> d = load_vec(da + r * F + c);
    Vec<T> og, ou;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float gf = to_f(g.e[e]);
      const float uf = to_f(u.e[e]);
      const float df = to_f(d.e[e]);
      const float sg = 1.f / (1.f + expf(-gf));
      og.e[e] = from_f<T>(df * uf * (sg * (1.f + gf * (1.f - sg))));
      ou.e[e] = from_f<T>(df * gf * sg);
    }
    store_vec(dgu + r * 2 * F + c, og);
    store_vec(dgu + r * 2 * F + F + c, ou);
  }
}

// ----------------------------------------------------------------- embedding backward
// ids sorted ascending (with their source rows); the block at the first
// position of each run of equal ids sums that run's rows in order and adds
// scale * sum into target[id]. No two blocks touch the same target row.
template <typename T>
__global__ void embedding_bwd_kernel(const int64_t* __restrict__ sorted_ids, const int64_t* __restrict__ order,
                                     const T* __restrict__ dy, float* __restrict__ target, int n, int D, float scale,
                                     int64_t vocab) {
  const int i = blockIdx.x;
  if (i >= n) return;
  const int64_t id = sorted_ids[i];
  TS_BOUND(id >= 0 && id < vocab, kSiteEmbeddingId, id);  // a token id outside the embedding table
  if (i > 0 && sorted_ids[i - 1] == id) return;
  int j_end = i + 1;
  while (j_end < n && sorted_ids[j_end] == id) ++j_end;
  for (int c = threadIdx.x; c < D; c += blockDim.x) {
    float s = 0.f;
    for (int j = i; j < j_end; ++j) s += to_f(dy[(size_t)order[j] * D + c]);
    target[(size_t)id * D + c] += scale * s;
  }
}

}  // namespace

// =================================================================== host API
std::vector<at::Tensor> rms_norm_fwd(const at::Tensor& x, const at::Tensor& w, double eps, bool unit) {
  check_cuda(x, "x");
  check_cuda(w, "w");
  TS_CHECK(x.dim() == 2 && w.dim() == 1 && w.size(0) == x.size(1), "rms_norm_fwd shapes");
  TS_CHECK(x.scalar_type() == w.scalar_type(), "rms_norm_fwd: x and w dtype differ");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = at::empty_like(x);
  auto rstd = at::empty({x.size(0)}, x.options().dtype(at::kFloat));
  if (x.size(0) == 0) return {y, rstd};
  const int H = x.size(1);
  if (x.scalar_type() == at::kBFloat16) {
    TS_CHECK(H % 8 == 0, "row width must be a multiple of 8");
    rms_fwd_dispatch<__nv_bfloat16>(x, w, y, rstd, (float)eps, unit ? 1 : 0);
  } else if (x.scalar_type() == at::kFloat) {
    TS_CHECK(H % 4 == 0, "row width must be a multiple of 4");
    rms_fwd_dispatch<float>(x, w, y, rstd, (float)eps, unit ? 1 : 0);
  } else {
    TS_CHECK(false, "rms_norm_fwd: unsupported dtype");
  }
  TS_LAUNCH_CHECK();
  return {y, rstd};
}

// dres (optional): gradient of a residual branch added to dx before its rounding.
// dw_acc (optional, fp32 [H]): the weight gradient is added into it (times dw_scale) and returned.
std::vector<at::Tensor> rms_norm_bwd(const at::Tensor& dy, const at::Tensor& x, const at::Tensor& w,
                                     const at::Tensor& rstd, bool unit, const c10::optional<at::Tensor>& dres,
                                     const c10::optional<at::Tensor>& dw_acc, double dw_scale) {
  check_cuda(dy, "dy");
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  auto dx = at::empty_like(x);
  at::Tensor dw;
  const int H = x.size(1);
  if (dres) {
    TS_CHECK(dres->is_contiguous() && dres->sizes() == x.sizes() && dres->scalar_type() == x.scalar_type(),
             "rms_norm_bwd: dres must be a contiguous tensor shaped and typed like x");
  }
  if (dw_acc) {
    TS_CHECK(dw_acc->scalar_type() == at::kFloat && dw_acc->is_contiguous() && dw_acc->numel() == H,
             "rms_norm_bwd: dw_acc must be a contiguous fp32 tensor of the row width");
  }
  const float sc = (float)dw_scale;
  if (x.size(0) == 0) return {dx, dw_acc ? *dw_acc : at::zeros({H}, x.options().dtype(at::kFloat))};
  if (x.scalar_type() == at::kBFloat16) {
    TS_CHECK(H % 8 == 0, "row width must be a multiple of 8");
    using T = __nv_bfloat16;
    dw = rms_bwd_fused_dispatch<T>(dy, x, w, rstd, dres ? (const T*)dres->data_ptr() : nullptr, dx,
                                   unit ? 1.f : 0.f, dw_acc, sc);
    if (!dw.defined()) {
      rms_dx_dispatch<T>(dy, x, w, rstd, dx, unit ? 1.f : 0.f);
      dw = column_weight_grad<T>(dy, x, rstd);
      if (dres) dx.add_(*dres);
      if (dw_acc) dw = dw_acc->add_(dw, sc);
    }
  } else if (x.scalar_type() == at::kFloat) {
    TS_CHECK(H % 4 == 0, "row width must be a multiple of 4");
    dw = rms_bwd_fused_dispatch<float>(dy, x, w, rstd, dres ? dres->data_ptr<float>() : nullptr, dx,
                                       unit ? 1.f : 0.f, dw_acc, sc);
    if (!dw.defined()) {
      rms_dx_dispatch<float>(dy, x, w, rstd, dx, unit ? 1.f : 0.f);
      dw = column_weight_grad<float>(dy, x, rstd);
      if (dres) dx.add_(*dres);
      if (dw_acc) dw = dw_acc->add_(dw, sc);
    }
  } else {
    TS_CHECK(false, "rms_norm_bwd: unsupported dtype");
  }
  TS_LAUNCH_CHECK();
  return {dx, dw};
}

template <typename T, int D>
static void qk_fwd_launch(const at::Tensor& qkv, const c10::optional<at::Tensor>& qw,
                          const c10::optional<at::Tensor>& kw, const at::Tensor& pos, const at::Tensor& inv_freq,
                          at::Tensor& q, at::Tensor& k, at::Tensor& v, int hq, int hkv, float eps, int unit,
                          int rot_lanes, const float* ct, const float* st, int tl) {
  const int tokens = qkv.size(0);
  const long long items = (long long)tokens * (hq + 2 * hkv);
  const int blocks = (int)((items + kWarps - 1) / kWarps);
  qk_norm_rope_fwd_kernel<T, D><<<blocks, kWarps * 32, 0, stream()>>>(
      (const T*)qkv.data_ptr(), qw ? (const T*)qw->data_ptr() : nullptr, kw ? (const T*)kw->data_ptr() : nullptr,
      pos.data_ptr<int64_t>(), inv_freq.data_ptr<float>(), ct, st, tl, (T*)q.data_ptr(), (T*)k.data_ptr(),
      (T*)v.data_ptr(), tokens, hq, hkv, eps, unit, rot_lanes);
}

#define TS_DISPATCH_HEAD(D, FN, T, ...)                                \
  do {                                                                 \
    if ((D) == 64) FN<T, 64>(__VA_ARGS__);                             \
    else if ((D) == 128) FN<T, 128>(__VA_ARGS__);                      \
    else if ((D) == 256) FN<T, 256>(__VA_ARGS__);                      \
    else TS_CHECK(false, "head_dim ", D, " unsupported (64/128/256)"); \
  } while (0)

std::vector<at::Tensor> qk_norm_rope_fwd(const at::Tensor& qkv, const c10::optional<at::Tensor>& qw,
                                         const c10::optional<at::Tensor>& kw, const at::Tensor& pos,
                                         const at::Tensor& inv_freq, int64_t hq, int64_t hkv, int64_t d,
                                         double eps, bool unit, const c10::optional<at::Tensor>& cos_tab,
                                         const c10::optional<at::Tensor>& sin_tab,
                                         const c10::optional<at::Tensor>& k_out,
                                         const c10::optional<at::Tensor>& v_out) {
  const float* ct = cos_tab ? cos_tab->data_ptr<float>() : nullptr;
  const float* st = sin_tab ? sin_tab->data_ptr<float>() : nullptr;
  const int tl = cos_tab ? (int)cos_tab->size(0) : 0;
  TS_CHECK(!cos_tab || (sin_tab && cos_tab->is_contiguous() && sin_tab->is_contiguous() &&
                        cos_tab->size(1) == inv_freq.numel() && sin_tab->sizes() == cos_tab->sizes() &&
                        cos_tab->scalar_type() == at::kFloat),
           "rope tables must be fp32 [positions, rotary_dim / 2] cos and sin");
  check_cuda(qkv, "qkv");
  const int epl = (int)d / 32;
  const int rot_lanes = (int)(2 * inv_freq.numel()) / epl;
  TS_CHECK(2 * inv_freq.numel() <= d && (2 * inv_freq.numel()) % (2 * epl) == 0 && rot_lanes >= 2 &&
               (rot_lanes & (rot_lanes - 1)) == 0,
           "rotary dims must be a power-of-two multiple of 2 * head_dim / 32");
  TS_CHECK(qkv.dim() == 2 && qkv.size(1) == (hq + 2 * hkv) * d, "qkv shape");
  TS_CHECK(pos.scalar_type() == at::kLong && inv_freq.scalar_type() == at::kFloat, "pos/inv_freq dtype");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int64_t t = qkv.size(0);
  auto q = at::empty({t, hq, d}, qkv.options());
  // k_out / v_out: contiguous [t, hkv, d] destinations (rows of a key/value buffer that also holds ancestors)
  for (const auto* o : {&k_out, &v_out}) {
    if (*o) {
      TS_CHECK((*o)->is_contiguous() && (*o)->dim() == 3 && (*o)->size(0) == t && (*o)->size(1) == hkv &&
                   (*o)->size(2) == d && (*o)->scalar_type() == qkv.scalar_type() && (*o)->device() == qkv.device(),
               "qk_norm_rope_fwd: k_out / v_out must be contiguous [t, hkv, d] tensors like qkv");
    }
  }
  auto k = k_out ? *k_out : at::empty({t, hkv, d}, qkv.options());
  auto v = v_out ? *v_out : at::empty({t, hkv, d}, qkv.options());
  if (t == 0) return {q, k, v};
  if (qkv.scalar_type() == at::kBFloat16) {
    TS_DISPATCH_HEAD(d, qk_fwd_launch, __nv_bfloat16, qkv, qw, kw, pos, inv_freq, q, k, v, hq, hkv, (float)eps,
                     unit ? 1 : 0, rot_lanes, ct, st, tl);
  } else if (qkv.scalar_type() == at::kFloat) {
    TS_DISPATCH_HEAD(d, qk_fwd_launch, float, qkv, qw, kw, pos, inv_freq, q, k, v, hq, hkv, (float)eps, unit ? 1 : 0,
                     rot_lanes, ct, st, tl);
  } else {
    TS_CHECK(false, "qk_norm_rope_fwd: unsupported dtype");
  }
  TS_LAUNCH_CHECK();
  return {q, k, v};
}

template <typename T, int D>
static void qk_bwd_launch(const at::Tensor& dq, const at::Tensor& dk, const at::Tensor& dv, const at::Tensor& qkv,
                          const c10::optional<at::Tensor>& qw, const c10::optional<at::Tensor>& kw,
                          const at::Tensor& pos, const at::Tensor& inv_freq, at::Tensor& dqkv, at::Tensor& pqk,
                          int hq, int hkv, float eps, int blocks, int per_block, int unit,
                          int rot_lanes, const float* ct, const float* st, int tl) {
  qk_norm_rope_bwd_kernel<T, D><<<blocks, kWarps * 32, 0, stream()>>>(
      (const T*)dq.data_ptr(), (const T*)dk.data_ptr(), (const T*)dv.data_ptr(), (const T*)qkv.data_ptr(),
      qw ? (const T*)qw->data_ptr() : nullptr, kw ? (const T*)kw->data_ptr() : nullptr, pos.data_ptr<int64_t>(),
      inv_freq.data_ptr<float>(), ct, st, tl, (T*)dqkv.data_ptr(), pqk.data_ptr<float>(), pqk.data_ptr<float>() + D,
      qkv.size(0), hq, hkv, eps, per_block, unit, rot_lanes, 2 * D);
}

std::vector<c10::optional<at::Tensor>> qk_norm_rope_bwd(const at::Tensor& dq, const at::Tensor& dk,
                                                        const at::Tensor& dv, const at::Tensor& qkv,
                                                        const c10::optional<at::Tensor>& qw,
                                                        const c10::optional<at::Tensor>& kw, const at::Tensor& pos,
                                                        const at::Tensor& inv_freq, int64_t hq, int64_t hkv,
                                                        int64_t d, double eps, bool unit,
                                                        const c10::optional<at::Tensor>& cos_tab,
                                                        const c10::optional<at::Tensor>& sin_tab,
                                                        const c10::optional<at::Tensor>& dqw_acc,
                                                        const c10::optional<at::Tensor>& dkw_acc, double dw_scale) {
  check_cuda(qkv, "qkv");
  const float* ct = cos_tab ? cos_tab->data_ptr<float>() : nullptr;
  const float* st = sin_tab ? sin_tab->data_ptr<float>() : nullptr;
  const int tl = cos_tab ? (int)cos_tab->size(0) : 0;
  const int rot_lanes = (int)(2 * inv_freq.numel()) / ((int)d / 32);
  check_cuda(dq, "dq");
  check_cuda(dk, "dk");
  check_cuda(dv, "dv");
  const c10::cuda::CUDAGuard guard(qkv.device());
  const int64_t t = qkv.size(0);
  auto dqkv = at::empty_like(qkv);
  const long long items = (long long)t * (hq + 2 * hkv);
  const int target = 4 * sm_count(qkv.get_device());
  int per_block = (int)std::max<long long>(kWarps, (items + target - 1) / target);
  int blocks = (int)std::max<long long>(1, (items + per_block - 1) / per_block);
  // every block writes its whole partial row: [q-norm weight | k-norm weight] partials side by side
  auto pqk = at::empty({blocks, 2 * d}, qkv.options().dtype(at::kFloat));
  if (t > 0) {
    if (qkv.scalar_type() == at::kBFloat16) {
      TS_DISPATCH_HEAD(d, qk_bwd_launch, __nv_bfloat16, dq, dk, dv, qkv, qw, kw, pos, inv_freq, dqkv, pqk, hq, hkv,
                       (float)eps, blocks, per_block, unit ? 1 : 0, rot_lanes, ct, st, tl);
    } else if (qkv.scalar_type() == at::kFloat) {
      TS_DISPATCH_HEAD(d, qk_bwd_launch, float, dq, dk, dv, qkv, qw, kw, pos, inv_freq, dqkv, pqk, hq, hkv,
                       (float)eps, blocks, per_block, unit ? 1 : 0, rot_lanes, ct, st, tl);
    } else {
      TS_CHECK(false, "qk_norm_rope_bwd: unsupported dtype");
    }
    TS_LAUNCH_CHECK();
  }
  c10::optional<at::Tensor> dqw, dkw;
  if (qw) {
    if (t == 0) pqk.zero_();
    for (const auto* acc : {&dqw_acc, &dkw_acc}) {
      if (*acc) {
        TS_CHECK((*acc)->scalar_type() == at::kFloat && (*acc)->is_contiguous() && (*acc)->numel() == d,
                 "qk_norm_rope_bwd: weight-gradient targets must be contiguous fp32 tensors of the head size");
      }
    }
    at::Tensor oq, ok;
    const bool adjacent = dqw_acc && dkw_acc && dkw_acc->data_ptr<float>() == dqw_acc->data_ptr<float>() + d;
    if (adjacent || (!dqw_acc && !dkw_acc)) {
      // one reduction over both weights (sink targets that sit back to back, or fresh outputs)
      at::Tensor both = adjacent ? at::from_blob(dqw_acc->data_ptr<float>(), {2 * d}, dqw_acc->options())
                                 : at::empty({2 * d}, qkv.options().dtype(at::kFloat));
      sum_partials_kernel<<<(2 * d + 31) / 32, dim3(32, kSumRows), 0, stream()>>>(
          pqk.data_ptr<float>(), both.data_ptr<float>(), blocks, 2 * d, (float)dw_scale, adjacent ? 1 : 0);
      oq = adjacent ? *dqw_acc : both.narrow(0, 0, d);
      ok = adjacent ? *dkw_acc : both.narrow(0, d, d);
    } else {
      auto pq = pqk.narrow(1, 0, d).contiguous();
      auto pk = pqk.narrow(1, d, d).contiguous();
      oq = dqw_acc ? *dqw_acc : at::empty({d}, qkv.options().dtype(at::kFloat));
      ok = dkw_acc ? *dkw_acc : at::empty({d}, qkv.options().dtype(at::kFloat));
      sum_partials_kernel<<<(d + 31) / 32, dim3(32, kSumRows), 0, stream()>>>(pq.data_ptr<float>(), oq.data_ptr<float>(),
                                                                      blocks, d, (float)dw_scale, dqw_acc ? 1 : 0);
      sum_partials_kernel<<<(d + 31) / 32, dim3(32, kSumRows), 0, stream()>>>(pk.data_ptr<float>(), ok.data_ptr<float>(),
                                                                      blocks, d, (float)dw_scale, dkw_acc ? 1 : 0);
    }
    TS_LAUNCH_CHECK();
    dqw = oq;
    dkw = ok;
  }
  return {dqkv, dqw, dkw};
}

at::Tensor swiglu_fwd(const at::Tensor& gu) {
  check_cuda(gu, "gu");
  const c10::cuda::CUDAGuard guard(gu.device());
  const long long rows = gu.numel() / gu.size(-1);
  const int F = gu.size(-1) / 2;
  auto sizes = gu.sizes().vec();
  sizes.back() = F;
  auto a = at::empty(sizes, gu.options());
  if (rows == 0) return a;
  const int blocks = 4 * sm_count(gu.get_device());
  if (gu.scalar_type() == at::kBFloat16) {
    TS_CHECK(F % 8 == 0, "ffn width must be a multiple of 8");
    swiglu_fwd_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>((const __nv_bfloat16*)gu.data_ptr(),
                                                                     (__nv_bfloat16*)a.data_ptr(), rows, F);
  } else if (gu.scalar_type() == at::kFloat) {
    TS_CHECK(F % 4 == 0, "ffn width must be a multiple of 4");
    swiglu_fwd_kernel<float><<<blocks, 256, 0, stream()>>>((const float*)gu.data_ptr(), (float*)a.data_ptr(), rows, F);
  } else {
    TS_CHECK(false, "swiglu_fwd: unsupported dtype");
  }
  TS_LAUNCH_CHECK();
  return a;
}

at::Tensor swiglu_bwd(const at::Tensor& da, const at::Tensor& gu) {
  check_cuda(gu, "gu");
  check_cuda(da, "da");
  const c10::cuda::CUDAGuard guard(gu.device());
  const long long rows = gu.numel() / gu.size(-1);
  const int F = gu.size(-1) / 2;
  auto dgu = at::empty_like(gu);
  if (rows == 0) return dgu;
  const int blocks = 4 * sm_count(gu.get_device());
  if (gu.scalar_type() == at::kBFloat16) {
    swiglu_bwd_kernel<__nv_bfloat16><<<blocks, 256, 0, stream()>>>(
        (const __nv_bfloat16*)da.data_ptr(), (const __nv_bfloat16*)gu.data_ptr(), (__nv_bfloat16*)dgu.data_ptr(), rows, F);
  } else if (gu.scalar_type() == at::kFloat) {
    swiglu_bwd_kernel<float><<<blocks, 256, 0, stream()>>>((const float*)da.data_ptr(), (const float*)gu.data_ptr(),
                                                           (float*)dgu.data_ptr(), rows, F);
  } else {
    TS_CHECK(false, "swiglu_bwd: unsupported dtype");
  }
  TS_LAUNCH_CHECK();
  return dgu;
}

void embedding_bwd_accumulate(at::Tensor& target, const at::Tensor& ids, const at::Tensor& dy, double scale) {
  check_cuda(target, "target");
  check_cuda(ids, "ids");
  check_cuda(dy, "dy");
  TS_CHECK(target.scalar_type() == at::kFloat, "embedding gradient target must be fp32");
  const c10::cuda::CUDAGuard guard(dy.device());
  const int n = ids.size(0);
  if (n == 0) return;
  const int D = dy.size(1);
  auto sorted = at::sort(ids, /*stable=*/true, /*dim=*/0, /*descending=*/false);
  auto sid = std::get<0>(sorted).contiguous();
  auto order = std::get<1>(sorted).contiguous();
  const int threads = D >= 1024 ? 512 : 256;
  if (dy.scalar_type() == at::kBFloat16) {
    embedding_bwd_kernel<__nv_bfloat16><<<n, threads, 0, stream()>>>(
        sid.data_ptr<int64_t>(), order.data_ptr<int64_t>(), (const __nv_bfloat16*)dy.data_ptr(),
        target.data_ptr<float>(), n, D, (float)scale, target.size(0));
  } else if (dy.scalar_type() == at::kFloat) {
    embedding_bwd_kernel<float><<<n, threads, 0, stream()>>>(sid.data_ptr<int64_t>(), order.data_ptr<int64_t>(),
                                                            (const float*)dy.data_ptr(), target.data_ptr<float>(), n,
                                                            D, (float)scale, target.size(0));
  } else {
    TS_CHECK(false, "embedding_bwd: unsupported dtype");
  }
  TS_LAUNCH_CHECK();
}

}  // namespace ts

// =================================================================== allocation-free entry point
// ts_rms_norm_bwd_noalloc (declared in noalloc.h) runs the same three kernels
// as rms_norm_bwd, but its per-chunk weight-gradient partials live in the
// file-scope array below instead of a caching-allocator buffer.
//
// * The array is a fixed 2 MiB (TS_NOALLOC_RMS_MAX_CHUNKS x
//   TS_NOALLOC_RMS_MAX_COLS_BF16 floats); every GPU that loads this library holds
//   it until the process exits.
// * Host code cannot pass the array's name to a kernel (on the host it is only
//   a stand-in symbol), so the first call on each device, with that device
//   current, looks up its device address with cudaGetSymbolAddress and caches
//   it. Make that first call before any stream capture.
// * Every call shares the one array and the last call's contents stay in it.
//   Each call writes every partial it later reads, so nothing has to start at
//   zero; calls whose kernels overlap on the GPU (different streams without
//   ordering) race on the array and must be serialised by the caller.
// * No cudaMalloc, cudaFree or allocating library routine is called.
namespace ts {
namespace {

static __device__ __align__(256) float g_noalloc_rms_partial[TS_NOALLOC_RMS_MAX_CHUNKS * TS_NOALLOC_RMS_MAX_COLS_BF16];

std::atomic<float*> g_noalloc_rms_ptr[64];
thread_local char g_noalloc_msg[256] = "";

int noalloc_fail(int code, const char* msg) {
  snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "%s", msg);
  return code;
}

template <typename T, int V>
void noalloc_dx(const T* dy, const T* x, const T* w, const float* rstd, T* dx, int rows, int H, cudaStream_t st) {
  rms_bwd_dx_kernel<T, V><<<(rows + kWarps - 1) / kWarps, kWarps * 32, 0, st>>>(dy, x, w, rstd, dx, rows, H, 0.f);
}

// No error was pending when the entry point started (it checks), so an error
// seen right after a launch belongs to that launch.
int noalloc_launch_status(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return 0;
  char buf[200];
  snprintf(buf, sizeof(buf), "ts_rms_norm_bwd_noalloc: %s launch failed: %s", what, cudaGetErrorString(e));
  return noalloc_fail(5, buf);
}

template <typename T>
int noalloc_run(const T* dy, const T* x, const T* w, const float* rstd, T* dx, float* dw, int rows, int H,
                float* partial, int device, cudaStream_t st) {
  constexpr int E = Vec<T>::N;
  const int nv = (H + 32 * E - 1) / (32 * E);
  if (nv <= 1) noalloc_dx<T, 1>(dy, x, w, rstd, dx, rows, H, st);
  else if (nv <= 2) noalloc_dx<T, 2>(dy, x, w, rstd, dx, rows, H, st);
  else if (nv <= 4) noalloc_dx<T, 4>(dy, x, w, rstd, dx, rows, H, st);
  else if (nv <= 8) noalloc_dx<T, 8>(dy, x, w, rstd, dx, rows, H, st);
  else if (nv <= 12) noalloc_dx<T, 12>(dy, x, w, rstd, dx, rows, H, st);
  else if (nv <= 16) noalloc_dx<T, 16>(dy, x, w, rstd, dx, rows, H, st);
  else return noalloc_fail(3, "ts_rms_norm_bwd_noalloc: row width too large for the register path");
  if (int rc = noalloc_launch_status("dx")) return rc;
  const int col_blocks = (H + 32 * E - 1) / (32 * E);
  const int target = 2 * sm_count(device);
  int chunks = std::max(1, std::min((rows + 7) / 8, target / std::max(col_blocks, 1)));
  chunks = std::min(chunks, TS_NOALLOC_RMS_MAX_CHUNKS);
  const int rows_per_chunk = (rows + chunks - 1) / chunks;
  chunks = (rows + rows_per_chunk - 1) / rows_per_chunk;
  rms_dw_partial_kernel<T><<<dim3(col_blocks, chunks), dim3(32, 8), 0, st>>>(dy, x, rstd, partial, rows, H,
                                                                            rows_per_chunk);
  if (int rc = noalloc_launch_status("weight-gradient partials")) return rc;
  sum_partials_kernel<<<(H + 31) / 32, dim3(32, kSumRows), 0, st>>>(partial, dw, chunks, H);
  return noalloc_launch_status("weight-gradient sum");
}

}  // namespace
}  // namespace ts

extern "C" __attribute__((visibility("default"))) const char* ts_noalloc_last_error(void) {
  return ts::g_noalloc_msg;
}

extern "C" __attribute__((visibility("default"))) int ts_rms_norm_bwd_noalloc(const void* dy, const void* x,
                                                                            const void* w, const float* rstd,
                                                                            void* dx, float* dw, int rows, int cols,
                                                                            int dtype, void* stream) {
  using namespace ts;
  g_noalloc_msg[0] = '\0';
  if (rows < 0 || cols <= 0) return noalloc_fail(1, "ts_rms_norm_bwd_noalloc: rows must be >= 0 and cols > 0");
  if (dtype != 0 && dtype != 1) return noalloc_fail(1, "ts_rms_norm_bwd_noalloc: dtype must be 0 (bf16) or 1 (fp32)");
  const int max_cols = dtype == 0 ? TS_NOALLOC_RMS_MAX_COLS_BF16 : TS_NOALLOC_RMS_MAX_COLS_FP32;
  if (cols > max_cols) {
    char buf[160];
    snprintf(buf, sizeof(buf), "ts_rms_norm_bwd_noalloc: cols=%d exceeds the limit of %d columns for %s", cols,
             max_cols, dtype == 0 ? "bf16" : "fp32");
    return noalloc_fail(2, buf);
  }
  if ((dtype == 0 && cols % 8) || (dtype == 1 && cols % 4))
    return noalloc_fail(1, "ts_rms_norm_bwd_noalloc: cols must be a multiple of 8 (bf16) or 4 (fp32)");
  // dw is always written; the row operands only when there are rows. The
  // kernels move rows in 16-byte vectors, so those pointers must be 16-byte
  // aligned (an offset view of a tensor may not be).
  auto misaligned = [](const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) != 0; };
  if (dw == nullptr || misaligned(dw, 4)) return noalloc_fail(1, "ts_rms_norm_bwd_noalloc: dw is null or not 4-byte aligned");
  if (rows > 0) {
    if (!dy || !x || !w || !dx || !rstd)
      return noalloc_fail(1, "ts_rms_norm_bwd_noalloc: dy, x, w, rstd and dx must not be null");
    if (misaligned(dy, 16) || misaligned(x, 16) || misaligned(w, 16) || misaligned(dx, 16))
      return noalloc_fail(1, "ts_rms_norm_bwd_noalloc: dy, x, w and dx must be 16-byte aligned");
    if (misaligned(rstd, 4)) return noalloc_fail(1, "ts_rms_norm_bwd_noalloc: rstd must be 4-byte aligned");
  }
  {
    // an error left by earlier work on this thread would otherwise be
    // reported (and cleared) as if one of this call's launches had failed
    const cudaError_t pending = cudaPeekAtLastError();
    if (pending != cudaSuccess) {
      char buf[200];
      snprintf(buf, sizeof(buf), "ts_rms_norm_bwd_noalloc: a CUDA error from earlier work is pending: %s",
               cudaGetErrorString(pending));
      return noalloc_fail(6, buf);
    }
  }
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64)
    return noalloc_fail(4, "ts_rms_norm_bwd_noalloc: no current CUDA device");
  float* scratch = g_noalloc_rms_ptr[device].load(std::memory_order_acquire);
  if (scratch == nullptr) {
    // once per device, with that device current: the array's device address.
    // Threads that race here all store the same address.
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_rms_partial);
    if (e != cudaSuccess || p == nullptr) return noalloc_fail(4, cudaGetErrorString(e));
    scratch = static_cast<float*>(p);
    g_noalloc_rms_ptr[device].store(scratch, std::memory_order_release);
  }
  if (rows == 0) {
    return cudaMemsetAsync(dw, 0, sizeof(float) * cols, static_cast<cudaStream_t>(stream)) == cudaSuccess
               ? 0
               : noalloc_fail(5, "ts_rms_norm_bwd_noalloc: clearing dw failed");
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == 0)
    return noalloc_run<__nv_bfloat16>((const __nv_bfloat16*)dy, (const __nv_bfloat16*)x, (const __nv_bfloat16*)w,
                                      rstd, (__nv_bfloat16*)dx, dw, rows, cols, scratch, device, st);
  return noalloc_run<float>((const float*)dy, (const float*)x, (const float*)w, rstd, (float*)dx, dw, rows, cols,
                            scratch, device, st);
}

TS_BOUNDS_ACCESSOR(bounds_word_rowops)
