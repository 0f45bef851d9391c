// Gated DeltaNet sequence mixing (K08', K09').
//
// conv1d_silu : causal depthwise conv over [tail; x] (width K) + SiLU, and the
//               new tail; backward gives dx, the tail's gradient and a
//               deterministic weight gradient (per-chunk partials summed in
//               chunk order).
// gdn         : the gated delta rule per head, exact recurrence in fp32:
//                 S <- exp(g_t) S;  d = beta_t (v_t - S^T k_t);  S <- S + k_t d^T;
//                 o_t = S^T q_t
//               with q, k L2-normalised (eps 1e-6) and q scaled by dk^-1/2.
//               One CTA per head; 512 threads hold the dk x dv fp32 state as
//               8x4 register tiles (16 row tiles x 32 column tiles). The
//               per-token reductions over rows (S^T k, S^T q) and over
//               columns (S do for the backward) go through shared memory.
//               The forward stores the state every kCk tokens; the backward
//               walks chunks in reverse, recomputes each chunk's per-token
//               states into a global scratch (L2-resident), and runs the
//               adjoint recurrence
//                 dS += q do^T;  a = k^T dS;  dv = beta a;
//                 dq = S_t do;   dk = dS d - beta e^g S_{t-1} a;
//                 dbeta = a . (v - e^g k^T S_{t-1});  dg = <S_t - beta k v^T, dS>;
//                 dS <- e^g (dS - beta k a^T)
//               then the L2-norm backward for q and k.
#include "common.cuh"
#include "common.h"

namespace ts {
namespace {

typedef __nv_bfloat16 bf16;

// ------------------------------------------------------------------ conv1d
// Row r of the padded input [tail; x] (r in [0, T+K-1)) is tail row r for
// r < K-1, else x row r-K+1. Output t reads padded rows t..t+K-1.
// Each thread owns two adjacent channels of one row chunk and walks the rows
// with a sliding window, so every input row is read once per chunk (plus a
// K-1 row halo) and all loads/stores are coalesced bf16x2 across channels.
constexpr int kConvRows = 64;

struct Pad {
  const bf16* x;
  const bf16* tail;
  int C, K;
  __device__ __forceinline__ float2 at(int r, int c) const {
    const __nv_bfloat162 v = r < K - 1 ? *reinterpret_cast<const __nv_bfloat162*>(tail + (long long)r * C + c)
                                       : *reinterpret_cast<const __nv_bfloat162*>(x + (long long)(r - K + 1) * C + c);
    return __bfloat1622float2(v);
  }
};

TS_DEVICE float silu_of(float a) { return a / (1.f + expf(-a)); }
TS_DEVICE float dsilu_of(float a) {
  const float s = 1.f / (1.f + expf(-a));
  return s * (1.f + a * (1.f - s));
}

template <int K>
__global__ void conv1d_fwd_kernel(const bf16* __restrict__ x, const bf16* __restrict__ w, const bf16* __restrict__ tail,
                                  bf16* __restrict__ y, bf16* __restrict__ new_tail, int T, int C) {
  const int c = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= C) return;
  const Pad in{x, tail, C, K};
  float w0[K], w1[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    w0[j] = __bfloat162float(w[c * K + j]);
    w1[j] = __bfloat162float(w[(c + 1) * K + j]);
  }
  const int t0 = blockIdx.y * kConvRows, t1 = min(T, t0 + kConvRows);
  float2 win[K];
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = t0 + j < T + K - 1 ? in.at(t0 + j, c) : make_float2(0.f, 0.f);
  for (int t = t0; t < t1; ++t) {
    win[K - 1] = in.at(t + K - 1, c);
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      a0 += w0[j] * win[j].x;
      a1 += w1[j] * win[j].y;
    }
    *reinterpret_cast<__nv_bfloat162*>(y + (long long)t * C + c) = __floats2bfloat162_rn(silu_of(a0), silu_of(a1));
#pragma unroll
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
  if (blockIdx.y == gridDim.y - 1) {  // the last K-1 padded rows become the new tail
    for (int r = 0; r < K - 1; ++r) {
      const float2 v = in.at(T + r, c);
      *reinterpret_cast<__nv_bfloat162*>(new_tail + (long long)r * C + c) = __floats2bfloat162_rn(v.x, v.y);
    }
  }
}

// One pass per (channel pair, row chunk): dpre[t] = dy[t] * silu'(pre[t]);
// d(pad)[r] = sum_j w[j] dpre[r-j] (+ the new tail's gradient for r >= T);
// dw partial[chunk][c][j] = sum_t dpre[t] * pad[t+j] over the chunk's t.
template <int K>
__global__ void conv1d_bwd_kernel(const bf16* __restrict__ dy, const bf16* __restrict__ dtail_out,
                                  const bf16* __restrict__ x, const bf16* __restrict__ w,
                                  const bf16* __restrict__ tail, bf16* __restrict__ dx, bf16* __restrict__ dtail,
                                  float* __restrict__ partial, int T, int C) {
  const int c = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (c >= C) return;
  const Pad in{x, tail, C, K};
  const int R = T + K - 1;
  float w0[K], w1[K], g0[K], g1[K];
#pragma unroll
  for (int j = 0; j < K; ++j) {
    w0[j] = __bfloat162float(w[c * K + j]);
    w1[j] = __bfloat162float(w[(c + 1) * K + j]);
    g0[j] = g1[j] = 0.f;
  }
  // padded rows owned by this chunk: [r0, r1); the last chunk also owns the tail rows >= T
  const int r0 = blockIdx.y * kConvRows;
  const int r1 = blockIdx.y == gridDim.y - 1 ? R : min(R, r0 + kConvRows);
  auto dpre_at = [&](int t, float2& v, float2 (&pw)[K]) {
    // pw: padded rows t..t+K-1
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      a0 += w0[j] * pw[j].x;
      a1 += w1[j] * pw[j].y;
    }
    const float2 d = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dy + (long long)t * C + c));
    v = make_float2(d.x * dsilu_of(a0), d.y * dsilu_of(a1));
  };
  // dq[k] holds dpre[r - k] for the current r (k = 0..K-1), zero outside [0, T)
  float2 dq[K];
  float2 win[K];  // padded rows r .. r+K-1
#pragma unroll
  for (int k = 0; k < K; ++k) dq[k] = make_float2(0.f, 0.f);
  // warm-up: dpre[r0-K+1 .. r0-1] into dq[K-1 .. 1]
  for (int k = K - 1; k >= 1; --k) {
    const int t = r0 - k;
    if (t >= 0 && t < T) {
      float2 pw[K];
#pragma unroll
      for (int j = 0; j < K; ++j) pw[j] = in.at(t + j, c);
      dpre_at(t, dq[k], pw);
    }
  }
#pragma unroll
  for (int j = 0; j < K - 1; ++j) win[j] = r0 + j < R ? in.at(r0 + j, c) : make_float2(0.f, 0.f);
  for (int r = r0; r < r1; ++r) {
    win[K - 1] = r + K - 1 < R ? in.at(r + K - 1, c) : make_float2(0.f, 0.f);
    float2 cur = make_float2(0.f, 0.f);
    if (r < T) {
      dpre_at(r, cur, win);
#pragma unroll
      for (int j = 0; j < K; ++j) {
        g0[j] += cur.x * win[j].x;
        g1[j] += cur.y * win[j].y;
      }
    }
    dq[0] = cur;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < K; ++j) {
      s0 += w0[j] * dq[j].x;
      s1 += w1[j] * dq[j].y;
    }
    if (r >= T) {
      const float2 d = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(dtail_out + (long long)(r - T) * C + c));
      s0 += d.x;
      s1 += d.y;
    }
    __nv_bfloat162* dst = r < K - 1 ? reinterpret_cast<__nv_bfloat162*>(dtail + (long long)r * C + c)
                                    : reinterpret_cast<__nv_bfloat162*>(dx + (long long)(r - K + 1) * C + c);
    *dst = __floats2bfloat162_rn(s0, s1);
#pragma unroll
    for (int k = K - 1; k >= 1; --k) dq[k] = dq[k - 1];
#pragma unroll
    for (int j = 0; j < K - 1; ++j) win[j] = win[j + 1];
  }
#pragma unroll
  for (int j = 0; j < K; ++j) {
    partial[((long long)blockIdx.y * C + c) * K + j] = g0[j];
    partial[((long long)blockIdx.y * C + c + 1) * K + j] = g1[j];
  }
}

__global__ void conv1d_dw_sum_kernel(const float* __restrict__ partial, float* __restrict__ dw, int chunks, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  float s = 0.f;
  for (int k = 0; k < chunks; ++k) s += partial[(long long)k * n + i];
  dw[i] = s;
}

// ------------------------------------------------------------------ gated delta rule
constexpr int kDk = 128, kDv = 128;
constexpr int kThreads = 512;       // 16 row tiles x 32 column tiles
constexpr int kTR = 8, kTC = 4;     // state tile per thread: 8 rows x 4 columns
constexpr int kCk = 64;             // checkpoint interval (tokens)

// q, k -> L2-normalised fp32 (q also scaled), one warp per (t, h) row of 128
__global__ void gdn_prep_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k, float* __restrict__ qn,
                                float* __restrict__ kn, float* __restrict__ rq, float* __restrict__ rk, long long rows,
                                float qscale) {
  const long long row = blockIdx.x * 8ll + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float a[4], b[4], sa = 0.f, sb = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    a[e] = __bfloat162float(q[row * kDk + lane * 4 + e]);
    b[e] = __bfloat162float(k[row * kDk + lane * 4 + e]);
    sa += a[e] * a[e];
    sb += b[e] * b[e];
  }
  sa = warp_sum(sa);
  sb = warp_sum(sb);
  const float ia = rsqrtf(sa + 1e-6f), ib = rsqrtf(sb + 1e-6f);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    qn[row * kDk + lane * 4 + e] = a[e] * ia * qscale;
    kn[row * kDk + lane * 4 + e] = b[e] * ib;
  }
  if (lane == 0) {
    rq[row] = ia;
    rk[row] = ib;
  }
}

// dq (bf16) from dqn (grad wrt normalised, scaled q): x_hat = x * r; dx = r (dxh - x_hat (x_hat . dxh))
__global__ void gdn_prep_bwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                    const float* __restrict__ dqn, const float* __restrict__ dkn,
                                    const float* __restrict__ rq, const float* __restrict__ rk, bf16* __restrict__ dq,
                                    bf16* __restrict__ dk, long long rows, float qscale) {
  const long long row = blockIdx.x * 8ll + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float ia = rq[row], ib = rk[row];
  float xa[4], xb[4], ga[4], gb[4], da = 0.f, db = 0.f;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    xa[e] = __bfloat162float(q[row * kDk + lane * 4 + e]) * ia;
    xb[e] = __bfloat162float(k[row * kDk + lane * 4 + e]) * ib;
    ga[e] = dqn[row * kDk + lane * 4 + e] * qscale;
    gb[e] = dkn[row * kDk + lane * 4 + e];
    da += xa[e] * ga[e];
    db += xb[e] * gb[e];
  }
  da = warp_sum(da);
  db = warp_sum(db);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    dq[row * kDk + lane * 4 + e] = __float2bfloat16_rn(ia * (ga[e] - xa[e] * da));
    dk[row * kDk + lane * 4 + e] = __float2bfloat16_rn(ib * (gb[e] - xb[e] * db));
  }
}

struct GdnSmem {
  float red[16][kDv];   // per-row-tile partial column sums (16 x 128)
  float colv[2][kDv];   // reduced column vectors
  float rowv[2][kDk];   // reduced row vectors
  float red2[32][kDk];  // per-column-tile partial row sums
  float scal[32];
};

// Block reduction over rows: each thread holds partials for its 4 columns; out[c] over all 128 columns.
TS_DEVICE void reduce_rows(GdnSmem& sm, const float (&part)[kTC], int rt, int ct, float* out) {
#pragma unroll
  for (int c = 0; c < kTC; ++c) sm.red[rt][ct * kTC + c] = part[c];
  __syncthreads();
  if (threadIdx.x < kDv) {
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < 16; ++r) s += sm.red[r][threadIdx.x];
    out[threadIdx.x] = s;
  }
  __syncthreads();
}

// Block reduction over columns: each thread holds partials for its 8 rows; out[r] over all 128 rows.
TS_DEVICE void reduce_cols(GdnSmem& sm, const float (&part)[kTR], int rt, int ct, float* out) {
#pragma unroll
  for (int r = 0; r < kTR; ++r) sm.red2[ct][rt * kTR + r] = part[r];
  __syncthreads();
  if (threadIdx.x < kDk) {
    float s = 0.f;
#pragma unroll 8
    for (int c = 0; c < 32; ++c) s += sm.red2[c][threadIdx.x];
    out[threadIdx.x] = s;
  }
  __syncthreads();
}

TS_DEVICE float block_sum(GdnSmem& sm, float v) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sm.scal[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < kThreads / 32; ++i) s += sm.scal[i];
  __syncthreads();
  return s;
}

// Forward: one CTA per head. ckpt[c] = state before token c*kCk; ckpt[n_ck] = final.
__global__ void __launch_bounds__(kThreads, 1) gdn_fwd_kernel(const float* __restrict__ qn, const float* __restrict__ kn,
                                                              const bf16* __restrict__ v, const float* __restrict__ g,
                                                              const float* __restrict__ beta,
                                                              const float* __restrict__ s0, bf16* __restrict__ o,
                                                              float* __restrict__ ckpt, int T, int H) {
  __shared__ GdnSmem sm;
  const int h = blockIdx.x;
  const int rt = threadIdx.x >> 5, ct = threadIdx.x & 31;  // row tile (warp), column tile (lane)
  const int r0 = rt * kTR, c0 = ct * kTC;
  const int n_ck = (T + kCk - 1) / kCk;
  float s[kTR][kTC];
#pragma unroll
  for (int i = 0; i < kTR; ++i)
#pragma unroll
    for (int j = 0; j < kTC; ++j) s[i][j] = s0[((long long)h * kDk + r0 + i) * kDv + c0 + j];
  for (int t = 0; t < T; ++t) {
    if (t % kCk == 0) {
      float* ck = ckpt + ((long long)(t / kCk) * H + h) * kDk * kDv;
#pragma unroll
      for (int i = 0; i < kTR; ++i)
#pragma unroll
        for (int j = 0; j < kTC; ++j) ck[(r0 + i) * kDv + c0 + j] = s[i][j];
    }
    const long long th = (long long)t * H + h;
    const float e = expf(g[th]);
    const float b = beta[th];
    float kr[kTR], qr[kTR];
#pragma unroll
    for (int i = 0; i < kTR; ++i) {
      kr[i] = kn[th * kDk + r0 + i];
      qr[i] = qn[th * kDk + r0 + i];
    }
    float part[kTC];
#pragma unroll
    for (int j = 0; j < kTC; ++j) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < kTR; ++i) {
        s[i][j] *= e;
        a += s[i][j] * kr[i];
      }
      part[j] = a;
    }
    reduce_rows(sm, part, rt, ct, sm.colv[0]);  // kv[j] = k^T S
    float dlt[kTC];
#pragma unroll
    for (int j = 0; j < kTC; ++j) dlt[j] = b * (__bfloat162float(v[th * kDv + c0 + j]) - sm.colv[0][c0 + j]);
#pragma unroll
    for (int j = 0; j < kTC; ++j) {
      float a = 0.f;
#pragma unroll
      for (int i = 0; i < kTR; ++i) {
        s[i][j] += kr[i] * dlt[j];
        a += s[i][j] * qr[i];
      }
      part[j] = a;
    }
    reduce_rows(sm, part, rt, ct, sm.colv[1]);  // o[j] = q^T S
    if (threadIdx.x < kDv) o[th * kDv + threadIdx.x] = __float2bfloat16_rn(sm.colv[1][threadIdx.x]);
  }
  float* ck = ckpt + ((long long)n_ck * H + h) * kDk * kDv;
#pragma unroll
  for (int i = 0; i < kTR; ++i)
#pragma unroll
    for (int j = 0; j < kTC; ++j) ck[(r0 + i) * kDv + c0 + j] = s[i][j];
}

// Backward: reverse over chunks; per chunk recompute the states S_{t-1} and the
// deltas into scratch, then the adjoint sweep.
__global__ void __launch_bounds__(kThreads, 1) gdn_bwd_kernel(
    const float* __restrict__ qn, const float* __restrict__ kn, const bf16* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, const float* __restrict__ ckpt, const bf16* __restrict__ dout,
    const float* __restrict__ dfinal, float* __restrict__ scratch, float* __restrict__ dqn, float* __restrict__ dkn,
    bf16* __restrict__ dv, float* __restrict__ dg, float* __restrict__ dbeta, float* __restrict__ ds0, int T, int H) {
  __shared__ GdnSmem sm;
  extern __shared__ float4 gdn_dyn[];  // [kCk][kDv] deltas, then [kCk][kDv] k^T S'
  float (*sdelta)[kDv] = reinterpret_cast<float (*)[kDv]>(gdn_dyn);
  float (*skv)[kDv] = reinterpret_cast<float (*)[kDv]>(reinterpret_cast<float*>(gdn_dyn) + kCk * kDv);
  const int h = blockIdx.x;
  const int rt = threadIdx.x >> 5, ct = threadIdx.x & 31;
  const int r0 = rt * kTR, c0 = ct * kTC;
  const int n_ck = (T + kCk - 1) / kCk;
  float* scr = scratch + (long long)h * kCk * kDk * kDv;  // [kCk][dk][dv] states before each token
  float ds[kTR][kTC];
#pragma unroll
  for (int i = 0; i < kTR; ++i)
#pragma unroll
    for (int j = 0; j < kTC; ++j) ds[i][j] = dfinal[((long long)h * kDk + r0 + i) * kDv + c0 + j];
  for (int c = n_ck - 1; c >= 0; --c) {
    const int t0 = c * kCk, t1 = min(T, t0 + kCk);
    // recompute the chunk forward, saving S_{t-1}, k^T S_{t-1} (after decay) and deltas
    float s[kTR][kTC];
    const float* ck = ckpt + ((long long)c * H + h) * kDk * kDv;
#pragma unroll
    for (int i = 0; i < kTR; ++i)
#pragma unroll
      for (int j = 0; j < kTC; ++j) s[i][j] = ck[(r0 + i) * kDv + c0 + j];
    for (int t = t0; t < t1; ++t) {
      float* st = scr + (long long)(t - t0) * kDk * kDv;
#pragma unroll
      for (int i = 0; i < kTR; ++i)
#pragma unroll
        for (int j = 0; j < kTC; ++j) st[(r0 + i) * kDv + c0 + j] = s[i][j];
      const long long th = (long long)t * H + h;
      const float e = expf(g[th]);
      const float b = beta[th];
      float kr[kTR];
#pragma unroll
      for (int i = 0; i < kTR; ++i) kr[i] = kn[th * kDk + r0 + i];
      float part[kTC];
#pragma unroll
      for (int j = 0; j < kTC; ++j) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < kTR; ++i) {
          s[i][j] *= e;
          a += s[i][j] * kr[i];
        }
        part[j] = a;
      }
      reduce_rows(sm, part, rt, ct, sm.colv[0]);
      if (threadIdx.x < kDv) {
        const float kvj = sm.colv[0][threadIdx.x];
        skv[t - t0][threadIdx.x] = kvj;
        sdelta[t - t0][threadIdx.x] = b * (__bfloat162float(v[th * kDv + threadIdx.x]) - kvj);
      }
      __syncthreads();
#pragma unroll
      for (int j = 0; j < kTC; ++j)
#pragma unroll
        for (int i = 0; i < kTR; ++i) s[i][j] += kr[i] * sdelta[t - t0][c0 + j];
    }
    __syncthreads();
    // adjoint sweep, last token first
    for (int t = t1 - 1; t >= t0; --t) {
      const long long th = (long long)t * H + h;
      const float e = expf(g[th]);
      const float b = beta[th];
      const float* st = scr + (long long)(t - t0) * kDk * kDv;
      float kr[kTR], qr[kTR], dor[kTC], dl[kTC], vr[kTC];
#pragma unroll
      for (int i = 0; i < kTR; ++i) {
        kr[i] = kn[th * kDk + r0 + i];
        qr[i] = qn[th * kDk + r0 + i];
      }
#pragma unroll
      for (int j = 0; j < kTC; ++j) {
        dor[j] = __bfloat162float(dout[th * kDv + c0 + j]);
        dl[j] = sdelta[t - t0][c0 + j];
        vr[j] = __bfloat162float(v[th * kDv + c0 + j]);
      }
      // S_t = e S_{t-1} + k d^T ; dS += q do^T ; a = k^T dS
      float sp[kTR][kTC], stt[kTR][kTC];
      float part[kTC];
#pragma unroll
      for (int j = 0; j < kTC; ++j) {
        float a = 0.f;
#pragma unroll
        for (int i = 0; i < kTR; ++i) {
          sp[i][j] = st[(r0 + i) * kDv + c0 + j];
          stt[i][j] = e * sp[i][j] + kr[i] * dl[j];
          ds[i][j] += qr[i] * dor[j];
          a += kr[i] * ds[i][j];
        }
        part[j] = a;
      }
      reduce_rows(sm, part, rt, ct, sm.colv[0]);  // a[j]
      float aj[kTC];
#pragma unroll
      for (int j = 0; j < kTC; ++j) aj[j] = sm.colv[0][c0 + j];
      if (threadIdx.x < kDv) dv[th * kDv + threadIdx.x] = __float2bfloat16_rn(b * sm.colv[0][threadIdx.x]);
      // dq = S_t do ; dk = dS d - b e S_{t-1} a   (column reductions)
      float pq[kTR], pk[kTR];
      float gpart = 0.f, bpart = 0.f;
#pragma unroll
      for (int i = 0; i < kTR; ++i) {
        float aq = 0.f, ak = 0.f;
#pragma unroll
        for (int j = 0; j < kTC; ++j) {
          aq += stt[i][j] * dor[j];
          ak += ds[i][j] * dl[j] - b * e * sp[i][j] * aj[j];
          gpart += (stt[i][j] - b * kr[i] * vr[j]) * ds[i][j];
        }
        pq[i] = aq;
        pk[i] = ak;
      }
      if (rt == 0) {
#pragma unroll
        for (int j = 0; j < kTC; ++j) bpart += aj[j] * (vr[j] - skv[t - t0][c0 + j]);
      }
      reduce_cols(sm, pq, rt, ct, sm.rowv[0]);
      if (threadIdx.x < kDk) dqn[th * kDk + threadIdx.x] = sm.rowv[0][threadIdx.x];
      reduce_cols(sm, pk, rt, ct, sm.rowv[1]);
      if (threadIdx.x < kDk) dkn[th * kDk + threadIdx.x] = sm.rowv[1][threadIdx.x];
      const float gs = block_sum(sm, gpart);
      const float bs = block_sum(sm, bpart);
      if (threadIdx.x == 0) {
        dg[th] = gs;
        dbeta[th] = bs;
      }
      // dS_{t-1} = e (dS - b k a^T)
#pragma unroll
      for (int i = 0; i < kTR; ++i)
#pragma unroll
        for (int j = 0; j < kTC; ++j) ds[i][j] = e * (ds[i][j] - b * kr[i] * aj[j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kTR; ++i)
#pragma unroll
    for (int j = 0; j < kTC; ++j) ds0[((long long)h * kDk + r0 + i) * kDv + c0 + j] = ds[i][j];
}

}  // namespace

std::vector<at::Tensor> conv1d_silu_fwd(const at::Tensor& x, const at::Tensor& w, const at::Tensor& tail) {
  check_cuda(x, "x");
  check_cuda(w, "w");
  check_cuda(tail, "tail");
  TS_CHECK(x.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && tail.scalar_type() == at::kBFloat16,
           "conv1d runs in bf16");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = x.size(0), C = x.size(1), K = w.size(1);
  TS_CHECK(K == 4, "conv1d kernel width 4 supported");
  TS_CHECK(C % 2 == 0, "conv1d needs an even channel count");
  auto y = at::empty_like(x);
  auto nt = at::empty({K - 1, C}, x.options());
  const int threads = 128;
  const dim3 grid((C / 2 + threads - 1) / threads, std::max(1, (T + kConvRows - 1) / kConvRows));
  conv1d_fwd_kernel<4><<<grid, threads, 0, stream()>>>((const bf16*)x.data_ptr(), (const bf16*)w.data_ptr(),
                                                       (const bf16*)tail.data_ptr(), (bf16*)y.data_ptr(),
                                                       (bf16*)nt.data_ptr(), T, C);
  TS_LAUNCH_CHECK();
  return {y, nt};
}

std::vector<at::Tensor> conv1d_silu_bwd(const at::Tensor& dy, const at::Tensor& dtail_out, const at::Tensor& x,
                                        const at::Tensor& w, const at::Tensor& tail) {
  check_cuda(dy, "dy");
  check_cuda(dtail_out, "dtail_out");
  check_cuda(x, "x");
  const c10::cuda::CUDAGuard guard(x.device());
  const int T = x.size(0), C = x.size(1), K = w.size(1);
  TS_CHECK(K == 4 && C % 2 == 0, "conv1d backward supports width 4 and even channel counts");
  auto dx = at::empty_like(x);
  auto dtail = at::empty_like(tail);
  const int R = T + K - 1;
  const int chunks = std::max(1, (R + kConvRows - 1) / kConvRows);
  auto partial = at::empty({chunks, C, K}, x.options().dtype(at::kFloat));
  auto dw = at::empty({C, K}, x.options().dtype(at::kFloat));
  const int threads = 128;
  conv1d_bwd_kernel<4><<<dim3((C / 2 + threads - 1) / threads, chunks), threads, 0, stream()>>>(
      (const bf16*)dy.data_ptr(), (const bf16*)dtail_out.data_ptr(), (const bf16*)x.data_ptr(),
      (const bf16*)w.data_ptr(), (const bf16*)tail.data_ptr(), (bf16*)dx.data_ptr(), (bf16*)dtail.data_ptr(),
      partial.data_ptr<float>(), T, C);
  conv1d_dw_sum_kernel<<<(C * K + 255) / 256, 256, 0, stream()>>>(partial.data_ptr<float>(), dw.data_ptr<float>(),
                                                                   chunks, C * K);
  TS_LAUNCH_CHECK();
  return {dx, dw, dtail};
}

std::vector<at::Tensor> gdn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                const at::Tensor& beta, const at::Tensor& state) {
  check_cuda(q, "q");
  check_cuda(k, "k");
  check_cuda(v, "v");
  check_cuda(g, "g");
  check_cuda(beta, "beta");
  check_cuda(state, "state");
  TS_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
           "gated delta rule takes bf16 q/k/v");
  TS_CHECK(g.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat && state.scalar_type() == at::kFloat,
           "gated delta rule takes fp32 g/beta/state");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T = q.size(0), H = q.size(1);
  TS_CHECK(q.size(2) == kDk && v.size(2) == kDv, "gated delta rule kernel supports head dims 128/128");
  const int n_ck = (T + kCk - 1) / kCk;
  auto o = at::empty_like(v);
  auto ckpt = at::empty({n_ck + 1, H, kDk, kDv}, q.options().dtype(at::kFloat));
  auto qn = at::empty({T, H, kDk}, q.options().dtype(at::kFloat));
  auto kn = at::empty({T, H, kDk}, q.options().dtype(at::kFloat));
  auto rq = at::empty({T, H}, q.options().dtype(at::kFloat));
  auto rk = at::empty({T, H}, q.options().dtype(at::kFloat));
  const long long rows = (long long)T * H;
  if (rows > 0)
    gdn_prep_kernel<<<(int)((rows + 7) / 8), 256, 0, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(),
                                                                 qn.data_ptr<float>(), kn.data_ptr<float>(),
                                                                 rq.data_ptr<float>(), rk.data_ptr<float>(), rows,
                                                                 1.f / sqrtf((float)kDk));
  gdn_fwd_kernel<<<H, kThreads, 0, stream()>>>(qn.data_ptr<float>(), kn.data_ptr<float>(), (const bf16*)v.data_ptr(),
                                               g.data_ptr<float>(), beta.data_ptr<float>(), state.data_ptr<float>(),
                                               (bf16*)o.data_ptr(), ckpt.data_ptr<float>(), T, H);
  TS_LAUNCH_CHECK();
  auto final_state = ckpt[n_ck].clone();
  // saved for the backward: checkpoints, normalised q/k and the norms
  auto saved = at::cat({ckpt.flatten(), qn.flatten(), kn.flatten(), rq.flatten(), rk.flatten()});
  return {o, final_state, saved};
}

std::vector<at::Tensor> gdn_bwd(const at::Tensor& dout, const at::Tensor& dfinal, const at::Tensor& q,
                                const at::Tensor& k, const at::Tensor& v, const at::Tensor& g, const at::Tensor& beta,
                                const at::Tensor& saved) {
  check_cuda(dout, "dout");
  check_cuda(dfinal, "dfinal");
  check_cuda(saved, "saved");
  const c10::cuda::CUDAGuard guard(q.device());
  const int T = q.size(0), H = q.size(1);
  const int n_ck = (T + kCk - 1) / kCk;
  const long long nck = (long long)(n_ck + 1) * H * kDk * kDv, nq = (long long)T * H * kDk, nr = (long long)T * H;
  auto ckpt = saved.narrow(0, 0, nck);
  auto qn = saved.narrow(0, nck, nq);
  auto kn = saved.narrow(0, nck + nq, nq);
  auto rq = saved.narrow(0, nck + 2 * nq, nr);
  auto rk = saved.narrow(0, nck + 2 * nq + nr, nr);
  auto scratch = at::empty({H, kCk, kDk, kDv}, q.options().dtype(at::kFloat));
  auto dqn = at::empty({T, H, kDk}, q.options().dtype(at::kFloat));
  auto dkn = at::empty({T, H, kDk}, q.options().dtype(at::kFloat));
  auto dv = at::empty_like(v);
  auto dg = at::empty({T, H}, q.options().dtype(at::kFloat));
  auto dbeta = at::empty({T, H}, q.options().dtype(at::kFloat));
  auto ds0 = at::empty({H, kDk, kDv}, q.options().dtype(at::kFloat));
  const int dyn = 2 * kCk * kDv * (int)sizeof(float);
  ensure_smem((const void*)gdn_bwd_kernel, (int)(dyn));
  gdn_bwd_kernel<<<H, kThreads, dyn, stream()>>>(qn.data_ptr<float>(), kn.data_ptr<float>(), (const bf16*)v.data_ptr(),
                                               g.data_ptr<float>(), beta.data_ptr<float>(), ckpt.data_ptr<float>(),
                                               (const bf16*)dout.data_ptr(), dfinal.data_ptr<float>(),
                                               scratch.data_ptr<float>(), dqn.data_ptr<float>(), dkn.data_ptr<float>(),
                                               (bf16*)dv.data_ptr(), dg.data_ptr<float>(), dbeta.data_ptr<float>(),
                                               ds0.data_ptr<float>(), T, H);
  auto dq = at::empty_like(q);
  auto dk = at::empty_like(k);
  const long long rows = (long long)T * H;
  if (rows > 0)
    gdn_prep_bwd_kernel<<<(int)((rows + 7) / 8), 256, 0, stream()>>>(
        (const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(), dqn.data_ptr<float>(), dkn.data_ptr<float>(),
        rq.data_ptr<float>(), rk.data_ptr<float>(), (bf16*)dq.data_ptr(), (bf16*)dk.data_ptr(), rows,
        1.f / sqrtf((float)kDk));
  TS_LAUNCH_CHECK();
  return {dq, dk, dv, dg, dbeta, ds0};
}

}  // namespace ts
