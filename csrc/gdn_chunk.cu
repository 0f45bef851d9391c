// Chunked (WY-form) gated delta rule, forward and backward (K09', S9).
//
// Per head, over chunks of C = 64 tokens with the chunk-start state S0
// ([dk, dv] = [128, 128], fp32), G the in-chunk inclusive cumsum of the log
// decay g and γ = G_C:
//
//   A_ij = β_i e^{G_i−G_j} (k_i·k_j) (i > j),  T = (I + A)^{-1}
//   W = T diag(β e^G) K,  U = T diag(β) V,  δ = U − W S0
//   P_ij = e^{G_i−G_j} (q_i·k_j) (j ≤ i)
//   O = diag(e^G) Q S0 + P δ,  S_C = e^γ S0 + Kᵀ diag(e^{γ−G}) δ
//
// with q, k L2-normalised (q also scaled by dk^-1/2) inside the kernels.
// The serial dependency runs over chunks, not tokens:
//
//   gdn_wy_kernel        chunk-parallel: A, T, W, U and the row-scaled keys
//                        Kd = diag(e^{γ−G}) K, Kb = diag(β e^G) K
//   gdn_state_fwd_kernel serial over chunks, one CTA per (head, 16 state
//                        columns), two products per chunk (δ = U − W S0,
//                        S_C = e^γ S0 + Kdᵀ δ) with the next chunk's operands
//                        streaming in by cp.async: δ, chunk-start states, final state
//   gdn_out_kernel       chunk-parallel: P and O = diag(e^G) Q S0 + P δ
//   gdn_bwd_pre_kernel   chunk-parallel: X1 = Pᵀ dO, X2 = Qᵀ diag(e^G) dO
//   gdn_state_bwd_kernel serial over chunks in reverse, per (head, 16 columns):
//                        dζ = Tᵀ(X1 + Kd dS'), dS0 = e^γ dS' + X2 − Kbᵀ dζ
//   gdn_grads_state_kernel / gdn_grads_local_kernel  chunk-parallel: dq, dk,
//                        dv, dβ, dg (terms through S0 / dS', then the C x C
//                        terms, the reverse cumsum and the L2-norm VJP)
//
// The algebra and the hand-derived backward are the ones of
// thundersync_b200/ops/gdn_chunked.py (checked there against autograd through
// the token recurrence). Every matrix product runs on the tensor cores as
// warp-level mma.sync m16n8k8 with tf32 operands split in two (x = hi + lo,
// a·b ≈ hi·hi + hi·lo + lo·hi, three MMAs per fragment): the dropped lo·lo
// term is below 2^-21 of the product, so the products keep fp32 accuracy and
// the final state stays within 1e-3 of the fp32 recurrence. The products are
// 64- and 128-row tiles held in registers by their epilogues (masks, decays,
// row sums), so they stay warp-level: each thread owns a fixed set of product
// elements (Tile) that the MMA fragments produce in place.
#include "common.cuh"
#include "common.h"

namespace ts {
namespace {

constexpr int C = 64;          // chunk length
constexpr int D = 128;         // dk = dv
constexpr int NT = 256;        // threads per CTA
constexpr int LD = D + 4;      // padded leading dimensions (≡ 4 mod 32: MMA fragment loads hit
constexpr int LC = C + 4;      // distinct banks, or two ways for transposed operands)
constexpr float kNormEps = 1e-6f;

typedef __nv_bfloat16 bf16;

// Ownership of a product's M x N elements: the CTA's 8 warps form a WM x WN grid of warp tiles of
// 8·TM rows x 4·TN columns, each covered by (TM/2) x (TN/2) m16n8 MMA fragments. Lane (g = lane/4,
// t = lane%4) owns rows g, g + 8 of every 16-row block and columns 2t, 2t + 1 of every 8-column
// block: element (r, c) of acc[TM][TN] is (row(r), col(c)). The 4 lanes of a quad (same g) and the
// WN warps of a warp row share each row.
template <int M, int N, int TM, int TN>
struct Tile {
  static constexpr int WM = M / (8 * TM), WN = N / (4 * TN);
  static_assert(WM * WN == NT / 32 && TM % 2 == 0 && TN % 2 == 0, "warp tiles must cover the product");
  TS_DEVICE static int wn() { return (threadIdx.x >> 5) % WN; }
  TS_DEVICE static int row(int r) {
    return ((threadIdx.x >> 5) / WN) * (8 * TM) + (r >> 1) * 16 + (r & 1) * 8 + ((threadIdx.x & 31) >> 2);
  }
  TS_DEVICE static int col(int c) {
    return ((threadIdx.x >> 5) % WN) * (4 * TN) + (c >> 1) * 8 + 2 * (threadIdx.x & 3) + (c & 1);
  }
};

// x = hi + lo with hi, lo tf32 (round to nearest; the low 13 bits cleared so hi is exact as fp32)
TS_DEVICE void tf32_split(float x, uint32_t& hi, uint32_t& lo) {
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
  h &= 0xffffe000u;
  const float rest = x - __uint_as_float(h);
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lo) : "f"(rest));
  hi = h;
}

TS_DEVICE void mma_tf32(float& d0, float& d1, float& d2, float& d3, const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

// acc[r][c] += Σ_k a(row(r), k) · b(k, col(c)) over k < K (a multiple of 8), with
// a(i, k) = TA ? A[k·lda + i] : A[i·lda + k] and b(k, j) = TB ? B[j·ldb + k] : B[k·ldb + j], fp32 operands
// in shared memory. Fragment layouts of m16n8k8 (PTX ISA): A a0 (g, t), a1 (g+8, t), a2 (g, t+4),
// a3 (g+8, t+4); B b0 (t, g), b1 (t+4, g); D d0, d1 (g, 2t + {0, 1}), d2, d3 (g+8, 2t + {0, 1}).
template <int M, int N, int TM, int TN, bool TA, bool TB>
TS_DEVICE void mm_acc(float (&acc)[TM][TN], const float* A, int lda, const float* B, int ldb, int K) {
  using Tl = Tile<M, N, TM, TN>;
  constexpr int MR = TM / 2, NC = TN / 2;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int r0 = ((threadIdx.x >> 5) / Tl::WN) * (8 * TM) + g;
  const int c0 = Tl::wn() * (4 * TN) + g;
  auto a_at = [&](int i, int k) { return TA ? A[k * lda + i] : A[i * lda + k]; };
  auto b_at = [&](int k, int j) { return TB ? B[j * ldb + k] : B[k * ldb + j]; };
#pragma unroll 2
  for (int k0 = 0; k0 < K; k0 += 8) {
    uint32_t ah[MR][4], al[MR][4], bh[NC][2], bl[NC][2];
#pragma unroll
    for (int i = 0; i < MR; ++i) {
      const int r = r0 + 16 * i;
      tf32_split(a_at(r, k0 + t), ah[i][0], al[i][0]);
      tf32_split(a_at(r + 8, k0 + t), ah[i][1], al[i][1]);
      tf32_split(a_at(r, k0 + t + 4), ah[i][2], al[i][2]);
      tf32_split(a_at(r + 8, k0 + t + 4), ah[i][3], al[i][3]);
    }
#pragma unroll
    for (int j = 0; j < NC; ++j) {
      const int c = c0 + 8 * j;
      tf32_split(b_at(k0 + t, c), bh[j][0], bl[j][0]);
      tf32_split(b_at(k0 + t + 4, c), bh[j][1], bl[j][1]);
    }
#pragma unroll
    for (int i = 0; i < MR; ++i)
#pragma unroll
      for (int j = 0; j < NC; ++j) {
        float& d0 = acc[2 * i][2 * j];
        float& d1 = acc[2 * i][2 * j + 1];
        float& d2 = acc[2 * i + 1][2 * j];
        float& d3 = acc[2 * i + 1][2 * j + 1];
        mma_tf32(d0, d1, d2, d3, al[i], bh[j]);  // small terms first
        mma_tf32(d0, d1, d2, d3, ah[i], bl[j]);
        mma_tf32(d0, d1, d2, d3, ah[i], bh[j]);
      }
  }
}

// Σ over the threads that own row Tl::row(r) of v[r]: the lanes of a quad by shuffles, then the Tl::WN
// warps of a warp row through part[WN][M] in warp order (fixed order: reproducible). Call with every
// thread of the CTA; part is complete after the caller's next __syncthreads.
template <class Tl, int TM>
TS_DEVICE void row_partials(float (&v)[TM], float* part, int M) {
#pragma unroll
  for (int r = 0; r < TM; ++r) {
    v[r] += __shfl_xor_sync(0xffffffffu, v[r], 1);
    v[r] += __shfl_xor_sync(0xffffffffu, v[r], 2);
  }
  if ((threadIdx.x & 3) == 0)
#pragma unroll
    for (int r = 0; r < TM; ++r) part[Tl::wn() * M + Tl::row(r)] = v[r];
}

template <int TM, int TN>
TS_DEVICE void zero(float (&acc)[TM][TN]) {
#pragma unroll
  for (int r = 0; r < TM; ++r)
#pragma unroll
    for (int c = 0; c < TN; ++c) acc[r][c] = 0.f;
}

// rows [0, n) of a [T, H, D] bf16 tensor (head h, from token t0) into dst[C][LD] fp32, rows >= n zeroed;
// with norm: rows are L2-normalised (rsqrt(|x|² + eps)) and scaled by `scale`
TS_DEVICE void load_rows(float* dst, const bf16* __restrict__ src, int t0, int n, int H, int h, bool norm,
                         float scale, float* rnorm = nullptr) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int r = warp; r < C; r += NT / 32) {
    float x[D / 32];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < D / 32; ++e) {
      x[e] = r < n ? __bfloat162float(src[((size_t)(t0 + r) * H + h) * D + lane + 32 * e]) : 0.f;
      ss += x[e] * x[e];
    }
    float m = scale;
    if (norm) {
      ss = warp_sum(ss);
      const float rs = rsqrtf(ss + kNormEps);
      m = rs * scale;
      if (rnorm != nullptr && lane == 0) rnorm[r] = rs;
    }
#pragma unroll
    for (int e = 0; e < D / 32; ++e) dst[r * LD + lane + 32 * e] = x[e] * m;
  }
}

// rows of an fp32 [T, H, D] tensor, columns [c0, c0 + W) into dst[C][ld]
template <int W>
TS_DEVICE void load_f32(float* dst, int ld, const float* __restrict__ src, int t0, int n, int H, int h, int c0) {
  for (int i = threadIdx.x; i < C * W; i += NT) {
    const int r = i / W, c = i % W;
    dst[r * ld + c] = r < n ? src[((size_t)(t0 + r) * H + h) * D + c0 + c] : 0.f;
  }
}
template <int W>
TS_DEVICE void load_bf16(float* dst, int ld, const bf16* __restrict__ src, int t0, int n, int H, int h, int c0) {
  for (int i = threadIdx.x; i < C * W; i += NT) {
    const int r = i / W, c = i % W;
    dst[r * ld + c] = r < n ? __bfloat162float(src[((size_t)(t0 + r) * H + h) * D + c0 + c]) : 0.f;
  }
}

// per-chunk scalars: G (inclusive cumsum of g), e^G, β, and γ = G at the last valid row
struct ChunkScalars {
  float G[C], eG[C], b[C];
};
TS_DEVICE void load_scalars(ChunkScalars& s, const float* __restrict__ g, const float* __restrict__ beta, int t0,
                            int n, int H, int h) {
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float g0 = lane < n ? g[(size_t)(t0 + lane) * H + h] : 0.f;
    float g1 = lane + 32 < n ? g[(size_t)(t0 + lane + 32) * H + h] : 0.f;
    // inclusive warp scans, then offset the upper half
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float a0 = __shfl_up_sync(0xffffffffu, g0, o);
      const float a1 = __shfl_up_sync(0xffffffffu, g1, o);
      if (lane >= o) {
        g0 += a0;
        g1 += a1;
      }
    }
    g1 += __shfl_sync(0xffffffffu, g0, 31);
    s.G[lane] = g0;
    s.G[lane + 32] = g1;
    s.eG[lane] = __expf(g0);
    s.eG[lane + 32] = __expf(g1);
    s.b[lane] = lane < n ? beta[(size_t)(t0 + lane) * H + h] : 0.f;
    s.b[lane + 32] = lane + 32 < n ? beta[(size_t)(t0 + lane + 32) * H + h] : 0.f;
  }
}

// ------------------------------------------------------------------ forward 1: WY factors
struct WySmem {
  float K[C * LD];
  float V[C * LD];
  float A[C * LC];
  float T[C * LC];
  ChunkScalars s;
};

__global__ void __launch_bounds__(NT) gdn_wy_kernel(const bf16* __restrict__ k, const bf16* __restrict__ v,
                                                    const float* __restrict__ g, const float* __restrict__ beta,
                                                    float* __restrict__ w_out, float* __restrict__ u_out,
                                                    float* __restrict__ t_out, float* __restrict__ kd_out,
                                                    float* __restrict__ kb_out, int Tn, int H) {
  extern __shared__ float smem_f[];
  WySmem& sm = *reinterpret_cast<WySmem*>(smem_f);
  const int ch = blockIdx.x, h = blockIdx.y;
  const int t0 = ch * C, n = min(C, Tn - t0);
  load_rows(sm.K, k, t0, n, H, h, true, 1.f);
  load_rows(sm.V, v, t0, n, H, h, false, 1.f);
  load_scalars(sm.s, g, beta, t0, n, H, h);
  __syncthreads();
  {  // A = strictly lower β_i e^{G_i − G_j} (k_i·k_j)
    using Tl = Tile<C, C, 4, 4>;
    float acc[4][4];
    zero(acc);
    mm_acc<C, C, 4, 4, false, true>(acc, sm.K, LD, sm.K, LD, D);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int i = Tl::row(r), j = Tl::col(c);
        sm.A[i * LC + j] = (i > j && i < n) ? sm.s.b[i] * __expf(sm.s.G[i] - sm.s.G[j]) * acc[r][c] : 0.f;
      }
  }
  __syncthreads();
  // T = (I + A)^{-1}: unit lower triangular; thread c owns column c and walks the rows in order
  if (threadIdx.x < C) {
    const int c = threadIdx.x;
    for (int i = 0; i < C; ++i) {
      float x = i == c ? 1.f : 0.f;
      if (i > c) {
        for (int j = c; j < i; ++j) x = fmaf(-sm.A[i * LC + j], sm.T[j * LC + c], x);
      }
      sm.T[i * LC + c] = x;
    }
  }
  // row scales: K rows by β e^G (kept: the state-gradient pass reads them), V rows by β; K rows by
  // e^{γ−G} go out for the state update
  {
    const float gam = sm.s.G[n - 1];
    for (int i = threadIdx.x; i < C * D; i += NT) {
      const int r = i / D, c = i % D;
      const float x = sm.K[r * LD + c];
      if (r < n) {
        const size_t o = ((size_t)(t0 + r) * H + h) * D + c;
        kd_out[o] = x * __expf(gam - sm.s.G[r]);
        kb_out[o] = x * sm.s.b[r] * sm.s.eG[r];
      }
      sm.K[r * LD + c] = x * sm.s.b[r] * sm.s.eG[r];
      sm.V[r * LD + c] *= sm.s.b[r];
    }
  }
  __syncthreads();
  using Tw = Tile<C, D, 4, 8>;
  {
    float acc[4][8];
    zero(acc);
    mm_acc<C, D, 4, 8, false, false>(acc, sm.T, LC, sm.K, LD, C);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = Tw::row(r);
      if (i < n)
#pragma unroll
        for (int c = 0; c < 8; ++c) w_out[((size_t)(t0 + i) * H + h) * D + Tw::col(c)] = acc[r][c];
    }
  }
  {
    float acc[4][8];
    zero(acc);
    mm_acc<C, D, 4, 8, false, false>(acc, sm.T, LC, sm.V, LD, C);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = Tw::row(r);
      if (i < n)
#pragma unroll
        for (int c = 0; c < 8; ++c) u_out[((size_t)(t0 + i) * H + h) * D + Tw::col(c)] = acc[r][c];
    }
  }
  float* tt = t_out + ((size_t)ch * H + h) * C * C;
  for (int i = threadIdx.x; i < C * C; i += NT) tt[i] = sm.T[(i / C) * LC + (i % C)];
}

// ------------------------------------------------------------------ asynchronous row copies
TS_DEVICE void cp_async16(void* dst, const void* src, bool valid) {
  const uint32_t d = (uint32_t)__cvta_generic_to_shared(dst);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
TS_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
TS_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// rows [0, C) (zero-filled from n) of W floats per row, from src + row·row_stride + c0, into dst[C][ld]
template <int W>
TS_DEVICE void prefetch_rows(float* dst, int ld, const float* __restrict__ src, size_t row_stride, int n, int c0) {
  constexpr int V = W / 4;  // 16-byte pieces per row
  for (int i = threadIdx.x; i < C * V; i += NT) {
    const int r = i / V, c = (i % V) * 4;
    cp_async16(dst + r * ld + c, src + (size_t)(r < n ? r : 0) * row_stride + c0 + c, r < n);
  }
}

// ------------------------------------------------------------------ forward 2: the serial state pass
// One CTA per (head, 16 state columns); per chunk only two products sit on the chain:
//   δ = U − W S,  S ← e^γ S + Kdᵀ δ   (Kd = diag(e^{γ−G}) K from gdn_wy_kernel)
// The next chunk's W, Kd and U slice stream into the other shared-memory buffer while this chunk computes.
constexpr int SF = 16;         // state columns per CTA
constexpr int LW = D + 4;      // 16-byte aligned rows for the asynchronous copies
constexpr int LU = SF + 4;
struct StateFwdSmem {
  float S[D * (SF + 1)];
  float W[2][C * LW];
  float K[2][C * LW];
  float U[2][C * LU];   // U slice, then δ
  float G[C];
};

__global__ void __launch_bounds__(NT) gdn_state_fwd_kernel(const float* __restrict__ g,
                                                           const float* __restrict__ w, const float* __restrict__ u,
                                                           const float* __restrict__ kd,
                                                           const float* __restrict__ s_in, float* __restrict__ s_out,
                                                           float* __restrict__ starts, float* __restrict__ delta,
                                                           int Tn, int H) {
  extern __shared__ __align__(16) float smem_f[];
  StateFwdSmem& sm = *reinterpret_cast<StateFwdSmem*>(smem_f);
  constexpr int LSF = SF + 1;
  const int h = blockIdx.x, j0 = blockIdx.y * SF;
  const int nch = (Tn + C - 1) / C;
  const size_t rs = (size_t)H * D;
  for (int i = threadIdx.x; i < D * SF; i += NT) sm.S[(i / SF) * LSF + i % SF] = s_in[((size_t)h * D + i / SF) * D + j0 + i % SF];
  auto issue = [&](int ch) {
    const int t0 = ch * C, n = min(C, Tn - t0), b = ch & 1;
    const size_t base = (size_t)t0 * rs + (size_t)h * D;
    prefetch_rows<D>(sm.W[b], LW, w + base, rs, n, 0);
    prefetch_rows<D>(sm.K[b], LW, kd + base, rs, n, 0);
    prefetch_rows<SF>(sm.U[b], LU, u + base, rs, n, j0);
    cp_async_commit();
  };
  issue(0);
  for (int ch = 0; ch < nch; ++ch) {
    const int t0 = ch * C, n = min(C, Tn - t0), b = ch & 1;
    if (ch + 1 < nch) {
      issue(ch + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    float* st = starts + ((size_t)ch * H + h) * D * D;
    for (int i = threadIdx.x; i < D * SF; i += NT) st[(i / SF) * D + j0 + i % SF] = sm.S[(i / SF) * LSF + i % SF];
    if (threadIdx.x < 32) {  // in-chunk cumsum of g (γ = G at the last valid row)
      const int lane = threadIdx.x;
      float g0 = lane < n ? g[(size_t)(t0 + lane) * H + h] : 0.f;
      float g1 = lane + 32 < n ? g[(size_t)(t0 + lane + 32) * H + h] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float a0 = __shfl_up_sync(0xffffffffu, g0, o), a1 = __shfl_up_sync(0xffffffffu, g1, o);
        if (lane >= o) g0 += a0, g1 += a1;
      }
      g1 += __shfl_sync(0xffffffffu, g0, 31);
      sm.G[lane] = g0;
      sm.G[lane + 32] = g1;
    }
    __syncthreads();
    using Td = Tile<C, SF, 2, 2>;
    {  // δ = U − W S
      float acc[2][2];
      zero(acc);
      mm_acc<C, SF, 2, 2, false, false>(acc, sm.W[b], LW, sm.S, LSF, D);
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int i = Td::row(r);
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int j = Td::col(c);
          const float d = i < n ? sm.U[b][i * LU + j] - acc[r][c] : 0.f;
          sm.U[b][i * LU + j] = d;
          if (i < n) delta[((size_t)(t0 + i) * H + h) * D + j0 + j] = d;
        }
      }
    }
    __syncthreads();
    {  // S = e^γ S + Kdᵀ δ
      using Ts = Tile<D, SF, 4, 2>;
      float acc[4][2];
      zero(acc);
      mm_acc<D, SF, 4, 2, true, false>(acc, sm.K[b], LW, sm.U[b], LU, C);
      const float eg = __expf(sm.G[n - 1]);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float& x = sm.S[Ts::row(r) * LSF + Ts::col(c)];
          x = fmaf(eg, x, acc[r][c]);  // each element is read and written by its own thread only
        }
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < D * SF; i += NT) s_out[((size_t)h * D + i / SF) * D + j0 + i % SF] = sm.S[(i / SF) * LSF + i % SF];
}

// ------------------------------------------------------------------ forward 3: outputs (chunk-parallel)
// O = diag(e^G) Q S0 + P δ with S0 the chunk-start state; P is also kept for the backward.
struct OutSmem {
  float S[D * LD];
  float Q[C * LD];
  float K[C * LD];   // K, then δ
  float P[C * LC];
  ChunkScalars s;
};

__global__ void __launch_bounds__(NT) gdn_out_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                     const float* __restrict__ g, const float* __restrict__ beta,
                                                     const float* __restrict__ delta, const float* __restrict__ starts,
                                                     bf16* __restrict__ o, float* __restrict__ p_out, int Tn, int H) {
  extern __shared__ float smem_f[];
  OutSmem& sm = *reinterpret_cast<OutSmem*>(smem_f);
  const int ch = blockIdx.x, h = blockIdx.y;
  const int t0 = ch * C, n = min(C, Tn - t0);
  const float* S0 = starts + ((size_t)ch * H + h) * D * D;
  for (int i = threadIdx.x; i < D * D; i += NT) sm.S[(i / D) * LD + i % D] = S0[i];
  load_rows(sm.Q, q, t0, n, H, h, true, rsqrtf((float)D));
  load_rows(sm.K, k, t0, n, H, h, true, 1.f);
  load_scalars(sm.s, g, beta, t0, n, H, h);
  __syncthreads();
  {
    using Tl = Tile<C, C, 4, 4>;
    float acc[4][4];
    zero(acc);
    mm_acc<C, C, 4, 4, false, true>(acc, sm.Q, LD, sm.K, LD, D);
    float* pp = p_out + ((size_t)ch * H + h) * C * C;
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int i = Tl::row(r), j = Tl::col(c);
        const float x = (j <= i && i < n) ? __expf(sm.s.G[i] - sm.s.G[j]) * acc[r][c] : 0.f;
        sm.P[i * LC + j] = x;
        pp[i * C + j] = x;
      }
  }
  using Tw = Tile<C, D, 4, 8>;
  float acc[4][8];
  zero(acc);
  mm_acc<C, D, 4, 8, false, false>(acc, sm.Q, LD, sm.S, LD, D);   // Q S0
#pragma unroll
  for (int r = 0; r < 4; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[r][c] *= sm.s.eG[Tw::row(r)];
  __syncthreads();
  load_f32<D>(sm.K, LD, delta, t0, n, H, h, 0);
  __syncthreads();
  mm_acc<C, D, 4, 8, false, false>(acc, sm.P, LC, sm.K, LD, C);   // + P δ
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = Tw::row(r);
    if (i < n)
#pragma unroll
      for (int c = 0; c < 8; ++c) o[((size_t)(t0 + i) * H + h) * D + Tw::col(c)] = __float2bfloat16_rn(acc[r][c]);
  }
}

// ------------------------------------------------------------------ backward 0: chain-free terms (chunk-parallel)
// X1 = Pᵀ dO  [C, D]  and  X2 = Qᵀ diag(e^G) dO  [D, D] per chunk: the parts of the state-gradient
// recursion that do not depend on the state gradient.
struct BwdPreSmem {
  float Q[C * LD];
  float X[C * LD];   // dO
  float P[C * LC];
  ChunkScalars s;
};

__global__ void __launch_bounds__(NT) gdn_bwd_pre_kernel(const bf16* __restrict__ q, const float* __restrict__ g,
                                                         const float* __restrict__ beta,
                                                         const bf16* __restrict__ dout, const float* __restrict__ p_sv,
                                                         float* __restrict__ x1, float* __restrict__ x2, int Tn,
                                                         int H) {
  extern __shared__ float smem_f[];
  BwdPreSmem& sm = *reinterpret_cast<BwdPreSmem*>(smem_f);
  const int ch = blockIdx.x, h = blockIdx.y;
  const int t0 = ch * C, n = min(C, Tn - t0);
  load_rows(sm.Q, q, t0, n, H, h, true, rsqrtf((float)D));
  load_bf16<D>(sm.X, LD, dout, t0, n, H, h, 0);
  load_scalars(sm.s, g, beta, t0, n, H, h);
  {
    const float* pp = p_sv + ((size_t)ch * H + h) * C * C;
    for (int i = threadIdx.x; i < C * C; i += NT) sm.P[(i / C) * LC + i % C] = pp[i];
  }
  __syncthreads();
  {
    using Tw = Tile<C, D, 4, 8>;
    float acc[4][8];
    zero(acc);
    mm_acc<C, D, 4, 8, true, false>(acc, sm.P, LC, sm.X, LD, C);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = Tw::row(r);
      if (i < n)
#pragma unroll
        for (int c = 0; c < 8; ++c) x1[((size_t)(t0 + i) * H + h) * D + Tw::col(c)] = acc[r][c];
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < C * D; i += NT) sm.X[(i / D) * LD + i % D] *= sm.s.eG[i / D];
  __syncthreads();
  using Tq = Tile<D, D, 8, 8>;
  float acc[8][8];
  zero(acc);
  mm_acc<D, D, 8, 8, true, false>(acc, sm.Q, LD, sm.X, LD, C);
  float* xx = x2 + ((size_t)ch * H + h) * D * D;
#pragma unroll
  for (int r = 0; r < 8; ++r)
#pragma unroll
    for (int c = 0; c < 8; ++c) xx[Tq::row(r) * D + Tq::col(c)] = acc[r][c];
}

// ------------------------------------------------------------------ backward 1: the serial state-gradient pass
// One CTA per (head, 16 columns), chunks in reverse; per chunk:
//   dd = X1 + Kd dS',  dζ = Tᵀ dd,  dS ← e^γ dS' + X2 − Kbᵀ dζ
// (Kd = diag(e^{γ−G}) K, Kb = diag(β e^G) K), with the next chunk's operands streaming in meanwhile.
constexpr int LT = C + 4;
struct StateBwdSmem {
  float dS[D * (SF + 1)];
  float Kd[2][C * LW];
  float Kb[2][C * LW];
  float T[2][C * LT];
  float X1[2][C * LU];   // X1 slice, then dd
  float X2[2][D * LU];
  float dz[C * (SF + 1)];
  float G[C];
};

__global__ void __launch_bounds__(NT) gdn_state_bwd_kernel(const float* __restrict__ g,
                                                           const float* __restrict__ kd, const float* __restrict__ kb,
                                                           const float* __restrict__ t_sv,
                                                           const float* __restrict__ x1, const float* __restrict__ x2,
                                                           const float* __restrict__ dfinal,
                                                           float* __restrict__ ds_sv, float* __restrict__ dz_out,
                                                           float* __restrict__ dstate, int Tn, int H) {
  extern __shared__ __align__(16) float smem_f[];
  StateBwdSmem& sm = *reinterpret_cast<StateBwdSmem*>(smem_f);
  constexpr int LSF = SF + 1;
  const int h = blockIdx.x, j0 = blockIdx.y * SF;
  const int nch = (Tn + C - 1) / C;
  const size_t rs = (size_t)H * D;
  for (int i = threadIdx.x; i < D * SF; i += NT) sm.dS[(i / SF) * LSF + i % SF] = dfinal[((size_t)h * D + i / SF) * D + j0 + i % SF];
  auto issue = [&](int ch) {
    const int t0 = ch * C, n = min(C, Tn - t0), b = ch & 1;
    const size_t base = (size_t)t0 * rs + (size_t)h * D;
    prefetch_rows<D>(sm.Kd[b], LW, kd + base, rs, n, 0);
    prefetch_rows<D>(sm.Kb[b], LW, kb + base, rs, n, 0);
    prefetch_rows<C>(sm.T[b], LT, t_sv + ((size_t)ch * H + h) * C * C, C, C, 0);
    prefetch_rows<SF>(sm.X1[b], LU, x1 + base, rs, n, j0);
    // X2 rows are the D state rows: two C-row halves
    const float* xx = x2 + ((size_t)ch * H + h) * D * D;
    prefetch_rows<SF>(sm.X2[b], LU, xx, D, C, j0);
    prefetch_rows<SF>(sm.X2[b] + C * LU, LU, xx + (size_t)C * D, D, C, j0);
    cp_async_commit();
  };
  issue(nch - 1);
  for (int ch = nch - 1; ch >= 0; --ch) {
    const int t0 = ch * C, n = min(C, Tn - t0), b = ch & 1;
    if (ch > 0) {
      issue(ch - 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    float* dsv = ds_sv + ((size_t)ch * H + h) * D * D;
    for (int i = threadIdx.x; i < D * SF; i += NT) dsv[(i / SF) * D + j0 + i % SF] = sm.dS[(i / SF) * LSF + i % SF];
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      float g0 = lane < n ? g[(size_t)(t0 + lane) * H + h] : 0.f;
      float g1 = lane + 32 < n ? g[(size_t)(t0 + lane + 32) * H + h] : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float a0 = __shfl_up_sync(0xffffffffu, g0, o), a1 = __shfl_up_sync(0xffffffffu, g1, o);
        if (lane >= o) g0 += a0, g1 += a1;
      }
      g1 += __shfl_sync(0xffffffffu, g0, 31);
      sm.G[lane] = g0;
      sm.G[lane + 32] = g1;
    }
    __syncthreads();
    using Td = Tile<C, SF, 2, 2>;
    {  // dd = X1 + Kd dS'
      float acc[2][2];
      zero(acc);
      mm_acc<C, SF, 2, 2, false, false>(acc, sm.Kd[b], LW, sm.dS, LSF, D);
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int i = Td::row(r), j = Td::col(c);
          sm.X1[b][i * LU + j] = i < n ? sm.X1[b][i * LU + j] + acc[r][c] : 0.f;
        }
    }
    __syncthreads();
    {  // dζ = Tᵀ dd
      float acc[2][2];
      zero(acc);
      mm_acc<C, SF, 2, 2, true, false>(acc, sm.T[b], LT, sm.X1[b], LU, C);
#pragma unroll
      for (int r = 0; r < 2; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int i = Td::row(r), j = Td::col(c);
          const float z = i < n ? acc[r][c] : 0.f;
          sm.dz[i * LSF + j] = z;
          if (i < n) dz_out[((size_t)(t0 + i) * H + h) * D + j0 + j] = z;
        }
    }
    __syncthreads();
    {  // dS = e^γ dS' + X2 − Kbᵀ dζ
      using Ts = Tile<D, SF, 4, 2>;
      float acc[4][2];
      zero(acc);
      mm_acc<D, SF, 4, 2, true, false>(acc, sm.Kb[b], LW, sm.dz, LSF, C);
      const float eg = __expf(sm.G[n - 1]);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int i = Ts::row(r), j = Ts::col(c);
          float& x = sm.dS[i * LSF + j];
          x = eg * x + sm.X2[b][i * LU + j] - acc[r][c];
        }
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < D * SF; i += NT) dstate[((size_t)h * D + i / SF) * D + j0 + i % SF] = sm.dS[(i / SF) * LSF + i % SF];
}

// ------------------------------------------------------------------ backward 2: terms through S0 and dS'
// Per chunk: with R = V − diag(e^G) K S0 and dR = diag(β) dζ,
//   dQ̂ += diag(e^G) dO S0ᵀ,  dK̂ += −diag(e^G) dR S0ᵀ + diag(e^{γ−G}) δ dS'ᵀ
//   dβ_i += Σ_v dζ_iv R_iv
//   dG_i += −e^{G_i} Σ_v (K S0)_iv dR_iv + e^{G_i} Σ_v dO_iv (Q S0)_iv − E_i,  E_i = e^{γ−G_i} Σ_v (K dS')_iv δ_iv
//   dγ    = e^γ ⟨S0, dS'⟩ + Σ_i E_i
struct GradStateSmem {
  float S[D * LD];   // S0, then dS'
  float K[C * LD];
  float Q[C * LD];   // Q, then δ
  float X[C * LD];   // dO
  float Z[C * LD];   // dζ
  float part[3][4][C];   // row partials (dβ, dG, E) per warp column of the C x D tiles
  float red[NT / 32];
  ChunkScalars s;
};

__global__ void __launch_bounds__(NT) gdn_grads_state_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, const bf16* __restrict__ dout, const float* __restrict__ starts,
    const float* __restrict__ ds_sv, const float* __restrict__ delta, const float* __restrict__ dz,
    float* __restrict__ dqh, float* __restrict__ dkh, float* __restrict__ dbeta, float* __restrict__ dG,
    float* __restrict__ dgam, int Tn, int H) {
  extern __shared__ float smem_f[];
  GradStateSmem& sm = *reinterpret_cast<GradStateSmem*>(smem_f);
  const int ch = blockIdx.x, h = blockIdx.y;
  const int t0 = ch * C, n = min(C, Tn - t0);
  const float* S0 = starts + ((size_t)ch * H + h) * D * D;
  for (int i = threadIdx.x; i < D * D; i += NT) sm.S[(i / D) * LD + i % D] = S0[i];
  load_rows(sm.K, k, t0, n, H, h, true, 1.f);
  load_rows(sm.Q, q, t0, n, H, h, true, rsqrtf((float)D));
  load_bf16<D>(sm.X, LD, dout, t0, n, H, h, 0);
  load_f32<D>(sm.Z, LD, dz, t0, n, H, h, 0);
  load_scalars(sm.s, g, beta, t0, n, H, h);
  __syncthreads();
  using Tw = Tile<C, D, 4, 8>;
  static_assert(Tw::WN == 4, "part[][4][] holds one partial per warp column");
  float dq[4][8], dk[4][8];
  float rb[4] = {0.f, 0.f, 0.f, 0.f}, rg[4] = {0.f, 0.f, 0.f, 0.f};
  {
    float ks[4][8], qs[4][8];
    zero(ks);
    zero(qs);
    mm_acc<C, D, 4, 8, false, false>(ks, sm.K, LD, sm.S, LD, D);   // K S0
    mm_acc<C, D, 4, 8, false, false>(qs, sm.Q, LD, sm.S, LD, D);   // Q S0
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = Tw::row(r);
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int j = Tw::col(c);
        const float vv = i < n ? __bfloat162float(v[((size_t)(t0 + i) * H + h) * D + j]) : 0.f;
        const float z = sm.Z[i * LD + j];
        const float R = vv - sm.s.eG[i] * ks[r][c];
        rb[r] = fmaf(z, R, rb[r]);
        rg[r] += -sm.s.eG[i] * ks[r][c] * sm.s.b[i] * z + sm.s.eG[i] * sm.X[i * LD + j] * qs[r][c];
      }
    }
  }
  zero(dq);
  zero(dk);
  mm_acc<C, D, 4, 8, false, true>(dq, sm.X, LD, sm.S, LD, D);   // dO S0ᵀ
  mm_acc<C, D, 4, 8, false, true>(dk, sm.Z, LD, sm.S, LD, D);   // dζ S0ᵀ
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = Tw::row(r);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      dq[r][c] *= sm.s.eG[i];
      dk[r][c] *= -sm.s.eG[i] * sm.s.b[i];
    }
  }
  // e^γ ⟨S0, dS'⟩ (this chunk's dS' is read straight from global memory)
  const float* dSp = ds_sv + ((size_t)ch * H + h) * D * D;
  float dot = 0.f;
  for (int i = threadIdx.x; i < D * D; i += NT) dot = fmaf(sm.S[(i / D) * LD + i % D], dSp[i], dot);
  __syncthreads();  // S0 and Q no longer needed
  for (int i = threadIdx.x; i < D * D; i += NT) sm.S[(i / D) * LD + i % D] = dSp[i];
  load_f32<D>(sm.Q, LD, delta, t0, n, H, h, 0);
  __syncthreads();
  const float gam = sm.s.G[n - 1];
  float re[4] = {0.f, 0.f, 0.f, 0.f};
  {
    float kd[4][8], dd[4][8];
    zero(kd);
    zero(dd);
    mm_acc<C, D, 4, 8, false, false>(kd, sm.K, LD, sm.S, LD, D);   // K dS'
    mm_acc<C, D, 4, 8, false, true>(dd, sm.Q, LD, sm.S, LD, D);    // δ dS'ᵀ
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = Tw::row(r);
      const float e = i < n ? __expf(gam - sm.s.G[i]) : 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        re[r] = fmaf(kd[r][c], sm.Q[i * LD + Tw::col(c)], re[r]);
        dk[r][c] = fmaf(e, dd[r][c], dk[r][c]);
      }
      re[r] *= e;
    }
  }
  // row sums: the quad's lanes, then one partial per warp column (summed in order below)
#pragma unroll
  for (int r = 0; r < 4; ++r) rg[r] -= re[r];
  row_partials<Tw>(rb, &sm.part[0][0][0], C);
  row_partials<Tw>(rg, &sm.part[1][0][0], C);
  row_partials<Tw>(re, &sm.part[2][0][0], C);
  // dγ: e^γ ⟨S0, dS'⟩ + Σ_i E_i
  dot = warp_sum(dot);
  if ((threadIdx.x & 31) == 0) sm.red[threadIdx.x >> 5] = dot;
  __syncthreads();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (int w = 0; w < NT / 32; ++w) tot += sm.red[w];
    float es = 0.f;
    for (int i = 0; i < n; ++i) es += ((sm.part[2][0][i] + sm.part[2][1][i]) + sm.part[2][2][i]) + sm.part[2][3][i];
    dgam[(size_t)ch * H + h] = __expf(gam) * tot + es;
  }
  for (int i = threadIdx.x; i < n; i += NT) {
    dbeta[(size_t)(t0 + i) * H + h] = ((sm.part[0][0][i] + sm.part[0][1][i]) + sm.part[0][2][i]) + sm.part[0][3][i];
    dG[(size_t)(t0 + i) * H + h] = ((sm.part[1][0][i] + sm.part[1][1][i]) + sm.part[1][2][i]) + sm.part[1][3][i];
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = Tw::row(r);
    if (i < n)
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const size_t x = ((size_t)(t0 + i) * H + h) * D + Tw::col(c);
        dqh[x] = dq[r][c];
        dkh[x] = dk[r][c];
      }
  }
}

// ------------------------------------------------------------------ backward 3: C x C terms, cumsum, L2-norm VJP
// dA = −dζ δᵀ (i > j), dP = dO δᵀ (j ≤ i); with A, P the forward's matrices:
//   dM = dA ⊙ β_i e^{G_i−G_j},  dN = dP ⊙ e^{G_i−G_j}
//   dK̂ += dM K + dMᵀ K + dNᵀ Q,  dQ̂ += dN K
//   dβ_i += Σ_j dA_ij e^{G_i−G_j} (k_i·k_j),  dG += rowsum(dA⊙A) − colsum(dA⊙A) + rowsum(dP⊙P) − colsum(dP⊙P)
//   dg = reverse cumsum of dG (+ dγ at the last row); dv = β ⊙ dζ
struct GradLocalSmem {
  float K[C * LD];
  float Q[C * LD];
  float X[C * LD];   // dO, then dζ
  float Y[C * LD];   // δ
  float dM[C * LC];
  float dN[C * LC];
  float rowacc[C][2];
  float part[4][C];   // dβ row partials per warp column of the C x C tiles
  ChunkScalars s;
};

__global__ void __launch_bounds__(NT) gdn_grads_local_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const float* __restrict__ g,
    const float* __restrict__ beta, const bf16* __restrict__ dout, const float* __restrict__ delta,
    const float* __restrict__ dz, const float* __restrict__ dqh, const float* __restrict__ dkh,
    const float* __restrict__ dbeta_s, const float* __restrict__ dG_s, const float* __restrict__ dgam,
    bf16* __restrict__ dq, bf16* __restrict__ dk, bf16* __restrict__ dv, float* __restrict__ dg,
    float* __restrict__ dbeta, int Tn, int H) {
  extern __shared__ float smem_f[];
  GradLocalSmem& sm = *reinterpret_cast<GradLocalSmem*>(smem_f);
  const int ch = blockIdx.x, h = blockIdx.y;
  const int t0 = ch * C, n = min(C, Tn - t0);
  load_rows(sm.K, k, t0, n, H, h, true, 1.f);
  load_rows(sm.Q, q, t0, n, H, h, true, rsqrtf((float)D));
  load_bf16<D>(sm.X, LD, dout, t0, n, H, h, 0);
  load_f32<D>(sm.Y, LD, delta, t0, n, H, h, 0);
  load_scalars(sm.s, g, beta, t0, n, H, h);
  for (int i = threadIdx.x; i < C * 2; i += NT) sm.rowacc[i / 2][i % 2] = 0.f;
  __syncthreads();
  using Tl = Tile<C, C, 4, 4>;
  float pdp[4][4];
  {  // dP = dO δᵀ and P = e^{G_i−G_j} q_i·k_j (j ≤ i)
    float dp[4][4], qk[4][4];
    zero(dp);
    zero(qk);
    mm_acc<C, C, 4, 4, false, true>(dp, sm.X, LD, sm.Y, LD, D);
    mm_acc<C, C, 4, 4, false, true>(qk, sm.Q, LD, sm.K, LD, D);
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int i = Tl::row(r), j = Tl::col(c);
        const bool on = j <= i && i < n;
        const float e = on ? __expf(sm.s.G[i] - sm.s.G[j]) : 0.f;
        sm.dN[i * LC + j] = on ? dp[r][c] * e : 0.f;
        pdp[r][c] = on ? dp[r][c] * e * qk[r][c] : 0.f;
      }
  }
  __syncthreads();
  load_f32<D>(sm.X, LD, dz, t0, n, H, h, 0);  // dO -> dζ
  __syncthreads();
  float ada[4][4];
  {  // dA = −dζ δᵀ (i > j); A = β_i e^{G_i−G_j} k_i·k_j
    float da[4][4], kk[4][4];
    zero(da);
    zero(kk);
    mm_acc<C, C, 4, 4, false, true>(da, sm.X, LD, sm.Y, LD, D);
    mm_acc<C, C, 4, 4, false, true>(kk, sm.K, LD, sm.K, LD, D);
    float rbeta[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = Tl::row(r);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j = Tl::col(c);
        const bool on = i > j && i < n;
        const float el = on ? __expf(sm.s.G[i] - sm.s.G[j]) : 0.f;
        const float dA = on ? -da[r][c] : 0.f;
        sm.dM[i * LC + j] = dA * sm.s.b[i] * el;
        ada[r][c] = dA * sm.s.b[i] * el * kk[r][c];
        rbeta[r] = fmaf(dA * el, kk[r][c], rbeta[r]);
      }
    }
    // row sums: the quad's lanes, then one partial per warp column (summed in order below; no atomics)
    static_assert(Tl::WN == 4, "part[4][] holds one partial per warp column");
    row_partials<Tl>(rbeta, &sm.part[0][0], C);
  }
  __syncthreads();
  // dG partial from the C x C terms: rowsum − colsum of (dA⊙A + dP⊙P); a column j's sum is over
  // the threads holding rows of column j — gather through the dN-sized scratch in Y (δ is no longer needed)
  {
    float* Mx = sm.Y;  // [C][LC] view
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) Mx[Tl::row(r) * LC + Tl::col(c)] = ada[r][c] + pdp[r][c];
  }
  __syncthreads();
  if (threadIdx.x < C) {
    const int i = threadIdx.x;
    const float* Mx = sm.Y;
    float rs = 0.f, cs = 0.f;
    for (int j = 0; j < C; ++j) {
      rs += Mx[i * LC + j];
      cs += Mx[j * LC + i];
    }
    sm.rowacc[i][1] = rs - cs;
    sm.rowacc[i][0] = ((sm.part[0][i] + sm.part[1][i]) + sm.part[2][i]) + sm.part[3][i];
  }
  __syncthreads();
  // dG total and the reverse cumsum (one warp, two values per lane)
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float a0 = 0.f, a1 = 0.f;
    if (lane < n) a0 = dG_s[(size_t)(t0 + lane) * H + h] + sm.rowacc[lane][1];
    if (lane + 32 < n) a1 = dG_s[(size_t)(t0 + lane + 32) * H + h] + sm.rowacc[lane + 32][1];
    if (lane == n - 1) a0 += dgam[(size_t)ch * H + h];
    if (lane + 32 == n - 1) a1 += dgam[(size_t)ch * H + h];
    // reverse inclusive scan over 64 values: suffix sums
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float b0 = __shfl_down_sync(0xffffffffu, a0, o);
      const float b1 = __shfl_down_sync(0xffffffffu, a1, o);
      if (lane + o < 32) {
        a0 += b0;
        a1 += b1;
      }
    }
    a0 += __shfl_sync(0xffffffffu, a1, 0);
    if (lane < n) dg[(size_t)(t0 + lane) * H + h] = a0;
    if (lane + 32 < n) dg[(size_t)(t0 + lane + 32) * H + h] = a1;
  }
  for (int i = threadIdx.x; i < n; i += NT)
    dbeta[(size_t)(t0 + i) * H + h] = dbeta_s[(size_t)(t0 + i) * H + h] + sm.rowacc[i][0];
  // dv = β ⊙ dζ
  for (int i = threadIdx.x; i < n * D; i += NT) {
    const int r = i / D, c = i % D;
    dv[((size_t)(t0 + r) * H + h) * D + c] = __float2bfloat16_rn(sm.s.b[r] * sm.X[r * LD + c]);
  }
  // dK̂ += dM K + dMᵀ K + dNᵀ Q ;  dQ̂ += dN K
  using Tw = Tile<C, D, 4, 8>;
  float ak[4][8], aq[4][8];
  zero(ak);
  zero(aq);
  mm_acc<C, D, 4, 8, false, false>(ak, sm.dM, LC, sm.K, LD, C);
  mm_acc<C, D, 4, 8, true, false>(ak, sm.dM, LC, sm.K, LD, C);
  mm_acc<C, D, 4, 8, true, false>(ak, sm.dN, LC, sm.Q, LD, C);
  mm_acc<C, D, 4, 8, false, false>(aq, sm.dN, LC, sm.K, LD, C);
  __syncthreads();
  // add the state terms, then stage dq̂ (scaled by dk^-1/2) and dk̂ rows in shared memory for the L2-norm VJP
  const float qscale = rsqrtf((float)D);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = Tw::row(r);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int j = Tw::col(c);
      const size_t x = ((size_t)(t0 + i) * H + h) * D + j;
      const float sq = i < n ? dqh[x] : 0.f, sk = i < n ? dkh[x] : 0.f;
      sm.Q[i * LD + j] = (aq[r][c] + sq) * qscale;
      sm.X[i * LD + j] = ak[r][c] + sk;
    }
  }
  __syncthreads();
  // L2-norm VJP per row: dx = r dy − r³ x (x·dy), r = rsqrt(|x|² + eps); one warp per row
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int rr = warp; rr < n; rr += NT / 32) {
    for (int which = 0; which < 2; ++which) {
      const bf16* src = which == 0 ? q : k;
      const float* dy = which == 0 ? sm.Q : sm.X;
      bf16* dst = which == 0 ? dq : dk;
      float x[D / 32], ss = 0.f, xd = 0.f;
#pragma unroll
      for (int e = 0; e < D / 32; ++e) {
        x[e] = __bfloat162float(src[((size_t)(t0 + rr) * H + h) * D + lane + 32 * e]);
        ss += x[e] * x[e];
        xd += x[e] * dy[rr * LD + lane + 32 * e];
      }
      ss = warp_sum(ss);
      xd = warp_sum(xd);
      const float r = rsqrtf(ss + kNormEps);
      const float r3 = r * r * r;
#pragma unroll
      for (int e = 0; e < D / 32; ++e)
        dst[((size_t)(t0 + rr) * H + h) * D + lane + 32 * e] =
            __float2bfloat16_rn(r * dy[rr * LD + lane + 32 * e] - r3 * x[e] * xd);
    }
  }
}

template <typename K>
void set_smem(K kernel, size_t bytes) {
  ensure_smem((const void*)kernel, (int)((int)bytes));
}

}  // namespace

// q, k, v [T, H, 128] bf16; g, beta [T, H] fp32; state [H, 128, 128] fp32.
// Returns (o, final_state, saved...) with saved = (chunk-start states, δ, T factors, P, Kd, Kb).
std::vector<at::Tensor> gdn_chunk_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                      const at::Tensor& g, const at::Tensor& beta, const at::Tensor& state) {
  check_cuda(q, "q");
  TS_CHECK(q.dim() == 3 && q.size(2) == D && k.sizes() == q.sizes() && v.sizes() == q.sizes(),
           "gdn_chunk_fwd: q, k, v must be [T, H, 128]");
  TS_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16 &&
               g.scalar_type() == at::kFloat && beta.scalar_type() == at::kFloat && state.scalar_type() == at::kFloat,
           "gdn_chunk_fwd: bf16 q/k/v, fp32 g/beta/state");
  TS_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous() && g.is_contiguous() && beta.is_contiguous() &&
               state.is_contiguous(),
           "gdn_chunk_fwd: contiguous inputs");
  const c10::cuda::CUDAGuard guard(q.device());
  const int Tn = q.size(0), H = q.size(1);
  const int nch = (Tn + C - 1) / C;
  auto f32 = q.options().dtype(at::kFloat);
  auto o = at::empty_like(v);
  auto fin = at::empty_like(state);
  auto starts = at::empty({std::max(nch, 1), H, D, D}, f32);
  auto delta = at::empty({Tn, H, D}, f32);
  auto tsv = at::empty({std::max(nch, 1), H, C, C}, f32);
  auto psv = at::empty({std::max(nch, 1), H, C, C}, f32);
  auto kd = at::empty({Tn, H, D}, f32);
  auto kb = at::empty({Tn, H, D}, f32);
  if (Tn == 0) {
    fin.copy_(state);
    return {o, fin, starts, delta, tsv, psv, kd, kb};
  }
  auto w = at::empty({Tn, H, D}, f32);
  auto u = at::empty({Tn, H, D}, f32);
  const bf16* qp = (const bf16*)q.data_ptr();
  const bf16* kp = (const bf16*)k.data_ptr();
  const bf16* vp = (const bf16*)v.data_ptr();
  set_smem(gdn_wy_kernel, sizeof(WySmem));
  gdn_wy_kernel<<<dim3(nch, H), NT, sizeof(WySmem), stream()>>>(kp, vp, g.data_ptr<float>(), beta.data_ptr<float>(),
                                                                 w.data_ptr<float>(), u.data_ptr<float>(),
                                                                 tsv.data_ptr<float>(), kd.data_ptr<float>(),
                                                                 kb.data_ptr<float>(), Tn, H);
  set_smem(gdn_state_fwd_kernel, sizeof(StateFwdSmem));
  gdn_state_fwd_kernel<<<dim3(H, D / SF), NT, sizeof(StateFwdSmem), stream()>>>(
      g.data_ptr<float>(), w.data_ptr<float>(), u.data_ptr<float>(), kd.data_ptr<float>(), state.data_ptr<float>(),
      fin.data_ptr<float>(), starts.data_ptr<float>(), delta.data_ptr<float>(), Tn, H);
  set_smem(gdn_out_kernel, sizeof(OutSmem));
  gdn_out_kernel<<<dim3(nch, H), NT, sizeof(OutSmem), stream()>>>(qp, kp, g.data_ptr<float>(), beta.data_ptr<float>(),
                                                                   delta.data_ptr<float>(), starts.data_ptr<float>(),
                                                                   (bf16*)o.data_ptr(), psv.data_ptr<float>(), Tn, H);
  TS_LAUNCH_CHECK();
  return {o, fin, starts, delta, tsv, psv, kd, kb};
}

// Returns (dq, dk, dv, dg, dbeta, dstate).
std::vector<at::Tensor> gdn_chunk_bwd(const at::Tensor& dout, const at::Tensor& dfinal, const at::Tensor& q,
                                      const at::Tensor& k, const at::Tensor& v, const at::Tensor& g,
                                      const at::Tensor& beta, const at::Tensor& starts, const at::Tensor& delta,
                                      const at::Tensor& tsv, const at::Tensor& psv, const at::Tensor& kd,
                                      const at::Tensor& kb) {
  check_cuda(q, "q");
  TS_CHECK(dout.is_contiguous() && dfinal.is_contiguous() && dout.scalar_type() == at::kBFloat16 &&
               dfinal.scalar_type() == at::kFloat && dout.sizes() == q.sizes(),
           "gdn_chunk_bwd: contiguous bf16 dout shaped like q, fp32 dfinal");
  const c10::cuda::CUDAGuard guard(q.device());
  const int Tn = q.size(0), H = q.size(1);
  const int nch = (Tn + C - 1) / C;
  auto f32 = q.options().dtype(at::kFloat);
  auto dq = at::empty_like(q);
  auto dk = at::empty_like(k);
  auto dv = at::empty_like(v);
  auto dg = at::empty({Tn, H}, f32);
  auto dbeta = at::empty({Tn, H}, f32);
  auto dstate = at::empty_like(dfinal);
  if (Tn == 0) {
    dstate.copy_(dfinal);
    return {dq, dk, dv, dg, dbeta, dstate};
  }
  auto dssv = at::empty({nch, H, D, D}, f32);
  auto x1 = at::empty({Tn, H, D}, f32);
  auto x2 = at::empty({nch, H, D, D}, f32);
  auto dz = at::empty({Tn, H, D}, f32);
  auto dqh = at::empty({Tn, H, D}, f32);
  auto dkh = at::empty({Tn, H, D}, f32);
  auto dbs = at::empty({Tn, H}, f32);
  auto dGs = at::empty({Tn, H}, f32);
  auto dgam = at::empty({nch, H}, f32);
  const bf16* qp = (const bf16*)q.data_ptr();
  const bf16* kp = (const bf16*)k.data_ptr();
  const bf16* dop = (const bf16*)dout.data_ptr();
  set_smem(gdn_bwd_pre_kernel, sizeof(BwdPreSmem));
  gdn_bwd_pre_kernel<<<dim3(nch, H), NT, sizeof(BwdPreSmem), stream()>>>(
      qp, g.data_ptr<float>(), beta.data_ptr<float>(), dop, psv.data_ptr<float>(), x1.data_ptr<float>(),
      x2.data_ptr<float>(), Tn, H);
  set_smem(gdn_state_bwd_kernel, sizeof(StateBwdSmem));
  gdn_state_bwd_kernel<<<dim3(H, D / SF), NT, sizeof(StateBwdSmem), stream()>>>(
      g.data_ptr<float>(), kd.data_ptr<float>(), kb.data_ptr<float>(), tsv.data_ptr<float>(), x1.data_ptr<float>(),
      x2.data_ptr<float>(), dfinal.data_ptr<float>(), dssv.data_ptr<float>(), dz.data_ptr<float>(),
      dstate.data_ptr<float>(), Tn, H);
  set_smem(gdn_grads_state_kernel, sizeof(GradStateSmem));
  gdn_grads_state_kernel<<<dim3(nch, H), NT, sizeof(GradStateSmem), stream()>>>(
      qp, kp, (const bf16*)v.data_ptr(), g.data_ptr<float>(), beta.data_ptr<float>(), dop, starts.data_ptr<float>(),
      dssv.data_ptr<float>(), delta.data_ptr<float>(), dz.data_ptr<float>(), dqh.data_ptr<float>(),
      dkh.data_ptr<float>(), dbs.data_ptr<float>(), dGs.data_ptr<float>(), dgam.data_ptr<float>(), Tn, H);
  set_smem(gdn_grads_local_kernel, sizeof(GradLocalSmem));
  gdn_grads_local_kernel<<<dim3(nch, H), NT, sizeof(GradLocalSmem), stream()>>>(
      qp, kp, g.data_ptr<float>(), beta.data_ptr<float>(), dop, delta.data_ptr<float>(), dz.data_ptr<float>(),
      dqh.data_ptr<float>(), dkh.data_ptr<float>(), dbs.data_ptr<float>(), dGs.data_ptr<float>(),
      dgam.data_ptr<float>(), (bf16*)dq.data_ptr(), (bf16*)dk.data_ptr(), (bf16*)dv.data_ptr(),
      dg.data_ptr<float>(), dbeta.data_ptr<float>(), Tn, H);
  TS_LAUNCH_CHECK();
  return {dq, dk, dv, dg, dbeta, dstate};
}

}  // namespace ts
