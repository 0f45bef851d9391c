// Bottom-right causal attention over a key/value chain, forward and backward.
//
// q [T, Hq, D], k/v [S, Hkv, D] (S >= T), bf16. Query i sees key j iff
// j <= i + (S - T). GQA: query head h reads KV head h / (Hq / Hkv).
// Forward writes O and the natural-log LSE [Hq, T]. Backward recomputes P from
// the LSE: one key-major pass produces dK/dV (looping over the group's query
// heads, no atomics) and one query-major pass produces dQ (no atomics), so the
// result is deterministic.
//
// Tiles: 64 queries x 64 keys per CTA step, 4 warps of 16 rows, bf16 MMAs with
// fp32 accumulation, cp.async double buffering, XOR-swizzled shared memory.
#include "common.cuh"
#include "common.h"

namespace ts {
namespace {

typedef __nv_bfloat16 bf16;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

TS_DEVICE uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

TS_DEVICE void mma16816(float* c, const uint32_t* a, const uint32_t* b) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}

TS_DEVICE void ldsm_x4(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
TS_DEVICE void ldsm_x4_t(uint32_t* r, uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

TS_DEVICE void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
TS_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> TS_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

TS_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of element (row, col) in a [rows][D] bf16 tile with 16-byte
// chunks XOR-swizzled by the row's low three bits (conflict-free ldmatrix).
template <int D> TS_DEVICE uint32_t swz(int row, int col) {
  return (uint32_t)(row * (D * 2) + ((((col >> 3) ^ (row & 7))) << 4) + ((col & 7) << 1));
}

// Async copy of `rows` rows x D from global (row stride `ld` elements) into a
// swizzled tile; rows >= limit are zero-filled.
template <int D, int ROWS, int THREADS>
TS_DEVICE void load_tile(uint32_t sbase, const bf16* g, long long ld, int row0, int limit) {
  constexpr int CH = D / 8;
#pragma unroll
  for (int c = threadIdx.x; c < ROWS * CH; c += THREADS) {
    const int r = c / CH, col = (c % CH) * 8;
    const int gr = row0 + r;
    const bool ok = gr < limit;
    const bf16* src = g + (long long)(ok ? gr : 0) * ld + col;
    cp_async16(sbase + swz<D>(r, col), src, ok);
  }
}

// ----------------------------------------------------------------------------- forward
template <int D>
__global__ void __launch_bounds__(128) attn_fwd_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                       const bf16* __restrict__ v, bf16* __restrict__ o,
                                                       float* __restrict__ lse, int T, int S, int Hq, int Hkv,
                                                       float sl2) {
  constexpr int BM = 64, BN = 64;
  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK = sQ + BM * D * 2;
  const uint32_t sV = sK + 2 * BN * D * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int q0 = blockIdx.x * BM;
  const int off = S - T;
  const long long ldq = (long long)Hq * D, ldk = (long long)Hkv * D;
  const int kv_end = min(S, q0 + BM + off);
  const int n_tiles = (kv_end + BN - 1) / BN;

  load_tile<D, BM, 128>(sQ, q + (long long)h * D, ldq, q0, T);
  load_tile<D, BN, 128>(sK, k + (long long)hk * D, ldk, 0, S);
  load_tile<D, BN, 128>(sV, v + (long long)hk * D, ldk, 0, S);
  cp_commit();

  float acc[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY}, l_r[2] = {0.f, 0.f};
  const int qr0 = q0 + warp * 16 + g;  // this thread's rows: qr0, qr0 + 8

  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) {
      const int nb = (j + 1) & 1;
      load_tile<D, BN, 128>(sK + nb * BN * D * 2, k + (long long)hk * D, ldk, (j + 1) * BN, S);
      load_tile<D, BN, 128>(sV + nb * BN * D * 2, v + (long long)hk * D, ldk, (j + 1) * BN, S);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t kb = sK + buf * BN * D * 2, vb = sV + buf * BN * D * 2;
    float s[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, sQ + swz<D>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8));
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t b[4];
        ldsm_x4(b, kb + swz<D>(np * 16 + (lane & 7) + ((lane >> 4) << 3), kk * 16 + ((lane >> 3) & 1) * 8));
        mma16816(s[2 * np], a, b);
        mma16816(s[2 * np + 1], a, b + 2);
      }
    }
    const int k0 = j * BN;
    const bool need_mask = (k0 + BN - 1 > q0 + off) || (k0 + BN > S);
    float mx[2] = {m_r[0], m_r[1]};
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[n][e] * sl2;
        if (need_mask) {
          const int key = k0 + n * 8 + 2 * tq + (e & 1);
          const int qi = qr0 + (e >> 1) * 8;
          if (key >= S || key > qi + off) x = -INFINITY;
        }
        s[n][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 1));
      mx[r] = fmaxf(mx[r], __shfl_xor_sync(0xffffffffu, mx[r], 2));
    }
    float alpha[2], ref[2];
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      ref[r] = mx[r] == -INFINITY ? 0.f : mx[r];
      alpha[r] = exp2f(m_r[r] - ref[r]);
      m_r[r] = mx[r];
      l_r[r] *= alpha[r];
    }
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      acc[i][0] *= alpha[0]; acc[i][1] *= alpha[0];
      acc[i][2] *= alpha[1]; acc[i][3] *= alpha[1];
    }
    uint32_t pa[BN / 16][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      float p0 = exp2f(s[n][0] - ref[0]), p1 = exp2f(s[n][1] - ref[0]);
      float p2 = exp2f(s[n][2] - ref[1]), p3 = exp2f(s[n][3] - ref[1]);
      l_r[0] += p0 + p1;
      l_r[1] += p2 + p3;
      pa[n >> 1][(n & 1) * 2 + 0] = pack_bf16(p0, p1);
      pa[n >> 1][(n & 1) * 2 + 1] = pack_bf16(p2, p3);
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t b[4];
        ldsm_x4_t(b, vb + swz<D>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dp * 16 + (lane >> 4) * 8));
        mma16816(acc[2 * dp], pa[kk], b);
        mma16816(acc[2 * dp + 1], pa[kk], b + 2);
      }
    }
    __syncthreads();
  }
  // epilogue
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 1);
    l_r[r] += __shfl_xor_sync(0xffffffffu, l_r[r], 2);
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qr0 + r * 8;
    if (qi >= T) continue;
    const float inv = 1.f / l_r[r];
    bf16* orow = o + (long long)qi * ldq + (long long)h * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<__nv_bfloat162*>(orow + i * 8 + 2 * tq) =
          __floats2bfloat162_rn(acc[i][2 * r] * inv, acc[i][2 * r + 1] * inv);
    }
    if (tq == 0) lse[(long long)h * T + qi] = (m_r[r] + log2f(l_r[r])) * kLn2;
  }
}

// ----------------------------------------------------------------------------- backward prep
// delta[h, i] = sum_d dO[i,h,d] * O[i,h,d]
template <int D>
__global__ void attn_bwd_delta_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout,
                                      float* __restrict__ delta, int T, int Hq) {
  const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= (long long)T * Hq) return;
  const int i = (int)(item / Hq), h = (int)(item % Hq);
  const bf16* po = o + item * D;
  const bf16* pd = dout + item * D;
  float s = 0.f;
  for (int d = lane; d < D; d += 32) s += __bfloat162float(po[d]) * __bfloat162float(pd[d]);
  s = warp_sum(s);
  if (lane == 0) delta[(long long)h * T + i] = s;
}

// ----------------------------------------------------------------------------- backward dK/dV
// CTA = 64 keys of one KV head (4 warps x 16 keys); loops over the group's
// query heads and the 32-query tiles that see these keys.
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_dkdv_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, const bf16* __restrict__ dout,
    const float* __restrict__ lse, const float* __restrict__ delta, bf16* __restrict__ dk, bf16* __restrict__ dv,
    int T, int S, int Hq, int Hkv, float scale) {
  constexpr int BN = 64, BQ = 32;
  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t sK = smem_u32(smem);
  const uint32_t sV = sK + BN * D * 2;
  const uint32_t sQ = sV + BN * D * 2;       // [2][BQ][D]
  const uint32_t sO = sQ + 2 * BQ * D * 2;   // dO [2][BQ][D]
  float* sL = reinterpret_cast<float*>(smem + (2 * BN + 4 * BQ) * D * 2);  // [2][BQ] lse*log2e
  float* sDl = sL + 2 * BQ;                                                 // [2][BQ] delta
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int hk = blockIdx.y;
  const int grp = Hq / Hkv;
  const int k0 = blockIdx.x * BN;
  const int off = S - T;
  const long long ldq = (long long)Hq * D, ldk = (long long)Hkv * D;
  const float sl2 = scale * kLog2e;

  load_tile<D, BN, 128>(sK, k + (long long)hk * D, ldk, k0, S);
  load_tile<D, BN, 128>(sV, v + (long long)hk * D, ldk, k0, S);
  cp_commit();

  float adk[D / 8][4], adv[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    adk[i][0] = adk[i][1] = adk[i][2] = adk[i][3] = 0.f;
    adv[i][0] = adv[i][1] = adv[i][2] = adv[i][3] = 0.f;
  }
  int qstart = k0 - off;
  if (qstart < 0) qstart = 0;
  qstart = (qstart / BQ) * BQ;
  const int n_qt = qstart < T ? (T - qstart + BQ - 1) / BQ : 0;
  const int total = n_qt * grp;
  const int kr0 = k0 + warp * 16 + g;  // this thread's key rows kr0, kr0 + 8

  auto issue = [&](int it, int b) {
    const int hh = hk * grp + it / n_qt;
    const int qt = qstart + (it % n_qt) * BQ;
    load_tile<D, BQ, 128>(sQ + b * BQ * D * 2, q + (long long)hh * D, ldq, qt, T);
    load_tile<D, BQ, 128>(sO + b * BQ * D * 2, dout + (long long)hh * D, ldq, qt, T);
    cp_commit();
  };
  if (total > 0) issue(0, 0);
  for (int it = 0; it < total; ++it) {
    const int b = it & 1;
    const int hh = hk * grp + it / n_qt;
    const int qt = qstart + (it % n_qt) * BQ;
    if (threadIdx.x < BQ) {
      const int qi = qt + threadIdx.x;
      sL[b * BQ + threadIdx.x] = qi < T ? lse[(long long)hh * T + qi] * kLog2e : 0.f;
      sDl[b * BQ + threadIdx.x] = qi < T ? delta[(long long)hh * T + qi] : 0.f;
    }
    if (it + 1 < total) {
      issue(it + 1, b ^ 1);
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t qb = sQ + b * BQ * D * 2, ob = sO + b * BQ * D * 2;
    // S^T = K Q^T : 16 keys x 32 queries per warp
    float st[BQ / 8][4], dpt[BQ / 8][4];
#pragma unroll
    for (int n = 0; n < BQ / 8; ++n) {
      st[n][0] = st[n][1] = st[n][2] = st[n][3] = 0.f;
      dpt[n][0] = dpt[n][1] = dpt[n][2] = dpt[n][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t ak[4], av[4];
      ldsm_x4(ak, sK + swz<D>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8));
      ldsm_x4(av, sV + swz<D>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8));
#pragma unroll
      for (int np = 0; np < BQ / 16; ++np) {
        uint32_t bq[4], bo[4];
        const int rr = np * 16 + (lane & 7) + ((lane >> 4) << 3), cc = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bq, qb + swz<D>(rr, cc));
        ldsm_x4(bo, ob + swz<D>(rr, cc));
        mma16816(st[2 * np], ak, bq);
        mma16816(st[2 * np + 1], ak, bq + 2);
        mma16816(dpt[2 * np], av, bo);
        mma16816(dpt[2 * np + 1], av, bo + 2);
      }
    }
    // P^T and dS^T
    uint32_t pa[BQ / 16][4], da[BQ / 16][4];
#pragma unroll
    for (int n = 0; n < BQ / 8; ++n) {
      float p[4], ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int qc = n * 8 + 2 * tq + (e & 1);  // query column within tile
        const int qi = qt + qc;
        const int key = kr0 + (e >> 1) * 8;
        const bool ok = qi < T && key < S && key <= qi + off;
        p[e] = ok ? exp2f(st[n][e] * sl2 - sL[b * BQ + qc]) : 0.f;
        ds[e] = p[e] * (dpt[n][e] - sDl[b * BQ + qc]);
      }
      pa[n >> 1][(n & 1) * 2 + 0] = pack_bf16(p[0], p[1]);
      pa[n >> 1][(n & 1) * 2 + 1] = pack_bf16(p[2], p[3]);
      da[n >> 1][(n & 1) * 2 + 0] = pack_bf16(ds[0], ds[1]);
      da[n >> 1][(n & 1) * 2 + 1] = pack_bf16(ds[2], ds[3]);
    }
    // dV += P^T dO ; dK += dS^T Q
#pragma unroll
    for (int kk = 0; kk < BQ / 16; ++kk) {
#pragma unroll
      for (int dp = 0; dp < D / 16; ++dp) {
        uint32_t bo[4], bq[4];
        const int rr = kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, cc = dp * 16 + (lane >> 4) * 8;
        ldsm_x4_t(bo, ob + swz<D>(rr, cc));
        ldsm_x4_t(bq, qb + swz<D>(rr, cc));
        mma16816(adv[2 * dp], pa[kk], bo);
        mma16816(adv[2 * dp + 1], pa[kk], bo + 2);
        mma16816(adk[2 * dp], da[kk], bq);
        mma16816(adk[2 * dp + 1], da[kk], bq + 2);
      }
    }
    __syncthreads();
  }
  if (total == 0) cp_wait<0>();
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int key = kr0 + r * 8;
    if (key >= S) continue;
    bf16* pk = dk + (long long)key * ldk + (long long)hk * D;
    bf16* pv = dv + (long long)key * ldk + (long long)hk * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<__nv_bfloat162*>(pk + i * 8 + 2 * tq) =
          __floats2bfloat162_rn(adk[i][2 * r] * scale, adk[i][2 * r + 1] * scale);
      *reinterpret_cast<__nv_bfloat162*>(pv + i * 8 + 2 * tq) =
          __floats2bfloat162_rn(adv[i][2 * r], adv[i][2 * r + 1]);
    }
  }
}

// ----------------------------------------------------------------------------- backward dQ
template <int D>
__global__ void __launch_bounds__(128) attn_bwd_dq_kernel(const bf16* __restrict__ q, const bf16* __restrict__ k,
                                                          const bf16* __restrict__ v, const bf16* __restrict__ dout,
                                                          const float* __restrict__ lse,
                                                          const float* __restrict__ delta, bf16* __restrict__ dq,
                                                          int T, int S, int Hq, int Hkv, float scale) {
  constexpr int BM = 64, BN = 64;
  extern __shared__ __align__(128) unsigned char smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sO = sQ + BM * D * 2;
  const uint32_t sK = sO + BM * D * 2;  // [2][BN][D]
  const uint32_t sV = sK + 2 * BN * D * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int q0 = blockIdx.x * BM;
  const int off = S - T;
  const long long ldq = (long long)Hq * D, ldk = (long long)Hkv * D;
  const float sl2 = scale * kLog2e;
  const int kv_end = min(S, q0 + BM + off);
  const int n_tiles = (kv_end + BN - 1) / BN;
  const int qr0 = q0 + warp * 16 + g;

  load_tile<D, BM, 128>(sQ, q + (long long)h * D, ldq, q0, T);
  load_tile<D, BM, 128>(sO, dout + (long long)h * D, ldq, q0, T);
  load_tile<D, BN, 128>(sK, k + (long long)hk * D, ldk, 0, S);
  load_tile<D, BN, 128>(sV, v + (long long)hk * D, ldk, 0, S);
  cp_commit();
  float L[2], Dl[2];
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qr0 + r * 8;
    L[r] = qi < T ? lse[(long long)h * T + qi] * kLog2e : 0.f;
    Dl[r] = qi < T ? delta[(long long)h * T + qi] : 0.f;
  }
  float adq[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) adq[i][0] = adq[i][1] = adq[i][2] = adq[i][3] = 0.f;

  for (int j = 0; j < n_tiles; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_tiles) {
      const int nb = (j + 1) & 1;
      load_tile<D, BN, 128>(sK + nb * BN * D * 2, k + (long long)hk * D, ldk, (j + 1) * BN, S);
      load_tile<D, BN, 128>(sV + nb * BN * D * 2, v + (long long)hk * D, ldk, (j + 1) * BN, S);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    const uint32_t kb = sK + buf * BN * D * 2, vb = sV + buf * BN * D * 2;
    float s[BN / 8][4], dp[BN / 8][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
      dp[n][0] = dp[n][1] = dp[n][2] = dp[n][3] = 0.f;
    }
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t aq[4], ao[4];
      ldsm_x4(aq, sQ + swz<D>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8));
      ldsm_x4(ao, sO + swz<D>(warp * 16 + (lane & 15), kk * 16 + (lane >> 4) * 8));
#pragma unroll
      for (int np = 0; np < BN / 16; ++np) {
        uint32_t bk[4], bv[4];
        const int rr = np * 16 + (lane & 7) + ((lane >> 4) << 3), cc = kk * 16 + ((lane >> 3) & 1) * 8;
        ldsm_x4(bk, kb + swz<D>(rr, cc));
        ldsm_x4(bv, vb + swz<D>(rr, cc));
        mma16816(s[2 * np], aq, bk);
        mma16816(s[2 * np + 1], aq, bk + 2);
        mma16816(dp[2 * np], ao, bv);
        mma16816(dp[2 * np + 1], ao, bv + 2);
      }
    }
    const int k0 = j * BN;
    uint32_t da[BN / 16][4];
#pragma unroll
    for (int n = 0; n < BN / 8; ++n) {
      float ds[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = k0 + n * 8 + 2 * tq + (e & 1);
        const int qi = qr0 + (e >> 1) * 8;
        const bool ok = key < S && key <= qi + off && qi < T;
        const float p = ok ? exp2f(s[n][e] * sl2 - L[e >> 1]) : 0.f;
        ds[e] = p * (dp[n][e] - Dl[e >> 1]);
      }
      da[n >> 1][(n & 1) * 2 + 0] = pack_bf16(ds[0], ds[1]);
      da[n >> 1][(n & 1) * 2 + 1] = pack_bf16(ds[2], ds[3]);
    }
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
#pragma unroll
      for (int dpi = 0; dpi < D / 16; ++dpi) {
        uint32_t b[4];
        ldsm_x4_t(b, kb + swz<D>(kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8, dpi * 16 + (lane >> 4) * 8));
        mma16816(adq[2 * dpi], da[kk], b);
        mma16816(adq[2 * dpi + 1], da[kk], b + 2);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 2; ++r) {
    const int qi = qr0 + r * 8;
    if (qi >= T) continue;
    bf16* pq = dq + (long long)qi * ldq + (long long)h * D;
#pragma unroll
    for (int i = 0; i < D / 8; ++i) {
      *reinterpret_cast<__nv_bfloat162*>(pq + i * 8 + 2 * tq) =
          __floats2bfloat162_rn(adq[i][2 * r] * scale, adq[i][2 * r + 1] * scale);
    }
  }
}

template <int D>
void fwd_launch(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
                float scale) {
  const int T = q.size(0), Hq = q.size(1), S = k.size(0), Hkv = k.size(1);
  const int smem = (64 + 4 * 64) * D * 2;
  auto kern = attn_fwd_kernel<D>;
  ensure_smem((const void*)kern, (int)(smem));
  dim3 grid((T + 63) / 64, Hq);
  kern<<<grid, 128, smem, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(),
                                      (const bf16*)v.data_ptr(), (bf16*)o.data_ptr(), lse.data_ptr<float>(), T, S, Hq,
                                      Hkv, scale * kLog2e);
}

template <int D>
void bwd_launch(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                const at::Tensor& o, const at::Tensor& lse, at::Tensor& dq, at::Tensor& dk, at::Tensor& dv,
                float scale) {
  const int T = q.size(0), Hq = q.size(1), S = k.size(0), Hkv = k.size(1);
  auto delta = at::empty({Hq, T}, q.options().dtype(at::kFloat));
  const long long items = (long long)T * Hq;
  attn_bwd_delta_kernel<D><<<(int)((items + 7) / 8), 256, 0, stream()>>>(
      (const bf16*)o.data_ptr(), (const bf16*)dout.data_ptr(), delta.data_ptr<float>(), T, Hq);
  {
    const int smem = (2 * 64 + 4 * 32) * D * 2 + 4 * 32 * 4;
    auto kern = attn_bwd_dkdv_kernel<D>;
    ensure_smem((const void*)kern, (int)(smem));
    dim3 grid((S + 63) / 64, Hkv);
    kern<<<grid, 128, smem, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(),
                                        (const bf16*)v.data_ptr(), (const bf16*)dout.data_ptr(),
                                        lse.data_ptr<float>(), delta.data_ptr<float>(), (bf16*)dk.data_ptr(),
                                        (bf16*)dv.data_ptr(), T, S, Hq, Hkv, scale);
  }
  {
    const int smem = (2 * 64 + 4 * 64) * D * 2;
    auto kern = attn_bwd_dq_kernel<D>;
    ensure_smem((const void*)kern, (int)(smem));
    dim3 grid((T + 63) / 64, Hq);
    kern<<<grid, 128, smem, stream()>>>((const bf16*)q.data_ptr(), (const bf16*)k.data_ptr(),
                                        (const bf16*)v.data_ptr(), (const bf16*)dout.data_ptr(),
                                        lse.data_ptr<float>(), delta.data_ptr<float>(), (bf16*)dq.data_ptr(), T, S,
                                        Hq, Hkv, scale);
  }
}

void check_attn(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  check_cuda(q, "q");
  check_cuda(k, "k");
  check_cuda(v, "v");
  TS_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
           "attention runs in bf16");
  TS_CHECK(q.dim() == 3 && k.dim() == 3 && v.dim() == 3, "attention expects [T,H,D] tensors");
  TS_CHECK(k.sizes() == v.sizes(), "k and v shapes differ");
  TS_CHECK(q.size(2) == k.size(2), "head dims differ");
  TS_CHECK(q.size(1) % k.size(1) == 0, "query heads must be a multiple of KV heads");
  TS_CHECK(k.size(0) >= q.size(0), "bottom-right attention needs S >= T");
}

}  // namespace

std::vector<at::Tensor> attn_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale) {
  check_attn(q, k, v);
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = at::empty_like(q);
  auto lse = at::empty({q.size(1), q.size(0)}, q.options().dtype(at::kFloat));
  if (q.size(0) == 0) return {o, lse};
  const int D = q.size(2);
  if (D == 64) fwd_launch<64>(q, k, v, o, lse, (float)scale);
  else if (D == 128) fwd_launch<128>(q, k, v, o, lse, (float)scale);
  else TS_CHECK(false, "attention head_dim ", D, " unsupported (64, 128)");
  TS_LAUNCH_CHECK();
  return {o, lse};
}

std::vector<at::Tensor> attn_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                 const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, double scale) {
  check_attn(q, k, v);
  check_cuda(dout, "dout");
  check_cuda(o, "o");
  const c10::cuda::CUDAGuard guard(q.device());
  auto dq = at::empty_like(q);
  auto dk = at::empty_like(k);
  auto dv = at::empty_like(v);
  if (q.size(0) == 0) return {dq, dk.zero_(), dv.zero_()};
  const int D = q.size(2);
  if (D == 64) bwd_launch<64>(dout, q, k, v, o, lse, dq, dk, dv, (float)scale);
  else if (D == 128) bwd_launch<128>(dout, q, k, v, o, lse, dq, dk, dv, (float)scale);
  else TS_CHECK(false, "attention head_dim ", D, " unsupported (64, 128)");
  TS_LAUNCH_CHECK();
  return {dq, dk, dv};
}

}  // namespace ts
