// Bottom-right causal attention forward on the 5th-generation tensor cores.
//
// One CTA computes a 128-query tile of one head (SW = 2 softmax warps per
// 32-row slab):
//   warp 4*SW    TMA producer: Q once, then K/V key tiles through a 2-stage
//                ring (128B-swizzled boxes of 64 columns)
//   warp 4*SW+1  MMA issuer (one thread): S = Q K^T into one of two TMEM
//                S buffers, O += P V into the TMEM O accumulator; commits
//                signal the other roles through mbarriers
//   warps 0..4*SW-1  softmax: the SW warps of a TMEM sub-partition share its
//                32 query rows and split each tile's key columns; each reads
//                its part of the S row, the partial maxima are exchanged
//                through shared memory (an mbarrier per slab), each
//                exponentiates its part (online max/sum in the log2 domain,
//                bottom-right mask) and writes P back into tensor memory as
//                bf16 pairs over the S columns it read -- the A operand of
//                O += P V -- and rescales its part of the O row only when the
//                row max moved
// The tensor core computes S(j+1) while the softmax warps work on S(j), and
// PV(j) while they work on S(j+1). Epilogue: O / l (bf16) and the natural-log
// LSE. Every mbarrier wait is bounded (see tc.cuh).
//
// Also here: a one-tile UMMA self-test (D = A B^T with K-major B and D = A B
// with MN-major B) that validates the descriptor encodings on the device.
#include <cudaTypedefs.h>

#include "common.h"
#include "tc.cuh"

namespace ts {
namespace {

typedef __nv_bfloat16 bf16;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 2^x with the SM's native ex2 unit (flush-to-zero); inputs here are <= 0 after the
// max/LSE shift, and outputs below the normal range contribute nothing in bf16.
TS_DEVICE float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
TS_DEVICE uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// One-lane wait, result broadcast so the whole warp agrees.
TS_DEVICE bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* err, int code) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = tc::mbar_wait(bar, parity, abort, err, code);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

// ------------------------------------------------------------------ packed (variable-length) work tables
// A pack holds several segments; queries of segment s are rows [q0_s, q0_s + T_s) of Q, and its keys are
// rows of one key buffer: zero or more *far* ranges (ancestors every query of s sees) and one *near* range
// whose key b is visible to local query i iff b <= i + off (bottom-right causal; off = length of an
// ancestor prefix stored right before the own keys, 0 when the own keys stand alone).
//
// Query-side item (forward and dQ; one per segment and BM-query tile), 8 ints:
//   q_row0 (Q row of the tile's first query), q_loc0 (its index within the segment), T, near_row0, off,
//   far0, nfar (slice of the far-range table, int2 {row0, len}), unused.
// Key-side item (dK/dV; one per key tile), 4 ints: k_row0, cnt (keys in the tile), cons0, ncons (slice of
// the consumer table). Consumer (4 ints): q_row0 and T of a segment whose queries read this tile, and
// vis_base: key row r of the tile is visible to that segment's local query i iff i >= vis_base + r
// (kFullVis: every query sees every key). A key tile lies inside one range with one consumer set, so a
// shared ancestor's dK/dV sum over every segment that reads it inside one CTA, without atomics.
// A launch without tables is the single-segment case: item = BM-tile of [0, T), near range = [0, S) with
// off = S - T, one consumer per key tile.
struct QItem {
  int q_row0, q_loc0, T, near_row0, off, far0, nfar, pad;
};
struct KItem {
  int k_row0, cnt, cons0, ncons;
};
constexpr int kFullVis = -(1 << 30);

TS_DEVICE QItem load_qitem(const int* tab, int idx) {
  const int4* p = reinterpret_cast<const int4*>(tab) + 2 * idx;
  const int4 a = p[0], b = p[1];
  return QItem{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
}
TS_DEVICE QItem dense_qitem(int BM, int T, int S) {
  const int n_qt = (T + BM - 1) / BM;
  const int qt = n_qt - 1 - (int)blockIdx.x;  // longest tiles first
  return QItem{qt * BM, qt * BM, T, 0, S - T, 0, 0, 0};
}

// The key tiles a query item visits, in order: every far range in BN-key tiles, then the near range up to
// the tile's last query. One walker per role; next() moves to the following tile.
template <int BN>
struct KeyWalk {
  const int2* far;
  int nfar, near_row0, off, T;
  int f, jj, row0, len;

  TS_DEVICE void init(const QItem& it, const int2* far_tab) {
    far = far_tab + it.far0;
    nfar = it.nfar;
    near_row0 = it.near_row0;
    off = it.off;
    T = it.T;
    f = 0;
    jj = 0;
    load();
  }
  TS_DEVICE void load() {
    while (f < nfar) {
      const int2 r = far[f];
      if (r.y > 0) {
        row0 = r.x;
        len = r.y;
        return;
      }
      ++f;
    }
    row0 = near_row0;
    len = off + T;
  }
  TS_DEVICE void next() {
    ++jj;
    if (f < nfar && jj * BN >= len) {
      ++f;
      jj = 0;
      load();
    }
  }
  TS_DEVICE int row() const { return row0 + jj * BN; }
  // keys of the current tile visible to local query qi (< T)
  TS_DEVICE int nvis(int qi) const {
    if (f < nfar) return min(BN, len - jj * BN);
    const int v = min(qi + off, off + T - 1) - jj * BN + 1;
    return v < 0 ? 0 : (v > BN ? BN : v);
  }
  // tiles for an item whose queries end at local index q_end (exclusive)
  TS_DEVICE int count(int q_end) const {
    int n = 0;
    for (int i = 0; i < nfar; ++i) n += (far[i].y + BN - 1) / BN;
    const int kv_end = min(off + T, off + q_end);
    return n + (kv_end + BN - 1) / BN;
  }
};

// Consumers of one key tile and the (head, consumer, query tile) steps a dK/dV CTA runs over them, heads
// outermost. Without a consumer table the single consumer is the one given to init.
template <int BQ>
struct StepWalk {
  const int4* cons;
  int ncons, hh, c, t, qstart, nqt;
  int4 cur;  // {q_row0, T, vis_base, 0} of the current consumer

  TS_DEVICE int4 consumer(int i) const { return cons != nullptr ? cons[i] : cur; }
  TS_DEVICE static int first_tile(int vis_base) {
    const int s = vis_base < 0 ? 0 : vis_base;
    return (s / BQ) * BQ;
  }
  TS_DEVICE static int tiles(const int4& cn) {
    const int s = first_tile(cn.z);
    return s < cn.y ? (cn.y - s + BQ - 1) / BQ : 0;
  }
  TS_DEVICE void init(const int4* cons_tab, int n, int4 dense_cons, int grp) {
    cons = cons_tab;
    ncons = n;
    cur = dense_cons;
    hh = 0;
    c = -1;
    t = 0;
    nqt = 0;
    advance_consumer(grp);
  }
  TS_DEVICE void advance_consumer(int grp) {
    for (;;) {
      ++c;
      if (c >= ncons) {
        c = 0;
        ++hh;
        if (hh >= grp || ncons == 0) return;
      }
      cur = consumer(c);
      nqt = tiles(cur);
      qstart = first_tile(cur.z);
      t = 0;
      if (nqt > 0) return;
    }
  }
  TS_DEVICE int per_head() const {
    int n = 0;
    for (int i = 0; i < ncons; ++i) n += tiles(consumer(i));
    return n;
  }
  TS_DEVICE void next(int grp) {
    ++t;
    if (t >= nqt) advance_consumer(grp);
  }
  TS_DEVICE int q_loc() const { return qstart + t * BQ; }  // local index of the step's first query
  TS_DEVICE int q_row() const { return cur.x + q_loc(); }  // its row in Q / dO
};

template <int D>
struct FwdLayout {
  // D = 256 halves the key tile so two K/V stages still fit in shared memory
  static constexpr int BM = 128, BN = D <= 128 ? 128 : 64;
  // softmax warps per TMEM sub-partition (32 query rows): each takes CW = BN / SW key columns of a tile and
  // D / SW columns of the O row. Two: four (16 softmax warps, 576 threads) measured 6-7% slower at head_dim
  // 128 (377 vs 403 TFLOP/s at T=2176, 586 vs 619 at T=9288).
  static constexpr int SW = 2;
  static constexpr int CW = BN / SW;
  static constexpr int SOFT = 4 * SW;                 // softmax warps
  static constexpr int PROD = SOFT, MMA = SOFT + 1;   // producer and MMA warps
  static constexpr int THREADS = 32 * (SOFT + 2);
  static constexpr int NB = D / 64;    // 64-column boxes per row
  static constexpr uint32_t Q = 0;
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t K_BYTES = BN * D * 2;
  static constexpr uint32_t K0 = Q + Q_BYTES;
  static constexpr uint32_t V0 = K0 + 2 * K_BYTES;
  static constexpr uint32_t BAR = V0 + 2 * K_BYTES;
  static constexpr uint32_t RED = BAR + 256;             // [SW][128] floats: the partial row sums
  static constexpr uint32_t XMAX = RED + SW * 512;       // [2 tile parities][SW][128] floats: partial row maxima
  static constexpr uint32_t TOTAL = XMAX + 2 * SW * 512;
  // TMEM columns: two S buffers (P is written back over the S columns its warp read, as bf16 pairs, and is
  // the A operand of O += P V from there) and the O accumulator
  static constexpr uint32_t S_COL0 = 0, S_COL1 = 128, O_COL = 256;
  // TMEM column of the A operand for the kk-th 16-key step of P: part w = kk*16 / CW lives at
  // S + w*CW (CW / 2 columns of bf16 pairs)
  static TS_DEVICE uint32_t p_col(int kk) { return (kk * 16 / CW) * CW + ((kk * 16) % CW) / 2; }
};
static_assert(FwdLayout<256>::TOTAL + 1024 <= 232448, "forward shared memory exceeds 227 KB");

struct FwdBars {
  uint64_t q, k_full[2], v_full[2], kv_empty[2], s_full[2], p_full[2], pv[2];
  uint64_t xbar[4][2];  // per TMEM sub-partition and tile parity: every warp of the row slab posted its max
  uint32_t tmem_slot;
  int abort;
};

static_assert(sizeof(FwdBars) <= 256, "forward barrier block");

template <int D>
__global__ void __launch_bounds__(FwdLayout<D>::THREADS, 1) attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tm_q,
                                                             const __grid_constant__ CUtensorMap tm_k,
                                                             const __grid_constant__ CUtensorMap tm_v,
                                                             bf16* __restrict__ out, float* __restrict__ lse,
                                                             int T_in, int S_in, int Hq, int Hkv, float sl2,
                                                             const int* __restrict__ qtab,
                                                             const int2* __restrict__ far_tab, int Ttot,
                                                             int* __restrict__ err) {
  using L = FwdLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FwdBars* bars = reinterpret_cast<FwdBars*>(smem + L::BAR);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const QItem it = qtab != nullptr ? load_qitem(qtab, blockIdx.x) : dense_qitem(L::BM, T_in, S_in);
  const int T = it.T;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int q0 = it.q_loc0;  // local index of the tile's first query
  KeyWalk<L::BN> walk;
  walk.init(it, far_tab);
  const int n = walk.count(q0 + L::BM);
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->q, 1);
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bars->k_full[i], 1);
      tc::mbar_init(&bars->v_full[i], 1);
      tc::mbar_init(&bars->kv_empty[i], 1);
      tc::mbar_init(&bars->s_full[i], 1);
      tc::mbar_init(&bars->p_full[i], 32 * L::SOFT);
      tc::mbar_init(&bars->pv[i], 1);
    }
    for (int i = 0; i < 4; ++i) {
      tc::mbar_init(&bars->xbar[i][0], 32 * L::SW);
      tc::mbar_init(&bars->xbar[i][1], 32 * L::SW);
    }
    bars->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == L::MMA) tc::tmem_alloc(&bars->tmem_slot, 512);
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == L::PROD) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tc::prefetch_tmap(&tm_q);
      tc::prefetch_tmap(&tm_k);
      tc::prefetch_tmap(&tm_v);
      tc::mbar_expect_tx(&bars->q, L::Q_BYTES);
      for (int b = 0; b < L::NB; ++b)
        tc::tma_load_2d(smem + L::Q + b * L::BM * 128, &tm_q, h * D + b * 64, it.q_row0, &bars->q);
      for (int j = 0; j < n; ++j, walk.next()) {
        const int s = j & 1;
        if (j >= 2 && !tc::mbar_wait(&bars->kv_empty[s], ((j - 2) >> 1) & 1, abort, err, 11)) break;
        const int krow = walk.row();
        tc::mbar_expect_tx(&bars->k_full[s], L::K_BYTES);
        for (int b = 0; b < L::NB; ++b)
          tc::tma_load_2d(smem + L::K0 + s * L::K_BYTES + b * L::BN * 128, &tm_k, hk * D + b * 64, krow,
                          &bars->k_full[s]);
        tc::mbar_expect_tx(&bars->v_full[s], L::K_BYTES);
        for (int b = 0; b < L::NB; ++b)
          tc::tma_load_2d(smem + L::V0 + s * L::K_BYTES + b * L::BN * 128, &tm_v, hk * D + b * 64, krow,
                          &bars->v_full[s]);
      }
    }
  } else if (warp == L::MMA) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_bf16(128, L::BN, false, false);
      const uint32_t id_o = tc::idesc_bf16(128, D, false, true);
      bool ok = tc::mbar_wait(&bars->q, 0, abort, err, 21);
      auto issue_s = [&](int j) -> bool {
        const int s = j & 1;
        if (!tc::mbar_wait(&bars->k_full[s], (j >> 1) & 1, abort, err, 22)) return false;
        tc::tc_fence_after();
        const uint32_t kb = sbase + L::K0 + s * L::K_BYTES;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t qoff = (kk >> 2) * L::BM * 128 + (kk & 3) * 32;
          const uint32_t koff = (kk >> 2) * L::BN * 128 + (kk & 3) * 32;
          const uint64_t a = tc::sdesc_sw128(sbase + L::Q + qoff, 16, 1024);
          const uint64_t b = tc::sdesc_sw128(kb + koff, 16, 1024);
          tc::mma_bf16(tmem + (s ? L::S_COL1 : L::S_COL0), a, b, id_s, kk > 0);
        }
        tc::mma_commit(&bars->s_full[s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n > 1) ok = issue_s(1);
      for (int j = 0; ok && j < n; ++j) {
        const int s = j & 1;
        if (!tc::mbar_wait(&bars->p_full[s], (j >> 1) & 1, abort, err, 23)) break;
        if (!tc::mbar_wait(&bars->v_full[s], (j >> 1) & 1, abort, err, 24)) break;
        tc::tc_fence_after();
        const uint32_t pcol = tmem + (s ? L::S_COL1 : L::S_COL0);
        const uint32_t vb = sbase + L::V0 + s * L::K_BYTES;
#pragma unroll
        for (int kk = 0; kk < L::BN / 16; ++kk) {
          const uint64_t b = tc::sdesc_sw128(vb + kk * 16 * 128, L::BN * 128, 1024);
          tc::mma_bf16_ts(tmem + L::O_COL, pcol + L::p_col(kk), b, id_o, j > 0 || kk > 0);
        }
        tc::mma_commit(&bars->pv[s]);
        tc::mma_commit(&bars->kv_empty[s]);
        if (j + 2 < n) ok = issue_s(j + 2);
      }
    }
  } else {
    // ------------------------------------------------------------ softmax (warps 0 .. SOFT-1)
    // warp w owns the rows of TMEM sub-partition (w & 3) and part pw = w >> 2 of each tile: key columns
    // [pw*CW, +CW) and O columns [pw*D/SW, +D/SW). The SW warps of a row slab exchange their partial maxima
    // per tile and their partial sums at the end through shared memory.
    const int r = (warp & 3) * 32 + lane;
    const int pw = warp >> 2;
    const int qi = q0 + r;  // local query index (rows at or past T belong to the next segment: not stored)
    const uint32_t lane_base = tmem + ((uint32_t)((warp & 3) * 32) << 16);
    constexpr int OCH = D / (32 * L::SW);  // 32-column chunks of the O row per warp
    float* lsum = reinterpret_cast<float*>(smem + L::RED);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    float* xmax = reinterpret_cast<float*>(smem + L::XMAX);
    uint64_t* xbar = bars->xbar[warp & 3];
    for (int j = 0; j < n && ok; ++j, walk.next()) {
      const int s = j & 1;
      if (!warp_wait(&bars->s_full[s], (j >> 1) & 1, abort, err, 31)) { ok = false; break; }
      tc::tc_fence_after();
      // this warp's part of the tile's columns
      float sv[L::CW];
      const uint32_t scol = s ? L::S_COL1 : L::S_COL0;
      const uint32_t pcol = lane_base + scol + pw * L::CW;
#pragma unroll
      for (int c = 0; c < L::CW; c += 32) tc::tmem_ld<(L::CW < 32 ? L::CW : 32)>(pcol + c, sv + c);
      tc::tmem_ld_wait();
      const int nv_part = walk.nvis(qi) - pw * L::CW;  // visible columns of this warp's part for this row
      // partial row max as 8 independent chains (a single fmaxf chain serialises on the instruction latency)
      float mx8[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) mx8[e] = -INFINITY;
      if (nv_part >= L::CW) {
#pragma unroll
        for (int i = 0; i < L::CW; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], sv[i]);
      } else {
#pragma unroll
        for (int i = 0; i < L::CW; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], i < nv_part ? sv[i] : -INFINITY);
      }
      const float pmax = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                               fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      // the slab's other warps post their partial maxima; all of them then hold the same row max
      xmax[(s * L::SW + pw) * 128 + r] = pmax;
      tc::mbar_arrive(&xbar[s]);
      if (!warp_wait(&xbar[s], (j >> 1) & 1, abort, err, 35)) { ok = false; break; }
      float raw = xmax[(s * L::SW) * 128 + r];
#pragma unroll
      for (int w2 = 1; w2 < L::SW; ++w2) raw = fmaxf(raw, xmax[(s * L::SW + w2) * 128 + r]);
      // the exponent reference moves only when the running max grows by more than 8 (a factor 2^8): P
      // stays <= 256 (exact in bf16's range, and the fp32 sums absorb it), and O is rescaled only then
      const float cand = fmaxf(m, raw * sl2);
      const bool bump = cand > m + 8.f;
      const float mx = bump ? cand : m;
      const float ref = mx == -INFINITY ? 0.f : mx;
      const float alpha = bump ? ex2(m - ref) : 1.f;
      // P of this part, as bf16 pairs over the first CW / 2 columns of the same part of S (columns this warp
      // has already read; the S(j + 2) MMA that next writes them is issued after PV(j) has read them)
      float rs8[8];  // 8 independent partial sums, for the same reason as the max
#pragma unroll
      for (int e = 0; e < 8; ++e) rs8[e] = 0.f;
      float pv_[L::CW / 2];
#pragma unroll
      for (int c8 = 0; c8 < L::CW / 8; ++c8) {
        float p[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int i = c8 * 8 + e;
          p[e] = i < nv_part ? ex2(fmaf(sv[i], sl2, -ref)) : 0.f;
          rs8[e] += p[e];
        }
#pragma unroll
        for (int q2 = 0; q2 < 4; ++q2) pv_[c8 * 4 + q2] = __uint_as_float(pack2(p[2 * q2], p[2 * q2 + 1]));
      }
      if constexpr (L::CW / 2 == 32) tc::tmem_st32(pcol, pv_);
      else tc::tmem_st16(pcol, pv_);
      const float rs = ((rs8[0] + rs8[1]) + (rs8[2] + rs8[3])) + ((rs8[4] + rs8[5]) + (rs8[6] + rs8[7]));
      l = l * alpha + rs;
      if (j > 0 && __any_sync(0xffffffffu, alpha < 1.f)) {
        if (!warp_wait(&bars->pv[(j - 1) & 1], ((j - 1) >> 1) & 1, abort, err, 32)) { ok = false; break; }
        tc::tc_fence_after();
#pragma unroll
        for (int c = pw * OCH; c < (pw + 1) * OCH; ++c) {
          float o[32];
          tc::tmem_ld32(lane_base + L::O_COL + c * 32, o);
          tc::tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tc::tmem_st32(lane_base + L::O_COL + c * 32, o);
        }
      }
      tc::tmem_st_wait();
      m = mx;
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->p_full[s]);
    }
    // the slab's partial sums: exchanged once through shared memory
    lsum[pw * 128 + r] = l;
    asm volatile("bar.sync 1, %0;\n" ::"n"(32 * L::SOFT) : "memory");
    float lt = lsum[r];
#pragma unroll
    for (int w2 = 1; w2 < L::SW; ++w2) lt += lsum[w2 * 128 + r];
    if (ok && warp_wait(&bars->pv[(n - 1) & 1], ((n - 1) >> 1) & 1, abort, err, 33)) {
      tc::tc_fence_after();
      const float inv = 1.f / lt;
#pragma unroll
      for (int c = pw * OCH; c < (pw + 1) * OCH; ++c) {
        float o[32];
        tc::tmem_ld32(lane_base + L::O_COL + c * 32, o);
        tc::tmem_ld_wait();
        if (qi < T) {
          bf16* dst = out + ((long long)(it.q_row0 + r) * Hq + h) * D + c * 32;
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            uint4 v;
            v.x = pack2(o[i] * inv, o[i + 1] * inv);
            v.y = pack2(o[i + 2] * inv, o[i + 3] * inv);
            v.z = pack2(o[i + 4] * inv, o[i + 5] * inv);
            v.w = pack2(o[i + 6] * inv, o[i + 7] * inv);
            *reinterpret_cast<uint4*>(dst + i) = v;
          }
        }
      }
      if (qi < T && pw == 0) lse[(long long)h * Ttot + it.q_row0 + r] = (m + log2f(lt)) * kLn2;
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == L::MMA) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ backward
// delta[h, i] = sum_d dO[i,h,d] * O[i,h,d] (fp32), one warp per (i, h).
__global__ void attn_delta_kernel(const bf16* __restrict__ o, const bf16* __restrict__ dout, float* __restrict__ delta,
                                  int T, int Hq, int D) {
  const long long item = (long long)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (item >= (long long)T * Hq) return;
  const int i = (int)(item / Hq), h = (int)(item % Hq);
  const bf16* po = o + item * D;
  const bf16* pd = dout + item * D;
  float s = 0.f;
  for (int d = lane * 2; d < D; d += 64) {
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(po + d));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(pd + d));
    s += a.x * b.x + a.y * b.y;
  }
  s = warp_sum(s);
  if (lane == 0) delta[(long long)h * T + i] = s;
}

// Sum of the per-split fp32 dK/dV partials in split order, scaled and rounded to bf16.
__global__ void attn_split_sum_kernel(const float* __restrict__ part, bf16* __restrict__ out, long long n,
                                      int nsplit, float scale) {
  const long long i4 = (blockIdx.x * (long long)blockDim.x + threadIdx.x) * 4;
  if (i4 >= n) return;
  float4 acc = *reinterpret_cast<const float4*>(part + i4);
  for (int z = 1; z < nsplit; ++z) {
    const float4 v = *reinterpret_cast<const float4*>(part + (long long)z * n + i4);
    acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
  }
  uint2 o;
  o.x = pack2(acc.x * scale, acc.y * scale);
  o.y = pack2(acc.z * scale, acc.w * scale);
  *reinterpret_cast<uint2*>(out + i4) = o;
}

// dK/dV for head dims 64 and 128 with 128-query steps (every MMA is 128 x 128 x 16 or wider: narrower MMAs
// leave the tensor pipe idle between instructions). Per step (query head, 128-query tile):
//   S^T = K Q^T and dP^T = V dO^T (A = K / V from shared memory) into two 128-column TMEM regions;
//   the compute warps load S^T, form P^T = exp2(S^T*sl2 - lse2) and write it back as bf16 pairs over the
//   first 64 columns of the S^T region; the MMA thread accumulates dV += P^T dO with P^T as a
//   tensor-memory A operand; meanwhile the compute warps load dP^T and write dS^T = P^T (dP^T - delta) the
//   same way, and the MMA thread accumulates dK += dS^T Q.
// MMA issue order dV(i), S(i+1), dK(i), dP(i+1): the tensor pipe computes S(i+1) while the compute warps
// form dS(i), and dP(i+1) / dV(i+1) while they form P(i+1). MMAs from one thread run in issue order, so
// S(i+1) overwrites P^T(i) only after dV(i) has read it. Q/dO tiles run NQ stages ahead.
template <int D>
struct DkvTLayout {
  static constexpr int BN = 128, BQ = 128, NB = D / 64, NQ = D <= 64 ? 4 : 2;
  static constexpr uint32_t KV_BYTES = BN * D * 2;
  static constexpr uint32_t QT_BYTES = BQ * D * 2;
  static constexpr uint32_t K = 0, V = KV_BYTES;
  static constexpr uint32_t Q0 = 2 * KV_BYTES;        // [NQ] Q tiles
  static constexpr uint32_t O0 = Q0 + NQ * QT_BYTES;  // [NQ] dO tiles
  static constexpr uint32_t LD0 = O0 + NQ * QT_BYTES; // [NQ][2][BQ] floats: lse2, delta
  static constexpr uint32_t BAR = LD0 + NQ * 2 * BQ * 4;
  static constexpr uint32_t TOTAL = BAR + 512;
  static constexpr uint32_t DK_COL = 0, DV_COL = D, S_COL = 2 * D, DP_COL = 2 * D + BQ;
  static_assert(DP_COL + BQ <= 512, "dK/dV tensor-memory columns");
};
static_assert(DkvTLayout<128>::TOTAL + 1024 <= 232448, "dK/dV shared memory exceeds 227 KB");
static_assert(DkvTLayout<64>::TOTAL + 1024 <= 232448, "dK/dV shared memory exceeds 227 KB");

struct DkvTBars {
  uint64_t kv, q_full[4], q_empty[4], s_full, dp_full, p_full, ds_full, fin;
  uint32_t tmem_slot;
  int abort;
  int4 info[4];  // per Q stage: {local index of the first query, T, vis_base, 0} of the step it holds
};
static_assert(sizeof(DkvTBars) <= 512, "dK/dV barrier block");

template <int D>
__global__ void __launch_bounds__(320, 1) attn_bwd_dkdv_t_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
    const float* __restrict__ lse, const float* __restrict__ delta, bf16* __restrict__ dk, bf16* __restrict__ dv,
    float* __restrict__ part_k, float* __restrict__ part_v, int T_in, int S_in, int Hq, int Hkv, float scale,
    const int* __restrict__ ktab, const int4* __restrict__ cons_tab, int Ttot, int Stot, int* __restrict__ err) {
  using L = DkvTLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DkvTBars* bars = reinterpret_cast<DkvTBars*>(smem + L::BAR);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.y, nsplit = gridDim.z, grp = Hq / Hkv / nsplit;
  const int hbase = hk * (Hq / Hkv) + blockIdx.z * grp;
  const KItem ki = ktab != nullptr ? reinterpret_cast<const KItem*>(ktab)[blockIdx.x]
                                    : KItem{(int)blockIdx.x * L::BN, min(L::BN, S_in - (int)blockIdx.x * L::BN), 0, 1};
  const int k0 = ki.k_row0;  // key row of the tile's first key
  const float sl2 = scale * kLog2e;
  StepWalk<L::BQ> steps;
  steps.init(ktab != nullptr ? cons_tab + ki.cons0 : nullptr, ki.ncons, make_int4(0, T_in, k0 - (S_in - T_in), 0),
             grp);
  const int total = steps.per_head() * grp;
  volatile int* abort = &bars->abort;
  float* ld = reinterpret_cast<float*>(smem + L::LD0);

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->kv, 1);
    for (int i = 0; i < L::NQ; ++i) {
      tc::mbar_init(&bars->q_full[i], 2);
      tc::mbar_init(&bars->q_empty[i], 1);
    }
    tc::mbar_init(&bars->s_full, 1);
    tc::mbar_init(&bars->dp_full, 1);
    tc::mbar_init(&bars->p_full, 256);
    tc::mbar_init(&bars->ds_full, 256);
    tc::mbar_init(&bars->fin, 1);
    bars->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 9) tc::tmem_alloc(&bars->tmem_slot, 512);
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 8) {
    // producer: K, V once; per step Q and dO tiles (TMA) plus lse2 / delta (plain loads, issued for the
    // next step before waiting for its stage so their latency overlaps the wait)
    if (lane == 0) {
      tc::mbar_expect_tx(&bars->kv, 2 * L::KV_BYTES);
      for (int b = 0; b < L::NB; ++b) {
        tc::tma_load_2d(smem + L::K + b * L::BN * 128, &tm_k, hk * D + b * 64, k0, &bars->kv);
        tc::tma_load_2d(smem + L::V + b * L::BN * 128, &tm_v, hk * D + b * 64, k0, &bars->kv);
      }
    }
    constexpr int PER = L::BQ / 32;
    float nl[PER], nd[PER];
    StepWalk<L::BQ> ahead = steps;  // one step ahead of `steps`: the lse / delta prefetch
    auto fetch = [&]() {
      const int hh = hbase + ahead.hh;
      const int qt = ahead.q_loc();
#pragma unroll
      for (int x = 0; x < PER; ++x) {
        const int qi = qt + x * 32 + lane;
        const long long at = (long long)hh * Ttot + ahead.cur.x + qi;
        nl[x] = qi < ahead.cur.y ? lse[at] : 0.f;
        nd[x] = qi < ahead.cur.y ? delta[at] : 0.f;
      }
      ahead.next(grp);
    };
    if (total > 0) fetch();
    for (int i = 0; i < total; ++i, steps.next(grp)) {
      const int qs = i % L::NQ;
      if (i >= L::NQ && !warp_wait(&bars->q_empty[qs], ((i - L::NQ) / L::NQ) & 1, abort, err, 151)) break;
      const int hh = hbase + steps.hh;
      const int qrow = steps.q_row();
      if (lane == 0) {
        tc::mbar_expect_tx(&bars->q_full[qs], 2 * L::QT_BYTES);
        for (int b = 0; b < L::NB; ++b) {
          tc::tma_load_2d(smem + L::Q0 + qs * L::QT_BYTES + b * L::BQ * 128, &tm_q, hh * D + b * 64, qrow,
                          &bars->q_full[qs]);
          tc::tma_load_2d(smem + L::O0 + qs * L::QT_BYTES + b * L::BQ * 128, &tm_do, hh * D + b * 64, qrow,
                          &bars->q_full[qs]);
        }
      }
#pragma unroll
      for (int x = 0; x < PER; ++x) {
        ld[(qs * 2 + 0) * L::BQ + x * 32 + lane] = nl[x] * kLog2e;
        ld[(qs * 2 + 1) * L::BQ + x * 32 + lane] = nd[x];
      }
      if (lane == 0) bars->info[qs] = make_int4(steps.q_loc(), steps.cur.y, steps.cur.z, 0);
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars->q_full[qs]);
      if (i + 1 < total) fetch();
    }
  } else if (warp == 9) {
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_bf16(128, L::BQ, false, false);
      const uint32_t id_acc = tc::idesc_bf16(128, D, false, true);
      // S^T / dP^T of one step: A = K or V (K-major, shared), B = Q or dO (K-major, shared)
      auto mma_t = [&](uint32_t col, uint32_t a_base, uint32_t b_base) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t kv_off = (kk >> 2) * L::BN * 128 + (kk & 3) * 32;
          const uint32_t q_off = (kk >> 2) * L::BQ * 128 + (kk & 3) * 32;
          tc::mma_bf16(tmem + col, tc::sdesc_sw128(a_base + kv_off, 16, 1024),
                       tc::sdesc_sw128(b_base + q_off, 16, 1024), id_s, kk > 0);
        }
      };
      // dV / dK accumulation: A = P^T / dS^T (bf16 pairs in TMEM: queries [64h, 64h + 64) of a step at
      // columns [64h, 64h + 32) of the region), B = dO / Q (MN-major, shared)
      auto mma_acc = [&](uint32_t dcol, uint32_t acol, uint32_t b_base, bool first) {
#pragma unroll
        for (int kk = 0; kk < L::BQ / 16; ++kk)
          tc::mma_bf16_ts(tmem + dcol, tmem + acol + (kk >> 2) * 64 + (kk & 3) * 8,
                          tc::sdesc_sw128(b_base + kk * 16 * 128, L::BQ * 128, 1024), id_acc, !first || kk > 0);
      };
      bool ok = tc::mbar_wait(&bars->kv, 0, abort, err, 161);
      if (ok && total > 0) {
        ok = tc::mbar_wait(&bars->q_full[0], 0, abort, err, 162);
        if (ok) {
          tc::tc_fence_after();
          mma_t(L::S_COL, sbase + L::K, sbase + L::Q0);
          tc::mma_commit(&bars->s_full);
          mma_t(L::DP_COL, sbase + L::V, sbase + L::O0);
          tc::mma_commit(&bars->dp_full);
        }
      }
      for (int i = 0; ok && i < total; ++i) {
        const int qs = i % L::NQ, qn = (i + 1) % L::NQ;
        const uint32_t qb = sbase + L::Q0 + qs * L::QT_BYTES, ob = sbase + L::O0 + qs * L::QT_BYTES;
        if (!tc::mbar_wait(&bars->p_full, i & 1, abort, err, 163)) { ok = false; break; }
        tc::tc_fence_after();
        mma_acc(L::DV_COL, L::S_COL, ob, i == 0);
        if (i + 1 < total) {
          if (!tc::mbar_wait(&bars->q_full[qn], ((i + 1) / L::NQ) & 1, abort, err, 164)) { ok = false; break; }
          tc::tc_fence_after();
          mma_t(L::S_COL, sbase + L::K, sbase + L::Q0 + qn * L::QT_BYTES);
          tc::mma_commit(&bars->s_full);
        }
        if (!tc::mbar_wait(&bars->ds_full, i & 1, abort, err, 165)) { ok = false; break; }
        tc::tc_fence_after();
        mma_acc(L::DK_COL, L::DP_COL, qb, i == 0);
        tc::mma_commit(&bars->q_empty[qs]);
        if (i + 1 < total) {
          mma_t(L::DP_COL, sbase + L::V, sbase + L::O0 + qn * L::QT_BYTES);
          tc::mma_commit(&bars->dp_full);
        }
      }
      if (ok) tc::mma_commit(&bars->fin);
    }
  } else {
    // warps 0-7: warp w reads TMEM lanes of sub-partition (w & 3) (key row r) and query columns
    // [64 * (w >> 2), +64) of each step, and writes its bf16 P^T / dS^T pairs over the first 32 of those
    // columns (its own: no warp waits for another's read).
    const int sp = warp & 3, hc = warp >> 2;
    const int r = sp * 32 + lane;
    const int kr = k0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(sp * 32) << 16);
    bool ok = true;
    for (int i = 0; i < total && ok; ++i) {
      const int qs = i % L::NQ;
      const float* l2p = ld + (qs * 2 + 0) * L::BQ + hc * 64;
      const float* dlp = ld + (qs * 2 + 1) * L::BQ + hc * 64;
      if (!warp_wait(&bars->q_full[qs], (i / L::NQ) & 1, abort, err, 171)) { ok = false; break; }
      const int4 inf = bars->info[qs];  // written by the producer before it released the stage
      const int qc0 = inf.x + hc * 64;
      const int lo = r < ki.cnt ? inf.z + r - qc0 : 64;  // local query qc0+c sees key kr iff c >= lo
      const int hi = inf.y - qc0;                        // and c < hi (query exists)
      if (!warp_wait(&bars->s_full, i & 1, abort, err, 172)) { ok = false; break; }
      tc::tc_fence_after();
      float p[64];
      tc::tmem_ld32(lane_base + L::S_COL + hc * 64, p);
      tc::tmem_ld32(lane_base + L::S_COL + hc * 64 + 32, p + 32);
      tc::tmem_ld_wait();
#pragma unroll
      for (int c4 = 0; c4 < 16; ++c4) {
        const float4 l = *reinterpret_cast<const float4*>(l2p + c4 * 4);
        const float lv[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = c4 * 4 + e;
          p[c] = (c >= lo && c < hi) ? ex2(fmaf(p[c], sl2, -lv[e])) : 0.f;
        }
      }
      {
        float w[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = __uint_as_float(pack2(p[2 * j], p[2 * j + 1]));
        tc::tmem_st32(lane_base + L::S_COL + hc * 64, w);
      }
      tc::tmem_st_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->p_full);

      if (!warp_wait(&bars->dp_full, i & 1, abort, err, 174)) { ok = false; break; }
      tc::tc_fence_after();
      {
        float dp[64];
        tc::tmem_ld32(lane_base + L::DP_COL + hc * 64, dp);
        tc::tmem_ld32(lane_base + L::DP_COL + hc * 64 + 32, dp + 32);
        tc::tmem_ld_wait();
#pragma unroll
        for (int c4 = 0; c4 < 16; ++c4) {
          const float4 d = *reinterpret_cast<const float4*>(dlp + c4 * 4);
          p[c4 * 4 + 0] *= dp[c4 * 4 + 0] - d.x;
          p[c4 * 4 + 1] *= dp[c4 * 4 + 1] - d.y;
          p[c4 * 4 + 2] *= dp[c4 * 4 + 2] - d.z;
          p[c4 * 4 + 3] *= dp[c4 * 4 + 3] - d.w;
        }
      }
      {
        float w[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) w[j] = __uint_as_float(pack2(p[2 * j], p[2 * j + 1]));
        tc::tmem_st32(lane_base + L::DP_COL + hc * 64, w);
      }
      tc::tmem_st_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->ds_full);
    }
    if (ok && total > 0 && warp_wait(&bars->fin, 0, abort, err, 176)) {
      tc::tc_fence_after();
#pragma unroll
      for (int c = hc * (D / 64); c < (hc + 1) * (D / 64); ++c) {
        float a[32], b[32];
        tc::tmem_ld32(lane_base + L::DK_COL + c * 32, a);
        tc::tmem_ld32(lane_base + L::DV_COL + c * 32, b);
        tc::tmem_ld_wait();
        if (r < ki.cnt && nsplit > 1) {
          const long long o = (((long long)blockIdx.z * Stot + kr) * Hkv + hk) * D + c * 32;
#pragma unroll
          for (int x = 0; x < 32; x += 4) {
            *reinterpret_cast<float4*>(part_k + o + x) = make_float4(a[x], a[x + 1], a[x + 2], a[x + 3]);
            *reinterpret_cast<float4*>(part_v + o + x) = make_float4(b[x], b[x + 1], b[x + 2], b[x + 3]);
          }
        } else if (r < ki.cnt) {
          bf16* pk = dk + ((long long)kr * Hkv + hk) * D + c * 32;
          bf16* pv = dv + ((long long)kr * Hkv + hk) * D + c * 32;
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 u, w;
            u.x = pack2(a[x] * scale, a[x + 1] * scale); u.y = pack2(a[x + 2] * scale, a[x + 3] * scale);
            u.z = pack2(a[x + 4] * scale, a[x + 5] * scale); u.w = pack2(a[x + 6] * scale, a[x + 7] * scale);
            w.x = pack2(b[x], b[x + 1]); w.y = pack2(b[x + 2], b[x + 3]);
            w.z = pack2(b[x + 4], b[x + 5]); w.w = pack2(b[x + 6], b[x + 7]);
            *reinterpret_cast<uint4*>(pk + x) = u;
            *reinterpret_cast<uint4*>(pv + x) = w;
          }
        }
      }
    } else if (ok && total == 0 && r < ki.cnt && nsplit > 1) {
      const long long o = (((long long)blockIdx.z * Stot + kr) * Hkv + hk) * D;
      for (int c = hc * (D / 2); c < (hc + 1) * (D / 2); c += 4) {
        *reinterpret_cast<float4*>(part_k + o + c) = make_float4(0.f, 0.f, 0.f, 0.f);
        *reinterpret_cast<float4*>(part_v + o + c) = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    } else if (ok && total == 0 && r < ki.cnt) {
      for (int c = hc * (D / 2); c < (hc + 1) * (D / 2); c += 8) {
        *reinterpret_cast<uint4*>(dk + ((long long)kr * Hkv + hk) * D + c) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(dv + ((long long)kr * Hkv + hk) * D + c) = make_uint4(0, 0, 0, 0);
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// dK (MODE 1) or dV (MODE 2) for head dim 256, whose dK and dV accumulators (256 TMEM columns each) do not
// fit together. CTA = 128 keys of one KV head; per step (query head, 64-query tile):
//   S^T = K Q^T with the CTA's K tile as a tensor-memory A operand (copied once from shared memory);
//   MODE 2: the compute warps write P^T back over the S^T columns (bf16 pairs) and the MMA thread
//           accumulates dV += P^T dO (N = 256) from there; two S^T buffers let S^T(i+1) run while the
//           compute warps exponentiate S^T(i);
//   MODE 1: dP^T = V dO^T (V resident in shared memory) into a second region; the compute warps write
//           dS^T = P^T (dP^T - delta) over the dP^T columns and the MMA thread accumulates dK += dS^T Q,
//           with issue order S^T(i+1), dK(i), dP^T(i+1).
// Q/dO tiles run NQ stages ahead; K is loaded into the last stage's space and copied to TMEM before that
// stage takes Q/dO.
template <int MODE>
struct Dkv256Layout {
  static constexpr int D = 256, BN = 128, BQ = 64, NB = 4, NQ = MODE == 1 ? 2 : 3;
  static constexpr uint32_t KV_BYTES = BN * D * 2;            // 64 KB
  static constexpr uint32_t QT_BYTES = BQ * D * 2;            // 32 KB
  static constexpr uint32_t ST_BYTES = 2 * QT_BYTES;          // one stage: Q tile, then dO tile
  static constexpr uint32_t V = 0;                            // MODE 1 only
  static constexpr uint32_t ST0 = MODE == 1 ? KV_BYTES : 0;   // [NQ] stages
  static constexpr uint32_t KLOAD = ST0 + (NQ - 1) * ST_BYTES;
  static constexpr uint32_t LD0 = ST0 + NQ * ST_BYTES;        // [NQ][2][BQ] floats: lse2, delta
  static constexpr uint32_t BAR = LD0 + NQ * 2 * BQ * 4;
  static constexpr uint32_t TOTAL = BAR + 512;
  static constexpr uint32_t ACC_COL = 0, KTM_COL = 256, S_COL = 384, DP_COL = 448;  // MODE 2: S buffers 384, 448
  static_assert(ST_BYTES == KV_BYTES, "K is staged through one Q/dO stage");
};
static_assert(Dkv256Layout<1>::TOTAL + 1024 <= 232448, "dK shared memory exceeds 227 KB");
static_assert(Dkv256Layout<2>::TOTAL + 1024 <= 232448, "dV shared memory exceeds 227 KB");

struct Dkv256Bars {
  uint64_t kv, kv_tm, q_full[3], q_empty[3], s_full[2], p_full[2], dp_full, s_free, fin;
  uint64_t rd[2][4];  // per buffer and TMEM sub-partition: warp (w & 3) has loaded its S^T / dP^T columns
  uint32_t tmem_slot;
  int abort;
};

template <int MODE>
__global__ void __launch_bounds__(320, 1) attn_bwd_dkdv256_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
    const float* __restrict__ lse, const float* __restrict__ delta, bf16* __restrict__ out,
    float* __restrict__ part, int T_in, int S_in, int Hq, int Hkv, float scale, const int* __restrict__ ktab,
    const int4* __restrict__ cons_tab, int Ttot, int Stot, int* __restrict__ err) {
  using L = Dkv256Layout<MODE>;
  constexpr int D = L::D;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Dkv256Bars* bars = reinterpret_cast<Dkv256Bars*>(smem + L::BAR);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hk = blockIdx.y, nsplit = gridDim.z, grp = Hq / Hkv / nsplit;
  const int hbase = hk * (Hq / Hkv) + blockIdx.z * grp;
  const KItem ki = ktab != nullptr ? reinterpret_cast<const KItem*>(ktab)[blockIdx.x]
                                    : KItem{(int)blockIdx.x * L::BN, min(L::BN, S_in - (int)blockIdx.x * L::BN), 0, 1};
  const int k0 = ki.k_row0;  // key row of the tile's first key
  const float sl2 = scale * kLog2e;
  StepWalk<L::BQ> steps;
  steps.init(ktab != nullptr ? cons_tab + ki.cons0 : nullptr, ki.ncons, make_int4(0, T_in, k0 - (S_in - T_in), 0),
             grp);
  const int total = steps.per_head() * grp;
  volatile int* abort = &bars->abort;
  float* ld = reinterpret_cast<float*>(smem + L::LD0);

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->kv, 1);
    tc::mbar_init(&bars->kv_tm, 256);
    for (int i = 0; i < L::NQ; ++i) {
      tc::mbar_init(&bars->q_full[i], 2);
      tc::mbar_init(&bars->q_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      tc::mbar_init(&bars->s_full[i], 1);
      tc::mbar_init(&bars->p_full[i], 256);
      for (int j = 0; j < 4; ++j) tc::mbar_init(&bars->rd[i][j], 32);
    }
    tc::mbar_init(&bars->dp_full, 1);
    tc::mbar_init(&bars->s_free, 256);
    tc::mbar_init(&bars->fin, 1);
    bars->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 9) tc::tmem_alloc(&bars->tmem_slot, 512);
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 8) {
    // producer: K (into the last stage's space) and, for dK, V once; per step Q and dO tiles plus
    // lse2 / delta (plain loads issued one step ahead)
    if (lane == 0) {
      tc::mbar_expect_tx(&bars->kv, (MODE == 1 ? 2 : 1) * L::KV_BYTES);
      for (int b = 0; b < L::NB; ++b) {
        tc::tma_load_2d(smem + L::KLOAD + b * L::BN * 128, &tm_k, hk * D + b * 64, k0, &bars->kv);
        if constexpr (MODE == 1)
          tc::tma_load_2d(smem + L::V + b * L::BN * 128, &tm_v, hk * D + b * 64, k0, &bars->kv);
      }
    }
    constexpr int PER = L::BQ / 32;
    float nl[PER], nd[PER];
    StepWalk<L::BQ> ahead = steps;  // one step ahead of `steps`: the lse / delta prefetch
    auto fetch = [&]() {
      const int hh = hbase + ahead.hh;
      const int qt = ahead.q_loc();
#pragma unroll
      for (int x = 0; x < PER; ++x) {
        const int qi = qt + x * 32 + lane;
        const long long at = (long long)hh * Ttot + ahead.cur.x + qi;
        nl[x] = qi < ahead.cur.y ? lse[at] : 0.f;
        nd[x] = qi < ahead.cur.y ? delta[at] : 0.f;
      }
      ahead.next(grp);
    };
    if (total > 0) fetch();
    for (int i = 0; i < total; ++i, steps.next(grp)) {
      const int qs = i % L::NQ;
      if (i == L::NQ - 1 && !warp_wait(&bars->kv_tm, 0, abort, err, 241)) break;  // K has left this stage
      if (i >= L::NQ && !warp_wait(&bars->q_empty[qs], ((i - L::NQ) / L::NQ) & 1, abort, err, 242)) break;
      const int hh = hbase + steps.hh;
      const int qrow = steps.q_row();
      uint8_t* st = smem + L::ST0 + qs * L::ST_BYTES;
      if (lane == 0) {
        tc::mbar_expect_tx(&bars->q_full[qs], 2 * L::QT_BYTES);
        for (int b = 0; b < L::NB; ++b) {
          tc::tma_load_2d(st + b * L::BQ * 128, &tm_q, hh * D + b * 64, qrow, &bars->q_full[qs]);
          tc::tma_load_2d(st + L::QT_BYTES + b * L::BQ * 128, &tm_do, hh * D + b * 64, qrow, &bars->q_full[qs]);
        }
      }
#pragma unroll
      for (int x = 0; x < PER; ++x) {
        ld[(qs * 2 + 0) * L::BQ + x * 32 + lane] = nl[x] * kLog2e;
        ld[(qs * 2 + 1) * L::BQ + x * 32 + lane] = nd[x];
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&bars->q_full[qs]);
      if (i + 1 < total) fetch();
    }
  } else if (warp == 9) {
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_bf16(128, L::BQ, false, false);
      const uint32_t id_acc = tc::idesc_bf16(128, D, false, true);
      auto stage = [&](int i) { return sbase + L::ST0 + (i % L::NQ) * L::ST_BYTES; };
      auto mma_st = [&](uint32_t col, uint32_t qb) {  // S^T = K Q^T, A = K from tensor memory
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::mma_bf16_ts(tmem + col, tmem + L::KTM_COL + kk * 8,
                          tc::sdesc_sw128(qb + (kk >> 2) * L::BQ * 128 + (kk & 3) * 32, 16, 1024), id_s, kk > 0);
      };
      auto mma_dpt = [&](uint32_t ob) {  // dP^T = V dO^T, A = V from shared memory
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::mma_bf16(tmem + L::DP_COL,
                       tc::sdesc_sw128(sbase + L::V + (kk >> 2) * L::BN * 128 + (kk & 3) * 32, 16, 1024),
                       tc::sdesc_sw128(ob + (kk >> 2) * L::BQ * 128 + (kk & 3) * 32, 16, 1024), id_s, kk > 0);
      };
      auto mma_acc = [&](uint32_t acol, uint32_t bb, bool first) {  // dK += dS^T Q or dV += P^T dO
#pragma unroll
        for (int kk = 0; kk < L::BQ / 16; ++kk)
          tc::mma_bf16_ts(tmem + L::ACC_COL, tmem + acol + kk * 8,
                          tc::sdesc_sw128(bb + kk * 16 * 128, L::BQ * 128, 1024), id_acc, !first || kk > 0);
      };
      bool ok = tc::mbar_wait(&bars->kv, 0, abort, err, 251);
      ok = ok && tc::mbar_wait(&bars->kv_tm, 0, abort, err, 252);
      tc::tc_fence_after();
      if constexpr (MODE == 2) {
        auto issue_s = [&](int i) -> bool {
          if (!tc::mbar_wait(&bars->q_full[i % L::NQ], (i / L::NQ) & 1, abort, err, 253)) return false;
          tc::tc_fence_after();
          mma_st(L::S_COL + (i & 1) * 64, stage(i));
          tc::mma_commit(&bars->s_full[i & 1]);
          return true;
        };
        if (ok && total > 0) ok = issue_s(0);
        if (ok && total > 1) ok = issue_s(1);
        for (int i = 0; ok && i < total; ++i) {
          if (!tc::mbar_wait(&bars->p_full[i & 1], (i >> 1) & 1, abort, err, 254)) { ok = false; break; }
          tc::tc_fence_after();
          mma_acc(L::S_COL + (i & 1) * 64, stage(i) + L::QT_BYTES, i == 0);
          tc::mma_commit(&bars->q_empty[i % L::NQ]);
          if (i + 2 < total) ok = issue_s(i + 2);
        }
      } else {
        if (ok && total > 0) {
          ok = tc::mbar_wait(&bars->q_full[0], 0, abort, err, 255);
          if (ok) {
            tc::tc_fence_after();
            mma_st(L::S_COL, stage(0));
            tc::mma_commit(&bars->s_full[0]);
            mma_dpt(stage(0) + L::QT_BYTES);
            tc::mma_commit(&bars->dp_full);
          }
        }
        for (int i = 0; ok && i < total; ++i) {
          if (i + 1 < total) {
            if (!tc::mbar_wait(&bars->s_free, i & 1, abort, err, 256)) { ok = false; break; }
            if (!tc::mbar_wait(&bars->q_full[(i + 1) % L::NQ], ((i + 1) / L::NQ) & 1, abort, err, 257)) {
              ok = false;
              break;
            }
            tc::tc_fence_after();
            mma_st(L::S_COL, stage(i + 1));
            tc::mma_commit(&bars->s_full[0]);
          }
          if (!tc::mbar_wait(&bars->p_full[0], i & 1, abort, err, 258)) { ok = false; break; }
          tc::tc_fence_after();
          mma_acc(L::DP_COL, stage(i), i == 0);
          tc::mma_commit(&bars->q_empty[i % L::NQ]);
          if (i + 1 < total) {
            mma_dpt(stage(i + 1) + L::QT_BYTES);
            tc::mma_commit(&bars->dp_full);
          }
        }
      }
      if (ok) tc::mma_commit(&bars->fin);
    }
  } else {
    // warps 0-7: key rows of sub-partition (w & 3), query columns [32 * (w >> 2), +32) of each step. The
    // bf16 pairs of warp hc = 1 land on columns that warp hc = 0 of the same sub-partition reads, so it
    // writes them once that warp has loaded its own.
    const int sp = warp & 3, hc = warp >> 2;
    const int r = sp * 32 + lane;
    const int kr = k0 + r;
    const uint32_t lane_base = tmem + ((uint32_t)(sp * 32) << 16);
    bool ok = true;
    // K tile -> tensor memory: warp hc copies D columns [128 hc, +128) of key row r
    if (warp_wait(&bars->kv, 0, abort, err, 261)) {
#pragma unroll
      for (int c0 = hc * 128; c0 < hc * 128 + 128; c0 += 64) {
        float w[32];
#pragma unroll
        for (int q8 = 0; q8 < 8; ++q8) {
          uint32_t a, b, c, d;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n"
                       : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
                       : "r"(sbase + L::KLOAD + tc::kmajor_off(r, c0 + q8 * 8, L::BN)));
          w[q8 * 4 + 0] = __uint_as_float(a);
          w[q8 * 4 + 1] = __uint_as_float(b);
          w[q8 * 4 + 2] = __uint_as_float(c);
          w[q8 * 4 + 3] = __uint_as_float(d);
        }
        tc::tmem_st32(lane_base + L::KTM_COL + c0 / 2, w);
      }
      tc::tmem_st_wait();
    }
    tc::tc_fence_before();
    tc::mbar_arrive(&bars->kv_tm);
    for (int i = 0; i < total && ok; ++i, steps.next(grp)) {
      const int qs = i % L::NQ, b = MODE == 2 ? (i & 1) : 0;
      const uint32_t scol = L::S_COL + b * 64;
      const int qc0 = steps.q_loc() + hc * 32;
      const int lo = r < ki.cnt ? steps.cur.z + r - qc0 : 32;  // local query qc0+c sees key kr iff c >= lo
      const int hi = steps.cur.y - qc0;                        // and c < hi (query exists)
      if (!warp_wait(&bars->q_full[qs], (i / L::NQ) & 1, abort, err, 262)) { ok = false; break; }
      if (!warp_wait(&bars->s_full[b], MODE == 2 ? (i >> 1) & 1 : i & 1, abort, err, 263)) { ok = false; break; }
      tc::tc_fence_after();
      float p[32];
      tc::tmem_ld32(lane_base + scol + hc * 32, p);
      tc::tmem_ld_wait();
      tc::tc_fence_before();
      if constexpr (MODE == 2) {
        if (hc == 0) tc::mbar_arrive(&bars->rd[b][sp]);
      } else {
        tc::mbar_arrive(&bars->s_free);
      }
      const float* l2p = ld + (qs * 2 + 0) * L::BQ + hc * 32;
#pragma unroll
      for (int c4 = 0; c4 < 8; ++c4) {
        const float4 l = *reinterpret_cast<const float4*>(l2p + c4 * 4);
        const float lv[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int c = c4 * 4 + e;
          p[c] = (c >= lo && c < hi) ? ex2(fmaf(p[c], sl2, -lv[e])) : 0.f;
        }
      }
      uint32_t wcol = scol;  // where this step's bf16 A operand goes
      if constexpr (MODE == 1) {
        if (!warp_wait(&bars->dp_full, i & 1, abort, err, 264)) { ok = false; break; }
        tc::tc_fence_after();
        float dp[32];
        tc::tmem_ld32(lane_base + L::DP_COL + hc * 32, dp);
        tc::tmem_ld_wait();
        if (hc == 0) {
          tc::tc_fence_before();
          tc::mbar_arrive(&bars->rd[0][sp]);
        }
        const float* dlp = ld + (qs * 2 + 1) * L::BQ + hc * 32;
#pragma unroll
        for (int c4 = 0; c4 < 8; ++c4) {
          const float4 d = *reinterpret_cast<const float4*>(dlp + c4 * 4);
          p[c4 * 4 + 0] *= dp[c4 * 4 + 0] - d.x;
          p[c4 * 4 + 1] *= dp[c4 * 4 + 1] - d.y;
          p[c4 * 4 + 2] *= dp[c4 * 4 + 2] - d.z;
          p[c4 * 4 + 3] *= dp[c4 * 4 + 3] - d.w;
        }
        wcol = L::DP_COL;
      }
      if (hc == 1 && !warp_wait(&bars->rd[b][sp], MODE == 2 ? (i >> 1) & 1 : i & 1, abort, err, 265)) {
        ok = false;
        break;
      }
      tc::tc_fence_after();
      {
        float w[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) w[x] = __uint_as_float(pack2(p[2 * x], p[2 * x + 1]));
        tc::tmem_st16(lane_base + wcol + hc * 16, w);
      }
      tc::tmem_st_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->p_full[b]);
    }
    const float osc = MODE == 1 ? scale : 1.f;
    if (ok && total > 0 && warp_wait(&bars->fin, 0, abort, err, 266)) {
      tc::tc_fence_after();
#pragma unroll
      for (int c = hc * 4; c < hc * 4 + 4; ++c) {
        float a[32];
        tc::tmem_ld32(lane_base + L::ACC_COL + c * 32, a);
        tc::tmem_ld_wait();
        if (r < ki.cnt && nsplit > 1) {
          const long long o = (((long long)blockIdx.z * Stot + kr) * Hkv + hk) * D + c * 32;
#pragma unroll
          for (int x = 0; x < 32; x += 4)
            *reinterpret_cast<float4*>(part + o + x) = make_float4(a[x], a[x + 1], a[x + 2], a[x + 3]);
        } else if (r < ki.cnt) {
          bf16* po = out + ((long long)kr * Hkv + hk) * D + c * 32;
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 u;
            u.x = pack2(a[x] * osc, a[x + 1] * osc); u.y = pack2(a[x + 2] * osc, a[x + 3] * osc);
            u.z = pack2(a[x + 4] * osc, a[x + 5] * osc); u.w = pack2(a[x + 6] * osc, a[x + 7] * osc);
            *reinterpret_cast<uint4*>(po + x) = u;
          }
        }
      }
    } else if (ok && total == 0 && r < ki.cnt && nsplit > 1) {
      const long long o = (((long long)blockIdx.z * Stot + kr) * Hkv + hk) * D;
      for (int c = hc * (D / 2); c < (hc + 1) * (D / 2); c += 4)
        *reinterpret_cast<float4*>(part + o + c) = make_float4(0.f, 0.f, 0.f, 0.f);
    } else if (ok && total == 0 && r < ki.cnt) {
      for (int c = hc * (D / 2); c < (hc + 1) * (D / 2); c += 8)
        *reinterpret_cast<uint4*>(out + ((long long)kr * Hkv + hk) * D + c) = make_uint4(0, 0, 0, 0);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// dQ for head dims 64 and 128 with 128-key steps (MMAs of N = 128). CTA = 128 queries of one head; thread
// r of warps 0-3 owns query row r. The CTA's Q and dO tiles sit in tensor memory as A operands of
// S = Q K^T and dP = dO V^T (two 128-column TMEM regions); the compute warps load S, release its region,
// exponentiate, load dP and write dS = P (dP - delta) back as bf16 pairs over the first 64 columns of the
// dP region, where the MMA thread reads it as the A operand of dQ += dS K.
// MMA issue order S(j+1), dQ(j), dP(j+1): S(j+1) runs while the compute warps exponentiate S(j), and
// dQ(j) / dP(j+1) while they exponentiate S(j+1). K/V tiles run NK stages ahead.
template <int D>
struct DqTLayout {
  static constexpr int BM = 128, BN = 128, NB = D / 64, NK = D <= 64 ? 4 : 2;
  // compute warps per TMEM sub-partition: each takes CW = BN / SW key columns of a step and D / SW columns
  // of the dQ row; it writes its dS pairs over the first CW / 2 of its own dP columns (no warp waits for
  // another's read). Two (four spill registers at 576 threads).
  static constexpr int SW = 2;
  static constexpr int CW = BN / SW;
  static constexpr int SOFT = 4 * SW, PROD = SOFT, MMA = SOFT + 1, THREADS = 32 * (SOFT + 2);
  static TS_DEVICE uint32_t ds_col(int kk) { return (kk * 16 / CW) * CW + ((kk * 16) % CW) / 2; }
  static constexpr uint32_t Q_BYTES = BM * D * 2;
  static constexpr uint32_t KT_BYTES = BN * D * 2;
  static constexpr uint32_t Q = 0, O = Q_BYTES;
  static constexpr uint32_t K0 = 2 * Q_BYTES;         // [NK] K tiles
  static constexpr uint32_t V0 = K0 + NK * KT_BYTES;  // [NK] V tiles
  static constexpr uint32_t BAR = V0 + NK * KT_BYTES;
  static constexpr uint32_t TOTAL = BAR + 512;
  static constexpr uint32_t DQ_COL = 0, S_COL = D, DP_COL = D + BN, QTM_COL = D + 2 * BN, OTM_COL = QTM_COL + D / 2;
  static_assert(OTM_COL + D / 2 <= 512, "dQ tensor-memory columns");
};
static_assert(DqTLayout<128>::TOTAL + 1024 <= 232448, "dQ shared memory exceeds 227 KB");
static_assert(DqTLayout<64>::TOTAL + 1024 <= 232448, "dQ shared memory exceeds 227 KB");

struct DqTBars {
  uint64_t q, kv_full[4], kv_empty[4], s_full, dp_full, s_free, ds_full, fin, qo_tm;
  uint64_t dp_read[4];  // head_dim 256 kernel: per TMEM sub-partition, warp (w & 3) has loaded its dP columns
  uint32_t tmem_slot;
  int abort;
};

template <int D>
__global__ void __launch_bounds__(DqTLayout<D>::THREADS, 1) attn_bwd_dq_t_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
    const float* __restrict__ lse, const float* __restrict__ delta, bf16* __restrict__ dq, int T_in, int S_in,
    int Hq, int Hkv, float scale, const int* __restrict__ qtab, const int2* __restrict__ far_tab, int Ttot,
    int* __restrict__ err) {
  using L = DqTLayout<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DqTBars* bars = reinterpret_cast<DqTBars*>(smem + L::BAR);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const QItem it = qtab != nullptr ? load_qitem(qtab, blockIdx.x) : dense_qitem(L::BM, T_in, S_in);
  const int T = it.T;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int q0 = it.q_loc0;
  KeyWalk<L::BN> walk;
  walk.init(it, far_tab);
  const int n = walk.count(q0 + L::BM);
  const float sl2 = scale * kLog2e;
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->q, 1);
    for (int i = 0; i < L::NK; ++i) {
      tc::mbar_init(&bars->kv_full[i], 1);
      tc::mbar_init(&bars->kv_empty[i], 1);
    }
    tc::mbar_init(&bars->s_full, 1);
    tc::mbar_init(&bars->dp_full, 1);
    tc::mbar_init(&bars->s_free, 32 * L::SOFT);
    tc::mbar_init(&bars->ds_full, 32 * L::SOFT);
    tc::mbar_init(&bars->fin, 1);
    tc::mbar_init(&bars->qo_tm, 128);
    for (int i = 0; i < 4; ++i) tc::mbar_init(&bars->dp_read[i], 32);
    bars->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == L::MMA) tc::tmem_alloc(&bars->tmem_slot, 512);
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == L::PROD) {
    if (lane == 0) {
      tc::mbar_expect_tx(&bars->q, 2 * L::Q_BYTES);
      for (int b = 0; b < L::NB; ++b) {
        tc::tma_load_2d(smem + L::Q + b * L::BM * 128, &tm_q, h * D + b * 64, it.q_row0, &bars->q);
        tc::tma_load_2d(smem + L::O + b * L::BM * 128, &tm_do, h * D + b * 64, it.q_row0, &bars->q);
      }
      for (int j = 0; j < n; ++j, walk.next()) {
        const int ks = j % L::NK;
        if (j >= L::NK && !tc::mbar_wait(&bars->kv_empty[ks], ((j - L::NK) / L::NK) & 1, abort, err, 181)) break;
        const int krow = walk.row();
        tc::mbar_expect_tx(&bars->kv_full[ks], 2 * L::KT_BYTES);
        for (int b = 0; b < L::NB; ++b) {
          tc::tma_load_2d(smem + L::K0 + ks * L::KT_BYTES + b * L::BN * 128, &tm_k, hk * D + b * 64, krow,
                          &bars->kv_full[ks]);
          tc::tma_load_2d(smem + L::V0 + ks * L::KT_BYTES + b * L::BN * 128, &tm_v, hk * D + b * 64, krow,
                          &bars->kv_full[ks]);
        }
      }
    }
  } else if (warp == L::MMA) {
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_bf16(128, L::BN, false, false);
      const uint32_t id_acc = tc::idesc_bf16(128, D, false, true);
      // S = Q K^T or dP = dO V^T: A = Q / dO (tensor memory), B = K / V tile (K-major, shared)
      auto mma_s = [&](uint32_t col, uint32_t a_col, uint32_t b_base) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::mma_bf16_ts(tmem + col, tmem + a_col + kk * 8,
                          tc::sdesc_sw128(b_base + (kk >> 2) * L::BN * 128 + (kk & 3) * 32, 16, 1024), id_s, kk > 0);
      };
      bool ok = tc::mbar_wait(&bars->q, 0, abort, err, 191);
      ok = ok && tc::mbar_wait(&bars->qo_tm, 0, abort, err, 192);
      if (ok && n > 0) {
        ok = tc::mbar_wait(&bars->kv_full[0], 0, abort, err, 193);
        if (ok) {
          tc::tc_fence_after();
          mma_s(L::S_COL, L::QTM_COL, sbase + L::K0);
          tc::mma_commit(&bars->s_full);
          mma_s(L::DP_COL, L::OTM_COL, sbase + L::V0);
          tc::mma_commit(&bars->dp_full);
        }
      }
      for (int j = 0; ok && j < n; ++j) {
        const int ks = j % L::NK, kn = (j + 1) % L::NK;
        if (j + 1 < n) {
          if (!tc::mbar_wait(&bars->s_free, j & 1, abort, err, 194)) { ok = false; break; }
          if (!tc::mbar_wait(&bars->kv_full[kn], ((j + 1) / L::NK) & 1, abort, err, 195)) { ok = false; break; }
          tc::tc_fence_after();
          mma_s(L::S_COL, L::QTM_COL, sbase + L::K0 + kn * L::KT_BYTES);
          tc::mma_commit(&bars->s_full);
        }
        if (!tc::mbar_wait(&bars->ds_full, j & 1, abort, err, 196)) { ok = false; break; }
        tc::tc_fence_after();
        const uint32_t kb = sbase + L::K0 + ks * L::KT_BYTES;
#pragma unroll
        for (int kk = 0; kk < L::BN / 16; ++kk)
          tc::mma_bf16_ts(tmem + L::DQ_COL, tmem + L::DP_COL + L::ds_col(kk),
                          tc::sdesc_sw128(kb + kk * 16 * 128, L::BN * 128, 1024), id_acc, j > 0 || kk > 0);
        tc::mma_commit(&bars->kv_empty[ks]);
        if (j + 1 < n) {
          mma_s(L::DP_COL, L::OTM_COL, sbase + L::V0 + kn * L::KT_BYTES);
          tc::mma_commit(&bars->dp_full);
        }
      }
      if (ok) tc::mma_commit(&bars->fin);
    }
  } else {
    // compute warps: sub-partition (w & 3) rows, key columns [CW * pw, +CW) of each step (pw = w >> 2); each
    // writes its bf16 dS pairs over the first CW / 2 of its own dP columns, where dQ += dS K reads them
    const int sp = warp & 3, pw = warp >> 2;
    const int r = sp * 32 + lane;
    const int qi = q0 + r;
    const long long lrow = (long long)h * Ttot + it.q_row0 + r;
    const float l2 = qi < T ? lse[lrow] * kLog2e : 0.f;
    const float dl = qi < T ? delta[lrow] : 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)(sp * 32) << 16);
    bool ok = true;
    // warps 0-3: copy this row of the Q and dO tiles (K-major, 128B-swizzled in shared memory) into the
    // A-operand columns of tensor memory, bf16 pairs per 32-bit column
    if (pw == 0) {
      if (warp_wait(&bars->q, 0, abort, err, 204)) {
#pragma unroll
        for (int which = 0; which < 2; ++which) {
          const uint32_t base = sbase + (which ? L::O : L::Q);
#pragma unroll
          for (int c0 = 0; c0 < D; c0 += 64) {
            float w[32];
#pragma unroll
            for (int q8 = 0; q8 < 8; ++q8) {
              uint32_t a, b, c, d;
              asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n"
                           : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
                           : "r"(base + tc::kmajor_off(r, c0 + q8 * 8, L::BM)));
              w[q8 * 4 + 0] = __uint_as_float(a);
              w[q8 * 4 + 1] = __uint_as_float(b);
              w[q8 * 4 + 2] = __uint_as_float(c);
              w[q8 * 4 + 3] = __uint_as_float(d);
            }
            tc::tmem_st32(lane_base + (which ? L::OTM_COL : L::QTM_COL) + c0 / 2, w);
          }
        }
        tc::tmem_st_wait();
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->qo_tm);
    }
    for (int j = 0; j < n && ok; ++j, walk.next()) {
      if (!warp_wait(&bars->s_full, j & 1, abort, err, 201)) { ok = false; break; }
      tc::tc_fence_after();
      constexpr int CW = L::CW;
      float p[CW];
#pragma unroll
      for (int c = 0; c < CW; c += 32) tc::tmem_ld32(lane_base + L::S_COL + pw * CW + c, p + c);
      tc::tmem_ld_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->s_free);
      // key pw*CW+c of the tile is visible iff c < nvis (the query exists and sees it)
      const int nvis = qi < T ? walk.nvis(qi) - pw * CW : 0;
#pragma unroll
      for (int c = 0; c < CW; ++c) p[c] = c < nvis ? ex2(fmaf(p[c], sl2, -l2)) : 0.f;
      if (!warp_wait(&bars->dp_full, j & 1, abort, err, 202)) { ok = false; break; }
      tc::tc_fence_after();
      {
        float dp[CW];
#pragma unroll
        for (int c = 0; c < CW; c += 32) tc::tmem_ld32(lane_base + L::DP_COL + pw * CW + c, dp + c);
        tc::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < CW; ++c) p[c] *= dp[c] - dl;
      }
      {
        float w[CW / 2];
#pragma unroll
        for (int x = 0; x < CW / 2; ++x) w[x] = __uint_as_float(pack2(p[2 * x], p[2 * x + 1]));
        if constexpr (CW / 2 == 32) tc::tmem_st32(lane_base + L::DP_COL + pw * CW, w);
        else tc::tmem_st16(lane_base + L::DP_COL + pw * CW, w);
      }
      tc::tmem_st_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->ds_full);
    }
    if (ok && warp_wait(&bars->fin, 0, abort, err, 205)) {
      tc::tc_fence_after();
#pragma unroll
      for (int c = pw * (D / (32 * L::SW)); c < (pw + 1) * (D / (32 * L::SW)); ++c) {
        float a[32];
        tc::tmem_ld32(lane_base + L::DQ_COL + c * 32, a);
        tc::tmem_ld_wait();
        if (qi < T) {
          bf16* pq = dq + ((long long)(it.q_row0 + r) * Hq + h) * D + c * 32;
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 u;
            u.x = pack2(a[x] * scale, a[x + 1] * scale); u.y = pack2(a[x + 2] * scale, a[x + 3] * scale);
            u.z = pack2(a[x + 4] * scale, a[x + 5] * scale); u.w = pack2(a[x + 6] * scale, a[x + 7] * scale);
            *reinterpret_cast<uint4*>(pq + x) = u;
          }
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == L::MMA) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// dQ for head dim 256 with 64-key steps. TMEM columns: dQ [0, 256), the CTA's Q tile as the A operand of
// S = Q K^T [256, 384), S [384, 448), dP [448, 512). dP = dO V^T takes dO from shared memory. The compute
// warps load S (releasing its columns), exponentiate, load dP and write dS = P (dP - delta) back as bf16
// pairs over the first 32 dP columns, where dQ += dS K (N = 256) reads it as its A operand. Shared memory
// holds dO and two K/V stages (192 KB); Q arrives in the second stage's space and is copied to TMEM
// before that stage takes K/V. MMA issue order S(j+1), dQ(j), dP(j+1), as in attn_bwd_dq_t_kernel.
struct Dq256Layout {
  static constexpr int D = 256, BM = 128, BN = 64, NB = 4, NK = 2;
  static constexpr uint32_t Q_BYTES = BM * D * 2;     // 64 KB
  static constexpr uint32_t KT_BYTES = BN * D * 2;    // 32 KB
  static constexpr uint32_t ST_BYTES = 2 * KT_BYTES;  // one K/V stage
  static constexpr uint32_t O = 0;
  static constexpr uint32_t ST0 = Q_BYTES;            // [NK] stages: K tile, then V tile
  static constexpr uint32_t QLOAD = ST0 + ST_BYTES;   // Q lands in stage 1 first
  static constexpr uint32_t BAR = ST0 + NK * ST_BYTES;
  static constexpr uint32_t TOTAL = BAR + 512;
  static constexpr uint32_t DQ_COL = 0, QTM_COL = 256, S_COL = 384, DP_COL = 448;
  static_assert(Q_BYTES == ST_BYTES, "Q is staged through one K/V stage");
};
static_assert(Dq256Layout::TOTAL + 1024 <= 232448, "dQ shared memory exceeds 227 KB");

template <int D_>
__global__ void __launch_bounds__(320, 1) attn_bwd_dq256_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
    const float* __restrict__ lse, const float* __restrict__ delta, bf16* __restrict__ dq, int T_in, int S_in,
    int Hq, int Hkv, float scale, const int* __restrict__ qtab, const int2* __restrict__ far_tab, int Ttot,
    int* __restrict__ err) {
  using L = Dq256Layout;
  constexpr int D = L::D;
  static_assert(D_ == D, "head dim 256 only");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DqTBars* bars = reinterpret_cast<DqTBars*>(smem + L::BAR);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const QItem it = qtab != nullptr ? load_qitem(qtab, blockIdx.x) : dense_qitem(L::BM, T_in, S_in);
  const int T = it.T;
  const int h = blockIdx.y, hk = h / (Hq / Hkv);
  const int q0 = it.q_loc0;
  KeyWalk<L::BN> walk;
  walk.init(it, far_tab);
  const int n = walk.count(q0 + L::BM);
  const float sl2 = scale * kLog2e;
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    tc::mbar_init(&bars->q, 1);
    for (int i = 0; i < L::NK; ++i) {
      tc::mbar_init(&bars->kv_full[i], 1);
      tc::mbar_init(&bars->kv_empty[i], 1);
    }
    tc::mbar_init(&bars->s_full, 1);
    tc::mbar_init(&bars->dp_full, 1);
    tc::mbar_init(&bars->s_free, 256);
    tc::mbar_init(&bars->ds_full, 256);
    tc::mbar_init(&bars->fin, 1);
    tc::mbar_init(&bars->qo_tm, 128);
    for (int i = 0; i < 4; ++i) tc::mbar_init(&bars->dp_read[i], 32);
    bars->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 9) tc::tmem_alloc(&bars->tmem_slot, 512);
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 8) {
    if (lane == 0) {
      tc::mbar_expect_tx(&bars->q, 2 * L::Q_BYTES);
      for (int b = 0; b < L::NB; ++b) {
        tc::tma_load_2d(smem + L::QLOAD + b * L::BM * 128, &tm_q, h * D + b * 64, it.q_row0, &bars->q);
        tc::tma_load_2d(smem + L::O + b * L::BM * 128, &tm_do, h * D + b * 64, it.q_row0, &bars->q);
      }
      for (int j = 0; j < n; ++j, walk.next()) {
        const int ks = j % L::NK;
        if (j == 1 && !tc::mbar_wait(&bars->qo_tm, 0, abort, err, 211)) break;  // Q has left stage 1
        if (j >= L::NK && !tc::mbar_wait(&bars->kv_empty[ks], ((j - L::NK) / L::NK) & 1, abort, err, 212)) break;
        uint8_t* st = smem + L::ST0 + ks * L::ST_BYTES;
        const int krow = walk.row();
        tc::mbar_expect_tx(&bars->kv_full[ks], 2 * L::KT_BYTES);
        for (int b = 0; b < L::NB; ++b) {
          tc::tma_load_2d(st + b * L::BN * 128, &tm_k, hk * D + b * 64, krow, &bars->kv_full[ks]);
          tc::tma_load_2d(st + L::KT_BYTES + b * L::BN * 128, &tm_v, hk * D + b * 64, krow,
                          &bars->kv_full[ks]);
        }
      }
    }
  } else if (warp == 9) {
    if (lane == 0) {
      const uint32_t id_s = tc::idesc_bf16(128, L::BN, false, false);
      const uint32_t id_acc = tc::idesc_bf16(128, D, false, true);
      auto mma_s = [&](uint32_t kb) {  // S = Q K^T, A = Q from tensor memory
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::mma_bf16_ts(tmem + L::S_COL, tmem + L::QTM_COL + kk * 8,
                          tc::sdesc_sw128(kb + (kk >> 2) * L::BN * 128 + (kk & 3) * 32, 16, 1024), id_s, kk > 0);
      };
      auto mma_dp = [&](uint32_t vb) {  // dP = dO V^T, A = dO from shared memory
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          tc::mma_bf16(tmem + L::DP_COL, tc::sdesc_sw128(sbase + L::O + (kk >> 2) * L::BM * 128 + (kk & 3) * 32, 16, 1024),
                       tc::sdesc_sw128(vb + (kk >> 2) * L::BN * 128 + (kk & 3) * 32, 16, 1024), id_s, kk > 0);
      };
      bool ok = tc::mbar_wait(&bars->q, 0, abort, err, 221);
      ok = ok && tc::mbar_wait(&bars->qo_tm, 0, abort, err, 222);
      if (ok && n > 0) {
        ok = tc::mbar_wait(&bars->kv_full[0], 0, abort, err, 223);
        if (ok) {
          tc::tc_fence_after();
          mma_s(sbase + L::ST0);
          tc::mma_commit(&bars->s_full);
          mma_dp(sbase + L::ST0 + L::KT_BYTES);
          tc::mma_commit(&bars->dp_full);
        }
      }
      for (int j = 0; ok && j < n; ++j) {
        const int ks = j % L::NK, kn = (j + 1) % L::NK;
        const uint32_t sn = sbase + L::ST0 + kn * L::ST_BYTES;
        if (j + 1 < n) {
          if (!tc::mbar_wait(&bars->s_free, j & 1, abort, err, 224)) { ok = false; break; }
          if (!tc::mbar_wait(&bars->kv_full[kn], ((j + 1) / L::NK) & 1, abort, err, 225)) { ok = false; break; }
          tc::tc_fence_after();
          mma_s(sn);
          tc::mma_commit(&bars->s_full);
        }
        if (!tc::mbar_wait(&bars->ds_full, j & 1, abort, err, 226)) { ok = false; break; }
        tc::tc_fence_after();
        const uint32_t kb = sbase + L::ST0 + ks * L::ST_BYTES;
#pragma unroll
        for (int kk = 0; kk < L::BN / 16; ++kk)
          tc::mma_bf16_ts(tmem + L::DQ_COL, tmem + L::DP_COL + kk * 8,
                          tc::sdesc_sw128(kb + kk * 16 * 128, L::BN * 128, 1024), id_acc, j > 0 || kk > 0);
        tc::mma_commit(&bars->kv_empty[ks]);
        if (j + 1 < n) {
          mma_dp(sn + L::KT_BYTES);
          tc::mma_commit(&bars->dp_full);
        }
      }
      if (ok) tc::mma_commit(&bars->fin);
    }
  } else {
    // warps 0-7: sub-partition (w & 3) rows, key columns [32 * (w >> 2), +32) of each step; warp hc = 1
    // writes its dS pairs over dP columns of warp hc = 0, once that warp has loaded them.
    const int sp = warp & 3, hc = warp >> 2;
    const int r = sp * 32 + lane;
    const int qi = q0 + r;
    const long long lrow = (long long)h * Ttot + it.q_row0 + r;
    const float l2 = qi < T ? lse[lrow] * kLog2e : 0.f;
    const float dl = qi < T ? delta[lrow] : 0.f;
    const uint32_t lane_base = tmem + ((uint32_t)(sp * 32) << 16);
    bool ok = true;
    if (hc == 0) {
      // warps 0-3: copy this row of Q (K-major, 128B-swizzled, in stage 1) into tensor memory
      if (warp_wait(&bars->q, 0, abort, err, 234)) {
#pragma unroll
        for (int c0 = 0; c0 < D; c0 += 64) {
          float w[32];
#pragma unroll
          for (int q8 = 0; q8 < 8; ++q8) {
            uint32_t a, b, c, d;
            asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];\n"
                         : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
                         : "r"(sbase + L::QLOAD + tc::kmajor_off(r, c0 + q8 * 8, L::BM)));
            w[q8 * 4 + 0] = __uint_as_float(a);
            w[q8 * 4 + 1] = __uint_as_float(b);
            w[q8 * 4 + 2] = __uint_as_float(c);
            w[q8 * 4 + 3] = __uint_as_float(d);
          }
          tc::tmem_st32(lane_base + L::QTM_COL + c0 / 2, w);
        }
        tc::tmem_st_wait();
      }
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->qo_tm);
    }
    for (int j = 0; j < n && ok; ++j, walk.next()) {
      if (!warp_wait(&bars->s_full, j & 1, abort, err, 231)) { ok = false; break; }
      tc::tc_fence_after();
      float p[32];
      tc::tmem_ld32(lane_base + L::S_COL + hc * 32, p);
      tc::tmem_ld_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->s_free);
      const int nvis = qi < T ? walk.nvis(qi) - hc * 32 : 0;  // key hc*32+c of the tile visible iff c < nvis
#pragma unroll
      for (int c = 0; c < 32; ++c) p[c] = c < nvis ? ex2(fmaf(p[c], sl2, -l2)) : 0.f;
      if (!warp_wait(&bars->dp_full, j & 1, abort, err, 232)) { ok = false; break; }
      tc::tc_fence_after();
      {
        float dp[32];
        tc::tmem_ld32(lane_base + L::DP_COL + hc * 32, dp);
        tc::tmem_ld_wait();
        if (hc == 0) {
          tc::tc_fence_before();
          tc::mbar_arrive(&bars->dp_read[sp]);
        }
#pragma unroll
        for (int c = 0; c < 32; ++c) p[c] *= dp[c] - dl;
      }
      if (hc == 1 && !warp_wait(&bars->dp_read[sp], j & 1, abort, err, 233)) { ok = false; break; }
      tc::tc_fence_after();
      {
        float w[16];
#pragma unroll
        for (int x = 0; x < 16; ++x) w[x] = __uint_as_float(pack2(p[2 * x], p[2 * x + 1]));
        tc::tmem_st16(lane_base + L::DP_COL + hc * 16, w);
      }
      tc::tmem_st_wait();
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->ds_full);
    }
    if (ok && warp_wait(&bars->fin, 0, abort, err, 235)) {
      tc::tc_fence_after();
#pragma unroll
      for (int c = hc * (D / 64); c < (hc + 1) * (D / 64); ++c) {
        float a[32];
        tc::tmem_ld32(lane_base + L::DQ_COL + c * 32, a);
        tc::tmem_ld_wait();
        if (qi < T) {
          bf16* pq = dq + ((long long)(it.q_row0 + r) * Hq + h) * D + c * 32;
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 u;
            u.x = pack2(a[x] * scale, a[x + 1] * scale); u.y = pack2(a[x + 2] * scale, a[x + 3] * scale);
            u.z = pack2(a[x + 4] * scale, a[x + 5] * scale); u.w = pack2(a[x + 6] * scale, a[x + 7] * scale);
            *reinterpret_cast<uint4*>(pq + x) = u;
          }
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ self-test
// D1 = A * Bk^T (Bk [N][K], K-major), D2 = A * Bm (Bm [K][N], MN-major); 128x128x128.
__global__ void __launch_bounds__(128, 1) tc_selftest_kernel(const __grid_constant__ CUtensorMap tm_a,
                                                             const __grid_constant__ CUtensorMap tm_bk,
                                                             const __grid_constant__ CUtensorMap tm_bm,
                                                             float* __restrict__ d1, float* __restrict__ d2,
                                                             int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = tc::smem_addr(smem);
  // A: 2 boxes x 16 KB, Bk: 2 boxes, Bm: 2 boxes (64-col boxes over N)
  uint64_t* bar_ld = reinterpret_cast<uint64_t*>(smem + 6 * 16384);
  uint64_t* bar_mma = bar_ld + 1;
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar_ld + 2);
  int* abort = reinterpret_cast<int*>(bar_ld + 3);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    tc::mbar_init(bar_ld, 1);
    tc::mbar_init(bar_mma, 1);
    *abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0) tc::tmem_alloc(slot, 256);
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    tc::mbar_expect_tx(bar_ld, 6 * 16384);
    for (int b = 0; b < 2; ++b) {
      tc::tma_load_2d(smem + b * 16384, &tm_a, b * 64, 0, bar_ld);
      tc::tma_load_2d(smem + 32768 + b * 16384, &tm_bk, b * 64, 0, bar_ld);
      tc::tma_load_2d(smem + 65536 + b * 16384, &tm_bm, b * 64, 0, bar_ld);
    }
    if (tc::mbar_wait(bar_ld, 0, abort, err, 41)) {
      tc::tc_fence_after();
      const uint32_t id1 = tc::idesc_bf16(128, 128, false, false);
      const uint32_t id2 = tc::idesc_bf16(128, 128, false, true);
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t boff = (kk >> 2) * 16384 + (kk & 3) * 32;
        tc::mma_bf16(tmem, tc::sdesc_sw128(sbase + boff, 16, 1024), tc::sdesc_sw128(sbase + 32768 + boff, 16, 1024),
                     id1, kk > 0);
        tc::mma_bf16(tmem + 128, tc::sdesc_sw128(sbase + boff, 16, 1024),
                     tc::sdesc_sw128(sbase + 65536 + kk * 16 * 128, 16384, 1024), id2, kk > 0);
      }
      tc::mma_commit(bar_mma);
    }
  }
  __syncwarp();
  bool ok = warp_wait(bar_mma, 0, abort, err, 42);
  if (ok) {
    tc::tc_fence_after();
    const uint32_t lb = tmem + ((uint32_t)(warp * 32) << 16);
    const int row = threadIdx.x;
    for (int c = 0; c < 4; ++c) {
      float v[32];
      tc::tmem_ld32(lb + c * 32, v);
      tc::tmem_ld_wait();
      for (int i = 0; i < 32; ++i) d1[row * 128 + c * 32 + i] = v[i];
      tc::tmem_ld32(lb + 128 + c * 32, v);
      tc::tmem_ld_wait();
      for (int i = 0; i < 32; ++i) d2[row * 128 + c * 32 + i] = v[i];
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 256);
  }
}

// ------------------------------------------------------------------ host helpers
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    TS_CUDA_CHECK(cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q));
    TS_CHECK(q == cudaDriverEntryPointSuccess && p != nullptr, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

}  // namespace

// 2-D bf16 map over [outer][inner] (row stride in elements), 128B-swizzled box of
// 64 x box_rows. The inner coordinate of every load is a multiple of 8 elements.
CUtensorMap make_bf16_map(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                          uint32_t box_rows) {
  TS_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TS_CHECK((row_stride_elems * 2) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_elems * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TS_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed with ", (int)r);
  return map;
}

CUtensorMap make_out_map(void* base, bool f32, uint64_t cols, uint64_t rows, uint64_t ld) {
  const uint64_t es = f32 ? 4 : 2;
  TS_CHECK(reinterpret_cast<uintptr_t>(base) % 16 == 0, "TMA base must be 16-byte aligned");
  TS_CHECK((ld * es) % 16 == 0, "TMA row stride must be a multiple of 16 bytes");
  CUtensorMap map;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {ld * es};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base,
                           dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           f32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TS_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled (output map) failed with ", (int)r);
  return map;
}

at::Tensor& tc_error_flag(const at::Device& dev) {
  static std::vector<at::Tensor> flags(64);
  const int i = dev.index();
  if (!flags[i].defined()) flags[i] = at::zeros({1}, at::TensorOptions().dtype(at::kInt).device(dev));
  return flags[i];
}

at::Tensor tc_status(const at::Tensor& like) { return tc_error_flag(like.device()); }

std::vector<at::Tensor> tc_selftest(const at::Tensor& a, const at::Tensor& bk, const at::Tensor& bm) {
  check_cuda(a, "a");
  const c10::cuda::CUDAGuard guard(a.device());
  TS_CHECK(a.sizes() == at::IntArrayRef({128, 128}) && bk.sizes() == a.sizes() && bm.sizes() == a.sizes(),
           "selftest takes 128x128 bf16 operands");
  auto d1 = at::empty({128, 128}, a.options().dtype(at::kFloat));
  auto d2 = at::empty({128, 128}, a.options().dtype(at::kFloat));
  CUtensorMap ma = make_bf16_map(a.data_ptr(), 128, 128, 128, 128);
  CUtensorMap mk = make_bf16_map(bk.data_ptr(), 128, 128, 128, 128);
  CUtensorMap mm = make_bf16_map(bm.data_ptr(), 128, 128, 128, 128);
  const int smem = 6 * 16384 + 64 + 1024;
  ensure_smem((const void*)tc_selftest_kernel, (int)(smem));
  tc_selftest_kernel<<<1, 128, smem, stream()>>>(ma, mk, mm, d1.data_ptr<float>(), d2.data_ptr<float>(),
                                                 tc_error_flag(a.device()).data_ptr<int>());
  TS_LAUNCH_CHECK();
  return {d1, d2};
}

// out (optional): a contiguous bf16 tensor shaped like q that receives O (e.g. rows of a larger buffer).
static at::Tensor out_or_new(const c10::optional<at::Tensor>& out, const at::Tensor& like, const char* what) {
  if (!out) return at::empty_like(like);
  TS_CHECK(out->is_contiguous() && out->sizes() == like.sizes() && out->scalar_type() == like.scalar_type() &&
               out->device() == like.device(),
           what, " must be a contiguous tensor shaped, typed and placed like its input");
  return *out;
}

namespace {

// Q-side / K-side work tables of a packed launch (all null for the single-segment launch).
struct PackTabs {
  const int* qtab = nullptr;
  const int2* far = nullptr;
  int nq = 0;
  const int* ktab = nullptr;
  const int4* cons = nullptr;
  int nk = 0;
};

template <int D>
void launch_fwd(dim3 grid, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, bf16* o,
                float* lse, int T, int S, int Hq, int Hkv, float sl2, const PackTabs& tb, int Ttot, int* err) {
  const int smem = FwdLayout<D>::TOTAL + 1024;
  ensure_smem((const void*)attn_fwd_tc_kernel<D>, smem);
  attn_fwd_tc_kernel<D><<<grid, FwdLayout<D>::THREADS, smem, stream()>>>(mq, mk, mv, o, lse, T, S, Hq, Hkv, sl2,
                                                                          tb.qtab, tb.far, Ttot, err);
}

void run_fwd(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, at::Tensor& o, at::Tensor& lse,
             double scale, const PackTabs& tb) {
  const int Ttot = q.size(0), Hq = q.size(1), D = q.size(2), S = k.size(0), Hkv = k.size(1);
  CUtensorMap mq = make_bf16_map(q.data_ptr(), (uint64_t)Hq * D, Ttot, (uint64_t)Hq * D, 128);
  const uint32_t kv_rows = D <= 128 ? 128 : 64;
  CUtensorMap mk = make_bf16_map(k.data_ptr(), (uint64_t)Hkv * D, S, (uint64_t)Hkv * D, kv_rows);
  CUtensorMap mv = make_bf16_map(v.data_ptr(), (uint64_t)Hkv * D, S, (uint64_t)Hkv * D, kv_rows);
  const dim3 grid(tb.qtab != nullptr ? tb.nq : (Ttot + 127) / 128, Hq);
  const float sl2 = (float)scale * kLog2e;
  int* err = tc_error_flag(q.device()).data_ptr<int>();
  bf16* po = (bf16*)o.data_ptr();
  float* pl = lse.data_ptr<float>();
  if (D == 128) launch_fwd<128>(grid, mq, mk, mv, po, pl, Ttot, S, Hq, Hkv, sl2, tb, Ttot, err);
  else if (D == 64) launch_fwd<64>(grid, mq, mk, mv, po, pl, Ttot, S, Hq, Hkv, sl2, tb, Ttot, err);
  else if (D == 256) launch_fwd<256>(grid, mq, mk, mv, po, pl, Ttot, S, Hq, Hkv, sl2, tb, Ttot, err);
  else TS_CHECK(false, "tcgen05 attention supports head_dim 64, 128 and 256");
  TS_LAUNCH_CHECK();
}

void check_attn_inputs(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v) {
  check_cuda(q, "q");
  check_cuda(k, "k");
  check_cuda(v, "v");
  TS_CHECK(q.scalar_type() == at::kBFloat16 && k.scalar_type() == at::kBFloat16 && v.scalar_type() == at::kBFloat16,
           "attention runs in bf16");
  TS_CHECK(q.dim() == 3 && k.dim() == 3 && k.sizes() == v.sizes() && k.size(2) == q.size(2) &&
               q.size(1) % k.size(1) == 0,
           "attention shapes: q [T, Hq, d], k/v [S, Hkv, d] with Hq a multiple of Hkv");
  TS_CHECK(q.is_contiguous() && k.is_contiguous() && v.is_contiguous(), "attention inputs must be contiguous");
}

// Reads the work tables of a packed launch: int32 CUDA tensors on q's device.
PackTabs pack_tabs(const at::Tensor& q, const at::Tensor& qtab, const at::Tensor& far,
                   const c10::optional<at::Tensor>& ktab, const c10::optional<at::Tensor>& cons) {
  auto ok = [&](const at::Tensor& t, int per) {
    return t.is_cuda() && t.device() == q.device() && t.scalar_type() == at::kInt && t.is_contiguous() &&
           t.numel() % per == 0 && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15) == 0;
  };
  TS_CHECK(ok(qtab, 8) && ok(far, 2), "packed attention: qtab (8 ints per item) and far (2 ints per range) must "
                                      "be contiguous, 16-byte aligned int32 CUDA tensors on q's device");
  PackTabs tb;
  tb.qtab = qtab.data_ptr<int>();
  tb.far = reinterpret_cast<const int2*>(far.data_ptr<int>());
  tb.nq = (int)(qtab.numel() / 8);
  if (ktab) {
    TS_CHECK(cons && ok(*ktab, 4) && ok(*cons, 4), "packed attention: ktab and cons (4 ints per entry) must be "
                                                   "contiguous, 16-byte aligned int32 CUDA tensors on q's device");
    tb.ktab = ktab->data_ptr<int>();
    tb.cons = reinterpret_cast<const int4*>(cons->data_ptr<int>());
    tb.nk = (int)(ktab->numel() / 4);
  }
  return tb;
}

}  // namespace

std::vector<at::Tensor> attn_fwd_tc(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v, double scale,
                                    const c10::optional<at::Tensor>& out) {
  check_attn_inputs(q, k, v);
  const c10::cuda::CUDAGuard guard(q.device());
  const int T = q.size(0), Hq = q.size(1), S = k.size(0);
  TS_CHECK(S >= T, "attention shapes: more queries than keys");
  auto o = out_or_new(out, q, "attention out");
  auto lse = at::empty({Hq, T}, q.options().dtype(at::kFloat));
  if (T == 0) return {o, lse};
  run_fwd(q, k, v, o, lse, scale, PackTabs{});
  return {o, lse};
}

// Packed forward: q [Ttot, Hq, d] holds every segment's queries, k/v [Stot, Hkv, d] every key range;
// qtab / far describe the work (see QItem). Rows of q no item covers are left untouched in `out` and lse.
std::vector<at::Tensor> attn_fwd_packed(const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                                        const at::Tensor& qtab, const at::Tensor& far, double scale,
                                        const c10::optional<at::Tensor>& out) {
  check_attn_inputs(q, k, v);
  const c10::cuda::CUDAGuard guard(q.device());
  auto o = out_or_new(out, q, "attention out");
  auto lse = at::empty({q.size(1), q.size(0)}, q.options().dtype(at::kFloat));
  const PackTabs tb = pack_tabs(q, qtab, far, c10::nullopt, c10::nullopt);
  if (q.size(0) == 0 || tb.nq == 0) return {o, lse};
  run_fwd(q, k, v, o, lse, scale, tb);
  return {o, lse};
}

namespace {
// Split the query heads of a KV head across CTAs when that fills the SMs' waves markedly better (the split
// costs an fp32 partial round trip and a sum kernel): e.g. 168 CTAs on 148 SMs run as two waves at 57%
// occupancy, 336 as three at 76%.
int dkdv_split(const dim3& g, int grp, int device) {
  const int sms = sm_count(device);
  const int ctas = (int)(g.x * g.y);
  auto util = [&](int n) {
    const int c = ctas * n;
    return (double)c / (double)(((c + sms - 1) / sms) * sms);
  };
  int nsplit = 1;
  double best = util(1);
  for (int n = 2; n <= grp && grp % n == 0; n *= 2) {
    if (util(n) > best * 1.15) {
      best = util(n);
      nsplit = n;
    }
  }
  return nsplit;
}

template <int D>
void launch_dkdv_t(dim3 g, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                   const CUtensorMap& mo, const at::Tensor& lse, const at::Tensor& delta, at::Tensor& dk,
                   at::Tensor& dv, int T, int S, int Hq, int Hkv, double scale, const PackTabs& tb, int* err) {
  const int nsplit = dkdv_split(g, Hq / Hkv, dk.get_device());
  g.z = nsplit;
  at::Tensor pk, pv;
  float* ppk = nullptr;
  float* ppv = nullptr;
  if (nsplit > 1) {
    pk = at::empty({nsplit, S, Hkv, D}, dk.options().dtype(at::kFloat));
    pv = at::empty({nsplit, S, Hkv, D}, dv.options().dtype(at::kFloat));
    ppk = pk.data_ptr<float>();
    ppv = pv.data_ptr<float>();
  }
  const int smem = DkvTLayout<D>::TOTAL + 1024;
  ensure_smem((const void*)attn_bwd_dkdv_t_kernel<D>, smem);
  attn_bwd_dkdv_t_kernel<D><<<g, 320, smem, stream()>>>(mq, mk, mv, mo, lse.data_ptr<float>(),
                                                        delta.data_ptr<float>(), (bf16*)dk.data_ptr(),
                                                        (bf16*)dv.data_ptr(), ppk, ppv, T, S, Hq, Hkv, (float)scale,
                                                        tb.ktab, tb.cons, T, S, err);
  if (nsplit > 1) {
    // with tables the key items cover every key row (rows nobody reads get an item without consumers,
    // which writes zeros), so every partial row summed here was written
    const long long n = (long long)S * Hkv * D;
    const int blocks = (int)((n / 4 + 255) / 256);
    attn_split_sum_kernel<<<blocks, 256, 0, stream()>>>(ppk, (bf16*)dk.data_ptr(), n, nsplit, (float)scale);
    attn_split_sum_kernel<<<blocks, 256, 0, stream()>>>(ppv, (bf16*)dv.data_ptr(), n, nsplit, 1.f);
  }
}

template <int MODE>
void launch_dkdv256(dim3 g, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                    const CUtensorMap& mo, const at::Tensor& lse, const at::Tensor& delta, at::Tensor& out, int T,
                    int S, int Hq, int Hkv, double scale, const PackTabs& tb, int* err) {
  const int nsplit = dkdv_split(g, Hq / Hkv, out.get_device());
  g.z = nsplit;
  at::Tensor part;
  float* pp = nullptr;
  if (nsplit > 1) {
    part = at::empty({nsplit, S, Hkv, 256}, out.options().dtype(at::kFloat));
    pp = part.data_ptr<float>();
  }
  const int smem = Dkv256Layout<MODE>::TOTAL + 1024;
  ensure_smem((const void*)attn_bwd_dkdv256_kernel<MODE>, smem);
  attn_bwd_dkdv256_kernel<MODE><<<g, 320, smem, stream()>>>(mq, mk, mv, mo, lse.data_ptr<float>(),
                                                            delta.data_ptr<float>(), (bf16*)out.data_ptr(), pp, T, S,
                                                            Hq, Hkv, (float)scale, tb.ktab, tb.cons, T, S, err);
  if (nsplit > 1) {
    const long long n = (long long)S * Hkv * 256;
    const int blocks = (int)((n / 4 + 255) / 256);
    attn_split_sum_kernel<<<blocks, 256, 0, stream()>>>(pp, (bf16*)out.data_ptr(), n, nsplit,
                                                        MODE == 1 ? (float)scale : 1.f);
  }
}

template <int D>
void launch_dq_t(dim3 g, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
                 const at::Tensor& lse, const at::Tensor& delta, at::Tensor& dq, int T, int S, int Hq, int Hkv,
                 double scale, const PackTabs& tb, int* err) {
  const int smem = DqTLayout<D>::TOTAL + 1024;
  ensure_smem((const void*)attn_bwd_dq_t_kernel<D>, smem);
  attn_bwd_dq_t_kernel<D><<<g, DqTLayout<D>::THREADS, smem, stream()>>>(mq, mk, mv, mo, lse.data_ptr<float>(),
                                                      delta.data_ptr<float>(), (bf16*)dq.data_ptr(), T, S, Hq, Hkv,
                                                      (float)scale, tb.qtab, tb.far, T, err);
}

void launch_dq256(dim3 g, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mo,
                  const at::Tensor& lse, const at::Tensor& delta, at::Tensor& dq, int T, int S, int Hq, int Hkv,
                  double scale, const PackTabs& tb, int* err) {
  const int smem = Dq256Layout::TOTAL + 1024;
  ensure_smem((const void*)attn_bwd_dq256_kernel<256>, smem);
  attn_bwd_dq256_kernel<256><<<g, 320, smem, stream()>>>(mq, mk, mv, mo, lse.data_ptr<float>(),
                                                         delta.data_ptr<float>(), (bf16*)dq.data_ptr(), T, S, Hq, Hkv,
                                                         (float)scale, tb.qtab, tb.far, T, err);
}

// T / S: total query and key rows (one segment without tables)
void run_bwd(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
             const at::Tensor& o, const at::Tensor& lse, double scale, at::Tensor& dq, at::Tensor& dk,
             at::Tensor& dv, const PackTabs& tb) {
  const int T = q.size(0), Hq = q.size(1), D = q.size(2), S = k.size(0), Hkv = k.size(1);
  auto delta = at::empty({Hq, T}, q.options().dtype(at::kFloat));
  const long long items = (long long)T * Hq;
  attn_delta_kernel<<<(int)((items + 7) / 8), 256, 0, stream()>>>((const bf16*)o.data_ptr(),
                                                                  (const bf16*)dout.data_ptr(),
                                                                  delta.data_ptr<float>(), T, Hq, D);
  int* err = tc_error_flag(q.device()).data_ptr<int>();
  CUtensorMap mk128 = make_bf16_map(k.data_ptr(), (uint64_t)Hkv * D, S, (uint64_t)Hkv * D, 128);
  CUtensorMap mv128 = make_bf16_map(v.data_ptr(), (uint64_t)Hkv * D, S, (uint64_t)Hkv * D, 128);
  CUtensorMap mq128 = make_bf16_map(q.data_ptr(), (uint64_t)Hq * D, T, (uint64_t)Hq * D, 128);
  CUtensorMap mo128 = make_bf16_map(dout.data_ptr(), (uint64_t)Hq * D, T, (uint64_t)Hq * D, 128);
  const bool packed = tb.qtab != nullptr;
  dim3 g1(packed ? tb.nk : (S + 127) / 128, Hkv), g2(packed ? tb.nq : (T + 127) / 128, Hq);
  if (D == 128) {
    if (g1.x) launch_dkdv_t<128>(g1, mq128, mk128, mv128, mo128, lse, delta, dk, dv, T, S, Hq, Hkv, scale, tb, err);
    if (g2.x) launch_dq_t<128>(g2, mq128, mk128, mv128, mo128, lse, delta, dq, T, S, Hq, Hkv, scale, tb, err);
  } else if (D == 64) {
    if (g1.x) launch_dkdv_t<64>(g1, mq128, mk128, mv128, mo128, lse, delta, dk, dv, T, S, Hq, Hkv, scale, tb, err);
    if (g2.x) launch_dq_t<64>(g2, mq128, mk128, mv128, mo128, lse, delta, dq, T, S, Hq, Hkv, scale, tb, err);
  } else {
    // dK and dV passes step over 64-query tiles, dQ over 64-key tiles
    CUtensorMap mq64 = make_bf16_map(q.data_ptr(), (uint64_t)Hq * D, T, (uint64_t)Hq * D, 64);
    CUtensorMap mo64 = make_bf16_map(dout.data_ptr(), (uint64_t)Hq * D, T, (uint64_t)Hq * D, 64);
    if (g1.x) {
      launch_dkdv256<1>(g1, mq64, mk128, mv128, mo64, lse, delta, dk, T, S, Hq, Hkv, scale, tb, err);
      launch_dkdv256<2>(g1, mq64, mk128, mv128, mo64, lse, delta, dv, T, S, Hq, Hkv, scale, tb, err);
    }
    CUtensorMap mk64 = make_bf16_map(k.data_ptr(), (uint64_t)Hkv * D, S, (uint64_t)Hkv * D, 64);
    CUtensorMap mv64 = make_bf16_map(v.data_ptr(), (uint64_t)Hkv * D, S, (uint64_t)Hkv * D, 64);
    if (g2.x) launch_dq256(g2, mq128, mk64, mv64, mo128, lse, delta, dq, T, S, Hq, Hkv, scale, tb, err);
  }
  TS_LAUNCH_CHECK();
}

void check_bwd_inputs(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k, const at::Tensor& v,
                      const at::Tensor& o, const at::Tensor& lse) {
  check_attn_inputs(q, k, v);
  check_cuda(o, "o");
  check_cuda(dout, "dout");
  check_cuda(lse, "lse");
  const int D = q.size(2);
  TS_CHECK(D == 64 || D == 128 || D == 256, "attention backward: head_dim 64, 128 or 256");
  TS_CHECK(o.sizes() == q.sizes() && dout.sizes() == q.sizes() && o.is_contiguous() && dout.is_contiguous(),
           "attention backward: o and dout must be contiguous and shaped like q");
  TS_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.dim() == 2 && lse.size(0) == q.size(1) &&
               lse.size(1) == q.size(0),
           "attention backward: lse must be a contiguous fp32 [Hq, T] tensor");
}

}  // namespace

// dq/dk/dv (optional): contiguous tensors shaped like q/k/v that receive the gradients.
std::vector<at::Tensor> attn_bwd_tc(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                    const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse, double scale,
                                    const c10::optional<at::Tensor>& dq_out, const c10::optional<at::Tensor>& dk_out,
                                    const c10::optional<at::Tensor>& dv_out) {
  check_bwd_inputs(dout, q, k, v, o, lse);
  const c10::cuda::CUDAGuard guard(q.device());
  TS_CHECK(k.size(0) >= q.size(0), "attention backward: more queries than keys");
  auto dq = out_or_new(dq_out, q, "attention dq");
  auto dk = out_or_new(dk_out, k, "attention dk");
  auto dv = out_or_new(dv_out, v, "attention dv");
  if (q.size(0) == 0) return {dq, dk.zero_(), dv.zero_()};
  run_bwd(dout, q, k, v, o, lse, scale, dq, dk, dv, PackTabs{});
  return {dq, dk, dv};
}

// Packed backward over the tables of attn_fwd_packed plus the key-side tables (KItem / consumers). The key
// items must cover every row of k (an item without consumers writes zero gradients); rows of dq that no
// query item covers are left untouched.
std::vector<at::Tensor> attn_bwd_packed(const at::Tensor& dout, const at::Tensor& q, const at::Tensor& k,
                                        const at::Tensor& v, const at::Tensor& o, const at::Tensor& lse,
                                        const at::Tensor& qtab, const at::Tensor& far, const at::Tensor& ktab,
                                        const at::Tensor& cons, double scale,
                                        const c10::optional<at::Tensor>& dq_out,
                                        const c10::optional<at::Tensor>& dk_out,
                                        const c10::optional<at::Tensor>& dv_out) {
  check_bwd_inputs(dout, q, k, v, o, lse);
  const c10::cuda::CUDAGuard guard(q.device());
  auto dq = out_or_new(dq_out, q, "attention dq");
  auto dk = out_or_new(dk_out, k, "attention dk");
  auto dv = out_or_new(dv_out, v, "attention dv");
  const PackTabs tb = pack_tabs(q, qtab, far, ktab, cons);
  if (q.size(0) == 0 || (tb.nq == 0 && tb.nk == 0)) return {dq, dk, dv};
  run_bwd(dout, q, k, v, o, lse, scale, dq, dk, dv, tb);
  return {dq, dk, dv};
}

}  // namespace ts
