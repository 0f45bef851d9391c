// tcgen05 GEMM for the projection shapes of the decoder (S4).
//
//   C[M, N] (op)= A[M, K] · B[K, N]
//
// A is K-major ([M][K] row-major) or M-major ([K][M] row-major, i.e. a
// transposed operand); B is K-major ([N][K] row-major, an nn.Linear weight)
// or N-major ([K][N] row-major). That covers y = x·Wᵀ (A, B K-major),
// dx = dy·W (B N-major) and dW = dyᵀ·x (A M-major, B N-major) without a
// transpose copy. The epilogue writes bf16, writes fp32, or adds into an fp32
// C (the gradient-sink accumulate: beta = 1).
//
// Persistent kernel, one CTA per SM, 128 x 256 output tiles, 64-deep K
// blocks in a 4-stage TMA ring:
//   warp 0  TMA producer (one elected lane)
//   warp 1  MMA issuer (one elected lane): tcgen05.mma into one of two TMEM
//           accumulators (2 x 256 columns), so the epilogue of tile i overlaps
//           the main loop of tile i+1
//   warps 2-5  epilogue: tcgen05.ld of its 32-lane TMEM sub-partition (rows),
//           convert, store
// Every wait is bounded (tc::mbar_wait); TMEM is always freed.
#include "common.cuh"
#include "common.h"
#include "tc.cuh"

#include <cuda.h>

namespace ts {

CUtensorMap make_bf16_map(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                          uint32_t box_rows);
at::Tensor& tc_error_flag(const at::Device& dev);

namespace {

typedef __nv_bfloat16 bf16;

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
constexpr uint32_t kBarOff = kStages * kStageBytes;  // 192 KB
constexpr uint32_t kSmem = kBarOff + 256;

enum Epi { kStoreBf16 = 0, kStoreF32 = 1, kAccumF32 = 2, kLse = 3, kDlogits = 4 };

// Per-row data of the LM-head epilogues (C = hidden · Wᵀ are the logits).
// kLse: per (row, N tile) online max / sum of exp / sum of exp·x partials and
//   the target's logit, reduced by lse_reduce_kernel; the [rows, V] logits
//   never reach memory.
// kDlogits: dlogits = g·(onehot(target) − softmax) (entropy adds
//   −p·g_H·(log p + H)), written as bf16.
struct LmArgs {
  const int64_t* tgt;
  float* pm;   // [rows][ntiles] tile max (log2 units)
  float* ps;   // [rows][ntiles] sum of 2^(x·log2e − m)
  float* pt;   // [rows][ntiles] sum of 2^(x·log2e − m) · x  (entropy), or null
  float* tlogit;  // [rows] logit of the target
  const float* lse;
  const float* glp;
  const float* gent;  // or null
  const float* ent;   // or null
  int ntiles;
};
constexpr float kLog2eF = 1.4426950408889634f;

TS_DEVICE float ex2f(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct GemmBars {
  uint64_t full[kStages], empty[kStages], acc_full[2], acc_empty[2];
  uint32_t tmem_slot;
  int abort;
};

TS_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// tile t -> (m block, n block), grouped so that consecutive tiles of a CTA
// wave share B columns (L2 reuse of the weight)
TS_DEVICE void tile_coords(int t, int mt, int nt, int& mb, int& nb) {
  constexpr int G = 8;
  const int per_group = G * nt;
  const int g = t / per_group;
  const int first_m = g * G;
  const int gm = min(G, mt - first_m);
  const int r = t % per_group;
  mb = first_m + r % gm;
  nb = r / gm;
}

// Epilogue of one output tile for the calling thread's row: reads the row's kBN fp32 accumulator
// columns from tensor memory at `tacc` (32 at a time) and stores / accumulates / reduces them.
template <int EPI>
TS_DEVICE void epilogue_tile(uint32_t tacc, int row, int nb, int M, int N, int ldc, float alpha, void* c,
                             const LmArgs& lm) {
  const int col0 = nb * kBN;
  // LM-head row state (one row per thread)
  float run_m = -INFINITY, run_s = 0.f, run_t = 0.f, row_lse = 0.f, row_g = 0.f, row_ge = 0.f, row_h = 0.f;
  int64_t row_tgt = -1;
  if constexpr (EPI == kLse || EPI == kDlogits) {
    if (row < M) {
      row_tgt = lm.tgt[row];
      if constexpr (EPI == kDlogits) {
        row_lse = lm.lse[row];
        row_g = lm.glp[row];
        if (lm.gent != nullptr) {
          row_ge = lm.gent[row];
          row_h = lm.ent[row];
        }
      }
    }
  }
#pragma unroll 1
  for (int cc = 0; cc < kBN; cc += 32) {
    float v[32];
    tc::tmem_ld32(tacc + cc, v);
    tc::tmem_ld_wait();
    const int col = col0 + cc;
    if constexpr (EPI == kLse) {
      if (row < M && col < N) {
        float cm = -INFINITY;
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          if (col + x < N) cm = fmaxf(cm, v[x] * kLog2eF);
          if (col + x == row_tgt) lm.tlogit[row] = v[x];
        }
        if (cm > run_m) {
          const float r = ex2f(run_m - cm);
          run_s *= r;
          run_t *= r;
          run_m = cm;
        }
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          if (col + x < N) {
            const float e = ex2f(fmaf(v[x], kLog2eF, -run_m));
            run_s += e;
            run_t = fmaf(e, v[x], run_t);
          }
        }
      }
      continue;
    }
    if constexpr (EPI == kDlogits) {
      if (row < M && col < N) {
        bf16* p = reinterpret_cast<bf16*>(c) + (long long)row * ldc + col;
        const float l2 = row_lse * kLog2eF;
        float d[32];
#pragma unroll
        for (int x = 0; x < 32; ++x) {
          const float pr = ex2f(fmaf(v[x], kLog2eF, -l2));
          float g = row_g;
          if (lm.gent != nullptr) g += row_ge * ((v[x] - row_lse) + row_h);
          d[x] = -pr * g + (col + x == row_tgt ? row_g : 0.f);
        }
        if (col + 32 <= N) {
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 u;
            u.x = pack_bf16(d[x], d[x + 1]);
            u.y = pack_bf16(d[x + 2], d[x + 3]);
            u.z = pack_bf16(d[x + 4], d[x + 5]);
            u.w = pack_bf16(d[x + 6], d[x + 7]);
            *reinterpret_cast<uint4*>(p + x) = u;
          }
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x)
            if (col + x < N) p[x] = __float2bfloat16_rn(d[x]);
        }
      }
      continue;
    }
    if (row < M && col < N) {
      const bool full = col + 32 <= N;
      if constexpr (EPI == kStoreBf16) {
        bf16* p = reinterpret_cast<bf16*>(c) + (long long)row * ldc + col;
        if (full) {
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 u;
            u.x = pack_bf16(alpha * v[x], alpha * v[x + 1]);
            u.y = pack_bf16(alpha * v[x + 2], alpha * v[x + 3]);
            u.z = pack_bf16(alpha * v[x + 4], alpha * v[x + 5]);
            u.w = pack_bf16(alpha * v[x + 6], alpha * v[x + 7]);
            *reinterpret_cast<uint4*>(p + x) = u;
          }
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x)
            if (col + x < N) p[x] = __float2bfloat16_rn(alpha * v[x]);
        }
      } else {
        float* p = reinterpret_cast<float*>(c) + (long long)row * ldc + col;
        if (full) {
#pragma unroll
          for (int x = 0; x < 32; x += 4) {
            float4 o = make_float4(alpha * v[x], alpha * v[x + 1], alpha * v[x + 2], alpha * v[x + 3]);
            if constexpr (EPI == kAccumF32) {
              const float4 prev = *reinterpret_cast<const float4*>(p + x);
              o.x += prev.x; o.y += prev.y; o.z += prev.z; o.w += prev.w;
            }
            *reinterpret_cast<float4*>(p + x) = o;
          }
        } else {
#pragma unroll
          for (int x = 0; x < 32; ++x)
            if (col + x < N) p[x] = (EPI == kAccumF32 ? p[x] : 0.f) + alpha * v[x];
        }
      }
    }
  }
  if constexpr (EPI == kLse) {
    if (row < M) {
      const long long o = (long long)row * lm.ntiles + nb;
      lm.pm[o] = run_m;
      lm.ps[o] = run_s;
      if (lm.pt != nullptr) lm.pt[o] = run_t;
    }
  }
}

template <bool A_MN, bool B_MN, int EPI>
__global__ void __launch_bounds__(192, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a,
                                                         const __grid_constant__ CUtensorMap tm_b,
                                                         const __grid_constant__ CUtensorMap tm_a2,
                                                         const __grid_constant__ CUtensorMap tm_b2, int K2,
                                                         void* __restrict__ c,
                                                         int M, int N, int K, int ldc, float alpha,
                                                         int* __restrict__ err, LmArgs lm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmBars* bars = reinterpret_cast<GemmBars*>(smem + kBarOff);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = (M + kBM - 1) / kBM, nt = (N + kBN - 1) / kBN, kt1 = (K + kBK - 1) / kBK, kt = kt1 + (K2 + kBK - 1) / kBK;
  const int tiles = mt * nt;
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      tc::mbar_init(&bars->full[s], 1);
      tc::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&bars->acc_full[b], 1);
      tc::mbar_init(&bars->acc_empty[b], 128);
    }
    bars->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc(&bars->tmem_slot, 512);
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_tmap(&tm_a);
      tc::prefetch_tmap(&tm_b);
      if (K2 > 0) {
        tc::prefetch_tmap(&tm_a2);
        tc::prefetch_tmap(&tm_b2);
      }
      int it = 0;
      for (int t = blockIdx.x; t < tiles; t += gridDim.x) {
        int mb, nb;
        tile_coords(t, mt, nt, mb, nb);
        for (int kb = 0; kb < kt; ++kb, ++it) {
          const int s = it % kStages;
          if (it >= kStages && !tc::mbar_wait(&bars->empty[s], ((it - kStages) / kStages) & 1, abort, err, 201))
            goto producer_done;
          tc::mbar_expect_tx(&bars->full[s], kStageBytes);
          uint8_t* a = smem + s * kStageBytes;
          uint8_t* b = a + kABytes;
          // K blocks past the first source's come from the second (A2, B2): out = A·B + A2·B2
          const bool second = kb >= kt1;
          const CUtensorMap* pa = second ? &tm_a2 : &tm_a;
          const CUtensorMap* pb = second ? &tm_b2 : &tm_b;
          const int kx = (second ? kb - kt1 : kb) * kBK;
          if constexpr (!A_MN) {
            tc::tma_load_2d(a, pa, kx, mb * kBM, &bars->full[s]);  // box 64 (k) x 128 (m)
          } else {
            // [K][M]: two boxes of 64 m-columns x 64 k-rows
            tc::tma_load_2d(a, pa, mb * kBM, kx, &bars->full[s]);
            tc::tma_load_2d(a + 64 * 128, pa, mb * kBM + 64, kx, &bars->full[s]);
          }
          if constexpr (!B_MN) {
            tc::tma_load_2d(b, pb, kx, nb * kBN, &bars->full[s]);  // box 64 (k) x 256 (n)
          } else {
#pragma unroll
            for (int j = 0; j < kBN / 64; ++j)  // [K][N]: four boxes of 64 n-columns x 64 k-rows
              tc::tma_load_2d(b + j * 64 * 128, pb, nb * kBN + j * 64, kx, &bars->full[s]);
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_bf16(kBM, kBN, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !tc::mbar_wait(&bars->acc_empty[buf], ((local - 2) >> 1) & 1, abort, err, 211)) break;
        tc::tc_fence_after();
        const uint32_t acc = tmem + buf * kBN;
        for (int kb = 0; kb < kt; ++kb, ++it) {
          const int s = it % kStages;
          if (!tc::mbar_wait(&bars->full[s], (it / kStages) & 1, abort, err, 212)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a = sbase + s * kStageBytes;
          const uint32_t b = a + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            // K-major: +32 bytes per 16-element K step; MN-major: +16 rows of 128 bytes
            const uint64_t ad = A_MN ? tc::sdesc_sw128(a + kk * 16 * 128, 64 * 128, 1024)
                                     : tc::sdesc_sw128(a + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? tc::sdesc_sw128(b + kk * 16 * 128, 64 * 128, 1024)
                                     : tc::sdesc_sw128(b + kk * 32, 16, 1024);
            tc::mma_bf16(acc, ad, bd, idesc, kb > 0 || kk > 0);
          }
          tc::mma_commit(&bars->empty[s]);
        }
        if (ok) tc::mma_commit(&bars->acc_full[buf]);
      }
    }
  } else {
    // epilogue warps 2..5: TMEM sub-partition (warp & 3) -> rows 32*(warp&3) .. +32
    const int sub = warp & 3;
    const int row_in_tile = sub * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(sub * 32) << 16);
    int local = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int buf = local & 1;
      bool ok = true;
      if ((threadIdx.x & 31) == 0) ok = tc::mbar_wait(&bars->acc_full[buf], (local >> 1) & 1, abort, err, 221);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc::tc_fence_after();
      int mb, nb;
      tile_coords(t, mt, nt, mb, nb);
      epilogue_tile<EPI>(lane_base + buf * kBN, mb * kBM + row_in_tile, nb, M, N, ldc, alpha, c, lm);
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->acc_empty[buf]);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ CTA-pair kernel (cta_group::2)
// A cluster of two CTAs on two SMs computes a 256 x 256 tile: each CTA
// stages 128 rows of A and 128 rows (N) of B per K block, the even CTA
// issues tcgen05.mma.cta_group::2 (M = 256) over both CTAs' shared memory,
// and each CTA's tensor memory receives its 128 rows of the accumulator.
// Per SM that halves the B bytes staged per MMA against the single-CTA
// 128 x 256 tile (32 KB instead of 48 KB per 64-deep K block). Every TMA
// load of the pair counts its bytes on the even CTA's `full` barrier; the
// MMA completion arrives on the `empty` / `acc_full` barriers of both CTAs;
// the eight epilogue warps of the pair arrive on the even CTA's
// `acc_empty`. Loads have no multicast: each CTA reads its own rows.
constexpr int kStagesP = 6;
constexpr uint32_t kBHalfBytes = 128 * kBK * 2;                 // 16 KB
constexpr uint32_t kStagePBytes = kABytes + kBHalfBytes;        // 32 KB per CTA
constexpr uint32_t kBarOffP = kStagesP * kStagePBytes;          // 192 KB
constexpr uint32_t kSmemP = kBarOffP + 256;
static_assert(kSmemP + 1024 <= 232448, "pair GEMM shared memory");

struct PairBars {
  uint64_t full[kStagesP], empty[kStagesP], acc_full[2], acc_empty[2];
  uint32_t tmem_slot;
  int abort;
};

template <bool A_MN, bool B_MN, int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(192, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_a2, const __grid_constant__ CUtensorMap tm_b2, int K2,
                     void* __restrict__ c, int M, int N, int K, int ldc, float alpha, int* __restrict__ err,
                     LmArgs lm) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + kBarOffP);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_rank();
  const int mt = (M + 2 * kBM - 1) / (2 * kBM), nt = (N + kBN - 1) / kBN, kt1 = (K + kBK - 1) / kBK, kt = kt1 + (K2 + kBK - 1) / kBK;
  const int tiles = mt * nt;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  volatile int* abort = &bars->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesP; ++s) {
      tc::mbar_init(&bars->full[s], 1);
      tc::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&bars->acc_full[b], 1);
      tc::mbar_init(&bars->acc_empty[b], 8);  // one arrival per epilogue warp of the pair
    }
    bars->abort = 0;
    tc::fence_barrier_init();
  }
  if (warp == 1) tc::tmem_alloc_pair(&bars->tmem_slot, 512);
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // both CTAs' barriers exist before any remote arrive or byte count
  tc::tc_fence_after();
  const uint32_t tmem = bars->tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tc::prefetch_tmap(&tm_a);
      tc::prefetch_tmap(&tm_b);
      if (K2 > 0) {
        tc::prefetch_tmap(&tm_a2);
        tc::prefetch_tmap(&tm_b2);
      }
      int it = 0;
      for (int t = cid; t < tiles; t += ncl) {
        int mb, nb;
        tile_coords(t, mt, nt, mb, nb);
        const int arow = mb * 2 * kBM + (int)rank * kBM;
        const int bcol = nb * kBN + (int)rank * (kBN / 2);
        for (int kb = 0; kb < kt; ++kb, ++it) {
          const int s = it % kStagesP;
          if (it >= kStagesP && !tc::mbar_wait(&bars->empty[s], ((it - kStagesP) / kStagesP) & 1, abort, err, 231))
            goto producer_done;
          if (rank == 0) tc::mbar_expect_tx(&bars->full[s], 2 * kStagePBytes);
          const uint32_t full0 = tc::map_cluster(tc::smem_addr(&bars->full[s]), 0);
          uint8_t* a = smem + s * kStagePBytes;
          uint8_t* b = a + kABytes;
          const bool second = kb >= kt1;
          const CUtensorMap* pa = second ? &tm_a2 : &tm_a;
          const CUtensorMap* pb = second ? &tm_b2 : &tm_b;
          const int kx = (second ? kb - kt1 : kb) * kBK;
          if constexpr (!A_MN) {
            tc::tma_load_2d_pair(a, pa, kx, arow, full0);  // box 64 (k) x 128 (m)
          } else {
            tc::tma_load_2d_pair(a, pa, arow, kx, full0);  // [K][M]: 2 boxes of 64 m x 64 k
            tc::tma_load_2d_pair(a + 64 * 128, pa, arow + 64, kx, full0);
          }
          if constexpr (!B_MN) {
            tc::tma_load_2d_pair(b, pb, kx, bcol, full0);  // box 64 (k) x 128 (n)
          } else {
            tc::tma_load_2d_pair(b, pb, bcol, kx, full0);  // [K][N]: 2 boxes of 64 n x 64 k
            tc::tma_load_2d_pair(b + 64 * 128, pb, bcol + 64, kx, full0);
          }
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      const uint32_t idesc = tc::idesc_bf16(2 * kBM, kBN, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = cid; ok && t < tiles; t += ncl, ++local) {
        const int buf = local & 1;
        if (local >= 2 && !tc::mbar_wait(&bars->acc_empty[buf], ((local - 2) >> 1) & 1, abort, err, 241)) break;
        tc::tc_fence_after();
        const uint32_t acc = tmem + buf * kBN;
        for (int kb = 0; kb < kt; ++kb, ++it) {
          const int s = it % kStagesP;
          if (!tc::mbar_wait(&bars->full[s], (it / kStagesP) & 1, abort, err, 242)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint32_t a = sbase + s * kStagePBytes;
          const uint32_t b = a + kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? tc::sdesc_sw128(a + kk * 16 * 128, 64 * 128, 1024)
                                     : tc::sdesc_sw128(a + kk * 32, 16, 1024);
            const uint64_t bd = B_MN ? tc::sdesc_sw128(b + kk * 16 * 128, 64 * 128, 1024)
                                     : tc::sdesc_sw128(b + kk * 32, 16, 1024);
            tc::mma_bf16_pair(acc, ad, bd, idesc, kb > 0 || kk > 0);
          }
          tc::mma_commit_pair(&bars->empty[s]);
        }
        if (ok) tc::mma_commit_pair(&bars->acc_full[buf]);
      }
    }
  } else {
    const int sub = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(sub * 32) << 16);
    const uint32_t acc_empty0 = tc::map_cluster(tc::smem_addr(&bars->acc_empty[0]), 0);
    const uint32_t acc_empty1 = tc::map_cluster(tc::smem_addr(&bars->acc_empty[1]), 0);
    int local = 0;
    for (int t = cid; t < tiles; t += ncl, ++local) {
      const int buf = local & 1;
      bool ok = true;
      if (lane == 0) ok = tc::mbar_wait(&bars->acc_full[buf], (local >> 1) & 1, abort, err, 251);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc::tc_fence_after();
      int mb, nb;
      tile_coords(t, mt, nt, mb, nb);
      const int row = mb * 2 * kBM + (int)rank * kBM + sub * 32 + lane;
      epilogue_tile<EPI>(lane_base + buf * kBN, row, nb, M, N, ldc, alpha, c, lm);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive_cluster(buf ? acc_empty1 : acc_empty0);
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // no CTA leaves while its pair may still read its shared memory or arrive on it
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc_pair(tmem, 512);
  }
}

// 0: single-CTA 128 x 256 tiles; 1: CTA-pair 256 x 256 tiles (default)
int g_gemm_pair = 1;

template <bool A_MN, bool B_MN, int EPI>
void launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, void* c, int M, int N, int K, int ldc, float alpha,
                 int device, LmArgs lm, const CUtensorMap* ma2 = nullptr, const CUtensorMap* mb2 = nullptr,
                 int K2 = 0) {
  const int tiles = ((M + 2 * kBM - 1) / (2 * kBM)) * ((N + kBN - 1) / kBN);
  const int smem = kSmemP + 1024;
  static int resident[16] = {0};  // co-resident CTA pairs per device (persistent grid size)
  int& pairs = resident[device & 15];
  if (pairs == 0) {
    TS_CUDA_CHECK(cudaFuncSetAttribute(gemm_pair_kernel<A_MN, B_MN, EPI>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * sm_count(device));
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<A_MN, B_MN, EPI>, &cfg) != cudaSuccess || n <= 0) {
      (void)cudaGetLastError();
      n = sm_count(device) / 2;
    }
    pairs = std::min(n, sm_count(device) / 2);
  }
  const int clusters = std::max(1, std::min(tiles, pairs));
  gemm_pair_kernel<A_MN, B_MN, EPI><<<2 * clusters, 192, smem, stream()>>>(
      ma, mb, ma2 ? *ma2 : ma, mb2 ? *mb2 : mb, ma2 ? K2 : 0, c, M, N, K, ldc, alpha,
      tc_error_flag(at::Device(at::kCUDA, device)).data_ptr<int>(), lm);
}

template <bool A_MN, bool B_MN, int EPI>
void launch(const CUtensorMap& ma, const CUtensorMap& mb, void* c, int M, int N, int K, int ldc, float alpha,
            int device, LmArgs lm = LmArgs{}, const CUtensorMap* ma2 = nullptr, const CUtensorMap* mb2 = nullptr,
            int K2 = 0) {
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  const int grid = std::max(1, std::min(tiles, sm_count(device)));
  const int smem = kSmem + 1024;
  ensure_smem((const void*)gemm_tc_kernel<A_MN, B_MN, EPI>, smem);
  gemm_tc_kernel<A_MN, B_MN, EPI><<<grid, 192, smem, stream()>>>(ma, mb, ma2 ? *ma2 : ma, mb2 ? *mb2 : mb,
                                                                  ma2 ? K2 : 0, c, M, N, K, ldc, alpha,
                                                                  tc_error_flag(at::Device(at::kCUDA, device))
                                                                      .data_ptr<int>(),
                                                                  lm);
}

// One warp per row: combine the tile partials into lse (and entropy), lp = target logit − lse.
__global__ void lse_reduce_kernel(const float* __restrict__ pm, const float* __restrict__ ps,
                                  const float* __restrict__ pt, const float* __restrict__ tlogit,
                                  float* __restrict__ lp, float* __restrict__ lse, float* __restrict__ ent, int rows,
                                  int ntiles) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* m = pm + (long long)row * ntiles;
  const float* sm = ps + (long long)row * ntiles;
  float mx = -INFINITY;
  for (int i = lane; i < ntiles; i += 32) mx = fmaxf(mx, m[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = 0.f, t = 0.f;
  for (int i = lane; i < ntiles; i += 32) {
    const float r = ex2f(m[i] - mx);
    s = fmaf(sm[i], r, s);
    if (pt != nullptr) t = fmaf(pt[(long long)row * ntiles + i], r, t);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    t += __shfl_xor_sync(0xffffffffu, t, o);
  }
  if (lane == 0) {
    const float l = (mx + log2f(s)) * 0.6931471805599453f;  // natural-log LSE
    lse[row] = l;
    lp[row] = tlogit[row] - l;
    if (ent != nullptr) ent[row] = l - t / s;
  }
}

}  // namespace

// Select the GEMM kernel: 1 = CTA-pair 256 x 256 tiles, 0 = single-CTA 128 x 256 tiles. Returns the previous value.
int64_t gemm_tc_pair(int64_t on) {
  const int prev = g_gemm_pair;
  if (on >= 0) g_gemm_pair = on ? 1 : 0;
  return prev;
}

// Fused LM-head forward: lp[r] = log softmax(h W^T)[r, tgt[r]] (+ entropy), lse[r];
// h [R, D] bf16, w [V, D] bf16; the logits never reach memory.
std::vector<at::Tensor> lmhead_lse_tc(const at::Tensor& h, const at::Tensor& w, const at::Tensor& tgt,
                                      bool with_entropy) {
  check_cuda(h, "h");
  check_cuda(w, "w");
  check_cuda(tgt, "tgt");
  TS_CHECK(h.scalar_type() == at::kBFloat16 && w.scalar_type() == at::kBFloat16 && tgt.scalar_type() == at::kLong,
           "lmhead_lse_tc takes bf16 h, w and int64 targets");
  const c10::cuda::CUDAGuard guard(h.device());
  const int R = h.size(0), D = h.size(1), V = w.size(0);
  TS_CHECK(w.size(1) == D && D % 8 == 0 && V % 8 == 0, "lmhead_lse_tc shapes");
  auto f32 = h.options().dtype(at::kFloat);
  auto lp = at::empty({R}, f32), lse = at::empty({R}, f32);
  auto ent = with_entropy ? at::empty({R}, f32) : at::Tensor();
  if (R == 0) return {lp, lse, ent};
  const int ntiles = (V + kBN - 1) / kBN;
  auto pm = at::empty({R, ntiles}, f32), ps = at::empty({R, ntiles}, f32);
  auto pt = with_entropy ? at::empty({R, ntiles}, f32) : at::Tensor();
  auto tl = at::zeros({R}, f32);
  LmArgs lm{tgt.data_ptr<int64_t>(), pm.data_ptr<float>(), ps.data_ptr<float>(),
            with_entropy ? pt.data_ptr<float>() : nullptr, tl.data_ptr<float>(), nullptr, nullptr, nullptr, nullptr,
            ntiles};
  const bool pair = g_gemm_pair != 0;
  const CUtensorMap ma = make_bf16_map(h.data_ptr(), D, R, D, 128);
  const CUtensorMap mb = make_bf16_map(w.data_ptr(), D, V, D, pair ? 128 : 256);
  if (pair) launch_pair<false, false, kLse>(ma, mb, nullptr, R, V, D, V, 1.f, h.get_device(), lm);
  else launch<false, false, kLse>(ma, mb, nullptr, R, V, D, V, 1.f, h.get_device(), lm);
  lse_reduce_kernel<<<(R + 7) / 8, 256, 0, stream()>>>(pm.data_ptr<float>(), ps.data_ptr<float>(),
                                                       with_entropy ? pt.data_ptr<float>() : nullptr,
                                                       tl.data_ptr<float>(), lp.data_ptr<float>(),
                                                       lse.data_ptr<float>(),
                                                       with_entropy ? ent.data_ptr<float>() : nullptr, R, ntiles);
  TS_LAUNCH_CHECK();
  return {lp, lse, ent};
}

// Fused LM-head backward epilogue: dlogits [R, V] bf16 from recomputed logits.
at::Tensor lmhead_dlogits_tc(const at::Tensor& h, const at::Tensor& w, const at::Tensor& tgt, const at::Tensor& lse,
                             const at::Tensor& glp, const c10::optional<at::Tensor>& gent,
                             const c10::optional<at::Tensor>& ent) {
  check_cuda(h, "h");
  check_cuda(w, "w");
  const c10::cuda::CUDAGuard guard(h.device());
  const int R = h.size(0), D = h.size(1), V = w.size(0);
  auto d = at::empty({R, V}, h.options());
  if (R == 0) return d;
  LmArgs lm{tgt.data_ptr<int64_t>(), nullptr, nullptr, nullptr, nullptr, lse.data_ptr<float>(), glp.data_ptr<float>(),
            gent ? gent->data_ptr<float>() : nullptr, ent ? ent->data_ptr<float>() : nullptr, 0};
  const bool pair = g_gemm_pair != 0;
  const CUtensorMap ma = make_bf16_map(h.data_ptr(), D, R, D, 128);
  const CUtensorMap mb = make_bf16_map(w.data_ptr(), D, V, D, pair ? 128 : 256);
  if (pair) launch_pair<false, false, kDlogits>(ma, mb, d.data_ptr(), R, V, D, V, 1.f, h.get_device(), lm);
  else launch<false, false, kDlogits>(ma, mb, d.data_ptr(), R, V, D, V, 1.f, h.get_device(), lm);
  TS_LAUNCH_CHECK();
  return d;
}

// out (op)= a · b, with a = a_t ? aᵀ : a and b = b_t ? bᵀ : b as seen by the
// math: a_t = false takes a as [M, K]; a_t = true takes a as [K, M].
// b_t = true takes b as [N, K] (nn.Linear weight); b_t = false as [K, N].
// mode 0: out bf16 [M, N] = alpha·a·b; mode 1: out fp32 = alpha·a·b;
// mode 2: out fp32 += alpha·a·b.
// out (op)= alpha · (a · b [+ a2 · b2]): the optional second operand pair shares M and N (and the
// transposition flags) and extends the contraction, its K blocks following the first pair's in the
// same main loop (a LoRA projection is x·Wᵀ + (s·x·Aᵀ)·Bᵀ in one kernel). With a second pair the
// first pair's K must be a multiple of 64.
void gemm_tc_cat(at::Tensor& out, const at::Tensor& a, const at::Tensor& b, const c10::optional<at::Tensor>& a2,
                 const c10::optional<at::Tensor>& b2, bool a_t, bool b_t, int64_t mode, double alpha) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  check_cuda(out, "out");
  TS_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_tc takes bf16 operands");
  TS_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm_tc takes matrices");
  TS_CHECK(a.is_contiguous() && b.is_contiguous(), "gemm_tc takes contiguous operands");
  const int M = a_t ? a.size(1) : a.size(0);
  const int K = a_t ? a.size(0) : a.size(1);
  const int N = b_t ? b.size(0) : b.size(1);
  TS_CHECK((b_t ? b.size(1) : b.size(0)) == K, "gemm_tc inner dimensions differ");
  TS_CHECK(out.size(0) == M && out.size(1) == N, "gemm_tc output shape");
  TS_CHECK(mode == 0 ? out.scalar_type() == at::kBFloat16 : out.scalar_type() == at::kFloat, "gemm_tc output dtype");
  // 16-byte TMA strides for every operand layout and 16-byte vector stores of C rows
  TS_CHECK(K % 8 == 0 && N % 8 == 0 && (!a_t || M % 8 == 0), "gemm_tc needs K, N (and M when a is [K, M]) "
           "to be multiples of 8");
  const bool two = a2.has_value();
  TS_CHECK(two == b2.has_value(), "gemm_tc: give both second operands or neither");
  int K2 = 0;
  if (two) {
    TS_CHECK(a2->scalar_type() == at::kBFloat16 && b2->scalar_type() == at::kBFloat16 && a2->is_contiguous() &&
                 b2->is_contiguous() && a2->dim() == 2 && b2->dim() == 2,
             "gemm_tc: second operands must be contiguous bf16 matrices");
    K2 = a_t ? a2->size(0) : a2->size(1);
    TS_CHECK((a_t ? a2->size(1) : a2->size(0)) == M && (b_t ? b2->size(0) : b2->size(1)) == N &&
                 (b_t ? b2->size(1) : b2->size(0)) == K2,
             "gemm_tc: second operand pair shapes");
    TS_CHECK(K % 64 == 0 && K2 % 8 == 0 && K2 > 0, "gemm_tc: with a second pair, K must be a multiple of 64");
  }
  const c10::cuda::CUDAGuard guard(a.device());
  if (M == 0 || N == 0) return;
  if (K == 0 && K2 == 0) {
    if (mode != 2) out.zero_();
    return;
  }
  // tensor maps: inner dimension first; boxes of 64 inner elements
  const bool pair = g_gemm_pair != 0;
  auto amap = [&](const at::Tensor& t, int k) {
    return a_t ? make_bf16_map(t.data_ptr(), M, k, M, 64) : make_bf16_map(t.data_ptr(), k, M, k, 128);
  };
  auto bmap = [&](const at::Tensor& t, int k) {
    return b_t ? make_bf16_map(t.data_ptr(), k, N, k, pair ? 128 : 256) : make_bf16_map(t.data_ptr(), N, k, N, 64);
  };
  const CUtensorMap ma = amap(a, K), mb = bmap(b, K);
  CUtensorMap ma2 = ma, mb2 = mb;
  if (two) {
    ma2 = amap(*a2, K2);
    mb2 = bmap(*b2, K2);
  }
  const CUtensorMap* pa2 = two ? &ma2 : nullptr;
  const CUtensorMap* pb2 = two ? &mb2 : nullptr;
  const int dev = a.get_device();
  void* c = out.data_ptr();
  const float al = (float)alpha;
  const LmArgs none{};
#define TS_GEMM_CASE(AM, BM)                                                                                  \
  if (pair) {                                                                                                 \
    if (mode == 0) launch_pair<AM, BM, kStoreBf16>(ma, mb, c, M, N, K, (int)N, al, dev, none, pa2, pb2, K2);  \
    else if (mode == 1) launch_pair<AM, BM, kStoreF32>(ma, mb, c, M, N, K, (int)N, al, dev, none, pa2, pb2, K2); \
    else launch_pair<AM, BM, kAccumF32>(ma, mb, c, M, N, K, (int)N, al, dev, none, pa2, pb2, K2);             \
  } else {                                                                                                    \
    if (mode == 0) launch<AM, BM, kStoreBf16>(ma, mb, c, M, N, K, (int)N, al, dev, none, pa2, pb2, K2);       \
    else if (mode == 1) launch<AM, BM, kStoreF32>(ma, mb, c, M, N, K, (int)N, al, dev, none, pa2, pb2, K2);   \
    else launch<AM, BM, kAccumF32>(ma, mb, c, M, N, K, (int)N, al, dev, none, pa2, pb2, K2);                  \
  }
  if (!a_t && b_t) {
    TS_GEMM_CASE(false, false)
  } else if (!a_t && !b_t) {
    TS_GEMM_CASE(false, true)
  } else if (a_t && !b_t) {
    TS_GEMM_CASE(true, true)
  } else {
    TS_GEMM_CASE(true, false)
  }
#undef TS_GEMM_CASE
  TS_LAUNCH_CHECK();
}

void gemm_tc(at::Tensor& out, const at::Tensor& a, const at::Tensor& b, bool a_t, bool b_t, int64_t mode,
             double alpha) {
  gemm_tc_cat(out, a, b, c10::nullopt, c10::nullopt, a_t, b_t, mode, alpha);
}

}  // namespace ts
