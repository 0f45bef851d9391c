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
//           convert, stage 32 x 32 chunks in swizzled shared memory and write
//           them with TMA stores (fp32 gradient accumulation: TMA reduce-add,
//           so the sink is never read by the SM); an optional bf16 residual
//           operand is added before the store (out = alpha·A·B + R)
// Every wait is bounded (tc::mbar_wait); TMEM is always freed.
#include "common.cuh"
#include "common.h"
#include "tc.cuh"

#include <cuda.h>

namespace ts {

CUtensorMap make_bf16_map(const void* base, uint64_t inner, uint64_t outer, uint64_t row_stride_elems,
                          uint32_t box_rows);
// Output map of the GEMM epilogue: [rows][cols] with a row stride of `ld` elements, 32 x 32 boxes,
// SWIZZLE_64B for bf16 (64-byte box rows) and SWIZZLE_128B for fp32 (128-byte box rows).
CUtensorMap make_out_map(void* base, bool f32, uint64_t cols, uint64_t rows, uint64_t ld);
at::Tensor& tc_error_flag(const at::Device& dev);

namespace {

typedef __nv_bfloat16 bf16;

constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr uint32_t kABytes = kBM * kBK * 2;  // 16 KB
constexpr uint32_t kBBytes = kBN * kBK * 2;  // 32 KB
constexpr uint32_t kStageBytes = kABytes + kBBytes;
// epilogue staging: 4 warps x 2 buffers x (32 rows x 128 B), 1024-aligned for the 128B swizzle
constexpr uint32_t kEpiBufBytes = 4096;
constexpr uint32_t kEpiBytes = 4 * 2 * kEpiBufBytes;  // 32 KB
constexpr uint32_t kEpiOff = kStages * kStageBytes;  // 192 KB
constexpr uint32_t kBarOff = kEpiOff + kEpiBytes;
constexpr uint32_t kSmem = kBarOff + 256;
static_assert(kSmem + 1024 <= 232448, "GEMM shared memory");

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

// ---- TMA store of a staged 32 x 32 chunk (issued by one lane after the warp's writes are fenced)
TS_DEVICE void tma_store_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(map), "r"(src),
               "r"(x), "r"(y)
               : "memory");
}
TS_DEVICE void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(
                   map),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
TS_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// at most one committed store group still reading shared memory
TS_DEVICE void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;\n" ::: "memory"); }
TS_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

TS_DEVICE void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;\n" ::: "memory"); }

// Per-warp epilogue state: `nbuf` (1 or 2) staging buffers of `stride` bytes used in turn.
struct EpiStage {
  uint32_t buf0;  // shared::cta address of buffer 0
  int n;          // chunks issued so far
  uint32_t stride = kEpiBufBytes;
  int nbuf = 2;
};

// Stage this lane's 32 values (row `lane` of the chunk) and TMA-store the 32 x 32 chunk at (col, row0).
// bf16 rows are 64 B (SWIZZLE_64B: 16-byte chunk j of row r sits at j ^ ((r >> 1) & 3)); fp32 rows are
// 128 B (SWIZZLE_128B: j ^ (r & 7)). Both placements are bank-conflict free for the row-per-lane writes.
template <int EPI>
TS_DEVICE void emit_chunk(EpiStage& st, const CUtensorMap* tm_c, const float* o, int col, int row0) {
  const int lane = threadIdx.x & 31;
  const uint32_t buf = st.buf0 + (uint32_t)(st.nbuf == 2 ? (st.n & 1) : 0) * st.stride;
  if (st.n >= st.nbuf) {
    // the store that last used this buffer has read it
    if (lane == 0) {
      if (st.nbuf == 2) bulk_wait_read1();
      else bulk_wait_read0();
    }
    __syncwarp();
  }
  if constexpr (EPI == kStoreF32 || EPI == kAccumF32) {
    const uint32_t rowb = buf + (uint32_t)lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t a = rowb + (uint32_t)((j ^ (lane & 7)) << 4);
      asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"r"(a), "f"(o[4 * j]), "f"(o[4 * j + 1]),
                   "f"(o[4 * j + 2]), "f"(o[4 * j + 3])
                   : "memory");
    }
  } else {
    const uint32_t rowb = buf + (uint32_t)lane * 64;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t a = rowb + (uint32_t)((j ^ ((lane >> 1) & 3)) << 4);
      asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};\n" ::"r"(a), "r"(pack_bf16(o[8 * j], o[8 * j + 1])),
                   "r"(pack_bf16(o[8 * j + 2], o[8 * j + 3])), "r"(pack_bf16(o[8 * j + 4], o[8 * j + 5])),
                   "r"(pack_bf16(o[8 * j + 6], o[8 * j + 7]))
                   : "memory");
    }
  }
  tc::fence_async_smem();
  __syncwarp();
  if (lane == 0) {
    if constexpr (EPI == kAccumF32) tma_reduce_add_2d(tm_c, buf, col, row0);
    else tma_store_2d(tm_c, buf, col, row0);
    bulk_commit();
  }
  ++st.n;
}

// Direct epilogue (no shared-memory staging, which leaves room for a deeper TMA ring): this lane's 32
// values go straight to row `row` of the output with 16-byte vector stores; the fp32 accumulate mode adds
// them with vector reductions at L2 (red.global.add.v4.f32: one add per element per GEMM, so the sum is
// deterministic), never reading the sink into the SM.
template <int EPI>
TS_DEVICE void emit_direct(void* c, int ldc, const float* o, int row, int col, int M, int N) {
  if (row >= M) return;
  const bool full = col + 32 <= N;
  if constexpr (EPI == kStoreF32 || EPI == kAccumF32) {
    float* p = reinterpret_cast<float*>(c) + (long long)row * ldc + col;
    if (full) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if constexpr (EPI == kAccumF32) {
          asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"l"(p + 4 * j), "f"(o[4 * j]),
                       "f"(o[4 * j + 1]), "f"(o[4 * j + 2]), "f"(o[4 * j + 3])
                       : "memory");
        } else {
          *reinterpret_cast<float4*>(p + 4 * j) = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
        }
      }
    } else {
      for (int x = 0; x < 32 && col + x < N; ++x) {
        if constexpr (EPI == kAccumF32) atomicAdd(p + x, o[x]);
        else p[x] = o[x];
      }
    }
  } else {
    bf16* p = reinterpret_cast<bf16*>(c) + (long long)row * ldc + col;
    if (full) {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        uint4 u;
        u.x = pack_bf16(o[8 * j], o[8 * j + 1]);
        u.y = pack_bf16(o[8 * j + 2], o[8 * j + 3]);
        u.z = pack_bf16(o[8 * j + 4], o[8 * j + 5]);
        u.w = pack_bf16(o[8 * j + 6], o[8 * j + 7]);
        *reinterpret_cast<uint4*>(p + 8 * j) = u;
      }
    } else {
      for (int x = 0; x < 32 && col + x < N; ++x) p[x] = __float2bfloat16_rn(o[x]);
    }
  }
}

// Epilogue of one output tile for the calling thread's row: reads the row's kBN fp32 accumulator
// columns from tensor memory at `tacc` (32 at a time) and stores / accumulates / reduces them.
// `row0` is the first row of the warp's 32-row slab (the chunk's TMA row coordinate). DIRECT: vector
// stores / reductions from registers instead of TMA stores of staged chunks (`c` is the output).
template <int EPI, bool DIRECT = false>
TS_DEVICE void epilogue_tile(uint32_t tacc, int row, int row0, int nb, int M, int N, int ldc, float alpha,
                             const bf16* __restrict__ res, const CUtensorMap* tm_c, EpiStage& st, const LmArgs& lm,
                             void* c = nullptr, int c_begin = 0, int c_end = kBN) {
  if (row0 >= M || c_begin >= c_end) return;  // warp-uniform: nothing of the output in this slab / range
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
  // one 32-column chunk: `v` holds its accumulators, `r4` its residual segment (kStoreBf16 with res)
  auto process = [&](float* v, int col, const uint4* r4) {
    if constexpr (EPI == kLse) {
      if (row < M) {
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
      return;
    }
    if constexpr (EPI == kDlogits) {
      const float l2 = row_lse * kLog2eF;
#pragma unroll
      for (int x = 0; x < 32; ++x) {
        const float pr = ex2f(fmaf(v[x], kLog2eF, -l2));
        float g = row_g;
        if (lm.gent != nullptr) g += row_ge * ((v[x] - row_lse) + row_h);
        v[x] = -pr * g + (col + x == row_tgt ? row_g : 0.f);
      }
    } else {
#pragma unroll
      for (int x = 0; x < 32; ++x) v[x] *= alpha;
      if constexpr (EPI == kStoreBf16) {
        if (res != nullptr) {
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(&r4[j]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const float2 f = __bfloat1622float2(h2[q]);
              v[8 * j + 2 * q] += f.x;
              v[8 * j + 2 * q + 1] += f.y;
            }
          }
        }
      }
    }
    if constexpr (DIRECT) emit_direct<EPI>(c, ldc, v, row, col, M, N);
    else emit_chunk<EPI>(st, tm_c, v, col, row0);
  };
  auto load_res = [&](uint4* r4, int col) {
    if constexpr (EPI == kStoreBf16) {
      if (res != nullptr) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          r4[j] = make_uint4(0, 0, 0, 0);
          if (row < M && col + 8 * j < N)
            r4[j] = __ldg(reinterpret_cast<const uint4*>(res + (long long)row * ldc + col + 8 * j));
        }
      }
    }
  };
  // two chunks per round: both TMEM loads (and residual loads) are in flight together, one wait
#pragma unroll 1
  for (int cc = c_begin; cc < c_end; cc += 64) {
    const int col = col0 + cc;
    if (col >= N) break;  // warp-uniform: nothing of this pair of chunks is inside the output
    const bool second = col + 32 < N;
    uint4 ra[4], rb[4];
    load_res(ra, col);
    if (second) load_res(rb, col + 32);
    float va[32], vb[32];
    tc::tmem_ld32(tacc + cc, va);
    tc::tmem_ld32(tacc + cc + 32, vb);
    tc::tmem_ld_wait();
    process(va, col, ra);
    if (second) process(vb, col + 32, rb);
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
                                                         const __grid_constant__ CUtensorMap tm_c,
                                                         const bf16* __restrict__ res,
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
  // Programmatic dependent launch: the set-up above (barriers, TMEM, tensor-map prefetch) may overlap the
  // previous kernel's tail; no global operand is read or written before that kernel has completed. The
  // next GEMM may then be scheduled as this one's CTAs retire.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

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
    EpiStage est{sbase + kEpiOff + (uint32_t)sub * 2 * kEpiBufBytes, 0};
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
      epilogue_tile<EPI>(lane_base + buf * kBN, mb * kBM + row_in_tile, mb * kBM + sub * 32, nb, M, N, ldc, alpha,
                         res, &tm_c, est, lm);
      tc::tc_fence_before();
      tc::mbar_arrive(&bars->acc_empty[buf]);
    }
    if (lane == 0) bulk_wait_all();  // staged stores done before shared memory goes away
    __syncwarp();
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
// Pair-kernel shapes: NT 256-column sub-tiles per pair tile. NT = 1: 256 x 256 tiles, 6-stage ring of
// 32 KB, two TMEM accumulators (the epilogue of tile i overlaps the main loop of tile i + 1). NT = 2
// ("wide"): 256 x 512 tiles, 4-stage ring of 48 KB; each A tile feeds two MMAs, so every SM stages 25%
// fewer bytes per FLOP from L2, and the two 256-column accumulators fill TMEM: the epilogue releases
// sub-tile 0 as soon as it has read it, and the next tile's MMAs into sub-tile 1 wait only for that half.
// DIRECT: the epilogue stores from registers, so the 32 KB of staging buffers become a 7th stage
// (the ring then holds 3.5k tensor-core cycles of loads instead of 3k, which covers the TMA latency
// measured under full load).
template <int NT, bool DIRECT = false>
struct PairCfg {
  static constexpr int kStages = NT == 1 ? (DIRECT ? 7 : 6) : 4;
  static constexpr uint32_t kBHalf = 128 * kBK * 2;               // 16 KB: 128 n-rows x 64 k
  static constexpr uint32_t kStage = kABytes + NT * kBHalf;       // per CTA
  static constexpr uint32_t kEpiOff = kStages * kStage;
  static constexpr uint32_t kBarOff = kEpiOff + (DIRECT ? 0u : kEpiBytes);
  static constexpr uint32_t kSmem = kBarOff + 256;
  static_assert(kSmem + 1024 <= 232448, "pair GEMM shared memory");
};

struct PairBars {
  uint64_t full[7], empty[7], acc_full[2], acc_empty[2];
  uint32_t tmem_slot;
  int abort;
};

// Optional pipeline timing of the pair kernel (off unless gemm_tc_profile(1)): per cluster, SM-clock cycles
// the producer waited for free stages, the MMA issuer waited for loaded stages and for drained
// accumulators, and the MMA issuer's whole span. Read by gemm_tc_profile_read.
constexpr int kProfSlots = 11;
__device__ unsigned long long g_gemm_prof[128 * kProfSlots];

TS_DEVICE unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ int g_gemm_prof_on = 0;

// The pair kernel's epilogue runs on `epi_warps` warps, 4 or 8 (chosen per launch). With 8, two warps
// share each TMEM sub-partition and take half of a tile's columns each; staging per warp is two 2 KB
// buffers for bf16 chunks or one 4 KB buffer for fp32 chunks. With 4 (and in the LM-head modes, which
// keep a row's online reduction in one warp), one warp per sub-partition covers all columns with two 4 KB
// buffers. Either way the staging takes 32 KB.
constexpr int kPairEpiWarps = 8;  // most epilogue warps of a launch
constexpr int kPairThreads = 64 + 32 * kPairEpiWarps;

template <bool A_MN, bool B_MN, int EPI, int NT, bool DIRECT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPairThreads, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                     const __grid_constant__ CUtensorMap tm_a2, const __grid_constant__ CUtensorMap tm_b2, int K2,
                     const __grid_constant__ CUtensorMap tm_c, const bf16* __restrict__ res, int M, int N, int K,
                     int ldc, float alpha, int* __restrict__ err, LmArgs lm, void* __restrict__ c, int epi_warps) {
  using C = PairCfg<NT, DIRECT>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + C::kBarOff);
  const uint32_t sbase = tc::smem_addr(smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_rank();
  constexpr int kTileN = NT * kBN;
  const int mt = (M + 2 * kBM - 1) / (2 * kBM), nt = (N + kTileN - 1) / kTileN, kt1 = (K + kBK - 1) / kBK,
            kt = kt1 + (K2 + kBK - 1) / kBK;
  const int tiles = mt * nt;
  const int cid = blockIdx.x >> 1, ncl = gridDim.x >> 1;
  volatile int* abort = &bars->abort;
  const bool prof = g_gemm_prof_on != 0 && cid < 128;
  __shared__ unsigned long long t_entry_s;
  if (prof && threadIdx.x == 0) t_entry_s = gtime();  // kernel entry, before barrier/TMEM set-up

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      tc::mbar_init(&bars->full[s], 1);
      tc::mbar_init(&bars->empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&bars->acc_full[b], 1);
      tc::mbar_init(&bars->acc_empty[b], 2 * epi_warps);  // one arrival per epilogue warp of the pair
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
  // Programmatic dependent launch: the set-up above (barriers, TMEM, tensor-map prefetch) may overlap the
  // previous kernel's tail; no global operand is read or written before that kernel has completed. The
  // next GEMM may then be scheduled as this one's CTAs retire.
  asm volatile("griddepcontrol.wait;\n" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      long long t_prod_wait = 0;
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
        for (int kb = 0; kb < kt; ++kb, ++it) {
          const int s = it % S;
          const long long w0 = prof ? clock64() : 0;
          if (it >= S && !tc::mbar_wait(&bars->empty[s], ((it - S) / S) & 1, abort, err, 231))
            goto producer_done;
          if (prof) t_prod_wait += clock64() - w0;
          if (rank == 0) tc::mbar_expect_tx(&bars->full[s], 2 * C::kStage);
          const uint32_t full0 = tc::map_cluster(tc::smem_addr(&bars->full[s]), 0);
          uint8_t* a = smem + s * C::kStage;
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
#pragma unroll
          for (int j = 0; j < NT; ++j) {
            uint8_t* b = a + kABytes + j * C::kBHalf;
            const int bcol = nb * kTileN + j * kBN + (int)rank * (kBN / 2);
            if constexpr (!B_MN) {
              tc::tma_load_2d_pair(b, pb, kx, bcol, full0);  // box 64 (k) x 128 (n)
            } else {
              tc::tma_load_2d_pair(b, pb, bcol, kx, full0);  // [K][N]: 2 boxes of 64 n x 64 k
              tc::tma_load_2d_pair(b + 64 * 128, pb, bcol + 64, kx, full0);
            }
          }
        }
      }
    producer_done:;
      if (prof && rank == 0) atomicAdd(&g_gemm_prof[cid * kProfSlots + 0], (unsigned long long)t_prod_wait);
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      long long t_full = 0, t_acc = 0;
      const long long t_begin = clock64();
      unsigned long long t_first = 0;
      const uint32_t idesc = tc::idesc_bf16(2 * kBM, kBN, A_MN, B_MN);
      int it = 0, local = 0;
      bool ok = true;
      for (int t = cid; ok && t < tiles; t += ncl, ++local) {
        // NT = 1: alternate between two accumulators; NT = 2: one accumulator of two halves
        const int buf = NT == 1 ? (local & 1) : 0;
        if constexpr (NT == 1) {
          const long long w0 = clock64();
          if (local >= 2 && !tc::mbar_wait(&bars->acc_empty[buf], ((local - 2) >> 1) & 1, abort, err, 241)) break;
          t_acc += clock64() - w0;
          tc::tc_fence_after();
        }
        const uint32_t acc = tmem + buf * kBN;
        for (int kb = 0; kb < kt; ++kb, ++it) {
          const int s = it % S;
          const long long w1 = clock64();
          if (!tc::mbar_wait(&bars->full[s], (it / S) & 1, abort, err, 242)) {
            ok = false;
            break;
          }
          t_full += clock64() - w1;
          tc::tc_fence_after();
          const uint32_t a = sbase + s * C::kStage;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk) {
            const uint64_t ad = A_MN ? tc::sdesc_sw128(a + kk * 16 * 128, 64 * 128, 1024)
                                     : tc::sdesc_sw128(a + kk * 32, 16, 1024);
#pragma unroll
            for (int j = 0; j < NT; ++j) {
              if constexpr (NT == 2) {
                // before the first write of this tile into half j, the epilogue must have read it
                if (kb == 0 && kk == 0 && local >= 1) {
                  if (!tc::mbar_wait(&bars->acc_empty[j], (local - 1) & 1, abort, err, 243)) {
                    ok = false;
                    break;
                  }
                  tc::tc_fence_after();
                }
              }
              const uint32_t b = a + kABytes + j * C::kBHalf;
              const uint64_t bd = B_MN ? tc::sdesc_sw128(b + kk * 16 * 128, 64 * 128, 1024)
                                       : tc::sdesc_sw128(b + kk * 32, 16, 1024);
              if (prof && t_first == 0) t_first = gtime();
              tc::mma_bf16_pair(acc + j * kBN, ad, bd, idesc, kb > 0 || kk > 0);
            }
            if (!ok) break;
          }
          if (!ok) break;
          tc::mma_commit_pair(&bars->empty[s]);
        }
        if (ok) tc::mma_commit_pair(&bars->acc_full[buf]);
      }
      if (prof) {
        unsigned long long* slot = &g_gemm_prof[cid * kProfSlots];
        atomicAdd(slot + 1, (unsigned long long)t_full);
        atomicAdd(slot + 2, (unsigned long long)t_acc);
        atomicAdd(slot + 3, (unsigned long long)(clock64() - t_begin));
        atomicAdd(slot + 4, (unsigned long long)it);  // k-blocks issued
        atomicAdd(slot + 5, 1ull);                    // launches
        atomicAdd(slot + 7, t_first - t_entry_s);     // entry -> first MMA (ns)
        atomicAdd(slot + 8, gtime() - t_entry_s);     // entry -> last commit issued (ns)
      }
    }
  } else {
    const int sub = warp & 3;
    const int ew = warp - 2;         // epilogue warp 0 .. epi_warps-1
    const int colhalf = ew >> 2;     // with 8 warps: 0 for columns [0, 128) of a tile, 1 for [128, 256)
    const bool split = epi_warps == 8 && !(EPI == kLse || EPI == kDlogits);
    const int c_begin = split ? colhalf * (kBN / 2) : (colhalf ? kBN : 0);
    const int c_end = split ? c_begin + kBN / 2 : kBN;
    const uint32_t lane_base = tmem + ((uint32_t)(sub * 32) << 16);
    const uint32_t acc_empty0 = tc::map_cluster(tc::smem_addr(&bars->acc_empty[0]), 0);
    const uint32_t acc_empty1 = tc::map_cluster(tc::smem_addr(&bars->acc_empty[1]), 0);
    constexpr bool kF32Out = EPI == kStoreF32 || EPI == kAccumF32;
    EpiStage est = split ? EpiStage{sbase + C::kEpiOff + (uint32_t)ew * (kEpiBytes / 8), 0,
                                    kF32Out ? kEpiBufBytes : kEpiBufBytes / 2, kF32Out ? 1 : 2}
                         : EpiStage{sbase + C::kEpiOff + (uint32_t)(ew & 3) * (kEpiBytes / 4), 0, kEpiBufBytes, 2};
    int local = 0;
    for (int t = cid; t < tiles; t += ncl, ++local) {
      const int buf = NT == 1 ? (local & 1) : 0;
      const uint32_t parity = NT == 1 ? ((local >> 1) & 1) : (local & 1);
      bool ok = true;
      if (lane == 0) ok = tc::mbar_wait(&bars->acc_full[buf], parity, abort, err, 251);
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      if (!ok) break;
      tc::tc_fence_after();
      int mb, nb;
      tile_coords(t, mt, nt, mb, nb);
      const int row0 = mb * 2 * kBM + (int)rank * kBM + sub * 32;
#pragma unroll 1
      for (int j = 0; j < NT; ++j) {
        const int half = NT == 1 ? buf : j;
        epilogue_tile<EPI, DIRECT>(lane_base + half * kBN, row0 + lane, row0, nb * NT + j, M, N, ldc, alpha, res,
                                   &tm_c, est, lm, c, c_begin, c_end);
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cluster(half ? acc_empty1 : acc_empty0);
      }
    }
    if (!DIRECT && lane == 0) bulk_wait_all();  // staged stores done before shared memory goes away
    __syncwarp();
    if (prof && rank == 0 && lane == 0 && ew == 0) atomicAdd(&g_gemm_prof[cid * kProfSlots + 9], gtime() - t_entry_s);
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::cluster_sync();  // no CTA leaves while its pair may still read its shared memory or arrive on it
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc_pair(tmem, 512);
  }
  if (prof && rank == 0 && threadIdx.x == 0) atomicAdd(&g_gemm_prof[cid * kProfSlots + 10], gtime() - t_entry_s);
}

// 0: single-CTA 128 x 256 tiles; 1: CTA-pair 256 x 256 tiles; 2 (default): by output mode -- single-CTA
// tiles for bf16 / fp32 stores (projections, dx), CTA pairs for fp32 accumulation into a gradient sink
// (dW) and the LM-head epilogues. Interleaved measurements at the decoder's shapes
// (benchmarks/bench_kernels.py gemm_ab): the single-CTA kernel is 9-16% faster on the forward projections
// at 2304 rows and 19-80% faster at 1152 rows (twice the tiles: far better wave fill for short packs),
// the pair kernel 3-7% faster on the fp32-accumulate dW products.
int g_gemm_pair = 2;

inline bool use_pair(int epi) { return g_gemm_pair == 1 || (g_gemm_pair == 2 && epi != kStoreBf16 && epi != kStoreF32); }

// 0: never the wide (256 x 512) pair tile (default: measured slower than 256 x 256 at every decoder
// shape); 1: when it fills the SMs' waves at least as well; 2: always (measurement)
int g_gemm_wide = 0;

// 1: the pair kernel's epilogue stores from registers and the ring has 7 stages; 0 (default): TMA-store
// epilogue through shared memory with 6 stages (measured faster: the deeper ring did not shorten the MMA
// issuer's waits for loads).
int g_gemm_direct = 0;

template <bool A_MN, bool B_MN, int EPI, int NT, bool DIRECT>
int resident_pairs(int device, int smem) {
  static int resident[16] = {0};  // co-resident CTA pairs per device (persistent grid size)
  int& pairs = resident[device & 15];
  if (pairs == 0) {
    TS_CUDA_CHECK(cudaFuncSetAttribute(gemm_pair_kernel<A_MN, B_MN, EPI, NT, DIRECT>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * sm_count(device));
    cfg.blockDim = dim3(kPairThreads);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<A_MN, B_MN, EPI, NT, DIRECT>, &cfg) != cudaSuccess ||
        n <= 0) {
      (void)cudaGetLastError();
      n = sm_count(device) / 2;
    }
    pairs = std::min(n, sm_count(device) / 2);
  }
  return pairs;
}

// Epilogue warps of the pair kernel: 0 = four everywhere; 1 (default) = eight for bf16 outputs (fp32 and
// LM-head modes keep four with double-buffered 4 KB staging); 2 = eight for every store / accumulate mode.
int g_gemm_epi8 = 1;

// 1 (default): launch the GEMM kernels with programmatic stream serialization, so a GEMM's launch and set-up
// overlap the previous kernel's completion when that kernel allows it (ours do); 0: plain stream order.
int g_gemm_pdl = 1;

template <typename... KArgs, typename... Args>
void launch_pdl(void (*kernel)(KArgs...), int grid, int block, int smem, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_gemm_pdl ? 1 : 0;
  TS_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...));
}

// Fraction of the pairs' tile slots a grid of `tiles` uses over its waves.
inline double wave_fill(int tiles, int pairs) {
  const int waves = (tiles + pairs - 1) / pairs;
  return double(tiles) / double(std::max(1, waves * pairs));
}

template <bool A_MN, bool B_MN, int EPI, int NT, bool DIRECT>
void launch_pair_cfg(int tiles, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const bf16* res,
                     int M, int N, int K, int ldc, float alpha, int device, LmArgs lm, const CUtensorMap* ma2,
                     const CUtensorMap* mb2, int K2, void* c) {
  const int smem = PairCfg<NT, DIRECT>::kSmem + 1024;
  const int pairs = resident_pairs<A_MN, B_MN, EPI, NT, DIRECT>(device, smem);
  const int clusters = std::max(1, std::min(tiles, pairs));
  const CUtensorMap& a2 = ma2 ? *ma2 : ma;
  const CUtensorMap& b2 = mb2 ? *mb2 : mb;
  int epi = 4;
  if (!DIRECT && ((g_gemm_epi8 >= 1 && EPI == kStoreBf16) ||
                  (g_gemm_epi8 == 2 && (EPI == kStoreF32 || EPI == kAccumF32))))
    epi = 8;
  launch_pdl(gemm_pair_kernel<A_MN, B_MN, EPI, NT, DIRECT>, 2 * clusters, 64 + 32 * epi, smem, ma, mb, a2, b2,
             ma2 ? K2 : 0, mc, res, M, N, K, ldc, alpha, tc_error_flag(at::Device(at::kCUDA, device)).data_ptr<int>(),
             lm, c, epi);
}

template <bool A_MN, bool B_MN, int EPI>
void launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const bf16* res, int M, int N,
                 int K, int ldc, float alpha, int device, LmArgs lm, const CUtensorMap* ma2 = nullptr,
                 const CUtensorMap* mb2 = nullptr, int K2 = 0, void* c = nullptr) {
  const int mt = (M + 2 * kBM - 1) / (2 * kBM);
  const int tiles1 = mt * ((N + kBN - 1) / kBN), tiles2 = mt * ((N + 2 * kBN - 1) / (2 * kBN));
  bool wide = false;
  if (g_gemm_wide == 2) {
    wide = true;
  } else if (g_gemm_wide == 1 && N > kBN) {
    const int p1 = resident_pairs<A_MN, B_MN, EPI, 1, true>(device, PairCfg<1, true>::kSmem + 1024);
    const int p2 = resident_pairs<A_MN, B_MN, EPI, 2, false>(device, PairCfg<2, false>::kSmem + 1024);
    wide = wave_fill(tiles2, p2) * 1.15 >= wave_fill(tiles1, p1);
  }
  if (wide) {
    launch_pair_cfg<A_MN, B_MN, EPI, 2, false>(tiles2, ma, mb, mc, res, M, N, K, ldc, alpha, device, lm, ma2, mb2, K2,
                                               c);
  } else if (g_gemm_direct) {
    launch_pair_cfg<A_MN, B_MN, EPI, 1, true>(tiles1, ma, mb, mc, res, M, N, K, ldc, alpha, device, lm, ma2, mb2, K2,
                                              c);
  } else {
    launch_pair_cfg<A_MN, B_MN, EPI, 1, false>(tiles1, ma, mb, mc, res, M, N, K, ldc, alpha, device, lm, ma2, mb2,
                                               K2, c);
  }
}

template <bool A_MN, bool B_MN, int EPI>
void launch(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, const bf16* res, int M, int N, int K,
            int ldc, float alpha, int device, LmArgs lm = LmArgs{}, const CUtensorMap* ma2 = nullptr,
            const CUtensorMap* mb2 = nullptr, int K2 = 0) {
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  const int grid = std::max(1, std::min(tiles, sm_count(device)));
  const int smem = kSmem + 1024;
  ensure_smem((const void*)gemm_tc_kernel<A_MN, B_MN, EPI>, smem);
  const CUtensorMap& a2 = ma2 ? *ma2 : ma;
  const CUtensorMap& b2 = mb2 ? *mb2 : mb;
  launch_pdl(gemm_tc_kernel<A_MN, B_MN, EPI>, grid, 192, smem, ma, mb, a2, b2, ma2 ? K2 : 0, mc, res, M, N, K, ldc,
             alpha, tc_error_flag(at::Device(at::kCUDA, device)).data_ptr<int>(), lm);
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

// Pipeline timing of the pair kernel: on = 1 clears the counters and switches timing on, 0 switches it off.
void gemm_tc_profile(int64_t on) {
  const int v = on ? 1 : 0;
  TS_CUDA_CHECK(cudaMemcpyToSymbol(g_gemm_prof_on, &v, sizeof(v)));
  if (on) {
    static const unsigned long long zero[128 * kProfSlots] = {0};
    TS_CUDA_CHECK(cudaMemcpyToSymbol(g_gemm_prof, zero, sizeof(zero)));
  }
}

// [clusters][producer wait for free stages, MMA wait for loaded stages, MMA wait for drained accumulators,
// MMA issuer span, k-blocks, launches] summed over the launches since gemm_tc_profile(1).
at::Tensor gemm_tc_profile_read() {
  auto out = at::empty({128, kProfSlots}, at::TensorOptions().dtype(at::kLong));
  TS_CUDA_CHECK(cudaMemcpyFromSymbol(out.data_ptr(), g_gemm_prof, sizeof(unsigned long long) * 128 * kProfSlots));
  return out;
}

// Programmatic dependent launch of the GEMM kernels: 1 on (default), 0 off. Returns the previous value.
int64_t gemm_tc_pdl(int64_t on) {
  const int prev = g_gemm_pdl;
  if (on >= 0) g_gemm_pdl = on ? 1 : 0;
  return prev;
}

// Pair-kernel epilogue: 1 = register stores with a 7-stage ring, 0 = TMA-store epilogue with 6 stages (default).
int64_t gemm_tc_direct(int64_t on) {
  const int prev = g_gemm_direct;
  if (on >= 0) g_gemm_direct = on ? 1 : 0;
  return prev;
}

// Wide pair tiles (256 x 512): 0 never (default), 1 when the waves fill as well, 2 always. Returns the previous value.
int64_t gemm_tc_wide(int64_t mode) {
  const int prev = g_gemm_wide;
  if (mode >= 0) g_gemm_wide = (int)std::min<int64_t>(mode, 2);
  return prev;
}

// Epilogue warps of the pair kernel (see g_gemm_epi8): 0, 1 or 2; returns the previous value (-1 reads it).
int64_t gemm_tc_epi8(int64_t mode) {
  const int prev = g_gemm_epi8;
  if (mode >= 0) g_gemm_epi8 = (int)std::min<int64_t>(mode, 2);
  return prev;
}

// Select the GEMM kernel: 1 = CTA-pair 256 x 256 tiles, 0 = single-CTA 128 x 256 tiles, 2 = by output mode
// (g_gemm_pair). Returns the previous value (-1 reads it).
int64_t gemm_tc_pair(int64_t on) {
  const int prev = g_gemm_pair;
  if (on >= 0) g_gemm_pair = (int)std::min<int64_t>(on, 2);
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
  const bool pair = use_pair(kLse);
  const CUtensorMap ma = make_bf16_map(h.data_ptr(), D, R, D, 128);
  const CUtensorMap mb = make_bf16_map(w.data_ptr(), D, V, D, pair ? 128 : 256);
  // the LSE epilogue stores nothing; its output map is a placeholder
  if (pair) launch_pair<false, false, kLse>(ma, mb, ma, nullptr, R, V, D, V, 1.f, h.get_device(), lm);  // no output
  else launch<false, false, kLse>(ma, mb, ma, nullptr, R, V, D, V, 1.f, h.get_device(), lm);
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
  const bool pair = use_pair(kDlogits);
  const CUtensorMap ma = make_bf16_map(h.data_ptr(), D, R, D, 128);
  const CUtensorMap mb = make_bf16_map(w.data_ptr(), D, V, D, pair ? 128 : 256);
  const CUtensorMap md = make_out_map(d.data_ptr(), false, V, R, V);
  if (pair)
    launch_pair<false, false, kDlogits>(ma, mb, md, nullptr, R, V, D, V, 1.f, h.get_device(), lm, nullptr, nullptr, 0,
                                        d.data_ptr());
  else launch<false, false, kDlogits>(ma, mb, md, nullptr, R, V, D, V, 1.f, h.get_device(), lm);
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
                 const c10::optional<at::Tensor>& b2, bool a_t, bool b_t, int64_t mode, double alpha,
                 const c10::optional<at::Tensor>& residual) {
  check_cuda(a, "a");
  check_cuda(b, "b");
  // the output may be a row-strided view (rows contiguous, checked below): the TMA store writes only it
  TS_CHECK(out.is_cuda() && out.device() == a.device(), "gemm_tc: out must be a CUDA tensor on a's device");
  TS_CHECK(a.scalar_type() == at::kBFloat16 && b.scalar_type() == at::kBFloat16, "gemm_tc takes bf16 operands");
  TS_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm_tc takes matrices");
  TS_CHECK(a.is_contiguous() && b.is_contiguous(), "gemm_tc takes contiguous operands");
  const int M = a_t ? a.size(1) : a.size(0);
  const int K = a_t ? a.size(0) : a.size(1);
  const int N = b_t ? b.size(0) : b.size(1);
  TS_CHECK((b_t ? b.size(1) : b.size(0)) == K, "gemm_tc inner dimensions differ");
  TS_CHECK(out.size(0) == M && out.size(1) == N, "gemm_tc output shape");
  TS_CHECK(mode == 0 ? out.scalar_type() == at::kBFloat16 : out.scalar_type() == at::kFloat, "gemm_tc output dtype");
  // 16-byte TMA strides for every operand layout and the output rows
  TS_CHECK(K % 8 == 0 && N % 8 == 0 && (!a_t || M % 8 == 0), "gemm_tc needs K, N (and M when a is [K, M]) "
           "to be multiples of 8");
  const int64_t ldc = out.size(0) > 1 ? out.stride(0) : N;
  TS_CHECK(out.size(1) <= 1 || out.stride(1) == 1, "gemm_tc: output rows must be contiguous");
  TS_CHECK((ldc * out.element_size()) % 16 == 0 && reinterpret_cast<uintptr_t>(out.data_ptr()) % 16 == 0,
           "gemm_tc: output base and row stride must be 16-byte aligned");
  const bf16* res = nullptr;
  if (residual.has_value()) {
    TS_CHECK(mode == 0, "gemm_tc: a residual operand needs the bf16 output mode");
    TS_CHECK(residual->scalar_type() == at::kBFloat16 && residual->dim() == 2 && residual->size(0) == M &&
                 residual->size(1) == N && residual->stride(1) == 1 && (M <= 1 || residual->stride(0) == ldc) &&
                 reinterpret_cast<uintptr_t>(residual->data_ptr()) % 16 == 0,
             "gemm_tc: the residual must be bf16 [M, N], 16-byte aligned, with the output's row stride");
    res = reinterpret_cast<const bf16*>(residual->data_ptr());
  }
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
    if (mode == 2) return;
    if (res != nullptr) out.copy_(*residual);
    else out.zero_();
    return;
  }
  // tensor maps: inner dimension first; boxes of 64 inner elements
  const bool pair = use_pair(mode == 0 ? kStoreBf16 : mode == 1 ? kStoreF32 : kAccumF32);
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
  const CUtensorMap mc = make_out_map(out.data_ptr(), mode != 0, N, M, ldc);
  const CUtensorMap* pa2 = two ? &ma2 : nullptr;
  const CUtensorMap* pb2 = two ? &mb2 : nullptr;
  const int dev = a.get_device();
  const float al = (float)alpha;
  const int ld = (int)ldc;
  void* cp = out.data_ptr();
  const LmArgs none{};
#define TS_GEMM_CASE(AM, BM)                                                                                     \
  if (pair) {                                                                                                    \
    if (mode == 0) launch_pair<AM, BM, kStoreBf16>(ma, mb, mc, res, M, N, K, ld, al, dev, none, pa2, pb2, K2, cp); \
    else if (mode == 1) launch_pair<AM, BM, kStoreF32>(ma, mb, mc, res, M, N, K, ld, al, dev, none, pa2, pb2, K2, cp); \
    else launch_pair<AM, BM, kAccumF32>(ma, mb, mc, res, M, N, K, ld, al, dev, none, pa2, pb2, K2, cp);            \
  } else {                                                                                                       \
    if (mode == 0) launch<AM, BM, kStoreBf16>(ma, mb, mc, res, M, N, K, ld, al, dev, none, pa2, pb2, K2);        \
    else if (mode == 1) launch<AM, BM, kStoreF32>(ma, mb, mc, res, M, N, K, ld, al, dev, none, pa2, pb2, K2);    \
    else launch<AM, BM, kAccumF32>(ma, mb, mc, res, M, N, K, ld, al, dev, none, pa2, pb2, K2);                   \
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
             double alpha, const c10::optional<at::Tensor>& residual) {
  gemm_tc_cat(out, a, b, c10::nullopt, c10::nullopt, a_t, b_t, mode, alpha, residual);
}

}  // namespace ts
