// Device-side index checks that never trap.
//
// TS_BOUND(cond, site, index): when `cond` is false the calling thread records
// (site, index) in this translation unit's status word -- the first failure
// wins -- and returns, so the out-of-range access never happens. These guard
// indices that come from user data (token ids, target ids) and are always
// compiled in: one compare per row.
//
// TS_BOUND_DEBUG(cond, site, index): the same check on index arithmetic that
// is correct by construction; it is compiled only into the bounds-checked
// debug build (`TS_BOUNDS_CHECK=1 python setup.py build_ext --inplace`).
//
// The host reads (and clears) the words through `bounds_status()`; a nonzero
// word is (site << 48) | (index & 0xFFFFFFFFFFFF).
#pragma once

#include <stdint.h>

namespace ts {
namespace {
__device__ unsigned long long g_bounds_word = 0ull;
}  // namespace
}  // namespace ts

// Record a failed check without leaving the thread (the caller writes a defined fallback instead).
#define TS_BOUND_RECORD(site, index)                                                                        \
  atomicCAS(&::ts::g_bounds_word, 0ull,                                                                     \
            ((unsigned long long)(site) << 48) | ((unsigned long long)(index) & 0xFFFFFFFFFFFFull))

#define TS_BOUND(cond, site, index)                                                                         \
  do {                                                                                                      \
    if (!(cond)) {                                                                                          \
      TS_BOUND_RECORD(site, index);                                                                         \
      return;                                                                                               \
    }                                                                                                       \
  } while (0)

#ifdef TS_BOUNDS_CHECK
#define TS_BOUND_DEBUG(cond, site, index) TS_BOUND(cond, site, index)
#else
#define TS_BOUND_DEBUG(cond, site, index) ((void)0)
#endif

// One host accessor per translation unit: returns this unit's word and clears it when `reset`.
#define TS_BOUNDS_ACCESSOR(fn)                                                                              \
  namespace ts {                                                                                            \
  uint64_t fn(bool reset) {                                                                                 \
    unsigned long long w = 0;                                                                               \
    TS_CUDA_CHECK(cudaMemcpyFromSymbol(&w, g_bounds_word, sizeof(w)));                                      \
    if (reset && w != 0) {                                                                                  \
      const unsigned long long z = 0;                                                                       \
      TS_CUDA_CHECK(cudaMemcpyToSymbol(g_bounds_word, &z, sizeof(z)));                                      \
    }                                                                                                       \
    return (uint64_t)w;                                                                                     \
  }                                                                                                         \
  }
