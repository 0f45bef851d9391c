// Page-locked host slabs for offloaded GRPO sources and statistics (C31).
//
// A slab is one 2 MiB-aligned anonymous host allocation, advised for
// transparent huge pages, and registered with cudaHostRegister in pieces of
// at most `piece_bytes` (the kernel pins each piece with its own page array,
// so a small piece keeps every pin's array at a low allocation order even
// on a fragmented host). Registration is all or nothing: a failing piece
// unregisters the pieces before it and frees the slab. The returned uint8
// tensor owns the slab; its deleter unregisters every piece (on the device
// current at registration) and frees the memory. device < 0 skips
// registration (pageable slab), which is what hosts without a GPU use.
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <sys/mman.h>

#include <cstdlib>
#include <vector>

#include "common.h"

namespace py = pybind11;

namespace ts {
namespace {

constexpr size_t kSlabAlign = size_t(2) << 20;

struct Slab {
  void* base = nullptr;
  size_t bytes = 0;
  int device = -1;
  std::vector<char*> pieces;
};

void release(Slab* s) {
  if (s->device >= 0) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    for (char* p : s->pieces) cudaHostUnregister(p);
    cudaSetDevice(prev);
  }
  std::free(s->base);
  delete s;
}

}  // namespace

py::tuple pinned_slab_alloc(int64_t capacity, int64_t piece_bytes, int64_t device) {
  TS_CHECK(capacity > 0, "a pinned slab needs a positive capacity");
  TS_CHECK(piece_bytes > 0, "piece_bytes must be positive");
  const size_t bytes = ((size_t)capacity + kSlabAlign - 1) / kSlabAlign * kSlabAlign;
  void* base = nullptr;
  TS_CHECK(posix_memalign(&base, kSlabAlign, bytes) == 0, "host allocation of ", bytes, " bytes failed");
#ifdef MADV_HUGEPAGE
  madvise(base, bytes, MADV_HUGEPAGE);
#endif
  auto* s = new Slab{base, bytes, (int)device, {}};
  if (device >= 0) {
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice((int)device);
    for (size_t off = 0; e == cudaSuccess && off < (size_t)capacity; off += (size_t)piece_bytes) {
      const size_t n = std::min((size_t)piece_bytes, (size_t)capacity - off);
      char* p = static_cast<char*>(base) + off;
      e = cudaHostRegister(p, n, cudaHostRegisterDefault);
      if (e == cudaSuccess) s->pieces.push_back(p);
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
      cudaGetLastError();
      release(s);
      TS_CHECK(false, "cudaHostRegister of a pinned slab piece failed: ", cudaGetErrorString(e));
    }
  }
  const int64_t pieces = (int64_t)s->pieces.size();
  auto t = torch::from_blob(
      base, {capacity}, [s](void*) { release(s); }, torch::TensorOptions().dtype(torch::kUInt8));
  return py::make_tuple(t, pieces);
}

void register_pinned(py::module& m) { m.def("pinned_slab_alloc", &pinned_slab_alloc); }

}  // namespace ts
