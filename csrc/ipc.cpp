// Peer-mapped device buffers for the native collectives (N0).
//
// Each rank allocates a dedicated device buffer with cudaMalloc (outside
// torch's caching allocator, so the exported allocation is exactly the
// buffer), exports a CUDA IPC handle, and opens every peer's handle to obtain
// a device pointer it can load from and store to over NVLink. Plain peer
// mappings only: no NVLink multicast object is created or bound.
#include <cuda_runtime.h>
#include <pybind11/pybind11.h>

#include <cstring>

#include "common.h"

namespace py = pybind11;

namespace ts {

py::tuple ipc_alloc(int64_t nbytes, int64_t device) {
  TS_CHECK(nbytes > 0, "ipc_alloc needs a positive size");
  TS_CUDA_CHECK(cudaSetDevice((int)device));
  void* p = nullptr;
  TS_CUDA_CHECK(cudaMalloc(&p, (size_t)nbytes));
  TS_CUDA_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  TS_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  auto t = torch::from_blob(
      p, {nbytes}, [](void* q) { cudaFree(q); },
      torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, (int)device));
  return py::make_tuple(t, py::bytes(reinterpret_cast<const char*>(&h), sizeof(h)));
}

int64_t ipc_open(const py::bytes& handle, int64_t device) {
  std::string s = handle;
  TS_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  TS_CUDA_CHECK(cudaSetDevice((int)device));
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  void* p = nullptr;
  TS_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) {
  if (ptr) TS_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)));
}

void register_ipc(py::module& m) {
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
}

}  // namespace ts
