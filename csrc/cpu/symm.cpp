// Symmetric-memory heap: one cudaMalloc'd region per rank, shared with the other ranks of
// the node through CUDA IPC handles, so kernels can load/store peers' buffers directly over
// NVLink (the intra-node data plane of the fused collective kernels).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstring>

namespace syn {

#define SYMM_CHECK(expr)                                                                      \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    TORCH_CHECK(_e == cudaSuccess, #expr " failed: ", cudaGetErrorString(_e));                \
  } while (0)

// Allocates `nbytes` (zeroed) on the current device.  Returns (uint8 tensor that owns the
// allocation, 64-byte IPC handle as a uint8 CPU tensor).
std::vector<torch::Tensor> symm_alloc(int64_t nbytes) {
  TORCH_CHECK(nbytes > 0, "symm_alloc: nbytes must be positive");
  int dev;
  SYMM_CHECK(cudaGetDevice(&dev));
  void* p = nullptr;
  SYMM_CHECK(cudaMalloc(&p, (size_t)nbytes));
  SYMM_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  cudaIpcMemHandle_t h;
  SYMM_CHECK(cudaIpcGetMemHandle(&h, p));
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, dev);
  auto t = torch::from_blob(p, {nbytes}, [](void* q) { cudaFree(q); }, opts);
  auto hb = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  memcpy(hb.data_ptr(), &h, sizeof(h));
  return {t, hb};
}

// Maps a peer's allocation; returns its device address in this process.
int64_t symm_open(torch::Tensor handle) {
  TORCH_CHECK(handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle.data_ptr(), sizeof(h));
  void* p = nullptr;
  SYMM_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return (int64_t)(uintptr_t)p;
}

void symm_close(int64_t ptr) { SYMM_CHECK(cudaIpcCloseMemHandle((void*)(uintptr_t)ptr)); }

// Whether device a can access device b's memory directly.
bool p2p_access(int64_t a, int64_t b) {
  int ok = 0;
  SYMM_CHECK(cudaDeviceCanAccessPeer(&ok, (int)a, (int)b));
  return ok != 0;
}

}  // namespace syn
