// Fixed device scratch for the allocation-free matmul entry point (mk_matmul_noalloc): a file-scope __device__
// array in this library's own module, so a call makes no cudaMalloc / cudaFree. Its address is looked up once per
// device with that device current and kept for the life of the process (it does not survive cudaDeviceReset).
#include <cuda_runtime.h>

#include <mutex>

#include "kernels.hpp"

namespace mkb {

namespace {

constexpr size_t kNoAllocBytes = size_t{16} << 20;  // 16 MiB per device
__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

}  // namespace

size_t noalloc_scratch_bytes() { return kNoAllocBytes; }

uint8_t* noalloc_scratch(cudaError_t* err) {
  static std::mutex mu;
  static void* addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *err = e;
    return nullptr;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    *err = cudaErrorInvalidDevice;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      *err = e;
      return nullptr;
    }
    addr[dev] = p;
  }
  *err = cudaSuccess;
  return static_cast<uint8_t*>(addr[dev]);
}

}  // namespace mkb
