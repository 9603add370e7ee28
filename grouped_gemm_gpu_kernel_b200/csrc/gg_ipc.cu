// gg_ipc.cu -- device memory shared between the processes of one node (CUDA IPC), for the
// multi-GPU gather of D fused into the grouped kernel: the root rank exports its D buffer, the
// other ranks map it and build executors whose D pointers lie in it, so their epilogues store
// straight into the root's memory over NVLink. Host code only.
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstring>
#include <mutex>
#include <vector>

#include "gg_internal.h"
#include "grouped_gemm_b200.h"

namespace {

static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(gg_ipc_handle{}.handle), "IPC handle size");

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuMemGetAddressRange_v3020>(nullptr);
    return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  }();
  return fn;
}

struct Mapping {
  char* base;  // what cudaIpcOpenMemHandle returned
  char* end;   // base + the exported allocation's size
};

std::mutex g_mu;
std::vector<Mapping> g_open;  // mappings made by gg_ipc_open, closed by gg_ipc_close
std::atomic<unsigned> g_generation{0};

}  // namespace

namespace gg {
unsigned ipc_mapping_generation() { return g_generation.load(std::memory_order_acquire); }
}  // namespace gg

extern "C" {

int gg_ipc_export(const void* ptr, gg_ipc_handle* out) {
  if (!ptr || !out) return cudaErrorInvalidValue;
  PFN_cuMemGetAddressRange_v3020 range = address_range_fn();
  if (!range) return cudaErrorNotSupported;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  cudaIpcMemHandle_t h;
  const cudaError_t st = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (st != cudaSuccess) return st;
  std::memcpy(out->handle, &h, sizeof h);
  out->offset = static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  out->bytes = static_cast<unsigned long long>(size) - out->offset;
  return cudaSuccess;
}

int gg_ipc_open(const gg_ipc_handle* handle, void** ptr) {
  if (!handle || !ptr) return cudaErrorInvalidValue;
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->handle, sizeof h);
  void* base = nullptr;
  const cudaError_t st = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (st != cudaSuccess) return st;
  g_generation.fetch_add(1, std::memory_order_acq_rel);
  char* b = static_cast<char*>(base);
  {
    std::lock_guard<std::mutex> lock(g_mu);
    g_open.push_back(Mapping{b, b + handle->offset + handle->bytes});
  }
  *ptr = b + handle->offset;
  return cudaSuccess;
}

int gg_ipc_close(void* ptr) {
  if (!ptr) return cudaErrorInvalidValue;
  char* p = static_cast<char*>(ptr);
  char* base = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    for (size_t i = 0; i < g_open.size(); ++i) {
      if (p >= g_open[i].base && p < g_open[i].end) {
        base = g_open[i].base;
        g_open.erase(g_open.begin() + static_cast<std::ptrdiff_t>(i));
        break;
      }
    }
  }
  if (!base) return cudaErrorInvalidValue;
  const cudaError_t st = cudaIpcCloseMemHandle(base);
  g_generation.fetch_add(1, std::memory_order_acq_rel);
  return st;
}

}  // extern "C"
