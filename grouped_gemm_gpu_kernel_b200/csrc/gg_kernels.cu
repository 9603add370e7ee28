// gg_kernels.cu -- instantiates the sm_100a grouped GEMM kernel for each tile variant and owns
// the launch / attribute / occupancy plumbing (the role of reference src/grouped_gemm.cu:691-910).
#include <atomic>
#include <cstdint>

#include "gg_internal.h"
#include "gg_kernel.cuh"

namespace gg {

namespace {

template <int BM, int BN>
struct VariantTraits {
  static constexpr int kSmem = SmemLayout<BM, BN>::kDynamicSmem;
  static void* kernel() { return reinterpret_cast<void*>(&grouped_gemm_sm100_kernel<BM, BN>); }
};

// One bit per device: the dynamic shared-memory attribute has been raised there.
std::atomic<unsigned long long> g_attr_done[static_cast<int>(Variant::kCount)];

template <typename Fn>
auto dispatch(Variant v, Fn&& fn) {
  switch (v) {
    case Variant::k64x64:
      return fn(VariantTraits<64, 64>{});
    case Variant::k128x64:
      return fn(VariantTraits<128, 64>{});
    case Variant::k64x128:
      return fn(VariantTraits<64, 128>{});
    case Variant::k128x128:
      return fn(VariantTraits<128, 128>{});
    case Variant::k128x256:
    default:
      return fn(VariantTraits<128, 256>{});
  }
}

bool valid(Variant v) { return static_cast<int>(v) >= 0 && static_cast<int>(v) < static_cast<int>(Variant::kCount); }

}  // namespace

Variant resolve_variant(int cta_m, int cta_n, int cta_k, int threads) {
  if (threads != kThreads) return Variant::kUnsupported;
  // the reference's shapes (same tile decomposition, cta_k names the variant only)
  if (cta_m == 64 && cta_n == 64 && cta_k == 16) return Variant::k64x64;
  if (cta_m == 128 && cta_n == 64 && cta_k == 32) return Variant::k128x64;
  if (cta_m == 64 && cta_n == 128 && cta_k == 32) return Variant::k64x128;
  // sm_100a-native shapes
  if (cta_m == 128 && cta_n == 128 && cta_k == 64) return Variant::k128x128;
  if (cta_m == 128 && cta_n == 256 && cta_k == 64) return Variant::k128x256;
  if (cta_m == 128 && cta_n == 64 && cta_k == 64) return Variant::k128x64;
  return Variant::kUnsupported;
}

int variant_bm(Variant v) {
  return (v == Variant::k64x64 || v == Variant::k64x128) ? 64 : 128;
}

int variant_bn(Variant v) {
  switch (v) {
    case Variant::k64x64:
    case Variant::k128x64:
      return 64;
    case Variant::k64x128:
    case Variant::k128x128:
      return 128;
    default:
      return 256;
  }
}

int variant_dynamic_smem(Variant v) {
  if (!valid(v)) return 0;
  return dispatch(v, [](auto t) { return decltype(t)::kSmem; });
}

cudaError_t prepare_kernel(Variant v) {
  if (!valid(v)) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  const unsigned long long bit = 1ull << (dev & 63);
  auto& done = g_attr_done[static_cast<int>(v)];
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  st = dispatch(v, [](auto t) {
    return cudaFuncSetAttribute(decltype(t)::kernel(), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                decltype(t)::kSmem);
  });
  if (st == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
  return st;
}

cudaError_t launch_grouped_kernel(Variant v, const KernelParams& params, int grid, cudaStream_t stream) {
  cudaError_t st = prepare_kernel(v);
  if (st != cudaSuccess) return st;
  switch (v) {
    case Variant::k64x64:
      grouped_gemm_sm100_kernel<64, 64><<<grid, kThreads, VariantTraits<64, 64>::kSmem, stream>>>(params);
      break;
    case Variant::k128x64:
      grouped_gemm_sm100_kernel<128, 64><<<grid, kThreads, VariantTraits<128, 64>::kSmem, stream>>>(params);
      break;
    case Variant::k64x128:
      grouped_gemm_sm100_kernel<64, 128><<<grid, kThreads, VariantTraits<64, 128>::kSmem, stream>>>(params);
      break;
    case Variant::k128x128:
      grouped_gemm_sm100_kernel<128, 128><<<grid, kThreads, VariantTraits<128, 128>::kSmem, stream>>>(params);
      break;
    case Variant::k128x256:
      grouped_gemm_sm100_kernel<128, 256><<<grid, kThreads, VariantTraits<128, 256>::kSmem, stream>>>(params);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t kernel_occupancy(Variant v, int* active_blocks_per_sm, cudaFuncAttributes* attrs) {
  cudaError_t st = prepare_kernel(v);
  if (st != cudaSuccess) return st;
  st = dispatch(v, [&](auto t) {
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(active_blocks_per_sm, decltype(t)::kernel(), kThreads,
                                                         decltype(t)::kSmem);
  });
  if (st != cudaSuccess) return st;
  return dispatch(v, [&](auto t) { return cudaFuncGetAttributes(attrs, decltype(t)::kernel()); });
}

cudaError_t launch_wait_selftest(int* status, unsigned long long timeout_ns, cudaStream_t stream) {
  wait_timeout_selftest_kernel<<<1, 32, 0, stream>>>(status, timeout_ns);
  return cudaGetLastError();
}

}  // namespace gg
