// gg_kernels.cu -- instantiates the sm_100a grouped GEMM kernel for each tile variant and owns
// the launch / attribute / occupancy plumbing (the role of reference src/grouped_gemm.cu:691-910).
#include <atomic>
#include <cstdint>

#include "gg_internal.h"
#include "gg_kernel.cuh"
#include "gg_kernel_pair.cuh"

namespace gg {

namespace {

template <int BM, int BN>
struct VariantTraits {
  static constexpr int kSmem = SmemLayout<BM, BN>::kDynamicSmem;
  static void* kernel() { return reinterpret_cast<void*>(&grouped_gemm_sm100_kernel<BM, BN>); }
};

template <int BN>
struct PairTraits {
  static constexpr int kSmem = PairLayout<BN>::kDynamicSmem;
  static void* kernel() { return reinterpret_cast<void*>(&grouped_gemm_sm100_pair_kernel<BN>); }
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
    case Variant::k256x128:
      return fn(PairTraits<128>{});
    case Variant::k256x256:
      return fn(PairTraits<256>{});
    case Variant::k128x256:
    default:
      return fn(VariantTraits<128, 256>{});
  }
}

// Launch configuration of a pair variant: clusters of two CTAs along x.
cudaLaunchConfig_t pair_config(int grid, size_t smem, cudaStream_t stream, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

bool valid(Variant v) { return static_cast<int>(v) >= 0 && static_cast<int>(v) < static_cast<int>(Variant::kCount); }

}  // namespace

Variant resolve_variant(int cta_m, int cta_n, int cta_k, int threads) {
  if (threads != kConfigThreads) return Variant::kUnsupported;
  // the reference's shapes (same tile decomposition, cta_k names the variant only)
  if (cta_m == 64 && cta_n == 64 && cta_k == 16) return Variant::k64x64;
  if (cta_m == 128 && cta_n == 64 && cta_k == 32) return Variant::k128x64;
  if (cta_m == 64 && cta_n == 128 && cta_k == 32) return Variant::k64x128;
  // sm_100a-native shapes
  if (cta_m == 256 && cta_n == 128 && cta_k == 64) return Variant::k256x128;
  if (cta_m == 256 && cta_n == 256 && cta_k == 64) return Variant::k256x256;
  if (cta_m == 128 && cta_n == 128 && cta_k == 64) return Variant::k128x128;
  if (cta_m == 128 && cta_n == 256 && cta_k == 64) return Variant::k128x256;
  if (cta_m == 128 && cta_n == 64 && cta_k == 64) return Variant::k128x64;
  return Variant::kUnsupported;
}

int variant_bm(Variant v) {
  if (v == Variant::k64x64 || v == Variant::k64x128) return 64;
  if (v == Variant::k256x128 || v == Variant::k256x256) return 256;
  return 128;
}

int variant_bn(Variant v) {
  switch (v) {
    case Variant::k64x64:
    case Variant::k128x64:
      return 64;
    case Variant::k64x128:
    case Variant::k128x128:
    case Variant::k256x128:
      return 128;
    default:
      return 256;
  }
}

bool variant_is_pair(Variant v) { return v == Variant::k256x128 || v == Variant::k256x256; }
int variant_cta_rows(Variant v) { return variant_is_pair(v) ? 128 : variant_bm(v); }
int variant_cta_cols(Variant v) { return variant_is_pair(v) ? variant_bn(v) / 2 : variant_bn(v); }
int variant_ctas_per_tile(Variant v) { return variant_is_pair(v) ? 2 : 1; }

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

// Launch of a one-CTA variant that may start while the previous kernel on the stream (a CTA-pair
// launch that triggers its dependents at start) still runs: the two work on disjoint outputs, so
// this grid's CTAs take SMs as the previous grid's CTAs retire (programmatic stream serialisation;
// the grid never waits on the previous one's results).
template <int BM, int BN>
cudaError_t launch_overlapping(const KernelParams& params, int grid, cudaStream_t stream) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = VariantTraits<BM, BN>::kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, grouped_gemm_sm100_kernel<BM, BN>, params);
}

cudaError_t launch_grouped_kernel(Variant v, const KernelParams& params, int grid, cudaStream_t stream,
                                  bool overlap_previous) {
  cudaError_t st = prepare_kernel(v);
  if (st != cudaSuccess) return st;
  if (overlap_previous) {
    switch (v) {
      case Variant::k128x128:
        return launch_overlapping<128, 128>(params, grid, stream);
      case Variant::k128x256:
        return launch_overlapping<128, 256>(params, grid, stream);
      default:
        return cudaErrorInvalidValue;
    }
  }
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
    case Variant::k256x128: {
      if (grid % 2) return cudaErrorInvalidValue;
      cudaLaunchAttribute attr[1];
      const cudaLaunchConfig_t cfg = pair_config(grid, PairTraits<128>::kSmem, stream, attr);
      return cudaLaunchKernelEx(&cfg, grouped_gemm_sm100_pair_kernel<128>, params);
    }
    case Variant::k256x256: {
      if (grid % 2) return cudaErrorInvalidValue;
      cudaLaunchAttribute attr[1];
      const cudaLaunchConfig_t cfg = pair_config(grid, PairTraits<256>::kSmem, stream, attr);
      return cudaLaunchKernelEx(&cfg, grouped_gemm_sm100_pair_kernel<256>, params);
    }
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t kernel_resident_ctas(Variant v, int* ctas) {
  cudaError_t st = prepare_kernel(v);
  if (st != cudaSuccess) return st;
  int dev = 0;
  st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  int sms = 0;
  st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (st != cudaSuccess) return st;
  if (!variant_is_pair(v)) {
    int active = 0;
    cudaFuncAttributes fa{};
    st = kernel_occupancy(v, &active, &fa);
    if (st != cudaSuccess) return st;
    *ctas = sms * (active > 0 ? active : 1);
    return cudaSuccess;
  }
  int clusters = 0;
  st = dispatch(v, [&](auto t) {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = pair_config(2, decltype(t)::kSmem, nullptr, attr);
    return cudaOccupancyMaxActiveClusters(&clusters, decltype(t)::kernel(), &cfg);
  });
  if (st != cudaSuccess) return st;
  *ctas = 2 * (clusters > 0 ? clusters : 1);
  return cudaSuccess;
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
