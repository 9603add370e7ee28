// gg_internal.h -- declarations shared by the kernel unit (gg_kernels.cu) and the host runtime
// (gg_host.cu). Not installed; callers use grouped_gemm_b200.h or grouped_gemm/grouped_gemm.cuh.
#pragma once

#include <cuda_runtime.h>
#include <cstddef>

#include "gg_params.cuh"

namespace gg {

// Compiled tile variants (BM x BN output tiles; K is always consumed 64 deep).
enum class Variant : int {
  k64x64 = 0,
  k128x64 = 1,
  k64x128 = 2,
  k128x128 = 3,
  k128x256 = 4,
  k256x128 = 5,  // CTA pair (cta_group::2), 128 rows per CTA
  k256x256 = 6,  // CTA pair (cta_group::2), 128 rows per CTA
  kCount = 7,
  kUnsupported = -1,
};

// Maps a (cta_m, cta_n, cta_k, threads) request to a variant, kUnsupported otherwise. Accepts the
// reference's three shapes (reference src/grouped_gemm.cu:67-81) and the sm_100a-native ones.
Variant resolve_variant(int cta_m, int cta_n, int cta_k, int threads);
int variant_bm(Variant v);   // output tile rows
int variant_bn(Variant v);   // output tile columns
bool variant_is_pair(Variant v);
int variant_cta_rows(Variant v);  // A / D rows one CTA loads and stores (the TMA box height)
int variant_cta_cols(Variant v);  // B columns one CTA loads
int variant_dynamic_smem(Variant v);
int variant_ctas_per_tile(Variant v);

// Raises the kernel's dynamic shared-memory limit on the current device (once per device).
cudaError_t prepare_kernel(Variant v);
// overlap_previous: the grid may start while the previous kernel on the stream (a CTA-pair launch of
// the same executor) still runs (one-CTA 128-row variants only).
cudaError_t launch_grouped_kernel(Variant v, const KernelParams& params, int grid, cudaStream_t stream,
                                  bool overlap_previous = false);
cudaError_t kernel_occupancy(Variant v, int* active_blocks_per_sm, cudaFuncAttributes* attrs);
// CTAs of this variant that can be resident on the device at once (whole pairs for pair variants).
cudaError_t kernel_resident_ctas(Variant v, int* ctas);
cudaError_t launch_wait_selftest(int* status, unsigned long long timeout_ns, cudaStream_t stream);

// Count of IPC mappings opened or closed in this process (gg_ipc.cu); a cached answer about which
// GPU owns an address is stale once it changes.
unsigned ipc_mapping_generation();

// CUDA-core path (use_tensor_cores = false), gg_simt.cu: same parameters and tile numbering,
// the variant only fixes the tile shape.
// One operand copied into a 16-byte-aligned scratch matrix so that TMA can load it: `rows` rows of
// `row_bytes` bytes, from `src` (any alignment, pitch src_pitch bytes) to `dst` (16-byte aligned,
// pitch dst_pitch bytes, a multiple of 16).
struct RealignJob {
  const unsigned char* src;
  unsigned char* dst;
  long long src_pitch;
  long long dst_pitch;
  int rows;
  int row_bytes;
};

// Runs every job of the device array `jobs` in one launch on `stream` (max_units: the most
// 16-byte destination chunks of any job, which sizes the grid).
cudaError_t launch_realign(const RealignJob* jobs, int count, long long max_units, cudaStream_t stream);

// overlap_previous: launched with programmatic stream serialisation, so its CTAs may start on
// the SMs the previous grid of the stream leaves free (that grid must not produce its inputs).
cudaError_t launch_simt_kernel(Variant v, const KernelParams& params, int grid, cudaStream_t stream,
                               bool overlap_previous = false);
cudaError_t simt_resident_ctas(int* ctas);
cudaError_t simt_occupancy(int* active_blocks_per_sm, cudaFuncAttributes* attrs);
int simt_threads();

}  // namespace gg
