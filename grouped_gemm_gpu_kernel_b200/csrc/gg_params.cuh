// gg_params.cuh -- constants, shared-memory layout and launch parameters of the grouped GEMM
// kernel, shared by the kernel unit and the host runtime (no device code here).
#pragma once

#include <cuda.h>
#include <cstddef>
#include <cstdint>

#include "grouped_gemm/device_problem_desc.cuh"

namespace gg {

using grouped_gemm::DeviceProblemDesc;

constexpr int kThreads = 384;  // 12 warps: 8 epilogue, MMA, scheduler, 2 producers
constexpr int kBK = 64;     // K elements per pipeline stage: one 128-byte swizzle row of FP16
constexpr int kMmaM = 128;  // tcgen05 M used by every variant
constexpr int kMmaK = 16;   // tcgen05 K for 16-bit inputs
constexpr int kRing = 4;    // scheduler ring depth
constexpr int kConfigThreads = 256;  // KernelConfig::threads accepted (the reference's default)
constexpr int kEpiWarps = 8;         // two per TMEM lane quarter, each with half the tile's columns
constexpr int kMmaWarp = 8;
constexpr int kSchedWarp = 9;
constexpr int kProdWarp0 = 10;
constexpr int kProdThreads = 64;
constexpr int kRingConsumerWarps = kEpiWarps + 1 + 2;  // arrivals that free one ring slot
constexpr int kEpiTileBytes = 128 * 128;               // 8 warps x one 4 KB staging tile (32 x 32 FP32)
constexpr int kEpiWarpBytes = 2 * kEpiTileBytes / kEpiWarps;
constexpr int kEpiThreads = kEpiWarps * 32;
// Tensor maps per problem, in this order: A (64 K x BM rows), B by 64-column chunk (64 N x 64 K),
// B as one 3-D box per stage (64 N x 64 K x BN/64 chunks; full chunks only), D (32 cols x BM rows).
constexpr int kMapsPerProblem = 4;
constexpr int kMapA = 0;
constexpr int kMapB = 1;
constexpr int kMapB3 = 2;
constexpr int kMapD = 3;
constexpr int kDescWords = static_cast<int>(sizeof(DeviceProblemDesc) / 4);

struct TileSlot {
  int problem;  // sorted problem index; -1 = no more work for this CTA
  int tile_m;
  int tile_n;
  int reserved;
  DeviceProblemDesc desc;
};

template <int BN>
struct StageCount {
  static constexpr int value = BN >= 256 ? 4 : 6;
};

// TMEM accumulators per CTA: BN FP32 columns each, 512 columns in all. More than two let the MMA
// run several tiles ahead of an epilogue that is waiting on the SM's store bandwidth.
template <int BN>
struct AccCount {
  static constexpr int value = BN <= 128 ? 4 : 2;
};

template <int BM, int BN>
struct SmemLayout {
  static constexpr int kStages = StageCount<BN>::value;
  static constexpr int kAcc = AccCount<BN>::value;
  static constexpr int kABytes = kMmaM * 128;
  static constexpr int kBBytes = BN * 128;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = kStages * kStageBytes;
  static constexpr int kEpiBytes = 2 * kEpiTileBytes;  // double-buffered staging tile
  static constexpr int kRingOffset = kEpiOffset + kEpiBytes;
  static constexpr int kBarOffset = kRingOffset + kRing * static_cast<int>(sizeof(TileSlot));
  static constexpr int kNumBars = 2 * kStages + 2 * kAcc + 2 * kRing + 1;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kBytes = kMiscOffset + 32;
  static constexpr int kDynamicSmem = kBytes + 1024;  // slack to align the base to 1024 bytes
  static constexpr uint32_t kATxBytes = static_cast<uint32_t>(BM) * 128;
  static constexpr uint32_t kBTxBytes = static_cast<uint32_t>(BN) * 128;
  static constexpr uint32_t kTmemCols = kAcc * BN;
  static_assert(kRingOffset % 1024 == 0, "stage and staging tiles stay 1024-byte aligned");
  static_assert(kBarOffset % 8 == 0, "mbarriers are 8-byte aligned");
  static_assert(kDynamicSmem <= 232448, "fits the 227 KB opt-in shared memory of a CTA");
  static_assert(kDynamicSmem > 232448 / 2 + 1024, "one CTA per SM, so TMEM allocation never contends");
  static_assert(kTmemCols >= 32 && kTmemCols <= 512 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM alloc size");
};

struct KernelParams {
  CUtensorMap single_maps[kMapsPerProblem];  // baseline launch: the maps of its one problem
  DeviceProblemDesc single_desc;      // baseline launch: its one problem
  const DeviceProblemDesc* problems;  // grouped launch: problem table in sorted order
  const CUtensorMap* tmaps;           // grouped launch: kMapsPerProblem maps per problem (64-byte aligned)
  const int* tile_offsets;            // grouped launch: problem_count + 1 prefix sums
  int* tile_counter;                  // grouped launch: claim counter, zero at launch
  int* done_counter;                  // when set: CTAs of the launch that have finished; the last one
                                      // sets tile_counter and this back to zero for the next launch
                                      // (null: the host clears tile_counter before every launch)
  const int* total_tiles_dev;         // when set: the tile count, written on the device by an
                                      // earlier launch (device-side preparation); else total_tiles
  int* status;                        // GG_STATUS_* bits
  unsigned long long timeout_ns;      // limit of every wait
  int problem_count;
  int total_tiles;
  int raster_group;  // M-tiles per raster group inside a problem (L2 reuse of A and B panels)
  int single_mode;   // 1: baseline launch, tiles blockIdx.x + i*gridDim.x of single_desc
  int input_format;   // A and B element type: 0 = FP16, 1 = BF16 (GG_INPUT_*)
  int output_format;  // C and D element type: 0 = FP32, 1 = FP16, 2 = BF16 (GG_OUTPUT_*)
  int activation;     // GG_ACT_* applied to D after the bias
  int layout;         // bit 0: every A stored column-major (k x m); bit 1: every B column-major (n x k)
  const float* const* bias;  // per map slot: that problem's bias (n FP32 values) or null; null: none
};

#ifdef __CUDACC__
// Called once per CTA (one thread) after the CTA's last tile claim: the last CTA of the grid to
// get here clears the claim counter and the finished count, so the next launch with the same
// counters needs no host-side reset before it.
__device__ __forceinline__ void finish_launch(const KernelParams& p) {
  if (!p.done_counter) return;
  __threadfence();
  if (atomicAdd(p.done_counter, 1) == static_cast<int>(gridDim.x) - 1) {
    atomicExch(p.tile_counter, 0);
    atomicExch(p.done_counter, 0);
  }
}
#endif

}  // namespace gg
