// grouped_gemm/grouped_gemm.cuh -- C++ API of the B200 grouped GEMM, a drop-in for the
// reference's header of the same path (reference include/grouped_gemm/grouped_gemm.cuh:1-132):
// same namespace, types, fields, signatures and error convention (cudaError_t, no exceptions).
// A program written against the reference compiles unchanged against this header and links to
// libgrouped_gemm_b200.so. Every function is a thin wrapper over the C-ABI in
// grouped_gemm_b200.h; the kernels underneath are hand-written sm_100a (tcgen05 + TMA) code.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

namespace grouped_gemm {

// Problem ordering applied by prepare_problem_set before tiles are numbered.
enum class SortMode {
  kNone = 0,
  kByK = 1,
  kByTiles = 2,
  kByTilesThenK = 3,
};

// One GEMM: D = alpha * A x B + beta * C. A is m x k FP16 (row stride lda), B is k x n FP16
// (ldb), C and D are m x n FP32 (ldc, ldd). C is read only when c != nullptr and beta != 0.
struct ProblemDesc {
  int m;
  int n;
  int k;

  const __half* a;
  const __half* b;
  const float* c;
  float* d;

  int lda;
  int ldb;
  int ldc;
  int ldd;

  float alpha = 1.0f;
  float beta = 0.0f;
};

// Tile shape and launch shape. The defaults are the reference's; the sm_100a-native shapes
// 128x128x64, 128x256x64, 128x64x64 and the CTA-pair shapes 256x128x64, 256x256x64 are also
// accepted (threads must be 256, the reference default; the kernel itself launches 384-thread
// blocks, which query_occupancy reports).
struct KernelConfig {
  int cta_m = 64;
  int cta_n = 64;
  int cta_k = 16;
  int threads = 256;

  int persistent_ctas = 0;
  bool use_tensor_cores = true;
};

// Problems in scheduling order, the map back to input order, and the tile prefix sum
// (tile_offsets.size() == sorted_problems.size() + 1, tile_offsets[0] == 0).
struct PreparedProblemSet {
  std::vector<ProblemDesc> sorted_problems;
  std::vector<int> sorted_to_original;
  std::vector<int> tile_offsets;
  int total_tiles = 0;
};

// Resource usage of the kernel a config selects: occupancy, shared memory, registers.
struct OccupancyInfo {
  int sm_count = 0;
  int max_blocks_per_sm = 0;
  int active_blocks_per_sm = 0;

  int threads_per_block = 0;
  int max_threads_per_sm = 0;
  int warps_per_block = 0;
  int max_warps_per_sm = 0;
  int active_warps_per_sm = 0;

  int max_registers_per_sm = 0;
  int max_registers_per_block = 0;

  // Model estimate (see query_occupancy).
  int estimated_registers_per_thread = 0;
  int estimated_registers_per_block = 0;

  // Compiler-reported values (cudaFuncGetAttributes).
  int registers_per_thread = 0;
  int registers_per_block = 0;
  int register_limited_blocks_per_sm = 0;

  int static_shared_bytes = 0;
  int dynamic_shared_bytes = 0;

  float theoretical_occupancy = 0.0f;
  bool using_tensor_cores = false;
};

PreparedProblemSet prepare_problem_set(
    const std::vector<ProblemDesc>& problems,
    const KernelConfig& config,
    SortMode sort_mode);

const char* sort_mode_name(SortMode sort_mode);

cudaError_t query_occupancy(const KernelConfig& config, OccupancyInfo* info);

// Owns the device-side problem table, TMA descriptors, tile offsets and tile counter of one
// prepared problem set. Move-only. One executor per concurrently running stream.
class GroupedGemmExecutor {
 public:
  GroupedGemmExecutor();
  ~GroupedGemmExecutor();

  GroupedGemmExecutor(const GroupedGemmExecutor&) = delete;
  GroupedGemmExecutor& operator=(const GroupedGemmExecutor&) = delete;

  GroupedGemmExecutor(GroupedGemmExecutor&& other) noexcept;
  GroupedGemmExecutor& operator=(GroupedGemmExecutor&& other) noexcept;

  cudaError_t build(const PreparedProblemSet& prepared, const KernelConfig& config);
  cudaError_t run(cudaStream_t stream = nullptr) const;

  int problem_count() const;
  int total_tiles() const;
  int grid_ctas() const;

 private:
  struct Impl;
  Impl* impl_;
};

cudaError_t run_grouped_gemm_once(
    const std::vector<ProblemDesc>& problems,
    SortMode sort_mode,
    const KernelConfig& config,
    cudaStream_t stream = nullptr);

cudaError_t run_baseline_per_problem(
    const std::vector<ProblemDesc>& problems,
    const KernelConfig& config,
    cudaStream_t stream = nullptr);

int count_non_empty_problems(
    const std::vector<ProblemDesc>& problems,
    const KernelConfig& config);

}  // namespace grouped_gemm
