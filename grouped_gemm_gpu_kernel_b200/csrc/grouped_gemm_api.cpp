// grouped_gemm_api.cpp -- the reference's C++ API (namespace grouped_gemm, header
// grouped_gemm/grouped_gemm.cuh) implemented as thin wrappers over the C-ABI entry points of
// grouped_gemm_b200.h, so C++ callers and foreign-language callers reach the same code.
#include "grouped_gemm/grouped_gemm.cuh"

#include <new>
#include <type_traits>

#include "grouped_gemm_b200.h"

namespace grouped_gemm {

static_assert(sizeof(ProblemDesc) == sizeof(gg_problem), "ProblemDesc and gg_problem share one layout");
static_assert(offsetof(ProblemDesc, a) == offsetof(gg_problem, a), "ProblemDesc::a");
static_assert(offsetof(ProblemDesc, d) == offsetof(gg_problem, d), "ProblemDesc::d");
static_assert(offsetof(ProblemDesc, lda) == offsetof(gg_problem, lda), "ProblemDesc::lda");
static_assert(offsetof(ProblemDesc, alpha) == offsetof(gg_problem, alpha), "ProblemDesc::alpha");
static_assert(offsetof(ProblemDesc, beta) == offsetof(gg_problem, beta), "ProblemDesc::beta");
static_assert(std::is_trivially_copyable<ProblemDesc>::value, "ProblemDesc is passed by bytes");

namespace {

const gg_problem* as_c(const ProblemDesc* p) { return reinterpret_cast<const gg_problem*>(p); }
gg_problem* as_c(ProblemDesc* p) { return reinterpret_cast<gg_problem*>(p); }

gg_config to_c(const KernelConfig& c) {
  gg_config g{};
  g.cta_m = c.cta_m;
  g.cta_n = c.cta_n;
  g.cta_k = c.cta_k;
  g.threads = c.threads;
  g.persistent_ctas = c.persistent_ctas;
  g.use_tensor_cores = c.use_tensor_cores ? 1 : 0;
  // the reference's API is FP16 in, FP32 out, row-major, no fused bias or activation; the rest are
  // C-ABI extensions
  g.input_type = GG_INPUT_F16;
  g.output_type = GG_OUTPUT_F32;
  g.activation = GG_ACT_NONE;
  g.a_layout = GG_LAYOUT_ROW_MAJOR;
  g.b_layout = GG_LAYOUT_ROW_MAJOR;
  return g;
}

}  // namespace

PreparedProblemSet prepare_problem_set(const std::vector<ProblemDesc>& problems, const KernelConfig& config,
                                       SortMode sort_mode) {
  PreparedProblemSet out;
  const int count = static_cast<int>(problems.size());
  out.sorted_problems.resize(problems.size());
  out.sorted_to_original.resize(problems.size());
  out.tile_offsets.resize(problems.size() + 1);
  const gg_config cfg = to_c(config);
  int total = 0;
  if (gg_prepare(as_c(problems.data()), count, &cfg, static_cast<int>(sort_mode), as_c(out.sorted_problems.data()),
                 out.sorted_to_original.data(), out.tile_offsets.data(), &total) != 0) {
    // Only a non-positive tile extent gets here; the reference would divide by it.
    out.tile_offsets.assign(problems.size() + 1, 0);
  }
  out.total_tiles = total;
  return out;
}

const char* sort_mode_name(SortMode sort_mode) { return gg_sort_mode_name(static_cast<int>(sort_mode)); }

cudaError_t query_occupancy(const KernelConfig& config, OccupancyInfo* info) {
  if (info == nullptr) return cudaErrorInvalidValue;
  const gg_config cfg = to_c(config);
  gg_occupancy o{};
  const int st = gg_query_occupancy(&cfg, &o);
  if (st != 0) return static_cast<cudaError_t>(st);
  info->sm_count = o.sm_count;
  info->max_blocks_per_sm = o.max_blocks_per_sm;
  info->active_blocks_per_sm = o.active_blocks_per_sm;
  info->threads_per_block = o.threads_per_block;
  info->max_threads_per_sm = o.max_threads_per_sm;
  info->warps_per_block = o.warps_per_block;
  info->max_warps_per_sm = o.max_warps_per_sm;
  info->active_warps_per_sm = o.active_warps_per_sm;
  info->max_registers_per_sm = o.max_registers_per_sm;
  info->max_registers_per_block = o.max_registers_per_block;
  info->estimated_registers_per_thread = o.estimated_registers_per_thread;
  info->estimated_registers_per_block = o.estimated_registers_per_block;
  info->registers_per_thread = o.registers_per_thread;
  info->registers_per_block = o.registers_per_block;
  info->register_limited_blocks_per_sm = o.register_limited_blocks_per_sm;
  info->static_shared_bytes = o.static_shared_bytes;
  info->dynamic_shared_bytes = o.dynamic_shared_bytes;
  info->theoretical_occupancy = o.theoretical_occupancy;
  info->using_tensor_cores = o.using_tensor_cores != 0;
  return cudaSuccess;
}

struct GroupedGemmExecutor::Impl {
  gg_executor* handle = nullptr;
};

GroupedGemmExecutor::GroupedGemmExecutor() : impl_(new (std::nothrow) Impl()) {
  if (impl_ != nullptr && gg_executor_create(&impl_->handle) != 0) impl_->handle = nullptr;
}

GroupedGemmExecutor::~GroupedGemmExecutor() {
  if (impl_ != nullptr) {
    gg_executor_destroy(impl_->handle);
    delete impl_;
    impl_ = nullptr;
  }
}

GroupedGemmExecutor::GroupedGemmExecutor(GroupedGemmExecutor&& other) noexcept : impl_(other.impl_) {
  other.impl_ = nullptr;
}

GroupedGemmExecutor& GroupedGemmExecutor::operator=(GroupedGemmExecutor&& other) noexcept {
  if (this != &other) {
    if (impl_ != nullptr) {
      gg_executor_destroy(impl_->handle);
      delete impl_;
    }
    impl_ = other.impl_;
    other.impl_ = nullptr;
  }
  return *this;
}

cudaError_t GroupedGemmExecutor::build(const PreparedProblemSet& prepared, const KernelConfig& config) {
  if (impl_ == nullptr || impl_->handle == nullptr) return cudaErrorInvalidDevicePointer;
  const gg_config cfg = to_c(config);
  return static_cast<cudaError_t>(gg_executor_build(
      impl_->handle, as_c(prepared.sorted_problems.data()), static_cast<int>(prepared.sorted_problems.size()),
      prepared.tile_offsets.data(), static_cast<int>(prepared.tile_offsets.size()), prepared.total_tiles, &cfg));
}

cudaError_t GroupedGemmExecutor::run(cudaStream_t stream) const {
  if (impl_ == nullptr || impl_->handle == nullptr) return cudaErrorInvalidDevicePointer;
  return static_cast<cudaError_t>(gg_executor_run(impl_->handle, stream));
}

int GroupedGemmExecutor::problem_count() const {
  return impl_ != nullptr ? gg_executor_problem_count(impl_->handle) : 0;
}

int GroupedGemmExecutor::total_tiles() const { return impl_ != nullptr ? gg_executor_total_tiles(impl_->handle) : 0; }

int GroupedGemmExecutor::grid_ctas() const { return impl_ != nullptr ? gg_executor_grid_ctas(impl_->handle) : 0; }

cudaError_t run_grouped_gemm_once(const std::vector<ProblemDesc>& problems, SortMode sort_mode,
                                  const KernelConfig& config, cudaStream_t stream) {
  const gg_config cfg = to_c(config);
  return static_cast<cudaError_t>(gg_run_grouped_gemm_once(as_c(problems.data()), static_cast<int>(problems.size()),
                                                           static_cast<int>(sort_mode), &cfg, stream));
}

cudaError_t run_baseline_per_problem(const std::vector<ProblemDesc>& problems, const KernelConfig& config,
                                     cudaStream_t stream) {
  const gg_config cfg = to_c(config);
  return static_cast<cudaError_t>(
      gg_run_baseline_per_problem(as_c(problems.data()), static_cast<int>(problems.size()), &cfg, stream));
}

int count_non_empty_problems(const std::vector<ProblemDesc>& problems, const KernelConfig& config) {
  const gg_config cfg = to_c(config);
  return gg_count_non_empty_problems(as_c(problems.data()), static_cast<int>(problems.size()), &cfg);
}

}  // namespace grouped_gemm
