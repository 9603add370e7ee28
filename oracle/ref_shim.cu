// C-ABI shim around the reference implementation, compiled together with the reference's own
// sources (unmodified, from where they lie) by oracle/Makefile into oracle/_ref/libgg_ref.so.
// TEST INFRASTRUCTURE ONLY: the product never links or loads this library.
//
// The reference namespace is renamed at compile time (-Dgrouped_gemm=grouped_gemm_ref) so that
// its symbols cannot collide with the B200 library when both are loaded into one process.
//
// What it exposes:
//   - the reference host preparation (src/grouped_gemm.cu:952-1022, 1319-1329), runnable on CPU;
//   - the reference host GEMM compute_reference (tests/test_correctness.cu:85-102), reached by
//     including the test translation unit with its main() renamed, timed single- or multi-thread;
//   - the reference test's input generator (tests/test_correctness.cu:106-197), GPU box only,
//     used to pin the committed golden inputs;
//   - the reference's own CUDA kernels (src/grouped_gemm.cu:640-688) built for sm_100a, GPU only.

#define main reference_test_main
#include "tests/test_correctness.cu"
#undef main

#include <atomic>
#include <chrono>
#include <cstring>
#include <thread>
#include <vector>

// Layout of gg_problem / grouped_gemm::ProblemDesc. Declared outside any anonymous namespace so
// that the extern "C" entry points taking it keep external linkage.
struct RefProblem {
  int m, n, k;
  const void* a;
  const void* b;
  const float* c;
  float* d;
  int lda, ldb, ldc, ldd;
  float alpha, beta;
};

namespace {

grouped_gemm_ref::KernelConfig make_cfg(int cta_m, int cta_n, int cta_k, int use_tc) {
  grouped_gemm_ref::KernelConfig cfg{};
  cfg.cta_m = cta_m;
  cfg.cta_n = cta_n;
  cfg.cta_k = cta_k;
  cfg.threads = 256;
  cfg.persistent_ctas = 0;
  cfg.use_tensor_cores = use_tc != 0;
  return cfg;
}

std::vector<grouped_gemm_ref::ProblemDesc> to_ref(const RefProblem* ps, int count) {
  std::vector<grouped_gemm_ref::ProblemDesc> v(static_cast<size_t>(count > 0 ? count : 0));
  for (int i = 0; i < count; ++i) {
    grouped_gemm_ref::ProblemDesc p{};
    p.m = ps[i].m;
    p.n = ps[i].n;
    p.k = ps[i].k;
    p.a = static_cast<const __half*>(ps[i].a);
    p.b = static_cast<const __half*>(ps[i].b);
    p.c = ps[i].c;
    p.d = ps[i].d;
    p.lda = ps[i].lda;
    p.ldb = ps[i].ldb;
    p.ldc = ps[i].ldc;
    p.ldd = ps[i].ldd;
    p.alpha = ps[i].alpha;
    p.beta = ps[i].beta;
    v[static_cast<size_t>(i)] = p;
  }
  return v;
}

size_t elems(int rows, int cols) { return safe_matrix_elems(rows, cols); }

// Host buffers of one problem in the reference test's own fixture type.
void fill_buffer(ProblemBuffer& pb, const RefProblem& p, const uint16_t* a, const uint16_t* b,
                 const float* c) {
  pb.m = p.m;
  pb.n = p.n;
  pb.k = p.k;
  pb.lda = p.lda;
  pb.ldb = p.ldb;
  pb.ldc = p.ldc;
  pb.ldd = p.ldd;
  pb.alpha = p.alpha;
  pb.beta = p.beta;
  pb.h_a.resize(elems(p.m, p.lda));
  pb.h_b.resize(elems(p.k, p.ldb));
  pb.h_c.resize(elems(p.m, p.ldc));
  pb.h_ref.assign(elems(p.m, p.ldd), 0.0f);
  std::memcpy(pb.h_a.data(), a, pb.h_a.size() * sizeof(uint16_t));
  std::memcpy(pb.h_b.data(), b, pb.h_b.size() * sizeof(uint16_t));
  std::memcpy(pb.h_c.data(), c, pb.h_c.size() * sizeof(float));
}

}  // namespace

extern "C" {

// ---- host preparation (CPU) ----------------------------------------------------------------

int ref_prepare(const RefProblem* problems, int count, int cta_m, int cta_n, int cta_k, int mode,
                int* sorted_to_original, int* tile_offsets) {
  const auto v = to_ref(problems, count);
  const auto cfg = make_cfg(cta_m, cta_n, cta_k, 1);
  const grouped_gemm_ref::PreparedProblemSet prep =
      grouped_gemm_ref::prepare_problem_set(v, cfg, static_cast<grouped_gemm_ref::SortMode>(mode));
  for (size_t i = 0; i < prep.sorted_to_original.size(); ++i) sorted_to_original[i] = prep.sorted_to_original[i];
  for (size_t i = 0; i < prep.tile_offsets.size(); ++i) tile_offsets[i] = prep.tile_offsets[i];
  return prep.total_tiles;
}

const char* ref_sort_mode_name(int mode) {
  return grouped_gemm_ref::sort_mode_name(static_cast<grouped_gemm_ref::SortMode>(mode));
}

int ref_count_non_empty(const RefProblem* problems, int count, int cta_m, int cta_n, int cta_k) {
  return grouped_gemm_ref::count_non_empty_problems(to_ref(problems, count), make_cfg(cta_m, cta_n, cta_k, 1));
}

// ---- the reference host GEMM (CPU) -----------------------------------------------------------
// a/b/c/d are the per-problem host arrays (FP16 bits, FP16 bits, FP32, FP32), packed with the
// problem's own leading dimensions. Runs compute_reference over all problems on `threads`
// host threads (problems handed out dynamically) and returns the seconds spent in that loop
// only; buffer set-up and copies are outside the timed region.
double ref_host_gemm_batch(const RefProblem* problems, int count, const uint16_t* const* a,
                           const uint16_t* const* b, const float* const* c, float* const* d,
                           int threads) {
  std::vector<ProblemBuffer> bufs(static_cast<size_t>(count));
  for (int i = 0; i < count; ++i) fill_buffer(bufs[static_cast<size_t>(i)], problems[i], a[i], b[i], c[i]);
  if (threads < 1) threads = 1;
  std::atomic<int> next{0};
  auto worker = [&]() {
    for (;;) {
      const int i = next.fetch_add(1);
      if (i >= count) return;
      compute_reference(bufs[static_cast<size_t>(i)]);
    }
  };
  const auto t0 = std::chrono::steady_clock::now();
  if (threads == 1) {
    worker();
  } else {
    std::vector<std::thread> pool;
    for (int t = 0; t < threads; ++t) pool.emplace_back(worker);
    for (auto& th : pool) th.join();
  }
  const auto t1 = std::chrono::steady_clock::now();
  for (int i = 0; i < count; ++i) {
    const ProblemBuffer& pb = bufs[static_cast<size_t>(i)];
    if (d[i] != nullptr) std::memcpy(d[i], pb.h_ref.data(), pb.h_ref.size() * sizeof(float));
  }
  return std::chrono::duration<double>(t1 - t0).count();
}

// ---- the reference test's input generator (needs a GPU: it allocates device buffers) -------
// Runs init_problem_buffers (tests/test_correctness.cu:106-197) on the given shapes and copies
// the host-side inputs and the host reference result out, packed problem after problem with
// safe_matrix_elems sizes. Returns 0 on success.
int ref_test_inputs(const int* shapes_mnk, int count, uint16_t* a_out, uint16_t* b_out, float* c_out,
                    float* alpha_out, float* beta_out, float* ref_out) {
  std::vector<std::tuple<int, int, int>> shapes;
  for (int i = 0; i < count; ++i)
    shapes.emplace_back(shapes_mnk[3 * i], shapes_mnk[3 * i + 1], shapes_mnk[3 * i + 2]);
  std::vector<ProblemBuffer> buffers;
  std::vector<grouped_gemm_ref::ProblemDesc> problems;
  if (!init_problem_buffers(shapes, &buffers, &problems)) return 1;
  size_t oa = 0, ob = 0, oc = 0, od = 0;
  for (int i = 0; i < count; ++i) {
    const ProblemBuffer& pb = buffers[static_cast<size_t>(i)];
    std::memcpy(a_out + oa, pb.h_a.data(), pb.h_a.size() * sizeof(uint16_t));
    std::memcpy(b_out + ob, pb.h_b.data(), pb.h_b.size() * sizeof(uint16_t));
    std::memcpy(c_out + oc, pb.h_c.data(), pb.h_c.size() * sizeof(float));
    std::memcpy(ref_out + od, pb.h_ref.data(), pb.h_ref.size() * sizeof(float));
    oa += pb.h_a.size();
    ob += pb.h_b.size();
    oc += pb.h_c.size();
    od += pb.h_ref.size();
    alpha_out[i] = pb.alpha;
    beta_out[i] = pb.beta;
  }
  return 0;
}

// CPU-only restatement of the host half of init_problem_buffers (tests/test_correctness.cu:114-152):
// the same std::mt19937 seed, the same uniform_real_distribution<float>(-1, 1) draw order
// (alpha, beta, then A, B, C element by element) and the same packed leading dimensions, followed
// by the reference's own compute_reference. Same output packing as ref_test_inputs; the GPU test
// suite checks that both produce identical bytes, which pins the committed fixtures.
int ref_test_inputs_host(const int* shapes_mnk, int count, unsigned seed, uint16_t* a_out,
                         uint16_t* b_out, float* c_out, float* alpha_out, float* beta_out,
                         float* ref_out) {
  std::mt19937 rng(seed);
  std::uniform_real_distribution<float> dist(-1.0f, 1.0f);
  size_t oa = 0, ob = 0, oc = 0, od = 0;
  for (int i = 0; i < count; ++i) {
    ProblemBuffer pb;
    pb.m = shapes_mnk[3 * i];
    pb.n = shapes_mnk[3 * i + 1];
    pb.k = shapes_mnk[3 * i + 2];
    pb.lda = std::max(1, pb.k);
    pb.ldb = std::max(1, pb.n);
    pb.ldc = std::max(1, pb.n);
    pb.ldd = std::max(1, pb.n);
    pb.alpha = dist(rng);
    pb.beta = dist(rng);
    pb.h_a.resize(elems(pb.m, pb.lda));
    pb.h_b.resize(elems(pb.k, pb.ldb));
    pb.h_c.resize(elems(pb.m, pb.ldc));
    pb.h_ref.assign(elems(pb.m, pb.ldd), 0.0f);
    for (auto& x : pb.h_a) x = __float2half_rn(dist(rng));
    for (auto& x : pb.h_b) x = __float2half_rn(dist(rng));
    for (auto& x : pb.h_c) x = dist(rng);
    compute_reference(pb);
    std::memcpy(a_out + oa, pb.h_a.data(), pb.h_a.size() * sizeof(uint16_t));
    std::memcpy(b_out + ob, pb.h_b.data(), pb.h_b.size() * sizeof(uint16_t));
    std::memcpy(c_out + oc, pb.h_c.data(), pb.h_c.size() * sizeof(float));
    std::memcpy(ref_out + od, pb.h_ref.data(), pb.h_ref.size() * sizeof(float));
    oa += pb.h_a.size();
    ob += pb.h_b.size();
    oc += pb.h_c.size();
    od += pb.h_ref.size();
    alpha_out[i] = pb.alpha;
    beta_out[i] = pb.beta;
  }
  return 0;
}

// ---- the reference's own CUDA kernels, built for sm_100a (GPU only) -------------------------

int ref_run_grouped_once(const RefProblem* problems, int count, int mode, int cta_m, int cta_n,
                         int cta_k, int use_tc, void* stream) {
  return static_cast<int>(grouped_gemm_ref::run_grouped_gemm_once(
      to_ref(problems, count), static_cast<grouped_gemm_ref::SortMode>(mode),
      make_cfg(cta_m, cta_n, cta_k, use_tc), static_cast<cudaStream_t>(stream)));
}

int ref_run_baseline(const RefProblem* problems, int count, int cta_m, int cta_n, int cta_k,
                     int use_tc, void* stream) {
  return static_cast<int>(grouped_gemm_ref::run_baseline_per_problem(
      to_ref(problems, count), make_cfg(cta_m, cta_n, cta_k, use_tc), static_cast<cudaStream_t>(stream)));
}

// Times executor.run like the reference bench (bench/benchmark_grouped_gemm.cu:540-566): prepare
// and build once, `warmup` untimed runs, then `iters` runs between two events on `stream`.
int ref_time_grouped(const RefProblem* problems, int count, int mode, int cta_m, int cta_n,
                     int cta_k, int use_tc, int warmup, int iters, void* stream, float* ms_per_run,
                     int* total_tiles, int* grid_ctas) {
  const auto cfg = make_cfg(cta_m, cta_n, cta_k, use_tc);
  const auto prep = grouped_gemm_ref::prepare_problem_set(
      to_ref(problems, count), cfg, static_cast<grouped_gemm_ref::SortMode>(mode));
  grouped_gemm_ref::GroupedGemmExecutor ex;
  cudaError_t st = ex.build(prep, cfg);
  if (st != cudaSuccess) return static_cast<int>(st);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int i = 0; i < warmup; ++i) {
    st = ex.run(s);
    if (st != cudaSuccess) return static_cast<int>(st);
  }
  cudaEvent_t e0, e1;
  cudaEventCreate(&e0);
  cudaEventCreate(&e1);
  cudaEventRecord(e0, s);
  for (int i = 0; i < iters; ++i) {
    st = ex.run(s);
    if (st != cudaSuccess) break;
  }
  cudaEventRecord(e1, s);
  cudaEventSynchronize(e1);
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (st != cudaSuccess) return static_cast<int>(st);
  *ms_per_run = ms / static_cast<float>(iters > 0 ? iters : 1);
  *total_tiles = ex.total_tiles();
  *grid_ctas = ex.grid_ctas();
  return static_cast<int>(cudaDeviceSynchronize());
}

}  // extern "C"
