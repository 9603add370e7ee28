/*
 * grouped_gemm_b200.h -- C-ABI of the B200 (sm_100a) grouped GEMM library libgrouped_gemm_b200.so.
 *
 * One launch runs many independent GEMMs  D_i = alpha_i * A_i x B_i + beta_i * C_i  with
 * A_i (m x k) and B_i (k x n) FP16 row-major, C_i and D_i FP32 row-major, FP32 accumulation
 * (the reference's contract). Extensions, all off by default: BF16 or FP8 A/B (gg_config.input_type),
 * FP16/BF16 C/D (gg_config.output_type), a per-column bias and an activation fused into the
 * epilogue (gg_executor_build_with_bias, gg_config.activation), column-major A and/or B
 * (gg_config.a_layout / b_layout).
 * This is the boundary a foreign-language caller binds (ctypes, cgo, JNI, ...): plain C types,
 * opaque handles, device pointers as void*, CUDA streams as void* (cudaStream_t; NULL = legacy
 * default stream). Every function that can fail returns an int holding a cudaError_t value:
 *   0  cudaSuccess
 *   1  cudaErrorInvalidValue          unsupported config, negative dims, inconsistent prepared set,
 *                                     null output argument
 *   17 cudaErrorInvalidDevicePointer  null a/b/d in a problem, or a null/destroyed executor
 *   702 cudaErrorLaunchTimeout        (gg_run_grouped_gemm_once only) a bounded wait inside the
 *                                     kernel ran out; D may be partly written
 *   other values are CUDA runtime errors passed through unchanged.
 * Asynchronous launches report such a timeout through a status word instead, read with
 * gg_executor_status, gg_baseline_status, gg_noalloc_status or gg_moe_plan_status.
 * An empty problem set (or one with zero tiles) is a successful no-op that launches nothing.
 *
 * Each entry point replaces one function of the reference C++ API
 * (reference include/grouped_gemm/grouped_gemm.cuh, implemented in src/grouped_gemm.cu); the
 * citation is given beside each. The C++ API itself is provided on top of this ABI by
 * include/grouped_gemm/grouped_gemm.cuh.
 */
#ifndef GROUPED_GEMM_B200_H_
#define GROUPED_GEMM_B200_H_

#ifdef __cplusplus
extern "C" {
#endif

#define GG_ABI_VERSION 2

/* Sort modes; reference grouped_gemm.cuh:11-16 (SortMode). */
#define GG_SORT_NONE 0
#define GG_SORT_BY_K 1
#define GG_SORT_BY_TILES 2
#define GG_SORT_BY_TILES_THEN_K 3

/* Bits of the device status word (gg_executor_status): a bounded wait inside the kernel ran out.
 * The kernel then stops, frees its tensor memory and returns instead of hanging. */
#define GG_STATUS_TIMEOUT_PRODUCER 0x1
#define GG_STATUS_TIMEOUT_MMA 0x2
#define GG_STATUS_TIMEOUT_EPILOGUE 0x4
#define GG_STATUS_TIMEOUT_SCHEDULER 0x8

/* One GEMM problem. Layout-identical to the reference's ProblemDesc (grouped_gemm.cuh:18-35);
 * a and b point to FP16 (__half) device memory (BF16 / FP8 with input_type), c and d to FP32 (FP16
 * or BF16 with GG_OUTPUT_F16 / GG_OUTPUT_BF16). c may be NULL; it is read only when beta != 0. */
typedef struct gg_problem {
  int m;
  int n;
  int k;
  const void* a;
  const void* b;
  const void* c;
  void* d;
  int lda;
  int ldb;
  int ldc;
  int ldd;
  float alpha;
  float beta;
} gg_problem;

/* Kernel configuration; the reference's KernelConfig (grouped_gemm.cuh:37-45) with the bool as
 * an int. Accepted (cta_m, cta_n, cta_k) with threads == 256:
 *   sm_100a-native tiles   128x128x64, 128x256x64, 128x64x64 (one CTA per tile), and
 *                          256x128x64, 256x256x64 (a cluster of two CTAs per tile,
 *                          tcgen05 cta_group::2: 128 rows per CTA)
 *   the reference's tiles  64x64x16, 128x64x32, 64x128x32  (same tile decomposition, run on the
 *                          same tcgen05 kernel; cta_k only selects the variant)
 * use_tensor_cores != 0 runs the tcgen05 tensor-core kernel; 0 runs the CUDA-core kernel (FP16
 * operands widened to FP32, FP32 FMA; the reference's SIMT path) with the same tile numbering.
 * input_type (no reference counterpart; the reference is FP16 only, and the C++ API of
 * grouped_gemm/grouped_gemm.cuh keeps the reference's KernelConfig and always passes FP16): the
 * element type of every A and B of the set: GG_INPUT_F16 (0), GG_INPUT_BF16, or the 8-bit floats
 * GG_INPUT_E4M3 (1 sign, 4 exponent bits with bias 7, 3 mantissa bits; no infinities, S.1111.111
 * is NaN) and GG_INPUT_E5M2 (1-5-2, bias 15, IEEE-style infinities and NaNs), one byte per element,
 * multiplied exactly and accumulated in FP32 (tcgen05 kind::f8f6f4). With 8-bit inputs the tensor
 * -core path needs tiles whose per-CTA B width is a multiple of 128 (128x128, 128x256, 64x128,
 * 256x256; others are an invalid config, unless B is column-major, see b_layout); any pointer
 * alignment and pitch is taken (16-byte aligned rows load by TMA, others by the zero-fill loader).
 * The CUDA-core path takes any tile.
 * output_type (no reference counterpart): the element type of every C and D of the set,
 * GG_OUTPUT_F32 (0, the reference's), GG_OUTPUT_F16 or GG_OUTPUT_BF16. The accumulation and the
 * epilogue arithmetic stay FP32; D is rounded to nearest even once, at the store.
 * activation (no reference counterpart): applied to every element of D after the bias,
 *   D = act(alpha * A x B + beta * C + bias):
 *   GG_ACT_NONE (0), GG_ACT_RELU (max(x, 0)), GG_ACT_GELU (tanh form,
 *   0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3))), the approximation of Hendrycks and Gimpel).
 * a_layout / b_layout (no reference counterpart, whose operands are row-major): GG_LAYOUT_ROW_MAJOR
 *   (0: A is m x k with row pitch lda >= k, B is k x n with ldb >= n) or GG_LAYOUT_COL_MAJOR
 *   (A stored as its transpose, k x m with lda >= m; B stored as n x k with ldb >= k, the layout of
 *   a [out_features][in_features] weight). The tensor cores read either form directly (K-major or
 *   MN-major shared-memory operands). With 8-bit inputs a column-major A needs 128-row tiles
 *   per CTA (not 64x128), and a column-major B lifts the 128-column rule. The mixture-of-experts
 *   plan takes a row-major A only.
 * tile_classes (no reference counterpart, whose launch uses one tile shape): GG_TILE_CLASSES_NONE
 *   (0: every problem is tiled with the config's tile) or, with a CTA-pair config (256x128x64,
 *   256x256x64) on the tensor cores, GG_TILE_CLASSES_PAIR_BLOCKS: an executor cuts every problem
 *   into its whole 256-row blocks, computed by CTA pairs, and the rows left over (fewer than 256),
 *   computed by one-CTA tiles of 128 rows and the same width; the two launches of a run may
 *   overlap on the GPU (the second takes SMs as the first retires). Large problems get the pair
 *   tiles (half the B bytes per SM), and no pair tile is padded past a problem's last row. The
 *   prepared set, its tile offsets and the executor's problem_count / total_tiles keep the config's
 *   256-row tiling. GG_TILE_CLASSES_SMALL_ON_CUDA_CORES, with any tensor-core config: problems
 *   whose m, n and k are all at most GG_SMALL_PROBLEM_DIM, and problems of at most
 *   GG_SMALL_ZERO_FILL_VOLUME multiply-adds (m * n * k) whose A or B TMA cannot load (a row pitch
 *   or base not 16-byte aligned), run on the CUDA-core kernel with 64 x 64 tiles; the others on
 *   the tensor cores with the config's tile, where an A or B that TMA cannot load is copied by
 *   every run, before the tensor-core launch, into a scratch matrix with 16-byte-aligned rows
 *   that the executor allocates at build time (rows x the row's bytes rounded up to 16, per
 *   such operand) and loaded from there by TMA (D is bit-identical to the zero-fill loader's).
 *   The CUDA-core launch starts on the SMs the tensor-core launch leaves free. Measured on B200
 *   with L2 flushed before every run: 4096 problems of 1..64, 76 us against 241 us on the tensor
 *   cores; 64 problems of 65^3, 20 against 43 us, of 257^3, 136 against 227 us, and 512 of 385^3,
 *   2.5 against 3.8 ms (odd pitches), while with aligned pitches the tensor cores win from 96^3
 *   up. Executors only: the no-allocation entry point, the per-problem baseline and the
 *   mixture-of-experts plan run the config's tile and path everywhere.
 * Any other value of these fields is an invalid config. The C++ API of
 * grouped_gemm/grouped_gemm.cuh keeps the reference's KernelConfig and always passes 0 for all
 * of them. */
#define GG_INPUT_F16 0
#define GG_INPUT_BF16 1
#define GG_INPUT_E4M3 2
#define GG_INPUT_E5M2 3
#define GG_OUTPUT_F32 0
#define GG_OUTPUT_F16 1
#define GG_OUTPUT_BF16 2
#define GG_ACT_NONE 0
#define GG_ACT_RELU 1
#define GG_ACT_GELU 2
#define GG_LAYOUT_ROW_MAJOR 0
#define GG_LAYOUT_COL_MAJOR 1
#define GG_TILE_CLASSES_NONE 0
#define GG_TILE_CLASSES_PAIR_BLOCKS 1
#define GG_TILE_CLASSES_SMALL_ON_CUDA_CORES 2
#define GG_SMALL_PROBLEM_DIM 64
#define GG_SMALL_ZERO_FILL_VOLUME (1LL << 25)
typedef struct gg_config {
  int cta_m;
  int cta_n;
  int cta_k;
  int threads;
  int persistent_ctas; /* > 0: fixed persistent grid size; 0: one CTA per SM slot, capped by tiles */
  int use_tensor_cores;
  int input_type;      /* GG_INPUT_F16, GG_INPUT_BF16, GG_INPUT_E4M3 or GG_INPUT_E5M2 */
  int output_type;     /* GG_OUTPUT_F32, GG_OUTPUT_F16 or GG_OUTPUT_BF16 */
  int activation;      /* GG_ACT_NONE, GG_ACT_RELU or GG_ACT_GELU */
  int a_layout;        /* GG_LAYOUT_ROW_MAJOR or GG_LAYOUT_COL_MAJOR */
  int b_layout;        /* GG_LAYOUT_ROW_MAJOR or GG_LAYOUT_COL_MAJOR */
  int tile_classes;    /* GG_TILE_CLASSES_NONE, _PAIR_BLOCKS or _SMALL_ON_CUDA_CORES */
} gg_config;

/* Resource report; field-for-field the reference's OccupancyInfo (grouped_gemm.cuh:54-83). */
typedef struct gg_occupancy {
  int sm_count;
  int max_blocks_per_sm;
  int active_blocks_per_sm;
  int threads_per_block;
  int max_threads_per_sm;
  int warps_per_block;
  int max_warps_per_sm;
  int active_warps_per_sm;
  int max_registers_per_sm;
  int max_registers_per_block;
  int estimated_registers_per_thread;
  int estimated_registers_per_block;
  int registers_per_thread;
  int registers_per_block;
  int register_limited_blocks_per_sm;
  int static_shared_bytes;
  int dynamic_shared_bytes;
  float theoretical_occupancy;
  int using_tensor_cores;
} gg_occupancy;

/* A contiguous piece of one problem assigned to one GPU by gg_partition: rows
 * [row0, row0+rows) x columns [col0, col0+cols) of problem `problem` (index into the input). */
typedef struct gg_shard_piece {
  int problem;
  int row0;
  int rows;
  int col0;
  int cols;
} gg_shard_piece;

typedef struct gg_executor gg_executor;

int gg_abi_version(void);

/* reference src/grouped_gemm.cu:952-965 (sort_mode_name): "none", "sort_by_k", "sort_by_tiles",
 * "sort_by_tiles_then_k", or "unknown". */
const char* gg_sort_mode_name(int sort_mode);

/* reference src/grouped_gemm.cu:58-65 (tile_count_for_problem): 0 when m <= 0 or n <= 0,
 * else ceil(m/cta_m) * ceil(n/cta_n). K = 0 still owns tiles (D = beta*C there). */
int gg_tile_count(const gg_problem* problem, const gg_config* config);

/* reference src/grouped_gemm.cu:967-1022 (prepare_problem_set). Host only, no CUDA call.
 * Writes count entries to sorted_problems and sorted_to_original, count+1 to tile_offsets
 * (tile_offsets[0] = 0) and the total to *total_tiles. Bit-identical to the reference. */
int gg_prepare(const gg_problem* problems, int count, const gg_config* config, int sort_mode,
               gg_problem* sorted_problems, int* sorted_to_original, int* tile_offsets,
               int* total_tiles);

/* reference src/grouped_gemm.cu:1024-1083 (query_occupancy) for the kernel the config selects. */
int gg_query_occupancy(const gg_config* config, gg_occupancy* info);

/* reference src/grouped_gemm.cu:1099-1130 (GroupedGemmExecutor constructor / destructor). */
int gg_executor_create(gg_executor** out);
void gg_executor_destroy(gg_executor* executor);

/* reference src/grouped_gemm.cu:1132-1239 (GroupedGemmExecutor::build). Takes the fields of a
 * PreparedProblemSet: `count` sorted problems, `offsets_len` tile offsets (must be count+1) and
 * total_tiles (must equal the last offset). Validates, encodes per-problem TMA descriptors and
 * uploads the problem table; the device state is owned by the executor. */
int gg_executor_build(gg_executor* executor, const gg_problem* sorted_problems, int count,
                      const int* tile_offsets, int offsets_len, int total_tiles,
                      const gg_config* config);

/* No reference counterpart. gg_executor_build plus a per-column bias fused into the epilogue:
 * bias is a host array of `count` device pointers in the order of sorted_problems, entry i
 * pointing to n_i FP32 values (any alignment) added to every row of D_i before the activation;
 * a NULL entry means no bias for that problem, and bias == NULL is gg_executor_build. The
 * pointers are copied into the executor's device table; the values are read at run time. */
int gg_executor_build_with_bias(gg_executor* executor, const gg_problem* sorted_problems, int count,
                                const int* tile_offsets, int offsets_len, int total_tiles,
                                const gg_config* config, const float* const* bias);

/* reference src/grouped_gemm.cu:1241-1265 (GroupedGemmExecutor::run): launches the persistent
 * kernel on `stream` (with tile classes, its parts; see gg_executor_launches). The reference
 * resets the tile counter with a memset before every launch; here the last CTA of each launch
 * sets it back to zero for the next run, so a run is its kernel launches alone. Runs of one
 * executor on two streams at the same time race on its tile counter: use one executor per
 * concurrent stream. */
int gg_executor_run(const gg_executor* executor, void* stream);

/* reference src/grouped_gemm.cu:1267-1277 (problem_count / total_tiles / grid_ctas). */
int gg_executor_problem_count(const gg_executor* executor);
int gg_executor_total_tiles(const gg_executor* executor);
int gg_executor_grid_ctas(const gg_executor* executor);
/* No reference counterpart (its run is one launch). Kernel launches one gg_executor_run makes: 0
 * with nothing to compute, 1, or with tile classes one per non-empty part plus one for the
 * operand copies of the small-problem class. */
int gg_executor_launches(const gg_executor* executor);

/* No reference counterpart (the reference kernels cannot time out). Synchronises the device and
 * returns in *device_status the GG_STATUS_* bits raised by this executor's launches so far, then
 * clears them. */
int gg_executor_status(const gg_executor* executor, int* device_status);

/* reference src/grouped_gemm.cu:1279-1291 (run_grouped_gemm_once): prepare + build + run. Like
 * the reference, the temporary executor is freed before returning, which synchronises; before
 * that its status word is read, and a bounded wait that ran out inside the kernel returns
 * cudaErrorLaunchTimeout (702) instead of success. */
int gg_run_grouped_gemm_once(const gg_problem* problems, int count, int sort_mode,
                             const gg_config* config, void* stream);

/* reference src/grouped_gemm.cu:1293-1317 (run_baseline_per_problem): one kernel launch per
 * non-empty problem, in input order, on the same tile code. Asynchronous: the launches share one
 * status word per device, read with gg_baseline_status. */
int gg_run_baseline_per_problem(const gg_problem* problems, int count, const gg_config* config,
                                void* stream);

/* No reference counterpart (the reference kernels cannot time out). Synchronises the current
 * device and returns in *device_status the GG_STATUS_* bits raised by gg_run_baseline_per_problem
 * launches on it since the last query (0 when none ran), then clears them. */
int gg_baseline_status(int* device_status);

/* reference src/grouped_gemm.cu:1319-1329 (count_non_empty_problems). */
int gg_count_non_empty_problems(const gg_problem* problems, int count, const gg_config* config);

/* No reference counterpart (the reference is single-GPU). Splits the problem set over
 * world_size GPUs: every output tile of the config's tiling is weighted by its 64-deep K blocks
 * plus a fixed epilogue cost, tiles are numbered in input order (row-major inside a problem),
 * and each tile goes to the rank whose 1/world_size share of the total weight holds the tile's
 * midpoint. A rank therefore owns one contiguous tile range per problem, returned as at most
 * three rectangles (pieces). Writes the pieces of `rank` to out (at most capacity), their number
 * to *out_count and their weight to *out_weight (nullable). With out == NULL only the count is
 * returned. Host only. */
int gg_partition(const gg_problem* problems, int count, const gg_config* config, int world_size,
                 int rank, gg_shard_piece* out, int capacity, int* out_count, double* out_weight);

/* No reference counterpart. Runs the kernel's bounded-wait helper on an mbarrier that nothing
 * ever completes, with the given limit, and returns the device status it recorded in *status
 * (GG_STATUS_TIMEOUT_* expected). Shows that a stuck wait ends with an error code instead of a
 * hang and that the context stays usable. */
int gg_selftest_wait_timeout(unsigned long long timeout_ns, int* status);

/* No reference counterpart. The same self-test, recording into the status word that
 * gg_baseline_status (word GG_STATUS_WORD_BASELINE) or gg_noalloc_status (GG_STATUS_WORD_NOALLOC)
 * reads on the current device, so that a caller can check that a timeout on those paths reaches
 * the query. Synchronises. Unknown word -> cudaErrorInvalidValue. */
#define GG_STATUS_WORD_BASELINE 0
#define GG_STATUS_WORD_NOALLOC 1
int gg_selftest_wait_timeout_word(int word, unsigned long long timeout_ns);

/* No counterpart in the reference. The grouped GEMM of gg_run_grouped_gemm_once for callers that
 * cannot allocate device memory: code whose device memory is owned by a caching allocator or a
 * pool that forbids side allocations, latency-critical paths where cudaMalloc/cudaFree and the
 * synchronisation they imply are not acceptable, or processes that must not grow their device
 * footprint after start-up. It calls no cudaMalloc, cudaFree or other allocating routine, on
 * the device or the host: the problem table, TMA descriptors, tile offsets, tile counter and
 * status word live in one fixed device array of this library (616 KiB, held on every GPU that
 * loads the library until the process exits). The caller still provides A, B, C and D.
 *   - At most GG_NOALLOC_MAX_PROBLEMS problems; more returns cudaErrorMemoryAllocation (2) and
 *     launches nothing. Other errors as for gg_run_grouped_gemm_once.
 *   - The first call on a device looks up the array's device address (cudaGetSymbolAddress).
 *   - Every call uses the same array and it keeps the last call's contents (the tile counter
 *     and status word are cleared by each call). Calls whose work overlaps on the GPU -- on two
 *     streams, or from two host threads on different streams -- race on it: order them on one
 *     stream. Results match gg_run_grouped_gemm_once bit for bit. */
#define GG_NOALLOC_MAX_PROBLEMS 1024
int gg_run_grouped_gemm_noalloc(const gg_problem* problems, int count, int sort_mode,
                                const gg_config* config, void* stream);

/* No counterpart in the reference. Synchronises the current device and returns in *device_status
 * the GG_STATUS_* bits of the last gg_run_grouped_gemm_noalloc call on it (each call clears them
 * first; a bounded wait that ran out leaves D partly written), then clears them. Allocates nothing. */
int gg_noalloc_status(int* device_status);

/* ---- grouped GEMM with device-side preparation (mixture-of-experts routing) ----------------
 * No counterpart in the reference, whose problem set is prepared on the host. Here the number of
 * rows of every problem lives in device memory -- as in a mixture-of-experts layer, where a
 * router on the GPU decides how many tokens each expert gets -- and never travels to the host:
 * the problems share N and K, their rows are packed back to back in A, C and D (expert 0's rows,
 * then expert 1's, ...), and each has its own B. gg_moe_plan_create does the host work once per
 * layer (tensor maps of the packed A and D and of every B, the device tables); gg_moe_plan_run
 * launches a one-block preparation kernel that reads the row counts, prefix-sums rows and tiles,
 * writes the problem records and tile offsets, and then the persistent grouped kernel, which reads
 * the tile count from the device. No host synchronisation, no host copy per run, so a run can be
 * captured in a CUDA graph and replayed with new row counts. */
typedef struct gg_moe_problem {
  const void* a;          /* FP16 (config input_type), capacity_rows x k, row pitch lda: the problems' rows packed */
  const void* const* b;   /* host array of `experts` device pointers, each k x n FP16, row pitch ldb */
  const void* c;          /* optional FP32 (config output_type), packed like A, row pitch ldc (read when beta != 0) */
  void* d;                /* FP32 (config output_type), packed like A, row pitch ldd */
  int experts;            /* problems, >= 1 */
  int n;                  /* columns of every B and D, >= 0 */
  int k;                  /* inner dimension, >= 0 */
  int capacity_rows;      /* rows allocated in A, C and D; the row counts of a run must sum to at most this */
  int lda;
  int ldb;
  int ldc;
  int ldd;
  float alpha;
  float beta;
  const float* const* bias; /* optional host array of `experts` device pointers, each n FP32 values
                               added to every row of that expert's D (NULL entries: none); NULL: no bias */
} gg_moe_problem;

typedef struct gg_moe_plan gg_moe_plan;

/* Status bit set by gg_moe_plan_run's preparation when a row count is negative or their sum
 * exceeds capacity_rows; that run computes nothing. */
#define GG_STATUS_BAD_ROWS 0x100

/* Builds the plan (allocates its device tables, encodes the tensor maps). Errors: invalid config,
 * experts < 1, negative n/k/capacity, null a/b/d or a null B pointer -> cudaErrorInvalidValue
 * (checked before any device work); CUDA errors passed through. */
int gg_moe_plan_create(const gg_moe_problem* problem, const gg_config* config, gg_moe_plan** out);
/* rows: `experts` ints in device memory. Enqueues preparation + grouped kernel on `stream`. */
int gg_moe_plan_run(gg_moe_plan* plan, const int* rows, void* stream);
/* Synchronises, returns (then clears) the GG_STATUS_* bits of the plan's runs, and the tile count
 * of the last run in *total_tiles (nullable). */
int gg_moe_plan_status(gg_moe_plan* plan, int* status, int* total_tiles);
void gg_moe_plan_destroy(gg_moe_plan* plan);

/* ---- grouped GEMM prepared on the device ----------------------------------------------------
 * No counterpart in the reference, whose problem set is prepared on the host
 * (src/grouped_gemm.cu:967-1022 prepare_problem_set, 1132-1239 build). Here the problem
 * descriptors themselves -- an array of gg_problem -- and their count are in device memory (written
 * by an earlier kernel: a planner or router on the GPU) and never travel to the host. A run
 * enqueues a one-block preparation kernel, which checks the problems (the checks of
 * gg_executor_build, and that lda >= k, ldb >= n, ldd >= n and, when C is read, ldc >= n; a failure
 * computes nothing and raises GG_STATUS_BAD_PROBLEMS), orders them by
 * the sort mode's rules (the same stable order as gg_prepare), prefix-sums their tiles and writes
 * the problem records, and then the persistent grouped kernel. No host synchronisation, no host
 * copy per run: a run can be captured in a CUDA graph and replayed over new problems. The problems
 * get no TMA descriptors (those are encoded on the host): A and B rows that start 16-byte aligned
 * (base and pitch in bytes multiples of 16) load by 16-byte cp.async into the same swizzled stages,
 * other A and B by the zero-fill loader; D takes the masked stores. Both take fewer bytes per cycle
 * than TMA.
 * Configs: one-CTA tiles (not the CTA-pair shapes), row-major A and B, no tile classes; any input
 * and output type, activation, and the CUDA-core path. D must be this GPU's memory. */
#define GG_DEVICE_PLAN_MAX_PROBLEMS 4096
#define GG_STATUS_BAD_PROBLEMS 0x200
typedef struct gg_device_plan gg_device_plan;
/* Allocates the plan's device tables for up to max_problems (1..GG_DEVICE_PLAN_MAX_PROBLEMS)
 * problems and encodes its descriptor templates. Invalid config or size -> cudaErrorInvalidValue. */
int gg_device_plan_create(const gg_config* config, int max_problems, gg_device_plan** out);
/* problems: device array of gg_problem (device pointers inside); count: device int, at most the
 * plan's max_problems (else GG_STATUS_BAD_PROBLEMS); sort_mode: GG_SORT_*. Enqueues on `stream`.
 * Runs of one plan on two streams at once race on its tables. */
int gg_device_plan_run(gg_device_plan* plan, const gg_problem* problems, const int* count, int sort_mode,
                       void* stream);
/* Synchronises; returns (then clears) the GG_STATUS_* bits of the plan's runs and the tile count
 * of the last run (nullable). */
int gg_device_plan_status(gg_device_plan* plan, int* status, int* total_tiles);
/* Synchronises; copies the last run's sorted-to-original order (capacity entries, -1 past the
 * count) and tile offsets (capacity + 1 entries) to the host: what gg_prepare returns for the same
 * problems and sort mode. */
int gg_device_plan_prepared(gg_device_plan* plan, int* sorted_to_original, int* tile_offsets, int capacity);
void gg_device_plan_destroy(gg_device_plan* plan);

/* No counterpart in the reference (which is single-GPU). One FP32 rectangle of a strided
 * row-major matrix and its place in a packed buffer, for gg_copy_rects. */
typedef struct gg_rect_copy {
  float* strided;      /* first element of the rectangle in its matrix (device memory) */
  long long packed;    /* element offset of the rectangle in the packed buffer */
  int rows;            /* rectangle rows */
  int cols;            /* rectangle columns */
  int ld;              /* row pitch of the strided matrix, elements (>= cols) */
  int reserved;
} gg_rect_copy;

/* No reference counterpart. Copies `count` FP32 rectangles between strided matrices and one packed
 * buffer in a single kernel launch on `stream`: to_packed != 0 packs (strided -> packed, row-major,
 * each rectangle at its `packed` offset), to_packed == 0 unpacks (packed -> strided). `rects` is an
 * array of gg_rect_copy in DEVICE memory. Used by the optional multi-GPU gather of D (pack before
 * the send, unpack after the receive). count == 0 launches nothing; count < 0, a null packed or
 * rects pointer with count > 0 return cudaErrorInvalidValue. */
int gg_copy_rects(float* packed, const gg_rect_copy* rects, int count, int to_packed, void* stream);

/* ---- device memory shared between processes (the gather fused into the kernel) ---------------
 * No reference counterpart. A multi-GPU run that wants every D on one root GPU can skip the
 * separate gather: the root exports its D buffer, every other rank opens it and builds its
 * executor with d pointers (and ldd) into the root's matrices, so that the grouped kernel's
 * epilogue stores each D tile straight into the root's memory over NVLink while later tiles are
 * still computing. A D that lies on another GPU is always written with plain coalesced stores (the
 * kernel's direct-store path), never with TMA. The handle is CUDA IPC: the exporting allocation
 * must be cudaMalloc memory (the PyTorch caching allocator's default), and the handle is valid
 * only on the same node while the allocation lives. */
typedef struct gg_ipc_handle {
  unsigned char handle[64];   /* cudaIpcMemHandle_t of the allocation that holds the pointer */
  unsigned long long offset;  /* byte offset of the pointer in that allocation */
  unsigned long long bytes;   /* bytes of the allocation from the pointer on */
} gg_ipc_handle;

/* Fills *out for device pointer ptr (current device). cudaErrorInvalidValue for a null pointer or
 * argument; CUDA errors pass through. */
int gg_ipc_export(const void* ptr, gg_ipc_handle* out);
/* Maps an exported allocation into this process (peer access enabled lazily) and returns the
 * pointer that corresponds to the exported one. Opening a handle of this very process fails
 * (CUDA IPC is between processes). */
int gg_ipc_open(const gg_ipc_handle* handle, void** ptr);
/* Unmaps what gg_ipc_open mapped; ptr is the pointer it returned. */
int gg_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* GROUPED_GEMM_B200_H_ */
