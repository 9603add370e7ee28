// gg_host.cu -- host runtime of the B200 grouped GEMM and its C-ABI (grouped_gemm_b200.h):
// problem-set preparation, per-problem TMA descriptor encoding, the executor that owns the
// device problem table, the per-problem baseline, the occupancy report and the multi-GPU
// partitioner. The C++ API (grouped_gemm_api.cpp) is a wrapper over these entry points.
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <numeric>
#include <vector>

#include "gg_internal.h"
#include "grouped_gemm_b200.h"

using grouped_gemm::DeviceProblemDesc;

namespace gg {
namespace {

static_assert(sizeof(gg_problem) == 72, "gg_problem mirrors grouped_gemm::ProblemDesc");
static_assert(offsetof(gg_problem, a) == 16 && offsetof(gg_problem, lda) == 48 && offsetof(gg_problem, alpha) == 64,
              "gg_problem field offsets");

constexpr int kMaxDevices = 64;
constexpr int kDefaultRasterGroup = 16;

int ceil_div(int x, int y) { return (x + y - 1) / y; }

// ---- environment knobs -------------------------------------------------------------------------
unsigned long long wait_timeout_ns() {
  static const unsigned long long v = [] {
    const char* s = std::getenv("GG_WAIT_TIMEOUT_MS");
    const long long ms = s ? std::atoll(s) : 2000;
    return static_cast<unsigned long long>(ms > 0 ? ms : 2000) * 1000000ull;
  }();
  return v;
}

int raster_group() {
  static const int v = [] {
    const char* s = std::getenv("GG_RASTER_GROUP");
    const int g = s ? std::atoi(s) : kDefaultRasterGroup;
    return g > 0 ? g : kDefaultRasterGroup;
  }();
  return v;
}

// ---- tile counting and sorting (reference src/grouped_gemm.cu:54-65, 967-1022) -----------------
int tile_count(int m, int n, int cta_m, int cta_n) {
  if (m <= 0 || n <= 0) return 0;
  return ceil_div(m, cta_m) * ceil_div(n, cta_n);
}

// True when problem x is ordered strictly before problem y under the by-K rule: larger K first,
// equal K -> larger m*n first (64-bit product).
bool k_rule_before(const gg_problem& x, const gg_problem& y) {
  if (x.k != y.k) return x.k > y.k;
  return static_cast<int64_t>(x.m) * x.n > static_cast<int64_t>(y.m) * y.n;
}

void sorted_order(const gg_problem* ps, int count, int cta_m, int cta_n, int mode, std::vector<int>& order) {
  order.resize(static_cast<size_t>(count));
  std::iota(order.begin(), order.end(), 0);
  if (mode == GG_SORT_BY_K) {
    std::stable_sort(order.begin(), order.end(),
                     [ps](int x, int y) { return k_rule_before(ps[x], ps[y]); });
  } else if (mode == GG_SORT_BY_TILES || mode == GG_SORT_BY_TILES_THEN_K) {
    // by-tiles and by-tiles-then-K share one rule: more tiles first, ties by the K rule.
    std::vector<int> tiles(static_cast<size_t>(count));
    for (int i = 0; i < count; ++i) tiles[static_cast<size_t>(i)] = tile_count(ps[i].m, ps[i].n, cta_m, cta_n);
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
      const int tx = tiles[static_cast<size_t>(x)], ty = tiles[static_cast<size_t>(y)];
      if (tx != ty) return tx > ty;
      return k_rule_before(ps[x], ps[y]);
    });
  }
}

// ---- TMA descriptor encoding ----------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuTensorMapEncodeTiled_v12000>(nullptr);
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
  }();
  return fn;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 2-D row-major tensor (inner x outer elements, row pitch in bytes), swizzled boxes (128-byte
// swizzle unless given).
bool encode_2d(CUtensorMap* map, CUtensorMapDataType type, const void* base, int inner, int outer,
               int64_t row_bytes, int box_inner, int box_outer,
               CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc || inner <= 0 || outer <= 0 || row_bytes <= 0 || (row_bytes % 16) != 0 || !aligned16(base)) return false;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(inner), static_cast<cuuint64_t>(outer)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(box_inner), static_cast<cuuint32_t>(box_outer)};
  const cuuint32_t elem_strides[2] = {1, 1};
  const CUresult r = enc(map, type, 2, const_cast<void*>(base), dims, strides, box, elem_strides,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// False when p is device memory of another GPU (a peer buffer mapped into this process, e.g. the
// root's D of a gather fused into the kernel): such a D is written with plain stores, never TMA.
// A pointer whose device cannot be queried counts as another GPU's too (plain stores are correct
// for any device memory; a TMA store is not). The last allocation range looked up is cached, so a
// problem set whose D matrices share one buffer costs one query; opening or closing an IPC
// mapping invalidates the cache, since a mapping can reuse the addresses of a freed buffer.
bool on_this_device(const void* p) {
  static thread_local uintptr_t lo = 0, hi = 0;
  static thread_local int cached_dev = -1;
  static thread_local bool cached_local = false;
  static thread_local unsigned cached_gen = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;  // unknown: plain stores are correct for any device memory
  }
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  // A mapping opened or closed since the range was cached may reuse its addresses: look again.
  const unsigned gen = ipc_mapping_generation();
  if (dev == cached_dev && gen == cached_gen && a >= lo && a < hi) return cached_local;
  cudaPointerAttributes attr{};
  if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
    (void)cudaGetLastError();
    return false;
  }
  const bool local = !(attr.type == cudaMemoryTypeDevice && attr.device != dev);
  static PFN_cuMemGetAddressRange_v3020 range = [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return static_cast<PFN_cuMemGetAddressRange_v3020>(nullptr);
    return reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  }();
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range && range(&base, &size, static_cast<CUdeviceptr>(a)) == CUDA_SUCCESS) {
    lo = static_cast<uintptr_t>(base);
    hi = lo + size;
    cached_dev = dev;
    cached_local = local;
    cached_gen = gen;
  }
  return local;
}

// Bytes of one C or D element in output format `fmt` (GG_OUTPUT_*).
int out_bytes(int fmt) { return fmt == GG_OUTPUT_F32 ? 4 : 2; }

bool aligned8(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 7u) == 0; }

// The D store map: 32 columns x 32 rows per box, in the staging layout of the epilogue (128-byte
// rows with the 128-byte swizzle for FP32, 64-byte rows with the 64-byte swizzle for 16-bit D).
bool encode_d(CUtensorMap* map, int fmt, const void* base, int n, int rows, int ldd) {
  const CUtensorMapDataType t = fmt == GG_OUTPUT_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                : fmt == GG_OUTPUT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  return encode_2d(map, t, base, n, rows, static_cast<int64_t>(ldd) * out_bytes(fmt), 32, 32,
                   fmt == GG_OUTPUT_F32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
}

// Vector-access flags of C and D in format fmt: C read 16 bytes at a time (so 16-bit C needs
// rows a multiple of 8 elements apart), D written 4 elements at a time.
unsigned vector_flags(int fmt, const void* c, int ldc, const void* d, int ldd) {
  unsigned f = 0;
  if (aligned16(c) && (ldc % (fmt == GG_OUTPUT_F32 ? 4 : 8)) == 0) f |= grouped_gemm::kFlagCVec;
  if ((fmt == GG_OUTPUT_F32 ? aligned16(d) : aligned8(d)) && (ldd % 4) == 0) f |= grouped_gemm::kFlagDVec;
  return f;
}

// Operand geometry of an input type: a 128-byte swizzle row holds 64 16-bit or 128 8-bit values,
// so a K block is 64 or 128 deep and a B chunk 64 or 128 columns wide.
struct InGeom {
  bool f8;
  int bytes;        // per element
  int kblock;       // K elements per pipeline stage
  int chunk;        // B columns per shared-memory chunk
  CUtensorMapDataType type;
};

InGeom in_geom(int in_fmt) {
  const bool f8 = in_fmt == GG_INPUT_E4M3 || in_fmt == GG_INPUT_E5M2;
  return f8 ? InGeom{true, 1, 2 * kBK, 128, CU_TENSOR_MAP_DATA_TYPE_UINT8}
            : InGeom{false, 2, kBK, 64, CU_TENSOR_MAP_DATA_TYPE_FLOAT16};
}

// B (k x n, row pitch ldb) seen as g.chunk columns x k rows x (n / g.chunk) full column chunks, the
// chunk dimension 128 bytes apart: one box {chunk, kblock, chunks} fills a whole B stage in the
// layout the MMA reads (chunk-major, 8 or 16 KB per chunk). Only full chunks are mapped, so no box
// can read past a row end; tiles that reach past the last full chunk use the 2-D map instead.
bool encode_b_chunks(CUtensorMap* map, const InGeom& g, const void* base, int k, int n, int64_t row_bytes,
                     int chunks_per_box) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  const int full_chunks = n / g.chunk;
  if (!enc || k <= 0 || full_chunks <= 0 || chunks_per_box <= 0 || row_bytes <= 0 || (row_bytes % 16) != 0 ||
      !aligned16(base))
    return false;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(g.chunk), static_cast<cuuint64_t>(k),
                              static_cast<cuuint64_t>(full_chunks)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes), 128};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(g.chunk), static_cast<cuuint32_t>(g.kblock),
                             static_cast<cuuint32_t>(chunks_per_box)};
  const cuuint32_t elem_strides[3] = {1, 1, 1};
  const CUresult r = enc(map, g.type, 3, const_cast<void*>(base), dims, strides, box, elem_strides,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Device record of one problem plus its kMapsPerProblem tensor maps. TMA is used for A/B only
// when both operands qualify, for D when it qualifies; everything else takes the zero-fill load
// path and masked direct stores.
DeviceProblemDesc make_device_problem(const gg_problem& p, Variant v, const gg_config* cfg, CUtensorMap* maps,
                                      int map_slot) {
  const InGeom g = in_geom(cfg->input_type);
  const int out_fmt = cfg->output_type;
  const bool a_col = cfg->a_layout == GG_LAYOUT_COL_MAJOR, b_col = cfg->b_layout == GG_LAYOUT_COL_MAJOR;
  const int bm = variant_bm(v), bn = variant_bn(v);
  const int cta_rows = variant_cta_rows(v);  // A and D rows one CTA moves per tile
  const int cta_cols = variant_cta_cols(v);  // B columns one CTA loads per tile
  DeviceProblemDesc d{};
  d.m = p.m;
  d.n = p.n;
  d.k = p.k;
  d.a = static_cast<const __half*>(p.a);
  d.b = static_cast<const __half*>(p.b);
  d.c = p.c;
  d.d = p.d;
  d.lda = p.lda;
  d.ldb = p.ldb;
  d.ldc = p.ldc;
  d.ldd = p.ldd;
  d.alpha = p.alpha;
  d.beta = p.beta;
  d.map_slot = map_slot;
  const bool has_tiles = p.m > 0 && p.n > 0;
  d.tiles_m = has_tiles ? ceil_div(p.m, bm) : 0;
  d.tiles_n = has_tiles ? ceil_div(p.n, bn) : 0;
  d.k_blocks = p.k > 0 ? ceil_div(p.k, g.kblock) : 0;
  unsigned flags = 0;
  std::memset(maps, 0, kMapsPerProblem * sizeof(CUtensorMap));
  // A row-major: boxes of kblock K x cta_rows rows; column-major (k x m): chunk M x kblock K per
  // box. B row-major: chunk N x kblock K per box (+ the 3-D whole-stage map); column-major (n x k):
  // kblock K x cta_cols rows, the whole stage in one box.
  const int64_t a_pitch = static_cast<int64_t>(p.lda) * g.bytes, b_pitch = static_cast<int64_t>(p.ldb) * g.bytes;
  const bool a_ok = a_col ? encode_2d(&maps[kMapA], g.type, p.a, p.m, p.k, a_pitch, g.chunk, g.kblock)
                          : encode_2d(&maps[kMapA], g.type, p.a, p.k, p.m, a_pitch, g.kblock, cta_rows);
  if (has_tiles && p.k > 0 && a_ok &&
      (b_col ? encode_2d(&maps[kMapB], g.type, p.b, p.k, p.n, b_pitch, g.kblock, cta_cols)
             : encode_2d(&maps[kMapB], g.type, p.b, p.n, p.k, b_pitch, g.chunk, g.kblock))) {
    flags |= grouped_gemm::kFlagTmaAB;
    if (!b_col && encode_b_chunks(&maps[kMapB3], g, p.b, p.k, p.n, b_pitch, cta_cols / g.chunk))
      flags |= grouped_gemm::kFlagTmaB3;
  }
  if (has_tiles && on_this_device(p.d) && encode_d(&maps[kMapD], out_fmt, p.d, p.n, p.m, p.ldd))
    flags |= grouped_gemm::kFlagTmaD;
  if (p.c != nullptr && p.beta != 0.0f) flags |= grouped_gemm::kFlagReadC;
  flags |= vector_flags(out_fmt, p.c, p.ldc, p.d, p.ldd);
  d.flags = flags;
  return d;
}

// Per-device status word for launches that have no executor (the per-problem baseline).
// create = false: the word if it exists, else null (nothing was launched on the device yet).
int* device_status_word(bool create = true) {
  static std::mutex mu;
  static int* words[kMaxDevices] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!words[dev] && create) {
    int* w = nullptr;
    if (cudaMalloc(&w, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(w, 0, sizeof(int)) != cudaSuccess) {
      cudaFree(w);
      return nullptr;
    }
    words[dev] = w;
  }
  return words[dev];
}

// Persistent grid: whole CTA pairs for pair variants, at most one tile per CTA (pair) and at
// most what fits on the device at once; persistent_ctas > 0 overrides (rounded up to whole pairs).
cudaError_t persistent_grid(Variant v, int total_tiles, int persistent_ctas, int* grid) {
  const int per_tile = variant_ctas_per_tile(v);
  if (persistent_ctas > 0) {
    *grid = (persistent_ctas + per_tile - 1) / per_tile * per_tile;
    return cudaSuccess;
  }
  int resident = 0;
  const cudaError_t st = kernel_resident_ctas(v, &resident);
  if (st != cudaSuccess) return st;
  const int units = std::max(1, std::min(resident / per_tile, total_tiles));
  *grid = units * per_tile;
  return cudaSuccess;
}

// Grid and launch of the path a config selects: the tcgen05 kernel, or the CUDA-core kernel when
// use_tensor_cores is 0 (persistent either way: at most one tile per CTA, at most what fits).
cudaError_t path_grid(bool tc, Variant v, int total_tiles, int persistent_ctas, int* grid) {
  if (tc) return persistent_grid(v, total_tiles, persistent_ctas, grid);
  if (persistent_ctas > 0) {
    *grid = persistent_ctas;
    return cudaSuccess;
  }
  int resident = 0;
  const cudaError_t st = simt_resident_ctas(&resident);
  if (st != cudaSuccess) return st;
  *grid = std::max(1, std::min(resident, total_tiles));
  return cudaSuccess;
}

cudaError_t launch_path(bool tc, Variant v, const KernelParams& kp, int grid, cudaStream_t s) {
  return tc ? launch_grouped_kernel(v, kp, grid, s) : launch_simt_kernel(v, kp, grid, s);
}

Variant variant_of(const gg_config* c) {
  if (!c || c->input_type < GG_INPUT_F16 || c->input_type > GG_INPUT_E5M2) return Variant::kUnsupported;
  if (c->output_type != GG_OUTPUT_F32 && c->output_type != GG_OUTPUT_F16 && c->output_type != GG_OUTPUT_BF16)
    return Variant::kUnsupported;
  if (c->activation != GG_ACT_NONE && c->activation != GG_ACT_RELU && c->activation != GG_ACT_GELU)
    return Variant::kUnsupported;
  const auto layout_ok = [](int l) { return l == GG_LAYOUT_ROW_MAJOR || l == GG_LAYOUT_COL_MAJOR; };
  if (!layout_ok(c->a_layout) || !layout_ok(c->b_layout)) return Variant::kUnsupported;
  const Variant v = resolve_variant(c->cta_m, c->cta_n, c->cta_k, c->threads);
  // Tile classes: CTA-pair blocks and one-CTA rows (pair configs on the tensor cores), or the
  // small problems of a tensor-core config on the CUDA cores.
  if (c->tile_classes != GG_TILE_CLASSES_NONE &&
      !(c->tile_classes == GG_TILE_CLASSES_PAIR_BLOCKS && c->use_tensor_cores && variant_is_pair(v)) &&
      !(c->tile_classes == GG_TILE_CLASSES_SMALL_ON_CUDA_CORES && c->use_tensor_cores))
    return Variant::kUnsupported;
  // 8-bit MN-major operands fill 128-wide chunks: on the tensor cores a row-major B needs per-CTA
  // B widths of 128 or 256, a column-major A 128 rows per CTA.
  if (v != Variant::kUnsupported && c->use_tensor_cores && in_geom(c->input_type).f8 &&
      ((c->b_layout == GG_LAYOUT_ROW_MAJOR && variant_cta_cols(v) % 128 != 0) ||
       (c->a_layout == GG_LAYOUT_COL_MAJOR && variant_cta_rows(v) % 128 != 0)))
    return Variant::kUnsupported;
  return v;
}

// The data-type and epilogue fields of a launch, from a validated config.
void set_formats(KernelParams& kp, const gg_config* c) {
  kp.input_format = c->input_type;
  kp.output_format = c->output_type;
  kp.activation = c->activation;
  kp.layout = (c->a_layout == GG_LAYOUT_COL_MAJOR ? 1 : 0) | (c->b_layout == GG_LAYOUT_COL_MAJOR ? 2 : 0);
}

size_t round_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Waits for the device, copies the status word to *bits and clears it. A null word reads as 0.
cudaError_t take_status(int* word, int* bits) {
  *bits = 0;
  if (!word) return cudaSuccess;
  cudaError_t st = cudaDeviceSynchronize();
  if (st != cudaSuccess) return st;
  st = cudaMemcpy(bits, word, sizeof(int), cudaMemcpyDeviceToHost);
  if (st != cudaSuccess) return st;
  return cudaMemset(word, 0, sizeof(int));
}

}  // namespace
}  // namespace gg

// ---- the executor ------------------------------------------------------------------------------
namespace gg {
namespace {

// One launch of an executor: a kernel variant over its own table of problems.
struct Part {
  Variant variant = Variant::kUnsupported;
  bool use_tc = true;
  int problem_count = 0;
  int total_tiles = 0;
  int grid = 0;
  KernelParams params{};
};

// Host image of one part's device tables before upload: per problem its tensor maps and record,
// the tile offsets, and (when a bias is given) one bias pointer per problem.
struct PartImage {
  Variant variant = Variant::kUnsupported;
  std::vector<CUtensorMap> maps;
  std::vector<DeviceProblemDesc> descs;
  std::vector<int> offsets;
  std::vector<const float*> bias;
};

// A problem's rows [row0, row0 + rows) as a problem of its own: A, C and D advanced by row0 rows
// (A stored column-major: by row0 columns of its k x m storage).
gg_problem row_slice(const gg_problem& p, int row0, int rows, const gg_config* c) {
  gg_problem q = p;
  q.m = rows;
  const int64_t in_b = in_geom(c->input_type).bytes, out_b = out_bytes(c->output_type);
  const int64_t a_step = c->a_layout == GG_LAYOUT_COL_MAJOR ? in_b : static_cast<int64_t>(p.lda) * in_b;
  q.a = static_cast<const char*>(p.a) + row0 * a_step;
  if (p.c) q.c = static_cast<const char*>(p.c) + static_cast<int64_t>(row0) * p.ldc * out_b;
  q.d = static_cast<char*>(p.d) + static_cast<int64_t>(row0) * p.ldd * out_b;
  return q;
}

// Appends problem p (bias `bias`, nullable) to the part's image.
void add_problem(PartImage& img, const gg_problem& p, const gg_config* c, const float* bias) {
  const int slot = static_cast<int>(img.descs.size());
  img.maps.resize(img.maps.size() + kMapsPerProblem);
  img.descs.push_back(make_device_problem(p, img.variant, c, &img.maps[static_cast<size_t>(slot) * kMapsPerProblem], slot));
  if (img.offsets.empty()) img.offsets.push_back(0);
  img.offsets.push_back(img.offsets.back() + tile_count(p.m, p.n, variant_bm(img.variant), variant_bn(img.variant)));
  img.bias.push_back(bias);
}

}  // namespace
}  // namespace gg

struct gg_executor {
  void* block = nullptr;  // one device allocation: every part's maps | problems | offsets | bias table,
                          // then the tile counters (one per part) and the status word
  int* d_counters = nullptr;
  int* d_status = nullptr;
  int parts = 0;          // launches per run: 1, or 2 with tile classes (CTA pairs, then one-CTA tiles)
  gg::Part part[2];
  int problem_count = 0;  // the prepared set's figures, as the reference reports them
  int total_tiles = 0;
  int grid_ctas = 0;
  gg::Variant variant = gg::Variant::kUnsupported;
  bool use_tc = true;  // tcgen05 kernel; false: the CUDA-core kernel
  void* realign_scratch = nullptr;     // 16-byte-aligned copies of operands TMA cannot load
  const gg::RealignJob* d_jobs = nullptr;  // in `block`: the copies each run makes first
  int realign_jobs = 0;
  long long realign_max_units = 0;  // most 16-byte chunks of one copy

  void release() {
    if (block) cudaFree(block);
    if (realign_scratch) cudaFree(realign_scratch);
    block = nullptr;
    realign_scratch = nullptr;
    d_jobs = nullptr;
    realign_jobs = 0;
    realign_max_units = 0;
    d_counters = nullptr;
    d_status = nullptr;
    parts = 0;
  }
};

extern "C" {

int gg_abi_version(void) { return GG_ABI_VERSION; }

const char* gg_sort_mode_name(int sort_mode) {
  switch (sort_mode) {
    case GG_SORT_NONE:
      return "none";
    case GG_SORT_BY_K:
      return "sort_by_k";
    case GG_SORT_BY_TILES:
      return "sort_by_tiles";
    case GG_SORT_BY_TILES_THEN_K:
      return "sort_by_tiles_then_k";
    default:
      return "unknown";
  }
}

int gg_tile_count(const gg_problem* problem, const gg_config* config) {
  if (!problem || !config || config->cta_m <= 0 || config->cta_n <= 0) return 0;
  return gg::tile_count(problem->m, problem->n, config->cta_m, config->cta_n);
}

int gg_prepare(const gg_problem* problems, int count, const gg_config* config, int sort_mode,
               gg_problem* sorted_problems, int* sorted_to_original, int* tile_offsets, int* total_tiles) {
  if (count < 0 || !config || !tile_offsets || !total_tiles || config->cta_m <= 0 || config->cta_n <= 0)
    return cudaErrorInvalidValue;
  if (count > 0 && (!problems || !sorted_problems || !sorted_to_original)) return cudaErrorInvalidValue;
  std::vector<int> order;
  gg::sorted_order(problems, count, config->cta_m, config->cta_n, sort_mode, order);
  tile_offsets[0] = 0;
  for (int s = 0; s < count; ++s) {
    const int o = order[static_cast<size_t>(s)];
    sorted_to_original[s] = o;
    sorted_problems[s] = problems[o];
    tile_offsets[s + 1] = tile_offsets[s] + gg::tile_count(problems[o].m, problems[o].n, config->cta_m, config->cta_n);
  }
  *total_tiles = tile_offsets[count];
  return cudaSuccess;
}

int gg_query_occupancy(const gg_config* config, gg_occupancy* info) {
  if (!info) return cudaErrorInvalidValue;
  const gg::Variant v = gg::variant_of(config);
  if (v == gg::Variant::kUnsupported) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  auto attr = [&](cudaDeviceAttr a) {
    int x = 0;
    if (st == cudaSuccess) st = cudaDeviceGetAttribute(&x, a, dev);
    return x;
  };
  gg_occupancy o{};
  o.sm_count = attr(cudaDevAttrMultiProcessorCount);
  o.max_blocks_per_sm = attr(cudaDevAttrMaxBlocksPerMultiprocessor);
  o.max_threads_per_sm = attr(cudaDevAttrMaxThreadsPerMultiProcessor);
  const int warp_size = attr(cudaDevAttrWarpSize);
  o.max_registers_per_sm = attr(cudaDevAttrMaxRegistersPerMultiprocessor);
  o.max_registers_per_block = attr(cudaDevAttrMaxRegistersPerBlock);
  if (st != cudaSuccess) return st;
  const bool tc = config->use_tensor_cores != 0;
  const int threads = tc ? gg::kThreads : gg::simt_threads();
  o.threads_per_block = threads;
  o.warps_per_block = threads / (warp_size > 0 ? warp_size : 32);
  o.max_warps_per_sm = o.max_threads_per_sm / (warp_size > 0 ? warp_size : 32);
  // Register model of the widest role, an epilogue thread: one 32-column TMEM chunk (32), the
  // matching C values (32) and ~24 for addresses, flags and loop state.
  // (CUDA-core path: a 4 x 4 FP32 accumulator block (16), its 8 operands and ~24.)
  o.estimated_registers_per_thread = tc ? 32 + 32 + 24 : 16 + 8 + 24;
  o.estimated_registers_per_block = o.estimated_registers_per_thread * threads;
  o.dynamic_shared_bytes = tc ? gg::variant_dynamic_smem(v) : 0;
  o.using_tensor_cores = tc ? 1 : 0;
  cudaFuncAttributes fa{};
  st = tc ? gg::kernel_occupancy(v, &o.active_blocks_per_sm, &fa) : gg::simt_occupancy(&o.active_blocks_per_sm, &fa);
  if (st != cudaSuccess) return st;
  o.registers_per_thread = fa.numRegs;
  o.static_shared_bytes = static_cast<int>(fa.sharedSizeBytes);
  o.registers_per_block = o.registers_per_thread * o.threads_per_block;
  o.register_limited_blocks_per_sm =
      o.registers_per_block > 0 ? std::min(o.max_blocks_per_sm, o.max_registers_per_sm / o.registers_per_block)
                                : o.max_blocks_per_sm;
  o.active_warps_per_sm = o.active_blocks_per_sm * o.warps_per_block;
  o.theoretical_occupancy =
      o.max_warps_per_sm > 0 ? static_cast<float>(o.active_warps_per_sm) / static_cast<float>(o.max_warps_per_sm) : 0.0f;
  *info = o;
  return cudaSuccess;
}

int gg_executor_create(gg_executor** out) {
  if (!out) return cudaErrorInvalidValue;
  *out = new (std::nothrow) gg_executor();
  return *out ? cudaSuccess : cudaErrorMemoryAllocation;
}

void gg_executor_destroy(gg_executor* executor) {
  if (!executor) return;
  executor->release();
  delete executor;
}

int gg_executor_build(gg_executor* ex, const gg_problem* sorted_problems, int count, const int* tile_offsets,
                      int offsets_len, int total_tiles, const gg_config* config) {
  return gg_executor_build_with_bias(ex, sorted_problems, count, tile_offsets, offsets_len, total_tiles, config,
                                     nullptr);
}

int gg_executor_build_with_bias(gg_executor* ex, const gg_problem* sorted_problems, int count,
                                const int* tile_offsets, int offsets_len, int total_tiles, const gg_config* config,
                                const float* const* bias) {
  if (!ex) return cudaErrorInvalidDevicePointer;
  const gg::Variant v = gg::variant_of(config);
  if (v == gg::Variant::kUnsupported) return cudaErrorInvalidValue;
  if (count < 0 || offsets_len != count + 1) return cudaErrorInvalidValue;
  if (offsets_len > 0 && (!tile_offsets || tile_offsets[offsets_len - 1] != total_tiles)) return cudaErrorInvalidValue;
  if (count > 0 && !sorted_problems) return cudaErrorInvalidValue;

  ex->release();
  ex->problem_count = 0;
  ex->total_tiles = 0;
  ex->grid_ctas = 0;
  ex->variant = v;
  ex->use_tc = config->use_tensor_cores != 0;

  for (int i = 0; i < count; ++i) {
    const gg_problem& p = sorted_problems[i];
    if (p.m < 0 || p.n < 0 || p.k < 0) return cudaErrorInvalidValue;
    if (!p.a || !p.b || !p.d) return cudaErrorInvalidDevicePointer;
  }
  if (count == 0 || total_tiles <= 0) {
    ex->problem_count = count;
    ex->total_tiles = total_tiles > 0 ? total_tiles : 0;
    return cudaSuccess;  // nothing to launch
  }

  // The parts: one variant over the prepared set as given; or, with tile classes, either the small
  // problems on the CUDA cores and the rest on the tensor cores, or the whole 256-row blocks of
  // every problem on CTA pairs and the rows left over (fewer than 256, on one-CTA 128-row tiles of
  // the same width); each part in the prepared order.
  gg::PartImage img[2];
  bool part_tc[2] = {ex->use_tc, ex->use_tc};
  int parts = 1;
  std::vector<gg::RealignJob> jobs;
  if (config->tile_classes == GG_TILE_CLASSES_SMALL_ON_CUDA_CORES) {
    // On the CUDA-core kernel, with its own 64 x 64 tiles (several CTAs per SM hide the latency of
    // short problems): problems no larger than GG_SMALL_PROBLEM_DIM in m, n and k, and problems of
    // at most GG_SMALL_ZERO_FILL_VOLUME multiply-adds whose A or B TMA cannot load (the tensor
    // cores would fill their stages with the zero-fill loader). The others on the tensor cores;
    // of those, an A or B that TMA cannot load (base or row pitch not 16-byte aligned) is copied
    // by every run into a scratch matrix with 16-byte-aligned rows, which the tensor cores load
    // by TMA (one HBM-bound copy instead of the zero-fill loader).
    parts = 2;
    img[0].variant = v;
    img[1].variant = gg::Variant::k64x64;
    part_tc[1] = false;
    CUtensorMap scratch[gg::kMapsPerProblem];
    const int eb = gg::in_geom(config->input_type).bytes;
    const bool a_col = config->a_layout == GG_LAYOUT_COL_MAJOR, b_col = config->b_layout == GG_LAYOUT_COL_MAJOR;
    // An operand the realignment can copy: fewer than 2^31 16-byte chunks (32 GB).
    auto tma_ok = [&](const void* base, int ld) {
      return gg::aligned16(base) && (static_cast<long long>(ld) * eb) % 16 == 0;
    };
    auto copyable = [&](int rows, int cols) {
      return static_cast<long long>(rows) * ((static_cast<long long>(cols) * eb + 15) / 16) < (1LL << 31);
    };
    std::vector<int> klass(count, 0);  // 0 tensor cores, 1 CUDA cores, 2 tensor cores on realigned copies
    size_t scratch_bytes = 0;
    for (int i = 0; i < count; ++i) {
      const gg_problem& p = sorted_problems[i];
      const bool has_work = p.m > 0 && p.n > 0 && p.k > 0;
      bool small = p.m <= GG_SMALL_PROBLEM_DIM && p.n <= GG_SMALL_PROBLEM_DIM && p.k <= GG_SMALL_PROBLEM_DIM;
      if (!small && has_work && static_cast<long long>(p.m) * p.n * p.k <= GG_SMALL_ZERO_FILL_VOLUME) {
        const DeviceProblemDesc d = gg::make_device_problem(p, v, config, scratch, 0);
        small = (d.flags & grouped_gemm::kFlagTmaAB) == 0u;
      }
      if (small) {
        klass[i] = 1;
        continue;
      }
      if (!has_work || (tma_ok(p.a, p.lda) && tma_ok(p.b, p.ldb))) continue;
      if (!copyable(a_col ? p.k : p.m, a_col ? p.m : p.k) || !copyable(b_col ? p.n : p.k, b_col ? p.k : p.n)) continue;
      klass[i] = 2;
      if (!tma_ok(p.a, p.lda)) {
        const long long row_bytes = static_cast<long long>(a_col ? p.m : p.k) * eb;
        scratch_bytes += gg::round_up(static_cast<size_t>((a_col ? p.k : p.m) * gg::round_up(row_bytes, 16)), 256);
      }
      if (!tma_ok(p.b, p.ldb)) {
        const long long row_bytes = static_cast<long long>(b_col ? p.k : p.n) * eb;
        scratch_bytes += gg::round_up(static_cast<size_t>((b_col ? p.n : p.k) * gg::round_up(row_bytes, 16)), 256);
      }
    }
    if (scratch_bytes > 0) {
      const cudaError_t st = cudaMalloc(&ex->realign_scratch, scratch_bytes);
      if (st != cudaSuccess) {
        ex->realign_scratch = nullptr;
        return st;
      }
    }
    unsigned char* next = static_cast<unsigned char*>(ex->realign_scratch);
    // One operand into the scratch: returns its copy and sets the copy's pitch in elements.
    auto realign = [&](const void* src, int ld, int rows, int cols, int* new_ld) -> const void* {
      const long long row_bytes = static_cast<long long>(cols) * eb;
      const long long pitch = static_cast<long long>(gg::round_up(static_cast<size_t>(row_bytes), 16));
      gg::RealignJob j{};
      j.src = static_cast<const unsigned char*>(src);
      j.dst = next;
      j.src_pitch = static_cast<long long>(ld) * eb;
      j.dst_pitch = pitch;
      j.rows = rows;
      j.row_bytes = static_cast<int>(row_bytes);
      jobs.push_back(j);
      next += gg::round_up(static_cast<size_t>(rows * pitch), 256);
      *new_ld = static_cast<int>(pitch / eb);
      return j.dst;
    };
    for (int i = 0; i < count; ++i) {
      gg_problem p = sorted_problems[i];
      if (klass[i] == 2) {
        if (!tma_ok(p.a, p.lda)) p.a = realign(p.a, p.lda, a_col ? p.k : p.m, a_col ? p.m : p.k, &p.lda);
        if (!tma_ok(p.b, p.ldb)) p.b = realign(p.b, p.ldb, b_col ? p.n : p.k, b_col ? p.k : p.n, &p.ldb);
      }
      gg::add_problem(img[klass[i] == 1 ? 1 : 0], p, config, bias ? bias[i] : nullptr);
    }
  } else if (config->tile_classes == GG_TILE_CLASSES_PAIR_BLOCKS) {
    parts = 2;
    img[0].variant = v;
    img[1].variant = gg::variant_bn(v) == 256 ? gg::Variant::k128x256 : gg::Variant::k128x128;
    for (int i = 0; i < count; ++i) {
      const gg_problem& p = sorted_problems[i];
      if (gg::tile_count(p.m, p.n, 256, gg::variant_bn(v)) == 0) continue;
      const int blocks = p.m / 256 * 256;
      const float* b = bias ? bias[i] : nullptr;
      if (blocks > 0) gg::add_problem(img[0], gg::row_slice(p, 0, blocks, config), config, b);
      if (p.m > blocks) gg::add_problem(img[1], gg::row_slice(p, blocks, p.m - blocks, config), config, b);
    }
  } else {
    img[0].variant = v;
    for (int i = 0; i < count; ++i) gg::add_problem(img[0], sorted_problems[i], config, bias ? bias[i] : nullptr);
    img[0].offsets.assign(tile_offsets, tile_offsets + offsets_len);  // the prepared offsets, as given
  }

  // Device layout: per part [maps | records | offsets | bias table], then counters and status.
  struct Off {
    size_t maps, descs, offs, bias;
  } off[2]{};
  size_t bytes = 0;
  for (int j = 0; j < parts; ++j) {
    const gg::PartImage& im = img[j];
    off[j].maps = gg::round_up(bytes, 128);
    off[j].descs = gg::round_up(off[j].maps + im.maps.size() * sizeof(CUtensorMap), 128);
    off[j].offs = gg::round_up(off[j].descs + im.descs.size() * sizeof(DeviceProblemDesc), 128);
    off[j].bias = gg::round_up(off[j].offs + im.offsets.size() * sizeof(int), 128);
    bytes = off[j].bias + (bias ? im.bias.size() * sizeof(const float*) : 0);
  }
  const size_t counter_off = gg::round_up(bytes, 128);
  bytes = counter_off + 128;  // tile counters at +0 (one int per part), finished-CTA counts at +8,
                             // status word at +64; zero in the image, and every launch leaves them
                             // zero for the next run
  const size_t jobs_off = bytes;
  bytes += jobs.size() * sizeof(gg::RealignJob);
  std::vector<unsigned char> image(bytes, 0);
  if (!jobs.empty()) std::memcpy(image.data() + jobs_off, jobs.data(), jobs.size() * sizeof(gg::RealignJob));
  for (int j = 0; j < parts; ++j) {
    const gg::PartImage& im = img[j];
    if (!im.maps.empty()) std::memcpy(image.data() + off[j].maps, im.maps.data(), im.maps.size() * sizeof(CUtensorMap));
    if (!im.descs.empty())
      std::memcpy(image.data() + off[j].descs, im.descs.data(), im.descs.size() * sizeof(DeviceProblemDesc));
    if (!im.offsets.empty()) std::memcpy(image.data() + off[j].offs, im.offsets.data(), im.offsets.size() * sizeof(int));
    if (bias && !im.bias.empty())
      std::memcpy(image.data() + off[j].bias, im.bias.data(), im.bias.size() * sizeof(const float*));
  }

  gg::Part part[2];
  for (int j = 0; j < parts; ++j) {
    gg::Part& pt = part[j];
    pt.variant = img[j].variant;
    pt.use_tc = part_tc[j];
    pt.problem_count = static_cast<int>(img[j].descs.size());
    pt.total_tiles = img[j].offsets.empty() ? 0 : img[j].offsets.back();
    if (pt.total_tiles > 0) {
      const cudaError_t st = gg::path_grid(pt.use_tc, pt.variant, pt.total_tiles, config->persistent_ctas, &pt.grid);
      if (st != cudaSuccess) return st;
    }
  }

  cudaError_t st = cudaMalloc(&ex->block, bytes);
  if (st != cudaSuccess) {
    ex->block = nullptr;
    ex->release();
    return st;
  }
  st = cudaMemcpy(ex->block, image.data(), bytes, cudaMemcpyHostToDevice);
  if (st != cudaSuccess) {
    ex->release();
    return st;
  }
  unsigned char* base = static_cast<unsigned char*>(ex->block);
  ex->d_counters = reinterpret_cast<int*>(base + counter_off);
  ex->d_status = reinterpret_cast<int*>(base + counter_off + 64);
  ex->d_jobs = reinterpret_cast<const gg::RealignJob*>(base + jobs_off);
  ex->realign_jobs = static_cast<int>(jobs.size());
  for (const gg::RealignJob& j : jobs)
    ex->realign_max_units = std::max(ex->realign_max_units, static_cast<long long>(j.rows) * ((j.row_bytes + 15) / 16));
  for (int j = 0; j < parts; ++j) {
    gg::KernelParams& kp = part[j].params;
    std::memset(&kp, 0, sizeof(kp));
    kp.problems = reinterpret_cast<const DeviceProblemDesc*>(base + off[j].descs);
    kp.tmaps = reinterpret_cast<const CUtensorMap*>(base + off[j].maps);
    kp.tile_offsets = reinterpret_cast<const int*>(base + off[j].offs);
    kp.tile_counter = ex->d_counters + j;
    kp.done_counter = ex->d_counters + 2 + j;  // the kernel clears both for the next run
    kp.status = ex->d_status;
    kp.timeout_ns = gg::wait_timeout_ns();
    kp.problem_count = part[j].problem_count;
    kp.total_tiles = part[j].total_tiles;
    kp.raster_group = gg::raster_group();
    kp.single_mode = 0;
    gg::set_formats(kp, config);
    kp.bias = bias ? reinterpret_cast<const float* const*>(base + off[j].bias) : nullptr;
    ex->part[j] = part[j];
  }
  ex->parts = parts;
  ex->problem_count = count;
  ex->total_tiles = total_tiles;
  ex->grid_ctas = part[0].grid > 0 ? part[0].grid : part[1].grid;
  return cudaSuccess;
}

int gg_executor_run(const gg_executor* ex, void* stream) {
  if (!ex) return cudaErrorInvalidDevicePointer;
  if (ex->total_tiles == 0 || ex->problem_count == 0) return cudaSuccess;
  if (!ex->block) return cudaErrorInvalidDevicePointer;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // No counter reset here: the last CTA of each launch clears its part's counters (finish_launch).
  // this run's copies of the operands TMA cannot load, before the tensor-core part reads them
  cudaError_t st = gg::launch_realign(ex->d_jobs, ex->realign_jobs, ex->realign_max_units, s);
  if (st != cudaSuccess) return st;
  bool after_tc = false;  // a tensor-core part was launched before this one
  for (int j = 0; j < ex->parts; ++j) {
    const gg::Part& pt = ex->part[j];
    if (pt.total_tiles <= 0) continue;
    // The second part of a tile-class split (one-CTA rows after the pair blocks, or the small
    // problems on the CUDA cores) may start on the SMs the first part leaves free: the parts write
    // disjoint outputs and count tiles on their own counters.
    if (after_tc)
      st = pt.use_tc ? gg::launch_grouped_kernel(pt.variant, pt.params, pt.grid, s, true)
                     : gg::launch_simt_kernel(pt.variant, pt.params, pt.grid, s, true);
    else
      st = gg::launch_path(pt.use_tc, pt.variant, pt.params, pt.grid, s);
    if (st != cudaSuccess) return st;
    after_tc = pt.use_tc;
  }
  return cudaSuccess;
}

int gg_executor_problem_count(const gg_executor* ex) { return ex ? ex->problem_count : 0; }
int gg_executor_total_tiles(const gg_executor* ex) { return ex ? ex->total_tiles : 0; }
int gg_executor_grid_ctas(const gg_executor* ex) { return ex ? ex->grid_ctas : 0; }
int gg_executor_launches(const gg_executor* ex) {
  if (!ex || !ex->block || ex->total_tiles == 0 || ex->problem_count == 0) return 0;
  int n = ex->realign_jobs > 0 ? 1 : 0;
  for (int j = 0; j < ex->parts; ++j) n += ex->part[j].total_tiles > 0 ? 1 : 0;
  return n;
}

int gg_executor_status(const gg_executor* ex, int* device_status) {
  if (!ex) return cudaErrorInvalidDevicePointer;
  if (!device_status) return cudaErrorInvalidValue;
  return gg::take_status(ex->d_status, device_status);
}

int gg_run_grouped_gemm_once(const gg_problem* problems, int count, int sort_mode, const gg_config* config,
                             void* stream) {
  if (count < 0 || (count > 0 && !problems) || !config) return cudaErrorInvalidValue;
  std::vector<gg_problem> sorted(static_cast<size_t>(count > 0 ? count : 1));
  std::vector<int> s2o(sorted.size());
  std::vector<int> offs(static_cast<size_t>(count) + 1);
  int total = 0;
  int st = gg_prepare(problems, count, config, sort_mode, sorted.data(), s2o.data(), offs.data(), &total);
  if (st != cudaSuccess) return st;
  gg_executor ex;
  st = gg_executor_build(&ex, sorted.data(), count, offs.data(), count + 1, total, config);
  if (st == cudaSuccess) st = gg_executor_run(&ex, stream);
  // The call synchronises anyway (freeing the temporary state, as in the reference), so the
  // kernel's status word is read here: a bounded wait that ran out left D partly written, which
  // the caller learns as cudaErrorLaunchTimeout.
  if (st == cudaSuccess && ex.d_status) {
    int bits = 0;
    st = gg_executor_status(&ex, &bits);
    if (st == cudaSuccess && bits != 0) st = cudaErrorLaunchTimeout;
  }
  ex.release();
  return st;
}

int gg_run_baseline_per_problem(const gg_problem* problems, int count, const gg_config* config, void* stream) {
  const gg::Variant v = gg::variant_of(config);
  if (v == gg::Variant::kUnsupported) return cudaErrorInvalidValue;
  if (count < 0 || (count > 0 && !problems)) return cudaErrorInvalidValue;
  const int bm = gg::variant_bm(v), bn = gg::variant_bn(v);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = nullptr;
  gg::KernelParams kp;
  for (int i = 0; i < count; ++i) {
    const gg_problem& p = problems[i];
    // Checked problem by problem in input order, as the reference does (src/grouped_gemm.cu:1304-1313).
    if (!p.a || !p.b || !p.d) return cudaErrorInvalidDevicePointer;
    if (gg::tile_count(p.m, p.n, bm, bn) == 0) continue;
    if (!status) {
      status = gg::device_status_word();
      if (!status) return cudaErrorMemoryAllocation;
    }
    std::memset(&kp, 0, sizeof(kp));
    kp.single_desc = gg::make_device_problem(p, v, config, kp.single_maps, 0);
    const int tiles = kp.single_desc.tiles_m * kp.single_desc.tiles_n;
    kp.status = status;
    kp.timeout_ns = gg::wait_timeout_ns();
    kp.problem_count = 1;
    kp.total_tiles = tiles;
    kp.raster_group = gg::raster_group();
    kp.single_mode = 1;
    gg::set_formats(kp, config);
    int grid = 0;
    const bool tc = config->use_tensor_cores != 0;
    cudaError_t st = gg::path_grid(tc, v, tiles, 0, &grid);
    if (st != cudaSuccess) return st;
    st = gg::launch_path(tc, v, kp, grid, s);
    if (st != cudaSuccess) return st;
  }
  return cudaSuccess;
}

int gg_baseline_status(int* device_status) {
  if (!device_status) return cudaErrorInvalidValue;
  return gg::take_status(gg::device_status_word(false), device_status);
}

int gg_count_non_empty_problems(const gg_problem* problems, int count, const gg_config* config) {
  if (!problems || !config || count <= 0 || config->cta_m <= 0 || config->cta_n <= 0) return 0;
  int non_empty = 0;
  for (int i = 0; i < count; ++i)
    if (gg::tile_count(problems[i].m, problems[i].n, config->cta_m, config->cta_n) > 0) ++non_empty;
  return non_empty;
}

int gg_partition(const gg_problem* problems, int count, const gg_config* config, int world_size, int rank,
                 gg_shard_piece* out, int capacity, int* out_count, double* out_weight) {
  if (!config || !out_count || world_size < 1 || rank < 0 || rank >= world_size || count < 0 ||
      (count > 0 && !problems) || config->cta_m <= 0 || config->cta_n <= 0)
    return cudaErrorInvalidValue;
  const int cm = config->cta_m, cn = config->cta_n;
  // The epilogue of a tile writes cm*cn*4 bytes of D; a K block loads (cm+cn)*64*2 bytes. The
  // fixed per-tile cost is expressed in K-block units so that the weight tracks both.
  const double epi = std::max(1.0, (cm * cn * 4.0) / ((cm + cn) * gg::kBK * 2.0));
  std::vector<double> per_tile(static_cast<size_t>(count), 0.0);
  std::vector<int> tiles(static_cast<size_t>(count), 0);
  double total = 0.0;
  for (int i = 0; i < count; ++i) {
    const gg_problem& p = problems[i];
    tiles[static_cast<size_t>(i)] = gg::tile_count(p.m, p.n, cm, cn);
    per_tile[static_cast<size_t>(i)] = static_cast<double>(p.k > 0 ? gg::ceil_div(p.k, gg::kBK) : 0) + epi;
    total += per_tile[static_cast<size_t>(i)] * tiles[static_cast<size_t>(i)];
  }
  int n = 0;
  double weight = 0.0, cum = 0.0;
  auto emit = [&](int problem, int row0, int rows, int col0, int cols) {
    if (rows <= 0 || cols <= 0) return;
    if (out && n < capacity) out[n] = gg_shard_piece{problem, row0, rows, col0, cols};
    ++n;
  };
  for (int i = 0; i < count; ++i) {
    const int T = tiles[static_cast<size_t>(i)];
    const double w = per_tile[static_cast<size_t>(i)];
    if (T == 0) continue;
    // Tiles are taken in row-major order; each one goes to the rank whose share of the total
    // weight holds the tile's midpoint, so a rank owns one contiguous tile range per problem.
    int t0 = -1, t1 = -1;
    for (int t = 0; t < T; ++t) {
      const double mid = cum + (t + 0.5) * w;
      int owner = total > 0.0 ? static_cast<int>(std::floor(mid * world_size / total)) : 0;
      owner = std::min(std::max(owner, 0), world_size - 1);
      if (owner == rank) {
        if (t0 < 0) t0 = t;
        t1 = t + 1;
      }
    }
    cum += w * T;
    if (t0 < 0) continue;
    weight += w * (t1 - t0);
    // Cut the tile range [t0, t1) of the tm x tn tile grid into at most three rectangles: the
    // tail of the first row band, whole row bands, the head of the last row band.
    const gg_problem& p = problems[i];
    const int tn = gg::ceil_div(p.n, cn);
    auto col_end = [&](int c) { return std::min(p.n, c * cn); };
    auto row_end = [&](int r) { return std::min(p.m, r * cm); };
    int r_first = t0 / tn, c_first = t0 % tn;
    const int r_last = (t1 - 1) / tn, c_last = (t1 - 1) % tn;
    if (r_first == r_last) {
      emit(i, r_first * cm, row_end(r_first + 1) - r_first * cm, c_first * cn, col_end(c_last + 1) - c_first * cn);
      continue;
    }
    if (c_first != 0) {
      emit(i, r_first * cm, row_end(r_first + 1) - r_first * cm, c_first * cn, p.n - c_first * cn);
      ++r_first;
    }
    const int full_end = (c_last == tn - 1) ? r_last + 1 : r_last;  // bands [r_first, full_end) are whole
    if (full_end > r_first) emit(i, r_first * cm, row_end(full_end) - r_first * cm, 0, p.n);
    if (c_last != tn - 1) emit(i, r_last * cm, row_end(r_last + 1) - r_last * cm, 0, col_end(c_last + 1));
  }
  *out_count = n;
  if (out_weight) *out_weight = weight;
  if (out && n > capacity) return cudaErrorInvalidValue;
  return cudaSuccess;
}

int gg_selftest_wait_timeout(unsigned long long timeout_ns, int* status) {
  if (!status) return cudaErrorInvalidValue;
  int* d = nullptr;
  cudaError_t st = cudaMalloc(&d, sizeof(int));
  if (st != cudaSuccess) return st;
  st = cudaMemset(d, 0, sizeof(int));
  if (st == cudaSuccess) st = gg::launch_wait_selftest(d, timeout_ns, nullptr);
  if (st == cudaSuccess) st = cudaDeviceSynchronize();
  if (st == cudaSuccess) st = cudaMemcpy(status, d, sizeof(int), cudaMemcpyDeviceToHost);
  cudaFree(d);
  return st;
}

}  // extern "C"

// ---- grouped GEMM without any allocation ------------------------------------------------------
// For callers that cannot call cudaMalloc: code running under a caching allocator or a memory
// pool that owns the whole device and forbids side allocations, code on a latency-critical path
// where an allocation (and the synchronisation cudaFree implies) is not acceptable, or code that
// must not grow its memory footprint after start-up. Everything the persistent kernel needs
// besides the caller's A/B/C/D -- the problem table, the TMA descriptors, the tile offsets, the
// tile counter and the status word -- lives in one fixed file-scope device array, sized for at
// most GG_NOALLOC_MAX_PROBLEMS problems (616 KiB, held by every GPU that loads this library until
// the process exits). Host-side preparation uses fixed static buffers as well.
namespace gg {
namespace {

constexpr int kNoAllocMaxProblems = GG_NOALLOC_MAX_PROBLEMS;
constexpr size_t kNoAllocMapsBytes = static_cast<size_t>(kNoAllocMaxProblems) * kMapsPerProblem * sizeof(CUtensorMap);
constexpr size_t kNoAllocDescsOff = kNoAllocMapsBytes;
constexpr size_t kNoAllocOffsOff =
    (kNoAllocDescsOff + static_cast<size_t>(kNoAllocMaxProblems) * sizeof(DeviceProblemDesc) + 127) / 128 * 128;
constexpr size_t kNoAllocCounterOff =
    (kNoAllocOffsOff + static_cast<size_t>(kNoAllocMaxProblems + 1) * sizeof(int) + 127) / 128 * 128;
constexpr size_t kNoAllocBytes = (kNoAllocCounterOff + 128 + 4095) / 4096 * 4096;
static_assert(kNoAllocBytes == 616 * 1024, "the documented size of the no-allocation scratch");

// The scratch itself. Host code must never pass this name to a kernel: on the host it only
// names a stand-in, not device memory. Its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

std::mutex g_noalloc_mu;                           // guards the host staging buffers below
unsigned char g_noalloc_image[kNoAllocBytes];      // host image of the scratch, uploaded per call
int g_noalloc_order[kNoAllocMaxProblems];          // sorted_to_original
int g_noalloc_tmp[kNoAllocMaxProblems];            // merge-sort buffer
void* g_noalloc_dev_ptr[kMaxDevices] = {};         // device address of the scratch, per device

// Stable order of the problems for a sort mode: the reference's rule (src/grouped_gemm.cu:977-1005),
// applied with a bottom-up merge sort over fixed buffers (no heap use). On ties the element from
// the left run comes first, so equal keys keep their input order, as std::stable_sort does.
bool noalloc_before(const gg_problem* ps, int mode, int cta_m, int cta_n, int x, int y) {
  if (mode == GG_SORT_BY_TILES || mode == GG_SORT_BY_TILES_THEN_K) {
    const int tx = tile_count(ps[x].m, ps[x].n, cta_m, cta_n), ty = tile_count(ps[y].m, ps[y].n, cta_m, cta_n);
    if (tx != ty) return tx > ty;
  }
  return k_rule_before(ps[x], ps[y]);
}

void noalloc_sort(const gg_problem* ps, int count, int mode, int cta_m, int cta_n) {
  for (int i = 0; i < count; ++i) g_noalloc_order[i] = i;
  if (mode != GG_SORT_BY_K && mode != GG_SORT_BY_TILES && mode != GG_SORT_BY_TILES_THEN_K) return;
  int* src = g_noalloc_order;
  int* dst = g_noalloc_tmp;
  for (int width = 1; width < count; width *= 2) {
    for (int lo = 0; lo < count; lo += 2 * width) {
      const int mid = std::min(lo + width, count), hi = std::min(lo + 2 * width, count);
      int i = lo, j = mid, o = lo;
      while (i < mid && j < hi) dst[o++] = noalloc_before(ps, mode, cta_m, cta_n, src[j], src[i]) ? src[j++] : src[i++];
      while (i < mid) dst[o++] = src[i++];
      while (j < hi) dst[o++] = src[j++];
    }
    std::swap(src, dst);
  }
  if (src != g_noalloc_order) std::memcpy(g_noalloc_order, src, static_cast<size_t>(count) * sizeof(int));
}

// Device address of the scratch on the current device, looked up once per device.
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  if (!g_noalloc_dev_ptr[dev]) {
    void* p = nullptr;
    st = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (st != cudaSuccess) return st;
    g_noalloc_dev_ptr[dev] = p;
  }
  *out = g_noalloc_dev_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace gg

extern "C" int gg_run_grouped_gemm_noalloc(const gg_problem* problems, int count, int sort_mode,
                                           const gg_config* config, void* stream) {
  const gg::Variant v = gg::variant_of(config);
  if (v == gg::Variant::kUnsupported) return cudaErrorInvalidValue;
  if (count < 0 || (count > 0 && !problems)) return cudaErrorInvalidValue;
  if (count > gg::kNoAllocMaxProblems) return cudaErrorMemoryAllocation;  // does not fit the fixed scratch
  for (int i = 0; i < count; ++i) {
    if (problems[i].m < 0 || problems[i].n < 0 || problems[i].k < 0) return cudaErrorInvalidValue;
    if (!problems[i].a || !problems[i].b || !problems[i].d) return cudaErrorInvalidDevicePointer;
  }
  if (count == 0) return cudaSuccess;

  std::lock_guard<std::mutex> lock(gg::g_noalloc_mu);
  gg::noalloc_sort(problems, count, sort_mode, config->cta_m, config->cta_n);
  auto* maps = reinterpret_cast<CUtensorMap*>(gg::g_noalloc_image);
  auto* descs = reinterpret_cast<DeviceProblemDesc*>(gg::g_noalloc_image + gg::kNoAllocDescsOff);
  auto* offs = reinterpret_cast<int*>(gg::g_noalloc_image + gg::kNoAllocOffsOff);
  offs[0] = 0;
  for (int s = 0; s < count; ++s) {
    const gg_problem& p = problems[gg::g_noalloc_order[s]];
    offs[s + 1] = offs[s] + gg::tile_count(p.m, p.n, config->cta_m, config->cta_n);
    descs[s] = gg::make_device_problem(p, v, config, &maps[static_cast<size_t>(s) * gg::kMapsPerProblem], s);
  }
  const int total = offs[count];
  if (total == 0) return cudaSuccess;

  void* scratch = nullptr;
  cudaError_t st = gg::noalloc_scratch(&scratch);
  if (st != cudaSuccess) return st;
  int grid = 0;
  st = gg::path_grid(config->use_tensor_cores != 0, v, total, config->persistent_ctas, &grid);
  if (st != cudaSuccess) return st;

  cudaStream_t s = static_cast<cudaStream_t>(stream);
  unsigned char* dev = static_cast<unsigned char*>(scratch);
  // Only the used prefix of each region is uploaded. A pageable-source copy returns once the
  // host image has been staged, so the image can be refilled by the next call.
  st = cudaMemcpyAsync(dev, gg::g_noalloc_image, static_cast<size_t>(count) * gg::kMapsPerProblem * sizeof(CUtensorMap),
                       cudaMemcpyHostToDevice, s);
  if (st == cudaSuccess)
    st = cudaMemcpyAsync(dev + gg::kNoAllocDescsOff, gg::g_noalloc_image + gg::kNoAllocDescsOff,
                         static_cast<size_t>(count) * sizeof(DeviceProblemDesc), cudaMemcpyHostToDevice, s);
  if (st == cudaSuccess)
    st = cudaMemcpyAsync(dev + gg::kNoAllocOffsOff, gg::g_noalloc_image + gg::kNoAllocOffsOff,
                         static_cast<size_t>(count + 1) * sizeof(int), cudaMemcpyHostToDevice, s);
  // The tile counter and the status word must start at zero; the scratch keeps the last call's
  // contents otherwise.
  if (st == cudaSuccess) st = cudaMemsetAsync(dev + gg::kNoAllocCounterOff, 0, 2 * sizeof(int), s);
  if (st != cudaSuccess) return st;

  gg::KernelParams kp;
  std::memset(&kp, 0, sizeof(kp));
  kp.problems = reinterpret_cast<const DeviceProblemDesc*>(dev + gg::kNoAllocDescsOff);
  kp.tmaps = reinterpret_cast<const CUtensorMap*>(dev);
  kp.tile_offsets = reinterpret_cast<const int*>(dev + gg::kNoAllocOffsOff);
  kp.tile_counter = reinterpret_cast<int*>(dev + gg::kNoAllocCounterOff);
  kp.status = reinterpret_cast<int*>(dev + gg::kNoAllocCounterOff + sizeof(int));
  kp.timeout_ns = gg::wait_timeout_ns();
  kp.problem_count = count;
  kp.total_tiles = total;
  kp.raster_group = gg::raster_group();
  kp.single_mode = 0;
  gg::set_formats(kp, config);
  return gg::launch_path(config->use_tensor_cores != 0, v, kp, grid, s);
}

namespace gg {
namespace {
// The status word of the no-allocation entry point on the current device (in its fixed array).
cudaError_t noalloc_status_word(int** word) {
  void* scratch = nullptr;
  const cudaError_t st = noalloc_scratch(&scratch);
  if (st != cudaSuccess) return st;
  *word = reinterpret_cast<int*>(static_cast<unsigned char*>(scratch) + kNoAllocCounterOff + sizeof(int));
  return cudaSuccess;
}
}  // namespace
}  // namespace gg

extern "C" int gg_noalloc_status(int* device_status) {
  if (!device_status) return cudaErrorInvalidValue;
  *device_status = 0;
  int* word = nullptr;
  const cudaError_t st = gg::noalloc_status_word(&word);
  if (st != cudaSuccess) return st;
  return gg::take_status(word, device_status);
}

extern "C" int gg_selftest_wait_timeout_word(int word, unsigned long long timeout_ns) {
  int* target = nullptr;
  if (word == GG_STATUS_WORD_BASELINE) {
    target = gg::device_status_word();
    if (!target) return cudaErrorMemoryAllocation;
  } else if (word == GG_STATUS_WORD_NOALLOC) {
    const cudaError_t st = gg::noalloc_status_word(&target);
    if (st != cudaSuccess) return st;
  } else {
    return cudaErrorInvalidValue;
  }
  const cudaError_t st = gg::launch_wait_selftest(target, timeout_ns, nullptr);
  return st != cudaSuccess ? st : cudaDeviceSynchronize();
}

// ---- grouped GEMM with device-side preparation (mixture-of-experts routing) ---------------------
// The problems share N and K and their rows are packed back to back in A, C and D; only the row
// counts change from run to run, and they live on the device. Everything that does not depend on
// them is built once on the host: one tensor map of the packed A and one of the packed D (each
// spanning all capacity_rows rows; a problem addresses them from its first row, tma_row0), the B
// maps of every expert, and a template problem record per expert. A run is a one-block
// preparation kernel (prefix sums of rows and tiles, problem records, tile offsets, tile count,
// counter reset) followed by the persistent kernel, which reads the tile count from the device.
namespace gg {
namespace {

constexpr int kMoePrepThreads = 1024;

// Exclusive prefix sum of v over the block (kMoePrepThreads threads); *total gets the sum.
template <typename T>
__device__ T block_exclusive_scan(T v, T* warp_sums, T* total) {
  const int lane = static_cast<int>(threadIdx.x & 31), warp = static_cast<int>(threadIdx.x >> 5);
  T x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    T w = lane < kMoePrepThreads / 32 ? warp_sums[lane] : T(0);
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    if (lane < kMoePrepThreads / 32) warp_sums[lane] = w;  // inclusive sums of the warps
  }
  __syncthreads();
  const T before = warp > 0 ? warp_sums[warp - 1] : T(0);
  *total = warp_sums[kMoePrepThreads / 32 - 1];
  __syncthreads();  // warp_sums is reused by the next call
  return before + x - v;
}

// Problem record of expert e whose rows start at row0 of the packed tensors.
__device__ __forceinline__ DeviceProblemDesc moe_record(const DeviceProblemDesc* templ, int e, int r, long long row0,
                                                        int tm, int tiles_n, int t, int capacity, const char* a,
                                                        int lda, int a_eb, const void* c, int ldc, void* d, int ldd,
                                                        int eb) {
  DeviceProblemDesc p = templ[e];
  p.m = r;
  p.a = reinterpret_cast<const __half*>(a + row0 * lda * a_eb);
  p.c = c ? static_cast<const char*>(c) + row0 * ldc * eb : nullptr;
  p.d = static_cast<char*>(d) + row0 * ldd * eb;
  p.tiles_m = t > 0 ? tm : 0;
  p.tiles_n = t > 0 ? tiles_n : 0;
  p.tma_row0 = static_cast<int>(row0 < capacity ? row0 : capacity);
  return p;
}

// One block. Rows are packed in expert order, so the row offsets are a prefix sum in that order.
// With at most kMoePrepThreads experts the problems are then ordered by tile count, largest
// first (ties by expert index; the by-tiles rule of the host preparation), which shortens the
// tail of the persistent schedule; larger sets keep expert order.
__global__ void __launch_bounds__(kMoePrepThreads) moe_prepare_kernel(
    const int* __restrict__ rows, int experts, int capacity, int bm, int tiles_n,
    const DeviceProblemDesc* __restrict__ templ, DeviceProblemDesc* __restrict__ descs, int* __restrict__ offsets,
    int* total_tiles, int* counter, int* status, const char* a, int lda, int a_eb, const void* c, int ldc,
    void* d, int ldd, int eb) {
  __shared__ long long s_rows[kMoePrepThreads / 32];
  __shared__ int s_tiles[kMoePrepThreads / 32];
  __shared__ long long s_key[kMoePrepThreads];
  __shared__ long long s_row0[kMoePrepThreads];
  const int tid = static_cast<int>(threadIdx.x);
  long long row_carry = 0;
  int tile_carry = 0;
  int bad = 0;
  if (experts <= kMoePrepThreads) {
    const int e = tid;
    int r = e < experts ? rows[e] : 0;
    if (r < 0) {
      bad = 1;
      r = 0;
    }
    const int tm = r > 0 ? (r + bm - 1) / bm : 0;
    const int t = tiles_n > 0 ? tm * tiles_n : 0;
    long long rows_total;
    const long long row0 = block_exclusive_scan<long long>(r, s_rows, &rows_total);
    row_carry = rows_total;
    s_row0[tid] = row0;
    // descending sort key: tile count, then the lower expert index first; padding sorts last
    s_key[tid] = e < experts ? (static_cast<long long>(t) << 32) | (0xffffffffll - e) : -1ll;
    __syncthreads();
    for (int k2 = 2; k2 <= kMoePrepThreads; k2 <<= 1) {
      for (int j = k2 >> 1; j > 0; j >>= 1) {
        const int ixj = tid ^ j;
        if (ixj > tid) {
          const long long x = s_key[tid], y = s_key[ixj];
          const bool desc = (tid & k2) == 0;
          if (desc ? (x < y) : (x > y)) {
            s_key[tid] = y;
            s_key[ixj] = x;
          }
        }
        __syncthreads();
      }
    }
    const long long key = s_key[tid];
    const int se = key < 0 ? -1 : static_cast<int>(0xffffffffll - (key & 0xffffffffll));
    const int st = key < 0 ? 0 : static_cast<int>(key >> 32);
    int tiles_total;
    const int t0 = block_exclusive_scan<int>(st, s_tiles, &tiles_total);
    tile_carry = tiles_total;
    if (se >= 0) {
      const int sr = max(rows[se], 0);
      const int stm = sr > 0 ? (sr + bm - 1) / bm : 0;
      descs[tid] =
          moe_record(templ, se, sr, s_row0[se], stm, tiles_n, st, capacity, a, lda, a_eb, c, ldc, d, ldd, eb);
      offsets[tid] = t0;
    }
  } else {
    for (int base = 0; base < experts; base += kMoePrepThreads) {
      const int e = base + tid;
      int r = e < experts ? rows[e] : 0;
      if (r < 0) {
        bad = 1;
        r = 0;
      }
      const int tm = r > 0 ? (r + bm - 1) / bm : 0;
      const int t = tiles_n > 0 ? tm * tiles_n : 0;
      long long rows_total;
      int tiles_total;
      const long long row0 = row_carry + block_exclusive_scan<long long>(r, s_rows, &rows_total);
      const int t0 = tile_carry + block_exclusive_scan<int>(t, s_tiles, &tiles_total);
      if (e < experts) {
        descs[e] = moe_record(templ, e, r, row0, tm, tiles_n, t, capacity, a, lda, a_eb, c, ldc, d, ldd, eb);
        offsets[e] = t0;
      }
      row_carry += rows_total;
      tile_carry += tiles_total;
    }
  }
  bad = __syncthreads_or(bad);
  if (tid == 0) {
    offsets[experts] = tile_carry;
    const bool ok = !bad && row_carry <= static_cast<long long>(capacity);
    *total_tiles = ok ? tile_carry : 0;
    *counter = 0;
    if (!ok) atomicOr(status, GG_STATUS_BAD_ROWS);
  }
}

}  // namespace
}  // namespace gg

struct gg_moe_plan {
  void* block = nullptr;  // maps | template records | records | offsets | total, counter, status
  const DeviceProblemDesc* d_templ = nullptr;
  DeviceProblemDesc* d_descs = nullptr;
  int* d_offsets = nullptr;
  int* d_total = nullptr;
  int* d_counter = nullptr;
  int* d_status = nullptr;
  gg_moe_problem problem{};
  gg::Variant variant = gg::Variant::kUnsupported;
  bool use_tc = true;
  int grid_ctas = 0;
  int tiles_n = 0;
  int in_bytes = 2;   // bytes of an A / B element
  int out_bytes = 4;  // bytes of a C / D element
  gg::KernelParams params{};
};

extern "C" {

int gg_moe_plan_create(const gg_moe_problem* problem, const gg_config* config, gg_moe_plan** out) {
  if (!out) return cudaErrorInvalidValue;
  *out = nullptr;
  const gg::Variant v = gg::variant_of(config);
  if (!problem || v == gg::Variant::kUnsupported) return cudaErrorInvalidValue;
  const gg_moe_problem& q = *problem;
  if (q.experts < 1 || q.n < 0 || q.k < 0 || q.capacity_rows < 0 || !q.a || !q.b || !q.d) return cudaErrorInvalidValue;
  // The packed rows are rows of a row-major A; B may be either layout (column-major: n x k).
  if (config->a_layout != GG_LAYOUT_ROW_MAJOR) return cudaErrorInvalidValue;
  const bool b_col = config->b_layout == GG_LAYOUT_COL_MAJOR;
  if (q.lda < std::max(1, q.k) || q.ldb < std::max(1, b_col ? q.k : q.n) || q.ldd < std::max(1, q.n) ||
      (q.c && q.ldc < std::max(1, q.n)))
    return cudaErrorInvalidValue;
  for (int e = 0; e < q.experts; ++e)
    if (!q.b[e]) return cudaErrorInvalidValue;

  const int bn = gg::variant_bn(v);
  const int cta_rows = gg::variant_cta_rows(v), cta_cols = gg::variant_cta_cols(v);
  const size_t E = static_cast<size_t>(q.experts);
  std::vector<CUtensorMap> maps(E * gg::kMapsPerProblem);
  std::vector<DeviceProblemDesc> templ(E);
  std::memset(maps.data(), 0, maps.size() * sizeof(CUtensorMap));
  CUtensorMap map_a{}, map_d{};
  const bool rows_exist = q.capacity_rows > 0 && q.n > 0;
  const gg::InGeom g = gg::in_geom(config->input_type);
  const bool tma_a = rows_exist && q.k > 0 &&
                     gg::encode_2d(&map_a, g.type, q.a, q.k, q.capacity_rows, static_cast<int64_t>(q.lda) * g.bytes,
                                   g.kblock, cta_rows);
  const bool tma_d = rows_exist && gg::on_this_device(q.d) &&
                     gg::encode_d(&map_d, config->output_type, q.d, q.n, q.capacity_rows, q.ldd);
  for (size_t e = 0; e < E; ++e) {
    CUtensorMap* m = &maps[e * gg::kMapsPerProblem];
    DeviceProblemDesc& p = templ[e];
    p.m = 0;
    p.n = q.n;
    p.k = q.k;
    p.a = static_cast<const __half*>(q.a);
    p.b = static_cast<const __half*>(q.b[e]);
    p.c = q.c;
    p.d = q.d;
    p.lda = q.lda;
    p.ldb = q.ldb;
    p.ldc = q.ldc;
    p.ldd = q.ldd;
    p.alpha = q.alpha;
    p.beta = q.beta;
    p.k_blocks = q.k > 0 ? gg::ceil_div(q.k, g.kblock) : 0;
    p.map_slot = static_cast<int>(e);  // the maps stay in expert order; the records are reordered
    unsigned flags = grouped_gemm::kFlagPackedRows;
    const int64_t b_pitch = static_cast<int64_t>(q.ldb) * g.bytes;
    if (tma_a && (b_col ? gg::encode_2d(&m[gg::kMapB], g.type, q.b[e], q.k, q.n, b_pitch, g.kblock, cta_cols)
                        : gg::encode_2d(&m[gg::kMapB], g.type, q.b[e], q.n, q.k, b_pitch, g.chunk, g.kblock))) {
      m[gg::kMapA] = map_a;
      flags |= grouped_gemm::kFlagTmaAB;
      if (!b_col && gg::encode_b_chunks(&m[gg::kMapB3], g, q.b[e], q.k, q.n, b_pitch, cta_cols / g.chunk))
        flags |= grouped_gemm::kFlagTmaB3;
    }
    if (tma_d) {
      m[gg::kMapD] = map_d;
      flags |= grouped_gemm::kFlagTmaD;
    }
    if (q.c != nullptr && q.beta != 0.0f) flags |= grouped_gemm::kFlagReadC;
    flags |= gg::vector_flags(config->output_type, q.c, q.ldc, q.d, q.ldd);
    p.flags = flags;
  }

  int grid = 0;
  const bool use_tc = config->use_tensor_cores != 0;
  cudaError_t st = gg::path_grid(use_tc, v, 1 << 30, config->persistent_ctas, &grid);
  if (st != cudaSuccess) return st;

  const size_t maps_bytes = maps.size() * sizeof(CUtensorMap);
  const size_t templ_off = gg::round_up(maps_bytes, 128);
  const size_t descs_off = gg::round_up(templ_off + E * sizeof(DeviceProblemDesc), 128);
  const size_t offs_off = gg::round_up(descs_off + E * sizeof(DeviceProblemDesc), 128);
  const size_t words_off = gg::round_up(offs_off + (E + 1) * sizeof(int), 128);
  const size_t bias_off = words_off + 128;  // bias table (one pointer per expert), when given
  const size_t bytes = bias_off + (q.bias ? E * sizeof(const float*) : 0);
  std::vector<unsigned char> image(bytes, 0);
  std::memcpy(image.data(), maps.data(), maps_bytes);
  std::memcpy(image.data() + templ_off, templ.data(), E * sizeof(DeviceProblemDesc));
  if (q.bias) std::memcpy(image.data() + bias_off, q.bias, E * sizeof(const float*));

  gg_moe_plan* plan = new (std::nothrow) gg_moe_plan();
  if (!plan) return cudaErrorMemoryAllocation;
  st = cudaMalloc(&plan->block, bytes);
  if (st != cudaSuccess) {
    delete plan;
    return st;
  }
  st = cudaMemcpy(plan->block, image.data(), bytes, cudaMemcpyHostToDevice);
  if (st != cudaSuccess) {
    cudaFree(plan->block);
    delete plan;
    return st;
  }
  unsigned char* base = static_cast<unsigned char*>(plan->block);
  plan->d_templ = reinterpret_cast<const DeviceProblemDesc*>(base + templ_off);
  plan->d_descs = reinterpret_cast<DeviceProblemDesc*>(base + descs_off);
  plan->d_offsets = reinterpret_cast<int*>(base + offs_off);
  plan->d_total = reinterpret_cast<int*>(base + words_off);
  plan->d_counter = reinterpret_cast<int*>(base + words_off + 4);
  plan->d_status = reinterpret_cast<int*>(base + words_off + 8);
  plan->problem = q;
  plan->problem.b = nullptr;  // the host arrays are not kept
  plan->problem.bias = nullptr;
  plan->out_bytes = gg::out_bytes(config->output_type);
  plan->in_bytes = g.bytes;
  plan->variant = v;
  plan->use_tc = use_tc;
  plan->grid_ctas = grid;
  plan->tiles_n = q.n > 0 ? gg::ceil_div(q.n, bn) : 0;

  gg::KernelParams& kp = plan->params;
  std::memset(&kp, 0, sizeof(kp));
  kp.problems = plan->d_descs;
  kp.tmaps = reinterpret_cast<const CUtensorMap*>(base);
  kp.tile_offsets = plan->d_offsets;
  kp.tile_counter = plan->d_counter;
  kp.total_tiles_dev = plan->d_total;
  kp.status = plan->d_status;
  kp.timeout_ns = gg::wait_timeout_ns();
  kp.problem_count = q.experts;
  kp.total_tiles = 0;
  kp.raster_group = gg::raster_group();
  kp.single_mode = 0;
  gg::set_formats(kp, config);
  kp.bias = q.bias ? reinterpret_cast<const float* const*>(base + bias_off) : nullptr;
  *out = plan;
  return cudaSuccess;
}

int gg_moe_plan_run(gg_moe_plan* plan, const int* rows, void* stream) {
  if (!plan || !plan->block) return cudaErrorInvalidDevicePointer;
  if (!rows) return cudaErrorInvalidValue;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const gg_moe_problem& q = plan->problem;
  gg::moe_prepare_kernel<<<1, gg::kMoePrepThreads, 0, s>>>(
      rows, q.experts, q.capacity_rows, gg::variant_bm(plan->variant), plan->tiles_n, plan->d_templ, plan->d_descs,
      plan->d_offsets, plan->d_total, plan->d_counter, plan->d_status, static_cast<const char*>(q.a), q.lda, plan->in_bytes,
      q.c, q.ldc, q.d, q.ldd, plan->out_bytes);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return st;
  return gg::launch_path(plan->use_tc, plan->variant, plan->params, plan->grid_ctas, s);
}

int gg_moe_plan_status(gg_moe_plan* plan, int* status, int* total_tiles) {
  if (!plan || !plan->block) return cudaErrorInvalidDevicePointer;
  if (!status) return cudaErrorInvalidValue;
  cudaError_t st = cudaDeviceSynchronize();
  if (st != cudaSuccess) return st;
  int words[3] = {0, 0, 0};
  st = cudaMemcpy(words, plan->d_total, sizeof(words), cudaMemcpyDeviceToHost);
  if (st != cudaSuccess) return st;
  *status = words[2];
  if (total_tiles) *total_tiles = words[0];
  return cudaMemset(plan->d_status, 0, sizeof(int));
}

void gg_moe_plan_destroy(gg_moe_plan* plan) {
  if (!plan) return;
  if (plan->block) cudaFree(plan->block);
  delete plan;
}

}  // extern "C"

// ---- grouped GEMM prepared on the device (problem descriptors in device memory) ---------------
// The problem set itself -- dims, pointers, leading dimensions, alpha and beta of every problem --
// lives in device memory (written by an earlier kernel, e.g. a router or a planner on the GPU),
// and so does the problem count. A run is a one-block preparation kernel and the persistent grouped
// kernel: the preparation validates the problems, orders them by the reference's sort rules
// (stable; the same order prepare_problem_set gives on the host), prefix-sums their tile counts
// and writes the problem records. No host synchronisation and no host copy per run. The problems
// have no TMA descriptors (those are encoded on the host): their operands take the zero-fill
// loader and D the masked coalesced stores, which work for any pitch and alignment.
namespace gg {
namespace {

constexpr int kDevPlanMax = GG_DEVICE_PLAN_MAX_PROBLEMS;
constexpr int kDevPrepThreads = kMoePrepThreads;  // block_exclusive_scan's block size

// Tile geometry the preparation needs (from the plan's config).
struct DevGeom {
  int bm, bn;   // tile
  int kblock;   // K elements per pipeline stage (64 for 16-bit inputs, 128 for 8-bit)
  int in_b;     // bytes per A / B element
  int out_fmt;  // GG_OUTPUT_*: element type of C and D
};

int next_pow2(int x) {
  int p = 1;
  while (p < x) p <<= 1;
  return p;
}

size_t dev_prep_smem(int max_problems) {
  return static_cast<size_t>(next_pow2(max_problems)) * (sizeof(long long) + 3 * sizeof(int));
}

// True when problem x goes before problem y under sort mode `mode`: the reference's rules
// (src/grouped_gemm.cu:977-1005: K descending, ties by m*n descending; by tiles: tile count
// descending, ties by the K rule), ties by input index (a stable sort); -1 (padding) goes last.
__device__ __forceinline__ bool dev_before(int x, int y, int mode, const int* tiles, const int* ks,
                                           const long long* mns) {
  if (x < 0) return false;
  if (y < 0) return true;
  const bool by_tiles = mode == GG_SORT_BY_TILES || mode == GG_SORT_BY_TILES_THEN_K;
  if (by_tiles && tiles[x] != tiles[y]) return tiles[x] > tiles[y];
  if (by_tiles || mode == GG_SORT_BY_K) {
    if (ks[x] != ks[y]) return ks[x] > ks[y];
    if (mns[x] != mns[y]) return mns[x] > mns[y];
  }
  return x < y;
}

__device__ __forceinline__ bool dev_aligned(const void* p, unsigned a) {
  return (reinterpret_cast<uintptr_t>(p) & (a - 1u)) == 0;
}

// One block. descs: one record per sorted slot; offsets: max_problems + 1 prefix sums (flat past
// the count); order: the sorted-to-input index of every slot (-1 past the count).
__global__ void __launch_bounds__(kDevPrepThreads) device_prepare_kernel(
    const gg_problem* __restrict__ problems, const int* __restrict__ count_ptr, int max_problems, int p2, int mode,
    DevGeom g, DeviceProblemDesc* __restrict__ descs, int* __restrict__ offsets, int* __restrict__ order,
    int* total_tiles, int* counter, int* status) {
  extern __shared__ __align__(16) unsigned char dsm[];
  long long* s_mn = reinterpret_cast<long long*>(dsm);
  int* s_tiles = reinterpret_cast<int*>(s_mn + p2);
  int* s_k = s_tiles + p2;
  int* s_idx = s_k + p2;
  __shared__ int s_warp[kDevPrepThreads / 32];
  const int tid = static_cast<int>(threadIdx.x);

  int count = *count_ptr;
  int bad = count < 0 || count > max_problems;
  if (bad) count = 0;
  for (int i = tid; i < p2; i += kDevPrepThreads) {
    int t = 0, k = 0, idx = -1;
    long long mn = 0;
    if (i < count) {
      const gg_problem q = problems[i];
      // the checks of GroupedGemmExecutor::build (src/grouped_gemm.cu:1169-1174) and of the pitches
      if (q.m < 0 || q.n < 0 || q.k < 0 || !q.a || !q.b || !q.d || q.lda < max(1, q.k) || q.ldb < max(1, q.n) ||
          q.ldd < max(1, q.n) || (q.c && q.beta != 0.0f && q.ldc < max(1, q.n)))
        bad = 1;
      t = (q.m > 0 && q.n > 0) ? ((q.m + g.bm - 1) / g.bm) * ((q.n + g.bn - 1) / g.bn) : 0;
      k = q.k;
      mn = static_cast<long long>(q.m) * q.n;
      idx = i;
    }
    s_tiles[i] = t;
    s_k[i] = k;
    s_mn[i] = mn;
    s_idx[i] = idx;
  }
  bad = __syncthreads_or(bad);
  if (bad) {  // nothing runs: zero tiles
    if (tid == 0) {
      *total_tiles = 0;
      *counter = 0;
      atomicOr(status, GG_STATUS_BAD_PROBLEMS);
    }
    return;
  }

  // Bitonic sort of the input indices; the order is total (ties by index), so the result is the
  // stable order of the reference's rules.
  if (mode == GG_SORT_BY_K || mode == GG_SORT_BY_TILES || mode == GG_SORT_BY_TILES_THEN_K) {
    for (int k2 = 2; k2 <= p2; k2 <<= 1) {
      for (int j = k2 >> 1; j > 0; j >>= 1) {
        for (int i = tid; i < p2; i += kDevPrepThreads) {
          const int ixj = i ^ j;
          if (ixj > i) {
            const int x = s_idx[i], y = s_idx[ixj];
            const bool up = (i & k2) == 0;
            if (up ? dev_before(y, x, mode, s_tiles, s_k, s_mn) : dev_before(x, y, mode, s_tiles, s_k, s_mn)) {
              s_idx[i] = y;
              s_idx[ixj] = x;
            }
          }
        }
        __syncthreads();
      }
    }
  }

  // Tile offsets in sorted order (flat past the count) and the order itself.
  int carry = 0;
  for (int base = 0; base < max(p2, kDevPrepThreads); base += kDevPrepThreads) {
    const int s = base + tid;
    const int x = s < p2 ? s_idx[s] : -1;
    int total;
    const int excl = block_exclusive_scan<int>(x >= 0 ? s_tiles[x] : 0, s_warp, &total);
    if (s < max_problems) {
      offsets[s] = carry + excl;
      order[s] = x;
    }
    carry += total;
  }

  // Problem records and TMA descriptors of the sorted slots.
  for (int s = tid; s < count; s += kDevPrepThreads) {
    const int x = s_idx[s];
    const gg_problem q = problems[x];
    DeviceProblemDesc d{};
    d.m = q.m;
    d.n = q.n;
    d.k = q.k;
    d.a = static_cast<const __half*>(q.a);
    d.b = static_cast<const __half*>(q.b);
    d.c = q.c;
    d.d = q.d;
    d.lda = q.lda;
    d.ldb = q.ldb;
    d.ldc = q.ldc;
    d.ldd = q.ldd;
    d.alpha = q.alpha;
    d.beta = q.beta;
    const bool has_tiles = q.m > 0 && q.n > 0;
    d.tiles_m = has_tiles ? (q.m + g.bm - 1) / g.bm : 0;
    d.tiles_n = has_tiles ? (q.n + g.bn - 1) / g.bn : 0;
    d.k_blocks = q.k > 0 ? (q.k + g.kblock - 1) / g.kblock : 0;
    d.tma_row0 = 0;
    d.map_slot = 0;  // no tensor maps: cp.async or zero-fill loads, masked stores
    unsigned flags = 0;
    // 16-byte copies for A and B when every row starts 16-byte aligned (the rules of TMA)
    if (has_tiles && q.k > 0 && dev_aligned(q.a, 16) && dev_aligned(q.b, 16) &&
        (static_cast<long long>(q.lda) * g.in_b) % 16 == 0 && (static_cast<long long>(q.ldb) * g.in_b) % 16 == 0)
      flags |= grouped_gemm::kFlagCpAsync;
    if (q.c != nullptr && q.beta != 0.0f) flags |= grouped_gemm::kFlagReadC;
    const bool f32 = g.out_fmt == GG_OUTPUT_F32;
    if (dev_aligned(q.c, 16) && q.ldc % (f32 ? 4 : 8) == 0) flags |= grouped_gemm::kFlagCVec;
    if (dev_aligned(q.d, f32 ? 16u : 8u) && q.ldd % 4 == 0) flags |= grouped_gemm::kFlagDVec;
    d.flags = flags;
    descs[s] = d;
  }
  if (tid == 0) {
    offsets[max_problems] = carry;
    *total_tiles = carry;
    *counter = 0;
  }
}

// Raises the preparation kernel's dynamic shared-memory limit on the current device to at least
// `bytes` (only above the 48 KB default; once per device and size).
cudaError_t dev_prep_reserve_smem(size_t bytes) {
  static std::mutex mu;
  static size_t raised[kMaxDevices] = {};
  if (bytes <= 48 * 1024) return cudaSuccess;
  int dev = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st != cudaSuccess) return st;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (raised[dev] >= bytes) return cudaSuccess;
  st = cudaFuncSetAttribute(device_prepare_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
  if (st == cudaSuccess) raised[dev] = bytes;
  return st;
}

}  // namespace
}  // namespace gg

struct gg_device_plan {
  void* block = nullptr;  // unused map group | records | offsets | order | total, counter, status
  DeviceProblemDesc* d_descs = nullptr;
  int* d_offsets = nullptr;
  int* d_order = nullptr;
  int* d_total = nullptr;
  int* d_counter = nullptr;
  int* d_status = nullptr;
  int max_problems = 0;
  int p2 = 1;
  gg::DevGeom geom{};
  gg::Variant variant = gg::Variant::kUnsupported;
  bool use_tc = true;
  int grid_ctas = 0;
  gg::KernelParams params{};
};

extern "C" {

int gg_device_plan_create(const gg_config* config, int max_problems, gg_device_plan** out) {
  if (!out) return cudaErrorInvalidValue;
  *out = nullptr;
  const gg::Variant v = gg::variant_of(config);
  if (v == gg::Variant::kUnsupported || gg::variant_is_pair(v) || config->tile_classes != GG_TILE_CLASSES_NONE ||
      config->a_layout != GG_LAYOUT_ROW_MAJOR || config->b_layout != GG_LAYOUT_ROW_MAJOR || max_problems < 1 ||
      max_problems > gg::kDevPlanMax)
    return cudaErrorInvalidValue;
  cudaError_t st = gg::dev_prep_reserve_smem(gg::dev_prep_smem(max_problems));
  if (st != cudaSuccess) return st;

  const gg::InGeom ig = gg::in_geom(config->input_type);
  const gg::DevGeom geom{gg::variant_bm(v), gg::variant_bn(v), ig.kblock, ig.bytes, config->output_type};
  const size_t M = static_cast<size_t>(max_problems);
  const size_t descs_off = gg::round_up(gg::kMapsPerProblem * sizeof(CUtensorMap), 128);  // one zeroed map group
  const size_t offs_off = gg::round_up(descs_off + M * sizeof(DeviceProblemDesc), 128);
  const size_t order_off = gg::round_up(offs_off + (M + 1) * sizeof(int), 128);
  const size_t words_off = gg::round_up(order_off + M * sizeof(int), 128);
  const size_t bytes = words_off + 128;

  gg_device_plan* plan = new (std::nothrow) gg_device_plan();
  if (!plan) return cudaErrorMemoryAllocation;
  st = cudaMalloc(&plan->block, bytes);
  if (st != cudaSuccess) {
    delete plan;
    return st;
  }
  st = cudaMemset(plan->block, 0, bytes);
  if (st != cudaSuccess) {
    cudaFree(plan->block);
    delete plan;
    return st;
  }
  unsigned char* base = static_cast<unsigned char*>(plan->block);
  const bool use_tc = config->use_tensor_cores != 0;
  int grid = 0;
  st = gg::path_grid(use_tc, v, 1 << 30, config->persistent_ctas, &grid);
  if (st != cudaSuccess) {
    cudaFree(plan->block);
    delete plan;
    return st;
  }
  plan->d_descs = reinterpret_cast<DeviceProblemDesc*>(base + descs_off);
  plan->d_offsets = reinterpret_cast<int*>(base + offs_off);
  plan->d_order = reinterpret_cast<int*>(base + order_off);
  plan->d_total = reinterpret_cast<int*>(base + words_off);
  plan->d_counter = reinterpret_cast<int*>(base + words_off + 4);
  plan->d_status = reinterpret_cast<int*>(base + words_off + 8);
  plan->max_problems = max_problems;
  plan->p2 = gg::next_pow2(max_problems);
  plan->geom = geom;
  plan->variant = v;
  plan->use_tc = use_tc;
  plan->grid_ctas = grid;

  gg::KernelParams& kp = plan->params;
  std::memset(&kp, 0, sizeof(kp));
  kp.problems = plan->d_descs;
  kp.tmaps = reinterpret_cast<const CUtensorMap*>(base);
  kp.tile_offsets = plan->d_offsets;
  kp.tile_counter = plan->d_counter;
  kp.total_tiles_dev = plan->d_total;
  kp.status = plan->d_status;
  kp.timeout_ns = gg::wait_timeout_ns();
  kp.problem_count = max_problems;  // slots past the count own no tiles
  kp.total_tiles = 0;
  kp.raster_group = gg::raster_group();
  kp.single_mode = 0;
  gg::set_formats(kp, config);
  *out = plan;
  return cudaSuccess;
}

int gg_device_plan_run(gg_device_plan* plan, const gg_problem* problems, const int* count, int sort_mode,
                       void* stream) {
  if (!plan || !plan->block) return cudaErrorInvalidDevicePointer;
  if (!problems || !count) return cudaErrorInvalidValue;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  gg::device_prepare_kernel<<<1, gg::kDevPrepThreads, gg::dev_prep_smem(plan->max_problems), s>>>(
      problems, count, plan->max_problems, plan->p2, sort_mode, plan->geom, plan->d_descs, plan->d_offsets,
      plan->d_order, plan->d_total, plan->d_counter, plan->d_status);
  cudaError_t st = cudaGetLastError();
  if (st != cudaSuccess) return st;
  return gg::launch_path(plan->use_tc, plan->variant, plan->params, plan->grid_ctas, s);
}

int gg_device_plan_status(gg_device_plan* plan, int* status, int* total_tiles) {
  if (!plan || !plan->block) return cudaErrorInvalidDevicePointer;
  if (!status) return cudaErrorInvalidValue;
  cudaError_t st = cudaDeviceSynchronize();
  if (st != cudaSuccess) return st;
  int words[3] = {0, 0, 0};
  st = cudaMemcpy(words, plan->d_total, sizeof(words), cudaMemcpyDeviceToHost);
  if (st != cudaSuccess) return st;
  *status = words[2];
  if (total_tiles) *total_tiles = words[0];
  return cudaMemset(plan->d_status, 0, sizeof(int));
}

int gg_device_plan_prepared(gg_device_plan* plan, int* sorted_to_original, int* tile_offsets, int capacity) {
  if (!plan || !plan->block) return cudaErrorInvalidDevicePointer;
  if (capacity < 0 || capacity > plan->max_problems || (capacity > 0 && !sorted_to_original) || !tile_offsets)
    return cudaErrorInvalidValue;
  cudaError_t st = cudaDeviceSynchronize();
  if (st != cudaSuccess) return st;
  if (capacity > 0) {
    st = cudaMemcpy(sorted_to_original, plan->d_order, static_cast<size_t>(capacity) * sizeof(int),
                    cudaMemcpyDeviceToHost);
    if (st != cudaSuccess) return st;
  }
  return cudaMemcpy(tile_offsets, plan->d_offsets, static_cast<size_t>(capacity + 1) * sizeof(int),
                    cudaMemcpyDeviceToHost);
}

void gg_device_plan_destroy(gg_device_plan* plan) {
  if (!plan) return;
  if (plan->block) cudaFree(plan->block);
  delete plan;
}

}  // extern "C"
