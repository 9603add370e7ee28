// gg_simt.cu -- the CUDA-core path of the grouped GEMM, taken when KernelConfig::use_tensor_cores
// is false: the reference's SIMT mainloop (compute_gemm_tile_simt, reference
// src/grouped_gemm.cu:373-482) restated for this library's problem records and scheduler.
//
// Same contract as the tensor-core kernel: the same tile_offsets and tile numbering (the config's
// cta_m x cta_n tiles), the same atomic tile claims and problem lookup (reference
// src/grouped_gemm.cu:219-234, 640-675), the same epilogue D = alpha*acc + beta*C with C read only
// when c != nullptr and beta != 0 (reference src/grouped_gemm.cu:460-481), with the tensor-core
// epilogue's extensions (output format, bias, activation; gg_epilogue_ops.cuh) and the operand
// layouts (row- or column-major A and B). FP16 (or BF16, FP8) operands
// are widened to FP32 and accumulated with FP32 FMA (a product of two 16-bit values is exact in
// FP32), so the result differs from the tensor-core path only in the order of the FP32 additions.
//
// A CTA computes its tile as 64 x 64 sub-tiles: 256 threads, each 4 x 4 outputs; K in steps of 64
// through shared memory (A stored k-major so a thread reads its 4 rows with one 16-byte load),
// operands loaded with plain zero-filled loads (any leading dimension, any alignment). No
// spin-waits: only atomics and block barriers.
//
// Small problems are a chain of dependent round trips per tile (claim, problem lookup, record,
// operands, C), so the kernel shortens the chain and keeps more chains in flight: four CTAs per SM;
// the next tile's claim in flight during the current tile; the lookup guessed in one round trip
// before any search; the problem record read once into shared memory by one warp; the tables
// brought into L2 at start; a problem of K <= 64 loaded in one step; C brought into L2 while the
// operands load; warps whose rows all lie past M skip the FMAs.
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "gg_epilogue_ops.cuh"
#include "gg_internal.h"

namespace gg {
namespace {

constexpr int kSimtThreads = 256;
constexpr int kSub = 64;     // sub-tile edge
constexpr int kSimtBK = 64;  // K per shared-memory step: a problem of K <= 64 loads in one step
constexpr int kPad = 4;      // keeps 16-byte alignment of every row, spreads banks
constexpr int kPerThread = kSub * kSimtBK / kSimtThreads;  // elements of each operand a thread loads per step
constexpr int kRowStep = kSimtThreads / kSub;                // stored rows between a thread's loads
static_assert(kSub == kSimtBK && kSimtThreads % kSub == 0, "square operand tiles, whole rows per pass");

// The raw bits of an operand element (two bytes, or one for the 8-bit formats), and their FP32
// value, exactly: FP16; BF16 (its bits are the top half of an FP32); E4M3 / E5M2 (every value of
// both is an FP16 value). Split so that a thread can issue all its loads of a K step before it
// needs the first value. Bits 0 widen to +0 in every format.
template <int kIn>
__device__ __forceinline__ unsigned load_bits(const char* x) {
  if constexpr (kIn == GG_INPUT_E4M3 || kIn == GG_INPUT_E5M2)
    return static_cast<unsigned>(*reinterpret_cast<const unsigned char*>(x));
  else
    return static_cast<unsigned>(*reinterpret_cast<const unsigned short*>(x));
}

template <int kIn>
__device__ __forceinline__ float widen_bits(unsigned v) {
  if constexpr (kIn == GG_INPUT_BF16) return __uint_as_float(v << 16);
  else if constexpr (kIn == GG_INPUT_E4M3 || kIn == GG_INPUT_E5M2)
    return __half2float(__half(__nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(v),
                                                       kIn == GG_INPUT_E4M3 ? __NV_E4M3 : __NV_E5M2)));
  else
    return __half2float(__ushort_as_half(static_cast<unsigned short>(v)));
}

// D = act(alpha * acc + (beta * C + bias)) for this thread's 4 x 4 outputs, C and D in format F.
// Every C and bias value is loaded before the first D store: a D store may alias a later C read
// as far as the compiler knows, so interleaved they would be one round trip per element.
template <int F>
__device__ __forceinline__ void store_block(const DeviceProblemDesc& d, const float* bias, int act, bool read_c,
                                            const float (&acc)[4][4], int r0, int c0) {
  float add[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gr = r0 + i;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gc = c0 + j;
      const bool in = gr < d.m && gc < d.n;
      float v = (in && read_c) ? d.beta * load_out<F>(d.c, static_cast<long long>(gr) * d.ldc + gc) : 0.0f;
      if (bias && in) v += __ldg(bias + gc);
      add[i][j] = v;
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gr = r0 + i;
    if (gr >= d.m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gc = c0 + j;
      if (gc >= d.n) continue;
      store_out<F>(d.d, static_cast<long long>(gr) * d.ldd + gc, activate(fmaf(d.alpha, acc[i][j], add[i][j]), act));
    }
  }
}

// Index q with offs[q] <= tile < offs[q+1] (warp-collective; offs has count + 1 entries and
// offs[count] = total > tile). One round trip when problem `guess` holds the tile (the caller
// guesses problem `tile`, right whenever every problem before it has one tile, as small problems
// do); otherwise a 32-ary search inside the bracket the guess leaves, one round trip per 32x.
__device__ int find_problem_warp(const int* __restrict__ offs, int count, int tile, int guess, int lane) {
  guess = min(max(guess, 0), count - 1);
  const int probe = lane < 2 ? __ldg(offs + guess + lane) : 0;
  const int g0 = __shfl_sync(0xffffffffu, probe, 0), g1 = __shfl_sync(0xffffffffu, probe, 1);
  if (g0 <= tile && tile < g1) return guess;
  int lo = g0 <= tile ? guess : 0, hi = g0 <= tile ? count : guess;  // offs[lo] <= tile < offs[hi]
  while (hi - lo > 1) {
    const int step = (hi - lo + 31) >> 5;
    const int idx = lo + lane * step;
    const bool le = idx < hi && __ldg(offs + idx) <= tile;
    const unsigned mask = __ballot_sync(0xffffffffu, le);
    const int last = mask ? 31 - __clz(static_cast<int>(mask)) : 0;
    lo += last * step;
    hi = min(hi, lo + step);
  }
  return lo;
}

// kIn: the input format (GG_INPUT_*), one instantiation each.
template <int kIn>
__global__ void __launch_bounds__(kSimtThreads, 3) grouped_gemm_simt_kernel(const __grid_constant__ KernelParams p,
                                                                           int bm, int bn) {
  __shared__ __align__(16) float As[kSimtBK][kSub + kPad];  // As[k][row]
  __shared__ __align__(16) float Bs[kSimtBK][kSub + kPad];  // Bs[k][col]
  __shared__ __align__(16) DeviceProblemDesc s_desc;        // the current tile's problem record
  __shared__ int s_work[3];                                 // problem, tile_m, tile_n

  const DeviceProblemDesc* problems = p.single_mode ? &p.single_desc : p.problems;
  const int total = p.total_tiles_dev ? *p.total_tiles_dev : p.total_tiles;
  const int tid = static_cast<int>(threadIdx.x);
  const int lane = tid & 31;
  // A warp computes a 16-row x 32-column band of the 64 x 64 sub-tile (8 x 4 threads of 4 x 4
  // outputs), so that it can skip the FMAs when its rows or its columns lie past the problem.
  const int warp = tid >> 5;
  const int rb = warp & 3, cb = warp >> 2;  // the warp's row band (16 rows) and column band (32 columns)
  const int ty = rb * 4 + (lane >> 3);      // rows ty * 4 .. ty * 4 + 3 of the sub-tile
  const int tx = cb * 8 + (lane & 7);       // columns tx * 4 .. tx * 4 + 3
  constexpr int eb = (kIn == GG_INPUT_E4M3 || kIn == GG_INPUT_E5M2) ? 1 : 2;  // bytes per A / B element
  const bool a_col = (p.layout & 1) != 0;  // A stored k x m
  const bool b_col = (p.layout & 2) != 0;  // B stored n x k
  // Warp 0 schedules. Lane 0 keeps one claim in flight (the next tile is claimed when the current
  // one is handed out, so the atomic's round trip overlaps the tile), and the warp caches the last
  // problem's tile range so that tiles of the same problem skip the search and the record load.
  int static_next = static_cast<int>(blockIdx.x);
  int claimed = 0;
  int cq = -1, cq_first = 0, cq_end = 0, ctm = 0, ctn = 0;  // cached problem, its range and grid
  if (tid < 32) {
    if (!p.single_mode && p.problem_count > 0) {
      // this CTA's share of the problem table and tile offsets, brought into L2 once
      const long long desc_lines = (static_cast<long long>(p.problem_count) * sizeof(DeviceProblemDesc) + 127) / 128;
      const long long offs_lines = (static_cast<long long>(p.problem_count + 1) * 4 + 127) / 128;
      const long long lines = desc_lines + offs_lines;
      const long long per = (lines + gridDim.x - 1) / gridDim.x;
      for (long long i = blockIdx.x * per + lane; i < min(lines, (blockIdx.x + 1) * per); i += 32) {
        const char* line = i < desc_lines ? reinterpret_cast<const char*>(p.problems) + 128 * i
                                          : reinterpret_cast<const char*>(p.tile_offsets) + 128 * (i - desc_lines);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(line));
      }
    }
    if (lane == 0) {
      if (p.single_mode) {
        claimed = static_next;
        static_next += static_cast<int>(gridDim.x);
      } else {
        claimed = static_cast<int>(blockIdx.x);  // a CTA's first tile is its index: no claim at start
      }
    }
  }

  for (;;) {
    if (tid < 32) {
      int q = -1, tm = 0, tn = 0;
      for (;;) {
        const int tile = __shfl_sync(0xffffffffu, claimed, 0);
        if (tile >= total) break;
        if (lane == 0) {  // the next claim, in flight while this tile is placed and computed
          if (p.single_mode) {
            claimed = static_next;
            static_next += static_cast<int>(gridDim.x);
          } else {
            claimed = static_cast<int>(gridDim.x) + atomicAdd(p.tile_counter, 1);
          }
        }
        if (!(cq >= 0 && tile >= cq_first && tile < cq_end)) {
          const int pq = p.single_mode ? 0 : find_problem_warp(p.tile_offsets, p.problem_count, tile, tile, lane);
          const int w = lane < kDescWords ? reinterpret_cast<const int*>(problems + pq)[lane] : 0;
          if (lane < kDescWords) reinterpret_cast<int*>(&s_desc)[lane] = w;
          cq = pq;
          cq_first = p.single_mode ? 0 : __ldg(p.tile_offsets + pq);
          cq_end = p.single_mode ? total : __ldg(p.tile_offsets + pq + 1);
          ctm = __shfl_sync(0xffffffffu, w, static_cast<int>(offsetof(DeviceProblemDesc, tiles_m) / 4));
          ctn = __shfl_sync(0xffffffffu, w, static_cast<int>(offsetof(DeviceProblemDesc, tiles_n) / 4));
        }
        const int local = tile - cq_first;
        // a tile outside its problem's grid (a prepared set inconsistent with the config) is
        // skipped, as the reference kernel does (src/grouped_gemm.cu:662-672)
        if (local < 0 || ctm <= 0 || ctn <= 0 || local >= ctm * ctn) continue;
        q = cq;
        tm = local / ctn;
        tn = local % ctn;
        break;
      }
      if (lane == 0) {
        s_work[0] = q;
        s_work[1] = tm;
        s_work[2] = tn;
      }
    }
    __syncthreads();
    const int q = s_work[0], tile_m = s_work[1], tile_n = s_work[2];
    if (q < 0) {
      if (tid == 0) finish_launch(p);  // warp 0 has made its last claim
      break;
    }
    const int m = s_desc.m, n = s_desc.n, k = s_desc.k;
    const __half* a = s_desc.a;
    const __half* b = s_desc.b;
    const int lda = s_desc.lda, ldb = s_desc.ldb;
    const bool read_c = (s_desc.flags & grouped_gemm::kFlagReadC) != 0u;
    DeviceProblemDesc d;  // the epilogue's fields
    d.m = m;
    d.n = n;
    d.c = s_desc.c;
    d.d = s_desc.d;
    d.ldc = s_desc.ldc;
    d.ldd = s_desc.ldd;
    d.alpha = s_desc.alpha;
    d.beta = s_desc.beta;
    const float* bias = p.bias ? p.bias[s_desc.map_slot] : nullptr;
    __syncthreads();  // s_work and s_desc are rewritten for the next tile only after every thread read them

    for (int sm = 0; sm < bm; sm += kSub) {
      const int row0 = tile_m * bm + sm;
      if (row0 >= m) break;
      for (int sn = 0; sn < bn; sn += kSub) {
        const int col0 = tile_n * bn + sn;
        if (col0 >= n) break;
        // the warp's band inside the problem: otherwise it skips the FMAs (it still loads and syncs)
        const bool warp_active = row0 + rb * 16 < m && col0 + cb * 32 < n;
        if (read_c) {  // C of this thread's 4 x 4 outputs into L2 while the operands load
          const int gr = row0 + ty * 4 + (lane & 3), gc = col0 + tx * 4;
          if (gr < m && gc < n)
            asm volatile("prefetch.global.L2 [%0];" ::"l"(static_cast<const char*>(d.c) +
                                                          (static_cast<long long>(gr) * d.ldc + gc) *
                                                              (p.output_format == kOutF32 ? 4 : 2)));
        }
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
        for (int k0 = 0; k0 < k; k0 += kSimtBK) {
          // Consecutive threads take consecutive elements of the stored layout (coalesced reads):
          // a thread keeps one index along the stored rows (u) and steps 4 rows at a time (o).
          // Every load of the step is issued before the first value is stored: one round trip.
          // Stored rows past the operand's edge, and warps whose 32 elements all lie past it, are
          // neither loaded nor stored: those shared-memory rows and columns feed only outputs
          // that are never written (rows past M, columns past N) or K values the FMA loop does
          // not reach, whatever they hold.
          unsigned va[kPerThread], vb[kPerThread];
          const int u = tid & (kSub - 1), o0 = tid / kSub;
          int na, nb;  // stored rows this thread loads, in steps of kRowStep
          {
            const int outer0 = a_col ? k0 : row0, inner0 = a_col ? row0 : k0;  // stored row, element
            const int outer_lim = a_col ? k : m, inner_lim = a_col ? m : k;
            const int rows = outer_lim - outer0 - o0;
            na = (rows <= 0 || inner0 + (u & ~31) >= inner_lim) ? 0 : min(kPerThread, (rows + kRowStep - 1) / kRowStep);
            const bool u_ok = inner0 + u < inner_lim;
            const char* pa = reinterpret_cast<const char*>(a) +
                             (static_cast<long long>(outer0 + o0) * lda + inner0 + u) * eb;
            const long long step = static_cast<long long>(kRowStep) * lda * eb;
#pragma unroll
            for (int j = 0; j < kPerThread; ++j) va[j] = (u_ok && j < na) ? load_bits<kIn>(pa + j * step) : 0u;
          }
          {
            const int outer0 = b_col ? col0 : k0, inner0 = b_col ? k0 : col0;
            const int outer_lim = b_col ? n : k, inner_lim = b_col ? k : n;
            const int rows = outer_lim - outer0 - o0;
            nb = (rows <= 0 || inner0 + (u & ~31) >= inner_lim) ? 0 : min(kPerThread, (rows + kRowStep - 1) / kRowStep);
            const bool u_ok = inner0 + u < inner_lim;
            const char* pb = reinterpret_cast<const char*>(b) +
                             (static_cast<long long>(outer0 + o0) * ldb + inner0 + u) * eb;
            const long long step = static_cast<long long>(kRowStep) * ldb * eb;
#pragma unroll
            for (int j = 0; j < kPerThread; ++j) vb[j] = (u_ok && j < nb) ? load_bits<kIn>(pb + j * step) : 0u;
          }
#pragma unroll
          for (int j = 0; j < kPerThread; ++j) {
            if (j >= na) break;
            const int o = o0 + kRowStep * j;
            if (a_col) As[o][u] = widen_bits<kIn>(va[j]);
            else As[u][o] = widen_bits<kIn>(va[j]);
          }
#pragma unroll
          for (int j = 0; j < kPerThread; ++j) {
            if (j >= nb) break;
            const int o = o0 + kRowStep * j;
            if (b_col) Bs[u][o] = widen_bits<kIn>(vb[j]);
            else Bs[o][u] = widen_bits<kIn>(vb[j]);
          }
          __syncthreads();
          if (warp_active) {
            const int kn = min(kSimtBK, k - k0);  // K values of this step
#pragma unroll 8
            for (int kk = 0; kk < kn; ++kk) {
              const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
              const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
              const float ar[4] = {av.x, av.y, av.z, av.w};
              const float br[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
              for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
            }
          }
          __syncthreads();
        }
        // C taken as 0 when it is not read
        if (p.output_format == kOutF16)
          store_block<kOutF16>(d, bias, p.activation, read_c, acc, row0 + ty * 4, col0 + tx * 4);
        else if (p.output_format == kOutBF16)
          store_block<kOutBF16>(d, bias, p.activation, read_c, acc, row0 + ty * 4, col0 + tx * 4);
        else
          store_block<kOutF32>(d, bias, p.activation, read_c, acc, row0 + ty * 4, col0 + tx * 4);
      }
    }
  }
}

}  // namespace

cudaError_t simt_resident_ctas(int* ctas) {
  int dev = 0, sms = 0, per_sm = 0;
  cudaError_t st = cudaGetDevice(&dev);
  if (st == cudaSuccess) st = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (st == cudaSuccess)
    st = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, grouped_gemm_simt_kernel<GG_INPUT_F16>, kSimtThreads,
                                                       0);
  if (st != cudaSuccess) return st;
  *ctas = sms * (per_sm > 0 ? per_sm : 1);
  return cudaSuccess;
}

cudaError_t simt_occupancy(int* active_blocks_per_sm, cudaFuncAttributes* attrs) {
  cudaError_t st = cudaFuncGetAttributes(attrs, grouped_gemm_simt_kernel<GG_INPUT_F16>);
  if (st != cudaSuccess) return st;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(active_blocks_per_sm, grouped_gemm_simt_kernel<GG_INPUT_F16>,
                                                       kSimtThreads, 0);
}

int simt_threads() { return kSimtThreads; }

template <int kIn>
cudaError_t launch_simt(Variant v, const KernelParams& params, int grid, cudaStream_t stream, bool overlap_previous) {
  if (!overlap_previous) {
    grouped_gemm_simt_kernel<kIn><<<grid, kSimtThreads, 0, stream>>>(params, variant_bm(v), variant_bn(v));
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kSimtThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, grouped_gemm_simt_kernel<kIn>, params, variant_bm(v), variant_bn(v));
}

cudaError_t launch_simt_kernel(Variant v, const KernelParams& params, int grid, cudaStream_t stream,
                               bool overlap_previous) {
  if (grid <= 0) return cudaSuccess;
  switch (params.input_format) {
    case GG_INPUT_BF16:
      return launch_simt<GG_INPUT_BF16>(v, params, grid, stream, overlap_previous);
    case GG_INPUT_E4M3:
      return launch_simt<GG_INPUT_E4M3>(v, params, grid, stream, overlap_previous);
    case GG_INPUT_E5M2:
      return launch_simt<GG_INPUT_E5M2>(v, params, grid, stream, overlap_previous);
    default:
      return launch_simt<GG_INPUT_F16>(v, params, grid, stream, overlap_previous);
  }
}

}  // namespace gg
