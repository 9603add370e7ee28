// gg_kernel.cuh -- the persistent grouped GEMM kernel for B200 (sm_100a).
//
// One CTA per SM (shared memory > half an SM's), 384 threads in five warp roles:
//
//   warps 0-7   epilogue   TMEM -> registers (tcgen05.ld), D = alpha*acc + beta*C. Warp w reads
//                          TMEM lanes 32(w%4)..+31 = tile rows 32(w%4)..+31 and stores half of the
//                          tile's columns (w/4 picks the half) on its own: per 32-column chunk one
//                          32x32 TMA store from a 128-byte-swizzled staging tile (clipped at the
//                          problem edge), or, when D is not TMA-eligible, coalesced masked stores
//                          read back from that tile.
//   warp 8      MMA        allocates 512 TMEM columns (2 accumulators of 256 columns or 4 of <= 128,
//                          so the epilogue of one tile overlaps the mainloops of the next); one
//                          thread issues tcgen05.mma.kind::f16 (M=128, N=BN, K=16; kind::f8f6f4,
//                          K=32, for 8-bit A/B) and tcgen05.commit.
//   warp 9      scheduler  claims global tile indices with atomicAdd (the reference's device
//                          scheduler, src/grouped_gemm.cu:640-675), finds the owning problem with a
//                          warp-parallel 32-ary search of tile_offsets (same answer as the
//                          reference's binary search, src/grouped_gemm.cu:219-234), copies the
//                          problem record into a 4-deep shared-memory ring read by every role.
//   warps 10-11 producers  fill a multi-stage ring of A/B shared-memory tiles: one thread issues
//                          TMA tensor loads for aligned problems (one box for A and, for tiles
//                          inside N, one 3-D box for all of B); all 64 threads load with zero
//                          fill for problems whose base or leading dimension TMA cannot take (the
//                          reference's scalar zero-fill path, src/grouped_gemm.cu:273-371),
//                          writing the same 128-byte-swizzled layout the TMA would.
//
// Shared-memory layout per stage: A as 128 rows x 64 K (K-major, 128-byte rows, SW128) and B as
// BN/64 column chunks of 64 K rows x 64 N (MN-major, SW128); with 8-bit A/B (kind::f8f6f4) the
// same bytes hold 128 rows x 128 K of A and BN/128 chunks of 128 K rows x 128 N of B. A 64-row tile (reference shapes
// 64xN) still runs an M=128 MMA; rows 64..127 of the accumulator are never stored.
//
// Every wait is bounded (timeout_ns from %globaltimer): a wait that runs out sets a status bit
// and a CTA-wide abort flag; all roles then leave their loops, the MMA thread drains its
// tensor-core work, the producer drains its TMA loads, the epilogue drains its TMA stores, and
// TMEM is freed before the CTA exits.
#pragma once

#include <cuda_fp16.h>
#include <cstddef>
#include <cstdint>

#include "gg_epilogue_ops.cuh"
#include "gg_params.cuh"
#include "gg_ptx.cuh"
#include "grouped_gemm_b200.h"

namespace gg {

// ---- bounded waits ---------------------------------------------------------------------------
__device__ __noinline__ bool wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                       unsigned long long timeout_ns, int code) {
  const uint64_t t0 = ptx::global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 31u) {
      if (*abort_flag) return false;
      if (ptx::global_timer_ns() - t0 > timeout_ns || i > 0x40000000u) {
        *abort_flag = 1;
        atomicOr(status, code);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool wait_phase(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                           unsigned long long timeout_ns, int code) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  return wait_slow(bar, parity, abort_flag, status, timeout_ns, code);
}

// Drain wait used after an abort: ignores the abort flag, gives up after `limit_ns`.
__device__ __noinline__ void wait_drain(uint32_t bar, uint32_t parity, unsigned long long limit_ns) {
  const uint64_t t0 = ptx::global_timer_ns();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (ptx::global_timer_ns() - t0 > limit_ns) return;
  }
}

// ---- scheduler helpers -----------------------------------------------------------------------
// Index q with offs[q] <= tile < offs[q+1] (empty problems are skipped because their two offsets
// are equal). Each round the 32 lanes probe 32 evenly spaced offsets, shrinking the bracket 32x.
__device__ __forceinline__ int find_problem_warp(const int* __restrict__ offs, int count, int tile, int lane) {
  int lo = 0, hi = count;  // invariant: offs[lo] <= tile < offs[hi] (offs[count] = total > tile)
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

// Raster inside a problem: groups of `group` M-tiles; inside a group M runs fastest, then N.
__device__ __forceinline__ void raster_tile(int local, int tiles_m, int tiles_n, int group, int& tm, int& tn) {
  const int span = group * tiles_n;
  const int g = local / span;
  const int first_m = g * group;
  const int gm = min(group, tiles_m - first_m);
  const int in_g = local - g * span;
  tm = first_m + in_g % gm;
  tn = in_g / gm;
}

// Scheduler state of one warp. Lane 0 keeps one tile claim in flight (the atomicAdd for the next
// tile is issued before the current tile is searched), and every lane keeps its word of the last
// problem's descriptor with that problem's tile range, so tiles claimed from the same problem skip
// the search and the descriptor load.
struct SchedState {
  int total;        // tiles of the launch
  int cur;          // lane 0: claimed tile not yet handed out
  int static_next;  // lane 0: next tile of the static order (baseline launches)
  int q;            // problem of the cached descriptor, -1 when none
  int q_first;      // its first tile
  int q_end;        // one past its last tile
  int w;            // this lane's 32-bit word of the cached descriptor
};

__device__ __forceinline__ int claim_tile(const KernelParams& p, SchedState& ss, int stride) {
  if (p.single_mode) {
    const int t = ss.static_next;
    ss.static_next += stride;
    return t;
  }
  return stride + atomicAdd(p.tile_counter, 1);  // tiles below stride are the CTAs' first tiles
}

__device__ __forceinline__ void sched_init(const KernelParams& p, SchedState& ss, int first_static, int stride,
                                           int lane) {
  ss.total = p.total_tiles_dev ? *p.total_tiles_dev : p.total_tiles;
  ss.static_next = first_static;
  ss.q = -1;
  ss.q_first = 0;
  ss.q_end = 0;
  ss.w = 0;
  ss.cur = 0;
  // the first tile of a CTA is its index (no claim on the start-up path); later claims count
  // from `stride`
  if (lane == 0) ss.cur = p.single_mode ? claim_tile(p, ss, stride) : first_static;
}

// Next tile of this CTA (warp-collective): returns false when the work is exhausted, else the
// problem index, the tile coordinates, and leaves the problem's descriptor words in ss.w.
__device__ __forceinline__ bool next_tile(const KernelParams& p, SchedState& ss, const DeviceProblemDesc* problems,
                                          int lane, int stride, int& q_out, int& tile_m, int& tile_n) {
  for (;;) {
    const int tile = __shfl_sync(0xffffffffu, ss.cur, 0);
    if (tile >= ss.total) return false;
    if (lane == 0) ss.cur = claim_tile(p, ss, stride);  // in flight while this tile is placed
    if (!(ss.q >= 0 && tile >= ss.q_first && tile < ss.q_end)) {
      const int q = p.single_mode ? 0 : find_problem_warp(p.tile_offsets, p.problem_count, tile, lane);
      ss.q = q;
      ss.q_first = p.single_mode ? 0 : p.tile_offsets[q];
      ss.q_end = p.single_mode ? ss.total : p.tile_offsets[q + 1];
      const int* src = reinterpret_cast<const int*>(problems + q);
      ss.w = lane < kDescWords ? src[lane] : 0;
    }
    const int local = tile - ss.q_first;
    const int tiles_m = __shfl_sync(0xffffffffu, ss.w, static_cast<int>(offsetof(DeviceProblemDesc, tiles_m) / 4));
    const int tiles_n = __shfl_sync(0xffffffffu, ss.w, static_cast<int>(offsetof(DeviceProblemDesc, tiles_n) / 4));
    // A tile index outside its problem's tile grid (a prepared set inconsistent with the config)
    // is skipped, as the reference kernel does (src/grouped_gemm.cu:662-672).
    if (local < 0 || tiles_m <= 0 || tiles_n <= 0 || local >= tiles_m * tiles_n) continue;
    raster_tile(local, tiles_m, tiles_n, p.raster_group, tile_m, tile_n);
    q_out = ss.q;
    return true;
  }
}

// At kernel start each CTA's scheduler brings its 1/gridDim share of the problem table and of the
// tile offsets into L2 (`part` of `parts`), so that the searches and record loads of every CTA hit
// L2 instead of DRAM once the first claims are out (cold tables cost one DRAM round trip per
// dependent load of the search otherwise).
__device__ __forceinline__ void prefetch_tables_l2(const KernelParams& p, int part, int parts, int lane) {
  if (p.single_mode || p.problem_count <= 0) return;
  const int64_t desc_bytes = static_cast<int64_t>(p.problem_count) * static_cast<int64_t>(sizeof(DeviceProblemDesc));
  const int64_t offs_bytes = static_cast<int64_t>(p.problem_count + 1) * 4;
  const int64_t desc_lines = (desc_bytes + 127) / 128, offs_lines = (offs_bytes + 127) / 128;
  const int64_t lines = desc_lines + offs_lines;
  const int64_t per = (lines + parts - 1) / parts;
  for (int64_t i = part * per + lane; i < min(lines, (part + 1) * per); i += 32) {
    const uint8_t* base = i < desc_lines ? reinterpret_cast<const uint8_t*>(p.problems) + 128 * i
                                         : reinterpret_cast<const uint8_t*>(p.tile_offsets) + 128 * (i - desc_lines);
    ptx::prefetch_l2(base);
  }
}

// Warms the tensor maps a tile of this problem will use (only those that were encoded).
__device__ __forceinline__ void prefetch_problem_maps(const CUtensorMap* maps, int q, unsigned flags, int lane) {
  const bool map_valid = (lane == kMapA || lane == kMapB) ? (flags & grouped_gemm::kFlagTmaAB) != 0u
                         : lane == kMapB3                 ? (flags & grouped_gemm::kFlagTmaB3) != 0u
                         : lane == kMapD                  ? (flags & grouped_gemm::kFlagTmaD) != 0u
                                                          : false;
  if (map_valid) ptx::prefetch_tensormap(maps + kMapsPerProblem * q + lane);
}

// ---- epilogue helper ---------------------------------------------------------------------
// What one epilogue warp needs of its tile.
struct EpiTile {
  int row0;            // first of the warp's 32 rows (>= m: the warp stores nothing)
  int m;
  int n;
  int col0;            // first column of the tile
  int c_begin;         // the warp's 32-column chunks: [c_begin, c_end)
  int c_end;
  int kb_count;        // K blocks; 0: the accumulator is taken as zero
  unsigned flags;      // DeviceProblemFlags
  float alpha;
  float beta;
  const void* c;       // output format, row pitch ldc
  int ldc;
  void* d;             // output format, row pitch ldd
  int ldd;
  const float* bias;   // n FP32 values, or null
  int act;             // GG_ACT_*
  const CUtensorMap* md;  // D map (kFlagTmaD)
  int tma_row0;
};

// One epilogue warp's share of a tile: rows row0..row0+31 (TMEM lanes of this warp's quarter) and
// chunks [c_begin, c_end) of 32 columns. D = act(alpha * acc + (beta * C + bias)), C taken as 0
// when it is not read (reference src/grouped_gemm.cu:614-621 for the FP32 form without bias and
// activation), in output format `fmt` (GG_OUTPUT_*; one body serves all formats: three inlined
// copies, one per format, would not fit the register budget together). `stage` is this warp's kEpiWarpBytes of shared memory: one
// FP32 or two 16-bit staging tiles of 32 rows x 32 columns (128-byte rows with the 128-byte
// swizzle for FP32, 64-byte rows with the 64-byte swizzle for 16-bit). The warp works alone, with
// no barrier across warps inside the tile:
//  - TMA-storable D: each chunk goes out in one 32x32 TMA store issued by lane 0; lane 0's bulk
//    groups say when a staging tile may be written again;
//  - any other D: the FP32 accumulator chunk is read back from the staging tile so that 8
//    consecutive lanes hold one 32-column row segment, and C is loaded and D stored with
//    coalesced accesses of 4 elements.
// `release` hands the accumulator back to the MMA warp after the last TMEM read.
template <typename Release>
__device__ __forceinline__ void epilogue_warp(int fmt, uint8_t* stage, uint32_t& store_count, uint32_t t_addr,
                                              int lane, const EpiTile& e, Release release) {
  const float* bias = e.bias;
  const int act = e.act;
  static_assert(kEpiWarpBytes == 4096, "one FP32 or two 16-bit staging tiles per epilogue warp");
  const bool out32 = fmt == kOutF32;
  const int eb = out32 ? 4 : 2;                // bytes per C / D element
  const int tile_bytes = 32 * 32 * eb;         // one staged chunk
  const bool two_tiles = !out32;               // 16-bit chunks: two staging tiles, alternating
  const int m = e.m, n = e.n, row0 = e.row0;
  const bool warp_rows = row0 < m;  // warp-uniform
  const bool read_c = (e.flags & grouped_gemm::kFlagReadC) != 0u;
  const bool cvec = (e.flags & grouped_gemm::kFlagCVec) != 0u;
  // With packed rows the D map spans every problem, so only a whole 32-row box may go out by TMA.
  const bool tma_d = (e.flags & grouped_gemm::kFlagTmaD) != 0u &&
                     ((e.flags & grouped_gemm::kFlagPackedRows) == 0u || row0 + 32 <= m);
  const int row = row0 + lane;
  if (tma_d) {
    // Two chunks per TMEM read (one 64-column tcgen05.ld and one wait), then one staging tile
    // and one TMA store per chunk, so that a store is always in flight while the next chunk is
    // prepared.
    for (int c = e.c_begin; c < e.c_end; c += 2) {
      const int nsub = c + 1 < e.c_end ? 2 : 1;
      uint32_t r[64];
      if (warp_rows && e.kb_count > 0) {
        if (nsub == 2) {
          ptx::tmem_load_64cols(t_addr + static_cast<uint32_t>(c * 32), r);
        } else {
          uint32_t h[32];
          ptx::tmem_load_32cols(t_addr + static_cast<uint32_t>(c * 32), h);
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = h[j];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 64; ++j) r[j] = 0u;
      }
      if (c + nsub >= e.c_end) {
        // This warp's last read of the accumulator: hand it back before the stores.
        ptx::tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) release();
      }
      if (!warp_rows) continue;
#pragma unroll
      for (int sub = 0; sub < 2; ++sub) {
        if (sub >= nsub) break;
        const int cc = e.col0 + (c + sub) * 32;
        // cv = beta * C + bias, the addend of alpha * acc
        float cv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) cv[j] = 0.0f;
        if (read_c && row < m) {
          const int64_t ci = static_cast<int64_t>(row) * e.ldc + cc;
          if (cvec && cc + 32 <= n) {
            const uint4* crow = reinterpret_cast<const uint4*>(static_cast<const char*>(e.c) + ci * eb);
            if (out32) {
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                const uint4 u = __ldg(crow + v);
                cv[4 * v] = __uint_as_float(u.x);
                cv[4 * v + 1] = __uint_as_float(u.y);
                cv[4 * v + 2] = __uint_as_float(u.z);
                cv[4 * v + 3] = __uint_as_float(u.w);
              }
            } else {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                const uint4 u = __ldg(crow + v);
                const float2 f0 = unpack2_rt(fmt, u.x), f1 = unpack2_rt(fmt, u.y), f2 = unpack2_rt(fmt, u.z),
                             f3 = unpack2_rt(fmt, u.w);
                cv[8 * v] = f0.x;
                cv[8 * v + 1] = f0.y;
                cv[8 * v + 2] = f1.x;
                cv[8 * v + 3] = f1.y;
                cv[8 * v + 4] = f2.x;
                cv[8 * v + 5] = f2.y;
                cv[8 * v + 6] = f3.x;
                cv[8 * v + 7] = f3.y;
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (cc + j < n) cv[j] = load_out_rt(fmt, e.c, ci + j);
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) cv[j] *= e.beta;
        }
        if (bias) {  // lane j loads column cc + j's bias (an L1 hit: prefetched); shuffles share it
          const float bl = cc + lane < n ? __ldg(bias + cc + lane) : 0.0f;
#pragma unroll
          for (int j = 0; j < 32; ++j) cv[j] += __shfl_sync(0xffffffffu, bl, j);
        }
        // the chunk's results, in cv: alpha * acc + (beta * C + bias), then the activation
#pragma unroll
        for (int j = 0; j < 32; ++j) cv[j] = fmaf(e.alpha, __uint_as_float(r[sub * 32 + j]), cv[j]);
        if (act != GG_ACT_NONE) {
#pragma unroll
          for (int j = 0; j < 32; ++j) cv[j] = activate(cv[j], act);
        }
        uint8_t* stile = stage + (two_tiles ? static_cast<int>(store_count & 1u) * tile_bytes : 0);
        if (lane == 0) {  // the store that last used this staging tile has read it
          if (two_tiles) ptx::bulk_wait_read_le1();
          else ptx::bulk_wait_all_read();
        }
        __syncwarp();
        if (out32) {
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4)
            *reinterpret_cast<float4*>(stile + lane * 128 + ((j4 ^ (lane & 7)) << 4)) =
                make_float4(cv[4 * j4], cv[4 * j4 + 1], cv[4 * j4 + 2], cv[4 * j4 + 3]);
        } else {
          // 64-byte rows, 64-byte swizzle: 16-byte unit j8 of row `lane` sits at j8 ^ ((lane >> 1) & 3)
#pragma unroll
          for (int j8 = 0; j8 < 4; ++j8)
            *reinterpret_cast<uint4*>(stile + lane * 64 + ((j8 ^ ((lane >> 1) & 3)) << 4)) =
                make_uint4(pack2_rt(fmt, cv[8 * j8], cv[8 * j8 + 1]), pack2_rt(fmt, cv[8 * j8 + 2], cv[8 * j8 + 3]),
                           pack2_rt(fmt, cv[8 * j8 + 4], cv[8 * j8 + 5]),
                           pack2_rt(fmt, cv[8 * j8 + 6], cv[8 * j8 + 7]));
        }
        ptx::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          ptx::tma_store_2d(e.md, ptx::smem_addr(stile), cc, e.tma_row0 + row0);  // rows past M are clipped
          ptx::bulk_commit_group();
        }
        ++store_count;
      }
    }
  } else {
    // Any other D: each chunk is read back from the staging tile so that 8 consecutive lanes
    // hold one 32-column row segment, then C is loaded and D stored with coalesced accesses.
    const int jj = lane & 7;
    const bool dvec = (e.flags & grouped_gemm::kFlagDVec) != 0u;
    if (warp_rows && lane == 0) ptx::bulk_wait_all_read();  // staging tile 0 is free
    for (int c = e.c_begin; c < e.c_end; ++c) {
      const int cc = e.col0 + c * 32;
      const int gcol = cc + 4 * jj;
      // beta * C, issued before the TMEM read so that its latency overlaps it.
      float cv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) cv[j] = 0.0f;
      if (read_c && warp_rows) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int grow = row0 + i * 4 + (lane >> 3);
          if (grow < m && gcol < n) {
            const int64_t ci = static_cast<int64_t>(grow) * e.ldc + gcol;
            if (cvec && gcol + 4 <= n) {
              const float4 v = load_out4_rt(fmt, static_cast<const char*>(e.c) + ci * eb);
              cv[4 * i] = v.x;
              cv[4 * i + 1] = v.y;
              cv[4 * i + 2] = v.z;
              cv[4 * i + 3] = v.w;
            } else {
#pragma unroll
              for (int q = 0; q < 4; ++q)
                if (gcol + q < n) cv[4 * i + q] = load_out_rt(fmt, e.c, ci + q);
            }
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) cv[j] *= e.beta;
      }
      uint32_t r[32];
      if (warp_rows && e.kb_count > 0) {
        ptx::tmem_load_32cols(t_addr + static_cast<uint32_t>(c * 32), r);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = 0u;
      }
      if (c == e.c_end - 1) {
        ptx::tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) release();
      }
      if (!warp_rows) continue;
#pragma unroll
      for (int j4 = 0; j4 < 8; ++j4)
        *reinterpret_cast<uint4*>(stage + lane * 128 + ((j4 ^ (lane & 7)) << 4)) =
            make_uint4(r[4 * j4], r[4 * j4 + 1], r[4 * j4 + 2], r[4 * j4 + 3]);
      __syncwarp();
      float bv[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      if (bias) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          if (gcol + q < n) bv[q] = __ldg(bias + gcol + q);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int rr = i * 4 + (lane >> 3);
        const float4 a4 = *reinterpret_cast<const float4*>(stage + rr * 128 + ((jj ^ (rr & 7)) << 4));
        const int grow = row0 + rr;
        if (grow < m && gcol < n) {
          float4 o = make_float4(fmaf(e.alpha, a4.x, cv[4 * i] + bv[0]), fmaf(e.alpha, a4.y, cv[4 * i + 1] + bv[1]),
                                 fmaf(e.alpha, a4.z, cv[4 * i + 2] + bv[2]), fmaf(e.alpha, a4.w, cv[4 * i + 3] + bv[3]));
          o = activate4(o, act);
          const int64_t di = static_cast<int64_t>(grow) * e.ldd + gcol;
          if (dvec && gcol + 4 <= n) {
            store_out4_rt(fmt, static_cast<char*>(e.d) + di * eb, o);
          } else {
            store_out_rt(fmt, e.d, di, o.x);
            if (gcol + 1 < n) store_out_rt(fmt, e.d, di + 1, o.y);
            if (gcol + 2 < n) store_out_rt(fmt, e.d, di + 2, o.z);
            if (gcol + 3 < n) store_out_rt(fmt, e.d, di + 3, o.w);
          }
        }
      }
      __syncwarp();
    }
  }
  if (e.c_begin >= e.c_end) {
    ptx::tc_fence_before_sync();
    __syncwarp();
    if (lane == 0) release();
  }
}

// Brings the bias of this warp's chunks into L1 before the accumulator wait (lane j: column
// col0 + c * 32 + j of each chunk c), so that the epilogue's loads of it hit L1 instead of waiting
// on L2 or DRAM; holds no registers across the wait.
__device__ __forceinline__ void epilogue_bias_prefetch(const EpiTile& e, int lane) {
  if (!e.bias) return;
  for (int c = e.c_begin; c < e.c_end; ++c) {
    const int col = e.col0 + c * 32 + lane;
    if (col < e.n) ptx::prefetch_l1(e.bias + col);
  }
}

// The chunk range [c_begin, c_end) of a tile's nchunks 32-column chunks that epilogue warp half
// `half` stores: whole 64-column pairs, the first half taking the larger share; a tile of two
// chunks gives one to each half, so that both halves work on narrow tiles.
__device__ __forceinline__ void epilogue_chunk_range(int nchunks, int half, int& c_begin, int& c_end) {
  const int split = nchunks == 2 ? 1 : min(nchunks, 2 * ((nchunks + 3) / 4));
  c_begin = half ? split : 0;
  c_end = half ? nchunks : split;
}

// ---- producer helpers ------------------------------------------------------------------------
// Zero-fill loader for problems TMA cannot take (odd leading dimension or base alignment). Fills
// one stage -- A rows [row0, row0+ROWS) and B columns [col0, col0+COLS) of K block kb -- in the
// same 128-byte-swizzled layouts the TMA loads produce. It works in bytes, so 16-bit (EB = 2) and
// 8-bit (EB = 1) operands share it: consecutive lanes read consecutive W-byte pieces of one row
// (coalesced; W = 4 when every row of the operand starts 4-byte aligned, else the widest the
// alignment allows), and each lane keeps up to 16 loads in flight before it stores them. Bytes
// past K (columns of A, rows of B) are written as zeros; rows of A past M and columns of B past N
// are not written at all: they only reach accumulator rows and columns that are never stored.
constexpr int kLsuBatch = 16;  // loads in flight per lane before their stores

// W bytes at src + bi, with every element at or past `limit` bytes read as zero (limit is a
// multiple of EB; bi and W are multiples of EB).
template <int W, int EB>
__device__ __forceinline__ uint32_t lsu_load(const uint8_t* src, int bi, int limit) {
  if (bi + W <= limit) {
    if (W == 4) return __ldg(reinterpret_cast<const unsigned int*>(src + bi));
    if (W == 2) return __ldg(reinterpret_cast<const unsigned short*>(src + bi));
    return __ldg(src + bi);
  }
  if constexpr (W == EB) {
    return 0u;  // one element, past the limit
  } else if constexpr (EB == 2) {
    return bi < limit ? static_cast<uint32_t>(__ldg(reinterpret_cast<const unsigned short*>(src + bi))) : 0u;
  } else {
    uint32_t v = 0u;  // 8-bit elements: the 1 to W-1 bytes before the limit
#pragma unroll
    for (int e = 0; e < W - 1; ++e)
      if (bi + e < limit) v |= static_cast<uint32_t>(__ldg(src + bi + e)) << (8 * e);
    return v;
  }
}

template <int W>
__device__ __forceinline__ void lsu_store(uint8_t* dst, uint32_t v) {
  if (W == 4) *reinterpret_cast<uint32_t*>(dst) = v;
  else if (W == 2) *reinterpret_cast<unsigned short*>(dst) = static_cast<unsigned short>(v);
  else *dst = static_cast<uint8_t>(v);
}

// K-major tile: ROWS rows of 128 bytes (the K block), row r at r * 128, 16-byte units XOR-swizzled
// by r & 7. Source row r starts at base + (row0 + r) * ld_bytes + k0_bytes; kbytes of it lie
// inside K.
template <int ROWS, int W, int EB>
__device__ __forceinline__ void lsu_fill_kmajor(uint8_t* dst, const uint8_t* base, int64_t ld_bytes, int rows,
                                                int kbytes, int row0, int64_t k0_bytes, int pw, int ln) {
  constexpr int kW = kProdThreads / 32;
  constexpr int kPer = 128 / (32 * W);  // loads per lane per row
  constexpr int kB = (kLsuBatch / kPer) < (ROWS / kW) ? (kLsuBatch / kPer) : (ROWS / kW);  // rows per batch
  const int klim = kbytes < 128 ? kbytes : 128;
#pragma unroll 1
  for (int rb = pw; rb < rows; rb += kW * kB) {
    uint32_t v[kB][kPer];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int r = rb + i * kW;
      const uint8_t* src = base + static_cast<int64_t>(row0 + (r < rows ? r : 0)) * ld_bytes + k0_bytes;
#pragma unroll
      for (int j = 0; j < kPer; ++j) v[i][j] = r < rows ? lsu_load<W, EB>(src, j * 32 * W + W * ln, klim) : 0u;
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int r = rb + i * kW;
      if (r < rows) {
        const int sw = (r & 7) << 4;
#pragma unroll
        for (int j = 0; j < kPer; ++j) lsu_store<W>(dst + r * 128 + ((j * 32 * W + W * ln) ^ sw), v[i][j]);
      }
    }
  }
}

// MN-major tile: KB K rows (the K block) x COLS_BYTES bytes of columns, stored as 128-byte-wide
// column chunks of KB rows (chunk c at c * KB * 128), row kr of a chunk at kr * 128, swizzled by
// kr & 7. Source K row kr starts at base + (k0 + kr) * ld_bytes + col0_bytes; cbytes of it lie
// inside N; rows at or past kvalid are zero.
template <int COLS_BYTES, int KB, int W, int EB>
__device__ __forceinline__ void lsu_fill_mnmajor(uint8_t* dst, const uint8_t* base, int64_t ld_bytes, int cbytes,
                                                 int kvalid, int64_t col0_bytes, int k0, int pw, int ln) {
  constexpr int kW = kProdThreads / 32;
  constexpr int kPer = COLS_BYTES / (32 * W);  // loads per lane per K row
  constexpr int kB = (kLsuBatch / kPer) < (KB / kW) ? (kLsuBatch / kPer) : (KB / kW);  // K rows per batch
#pragma unroll 1
  for (int rb = pw; rb < KB; rb += kW * kB) {
    uint32_t v[kB][kPer];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int kr = rb + i * kW;
      const bool kin = kr < kvalid;
      const uint8_t* src = base + static_cast<int64_t>(kin ? k0 + kr : 0) * ld_bytes + col0_bytes;
#pragma unroll
      for (int j = 0; j < kPer; ++j) v[i][j] = kin ? lsu_load<W, EB>(src, j * 32 * W + W * ln, cbytes) : 0u;
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int kr = rb + i * kW;
      const int sw = (kr & 7) << 4;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int c = j * 32 * W + W * ln;
        if (c < cbytes) lsu_store<W>(dst + (c >> 7) * (KB * 128) + kr * 128 + ((c & 127) ^ sw), v[i][j]);
      }
    }
  }
}

// Widest load (4, 2 or 1 bytes) that every row of an operand allows: base and row pitch in bytes.
__device__ __forceinline__ int lsu_width(const void* p, int64_t ld_bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p) | static_cast<uintptr_t>(ld_bytes);
  return (a & 3u) == 0u ? 4 : (a & 1u) == 0u ? 2 : 1;
}

// One operand of the stage. kmajor: a K-major tile of NV rows (row-major A, column-major B);
// else an MN-major tile of NV columns (row-major B, column-major A). nv_valid rows/columns from
// v0 on and K from k0 on lie inside the problem.
template <int NV, int EB>
__device__ __forceinline__ void lsu_fill_operand(uint8_t* dst, const void* p, int ld, bool kmajor, int nv_valid,
                                                 int k, int v0, int k0, int pw, int ln) {
  constexpr int KB = EB == 2 ? kBK : 2 * kBK;  // K values in one 128-byte row
  const uint8_t* base = static_cast<const uint8_t*>(p);
  const int64_t ld_bytes = static_cast<int64_t>(ld) * EB;
  const int w = lsu_width(p, ld_bytes);
  if (kmajor) {
    const int kbytes = (k - k0) * EB;
    const int64_t k0b = static_cast<int64_t>(k0) * EB;
    if (w == 4) lsu_fill_kmajor<NV, 4, EB>(dst, base, ld_bytes, nv_valid, kbytes, v0, k0b, pw, ln);
    else if (w == 2 || EB == 2) lsu_fill_kmajor<NV, 2, EB>(dst, base, ld_bytes, nv_valid, kbytes, v0, k0b, pw, ln);
    else lsu_fill_kmajor<NV, 1, EB>(dst, base, ld_bytes, nv_valid, kbytes, v0, k0b, pw, ln);
  } else if constexpr (NV * EB >= 128) {  // narrower MN-major 8-bit tiles are refused on the host
    const int cbytes = nv_valid * EB;
    const int kvalid = k - k0 < KB ? k - k0 : KB;
    const int64_t c0b = static_cast<int64_t>(v0) * EB;
    if (w == 4) lsu_fill_mnmajor<NV * EB, KB, 4, EB>(dst, base, ld_bytes, cbytes, kvalid, c0b, k0, pw, ln);
    else if (w == 2 || EB == 2)
      lsu_fill_mnmajor<NV * EB, KB, 2, EB>(dst, base, ld_bytes, cbytes, kvalid, c0b, k0, pw, ln);
    else lsu_fill_mnmajor<NV * EB, KB, 1, EB>(dst, base, ld_bytes, cbytes, kvalid, c0b, k0, pw, ln);
  }
}

// `col_a` / `col_b`: the operand is stored column-major, so A (k x m) fills the MN-major chunk
// layout of row-major B and B (n x k) the K-major row layout of row-major A. f8: 8-bit operands.
template <int ROWS, int COLS>
__device__ __forceinline__ void lsu_fill_stage(uint8_t* as, uint8_t* bs, const __half* a, int lda, const __half* b,
                                               int ldb, int m, int n, int k, int row0, int col0, int kb, int ptid,
                                               bool col_a, bool col_b, bool f8) {
  const int pw = ptid >> 5, ln = ptid & 31;
  const int rows = min(ROWS, m - row0);
  const int cols = min(COLS, n - col0);
  if (f8) {
    const int k0 = kb * 2 * kBK;
    lsu_fill_operand<ROWS, 1>(as, a, lda, !col_a, rows, k, row0, k0, pw, ln);
    if (cols > 0) lsu_fill_operand<COLS, 1>(bs, b, ldb, col_b, cols, k, col0, k0, pw, ln);
  } else {
    const int k0 = kb * kBK;
    lsu_fill_operand<ROWS, 2>(as, a, lda, !col_a, rows, k, row0, k0, pw, ln);
    if (cols > 0) lsu_fill_operand<COLS, 2>(bs, b, ldb, col_b, cols, k, col0, k0, pw, ln);
  }
}

// Stage fill with 16-byte cp.async, for row-major A and B whose rows start 16-byte aligned but that
// have no tensor maps (problem sets prepared on the device): the same 128-byte-swizzled layouts the
// TMA loads write. A: ROWS rows of one 128-byte K row each (K-major); B: the K block's rows of COLS
// columns as 128-byte-wide chunks (MN-major). Bytes of A past K and K rows of B past K are
// zero-filled by the copies themselves (source size below 16); rows of A past M and columns of B
// past N are not written (they only reach accumulator rows and columns that are never stored).
// The copies are issued, not awaited: the caller tracks them on the stage's mbarrier.
template <int ROWS, int COLS, bool F8>
__device__ __forceinline__ void cpasync_fill_stage(uint32_t as, uint32_t bs, const uint8_t* a, int64_t lda_b,
                                                   const uint8_t* b, int64_t ldb_b, int m, int n, int k, int row0,
                                                   int col0, int kb, int ptid) {
  constexpr int EB = F8 ? 1 : 2;
  constexpr int KB = F8 ? 2 * kBK : kBK;  // K values per 128-byte row, K rows of B per stage
  constexpr int kSegs = COLS * EB / 16;   // 16-byte pieces of one K row of B
  constexpr int kRowsB = kProdThreads / kSegs;  // K rows of B per pass of the producer threads
  static_assert(kProdThreads == 64 && kSegs <= kProdThreads && kProdThreads % kSegs == 0, "copy split");
  const int k0 = kb * KB;
  // A: thread = (row mod 8, 16-byte piece j); its swizzled column and source size stay fixed.
  {
    const int r0 = ptid >> 3, j = ptid & 7;
    const int sb = max(0, min(16, (k - k0) * EB - 16 * j));
    const int rows = min(ROWS, m - row0);
    uint32_t d = as + static_cast<uint32_t>(r0 * 128 + ((j ^ r0) << 4));
    const uint8_t* src = a + static_cast<int64_t>(row0 + r0) * lda_b + static_cast<int64_t>(k0) * EB + 16 * j;
    const int64_t step = 8 * lda_b;
#pragma unroll 4
    for (int r = r0; r < rows; r += 8) {
      ptx::cp_async_16(d, sb > 0 ? src : a, static_cast<uint32_t>(sb));
      d += 1024;
      src += step;
    }
  }
  // B: thread = (K row mod kRowsB, 16-byte piece of the row); columns past N are not written.
  {
    const int seg = ptid % kSegs, kr0 = ptid / kSegs;
    const int c = seg * 16;
    const int cbytes = min(COLS, n - col0) * EB;
    if (c < cbytes) {
      const int cb = min(16, cbytes - c);
      const int kvalid = min(KB, k - k0);
      const int cs = (c & 127) >> 4;
      const uint32_t dcol = bs + static_cast<uint32_t>((c >> 7) * (KB * 128));
      const uint8_t* src = b + static_cast<int64_t>(k0 + kr0) * ldb_b + static_cast<int64_t>(col0) * EB + c;
      const int64_t step = kRowsB * ldb_b;
#pragma unroll 8
      for (int kr = kr0; kr < KB; kr += kRowsB) {
        const int sb = kr < kvalid ? cb : 0;
        ptx::cp_async_16(dcol + static_cast<uint32_t>(kr * 128 + ((cs ^ (kr & 7)) << 4)), sb > 0 ? src : b,
                         static_cast<uint32_t>(sb));
        src += step;
      }
    }
  }
}

// ---- mainloop helpers ------------------------------------------------------------------------
// Operand modes of a launch, one bit each: 8-bit A/B, A stored column-major (k x m: MN-major in
// shared memory), B stored column-major (n x k: K-major in shared memory). The per-stage helpers
// below take them as template parameters so that the geometry folds; the roles pick the
// instantiation once per K block.
constexpr int kModeF8 = 1;
constexpr int kModeACol = 2;
constexpr int kModeBCol = 4;

__device__ __forceinline__ int operand_mode(const KernelParams& p) {
  return (p.input_format >= GG_INPUT_E4M3 ? kModeF8 : 0) | ((p.layout & 1) ? kModeACol : 0) |
         ((p.layout & 2) ? kModeBCol : 0);
}

// The four MMAs of one K block (one shared-memory stage). F8: kind::f8f6f4, K = 32 per MMA, else
// kind::f16, K = 16. A K-major operand (row-major A, column-major B) is 128-byte rows of K, SW128,
// one MMA's K step = 32 bytes inside the row, 8-row groups 1024 bytes apart. An MN-major operand
// (row-major B, column-major A) is column chunks of 64 (16-bit) or 128 (8-bit) values x K rows,
// SW128: one MMA's K rows = 2048 / 4096 bytes, chunks 8192 / 16384 bytes apart (leading byte
// offset), 8-row K groups 1024 bytes apart (stride offset).
template <bool F8, bool ACol, bool BCol, bool kPair>
__device__ __forceinline__ void mma_kblock(uint32_t d_tmem, uint32_t a0, uint32_t b0, uint32_t idesc, bool first) {
  constexpr uint32_t kMnStep = F8 ? 4096u : 2048u;
  constexpr uint32_t kMnLbo = F8 ? 16384u : 8192u;
#pragma unroll
  for (int kk = 0; kk < kBK / kMmaK; ++kk) {
    const uint64_t adesc = ACol ? ptx::smem_desc_sw128(a0 + kk * kMnStep, kMnLbo, 1024u)
                                : ptx::smem_desc_sw128(a0 + kk * 32u, 16u, 1024u);
    const uint64_t bdesc = BCol ? ptx::smem_desc_sw128(b0 + kk * 32u, 16u, 1024u)
                                : ptx::smem_desc_sw128(b0 + kk * kMnStep, kMnLbo, 1024u);
    const uint32_t acc = (!first || kk != 0) ? 1u : 0u;
    if constexpr (kPair) {
      if constexpr (F8) ptx::tc_mma_f8_pair(d_tmem, adesc, bdesc, idesc, acc);
      else ptx::tc_mma_f16_pair(d_tmem, adesc, bdesc, idesc, acc);
    } else {
      if constexpr (F8) ptx::tc_mma_f8(d_tmem, adesc, bdesc, idesc, acc);
      else ptx::tc_mma_f16(d_tmem, adesc, bdesc, idesc, acc);
    }
  }
}

template <bool kPair>
__device__ __forceinline__ void mma_kblock_any(int mode, uint32_t d_tmem, uint32_t a0, uint32_t b0, uint32_t idesc,
                                               bool first) {
  switch (mode) {
    case 0: mma_kblock<false, false, false, kPair>(d_tmem, a0, b0, idesc, first); break;
    case 1: mma_kblock<true, false, false, kPair>(d_tmem, a0, b0, idesc, first); break;
    case 2: mma_kblock<false, true, false, kPair>(d_tmem, a0, b0, idesc, first); break;
    case 3: mma_kblock<true, true, false, kPair>(d_tmem, a0, b0, idesc, first); break;
    case 4: mma_kblock<false, false, true, kPair>(d_tmem, a0, b0, idesc, first); break;
    case 5: mma_kblock<true, false, true, kPair>(d_tmem, a0, b0, idesc, first); break;
    case 6: mma_kblock<false, true, true, kPair>(d_tmem, a0, b0, idesc, first); break;
    default: mma_kblock<true, true, true, kPair>(d_tmem, a0, b0, idesc, first); break;
  }
}

// The TMA loads of one stage, completing on `bar`: ROWS rows of A starting at a_row and COLS
// columns of B starting at col0, K block kb. F8: 128-deep K blocks and 128-wide MN chunks of 16 KB,
// else 64 and 64 (8 KB). A row-major: one box {kblock, ROWS}; column-major: one box {chunk, kblock}
// per chunk of rows. B row-major: one 3-D box of the whole stage when b_one_box, else one box per
// column chunk; column-major: one box {kblock, COLS}. kPair: the cta_group::2 form whose bytes
// complete on the leader's barrier.
template <int ROWS, int COLS, bool F8, bool ACol, bool BCol, bool kPair>
__device__ __forceinline__ void load_stage_tma(uint32_t a_dst, uint32_t b_dst, const CUtensorMap* ma,
                                               const CUtensorMap* mb, const CUtensorMap* mb3, uint32_t bar, int kb,
                                               int a_row, int col0, bool b_one_box) {
  constexpr int kKb = F8 ? 2 * kBK : kBK;
  constexpr int kCw = F8 ? 128 : 64;
  constexpr uint32_t kChunk = F8 ? 16384u : 8192u;
  auto load2 = [&](uint32_t dst, const CUtensorMap* map, int x, int y) {
    if constexpr (kPair) ptx::tma_load_2d_pair(dst, map, bar, x, y);
    else ptx::tma_load_2d(dst, map, bar, x, y);
  };
  if constexpr (ACol) {
#pragma unroll
    for (int j = 0; j < ROWS / kCw; ++j) load2(a_dst + j * kChunk, ma, a_row + j * kCw, kb * kKb);
  } else {
    load2(a_dst, ma, kb * kKb, a_row);
  }
  if constexpr (BCol) {
    load2(b_dst, mb, kb * kKb, col0);
  } else if (b_one_box) {
    if constexpr (kPair) ptx::tma_load_3d_pair(b_dst, mb3, bar, 0, kb * kKb, col0 / kCw);
    else ptx::tma_load_3d(b_dst, mb3, bar, 0, kb * kKb, col0 / kCw);
  } else {
#pragma unroll
    for (int j = 0; j < COLS / kCw; ++j) load2(b_dst + j * kChunk, mb, col0 + j * kCw, kb * kKb);
  }
}

template <int ROWS, int COLS, bool kPair>
__device__ __forceinline__ void load_stage_tma_any(int mode, uint32_t a_dst, uint32_t b_dst, const CUtensorMap* ma,
                                                   const CUtensorMap* mb, const CUtensorMap* mb3, uint32_t bar,
                                                   int kb, int a_row, int col0, bool b_one_box) {
#define GG_LOAD_STAGE(F8, AC, BC) \
  load_stage_tma<ROWS, COLS, F8, AC, BC, kPair>(a_dst, b_dst, ma, mb, mb3, bar, kb, a_row, col0, b_one_box)
  switch (mode) {
    case 0: GG_LOAD_STAGE(false, false, false); break;
    case 1: GG_LOAD_STAGE(true, false, false); break;
    case 2: GG_LOAD_STAGE(false, true, false); break;
    case 3: GG_LOAD_STAGE(true, true, false); break;
    case 4: GG_LOAD_STAGE(false, false, true); break;
    case 5: GG_LOAD_STAGE(true, false, true); break;
    case 6: GG_LOAD_STAGE(false, true, true); break;
    default: GG_LOAD_STAGE(true, true, true); break;
  }
#undef GG_LOAD_STAGE
}

// ---- the kernel --------------------------------------------------------------------------------
template <int BM, int BN>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_sm100_kernel(const __grid_constant__ KernelParams p) {
  using L = SmemLayout<BM, BN>;
  constexpr int S = L::kStages;
  constexpr int kAcc = L::kAcc;
  static_assert(BM == 64 || BM == 128, "tile rows");
  static_assert(BN == 64 || BN == 128 || BN == 256, "tile columns");

  extern __shared__ uint8_t smem_dyn[];
  const uint32_t raw_addr = ptx::smem_addr(smem_dyn);
  uint8_t* smem = smem_dyn + ((1024u - (raw_addr & 1023u)) & 1023u);
  const uint32_t sbase = ptx::smem_addr(smem);

  TileSlot* ring = reinterpret_cast<TileSlot*>(smem + L::kRingOffset);
  const uint32_t bar0 = sbase + L::kBarOffset;
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto accf_bar = [&](int b) { return bar0 + 8u * (2 * S + b); };
  auto acce_bar = [&](int b) { return bar0 + 8u * (2 * S + kAcc + b); };
  auto ringf_bar = [&](int r) { return bar0 + 8u * (2 * S + 2 * kAcc + r); };
  auto ringe_bar = [&](int r) { return bar0 + 8u * (2 * S + 2 * kAcc + kRing + r); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 2 * kAcc + 2 * kRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kMiscOffset);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 4);
  volatile int* prod_go = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 8);
  volatile int* epi_go = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 12);  // two words

  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(full_bar(s), 1);
      ptx::mbar_init(empty_bar(s), 1);
    }
    for (int b = 0; b < kAcc; ++b) {
      ptx::mbar_init(accf_bar(b), 1);
      ptx::mbar_init(acce_bar(b), kEpiWarps);
    }
    for (int r = 0; r < kRing; ++r) {
      ptx::mbar_init(ringf_bar(r), 1);
      ptx::mbar_init(ringe_bar(r), kRingConsumerWarps);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *prod_go = 0;
    epi_go[0] = 0;
    epi_go[1] = 0;
    ptx::fence_mbar_init();
  }
  if (warp == kMmaWarp) {
    ptx::tmem_alloc(ptx::smem_addr(tmem_slot), L::kTmemCols);
    ptx::tmem_relinquish();
  }
  ptx::tc_fence_before_sync();
  __syncthreads();
  ptx::tc_fence_after_sync();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // A CUDA-core launch of the same executor may follow (its small problems): it works on other
  // problems' outputs, so it may take the SMs this grid leaves free.
  if (threadIdx.x == 0) ptx::launch_dependents();

  const DeviceProblemDesc* problems = p.single_mode ? &p.single_desc : p.problems;
  const CUtensorMap* maps = p.single_mode ? p.single_maps : p.tmaps;
  const unsigned long long tmo = p.timeout_ns;

  if (warp == kSchedWarp) {
    // ======================= scheduler =======================
    SchedState ss;
    sched_init(p, ss, static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x), lane);  // first claim in flight
    prefetch_tables_l2(p, static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x), lane);
    for (int t = 0;; ++t) {
      const int slot = t % kRing;
      const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
      int ok = 1;
      if (lane == 0) ok = wait_phase(ringe_bar(slot), par ^ 1u, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_SCHEDULER);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      TileSlot* s = &ring[slot];
      int pidx = -1, tile_m = 0, tile_n = 0;
      if (next_tile(p, ss, problems, lane, static_cast<int>(gridDim.x), pidx, tile_m, tile_n)) {
        if (lane < kDescWords) reinterpret_cast<int*>(&s->desc)[lane] = ss.w;
        const unsigned fl = static_cast<unsigned>(
            __shfl_sync(0xffffffffu, ss.w, static_cast<int>(offsetof(DeviceProblemDesc, flags) / 4)));
        const int slot_maps = __shfl_sync(0xffffffffu, ss.w, static_cast<int>(offsetof(DeviceProblemDesc, map_slot) / 4));
        prefetch_problem_maps(maps, slot_maps, fl, lane);
      } else {
        pidx = -1;
      }
      if (lane == 0) {
        s->problem = pidx;
        s->tile_m = tile_m;
        s->tile_n = tile_n;
      }
      __syncwarp();
      if (lane == 0) {
        __threadfence_block();
        ptx::mbar_arrive(ringf_bar(slot));
      }
      if (pidx < 0) break;
    }
  } else if (warp >= kProdWarp0) {
    // ======================= producers =======================
    const int ptid = static_cast<int>(threadIdx.x) - kProdWarp0 * 32;
    // Stage geometry: a 128-byte swizzle row holds 64 16-bit or 128 8-bit values, so a K block
    // is 64 (FP16/BF16) or 128 (FP8) deep and an MN chunk 64 or 128 wide (load_stage_tma); the
    // stage's bytes are the same either way.
    const int mode = operand_mode(p);
    const bool f8 = (mode & kModeF8) != 0;
    uint32_t it = 0;  // global k-block counter: stage = it % S, phase = (it / S) & 1
    bool aborted = false;
    for (int t = 0;; ++t) {
      const int slot = t % kRing;
      const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
      int ok = 1;
      if (lane == 0) ok = wait_phase(ringf_bar(slot), par, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_PRODUCER);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      const TileSlot* s = &ring[slot];
      const int q = s->problem;
      const int tile_m = s->tile_m, tile_n = s->tile_n;
      const int kb_count = s->desc.k_blocks;
      const unsigned flags = s->desc.flags;
      const int m = s->desc.m, n = s->desc.n, k = s->desc.k;
      const __half* a = s->desc.a;
      const __half* b = s->desc.b;
      const int lda = s->desc.lda, ldb = s->desc.ldb;
      const int a_row = s->desc.tma_row0 + tile_m * BM;  // first A row of the tile in the A map
      const int map_slot = s->desc.map_slot;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ringe_bar(slot));
      if (q < 0) break;

      if (flags & grouped_gemm::kFlagTmaAB) {
        if (ptid == 0) {
          const CUtensorMap* ma = maps + kMapsPerProblem * map_slot + kMapA;
          const CUtensorMap* mb = maps + kMapsPerProblem * map_slot + kMapB;
          const CUtensorMap* mb3 = maps + kMapsPerProblem * map_slot + kMapB3;
          // One 3-D box loads the whole B stage when every column chunk of the tile lies inside N;
          // an edge tile loads chunk by chunk so columns past N are zero-filled.
          const bool b_one_box = (flags & grouped_gemm::kFlagTmaB3) && (tile_n + 1) * BN <= n;
          for (int kb = 0; kb < kb_count; ++kb) {
            const int st = static_cast<int>(it % S);
            const uint32_t ph = (it / S) & 1u;
            if (!wait_phase(empty_bar(st), ph ^ 1u, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_PRODUCER)) {
              aborted = true;
              break;
            }
            const uint32_t a_dst = sbase + static_cast<uint32_t>(st * L::kStageBytes);
            const uint32_t b_dst = a_dst + L::kABytes;
            ptx::mbar_arrive_expect_tx(full_bar(st), L::kATxBytes + L::kBTxBytes);
            load_stage_tma_any<BM, BN, false>(mode, a_dst, b_dst, ma, mb, mb3, full_bar(st), kb, a_row, tile_n * BN,
                                              b_one_box);
            ++it;
          }
        } else {
          it += static_cast<uint32_t>(kb_count);
        }
        if (aborted) break;
      } else if (flags & grouped_gemm::kFlagCpAsync) {
        // 16-byte cp.async: every producer thread issues its copies and ties them to the stage's
        // full barrier (one pending arrival each, received when its copies land); after a named
        // barrier, one thread adds the barrier's expected arrival. The MMA thread fences the
        // generic-proxy writes before its tensor-core reads.
        for (int kb = 0; kb < kb_count; ++kb) {
          const int st = static_cast<int>(it % S);
          const uint32_t ph = (it / S) & 1u;
          if (ptid == 0) {
            const bool got = wait_phase(empty_bar(st), ph ^ 1u, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_PRODUCER);
            *prod_go = got ? 1 : 0;
          }
          ptx::named_bar_sync(1, kProdThreads);
          if (!*prod_go) {
            aborted = true;
            break;
          }
          const uint32_t as = sbase + static_cast<uint32_t>(st * L::kStageBytes);
          const uint32_t bs = as + L::kABytes;
          const int64_t lda_b = static_cast<int64_t>(lda) * (f8 ? 1 : 2), ldb_b = static_cast<int64_t>(ldb) * (f8 ? 1 : 2);
          if (f8)
            cpasync_fill_stage<BM, BN, true>(as, bs, reinterpret_cast<const uint8_t*>(a), lda_b,
                                             reinterpret_cast<const uint8_t*>(b), ldb_b, m, n, k, tile_m * BM,
                                             tile_n * BN, kb, ptid);
          else
            cpasync_fill_stage<BM, BN, false>(as, bs, reinterpret_cast<const uint8_t*>(a), lda_b,
                                              reinterpret_cast<const uint8_t*>(b), ldb_b, m, n, k, tile_m * BM,
                                              tile_n * BN, kb, ptid);
          ptx::cp_async_mbar_arrive(full_bar(st));
          ptx::named_bar_sync(1, kProdThreads);  // every pending arrival is registered
          if (ptid == 0) ptx::mbar_arrive(full_bar(st));
          ++it;
        }
        if (aborted) break;
      } else {
        for (int kb = 0; kb < kb_count; ++kb) {
          const int st = static_cast<int>(it % S);
          const uint32_t ph = (it / S) & 1u;
          if (ptid == 0) {
            const bool got = wait_phase(empty_bar(st), ph ^ 1u, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_PRODUCER);
            *prod_go = got ? 1 : 0;
          }
          ptx::named_bar_sync(1, kProdThreads);
          if (!*prod_go) {
            aborted = true;
            break;
          }
          uint8_t* as = smem + st * L::kStageBytes;
          uint8_t* bs = as + L::kABytes;
          lsu_fill_stage<BM, BN>(as, bs, a, lda, b, ldb, m, n, k, tile_m * BM, tile_n * BN, kb, ptid,
                                 (mode & kModeACol) != 0, (mode & kModeBCol) != 0, f8);
          ptx::fence_proxy_async_smem();
          ptx::named_bar_sync(1, kProdThreads);
          if (ptid == 0) ptx::mbar_arrive(full_bar(st));
          ++it;
        }
        if (aborted) break;
      }
    }
    ptx::cp_async_wait_all();  // this thread's 16-byte copies, if any, have landed
    if ((aborted || *abort_flag) && ptid == 0) {
      // TMA loads issued for the last stages may still be landing: wait for them before exit
      // (bounded: a stage that was never issued just runs out its short limit).
      const uint32_t n_back = it < static_cast<uint32_t>(S) ? it : static_cast<uint32_t>(S);
      for (uint32_t j = 1; j <= n_back; ++j) {
        const uint32_t i2 = it - j;
        wait_drain(full_bar(static_cast<int>(i2 % S)), (i2 / S) & 1u, 100000000ull);
      }
    }
  } else if (warp == kMmaWarp) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      const int mode = operand_mode(p);
      const uint32_t kIdesc = ptx::idesc_f32acc(
          kMmaM, BN, static_cast<uint32_t>((mode & kModeF8) ? p.input_format - GG_INPUT_E4M3 : p.input_format),
          (mode & kModeACol) != 0, (mode & kModeBCol) == 0);
      uint32_t it = 0;
      for (int t = 0;; ++t) {
        const int slot = t % kRing;
        const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
        if (!wait_phase(ringf_bar(slot), par, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_MMA)) break;
        const int q = ring[slot].problem;
        const int kb_count = ring[slot].desc.k_blocks;
        const bool cpasync_tile = (ring[slot].desc.flags & grouped_gemm::kFlagCpAsync) != 0u;
        ptx::mbar_arrive(ringe_bar(slot));
        if (q < 0) break;
        const int buf = t % kAcc;
        if (!wait_phase(acce_bar(buf), (static_cast<uint32_t>(t / kAcc) & 1u) ^ 1u, abort_flag, p.status, tmo,
                        GG_STATUS_TIMEOUT_MMA))
          break;
        ptx::tc_fence_after_sync();
        if (kb_count <= 0) {
          ptx::mbar_arrive(accf_bar(buf));  // K = 0: the epilogue uses a zero accumulator
          continue;
        }
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        bool aborted = false;
        for (int kb = 0; kb < kb_count; ++kb) {
          const int st = static_cast<int>(it % S);
          const uint32_t ph = (it / S) & 1u;
          if (!wait_phase(full_bar(st), ph, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_MMA)) {
            aborted = true;
            break;
          }
          ptx::tc_fence_after_sync();
          if (cpasync_tile) ptx::fence_proxy_async_smem();  // cp.async wrote the stage (generic proxy)
          const uint32_t a0 = sbase + static_cast<uint32_t>(st * L::kStageBytes);
          const uint32_t b0 = a0 + L::kABytes;
          mma_kblock_any<false>(mode, d_tmem, a0, b0, kIdesc, kb == 0);
          ptx::tc_commit(empty_bar(st));  // stage is free once these MMAs have read it
          ++it;
        }
        if (aborted) break;
        ptx::tc_commit(accf_bar(buf));  // accumulator ready for the epilogue
      }
      // Every MMA issued must complete before TMEM is freed (matters on the abort path).
      ptx::tc_commit(drain_bar);
      wait_drain(drain_bar, 0u, 100000000ull);
    }
    __syncwarp();
  } else {
    // ======================= epilogue (warps 0-7) =======================
    // The eight warps move in step: thread 0 waits on the ring and accumulator barriers and
    // broadcasts the outcome through epi_go after a named barrier, so a timed-out wait ends
    // the loop in every warp at the same point (no warp is left inside a named barrier).
    const int qw = warp & 3;    // TMEM lane quarter = tile rows 32*qw .. 32*qw+31
    const int half = warp >> 2;  // which half of the tile's columns this warp stores
    const int et = static_cast<int>(threadIdx.x);
    uint32_t store_count = 0;
    for (int t = 0;; ++t) {
      const int slot = t % kRing;
      const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
      if (et == 0)
        epi_go[0] = wait_phase(ringf_bar(slot), par, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_EPILOGUE) ? 1 : 0;
      ptx::named_bar_sync(2, kEpiThreads);
      if (!epi_go[0]) break;
      const TileSlot* s = &ring[slot];
      const int q = s->problem;
      const int tile_m = s->tile_m, tile_n = s->tile_n;
      const int m = s->desc.m, n = s->desc.n;
      const int kb_count = s->desc.k_blocks;
      const unsigned flags = s->desc.flags;
      EpiTile e;
      e.flags = flags;
      e.alpha = s->desc.alpha;
      e.beta = s->desc.beta;
      e.c = s->desc.c;
      e.ldc = s->desc.ldc;
      e.d = s->desc.d;
      e.ldd = s->desc.ldd;
      e.tma_row0 = s->desc.tma_row0;
      const int map_slot = s->desc.map_slot;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ringe_bar(slot));
      if (q < 0) break;
      const int nchunks = min(BN / 32, (n - tile_n * BN + 31) / 32);  // tile-uniform
      int c_begin, c_end;
      epilogue_chunk_range(nchunks, half, c_begin, c_end);
      // Warps whose 32 rows lie past BM (64-row tiles) or past M store nothing.
      e.row0 = qw * 32 < BM ? tile_m * BM + qw * 32 : m;
      e.m = m;
      e.n = n;
      e.col0 = tile_n * BN;
      e.c_begin = c_begin;
      e.c_end = c_end;
      e.kb_count = kb_count;
      e.bias = p.bias ? p.bias[map_slot] : nullptr;
      e.act = p.activation;
      e.md = maps + kMapsPerProblem * map_slot + kMapD;
      epilogue_bias_prefetch(e, lane);  // its latency hides behind the accumulator wait
      const int buf = t % kAcc;
      if (et == 0)
        epi_go[1] = wait_phase(accf_bar(buf), static_cast<uint32_t>(t / kAcc) & 1u, abort_flag, p.status, tmo,
                               GG_STATUS_TIMEOUT_EPILOGUE) ? 1 : 0;
      ptx::named_bar_sync(2, kEpiThreads);
      if (!epi_go[1]) break;
      ptx::tc_fence_after_sync();

      const uint32_t t_addr = tmem_base + static_cast<uint32_t>(buf * BN) + (static_cast<uint32_t>(qw * 32) << 16);
      epilogue_warp(p.output_format, smem + L::kEpiOffset + warp * kEpiWarpBytes, store_count, t_addr, lane, e,
                    [&] { ptx::mbar_arrive(acce_bar(buf)); });
    }
    if (lane == 0) ptx::bulk_wait_all();  // every warp issues its own TMA stores
    __syncwarp();
  }

  __syncthreads();
  if (threadIdx.x == 0) finish_launch(p);
  if (warp == kMmaWarp) {
    ptx::tc_fence_after_sync();
    ptx::tmem_dealloc(tmem_base, L::kTmemCols);
  }
}

// Runs the bounded wait on an mbarrier nothing completes; records the resulting status.
__global__ void wait_timeout_selftest_kernel(int* status, unsigned long long timeout_ns) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_word;
  if (threadIdx.x == 0) {
    ptx::mbar_init(ptx::smem_addr(&bar), 1);
    abort_word = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const bool ok = wait_phase(ptx::smem_addr(&bar), 0u, reinterpret_cast<volatile int*>(&abort_word), status,
                               timeout_ns, GG_STATUS_TIMEOUT_MMA);
    if (ok) atomicOr(status, 0x100);  // would mean the wait returned without the barrier completing
  }
}

}  // namespace gg
