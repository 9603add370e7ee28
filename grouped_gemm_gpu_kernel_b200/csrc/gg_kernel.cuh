// gg_kernel.cuh -- the persistent grouped GEMM kernel for B200 (sm_100a).
//
// One CTA per SM (shared memory > half an SM's), 256 threads in five warp roles:
//
//   warps 0-3  epilogue   TMEM -> registers (tcgen05.ld), D = alpha*acc + beta*C, then per 32-column
//                         chunk one 128-byte-swizzled staging tile of all BM rows that a single
//                         TMA store writes out (clipped at the problem edge), or masked direct
//                         stores when D is not TMA-eligible. Warp w reads TMEM lanes
//                         32w..32w+31 = tile rows 32w..32w+31.
//   warp 4     MMA        allocates 2*BN TMEM columns (two accumulators, so the epilogue of one
//                         tile overlaps the mainloop of the next); one thread issues
//                         tcgen05.mma.kind::f16 (M=128, N=BN, K=16) and tcgen05.commit.
//   warp 5     scheduler  claims global tile indices with atomicAdd (the reference's device
//                         scheduler, src/grouped_gemm.cu:640-675), finds the owning problem with a
//                         warp-parallel 32-ary search of tile_offsets (same answer as the
//                         reference's binary search, src/grouped_gemm.cu:219-234), copies the
//                         problem record into a 4-deep shared-memory ring read by every role.
//   warps 6-7  producers  fill a multi-stage ring of A/B shared-memory tiles: one thread issues
//                         TMA tensor loads for aligned problems (one box for A and, for tiles
//                         inside N, one 3-D box for all of B); all 64 threads load with zero
//                         fill for problems whose base or leading dimension TMA cannot take (the
//                         reference's scalar zero-fill path, src/grouped_gemm.cu:273-371), writing
//                         the same 128-byte-swizzled layout the TMA would.
//
// Shared-memory layout per stage: A as 128 rows x 64 K (K-major, 128-byte rows, SW128) and B as
// BN/64 column chunks of 64 K rows x 64 N (MN-major, SW128). A 64-row tile (reference shapes
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

// ---- producer helpers ------------------------------------------------------------------------
// Eight FP16 values of row `row`, columns col..col+7, with zero fill outside rows x cols.
__device__ __forceinline__ uint4 load8_zero_fill(const __half* base, int ld, int row, int col, int rows, int cols) {
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (row < rows && col < cols) {
    const unsigned short* src =
        reinterpret_cast<const unsigned short*>(base) + static_cast<int64_t>(row) * ld + col;
    if (col + 8 <= cols && (reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
      v = __ldg(reinterpret_cast<const uint4*>(src));
    } else {
      uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const uint32_t h = (col + i < cols) ? static_cast<uint32_t>(__ldg(src + i)) : 0u;
        w[i >> 1] |= h << ((i & 1) * 16);
      }
      v = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
  return v;
}

// ---- the kernel --------------------------------------------------------------------------------
template <int BM, int BN>
__global__ void __launch_bounds__(kThreads, 1) grouped_gemm_sm100_kernel(const __grid_constant__ KernelParams p) {
  using L = SmemLayout<BM, BN>;
  constexpr int S = L::kStages;
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
  auto acce_bar = [&](int b) { return bar0 + 8u * (2 * S + 2 + b); };
  auto ringf_bar = [&](int r) { return bar0 + 8u * (2 * S + 4 + r); };
  auto ringe_bar = [&](int r) { return bar0 + 8u * (2 * S + 4 + kRing + r); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 4 + 2 * kRing);
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
    for (int b = 0; b < 2; ++b) {
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

  const DeviceProblemDesc* problems = p.single_mode ? &p.single_desc : p.problems;
  const CUtensorMap* maps = p.single_mode ? p.single_maps : p.tmaps;
  const unsigned long long tmo = p.timeout_ns;

  if (warp == kSchedWarp) {
    // ======================= scheduler =======================
    int static_next = static_cast<int>(blockIdx.x);
    for (int t = 0;; ++t) {
      const int slot = t % kRing;
      const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
      int ok = 1;
      if (lane == 0) ok = wait_phase(ringe_bar(slot), par ^ 1u, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_SCHEDULER);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      TileSlot* s = &ring[slot];
      int pidx = -1, tile_m = 0, tile_n = 0;
      for (;;) {
        int tile = 0;
        if (lane == 0) {
          if (p.single_mode) {
            tile = static_next;
            static_next += static_cast<int>(gridDim.x);
          } else {
            tile = atomicAdd(p.tile_counter, 1);
          }
        }
        tile = __shfl_sync(0xffffffffu, tile, 0);
        if (tile >= p.total_tiles) break;
        const int q = p.single_mode ? 0 : find_problem_warp(p.tile_offsets, p.problem_count, tile, lane);
        const int local = tile - (p.single_mode ? 0 : __ldg(p.tile_offsets + q));
        const int* src = reinterpret_cast<const int*>(problems + q);
        const int w = lane < kDescWords ? src[lane] : 0;
        const int tiles_m = __shfl_sync(0xffffffffu, w, static_cast<int>(offsetof(DeviceProblemDesc, tiles_m) / 4));
        const int tiles_n = __shfl_sync(0xffffffffu, w, static_cast<int>(offsetof(DeviceProblemDesc, tiles_n) / 4));
        // A tile index outside its problem's tile grid (a prepared set inconsistent with the
        // config) is skipped, as the reference kernel does (src/grouped_gemm.cu:662-672).
        if (local < 0 || tiles_m <= 0 || tiles_n <= 0 || local >= tiles_m * tiles_n) continue;
        raster_tile(local, tiles_m, tiles_n, p.raster_group, tile_m, tile_n);
        if (lane < kDescWords) reinterpret_cast<int*>(&s->desc)[lane] = w;
        // Warm the tensor maps this tile will use (only those that were encoded) while the tile
        // waits in the ring.
        const unsigned fl = static_cast<unsigned>(
            __shfl_sync(0xffffffffu, w, static_cast<int>(offsetof(DeviceProblemDesc, flags) / 4)));
        const bool map_valid = (lane == kMapA || lane == kMapB) ? (fl & grouped_gemm::kFlagTmaAB) != 0u
                               : lane == kMapB3                 ? (fl & grouped_gemm::kFlagTmaB3) != 0u
                               : lane == kMapD                  ? (fl & grouped_gemm::kFlagTmaD) != 0u
                                                                : false;
        if (map_valid) ptx::prefetch_tensormap(maps + kMapsPerProblem * q + lane);
        pidx = q;
        break;
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
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ringe_bar(slot));
      if (q < 0) break;

      if (flags & grouped_gemm::kFlagTmaAB) {
        if (ptid == 0) {
          const CUtensorMap* ma = maps + kMapsPerProblem * q + kMapA;
          const CUtensorMap* mb = maps + kMapsPerProblem * q + kMapB;
          const CUtensorMap* mb3 = maps + kMapsPerProblem * q + kMapB3;
          // One 3-D box loads the whole B stage when every 64-column chunk of the tile lies
          // inside N; an edge tile loads chunk by chunk so columns past N are zero-filled.
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
            ptx::tma_load_2d(a_dst, ma, full_bar(st), kb * kBK, tile_m * BM);
            if (b_one_box) {
              ptx::tma_load_3d(b_dst, mb3, full_bar(st), 0, kb * kBK, tile_n * (BN / 64));
            } else {
#pragma unroll
              for (int j = 0; j < BN / 64; ++j)
                ptx::tma_load_2d(b_dst + j * 8192u, mb, full_bar(st), tile_n * BN + j * 64, kb * kBK);
            }
            ++it;
          }
        } else {
          it += static_cast<uint32_t>(kb_count);
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
          for (int idx = ptid; idx < BM * 8; idx += kProdThreads) {
            const int r = idx >> 3, j = idx & 7;
            const uint4 v = load8_zero_fill(a, lda, tile_m * BM + r, kb * kBK + j * 8, m, k);
            *reinterpret_cast<uint4*>(as + r * 128 + ((j ^ (r & 7)) << 4)) = v;
          }
          constexpr int kChunksPerRow = BN / 8;
          for (int idx = ptid; idx < kBK * kChunksPerRow; idx += kProdThreads) {
            const int kr = idx / kChunksPerRow, jn = idx % kChunksPerRow;
            const int c = jn >> 3, j = jn & 7;
            const uint4 v = load8_zero_fill(b, ldb, kb * kBK + kr, tile_n * BN + jn * 8, k, n);
            *reinterpret_cast<uint4*>(bs + c * 8192 + kr * 128 + ((j ^ (kr & 7)) << 4)) = v;
          }
          ptx::fence_proxy_async_smem();
          ptx::named_bar_sync(1, kProdThreads);
          if (ptid == 0) ptx::mbar_arrive(full_bar(st));
          ++it;
        }
        if (aborted) break;
      }
    }
    if (aborted && ptid == 0) {
      // TMA loads issued for the last stages may still be landing: wait for them before exit.
      const uint32_t n_back = it < static_cast<uint32_t>(S) ? it : static_cast<uint32_t>(S);
      for (uint32_t j = 1; j <= n_back; ++j) {
        const uint32_t i2 = it - j;
        wait_drain(full_bar(static_cast<int>(i2 % S)), (i2 / S) & 1u, 100000000ull);
      }
    }
  } else if (warp == kMmaWarp) {
    // ======================= MMA issuer =======================
    if (lane == 0) {
      constexpr uint32_t kIdesc = ptx::idesc_f16_f32_kA_mnB(kMmaM, BN);
      uint32_t it = 0;
      for (int t = 0;; ++t) {
        const int slot = t % kRing;
        const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
        if (!wait_phase(ringf_bar(slot), par, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_MMA)) break;
        const int q = ring[slot].problem;
        const int kb_count = ring[slot].desc.k_blocks;
        ptx::mbar_arrive(ringe_bar(slot));
        if (q < 0) break;
        const int buf = t & 1;
        if (!wait_phase(acce_bar(buf), (static_cast<uint32_t>(t >> 1) & 1u) ^ 1u, abort_flag, p.status, tmo,
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
          const uint32_t a0 = sbase + static_cast<uint32_t>(st * L::kStageBytes);
          const uint32_t b0 = a0 + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kMmaK; ++kk) {
            // A: K-major SW128, 16-element K step = 32 bytes inside the 128-byte row;
            //    8-row groups 1024 bytes apart.
            // B: MN-major SW128, 16-row K step = 2048 bytes; 64-column chunks 8192 bytes
            //    apart (leading byte offset), 8-row K groups 1024 bytes apart (stride offset).
            const uint64_t adesc = ptx::smem_desc_sw128(a0 + kk * 32u, 16u, 1024u);
            const uint64_t bdesc = ptx::smem_desc_sw128(b0 + kk * 2048u, 8192u, 1024u);
            ptx::tc_mma_f16(d_tmem, adesc, bdesc, kIdesc, (kb | kk) != 0 ? 1u : 0u);
          }
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
    // ======================= epilogue (warps 0-3) =======================
    // The four warps move in step: thread 0 waits on the ring and accumulator barriers and
    // broadcasts the outcome through epi_go after a named barrier, so a timed-out wait ends
    // the loop in every warp at the same point (no warp is left inside a named barrier).
    const int qw = warp;  // TMEM lane quarter = tile rows 32*qw .. 32*qw+31
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
      const float alpha = s->desc.alpha, beta = s->desc.beta;
      const float* cptr = s->desc.c;
      float* dptr = s->desc.d;
      const int ldc = s->desc.ldc, ldd = s->desc.ldd;
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(ringe_bar(slot));
      if (q < 0) break;
      const int buf = t & 1;
      if (et == 0)
        epi_go[1] = wait_phase(accf_bar(buf), static_cast<uint32_t>(t >> 1) & 1u, abort_flag, p.status, tmo,
                               GG_STATUS_TIMEOUT_EPILOGUE) ? 1 : 0;
      ptx::named_bar_sync(2, kEpiThreads);
      if (!epi_go[1]) break;
      ptx::tc_fence_after_sync();

      const int row0 = tile_m * BM + qw * 32;
      const int row = row0 + lane;
      const int col0 = tile_n * BN;
      const bool warp_rows = qw * 32 < BM && row0 < m;  // warp-uniform
      const int nchunks = min(BN / 32, (n - col0 + 31) / 32);  // tile-uniform
      const uint32_t t_addr = tmem_base + static_cast<uint32_t>(buf * BN) + (static_cast<uint32_t>(qw * 32) << 16);
      const bool read_c = (flags & grouped_gemm::kFlagReadC) != 0u;
      const bool tma_d = (flags & grouped_gemm::kFlagTmaD) != 0u;
      const CUtensorMap* md = maps + kMapsPerProblem * q + kMapD;

      for (int c = 0; c < nchunks; ++c) {
        float acc[32];
        if (warp_rows && kb_count > 0) {
          uint32_t r[32];
          ptx::tmem_load_32cols(t_addr + static_cast<uint32_t>(c * 32), r);
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = __uint_as_float(r[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) acc[j] = 0.0f;
        }
        if (c == nchunks - 1) {
          // Last read of this accumulator: hand it back to the MMA warp before the stores.
          ptx::tc_fence_before_sync();
          __syncwarp();
          if (lane == 0) ptx::mbar_arrive(acce_bar(buf));
        }
        const int cc = col0 + c * 32;
        float cv[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) cv[j] = 0.0f;
        if (read_c && warp_rows && row < m) {
          const float* crow = cptr + static_cast<int64_t>(row) * ldc + cc;
          if ((flags & grouped_gemm::kFlagCVec) && cc + 32 <= n) {
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              const float4 v = *reinterpret_cast<const float4*>(crow + 4 * j4);
              cv[4 * j4] = v.x;
              cv[4 * j4 + 1] = v.y;
              cv[4 * j4 + 2] = v.z;
              cv[4 * j4 + 3] = v.w;
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (cc + j < n) cv[j] = crow[j];
          }
        }
        // D = alpha * acc + beta * C, C taken as 0 when it is not read
        // (reference src/grouped_gemm.cu:614-621).
        float out[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) out[j] = alpha * acc[j] + beta * cv[j];

        if (tma_d) {
          // All BM rows of this 32-column chunk go out in one TMA store from a shared staging
          // tile (two tiles alternate; the store that used this one two chunks ago must have
          // finished reading it). Rows past M are clipped by the tensor map.
          uint8_t* stile = smem + L::kEpiOffset + static_cast<int>(store_count & 1u) * kEpiTileBytes;
          if (et == 0) ptx::bulk_wait_read_le1();
          ptx::named_bar_sync(2, kEpiThreads);
          if (qw * 32 < BM) {
            const int r = qw * 32 + lane;
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {
              *reinterpret_cast<float4*>(stile + r * 128 + ((j4 ^ (r & 7)) << 4)) =
                  make_float4(out[4 * j4], out[4 * j4 + 1], out[4 * j4 + 2], out[4 * j4 + 3]);
            }
          }
          ptx::fence_proxy_async_smem();
          ptx::named_bar_sync(2, kEpiThreads);
          if (et == 0) {
            ptx::tma_store_2d(md, ptx::smem_addr(stile), cc, tile_m * BM);
            ptx::bulk_commit_group();
          }
          ++store_count;
        } else if (warp_rows && row < m) {
          float* drow = dptr + static_cast<int64_t>(row) * ldd + cc;
          if ((flags & grouped_gemm::kFlagDVec) && cc + 32 <= n) {
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4)
              *reinterpret_cast<float4*>(drow + 4 * j4) =
                  make_float4(out[4 * j4], out[4 * j4 + 1], out[4 * j4 + 2], out[4 * j4 + 3]);
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (cc + j < n) drow[j] = out[j];
          }
        }
      }
      if (nchunks <= 0) {
        ptx::tc_fence_before_sync();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive(acce_bar(buf));
      }
    }
    if (et == 0) ptx::bulk_wait_all();
    __syncwarp();
  }

  __syncthreads();
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
