// gg_kernel_pair.cuh -- the persistent grouped GEMM kernel on CTA pairs (tcgen05 cta_group::2).
//
// A cluster of two CTAs on two SMs computes one 256 x BN output tile with M=256 MMAs: CTA rank r
// loads rows [256*tile_m + 128*r, +128) of A and columns [BN*tile_n + (BN/2)*r, +BN/2) of B into
// its own shared memory, the MMA reads both halves of both operands and leaves rows
// 128*r .. 128*r+127 of the accumulator in CTA r's tensor memory, and each CTA's epilogue stores
// its own 128 rows. Per SM this moves 3/4 (BN=256) or 2/3 (BN=128) of the operand bytes a one-CTA
// 128 x BN tile moves for the same tensor work, so the same shared memory holds more pipeline
// stages (6 x 32 KB or 8 x 24 KB) and covers more load latency.
//
// Roles are those of gg_kernel.cuh, with the pair split:
//   leader (rank 0)  the scheduler warp claims tiles and writes each ring slot into both CTAs'
//                    shared memory (remote stores, then a cluster-release arrive on the peer's
//                    ring barrier); the MMA thread issues tcgen05.mma.cta_group::2 and commits to
//                    the empty / accumulator barriers of both CTAs at once (commit multicast).
//   both CTAs        producers load their own halves; the TMA byte counts complete on the
//                    leader's stage barrier (cp.async.bulk.tensor.cta_group::2, no multicast) and
//                    each CTA's producer adds one arrival there, so TMA and zero-fill stages use
//                    the same count. Epilogues drain their own TMEM; the peer's release of an
//                    accumulator is a remote arrive on the leader's barrier.
// Waits stay bounded as in the one-CTA kernel; a cluster barrier precedes TMEM release and exit so
// neither CTA leaves while the other may still touch its shared memory.
#pragma once

#include "gg_kernel.cuh"

namespace gg {

template <int BN>
struct PairLayout {
  static constexpr int kBHalf = BN / 2;
  static constexpr int kStages = BN >= 256 ? 6 : 8;
  static constexpr int kAcc = AccCount<BN>::value;  // TMEM accumulators (BN columns each)
  static constexpr int kABytes = 128 * 128;     // 128 rows x 64 K
  static constexpr int kBBytes = kBHalf * 128;  // BN/2 columns (chunks of 64) x 64 K
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiOffset = kStages * kStageBytes;
  static constexpr int kEpiBytes = 2 * kEpiTileBytes;
  static constexpr int kRingOffset = kEpiOffset + kEpiBytes;
  static constexpr int kBarOffset = kRingOffset + kRing * static_cast<int>(sizeof(TileSlot));
  static constexpr int kNumBars = 2 * kStages + 2 * kAcc + 2 * kRing + 1;
  static constexpr int kMiscOffset = kBarOffset + kNumBars * 8;
  static constexpr int kBytes = kMiscOffset + 32;
  static constexpr int kDynamicSmem = kBytes + 1024;
  static constexpr uint32_t kStageTxPair = 2u * static_cast<uint32_t>(kStageBytes);  // both CTAs' halves
  static constexpr uint32_t kTmemCols = kAcc * BN;
  static_assert(kRingOffset % 1024 == 0, "stage and staging tiles stay 1024-byte aligned");
  static_assert(kDynamicSmem <= 232448, "fits the 227 KB opt-in shared memory of a CTA");
  static_assert(kDynamicSmem > 232448 / 2 + 1024, "one CTA per SM");
};

constexpr int kPairRingConsumersLeader = kEpiWarps + 1 + 2;  // epilogue, MMA, producers
constexpr int kPairRingConsumersPeer = kEpiWarps + 2;        // epilogue, producers

// Bounded wait with cluster-scope acquire (ring slots the leader wrote into this CTA remotely).
__device__ __noinline__ bool wait_slow_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* status,
                                               unsigned long long timeout_ns, int code) {
  const uint64_t t0 = ptx::global_timer_ns();
  for (uint32_t i = 0;; ++i) {
    if (ptx::mbar_try_wait_cluster(bar, parity)) return true;
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

__device__ __forceinline__ bool wait_phase_cluster(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                                   int* status, unsigned long long timeout_ns, int code) {
  if (ptx::mbar_try_wait_cluster(bar, parity)) return true;
  return wait_slow_cluster(bar, parity, abort_flag, status, timeout_ns, code);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_gemm_sm100_pair_kernel(const __grid_constant__ KernelParams p) {
  using L = PairLayout<BN>;
  constexpr int S = L::kStages;
  constexpr int kAcc = L::kAcc;
  constexpr int BM = 256;          // output rows per pair tile
  constexpr int HB = BN / 2;       // B columns per CTA
  static_assert(BN == 128 || BN == 256, "pair tile columns");

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
  volatile int* epi_go = reinterpret_cast<volatile int*>(smem + L::kMiscOffset + 12);

  const int warp = static_cast<int>(threadIdx.x >> 5);
  const int lane = static_cast<int>(threadIdx.x & 31);
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(full_bar(s), 2);   // leader producer (with the byte count) + peer producer
      ptx::mbar_init(empty_bar(s), 1);  // the MMA commit, multicast to both CTAs
    }
    for (int b = 0; b < kAcc; ++b) {
      ptx::mbar_init(accf_bar(b), 1);
      ptx::mbar_init(acce_bar(b), 2 * kEpiWarps);  // epilogue warps of both CTAs (leader's copy used)
    }
    for (int r = 0; r < kRing; ++r) {
      ptx::mbar_init(ringf_bar(r), 1);
      ptx::mbar_init(ringe_bar(r), kPairRingConsumersLeader + kPairRingConsumersPeer);
    }
    ptx::mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *prod_go = 0;
    epi_go[0] = 0;
    epi_go[1] = 0;
    ptx::fence_mbar_init();
  }
  ptx::cluster_sync();  // both CTAs' barriers exist before either touches the other's
  // A one-CTA launch of the same executor may follow (the rows the pair tiles leave): it works on
  // other problems' outputs, so it may start as soon as SMs free up.
  if (threadIdx.x == 0) ptx::launch_dependents();
  if (warp == kMmaWarp) {
    ptx::tmem_alloc_pair(ptx::smem_addr(tmem_slot), L::kTmemCols);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before_sync();
  __syncthreads();
  ptx::tc_fence_after_sync();
  const uint32_t tmem_base = *reinterpret_cast<volatile uint32_t*>(tmem_slot);

  const DeviceProblemDesc* problems = p.single_mode ? &p.single_desc : p.problems;
  const CUtensorMap* maps = p.single_mode ? p.single_maps : p.tmaps;
  const unsigned long long tmo = p.timeout_ns;
  // Ring slots are released on the leader's barrier; the peer arrives there remotely.
  auto release_slot = [&](int slot) {
    if (leader) ptx::mbar_arrive(ringe_bar(slot));
    else ptx::mbar_arrive_cluster(ptx::mapa_shared(ringe_bar(slot), 0));
  };

  if (warp == kSchedWarp) {
    // ======================= scheduler (leader only) =======================
    if (leader) {
      const int pair_id = static_cast<int>(blockIdx.x >> 1);
      const int pairs = static_cast<int>(gridDim.x >> 1);
      SchedState ss;
      sched_init(p, ss, pair_id, pairs, lane);
      prefetch_tables_l2(p, pair_id, pairs, lane);
      for (int t = 0;; ++t) {
        const int slot = t % kRing;
        const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
        int ok = 1;
        if (lane == 0)
          ok = wait_phase_cluster(ringe_bar(slot), par ^ 1u, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_SCHEDULER);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        TileSlot* s = &ring[slot];
        int pidx = -1, tile_m = 0, tile_n = 0;
        if (next_tile(p, ss, problems, lane, pairs, pidx, tile_m, tile_n)) {
          if (lane < kDescWords) reinterpret_cast<int*>(&s->desc)[lane] = ss.w;
          const unsigned fl = static_cast<unsigned>(
              __shfl_sync(0xffffffffu, ss.w, static_cast<int>(offsetof(DeviceProblemDesc, flags) / 4)));
          const int slot_maps =
              __shfl_sync(0xffffffffu, ss.w, static_cast<int>(offsetof(DeviceProblemDesc, map_slot) / 4));
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
          // Copy the slot into the peer's ring, then publish it on both sides. The remote arrive
          // releases at cluster scope, after this thread's remote stores.
          const uint32_t local_slot = ptx::smem_addr(s);
          const uint32_t remote_slot = ptx::mapa_shared(local_slot, 1);
          const uint32_t* words = reinterpret_cast<const uint32_t*>(s);
          for (int i = 0; i < static_cast<int>(sizeof(TileSlot) / 4); ++i)
            ptx::st_shared_cluster_u32(remote_slot + 4u * i, words[i]);
          __threadfence_block();
          ptx::mbar_arrive(ringf_bar(slot));
          ptx::mbar_arrive_cluster(ptx::mapa_shared(ringf_bar(slot), 1));
        }
        if (pidx < 0) break;
      }
    }
  } else if (warp >= kProdWarp0) {
    // ======================= producers (both CTAs) =======================
    const int ptid = static_cast<int>(threadIdx.x) - kProdWarp0 * 32;
    // 16-bit operands: 64-deep K blocks, 64-wide MN chunks; 8-bit: 128 and 128 (same bytes).
    const int mode = operand_mode(p);
    const bool f8 = (mode & kModeF8) != 0;
    const int cw = f8 ? 128 : 64;
    uint32_t it = 0;
    bool aborted = false;
    for (int t = 0;; ++t) {
      const int slot = t % kRing;
      const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
      int ok = 1;
      if (lane == 0)
        ok = wait_phase_cluster(ringf_bar(slot), par, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_PRODUCER);
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
      if (lane == 0) release_slot(slot);
      if (q < 0) break;
      const int row_base = tile_m * BM + static_cast<int>(rank) * 128;  // this CTA's rows of A
      const int a_row = s->desc.tma_row0 + row_base;                     // the same row in the A map
      const int map_slot = s->desc.map_slot;
      const int col_base = tile_n * BN + static_cast<int>(rank) * HB;   // this CTA's columns of B

      if (flags & grouped_gemm::kFlagTmaAB) {
        if (ptid == 0) {
          const CUtensorMap* ma = maps + kMapsPerProblem * map_slot + kMapA;
          const CUtensorMap* mb = maps + kMapsPerProblem * map_slot + kMapB;
          const CUtensorMap* mb3 = maps + kMapsPerProblem * map_slot + kMapB3;
          const bool b_one_box = HB > cw && (flags & grouped_gemm::kFlagTmaB3) && col_base + HB <= n;
          for (int kb = 0; kb < kb_count; ++kb) {
            const int st = static_cast<int>(it % S);
            const uint32_t ph = (it / S) & 1u;
            if (!wait_phase(empty_bar(st), ph ^ 1u, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_PRODUCER)) {
              aborted = true;
              break;
            }
            const uint32_t a_dst = sbase + static_cast<uint32_t>(st * L::kStageBytes);
            const uint32_t b_dst = a_dst + L::kABytes;
            const uint32_t bar_leader = ptx::mapa_shared(full_bar(st), 0);
            if (leader) ptx::mbar_arrive_expect_tx(full_bar(st), L::kStageTxPair);
            load_stage_tma_any<128, HB, true>(mode, a_dst, b_dst, ma, mb, mb3, bar_leader, kb, a_row, col_base,
                                              b_one_box);
            // The peer's arrival only counts: its TMA bytes are tracked by complete_tx.
            if (!leader) ptx::mbar_arrive_cluster_relaxed(bar_leader);
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
          lsu_fill_stage<128, HB>(as, bs, a, lda, b, ldb, m, n, k, row_base, col_base, kb, ptid,
                                  (mode & kModeACol) != 0, (mode & kModeBCol) != 0, f8);
          ptx::fence_proxy_async_all();  // the leader's tensor cores read this CTA's shared memory
          ptx::named_bar_sync(1, kProdThreads);
          if (ptid == 0) {
            if (leader) ptx::mbar_arrive(full_bar(st));
            else ptx::mbar_arrive_cluster(ptx::mapa_shared(full_bar(st), 0));
          }
          ++it;
        }
        if (aborted) break;
      }
    }
    if (aborted && ptid == 0 && leader) {
      // Loads issued for the last stages may still be landing: wait for them before exit.
      const uint32_t n_back = it < static_cast<uint32_t>(S) ? it : static_cast<uint32_t>(S);
      for (uint32_t j = 1; j <= n_back; ++j) {
        const uint32_t i2 = it - j;
        wait_drain(full_bar(static_cast<int>(i2 % S)), (i2 / S) & 1u, 100000000ull);
      }
    }
  } else if (warp == kMmaWarp) {
    // ======================= MMA issuer (leader only) =======================
    if (leader && lane == 0) {
      const int mode = operand_mode(p);
      const uint32_t kIdesc = ptx::idesc_f32acc(
          256, BN, static_cast<uint32_t>((mode & kModeF8) ? p.input_format - GG_INPUT_E4M3 : p.input_format),
          (mode & kModeACol) != 0, (mode & kModeBCol) == 0);
      uint32_t it = 0;
      for (int t = 0;; ++t) {
        const int slot = t % kRing;
        const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
        if (!wait_phase(ringf_bar(slot), par, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_MMA)) break;
        const int q = ring[slot].problem;
        const int kb_count = ring[slot].desc.k_blocks;
        // TMA stages are ordered by their byte counts (async proxy); zero-fill stages carry the
        // peer's generic stores and need the cluster-scope acquire.
        const bool lsu_tile = (ring[slot].desc.flags & grouped_gemm::kFlagTmaAB) == 0u;
        ptx::mbar_arrive(ringe_bar(slot));
        if (q < 0) break;
        const int buf = t % kAcc;
        if (!wait_phase_cluster(acce_bar(buf), (static_cast<uint32_t>(t / kAcc) & 1u) ^ 1u, abort_flag, p.status, tmo,
                                GG_STATUS_TIMEOUT_MMA))
          break;
        ptx::tc_fence_after_sync();
        if (kb_count <= 0) {
          ptx::mbar_arrive(accf_bar(buf));  // K = 0: both epilogues use a zero accumulator
          ptx::mbar_arrive_cluster(ptx::mapa_shared(accf_bar(buf), 1));
          continue;
        }
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(buf * BN);
        bool aborted = false;
        for (int kb = 0; kb < kb_count; ++kb) {
          const int st = static_cast<int>(it % S);
          const uint32_t ph = (it / S) & 1u;
          const bool got = lsu_tile ? wait_phase_cluster(full_bar(st), ph, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_MMA)
                                    : wait_phase(full_bar(st), ph, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_MMA);
          if (!got) {
            aborted = true;
            break;
          }
          ptx::tc_fence_after_sync();
          const uint32_t a0 = sbase + static_cast<uint32_t>(st * L::kStageBytes);
          const uint32_t b0 = a0 + L::kABytes;
          mma_kblock_any<true>(mode, d_tmem, a0, b0, kIdesc, kb == 0);
          ptx::tc_commit_pair_mc(empty_bar(st), 0x3);  // both CTAs' stage is free
          ++it;
        }
        if (aborted) break;
        ptx::tc_commit_pair_mc(accf_bar(buf), 0x3);  // both halves of the accumulator are ready
      }
      ptx::tc_commit_pair(drain_bar);
      wait_drain(drain_bar, 0u, 100000000ull);
    }
    __syncwarp();
  } else {
    // ======================= epilogue (warps 0-7, both CTAs) =======================
    const int qw = warp & 3;     // TMEM lane quarter
    const int half = warp >> 2;  // half of the tile's columns
    const int et = static_cast<int>(threadIdx.x);
    uint32_t store_count = 0;
    for (int t = 0;; ++t) {
      const int slot = t % kRing;
      const uint32_t par = static_cast<uint32_t>(t / kRing) & 1u;
      if (et == 0)
        epi_go[0] =
            wait_phase_cluster(ringf_bar(slot), par, abort_flag, p.status, tmo, GG_STATUS_TIMEOUT_EPILOGUE) ? 1 : 0;
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
      if (lane == 0) release_slot(slot);
      if (q < 0) break;
      const int nchunks = min(BN / 32, (n - tile_n * BN + 31) / 32);
      int c_begin, c_end;
      epilogue_chunk_range(nchunks, half, c_begin, c_end);
      e.row0 = tile_m * BM + static_cast<int>(rank) * 128 + qw * 32;  // this warp's first row
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
                    [&] {
                      if (leader) ptx::mbar_arrive(acce_bar(buf));
                      else ptx::mbar_arrive_cluster(ptx::mapa_shared(acce_bar(buf), 0));
                    });
    }
    if (lane == 0) ptx::bulk_wait_all();  // every warp issues its own TMA stores
    __syncwarp();
  }

  // Neither CTA leaves (or frees TMEM) while the other may still read or signal its shared memory.
  ptx::cluster_sync();
  if (threadIdx.x == 0) finish_launch(p);
  if (*abort_flag) {
    // After an abort, loads issued by the other CTA may still be landing here: give them time.
    const uint64_t t0 = ptx::global_timer_ns();
    while (ptx::global_timer_ns() - t0 < 200000ull) {
    }
  }
  if (warp == kMmaWarp) {
    ptx::tc_fence_after_sync();
    ptx::tmem_dealloc_pair(tmem_base, L::kTmemCols);
  }
}

}  // namespace gg
