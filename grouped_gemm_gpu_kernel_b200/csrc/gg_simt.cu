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
// A CTA computes its tile as 64 x 64 sub-tiles: 256 threads, each 4 x 4 outputs; K in steps of 32
// through shared memory (A stored k-major so a thread reads its 4 rows with one 16-byte load),
// operands loaded with plain zero-filled loads (any leading dimension, any alignment). No
// spin-waits: only atomics and block barriers.
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include "gg_epilogue_ops.cuh"
#include "gg_internal.h"

namespace gg {
namespace {

constexpr int kSimtThreads = 256;
constexpr int kSub = 64;     // sub-tile edge
constexpr int kSimtBK = 32;  // K per shared-memory step
constexpr int kPad = 4;      // keeps 16-byte alignment of every row, spreads banks

// Operand element i widened to FP32, exactly: FP16; BF16 (its bits are the top half of an FP32);
// E4M3 / E5M2 (one byte per element; every value of both is an FP16 value).
__device__ __forceinline__ float widen(const __half* x, long long i, int fmt) {
  if (fmt == GG_INPUT_BF16)
    return __uint_as_float(static_cast<unsigned>(reinterpret_cast<const unsigned short*>(x)[i]) << 16);
  if (fmt == GG_INPUT_E4M3 || fmt == GG_INPUT_E5M2) {
    const __nv_fp8_storage_t v = reinterpret_cast<const unsigned char*>(x)[i];
    return __half2float(__half(__nv_cvt_fp8_to_halfraw(v, fmt == GG_INPUT_E4M3 ? __NV_E4M3 : __NV_E5M2)));
  }
  return __half2float(x[i]);
}

// D = act(alpha * acc + (beta * C + bias)) for this thread's 4 x 4 outputs, C and D in format F.
template <int F>
__device__ __forceinline__ void store_block(const DeviceProblemDesc& d, const float* bias, int act, bool read_c,
                                            const float (&acc)[4][4], int r0, int c0) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gr = r0 + i;
    if (gr >= d.m) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gc = c0 + j;
      if (gc >= d.n) continue;
      float add = read_c ? d.beta * load_out<F>(d.c, static_cast<long long>(gr) * d.ldc + gc) : 0.0f;
      if (bias) add += __ldg(bias + gc);
      store_out<F>(d.d, static_cast<long long>(gr) * d.ldd + gc, activate(fmaf(d.alpha, acc[i][j], add), act));
    }
  }
}

// Last q with offs[q] <= tile (offs has count + 1 entries, offs[count] = total > tile).
__device__ int find_problem(const int* offs, int count, int tile) {
  int lo = 0, hi = count;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (offs[mid] <= tile) lo = mid;
    else hi = mid;
  }
  return lo;
}

__global__ void __launch_bounds__(kSimtThreads) grouped_gemm_simt_kernel(const __grid_constant__ KernelParams p,
                                                                        int bm, int bn) {
  __shared__ __align__(16) float As[kSimtBK][kSub + kPad];  // As[k][row]
  __shared__ __align__(16) float Bs[kSimtBK][kSub + kPad];  // Bs[k][col]
  __shared__ int s_work[3];                                 // problem, tile_m, tile_n

  const DeviceProblemDesc* problems = p.single_mode ? &p.single_desc : p.problems;
  const int total = p.total_tiles_dev ? *p.total_tiles_dev : p.total_tiles;
  const int tid = static_cast<int>(threadIdx.x);
  const int tx = tid & 15, ty = tid >> 4;
  const int in_fmt = p.input_format;
  const bool a_col = (p.layout & 1) != 0;  // A stored k x m
  const bool b_col = (p.layout & 2) != 0;  // B stored n x k
  int static_next = static_cast<int>(blockIdx.x);

  for (;;) {
    if (tid == 0) {
      int q = -1, tm = 0, tn = 0;
      for (;;) {
        int tile;
        if (p.single_mode) {
          tile = static_next;
          static_next += static_cast<int>(gridDim.x);
        } else {
          tile = atomicAdd(p.tile_counter, 1);
        }
        if (tile >= total) break;
        const int pq = p.single_mode ? 0 : find_problem(p.tile_offsets, p.problem_count, tile);
        const int local = tile - (p.single_mode ? 0 : p.tile_offsets[pq]);
        const int tiles_m = problems[pq].tiles_m, tiles_n = problems[pq].tiles_n;
        // a tile outside its problem's grid (a prepared set inconsistent with the config) is
        // skipped, as the reference kernel does (src/grouped_gemm.cu:662-672)
        if (local < 0 || tiles_m <= 0 || tiles_n <= 0 || local >= tiles_m * tiles_n) continue;
        q = pq;
        tm = local / tiles_n;
        tn = local % tiles_n;
        break;
      }
      s_work[0] = q;
      s_work[1] = tm;
      s_work[2] = tn;
    }
    __syncthreads();
    const int q = s_work[0], tile_m = s_work[1], tile_n = s_work[2];
    __syncthreads();  // s_work is rewritten for the next tile only after every thread read it
    if (q < 0) break;

    const DeviceProblemDesc& d = problems[q];
    const int m = d.m, n = d.n, k = d.k;
    const __half* a = d.a;
    const __half* b = d.b;
    const int lda = d.lda, ldb = d.ldb;
    const bool read_c = (d.flags & grouped_gemm::kFlagReadC) != 0u;
    const float* bias = p.bias ? p.bias[d.map_slot] : nullptr;

    for (int sm = 0; sm < bm; sm += kSub) {
      const int row0 = tile_m * bm + sm;
      if (row0 >= m) break;
      for (int sn = 0; sn < bn; sn += kSub) {
        const int col0 = tile_n * bn + sn;
        if (col0 >= n) break;
        float acc[4][4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[i][j] = 0.0f;
        for (int k0 = 0; k0 < k; k0 += kSimtBK) {
          // consecutive threads take consecutive elements of the stored layout (coalesced reads)
          for (int i = tid; i < kSub * kSimtBK; i += kSimtThreads) {
            const int r = a_col ? i % kSub : i / kSimtBK, kk = a_col ? i / kSub : i % kSimtBK;
            const int gr = row0 + r, gk = k0 + kk;
            const long long ai = a_col ? static_cast<long long>(gk) * lda + gr : static_cast<long long>(gr) * lda + gk;
            As[kk][r] = (gr < m && gk < k) ? widen(a, ai, in_fmt) : 0.0f;
          }
          for (int i = tid; i < kSimtBK * kSub; i += kSimtThreads) {
            const int kk = b_col ? i % kSimtBK : i / kSub, c = b_col ? i / kSimtBK : i % kSub;
            const int gk = k0 + kk, gc = col0 + c;
            const long long bi = b_col ? static_cast<long long>(gc) * ldb + gk : static_cast<long long>(gk) * ldb + gc;
            Bs[kk][c] = (gk < k && gc < n) ? widen(b, bi, in_fmt) : 0.0f;
          }
          __syncthreads();
#pragma unroll 8
          for (int kk = 0; kk < kSimtBK; ++kk) {
            const float4 av = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            const float4 bv = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
            const float ar[4] = {av.x, av.y, av.z, av.w};
            const float br[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
              for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(ar[i], br[j], acc[i][j]);
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
    st = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, grouped_gemm_simt_kernel, kSimtThreads, 0);
  if (st != cudaSuccess) return st;
  *ctas = sms * (per_sm > 0 ? per_sm : 1);
  return cudaSuccess;
}

cudaError_t simt_occupancy(int* active_blocks_per_sm, cudaFuncAttributes* attrs) {
  cudaError_t st = cudaFuncGetAttributes(attrs, grouped_gemm_simt_kernel);
  if (st != cudaSuccess) return st;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(active_blocks_per_sm, grouped_gemm_simt_kernel, kSimtThreads,
                                                       0);
}

int simt_threads() { return kSimtThreads; }

cudaError_t launch_simt_kernel(Variant v, const KernelParams& params, int grid, cudaStream_t stream) {
  if (grid <= 0) return cudaSuccess;
  grouped_gemm_simt_kernel<<<grid, kSimtThreads, 0, stream>>>(params, variant_bm(v), variant_bn(v));
  return cudaGetLastError();
}

}  // namespace gg
