// gg_copy.cu -- batched FP32 rectangle pack/unpack for the optional multi-GPU gather of D, and the
// operand realignment copy of executors with the small-problem tile class.
//
// One launch moves every rectangle of a rank's shard between its strided D matrices and the
// contiguous buffer NCCL sends or receives. Grid: x = rectangle, y = row slices; a block walks
// rows y, y + gridDim.y, ... of its rectangle and its threads stride over the columns, so every
// warp reads and writes consecutive addresses on both sides.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "gg_internal.h"
#include "grouped_gemm_b200.h"

namespace {

constexpr int kCopyThreads = 256;
constexpr int kRowSlices = 64;

__global__ void __launch_bounds__(kCopyThreads) copy_rects_kernel(float* __restrict__ packed,
                                                                  const gg_rect_copy* __restrict__ rects,
                                                                  int to_packed) {
  const gg_rect_copy r = rects[blockIdx.x];
  if (r.rows <= 0 || r.cols <= 0) return;
  for (int row = blockIdx.y; row < r.rows; row += gridDim.y) {
    float* s = r.strided + static_cast<long long>(row) * r.ld;
    float* p = packed + r.packed + static_cast<long long>(row) * r.cols;
    if (to_packed) {
      for (int c = threadIdx.x; c < r.cols; c += blockDim.x) p[c] = s[c];
    } else {
      for (int c = threadIdx.x; c < r.cols; c += blockDim.x) s[c] = p[c];
    }
  }
}

// Operand realignment: a row of blocks per job. A thread writes 16-byte chunks of the
// destination rows (16-byte aligned), each assembled from the two aligned 16-byte source granules
// it straddles (funnel shifts by the row's misalignment), with no branch, so that the loads of
// kRealignRows chunks are in flight before the stores. A granule is read only when it holds at
// least one byte of the source row (the first granule of a chunk always does); the bytes of a
// row's last chunk past row_bytes are written as zeros.
constexpr int kRealignRows = 4;

// Bytes [16 c, 16 c + 16) of a source row of row_bytes bytes (zeros past row_bytes), c < chunks.
__device__ __forceinline__ uint4 realign_chunk(const unsigned char* row, int c, int row_bytes) {
  const int b0 = 16 * c;
  const uintptr_t s = reinterpret_cast<uintptr_t>(row) + static_cast<uintptr_t>(b0);
  const int d = static_cast<int>(s & 15u);  // misalignment
  const uint4* g = reinterpret_cast<const uint4*>(s - static_cast<uintptr_t>(d));
  const uint4 g0 = *g;
  // the second granule starts 16 - d bytes into the chunk: read it only if the row reaches it
  const uint4 g1 = (d != 0 && b0 + 16 - d < row_bytes) ? g[1] : make_uint4(0u, 0u, 0u, 0u);
  const unsigned w[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
  const int q = d >> 2, sh = 8 * (d & 3);
  unsigned x[5];
#pragma unroll
  for (int i = 0; i < 5; ++i) x[i] = q == 0 ? w[i] : q == 1 ? w[i + 1] : q == 2 ? w[i + 2] : w[i + 3];
  unsigned o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // bytes of word i inside the row: 4, or 0..3 in the row's last chunk
    const int keep = min(4, max(0, row_bytes - b0 - 4 * i));
    const unsigned mask = keep >= 4 ? 0xffffffffu : ((1u << (8 * keep)) - 1u);
    o[i] = __funnelshift_r(x[i], x[i + 1], sh) & mask;
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void __launch_bounds__(kCopyThreads) realign_kernel(const gg::RealignJob* __restrict__ jobs) {
  const gg::RealignJob j = jobs[blockIdx.x];
  if (j.rows <= 0 || j.row_bytes <= 0) return;
  // the job's (row, chunk) units, strided over the blocks of its row of the grid (fewer than
  // 2^31 units per job: the host realigns no larger operand)
  const unsigned chunks = static_cast<unsigned>((j.row_bytes + 15) / 16);
  const unsigned units = static_cast<unsigned>(j.rows) * chunks;
  const unsigned stride = gridDim.y * blockDim.x;
  const unsigned char* __restrict__ src = j.src;
  unsigned char* __restrict__ dst = j.dst;
  for (unsigned u0 = blockIdx.y * blockDim.x + threadIdx.x; u0 < units; u0 += stride * kRealignRows) {
    uint4 v[kRealignRows];
    int row[kRealignRows], col[kRealignRows];
#pragma unroll
    for (int r = 0; r < kRealignRows; ++r) {
      const unsigned u = u0 + r * stride;  // no wrap: u0 + (kRealignRows - 1) * stride < 2^31 + 2^29
      row[r] = u < units ? static_cast<int>(u / chunks) : -1;
      col[r] = u < units ? static_cast<int>(u - static_cast<unsigned>(row[r]) * chunks) : 0;
      v[r] = row[r] >= 0 ? realign_chunk(src + static_cast<long long>(row[r]) * j.src_pitch, col[r], j.row_bytes)
                         : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int r = 0; r < kRealignRows; ++r)
      if (row[r] >= 0) reinterpret_cast<uint4*>(dst + static_cast<long long>(row[r]) * j.dst_pitch)[col[r]] = v[r];
  }
}

}  // namespace

namespace gg {

cudaError_t launch_realign(const RealignJob* jobs, int count, long long max_units, cudaStream_t stream) {
  if (count <= 0) return cudaSuccess;
  // blocks per job: two passes of kRealignRows units per thread for the largest job, at most 1024
  const long long per_block = 2LL * kCopyThreads * kRealignRows;
  const int slices = static_cast<int>(std::min<long long>(1024, std::max<long long>(1, (max_units + per_block - 1) / per_block)));
  realign_kernel<<<dim3(static_cast<unsigned>(count), static_cast<unsigned>(slices)), kCopyThreads, 0, stream>>>(jobs);
  return cudaGetLastError();
}

}  // namespace gg

extern "C" int gg_copy_rects(float* packed, const gg_rect_copy* rects, int count, int to_packed, void* stream) {
  if (count < 0) return static_cast<int>(cudaErrorInvalidValue);
  if (count == 0) return 0;
  if (packed == nullptr || rects == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  // gridDim.x is limited to 2^31-1 and gridDim.y to 65535; count fits an int.
  copy_rects_kernel<<<dim3(static_cast<unsigned>(count), kRowSlices), kCopyThreads, 0,
                      static_cast<cudaStream_t>(stream)>>>(packed, rects, to_packed);
  return static_cast<int>(cudaGetLastError());
}
