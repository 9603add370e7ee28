// gg_copy.cu -- batched FP32 rectangle pack/unpack for the optional multi-GPU gather of D.
//
// One launch moves every rectangle of a rank's shard between its strided D matrices and the
// contiguous buffer NCCL sends or receives. Grid: x = rectangle, y = row slices; a block walks
// rows y, y + gridDim.y, ... of its rectangle and its threads stride over the columns, so every
// warp reads and writes consecutive addresses on both sides.
#include <cuda_runtime.h>

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

}  // namespace

extern "C" int gg_copy_rects(float* packed, const gg_rect_copy* rects, int count, int to_packed, void* stream) {
  if (count < 0) return static_cast<int>(cudaErrorInvalidValue);
  if (count == 0) return 0;
  if (packed == nullptr || rects == nullptr) return static_cast<int>(cudaErrorInvalidValue);
  // gridDim.x is limited to 2^31-1 and gridDim.y to 65535; count fits an int.
  copy_rects_kernel<<<dim3(static_cast<unsigned>(count), kRowSlices), kCopyThreads, 0,
                      static_cast<cudaStream_t>(stream)>>>(packed, rects, to_packed);
  return static_cast<int>(cudaGetLastError());
}
