// grouped_gemm/device_problem_desc.cuh -- the per-problem record the B200 kernel reads from HBM.
//
// It extends the reference's DeviceProblemDesc (reference src/grouped_gemm.cu:25-45, internal
// there) -- the ProblemDesc fields followed by tiles_m / tiles_n -- with the k-block count of
// the kernel's K tiling, the problem's data-path flags and, for problem sets whose rows are
// packed in one tensor (experts of a mixture-of-experts layer), the problem's first row in that
// tensor, so the kernel never recomputes them per tile. 96 bytes, a multiple of 4 so a warp can
// copy it word by word.
#pragma once

#include <cuda_fp16.h>

namespace grouped_gemm {

enum DeviceProblemFlags : unsigned {
  kFlagTmaAB = 1u,   // A and B are loaded by TMA (16-byte aligned bases, lda and ldb % 8 == 0)
  kFlagTmaD = 2u,    // D is stored by TMA (16-byte aligned base, rows a multiple of 16 bytes apart)
  kFlagReadC = 4u,   // c != nullptr && beta != 0: the epilogue reads C
  kFlagCVec = 8u,    // C rows can be read as 16-byte vectors (16-bit C: and row pitch % 8 == 0)
  kFlagDVec = 16u,   // D rows can be written as 4-element vectors (direct-store path)
  kFlagTmaB3 = 32u,  // B also has a 3-D map that loads a whole stage of full 64-column chunks at once
  kFlagPackedRows = 64u,  // the A and D maps span the packed rows of every problem: TMA row
                          // coordinates add tma_row0, and D goes out by TMA only in whole
                          // 32-row boxes (a partial box would reach the next problem's rows)
  kFlagCpAsync = 128u,  // no tensor maps (prepared on the device), but A and B rows are 16-byte
                        // aligned: the producers copy stages with 16-byte cp.async (row-major A, B)
};

struct DeviceProblemDesc {
  int m;
  int n;
  int k;

  const __half* a;  // FP16, or BF16 bits (the launch's input format)
  const __half* b;
  const void* c;    // FP32, or FP16 / BF16 (the launch's output format)
  void* d;

  int lda;
  int ldb;
  int ldc;
  int ldd;

  float alpha;
  float beta;

  int tiles_m;   // ceil(m / cta_m), 0 when m <= 0 or n <= 0
  int tiles_n;   // ceil(n / cta_n), 0 when m <= 0 or n <= 0
  int k_blocks;  // ceil(k / 64): 64-deep K blocks of the tcgen05 mainloop
  unsigned flags;  // DeviceProblemFlags
  int tma_row0;    // first row of this problem in the packed A/D maps (kFlagPackedRows), else 0
  int map_slot;    // index of this problem's group of tensor maps in the map table
};

static_assert(sizeof(DeviceProblemDesc) == 96, "DeviceProblemDesc layout");
static_assert(sizeof(DeviceProblemDesc) % 4 == 0, "copied word by word");

}  // namespace grouped_gemm
