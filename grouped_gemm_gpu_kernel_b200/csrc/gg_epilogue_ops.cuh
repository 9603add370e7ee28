// gg_epilogue_ops.cuh -- element formats of C and D and the fused post-operation of the epilogue,
// shared by the tcgen05 kernels and the CUDA-core kernel.
//
// The reference stores FP32 D = alpha * acc + beta * C (src/grouped_gemm.cu:460-481, 614-621).
// The extensions here keep that arithmetic in FP32 and add, in this order: a per-column bias, an
// activation, and one round-to-nearest-even conversion to the output format at the store:
//   D = round_out(act(alpha * acc + (beta * C + bias))).
// C, when read, has the output format and is widened to FP32 exactly.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cstdint>
#include <cstring>

#include "grouped_gemm_b200.h"

namespace gg {

constexpr int kOutF32 = GG_OUTPUT_F32;
constexpr int kOutF16 = GG_OUTPUT_F16;
constexpr int kOutBF16 = GG_OUTPUT_BF16;

template <int F>
struct OutFormat {
  static constexpr int kBytes = F == kOutF32 ? 4 : 2;
};

// A 16-bit element of the output format widened to FP32 (exact: both are subsets of FP32).
template <int F>
__device__ __forceinline__ float widen16(unsigned short u) {
  if constexpr (F == kOutBF16) return __uint_as_float(static_cast<uint32_t>(u) << 16);
  else return __half2float(__ushort_as_half(u));
}

// Two 16-bit elements packed in one word, the lower address in the low half.
template <int F>
__device__ __forceinline__ float2 unpack2(uint32_t u) {
  return make_float2(widen16<F>(static_cast<unsigned short>(u & 0xffffu)),
                     widen16<F>(static_cast<unsigned short>(u >> 16)));
}

// Two FP32 values rounded to the 16-bit output format (nearest even) and packed, x first.
template <int F>
__device__ __forceinline__ uint32_t pack2(float x, float y) {
  uint32_t u;
  if constexpr (F == kOutBF16) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(x, y);
    memcpy(&u, &h, 4);
  } else {
    const __half2 h = __floats2half2_rn(x, y);
    memcpy(&u, &h, 4);
  }
  return u;
}

// Element i of an output-format array, as FP32 (read-only path).
template <int F>
__device__ __forceinline__ float load_out(const void* base, int64_t i) {
  if constexpr (F == kOutF32) return __ldg(static_cast<const float*>(base) + i);
  else return widen16<F>(__ldg(static_cast<const unsigned short*>(base) + i));
}

// Four consecutive elements at p, which is aligned to four elements (16 or 8 bytes).
template <int F>
__device__ __forceinline__ float4 load_out4(const void* p) {
  if constexpr (F == kOutF32) {
    return __ldg(static_cast<const float4*>(p));
  } else {
    const uint2 u = __ldg(static_cast<const uint2*>(p));
    const float2 lo = unpack2<F>(u.x), hi = unpack2<F>(u.y);
    return make_float4(lo.x, lo.y, hi.x, hi.y);
  }
}

template <int F>
__device__ __forceinline__ void store_out(void* base, int64_t i, float v) {
  if constexpr (F == kOutF32) static_cast<float*>(base)[i] = v;
  else if constexpr (F == kOutF16) static_cast<__half*>(base)[i] = __float2half_rn(v);
  else static_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
}

// Four consecutive elements to p, aligned to four elements.
template <int F>
__device__ __forceinline__ void store_out4(void* p, float4 o) {
  if constexpr (F == kOutF32) *static_cast<float4*>(p) = o;
  else *static_cast<uint2*>(p) = make_uint2(pack2<F>(o.x, o.y), pack2<F>(o.z, o.w));
}

// The same, for a format known only at run time (one kernel body serves every format).
__device__ __forceinline__ float2 unpack2_rt(int fmt, uint32_t u) {
  return fmt == kOutBF16 ? unpack2<kOutBF16>(u) : unpack2<kOutF16>(u);
}

__device__ __forceinline__ uint32_t pack2_rt(int fmt, float x, float y) {
  return fmt == kOutBF16 ? pack2<kOutBF16>(x, y) : pack2<kOutF16>(x, y);
}

__device__ __forceinline__ float load_out_rt(int fmt, const void* base, int64_t i) {
  if (fmt == kOutF32) return load_out<kOutF32>(base, i);
  const unsigned short u = __ldg(static_cast<const unsigned short*>(base) + i);
  return fmt == kOutBF16 ? widen16<kOutBF16>(u) : widen16<kOutF16>(u);
}

__device__ __forceinline__ float4 load_out4_rt(int fmt, const void* p) {
  if (fmt == kOutF32) return load_out4<kOutF32>(p);
  const uint2 u = __ldg(static_cast<const uint2*>(p));
  const float2 lo = unpack2_rt(fmt, u.x), hi = unpack2_rt(fmt, u.y);
  return make_float4(lo.x, lo.y, hi.x, hi.y);
}

__device__ __forceinline__ void store_out_rt(int fmt, void* base, int64_t i, float v) {
  if (fmt == kOutF32) store_out<kOutF32>(base, i, v);
  else if (fmt == kOutF16) store_out<kOutF16>(base, i, v);
  else store_out<kOutBF16>(base, i, v);
}

__device__ __forceinline__ void store_out4_rt(int fmt, void* p, float4 o) {
  if (fmt == kOutF32) store_out4<kOutF32>(p, o);
  else *static_cast<uint2*>(p) = make_uint2(pack2_rt(fmt, o.x, o.y), pack2_rt(fmt, o.z, o.w));
}

// GG_ACT_RELU: max(x, 0) (a NaN gives 0). GG_ACT_GELU: the tanh form of GELU (Hendrycks and
// Gimpel, "Gaussian Error Linear Units"), 0.5 x (1 + tanh(u)) with u = sqrt(2/pi) (x + 0.044715 x^3),
// evaluated through the identity 0.5 (1 + tanh(u)) = 1 / (1 + exp(-2u)) as x / (1 + exp(-2u)):
// one fast exponential and one fast division, a few instructions, so that the many unrolled copies
// in the epilogue stay small. The exponent is capped at 80 (exp(80) < 2^126, the range of
// __fdividef), where the result is below 1e-34 |x| either way. Relative error about 1e-5 at worst
// (the intrinsics' bounds), far inside the epilogue's accuracy bound.
__device__ __forceinline__ float gelu_tanh(float x) {
  const float minus_2u = -1.5957691216057308f * fmaf(0.044715f * x, x * x, x);
  return __fdividef(x, 1.0f + __expf(fminf(minus_2u, 80.0f)));
}

__device__ __forceinline__ float activate(float x, int act) {
  if (act == GG_ACT_RELU) return fmaxf(x, 0.0f);
  if (act == GG_ACT_GELU) return gelu_tanh(x);
  return x;
}

__device__ __forceinline__ float4 activate4(float4 v, int act) {
  if (act == GG_ACT_NONE) return v;
  return make_float4(activate(v.x, act), activate(v.y, act), activate(v.z, act), activate(v.w, act));
}

}  // namespace gg
