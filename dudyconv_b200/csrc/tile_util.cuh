// tile_util.cuh -- small register helpers shared by the tensor-core kernels: the 16-bit
// element funnel shift used for causal tap offsets, and 8-wide packed multiplies.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace dudy {
namespace tc {

// The 8 consecutive 16-bit elements that start `sh` (0..7) elements into the 16 elements
// (q0 | q1), q0 holding the lower addresses. Branch-free: output word m is input word
// m + sh/2 (picked by two selects on the bits of sh), funnel-shifted by 16 bits when sh is
// odd. Straight-line code keeps the callers' unrolled loops short (their first pass runs
// from a cold instruction cache).
__device__ __forceinline__ uint4 shift8(uint4 q0, uint4 q1, int sh) {
  const uint32_t w[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
  const bool k2 = (sh & 4) != 0, k1 = (sh & 2) != 0, odd = (sh & 1) != 0;
  uint32_t o[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const uint32_t t0 = k2 ? w[m + 2] : w[m];
    const uint32_t t1 = k2 ? w[m + 3] : w[m + 1];
    const uint32_t t2 = k2 ? (m + 4 < 8 ? w[m + 4] : 0u) : w[m + 2];
    const uint32_t base = k1 ? t1 : t0;
    const uint32_t next = k1 ? t2 : t1;
    o[m] = odd ? __byte_perm(base, next, 0x5432) : base;
  }
  return make_uint4(o[0], o[1], o[2], o[3]);
}

// Element-wise product of two packed pairs, rounded once to the element type. The exact
// product of two fp16 (or two bf16) values fits in fp32, so this equals the fp32 product
// rounded to 16 bits.
template <typename T>
__device__ __forceinline__ uint32_t mul2(uint32_t a, uint32_t b);

template <>
__device__ __forceinline__ uint32_t mul2<__half>(uint32_t a, uint32_t b) {
  __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&a), *reinterpret_cast<const __half2 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}

template <>
__device__ __forceinline__ uint32_t mul2<__nv_bfloat16>(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2(*reinterpret_cast<const __nv_bfloat162 *>(&a),
                             *reinterpret_cast<const __nv_bfloat162 *>(&b));
  return *reinterpret_cast<uint32_t *>(&r);
}

template <typename T>
__device__ __forceinline__ uint4 mul8(uint4 a, uint4 b) {
  return make_uint4(mul2<T>(a.x, b.x), mul2<T>(a.y, b.y), mul2<T>(a.z, b.z), mul2<T>(a.w, b.w));
}

// Exact two-term split of the element-wise product of two packed pairs:
//   hi = round(a*b)  and  lo = round(a*b - hi),  so that hi + lo == a*b.
// The product of two 16-bit values has at most 22 (fp16) or 16 (bf16) significant bits,
// so the residual a*b - hi has at most 11 (8) and is representable in the same type; the
// fused multiply-add forms it with a single rounding of an exactly representable value,
// i.e. exactly (for fp16 down to the subnormal range, where lo keeps an absolute error
// below 2^-25). Feeding hi and lo to two MMAs into one fp32 accumulator therefore
// contracts the exact products instead of products rounded to 16 bits.
template <typename T>
__device__ __forceinline__ void split_mul2(uint32_t a, uint32_t b, uint32_t &hi, uint32_t &lo);

template <>
__device__ __forceinline__ void split_mul2<__half>(uint32_t a, uint32_t b, uint32_t &hi,
                                                   uint32_t &lo) {
  const __half2 x = *reinterpret_cast<const __half2 *>(&a);
  const __half2 y = *reinterpret_cast<const __half2 *>(&b);
  const __half2 p = __hmul2(x, y);
  const __half2 r = __hfma2(x, y, __hneg2(p));
  hi = *reinterpret_cast<const uint32_t *>(&p);
  lo = *reinterpret_cast<const uint32_t *>(&r);
}

template <>
__device__ __forceinline__ void split_mul2<__nv_bfloat16>(uint32_t a, uint32_t b, uint32_t &hi,
                                                          uint32_t &lo) {
  const __nv_bfloat162 x = *reinterpret_cast<const __nv_bfloat162 *>(&a);
  const __nv_bfloat162 y = *reinterpret_cast<const __nv_bfloat162 *>(&b);
  const __nv_bfloat162 p = __hmul2(x, y);
  const __nv_bfloat162 r = __hfma2(x, y, __hneg2(p));
  hi = *reinterpret_cast<const uint32_t *>(&p);
  lo = *reinterpret_cast<const uint32_t *>(&r);
}

template <typename T>
__device__ __forceinline__ void split_mul8(uint4 a, uint4 b, uint4 &hi, uint4 &lo) {
  split_mul2<T>(a.x, b.x, hi.x, lo.x);
  split_mul2<T>(a.y, b.y, hi.y, lo.y);
  split_mul2<T>(a.z, b.z, hi.z, lo.z);
  split_mul2<T>(a.w, b.w, hi.w, lo.w);
}

// two fp32 values rounded to the element type and packed (lower element in the low half)
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);

template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  __half2 r = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&r);
}

template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 r = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&r);
}

}  // namespace tc
}  // namespace dudy
