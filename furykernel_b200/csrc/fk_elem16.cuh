// The 16-bit element types a model's weights and KV caches may hold: bfloat16
// and binary16 (weights: src/FuryKernel/Program/Check.hs:105-111; caches:
// CacheElem, src/FuryKernel/Program/Graph.hs:169-180). Both widen to binary32
// exactly where they are read; both narrow from binary32 where they are
// stored: to nearest, ties to even, with a NaN keeping its sign and top
// payload bits and coming out quiet (narrowBF16 and narrowF16,
// src/FuryKernel/Numerics.hs:41-48 and :100-130; the CPU target's
// conversions, src/FuryKernel/Cpu.hs:717-718).
//
// A kernel over either type takes the type as a tag, E::widen / E::widen4 /
// E::narrow; a pack of four elements is 8 bytes, element 0 the low half of
// the first word. Widening here does not quiet a NaN as the reference's
// does: a widened value is only ever an operand of arithmetic, whose NaN
// result is a NaN either way.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "fk_kernels.h"

namespace fk {

struct Bf16 {
  using Storage = uint16_t;
  static constexpr FkElem kElem = FK_BF16;
  __device__ static __forceinline__ float widen(uint16_t h) { return __uint_as_float((uint32_t)h << 16); }
  __device__ static __forceinline__ float4 widen4(uint2 r) {
    return make_float4(__uint_as_float(r.x << 16), __uint_as_float(r.x & 0xFFFF0000u), __uint_as_float(r.y << 16),
                       __uint_as_float(r.y & 0xFFFF0000u));
  }
  __device__ static __forceinline__ uint16_t narrow(float v) {
    const uint32_t w = __float_as_uint(v);
    if ((w & 0x7F800000u) == 0x7F800000u && (w & 0x007FFFFFu)) return (uint16_t)((w >> 16) | 0x0040u);
    return (uint16_t)((w + 0x7FFFu + ((w >> 16) & 1u)) >> 16);
  }
};

struct F16 {
  using Storage = uint16_t;
  static constexpr FkElem kElem = FK_F16;
  // Every binary16 value, subnormals included, is a binary32 value.
  __device__ static __forceinline__ float widen(uint16_t h) { return __half2float(__ushort_as_half(h)); }
  __device__ static __forceinline__ float2 widen2(uint32_t w) {
    __half2 h;
    memcpy(&h, &w, 4);
    return __half22float2(h);
  }
  __device__ static __forceinline__ float4 widen4(uint2 r) {
    const float2 a = widen2(r.x), b = widen2(r.y);
    return make_float4(a.x, a.y, b.x, b.y);
  }
  // cvt.rn.f16.f32: nearest, ties to even, gradual underflow, past the
  // largest finite value by half an ulp or more to infinity; a NaN as
  // narrowF16 has it (0x7E00 with the top 9 payload bits, the sign kept).
  __device__ static __forceinline__ uint16_t narrow(float v) {
    const uint32_t w = __float_as_uint(v);
    if ((w & 0x7F800000u) == 0x7F800000u && (w & 0x007FFFFFu))
      return (uint16_t)(((w >> 16) & 0x8000u) | 0x7E00u | ((w & 0x007FFFFFu) >> 13));
    return __half_as_ushort(__float2half_rn(v));
  }
};

// An f32 element, for the kernels that take f32 caches and tables as well.
struct F32 {
  using Storage = float;
  static constexpr FkElem kElem = FK_F32;
};

}  // namespace fk

// The launch for a 16-bit element type, CALL(tag); any other type is refused.
#define FK_BY_ELEM16(e, CALL) \
  ((e) == FK_BF16 ? CALL(fk::Bf16) : (e) == FK_F16 ? CALL(fk::F16) : cudaErrorInvalidValue)
