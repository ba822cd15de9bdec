// The reference's bf16 GEMV family itself (test/Test/FuryKernel/Gemv.hs):
// y[m, n] = x[m, k] W[n, k]^T with x, W and y bf16, the products and sums in
// binary32. The order contract (Gemv.hs:9-26, 118-191): virtual lane
// v = q * 32 + l of split q visits packs v, v + 32 s, ... of p elements
// (p = 4, 8 or 16); a pack's elements go four to a chain, chain c adding
// ((x0 w0 + x1 w1) + (x2 w2 + x3 w3)) from 0; a lane's chains are added left
// to right (inOrder, Gemv.hs:214-217), the lanes pairwise, neighbours first;
// the splits' partials in split order; y narrowed to bf16 by round to
// nearest even (narrowBF16, src/FuryKernel/Numerics.hs:41-48). Widening is
// exact (a bf16 is the top half of its binary32); the reference quiets a
// NaN input on widening, which changes no result here (the GPU's arithmetic
// turns any NaN into its canonical NaN), so a NaN's payload is the one
// thing not matched.
//
// Work: persistent blocks of 16 warps, a warp a row at a time (its splits
// one after another, as the order contract allows); weights streamed with
// 128-bit loads that skip L1, 2 to 4 packs in flight a lane, x read through
// L1 (every warp reads the same x).
#include "fk_common.cuh"
#include "fk_kernels.h"

namespace fk {

struct Bf16Args {
  const uint16_t* w;
  const uint16_t* x;
  uint16_t* y;
  uint32_t n, k, m, split, ldx, ldy;
};

__device__ __forceinline__ float widen(uint32_t bits16) { return __uint_as_float(bits16 << 16); }

__device__ __forceinline__ uint16_t narrow(float v) {
  const uint32_t w = __float_as_uint(v);
  if (isnan(v)) return (uint16_t)((w >> 16) | 0x0040u);
  return (uint16_t)((w + 0x7FFFu + ((w >> 16) & 1u)) >> 16);
}

// A pack of P bf16 elements, as P / 2 32-bit words.
template <int P>
struct Pack {
  uint32_t u[P / 2];
};

template <int P>
__device__ __forceinline__ Pack<P> load_pack(const uint16_t* p, bool stream) {
  Pack<P> r;
  if (P == 4) {
    const uint2 v = stream ? __ldcs(reinterpret_cast<const uint2*>(p)) : __ldg(reinterpret_cast<const uint2*>(p));
    r.u[0] = v.x, r.u[1] = v.y;
  } else {
#pragma unroll
    for (int h = 0; h < P / 8; ++h) {
      const uint4 v = stream ? __ldcs(reinterpret_cast<const uint4*>(p) + h) : __ldg(reinterpret_cast<const uint4*>(p) + h);
      r.u[4 * h] = v.x, r.u[4 * h + 1] = v.y, r.u[4 * h + 2] = v.z, r.u[4 * h + 3] = v.w;
    }
  }
  return r;
}

// Element e of a pack (little-endian halves).
template <int P>
__device__ __forceinline__ float elem(const Pack<P>& p, int e) {
  const uint32_t word = p.u[e >> 1];
  return widen((e & 1) ? (word >> 16) : (word & 0xFFFFu));
}

// One pack j of a row into the chains of every batch row.
template <int M, int P>
__device__ __forceinline__ void pack_chains(const Bf16Args& a, float (&acc)[M][P / 4], const Pack<P>& wp,
                                            uint32_t j) {
#pragma unroll
  for (int i = 0; i < M; ++i) {
    if (i >= (int)a.m) break;
    const Pack<P> xp = load_pack<P>(a.x + (size_t)i * a.ldx + (size_t)j * P, false);
#pragma unroll
    for (int c = 0; c < P / 4; ++c) {
      const float d01 = __fadd_rn(__fmul_rn(elem(xp, 4 * c), elem(wp, 4 * c)),
                                  __fmul_rn(elem(xp, 4 * c + 1), elem(wp, 4 * c + 1)));
      const float d23 = __fadd_rn(__fmul_rn(elem(xp, 4 * c + 2), elem(wp, 4 * c + 2)),
                                  __fmul_rn(elem(xp, 4 * c + 3), elem(wp, 4 * c + 3)));
      acc[i][c] = __fadd_rn(acc[i][c], __fadd_rn(d01, d23));
    }
  }
}

template <int M, int P>
__global__ void __launch_bounds__(512) gemv_bf16_kernel(Bf16Args a) {
  constexpr int C = P / 4;  // chains a lane
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t packs = a.k / P;
  const uint32_t stride = 32u * a.split;
  grid_wait();
  grid_launch_dependents();
  for (uint32_t row = blockIdx.x * 16 + warp; row < a.n; row += gridDim.x * 16) {
    const uint16_t* wr = a.w + (size_t)row * a.k;
    float total[M];
    for (uint32_t q = 0; q < a.split; ++q) {
      float acc[M][C];
#pragma unroll
      for (int i = 0; i < M; ++i)
#pragma unroll
        for (int c = 0; c < C; ++c) acc[i][c] = 0.0f;
      // The lane's packs in order, U weight packs in flight at a time.
      constexpr int U = P == 16 ? 2 : 4;
      uint32_t j = q * 32u + (uint32_t)lane;
      for (; j + (U - 1) * stride < packs; j += U * stride) {
        Pack<P> wp[U];
#pragma unroll
        for (int t = 0; t < U; ++t) wp[t] = load_pack<P>(wr + (size_t)(j + t * stride) * P, true);
#pragma unroll
        for (int t = 0; t < U; ++t) pack_chains<M, P>(a, acc, wp[t], j + t * stride);
      }
      for (; j < packs; j += stride) pack_chains<M, P>(a, acc, load_pack<P>(wr + (size_t)j * P, true), j);
#pragma unroll
      for (int i = 0; i < M; ++i) {
        float t = acc[i][0];
#pragma unroll
        for (int c = 1; c < C; ++c) t = __fadd_rn(t, acc[i][c]);
        const float part = warp_sum(t);
        total[i] = q == 0 ? part : __fadd_rn(total[i], part);
      }
    }
    if (lane == 0) {
#pragma unroll
      for (int i = 0; i < M; ++i)
        if (i < (int)a.m) a.y[(size_t)i * a.ldy + row] = narrow(total[i]);
    }
  }
}

template <int P>
static cudaError_t launch_p(const Bf16Args& a, int sms, cudaStream_t st, bool pdl) {
  uint32_t blocks = (a.n + 15) / 16;
  const uint32_t cap = (uint32_t)sms * 4;
  if (blocks > cap) blocks = cap;
  if (a.m <= 1) return fk_launch_ex(gemv_bf16_kernel<1, P>, dim3(blocks), dim3(512), 0, st, pdl, a);
  if (a.m <= 2) return fk_launch_ex(gemv_bf16_kernel<2, P>, dim3(blocks), dim3(512), 0, st, pdl, a);
  if (a.m <= 4) return fk_launch_ex(gemv_bf16_kernel<4, P>, dim3(blocks), dim3(512), 0, st, pdl, a);
  if (a.m <= 8) return fk_launch_ex(gemv_bf16_kernel<8, P>, dim3(blocks), dim3(512), 0, st, pdl, a);
  return fk_launch_ex(gemv_bf16_kernel<16, P>, dim3(blocks), dim3(512), 0, st, pdl, a);
}

}  // namespace fk

cudaError_t fk_launch_gemv_bf16(const uint16_t* w, const uint16_t* x, uint16_t* y, uint32_t n, uint32_t k,
                                uint32_t m, uint32_t pack, uint32_t split, uint32_t ldx, uint32_t ldy, int sms,
                                bool pdl, cudaStream_t st) {
  if (n == 0 || m == 0) return cudaSuccess;
  if (m > 16 || split == 0 || !(pack == 4 || pack == 8 || pack == 16) || k % pack != 0 || ldx % pack != 0)
    return cudaErrorInvalidValue;
  fk::Bf16Args a{w, x, y, n, k, m, split, ldx, ldy};
  if (pack == 4) return fk::launch_p<4>(a, sms, st, pdl);
  if (pack == 8) return fk::launch_p<8>(a, sms, st, pdl);
  return fk::launch_p<16>(a, sms, st, pdl);
}
