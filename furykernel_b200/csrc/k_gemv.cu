// Weight-streaming GEMV y = W x for decode: W [n, k] out_in in f32, x [m, k].
//
// The order of each output's arithmetic is the reference GEMV family's
// contract (test/Test/FuryKernel/Gemv.hs:9-26) at pack width 4 and split s:
// virtual lane v = q * 32 + l of split q visits packs v, v + 32 s, ...;
// each pack adds ((x0 w0 + x1 w1) + (x2 w2 + x3 w3)) to the lane's chain,
// which starts at 0; the lanes are summed pairwise, neighbours first; the
// splits' partials are added in split order (combineSplits,
// src/FuryKernel/Reduce.hs:97-125). The kernel keeps that order exactly, so
// its outputs are the CPU target's bits.
//
// A block is 8 warps, 8 / s output rows of s splits each; a warp streams its
// row's packs with 128-bit loads that bypass L1, 8 in flight a lane. The
// block first stages x in shared memory, computing on the way what the
// plan recomputes before the anchor: RMSNorm of a stored row (its scale by
// the 256-lane spec order of RmsNorm, then x * scale * gamma), or SiLU-gate
// of a stored gate/up row. After the rows' sums, an epilogue adds the
// residual (the plan's Add epilogue on the linear layer's tile).
#include "fk_common.cuh"
#include "fk_kernels.h"

namespace fk {

struct GemvArgs {
  const float* w;
  const float* x;
  const float* gamma;
  const float* r;
  float* y;
  uint32_t n, k, m, split;
  uint32_t ldx, ldr, ldy;
  uint32_t up_off;  // SiLU-gate: up at x + up_off, gate at x
  uint32_t kc;      // staged chunk of k, a multiple of 4
  float eps, factor;
};

enum { PRO_NONE = 0, PRO_RMSNORM = 1, PRO_SILU = 2 };

// RMSNorm's scale of one row of k floats, by a single warp computing the
// 256 spec lanes: lane l plays lanes l + 32 g, g < 8, each adding v*v over
// packs (l + 32 g) + 256 t in order; each group of 32 spec lanes is summed
// pairwise; the 8 sums combined as tgReduceSum does.
__device__ float rmsnorm_scale_warp(const float* __restrict__ xr, uint32_t k, float eps) {
  const int lane = threadIdx.x & 31;
  const uint32_t packs = k >> 2;
  const float4* x4 = reinterpret_cast<const float4*>(xr);
  float slots[8];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    float acc = 0.0f;
    for (uint32_t j = lane + 32u * g; j < packs; j += 256u) {
      float4 v = __ldg(x4 + j);
      acc = __fadd_rn(acc, __fmul_rn(v.x, v.x));
      acc = __fadd_rn(acc, __fmul_rn(v.y, v.y));
      acc = __fadd_rn(acc, __fmul_rn(v.z, v.z));
      acc = __fadd_rn(acc, __fmul_rn(v.w, v.w));
    }
    slots[g] = warp_sum(acc);
  }
  const float total = tg_sum8(slots);
  return rsqrt_rounded(__fadd_rn(__fdiv_rn(total, (float)k), eps));
}

__device__ __forceinline__ float silu_gate(float a, float b) {
  // silu(a) * b, silu(a) = a / (1 + exp(-a)), exp in binary64 rounded once.
  const float e = exp_rounded(-a);
  return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, e)), b);
}

template <int M, int PRO, bool ADD>
__global__ void __launch_bounds__(256) gemv_kernel(GemvArgs a) {
  extern __shared__ float4 xs4[];  // [m][kc / 4]
  __shared__ float scales[M];
  __shared__ float part[8][M];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t s = a.split;
  const uint32_t rows_per_block = 8u / s;
  const uint32_t row = blockIdx.x * rows_per_block + (uint32_t)warp / s;
  const uint32_t q = (uint32_t)warp % s;
  const uint32_t v = q * 32u + (uint32_t)lane;
  const uint32_t stride = 32u * s;
  const uint32_t packs = a.k >> 2;
  const bool active = row < a.n;
  const float4* wr = reinterpret_cast<const float4*>(a.w + (size_t)(active ? row : 0) * a.k);

  // Weights do not depend on earlier launches: prefetch this warp's first
  // packs into L2 before waiting on them.
  if (active && (lane & 7) == 0) {
    for (uint32_t j = v; j < packs && j < v + 8u * stride; j += stride)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(wr + j));
  }
  grid_wait();
  grid_launch_dependents();

  if (PRO == PRO_RMSNORM) {
    for (uint32_t i = warp; i < a.m; i += 8) {
      float sc = rmsnorm_scale_warp(a.x + (size_t)i * a.ldx, a.k, a.eps);
      if (lane == 0) scales[i] = sc;
    }
  }

  float acc[M];
#pragma unroll
  for (int i = 0; i < M; ++i) acc[i] = 0.0f;

  const uint32_t kc4 = a.kc >> 2;
  for (uint32_t c0 = 0; c0 < packs; c0 += kc4) {
    const uint32_t c1 = min(packs, c0 + kc4);
    const uint32_t width = c1 - c0;
    __syncthreads();
    // Stage x[:, c0:c1] (packs), transformed as the prologue says.
    for (uint32_t idx = threadIdx.x; idx < a.m * width; idx += 256u) {
      const uint32_t i = idx / width, p = idx - i * width, j = c0 + p;
      const float* xr = a.x + (size_t)i * a.ldx;
      float4 xv = __ldg(reinterpret_cast<const float4*>(xr) + j);
      if (PRO == PRO_RMSNORM) {
        const float sc = scales[i];
        xv = make_float4(__fmul_rn(xv.x, sc), __fmul_rn(xv.y, sc), __fmul_rn(xv.z, sc), __fmul_rn(xv.w, sc));
        if (a.gamma) {
          const float4 g = __ldg(reinterpret_cast<const float4*>(a.gamma) + j);
          xv = make_float4(__fmul_rn(xv.x, g.x), __fmul_rn(xv.y, g.y), __fmul_rn(xv.z, g.z), __fmul_rn(xv.w, g.w));
        }
        if (a.factor != 1.0f)
          xv = make_float4(__fmul_rn(xv.x, a.factor), __fmul_rn(xv.y, a.factor), __fmul_rn(xv.z, a.factor),
                           __fmul_rn(xv.w, a.factor));
      } else if (PRO == PRO_SILU) {
        const float4 u = __ldg(reinterpret_cast<const float4*>(xr + a.up_off) + j);
        xv = make_float4(silu_gate(xv.x, u.x), silu_gate(xv.y, u.y), silu_gate(xv.z, u.z), silu_gate(xv.w, u.w));
      }
      xs4[(size_t)i * kc4 + p] = xv;
    }
    __syncthreads();
    if (active) {
      // This lane's packs in [c0, c1): j = v (mod stride), in order.
      uint32_t j = c0 + ((v + stride - (c0 % stride)) % stride);
      for (; j + 7u * stride < c1; j += 8u * stride) {
        float4 wv[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) wv[u] = ld_stream(wr + j + u * stride);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
#pragma unroll
          for (int i = 0; i < M; ++i)
            if (i < (int)a.m) acc[i] = __fadd_rn(acc[i], pack_dot(xs4[(size_t)i * kc4 + (j + u * stride - c0)], wv[u]));
        }
      }
      for (; j < c1; j += stride) {
        const float4 wv = ld_stream(wr + j);
#pragma unroll
        for (int i = 0; i < M; ++i)
          if (i < (int)a.m) acc[i] = __fadd_rn(acc[i], pack_dot(xs4[(size_t)i * kc4 + (j - c0)], wv));
      }
    }
  }

#pragma unroll
  for (int i = 0; i < M; ++i) {
    float t = warp_sum(acc[i]);
    if (lane == 0 && i < (int)a.m) part[warp][i] = t;
  }
  __syncthreads();
  // Combine the splits in split order, then the epilogue.
  for (uint32_t idx = threadIdx.x; idx < rows_per_block * a.m; idx += 256u) {
    const uint32_t rl = idx / a.m, i = idx - rl * a.m;
    const uint32_t o = blockIdx.x * rows_per_block + rl;
    if (o >= a.n) continue;
    float t = part[rl * s][i];
    for (uint32_t qq = 1; qq < s; ++qq) t = __fadd_rn(t, part[rl * s + qq][i]);
    if (ADD) t = __fadd_rn(a.r[(size_t)i * a.ldr + o], t);
    a.y[(size_t)i * a.ldy + o] = t;
  }
}

template <int M, int PRO, bool ADD>
static cudaError_t launch_m(const GemvArgs& a, cudaStream_t st, bool pdl) {
  const uint32_t rows_per_block = 8u / a.split;
  const uint32_t blocks = (a.n + rows_per_block - 1) / rows_per_block;
  const size_t smem = (size_t)a.m * a.kc * sizeof(float);
  auto kern = gemv_kernel<M, PRO, ADD>;
  {
    cudaError_t e = fk_allow_smem(kern, smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int PRO, bool ADD>
static cudaError_t launch_pro(const GemvArgs& a, cudaStream_t st, bool pdl) {
  if (a.m <= 1) return launch_m<1, PRO, ADD>(a, st, pdl);
  if (a.m <= 2) return launch_m<2, PRO, ADD>(a, st, pdl);
  if (a.m <= 4) return launch_m<4, PRO, ADD>(a, st, pdl);
  if (a.m <= 8) return launch_m<8, PRO, ADD>(a, st, pdl);
  if (a.m <= 16) return launch_m<16, PRO, ADD>(a, st, pdl);
  if (a.m <= 32) return launch_m<32, PRO, ADD>(a, st, pdl);
  return cudaErrorInvalidValue;
}

}  // namespace fk

cudaError_t fk_launch_gemv(const FkGemv& g, cudaStream_t st) {
  if (g.n == 0 || g.m == 0) return cudaSuccess;
  if (g.k % 4 != 0 || !(g.split == 1 || g.split == 2 || g.split == 4 || g.split == 8)) return cudaErrorInvalidValue;
  if (g.m > 32) {
    // Batch rows are independent: 32 at a time.
    for (uint32_t i0 = 0; i0 < g.m; i0 += 32) {
      FkGemv part = g;
      part.m = g.m - i0 < 32 ? g.m - i0 : 32;
      part.x = g.x + (size_t)i0 * g.ldx;
      part.y = g.y + (size_t)i0 * g.ldy;
      if (g.r) part.r = g.r + (size_t)i0 * g.ldr;
      cudaError_t e = fk_launch_gemv(part, st);
      if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
  }
  fk::GemvArgs a;
  a.w = g.w;
  a.x = g.x;
  a.gamma = g.gamma;
  a.r = g.r;
  a.y = g.y;
  a.n = g.n;
  a.k = g.k;
  a.m = g.m;
  a.split = g.split;
  a.ldx = g.ldx;
  a.ldr = g.ldr;
  a.ldy = g.ldy;
  a.up_off = g.up_off;
  a.eps = g.eps;
  a.factor = g.factor;
  // Stage as much of x as 64 KiB holds (the whole row at m = 1 up to k = 16384).
  uint32_t kc = (64u * 1024u / 4u) / g.m;
  kc &= ~3u;
  if (kc > g.k) kc = g.k;
  a.kc = kc;
  const bool add = g.r != nullptr;
  switch (g.prologue) {
    case FK_PRO_NONE:
      return add ? fk::launch_pro<fk::PRO_NONE, true>(a, st, g.pdl) : fk::launch_pro<fk::PRO_NONE, false>(a, st, g.pdl);
    case FK_PRO_RMSNORM:
      return add ? fk::launch_pro<fk::PRO_RMSNORM, true>(a, st, g.pdl)
                 : fk::launch_pro<fk::PRO_RMSNORM, false>(a, st, g.pdl);
    case FK_PRO_SILU:
      return add ? fk::launch_pro<fk::PRO_SILU, true>(a, st, g.pdl) : fk::launch_pro<fk::PRO_SILU, false>(a, st, g.pdl);
    default:
      return cudaErrorInvalidValue;
  }
}
