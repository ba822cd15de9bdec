// The batched GEMV (k_gemv_batch.cu) for 16-bit weights, bf16 or f16: the
// same kernel, the same packed f32x2 arithmetic in the same order, with each
// weight pack of four 16-bit elements (8 bytes) and the RMSNorm gain widened
// to binary32 exactly where they are read (widenBF16 and widenF16,
// src/FuryKernel/Numerics.hs:33-38 and :51-66; the element type a tag,
// fk_elem16.cuh), so its outputs are the f32 kernel's over the widened
// weights. Derived from that file line for line; only the weight and gain
// loads differ.
#include "fk_common.cuh"
#include "fk_elem16.cuh"
#include "fk_kernels.h"

namespace fk {
namespace w16b {

struct BatchArgs {
  const uint16_t* w;
  const float* x;
  const uint16_t* gamma;
  const float* r;
  float* y;
  uint32_t n, k, m;
  uint32_t ldx, ldr, ldy;
  float eps, factor;
  float negzero;  // -0.0, unknown to the compiler (see prod2)
};

enum { BPRO_NONE = 0, BPRO_RMSNORM = 1 };
enum { BEPI_NONE = 0, BEPI_ADD = 1, BEPI_SILU_PAIR = 2 };
template <int M>
__host__ __device__ constexpr int batch_warps() {
  return M <= 8 ? 16 : 12;
}
constexpr int kBatchRows = 4;     // weight rows a warp
constexpr uint32_t kChunk = 256;  // packs of x a chunk
constexpr uint32_t kMaxBatch = 64;
constexpr uint32_t kAhead = 4;  // steps of L2 prefetch ahead of the loads

__device__ __forceinline__ float silu_pair_of(float a, float b) {
  const float e = exp_rounded(-a);
  return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, e)), b);
}

__device__ __forceinline__ uint2 ld_stream2(const uint2* p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// Packed binary32 pairs (PTX .f32x2, sm_100a): each half rounded to nearest
// even, as add.rn.f32 / mul.rn.f32 on its own.
__device__ __forceinline__ uint64_t pair(float lo, float hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(lo), "f"(hi));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// A packed product, rounded once, that the code generator cannot fuse into
// the add it feeds: ptxas contracts mul.rn.f32x2 followed by add.rn.f32x2
// into one fused multiply-add (measured on sm_100a, --fmad=false
// notwithstanding), which would skip the product's rounding. As
// fma(a, b, -0) with the -0 known only at run time it is a * b rounded once,
// signed zeros included (+0 + -0 = +0, -0 + -0 = -0).
__device__ __forceinline__ uint64_t prod2(uint64_t a, uint64_t b, uint64_t negzero) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(negzero));
  return d;
}
__device__ __forceinline__ float lo_of(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float hi_of(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// Copy chunk c of batch rows [row0, row0 + mp) into the raw buffer [M][kChunk].
__device__ __forceinline__ void copy_chunk(const BatchArgs& a, float4* raw, uint32_t row0, uint32_t mp, uint32_t c,
                                           uint32_t packs) {
  const uint32_t base = c * kChunk;
  const uint32_t len = min(kChunk, packs - base);
  for (uint32_t idx = threadIdx.x; idx < mp * kChunk; idx += blockDim.x) {
    const uint32_t i = idx / kChunk, j = idx % kChunk;
    if (j < len) cp_async16(raw + idx, a.x + (size_t)(row0 + i) * a.ldx + 4 * (size_t)(base + j));
  }
}

// RMSNorm's epilogue on one pack: x * scale * gamma (* factor), each product
// rounded, as the RmsNorm op computes it.
template <int PRO>
__device__ __forceinline__ float4 prologue(const BatchArgs& a, float4 v, float sc, float4 g) {
  if (PRO == BPRO_RMSNORM) {
    v = make_float4(__fmul_rn(v.x, sc), __fmul_rn(v.y, sc), __fmul_rn(v.z, sc), __fmul_rn(v.w, sc));
    if (a.gamma) v = make_float4(__fmul_rn(v.x, g.x), __fmul_rn(v.y, g.y), __fmul_rn(v.z, g.z), __fmul_rn(v.w, g.w));
    if (a.factor != 1.0f)
      v = make_float4(__fmul_rn(v.x, a.factor), __fmul_rn(v.y, a.factor), __fmul_rn(v.z, a.factor),
                      __fmul_rn(v.w, a.factor));
  }
  return v;
}

// Raw chunk -> compute buffer: plane 2p holds {x0, x0', x1, x1'} and plane
// 2p + 1 {x2, x2', x3, x3'} of batch rows 2p and 2p + 1 (rows past mp zero).
template <class E, int M, int PRO>
__device__ __forceinline__ void interleave_chunk(const BatchArgs& a, const float4* raw, float4* xs,
                                                 const float* scales, uint32_t row0, uint32_t mp, uint32_t c,
                                                 uint32_t packs) {
  const uint32_t base = c * kChunk;
  const uint32_t len = min(kChunk, packs - base);
  for (uint32_t idx = threadIdx.x; idx < (M / 2) * kChunk; idx += blockDim.x) {
    const uint32_t p = idx / kChunk, j = idx % kChunk;
    if (j >= len) continue;
    const uint32_t i0 = 2 * p, i1 = 2 * p + 1;
    float4 g = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (PRO == BPRO_RMSNORM && a.gamma) g = E::widen4(__ldg(reinterpret_cast<const uint2*>(a.gamma) + base + j));
    const float4 zero = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    const float4 u = i0 < mp ? prologue<PRO>(a, raw[i0 * kChunk + j], PRO == BPRO_RMSNORM ? scales[row0 + i0] : 0.0f, g)
                             : zero;
    const float4 v = i1 < mp ? prologue<PRO>(a, raw[i1 * kChunk + j], PRO == BPRO_RMSNORM ? scales[row0 + i1] : 0.0f, g)
                             : zero;
    xs[(2 * p) * kChunk + j] = make_float4(u.x, v.x, u.y, v.y);
    xs[(2 * p + 1) * kChunk + j] = make_float4(u.z, v.z, u.w, v.w);
  }
}

template <class E, int M, int PRO, int EPI>
__global__ void __launch_bounds__(batch_warps<M>() * 32, 1) gemv_batch_w16_kernel(BatchArgs a) {
  extern __shared__ float4 smem4[];  // raw [M][kChunk], then compute [2][M][kChunk]
  float4* raw = smem4;
  float4* comp = smem4 + (size_t)M * kChunk;
  __shared__ float scales[kMaxBatch];
  __shared__ float slots[kMaxBatch][8];
  constexpr int P = M / 2;  // packed batch-row pairs
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t packs = a.k >> 2;
  const uint32_t units = (a.n + kBatchRows - 1) / kBatchRows;
  const uint32_t G = gridDim.x;
  const uint32_t u_lo = (uint32_t)((uint64_t)units * blockIdx.x / G);
  const uint32_t u_hi = (uint32_t)((uint64_t)units * (blockIdx.x + 1) / G);
  const uint32_t chunks = (packs + kChunk - 1) / kChunk;

  // The weights depend on no earlier launch: start this warp's first unit
  // toward L2 while the previous kernel finishes.
  if (u_lo + (uint32_t)warp < u_hi) {
    const char* row = reinterpret_cast<const char*>(a.w + (size_t)(u_lo + warp) * kBatchRows * a.k);
    const size_t bytes = (size_t)min((uint32_t)kBatchRows, a.n - (u_lo + warp) * kBatchRows) * a.k * 2;
    for (size_t off = (size_t)lane * 128; off < bytes && off < 16384; off += 32 * 128)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(row + off));
  }
  grid_wait();
  grid_launch_dependents();

  if (PRO == BPRO_RMSNORM) {
    // Each row's scale by the spec's 256 lanes over packs t, t + 256, ...
    // (src/FuryKernel/Reduce.hs:59-85): the two halves of the block take
    // alternate rows, lane t of the spec at thread t of the half (a block
    // of fewer than 512 threads has one half).
    const uint32_t t = threadIdx.x & 255u, half = threadIdx.x >> 8, halves = blockDim.x >> 8;
    for (uint32_t i = half; half < halves && i < a.m; i += halves) {
      const float4* x4 = reinterpret_cast<const float4*>(a.x + (size_t)i * a.ldx);
      float acc = 0.0f;
      for (uint32_t j = t; j < packs; j += 256u) {
        const float4 v = __ldg(x4 + j);
        acc = __fadd_rn(acc, __fmul_rn(v.x, v.x));
        acc = __fadd_rn(acc, __fmul_rn(v.y, v.y));
        acc = __fadd_rn(acc, __fmul_rn(v.z, v.z));
        acc = __fadd_rn(acc, __fmul_rn(v.w, v.w));
      }
      acc = warp_sum(acc);
      if (lane == 0) slots[i][t >> 5] = acc;
    }
    __syncthreads();
    if (threadIdx.x < a.m)
      scales[threadIdx.x] = rsqrt_rounded(__fadd_rn(__fdiv_rn(tg_sum8(slots[threadIdx.x]), (float)a.k), a.eps));
    __syncthreads();
  }

  const uint2* w4 = reinterpret_cast<const uint2*>(a.w);
  const uint64_t nz = pair(a.negzero, a.negzero);
  for (uint32_t u0 = u_lo; u0 < u_hi; u0 += batch_warps<M>()) {
    const uint32_t u = u0 + (uint32_t)warp;
    const bool active = u < u_hi;
    const uint32_t row0 = u * kBatchRows;
    // Rows past n (the last unit's tail) read row n - 1 and store nothing.
    const uint2* wrow = w4 + (size_t)min(row0, a.n - 1) * packs;
    uint32_t roff[kBatchRows];
#pragma unroll
    for (int r = 0; r < kBatchRows; ++r) roff[r] = (min(row0 + r, a.n - 1) - min(row0, a.n - 1)) * packs;
    // The L2 prefetch a step issues: lane l < 16 takes line l & 3 (of 128
    // bytes) of row l >> 2's packs kAhead steps on.
    const uint32_t pf_row = (min(row0 + ((uint32_t)lane >> 2 & 3u), a.n - 1) - min(row0, a.n - 1)) * packs;
    const uint32_t pf_line = ((uint32_t)lane & 3u) * 8u;

    for (uint32_t p0 = 0; p0 < a.m; p0 += M) {
      const uint32_t mp = min((uint32_t)M, a.m - p0);
      uint64_t acc[kBatchRows][P];
#pragma unroll
      for (int r = 0; r < kBatchRows; ++r)
#pragma unroll
        for (int q = 0; q < P; ++q) acc[r][q] = 0;  // +0.0 in both halves

      copy_chunk(a, raw, p0, mp, 0, packs);
      cp_async_commit();
      float4 wv[kBatchRows];
      uint32_t g = (uint32_t)lane;
      if (active) {
        const uint32_t g0 = min(g, packs - 1);
#pragma unroll
        for (int r = 0; r < kBatchRows; ++r) wv[r] = E::widen4(ld_stream2(wrow + roff[r] + g0));
      }
      for (uint32_t c = 0; c < chunks; ++c) {
        float4* xs = comp + (size_t)(c & 1) * M * kChunk;
        cp_async_wait_all();
        __syncthreads();  // chunk c's copies are in; compute buffer c & 1 is free
        interleave_chunk<E, M, PRO>(a, raw, xs, scales, p0, mp, c, packs);
        __syncthreads();  // the raw buffer is free, chunk c is interleaved
        if (c + 1 < chunks) {
          copy_chunk(a, raw, p0, mp, c + 1, packs);
          cp_async_commit();
        }
        if (active) {
          const uint32_t end = min(packs, (c + 1) * kChunk);
          for (; g < end; g += 32) {
            uint64_t wd[kBatchRows][4];  // each weight element paired with itself
#pragma unroll
            for (int r = 0; r < kBatchRows; ++r) {
              wd[r][0] = pair(wv[r].x, wv[r].x);
              wd[r][1] = pair(wv[r].y, wv[r].y);
              wd[r][2] = pair(wv[r].z, wv[r].z);
              wd[r][3] = pair(wv[r].w, wv[r].w);
            }
            // Weights kAhead steps on toward L2, then the next step's packs
            // into registers (the last step reloads its own: no branch).
            {
              const uint32_t gp = g - (uint32_t)lane + 32u * kAhead + pf_line;
              if (lane < 16 && gp < packs) asm volatile("prefetch.global.L2 [%0];" ::"l"(wrow + pf_row + gp));
            }
            const uint32_t gn = min(g + 32, packs - 1);
#pragma unroll
            for (int r = 0; r < kBatchRows; ++r) wv[r] = E::widen4(ld_stream2(wrow + roff[r] + gn));
            // Each 128-bit load is two packed operands as they lie.
            const ulonglong2* xc = reinterpret_cast<const ulonglong2*>(xs) + (g - c * kChunk);
#pragma unroll
            for (int q = 0; q < P; ++q) {
              const ulonglong2 e = xc[(2 * q) * kChunk], f = xc[(2 * q + 1) * kChunk];
              const uint64_t x0 = e.x, x1 = e.y, x2 = f.x, x3 = f.y;
#pragma unroll
              for (int r = 0; r < kBatchRows; ++r) {
                // ((x0 w0 + x1 w1) + (x2 w2 + x3 w3)) added to the chain.
                const uint64_t s01 = add2(prod2(x0, wd[r][0], nz), prod2(x1, wd[r][1], nz));
                const uint64_t s23 = add2(prod2(x2, wd[r][2], nz), prod2(x3, wd[r][3], nz));
                acc[r][q] = add2(acc[r][q], add2(s01, s23));
              }
            }
          }
        }
      }
      __syncthreads();  // every warp is done with the compute buffers

      if (active) {
        // Lanes summed pairwise; lane i keeps batch row p0 + i's totals.
        float mine[kBatchRows];
#pragma unroll
        for (int r = 0; r < kBatchRows; ++r) {
          mine[r] = 0.0f;
#pragma unroll
          for (int q = 0; q < P; ++q) {
            const float t0 = warp_sum(lo_of(acc[r][q])), t1 = warp_sum(hi_of(acc[r][q]));
            if (lane == 2 * q) mine[r] = t0;
            if (lane == 2 * q + 1) mine[r] = t1;
          }
        }
        if ((uint32_t)lane < mp) {
          const uint32_t i = p0 + (uint32_t)lane;
          if (EPI == BEPI_SILU_PAIR) {
#pragma unroll
            for (int q = 0; q < kBatchRows / 2; ++q)
              if (row0 + 2 * q + 1 < a.n)
                a.y[(size_t)i * a.ldy + row0 / 2 + q] = silu_pair_of(mine[2 * q], mine[2 * q + 1]);
          } else {
#pragma unroll
            for (int r = 0; r < kBatchRows; ++r) {
              if (row0 + r >= a.n) break;
              float v = mine[r];
              if (EPI == BEPI_ADD) v = __fadd_rn(a.r[(size_t)i * a.ldr + row0 + r], v);
              a.y[(size_t)i * a.ldy + row0 + r] = v;
            }
          }
        }
      }
    }
  }
}

template <class E, int M, int PRO, int EPI>
static cudaError_t launch_batch(const BatchArgs& a, int sms, cudaStream_t st, bool pdl) {
  auto kern = gemv_batch_w16_kernel<E, M, PRO, EPI>;
  const size_t smem = 3 * (size_t)M * kChunk * sizeof(float4);
  cudaError_t e = fk_allow_smem(kern, smem);
  if (e != cudaSuccess) return e;
  const uint32_t units = (a.n + kBatchRows - 1) / kBatchRows;
  uint32_t blocks = (uint32_t)sms;
  if (blocks > units) blocks = units;
  return fk_launch_ex(kern, dim3(blocks), dim3(batch_warps<M>() * 32), smem, st, pdl, a);
}

template <class E, int PRO, int EPI>
static cudaError_t batch_m(const BatchArgs& a, int sms, cudaStream_t st, bool pdl) {
  if (a.m <= 8) return launch_batch<E, 8, PRO, EPI>(a, sms, st, pdl);
  return launch_batch<E, 16, PRO, EPI>(a, sms, st, pdl);
}

template <class E>
static cudaError_t batch(const BatchArgs& a, int prologue, int epi, int sms, cudaStream_t st, bool pdl) {
  switch (prologue * 4 + epi) {
    case FK_PRO_NONE * 4 + BEPI_NONE: return batch_m<E, BPRO_NONE, BEPI_NONE>(a, sms, st, pdl);
    case FK_PRO_NONE * 4 + BEPI_ADD: return batch_m<E, BPRO_NONE, BEPI_ADD>(a, sms, st, pdl);
    case FK_PRO_RMSNORM * 4 + BEPI_NONE: return batch_m<E, BPRO_RMSNORM, BEPI_NONE>(a, sms, st, pdl);
    case FK_PRO_RMSNORM * 4 + BEPI_SILU_PAIR: return batch_m<E, BPRO_RMSNORM, BEPI_SILU_PAIR>(a, sms, st, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace w16b
}  // namespace fk

bool fk_gemv_w16_batches(const FkGemv& g, const uint16_t* w) {
  return g.m >= 1 && g.m <= fk::w16b::kMaxBatch && g.split == 1 && !g.scatter && g.k % 4 == 0 && g.ldx % 4 == 0 &&
         (reinterpret_cast<uintptr_t>(g.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
         (g.prologue == FK_PRO_NONE || g.prologue == FK_PRO_RMSNORM) && !(g.silu_pair && (g.n % 2 != 0 || g.r));
}

cudaError_t fk_launch_gemv_batch_w16(const FkGemv& g, FkElem e, const uint16_t* w, const uint16_t* gamma, int sms,
                                     cudaStream_t st) {
  if (g.n == 0 || g.m == 0) return cudaSuccess;
  if (!fk_gemv_w16_batches(g, w)) return cudaErrorInvalidValue;
  fk::w16b::BatchArgs a;
  a.w = w;
  a.x = g.x;
  a.gamma = gamma;
  a.r = g.r;
  a.y = g.y;
  a.n = g.n;
  a.k = g.k;
  a.m = g.m;
  a.ldx = g.ldx;
  a.ldr = g.ldr;
  a.ldy = g.ldy;
  a.eps = g.eps;
  a.factor = g.factor;
  a.negzero = -0.0f;
  using namespace fk::w16b;
  const int epi = g.silu_pair ? BEPI_SILU_PAIR : (g.r ? BEPI_ADD : BEPI_NONE);
#define CALL(E) batch<E>(a, g.prologue, epi, sms, st, g.pdl)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}
