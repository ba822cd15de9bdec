// GEMV for decode batches of up to 64 rows: y[m, n] = x[m, k] W[n, k]^T in
// the GEMV order contract (test/Test/FuryKernel/Gemv.hs:9-26) at pack width
// 4 and split 1 -- lane l's chain over packs l, l + 32, ... from 0, the lanes
// summed pairwise, neighbours first -- so its outputs are the bits of the
// other GEMV kernels and of the CPU target.
//
// At a batch past 4 the f32 arithmetic outweighs the weight stream (two
// rounded operations per multiply-add, no fused form under the contract), so
// the kernel is built to keep the FP32 pipes issuing: a warp owns 4 weight
// rows and M batch rows at once (4 M chains a lane, every x pack read from
// shared memory used 4 times, every weight pack M times).
//
// Persistent blocks of 16 warps, one a SM. The units (4 consecutive rows)
// are cut into one contiguous range a block; a block takes its range 16
// units at a time, warp w the unit w of each round. Within a round the block
// walks k in chunks of 256 packs: the chunk of every batch row in the pass is
// copied to shared memory with cp.async (the next chunk's copies in flight
// while this one is used), RMSNorm's scale and gain applied in place by the
// thread that copied it; every warp's lanes then stream their rows' packs
// with 128-bit loads that skip L1, one step ahead. Batches past M run as
// passes of M rows over the same weight rows.
#include "fk_common.cuh"
#include "fk_kernels.h"

namespace fk {

struct BatchArgs {
  const float* w;
  const float* x;
  const float* gamma;
  const float* r;
  float* y;
  uint32_t n, k, m;
  uint32_t ldx, ldr, ldy;
  float eps, factor;
};

enum { BPRO_NONE = 0, BPRO_RMSNORM = 1 };
enum { BEPI_NONE = 0, BEPI_ADD = 1, BEPI_SILU_PAIR = 2 };
template <int M>
__host__ __device__ constexpr int batch_warps() { return M <= 8 ? 16 : 12; }
constexpr int kBatchRows = 4;     // weight rows a warp
constexpr uint32_t kChunk = 256;  // packs of x a chunk
constexpr uint32_t kMaxBatch = 64;

__device__ __forceinline__ float silu_pair_of(float a, float b) {
  const float e = exp_rounded(-a);
  return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, e)), b);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = (uint32_t)__cvta_generic_to_shared(smem);
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Copy chunk c of batch rows [row0, row0 + mp) into buffer xs; rows mp..M-1
// of the buffer (computed on, never stored) are zero.
template <int M>
__device__ __forceinline__ void stage_chunk(const BatchArgs& a, float4* xs, uint32_t row0, uint32_t mp, uint32_t c,
                                            uint32_t packs) {
  const uint32_t base = c * kChunk;
  const uint32_t len = min(kChunk, packs - base);
  for (uint32_t idx = threadIdx.x; idx < M * kChunk; idx += blockDim.x) {
    const uint32_t i = idx / kChunk, j = idx % kChunk;
    if (i >= mp)
      xs[idx] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    else if (j < len)
      cp_async16(xs + idx, a.x + (size_t)(row0 + i) * a.ldx + 4 * (size_t)(base + j));
  }
}

// RMSNorm of the copies this thread made: x * scale * gamma (* factor), each
// product rounded, as the RmsNorm op's epilogue.
__device__ __forceinline__ void normalize_chunk(const BatchArgs& a, float4* xs, const float* scales, uint32_t row0,
                                                uint32_t mp, uint32_t c, uint32_t packs) {
  const uint32_t base = c * kChunk;
  const uint32_t len = min(kChunk, packs - base);
  for (uint32_t idx = threadIdx.x; idx < mp * kChunk; idx += blockDim.x) {
    const uint32_t i = idx / kChunk, j = idx % kChunk;
    if (j >= len) continue;
    float4 v = xs[idx];
    const float sc = scales[row0 + i];
    v = make_float4(__fmul_rn(v.x, sc), __fmul_rn(v.y, sc), __fmul_rn(v.z, sc), __fmul_rn(v.w, sc));
    if (a.gamma) {
      const float4 g = __ldg(reinterpret_cast<const float4*>(a.gamma) + base + j);
      v = make_float4(__fmul_rn(v.x, g.x), __fmul_rn(v.y, g.y), __fmul_rn(v.z, g.z), __fmul_rn(v.w, g.w));
    }
    if (a.factor != 1.0f)
      v = make_float4(__fmul_rn(v.x, a.factor), __fmul_rn(v.y, a.factor), __fmul_rn(v.z, a.factor),
                      __fmul_rn(v.w, a.factor));
    xs[idx] = v;
  }
}

template <int M, int PRO, int EPI>
__global__ void __launch_bounds__(batch_warps<M>() * 32, 1) gemv_batch_kernel(BatchArgs a) {
  extern __shared__ float4 xbuf[];  // [2][M][kChunk]
  __shared__ float scales[kMaxBatch];
  __shared__ float slots[kMaxBatch][8];
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
    const size_t bytes = (size_t)min((uint32_t)kBatchRows, a.n - (u_lo + warp) * kBatchRows) * a.k * 4;
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

  const float4* w4 = reinterpret_cast<const float4*>(a.w);
  for (uint32_t u0 = u_lo; u0 < u_hi; u0 += batch_warps<M>()) {
    const uint32_t u = u0 + (uint32_t)warp;
    const bool active = u < u_hi;
    const uint32_t row0 = u * kBatchRows;
    // Rows past n (the last unit's tail) read row n - 1 and store nothing.
    const float4* wrow = w4 + (size_t)min(row0, a.n - 1) * packs;
    uint32_t roff[kBatchRows];
#pragma unroll
    for (int r = 0; r < kBatchRows; ++r) roff[r] = (min(row0 + r, a.n - 1) - min(row0, a.n - 1)) * packs;

    for (uint32_t p0 = 0; p0 < a.m; p0 += M) {
      const uint32_t mp = min((uint32_t)M, a.m - p0);
      float acc[kBatchRows][M];
#pragma unroll
      for (int r = 0; r < kBatchRows; ++r)
#pragma unroll
        for (int i = 0; i < M; ++i) acc[r][i] = 0.0f;

      stage_chunk<M>(a, xbuf, p0, mp, 0, packs);
      cp_async_commit();
      float4 wv[kBatchRows];
      uint32_t g = (uint32_t)lane;
      if (active && g < packs) {
#pragma unroll
        for (int r = 0; r < kBatchRows; ++r) wv[r] = ld_stream(wrow + roff[r] + g);
      }
      for (uint32_t c = 0; c < chunks; ++c) {
        float4* xs = xbuf + (size_t)(c & 1) * M * kChunk;
        if (c + 1 < chunks) {
          stage_chunk<M>(a, xbuf + (size_t)((c + 1) & 1) * M * kChunk, p0, mp, c + 1, packs);
          cp_async_commit();
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
        if (PRO == BPRO_RMSNORM) normalize_chunk(a, xs, scales, p0, mp, c, packs);
        __syncthreads();
        if (active) {
          const uint32_t end = min(packs, (c + 1) * kChunk);
          for (; g < end; g += 32) {
            // The next step's packs (the last step reloads its own: no branch).
            const uint32_t gn = min(g + 32, packs - 1);
            float4 wn[kBatchRows];
#pragma unroll
            for (int r = 0; r < kBatchRows; ++r) wn[r] = ld_stream(wrow + roff[r] + gn);
            // Every row of the pass's buffer, the zero rows past mp included:
            // no branch between the loads and the arithmetic.
            const float4* xc = xs + (g - c * kChunk);
#pragma unroll
            for (int i = 0; i < M; ++i) {
              const float4 xv = xc[i * kChunk];
#pragma unroll
              for (int r = 0; r < kBatchRows; ++r) acc[r][i] = __fadd_rn(acc[r][i], pack_dot(xv, wv[r]));
            }
#pragma unroll
            for (int r = 0; r < kBatchRows; ++r) wv[r] = wn[r];
          }
        }
        __syncthreads();
      }

      if (active) {
        // Lanes summed pairwise; lane i keeps batch row p0 + i's totals.
        float mine[kBatchRows];
#pragma unroll
        for (int r = 0; r < kBatchRows; ++r) {
          mine[r] = 0.0f;
#pragma unroll
          for (int i = 0; i < M; ++i) {
            const float t = warp_sum(acc[r][i]);
            if (lane == i) mine[r] = t;
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

template <int M, int PRO, int EPI>
static cudaError_t launch_batch(const BatchArgs& a, int sms, cudaStream_t st, bool pdl) {
  auto kern = gemv_batch_kernel<M, PRO, EPI>;
  const size_t smem = 2 * (size_t)M * kChunk * sizeof(float4);
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const uint32_t units = (a.n + kBatchRows - 1) / kBatchRows;
  uint32_t blocks = (uint32_t)sms;
  if (blocks > units) blocks = units;
  return fk_launch_ex(kern, dim3(blocks), dim3(batch_warps<M>() * 32), smem, st, pdl, a);
}

template <int PRO, int EPI>
static cudaError_t batch_m(const BatchArgs& a, int sms, cudaStream_t st, bool pdl) {
  if (a.m <= 8) return launch_batch<8, PRO, EPI>(a, sms, st, pdl);
  return launch_batch<16, PRO, EPI>(a, sms, st, pdl);
}

}  // namespace fk

bool fk_gemv_batches(const FkGemv& g) {
  return g.m >= 1 && g.m <= fk::kMaxBatch && g.split == 1 && !g.scatter && g.k % 4 == 0 && g.ldx % 4 == 0 &&
         (reinterpret_cast<uintptr_t>(g.x) & 15) == 0 && (reinterpret_cast<uintptr_t>(g.w) & 15) == 0 &&
         (g.prologue == FK_PRO_NONE || g.prologue == FK_PRO_RMSNORM) && !(g.silu_pair && (g.n % 2 != 0 || g.r));
}

cudaError_t fk_launch_gemv_batch(const FkGemv& g, int sms, cudaStream_t st) {
  if (g.n == 0 || g.m == 0) return cudaSuccess;
  if (!fk_gemv_batches(g)) return cudaErrorInvalidValue;
  fk::BatchArgs a;
  a.w = g.w;
  a.x = g.x;
  a.gamma = g.gamma;
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
  using namespace fk;
  const int epi = g.silu_pair ? BEPI_SILU_PAIR : (g.r ? BEPI_ADD : BEPI_NONE);
  switch (g.prologue * 4 + epi) {
    case FK_PRO_NONE * 4 + BEPI_NONE: return batch_m<BPRO_NONE, BEPI_NONE>(a, sms, st, g.pdl);
    case FK_PRO_NONE * 4 + BEPI_ADD: return batch_m<BPRO_NONE, BEPI_ADD>(a, sms, st, g.pdl);
    case FK_PRO_RMSNORM * 4 + BEPI_NONE: return batch_m<BPRO_RMSNORM, BEPI_NONE>(a, sms, st, g.pdl);
    case FK_PRO_RMSNORM * 4 + BEPI_SILU_PAIR: return batch_m<BPRO_RMSNORM, BEPI_SILU_PAIR>(a, sms, st, g.pdl);
    default: return cudaErrorInvalidValue;
  }
}
