// Threadgroup tree reduction (config 1) and the row kernels RMSNorm and
// softmax (config 2), each computing the bits of its spec kernel under the
// reference CPU target's semantics.
#include "fk_common.cuh"
#include "fk_kernels.h"

namespace fk {

// ---------------------------------------------------------------------------
// Pass 1: 256-element groups halved through threadgroup memory, one partial
// per group. A warp takes a whole group: lane l holds elements l + 32 j,
// j < 8, so the halvings by 128, 64 and 32 pair elements within a lane and
// those by 16 ... 1 are the butterfly's shuffles down: the same additions,
// in the same order, as the halving tree (x[i] + x[i + s] for i < s).
// Elements past n are -0, the identity of addition.
__global__ void __launch_bounds__(256) reduce_groups_kernel(const float* __restrict__ x, uint64_t n,
                                                            float* __restrict__ partials,
                                                            uint32_t groups) {
  const int lane = threadIdx.x & 31;
  const uint32_t warps_total = gridDim.x * (blockDim.x >> 5);
  for (uint32_t g = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); g < groups; g += warps_total) {
    const uint64_t base = (uint64_t)g * 256;
    float v[8];
    if (base + 256 <= n) {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[j] = __ldcs(x + base + lane + 32 * j);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        uint64_t at = base + lane + 32 * j;
        v[j] = at < n ? x[at] : -0.0f;
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(v[j], v[j + 4]);
    v[0] = __fadd_rn(v[0], v[2]);
    v[1] = __fadd_rn(v[1], v[3]);
    float t = __fadd_rn(v[0], v[1]);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) t = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, s));
    if (lane == 0) partials[g] = t;
  }
}

// Pass 2, one 256-lane group: lane l adds partials l, l + 256, ... from -0,
// then the lanes' sums are halved as in pass 1. Spread over `ctas` blocks
// that each compute 256 / ctas lanes' chains; the last block to finish
// halves them.
__global__ void __launch_bounds__(256) reduce_final_kernel(const float* __restrict__ partials,
                                                           uint32_t count, float* __restrict__ chains,
                                                           unsigned int* __restrict__ done,
                                                           float* __restrict__ y) {
  // Block b computes chains [32 b, 32 b + 32). The chains' terms come in
  // 64 at a time (warp w loads terms k0 + w + 8 i, i < 8, all in flight),
  // staged in shared memory; warp 0's lane l then adds chain 32 b + l's 64
  // terms in order.
  constexpr int kRows = 64;
  __shared__ float terms[kRows][32];
  __shared__ bool last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t chain = blockIdx.x * 32 + lane;
  float acc = -0.0f;
  const uint32_t per_chain = (count + 255) / 256;
  for (uint32_t k0 = 0; k0 < per_chain; k0 += kRows) {
#pragma unroll
    for (int i = 0; i < kRows / 8; ++i) {
      const uint32_t k = k0 + warp + 8 * i;
      const uint32_t at = chain + 256 * k;
      terms[warp + 8 * i][lane] = (k < per_chain && at < count) ? __ldcg(partials + at) : 0.0f;
    }
    __syncthreads();
    if (warp == 0) {
      const uint32_t rows = min((uint32_t)kRows, per_chain - k0);
      for (uint32_t j = 0; j < rows; ++j)
        if (chain + 256 * (k0 + j) < count) acc = __fadd_rn(acc, terms[j][lane]);
    }
    __syncthreads();
  }
  if (warp == 0) chains[chain] = acc;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  if (warp == 0) {
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) v[j] = __ldcg(chains + lane + 32 * j);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __fadd_rn(v[j], v[j + 4]);
    v[0] = __fadd_rn(v[0], v[2]);
    v[1] = __fadd_rn(v[1], v[3]);
    float t = __fadd_rn(v[0], v[1]);
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) t = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, s));
    if (lane == 0) {
      y[0] = t;
      *done = 0;  // ready for the next launch
    }
  }
}

// ---------------------------------------------------------------------------
// Row kernels: one 256-thread block per row; thread t takes packs t, t + 256,
// ... of four floats, held in registers between the passes (h <= 256 * 4 * PK).

template <int PK>
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const float* __restrict__ x,
                                                           const float* __restrict__ gamma,
                                                           float* __restrict__ y, uint32_t h,
                                                           float eps, float factor) {
  __shared__ float slots[8];
  const uint32_t row = blockIdx.x, t = threadIdx.x;
  const uint32_t packs = h >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * h);
  float4 v[PK];
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < PK; ++i) {
    uint32_t j = t + 256u * i;
    if (j < packs) {
      v[i] = __ldcs(xr + j);
      acc = __fadd_rn(acc, __fmul_rn(v[i].x, v[i].x));
      acc = __fadd_rn(acc, __fmul_rn(v[i].y, v[i].y));
      acc = __fadd_rn(acc, __fmul_rn(v[i].z, v[i].z));
      acc = __fadd_rn(acc, __fmul_rn(v[i].w, v[i].w));
    }
  }
  acc = warp_sum(acc);
  if ((t & 31) == 0) slots[t >> 5] = acc;
  __syncthreads();
  const float total = tg_sum8(slots);
  const float scale = rsqrt_rounded(__fadd_rn(__fdiv_rn(total, (float)h), eps));
  float4* yr = reinterpret_cast<float4*>(y + (size_t)row * h);
  const float4* g4 = reinterpret_cast<const float4*>(gamma);
#pragma unroll
  for (int i = 0; i < PK; ++i) {
    uint32_t j = t + 256u * i;
    if (j < packs) {
      float4 o = make_float4(__fmul_rn(v[i].x, scale), __fmul_rn(v[i].y, scale), __fmul_rn(v[i].z, scale),
                             __fmul_rn(v[i].w, scale));
      if (gamma) {
        float4 g = __ldg(g4 + j);
        o = make_float4(__fmul_rn(o.x, g.x), __fmul_rn(o.y, g.y), __fmul_rn(o.z, g.z), __fmul_rn(o.w, g.w));
      }
      if (factor != 1.0f)
        o = make_float4(__fmul_rn(o.x, factor), __fmul_rn(o.y, factor), __fmul_rn(o.z, factor),
                        __fmul_rn(o.w, factor));
      __stcs(yr + j, o);
    }
  }
}

template <int PK>
__global__ void __launch_bounds__(256) softmax_rows_kernel(const float* __restrict__ x,
                                                           float* __restrict__ y, uint32_t h) {
  __shared__ float slots[8];
  const uint32_t row = blockIdx.x, t = threadIdx.x;
  const uint32_t packs = h >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * h);
  float4 v[PK];
  float mx = -INFINITY;
#pragma unroll
  for (int i = 0; i < PK; ++i) {
    uint32_t j = t + 256u * i;
    if (j < packs) {
      v[i] = __ldcs(xr + j);
      mx = max_number(mx, v[i].x);
      mx = max_number(mx, v[i].y);
      mx = max_number(mx, v[i].z);
      mx = max_number(mx, v[i].w);
    }
  }
  mx = warp_max(mx);
  if ((t & 31) == 0) slots[t >> 5] = mx;
  __syncthreads();
  const float top = tg_max8(slots);
  __syncthreads();
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < PK; ++i) {
    uint32_t j = t + 256u * i;
    if (j < packs) {
      v[i].x = exp_rounded(__fsub_rn(v[i].x, top));
      acc = __fadd_rn(acc, v[i].x);
      v[i].y = exp_rounded(__fsub_rn(v[i].y, top));
      acc = __fadd_rn(acc, v[i].y);
      v[i].z = exp_rounded(__fsub_rn(v[i].z, top));
      acc = __fadd_rn(acc, v[i].z);
      v[i].w = exp_rounded(__fsub_rn(v[i].w, top));
      acc = __fadd_rn(acc, v[i].w);
    }
  }
  acc = warp_sum(acc);
  if ((t & 31) == 0) slots[t >> 5] = acc;
  __syncthreads();
  const float total = tg_sum8(slots);
  float4* yr = reinterpret_cast<float4*>(y + (size_t)row * h);
#pragma unroll
  for (int i = 0; i < PK; ++i) {
    uint32_t j = t + 256u * i;
    if (j < packs)
      __stcs(yr + j, make_float4(__fdiv_rn(v[i].x, total), __fdiv_rn(v[i].y, total), __fdiv_rn(v[i].z, total),
                                 __fdiv_rn(v[i].w, total)));
  }
}

}  // namespace fk

// ---------------------------------------------------------------------------
// Launchers

cudaError_t fk_launch_reduce_groups(const float* x, uint64_t n, float* partials, int sms, cudaStream_t s) {
  const uint32_t groups = (uint32_t)((n + 255) / 256);
  if (groups == 0) return cudaSuccess;
  // 8 warps a block, 8 blocks an SM resident: grid-stride over the groups.
  uint32_t blocks = (groups + 7) / 8;
  uint32_t cap = (uint32_t)sms * 8u;
  if (blocks > cap) blocks = cap;
  fk::reduce_groups_kernel<<<blocks, 256, 0, s>>>(x, n, partials, groups);
  return cudaGetLastError();
}

cudaError_t fk_launch_reduce_final(const float* partials, uint32_t count, float* chains, unsigned int* done,
                                   float* y, cudaStream_t s) {
  fk::reduce_final_kernel<<<8, 256, 0, s>>>(partials, count, chains, done, y);
  return cudaGetLastError();
}

cudaError_t fk_launch_rmsnorm_rows(const float* x, const float* gamma, float* y, uint32_t rows, uint32_t h,
                                   float eps, float factor, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const uint32_t packs = h / 4;
  if (packs <= 256)
    fk::rmsnorm_rows_kernel<1><<<rows, 256, 0, s>>>(x, gamma, y, h, eps, factor);
  else if (packs <= 1024)
    fk::rmsnorm_rows_kernel<4><<<rows, 256, 0, s>>>(x, gamma, y, h, eps, factor);
  else if (packs <= 4096)
    fk::rmsnorm_rows_kernel<16><<<rows, 256, 0, s>>>(x, gamma, y, h, eps, factor);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t fk_launch_softmax_rows(const float* x, float* y, uint32_t rows, uint32_t h, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  const uint32_t packs = h / 4;
  if (packs <= 256)
    fk::softmax_rows_kernel<1><<<rows, 256, 0, s>>>(x, y, h);
  else if (packs <= 1024)
    fk::softmax_rows_kernel<4><<<rows, 256, 0, s>>>(x, y, h);
  else if (packs <= 4096)
    fk::softmax_rows_kernel<16><<<rows, 256, 0, s>>>(x, y, h);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}
