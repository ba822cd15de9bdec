// Elementwise work, the embedding gather, the greedy pick, and the seeded
// fills that make a synthetic model's weights on the device.
#include <math.h>

#include "fk_common.cuh"
#include "fk_kernels.h"
#include "fk_peers.cuh"

namespace fk {

// Gather (src/FuryKernel/Program/Eval.hs:528-535), one token a row:
// y = table[token] * factor. Grid (ceil(width / 1024), m), 256 threads of
// one pack each.
__global__ void gather_kernel(const float* __restrict__ table, uint32_t width, const uint32_t* __restrict__ tokens,
                              float factor, float* __restrict__ y) {
  grid_wait();
  grid_launch_dependents();
  const uint32_t r = blockIdx.y;
  const uint32_t j = blockIdx.x * 256u + threadIdx.x;
  if (4 * j >= width) return;
  const float4* src = reinterpret_cast<const float4*>(table + (size_t)tokens[r] * width);
  float4 v = __ldg(src + j);
  if (factor != 1.0f) v = make_float4(__fmul_rn(v.x, factor), __fmul_rn(v.y, factor), __fmul_rn(v.z, factor),
                                      __fmul_rn(v.w, factor));
  reinterpret_cast<float4*>(y + (size_t)r * width)[j] = v;
}

// One thread's part of a row's first maximum: elements t, t + T, ... (or,
// with vec, packs of 4 at t, t + T, ..., four packs in flight, then the
// tail past the last whole pack), in increasing index order; an element is
// taken when greater than the best so far, or when it is the first
// candidate equal to it (-inf), never a NaN.
__device__ __forceinline__ void scan_first_max(const float* __restrict__ xr, uint32_t n, bool vec, float& bv,
                                               uint32_t& bi) {
  bv = -INFINITY;
  bi = 0xffffffffu;
  auto take = [&](float v, uint32_t j) {
    if (v > bv || (bi == 0xffffffffu && v == bv)) {
      bv = v;
      bi = j;
    }
  };
  const uint32_t T = blockDim.x;
  uint32_t j0 = 0;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(xr);
    const uint32_t packs = n / 4;
    uint32_t p = threadIdx.x;
    for (; p + 3 * T < packs; p += 4 * T) {
      float4 q[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) q[u] = __ldg(x4 + p + u * T);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t j = 4 * (p + u * T);
        take(q[u].x, j);
        take(q[u].y, j + 1);
        take(q[u].z, j + 2);
        take(q[u].w, j + 3);
      }
    }
    for (; p < packs; p += T) {
      const float4 q = __ldg(x4 + p);
      take(q.x, 4 * p);
      take(q.y, 4 * p + 1);
      take(q.z, 4 * p + 2);
      take(q.w, 4 * p + 3);
    }
    j0 = 4 * packs;
  }
  for (uint32_t j = j0 + threadIdx.x; j < n; j += T) take(xr[j], j);
}

// ArgMax (Eval.hs:545-548, 684-685): the fold keeps the first index whose
// value is greater than all before it, so NaNs past the first element are
// never taken and a NaN first element is the answer. Each thread scans its
// elements in index order (scan_first_max); pairs combine by "greater, or
// equal at a lower index". Grid m, 1024 threads.
__global__ void __launch_bounds__(1024) argmax_kernel(const float* __restrict__ x, uint32_t n, uint32_t ldx,
                                                      uint32_t* __restrict__ ids) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  grid_wait();
  grid_launch_dependents();
  const uint32_t r = blockIdx.x;
  const float* xr = x + (size_t)r * ldx;
  float bv;
  uint32_t bi;
  scan_first_max(xr, n, ((uintptr_t)x % 16 == 0) && ldx % 4 == 0, bv, bi);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0xffffffffu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) ids[r] = isnan(xr[0]) || bi == 0xffffffffu ? 0u : bi;
  }
}

// A vocabulary shard's greedy candidate per row: its largest value and
// that value's index plus the shard's offset, as argmax_kernel finds it
// (first index of the maximum; a NaN first element wins). Grid m, 1024 threads.
__global__ void __launch_bounds__(1024) argmax_pairs_kernel(const float* __restrict__ x, uint32_t n, uint32_t ldx,
                                                            uint32_t offset, uint32_t* __restrict__ pairs,
                                                            FkPeers peers, int scatter) {
  __shared__ float sv[32];
  __shared__ uint32_t si[32];
  grid_wait();
  grid_launch_dependents();
  const uint32_t r = blockIdx.x;
  const float* xr = x + (size_t)r * ldx;
  float bv;
  uint32_t bi;
  scan_first_max(xr, n, ((uintptr_t)x % 16 == 0) && ldx % 4 == 0, bv, bi);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_down_sync(0xffffffffu, bv, o);
    const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = bv;
    si[warp] = bi;
  }
  __syncthreads();
  if (warp == 0) {
    bv = lane < (int)(blockDim.x >> 5) ? sv[lane] : -INFINITY;
    bi = lane < (int)(blockDim.x >> 5) ? si[lane] : 0xffffffffu;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_down_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if (lane == 0) {
      // Only the row's first element, in the first shard, wins as a NaN;
      // a shard of NaNs alone offers no candidate (index 0xffffffff).
      if (offset == 0 && isnan(xr[0])) {
        bv = xr[0];
        bi = 0;
      }
      const uint32_t idx = bi == 0xffffffffu ? bi : bi + offset;
      if (scatter) {  // into every rank's exchange buffer 2, this rank's slot
        for (uint32_t q = 0; q < peers.world; ++q) {
          uint32_t* slot = reinterpret_cast<uint32_t*>(xdata(peers.base[q], 2, peers.rank));
          slot[2 * r] = __float_as_uint(bv);
          slot[2 * r + 1] = idx;
        }
      } else {
        pairs[2 * r] = __float_as_uint(bv);
        pairs[2 * r + 1] = idx;
      }
    }
  }
  if (scatter) peers_signal(peers, 2, (threadIdx.x & 31) == 0);
}

// The greedy id from the shards' candidates, [shards][m][2], in shard order:
// the fold over the whole row keeps the first shard's NaN-first candidate,
// else the largest value, ties to the lower index.
__global__ void argmax_pick_kernel(const uint32_t* __restrict__ pairs, uint32_t shards, uint32_t m,
                                   uint32_t* __restrict__ ids, FkPeers peers, int gather, int* err) {
  grid_wait();
  grid_launch_dependents();
  if (gather) peers_wait(peers, 2, err);
  // Shard s's candidates: gathered by NCCL at pairs + 2 s m, or in this
  // rank's exchange buffer 2, slot s.
  auto src = [&](uint32_t s) -> const uint32_t* {
    return gather ? reinterpret_cast<const uint32_t*>(xdata(peers.base[peers.rank], 2, s)) : pairs + (size_t)s * m * 2;
  };
  for (uint32_t r = threadIdx.x; r < m; r += blockDim.x) {
    float bv = __uint_as_float(src(0)[2 * r]);
    uint32_t bi = src(0)[2 * r + 1];
    if (!isnan(bv)) {
      for (uint32_t s = 1; s < shards; ++s) {
        const float v = __uint_as_float(src(s)[2 * r]);
        const uint32_t i = src(s)[2 * r + 1];
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
    }
    ids[r] = bi;
  }
}

__global__ void add_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                           uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x)
    y[i] = __fadd_rn(a[i], b[i]);
}

// The same sums, four a thread with 16-byte loads and stores (n4 = n / 4;
// every array 16-byte aligned).
__global__ void add4_kernel(const float4* __restrict__ a, const float4* __restrict__ b, float4* __restrict__ y,
                            uint64_t n4) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n4; i += (uint64_t)gridDim.x * blockDim.x) {
    const float4 u = a[i], v = b[i];
    y[i] = make_float4(__fadd_rn(u.x, v.x), __fadd_rn(u.y, v.y), __fadd_rn(u.z, v.z), __fadd_rn(u.w, v.w));
  }
}

// SiLU-gate, silu(a) * b with silu(a) = a / (1 + exp(-a)).
__global__ void silu_mul_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ y,
                                uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const float e = exp_rounded(-a[i]);
    y[i] = __fmul_rn(__fdiv_rn(a[i], __fadd_rn(1.0f, e)), b[i]);
  }
}

// The SiLU-gate of interleaved (gate, up) pairs, as silu_mul computes it:
// y[i] = silu(x[2i]) * x[2i + 1] (a GEMM over gate/up rows interleaved).
__global__ void silu_pairs_kernel(const float2* __restrict__ x, float* __restrict__ y, uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const float2 gu = x[i];
    const float e = exp_rounded(-gu.x);
    y[i] = __fmul_rn(__fdiv_rn(gu.x, __fadd_rn(1.0f, e)), gu.y);
  }
}

// Seeded inputs: SplitMix's finaliser of seed * golden + i, i from 1
// (test/cpu/Cases.hs:885-892). N(mu, sigma) by Box-Muller on consecutive
// words, in binary64 rounded once; U(a, b) from the top 24 bits.
__device__ __forceinline__ uint64_t splitmix(uint64_t seed, uint64_t i) {
  uint64_t z = seed * 0x9E3779B97F4A7C15ULL + i;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__global__ void fill_normal_kernel(float* __restrict__ out, uint64_t n, uint64_t seed, double mu, double sigma) {
  const uint64_t pairs = (n + 1) / 2;
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < pairs;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t w1 = splitmix(seed, 2 * p + 1), w2 = splitmix(seed, 2 * p + 2);
    const double u1 = ((double)(w1 >> 11) + 1.0) * 0x1p-53;
    const double u2 = (double)(w2 >> 11) * 0x1p-53;
    const double rr = sqrt(-2.0 * log(u1));
    const double t = 6.283185307179586 * u2;
    out[2 * p] = (float)(mu + sigma * (rr * cos(t)));
    if (2 * p + 1 < n) out[2 * p + 1] = (float)(mu + sigma * (rr * sin(t)));
  }
}

__global__ void fill_uniform_kernel(float* __restrict__ out, uint64_t n, uint64_t seed, double a, double b) {
  for (uint64_t j = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; j < n; j += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t w = splitmix(seed, j + 1);
    out[j] = (float)(a + (b - a) * ((double)(w >> 40) * 0x1p-24));
  }
}

// The engine's greedy feedback between decode steps: each row's next token
// is its greedy id and its position advances by one.
__global__ void advance_kernel(const uint32_t* __restrict__ ids, uint32_t* __restrict__ tokens,
                               uint32_t* __restrict__ pos, uint32_t m) {
  grid_wait();
  grid_launch_dependents();
  for (uint32_t r = threadIdx.x; r < m; r += blockDim.x) {
    tokens[r] = ids[r];
    pos[r] = pos[r] + 1u;
  }
}

}  // namespace fk

cudaError_t fk_launch_argmax_pairs(const float* x, uint32_t m, uint32_t n, uint32_t ldx, uint32_t offset,
                                   uint32_t* pairs, const FkPeers* peers, bool pdl, cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (n == 0 || (peers && 2 * (size_t)m > FK_XSLOT)) return cudaErrorInvalidValue;
  FkPeers none = {};
  return fk_launch_ex(fk::argmax_pairs_kernel, dim3(m), dim3(1024), 0, s, pdl, x, n, ldx, offset, pairs,
                      peers ? *peers : none, peers ? 1 : 0);
}

cudaError_t fk_launch_argmax_pick(const uint32_t* pairs, uint32_t shards, uint32_t m, uint32_t* ids,
                                  const FkPeers* peers, int* err, bool pdl, cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (peers && shards != peers->world) return cudaErrorInvalidValue;
  FkPeers none = {};
  return fk_launch_ex(fk::argmax_pick_kernel, dim3(1), dim3(256), 0, s, pdl, pairs, shards, m, ids,
                      peers ? *peers : none, peers ? 1 : 0, err);
}

cudaError_t fk_launch_advance(const uint32_t* ids, uint32_t* tokens, uint32_t* pos, uint32_t m, bool pdl,
                              cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  return fk_launch_ex(fk::advance_kernel, dim3(1), dim3(256), 0, s, pdl, ids, tokens, pos, m);
}

cudaError_t fk_launch_gather(const float* table, uint32_t width, const uint32_t* tokens, uint32_t m, float factor,
                             float* y, bool pdl, cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (width % 4 != 0) return cudaErrorInvalidValue;
  return fk_launch_ex(fk::gather_kernel, dim3((width / 4 + 255) / 256, m), dim3(256), 0, s, pdl, table, width, tokens,
                      factor, y);
}

cudaError_t fk_launch_argmax(const float* x, uint32_t m, uint32_t n, uint32_t ldx, uint32_t* ids, bool pdl,
                             cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (n == 0) return cudaErrorInvalidValue;
  return fk_launch_ex(fk::argmax_kernel, dim3(m), dim3(1024), 0, s, pdl, x, n, ldx, ids);
}

static unsigned grid_for(uint64_t n) {
  uint64_t b = (n + 255) / 256;
  return (unsigned)(b > 148ull * 64 ? 148ull * 64 : (b == 0 ? 1 : b));
}

cudaError_t fk_launch_add(const float* a, const float* b, float* y, uint64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (n % 4 == 0 && (((uintptr_t)a | (uintptr_t)b | (uintptr_t)y) & 15) == 0)
    fk::add4_kernel<<<grid_for(n / 4), 256, 0, s>>>(reinterpret_cast<const float4*>(a),
                                                    reinterpret_cast<const float4*>(b), reinterpret_cast<float4*>(y),
                                                    n / 4);
  else
    fk::add_kernel<<<grid_for(n), 256, 0, s>>>(a, b, y, n);
  return cudaGetLastError();
}

cudaError_t fk_launch_silu_mul(const float* a, const float* b, float* y, uint64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fk::silu_mul_kernel<<<grid_for(n), 256, 0, s>>>(a, b, y, n);
  return cudaGetLastError();
}

cudaError_t fk_launch_silu_pairs(const float* x, float* y, uint64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  if (reinterpret_cast<uintptr_t>(x) & 7) return cudaErrorInvalidValue;
  fk::silu_pairs_kernel<<<grid_for(n), 256, 0, s>>>(reinterpret_cast<const float2*>(x), y, n);
  return cudaGetLastError();
}

cudaError_t fk_launch_fill_normal(float* out, uint64_t n, uint64_t seed, double mu, double sigma, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fk::fill_normal_kernel<<<grid_for((n + 1) / 2), 256, 0, s>>>(out, n, seed, mu, sigma);
  return cudaGetLastError();
}

cudaError_t fk_launch_fill_uniform(float* out, uint64_t n, uint64_t seed, double a, double b, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fk::fill_uniform_kernel<<<grid_for(n), 256, 0, s>>>(out, n, seed, a, b);
  return cudaGetLastError();
}
