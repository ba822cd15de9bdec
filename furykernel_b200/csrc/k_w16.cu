// A decode step whose weights are 16-bit: bf16, the element type the
// reference's program builder gives a model's weights (`weight`,
// src/FuryKernel/Program/Build.hs:171-175), or f16, the other 16-bit type a
// weight may hold (src/FuryKernel/Program/Check.hs:105-111). Activations,
// sums and outputs stay binary32, and every weight is widened to binary32
// where it is read, exactly (widenBF16 and widenF16,
// src/FuryKernel/Numerics.hs:33-38 and :51-66; fk_elem16.cuh). So each kernel here
// keeps the arithmetic and the order of its f32 counterpart over the widened
// weights -- the GEMV order contract at pack 4 and split s
// (test/Test/FuryKernel/Gemv.hs:9-26), RMSNorm's 256-lane order, the
// SiLU-gate -- and the f32 oracle over the widened weights gives its bits,
// while the weights' HBM bytes halve.
//
// Widening does not quiet a NaN here (the reference's widening does): a NaN
// weight makes a NaN sum either way. Each kernel takes the element type as
// a tag (fk::Bf16, fk::F16).
//
// Kernels: the weight-streaming GEMV for batches of up to 4 rows
// (gemv_stream_w16_kernel, persistent, x staged once a block with its
// prologue, every epilogue including the tensor-parallel scatter and the
// reduce-then-normalize prologue), the packed batched GEMV for up to 64 rows
// at split 1 (k_w16_batch.cu), the chunked GEMV for the rest
// (gemv_chunk_w16_kernel, 32 rows a launch), the embedding gather, RMSNorm
// rows with a 16-bit gain, the TF32 split of 16-bit weights (exact: a bf16
// value has 8 significant bits, an f16 value 11 and a TF32 value 11, and
// f16's exponents are within TF32's, so the low half is 0), and the seeded
// normal fill rounded to the weights' type.
#include "fk_common.cuh"
#include "fk_elem16.cuh"
#include "fk_kernels.h"
#include "fk_peers.cuh"

namespace fk {
namespace w16 {

// Streaming load of a pack's raw bits: read once, no L1 allocation.
__device__ __forceinline__ uint2 ld_stream2(const uint2* p) {
  uint2 v;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
  return v;
}

// Pack j of a 16-bit gain, widened.
template <class E>
__device__ __forceinline__ float4 gain4(const uint16_t* gamma, uint32_t j) {
  return E::widen4(__ldg(reinterpret_cast<const uint2*>(gamma) + j));
}

struct StreamArgs {
  const uint16_t* w;
  const float* x;
  const uint16_t* gamma;
  const float* r;
  float* y;
  uint32_t n, k, m, split;
  uint32_t ldx, ldr, ldy;
  uint32_t up_off;
  float eps, factor;
  FkPeers peers;
  uint32_t xbuf;
  float* xout;
  int* err;
  size_t prefetch;  // bulk L2 prefetch budget of the launch (FkGemv::prefetch)
};

enum { SPRO_NONE = 0, SPRO_RMSNORM = 1, SPRO_SILU = 2, SPRO_REDUCE_RMSNORM = 3 };
enum { SEPI_NONE = 0, SEPI_ADD = 1, SEPI_SILU_PAIR = 2, SEPI_SCATTER = 3 };
constexpr int kStreamWarps = 16;
constexpr uint32_t kScatterRows = 128;
constexpr int kInFlight = 16;  // packs of 8 bytes a lane has requested at once

__device__ __forceinline__ float silu_of(float a, float b) {
  const float e = exp_rounded(-a);
  return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, e)), b);
}

// One row's totals for the staged rows of x, in the contract's order: split
// q, lane l visits packs q*32 + l, + 32 s, ...; chains from 0; lanes summed
// pairwise; splits added in order.
template <class E, int M>
__device__ __forceinline__ void row_totals(const uint2* __restrict__ wr, const float4* __restrict__ xs4,
                                           uint32_t packs, uint32_t m, uint32_t s, int lane, float (&total)[M]) {
  const uint32_t stride = 32u * s;
  for (uint32_t q = 0; q < s; ++q) {
    float acc[M];
#pragma unroll
    for (int i = 0; i < M; ++i) acc[i] = 0.0f;
    uint32_t j = q * 32u + (uint32_t)lane;
    for (; j + (kInFlight - 1) * stride < packs; j += kInFlight * stride) {
      uint2 raw[kInFlight];
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) raw[u] = ld_stream2(wr + j + u * stride);
#pragma unroll
      for (int u = 0; u < kInFlight; ++u) {
        const float4 wv = E::widen4(raw[u]);
#pragma unroll
        for (int i = 0; i < M; ++i)
          if (i < (int)m) acc[i] = __fadd_rn(acc[i], pack_dot(xs4[(size_t)i * packs + j + u * stride], wv));
      }
    }
    for (; j < packs; j += stride) {
      const float4 wv = E::widen4(ld_stream2(wr + j));
#pragma unroll
      for (int i = 0; i < M; ++i)
        if (i < (int)m) acc[i] = __fadd_rn(acc[i], pack_dot(xs4[(size_t)i * packs + j], wv));
    }
#pragma unroll
    for (int i = 0; i < M; ++i) {
      const float part = warp_sum(acc[i]);
      total[i] = q == 0 ? part : __fadd_rn(total[i], part);
    }
  }
}

// Two rows' totals at once (a gate/up pair, or two units of a warp), each
// in row_totals' order: their loads interleaved, 8 packs of each row in
// flight a lane, so that a warp has as many bytes in flight as with one
// row but pays the pause between rows (the last loads' latency, the lanes'
// sums) once for the two.
template <class E, int M>
__device__ __forceinline__ void row_totals2(const uint2* __restrict__ wa, const uint2* __restrict__ wb,
                                            const float4* __restrict__ xs4, uint32_t packs, uint32_t m, uint32_t s,
                                            int lane, float (&ta)[M], float (&tb)[M]) {
  constexpr int F = kInFlight / 2;
  const uint32_t stride = 32u * s;
  for (uint32_t q = 0; q < s; ++q) {
    float acca[M], accb[M];
#pragma unroll
    for (int i = 0; i < M; ++i) acca[i] = accb[i] = 0.0f;
    uint32_t j = q * 32u + (uint32_t)lane;
    for (; j + (F - 1) * stride < packs; j += F * stride) {
      uint2 ra[F], rb[F];
#pragma unroll
      for (int u = 0; u < F; ++u) {
        ra[u] = ld_stream2(wa + j + u * stride);
        rb[u] = ld_stream2(wb + j + u * stride);
      }
#pragma unroll
      for (int u = 0; u < F; ++u) {
        const float4 va = E::widen4(ra[u]), vb = E::widen4(rb[u]);
#pragma unroll
        for (int i = 0; i < M; ++i)
          if (i < (int)m) {
            const float4 xv = xs4[(size_t)i * packs + j + u * stride];
            acca[i] = __fadd_rn(acca[i], pack_dot(xv, va));
            accb[i] = __fadd_rn(accb[i], pack_dot(xv, vb));
          }
      }
    }
    for (; j < packs; j += stride) {
      const float4 va = E::widen4(ld_stream2(wa + j)), vb = E::widen4(ld_stream2(wb + j));
#pragma unroll
      for (int i = 0; i < M; ++i)
        if (i < (int)m) {
          const float4 xv = xs4[(size_t)i * packs + j];
          acca[i] = __fadd_rn(acca[i], pack_dot(xv, va));
          accb[i] = __fadd_rn(accb[i], pack_dot(xv, vb));
        }
    }
#pragma unroll
    for (int i = 0; i < M; ++i) {
      const float pa = warp_sum(acca[i]), pb = warp_sum(accb[i]);
      ta[i] = q == 0 ? pa : __fadd_rn(ta[i], pa);
      tb[i] = q == 0 ? pb : __fadd_rn(tb[i], pb);
    }
  }
}

// Persistent blocks of 16 warps; unit u (a row, or a gate/up row pair) goes
// to block u mod G and, within it, warp (u / G) mod 16; a scattering block
// owns the contiguous rows [s_lo, s_hi) instead.
template <class E, int M, int PRO, int EPI>
__global__ void __launch_bounds__(512, 2) gemv_stream_w16_kernel(StreamArgs a) {
  extern __shared__ float4 xs4[];  // [m][k / 4]
  __shared__ float scales[M];
  __shared__ float slots[8];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t packs = a.k >> 2;
  const uint32_t per_unit = EPI == SEPI_SILU_PAIR ? 2u : 1u;
  const uint32_t units = a.n / per_unit;
  const uint32_t G = gridDim.x;

  // The weights depend on no earlier launch: while the previous kernels
  // finish, start this block's rows toward L2. With a prefetch budget
  // (fkc_set_prefetch), the copy engine brings the block's units in the
  // order its warps read them (warp w: slots w, w + 16, ...) up to the
  // block's share of the budget; otherwise each warp's first 8 KB.
  {
    const size_t unit_bytes = (size_t)per_unit * a.k * 2;
    if (a.prefetch > 0) {
      const uint32_t p_lo = EPI == SEPI_SCATTER ? (uint32_t)((uint64_t)units * blockIdx.x / G) : 0u;
      const uint32_t p_hi = EPI == SEPI_SCATTER ? (uint32_t)((uint64_t)units * (blockIdx.x + 1) / G) : 0u;
      const size_t budget = a.prefetch / G;
      if (lane == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 && unit_bytes % 16 == 0 && unit_bytes <= 0xFFFFFFF0u) {
        for (uint32_t slot = (uint32_t)warp; (size_t)slot * unit_bytes < budget; slot += kStreamWarps) {
          const uint32_t u = EPI == SEPI_SCATTER ? p_lo + slot : blockIdx.x + slot * G;
          if (EPI == SEPI_SCATTER ? u >= p_hi : u >= units) break;
          prefetch_l2_bulk(a.w + (size_t)u * per_unit * a.k, (uint32_t)unit_bytes);
        }
      }
    } else {
      const uint32_t u0 = EPI == SEPI_SCATTER ? (uint32_t)((uint64_t)units * blockIdx.x / G) + (uint32_t)warp
                                              : blockIdx.x + (uint32_t)warp * G;
      if (u0 < units) {
        const char* row = reinterpret_cast<const char*>(a.w + (size_t)u0 * per_unit * a.k);
        for (size_t off = (size_t)lane * 128; off < unit_bytes && off < 8192; off += 32 * 128)
          asm volatile("prefetch.global.L2 [%0];" ::"l"(row + off));
      }
    }
  }
  grid_wait();
  grid_launch_dependents();

  constexpr bool NORM = PRO == SPRO_RMSNORM || PRO == SPRO_REDUCE_RMSNORM;
  if (PRO == SPRO_REDUCE_RMSNORM) peers_wait_rows(a.peers, a.xbuf, a.k, a.err);
  for (uint32_t idx = threadIdx.x; idx < a.m * packs; idx += blockDim.x) {
    const uint32_t i = idx / packs, j = idx - i * packs;
    const float* xr = a.x + (size_t)i * a.ldx;
    float4 v = __ldg(reinterpret_cast<const float4*>(xr) + j);
    if (PRO == SPRO_SILU) {
      const float4 u = __ldg(reinterpret_cast<const float4*>(xr + a.up_off) + j);
      v = make_float4(silu_of(v.x, u.x), silu_of(v.y, u.y), silu_of(v.z, u.z), silu_of(v.w, u.w));
    } else if (PRO == SPRO_REDUCE_RMSNORM) {
      char* me = a.peers.base[a.peers.rank];
      float4 s = reinterpret_cast<const float4*>(xdata(me, a.xbuf, 0) + (size_t)i * a.k)[j];
      for (uint32_t q = 1; q < a.peers.world; ++q) {
        const float4 p = reinterpret_cast<const float4*>(xdata(me, a.xbuf, q) + (size_t)i * a.k)[j];
        s = make_float4(__fadd_rn(s.x, p.x), __fadd_rn(s.y, p.y), __fadd_rn(s.z, p.z), __fadd_rn(s.w, p.w));
      }
      v = make_float4(__fadd_rn(v.x, s.x), __fadd_rn(v.y, s.y), __fadd_rn(v.z, s.z), __fadd_rn(v.w, s.w));
      if (blockIdx.x == 0) reinterpret_cast<float4*>(a.xout + (size_t)i * a.k)[j] = v;
    }
    xs4[(size_t)i * packs + j] = v;
  }
  __syncthreads();
  if (NORM) {
    // RMSNorm of each staged row: threads 0..255 are the spec's 256 lanes
    // over packs t, t + 256, ... (src/FuryKernel/Reduce.hs:59-85); then
    // x * scale * gamma (* factor) in place, gamma widened.
    for (uint32_t i = 0; i < a.m; ++i) {
      if (threadIdx.x < 256) {
        float acc = 0.0f;
        for (uint32_t j = threadIdx.x; j < packs; j += 256u) {
          const float4 v = xs4[(size_t)i * packs + j];
          acc = __fadd_rn(acc, __fmul_rn(v.x, v.x));
          acc = __fadd_rn(acc, __fmul_rn(v.y, v.y));
          acc = __fadd_rn(acc, __fmul_rn(v.z, v.z));
          acc = __fadd_rn(acc, __fmul_rn(v.w, v.w));
        }
        acc = warp_sum(acc);
        if (lane == 0) slots[warp] = acc;
      }
      __syncthreads();
      if (threadIdx.x == 0) scales[i] = rsqrt_rounded(__fadd_rn(__fdiv_rn(tg_sum8(slots), (float)a.k), a.eps));
      __syncthreads();
    }
    for (uint32_t idx = threadIdx.x; idx < a.m * packs; idx += blockDim.x) {
      const uint32_t i = idx / packs, j = idx - i * packs;
      float4 v = xs4[(size_t)i * packs + j];
      const float sc = scales[i];
      v = make_float4(__fmul_rn(v.x, sc), __fmul_rn(v.y, sc), __fmul_rn(v.z, sc), __fmul_rn(v.w, sc));
      if (a.gamma) {
        const float4 g = gain4<E>(a.gamma, j);
        v = make_float4(__fmul_rn(v.x, g.x), __fmul_rn(v.y, g.y), __fmul_rn(v.z, g.z), __fmul_rn(v.w, g.w));
      }
      if (a.factor != 1.0f)
        v = make_float4(__fmul_rn(v.x, a.factor), __fmul_rn(v.y, a.factor), __fmul_rn(v.z, a.factor),
                        __fmul_rn(v.w, a.factor));
      xs4[(size_t)i * packs + j] = v;
    }
    __syncthreads();
  }

  __shared__ float outs[EPI == SEPI_SCATTER ? M : 1][EPI == SEPI_SCATTER ? kScatterRows : 1];
  const uint32_t s_lo = (uint32_t)((uint64_t)units * blockIdx.x / G);
  const uint32_t s_hi = (uint32_t)((uint64_t)units * (blockIdx.x + 1) / G);
  // Weight rows are k bf16 = k / 4 packs of 8 bytes.
  const uint2* w2 = reinterpret_cast<const uint2*>(a.w);
  // A unit's totals out: staged (scatter), or through the epilogue to y.
  auto emit = [&](uint32_t u, const float(&t0)[M], const float(&t1)[M]) {
    if (lane != 0) return;
#pragma unroll
    for (int i = 0; i < M; ++i) {
      if (i >= (int)a.m) break;
      if (EPI == SEPI_SCATTER) {
        outs[i][u - s_lo] = t0[i];
        continue;
      }
      float v;
      if (EPI == SEPI_SILU_PAIR)
        v = silu_of(t0[i], t1[i]);
      else if (EPI == SEPI_ADD)
        v = __fadd_rn(a.r[(size_t)i * a.ldr + u], t0[i]);
      else
        v = t0[i];
      a.y[(size_t)i * a.ldy + u] = v;
    }
  };
  // At batch 1 a warp takes its slots two at a time (a gate/up unit's two
  // rows, or two one-row units), their rows' loads interleaved
  // (row_totals2); larger batches keep one row at a time, whose
  // accumulators would not fit twice in the 64 registers a thread has.
  constexpr bool PAIRED = M == 1;
  auto unit_of = [&](uint32_t slot) { return EPI == SEPI_SCATTER ? s_lo + slot : blockIdx.x + slot * G; };
  auto live = [&](uint32_t u) { return EPI == SEPI_SCATTER ? u < s_hi : u < units; };
  for (uint32_t slot = (uint32_t)warp;; slot += (EPI == SEPI_SILU_PAIR || !PAIRED ? 1u : 2u) * kStreamWarps) {
    const uint32_t u = unit_of(slot);
    if (!live(u)) break;
    float t0[M], t1[M];
    if (EPI == SEPI_SILU_PAIR) {
      if (PAIRED) {
        row_totals2<E, M>(w2 + (size_t)u * 2 * packs, w2 + ((size_t)u * 2 + 1) * packs, xs4, packs, a.m, a.split,
                          lane, t0, t1);
      } else {
        row_totals<E, M>(w2 + (size_t)u * 2 * packs, xs4, packs, a.m, a.split, lane, t0);
        row_totals<E, M>(w2 + ((size_t)u * 2 + 1) * packs, xs4, packs, a.m, a.split, lane, t1);
      }
      emit(u, t0, t1);
    } else if (!PAIRED) {
      row_totals<E, M>(w2 + (size_t)u * packs, xs4, packs, a.m, a.split, lane, t0);
      emit(u, t0, t0);
    } else {
      const uint32_t u2 = unit_of(slot + kStreamWarps);
      if (live(u2)) {
        row_totals2<E, M>(w2 + (size_t)u * packs, w2 + (size_t)u2 * packs, xs4, packs, a.m, a.split, lane, t0, t1);
        emit(u, t0, t1);
        emit(u2, t1, t1);
      } else {
        row_totals<E, M>(w2 + (size_t)u * packs, xs4, packs, a.m, a.split, lane, t0);
        emit(u, t0, t0);
      }
    }
  }
  if (EPI == SEPI_SCATTER) {
    // This rank's partial rows [s_lo, s_hi) into its slot of every rank's
    // region, then counted in (fk_peers.cuh).
    __syncthreads();
    const uint32_t cnt = s_hi - s_lo;
    for (uint32_t q = 0; q < a.peers.world; ++q) {
      float* dst = xdata(a.peers.base[q], a.xbuf, a.peers.rank);
      for (uint32_t idx = threadIdx.x; idx < a.m * cnt; idx += blockDim.x) {
        const uint32_t i = idx / cnt, j = idx - i * cnt;
        dst[(size_t)i * a.n + s_lo + j] = outs[i][j];
      }
    }
    peers_count_rows(a.peers, a.xbuf, units);
  }
}

template <class E, int M, int PRO, int EPI>
static cudaError_t launch_stream(const StreamArgs& a, int sms, cudaStream_t st, bool pdl) {
  auto kern = gemv_stream_w16_kernel<E, M, PRO, EPI>;
  const size_t smem = (size_t)a.m * a.k * sizeof(float);
  cudaError_t e = fk_allow_smem(kern, smem);
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 512, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidValue;
  if (per_sm > 2) per_sm = 2;
  const uint32_t units = EPI == SEPI_SILU_PAIR ? a.n / 2 : a.n;
  uint32_t blocks = (uint32_t)(sms * per_sm);
  if (blocks > units) blocks = units;
  if (EPI == SEPI_SCATTER && (units + blocks - 1) / blocks > kScatterRows) return cudaErrorInvalidValue;
  return fk_launch_ex(kern, dim3(blocks), dim3(512), smem, st, pdl, a);
}

template <class E, int PRO, int EPI>
static cudaError_t stream_m(const StreamArgs& a, int sms, cudaStream_t st, bool pdl) {
  if (a.m <= 1) return launch_stream<E, 1, PRO, EPI>(a, sms, st, pdl);
  if (a.m <= 2) return launch_stream<E, 2, PRO, EPI>(a, sms, st, pdl);
  return launch_stream<E, 4, PRO, EPI>(a, sms, st, pdl);
}

// ---------------------------------------------------------------------------
// The chunked GEMV (batches past 4 rows): blocks of 8 warps, 8 / s rows of s
// splits each; x staged a chunk of k at a time with its prologue.

struct ChunkArgs {
  const uint16_t* w;
  const float* x;
  const uint16_t* gamma;
  const float* r;
  float* y;
  uint32_t n, k, m, split;
  uint32_t ldx, ldr, ldy;
  uint32_t up_off;
  uint32_t kc;  // staged chunk of k, a multiple of 4
  float eps, factor;
};

enum { PRO_NONE = 0, PRO_RMSNORM = 1, PRO_SILU = 2 };

// RMSNorm's scale of one row by one warp playing the 256 spec lanes: lane l
// plays lanes l + 32 g, g < 8, each over packs (l + 32 g) + 256 t in order;
// each group of 32 summed pairwise; the 8 sums combined as tgReduceSum.
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
  return rsqrt_rounded(__fadd_rn(__fdiv_rn(tg_sum8(slots), (float)k), eps));
}

template <class E, int M, int PRO, bool ADD>
__global__ void __launch_bounds__(256) gemv_chunk_w16_kernel(ChunkArgs a) {
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
  const uint2* wr = reinterpret_cast<const uint2*>(a.w) + (size_t)(active ? row : 0) * packs;

  if (active && (lane & 15) == 0) {
    for (uint32_t j = v; j < packs && j < v + 8u * stride; j += stride)
      asm volatile("prefetch.global.L2 [%0];" ::"l"(wr + j));
  }
  grid_wait();
  grid_launch_dependents();

  if (PRO == PRO_RMSNORM) {
    for (uint32_t i = warp; i < a.m; i += 8) {
      const float sc = rmsnorm_scale_warp(a.x + (size_t)i * a.ldx, a.k, a.eps);
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
    for (uint32_t idx = threadIdx.x; idx < a.m * width; idx += 256u) {
      const uint32_t i = idx / width, p = idx - i * width, j = c0 + p;
      const float* xr = a.x + (size_t)i * a.ldx;
      float4 xv = __ldg(reinterpret_cast<const float4*>(xr) + j);
      if (PRO == PRO_RMSNORM) {
        const float sc = scales[i];
        xv = make_float4(__fmul_rn(xv.x, sc), __fmul_rn(xv.y, sc), __fmul_rn(xv.z, sc), __fmul_rn(xv.w, sc));
        if (a.gamma) {
          const float4 g = gain4<E>(a.gamma, j);
          xv = make_float4(__fmul_rn(xv.x, g.x), __fmul_rn(xv.y, g.y), __fmul_rn(xv.z, g.z), __fmul_rn(xv.w, g.w));
        }
        if (a.factor != 1.0f)
          xv = make_float4(__fmul_rn(xv.x, a.factor), __fmul_rn(xv.y, a.factor), __fmul_rn(xv.z, a.factor),
                           __fmul_rn(xv.w, a.factor));
      } else if (PRO == PRO_SILU) {
        const float4 u = __ldg(reinterpret_cast<const float4*>(xr + a.up_off) + j);
        xv = make_float4(silu_of(xv.x, u.x), silu_of(xv.y, u.y), silu_of(xv.z, u.z), silu_of(xv.w, u.w));
      }
      xs4[(size_t)i * kc4 + p] = xv;
    }
    __syncthreads();
    if (active) {
      // This lane's packs in [c0, c1): j = v (mod stride), in order.
      uint32_t j = c0 + ((v + stride - (c0 % stride)) % stride);
      for (; j + (kInFlight - 1) * stride < c1; j += kInFlight * stride) {
        uint2 raw[kInFlight];
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) raw[u] = ld_stream2(wr + j + u * stride);
#pragma unroll
        for (int u = 0; u < kInFlight; ++u) {
          const float4 wv = E::widen4(raw[u]);
#pragma unroll
          for (int i = 0; i < M; ++i)
            if (i < (int)a.m) acc[i] = __fadd_rn(acc[i], pack_dot(xs4[(size_t)i * kc4 + (j + u * stride - c0)], wv));
        }
      }
      for (; j < c1; j += stride) {
        const float4 wv = E::widen4(ld_stream2(wr + j));
#pragma unroll
        for (int i = 0; i < M; ++i)
          if (i < (int)a.m) acc[i] = __fadd_rn(acc[i], pack_dot(xs4[(size_t)i * kc4 + (j - c0)], wv));
      }
    }
  }

#pragma unroll
  for (int i = 0; i < M; ++i) {
    const float t = warp_sum(acc[i]);
    if (lane == 0 && i < (int)a.m) part[warp][i] = t;
  }
  __syncthreads();
  // The splits in split order, then the epilogue.
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

template <class E, int M, int PRO, bool ADD>
static cudaError_t launch_chunk_m(const ChunkArgs& a, cudaStream_t st, bool pdl) {
  const uint32_t rows_per_block = 8u / a.split;
  const uint32_t blocks = (a.n + rows_per_block - 1) / rows_per_block;
  const size_t smem = (size_t)a.m * a.kc * sizeof(float);
  auto kern = gemv_chunk_w16_kernel<E, M, PRO, ADD>;
  cudaError_t e = fk_allow_smem(kern, smem);
  if (e != cudaSuccess) return e;
  return fk_launch_ex(kern, dim3(blocks), dim3(256), smem, st, pdl, a);
}

template <class E, int PRO, bool ADD>
static cudaError_t launch_chunk(const ChunkArgs& a, cudaStream_t st, bool pdl) {
  if (a.m <= 1) return launch_chunk_m<E, 1, PRO, ADD>(a, st, pdl);
  if (a.m <= 2) return launch_chunk_m<E, 2, PRO, ADD>(a, st, pdl);
  if (a.m <= 4) return launch_chunk_m<E, 4, PRO, ADD>(a, st, pdl);
  if (a.m <= 8) return launch_chunk_m<E, 8, PRO, ADD>(a, st, pdl);
  if (a.m <= 16) return launch_chunk_m<E, 16, PRO, ADD>(a, st, pdl);
  if (a.m <= 32) return launch_chunk_m<E, 32, PRO, ADD>(a, st, pdl);
  return cudaErrorInvalidValue;
}

// ---------------------------------------------------------------------------
// Elementwise.

// The embedding gather: row tokens[r] of a 16-bit table, widened, times the
// factor. Grid (width / 4 / 256, m).
template <class E>
__global__ void gather_w16_kernel(const uint16_t* __restrict__ table, uint32_t width,
                                  const uint32_t* __restrict__ tokens, float factor, float* __restrict__ y) {
  grid_wait();
  grid_launch_dependents();
  const uint32_t r = blockIdx.y;
  const uint32_t j = blockIdx.x * 256u + threadIdx.x;
  if (4 * j >= width) return;
  const uint2* src = reinterpret_cast<const uint2*>(table + (size_t)tokens[r] * width);
  float4 v = E::widen4(__ldg(src + j));
  if (factor != 1.0f)
    v = make_float4(__fmul_rn(v.x, factor), __fmul_rn(v.y, factor), __fmul_rn(v.z, factor), __fmul_rn(v.w, factor));
  reinterpret_cast<float4*>(y + (size_t)r * width)[j] = v;
}

// RMSNorm rows (prefill) with a 16-bit gain: the 256 spec lanes over packs
// t, t + 256, ...; y = x * scale * gamma (* factor). A block a row.
template <class E, int PK>
__global__ void __launch_bounds__(256) rmsnorm_rows_w16_kernel(const float* __restrict__ x,
                                                               const uint16_t* __restrict__ gamma,
                                                               float* __restrict__ y, uint32_t h, float eps,
                                                               float factor) {
  __shared__ float slots[8];
  const uint32_t row = blockIdx.x, t = threadIdx.x;
  const uint32_t packs = h >> 2;
  const float4* xr = reinterpret_cast<const float4*>(x + (size_t)row * h);
  float4 v[PK];
  float acc = 0.0f;
#pragma unroll
  for (int i = 0; i < PK; ++i) {
    const uint32_t j = t + 256u * i;
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
  const float scale = rsqrt_rounded(__fadd_rn(__fdiv_rn(tg_sum8(slots), (float)h), eps));
  float4* yr = reinterpret_cast<float4*>(y + (size_t)row * h);
#pragma unroll
  for (int i = 0; i < PK; ++i) {
    const uint32_t j = t + 256u * i;
    if (j < packs) {
      float4 o = make_float4(__fmul_rn(v[i].x, scale), __fmul_rn(v[i].y, scale), __fmul_rn(v[i].z, scale),
                             __fmul_rn(v[i].w, scale));
      const float4 g = gain4<E>(gamma, j);
      o = make_float4(__fmul_rn(o.x, g.x), __fmul_rn(o.y, g.y), __fmul_rn(o.z, g.z), __fmul_rn(o.w, g.w));
      if (factor != 1.0f)
        o = make_float4(__fmul_rn(o.x, factor), __fmul_rn(o.y, factor), __fmul_rn(o.z, factor),
                        __fmul_rn(o.w, factor));
      yr[j] = o;
    }
  }
}

// The TF32 halves of 16-bit weights for the prefill GEMM: the widened value
// is a TF32 value, so hi is it and lo is 0.
template <class E>
__global__ void split_tf32_w16_kernel(const uint16_t* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                      uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    hi[i] = E::widen(x[i]);
    lo[i] = 0.0f;
  }
}

// Seeded normals as the f32 fill draws them (SplitMix's finaliser of
// seed * golden + i, i from 1, test/cpu/Cases.hs:885-892; Box-Muller on
// consecutive words in binary64, rounded once to binary32), then rounded to
// the 16-bit type: the f32 fill's values, narrowed.
__device__ __forceinline__ uint64_t splitmix(uint64_t seed, uint64_t i) {
  uint64_t z = seed * 0x9E3779B97F4A7C15ULL + i;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

template <class E>
__global__ void fill_normal_w16_kernel(uint16_t* __restrict__ out, uint64_t n, uint64_t seed, double mu,
                                       double sigma) {
  const uint64_t pairs = (n + 1) / 2;
  for (uint64_t p = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; p < pairs;
       p += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t w1 = splitmix(seed, 2 * p + 1), w2 = splitmix(seed, 2 * p + 2);
    const double u1 = ((double)(w1 >> 11) + 1.0) * 0x1p-53;
    const double u2 = (double)(w2 >> 11) * 0x1p-53;
    const double rr = sqrt(-2.0 * log(u1));
    const double t = 6.283185307179586 * u2;
    out[2 * p] = E::narrow((float)(mu + sigma * (rr * cos(t))));
    if (2 * p + 1 < n) out[2 * p + 1] = E::narrow((float)(mu + sigma * (rr * sin(t))));
  }
}

static unsigned grid_for(uint64_t n) {
  const uint64_t b = (n + 255) / 256;
  return (unsigned)(b > 148ull * 64 ? 148ull * 64 : (b == 0 ? 1 : b));
}

template <class E>
static cudaError_t gemv(const FkGemv& g, const uint16_t* w, const uint16_t* gamma, int sms, cudaStream_t st) {
  if (g.k % 4 != 0 || g.split == 0 || !w) return cudaErrorInvalidValue;
  const bool peer = g.scatter || g.prologue == FK_PRO_REDUCE_RMSNORM;
  if (fk_gemv_streams(g)) {
    if (g.silu_pair && (g.n % 2 != 0 || g.r)) return cudaErrorInvalidValue;
    if (peer && (g.peers.world < 1 || g.xbuf >= FK_XBUFS || (size_t)g.m * (g.scatter ? g.n : g.k) > FK_XSLOT ||
                 (g.prologue == FK_PRO_REDUCE_RMSNORM && !g.xout)))
      return cudaErrorInvalidValue;
    StreamArgs a;
    a.w = w;
    a.x = g.x;
    a.gamma = gamma;
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
    a.peers = g.peers;
    a.xbuf = g.xbuf;
    a.xout = g.xout;
    a.err = g.err;
    a.prefetch = g.prefetch;
    const int epi = g.scatter ? SEPI_SCATTER : g.silu_pair ? SEPI_SILU_PAIR : (g.r ? SEPI_ADD : SEPI_NONE);
    switch (g.prologue * 4 + epi) {
      case FK_PRO_NONE * 4 + SEPI_NONE: return stream_m<E, SPRO_NONE, SEPI_NONE>(a, sms, st, g.pdl);
      case FK_PRO_NONE * 4 + SEPI_ADD: return stream_m<E, SPRO_NONE, SEPI_ADD>(a, sms, st, g.pdl);
      case FK_PRO_NONE * 4 + SEPI_SCATTER: return stream_m<E, SPRO_NONE, SEPI_SCATTER>(a, sms, st, g.pdl);
      case FK_PRO_RMSNORM * 4 + SEPI_NONE: return stream_m<E, SPRO_RMSNORM, SEPI_NONE>(a, sms, st, g.pdl);
      case FK_PRO_RMSNORM * 4 + SEPI_SILU_PAIR: return stream_m<E, SPRO_RMSNORM, SEPI_SILU_PAIR>(a, sms, st, g.pdl);
      case FK_PRO_SILU * 4 + SEPI_NONE: return stream_m<E, SPRO_SILU, SEPI_NONE>(a, sms, st, g.pdl);
      case FK_PRO_SILU * 4 + SEPI_ADD: return stream_m<E, SPRO_SILU, SEPI_ADD>(a, sms, st, g.pdl);
      case FK_PRO_REDUCE_RMSNORM * 4 + SEPI_NONE:
        return stream_m<E, SPRO_REDUCE_RMSNORM, SEPI_NONE>(a, sms, st, g.pdl);
      case FK_PRO_REDUCE_RMSNORM * 4 + SEPI_SILU_PAIR:
        return stream_m<E, SPRO_REDUCE_RMSNORM, SEPI_SILU_PAIR>(a, sms, st, g.pdl);
      default: return cudaErrorInvalidValue;
    }
  }
  // Batches up to 64 rows at split 1: the packed batched kernel
  // (k_w16_batch.cu), which has the row-pair form.
  if (!peer && fk_gemv_w16_batches(g, w)) return fk_launch_gemv_batch_w16(g, E::kElem, w, gamma, sms, st);
  // Past those: the chunked kernel, which has no row-pair or peer forms, 32
  // batch rows a launch.
  if (g.silu_pair || peer || !(g.split == 1 || g.split == 2 || g.split == 4 || g.split == 8))
    return cudaErrorInvalidValue;
  for (uint32_t i0 = 0; i0 < g.m; i0 += 32) {
    ChunkArgs a;
    a.m = g.m - i0 < 32 ? g.m - i0 : 32;
    a.w = w;
    a.x = g.x + (size_t)i0 * g.ldx;
    a.gamma = gamma;
    a.r = g.r ? g.r + (size_t)i0 * g.ldr : nullptr;
    a.y = g.y + (size_t)i0 * g.ldy;
    a.n = g.n;
    a.k = g.k;
    a.split = g.split;
    a.ldx = g.ldx;
    a.ldr = g.ldr;
    a.ldy = g.ldy;
    a.up_off = g.up_off;
    a.eps = g.eps;
    a.factor = g.factor;
    // As much of x as 64 KiB holds.
    uint32_t kc = (64u * 1024u / 4u) / a.m;
    kc &= ~3u;
    if (kc > g.k) kc = g.k;
    a.kc = kc;
    const bool add = a.r != nullptr;
    cudaError_t e;
    switch (g.prologue) {
      case FK_PRO_NONE: e = add ? launch_chunk<E, PRO_NONE, true>(a, st, g.pdl) : launch_chunk<E, PRO_NONE, false>(a, st, g.pdl); break;
      case FK_PRO_RMSNORM:
        e = add ? launch_chunk<E, PRO_RMSNORM, true>(a, st, g.pdl) : launch_chunk<E, PRO_RMSNORM, false>(a, st, g.pdl);
        break;
      case FK_PRO_SILU: e = add ? launch_chunk<E, PRO_SILU, true>(a, st, g.pdl) : launch_chunk<E, PRO_SILU, false>(a, st, g.pdl); break;
      default: return cudaErrorInvalidValue;
    }
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

template <class E>
static cudaError_t rmsnorm_rows(const float* x, const uint16_t* gamma, float* y, uint32_t rows, uint32_t h, float eps,
                                float factor, cudaStream_t s) {
  const uint32_t packs = h / 4;
  if (packs <= 256)
    rmsnorm_rows_w16_kernel<E, 1><<<rows, 256, 0, s>>>(x, gamma, y, h, eps, factor);
  else if (packs <= 1024)
    rmsnorm_rows_w16_kernel<E, 4><<<rows, 256, 0, s>>>(x, gamma, y, h, eps, factor);
  else if (packs <= 4096)
    rmsnorm_rows_w16_kernel<E, 16><<<rows, 256, 0, s>>>(x, gamma, y, h, eps, factor);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

template <class E>
static cudaError_t split_tf32(const uint16_t* x, float* hi, float* lo, uint64_t n, cudaStream_t s) {
  split_tf32_w16_kernel<E><<<grid_for(n), 256, 0, s>>>(x, hi, lo, n);
  return cudaGetLastError();
}

template <class E>
static cudaError_t fill_normal(uint16_t* out, uint64_t n, uint64_t seed, double mu, double sigma, cudaStream_t s) {
  fill_normal_w16_kernel<E><<<grid_for((n + 1) / 2), 256, 0, s>>>(out, n, seed, mu, sigma);
  return cudaGetLastError();
}

}  // namespace w16
}  // namespace fk

cudaError_t fk_launch_gemv_w16(const FkGemv& g, FkElem e, const uint16_t* w, const uint16_t* gamma, int sms,
                               cudaStream_t st) {
  if (g.n == 0 || g.m == 0) return cudaSuccess;
#define CALL(E) fk::w16::gemv<E>(g, w, gamma, sms, st)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}

cudaError_t fk_launch_gather_w16(FkElem e, const uint16_t* table, uint32_t width, const uint32_t* tokens, uint32_t m,
                                 float factor, float* y, bool pdl, cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (width % 4 != 0) return cudaErrorInvalidValue;
#define CALL(E)                                                                                                     \
  fk_launch_ex(fk::w16::gather_w16_kernel<E>, dim3((width / 4 + 255) / 256, m), dim3(256), 0, s, pdl, table, width, \
               tokens, factor, y)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}

cudaError_t fk_launch_rmsnorm_rows_w16(FkElem e, const float* x, const uint16_t* gamma, float* y, uint32_t rows,
                                       uint32_t h, float eps, float factor, cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  if (h % 4 != 0) return cudaErrorInvalidValue;
#define CALL(E) fk::w16::rmsnorm_rows<E>(x, gamma, y, rows, h, eps, factor, s)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}

cudaError_t fk_launch_split_tf32_w16(FkElem e, const uint16_t* x, float* hi, float* lo, uint64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
#define CALL(E) fk::w16::split_tf32<E>(x, hi, lo, n, s)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}

cudaError_t fk_launch_fill_normal_w16(FkElem e, uint16_t* out, uint64_t n, uint64_t seed, double mu, double sigma,
                                      cudaStream_t s) {
  if (n == 0) return cudaSuccess;
#define CALL(E) fk::w16::fill_normal<E>(out, n, seed, mu, sigma, s)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}
