// Weight-streaming GEMV for decode batches of up to 4 rows: persistent
// blocks, one prologue a block, rows handed out block-major.
//
// Arithmetic: the GEMV order contract (test/Test/FuryKernel/Gemv.hs:9-26) at
// pack width 4 and split s, as k_gemv.cu: a warp computes a row's splits one
// after another (split q: lane l over packs q*32 + l, q*32 + l + 32 s, ...;
// chains from 0, lanes summed pairwise, splits added in order), so the split
// changes the bits, never the parallel work.
//
// Work: 16 warps a block, blocks resident at once; unit u (a row, or a
// gate/up row pair) goes to block u mod G and, within it, warp (u / G) mod
// 16, so every block's share differs by at most one unit whatever the rows'
// count. A block stages x once, with its prologue applied (RMSNorm's scale by
// the spec order of 256 lanes over packs, then x * scale * gamma; or the
// SiLU-gate of a gate/up row), in shared memory; warps stream their rows'
// weights with 128-bit loads that skip L1, 8 in flight a lane.
//
// Epilogues: none; the residual add (the plan's Add on the tile); or the
// SiLU-gate of a row pair, for weights whose rows interleave gate and up
// (row 2i gate_i, row 2i+1 up_i): y_i = silu(gate_i) * up_i, computed on the
// pair's tile instead of in the next step's prologue (the same bits, once).
//
// Tensor parallelism (fk_peers.cuh): the row-parallel projections scatter
// their partial rows into every rank's exchange region (SEPI_SCATTER: a
// block owns a contiguous run of rows, stages them in shared memory, writes
// the run into this rank's slot of every region and counts itself in; the
// launch's last block publishes all rows to every rank with one
// system-scope fence); the
// next GEMV's prologue (SPRO_REDUCE_RMSNORM) waits for every rank's rows,
// forms the residual row x_new = r + (((P_0 + P_1) + P_2) + ...), ranks in
// order, so that every rank holds the same bits, stores it (block 0), and
// normalizes it as SPRO_RMSNORM does.
#include "fk_common.cuh"
#include "fk_kernels.h"
#include "fk_peers.cuh"

namespace fk {

struct StreamArgs {
  const float* w;
  const float* x;
  const float* gamma;
  const float* r;
  float* y;
  uint32_t n, k, m, split;
  uint32_t ldx, ldr, ldy;
  uint32_t up_off;
  float eps, factor;
  FkPeers peers;
  uint32_t xbuf;  // the exchange buffer scattered into, or reduced from
  float* xout;    // the reduced residual rows [m, k], stored by block 0
  int* err;
  size_t prefetch;  // bulk L2 prefetch budget of the launch (FkGemv::prefetch)
};

enum { SPRO_NONE = 0, SPRO_RMSNORM = 1, SPRO_SILU = 2, SPRO_REDUCE_RMSNORM = 3 };
enum { SEPI_NONE = 0, SEPI_ADD = 1, SEPI_SILU_PAIR = 2, SEPI_SCATTER = 3 };
constexpr int kStreamWarps = 16;
constexpr uint32_t kScatterRows = 128;  // a scattering block's most output rows

__device__ __forceinline__ float silu_of(float a, float b) {
  const float e = exp_rounded(-a);
  return __fmul_rn(__fdiv_rn(a, __fadd_rn(1.0f, e)), b);
}

// One row's totals for the staged rows of x, in the contract's order.
template <int M>
__device__ __forceinline__ void row_totals(const float4* __restrict__ wr, const float4* __restrict__ xs4,
                                           uint32_t packs, uint32_t m, uint32_t s, int lane, float (&total)[M]) {
  const uint32_t stride = 32u * s;
  for (uint32_t q = 0; q < s; ++q) {
    float acc[M];
#pragma unroll
    for (int i = 0; i < M; ++i) acc[i] = 0.0f;
    uint32_t j = q * 32u + (uint32_t)lane;
    for (; j + 7u * stride < packs; j += 8u * stride) {
      float4 wv[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) wv[u] = ld_stream(wr + j + u * stride);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
#pragma unroll
        for (int i = 0; i < M; ++i)
          if (i < (int)m) acc[i] = __fadd_rn(acc[i], pack_dot(xs4[(size_t)i * packs + j + u * stride], wv[u]));
      }
    }
    for (; j < packs; j += stride) {
      const float4 wv = ld_stream(wr + j);
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

template <int M, int PRO, int EPI>
__global__ void __launch_bounds__(512, 2) gemv_stream_kernel(StreamArgs a) {
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
    const size_t unit_bytes = (size_t)per_unit * a.k * 4;
    if (a.prefetch > 0) {
      const uint32_t p_lo = EPI == SEPI_SCATTER ? (uint32_t)((uint64_t)units * blockIdx.x / G) : 0u;
      const uint32_t p_hi = EPI == SEPI_SCATTER ? (uint32_t)((uint64_t)units * (blockIdx.x + 1) / G) : 0u;
      const size_t budget = a.prefetch / G;
      if (lane == 0 && (reinterpret_cast<uintptr_t>(a.w) & 15) == 0 && unit_bytes <= 0xFFFFFFF0u) {
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
  // Stage x: as given, the SiLU-gate of a gate/up row, or the residual plus
  // every rank's partial, in rank order.
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
    // RMSNorm of each staged row: threads 0..255 are the spec's 256 lanes,
    // each over packs t, t + 256, ... (src/FuryKernel/Reduce.hs:59-85); then
    // x * scale * gamma (* factor) in place.
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
        const float4 g = __ldg(reinterpret_cast<const float4*>(a.gamma) + j);
        v = make_float4(__fmul_rn(v.x, g.x), __fmul_rn(v.y, g.y), __fmul_rn(v.z, g.z), __fmul_rn(v.w, g.w));
      }
      if (a.factor != 1.0f)
        v = make_float4(__fmul_rn(v.x, a.factor), __fmul_rn(v.y, a.factor), __fmul_rn(v.z, a.factor),
                        __fmul_rn(v.w, a.factor));
      xs4[(size_t)i * packs + j] = v;
    }
    __syncthreads();
  }

  // Scattering blocks own contiguous output rows [s_lo, s_hi), staged in
  // shared memory and written to every rank in contiguous runs.
  __shared__ float outs[EPI == SEPI_SCATTER ? M : 1][EPI == SEPI_SCATTER ? kScatterRows : 1];
  const uint32_t s_lo = (uint32_t)((uint64_t)units * blockIdx.x / G);
  const uint32_t s_hi = (uint32_t)((uint64_t)units * (blockIdx.x + 1) / G);
  for (uint32_t slot = (uint32_t)warp;; slot += kStreamWarps) {
    const uint32_t u = EPI == SEPI_SCATTER ? s_lo + slot : blockIdx.x + slot * G;
    if (EPI == SEPI_SCATTER ? u >= s_hi : u >= units) break;
    float t0[M], t1[M];
    row_totals<M>(reinterpret_cast<const float4*>(a.w + (size_t)u * per_unit * a.k), xs4, packs, a.m, a.split,
                  lane, t0);
    if (EPI == SEPI_SILU_PAIR)
      row_totals<M>(reinterpret_cast<const float4*>(a.w + ((size_t)u * 2 + 1) * a.k), xs4, packs, a.m, a.split,
                    lane, t1);
    if (lane == 0) {
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
    }
  }
  if (EPI == SEPI_SCATTER) {
    // This rank's partial rows [s_lo, s_hi) into its slot of every rank's
    // region (contiguous runs), counted in (fk_peers.cuh).
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

template <int M, int PRO, int EPI>
static cudaError_t launch_stream(const StreamArgs& a, int sms, cudaStream_t st, bool pdl) {
  auto kern = gemv_stream_kernel<M, PRO, EPI>;
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

template <int PRO, int EPI>
static cudaError_t stream_m(const StreamArgs& a, int sms, cudaStream_t st, bool pdl) {
  if (a.m <= 1) return launch_stream<1, PRO, EPI>(a, sms, st, pdl);
  if (a.m <= 2) return launch_stream<2, PRO, EPI>(a, sms, st, pdl);
  return launch_stream<4, PRO, EPI>(a, sms, st, pdl);
}

}  // namespace fk

bool fk_gemv_streams(const FkGemv& g) {
  return g.m <= 4 && (size_t)g.m * g.k * sizeof(float) <= 200 * 1024;
}

cudaError_t fk_launch_gemv_stream(const FkGemv& g, int sms, cudaStream_t st) {
  if (g.n == 0 || g.m == 0) return cudaSuccess;
  if (!fk_gemv_streams(g) || g.k % 4 != 0 || g.split == 0 || (g.silu_pair && (g.n % 2 != 0 || g.r)))
    return cudaErrorInvalidValue;
  fk::StreamArgs a;
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
  a.peers = g.peers;
  a.xbuf = g.xbuf;
  a.xout = g.xout;
  a.err = g.err;
  a.prefetch = g.prefetch;
  using namespace fk;
  const bool peer = g.scatter || g.prologue == FK_PRO_REDUCE_RMSNORM;
  if (peer && (g.peers.world < 1 || g.xbuf >= FK_XBUFS || (size_t)g.m * (g.scatter ? g.n : g.k) > FK_XSLOT ||
               (g.prologue == FK_PRO_REDUCE_RMSNORM && !g.xout)))
    return cudaErrorInvalidValue;
  const int epi = g.scatter ? SEPI_SCATTER : g.silu_pair ? SEPI_SILU_PAIR : (g.r ? SEPI_ADD : SEPI_NONE);
  switch (g.prologue * 4 + epi) {
    case FK_PRO_NONE * 4 + SEPI_NONE: return stream_m<SPRO_NONE, SEPI_NONE>(a, sms, st, g.pdl);
    case FK_PRO_NONE * 4 + SEPI_ADD: return stream_m<SPRO_NONE, SEPI_ADD>(a, sms, st, g.pdl);
    case FK_PRO_NONE * 4 + SEPI_SCATTER: return stream_m<SPRO_NONE, SEPI_SCATTER>(a, sms, st, g.pdl);
    case FK_PRO_RMSNORM * 4 + SEPI_NONE: return stream_m<SPRO_RMSNORM, SEPI_NONE>(a, sms, st, g.pdl);
    case FK_PRO_RMSNORM * 4 + SEPI_SILU_PAIR: return stream_m<SPRO_RMSNORM, SEPI_SILU_PAIR>(a, sms, st, g.pdl);
    case FK_PRO_SILU * 4 + SEPI_NONE: return stream_m<SPRO_SILU, SEPI_NONE>(a, sms, st, g.pdl);
    case FK_PRO_SILU * 4 + SEPI_ADD: return stream_m<SPRO_SILU, SEPI_ADD>(a, sms, st, g.pdl);
    case FK_PRO_REDUCE_RMSNORM * 4 + SEPI_NONE: return stream_m<SPRO_REDUCE_RMSNORM, SEPI_NONE>(a, sms, st, g.pdl);
    case FK_PRO_REDUCE_RMSNORM * 4 + SEPI_SILU_PAIR:
      return stream_m<SPRO_REDUCE_RMSNORM, SEPI_SILU_PAIR>(a, sms, st, g.pdl);
    default: return cudaErrorInvalidValue;
  }
}
