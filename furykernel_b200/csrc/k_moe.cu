// Routed experts (Graph.hs:306-340; their meaning, Eval.hs:291-320,
// 356-416, 648-659) for decode batches: the route (each row's top k of its
// router logits and their softmax weights), the routed GEMV (each row's k
// experts' rows times its input), the GELU-tanh gate of the experts'
// gate/up halves, and the rank-weighted combine with the residual.
//
// Arithmetic, which the oracle's fko_route_topk / fko_gemv_routed /
// fko_gated_gelu / fko_combine_ranks_add restate:
// - route: the top k, a logit taken where it is greater than the best so
//   far in index order (ties to the lower index; a NaN first untaken logit
//   is taken, a later NaN never); e_j = exp(x_j - best) (the difference in
//   binary32, exp in binary64 rounded once), their sum in rank order,
//   w_j = e_j / sum, times the expert scale when given;
// - routed GEMV: the GEMV order contract at pack 4 and split s for each
//   (row, rank) with its expert's rows;
// - GELU-tanh: (0.5 x)(1 + tanh(c (x + ((0.044715 x) x) x))), c = sqrt(2/pi)
//   in binary32, tanh in binary64 rounded once; the gate gelu(a) b;
// - combine: ((w_0 s_0 + w_1 s_1) + ...) in rank order, then r + that.
#include "fk_common.cuh"
#include "fk_elem16.cuh"
#include "fk_kernels.h"

namespace fk {
namespace moe {

constexpr uint32_t kMaxRanks = 8;
constexpr uint32_t kPairWindow = 1024;  // (row, rank) pairs a block lists at a time

// An expert's scale: f32, or a 16-bit type widened exactly.
template <class E>
__device__ __forceinline__ float scale_of(const void* scale, uint32_t i) {
  if constexpr (E::kElem == FK_F32)
    return static_cast<const float*>(scale)[i];
  else
    return E::widen(static_cast<const uint16_t*>(scale)[i]);
}

// The route: a warp a row; lane l holds logits l, l + 32, ... (n <= 1024).
// E: the expert scales' element type (scale null: no scales).
template <class E>
__global__ void __launch_bounds__(32) route_topk_kernel(const float* __restrict__ x, uint32_t n, uint32_t k,
                                                        uint32_t ldx, const void* __restrict__ scale,
                                                        uint32_t* __restrict__ ids, float* __restrict__ ws) {
  grid_wait();
  grid_launch_dependents();
  const uint32_t r = blockIdx.x, lane = threadIdx.x;
  const float* xr = x + (size_t)r * ldx;
  uint32_t taken = 0;  // bit t: logit lane + 32 t is taken
  uint32_t picked[kMaxRanks];
  for (uint32_t j = 0; j < k; ++j) {
    // This lane's best untaken non-NaN logit (ties to the lower index), and
    // its first untaken index.
    float bv = 0.0f;
    uint32_t bi = 0xffffffffu, first = 0xffffffffu;
    for (uint32_t t = 0, i = lane; i < n; ++t, i += 32) {
      if (taken & (1u << t)) continue;
      if (first == 0xffffffffu) first = i;
      const float v = xr[i];
      if (isnan(v)) continue;
      if (bi == 0xffffffffu || v > bv) {
        bv = v;
        bi = i;
      }
    }
    // The warp's: the greater logit, or the lower index among equals.
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const uint32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != 0xffffffffu && (bi == 0xffffffffu || ov > bv || (ov == bv && oi < bi))) {
        bv = ov;
        bi = oi;
      }
      first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
    }
    // A NaN at the first untaken index is taken (nothing is greater than it).
    const uint32_t pick = (first != 0xffffffffu && isnan(xr[first])) || bi == 0xffffffffu ? first : bi;
    picked[j] = pick;
    if (pick != 0xffffffffu && pick % 32 == lane) taken |= 1u << (pick / 32);
  }
  if (lane == 0) {
    float e[kMaxRanks];
    const float top = xr[picked[0]];
    float total = 0.0f;
    for (uint32_t j = 0; j < k; ++j) {
      e[j] = exp_rounded(__fsub_rn(xr[picked[j]], top));
      total = j == 0 ? e[j] : __fadd_rn(total, e[j]);
    }
    for (uint32_t j = 0; j < k; ++j) {
      float w = __fdiv_rn(e[j], total);
      if (scale) w = __fmul_rn(w, scale_of<E>(scale, picked[j]));
      ids[(size_t)r * k + j] = picked[j];
      ws[(size_t)r * k + j] = w;
    }
  }
}

struct RoutedArgs {
  const void* table;   // [entries, n, kk], f32, bf16 or f16
  const uint32_t* ids; // [m, k]
  const float* x;      // [m, ldx]: one segment of kk every rank takes, or k of them
  float* y;            // [m, ldy]: a segment of n a rank
  uint32_t entries, n, kk, m, k, split, ldx, ldy;
  bool per_rank;
};

constexpr int kPairsAPass = 4;

// A pack of four table weights: f32, or a 16-bit type widened exactly.
template <class E>
__device__ __forceinline__ float4 ld_pack(const typename E::Storage* row, uint32_t j) {
  if constexpr (E::kElem == FK_F32) {
    return ld_stream(reinterpret_cast<const float4*>(row) + j);
  } else {
    uint2 v;
    asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
        : "=r"(v.x), "=r"(v.y)
        : "l"(reinterpret_cast<const uint2*>(row) + j));
    return E::widen4(v);
  }
}

// The routed GEMV: a block a (expert, 8 output rows), a warp a row. The
// block walks the (row, rank) pairs in windows of kPairWindow, lists those
// whose route chose its expert and, for up to 4 pairs at a time, streams
// the expert's row once for them, each pair's dot in the GEMV contract's
// order (a pair's result does not depend on which pairs share its pass).
// Experts no row chose read no weights. E: the table's element type, f32,
// bf16 or f16 (widened where read).
template <class E>
__global__ void __launch_bounds__(256) gemv_routed_kernel(RoutedArgs a) {
  __shared__ uint32_t pairs[kPairWindow];
  __shared__ uint32_t npairs;
  const uint32_t e = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  grid_wait();
  grid_launch_dependents();
  const uint32_t all = a.m * a.k;
  const uint32_t o = blockIdx.y * 8u + (uint32_t)warp;
  const uint32_t packs = a.kk >> 2;
  const uint32_t stride = 32u * a.split;
  const typename E::Storage* wr =
      reinterpret_cast<const typename E::Storage*>(a.table) + ((size_t)e * a.n + (o < a.n ? o : 0)) * a.kk;
  for (uint32_t w0 = 0; w0 < all; w0 += kPairWindow) {
    const uint32_t w1 = min(all, w0 + kPairWindow);
    __syncthreads();  // every warp is done with the last window's list
    if (warp == 0) {  // the window's pairs that chose e, in order: a ballot per 32
      uint32_t c = 0;
      for (uint32_t base = w0; base < w1; base += 32u) {
        const uint32_t p = base + (uint32_t)lane;
        const bool hit = p < w1 && a.ids[p] == e;
        const uint32_t mask = __ballot_sync(0xffffffffu, hit);
        if (hit) pairs[c + __popc(mask & ((1u << lane) - 1u))] = p;
        c += __popc(mask);
      }
      if (lane == 0) npairs = c;
    }
    __syncthreads();
    const uint32_t P = npairs;
    if (P == 0 || o >= a.n) continue;
    for (uint32_t p0 = 0; p0 < P; p0 += kPairsAPass) {
      const uint32_t np = min((uint32_t)kPairsAPass, P - p0);
      const float4* xs[kPairsAPass];
#pragma unroll
      for (int q = 0; q < kPairsAPass; ++q) {
        const uint32_t pr = pairs[p0 + min((uint32_t)q, np - 1)];
        const uint32_t r = pr / a.k, j = pr % a.k;
        xs[q] = reinterpret_cast<const float4*>(a.x + (size_t)r * a.ldx + (a.per_rank ? (size_t)j * a.kk : 0));
      }
      float total[kPairsAPass];
      for (uint32_t sq = 0; sq < a.split; ++sq) {
        float acc[kPairsAPass];
#pragma unroll
        for (int q = 0; q < kPairsAPass; ++q) acc[q] = 0.0f;
        for (uint32_t jj = sq * 32u + (uint32_t)lane; jj < packs; jj += stride) {
          const float4 wv = ld_pack<E>(wr, jj);
#pragma unroll
          for (int q = 0; q < kPairsAPass; ++q)
            if ((uint32_t)q < np) acc[q] = __fadd_rn(acc[q], pack_dot(__ldg(xs[q] + jj), wv));
        }
#pragma unroll
        for (int q = 0; q < kPairsAPass; ++q) {
          const float part = warp_sum(acc[q]);
          total[q] = sq == 0 ? part : __fadd_rn(total[q], part);
        }
      }
      if (lane == 0) {
#pragma unroll
        for (int q = 0; q < kPairsAPass; ++q)
          if ((uint32_t)q < np) {
            const uint32_t pr = pairs[p0 + q];
            const uint32_t r = pr / a.k, j = pr % a.k;
            a.y[(size_t)r * a.ldy + (size_t)j * a.n + o] = total[q];
          }
      }
    }
  }
}

__device__ __forceinline__ float gelu_tanh(float x) {
  const float c = 0.79788456080286535588f;
  float p = __fmul_rn(0.044715f, x);
  p = __fmul_rn(p, x);
  p = __fmul_rn(p, x);
  const float u = __fmul_rn(c, __fadd_rn(x, p));
  const float t = (float)tanh((double)u);
  return __fmul_rn(__fmul_rn(0.5f, x), __fadd_rn(1.0f, t));
}

// GatedGelu: per segment of 2 f, gelu(a_i) b_i of its halves.
__global__ void gated_gelu_kernel(const float* __restrict__ x, uint64_t segments, uint32_t f, float* __restrict__ y) {
  grid_wait();
  grid_launch_dependents();
  const uint64_t total = segments * f;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint64_t s = i / f, c = i - s * f;
    y[i] = __fmul_rn(gelu_tanh(x[s * 2 * f + c]), x[s * 2 * f + f + c]);
  }
}

// CombineRanks then the residual: y = r + ((w_0 s_0 + w_1 s_1) + ...).
__global__ void combine_ranks_add_kernel(const float* __restrict__ r, const float* __restrict__ ws,
                                         const float* __restrict__ segs, uint32_t m, uint32_t k, uint32_t d,
                                         float* __restrict__ y) {
  grid_wait();
  grid_launch_dependents();
  const uint64_t total = (uint64_t)m * d;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < total; i += (uint64_t)gridDim.x * blockDim.x) {
    const uint32_t row = (uint32_t)(i / d), c = (uint32_t)(i - (uint64_t)row * d);
    const float* w = ws + (size_t)row * k;
    const float* s = segs + (size_t)row * k * d + c;
    float acc = __fmul_rn(w[0], s[0]);
    for (uint32_t j = 1; j < k; ++j) acc = __fadd_rn(acc, __fmul_rn(w[j], s[(size_t)j * d]));
    y[i] = __fadd_rn(r[i], acc);
  }
}

static unsigned grid_for(uint64_t n) {
  const uint64_t b = (n + 255) / 256;
  return (unsigned)(b > 148ull * 64 ? 148ull * 64 : (b == 0 ? 1 : b));
}

}  // namespace moe
}  // namespace fk

cudaError_t fk_launch_route_topk(const float* x, uint32_t m, uint32_t n, uint32_t k, uint32_t ldx,
                                 const void* scale, FkElem scale_elem, uint32_t* ids, float* ws, bool pdl,
                                 cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (n == 0 || n > 1024 || k == 0 || k > fk::moe::kMaxRanks || k > n || ldx < n) return cudaErrorInvalidValue;
  switch (scale_elem) {
    case FK_F32:
      return fk_launch_ex(fk::moe::route_topk_kernel<fk::F32>, dim3(m), dim3(32), 0, s, pdl, x, n, k, ldx, scale,
                          ids, ws);
    case FK_BF16:
      return fk_launch_ex(fk::moe::route_topk_kernel<fk::Bf16>, dim3(m), dim3(32), 0, s, pdl, x, n, k, ldx, scale,
                          ids, ws);
    case FK_F16:
      return fk_launch_ex(fk::moe::route_topk_kernel<fk::F16>, dim3(m), dim3(32), 0, s, pdl, x, n, k, ldx, scale,
                          ids, ws);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t fk_launch_gemv_routed(const void* table, FkElem el, uint32_t entries, uint32_t n, uint32_t kk,
                                  const uint32_t* ids, uint32_t m, uint32_t k, const float* x, uint32_t ldx,
                                  bool per_rank, uint32_t split, float* y, uint32_t ldy, bool pdl, cudaStream_t s) {
  if (m == 0 || n == 0) return cudaSuccess;
  if (kk % 4 != 0 || kk == 0 || k == 0 || entries == 0 || (uint64_t)m * k > 0xFFFFFFFFull || split == 0 ||
      ldx < (per_rank ? k * kk : kk) || ldy < k * n)
    return cudaErrorInvalidValue;
  fk::moe::RoutedArgs a;
  a.table = table;
  a.ids = ids;
  a.x = x;
  a.y = y;
  a.entries = entries;
  a.n = n;
  a.kk = kk;
  a.m = m;
  a.k = k;
  a.split = split;
  a.ldx = ldx;
  a.ldy = ldy;
  a.per_rank = per_rank;
  const dim3 grid(entries, (n + 7) / 8);
  switch (el) {
    case FK_F32: return fk_launch_ex(fk::moe::gemv_routed_kernel<fk::F32>, grid, dim3(256), 0, s, pdl, a);
    case FK_BF16: return fk_launch_ex(fk::moe::gemv_routed_kernel<fk::Bf16>, grid, dim3(256), 0, s, pdl, a);
    case FK_F16: return fk_launch_ex(fk::moe::gemv_routed_kernel<fk::F16>, grid, dim3(256), 0, s, pdl, a);
    default: return cudaErrorInvalidValue;
  }
}

cudaError_t fk_launch_gated_gelu(const float* x, uint64_t segments, uint32_t f, float* y, bool pdl, cudaStream_t s) {
  if (segments == 0 || f == 0) return cudaSuccess;
  return fk_launch_ex(fk::moe::gated_gelu_kernel, dim3(fk::moe::grid_for(segments * f)), dim3(256), 0, s, pdl, x,
                      segments, f, y);
}

cudaError_t fk_launch_combine_ranks_add(const float* r, const float* ws, const float* segs, uint32_t m, uint32_t k,
                                        uint32_t d, float* y, bool pdl, cudaStream_t s) {
  if (m == 0 || d == 0) return cudaSuccess;
  if (k == 0) return cudaErrorInvalidValue;
  return fk_launch_ex(fk::moe::combine_ranks_add_kernel, dim3(fk::moe::grid_for((uint64_t)m * d)), dim3(256), 0, s,
                      pdl, r, ws, segs, m, k, d, y);
}
