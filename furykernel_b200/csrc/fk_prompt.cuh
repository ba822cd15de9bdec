// Attention over a prompt's rows (prefill) on the CUDA cores, shared by the
// Ring f32, Ring 16-bit and paged caches: each kernel supplies where a
// position's key and value are (a source with k4 / v4, four elements of a
// position widened to f32) and runs attend_prompt_body.
//
// A block takes (64 query rows, head); 256 threads, thread (ty, tx) =
// (tid / 16, tid % 16) owning rows 4ty..4ty+3. Positions go 64 at a time
// through shared memory: the round's keys (rows padded to 132 floats, so
// that the 16-byte reads of consecutive keys fall in distinct banks) and
// values. The scores are a register tile, 4 rows x 4 positions a thread
// (positions tx, tx + 16, tx + 32, tx + 48 of the round), each a chain of
// fused multiply-adds over the head's dimensions, times the scale. The
// softmax is online (the running maximum of a row, its weights' sum and
// its output rescaled by exp(m_old - m_new) when the maximum grows): the
// weights exp(s - m) go to shared memory over the keys' buffer, and the
// weighted values accumulate into 4 rows x 8 dimensions a thread. The
// values' rows are stored permuted (position tx + 16j of the round at row
// 4tx + j) so that a thread's weights, four consecutive floats, meet them
// in order.
//
// The blocks' order balances the causal work across the SMs: a tile of the
// prompt's late rows sees up to 8 times the positions of an early one, and
// two blocks share an SM. Block L (in launch order) of the first wave (one
// block an SM) takes the L-th heaviest (tile, head); block S + j of the
// second takes the j-th lightest, which lands on the SM whose first block
// took the j-th heaviest, so each SM's two tiles add up to about the same
// number of positions (measured on config 5: the busiest SM's FMA pipe at
// 89% while the average SM's was at 43%, with the tiles launched heavy
// first in tile order).
//
// The orders, the fused products and expf differ from the decode kernels'
// and from the CPU target's, so prefill attention is held to the f64
// evaluator's bounds (src/FuryKernel/Program/Eval.hs:474-527 and
// attendBounds :900-919: each score's error, the weights' and the sum's
// rounding), like the prefill GEMMs, not to bits.
#pragma once

#include <cstdint>

#include "fk_common.cuh"
#include "fk_kernels.h"

namespace fk {
namespace prompt {

constexpr uint32_t kRows = 64;     // query rows a block
constexpr uint32_t kKeys = 64;     // positions a round
constexpr uint32_t kDim = 128;     // the head's dimensions (the only one the target plans)
constexpr uint32_t kThreads = 256;
constexpr uint32_t kKStride = 132;  // a key's row in shared memory, padded
constexpr size_t kSmemBytes = (size_t)(kRows * kDim + kKeys * kKStride + kKeys * kDim) * 4;
static_assert(kRows * kKeys <= kKeys * kKStride, "the weights overlay the keys' buffer");

// RoPE of pair (i, i + half) of one head (halves pairing, Eval.hs:634-645):
// the arithmetic of the decode kernels' rotation.
__device__ __forceinline__ void rope_q(const float* __restrict__ src, uint32_t i, uint32_t half, uint32_t rotated,
                                       const float* __restrict__ cos_row, const float* __restrict__ sin_row,
                                       float& lo, float& hi) {
  const float a = src[i], b = src[i + half];
  if (i < rotated) {
    const float c = __ldg(cos_row + i), s = __ldg(sin_row + i);
    lo = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    hi = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
  } else {
    lo = a;
    hi = b;
  }
}

__device__ __forceinline__ void fma4(float& acc, const float4 q, const float4 k) {
  acc = fmaf(q.x, k.x, acc);
  acc = fmaf(q.y, k.y, acc);
  acc = fmaf(q.z, k.z, acc);
  acc = fmaf(q.w, k.w, acc);
}

// The body, one block a (tile, head): a.m rows at positions a.pos, q in
// a.qkv's rows (column a.q_off + head * 128, rotated here), every row over
// the positions 0..its own that are also <= max_pos. src.bind(a, kv
// head), once the block's predecessor is done (it may have written the
// rows' slots); then src.k4(t, dd) and src.v4(t, dd): dimensions dd..dd+3
// of position t's key and value (t at most the tile's largest position).
template <class Src>
__device__ __forceinline__ void attend_prompt_body(const FkAttend& a, Src src, float* __restrict__ out, uint32_t ldo,
                                                   uint32_t max_pos) {
  extern __shared__ float4 prompt_smem4[];
  float* qs = reinterpret_cast<float*>(prompt_smem4);  // [64][128] rotated queries
  float* ks = qs + kRows * kDim;                       // [64][132] the round's keys; then the weights [64][64]
  float* vs = ks + kKeys * kKStride;                   // [64][128] the round's values, rows permuted
  float* ps = ks;
  const uint32_t tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const uint32_t lane = tid & 31, warp = tid >> 5;
  // The grid is (S, waves): S the first wave's blocks (prompt_grid).
  const uint32_t T = (a.m + kRows - 1) / kRows, H = a.heads, N = T * H, S = gridDim.x;
  const uint32_t L = blockIdx.x + S * blockIdx.y;
  if (L >= N) return;  // the last wave's padding
  const uint32_t o = L < S ? L : N - 1 - (L - S);  // the item's rank, heaviest first
  const uint32_t tile = T - 1 - o / H, h = o % H;
  const uint32_t r0 = tile * kRows;
  const uint32_t rows = min(kRows, a.m - r0);
  const uint32_t ncols = max_pos + 1;
  grid_wait();
  grid_launch_dependents();
  src.bind(a, h / (a.heads / a.kv_heads));

  for (uint32_t i = warp; i < kRows; i += kThreads / 32) {
    for (uint32_t c = lane; c < kDim / 2; c += 32) {
      float q0 = 0.0f, q1 = 0.0f;
      if (i < rows) {
        const uint32_t r = r0 + i, p = a.pos[r];
        rope_q(a.qkv + (size_t)r * a.ldq + a.q_off + (size_t)h * kDim, c, kDim / 2, a.rotated,
               a.cos_t + (size_t)p * a.rotated, a.sin_t + (size_t)p * a.rotated, q0, q1);
      }
      qs[i * kDim + c] = q0;
      qs[i * kDim + c + kDim / 2] = q1;
    }
  }
  // A row past the tile's end sees position 0 only, so that its (unstored)
  // arithmetic stays finite.
  uint32_t prow[4];
#pragma unroll
  for (int ri = 0; ri < 4; ++ri) {
    const uint32_t i = 4 * ty + ri;
    prow[ri] = i < rows ? a.pos[r0 + i] : 0u;
  }
  uint32_t tile_max = 0;
  for (uint32_t i = 0; i < rows; ++i) tile_max = max(tile_max, a.pos[r0 + i]);
  const uint32_t keys = min(tile_max + 1, ncols);  // positions past max_pos are the caller's error: not read

  float mrow[4], lpart[4], acc[4][8];
#pragma unroll
  for (int ri = 0; ri < 4; ++ri) {
    mrow[ri] = -INFINITY;
    lpart[ri] = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[ri][j] = 0.0f;
  }
  __syncthreads();

  for (uint32_t c0 = 0; c0 < keys; c0 += kKeys) {
    // The round's keys and values, 16 bytes a thread at a time.
    for (uint32_t e = tid; e < kKeys * (kDim / 4); e += kThreads) {
      const uint32_t kk = e / (kDim / 4), dd = 4 * (e % (kDim / 4));
      const uint32_t t = c0 + kk;
      const bool live = t < keys;
      const float4 kv = live ? src.k4(t, dd) : make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 vv = live ? src.v4(t, dd) : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(ks + kk * kKStride + dd) = kv;
      *reinterpret_cast<float4*>(vs + (4 * (kk % 16) + kk / 16) * kDim + dd) = vv;
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int ri = 0; ri < 4; ++ri)
#pragma unroll
      for (int kj = 0; kj < 4; ++kj) s[ri][kj] = 0.0f;
#pragma unroll 4
    for (uint32_t dd = 0; dd < kDim; dd += 4) {
      float4 q[4], k[4];
#pragma unroll
      for (int ri = 0; ri < 4; ++ri) q[ri] = *reinterpret_cast<const float4*>(qs + (4 * ty + ri) * kDim + dd);
#pragma unroll
      for (int kj = 0; kj < 4; ++kj) k[kj] = *reinterpret_cast<const float4*>(ks + (tx + 16 * kj) * kKStride + dd);
#pragma unroll
      for (int ri = 0; ri < 4; ++ri)
#pragma unroll
        for (int kj = 0; kj < 4; ++kj) fma4(s[ri][kj], q[ri], k[kj]);
    }
    __syncthreads();  // every read of the keys done: the weights overwrite them

#pragma unroll
    for (int ri = 0; ri < 4; ++ri) {
      float cm = -INFINITY;
#pragma unroll
      for (int kj = 0; kj < 4; ++kj) {
        const uint32_t t = c0 + tx + 16 * kj;
        s[ri][kj] = t <= prow[ri] && t < ncols ? __fmul_rn(s[ri][kj], a.scale) : -INFINITY;
        cm = fmaxf(cm, s[ri][kj]);
      }
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
      // Position 0 is every row's from the first round on, so m_new is finite.
      const float mnew = fmaxf(mrow[ri], cm);
      const float alpha = expf(mrow[ri] - mnew);
      mrow[ri] = mnew;
      float p[4];
#pragma unroll
      for (int kj = 0; kj < 4; ++kj) p[kj] = s[ri][kj] == -INFINITY ? 0.0f : expf(s[ri][kj] - mnew);
      lpart[ri] = fmaf(lpart[ri], alpha, (p[0] + p[1]) + (p[2] + p[3]));
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[ri][j] *= alpha;
      *reinterpret_cast<float4*>(ps + (4 * ty + ri) * kKeys + 4 * tx) = make_float4(p[0], p[1], p[2], p[3]);
    }
    __syncthreads();

#pragma unroll 2
    for (uint32_t j = 0; j < kKeys; j += 4) {
      float4 pr[4];
#pragma unroll
      for (int ri = 0; ri < 4; ++ri) pr[ri] = *reinterpret_cast<const float4*>(ps + (4 * ty + ri) * kKeys + j);
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float4 va = *reinterpret_cast<const float4*>(vs + (j + jj) * kDim + 4 * tx);
        const float4 vb = *reinterpret_cast<const float4*>(vs + (j + jj) * kDim + kDim / 2 + 4 * tx);
#pragma unroll
        for (int ri = 0; ri < 4; ++ri) {
          const float w = jj == 0 ? pr[ri].x : jj == 1 ? pr[ri].y : jj == 2 ? pr[ri].z : pr[ri].w;
          acc[ri][0] = fmaf(w, va.x, acc[ri][0]);
          acc[ri][1] = fmaf(w, va.y, acc[ri][1]);
          acc[ri][2] = fmaf(w, va.z, acc[ri][2]);
          acc[ri][3] = fmaf(w, va.w, acc[ri][3]);
          acc[ri][4] = fmaf(w, vb.x, acc[ri][4]);
          acc[ri][5] = fmaf(w, vb.y, acc[ri][5]);
          acc[ri][6] = fmaf(w, vb.z, acc[ri][6]);
          acc[ri][7] = fmaf(w, vb.w, acc[ri][7]);
        }
      }
    }
    __syncthreads();  // before the next round overwrites keys, weights and values
  }

#pragma unroll
  for (int ri = 0; ri < 4; ++ri) {
    float l = lpart[ri];
#pragma unroll
    for (int o = 8; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    const uint32_t i = 4 * ty + ri;
    if (i < rows) {
      float* o = out + (size_t)(r0 + i) * ldo + (size_t)h * kDim;
      *reinterpret_cast<float4*>(o + 4 * tx) =
          make_float4(acc[ri][0] / l, acc[ri][1] / l, acc[ri][2] / l, acc[ri][3] / l);
      *reinterpret_cast<float4*>(o + kDim / 2 + 4 * tx) =
          make_float4(acc[ri][4] / l, acc[ri][5] / l, acc[ri][6] / l, acc[ri][7] / l);
    }
  }
}

// The launch grid for m rows and `heads` heads: (S, waves), S the first
// wave (the SM count, or fewer blocks), the blocks past m's items idle.
inline dim3 prompt_grid(uint32_t m, uint32_t heads) {
  static int sms[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  if (!sms[dev]) {
    int n = 148;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n < 1) n = 148;
    sms[dev] = n;
  }
  const uint32_t items = (m + kRows - 1) / kRows * heads;
  const uint32_t S = items < (uint32_t)sms[dev] ? items : (uint32_t)sms[dev];
  return dim3(S, (items + S - 1) / S);
}

}  // namespace prompt
}  // namespace fk
