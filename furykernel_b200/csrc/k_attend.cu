// Decode attention over Ring KV caches, as the plan runs it: the KV store
// step (RoPE of k recomputed, then k and v stored at each row's position),
// the attention anchor in splits of positions (RoPE of q recomputed; each
// split's maximum, sum and accumulator stored as partials, the Partials
// form of src/FuryKernel/Program/Plan.hs:174-181), and the combine step.
//
// Arithmetic, which the oracle's fko_attend_split / fko_attend_combine
// restate: a score is lane l's chain over packs l, l + 32, ... of q*k from
// 0, summed pairwise over the lanes, times the scale (Eval.hs:474-527: the
// scale on the dot product). A split's weights are exp(s - max) in binary64
// rounded once; warp w of 4 takes positions w, w + 4, ... of the split,
// adding e and e * v from 0, and the warps' sums are added in warp order.
// The combine rescales each split by exp(m - M), M the largest maximum, and
// adds the splits in order before dividing.
#include <algorithm>

#include "fk_common.cuh"
#include "fk_kernels.h"
#include "fk_prompt.cuh"

namespace fk {

constexpr int kAttWarps = 4;
constexpr int kHeadDim = 128;  // one float4 pack a lane
constexpr int kMaxChunk = 256;
constexpr uint32_t kMaxAttendRows = 16384;  // rows of one launch (prefill), first[] in shared memory

// RoPE of one head (halves pairing, Eval.hs:634-645): thread i < d/2 turns
// pair (i, i + d/2) by the position's table entry; pairs past `rotated` stay.
__device__ __forceinline__ void rope_pair(const float* __restrict__ src, float* __restrict__ dst, uint32_t i,
                                          uint32_t half, uint32_t rotated, const float* __restrict__ cos_row,
                                          const float* __restrict__ sin_row) {
  const float a = src[i], b = src[i + half];
  if (i < rotated) {
    const float c = __ldg(cos_row + i), s = __ldg(sin_row + i);
    dst[i] = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    dst[i + half] = __fadd_rn(__fmul_rn(b, c), __fmul_rn(a, s));
  } else {
    dst[i] = a;
    dst[i + half] = b;
  }
}

// The KV store step: grid (ceil(kv_heads / hb), m), hb * d / 2 threads, hb
// heads a block (4 at d = 128: a prompt's rows in blocks of 256 threads, not
// thousands of 64-thread blocks).
__global__ void kv_store_kernel(FkKvStore a) {
  grid_wait();
  grid_launch_dependents();
  const uint32_t half = a.d / 2;
  const uint32_t h = blockIdx.x * (blockDim.x / half) + threadIdx.x / half, r = blockIdx.y, i = threadIdx.x % half;
  if (h >= a.kv_heads) return;
  const uint32_t p = a.pos[r];
  const size_t at = (((size_t)a.slot[r] * a.kv_heads + h) * a.length + p % a.length) * a.d;
  const float* krow = a.qkv + (size_t)r * a.ldq + a.k_off + (size_t)h * a.d;
  const float* vrow = a.qkv + (size_t)r * a.ldq + a.v_off + (size_t)h * a.d;
  rope_pair(krow, a.kc + at, i, half, a.rotated, a.cos_t + (size_t)p * a.rotated, a.sin_t + (size_t)p * a.rotated);
  a.vc[at + i] = vrow[i];
  a.vc[at + i + half] = vrow[i + half];
}

// The attention anchor: persistent blocks of 4 warps over the step's items
// (row, head, split), item i at block i mod G. A warp takes positions w,
// w + 4, ... of its split, 8 at a time. The first 8 keys and values are
// requested before q is rotated, so that their latency hides the rotation's;
// a split's weights exp(s - max) are computed once a position, 32 positions
// across the lanes, and handed to the warp that adds them by shuffle.
//
// FUSED (attend_decode, a decode step's rows in distinct slots): the plan's
// KV store step and its attention in one launch. An item whose positions
// land on the ring slot of its row's position p rotates the row's new key
// (and reads its new value) itself and uses them there, so no item waits
// for the store; one item a (row, KV head) -- the last split, the group's
// first head -- writes them to the caches. The same arithmetic, so the
// same bits, as the two kernels. (Counting items in for an in-kernel
// combine cost more, a release-acquire atomic an item, than the combine
// launch it saved.)
template <bool FUSED>
__global__ void __launch_bounds__(128, 4) attend_kernel(FkAttendDecode f) {
  const FkAttend& a = f.a;
  __shared__ float qrot[kHeadDim];
  __shared__ float krot[FUSED ? kHeadDim : 1];
  __shared__ float vnew[FUSED ? kHeadDim : 1];
  __shared__ float scores[kMaxChunk];
  __shared__ float4 accw[kAttWarps][kHeadDim / 4];
  __shared__ float lw[kAttWarps];
  extern __shared__ uint32_t first[];  // [m + 1]: items before row r

  prefetch_l2_slice(a.pf, a.pf_bytes);
  // FUSED: the cached keys and values an item reads were stored by earlier
  // steps (this step's own key and value are substituted where the item
  // reads them, below), and the positions and slots were set before the
  // step's first launch: the block's first keys and values are requested
  // before it waits for the q/k/v GEMV, so that their latency hides under
  // that launch's end. The unfused kernel follows the KV store step and
  // waits first.
  bool waited = !FUSED;
  if (!FUSED) {
    grid_wait();
    grid_launch_dependents();
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    uint32_t acc = 0;
    for (uint32_t r = 0; r < a.m; ++r) {
      first[r] = acc;
      acc += a.heads * ((a.pos[r] + 1 + a.chunk - 1) / a.chunk);
    }
    first[a.m] = acc;
  }
  __syncthreads();
  const uint32_t items = first[a.m];
  const float4* kc4 = reinterpret_cast<const float4*>(a.kc);
  const float4* vc4 = reinterpret_cast<const float4*>(a.vc);
  constexpr int B = 8;  // positions in flight a warp
  constexpr uint32_t kStep = B * kAttWarps;
  const uint32_t group = a.heads / a.kv_heads;

  for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
    // The row whose items hold it: the last r with first[r] <= it.
    uint32_t lo = 0, hi = a.m - 1;
    while (lo < hi) {
      const uint32_t mid = (lo + hi + 1) / 2;
      if (first[mid] <= it) lo = mid; else hi = mid - 1;
    }
    const uint32_t r = lo;
    const uint32_t p = a.pos[r];
    const uint32_t splits = (p + 1 + a.chunk - 1) / a.chunk;
    const uint32_t local = it - first[r];
    const uint32_t h = local / splits, j = local - h * splits;
    const uint32_t t0 = j * a.chunk;
    const uint32_t t1 = min(p + 1, t0 + a.chunk);
    const uint32_t kvh = h / group;
    const size_t base = ((size_t)a.slot[r] * a.kv_heads + kvh) * a.length;
    const uint32_t pslot = p % a.length;  // where the row's new key and value land
    // Whether one of this item's positions lands on that ring slot (the
    // last split always; earlier ones only once the ring has wrapped).
    const uint32_t alias = t0 + (pslot + a.length - t0 % a.length) % a.length;
    const bool fresh = FUSED && alias < t1;

    // This warp's first keys and values: they depend on nothing below.
    float4 kv[B], vv[B];
#pragma unroll
    for (int u = 0; u < B; ++u) {
      const uint32_t tt = t0 + warp + u * kAttWarps;
      const size_t at = (base + tt % a.length) * (kHeadDim / 4) + lane;
      kv[u] = tt < t1 ? __ldcs(kc4 + at) : make_float4(0, 0, 0, 0);
      vv[u] = tt < t1 ? __ldcs(vc4 + at) : make_float4(0, 0, 0, 0);
    }
    if (!waited) {  // q, the new key and value: the q/k/v GEMV's outputs
      grid_wait();
      grid_launch_dependents();
      waited = true;
    }

    __syncthreads();  // the previous item's shared arrays are free
    const float* cos_row = a.cos_t + (size_t)p * a.rotated;
    const float* sin_row = a.sin_t + (size_t)p * a.rotated;
    if (threadIdx.x < kHeadDim / 2)
      rope_pair(a.qkv + (size_t)r * a.ldq + a.q_off + (size_t)h * kHeadDim, qrot, threadIdx.x, kHeadDim / 2,
                a.rotated, cos_row, sin_row);
    if (fresh) {
      const float* krow = a.qkv + (size_t)r * a.ldq + f.k_off + (size_t)kvh * kHeadDim;
      const float* vrow = a.qkv + (size_t)r * a.ldq + f.v_off + (size_t)kvh * kHeadDim;
      if (threadIdx.x >= kHeadDim / 2)
        rope_pair(krow, krot, threadIdx.x - kHeadDim / 2, kHeadDim / 2, a.rotated, cos_row, sin_row);
      vnew[threadIdx.x] = vrow[threadIdx.x];
    }
    __syncthreads();
    if (FUSED && j == splits - 1 && h % group == 0) {  // the KV store step, once a (row, KV head)
      const size_t at = (base + pslot) * kHeadDim + threadIdx.x;
      f.kc_w[at] = krot[threadIdx.x];
      f.vc_w[at] = vnew[threadIdx.x];
    }
    const float4 qv = reinterpret_cast<const float4*>(qrot)[lane];

    // Scores: warp w takes positions t0 + w + 4 u, eight at a time.
    for (uint32_t t = t0 + warp; t < t1; t += kStep) {
      if (t != t0 + warp) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          const uint32_t tt = t + u * kAttWarps;
          kv[u] = tt < t1 ? __ldcs(kc4 + (base + tt % a.length) * (kHeadDim / 4) + lane) : make_float4(0, 0, 0, 0);
        }
      }
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const uint32_t tt = t + u * kAttWarps;
        float4 kk = kv[u];
        if (fresh && tt < t1 && tt % a.length == pslot) kk = reinterpret_cast<const float4*>(krot)[lane];
        const float sc = __fmul_rn(warp_sum(__fadd_rn(0.0f, pack_dot(qv, kk))), a.scale);
        if (lane == 0 && tt < t1) scores[tt - t0] = sc;
      }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (uint32_t i = lane; i < t1 - t0; i += 32) mx = max_number(mx, scores[i]);
    mx = warp_max(mx);

    // Weighted sums: warp w over positions t0 + w, t0 + w + 4, ..., in order.
    float l = 0.0f;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (uint32_t t = t0 + warp; t < t1; t += kStep) {
      if (t != t0 + warp) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          const uint32_t tt = t + u * kAttWarps;
          vv[u] = tt < t1 ? __ldcs(vc4 + (base + tt % a.length) * (kHeadDim / 4) + lane) : make_float4(0, 0, 0, 0);
        }
      }
      // The 32 positions from t - warp: lane i's weight is position i's.
      const uint32_t g0 = t - (uint32_t)warp - t0;
      const float e_lane = g0 + lane < t1 - t0 ? exp_rounded(__fsub_rn(scores[g0 + lane], mx)) : 0.0f;
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const uint32_t tt = t + u * kAttWarps;
        const float e = __shfl_sync(0xffffffffu, e_lane, warp + u * kAttWarps);
        if (tt < t1) {
          float4 v4 = vv[u];
          if (fresh && tt % a.length == pslot) v4 = reinterpret_cast<const float4*>(vnew)[lane];
          l = __fadd_rn(l, e);
          acc.x = __fadd_rn(acc.x, __fmul_rn(e, v4.x));
          acc.y = __fadd_rn(acc.y, __fmul_rn(e, v4.y));
          acc.z = __fadd_rn(acc.z, __fmul_rn(e, v4.z));
          acc.w = __fadd_rn(acc.w, __fmul_rn(e, v4.w));
        }
      }
    }
    accw[warp][lane] = acc;
    if (lane == 0) lw[warp] = l;
    __syncthreads();
    const size_t at = ((size_t)r * a.heads + h) * a.max_splits + j;
    const float* accf = reinterpret_cast<const float*>(accw);
    const uint32_t i = threadIdx.x;  // one dimension a thread
    float o = accf[i];
#pragma unroll
    for (int w = 1; w < kAttWarps; ++w) o = __fadd_rn(o, accf[w * kHeadDim + i]);
    a.part_acc[at * kHeadDim + i] = o;
    if (threadIdx.x == 0) {
      float lt = lw[0];
#pragma unroll
      for (int w = 1; w < kAttWarps; ++w) lt = __fadd_rn(lt, lw[w]);
      a.part_l[at] = lt;
      a.part_m[at] = mx;
    }
  }
  if (!waited) grid_launch_dependents();  // a block without items
}

// Attention over a prompt's rows (prefill), all rows in one slot, each row
// over the positions <= its own (stored before, by kv_store_ring): the
// register-tiled body of fk_prompt.cuh over the Ring f32 caches.
struct RingPromptSrc {
  const float* kc;
  const float* vc;
  size_t base;  // position 0 of the rows' (slot, KV head), in elements / d
  __device__ __forceinline__ void bind(const FkAttend& a, uint32_t kvh) {
    kc = a.kc;
    vc = a.vc;
    base = ((size_t)a.slot[0] * a.kv_heads + kvh) * a.length;
  }
  __device__ __forceinline__ float4 k4(uint32_t t, uint32_t dd) const {
    return __ldg(reinterpret_cast<const float4*>(kc + (base + t) * kHeadDim + dd));
  }
  __device__ __forceinline__ float4 v4(uint32_t t, uint32_t dd) const {
    return __ldg(reinterpret_cast<const float4*>(vc + (base + t) * kHeadDim + dd));
  }
};

__global__ void __launch_bounds__(prompt::kThreads) attend_prompt_kernel(FkAttend a, float* __restrict__ out,
                                                                         uint32_t ldo, uint32_t max_pos) {
  prompt::attend_prompt_body(a, RingPromptSrc{}, out, ldo, max_pos);
}

// The combine step: grid (heads, m), d threads. The largest maximum M (the
// maximum is exact in any order) and each split's weight exp(m_j - M) are
// computed once a block, into shared memory; every thread then adds the
// splits in order for its dimension. A thread's first kCombineHeld
// accumulators are requested together with the maxima, so that a decode
// step's few splits cost one round trip to L2, not one for every 8.
constexpr int kCombineHeld = 32;
__global__ void combine_kernel(FkCombine a) {
  extern __shared__ float wsplit[];  // [max_splits] weights, then [max_splits] sums
  float* lsplit = wsplit + a.max_splits;
  grid_wait();
  grid_launch_dependents();
  const uint32_t h = blockIdx.x, r = blockIdx.y, i = threadIdx.x;
  const uint32_t splits = (a.pos[r] + 1 + a.chunk - 1) / a.chunk;
  const size_t at = ((size_t)r * a.heads + h) * a.max_splits;
  float held[kCombineHeld];
#pragma unroll
  for (int u = 0; u < kCombineHeld; ++u) held[u] = (uint32_t)u < splits ? a.part_acc[(at + u) * a.d + i] : 0.0f;
  if (threadIdx.x < 32) {  // one warp: M, then the weights and sums (lane j's first split kept in registers)
    const uint32_t j0 = threadIdx.x;
    const float m0 = j0 < splits ? a.part_m[at + j0] : -INFINITY;
    const float l0 = j0 < splits ? a.part_l[at + j0] : 0.0f;
    float top = j0 < splits ? max_number(-INFINITY, m0) : -INFINITY;
    for (uint32_t j = j0 + 32; j < splits; j += 32) top = max_number(top, a.part_m[at + j]);
    top = warp_max(top);
    if (j0 < splits) {
      wsplit[j0] = exp_rounded(__fsub_rn(m0, top));
      lsplit[j0] = l0;
    }
    for (uint32_t j = j0 + 32; j < splits; j += 32) {
      wsplit[j] = exp_rounded(__fsub_rn(a.part_m[at + j], top));
      lsplit[j] = a.part_l[at + j];
    }
  }
  __syncthreads();
  const float w0 = wsplit[0];
  float l = __fmul_rn(lsplit[0], w0);
  float o = __fmul_rn(held[0], w0);
  // The splits in order: the held ones, then the rest 8 loads at a time in flight.
#pragma unroll
  for (int u = 1; u < kCombineHeld; ++u) {
    if ((uint32_t)u < splits) {
      l = __fadd_rn(l, __fmul_rn(lsplit[u], wsplit[u]));
      o = __fadd_rn(o, __fmul_rn(held[u], wsplit[u]));
    }
  }
  uint32_t j = kCombineHeld;
  for (; j + 8 <= splits; j += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) v[u] = a.part_acc[(at + j + u) * a.d + i];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      l = __fadd_rn(l, __fmul_rn(lsplit[j + u], wsplit[j + u]));
      o = __fadd_rn(o, __fmul_rn(v[u], wsplit[j + u]));
    }
  }
  for (; j < splits; ++j) {
    const float w = wsplit[j];
    l = __fadd_rn(l, __fmul_rn(lsplit[j], w));
    o = __fadd_rn(o, __fmul_rn(a.part_acc[(at + j) * a.d + i], w));
  }
  a.out[(size_t)r * a.ldo + (size_t)h * a.d + i] = __fdiv_rn(o, l);
}

// A standalone RoPE of every head: grid (heads, m), d / 2 threads.
__global__ void rope_kernel(const float* __restrict__ x, uint32_t heads, uint32_t d, uint32_t rotated, uint32_t ldx,
                            const uint32_t* __restrict__ pos, const float* __restrict__ cos_t,
                            const float* __restrict__ sin_t, float* __restrict__ y, uint32_t ldy) {
  const uint32_t h = blockIdx.x, r = blockIdx.y, p = pos[r];
  rope_pair(x + (size_t)r * ldx + (size_t)h * d, y + (size_t)r * ldy + (size_t)h * d, threadIdx.x, d / 2, rotated,
            cos_t + (size_t)p * rotated, sin_t + (size_t)p * rotated);
}

}  // namespace fk

cudaError_t fk_launch_kv_store(const FkKvStore& a, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d % 2 != 0 || a.d > 2048 || a.kv_heads == 0) return cudaErrorInvalidValue;
  const uint32_t half = a.d / 2;
  const uint32_t hb = std::max(1u, std::min(a.kv_heads, 256u / half));  // heads a block
  return fk_launch_ex(fk::kv_store_kernel, dim3((a.kv_heads + hb - 1) / hb, a.m), dim3(hb * half), 0, s, a.pdl, a);
}

namespace {
template <bool FUSED>
cudaError_t launch_attend(const FkAttendDecode& f, cudaStream_t s) {
  const FkAttend& a = f.a;
  if (a.m == 0) return cudaSuccess;
  if (a.d != fk::kHeadDim || a.chunk == 0 || a.chunk > fk::kMaxChunk || a.kv_heads == 0 ||
      a.heads % a.kv_heads != 0 || a.m > fk::kMaxAttendRows || (uint64_t)a.m * a.heads * a.max_splits >= (1ull << 32))
    return cudaErrorInvalidValue;
  if (FUSED && (!f.kc_w || !f.vc_w)) return cudaErrorInvalidValue;
  // Blocks for the most items a step can have, as many as are resident at
  // once; each loops over its items.
  auto kern = fk::attend_kernel<FUSED>;
  int dev = 0, sms = 148, per_sm = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const size_t smem = ((size_t)a.m + 1) * sizeof(uint32_t);
  cudaError_t e = fk_allow_smem(kern, smem);
  if (e != cudaSuccess) return e;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, smem);
  if (e != cudaSuccess) return e;
  if (per_sm < 1) return cudaErrorInvalidConfiguration;
  const uint64_t most = (uint64_t)a.m * a.heads * a.max_splits;
  const uint64_t resident = (uint64_t)sms * per_sm;
  const uint32_t blocks = (uint32_t)(most < resident ? most : resident);
  return fk_launch_ex(kern, dim3(blocks), dim3(128), smem, s, a.pdl, f);
}
}  // namespace

cudaError_t fk_launch_attend(const FkAttend& a, cudaStream_t s) {
  FkAttendDecode f = {};
  f.a = a;
  return launch_attend<false>(f, s);
}

cudaError_t fk_launch_attend_decode(const FkAttendDecode& f, cudaStream_t s) { return launch_attend<true>(f, s); }

cudaError_t fk_launch_attend_prompt(const FkAttend& a, float* out, uint32_t ldo, uint32_t max_pos, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d != fk::kHeadDim || a.kv_heads == 0 || a.heads % a.kv_heads != 0 || max_pos >= a.length) return cudaErrorInvalidValue;
  if (ldo % 4 != 0 || ((uintptr_t)out | (uintptr_t)a.kc | (uintptr_t)a.vc) % 16 != 0)
    return cudaErrorInvalidValue;  // 16-byte loads and stores
  const size_t smem = fk::prompt::kSmemBytes;
  cudaError_t e = fk_allow_smem(fk::attend_prompt_kernel, smem);
  if (e != cudaSuccess) return e;
  const dim3 grid = fk::prompt::prompt_grid(a.m, a.heads);
  return fk_launch_ex(fk::attend_prompt_kernel, grid, dim3(fk::prompt::kThreads), smem, s, a.pdl, a, out, ldo,
                      max_pos);
}

cudaError_t fk_launch_combine(const FkCombine& a, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d > 1024 || a.d < 32 || a.max_splits == 0 || a.max_splits > 24576) return cudaErrorInvalidValue;
  const size_t smem = 2 * (size_t)a.max_splits * sizeof(float);
  cudaError_t e = fk_allow_smem(fk::combine_kernel, smem);
  if (e != cudaSuccess) return e;
  return fk_launch_ex(fk::combine_kernel, dim3(a.heads, a.m), dim3(a.d), smem, s, a.pdl, a);
}

cudaError_t fk_launch_rope(const float* x, uint32_t m, uint32_t heads, uint32_t d, uint32_t rotated, uint32_t ldx,
                           const uint32_t* pos, const float* cos_t, const float* sin_t, float* y, uint32_t ldy,
                           cudaStream_t s) {
  if (m == 0) return cudaSuccess;
  if (d % 2 != 0 || d > 2048) return cudaErrorInvalidValue;
  fk::rope_kernel<<<dim3(heads, m), d / 2, 0, s>>>(x, heads, d, rotated, ldx, pos, cos_t, sin_t, y, ldy);
  return cudaGetLastError();
}
