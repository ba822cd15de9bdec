// Decode attention over 16-bit Ring KV caches: bf16, the element type the
// reference's program builder gives a cache (`cache = cacheOf CacheBF16`,
// src/FuryKernel/Program/Build.hs:188-194), or f16 (CacheF16; CacheElem,
// Graph.hs:165-180): "a KV cache holds each stored element rounded to its
// element type" (src/FuryKernel/Program/Eval.hs:9). So the KV store rounds
// each rotated key and each value to the cache's type (narrowBF16 or
// narrowF16: nearest, ties to even, src/FuryKernel/Numerics.hs:41-48 and
// :100-130; the type a tag, fk_elem16.cuh), and the attention reads them widened,
// exactly; everything else -- RoPE, the scores' chains and lane sums, the
// weights exp(s - max) in binary64 rounded once, the warps' sums in warp
// order, the partials -- is the f32 kernels' arithmetic in the f32 kernels'
// order (k_attend.cu). The oracle's f32 attention over caches that hold the
// rounded values gives the bits; the caches' HBM bytes halve.
//
// The fused decode form (attend_decode) uses the row's new key and value
// rounded as the store rounds them, which is what the two-kernel form reads
// back from the cache: the same bits either way.
#include "fk_common.cuh"
#include "fk_elem16.cuh"
#include "fk_kernels.h"
#include "fk_prompt.cuh"

namespace fk {
namespace kv16 {

constexpr int kAttWarps = 4;
constexpr int kHeadDim = 128;  // one pack of 4 a lane
constexpr int kMaxChunk = 256;
constexpr uint32_t kMaxAttendRows = 16384;

// A value as the cache holds it.
template <class E>
__device__ __forceinline__ float rounded(float v) {
  return E::widen(E::narrow(v));
}

// RoPE of pair (i, i + half) of one head (halves pairing, Eval.hs:634-645),
// as k_attend.cu's rope_pair computes it; pairs past `rotated` stay.
__device__ __forceinline__ void rope2(const float* __restrict__ src, uint32_t i, uint32_t half, uint32_t rotated,
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

struct Store16 {
  FkKvStore a;  // a.kc / a.vc unused
  uint16_t* kc;
  uint16_t* vc;
};

// The KV store step: grid (ceil(kv_heads / hb), m), hb * d / 2 threads, hb
// heads a block (4 at d = 128).
template <class E>
__global__ void kv_store16_kernel(Store16 s) {
  const FkKvStore& a = s.a;
  grid_wait();
  grid_launch_dependents();
  const uint32_t half = a.d / 2;
  const uint32_t h = blockIdx.x * (blockDim.x / half) + threadIdx.x / half, r = blockIdx.y, i = threadIdx.x % half;
  if (h >= a.kv_heads) return;
  const uint32_t p = a.pos[r];
  const size_t at = (((size_t)a.slot[r] * a.kv_heads + h) * a.length + p % a.length) * a.d;
  const float* krow = a.qkv + (size_t)r * a.ldq + a.k_off + (size_t)h * a.d;
  const float* vrow = a.qkv + (size_t)r * a.ldq + a.v_off + (size_t)h * a.d;
  float lo, hi;
  rope2(krow, i, half, a.rotated, a.cos_t + (size_t)p * a.rotated, a.sin_t + (size_t)p * a.rotated, lo, hi);
  s.kc[at + i] = E::narrow(lo);
  s.kc[at + i + half] = E::narrow(hi);
  s.vc[at + i] = E::narrow(vrow[i]);
  s.vc[at + i + half] = E::narrow(vrow[i + half]);
}

struct Attend16 {
  FkAttend a;  // a.kc / a.vc unused
  const uint16_t* kc;
  const uint16_t* vc;
  uint32_t k_off, v_off;  // FUSED: the new key's and value's columns in a qkv row
  uint16_t* kc_w;
  uint16_t* vc_w;  // FUSED: the caches, written
};

// The attention anchor (k_attend.cu's attend_kernel over bf16 caches):
// persistent blocks of 4 warps over the step's items (row, head, split),
// item i at block i mod G; a warp takes positions w, w + 4, ... of its
// split, 8 at a time, their raw bits requested before q is rotated.
template <class E, bool FUSED>
__global__ void __launch_bounds__(128, 4) attend16_kernel(Attend16 f) {
  const FkAttend& a = f.a;
  __shared__ float qrot[kHeadDim];
  __shared__ float krot[FUSED ? kHeadDim : 1];
  __shared__ float vnew[FUSED ? kHeadDim : 1];
  __shared__ float scores[kMaxChunk];
  __shared__ float4 accw[kAttWarps][kHeadDim / 4];
  __shared__ float lw[kAttWarps];
  extern __shared__ uint32_t first[];  // [m + 1]: items before row r

  prefetch_l2_slice(a.pf, a.pf_bytes);
  // FUSED: the block's first keys and values are requested before it waits
  // for the q/k/v GEMV (k_attend.cu's attend_kernel says why that is sound).
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
  const uint2* kc2 = reinterpret_cast<const uint2*>(f.kc);
  const uint2* vc2 = reinterpret_cast<const uint2*>(f.vc);
  constexpr int B = 8;
  constexpr uint32_t kStep = B * kAttWarps;
  const uint32_t group = a.heads / a.kv_heads;
  const uint2 zero2 = make_uint2(0u, 0u);

  for (uint32_t it = blockIdx.x; it < items; it += gridDim.x) {
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
    const uint32_t pslot = p % a.length;
    const uint32_t alias = t0 + (pslot + a.length - t0 % a.length) % a.length;
    const bool fresh = FUSED && alias < t1;

    uint2 kv[B], vv[B];
#pragma unroll
    for (int u = 0; u < B; ++u) {
      const uint32_t tt = t0 + warp + u * kAttWarps;
      const size_t at = (base + tt % a.length) * (kHeadDim / 4) + lane;
      kv[u] = tt < t1 ? __ldcs(kc2 + at) : zero2;
      vv[u] = tt < t1 ? __ldcs(vc2 + at) : zero2;
    }
    if (!waited) {
      grid_wait();
      grid_launch_dependents();
      waited = true;
    }

    __syncthreads();  // the previous item's shared arrays are free
    const float* cos_row = a.cos_t + (size_t)p * a.rotated;
    const float* sin_row = a.sin_t + (size_t)p * a.rotated;
    if (threadIdx.x < kHeadDim / 2) {
      float q0, q1;
      rope2(a.qkv + (size_t)r * a.ldq + a.q_off + (size_t)h * kHeadDim, threadIdx.x, kHeadDim / 2, a.rotated,
            cos_row, sin_row, q0, q1);
      qrot[threadIdx.x] = q0;
      qrot[threadIdx.x + kHeadDim / 2] = q1;
    }
    if (fresh) {
      const float* krow = a.qkv + (size_t)r * a.ldq + f.k_off + (size_t)kvh * kHeadDim;
      const float* vrow = a.qkv + (size_t)r * a.ldq + f.v_off + (size_t)kvh * kHeadDim;
      if (threadIdx.x >= kHeadDim / 2) {
        const uint32_t i = threadIdx.x - kHeadDim / 2;
        float k0, k1;
        rope2(krow, i, kHeadDim / 2, a.rotated, cos_row, sin_row, k0, k1);
        krot[i] = rounded<E>(k0);
        krot[i + kHeadDim / 2] = rounded<E>(k1);
      }
      vnew[threadIdx.x] = rounded<E>(vrow[threadIdx.x]);
    }
    __syncthreads();
    if (FUSED && j == splits - 1 && h % group == 0) {  // the KV store step, once a (row, KV head)
      const size_t at = (base + pslot) * kHeadDim + threadIdx.x;
      f.kc_w[at] = E::narrow(krot[threadIdx.x]);
      f.vc_w[at] = E::narrow(vnew[threadIdx.x]);
    }
    const float4 qv = reinterpret_cast<const float4*>(qrot)[lane];

    for (uint32_t t = t0 + warp; t < t1; t += kStep) {
      if (t != t0 + warp) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          const uint32_t tt = t + u * kAttWarps;
          kv[u] = tt < t1 ? __ldcs(kc2 + (base + tt % a.length) * (kHeadDim / 4) + lane) : zero2;
        }
      }
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const uint32_t tt = t + u * kAttWarps;
        float4 kk = E::widen4(kv[u]);
        if (fresh && tt < t1 && tt % a.length == pslot) kk = reinterpret_cast<const float4*>(krot)[lane];
        const float sc = __fmul_rn(warp_sum(__fadd_rn(0.0f, pack_dot(qv, kk))), a.scale);
        if (lane == 0 && tt < t1) scores[tt - t0] = sc;
      }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (uint32_t i = lane; i < t1 - t0; i += 32) mx = max_number(mx, scores[i]);
    mx = warp_max(mx);

    float l = 0.0f;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    for (uint32_t t = t0 + warp; t < t1; t += kStep) {
      if (t != t0 + warp) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          const uint32_t tt = t + u * kAttWarps;
          vv[u] = tt < t1 ? __ldcs(vc2 + (base + tt % a.length) * (kHeadDim / 4) + lane) : zero2;
        }
      }
      const uint32_t g0 = t - (uint32_t)warp - t0;
      const float e_lane = g0 + lane < t1 - t0 ? exp_rounded(__fsub_rn(scores[g0 + lane], mx)) : 0.0f;
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const uint32_t tt = t + u * kAttWarps;
        const float e = __shfl_sync(0xffffffffu, e_lane, warp + u * kAttWarps);
        if (tt < t1) {
          float4 v4 = E::widen4(vv[u]);
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
    const uint32_t i = threadIdx.x;
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

// Attention over a prompt's rows in one slot (prefill): the register-tiled
// body of fk_prompt.cuh over 16-bit Ring caches, four elements a load,
// widened.
template <class E>
struct Ring16PromptSrc {
  const uint16_t* kc;
  const uint16_t* vc;
  size_t base;  // position 0 of the rows' (slot, KV head), in elements / d
  __device__ __forceinline__ void bind(const FkAttend& a, uint32_t kvh) {
    base = ((size_t)a.slot[0] * a.kv_heads + kvh) * a.length;
  }
  __device__ __forceinline__ float4 k4(uint32_t t, uint32_t dd) const {
    return E::widen4(__ldg(reinterpret_cast<const uint2*>(kc + (base + t) * kHeadDim + dd)));
  }
  __device__ __forceinline__ float4 v4(uint32_t t, uint32_t dd) const {
    return E::widen4(__ldg(reinterpret_cast<const uint2*>(vc + (base + t) * kHeadDim + dd)));
  }
};

template <class E>
__global__ void __launch_bounds__(prompt::kThreads) attend_prompt16_kernel(Attend16 f, float* __restrict__ out,
                                                                           uint32_t ldo, uint32_t max_pos) {
  prompt::attend_prompt_body(f.a, Ring16PromptSrc<E>{f.kc, f.vc, 0}, out, ldo, max_pos);
}

template <class E, bool FUSED>
cudaError_t launch_attend16(const Attend16& f, cudaStream_t s) {
  const FkAttend& a = f.a;
  if (a.m == 0) return cudaSuccess;
  if (a.d != kHeadDim || a.chunk == 0 || a.chunk > kMaxChunk || a.kv_heads == 0 || a.heads % a.kv_heads != 0 ||
      a.m > kMaxAttendRows || (uint64_t)a.m * a.heads * a.max_splits >= (1ull << 32) || !f.kc || !f.vc)
    return cudaErrorInvalidValue;
  if (FUSED && (!f.kc_w || !f.vc_w)) return cudaErrorInvalidValue;
  auto kern = attend16_kernel<E, FUSED>;
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

template <class E>
cudaError_t launch_prompt16(const Attend16& f, float* out, uint32_t ldo, uint32_t max_pos, cudaStream_t s) {
  const size_t smem = prompt::kSmemBytes;
  cudaError_t e = fk_allow_smem(attend_prompt16_kernel<E>, smem);
  if (e != cudaSuccess) return e;
  const dim3 grid = prompt::prompt_grid(f.a.m, f.a.heads);
  return fk_launch_ex(attend_prompt16_kernel<E>, grid, dim3(prompt::kThreads), smem, s, f.a.pdl, f, out, ldo,
                      max_pos);
}

}  // namespace kv16
}  // namespace fk

cudaError_t fk_launch_kv_store16(const FkKvStore& a, FkElem e, uint16_t* kc, uint16_t* vc, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d % 2 != 0 || a.d > 2048 || a.kv_heads == 0 || !kc || !vc) return cudaErrorInvalidValue;
  fk::kv16::Store16 st;
  st.a = a;
  st.kc = kc;
  st.vc = vc;
  const uint32_t half = a.d / 2;
  const uint32_t hb = half >= 256 ? 1u : (a.kv_heads < 256u / half ? a.kv_heads : 256u / half);  // heads a block
#define CALL(E) \
  fk_launch_ex(fk::kv16::kv_store16_kernel<E>, dim3((a.kv_heads + hb - 1) / hb, a.m), dim3(hb * half), 0, s, a.pdl, st)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}

cudaError_t fk_launch_attend16(const FkAttend& a, FkElem e, const uint16_t* kc, const uint16_t* vc, cudaStream_t s) {
  fk::kv16::Attend16 f = {};
  f.a = a;
  f.kc = kc;
  f.vc = vc;
#define CALL(E) fk::kv16::launch_attend16<E, false>(f, s)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}

cudaError_t fk_launch_attend_decode16(const FkAttend& a, FkElem e, uint32_t k_off, uint32_t v_off, uint16_t* kc,
                                      uint16_t* vc, cudaStream_t s) {
  fk::kv16::Attend16 f = {};
  f.a = a;
  f.kc = kc;
  f.vc = vc;
  f.k_off = k_off;
  f.v_off = v_off;
  f.kc_w = kc;
  f.vc_w = vc;
#define CALL(E) fk::kv16::launch_attend16<E, true>(f, s)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}

cudaError_t fk_launch_attend_prompt16(const FkAttend& a, FkElem e, const uint16_t* kc, const uint16_t* vc, float* out,
                                      uint32_t ldo, uint32_t max_pos, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d != fk::kv16::kHeadDim || a.kv_heads == 0 || a.heads % a.kv_heads != 0 || max_pos >= a.length || !kc ||
      !vc)
    return cudaErrorInvalidValue;
  if (ldo % 4 != 0 || ((uintptr_t)out % 16 | (uintptr_t)kc % 8 | (uintptr_t)vc % 8) != 0)
    return cudaErrorInvalidValue;  // 16-byte stores, 8-byte loads
  fk::kv16::Attend16 f = {};
  f.a = a;
  f.kc = kc;
  f.vc = vc;
#define CALL(E) fk::kv16::launch_prompt16<E>(f, out, ldo, max_pos, s)
  return FK_BY_ELEM16(e, CALL);
#undef CALL
}
