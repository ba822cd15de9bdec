// Attention over paged KV caches (Paged blocks blockSize kvHeads headDim,
// src/FuryKernel/Program/Graph.hs:144-152): a cache is `blocks` blocks of
// `block_size` positions, each an array of its own wherever the engine
// allocated it, reached through a table of the blocks' addresses (the
// launch's k_cache and v_cache tables: u64 entries, IR.hs:400-429); each
// row lists its sequence's blocks by index in a block table of `table_len`
// u32 entries. Position p, KV head h of a row is at element
// (h * block_size + p mod block_size) * d of block table[p / block_size]
// (cacheIndex, src/FuryKernel/Program/Eval.hs:592-602).
//
// Arithmetic: the ring kernels' (k_attend.cu), position for position -- the
// KV store rotates each key and stores it and the value at the row's
// position; a score is a chain over the lanes' packs summed pairwise, times
// the scale; a split's weights exp(s - max) in binary64 rounded once, the
// warps' sums in warp order; the prompt attention's two passes. Only where
// a position's key and value live differs, so the oracle's ring attention
// over the blocks gathered in table order gives the bits. Elements are f32,
// bf16 or f16 (stores rounded to the cache's type, nearest even, reads
// widened: Eval.hs:9; the type a tag, fk_elem16.cuh).
//
// A block-table entry at or past `blocks` is not read or written: its keys
// and values read as 0 and its stores are dropped (the engine checks the
// tables it uploads; this keeps a bad entry from reaching past the address
// tables). The addresses themselves are the caller's: each must point at a
// block of kv_heads * block_size * d elements of the cache's type.
#include "fk_common.cuh"
#include "fk_elem16.cuh"
#include "fk_kernels.h"
#include "fk_prompt.cuh"

namespace fk {
namespace paged {

constexpr int kAttWarps = 4;
constexpr int kHeadDim = 128;
constexpr int kMaxChunk = 256;
constexpr uint32_t kMaxAttendRows = 16384;

// The element forms of a cache of type E: a pack of four elements widened
// to f32, an element widened, an element stored (16-bit types: rounded to
// nearest even).
template <class E>
using St = typename E::Storage;
template <class E>
__device__ __forceinline__ float4 ld_pack(const St<E>* p) {
  if constexpr (E::kElem == FK_F32)
    return __ldcs(reinterpret_cast<const float4*>(p));
  else
    return E::widen4(__ldcs(reinterpret_cast<const uint2*>(p)));
}
template <class E>
__device__ __forceinline__ float ld_elem(const St<E>* p) {
  if constexpr (E::kElem == FK_F32)
    return *p;
  else
    return E::widen(*p);
}
template <class E>
__device__ __forceinline__ void st_elem(St<E>* p, float v) {
  if constexpr (E::kElem == FK_F32)
    *p = v;
  else
    *p = E::narrow(v);
}

// RoPE of pair (i, i + half) of one head (halves pairing, Eval.hs:634-645),
// k_attend.cu's rope_pair arithmetic.
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

struct Pool {
  const uint32_t* table;  // [m, table_len] each row's blocks, by index
  const uint64_t* kblk;   // [blocks] each block's address: keys
  const uint64_t* vblk;   // and values
  uint32_t block_size, table_len, blocks;
};

// Where (row r, position t, KV head h, element 0) is: the block's index in
// the high word, the element within the block in the low word; UINT64_MAX
// where the row's table has no block there.
__device__ __forceinline__ uint64_t at_of(const Pool& P, uint32_t r, uint32_t t, uint32_t h, uint32_t kv_heads,
                                          uint32_t d) {
  const uint32_t slot = t / P.block_size;
  if (slot >= P.table_len) return ~0ull;
  const uint32_t block = __ldg(P.table + (size_t)r * P.table_len + slot);
  if (block >= P.blocks) return ~0ull;
  return ((uint64_t)block << 32) | ((h * P.block_size + t % P.block_size) * d);
}

// The element `at` (from at_of) of a cache through its blocks' addresses.
template <class E>
__device__ __forceinline__ St<E>* elem_at(const uint64_t* blk, uint64_t at) {
  return reinterpret_cast<St<E>*>(__ldg(reinterpret_cast<const unsigned long long*>(blk) + (at >> 32))) +
         (uint32_t)at;
}

template <class E>
struct StoreArgs {
  FkKvStore a;  // a.slot, a.kc, a.vc, a.length unused
  Pool P;
};

// The KV store step: grid (ceil(kv_heads / hb), m), hb * d / 2 threads, hb
// heads a block (4 at d = 128).
template <class E>
__global__ void kv_store_paged_kernel(StoreArgs<E> s) {
  const FkKvStore& a = s.a;
  grid_wait();
  grid_launch_dependents();
  const uint32_t half = a.d / 2;
  const uint32_t h = blockIdx.x * (blockDim.x / half) + threadIdx.x / half, r = blockIdx.y, i = threadIdx.x % half;
  if (h >= a.kv_heads) return;
  const uint32_t p = a.pos[r];
  const uint64_t at = at_of(s.P, r, p, h, a.kv_heads, a.d);
  if (at == ~0ull) return;
  const float* krow = a.qkv + (size_t)r * a.ldq + a.k_off + (size_t)h * a.d;
  const float* vrow = a.qkv + (size_t)r * a.ldq + a.v_off + (size_t)h * a.d;
  float lo, hi;
  rope2(krow, i, half, a.rotated, a.cos_t + (size_t)p * a.rotated, a.sin_t + (size_t)p * a.rotated, lo, hi);
  St<E>* kp = elem_at<E>(s.P.kblk, at);
  St<E>* vp = elem_at<E>(s.P.vblk, at);
  st_elem<E>(kp + i, lo);
  st_elem<E>(kp + i + half, hi);
  st_elem<E>(vp + i, vrow[i]);
  st_elem<E>(vp + i + half, vrow[i + half]);
}

template <class E>
struct AttendArgs {
  FkAttend a;  // a.slot, a.kc, a.vc, a.length unused
  Pool P;
  uint32_t k_off, v_off;  // FUSED: the new key's and value's columns in a qkv row
};

// A value as a cache of type E holds it.
template <class E>
__device__ __forceinline__ float as_held(float v) {
  if constexpr (E::kElem == FK_F32)
    return v;
  else
    return E::widen(E::narrow(v));
}

// The attention anchor: persistent blocks of 4 warps over the step's items
// (row, head, split), item i at block i mod G; warp w takes positions w,
// w + 4, ... of its split, 8 at a time (the ring kernel's order).
//
// FUSED (attend_decode_paged): the KV store folded in, as the ring's
// attend_decode does it. The split that holds the row's position p uses
// the new key (rotated) and value as the cache holds them, in place of what
// it loads at p, and one block a (row, KV head) stores them. The same bits
// as the store then the attention, when no row reads an element another
// row stores in the same step: every block-table entry distinct (the
// engine checks its tables for that).
template <class E, bool FUSED>
__global__ void __launch_bounds__(128, 4) attend_paged_kernel(AttendArgs<E> f) {
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
  constexpr int B = 8;
  constexpr uint32_t kStep = B * kAttWarps;
  const uint32_t group = a.heads / a.kv_heads;
  const float4 zero4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);

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
    const bool fresh = FUSED && j == splits - 1;  // the split that holds p

    float4 kv[B], vv[B];
#pragma unroll
    for (int u = 0; u < B; ++u) {
      const uint32_t tt = t0 + warp + u * kAttWarps;
      const uint64_t at = tt < t1 ? at_of(f.P, r, tt, kvh, a.kv_heads, kHeadDim) : ~0ull;
      kv[u] = at != ~0ull ? ld_pack<E>(elem_at<E>(f.P.kblk, at) + 4 * lane) : zero4;
      vv[u] = at != ~0ull ? ld_pack<E>(elem_at<E>(f.P.vblk, at) + 4 * lane) : zero4;
    }
    if (!waited) {
      grid_wait();
      grid_launch_dependents();
      waited = true;
    }

    __syncthreads();  // the previous item's shared arrays are free
    if (threadIdx.x < kHeadDim / 2) {
      float q0, q1;
      rope2(a.qkv + (size_t)r * a.ldq + a.q_off + (size_t)h * kHeadDim, threadIdx.x, kHeadDim / 2, a.rotated,
            a.cos_t + (size_t)p * a.rotated, a.sin_t + (size_t)p * a.rotated, q0, q1);
      qrot[threadIdx.x] = q0;
      qrot[threadIdx.x + kHeadDim / 2] = q1;
    }
    if (fresh) {
      const float* krow = a.qkv + (size_t)r * a.ldq + f.k_off + (size_t)kvh * kHeadDim;
      const float* vrow = a.qkv + (size_t)r * a.ldq + f.v_off + (size_t)kvh * kHeadDim;
      if (threadIdx.x >= kHeadDim / 2) {
        const uint32_t i = threadIdx.x - kHeadDim / 2;
        float k0, k1;
        rope2(krow, i, kHeadDim / 2, a.rotated, a.cos_t + (size_t)p * a.rotated, a.sin_t + (size_t)p * a.rotated,
              k0, k1);
        krot[i] = as_held<E>(k0);
        krot[i + kHeadDim / 2] = as_held<E>(k1);
      }
      vnew[threadIdx.x] = as_held<E>(vrow[threadIdx.x]);
    }
    __syncthreads();
    if (fresh && h % group == 0) {  // the KV store, once a (row, KV head)
      const uint64_t at = at_of(f.P, r, p, kvh, a.kv_heads, kHeadDim);
      if (at != ~0ull) {
        st_elem<E>(elem_at<E>(f.P.kblk, at) + threadIdx.x, krot[threadIdx.x]);
        st_elem<E>(elem_at<E>(f.P.vblk, at) + threadIdx.x, vnew[threadIdx.x]);
      }
    }
    const float4 qv = reinterpret_cast<const float4*>(qrot)[lane];

    for (uint32_t t = t0 + warp; t < t1; t += kStep) {
      if (t != t0 + warp) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          const uint32_t tt = t + u * kAttWarps;
          const uint64_t at = tt < t1 ? at_of(f.P, r, tt, kvh, a.kv_heads, kHeadDim) : ~0ull;
          kv[u] = at != ~0ull ? ld_pack<E>(elem_at<E>(f.P.kblk, at) + 4 * lane) : zero4;
        }
      }
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const uint32_t tt = t + u * kAttWarps;
        float4 kk = kv[u];
        if (fresh && tt == p) kk = reinterpret_cast<const float4*>(krot)[lane];
        const float sc = __fmul_rn(warp_sum(__fadd_rn(0.0f, pack_dot(qv, kk))), a.scale);
        if (lane == 0 && tt < t1) scores[tt - t0] = sc;
      }
    }
    __syncthreads();
    float mx = -INFINITY;
    for (uint32_t i = lane; i < t1 - t0; i += 32) mx = max_number(mx, scores[i]);
    mx = warp_max(mx);

    float l = 0.0f;
    float4 acc = zero4;
    for (uint32_t t = t0 + warp; t < t1; t += kStep) {
      if (t != t0 + warp) {
#pragma unroll
        for (int u = 0; u < B; ++u) {
          const uint32_t tt = t + u * kAttWarps;
          const uint64_t at = tt < t1 ? at_of(f.P, r, tt, kvh, a.kv_heads, kHeadDim) : ~0ull;
          vv[u] = at != ~0ull ? ld_pack<E>(elem_at<E>(f.P.vblk, at) + 4 * lane) : zero4;
        }
      }
      const uint32_t g0 = t - (uint32_t)warp - t0;
      const float e_lane = g0 + lane < t1 - t0 ? exp_rounded(__fsub_rn(scores[g0 + lane], mx)) : 0.0f;
#pragma unroll
      for (int u = 0; u < B; ++u) {
        const uint32_t tt = t + u * kAttWarps;
        const float e = __shfl_sync(0xffffffffu, e_lane, warp + u * kAttWarps);
        if (tt < t1) {
          const float4 v4 = fresh && tt == p ? reinterpret_cast<const float4*>(vnew)[lane] : vv[u];
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

// Attention over a prompt's rows of one sequence (prefill): the
// register-tiled body of fk_prompt.cuh, positions through row 0's block
// table (the prompt's rows share their sequence's table). A position whose
// block is not in the table reads as zeros.
template <class E>
struct PagedPromptSrc {
  Pool P;
  uint32_t kvh, kv_heads;
  __device__ __forceinline__ void bind(const FkAttend& a, uint32_t h) {
    kvh = h;
    kv_heads = a.kv_heads;
  }
  __device__ __forceinline__ float4 load(const uint64_t* blk, uint32_t t, uint32_t dd) const {
    const uint64_t at = at_of(P, 0, t, kvh, kv_heads, kHeadDim);
    if (at == ~0ull) return make_float4(0.f, 0.f, 0.f, 0.f);
    const St<E>* p = elem_at<E>(blk, at) + dd;
    if constexpr (E::kElem == FK_F32)
      return __ldg(reinterpret_cast<const float4*>(p));
    else
      return E::widen4(__ldg(reinterpret_cast<const uint2*>(p)));
  }
  __device__ __forceinline__ float4 k4(uint32_t t, uint32_t dd) const { return load(P.kblk, t, dd); }
  __device__ __forceinline__ float4 v4(uint32_t t, uint32_t dd) const { return load(P.vblk, t, dd); }
};

template <class E>
__global__ void __launch_bounds__(prompt::kThreads) attend_prompt_paged_kernel(AttendArgs<E> f, float* __restrict__ out,
                                                                               uint32_t ldo, uint32_t max_pos) {
  prompt::attend_prompt_body(f.a, PagedPromptSrc<E>{f.P, 0, 0}, out, ldo, max_pos);
}

template <class E>
cudaError_t launch_store(const FkKvStore& a, const FkPaged& pg, void* kc, void* vc, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d % 2 != 0 || a.d > 2048 || a.kv_heads == 0 || pg.block_size == 0 || pg.table_len == 0 || !pg.table || !kc ||
      !vc)
    return cudaErrorInvalidValue;
  if ((uint64_t)a.kv_heads * pg.block_size * a.d >= (1ull << 32)) return cudaErrorInvalidValue;
  StoreArgs<E> st;
  st.a = a;
  st.P = Pool{pg.table, static_cast<const uint64_t*>(kc), static_cast<const uint64_t*>(vc), pg.block_size,
              pg.table_len, pg.blocks};
  const uint32_t half = a.d / 2;
  const uint32_t hb = half >= 256 ? 1u : (a.kv_heads < 256u / half ? a.kv_heads : 256u / half);  // heads a block
  return fk_launch_ex(kv_store_paged_kernel<E>, dim3((a.kv_heads + hb - 1) / hb, a.m), dim3(hb * half), 0, s, a.pdl,
                      st);
}

template <class E, bool FUSED>
cudaError_t launch_attend(const FkAttend& a, const FkPaged& pg, const void* kc, const void* vc, uint32_t k_off,
                          uint32_t v_off, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d != kHeadDim || a.chunk == 0 || a.chunk > kMaxChunk || a.kv_heads == 0 || a.heads % a.kv_heads != 0 ||
      a.m > kMaxAttendRows || (uint64_t)a.m * a.heads * a.max_splits >= (1ull << 32) || pg.block_size == 0 ||
      pg.table_len == 0 || !pg.table || !kc || !vc)
    return cudaErrorInvalidValue;
  if ((uint64_t)a.kv_heads * pg.block_size * kHeadDim >= (1ull << 32)) return cudaErrorInvalidValue;
  AttendArgs<E> f = {};
  f.a = a;
  f.P = Pool{pg.table, static_cast<const uint64_t*>(kc), static_cast<const uint64_t*>(vc), pg.block_size,
             pg.table_len, pg.blocks};
  if (FUSED) {
    if (a.rotated > kHeadDim / 2) return cudaErrorInvalidValue;
    f.k_off = k_off;
    f.v_off = v_off;
  }
  auto kern = attend_paged_kernel<E, FUSED>;
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
cudaError_t launch_prompt(const FkAttend& a, const FkPaged& pg, const void* kc, const void* vc, float* out, uint32_t ldo,
                          uint32_t max_pos, cudaStream_t s) {
  if (a.m == 0) return cudaSuccess;
  if (a.d != kHeadDim || a.kv_heads == 0 || a.heads % a.kv_heads != 0 || pg.block_size == 0 ||
      pg.table_len == 0 || !pg.table || !kc || !vc || (uint64_t)max_pos >= (uint64_t)pg.table_len * pg.block_size)
    return cudaErrorInvalidValue;
  if (ldo % 4 != 0 || (uintptr_t)out % 16 != 0) return cudaErrorInvalidValue;  // 16-byte stores
  const size_t smem = prompt::kSmemBytes;
  auto kern = attend_prompt_paged_kernel<E>;
  cudaError_t e = fk_allow_smem(kern, smem);
  if (e != cudaSuccess) return e;
  if ((uint64_t)a.kv_heads * pg.block_size * kHeadDim >= (1ull << 32)) return cudaErrorInvalidValue;
  AttendArgs<E> f = {};
  f.a = a;
  f.P = Pool{pg.table, static_cast<const uint64_t*>(kc), static_cast<const uint64_t*>(vc), pg.block_size,
             pg.table_len, pg.blocks};
  const dim3 grid = prompt::prompt_grid(a.m, a.heads);
  return fk_launch_ex(kern, grid, dim3(prompt::kThreads), smem, s, a.pdl, f, out, ldo, max_pos);
}

}  // namespace paged
}  // namespace fk

// The launch for a cache of element type e: f32, bf16 or f16.
#define FK_BY_ELEM(e, CALL)                          \
  ((e) == FK_F32    ? CALL(fk::F32)                  \
   : (e) == FK_BF16 ? CALL(fk::Bf16)                 \
   : (e) == FK_F16  ? CALL(fk::F16)                  \
                    : cudaErrorInvalidValue)

cudaError_t fk_launch_kv_store_paged(const FkKvStore& a, const FkPaged& pg, void* kc, void* vc, FkElem e,
                                     cudaStream_t s) {
#define CALL(E) fk::paged::launch_store<E>(a, pg, kc, vc, s)
  return FK_BY_ELEM(e, CALL);
#undef CALL
}

cudaError_t fk_launch_attend_paged(const FkAttend& a, const FkPaged& pg, const void* kc, const void* vc, FkElem e,
                                   cudaStream_t s) {
#define CALL(E) fk::paged::launch_attend<E, false>(a, pg, kc, vc, 0, 0, s)
  return FK_BY_ELEM(e, CALL);
#undef CALL
}

cudaError_t fk_launch_attend_decode_paged(const FkAttend& a, const FkPaged& pg, void* kc, void* vc, FkElem e,
                                          uint32_t k_off, uint32_t v_off, cudaStream_t s) {
#define CALL(E) fk::paged::launch_attend<E, true>(a, pg, kc, vc, k_off, v_off, s)
  return FK_BY_ELEM(e, CALL);
#undef CALL
}

cudaError_t fk_launch_attend_prompt_paged(const FkAttend& a, const FkPaged& pg, const void* kc, const void* vc,
                                          FkElem e, float* out, uint32_t ldo, uint32_t max_pos, cudaStream_t s) {
#define CALL(E) fk::paged::launch_prompt<E>(a, pg, kc, vc, out, ldo, max_pos, s)
  return FK_BY_ELEM(e, CALL);
#undef CALL
}
