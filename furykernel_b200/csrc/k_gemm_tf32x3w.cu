// Prefill GEMM on the 5th-generation tensor cores, the weights as they lie:
// C[M, N] = A[M, K] W[N, K]^T in f32 as three TF32 products (3xTF32),
// C = A_hi W_hi + A_hi W_lo + A_lo W_hi, each operand x = x_hi + x_lo with
// x_hi = tf32(x) and x_lo = tf32(x - x_hi) (round to nearest, ties away:
// the split of split_tf32, so the products are those of gemm_tf32x3). A,
// the small operand (the prompt's rows), comes split by the launcher; W is
// read once as f32 and split inside the kernel, so no TF32 copies of the
// weights exist in HBM. Held to the f64 evaluator's binary32 bounds
// (src/FuryKernel/Program/Eval.hs: dotA, the products added in any order),
// not to the CPU target's gemmTile order (src/FuryKernel/Tile.hs:76-157).
//
// A CTA computes one 128 x tn tile of C, tn a multiple of 16 up to 256
// chosen per shape by the launcher so that the tiles fill the SMs in as few
// rounds as possible (config 3c, M 512, N 11008: tn 160, 276 tiles, two
// rounds on 148 SMs, where 128-wide tiles take three). K moves in slabs of
// 32 floats (one 128-byte swizzled row a matrix row) through a ring of
// `stages` buffers:
//   warp 4      TMA: A_hi, A_lo (128 rows) and W (tn rows) of the slab;
//   warps 6..9  the W split: each float of the slab rewritten in place as
//               its TF32 high part, its low part into a twin buffer (the
//               same swizzled byte offset), then the async-proxy fence;
//   warp 5      one thread issues tcgen05.mma kind::tf32 (128 x tn x 8,
//               K-major) into a TMEM accumulator: hi*hi, hi*lo, lo*hi;
//   warps 0..3  the epilogue: warp w reads TMEM lanes 32w..32w+31 by
//               tcgen05.ld and stores C.
// Every wait is bounded: past its bound the kernel records a status code
// (fkc_status), waits (bounded) for its own TMA loads in flight, frees its
// TMEM and returns. No TMA multicast: every load reads this GPU's memory.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "fk_common.cuh"
#include "fk_kernels.h"
#include "fk_tcgen05.cuh"

namespace fk {
namespace gw {

using namespace tc;

constexpr uint32_t kBM = 128, kBK = 32;
constexpr uint32_t kMaxN = 256;
constexpr uint32_t kTileA = kBM * kBK * 4;  // 16 KiB
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kThreads = 320;          // 10 warps
constexpr uint32_t kMaxStages = 6;
constexpr uint32_t kSmemBudget = 220 * 1024;

// Status codes (first one wins), after gemm_tf32x3's 1..3.
enum { GW_TIMEOUT_EMPTY = 4, GW_TIMEOUT_FULL = 5, GW_TIMEOUT_SPLIT = 6, GW_TIMEOUT_ACCUM = 7 };

__host__ __device__ constexpr uint32_t stage_bytes(uint32_t tn) { return 2 * kTileA + 2 * tn * kBK * 4; }

__device__ __forceinline__ uint32_t tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3w_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                        const __grid_constant__ CUtensorMap tw, float* __restrict__ c, uint32_t M, uint32_t N,
                        uint32_t K, uint32_t ldc, uint32_t tn, uint32_t stages, long long wait_cycles,
                        int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = stage_bytes(tn);
  // Barriers after the ring: full[S] (TMA bytes), split[S] (the four split
  // warps), empty[S] (the MMAs of the slab done), accum (all MMAs done).
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + stages * sb);
  uint64_t* full = bars;
  uint64_t* split = bars + kMaxStages;
  uint64_t* empty = bars + 2 * kMaxStages;
  uint64_t* accum = bars + 3 * kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * kMaxStages + 1);
  __shared__ int aborted;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // M tiles vary fastest: the CTAs that share a weight tile run together,
  // so the tile crosses HBM once and is reused from L2.
  const uint32_t m0 = blockIdx.x * kBM, n0 = blockIdx.y * tn;
  const uint32_t kblocks = K / kBK;
  const uint32_t w_bytes = tn * kBK * 4;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (uint32_t s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&split[s]), 4);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(accum), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 5) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4 && lane == 0) {
    // The producer. `issued` counts the slabs whose loads went out, so that
    // after an abort it can wait for the ones still in flight.
    uint32_t issued = 0;
    for (uint32_t kb = 0; kb < kblocks; ++kb) {
      const uint32_t s = kb % stages, use = kb / stages;
      if (use > 0 && !mbar_wait(smem_u32(&empty[s]), (use - 1) & 1, wait_cycles)) {
        record(err, GW_TIMEOUT_EMPTY);
        aborted = 1;
        break;
      }
      if (*reinterpret_cast<volatile int*>(&aborted)) break;
      uint8_t* st = smem + s * sb;
      const uint32_t bar = smem_u32(&full[s]);
      mbar_expect_tx(bar, sb - w_bytes);  // A_hi, A_lo, W (the low-part twin is written here)
      const int x = (int)(kb * kBK);
      tma_load_2d(smem_u32(st), &ta_hi, x, (int)m0, bar);
      tma_load_2d(smem_u32(st + kTileA), &ta_lo, x, (int)m0, bar);
      tma_load_2d(smem_u32(st + 2 * kTileA), &tw, x, (int)n0, bar);
      ++issued;
    }
    // Loads in flight finish before the CTA leaves (bounded).
    const uint32_t first = issued > stages ? issued - stages : 0;
    for (uint32_t kb = first; kb < issued; ++kb)
      if (!mbar_wait(smem_u32(&full[kb % stages]), (kb / stages) & 1, wait_cycles)) record(err, GW_TIMEOUT_FULL);
  } else if (warp >= 6) {
    // The W split: thread t of the 128 takes 16-byte chunks t, t + 128, ...
    // of the slab's W tile (an element-wise map, so the swizzle is kept).
    const uint32_t t = threadIdx.x - 192;
    const uint32_t chunks = w_bytes / 16;
    for (uint32_t kb = 0; kb < kblocks; ++kb) {
      const uint32_t s = kb % stages, use = kb / stages;
      if (!mbar_wait(smem_u32(&full[s]), use & 1, wait_cycles)) {
        record(err, GW_TIMEOUT_FULL);
        aborted = 1;
        break;
      }
      float4* w = reinterpret_cast<float4*>(smem + s * sb + 2 * kTileA);
      float4* wlo = reinterpret_cast<float4*>(smem + s * sb + 2 * kTileA + w_bytes);
      for (uint32_t i = t; i < chunks; i += 128) {
        const float4 v = w[i];
        const uint32_t hx = tf32_rna(v.x), hy = tf32_rna(v.y), hz = tf32_rna(v.z), hw = tf32_rna(v.w);
        const float4 lo = make_float4(__uint_as_float(tf32_rna(__fsub_rn(v.x, __uint_as_float(hx)))),
                                      __uint_as_float(tf32_rna(__fsub_rn(v.y, __uint_as_float(hy)))),
                                      __uint_as_float(tf32_rna(__fsub_rn(v.z, __uint_as_float(hz)))),
                                      __uint_as_float(tf32_rna(__fsub_rn(v.w, __uint_as_float(hw)))));
        w[i] = make_float4(__uint_as_float(hx), __uint_as_float(hy), __uint_as_float(hz), __uint_as_float(hw));
        wlo[i] = lo;
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&split[s]));
    }
  } else if (warp == 5 && lane == 0) {
    // The MMA issuer: three TF32 products a K step of 8, 4 steps a slab.
    const uint32_t idesc = tf32_idesc(tn);
    bool ok = true;
    for (uint32_t kb = 0; kb < kblocks && ok; ++kb) {
      const uint32_t s = kb % stages, use = kb / stages;
      if (!mbar_wait(smem_u32(&split[s]), use & 1, wait_cycles)) {
        record(err, GW_TIMEOUT_SPLIT);
        ok = false;
        break;
      }
      fence_after();
      const uint32_t a_hi = smem_u32(smem + s * sb);
      const uint32_t a_lo = a_hi + kTileA;
      const uint32_t w_hi = a_hi + 2 * kTileA;
      const uint32_t w_lo = w_hi + w_bytes;
#pragma unroll
      for (uint32_t kk = 0; kk < kBK / 8; ++kk) {
        const uint32_t off = kk * 32;  // 8 floats of K within the 128-byte row
        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
        mma_tf32(tmem, sw128_desc(a_hi + off), sw128_desc(w_hi + off), idesc, acc);
        mma_tf32(tmem, sw128_desc(a_hi + off), sw128_desc(w_lo + off), idesc, 1u);
        mma_tf32(tmem, sw128_desc(a_lo + off), sw128_desc(w_hi + off), idesc, 1u);
      }
      mma_commit(smem_u32(&empty[s]));  // the slab's buffers are free once these finish
    }
    mma_commit(smem_u32(accum));  // the accumulator, once every MMA issued finishes
    if (!ok) aborted = 1;
  }

  if (warp < 4) {
    // The epilogue: warp w reads TMEM lanes (rows) 32w .. 32w + 31, 32
    // columns at a time (16 for the last piece of a tile of 16 * odd).
    if (!mbar_wait(smem_u32(accum), 0, wait_cycles)) {
      record(err, GW_TIMEOUT_ACCUM);
    } else if (!*reinterpret_cast<volatile int*>(&aborted)) {
      fence_after();
      const uint32_t row = m0 + 32 * warp + lane;
      float* out = c + (size_t)row * ldc;
      const bool vec = (ldc & 3) == 0;
#pragma unroll 1
      for (uint32_t cc = 0; cc < tn; cc += 32) {
        const uint32_t taddr = tmem + ((32 * warp) << 16) + cc;
        const uint32_t col0 = n0 + cc;
        if (cc + 32 <= tn) {
          uint32_t r[32];
          tmem_ld32(taddr, r);
          if (row < M) {
            if (vec && col0 + 32 <= N) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<float4*>(out + col0 + j) =
                    make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]), __uint_as_float(r[j + 2]),
                                __uint_as_float(r[j + 3]));
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < N) out[col0 + j] = __uint_as_float(r[j]);
            }
          }
        } else {
          uint32_t r[16];
          tmem_ld16(taddr, r);
          if (row < M)
            for (int j = 0; j < 16; ++j)
              if (col0 + j < N) out[col0 + j] = __uint_as_float(r[j]);
        }
      }
    }
  }
  fence_before();
  __syncthreads();
  fence_after();
  if (warp == 5)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace gw
}  // namespace fk

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_w() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// A row-major [rows, K] f32 matrix as TMA tiles of 32 x box_rows (x = K),
// 128-byte swizzle; rows past the matrix read as zeros.
bool make_map_w(CUtensorMap* map, const float* base, uint32_t rows, uint32_t K, uint32_t box_rows) {
  auto fn = encode_fn_w();
  if (!fn) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 4};
  cuuint32_t box[2] = {fk::gw::kBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// The tile width for M x N on `sms` SMs: among 16, 32, ..., 256, the one
// whose tiles take the fewest column-rounds, rounds x (tn + 24) (a tile's
// fixed cost counted as 24 columns), the wider on a tie.
uint32_t fk_gemm_tf32x3w_tile(uint32_t M, uint32_t N, int sms) {
  const uint64_t mt = (M + fk::gw::kBM - 1) / fk::gw::kBM;
  uint32_t best = 256;
  uint64_t best_cost = ~0ull;
  for (uint32_t tn = 256; tn >= 16; tn -= 16) {
    const uint64_t tiles = mt * ((N + tn - 1) / tn);
    const uint64_t rounds = (tiles + (uint64_t)sms - 1) / (uint64_t)sms;
    const uint64_t cost = rounds * (tn + 24);
    if (cost < best_cost) {
      best_cost = cost;
      best = tn;
    }
  }
  return best;
}

cudaError_t fk_launch_gemm_tf32x3w(const float* a_hi, const float* a_lo, const float* w, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, uint32_t ldc, uint32_t tn, long long wait_cycles, int* err,
                                   cudaStream_t s) {
  using namespace fk::gw;
  if (M == 0 || N == 0) return cudaSuccess;
  if (K == 0 || K % kBK != 0 || tn == 0 || tn % 16 != 0 || tn > kMaxN || ldc < N ||
      ((uintptr_t)a_hi | (uintptr_t)a_lo | (uintptr_t)w) & 15)
    return cudaErrorInvalidValue;
  uint32_t stages = kSmemBudget / stage_bytes(tn);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return cudaErrorInvalidValue;
  const size_t smem = 1024 + (size_t)stages * stage_bytes(tn) + 256;
  CUtensorMap ma_hi, ma_lo, mw;
  if (!make_map_w(&ma_hi, a_hi, M, K, kBM) || !make_map_w(&ma_lo, a_lo, M, K, kBM) || !make_map_w(&mw, w, N, K, tn))
    return cudaErrorInvalidValue;
  cudaError_t e = fk_allow_smem(gemm_tf32x3w_kernel, smem);
  if (e != cudaSuccess) return e;
  const uint32_t ntiles = (N + tn - 1) / tn;
  if (ntiles > 65535) return cudaErrorInvalidValue;
  dim3 grid((M + kBM - 1) / kBM, ntiles);
  gemm_tf32x3w_kernel<<<grid, kThreads, smem, s>>>(ma_hi, ma_lo, mw, c, M, N, K, ldc, tn, stages,
                                                    wait_cycles > 0 ? wait_cycles : 4000000000LL, err);
  return cudaGetLastError();
}
