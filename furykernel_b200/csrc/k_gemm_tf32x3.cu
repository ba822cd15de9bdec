// Prefill GEMM on the 5th-generation tensor cores: C[M, N] = A[M, K] W[N, K]^T
// in f32, as three TF32 products (3xTF32): each operand x = x_hi + x_lo, its
// two parts TF32 values (rounded to nearest from x, then from x - x_hi), and
// C = A_hi W_hi + A_hi W_lo + A_lo W_hi accumulated in f32 in tensor memory.
// The product dropped, A_lo W_lo, is below 2^-22 of |A||W|; the sums are the
// tensor cores' own order, so results are held to the f64 evaluator's bounds
// (src/FuryKernel/Program/Eval.hs:747-754) rather than to the CPU target's
// bits (the gemmTile of src/FuryKernel/Tile.hs:76-157 fixes an order this
// kernel does not keep).
//
// A CTA computes one 128 x 128 tile of C: warp 4 moves K slabs of 32 floats
// of A_hi, A_lo, W_hi, W_lo into a 3-stage ring of shared memory by TMA (128B
// swizzle); one thread of warp 5 issues tcgen05.mma kind::tf32 (128 x 128 x
// 8, K-major operands) into a 128-column TMEM accumulator and commits each
// stage back to the producer; warps 0-3 read the accumulator out by
// tcgen05.ld (warp w owns TMEM lanes 32w..32w+31) and store C. Every wait is
// bounded in time: past it the kernel records an error code and leaves.
// No TMA multicast: the loads read this GPU's memory only, one CTA each.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include "fk_common.cuh"
#include "fk_kernels.h"
#include "fk_tcgen05.cuh"

namespace fk {

constexpr int kGM = 128, kGN = 128, kGK = 32, kStages = 3;
constexpr int kTileA = kGM * kGK * 4;  // 16 KiB
constexpr int kTileB = kGN * kGK * 4;  // 16 KiB
constexpr int kStageBytes = 2 * kTileA + 2 * kTileB;
constexpr int kGemmSmem = kStages * kStageBytes + 1024 /* align */ + 256 /* barriers */;
constexpr int kTmemCols = 128;
constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at the B200's clock

// Error codes the kernel records (first one wins).
enum { GEMM_OK = 0, GEMM_TIMEOUT_FULL = 1, GEMM_TIMEOUT_EMPTY = 2, GEMM_TIMEOUT_ACCUM = 3 };

using namespace tc;

__global__ void __launch_bounds__(192, 1)
    gemm_tf32x3_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                       const __grid_constant__ CUtensorMap tw_hi, const __grid_constant__ CUtensorMap tw_lo,
                       float* __restrict__ c, uint32_t M, uint32_t N, uint32_t K, uint32_t ldc,
                       int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  // bars[0..S): full, bars[S..2S): empty, bars[2S]: accumulator ready.
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 1);
  __shared__ int aborted;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // M tiles vary fastest: the CTAs that share a weight tile (one N tile,
  // every M tile) run together, so the tile crosses HBM once and is reused
  // from L2.
  const uint32_t m0 = blockIdx.x * kGM, n0 = blockIdx.y * kGN;
  const uint32_t kblocks = K / kGK;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bars[s]), 1);
      mbar_init(smem_u32(&bars[kStages + s]), 1);
    }
    mbar_init(smem_u32(&bars[2 * kStages]), 1);
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
    // The producer: K slabs of the four operand tiles into the ring.
    for (uint32_t kb = 0; kb < kblocks; ++kb) {
      const uint32_t s = kb % kStages, use = kb / kStages;
      if (use > 0 && !mbar_wait(smem_u32(&bars[kStages + s]), (use - 1) & 1, kWaitCycles)) {
        record(err, GEMM_TIMEOUT_EMPTY);
        aborted = 1;
        break;
      }
      uint8_t* st = smem + s * kStageBytes;
      const uint32_t full = smem_u32(&bars[s]);
      mbar_expect_tx(full, kStageBytes);
      const int x = (int)(kb * kGK);
      tma_load_2d(smem_u32(st), &ta_hi, x, (int)m0, full);
      tma_load_2d(smem_u32(st + kTileA), &ta_lo, x, (int)m0, full);
      tma_load_2d(smem_u32(st + 2 * kTileA), &tw_hi, x, (int)n0, full);
      tma_load_2d(smem_u32(st + 2 * kTileA + kTileB), &tw_lo, x, (int)n0, full);
    }
  } else if (warp == 5 && lane == 0) {
    // The MMA issuer: three TF32 products a K step, 4 steps a slab.
    bool ok = true;
    for (uint32_t kb = 0; kb < kblocks && ok; ++kb) {
      const uint32_t s = kb % kStages, use = kb / kStages;
      if (!mbar_wait(smem_u32(&bars[s]), use & 1, kWaitCycles)) {
        record(err, GEMM_TIMEOUT_FULL);
        ok = false;
        break;
      }
      fence_after();
      const uint32_t a_hi = smem_u32(smem + s * kStageBytes);
      const uint32_t a_lo = a_hi + kTileA;
      const uint32_t w_hi = a_hi + 2 * kTileA;
      const uint32_t w_lo = w_hi + kTileB;
#pragma unroll
      for (uint32_t kk = 0; kk < kGK / 8; ++kk) {
        const uint32_t off = kk * 32;  // 8 floats of K within the 128-byte row
        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
        mma_tf32(tmem, sw128_desc(a_hi + off), sw128_desc(w_hi + off), tf32_idesc(kGN), acc);
        mma_tf32(tmem, sw128_desc(a_hi + off), sw128_desc(w_lo + off), tf32_idesc(kGN), 1u);
        mma_tf32(tmem, sw128_desc(a_lo + off), sw128_desc(w_hi + off), tf32_idesc(kGN), 1u);
      }
      mma_commit(smem_u32(&bars[kStages + s]));  // the stage is free once these finish
    }
    mma_commit(smem_u32(&bars[2 * kStages]));  // the accumulator, once all finish
    if (!ok) aborted = 1;
  }

  if (warp < 4) {
    // The epilogue: warp w reads TMEM lanes (rows) 32w .. 32w + 31.
    if (!mbar_wait(smem_u32(&bars[2 * kStages]), 0, kWaitCycles)) {
      record(err, GEMM_TIMEOUT_ACCUM);
    } else if (!aborted) {
      fence_after();
      const uint32_t row = m0 + 32 * warp + lane;
#pragma unroll 1
      for (int cc = 0; cc < kGN / 32; ++cc) {
        uint32_t r[32];
        tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)(cc * 32), r);
        const uint32_t col0 = n0 + cc * 32;
        if (row < M) {
          float* out = c + (size_t)row * ldc + col0;
          if (col0 + 32 <= N && ((ldc & 3) == 0)) {
#pragma unroll
            for (int j = 0; j < 32; j += 4)
              *reinterpret_cast<float4*>(out + j) = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                                                __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < N) out[j] = __uint_as_float(r[j]);
          }
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

// x = hi + lo, each a TF32 value rounded to nearest (ties away) in turn.
__device__ __forceinline__ void split_one(float v, float& h, float& l) {
  uint32_t hb, lb;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(hb) : "f"(v));
  const float rest = __fsub_rn(v, __uint_as_float(hb));
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(lb) : "f"(rest));
  h = __uint_as_float(hb);
  l = __uint_as_float(lb);
}

// With vec (n a multiple of 4, the arrays on 16 bytes), 16-byte loads and
// stores, two in flight a thread; else an element at a time.
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  uint64_t n, int vec) {
  const uint64_t T = (uint64_t)gridDim.x * blockDim.x, t = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* h4 = reinterpret_cast<float4*>(hi);
    float4* l4 = reinterpret_cast<float4*>(lo);
    const uint64_t n4 = n / 4;
    for (uint64_t i = t; i < n4; i += 2 * T) {
      const bool two = i + T < n4;
      const float4 a = __ldcs(x4 + i);
      const float4 b = two ? __ldcs(x4 + i + T) : a;
      float4 ah, al, bh, bl;
      split_one(a.x, ah.x, al.x);
      split_one(a.y, ah.y, al.y);
      split_one(a.z, ah.z, al.z);
      split_one(a.w, ah.w, al.w);
      h4[i] = ah;
      l4[i] = al;
      if (two) {
        split_one(b.x, bh.x, bl.x);
        split_one(b.y, bh.y, bl.y);
        split_one(b.z, bh.z, bl.z);
        split_one(b.w, bh.w, bl.w);
        h4[i + T] = bh;
        l4[i + T] = bl;
      }
    }
    return;
  }
  for (uint64_t i = t; i < n; i += T) split_one(x[i], hi[i], lo[i]);
}

}  // namespace fk

namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
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

// A row-major [rows, K] f32 matrix as TMA tiles of 32 x 128 (x = K), 128B swizzle.
bool make_map(CUtensorMap* map, const float* base, uint32_t rows, uint32_t K, uint32_t box_rows) {
  auto fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 4};
  cuuint32_t box[2] = {(cuuint32_t)fk::kGK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

cudaError_t fk_launch_split_tf32(const float* x, float* hi, float* lo, uint64_t n, cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  const int vec = n % 4 == 0 && (((uintptr_t)x | (uintptr_t)hi | (uintptr_t)lo) & 15) == 0;
  uint64_t blocks = ((vec ? n / 8 : n) + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks == 0) blocks = 1;
  fk::split_tf32_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, hi, lo, n, vec);
  return cudaGetLastError();
}

cudaError_t fk_launch_gemm_tf32x3(const float* a_hi, const float* a_lo, const float* w_hi, const float* w_lo,
                                  float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t ldc, int* err,
                                  cudaStream_t s) {
  if (M == 0 || N == 0) return cudaSuccess;
  if (K == 0 || K % fk::kGK != 0 || ((uintptr_t)a_hi | (uintptr_t)a_lo | (uintptr_t)w_hi | (uintptr_t)w_lo) & 15)
    return cudaErrorInvalidValue;
  CUtensorMap ma_hi, ma_lo, mw_hi, mw_lo;
  if (!make_map(&ma_hi, a_hi, M, K, fk::kGM) || !make_map(&ma_lo, a_lo, M, K, fk::kGM) ||
      !make_map(&mw_hi, w_hi, N, K, fk::kGN) || !make_map(&mw_lo, w_lo, N, K, fk::kGN))
    return cudaErrorInvalidValue;
  {
    cudaError_t e = fk_allow_smem(fk::gemm_tf32x3_kernel, fk::kGemmSmem);
    if (e != cudaSuccess) return e;
  }
  if ((N + fk::kGN - 1) / fk::kGN > 65535) return cudaErrorInvalidValue;
  dim3 grid((M + fk::kGM - 1) / fk::kGM, (N + fk::kGN - 1) / fk::kGN);
  fk::gemm_tf32x3_kernel<<<grid, 192, fk::kGemmSmem, s>>>(ma_hi, ma_lo, mw_hi, mw_lo, c, M, N, K, ldc, err);
  return cudaGetLastError();
}
