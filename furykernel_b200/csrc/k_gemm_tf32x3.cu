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

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}

__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the barrier's phase, at most kWaitCycles; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity))
    if (clock64() - t0 > kWaitCycles) return false;
  return true;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(map), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// The shared-memory matrix descriptor of a K-major operand tile in the
// 128-byte-swizzled canonical layout: rows of 128 bytes, 8-row atoms 1024
// bytes apart (stride byte offset), descriptor version 1, swizzle mode 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(1024u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// The instruction descriptor of kind::tf32: f32 accumulators, TF32 A and B,
// both K-major, N = kGN, M = kGM.
__host__ __device__ constexpr uint32_t tf32_idesc() {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(kGN >> 3) << 17) | ((uint32_t)(kGM >> 4) << 24);
}

__device__ __forceinline__ void mma_tf32(uint32_t tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem),
      "l"(da), "l"(db), "r"(tf32_idesc()), "r"(accumulate));
}

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void record(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

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
      if (use > 0 && !mbar_wait(smem_u32(&bars[kStages + s]), (use - 1) & 1)) {
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
      if (!mbar_wait(smem_u32(&bars[s]), use & 1)) {
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
        mma_tf32(tmem, sw128_desc(a_hi + off), sw128_desc(w_hi + off), acc);
        mma_tf32(tmem, sw128_desc(a_hi + off), sw128_desc(w_lo + off), 1u);
        mma_tf32(tmem, sw128_desc(a_lo + off), sw128_desc(w_hi + off), 1u);
      }
      mma_commit(smem_u32(&bars[kStages + s]));  // the stage is free once these finish
    }
    mma_commit(smem_u32(&bars[2 * kStages]));  // the accumulator, once all finish
    if (!ok) aborted = 1;
  }

  if (warp < 4) {
    // The epilogue: warp w reads TMEM lanes (rows) 32w .. 32w + 31.
    if (!mbar_wait(smem_u32(&bars[2 * kStages]), 0)) {
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
__global__ void split_tf32_kernel(const float* __restrict__ x, float* __restrict__ hi, float* __restrict__ lo,
                                  uint64_t n) {
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += (uint64_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    uint32_t h, l;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
    const float rest = __fsub_rn(v, __uint_as_float(h));
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(l) : "f"(rest));
    hi[i] = __uint_as_float(h);
    lo[i] = __uint_as_float(l);
  }
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
  uint64_t blocks = (n + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  fk::split_tf32_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, hi, lo, n);
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
