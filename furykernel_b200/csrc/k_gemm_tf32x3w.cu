// Prefill GEMM on the 5th-generation tensor cores, the weights as they lie:
// C[M, N] = A[M, K] W[N, K]^T in f32 as three TF32 products (3xTF32),
// C = A_hi W_hi + A_hi W_lo + A_lo W_hi, each operand x = x_hi + x_lo with
// x_hi = tf32(x) and x_lo = tf32(x - x_hi) (round to nearest, ties away:
// the split of split_tf32, so the products are those of gemm_tf32x3). A,
// the small operand (the prompt's rows), comes split by the launcher; W is
// read once as f32 and split on the chip, so no TF32 copies of the weights
// exist in HBM. Held to the f64 evaluator's binary32 bounds
// (src/FuryKernel/Program/Eval.hs: dotA, the products added in any order),
// not to the CPU target's gemmTile order (src/FuryKernel/Tile.hs:76-157).
//
// The MMA computes the tile transposed, D = W A^T: a CTA owns 128 rows of W
// (the MMA's M, one TMEM lane each) and tm rows of A (the MMA's N, tm a
// multiple of 16 up to 256). W is the MMA's A operand and lives in tensor
// memory: its split never touches shared memory's MMA operand path, whose
// bandwidth the MMA's B operand needs. K moves in slabs of 16 floats
// (64-byte rows, 64-byte swizzle) through `stages` buffers:
//   warp 4      TMA: the slab's A_hi and A_lo rows and its 128 W rows;
//   warps 0..3  the W split: thread t reads row t of the W slab (its four
//               16-byte chunks, where the swizzle put them), splits the 16
//               floats in registers and stores the high and low parts into
//               16 + 16 columns of its TMEM lane (tcgen05.st); after the
//               last slab, the epilogue: warp w reads lanes 32w..32w+31 of
//               the accumulator (tcgen05.ld) and stores C, the lanes'
//               consecutive columns of a row of C together;
//   warp 5      one thread issues tcgen05.mma kind::tf32 (128 x tm x 8, A
//               from TMEM, B K-major from shared memory): hi*hi, lo*hi,
//               hi*lo, into a TMEM accumulator of tm columns.
// A kind::tf32 MMA costs about 140 SM cycles up to N = 176 and 168 at
// N = 256 (measured on a B200, K 8): the wide tile nearly doubles the
// flops an instruction, and 16-float slabs keep 5 stages of a 256-row
// tile in shared memory. Shapes with fewer tiles than SMs split K in two
// (grid z): each half adds its partial tile into C, which the launcher
// zeroes first; two additions onto zero give the same bits in either
// order, so the result does not depend on which half lands first.
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

constexpr uint32_t kBW = 128, kBK = 16;  // W rows a tile (TMEM lanes), K a slab
constexpr uint32_t kRowBytes = kBK * 4;   // a slab's row: 64 bytes
constexpr uint32_t kMaxTm = 256;
constexpr uint32_t kTmemCols = 512;       // accumulator [0, 256), W stages from 256, 32 columns each
constexpr uint32_t kWCol0 = 256;
constexpr uint32_t kThreads = 192;        // 6 warps
constexpr uint32_t kMaxStages = 8;
constexpr uint32_t kSmemBudget = 216 * 1024;
constexpr uint32_t kSmemFloor = 120 * 1024;  // one CTA an SM: its TMEM allocation is all of TMEM

// Status codes (first one wins), after gemm_tf32x3's 1..3.
enum { GW_TIMEOUT_EMPTY = 4, GW_TIMEOUT_FULL = 5, GW_TIMEOUT_SPLIT = 6, GW_TIMEOUT_ACCUM = 7 };

// A stage: A_hi then A_lo, tm rows of 64 bytes each, then the W slab's 128
// rows.
constexpr uint32_t kWSlab = kBW * kRowBytes;  // 8 KiB
__host__ __device__ constexpr uint32_t stage_bytes(uint32_t tm) { return 2 * tm * kRowBytes + kWSlab; }

__device__ __forceinline__ uint32_t tf32_rna(float v) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(v));
  return r;
}

// The shared-memory matrix descriptor of a K-major operand tile in the
// 64-byte-swizzled canonical layout: rows of 64 bytes, 8-row atoms 512 bytes
// apart (stride byte offset), descriptor version 1, swizzle mode 4.
__device__ __forceinline__ uint64_t sw64_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);
  d |= (uint64_t)(16u >> 4) << 16;
  d |= (uint64_t)(512u >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)4 << 61;
  return d;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3w_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                        const __grid_constant__ CUtensorMap tw, float* __restrict__ c, uint32_t M, uint32_t N,
                        uint32_t K, uint32_t ldc, uint32_t tm, uint32_t stages, long long wait_cycles,
                        int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = stage_bytes(tm);
  // Barriers after the ring: full[S] (the slab's TMA bytes), split[S] (the
  // four split warps stored the W slab), empty[S] (the slab's MMAs done:
  // its shared and tensor memory free), accum (every MMA done).
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + stages * sb);
  uint64_t* full = bars;
  uint64_t* split = bars + kMaxStages;
  uint64_t* empty = bars + 2 * kMaxStages;
  uint64_t* accum = bars + 3 * kMaxStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 3 * kMaxStages + 1);
  __shared__ int aborted;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // A tiles vary fastest: the CTAs that share a W tile run together, so it
  // crosses HBM once and is reused from L2. blockIdx.z: the K half.
  const uint32_t m0 = blockIdx.x * tm, n0 = blockIdx.y * kBW;
  const uint32_t kblocks = K / kBK, per = (kblocks + gridDim.z - 1) / gridDim.z;
  const uint32_t kbeg = blockIdx.z * per, kend = min(kblocks, kbeg + per);
  const uint32_t nk = kend > kbeg ? kend - kbeg : 0;

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

  if (warp < 4) {
    // The W split, a row a thread (TMEM lane 32 warp + lane). Chunk j of
    // row r sits at chunk j ^ ((r / 2) % 4) of the row (64-byte swizzle).
    const uint32_t row = 32 * warp + lane;
    const uint32_t lane_addr = tmem + ((32 * warp) << 16);
    for (uint32_t i = 0; i < nk; ++i) {
      const uint32_t s = i % stages, use = i / stages;
      // One lane waits and tells the others, so that the warp stays together
      // for its warp-wide TMEM stores.
      int ready = 0;
      if (lane == 0) ready = mbar_wait(smem_u32(&full[s]), use & 1, wait_cycles) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, ready, 0)) {
        if (lane == 0) record(err, GW_TIMEOUT_FULL);
        aborted = 1;
        break;
      }
      const float4* wr = reinterpret_cast<const float4*>(smem + s * sb + 2 * tm * kRowBytes + row * kRowBytes);
      uint32_t hl[32];  // the high parts, then the low parts
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 v = wr[j ^ ((row >> 1) & 3)];
        const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          hl[4 * j + q] = tf32_rna(x[q]);
          hl[16 + 4 * j + q] = tf32_rna(__fsub_rn(x[q], __uint_as_float(hl[4 * j + q])));
        }
      }
      tmem_st32(lane_addr + kWCol0 + 32 * s, hl);
      tmem_wait_st();
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&split[s]));
    }
  } else if (warp == 4 && lane == 0) {
    // The producer. `issued` counts the slabs whose loads went out, so that
    // after an abort it can wait for the ones still in flight.
    uint32_t issued = 0;
    for (uint32_t i = 0; i < nk; ++i) {
      const uint32_t s = i % stages, use = i / stages;
      if (use > 0 && !mbar_wait(smem_u32(&empty[s]), (use - 1) & 1, wait_cycles)) {
        record(err, GW_TIMEOUT_EMPTY);
        aborted = 1;
        break;
      }
      if (*reinterpret_cast<volatile int*>(&aborted)) break;
      uint8_t* st = smem + s * sb;
      const uint32_t bar = smem_u32(&full[s]);
      mbar_expect_tx(bar, sb);
      const int x = (int)((kbeg + i) * kBK);
      tma_load_2d(smem_u32(st), &ta_hi, x, (int)m0, bar);
      tma_load_2d(smem_u32(st + tm * kRowBytes), &ta_lo, x, (int)m0, bar);
      tma_load_2d(smem_u32(st + 2 * tm * kRowBytes), &tw, x, (int)n0, bar);
      ++issued;
    }
    // Loads in flight finish before the CTA leaves (bounded).
    const uint32_t first = issued > stages ? issued - stages : 0;
    for (uint32_t i = first; i < issued; ++i)
      if (!mbar_wait(smem_u32(&full[i % stages]), (i / stages) & 1, wait_cycles)) record(err, GW_TIMEOUT_FULL);
  } else if (warp == 5 && lane == 0) {
    // The MMA issuer: three TF32 products a K step of 8, 2 steps a slab.
    const uint32_t idesc = tf32_idesc(tm, kBW);
    bool ok = true;
    for (uint32_t i = 0; i < nk && ok; ++i) {
      const uint32_t s = i % stages, use = i / stages;
      if (!mbar_wait(smem_u32(&split[s]), use & 1, wait_cycles)) {
        record(err, GW_TIMEOUT_SPLIT);
        ok = false;
        break;
      }
      fence_after();
      const uint32_t b_hi = smem_u32(smem + s * sb);
      const uint32_t b_lo = b_hi + tm * kRowBytes;
      const uint32_t w_hi = tmem + kWCol0 + 32 * s, w_lo = w_hi + 16;
#pragma unroll
      for (uint32_t kk = 0; kk < kBK / 8; ++kk) {
        const uint32_t off = kk * 32;  // 8 floats of K within the 64-byte row
        const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
        mma_tf32_ts(tmem, w_hi + 8 * kk, sw64_desc(b_hi + off), idesc, acc);
        mma_tf32_ts(tmem, w_lo + 8 * kk, sw64_desc(b_hi + off), idesc, 1u);
        mma_tf32_ts(tmem, w_hi + 8 * kk, sw64_desc(b_lo + off), idesc, 1u);
      }
      mma_commit(smem_u32(&empty[s]));  // the slab's buffers are free once these finish
    }
    mma_commit(smem_u32(accum));  // the accumulator, once every MMA issued finishes
    if (!ok) aborted = 1;
  }

  if (warp < 4 && nk > 0) {
    // The epilogue: lane 32w + l of the accumulator is W row n0 + 32w + l,
    // column j is A row m0 + j; C[m0 + j][n] from each, a row of C's 32
    // consecutive columns a store (or, K split, an addition) across the warp.
    int done = 0;
    if (lane == 0) done = mbar_wait(smem_u32(accum), 0, wait_cycles) ? 1 : 0;
    done = __shfl_sync(0xffffffffu, done, 0);
    if (!done) {
      if (lane == 0) record(err, GW_TIMEOUT_ACCUM);
    } else if (!__shfl_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&aborted), 0)) {
      fence_after();
      const uint32_t n = n0 + 32 * warp + lane;
      const bool live = n < N, add = gridDim.z > 1;
#pragma unroll 1
      for (uint32_t cc = 0; cc < tm; cc += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + ((32 * warp) << 16) + cc, r);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (live && m0 + cc + j < M) {
            float* at = c + (size_t)(m0 + cc + j) * ldc + n;
            if (add)
              atomicAdd(at, __uint_as_float(r[j]));
            else
              *at = __uint_as_float(r[j]);
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

// A row-major [rows, K] f32 matrix as TMA tiles of 16 x box_rows (x = K),
// 64-byte swizzle; rows past the matrix read as zeros.
bool make_map_w(CUtensorMap* map, const float* base, uint32_t rows, uint32_t K, uint32_t box_rows) {
  auto fn = encode_fn_w();
  if (!fn) return false;
  cuuint64_t dims[2] = {K, rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 4};
  cuuint32_t box[2] = {fk::gw::kBK, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

// The tile for M x N x K on `sms` SMs: tm among 16, 32, ..., 256 and K
// split in 1 or 2, the least modelled time: rounds of CTAs x (slabs a CTA x
// a slab's cost + the epilogue), with a 16-float slab's cost 350 + 0.62 tm
// SM cycles (from the measured MMA costs above) and an epilogue of
// 8 tm cycles, twice that when it adds.
FkGemmTile fk_gemm_tf32x3w_tile(uint32_t M, uint32_t N, uint32_t K, int sms) {
  FkGemmTile best = {256, 1};
  double best_cost = 1e300;
  const uint64_t wt = (N + fk::gw::kBW - 1) / fk::gw::kBW, kblocks = K / fk::gw::kBK;
  for (uint32_t split = 1; split <= 2; ++split) {
    if (split == 2 && kblocks < 8) break;
    for (uint32_t tm = 256; tm >= 16; tm -= 16) {
      const uint64_t ctas = wt * ((M + tm - 1) / tm) * split;
      const uint64_t rounds = (ctas + (uint64_t)sms - 1) / (uint64_t)sms;
      const double slab = 693.0 + 1.23 * tm;
      const double cost = (double)rounds * ((double)((kblocks + split - 1) / split) * slab + 8.0 * tm * split);
      if (cost < best_cost) {
        best_cost = cost;
        best = {tm, split};
      }
    }
  }
  return best;
}

cudaError_t fk_launch_gemm_tf32x3w(const float* a_hi, const float* a_lo, const float* w, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, uint32_t ldc, FkGemmTile tile, long long wait_cycles,
                                   int* err, cudaStream_t s) {
  using namespace fk::gw;
  if (M == 0 || N == 0) return cudaSuccess;
  const uint32_t tm = tile.tm;
  if (K == 0 || K % kBK != 0 || tm == 0 || tm % 16 != 0 || tm > kMaxTm || ldc < N ||
      (tile.split != 1 && tile.split != 2) || ((uintptr_t)a_hi | (uintptr_t)a_lo | (uintptr_t)w) & 15)
    return cudaErrorInvalidValue;
  uint32_t stages = kSmemBudget / stage_bytes(tm);
  if (stages > kMaxStages) stages = kMaxStages;
  if (stages < 2) return cudaErrorInvalidValue;
  size_t smem = 1024 + (size_t)stages * stage_bytes(tm) + 256;
  if (smem < kSmemFloor) smem = kSmemFloor;
  CUtensorMap ma_hi, ma_lo, mw;
  if (!make_map_w(&ma_hi, a_hi, M, K, tm) || !make_map_w(&ma_lo, a_lo, M, K, tm) || !make_map_w(&mw, w, N, K, kBW))
    return cudaErrorInvalidValue;
  cudaError_t e = fk_allow_smem(gemm_tf32x3w_kernel, smem);
  if (e != cudaSuccess) return e;
  const uint32_t wtiles = (N + kBW - 1) / kBW;
  if (wtiles > 65535) return cudaErrorInvalidValue;
  if (tile.split > 1) {
    // The halves add into C: zero it first (in the launch's stream order).
    e = cudaMemset2DAsync(c, (size_t)ldc * 4, 0, (size_t)N * 4, M, s);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((M + tm - 1) / tm, wtiles, tile.split);
  gemm_tf32x3w_kernel<<<grid, kThreads, smem, s>>>(ma_hi, ma_lo, mw, c, M, N, K, ldc, tm, stages,
                                                    wait_cycles > 0 ? wait_cycles : 4000000000LL, err);
  return cudaGetLastError();
}
