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
// tile in shared memory. The grid is persistent when the tiles outnumber
// the SMs: CTA j takes slabs [j U / G, (j + 1) U / G) of all U tiles' slabs
// in tile order, so every SM gets the same work and a tile lies in at most
// two CTAs; with fewer tiles, a tile a CTA or two K halves a tile. Parts
// of a tile add into C, which the launcher zeroes first; two additions
// onto zero give the same bits in either order, so the result does not
// depend on which part lands first.
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

// Where a CTA's work lies: `units` = tiles x slabs a tile, in tile order
// (a tile's slabs in K order, A tiles varying fastest so that the CTAs
// sharing a W tile run together and it crosses HBM once); CTA j takes units
// [j U / G, (j + 1) U / G). A piece is a run of one tile's slabs; a CTA's
// pieces are its tiles, the first and last possibly partial.
struct Work {
  uint32_t atiles, slabs;  // A tiles, slabs a tile
  uint64_t units;
};

__device__ __forceinline__ void unit_range(const Work& w, uint64_t& u0, uint64_t& u1) {
  u0 = (uint64_t)blockIdx.x * w.units / gridDim.x;
  u1 = (uint64_t)(blockIdx.x + 1) * w.units / gridDim.x;
}

__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32x3w_kernel(const __grid_constant__ CUtensorMap ta_hi, const __grid_constant__ CUtensorMap ta_lo,
                        const __grid_constant__ CUtensorMap tw, float* __restrict__ c, uint32_t M, uint32_t N,
                        uint32_t ldc, uint32_t tm, uint32_t stages, Work work, long long wait_cycles,
                        int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = stage_bytes(tm);
  // Barriers after the ring: full[S] (the slab's TMA bytes), split[S] (the
  // four split warps stored the W slab), empty[S] (the slab's MMAs done:
  // its shared and tensor memory free), accum (a piece's MMAs done: one
  // phase a piece), drained (the epilogue warps read the accumulator).
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + stages * sb);
  uint64_t* full = bars;
  uint64_t* split = bars + kMaxStages;
  uint64_t* empty = bars + 2 * kMaxStages;
  uint64_t* accum = bars + 3 * kMaxStages;
  uint64_t* drained = accum + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drained + 1);
  __shared__ int aborted;

  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t u0, u1;
  unit_range(work, u0, u1);
  const uint32_t S = work.slabs;

  if (threadIdx.x == 0) {
    aborted = 0;
    for (uint32_t s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&split[s]), 4);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    mbar_init(smem_u32(accum), 1);
    mbar_init(smem_u32(drained), 4);
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

  // The epilogue of one piece (of tile t), by warps 0..3 after its MMAs:
  // warp w reads TMEM lanes 32w.. of the accumulator (W rows n0 + those),
  // column j is A row m0 + j; a row of C's 32 consecutive columns a store
  // across the warp. A whole tile is stored; a piece of a tile (the tile's
  // two pieces lie in two CTAs) is added into C, which the launcher zeroed:
  // two additions onto zero, the same bits in either order. Then the
  // accumulator is free for the next piece. False when the wait ran out.
  auto epilogue = [&](uint32_t t, bool whole, uint32_t piece, uint32_t lane, uint32_t warp) -> bool {
    int done = 0;
    if (lane == 0) done = mbar_wait(smem_u32(accum), piece & 1, wait_cycles) ? 1 : 0;
    done = __shfl_sync(0xffffffffu, done, 0);
    if (!done) {
      if (lane == 0) record(err, GW_TIMEOUT_ACCUM);
      return false;
    }
    fence_after();
    if (!__shfl_sync(0xffffffffu, *reinterpret_cast<volatile int*>(&aborted), 0)) {
      const uint32_t m0 = (t % work.atiles) * tm, n = (t / work.atiles) * kBW + 32 * warp + lane;
      const bool live = n < N;
#pragma unroll 1
      for (uint32_t cc = 0; cc < tm; cc += 16) {
        uint32_t r[16];
        tmem_ld16(tmem + ((32 * warp) << 16) + cc, r);
#pragma unroll
        for (int j = 0; j < 16; ++j)
          if (live && m0 + cc + j < M) {
            float* at = c + (size_t)(m0 + cc + j) * ldc + n;
            if (whole)
              *at = __uint_as_float(r[j]);
            else
              atomicAdd(at, __uint_as_float(r[j]));
          }
      }
    }
    fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(drained));
    return true;
  };

  // The CTA's pieces in order: piece p covers slabs [kb, kb + n) of tile t.
  // Each role walks them with the same slab counter i (its ring stage and
  // phase), a tight loop over a piece's slabs inside.
  if (warp < 4) {
    // The W split, a row a thread (TMEM lane 32 warp + lane), then after
    // each piece its epilogue. Chunk j of row r sits at chunk
    // j ^ ((r / 2) % 4) of the row (64-byte swizzle).
    const uint32_t row = 32 * warp + lane;
    const uint32_t lane_addr = tmem + ((32 * warp) << 16);
    const uint32_t wr_off = 2 * tm * kRowBytes + row * kRowBytes;
    uint32_t i = 0, piece = 0;
    bool ok = true;
    for (uint64_t u = u0; u < u1 && ok; ++piece) {
      const uint32_t t = (uint32_t)(u / S), kb = (uint32_t)(u % S);
      const uint32_t n = (uint32_t)min((uint64_t)(S - kb), u1 - u);
      u += n;
      for (uint32_t j = 0; j < n; ++j, ++i) {
        const uint32_t s = i % stages, use = i / stages;
        // One lane waits and tells the others, so that the warp stays
        // together for its warp-wide TMEM stores.
        int ready = 0;
        if (lane == 0) ready = mbar_wait(smem_u32(&full[s]), use & 1, wait_cycles) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, ready, 0)) {
          if (lane == 0) record(err, GW_TIMEOUT_FULL);
          aborted = 1;
          ok = false;
          break;
        }
        const float4* wr = reinterpret_cast<const float4*>(smem + s * sb + wr_off);
        uint32_t hl[32];  // the high parts, then the low parts
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const float4 v = wr[c4 ^ ((row >> 1) & 3)];
          const float x[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            hl[4 * c4 + q] = tf32_rna(x[q]);
            hl[16 + 4 * c4 + q] = tf32_rna(__fsub_rn(x[q], __uint_as_float(hl[4 * c4 + q])));
          }
        }
        tmem_st32(lane_addr + kWCol0 + 32 * s, hl);
        tmem_wait_st();
        fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&split[s]));
      }
      if (ok) ok = epilogue(t, kb == 0 && n == S, piece, lane, warp);
    }
  } else if (warp == 4 && lane == 0) {
    // The producer. `issued` counts the slabs whose loads went out, so that
    // after an abort it can wait for the ones still in flight.
    uint32_t i = 0;
    bool ok = true;
    for (uint64_t u = u0; u < u1 && ok;) {
      const uint32_t t = (uint32_t)(u / S), kb = (uint32_t)(u % S);
      const uint32_t n = (uint32_t)min((uint64_t)(S - kb), u1 - u);
      const int m0 = (int)((t % work.atiles) * tm), n0 = (int)((t / work.atiles) * kBW);
      u += n;
      for (uint32_t j = 0; j < n; ++j, ++i) {
        const uint32_t s = i % stages, use = i / stages;
        if (use > 0 && !mbar_wait(smem_u32(&empty[s]), (use - 1) & 1, wait_cycles)) {
          record(err, GW_TIMEOUT_EMPTY);
          aborted = 1;
          ok = false;
          break;
        }
        if (*reinterpret_cast<volatile int*>(&aborted)) {
          ok = false;
          break;
        }
        uint8_t* st = smem + s * sb;
        const uint32_t bar = smem_u32(&full[s]);
        mbar_expect_tx(bar, sb);
        const int x = (int)((kb + j) * kBK);
        tma_load_2d(smem_u32(st), &ta_hi, x, m0, bar);
        tma_load_2d(smem_u32(st + tm * kRowBytes), &ta_lo, x, m0, bar);
        tma_load_2d(smem_u32(st + 2 * tm * kRowBytes), &tw, x, n0, bar);
      }
    }
    // Loads in flight finish before the CTA leaves (bounded).
    const uint32_t issued = i;
    const uint32_t first = issued > stages ? issued - stages : 0;
    for (uint32_t q = first; q < issued; ++q)
      if (!mbar_wait(smem_u32(&full[q % stages]), (q / stages) & 1, wait_cycles)) record(err, GW_TIMEOUT_FULL);
  } else if (warp == 5 && lane == 0) {
    // The MMA issuer: three TF32 products a K step of 8, 2 steps a slab; a
    // piece starts a fresh accumulator, once the epilogue has read the
    // previous piece's, and commits it after its last slab.
    const uint32_t idesc = tf32_idesc(tm, kBW);
    bool ok = true;
    uint32_t i = 0, piece = 0;
    for (uint64_t u = u0; u < u1 && ok; ++piece) {
      const uint32_t n = (uint32_t)min((uint64_t)(S - (uint32_t)(u % S)), u1 - u);
      u += n;
      if (piece > 0 && !mbar_wait(smem_u32(drained), (piece - 1) & 1, wait_cycles)) {
        record(err, GW_TIMEOUT_ACCUM);
        ok = false;
        break;
      }
      for (uint32_t j = 0; j < n; ++j, ++i) {
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
          const uint32_t acc = (j > 0 || kk > 0) ? 1u : 0u;
          mma_tf32_ts(tmem, w_hi + 8 * kk, sw64_desc(b_hi + off), idesc, acc);
          mma_tf32_ts(tmem, w_lo + 8 * kk, sw64_desc(b_hi + off), idesc, 1u);
          mma_tf32_ts(tmem, w_hi + 8 * kk, sw64_desc(b_lo + off), idesc, 1u);
        }
        mma_commit(smem_u32(&empty[s]));  // the slab's buffers are free once these finish
      }
      if (ok) mma_commit(smem_u32(accum));  // the piece's accumulator, once its MMAs finish
    }
    if (!ok) {
      // The MMAs issued so far finish before the CTA frees its TMEM (a
      // commit and a bounded wait for it); an epilogue waiting for it sees
      // `aborted` and stores nothing.
      aborted = 1;
      __threadfence_block();
      mma_commit(smem_u32(accum));
      mbar_wait(smem_u32(accum), (piece - 1) & 1, wait_cycles);
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

// The tile and grid for M x N x K on `sms` SMs: tm among 16, 32, ..., 256
// (tiles of 128 W rows x tm A rows) and G CTAs, one an SM at most: G =
// tiles (a tile a CTA), G = 2 tiles (each tile in two halves of its K
// slabs), or, with more tiles than SMs, G = sms (every CTA an equal share
// of the tiles' slabs, so a tile lies in at most two CTAs). The least
// modelled time: a CTA's slabs x a 16-float slab's cost (6 MMAs at about
// 138 + 0.117 tm SM cycles each, measured) + its pieces x an epilogue of
// 500 + 8 tm cycles.
FkGemmTile fk_gemm_tf32x3w_tile(uint32_t M, uint32_t N, uint32_t K, int sms) {
  FkGemmTile best = {256, 1};
  double best_cost = 1e300;
  const uint64_t wt = (N + fk::gw::kBW - 1) / fk::gw::kBW, S = K / fk::gw::kBK;
  for (uint32_t tm = 256; tm >= 16; tm -= 16) {
    const uint64_t tiles = wt * ((M + tm - 1) / tm);
    const double slab = 6.0 * (138.0 + 0.117 * tm), epi = 500.0 + 8.0 * tm;
    const uint64_t grids[3] = {tiles, 2 * tiles, (uint64_t)sms};
    for (int g = 0; g < 3; ++g) {
      const uint64_t G = grids[g];
      if (G == 0 || G > (uint64_t)sms || (g == 1 && S < 2) || (g == 2 && tiles <= (uint64_t)sms)) continue;
      const uint64_t per = (tiles * S + G - 1) / G;
      const double pieces = g == 0 ? 1.0 : g == 1 ? 1.0 : (double)(per + S - 1) / S + 1.0;
      const double cost = (double)per * slab + pieces * epi;
      if (cost < best_cost) {
        best_cost = cost;
        best = {tm, (uint32_t)G};
      }
    }
  }
  // More tiles than SMs at tm 16 still: a tile a CTA, in rounds.
  if (best_cost == 1e300) best = {16, (uint32_t)(wt * ((M + 15) / 16))};
  return best;
}

cudaError_t fk_launch_gemm_tf32x3w(const float* a_hi, const float* a_lo, const float* w, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, uint32_t ldc, FkGemmTile tile, long long wait_cycles,
                                   int* err, cudaStream_t s) {
  using namespace fk::gw;
  if (M == 0 || N == 0) return cudaSuccess;
  const uint32_t tm = tile.tm;
  if (K == 0 || K % kBK != 0 || tm == 0 || tm % 16 != 0 || tm > kMaxTm || ldc < N ||
      ((uintptr_t)a_hi | (uintptr_t)a_lo | (uintptr_t)w) & 15)
    return cudaErrorInvalidValue;
  Work work;
  work.atiles = (M + tm - 1) / tm;
  work.slabs = K / kBK;
  const uint64_t tiles = (uint64_t)((N + kBW - 1) / kBW) * work.atiles;
  work.units = tiles * work.slabs;
  // G CTAs: a tile each (G = tiles), two halves each (2 tiles), or an equal
  // share each with at most two CTAs a tile (G <= tiles). Anything else
  // could give a tile three pieces, whose additions would round in the
  // order they land.
  const uint64_t G = tile.grid;
  if (G == 0 || G > 0x7fffffffull || !(G <= tiles || G == 2 * tiles)) return cudaErrorInvalidValue;
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
  if (G != tiles) {
    // Pieces of tiles add into C: zero it first (in the launch's stream order).
    e = cudaMemset2DAsync(c, (size_t)ldc * 4, 0, (size_t)N * 4, M, s);
    if (e != cudaSuccess) return e;
  }
  gemm_tf32x3w_kernel<<<(uint32_t)G, kThreads, smem, s>>>(ma_hi, ma_lo, mw, c, M, N, ldc, tm, stages, work,
                                                           wait_cycles > 0 ? wait_cycles : 4000000000LL, err);
  return cudaGetLastError();
}
