// Host-side launchers of the furykernel-cuda kernels (internal to the
// library; the public boundary is include/furykernel_cuda.h).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <mutex>
#include <utility>

enum { FK_PRO_NONE = 0, FK_PRO_RMSNORM = 1, FK_PRO_SILU = 2, FK_PRO_REDUCE_RMSNORM = 3 };

// The element type of a model's weights or KV caches (fk_elem16.cuh).
enum FkElem { FK_F32 = 0, FK_BF16 = 1, FK_F16 = 2 };

// Tensor-parallel exchange over NVLink peer memory. Every rank owns one
// region, mapped into every other rank's process; by byte offset:
//   0    u32 flags[FK_XBUFS][FK_MAX_PEERS]  buffers 0, 1: the rows rank q has written here, all uses;
//                                            buffer 2: the epoch rank q last signalled into this region
//   128  u32 epoch[FK_XBUFS]                this rank's uses of each buffer so far
//   160  u32 counter[FK_XBUFS]              blocks of the running producer that have finished
//   256  f32 data[FK_XBUFS][FK_MAX_PEERS][FK_XSLOT]  rank q's partial rows, by buffer
// Buffers: 0 the attention output projection's partials, 1 the down
// projection's, 2 the vocabulary shards' greedy candidates.
constexpr int FK_MAX_PEERS = 8;
constexpr int FK_XBUFS = 3;
constexpr unsigned FK_XSLOT = 65536;  // floats of a rank's slot: 4 rows of 16384
constexpr size_t FK_XREGION = 256 + (size_t)FK_XBUFS * FK_MAX_PEERS * FK_XSLOT * 4;

struct FkPeers {
  char* base[FK_MAX_PEERS];  // each rank's region as this process maps it
  unsigned world, rank;
  long long wait_cycles;  // a wait's bound in SM clock cycles (the context's setting)
  unsigned long long* stats;  // null, or [ns waited, waits]: each block's wait added by its thread 0
};

struct FkGemv {
  const float* w;      // [n, k] out_in
  const float* x;      // [m, ldx]
  const float* gamma;  // RMSNorm prologue's gain, [k], or null
  const float* r;      // residual [m, ldr] added in the epilogue, or null
  float* y;            // [m, ldy]
  uint32_t n, k, m, split;
  uint32_t ldx, ldr, ldy;
  uint32_t up_off;  // SiLU-gate prologue: the up half's offset in a row of x
  int prologue;     // FK_PRO_*
  float eps, factor;
  bool pdl;        // launch as a programmatic dependent of the previous kernel
  bool silu_pair;  // rows interleave gate and up: y_i = silu(row 2i) * row 2i+1
  // Tensor parallelism over peer memory (streaming kernel only):
  bool scatter;    // write the partial rows into every rank's exchange buffer xbuf
  FkPeers peers;
  unsigned xbuf;
  float* xout;     // FK_PRO_REDUCE_RMSNORM: where block 0 stores the reduced rows
  int* err;        // the context's status word
  // Weight bytes (all blocks together) the streaming kernel brings toward
  // L2 by bulk prefetch before it waits for its predecessor
  // (fkc_set_prefetch). 0: only the first lines of each warp's first row.
  size_t prefetch;
};

struct FkAttend {
  const float* qkv;  // rows of [q | k | v]; q at column q_off, ld = ldq
  const float* cos_t;
  const float* sin_t;  // [positions, rotated]
  const uint32_t* pos;
  const uint32_t* slot;
  const float* kc;
  const float* vc;  // Ring caches [slots, kv_heads, length, d]
  float* part_m;    // [m, heads, max_splits]
  float* part_l;
  float* part_acc;  // [m, heads, max_splits, d]
  uint32_t m, heads, kv_heads, d, length, rotated, chunk, max_splits;
  uint32_t ldq, q_off;
  float scale;
  bool pdl;
  // A range the launch's blocks bring toward L2 (bulk prefetch, a slice a
  // block) before they wait for their predecessor: the next GEMV's weights,
  // which then stream while the attention runs (fkc_set_l2_prefetch). Null:
  // none.
  const void* pf;
  unsigned long long pf_bytes;
};

// The decode step's KV store and attention in one launch (rows in distinct
// slots): FkAttend plus where the new key and value sit in a qkv row and the
// caches to write.
struct FkAttendDecode {
  FkAttend a;
  uint32_t k_off, v_off;  // columns of k and v in a qkv row (ld = a.ldq)
  float* kc_w;
  float* vc_w;  // the caches a.kc / a.vc, written
};

struct FkKvStore {
  const float* qkv;  // k at column k_off, v at column v_off, ld = ldq
  const float* cos_t;
  const float* sin_t;
  const uint32_t* pos;
  const uint32_t* slot;
  float* kc;
  float* vc;
  uint32_t m, kv_heads, d, length, rotated;
  uint32_t ldq, k_off, v_off;
  bool pdl;
};

// A paged cache's block tables: row r's entries at table + r * table_len,
// each a block of the pool (< blocks) of block_size positions.
struct FkPaged {
  const uint32_t* table;
  uint32_t block_size, table_len, blocks;
};

struct FkCombine {
  const float* part_m;
  const float* part_l;
  const float* part_acc;
  const uint32_t* pos;
  float* out;  // [m, ldo]
  uint32_t m, heads, d, chunk, max_splits, ldo;
  bool pdl;
};

cudaError_t fk_launch_reduce_groups(const float* x, uint64_t n, float* partials, int sms, cudaStream_t s);
cudaError_t fk_launch_reduce_final(const float* partials, uint32_t count, float* chains, unsigned int* done,
                                   float* y, cudaStream_t s);
cudaError_t fk_launch_rmsnorm_rows(const float* x, const float* gamma, float* y, uint32_t rows, uint32_t h,
                                   float eps, float factor, cudaStream_t s);
cudaError_t fk_launch_softmax_rows(const float* x, float* y, uint32_t rows, uint32_t h, cudaStream_t s);
cudaError_t fk_launch_gemv(const FkGemv& g, cudaStream_t s);
bool fk_gemv_streams(const FkGemv& g);
cudaError_t fk_launch_gemv_stream(const FkGemv& g, int sms, cudaStream_t s);
bool fk_gemv_batches(const FkGemv& g);
cudaError_t fk_launch_gemv_batch(const FkGemv& g, int sms, cudaStream_t s);
cudaError_t fk_launch_kv_store(const FkKvStore& a, cudaStream_t s);
cudaError_t fk_launch_attend(const FkAttend& a, cudaStream_t s);
cudaError_t fk_launch_attend_decode(const FkAttendDecode& f, cudaStream_t s);
cudaError_t fk_launch_attend_prompt(const FkAttend& a, float* out, uint32_t ldo, uint32_t max_pos, cudaStream_t s);
cudaError_t fk_launch_combine(const FkCombine& a, cudaStream_t s);
cudaError_t fk_launch_gather(const float* table, uint32_t width, const uint32_t* tokens, uint32_t m, float factor,
                             float* y, bool pdl, cudaStream_t s);
cudaError_t fk_launch_argmax(const float* x, uint32_t m, uint32_t n, uint32_t ldx, uint32_t* ids, bool pdl,
                             cudaStream_t s);
cudaError_t fk_launch_rope(const float* x, uint32_t m, uint32_t heads, uint32_t d, uint32_t rotated, uint32_t ldx,
                           const uint32_t* pos, const float* cos_t, const float* sin_t, float* y, uint32_t ldy,
                           cudaStream_t s);
cudaError_t fk_launch_add(const float* a, const float* b, float* y, uint64_t n, cudaStream_t s);
cudaError_t fk_launch_silu_mul(const float* a, const float* b, float* y, uint64_t n, cudaStream_t s);
cudaError_t fk_launch_silu_pairs(const float* x, float* y, uint64_t n, cudaStream_t s);
cudaError_t fk_launch_gemv_bf16(const uint16_t* w, const uint16_t* x, uint16_t* y, uint32_t n, uint32_t k,
                                uint32_t m, uint32_t pack, uint32_t split, uint32_t ldx, uint32_t ldy, int sms,
                                bool pdl, cudaStream_t s);
cudaError_t fk_launch_argmax_pairs(const float* x, uint32_t m, uint32_t n, uint32_t ldx, uint32_t offset,
                                   uint32_t* pairs, const FkPeers* peers, bool pdl, cudaStream_t s);
cudaError_t fk_launch_argmax_pick(const uint32_t* pairs, uint32_t shards, uint32_t m, uint32_t* ids,
                                  const FkPeers* peers, int* err, bool pdl, cudaStream_t s);
cudaError_t fk_launch_advance(const uint32_t* ids, uint32_t* tokens, uint32_t* pos, uint32_t m, bool pdl,
                              cudaStream_t s);
cudaError_t fk_launch_split_tf32(const float* x, float* hi, float* lo, uint64_t n, cudaStream_t s);
cudaError_t fk_launch_gemm_tf32x3(const float* a_hi, const float* a_lo, const float* w_hi, const float* w_lo,
                                  float* c, uint32_t M, uint32_t N, uint32_t K, uint32_t ldc, int* err,
                                  cudaStream_t s);
// The 3xTF32 GEMM over f32 weights as they lie (W split inside the kernel):
// tiles of 128 W rows x tm A rows on `grid` CTAs, each an equal share of
// the tiles' K slabs (grid = tiles: a tile each; 2 tiles: two halves each;
// fewer than the tiles: at most two CTAs a tile, their parts added into
// C); fk_gemm_tf32x3w_tile picks one for a shape.
struct FkGemmTile {
  uint32_t tm;
  uint32_t grid;
};
FkGemmTile fk_gemm_tf32x3w_tile(uint32_t M, uint32_t N, uint32_t K, int sms);
cudaError_t fk_launch_gemm_tf32x3w(const float* a_hi, const float* a_lo, const float* w, float* c, uint32_t M,
                                   uint32_t N, uint32_t K, uint32_t ldc, FkGemmTile tile, long long wait_cycles,
                                   int* err, cudaStream_t s);
cudaError_t fk_launch_fill_normal(float* out, uint64_t n, uint64_t seed, double mu, double sigma, cudaStream_t s);
cudaError_t fk_launch_fill_uniform(float* out, uint64_t n, uint64_t seed, double a, double b, cudaStream_t s);
// 16-bit weights, bf16 or f16 (k_w16.cu): the f32 kernels' arithmetic over
// widened weights.
cudaError_t fk_launch_gemv_w16(const FkGemv& g, FkElem e, const uint16_t* w, const uint16_t* gamma, int sms,
                               cudaStream_t s);
bool fk_gemv_w16_batches(const FkGemv& g, const uint16_t* w);
cudaError_t fk_launch_gemv_batch_w16(const FkGemv& g, FkElem e, const uint16_t* w, const uint16_t* gamma, int sms,
                                     cudaStream_t s);
cudaError_t fk_launch_gather_w16(FkElem e, const uint16_t* table, uint32_t width, const uint32_t* tokens, uint32_t m,
                                 float factor, float* y, bool pdl, cudaStream_t s);
cudaError_t fk_launch_rmsnorm_rows_w16(FkElem e, const float* x, const uint16_t* gamma, float* y, uint32_t rows,
                                       uint32_t h, float eps, float factor, cudaStream_t s);
cudaError_t fk_launch_split_tf32_w16(FkElem e, const uint16_t* x, float* hi, float* lo, uint64_t n, cudaStream_t s);
cudaError_t fk_launch_fill_normal_w16(FkElem e, uint16_t* out, uint64_t n, uint64_t seed, double mu, double sigma,
                                      cudaStream_t s);
// 16-bit KV caches, bf16 or f16 (k_attend_kv16.cu): stores rounded to the
// cache's type, reads widened.
cudaError_t fk_launch_kv_store16(const FkKvStore& a, FkElem e, uint16_t* kc, uint16_t* vc, cudaStream_t s);
cudaError_t fk_launch_attend16(const FkAttend& a, FkElem e, const uint16_t* kc, const uint16_t* vc, cudaStream_t s);
cudaError_t fk_launch_attend_decode16(const FkAttend& a, FkElem e, uint32_t k_off, uint32_t v_off, uint16_t* kc,
                                      uint16_t* vc, cudaStream_t s);
cudaError_t fk_launch_attend_prompt16(const FkAttend& a, FkElem e, const uint16_t* kc, const uint16_t* vc, float* out,
                                      uint32_t ldo, uint32_t max_pos, cudaStream_t s);
// Paged KV caches (k_attend_paged.cu), f32, bf16 or f16 elements.
cudaError_t fk_launch_kv_store_paged(const FkKvStore& a, const FkPaged& pg, void* kc, void* vc, FkElem e,
                                     cudaStream_t s);
cudaError_t fk_launch_attend_paged(const FkAttend& a, const FkPaged& pg, const void* kc, const void* vc, FkElem e,
                                   cudaStream_t s);
cudaError_t fk_launch_attend_prompt_paged(const FkAttend& a, const FkPaged& pg, const void* kc, const void* vc,
                                          FkElem e, float* out, uint32_t ldo, uint32_t max_pos, cudaStream_t s);
// The KV store folded into the split attention (every table entry distinct).
cudaError_t fk_launch_attend_decode_paged(const FkAttend& a, const FkPaged& pg, void* kc, void* vc, FkElem e,
                                          uint32_t k_off, uint32_t v_off, cudaStream_t s);
// Routed experts (k_moe.cu); the experts' table f32, bf16 or f16.
// scale: the experts' scales of element type scale_elem, or null.
cudaError_t fk_launch_route_topk(const float* x, uint32_t m, uint32_t n, uint32_t k, uint32_t ldx,
                                 const void* scale, FkElem scale_elem, uint32_t* ids, float* ws, bool pdl,
                                 cudaStream_t s);
cudaError_t fk_launch_gemv_routed(const void* table, FkElem e, uint32_t entries, uint32_t n, uint32_t kk,
                                  const uint32_t* ids, uint32_t m, uint32_t k, const float* x, uint32_t ldx,
                                  bool per_rank, uint32_t split, float* y, uint32_t ldy, bool pdl, cudaStream_t s);
cudaError_t fk_launch_gated_gelu(const float* x, uint64_t segments, uint32_t f, float* y, bool pdl, cudaStream_t s);
cudaError_t fk_launch_combine_ranks_add(const float* r, const float* ws, const float* segs, uint32_t m, uint32_t k,
                                        uint32_t d, float* y, bool pdl, cudaStream_t s);
cudaError_t fk_launch_rope_tables(float* cos_t, float* sin_t, double theta, uint32_t d, uint32_t rotated,
                                  uint32_t positions, cudaStream_t s);

// Lets `func` take `bytes` of dynamic shared memory on the current device:
// cudaFuncSetAttribute is per device, so it is set once per (function,
// device) and raised when a launch asks for more.
template <typename F>
inline cudaError_t fk_allow_smem(F func, size_t bytes) {
  if (bytes <= 48 * 1024) return cudaSuccess;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, size_t> allowed;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  size_t& have = allowed[{reinterpret_cast<const void*>(func), dev}];
  if (bytes <= have) return cudaSuccess;
  e = cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess) have = bytes;
  return e;
}

// Launch helper for kernels that take part in programmatic dependent launch.
template <typename... KArgs, typename... Args>
static inline cudaError_t fk_launch_ex(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                                       bool pdl, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}
