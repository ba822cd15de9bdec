/*
 * furykernel-cuda: the C ABI of a B200-native (sm_100a) target for
 * FuryKernel programs.
 *
 * The reference's targets implement `Backend t` (src/FuryKernel/Backend.hs:
 * 156-162): `backendLower` turns checked kernels into one translation unit
 * plus a `LoweredKernel` launch table each (Backend.hs:203-228), and the
 * CPU target's generated functions take the parameter struct's bytes, then
 * the buffers in declaration order (src/FuryKernel/Cpu.hs:34-38, 271-278).
 * This library is the runtime half of a CUDA target: its kernels are
 * prebuilt for sm_100a, so `backendLower` for it resolves each checked
 * kernel to an entry of the table below by name and ABI hash, and the
 * engine launches entries with the same call convention the CPU target's
 * functions have: parameter bytes in C layout (src/FuryKernel/Abi.hs:
 * 113-133), then buffers in declaration order.
 *
 * Conventions:
 *  - Every entry point returns FKC_OK or an error code and never aborts; the
 *    message of the last failure on the calling thread is fkc_last_error().
 *  - A launch whose dimension lies outside its declared range is refused
 *    with the CPU target's exact text, "<kernel>: the dimension <d> is <v>,
 *    outside its range <r>." (src/FuryKernel/Emit/Rust.hs:94-104), and runs
 *    nothing. A launch whose grid comes to 0 threadgroups is skipped
 *    (Backend.hs:208-215).
 *  - Pointers to device memory are plain `void *` from fkc_buf_alloc (or
 *    any cudaMalloc'd memory of the context's device). No torch types cross
 *    this boundary.
 *  - One context per device; a context's entry points are not reentrant
 *    with each other, contexts are independent.
 */
#ifndef FURYKERNEL_CUDA_H
#define FURYKERNEL_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FKC_OK 0
#define FKC_ERR_ARGUMENT 1 /* refused: a dimension, an unknown kernel, an ABI mismatch */
#define FKC_ERR_CUDA 2
#define FKC_ERR_NCCL 3
#define FKC_ERR_STATE 4 /* e.g. capture not begun, no communicator */

typedef struct fkc_ctx fkc_ctx;
typedef struct fkc_graph fkc_graph;

/* The message of the calling thread's last failure ("" if none). Replaces
 * the reference's panics and `Left [Finding]` (src/FuryKernel/Finding.hs:
 * 11-17) at the C boundary. */
const char *fkc_last_error(void);
int fkc_version(void);

/* ---- device and context ------------------------------------------------ */
/* A context on one device: its compute stream, scratch and communicator.
 * The runtime half of `cpu :: Backend Cpu` (Cpu.hs:84-91), for a GPU. */
int fkc_open(int device, fkc_ctx **out);
int fkc_close(fkc_ctx *ctx);
/* The context's cudaStream_t, for callers that order their own work. */
int fkc_stream(fkc_ctx *ctx, void **stream);
/* Number of SMs of the context's device. */
int fkc_sm_count(fkc_ctx *ctx, int *sms);
/* Launch later kernels as programmatic dependents of the previous launch
 * (overlaps a launch's start with its predecessor's end). Default off. */
int fkc_set_pdl(fkc_ctx *ctx, int enabled);
/* The weight bytes each later weight-streaming GEMV launch (decode batches
 * of up to 4 rows) brings toward L2 by bulk prefetch, all its blocks
 * together, in the order its warps read them, before it waits for its
 * predecessor; 0 (the default): only the first lines of each warp's first
 * row. The blocks that become resident while the previous launch drains
 * start their weight stream early (measured on the 32-layer decode step:
 * 64 MiB takes about 2% off a batch-1 step, adds about 2% at batch 4). A
 * launch setting like fkc_set_pdl: captured into graphs as it stands. */
int fkc_set_prefetch(fkc_ctx *ctx, unsigned long long bytes);
/* A device range (16-byte aligned, whole 16 bytes) that later decode
 * attention launches (attend_split, attend_decode and their 16-bit and
 * paged forms) bring toward L2 by bulk prefetch, a slice a block, before
 * they wait for their predecessor: the next GEMV's weights, which then
 * stream from HBM while the latency-bound attention runs. p NULL or bytes 0:
 * none (the default). A launch setting like fkc_set_pdl. */
int fkc_set_l2_prefetch(fkc_ctx *ctx, const void *p, unsigned long long bytes);
/* The tile of later gemm_tf32x3w launches: tm A rows (a multiple of 16 up
 * to 256) against 128 W rows, and how the tiles' K slabs go to CTAs: parts
 * 1, a tile a CTA; 2, each tile in two halves; 0, an equal share of all
 * the slabs to each of min(tiles, SMs) CTAs (a tile in at most two). Parts
 * of a tile add into C (zeroed first). tm 0 (the default): each launch
 * picks its shape's tile. A launch setting like fkc_set_pdl, for tuning
 * and tests. */
int fkc_set_gemm_tile(fkc_ctx *ctx, unsigned tm, unsigned parts);
int fkc_sync(fkc_ctx *ctx);
/* Synchronizes, then reads and clears the context's device status word:
 * 0, or the code a kernel with bounded waits recorded when one ran out
 * (the tensor-core GEMM: 1 a stage never filled, 2 a stage never freed,
 * 3 the accumulator never completed; the tensor-parallel exchange: 10 + the
 * exchange buffer whose peers' rows or signal never came). */
int fkc_status(fkc_ctx *ctx, int *code);
/* The bound of each wait on another rank (the tensor-parallel exchange's),
 * in microseconds at the device's highest SM clock; 0 restores the default
 * of about 2 s. A wait that runs out records its status (fkc_status) and
 * the kernel goes on with what it has, so that the context stays usable.
 * Applies to launches made after the call (a captured graph keeps the
 * bound it was captured with). */
int fkc_set_wait_limit(fkc_ctx *ctx, unsigned microseconds);
/* Statistics of those waits, for finding what limits tensor-parallel steps:
 * while on, every block that waits on its peers adds the time it waited
 * (device clock, nanoseconds) and one wait to the context's totals, which
 * fkc_read_wait_stats synchronizes, returns and clears. Off by default (the
 * totals cost two atomics a block a wait); applies to launches made, or
 * graphs captured, after the call; not during a capture. */
int fkc_set_wait_stats(fkc_ctx *ctx, int enabled);
int fkc_read_wait_stats(fkc_ctx *ctx, unsigned long long *ns_waited, unsigned long long *waits);

/* ---- memory ------------------------------------------------------------- */
/* Buffers the engine binds to kernels (the reference's caller-owned slices,
 * Cpu.hs:34-38), owned here, freed by fkc_buf_free or fkc_close. */
int fkc_buf_alloc(fkc_ctx *ctx, size_t bytes, void **dptr);
int fkc_buf_free(fkc_ctx *ctx, void *dptr);
int fkc_buf_zero(fkc_ctx *ctx, void *dptr, size_t bytes);
/* Copies on the context's stream; download waits for it. */
int fkc_buf_upload(fkc_ctx *ctx, void *dptr, const void *host, size_t bytes);
int fkc_buf_download(fkc_ctx *ctx, void *host, const void *dptr, size_t bytes);
/* Pinned host memory for per-step inputs and outputs. */
int fkc_host_alloc(size_t bytes, void **host);
int fkc_host_free(void *host);
/* A persistent KV arena of Ring caches (src/FuryKernel/Program/Graph.hs:
 * 137-143): per layer, keys then values, each [slots, kv_heads, length,
 * head_dim] f32; *k_base and *v_base point at layer 0's, the layer stride
 * is slots * kv_heads * length * head_dim elements. */
int fkc_kv_arena(fkc_ctx *ctx, uint32_t layers, uint32_t slots, uint32_t kv_heads, uint32_t length,
                 uint32_t head_dim, void **k_base, void **v_base);
/* The same arena with elements of elem_bytes: 4 (f32) or 2 (bf16 or f16, the
 * element types the reference gives a cache, CacheBF16 and CacheF16,
 * Graph.hs:165-180; the *_kvbf16 and *_kvf16 table entries read and write
 * it). The layer stride is slots * kv_heads * length * head_dim elements of
 * that size. */
int fkc_kv_arena_elem(fkc_ctx *ctx, uint32_t layers, uint32_t slots, uint32_t kv_heads, uint32_t length,
                      uint32_t head_dim, uint32_t elem_bytes, void **k_base, void **v_base);
/* RoPE tables: the cosine and sine of p * theta^(-2i/d) for p < positions,
 * i < rotated, each rounded once from binary64 (the engine's tables that
 * Eval.hs:36-68 allows), [positions, rotated] f32 each. */
int fkc_rope_tables(fkc_ctx *ctx, double theta, uint32_t d, uint32_t rotated, uint32_t positions, void **cos_t,
                    void **sin_t);
/* Seeded synthetic inputs on the device: SplitMix's finaliser
 * (test/cpu/Cases.hs:885-892), normals by Box-Muller in binary64. */
int fkc_fill_normal(fkc_ctx *ctx, void *dptr, uint64_t n, uint64_t seed, double mu, double sigma);
int fkc_fill_uniform(fkc_ctx *ctx, void *dptr, uint64_t n, uint64_t seed, double a, double b);
/* fkc_fill_normal's values rounded to bf16 (nearest, ties to even: narrowBF16,
 * src/FuryKernel/Numerics.hs:41-48), n bf16 elements at dptr. */
int fkc_fill_normal_bf16(fkc_ctx *ctx, void *dptr, uint64_t n, uint64_t seed, double mu, double sigma);
/* The same values rounded to f16 (nearest, ties to even, gradual underflow:
 * narrowF16, src/FuryKernel/Numerics.hs:100-130), n f16 elements at dptr. */
int fkc_fill_normal_f16(fkc_ctx *ctx, void *dptr, uint64_t n, uint64_t seed, double mu, double sigma);

/* ---- the kernel table (LoweredKernel, Backend.hs:203-228) ----------------- */
int fkc_kernel_count(void);
/* Entry i: its name, the canonical ABI text the hash covers
 * (abiDescription, Abi.hs:136-159), the hash (FNV-1a 64, Abi.hs:259-262),
 * the spec's threads per threadgroup, and the parameter struct's size. */
int fkc_kernel_describe(int id, const char **name, const char **abi_description, uint64_t *abi_hash,
                        uint32_t *threads, uint32_t *params_size, uint32_t *buffers);
/* Resolves a checked kernel to an entry: same name and same ABI hash, else
 * refused with the ABI difference, as checkOverrides words it
 * (Abi.hs:172-190). */
int fkc_kernel_find(const char *name, uint64_t abi_hash, int *id);
/* 64-bit FNV-1a of bytes (fnv1a64, Abi.hs:259-262). */
uint64_t fkc_fnv1a64(const void *bytes, size_t n);

/* ---- launches (the generated kernel fn, Cpu.hs:242-315) ------------------- */
/* Runs entry `kernel` on the context's stream: params are the parameter
 * struct's bytes in C layout, bufs the buffers in declaration order. The
 * dimensions are checked against their ranges first. */
int fkc_launch(fkc_ctx *ctx, int kernel, const void *params, size_t params_len, void *const *bufs, int nbufs);

/* ---- the tree reduction without allocation --------------------------------- */
/* No counterpart in the reference. The sum of n f32 values at x into *y, with
 * exactly the bits of the reduce_groups + reduce_final launches, for callers
 * that cannot call cudaMalloc: code that runs inside a host whose allocator
 * owns every byte of device memory (a serving engine's fixed arena, a memory
 * pool with a hard budget), or on a path where an allocation's implicit
 * synchronization or failure is not acceptable. The caller passes the input
 * and the output; the scratch (the groups' partials, the final pass's sums
 * and counter) is a static device array of the library, about 1 MiB, which
 * every GPU that loads the library holds until the process exits; n may be
 * at most 2^26 (67,108,864), larger n is refused with FKC_ERR_ARGUMENT.
 * Runs on the current device, on `stream` (a cudaStream_t, NULL for the
 * default stream). The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress) with that device current: make that first
 * call before any stream capture. The address found is kept for the life of
 * the process: after a cudaDeviceReset of a device (which ends the memory
 * of its primary context) this entry point must not be called on that
 * device again in the same process. Every call on a device shares the one
 * array, which keeps the last call's contents; calls that overlap on the GPU
 * (on different streams without ordering between them) race and must not
 * be made. Nothing here calls cudaMalloc, cudaFree or any allocating
 * routine. */
int fkc_reduce_sum_f32_noalloc(const void *x, uint64_t n, void *y, void *stream);

/* ---- a plan's launch sequence as one CUDA graph ---------------------------- */
/* Launches between begin and end are captured, not run; replay runs them all
 * (the steps of src/FuryKernel/Program/Plan.hs:109-121, one launch each). */
int fkc_capture_begin(fkc_ctx *ctx);
int fkc_capture_end(fkc_ctx *ctx, fkc_graph **out);
int fkc_graph_launch(fkc_ctx *ctx, fkc_graph *g);
int fkc_graph_destroy(fkc_graph *g);
/* One engine step end to end: host inputs copied in, the graph replayed,
 * outputs copied back, the stream synchronized. */
int fkc_step(fkc_ctx *ctx, fkc_graph *g, const void *host_in, void *dev_in, size_t in_bytes, void *host_out,
             const void *dev_out, size_t out_bytes);
/* Device time of `iters` replays after `warmup`, by CUDA events on the
 * context's stream, in milliseconds (total). */
int fkc_time_graph(fkc_ctx *ctx, fkc_graph *g, int warmup, int iters, float *ms);

/* ---- tensor parallelism over NCCL ---------------------------------------- */
/* The reference has no collectives; a row-parallel projection's partial
 * outputs are summed across the ranks of one box over NVLink. */
int fkc_comm_unique_id(void *id128);
int fkc_comm_init(fkc_ctx *ctx, int nranks, int rank, const void *id128);
int fkc_allreduce_sum_f32(fkc_ctx *ctx, void *dptr, size_t count);
/* Each rank's `count` 32-bit words, gathered in rank order into recv
 * (nranks * count words): the vocabulary shards' greedy candidates. */
int fkc_allgather_u32(fkc_ctx *ctx, const void *send, void *recv, size_t count);
/* The context's rank and number of ranks (0 and 1 without a communicator). */
int fkc_comm_rank(fkc_ctx *ctx, int *rank, int *nranks);

/* ---- tensor parallelism over NVLink peer memory ---------------------------- */
/* The row-parallel projections' partial sums travel by stores into every
 * rank's exchange region, and the next GEMV's prologue adds them in rank
 * order: every rank gets the same bits, with no collective launch.
 * fkc_peer_alloc: this rank's region (bytes: the library's region size,
 * fkc_peer_region_bytes) and its 64-byte IPC handle; fkc_peer_open: a peer's
 * region from its handle; fkc_peer_set: every rank's region as this process
 * maps it, by rank (this rank's own included). The table's gemv_scatter,
 * gemv_reduce_rmsnorm(_silu), argmax_scatter and argmax_gather_pick use the
 * set; their waits are bounded and report through fkc_status. */
size_t fkc_peer_region_bytes(void);
int fkc_peer_alloc(fkc_ctx *ctx, size_t bytes, void **local, void *handle64);
int fkc_peer_open(fkc_ctx *ctx, const void *handle64, void **peer);
int fkc_peer_set(fkc_ctx *ctx, int world, int rank, void *const *regions);
int fkc_comm_destroy(fkc_ctx *ctx);

#ifdef __cplusplus
}
#endif
#endif
