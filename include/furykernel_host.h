/* furykernel-cuda's host side in C++ (libfurykernel_host.so): FuryKernel's
 * programs, its planner and the lowering of a plan to launches of the CUDA
 * target's kernel table, behind a C ABI.
 *
 * The reference computes these in Haskell before its target runs anything:
 * the program a model is written as (FuryKernel.Program.Graph, Build:
 * src/FuryKernel/Program/Graph.hs:299-360, Build.hs), the plan
 * (FuryKernel.Program.Plan.plan, src/FuryKernel/Program/Plan.hs), and a
 * backend's launches for the plan's steps (Backend.hs:203-228, the
 * LoweredKernel list a backend runs). A FuryKernel.Cuda module binds the
 * entries below where it would otherwise call its own planner on a program
 * the CUDA target runs; the launch list it gets back names entries of
 * libfurykernel_cuda.so's kernel table (fkc_kernel_find) with their
 * parameters and buffers, ready for fkc_launch or a captured graph.
 *
 * Errors: every entry returns 0 (FKH_OK) or a nonzero code, and writes the
 * refusal's text (the planner's or the lowering's words) into `err`
 * (NUL-terminated, truncated to `err_cap` bytes) when `err` is not NULL. */
#ifndef FURYKERNEL_HOST_H
#define FURYKERNEL_HOST_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FKH_API __attribute__((visibility("default")))
#else
#define FKH_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FKH_OK = 0,
  FKH_ERR_ARGUMENT = 1, /* a refusal: the text says why */
  FKH_ERR_SPACE = 2,    /* an output buffer too small: *len holds the size */
  FKH_ERR_INTERNAL = 3
};

/* The library's ABI version (this header's FKH_ABI_VERSION). */
#define FKH_ABI_VERSION 9
FKH_API int fkh_abi_version(void);

/* A Llama-shaped model (the shapes of the programs the engine plans). */
typedef struct {
  uint64_t d_model, heads, kv_heads, head_dim, ffn, vocab, layers;
  double theta, eps;
  uint64_t slots, length, positions;
  /* Element types: 0 f32, 1 bf16, 2 f16 (weights: Check.hs:105-111, bf16 the
   * reference's own; caches: CacheElem, Graph.hs:169-180). */
  int weights_type; /* every weight's */
  int cache_type;   /* the KV caches' */
  /* A paged cache (Paged, Graph.hs:144-152): a pool of `blocks` blocks of
   * `block_size` positions a layer, each row's block table of
   * ceil(positions / block_size) entries; block_size 0: the ring. */
  uint64_t blocks, block_size;
  /* Routed experts in place of the dense FFN: `experts` of ffn each, every
   * row its top_k (experts 0: the dense FFN). */
  uint64_t experts, top_k;
  /* Each chosen expert's weight times its scale, a weight [experts] after
   * the router (the route's expert scale, RouteSpec, Graph.hs:249-257). */
  int expert_scale;
} fkh_llama_shape;

/* The planner's options (PlanOptions, src/FuryKernel/Program/Plan.hs:243-268). */
typedef struct {
  int horizontal, gated, store_gelus;
  uint64_t sequence_rows;
} fkh_plan_options;

/* Texts: a program as the reference's renderProgram lays it out
 * (Graph.hs:445-528) and a plan as renderPlan does (Plan.hs:815-843). The
 * text is written to buf (NUL-terminated) when cap is large enough; *len is
 * its length without the NUL either way (FKH_ERR_SPACE when it did not fit).
 * which: 0 the embedding, 1 one decoder layer, 2 the head. */
FKH_API int fkh_llama_program_text(const fkh_llama_shape *shape, int which, char *buf, size_t cap, size_t *len, char *err,
                           size_t err_cap);
/* Parses a program text (the renderer's layout) and renders it back. */
FKH_API int fkh_program_roundtrip(const char *program_text, char *buf, size_t cap, size_t *len, char *err, size_t err_cap);
/* Parses a program text, plans it with the options and renders the plan. */
FKH_API int fkh_plan_text(const char *program_text, const fkh_plan_options *opts, char *buf, size_t cap, size_t *len,
                  char *err, size_t err_cap);

/* The Llama engine's decode step: the shape, the batch, this rank of the
 * tensor-parallel group, the choices, and the device addresses of every
 * buffer the launches bind (furykernel_b200/engine.py's Llama holds the
 * same fields). */
typedef struct {
  fkh_llama_shape full; /* the whole model; each rank holds heads, kv_heads, ffn and vocab / world */
  uint64_t batch, rank, world, sms, chunk;
  int gate_up_interleaved, peer_exchange, fuse_attention;
  /* the weight arena: per layer q k v o gate up down attn_norm mlp_norm,
   * then the whole embedding table and the final norm; the Ring KV arena's
   * key and value bases (fkc_kv_arena), or, for a paged cache, the keys' and
   * the values' tables of block addresses, [layers][blocks] u64 each (every
   * block an array of kv_heads * block_size * head_dim elements, wherever
   * it lies) */
  uint64_t arena, kbase, vbase;
  uint64_t cos_t, sin_t;           /* fkc_rope_tables */
  uint64_t tokens, pos, slot;      /* [batch] u32 each */
  uint64_t x, x1, qkv, att, gu, act, logits, out_ids;
  uint64_t partial, pairs, pairs_all; /* NCCL tensor parallelism */
  uint64_t part[3];                   /* split attention's partials */
  /* A committed selection's split-K for GEMV shapes: nsplits triples
   * (n, k, split), the same split at every batch; NULL for the default. */
  const uint32_t *splits;
  size_t nsplits;
  /* Routed experts: the normed row [batch, d], the router's logits
   * [batch, experts], the route's ids (u32) and weights [batch, top_k], the
   * experts' gate/up rows [batch, top_k * 2 ffn], their gate
   * [batch, top_k * ffn], their outputs [batch, top_k * d]. */
  uint64_t mlp_in, router_logits, route_ids, route_weights, experts_gu, experts_act, experts_out;
  /* The layer's plan options (PlanOptions, Plan.hs:243-268): a route in a
   * step of its own (optGated), gelus stored by their own step
   * (optStoreGelus). */
  int gated, store_gelus;
} fkh_llama_desc;

/* A launch list: kernel names of the CUDA target's table, parameters by
 * name (numbers as double: every table parameter is an integer below 2^53
 * or an f32), buffers as device addresses in declaration order. Two
 * pseudo-kernels stand for NCCL calls: "__allreduce__" (count; the buffer
 * summed in place) and "__allgather__" (count; send, receive). */
typedef struct fkh_launches fkh_launches;

FKH_API int fkh_llama_launches(const fkh_llama_desc *desc, fkh_launches **out, char *err, size_t err_cap);
FKH_API size_t fkh_launches_count(const fkh_launches *l);
FKH_API const char *fkh_launch_kernel(const fkh_launches *l, size_t i);
FKH_API size_t fkh_launch_param_count(const fkh_launches *l, size_t i);
FKH_API const char *fkh_launch_param_name(const fkh_launches *l, size_t i, size_t j);
FKH_API double fkh_launch_param_value(const fkh_launches *l, size_t i, size_t j);
FKH_API size_t fkh_launch_buf_count(const fkh_launches *l, size_t i);
FKH_API uint64_t fkh_launch_buf(const fkh_launches *l, size_t i, size_t j);
FKH_API void fkh_launches_free(fkh_launches *l);

/* The prompt prefill in front of a decode step: every prompt row through
 * the layers at once, the linears as tcgen05 3xTF32 GEMM tiles
 * (gemm_tf32x3, the reference's gemmTile: src/FuryKernel/Tile.hs:76-157),
 * each row's keys and values stored in the Ring caches
 * (furykernel_b200/prefill.py holds the same fields). */
typedef struct {
  uint64_t rows;      /* the most rows a launch list takes */
  uint64_t chunk;     /* attention positions a split covers */
  uint64_t positions; /* the bound of the positions a prefill stores */
  int one_slot;       /* every run's rows in one slot: the query-tiled attend_prompt */
  uint64_t w_hi, w_lo; /* the weights' TF32 halves, laid out as the weight arena */
  uint64_t tokens, pos, slot; /* [rows] u32 each */
  uint64_t x, a, a_hi, a_lo, qkv, att, tmp, x1, gu, act;
  uint64_t part[3];
  /* Routed experts over the rows (the decode step's kernels): the router's
   * logits [rows, experts], the route's ids (u32) and weights [rows, top_k],
   * the experts' gate/up rows [rows, top_k * 2 ffn], their gate
   * [rows, top_k * ffn], their outputs [rows, top_k * d]. */
  uint64_t router_logits, route_ids, route_weights, experts_gu, experts_act, experts_out;
} fkh_prefill_desc;

/* The prefill of m rows (1..rows); `desc` is the decode step's, whose own
 * launches are the templates of the gather, the KV stores and the attention. */
FKH_API int fkh_llama_prefill_launches(const fkh_llama_desc *desc, const fkh_prefill_desc *prefill, uint64_t m,
                                       fkh_launches **out, char *err, size_t err_cap);

/* Split-K for a GEMV of n rows of k on `sms` SMs (the chunked kernel's). */
FKH_API uint64_t fkh_split_for(uint64_t n_rows, uint64_t k, uint64_t sms);

/* ---- variant spaces and selections ---------------------------------------
 * JSON as the reference writes it (src/FuryKernel/Json.hs): parsed and
 * rendered back, or the parse error and its character. */
FKH_API int fkh_json_roundtrip(const char *text, char *buf, size_t cap, size_t *len, char *err, size_t err_cap);
/* A selection (src/FuryKernel/Selection.hs:8-36, the format, version 1)
 * parsed and rendered back, or what is wrong with its format. */
FKH_API int fkh_selection_roundtrip(const char *text, char *buf, size_t cap, size_t *len, char *err,
                                    size_t err_cap);
/* A variant space given as JSON ({"family", "axes": [{"name", "prefix",
 * "values", "order"}], "classes": [{dimension: value}], "batch"}): what
 * checkSpace refuses (Variant.hs), one a line; an axis key read back (or
 * parseAxisKey's message); every variant's name, each marked where it does
 * not read back. */
FKH_API int fkh_space_check(const char *space_json, char *buf, size_t cap, size_t *len, char *err, size_t err_cap);
FKH_API int fkh_space_parse_key(const char *space_json, const char *key, char *buf, size_t cap, size_t *len,
                                char *err, size_t err_cap);
FKH_API int fkh_space_names(const char *space_json, char *buf, size_t cap, size_t *len, char *err, size_t err_cap);
/* splitJoin (Variant.hs): a name split at the first _x_ whose right side is
 * right_prefix and digits -- or, where right_prefix is "", a plan step's name
 * (isStepName, Program/Plan.hs:162-165) -- as "left\nright"; empty where
 * none is. */
FKH_API int fkh_split_join(const char *name, const char *right_prefix, char *buf, size_t cap, size_t *len, char *err,
                           size_t err_cap);
/* This target's GEMV family (classes n_k_m, m the batch; one axis, the
 * split-K s, which orders the reduction): what pruning makes of a point
 * (kind: 0 kept, 1 illegal, 2 indivisible, 3 too few work units; the
 * launch's work units; the kernel identity the selection records as its IR
 * hash; the reasons); a selection of the given splits rendered; a
 * selection validated against classes (n, k, m triples) on a GPU of `cores`
 * SMs, giving each class's split, or every problem, one a line. */
FKH_API int fkh_gemv_consider(uint32_t n, uint32_t k, uint32_t m, uint32_t split, uint32_t cores, int *kind,
                              uint64_t *groups, uint64_t *hash, char *reasons, size_t reasons_cap);
FKH_API int fkh_gemv_selection_render(const uint32_t *classes, const uint32_t *splits, size_t count, uint32_t cores,
                                      char *buf, size_t cap, size_t *len, char *err, size_t err_cap);
FKH_API int fkh_gemv_selection_validate(const char *text, const uint32_t *classes, size_t count, uint32_t cores,
                                        uint32_t *splits, char *err, size_t err_cap);

#ifdef __cplusplus
}
#endif
#endif
