/*
 * TEST INFRASTRUCTURE -- not part of the product.
 *
 * A CPU restatement of the FuryKernel reference's semantics for the decode
 * and prefill path, used only by tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / reference arm, as the checker and as the timed
 * CPU baseline. Nothing in furykernel_b200/ links, loads or calls it.
 *
 * Two layers:
 *   fko_*  what the reference's CPU target (src/FuryKernel/Cpu.hs) computes
 *          for the spec kernels of this path: binary32 arithmetic, no fused
 *          multiply-add, SIMD reductions pairwise neighbours first
 *          (Cpu.hs:469-505), threadgroup reductions in Reduce.hs order,
 *          transcendentals in binary64 rounded once (Cpu.hs:639-660).
 *          The CUDA kernels are written to compute these bits.
 *   fkr_*  the f64 evaluator (src/FuryKernel/Program/Eval.hs): each element's
 *          value in f64 and its binary32 error bound, the accuracy referee.
 *
 * Parity pins: the generator follows test/cpu/Cases.hs:885-892; the
 * reduction orders are pinned by the known answers of
 * test/Test/FuryKernel/InterpTest.hs:50-58 and ReduceTest.hs:46-59 (see
 * tests/test_oracle_pins.py). The reference's own CPU target cannot be built
 * here (no GHC, no rustc), so no bits come from running it.
 */
#ifndef FKO_H
#define FKO_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded inputs (test/cpu/Cases.hs:885-892) ---- */
uint64_t fko_random(uint64_t seed, uint64_t i);
void fko_fill_uniform(uint64_t seed, uint64_t n, double a, double b, float *out);
void fko_fill_normal(uint64_t seed, uint64_t n, double mu, double sigma, float *out);
void fko_fill_ints(uint64_t seed, uint64_t n, uint32_t bound, uint32_t *out);

/* ---- CPU-target arithmetic helpers ---- */
float fko_max(float a, float b);
float fko_min(float a, float b);
float fko_simd_sum(const float *v, int n);
float fko_simd_max(const float *v, int n);
float fko_tg_reduce_sum(const float *lanes, int threads);
float fko_tg_reduce_max(const float *lanes, int threads);
float fko_rsqrt(float v);
float fko_exp(float v);

/* ---- spec kernels (CPU-target semantics); threads = OpenMP threads ---- */
void fko_reduce_pass1(const float *x, uint64_t n, float *partials, int threads);
void fko_reduce_pass2(const float *partials, uint32_t count, float *y);
float fko_reduce_sum(const float *x, uint64_t n, int threads);

void fko_rmsnorm_rows(const float *x, uint32_t rows, uint32_t h, const float *gamma,
                      float eps, float factor, float *y, int threads);
void fko_softmax_rows(const float *x, uint32_t rows, uint32_t h, float *y, int threads);

void fko_gemm_tile(const float *a, uint32_t M, uint32_t K, const float *b, uint32_t N, float *c, int threads);
float fko_widen_bf16(uint16_t b);
uint16_t fko_narrow_bf16(float x);
float fko_widen_f16(uint16_t h);
uint16_t fko_narrow_f16(float x);
void fko_gemv_bf16(const uint16_t *w, uint32_t n, uint32_t k, const uint16_t *x, uint32_t m, uint32_t pack,
                   uint32_t split, uint16_t *y, int threads);
void fko_gemv(const float *w, uint32_t n, uint32_t k, const float *x, uint32_t m,
              uint32_t split, float *y, int threads);

void fko_rope_tables(double theta, uint32_t d, uint32_t rotated, uint32_t positions,
                     float *cos_t, float *sin_t);
void fko_rope(const float *x, uint32_t m, uint32_t heads, uint32_t d, uint32_t rotated,
              const uint32_t *pos, const float *cos_t, const float *sin_t, float *y);
void fko_kv_store_ring(const float *x, uint32_t m, uint32_t kv_heads, uint32_t d,
                       uint32_t length, const uint32_t *pos, const uint32_t *slot,
                       float *cache);
void fko_attend_split(const float *q, uint32_t m, uint32_t heads, uint32_t kv_heads,
                      uint32_t d, uint32_t length, const uint32_t *pos,
                      const uint32_t *slot, const float *kc, const float *vc,
                      float scale, uint32_t chunk, uint32_t warps, uint32_t max_splits,
                      float *part_m, float *part_l, float *part_acc, int threads);
void fko_attend_combine(uint32_t m, uint32_t heads, uint32_t d, const uint32_t *pos,
                        uint32_t chunk, uint32_t max_splits, const float *part_m,
                        const float *part_l, const float *part_acc, float *out);
void fko_silu_mul(const float *a, const float *b, uint64_t n, float *y);
float fko_gelu_tanh(float x);
void fko_route_topk(const float *x, uint32_t m, uint32_t n, uint32_t k, const float *scale, uint32_t *ids,
                    float *ws);
void fko_gemv_routed(const float *table, uint32_t entries, uint32_t n, uint32_t kk, const uint32_t *ids, uint32_t m,
                     uint32_t k, const float *x, uint32_t xw, uint32_t split, float *y, int threads);
void fko_gated_gelu(const float *x, uint64_t segments, uint32_t f, float *y);
void fko_combine_ranks_add(const float *r, const float *ws, const float *segs, uint32_t m, uint32_t k, uint32_t d,
                           float *y);
void fko_add(const float *a, const float *b, uint64_t n, float *y);
void fko_gather(const float *table, uint32_t width, const uint32_t *tokens, uint32_t m,
                float factor, float *y);
void fko_argmax(const float *x, uint32_t m, uint32_t n, uint32_t *ids);

/* ---- f64 evaluator with binary32 bounds (Program/Eval.hs) ---- */
double fkr_settle(double x, double e);
double fkr_widened(double e);
void fkr_input(const float *x, uint64_t n, double *v, double *b);
void fkr_linear(const float *w, uint32_t n, uint32_t k, const double *x, const double *xb,
                uint32_t m, double *y, double *yb, int threads);
void fkr_rmsnorm(const double *x, const double *xb, uint32_t m, uint32_t width,
                 uint32_t seg, const float *gamma, double eps, double factor, double *y,
                 double *yb);
void fkr_add(const double *a, const double *ab, const double *c, const double *cb,
             uint64_t n, double *y, double *yb);
void fkr_silu_mul(const double *a, const double *ab, const double *c, const double *cb,
                  uint64_t n, double *y, double *yb);
void fkr_rope(const double *x, const double *xb, uint32_t m, uint32_t width, uint32_t d,
              uint32_t rotated, double theta, const uint32_t *pos, double *y, double *yb);
void fkr_attend(const double *q, const double *qb, uint32_t m, uint32_t heads,
                uint32_t kv_heads, uint32_t d, uint32_t length, const uint32_t *pos,
                const uint32_t *slot, const double *kc, const double *kcb,
                const double *vc, const double *vcb, double scale, double *y, double *yb,
                int threads);
void fkr_gather(const float *table, uint32_t width, const uint32_t *tokens, uint32_t m,
                double factor, double *y, double *yb);
void fkr_argmax(const double *x, const double *xb, uint32_t m, uint32_t n, uint32_t *ids,
                int *decided);
void fkr_softmax(const double *x, const double *xb, uint32_t m, uint32_t n, double *y,
                 double *yb);
void fkr_sum(const float *x, uint64_t n, double *y, double *yb);

#ifdef __cplusplus
}
#endif
#endif
