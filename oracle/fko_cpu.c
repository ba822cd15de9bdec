/*
 * TEST INFRASTRUCTURE -- not part of the product (see fko.h).
 *
 * What the reference's CPU target computes for the spec kernels of the
 * decode/prefill path. Built with -ffp-contract=off and without fast math,
 * so that every operation below is one binary32 rounding, as the CPU
 * target's Rust is (src/FuryKernel/Cpu.hs:1-40). Each function names the
 * reference lines it follows.
 */
#include "fko.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* Seeded inputs: SplitMix's finaliser over seed * golden + i, i from 1      */
/* (test/cpu/Cases.hs:885-892).                                              */

static inline uint64_t fko_mix(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

uint64_t fko_random(uint64_t seed, uint64_t i) {
  return fko_mix(seed * 0x9E3779B97F4A7C15ULL + i);
}

/* U(a, b) from the top 24 bits of element j's word (word j + 1). */
void fko_fill_uniform(uint64_t seed, uint64_t n, double a, double b, float *out) {
#pragma omp parallel for schedule(static)
  for (int64_t j = 0; j < (int64_t)n; ++j) {
    uint64_t w = fko_random(seed, (uint64_t)j + 1);
    out[j] = (float)(a + (b - a) * ((double)(w >> 40) * 0x1p-24));
  }
}

/* N(mu, sigma) by Box-Muller on consecutive pairs of words: elements 2p and
 * 2p+1 from words 2p+1 and 2p+2, u1 in (0, 1], u2 in [0, 1), in binary64,
 * rounded once to binary32. */
void fko_fill_normal(uint64_t seed, uint64_t n, double mu, double sigma, float *out) {
  const int64_t pairs = (int64_t)((n + 1) / 2);
#pragma omp parallel for schedule(static)
  for (int64_t p = 0; p < pairs; ++p) {
    uint64_t w1 = fko_random(seed, 2 * (uint64_t)p + 1);
    uint64_t w2 = fko_random(seed, 2 * (uint64_t)p + 2);
    double u1 = ((double)(w1 >> 11) + 1.0) * 0x1p-53;
    double u2 = (double)(w2 >> 11) * 0x1p-53;
    double r = sqrt(-2.0 * log(u1));
    double t = 6.283185307179586 * u2;
    out[2 * p] = (float)(mu + sigma * (r * cos(t)));
    if (2 * p + 1 < (int64_t)n) out[2 * p + 1] = (float)(mu + sigma * (r * sin(t)));
  }
}

/* U[0, bound) from the top 32 bits: floor(hi32 * bound / 2^32). */
void fko_fill_ints(uint64_t seed, uint64_t n, uint32_t bound, uint32_t *out) {
  for (uint64_t j = 0; j < n; ++j) {
    uint64_t w = fko_random(seed, j + 1);
    out[j] = (uint32_t)(((w >> 32) * (uint64_t)bound) >> 32);
  }
}

/* ------------------------------------------------------------------------ */
/* Arithmetic of the CPU target                                              */

static inline uint32_t bits_of(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
}
static inline float of_bits(uint32_t u) {
  float f;
  memcpy(&f, &u, 4);
  return f;
}

/* IEEE 754-2019 maximumNumber / minimumNumber (Cpu.hs:157-183). */
float fko_max(float a, float b) {
  if (isnan(a)) return isnan(b) ? of_bits(0x7fc00000u) : b;
  if (isnan(b) || a > b) return a;
  if (b > a) return b;
  return of_bits(bits_of(a) & bits_of(b));
}

float fko_min(float a, float b) {
  if (isnan(a)) return isnan(b) ? of_bits(0x7fc00000u) : b;
  if (isnan(b) || a < b) return a;
  if (b < a) return b;
  return of_bits(bits_of(a) | bits_of(b));
}

/* A SIMD group's reduction: pairwise, neighbours first; an odd one out moves
 * up unchanged (Cpu.hs:469-505, IR.hs:277-289). */
float fko_simd_sum(const float *v, int n) {
  float t[64];
  memcpy(t, v, (size_t)n * sizeof(float));
  while (n > 1) {
    for (int k = 0; k < n / 2; ++k) t[k] = t[2 * k] + t[2 * k + 1];
    if (n % 2 == 1) t[n / 2] = t[n - 1];
    n = (n + 1) / 2;
  }
  return t[0];
}

float fko_simd_max(const float *v, int n) {
  float t[64];
  memcpy(t, v, (size_t)n * sizeof(float));
  while (n > 1) {
    for (int k = 0; k < n / 2; ++k) t[k] = fko_max(t[2 * k], t[2 * k + 1]);
    if (n % 2 == 1) t[n / 2] = t[n - 1];
    n = (n + 1) / 2;
  }
  return t[0];
}

/* tgReduce (src/FuryKernel/Reduce.hs:59-85) at SIMD width 32: each SIMD
 * group's lanes reduced into its slot; lane l of the first group combines
 * slots l, l + 32, ... from the identity; the first group's lanes reduced
 * once more. */
static float tg_reduce(const float *lanes, int threads, int is_max) {
  float slots[32];
  const int groups = (threads + 31) / 32;
  for (int g = 0; g < groups; ++g) {
    int n = threads - 32 * g < 32 ? threads - 32 * g : 32;
    slots[g] = is_max ? fko_simd_max(lanes + 32 * g, n) : fko_simd_sum(lanes + 32 * g, n);
  }
  const int first = threads < 32 ? threads : 32;
  float acc[32];
  for (int l = 0; l < first; ++l) {
    float a = is_max ? -INFINITY : -0.0f;
    for (int k = l; k < groups; k += 32) a = is_max ? fko_max(a, slots[k]) : a + slots[k];
    acc[l] = a;
  }
  return is_max ? fko_simd_max(acc, first) : fko_simd_sum(acc, first);
}

float fko_tg_reduce_sum(const float *lanes, int threads) { return tg_reduce(lanes, threads, 0); }
float fko_tg_reduce_max(const float *lanes, int threads) { return tg_reduce(lanes, threads, 1); }

/* Rsqrt and Exp in binary64, rounded once to binary32 (Cpu.hs:639-660). */
float fko_rsqrt(float v) { return (float)(1.0 / sqrt((double)v)); }
float fko_exp(float v) { return (float)exp((double)v); }

/* ------------------------------------------------------------------------ */
/* Threadgroup tree reduction: the config-1 spec kernel. 256-lane groups    */
/* halve through threadgroup memory with a barrier per step; lanes past n   */
/* hold -0, the identity of addition. Pass 2 is one group whose lane l adds */
/* partials l, l + 256, ... from -0, then halves the same way.              */

static float halve256(float *t) {
  for (int s = 128; s > 0; s >>= 1)
    for (int i = 0; i < s; ++i) t[i] = t[i] + t[i + s];
  return t[0];
}

void fko_reduce_pass1(const float *x, uint64_t n, float *partials, int threads) {
  const int64_t groups = (int64_t)((n + 255) / 256);
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t g = 0; g < groups; ++g) {
    float t[256];
    for (int i = 0; i < 256; ++i) {
      uint64_t at = (uint64_t)g * 256 + (uint64_t)i;
      t[i] = at < n ? x[at] : -0.0f;
    }
    partials[g] = halve256(t);
  }
}

void fko_reduce_pass2(const float *partials, uint32_t count, float *y) {
  float t[256];
  for (uint32_t l = 0; l < 256; ++l) {
    float acc = -0.0f;
    for (uint32_t i = l; i < count; i += 256) acc = acc + partials[i];
    t[l] = acc;
  }
  y[0] = halve256(t);
}

float fko_reduce_sum(const float *x, uint64_t n, int threads) {
  uint32_t groups = (uint32_t)((n + 255) / 256);
  float *p = (float *)malloc((size_t)groups * sizeof(float));
  float y;
  fko_reduce_pass1(x, n, p, threads);
  fko_reduce_pass2(p, groups, &y);
  free(p);
  return y;
}

/* ------------------------------------------------------------------------ */
/* Row kernels, one 256-lane group per row, packs of four f32 (16 bytes, the */
/* CPU target's LaneLoadMax, Cpu.hs:71-78): lane t takes packs t, t + 256,  */
/* ... in order.                                                            */

/* RMSNorm: the pattern of test/Test/FuryKernel/Kernels.hs:53-75 over f32:
 * acc += v*v per element, tgReduceSum, scale = rsqrt(total / h + eps),
 * y = x * scale * gamma (* factor when it is not 1). */
void fko_rmsnorm_rows(const float *x, uint32_t rows, uint32_t h, const float *gamma,
                      float eps, float factor, float *y, int threads) {
  const uint32_t packs = h / 4;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t r = 0; r < (int64_t)rows; ++r) {
    const float *xr = x + (size_t)r * h;
    float lanes[256];
    for (uint32_t t = 0; t < 256; ++t) {
      float acc = 0.0f;
      for (uint32_t j = t; j < packs; j += 256)
        for (int e = 0; e < 4; ++e) {
          float v = xr[4 * j + e];
          acc = acc + v * v;
        }
      lanes[t] = acc;
    }
    float total = fko_tg_reduce_sum(lanes, 256);
    float scale = fko_rsqrt(total / (float)h + eps);
    float *yr = y + (size_t)r * h;
    for (uint32_t j = 0; j < h; ++j) {
      float v = xr[j] * scale;
      if (gamma) v = v * gamma[j];
      if (factor != 1.0f) v = v * factor;
      yr[j] = v;
    }
  }
}

/* Softmax, max-subtracted: tgReduceMax of the lanes' maxima
 * (Reduce.hs:48-51), exp in binary64 of x - max, tgReduceSum of the lanes'
 * sums, each e over the total. */
void fko_softmax_rows(const float *x, uint32_t rows, uint32_t h, float *y, int threads) {
  const uint32_t packs = h / 4;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t r = 0; r < (int64_t)rows; ++r) {
    const float *xr = x + (size_t)r * h;
    float *yr = y + (size_t)r * h;
    float lanes[256];
    for (uint32_t t = 0; t < 256; ++t) {
      float mx = -INFINITY;
      for (uint32_t j = t; j < packs; j += 256)
        for (int e = 0; e < 4; ++e) mx = fko_max(mx, xr[4 * j + e]);
      lanes[t] = mx;
    }
    float top = fko_tg_reduce_max(lanes, 256);
    for (uint32_t t = 0; t < 256; ++t) {
      float acc = 0.0f;
      for (uint32_t j = t; j < packs; j += 256)
        for (int e = 0; e < 4; ++e) {
          float ev = fko_exp(xr[4 * j + e] - top);
          yr[4 * j + e] = ev;
          acc = acc + ev;
        }
      lanes[t] = acc;
    }
    float total = fko_tg_reduce_sum(lanes, 256);
    for (uint32_t j = 0; j < h; ++j) yr[j] = yr[j] / total;
  }
}

/* ------------------------------------------------------------------------ */
/* GEMV y = W x, W [n, k] out_in, x [m, k], y [m, n]: the per-row order of   */
/* test/Test/FuryKernel/Gemv.hs:9-26 at pack width 4 and split s. Virtual    */
/* lane v = q * 32 + l visits packs v, v + 32 s, ...; a pack adds            */
/* ((x0 w0 + x1 w1) + (x2 w2 + x3 w3)) to the lane's chain, which starts at  */
/* 0; the lanes are summed pairwise; the splits' partials in split order.    */

void fko_gemv(const float *w, uint32_t n, uint32_t k, const float *x, uint32_t m,
              uint32_t split, float *y, int threads) {
  const uint32_t packs = k / 4;
  const uint32_t stride = 32 * split;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t o = 0; o < (int64_t)n; ++o) {
    const float *wr = w + (size_t)o * k;
    for (uint32_t i = 0; i < m; ++i) {
      const float *xr = x + (size_t)i * k;
      float total = 0.0f;
      for (uint32_t q = 0; q < split; ++q) {
        float lanes[32];
        for (uint32_t l = 0; l < 32; ++l) {
          float acc = 0.0f;
          for (uint32_t j = q * 32 + l; j < packs; j += stride) {
            const float *xp = xr + 4 * (size_t)j;
            const float *wp = wr + 4 * (size_t)j;
            float c = (xp[0] * wp[0] + xp[1] * wp[1]) + (xp[2] * wp[2] + xp[3] * wp[3]);
            acc = acc + c;
          }
          lanes[l] = acc;
        }
        float part = fko_simd_sum(lanes, 32);
        total = q == 0 ? part : total + part;
      }
      y[(size_t)i * n + (size_t)o] = total;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* gemmTile (src/FuryKernel/Tile.hs:76-157) as the CPU target runs it:      */
/* C = A B^T, an element's sum over k in order, 8 at a time through the     */
/* fragment product (Cpu.hs:549-560: acc = acc + a * b, each product and    */
/* sum rounded), from 0 -- so a sequential binary32 dot over k.             */

void fko_gemm_tile(const float *a, uint32_t M, uint32_t K, const float *b, uint32_t N, float *c, int threads) {
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t i = 0; i < (int64_t)M; ++i) {
    const float *ar = a + (size_t)i * K;
    for (uint32_t j = 0; j < N; ++j) {
      const float *br = b + (size_t)j * K;
      float acc = 0.0f;
      for (uint32_t k = 0; k < K; ++k) acc = acc + ar[k] * br[k];
      c[(size_t)i * N + j] = acc;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* The bf16 GEMV family itself (test/Test/FuryKernel/Gemv.hs:118-191): x, W  */
/* and y bf16, widened exactly to binary32 (a NaN quieted, Numerics.hs:      */
/* 33-38); pack width p (4, 8, 16): a lane's pack goes four elements to a    */
/* chain, chain c adding ((x0 w0 + x1 w1) + (x2 w2 + x3 w3)) from 0; a       */
/* lane's chains added left to right (inOrder, Gemv.hs:214-217), then the    */
/* SIMD sum; the splits' partials in split order; y narrowed to bf16 by     */
/* round-to-nearest-even (narrowBF16, Numerics.hs:41-48).                    */

float fko_widen_bf16(uint16_t b) {
  uint32_t w = (uint32_t)b << 16;
  if ((w & 0x7F800000u) == 0x7F800000u && (w & 0x007FFFFFu)) w |= 0x00400000u;
  float f;
  memcpy(&f, &w, 4);
  return f;
}

uint16_t fko_narrow_bf16(float x) {
  uint32_t w;
  memcpy(&w, &x, 4);
  if (x != x) return (uint16_t)((w >> 16) | 0x0040u);
  const uint32_t lsb = (w >> 16) & 1u;
  return (uint16_t)((w + 0x7FFFu + lsb) >> 16);
}

/* binary16 <-> binary32. Widening is exact; a NaN comes out quiet, its sign */
/* and payload kept (widenF16, Numerics.hs:51-66). Narrowing rounds to       */
/* nearest, ties to even, with gradual underflow; past the largest finite    */
/* value by half an ulp or more to infinity; a NaN keeps its sign and top 9  */
/* payload bits and comes out quiet (narrowF16, Numerics.hs:100-130).        */

float fko_widen_f16(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  uint32_t m = h & 0x3FFu, w;
  if (e == 0x1F)
    w = m ? 0x7FC00000u | (m << 13) : 0x7F800000u;
  else if (e)
    w = ((e + 112u) << 23) | (m << 13);
  else if (!m)
    w = 0;
  else {
    /* m * 2^-24 = (m << s) * 2^(-24 - s): with the leading 1 at bit 10 that */
    /* is 1.f * 2^(-14 - s), biased exponent 113 - s.                         */
    uint32_t s = 0;
    while (!(m & 0x400u)) {
      m <<= 1;
      ++s;
    }
    w = ((113u - s) << 23) | ((m & 0x3FFu) << 13);
  }
  w |= sign;
  float f;
  memcpy(&f, &w, 4);
  return f;
}

/* kept rounded up when what was shifted off is past half, or half and kept */
/* odd.                                                                     */
static uint32_t round_even(uint32_t kept, uint32_t rest, uint32_t half) {
  return rest > half || (rest == half && (kept & 1u)) ? kept + 1u : kept;
}

uint16_t fko_narrow_f16(float x) {
  uint32_t w;
  memcpy(&w, &x, 4);
  const uint16_t sign = (uint16_t)((w >> 16) & 0x8000u);
  const int e = (int)((w >> 23) & 0xFFu);
  const uint32_t m = w & 0x7FFFFFu;
  if (e == 0xFF) return (uint16_t)(sign | (m ? 0x7E00u | (m >> 13) : 0x7C00u));
  const int unbiased = e - 127;
  if (unbiased >= 16) return (uint16_t)(sign | 0x7C00u);
  if (unbiased >= -14) /* a carry out of the mantissa moves the exponent, up to infinity */
    return (uint16_t)(sign | round_even(((uint32_t)(unbiased + 15) << 10) | (m >> 13), m & 0x1FFFu, 0x1000u));
  /* Subnormal or zero: in units of 2^-24 the value is (1.m) * 2^(unbiased + 24). */
  const int shift = -(unbiased + 1);
  if (e == 0 || shift > 24) return sign;
  const uint32_t full = m | 0x800000u;
  return (uint16_t)(sign | round_even(full >> shift, full & ((1u << shift) - 1u), 1u << (shift - 1)));
}

void fko_gemv_bf16(const uint16_t *w, uint32_t n, uint32_t k, const uint16_t *x, uint32_t m, uint32_t pack,
                   uint32_t split, uint16_t *y, int threads) {
  const uint32_t packs = k / pack, chains = pack / 4;
  const uint32_t stride = 32 * split;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t o = 0; o < (int64_t)n; ++o) {
    const uint16_t *wr = w + (size_t)o * k;
    for (uint32_t i = 0; i < m; ++i) {
      const uint16_t *xr = x + (size_t)i * k;
      float total = 0.0f;
      for (uint32_t q = 0; q < split; ++q) {
        float lanes[32];
        for (uint32_t l = 0; l < 32; ++l) {
          float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
          for (uint32_t j = q * 32 + l; j < packs; j += stride)
            for (uint32_t c = 0; c < chains; ++c) {
              const size_t at = (size_t)j * pack + 4 * c;
              float x0 = fko_widen_bf16(xr[at]), x1 = fko_widen_bf16(xr[at + 1]);
              float x2 = fko_widen_bf16(xr[at + 2]), x3 = fko_widen_bf16(xr[at + 3]);
              float w0 = fko_widen_bf16(wr[at]), w1 = fko_widen_bf16(wr[at + 1]);
              float w2 = fko_widen_bf16(wr[at + 2]), w3 = fko_widen_bf16(wr[at + 3]);
              acc[c] = acc[c] + ((x0 * w0 + x1 * w1) + (x2 * w2 + x3 * w3));
            }
          float t = acc[0];
          for (uint32_t c = 1; c < chains; ++c) t = t + acc[c];
          lanes[l] = t;
        }
        float part = fko_simd_sum(lanes, 32);
        total = q == 0 ? part : total + part;
      }
      y[(size_t)i * n + (size_t)o] = fko_narrow_bf16(total);
    }
  }
}

/* ------------------------------------------------------------------------ */
/* RoPE, halves pairing (Eval.hs:634-645): tables of each position's cosine  */
/* and sine of p * theta^(-2i/d), rounded once from binary64; each pair      */
/* (i, i + d/2), i < rotated, turned as x_i c - x_{i+d/2} s and              */
/* x_{i+d/2} c + x_i s in binary32.                                          */

void fko_rope_tables(double theta, uint32_t d, uint32_t rotated, uint32_t positions,
                     float *cos_t, float *sin_t) {
  for (uint32_t p = 0; p < positions; ++p)
    for (uint32_t i = 0; i < rotated; ++i) {
      double angle = (double)p * pow(theta, -((double)(2 * i) / (double)d));
      cos_t[(size_t)p * rotated + i] = (float)cos(angle);
      sin_t[(size_t)p * rotated + i] = (float)sin(angle);
    }
}

void fko_rope(const float *x, uint32_t m, uint32_t heads, uint32_t d, uint32_t rotated,
              const uint32_t *pos, const float *cos_t, const float *sin_t, float *y) {
  const uint32_t half = d / 2;
  for (uint32_t r = 0; r < m; ++r)
    for (uint32_t h = 0; h < heads; ++h) {
      const float *xh = x + ((size_t)r * heads + h) * d;
      float *yh = y + ((size_t)r * heads + h) * d;
      for (uint32_t i = 0; i < half; ++i) {
        if (i < rotated) {
          float c = cos_t[(size_t)pos[r] * rotated + i];
          float s = sin_t[(size_t)pos[r] * rotated + i];
          float a = xh[i], b = xh[i + half];
          yh[i] = a * c - b * s;
          yh[i + half] = b * c + a * s;
        } else {
          yh[i] = xh[i];
          yh[i + half] = xh[i + half];
        }
      }
    }
}

/* KvStore into a Ring (Graph.hs:137-143, Eval.hs:415-473): row r's head h
 * at ((slot * H + h) * L + pos mod L) * d, an exact copy in an f32 cache. */
void fko_kv_store_ring(const float *x, uint32_t m, uint32_t kv_heads, uint32_t d,
                       uint32_t length, const uint32_t *pos, const uint32_t *slot,
                       float *cache) {
  for (uint32_t r = 0; r < m; ++r)
    for (uint32_t h = 0; h < kv_heads; ++h) {
      size_t at = (((size_t)slot[r] * kv_heads + h) * length + pos[r] % length) * d;
      memcpy(cache + at, x + ((size_t)r * kv_heads + h) * d, (size_t)d * sizeof(float));
    }
}

/* ------------------------------------------------------------------------ */
/* Decode attention in splits of `chunk` positions, then their combine: the  */
/* Partials form of Plan.hs:174-181 with the order the CUDA kernel keeps.    */
/* Per position, lane l's chain over packs l, l + 32, ... of q*k from 0,     */
/* summed pairwise over the lanes, times the scale. A split's maximum, its   */
/* weights exp(s - max) in binary64 rounded once; warp w of `warps` takes    */
/* positions w, w + warps, ... adding e and e * v from 0; the warps' sums    */
/* added in warp order. The combine: the largest maximum M, each split's     */
/* exp(m - M), the rescaled sums added in split order, acc over l.           */

void fko_attend_split(const float *q, uint32_t m, uint32_t heads, uint32_t kv_heads,
                      uint32_t d, uint32_t length, const uint32_t *pos,
                      const uint32_t *slot, const float *kc, const float *vc,
                      float scale, uint32_t chunk, uint32_t warps, uint32_t max_splits,
                      float *part_m, float *part_l, float *part_acc, int threads) {
  const uint32_t group = heads / kv_heads;
  const uint32_t packs = d / 4;
#pragma omp parallel for collapse(2) schedule(dynamic) num_threads(threads > 0 ? threads : 1)
  for (int64_t r = 0; r < (int64_t)m; ++r)
    for (int64_t h = 0; h < (int64_t)heads; ++h) {
      const uint32_t npos = pos[r] + 1;
      const uint32_t splits = (npos + chunk - 1) / chunk;
      const uint32_t kvh = (uint32_t)h / group;
      const float *qh = q + ((size_t)r * heads + h) * d;
      const size_t base = ((size_t)slot[r] * kv_heads + kvh) * length;
      float *scores = (float *)malloc(chunk * sizeof(float));
      float *accw = (float *)malloc((size_t)warps * d * sizeof(float));
      float *lw = (float *)malloc(warps * sizeof(float));
      for (uint32_t j = 0; j < splits; ++j) {
        const uint32_t t0 = j * chunk;
        const uint32_t t1 = t0 + chunk < npos ? t0 + chunk : npos;
        float mx = -INFINITY;
        for (uint32_t t = t0; t < t1; ++t) {
          const float *kt = kc + (base + t % length) * d;
          float lanes[32];
          for (uint32_t l = 0; l < 32; ++l) {
            float acc = 0.0f;
            for (uint32_t p = l; p < packs; p += 32) {
              const float *a = qh + 4 * p;
              const float *b = kt + 4 * p;
              acc = acc + ((a[0] * b[0] + a[1] * b[1]) + (a[2] * b[2] + a[3] * b[3]));
            }
            lanes[l] = acc;
          }
          scores[t - t0] = fko_simd_sum(lanes, 32) * scale;
          mx = fko_max(mx, scores[t - t0]);
        }
        for (uint32_t w = 0; w < warps; ++w) {
          lw[w] = 0.0f;
          for (uint32_t i = 0; i < d; ++i) accw[(size_t)w * d + i] = 0.0f;
          for (uint32_t t = t0 + w; t < t1; t += warps) {
            const float *vt = vc + (base + t % length) * d;
            float e = fko_exp(scores[t - t0] - mx);
            lw[w] = lw[w] + e;
            for (uint32_t i = 0; i < d; ++i)
              accw[(size_t)w * d + i] = accw[(size_t)w * d + i] + e * vt[i];
          }
        }
        const size_t at = ((size_t)r * heads + h) * max_splits + j;
        float l = lw[0];
        for (uint32_t w = 1; w < warps; ++w) l = l + lw[w];
        part_m[at] = mx;
        part_l[at] = l;
        for (uint32_t i = 0; i < d; ++i) {
          float a = accw[i];
          for (uint32_t w = 1; w < warps; ++w) a = a + accw[(size_t)w * d + i];
          part_acc[at * d + i] = a;
        }
      }
      free(scores);
      free(accw);
      free(lw);
    }
}

void fko_attend_combine(uint32_t m, uint32_t heads, uint32_t d, const uint32_t *pos,
                        uint32_t chunk, uint32_t max_splits, const float *part_m,
                        const float *part_l, const float *part_acc, float *out) {
  for (uint32_t r = 0; r < m; ++r)
    for (uint32_t h = 0; h < heads; ++h) {
      const uint32_t splits = (pos[r] + 1 + chunk - 1) / chunk;
      const size_t at = ((size_t)r * heads + h) * max_splits;
      float top = -INFINITY;
      for (uint32_t j = 0; j < splits; ++j) top = fko_max(top, part_m[at + j]);
      float wts[4096];
      for (uint32_t j = 0; j < splits; ++j) wts[j] = fko_exp(part_m[at + j] - top);
      float l = part_l[at] * wts[0];
      for (uint32_t j = 1; j < splits; ++j) l = l + part_l[at + j] * wts[j];
      float *o = out + ((size_t)r * heads + h) * d;
      for (uint32_t i = 0; i < d; ++i) {
        float a = part_acc[at * d + i] * wts[0];
        for (uint32_t j = 1; j < splits; ++j) a = a + part_acc[(at + j) * d + i] * wts[j];
        o[i] = a / l;
      }
    }
}

/* ------------------------------------------------------------------------ */
/* Elementwise work and the greedy pick.                                     */

/* SiLU-gate: silu(a) * b, silu(a) = a / (1 + exp(-a)), exp in binary64. */
void fko_silu_mul(const float *a, const float *b, uint64_t n, float *y) {
  for (uint64_t i = 0; i < n; ++i) {
    float e = fko_exp(-a[i]);
    float s = a[i] / (1.0f + e);
    y[i] = s * b[i];
  }
}

/* ------------------------------------------------------------------------ */
/* Routed experts (Graph.hs:306-340; their meaning, Eval.hs:291-320, 356-416, */
/* 648-656), in this target's binary32 order.                               */

/* GELU, the tanh form (geluTanh, Eval.hs:658-659), evaluated as written,  */
/* left to right in binary32: (0.5 x) (1 + tanh(c (x + ((0.044715 x) x) x))),*/
/* c = sqrt(2/pi) rounded to binary32, tanh in binary64 rounded once.       */
float fko_gelu_tanh(float x) {
  const float c = (float)0.79788456080286535588;
  float p = 0.044715f * x;
  p = p * x;
  p = p * x;
  const float u = c * (x + p);
  const float t = (float)tanh((double)u);
  return (0.5f * x) * (1.0f + t);
}

/* Route (routeRow SoftmaxOfTopK, Eval.hs:648-656): each row's top k of its */
/* n logits, ties to the lower index (a logit is taken where it is greater  */
/* than the best so far); e_j = exp(x_j - best) (the difference in binary32,*/
/* exp in binary64 rounded once), their sum in rank order, w_j = e_j / sum, */
/* times scale[id] where an expert scale is given.                          */
void fko_route_topk(const float *x, uint32_t m, uint32_t n, uint32_t k, const float *scale, uint32_t *ids,
                    float *ws) {
  for (uint32_t r = 0; r < m; ++r) {
    const float *xr = x + (size_t)r * n;
    uint32_t *ir = ids + (size_t)r * k;
    float *wr = ws + (size_t)r * k;
    for (uint32_t j = 0; j < k; ++j) {
      uint32_t best = n;
      for (uint32_t i = 0; i < n; ++i) {
        int taken = 0;
        for (uint32_t q = 0; q < j; ++q) taken |= ir[q] == i;
        if (taken) continue;
        if (best == n || xr[i] > xr[best]) best = i;
      }
      ir[j] = best;
    }
    float e[64];
    const float top = xr[ir[0]];
    float total = 0.0f;
    for (uint32_t j = 0; j < k; ++j) {
      e[j] = (float)exp((double)(xr[ir[j]] - top));
      total = j == 0 ? e[j] : total + e[j];
    }
    for (uint32_t j = 0; j < k; ++j) {
      float w = e[j] / total;
      if (scale) w = w * scale[ir[j]];
      wr[j] = w;
    }
  }
}

/* LinearRouted (Eval.hs:291-320): per row r and rank j, y[r, j n + o] =   */
/* W[ids[r, j]] row o . x[r, base : base + kk], base 0 when every rank     */
/* takes the row's one segment (xw == kk), else j kk; the GEMV order       */
/* contract at pack 4 and split s, as fko_gemv.                             */
void fko_gemv_routed(const float *table, uint32_t entries, uint32_t n, uint32_t kk, const uint32_t *ids, uint32_t m,
                     uint32_t k, const float *x, uint32_t xw, uint32_t split, float *y, int threads) {
  const uint32_t packs = kk / 4;
  const uint32_t stride = 32 * split;
#pragma omp parallel for schedule(static) num_threads(threads > 0 ? threads : 1)
  for (int64_t rj = 0; rj < (int64_t)m * k; ++rj) {
    const uint32_t r = (uint32_t)(rj / k), j = (uint32_t)(rj % k);
    const uint32_t e = ids[(size_t)r * k + j];
    const float *xr = x + (size_t)r * xw + (xw == kk ? 0 : (size_t)j * kk);
    float *yr = y + (size_t)r * k * n + (size_t)j * n;
    if (e >= entries) {
      for (uint32_t o = 0; o < n; ++o) yr[o] = NAN;
      continue;
    }
    for (uint32_t o = 0; o < n; ++o) {
      const float *wr = table + ((size_t)e * n + o) * kk;
      float total = 0.0f;
      for (uint32_t q = 0; q < split; ++q) {
        float lanes[32];
        for (uint32_t l = 0; l < 32; ++l) {
          float acc = 0.0f;
          for (uint32_t jj = q * 32 + l; jj < packs; jj += stride) {
            const float *xp = xr + 4 * (size_t)jj;
            const float *wp = wr + 4 * (size_t)jj;
            float c = (xp[0] * wp[0] + xp[1] * wp[1]) + (xp[2] * wp[2] + xp[3] * wp[3]);
            acc = acc + c;
          }
          lanes[l] = acc;
        }
        float part = fko_simd_sum(lanes, 32);
        total = q == 0 ? part : total + part;
      }
      yr[o] = total;
    }
  }
}

/* GatedGelu (Eval.hs:356-362): per segment of 2 f, gelu(a_i) b_i of its  */
/* halves a and b; the output's segments are f wide.                       */
void fko_gated_gelu(const float *x, uint64_t segments, uint32_t f, float *y) {
  for (uint64_t s = 0; s < segments; ++s)
    for (uint32_t i = 0; i < f; ++i) {
      const float a = x[s * 2 * f + i], b = x[s * 2 * f + f + i];
      y[s * f + i] = fko_gelu_tanh(a) * b;
    }
}

/* CombineRanks then the residual Add (Eval.hs:405-416, 336-343): per row, */
/* ((w_0 s_0 + w_1 s_1) + w_2 s_2) + ... in rank order, then r + that.     */
void fko_combine_ranks_add(const float *r, const float *ws, const float *segs, uint32_t m, uint32_t k, uint32_t d,
                           float *y) {
  for (uint32_t row = 0; row < m; ++row)
    for (uint32_t i = 0; i < d; ++i) {
      float acc = ws[(size_t)row * k] * segs[(size_t)row * k * d + i];
      for (uint32_t j = 1; j < k; ++j)
        acc = acc + ws[(size_t)row * k + j] * segs[(size_t)row * k * d + (size_t)j * d + i];
      y[(size_t)row * d + i] = r[(size_t)row * d + i] + acc;
    }
}

void fko_add(const float *a, const float *b, uint64_t n, float *y) {
  for (uint64_t i = 0; i < n; ++i) y[i] = a[i] + b[i];
}

/* Gather (Eval.hs:528-535) of one token per row, times the factor. */
void fko_gather(const float *table, uint32_t width, const uint32_t *tokens, uint32_t m,
                float factor, float *y) {
  for (uint32_t r = 0; r < m; ++r)
    for (uint32_t j = 0; j < width; ++j) {
      float v = table[(size_t)tokens[r] * width + j];
      y[(size_t)r * width + j] = factor != 1.0f ? v * factor : v;
    }
}

/* ArgMax (Eval.hs:545-548, 684-685): the fold keeps the first index whose
 * value is greater than every one before it. */
void fko_argmax(const float *x, uint32_t m, uint32_t n, uint32_t *ids) {
  for (uint32_t r = 0; r < m; ++r) {
    const float *xr = x + (size_t)r * n;
    uint32_t best = 0;
    float bx = xr[0];
    for (uint32_t j = 1; j < n; ++j)
      if (xr[j] > bx) {
        best = j;
        bx = xr[j];
      }
    ids[r] = best;
  }
}
