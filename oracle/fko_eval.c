/*
 * TEST INFRASTRUCTURE -- not part of the product (see fko.h).
 *
 * The f64 evaluator of src/FuryKernel/Program/Eval.hs for the operations of
 * the decode/prefill path: each element's value in binary64, in the order of
 * the program, and its bound, how far from it a kernel's binary32 value can
 * be (Eval.hs:26-68). A kernel's element passes when it lies within
 * fkr_widened(bound) of the value, as Eval.hs:940-944 compares stores.
 *
 * Two operations are this build's additions, with meanings in the style of
 * their neighbours: SiLU-gate (silu(a) * b, bounded like GeluMul at
 * Eval.hs:363-371) and softmax over a whole row (bounded as a route's
 * softmax weights are, Eval.hs:867-875).
 */
#include "fko.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
  double x; /* exact value */
  double e; /* bound */
} approx;

static const double UNIT = 0x1p-24;   /* binary32's unit roundoff */
static const double FLUSH = 0x1p-126; /* the least normal */

static double overflow_at(void) { return ldexp(1.0, 128) - ldexp(1.0, 103); }

/* settle (Eval.hs:728-737). */
double fkr_settle(double x, double e) {
  if (isnan(x)) return e;
  if (isnan(e) || fabs(x) + e >= overflow_at()) return INFINITY;
  if (fabs(x) - e < FLUSH) return fmax(e, fabs(x));
  return e;
}

static approx settle(approx a) {
  a.e = fkr_settle(a.x, a.e);
  return a;
}

/* widened (Eval.hs:921-922). */
double fkr_widened(double e) { return e * (1.0 + 0x1p-20); }

/* gammaN (Eval.hs:701-706). */
static double gamma_n(double n) {
  if (n <= 0) return 0;
  double nu = n * UNIT;
  if (nu >= 0.5) return INFINITY;
  return nu / (1.0 - nu);
}

static double mag(approx a) { return fabs(a.x) + a.e; }
static approx exact_a(double x) { return (approx){x, 0.0}; }
static approx const_a(double c) { return settle((approx){c, fabs(c - (double)(float)c)}); }
static approx neg_a(approx a) { return (approx){-a.x, a.e}; }

/* sumA (Eval.hs:739-745). */
static approx sum_a(const approx *t, int n) {
  double s = 0, eb = 0, m = 0;
  for (int i = 0; i < n; ++i) {
    s += t[i].x;
    eb += t[i].e;
    m += mag(t[i]);
  }
  return settle((approx){s, eb + gamma_n(n - 1) * m + 2.0 * n * FLUSH});
}

/* dotA (Eval.hs:747-754), over pairs given as two arrays. */
static approx dot_a(const approx *a, const approx *c, int64_t n) {
  double s = 0, spread = 0, m = 0;
  for (int64_t i = 0; i < n; ++i) {
    s += a[i].x * c[i].x;
    spread += fabs(a[i].x) * c[i].e + a[i].e * fabs(c[i].x) + a[i].e * c[i].e;
    m += mag(a[i]) * mag(c[i]);
  }
  return settle((approx){s, spread + gamma_n((double)n) * m + 4.0 * (double)n * FLUSH});
}

/* productA (Eval.hs:759-767). */
static approx product_a(const approx *f, int n) {
  double p = 1, whole = 1, spread = 0, mx = 1;
  for (int i = 0; i < n; ++i) {
    p *= f[i].x;
    spread = spread * mag(f[i]) + whole * f[i].e;
    whole = whole * fabs(f[i].x);
    mx *= fmax(1.0, mag(f[i]));
  }
  return settle((approx){p, spread + gamma_n(n - 1) * (whole + spread) + 2.0 * n * FLUSH * mx});
}

/* quotientA (Eval.hs:769-777). */
static approx quotient_a(approx a, approx c) {
  double q = a.x / c.x;
  if (isnan(c.x) || isnan(c.e) || fabs(c.x) <= c.e) return (approx){q, INFINITY};
  double low = fabs(c.x) - c.e;
  return settle((approx){q, (fabs(a.x) * c.e + a.e * fabs(c.x)) / (fabs(c.x) * low) +
                                UNIT * mag(a) / low + FLUSH});
}

static double worst2(double a, double b) {
  if (isnan(a) || isnan(b)) return NAN;
  return fmax(0.0, fmax(a, b));
}

/* monotoneA (Eval.hs:780-787). */
static approx monotone_a(double k, double (*f)(double), approx a) {
  double y = f(a.x);
  if (isinf(a.e)) return (approx){y, INFINITY};
  double lo = f(a.x - a.e), hi = f(a.x + a.e);
  return settle((approx){y, worst2(fabs(lo - y), fabs(hi - y)) +
                                2.0 * k * UNIT * worst2(fabs(lo), fabs(hi)) + FLUSH});
}

static double inv_sqrt(double v) { return 1.0 / sqrt(v); }

/* ------------------------------------------------------------------------ */

/* Input (Eval.hs:270-280): read as binary32, which an f32 input already is. */
void fkr_input(const float *x, uint64_t n, double *v, double *b) {
  for (uint64_t i = 0; i < n; ++i) {
    v[i] = (double)x[i];
    b[i] = fkr_settle(v[i], 0.0);
  }
}

/* Linear (Eval.hs:281-290): a dot product per output, weights exact. */
void fkr_linear(const float *w, uint32_t n, uint32_t k, const double *x, const double *xb,
                uint32_t m, double *y, double *yb, int threads) {
#pragma omp parallel num_threads(threads > 0 ? threads : 1)
  {
    approx *wa = (approx *)malloc((size_t)k * sizeof(approx));
    approx *xa = (approx *)malloc((size_t)k * sizeof(approx));
#pragma omp for schedule(static) collapse(2)
    for (int64_t r = 0; r < (int64_t)m; ++r)
      for (int64_t j = 0; j < (int64_t)n; ++j) {
        for (uint32_t i = 0; i < k; ++i) {
          wa[i] = exact_a((double)w[(size_t)j * k + i]);
          xa[i] = (approx){x[(size_t)r * k + i], xb[(size_t)r * k + i]};
        }
        approx d = dot_a(wa, xa, k);
        y[(size_t)r * n + j] = d.x;
        yb[(size_t)r * n + j] = d.e;
      }
    free(wa);
    free(xa);
  }
}

/* RmsNorm (Eval.hs:322-335) and normBounds (Eval.hs:809-815), per segment. */
void fkr_rmsnorm(const double *x, const double *xb, uint32_t m, uint32_t width,
                 uint32_t seg, const float *gamma, double eps, double factor, double *y,
                 double *yb) {
  approx *xa = (approx *)malloc((size_t)seg * sizeof(approx));
  for (uint32_t r = 0; r < m; ++r)
    for (uint32_t s0 = 0; s0 < width; s0 += seg) {
      const double *xs = x + (size_t)r * width + s0;
      const double *bs = xb + (size_t)r * width + s0;
      double ss = 0;
      for (uint32_t i = 0; i < seg; ++i) {
        ss += xs[i] * xs[i];
        xa[i] = (approx){xs[i], bs[i]};
      }
      double ms = ss / (double)seg;
      double s = pow(ms + eps, -0.5);
      approx sq = dot_a(xa, xa, seg);
      approx f2[2] = {sq, const_a(1.0 / (double)seg)};
      approx mean_square = product_a(f2, 2);
      approx t2[2] = {mean_square, const_a(eps)};
      approx rr = monotone_a(2.0, inv_sqrt, sum_a(t2, 2));
      for (uint32_t i = 0; i < seg; ++i) {
        double g = gamma ? (double)gamma[i] : 1.0;
        y[(size_t)r * width + s0 + i] = xs[i] * s * g * factor;
        approx fs[4] = {xa[i], rr, const_a(factor), exact_a(g)};
        yb[(size_t)r * width + s0 + i] = product_a(fs, gamma ? 4 : 3).e;
      }
    }
  free(xa);
}

/* Add (Eval.hs:336-345). */
void fkr_add(const double *a, const double *ab, const double *c, const double *cb,
             uint64_t n, double *y, double *yb) {
  for (uint64_t i = 0; i < n; ++i) {
    approx t[2] = {{a[i], ab[i]}, {c[i], cb[i]}};
    y[i] = a[i] + c[i];
    yb[i] = sum_a(t, 2).e;
  }
}

/* SiLU-gate, silu(a) * c with silu(a) = a / (1 + exp(-a)): this build's
 * operation, bounded as GeluMul is (Eval.hs:363-371) through the contract's
 * pieces: exp within 4 ulp, a correctly rounded sum, quotient and product. */
void fkr_silu_mul(const double *a, const double *ab, const double *c, const double *cb,
                  uint64_t n, double *y, double *yb) {
  for (uint64_t i = 0; i < n; ++i) {
    approx u = {a[i], ab[i]}, v = {c[i], cb[i]};
    y[i] = a[i] / (1.0 + exp(-a[i])) * c[i];
    approx den[2] = {exact_a(1.0), monotone_a(4.0, exp, neg_a(u))};
    approx pr[2] = {quotient_a(u, sum_a(den, 2)), v};
    yb[i] = product_a(pr, 2).e;
  }
}

/* ropeTrig (Eval.hs:819-830). */
static void rope_trig(double theta, uint32_t d, uint32_t i, double position, approx *c,
                      approx *s) {
  double freq = pow(theta, -((double)(2 * i) / (double)d));
  approx f2[2] = {const_a(position), settle((approx){freq, 8.0 * UNIT * freq + FLUSH})};
  approx angle = product_a(f2, 2);
  double yc = cos(angle.x), ys = sin(angle.x);
  if (isinf(angle.e)) {
    *c = (approx){yc, INFINITY};
    *s = (approx){ys, INFINITY};
    return;
  }
  double e = angle.e;
  *c = settle((approx){yc, fmin(2.0, e) + 8.0 * UNIT * fmin(1.0, fabs(yc) + e) + FLUSH});
  *s = settle((approx){ys, fmin(2.0, e) + 8.0 * UNIT * fmin(1.0, fabs(ys) + e) + FLUSH});
}

/* Rope (Eval.hs:372-383, rotate :634-645, rotationBounds :832-841), one axis. */
void fkr_rope(const double *x, const double *xb, uint32_t m, uint32_t width, uint32_t d,
              uint32_t rotated, double theta, const uint32_t *pos, double *y, double *yb) {
  const uint32_t half = d / 2;
  for (uint32_t r = 0; r < m; ++r) {
    const double p = (double)pos[r];
    for (uint32_t h0 = 0; h0 < width; h0 += d) {
      const double *a = x + (size_t)r * width + h0;
      const double *ae = xb + (size_t)r * width + h0;
      double *o = y + (size_t)r * width + h0;
      double *oe = yb + (size_t)r * width + h0;
      for (uint32_t j = 0; j < d; ++j) {
        uint32_t i = j < half ? j : j - half;
        double t = i < rotated ? p * pow(theta, -((double)(2 * i) / (double)d)) : 0.0;
        if (j < half)
          o[j] = a[j] * cos(t) - a[j + half] * sin(t);
        else
          o[j] = a[j] * cos(t) + a[i] * sin(t);
        if (i < rotated) {
          approx c, s;
          rope_trig(theta, d, i, p, &c, &s);
          approx l[2], rr[2] = {c, s};
          l[0] = (approx){a[j], ae[j]};
          l[1] = j < half ? neg_a((approx){a[j + half], ae[j + half]}) : (approx){a[i], ae[i]};
          oe[j] = dot_a(l, rr, 2).e;
        } else {
          oe[j] = ae[j];
        }
      }
    }
  }
}

/* attendBounds (Eval.hs:900-919): the output elements' bounds from each
 * key's score and the keys' values, element by element. */
static void attend_bounds(const approx *scores, int64_t t, const double *vx,
                          const double *ve, uint32_t d, double *out_b) {
  double top = -INFINITY, highest = 0, tot = 0;
  for (int64_t i = 0; i < t; ++i) {
    top = fmax(top, scores[i].x);
    highest = fmax(highest, mag(scores[i]));
  }
  double *ps = (double *)malloc((size_t)t * sizeof(double));
  double *rhos = (double *)malloc((size_t)t * sizeof(double));
  double *gs = (double *)malloc((size_t)t * sizeof(double));
  for (int64_t i = 0; i < t; ++i) {
    ps[i] = exp(scores[i].x - top);
    tot += ps[i];
  }
  double gbar = 0;
  for (int64_t i = 0; i < t; ++i) {
    ps[i] /= tot;
    rhos[i] = scores[i].e + 2.0 * UNIT * (mag(scores[i]) + highest) +
              12.0 * ((double)t + 1.0) * UNIT + FLUSH;
    gs[i] = exp(rhos[i]) - 1.0;
    gbar += ps[i] * gs[i];
  }
  for (uint32_t c = 0; c < d; ++c) {
    if (isnan(gbar) || gbar >= 1.0) {
      out_b[c] = INFINITY;
      continue;
    }
    double o = 0, s1 = 0, s2 = 0, vm = 0;
    for (int64_t i = 0; i < t; ++i) {
      double v = vx[(size_t)i * d + c], e = ve[(size_t)i * d + c];
      o += ps[i] * v;
      s1 += ps[i] * (gs[i] + gbar) * fabs(v);
      s2 += ps[i] * exp(rhos[i]) * e;
      vm = fmax(vm, fabs(v) + e);
    }
    double spread = (s1 + s2) / (1.0 - gbar) + 4.0 * (double)t * FLUSH * vm;
    out_b[c] = fkr_settle(o, spread + UNIT * (fabs(o) + spread) + FLUSH);
  }
  free(ps);
  free(rhos);
  free(gs);
}

/* Attend (Eval.hs:474-527) over a Ring, no window, no reach: each row's
 * positions 0..pos of its slot, the caches as the kernels left them
 * (evaluateStored, Eval.hs:186-198): kc/vc are [slots, kv_heads, length, d]
 * with their bounds. */
void fkr_attend(const double *q, const double *qb, uint32_t m, uint32_t heads,
                uint32_t kv_heads, uint32_t d, uint32_t length, const uint32_t *pos,
                const uint32_t *slot, const double *kc, const double *kcb,
                const double *vc, const double *vcb, double scale, double *y, double *yb,
                int threads) {
  const uint32_t group = heads / kv_heads;
#pragma omp parallel for collapse(2) schedule(dynamic) num_threads(threads > 0 ? threads : 1)
  for (int64_t r = 0; r < (int64_t)m; ++r)
    for (int64_t h = 0; h < (int64_t)heads; ++h) {
      const int64_t t = (int64_t)pos[r] + 1;
      const uint32_t kvh = (uint32_t)h / group;
      const size_t base = ((size_t)slot[r] * kv_heads + kvh) * length;
      const double *qh = q + ((size_t)r * heads + h) * d;
      const double *qe = qb + ((size_t)r * heads + h) * d;
      approx *qa = (approx *)malloc(d * sizeof(approx));
      approx *qs = (approx *)malloc(d * sizeof(approx));
      approx *ka = (approx *)malloc(d * sizeof(approx));
      approx *sc = (approx *)malloc((size_t)t * sizeof(approx));
      double *vx = (double *)malloc((size_t)t * d * sizeof(double));
      double *ve = (double *)malloc((size_t)t * d * sizeof(double));
      approx cs = const_a(scale);
      for (uint32_t i = 0; i < d; ++i) {
        qa[i] = (approx){qh[i], qe[i]};
        approx pr[2] = {qa[i], cs};
        qs[i] = product_a(pr, 2);
      }
      double top = -INFINITY;
      for (int64_t p = 0; p < t; ++p) {
        size_t at = (base + (size_t)p % length) * d;
        double dot = 0;
        for (uint32_t i = 0; i < d; ++i) {
          ka[i] = (approx){kc[at + i], kcb ? kcb[at + i] : 0.0};
          dot += qh[i] * kc[at + i];
          vx[(size_t)p * d + i] = vc[at + i];
          ve[(size_t)p * d + i] = vcb ? vcb[at + i] : 0.0;
        }
        approx dq = dot_a(qa, ka, d);
        approx pr[2] = {dq, cs};
        double b1 = product_a(pr, 2).e;
        double b2 = dot_a(qs, ka, d).e;
        sc[p] = (approx){scale * dot, fmax(b1, b2)};
        top = fmax(top, sc[p].x);
      }
      double total = 0;
      for (int64_t p = 0; p < t; ++p) total += exp(sc[p].x - top);
      double *o = y + ((size_t)r * heads + h) * d;
      for (uint32_t i = 0; i < d; ++i) {
        double acc = 0;
        for (int64_t p = 0; p < t; ++p) acc += exp(sc[p].x - top) / total * vx[(size_t)p * d + i];
        o[i] = acc;
      }
      attend_bounds(sc, t, vx, ve, d, yb + ((size_t)r * heads + h) * d);
      free(qa);
      free(qs);
      free(ka);
      free(sc);
      free(vx);
      free(ve);
    }
}

/* Gather (Eval.hs:528-535) with gatherA (Eval.hs:883-887), one token a row. */
void fkr_gather(const float *table, uint32_t width, const uint32_t *tokens, uint32_t m,
                double factor, double *y, double *yb) {
  for (uint32_t r = 0; r < m; ++r)
    for (uint32_t j = 0; j < width; ++j) {
      double w = (double)table[(size_t)tokens[r] * width + j];
      y[(size_t)r * width + j] = w * factor;
      approx a = exact_a(w), f = const_a(factor);
      double by_dot = dot_a(&a, &f, 1).e;
      approx s = sum_a(&a, 1);
      approx pr[2] = {s, f};
      double by_sum = product_a(pr, 2).e;
      yb[(size_t)r * width + j] = fmax(by_dot, by_sum);
    }
}

/* ArgMax (Eval.hs:545-548) and argMaxDecided (Eval.hs:877-880): decided when
 * the best is certainly before every other (certainlyBefore, Eval.hs:851-855). */
void fkr_argmax(const double *x, const double *xb, uint32_t m, uint32_t n, uint32_t *ids,
                int *decided) {
  for (uint32_t r = 0; r < m; ++r) {
    const double *xr = x + (size_t)r * n;
    const double *br = xb + (size_t)r * n;
    uint32_t best = 0;
    for (uint32_t j = 1; j < n; ++j)
      if (xr[j] > xr[best]) best = j;
    ids[r] = best;
    /* ranked's first: the largest exact value, ties to the lower index. */
    double lo = xr[best] - br[best];
    int ok = 1;
    for (uint32_t j = 0; j < n && ok; ++j) {
      if (j == best) continue;
      double hi = xr[j] + br[j];
      if (!(lo > hi || (lo == hi && best < j))) ok = 0;
    }
    decided[r] = ok;
  }
}

/* Softmax over a row: this build's row kernel, bounded as a route's softmax
 * weights are (routeWeightBounds, Eval.hs:867-875, every element taken). */
void fkr_softmax(const double *x, const double *xb, uint32_t m, uint32_t n, double *y,
                 double *yb) {
  approx *es = (approx *)malloc((size_t)n * sizeof(approx));
  for (uint32_t r = 0; r < m; ++r) {
    const double *xr = x + (size_t)r * n;
    const double *br = xb + (size_t)r * n;
    uint32_t best = 0;
    for (uint32_t j = 1; j < n; ++j)
      if (xr[j] > xr[best]) best = j;
    approx b = {xr[best], br[best]};
    double tot = 0;
    for (uint32_t j = 0; j < n; ++j) tot += exp(xr[j] - xr[best]);
    for (uint32_t j = 0; j < n; ++j) {
      approx t2[2] = {{xr[j], br[j]}, neg_a(b)};
      es[j] = monotone_a(4.0, exp, sum_a(t2, 2));
    }
    /* sumA over n terms, in one pass. */
    double s = 0, eb = 0, mg = 0;
    for (uint32_t j = 0; j < n; ++j) {
      s += es[j].x;
      eb += es[j].e;
      mg += mag(es[j]);
    }
    approx total = settle((approx){s, eb + gamma_n((double)n - 1) * mg + 2.0 * n * FLUSH});
    for (uint32_t j = 0; j < n; ++j) {
      y[(size_t)r * n + j] = exp(xr[j] - xr[best]) / tot;
      yb[(size_t)r * n + j] = quotient_a(es[j], total).e;
    }
  }
  free(es);
}

/* A sum of exact binary32 terms (sumA, Eval.hs:739-745). */
void fkr_sum(const float *x, uint64_t n, double *y, double *yb) {
  double s = 0, m = 0;
  for (uint64_t i = 0; i < n; ++i) {
    s += (double)x[i];
    m += fabs((double)x[i]);
  }
  *y = s;
  *yb = fkr_settle(s, gamma_n((double)n - 1) * m + 2.0 * (double)n * FLUSH);
}
