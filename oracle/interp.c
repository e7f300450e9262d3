/*
 * ORACLE -- test infrastructure only.  Only tests/, __graft_entry__.smoke()
 * and bench.py's CPU legs may load this; the product path never does.
 *
 * A C restatement of the reference's float64 interpreter (src/interp.js:1-162)
 * and of its float32 error budget (src/gpu/bounds.js:13-136, amendment 8).
 *
 *  - tco_evaluate(..., with_bounds = 0): interp.js `evaluate`.  Every value is
 *    float64, loops run in index order and every reduction sums first to last
 *    (src/interp.js:29-45, :67-84), max starts at -inf, relu/step test x > 0.
 *  - tco_evaluate(..., with_bounds = 1): bounds.js `referenceWithBounds`.
 *    Inputs and constants are rounded to float32 first (bounds.js:107, :111)
 *    unless an input carries its own bound (bounds.js:97-102, the `carried`
 *    form); every node gets a first-order bound E per element.
 *
 * Intermediates are freed after their last use, so the peak memory is the
 * live set, not the whole graph (the idea of workloads.js:275-301's
 * streamingReference, which gives the same values and bounds).
 *
 * Single-threaded, no SIMD intrinsics: this is also the timed CPU baseline.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "interp.h"

static const double U = 5.9604644775390625e-08;      /* 2^-24 */
static const double EPS = 1.1920928955078125e-07;    /* 2^-23 */
static const double TAU = 1.1754943508222875e-38;    /* 2^-126 */

static double gamma_n(double n) { return (n * U) / (1 - n * U); }
static double ftz(double r) { return (r != 0 && fabs(r) < TAU) ? TAU : 0; }
static double fround(double v) { return (double)(float)v; }

static int64_t nsize(const tco_node* n) {
  int64_t s = 1;
  for (int i = 0; i < n->rank; i++) s *= n->shape[i];
  return s;
}

static void set_err(char* err, int errlen, const char* msg, int node) {
  if (err && errlen > 0) snprintf(err, (size_t)errlen, "node %d: %s", node, msg);
}

/* ---- index helpers (src/interp.js:9-14, :89-126) ---- */
static void strides_of(const int64_t* shape, int rank, int64_t* st) {
  int64_t acc = 1;
  for (int i = rank - 1; i >= 0; i--) { st[i] = acc; acc *= shape[i]; }
}

static void k_broadcast(const tco_node* nd, const tco_node* src, const double* x, double* out) {
  int64_t fs[TCO_MAX_RANK], ts[TCO_MAX_RANK];
  strides_of(src->shape, src->rank, fs);
  strides_of(nd->shape, nd->rank, ts);
  int lead = nd->rank - src->rank;
  int64_t n = nsize(nd);
  for (int64_t i = 0; i < n; i++) {
    int64_t s = 0;
    for (int d = 0; d < src->rank; d++) {
      if (src->shape[d] == 1) continue;
      int64_t coord = (i / ts[lead + d]) % nd->shape[lead + d];
      s += coord * fs[d];
    }
    out[i] = x[s];
  }
}

static void k_transpose(const tco_node* nd, const tco_node* src, const double* x, double* out) {
  int64_t fs[TCO_MAX_RANK], ts[TCO_MAX_RANK];
  strides_of(src->shape, src->rank, fs);
  strides_of(nd->shape, nd->rank, ts);
  int64_t n = nsize(nd);
  for (int64_t i = 0; i < n; i++) {
    int64_t s = 0;
    for (int d = 0; d < nd->rank; d++) {
      int64_t coord = (i / ts[d]) % nd->shape[d];
      s += coord * fs[nd->perm[d]];
    }
    out[i] = x[s];
  }
}

static void reduce_dims(const tco_node* src, int axis, int64_t* outer, int64_t* n, int64_t* inner) {
  int64_t o = 1, in = 1;
  for (int i = 0; i < axis; i++) o *= src->shape[i];
  for (int i = axis + 1; i < src->rank; i++) in *= src->shape[i];
  *outer = o; *n = src->shape[axis]; *inner = in;
}

/* sum or max; `absval` sums |x| (the budget's mass term) */
static void k_reduce(const tco_node* nd, const tco_node* src, const double* x, double* out, int is_max, int absval) {
  int64_t outer, n, inner;
  reduce_dims(src, nd->axis, &outer, &n, &inner);
  for (int64_t o = 0; o < outer; o++) {
    for (int64_t i = 0; i < inner; i++) {
      double acc = is_max ? -INFINITY : 0.0;
      const double* p = x + o * n * inner + i;
      for (int64_t k = 0; k < n; k++) {
        double v = p[k * inner];
        if (absval) v = fabs(v);
        if (is_max) { if (v > acc) acc = v; }
        else acc = acc + v;
      }
      out[o * inner + i] = acc;
    }
  }
}

/* matmul; `absmode` bit 0: |a|, bit 1: |b| */
static void k_matmul(const tco_node* nd, const tco_node* na, const tco_node* nb, const double* a, const double* b,
                     double* out, int absmode) {
  int64_t m = na->shape[na->rank - 2], k = na->shape[na->rank - 1], n = nb->shape[nb->rank - 1];
  int64_t batch = 1;
  for (int i = 0; i < na->rank - 2; i++) batch *= na->shape[i];
  (void)nd;
  for (int64_t t = 0; t < batch; t++) {
    const double* A = a + t * m * k;
    const double* B = b + t * k * n;
    double* O = out + t * m * n;
    for (int64_t i = 0; i < m; i++) {
      for (int64_t j = 0; j < n; j++) {
        double acc = 0;
        for (int64_t p = 0; p < k; p++) {
          double av = A[i * k + p], bv = B[p * n + j];
          if (absmode & 1) av = fabs(av);
          if (absmode & 2) bv = fabs(bv);
          acc += av * bv;
        }
        O[i * n + j] = acc;
      }
    }
  }
}

static double ew1(int op, double x) {
  switch (op) {
    case TCO_NEG: return -x;
    case TCO_EXP: return exp(x);
    case TCO_LOG: return log(x);
    case TCO_RELU: return x > 0 ? x : 0;
    case TCO_TANH: return tanh(x);
    case TCO_SQRT: return sqrt(x);
    case TCO_STEP: return x > 0 ? 1 : 0;
    case TCO_STOPGRAD: return x;
  }
  return NAN;
}

static double ew2(int op, double a, double b) {
  switch (op) {
    case TCO_ADD: return a + b;
    case TCO_SUB: return a - b;
    case TCO_MUL: return a * b;
    case TCO_DIV: return a / b;
  }
  return NAN;
}

/* amendment 8's elementwise rules (src/gpu/bounds.js:25-55) */
static double bound1(int op, double r, double x, double ex) {
  switch (op) {
    case TCO_NEG: case TCO_RELU: case TCO_STOPGRAD: return ex;
    case TCO_EXP: {
      double grow = exp(ex);
      return fabs(r) * (grow - 1) + (3 + 2 * (fabs(x) + ex)) * EPS * fabs(r) * grow;
    }
    case TCO_LOG: {
      if (!(x > 0) || ex >= x) return INFINITY;
      double inherited = -log1p(-ex / x);
      double floor_ = 4.76837158203125e-07; /* 2^-21 */
      double rel = 3 * EPS * (fabs(r) + inherited);
      return inherited + (floor_ > rel ? floor_ : rel);
    }
    case TCO_TANH: {
      double rel = (9.5 + 4 * (fabs(x) + ex)) * EPS;
      return ex + (1e-5 > rel ? 1e-5 : rel);
    }
    case TCO_SQRT: {
      if (x < 0) return INFINITY;
      double inherited;
      if (x > 0) { double s1 = sqrt(ex), s2 = ex / sqrt(x); inherited = s1 < s2 ? s1 : s2; }
      else inherited = sqrt(ex);
      return inherited + 4.5 * EPS * fabs(r);
    }
    case TCO_STEP: return (ex > 0 && fabs(x) <= ex) ? 1 : 0;
  }
  return INFINITY;
}

static double bound2(int op, double r, double a, double b, double ea, double eb) {
  switch (op) {
    case TCO_ADD: case TCO_SUB: return ea + eb + U * fabs(r);
    case TCO_MUL: return fabs(b) * ea + fabs(a) * eb + ea * eb + U * fabs(r);
    case TCO_DIV: {
      double m = fabs(b);
      if (eb >= m || m < 1.1754943508222875e-38 || m > 8.507059173023462e37) return INFINITY;
      return (ea + fabs(r) * eb) / (m - eb) + 2.5 * EPS * fabs(r);
    }
  }
  return INFINITY;
}

static int all_zero(const double* x, int64_t n) {
  for (int64_t i = 0; i < n; i++) if (x[i] != 0) return 0;
  return 1;
}

int tco_abi_version(void) { return 1; }

/* One node's value (and bound).  Returns 0 or -1. */
static int eval_node(tco_node* nodes, int id, double** vals, double** bnds, int with_bounds, char* err, int errlen) {
  tco_node* nd = &nodes[id];
  int64_t n = nsize(nd);
  double* v = vals[id];
  double* e = with_bounds ? bnds[id] : NULL;
  if (nd->op == TCO_CONST) {
    for (int64_t i = 0; i < n; i++) {
      double c = nd->data ? nd->data[i] : nd->scalar;
      v[i] = with_bounds ? fround(c) : c;
      if (e) e[i] = ftz(v[i]);
    }
    return 0;
  }
  const tco_node* na = &nodes[nd->in0];
  const tco_node* nb = nd->n_in > 1 ? &nodes[nd->in1] : NULL;
  const double* a = vals[nd->in0];
  const double* b = nb ? vals[nd->in1] : NULL;
  const double* ea = with_bounds ? bnds[nd->in0] : NULL;
  const double* eb = (with_bounds && nb) ? bnds[nd->in1] : NULL;
  switch (nd->op) {
    case TCO_ADD: case TCO_SUB: case TCO_MUL: case TCO_DIV:
      for (int64_t i = 0; i < n; i++) v[i] = ew2(nd->op, a[i], b[i]);
      if (e) for (int64_t i = 0; i < n; i++) e[i] = bound2(nd->op, v[i], a[i], b[i], ea[i], eb[i]);
      break;
    case TCO_NEG: case TCO_EXP: case TCO_LOG: case TCO_RELU: case TCO_TANH: case TCO_STEP: case TCO_STOPGRAD:
    case TCO_SQRT:
      for (int64_t i = 0; i < n; i++) v[i] = ew1(nd->op, a[i]);
      if (e) for (int64_t i = 0; i < n; i++) e[i] = bound1(nd->op, v[i], a[i], ea[i]);
      break;
    case TCO_MATMUL: {
      k_matmul(nd, na, nb, a, b, v, 0);
      if (e) {
        int64_t K = na->shape[na->rank - 1];
        double g = gamma_n((double)K);
        int64_t na_n = nsize(na), nb_n = nsize(nb);
        int za = all_zero(ea, na_n), zb = all_zero(eb, nb_n);
        double* t = (double*)malloc(sizeof(double) * (size_t)(n ? n : 1));
        if (!t) { set_err(err, errlen, "out of host memory", id); return -1; }
        /* bound = |a|.eb + ea.|b| + ea.eb + gamma(K) |a|.|b|  (bounds.js:68-74) */
        for (int64_t i = 0; i < n; i++) e[i] = 0;
        if (!zb) { k_matmul(nd, na, nb, a, eb, t, 1); for (int64_t i = 0; i < n; i++) e[i] += t[i]; }
        if (!za) { k_matmul(nd, na, nb, ea, b, t, 2); for (int64_t i = 0; i < n; i++) e[i] += t[i]; }
        if (!za && !zb) { k_matmul(nd, na, nb, ea, eb, t, 0); for (int64_t i = 0; i < n; i++) e[i] += t[i]; }
        k_matmul(nd, na, nb, a, b, t, 3);
        for (int64_t i = 0; i < n; i++) e[i] += g * t[i];
        free(t);
      }
      break;
    }
    case TCO_SUM: case TCO_MAX: {
      int is_max = nd->op == TCO_MAX;
      k_reduce(nd, na, a, v, is_max, 0);
      if (e) {
        if (is_max) k_reduce(nd, na, ea, e, 1, 0);
        else {
          int64_t outer, cnt, inner;
          reduce_dims(na, nd->axis, &outer, &cnt, &inner);
          double g = gamma_n((double)cnt);
          double* t = (double*)malloc(sizeof(double) * (size_t)(n ? n : 1));
          if (!t) { set_err(err, errlen, "out of host memory", id); return -1; }
          k_reduce(nd, na, ea, e, 0, 0);
          k_reduce(nd, na, a, t, 0, 1);
          for (int64_t i = 0; i < n; i++) e[i] = e[i] + g * t[i];
          free(t);
        }
      }
      break;
    }
    case TCO_BROADCAST:
      k_broadcast(nd, na, a, v);
      if (e) k_broadcast(nd, na, ea, e);
      break;
    case TCO_RESHAPE:
      memcpy(v, a, sizeof(double) * (size_t)n);
      if (e) memcpy(e, ea, sizeof(double) * (size_t)n);
      break;
    case TCO_TRANSPOSE:
      k_transpose(nd, na, a, v);
      if (e) k_transpose(nd, na, ea, e);
      break;
    default:
      set_err(err, errlen, "no kernel for this op", id);
      return -1;
  }
  if (e) for (int64_t i = 0; i < n; i++) e[i] += ftz(v[i]);
  return 0;
}

int tco_evaluate(tco_node* nodes, int n, int with_bounds, char* err, int errlen) {
  int rc = -1;
  double** vals = (double**)calloc((size_t)n + 1, sizeof(double*));
  double** bnds = (double**)calloc((size_t)n + 1, sizeof(double*));
  char* owned_v = (char*)calloc((size_t)n + 1, 1);
  char* owned_b = (char*)calloc((size_t)n + 1, 1);
  int* last_use = (int*)malloc(sizeof(int) * ((size_t)n + 1));
  if (!vals || !bnds || !owned_v || !owned_b || !last_use) { set_err(err, errlen, "out of host memory", -1); goto done; }
  for (int i = 0; i < n; i++) last_use[i] = -1;
  for (int i = 0; i < n; i++) {
    if (nodes[i].n_in > 0) last_use[nodes[i].in0] = i;
    if (nodes[i].n_in > 1) last_use[nodes[i].in1] = i;
  }
  for (int id = 0; id < n; id++) {
    tco_node* nd = &nodes[id];
    int64_t sz = nsize(nd);
    size_t bytes = sizeof(double) * (size_t)(sz ? sz : 1);
    if (nd->op == TCO_INPUT) {
      if (!nd->data) { set_err(err, errlen, "no value for input", id); goto done; }
      if (!with_bounds || nd->data_bound) {
        vals[id] = (double*)nd->data;  /* used as given (never written) */
      } else {
        vals[id] = (double*)malloc(bytes);
        if (!vals[id]) { set_err(err, errlen, "out of host memory", id); goto done; }
        owned_v[id] = 1;
        for (int64_t i = 0; i < sz; i++) vals[id][i] = fround(nd->data[i]);
      }
      if (with_bounds) {
        if (nd->data_bound) bnds[id] = (double*)nd->data_bound;
        else {
          bnds[id] = (double*)malloc(bytes);
          if (!bnds[id]) { set_err(err, errlen, "out of host memory", id); goto done; }
          owned_b[id] = 1;
          for (int64_t i = 0; i < sz; i++) bnds[id][i] = ftz(vals[id][i]);
        }
      }
    } else {
      if (nd->out) vals[id] = nd->out;
      else {
        vals[id] = (double*)malloc(bytes);
        if (!vals[id]) { set_err(err, errlen, "out of host memory", id); goto done; }
        owned_v[id] = 1;
      }
      if (with_bounds) {
        if (nd->out_bound) bnds[id] = nd->out_bound;
        else {
          bnds[id] = (double*)malloc(bytes);
          if (!bnds[id]) { set_err(err, errlen, "out of host memory", id); goto done; }
          owned_b[id] = 1;
        }
      }
      if (eval_node(nodes, id, vals, bnds, with_bounds, err, errlen) != 0) goto done;
    }
    /* requested copies of inputs */
    if (nd->op == TCO_INPUT && nd->out) memcpy(nd->out, vals[id], bytes);
    if (nd->op == TCO_INPUT && with_bounds && nd->out_bound) memcpy(nd->out_bound, bnds[id], bytes);
    /* free operands whose last use this was */
    for (int k = 0; k < nd->n_in; k++) {
      int src = k == 0 ? nd->in0 : nd->in1;
      if (last_use[src] == id) {
        if (owned_v[src]) { free(vals[src]); owned_v[src] = 0; }
        if (owned_b[src]) { free(bnds[src]); owned_b[src] = 0; }
        vals[src] = NULL; bnds[src] = NULL;
      }
    }
  }
  rc = 0;
done:
  if (vals) for (int i = 0; i < n; i++) if (owned_v && owned_v[i]) free(vals[i]);
  if (bnds) for (int i = 0; i < n; i++) if (owned_b && owned_b[i]) free(bnds[i]);
  free(vals); free(bnds); free(owned_v); free(owned_b); free(last_use);
  return rc;
}
