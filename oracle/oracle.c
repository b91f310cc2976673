/* oracle.c — CPU restatement of the reference's small-op path.
 * TEST INFRASTRUCTURE ONLY (see oracle.h for scope and citations).
 *
 * Built with -ffp-contract=off: every a*b+c below rounds twice unless it is
 * written as fmaf(), which marks the places where the CUDA compiler's
 * default contraction (fmad=true in NVRTC and nvcc) fuses the reference's
 * expression.
 */
#include "oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ---- fp16 / bf16 conversions (IEEE 754 binary16, round to nearest even) ---- */
uint16_t oracle_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const uint32_t exp = (x >> 23) & 0xffu;
  uint32_t man = x & 0x7fffffu;
  if (exp == 0xffu) return (uint16_t)(sign | 0x7c00u | (man ? 0x200u | (man >> 13) : 0u));
  const int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7c00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    const int shift = 14 - e;
    uint32_t h = man >> shift;
    const uint32_t rem = man & ((1u << shift) - 1u), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)e << 10) | (man >> 13);
  const uint32_t rem = man & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}

float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu, x;
  if (exp == 0x1fu) {
    x = sign | 0x7f800000u | (man << 13);
  } else if (exp == 0) {
    if (man == 0) {
      x = sign;
    } else {
      int e = -1;
      do { ++e; man <<= 1; } while (!(man & 0x400u));
      x = sign | ((uint32_t)(127 - 15 - e) << 23) | ((man & 0x3ffu) << 13);
    }
  } else {
    x = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

uint16_t oracle_f32_to_bf16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

float oracle_bf16_to_f32(uint16_t h) {
  const uint32_t x = (uint32_t)h << 16;
  float f;
  memcpy(&f, &x, 4);
  return f;
}

static inline float ld(const void* base, int dt, int64_t off) {
  if (dt == 0) return ((const float*)base)[off];
  if (dt == 4) return (float)((const double*)base)[off];
  if (dt == 1) return oracle_f16_to_f32(((const uint16_t*)base)[off]);
  return oracle_bf16_to_f32(((const uint16_t*)base)[off]);
}

static inline void st(void* base, int dt, int64_t off, float v) {
  if (dt == 0) ((float*)base)[off] = v;
  else if (dt == 1) ((uint16_t*)base)[off] = oracle_f32_to_f16(v);
  else ((uint16_t*)base)[off] = oracle_f32_to_bf16(v);
}

/* ---- operator formulas ---------------------------------------------------- */
float oracle_op1(int v, float A, float B, float p0, float p1) {
  switch (v) {
    case OR_ADD: return A + B;
    case OR_MUL: return A * B;
    case OR_SUB: return A - B;
    case OR_DIV0: return (B != 0.f) ? (A / B) : 0.f;
    case OR_DIV: return A / B;
    case OR_MAX: return A > B ? A : B;
    case OR_MIN: return A < B ? A : B;
    case OR_POW: return powf(A, B);
    case OR_RELU: return A > 0.f ? A : 0.f;
    case OR_SIGMOID: return 1.f / (1.f + expf(-A));
    case OR_TANH: return tanhf(A);
    case OR_EXP: return expf(A);
    case OR_LOG: return logf(A);
    case OR_SQRT: return sqrtf(A);
    case OR_ABS: return fabsf(A);
    case OR_HARDSIGMOID: return fminf(fmaxf(fmaf(0.2f, A, 0.5f), 0.f), 1.f);
    case OR_HARDSWISH: return A * fminf(fmaxf(A / 6.f + 0.5f, 0.f), 1.f);
    case OR_GELU: {
      const float inner = fmaf(0.044715f * A * A, A, A);
      return 0.5f * A * (1.f + tanhf(0.79788456f * inner));
    }
    case OR_SIN: return sinf(A);
    case OR_COS: return cosf(A);
    case OR_LEAKY_RELU: return A >= 0.f ? A : p0 * A;
    case OR_CLAMP: return fminf(fmaxf(A, p0), p1);
    case OR_ELU: return A > 0.f ? A : p0 * (expf(A) - 1.f);
    case OR_SOFTPLUS: return log1pf(expf(p0 * A)) / p0;
    case OR_CLAMP_MIN: return fmaxf(A, p0);
    case OR_CLAMP_MAX: return fminf(A, p0);
    default: return A; /* OR_COPY */
  }
}

/* The same formulas evaluated in double precision (no intermediate fp32
 * rounding): the exact value the fp32 results are measured against. */
double oracle_op1_exact(int v, double A, double B, double p0, double p1) {
  switch (v) {
    case OR_ADD: return A + B;
    case OR_MUL: return A * B;
    case OR_SUB: return A - B;
    case OR_DIV0: return (B != 0.0) ? (A / B) : 0.0;
    case OR_DIV: return A / B;
    case OR_MAX: return A > B ? A : B;
    case OR_MIN: return A < B ? A : B;
    case OR_POW: return pow(A, B);
    case OR_RELU: return A > 0.0 ? A : 0.0;
    case OR_SIGMOID: return 1.0 / (1.0 + exp(-A));
    case OR_TANH: return tanh(A);
    case OR_EXP: return exp(A);
    case OR_LOG: return log(A);
    case OR_SQRT: return sqrt(A);
    case OR_ABS: return fabs(A);
    case OR_HARDSIGMOID: return fmin(fmax(0.2f * A + 0.5, 0.0), 1.0);
    case OR_HARDSWISH: return A * fmin(fmax(A / 6.0 + 0.5, 0.0), 1.0);
    case OR_GELU: return 0.5 * A * (1.0 + tanh((double)0.79788456f * (A + (double)0.044715f * A * A * A)));
    case OR_SIN: return sin(A);
    case OR_COS: return cos(A);
    case OR_LEAKY_RELU: return A >= 0.0 ? A : p0 * A;
    case OR_CLAMP: return fmin(fmax(A, p0), p1);
    case OR_ELU: return A > 0.0 ? A : p0 * (exp(A) - 1.0);
    case OR_SOFTPLUS: return log1p(exp(p0 * A)) / p0;
    case OR_CLAMP_MIN: return fmax(A, p0);
    case OR_CLAMP_MAX: return fmin(A, p0);
    default: return A;
  }
}

static inline double ldd(const void* base, int dt, int64_t off) {
  if (dt == 4) return ((const double*)base)[off];
  return (double)ld(base, dt, off);
}

/* torch broadcasting of t onto out's shape: per-out-dim strides */
static int bcast(const or_tensor* t, const or_tensor* out, int64_t* s) {
  const int nd = out->ndim;
  for (int d = 0; d < t->ndim - nd; ++d)
    if (t->sizes[d] != 1) return -1;
  for (int d = 0; d < nd; ++d) {
    const int od = nd - 1 - d, id = t->ndim - 1 - d;
    const int64_t sz = id >= 0 ? t->sizes[id] : 1, str = id >= 0 ? t->strides[id] : 0;
    if (sz == out->sizes[od]) s[od] = sz == 1 ? 0 : str;
    else if (sz == 1) s[od] = 0;
    else return -1;
  }
  return 0;
}

int oracle_ew(int v, float p0, float p1, const or_tensor* a, const or_tensor* b,
              const or_tensor* out) {
  int64_t sa[8] = {0}, sb[8] = {0};
  if (bcast(a, out, sa)) return -1;
  if (b && bcast(b, out, sb)) return -1;
  const int nd = out->ndim;
  int64_t n = 1;
  for (int d = 0; d < nd; ++d) n *= out->sizes[d];
  int64_t idx[8] = {0};
  int64_t oa = 0, ob = 0, oo = 0;
  for (int64_t e = 0; e < n; ++e) {
    const float A = ld(a->data, a->dtype, oa);
    const float B = b ? ld(b->data, b->dtype, ob) : 0.f;
    st(out->data, out->dtype, oo, oracle_op1(v, A, B, p0, p1));
    for (int d = nd - 1; d >= 0; --d) { /* odometer, last dim fastest */
      ++idx[d];
      oa += sa[d]; ob += sb[d]; oo += out->strides[d];
      if (idx[d] < out->sizes[d]) break;
      oa -= sa[d] * idx[d]; ob -= sb[d] * idx[d]; oo -= out->strides[d] * idx[d];
      idx[d] = 0;
    }
  }
  return 0;
}

int oracle_ew_exact(int v, float p0, float p1, const or_tensor* a, const or_tensor* b,
                    const or_tensor* out) {
  int64_t sa[8] = {0}, sb[8] = {0};
  if (out->dtype != 4) return -1;
  if (bcast(a, out, sa)) return -1;
  if (b && bcast(b, out, sb)) return -1;
  const int nd = out->ndim;
  int64_t n = 1;
  for (int d = 0; d < nd; ++d) n *= out->sizes[d];
  int64_t idx[8] = {0};
  int64_t oa = 0, ob = 0, oo = 0;
  for (int64_t e = 0; e < n; ++e) {
    const double A = ldd(a->data, a->dtype, oa);
    const double B = b ? ldd(b->data, b->dtype, ob) : 0.0;
    ((double*)out->data)[oo] = oracle_op1_exact(v, A, B, p0, p1);
    for (int d = nd - 1; d >= 0; --d) {
      ++idx[d];
      oa += sa[d]; ob += sb[d]; oo += out->strides[d];
      if (idx[d] < out->sizes[d]) break;
      oa -= sa[d] * idx[d]; ob -= sb[d] * idx[d]; oo -= out->strides[d] * idx[d];
      idx[d] = 0;
    }
  }
  return 0;
}

/* the reference's decomposition: every operand's offset comes from the linear
 * output index decomposed over that operand's own aligned sizes */
static int64_t ref_offset(const int64_t* sizes, const int64_t* strides, int nd, int64_t idx) {
  int64_t off = 0;
  for (int d = nd - 1; d >= 0; --d) {
    const int64_t dim = sizes[d] > 0 ? sizes[d] : 1;
    off += (idx % dim) * strides[d];
    idx /= dim;
  }
  return off;
}

static void ref_align(const or_tensor* t, int nd, int64_t* sz, int64_t* st_) {
  for (int d = 0; d < nd; ++d) {
    const int od = nd - 1 - d, id = t->ndim - 1 - d;
    const int64_t s = id >= 0 ? t->sizes[id] : 1, str = id >= 0 ? t->strides[id] : 0;
    sz[od] = s;
    st_[od] = s == 1 ? 0 : str;
  }
}

int oracle_ew_refindex(int v, float p0, float p1, const or_tensor* a, const or_tensor* b,
                       const or_tensor* out) {
  const int nd = out->ndim;
  int64_t asz[8], ast[8], bsz[8], bst[8], ost[8];
  ref_align(a, nd, asz, ast);
  if (b) ref_align(b, nd, bsz, bst);
  int64_t n = 1;
  for (int d = nd - 1; d >= 0; --d) { ost[d] = n; n *= out->sizes[d]; }
  for (int64_t e = 0; e < n; ++e) {
    const float A = ld(a->data, a->dtype, ref_offset(asz, ast, nd, e));
    const float B = b ? ld(b->data, b->dtype, ref_offset(bsz, bst, nd, e)) : 0.f;
    st(out->data, out->dtype, ref_offset(out->sizes, ost, nd, e), oracle_op1(v, A, B, p0, p1));
  }
  return 0;
}

/* ---- reductions ------------------------------------------------------------ */
int oracle_reduce(int mean, const or_tensor* x, const or_tensor* out, const int32_t* axes,
                  int naxes, int keepdim, int threads) {
  const int nd = x->ndim;
  int red[8] = {0}, rax[8], nr = 0;
  for (int i = 0; i < naxes; ++i) {
    int ax = axes[i] < 0 ? axes[i] + nd : axes[i];
    if (ax < 0 || ax >= nd) return -1;
    red[ax] = 1;
  }
  for (int i = 0; i < naxes; ++i) { /* reduced axes in the order given (deduplicated) */
    int ax = axes[i] < 0 ? axes[i] + nd : axes[i], dup = 0;
    for (int j = 0; j < nr; ++j) dup |= rax[j] == ax;
    if (!dup) rax[nr++] = ax;
  }
  int64_t ksz[8], kst[8], kso[8], nk = 0, od = 0;
  for (int d = 0; d < nd; ++d) {
    if (red[d]) { if (keepdim) ++od; continue; }
    ksz[nk] = x->sizes[d];
    kst[nk] = x->strides[d];
    kso[nk] = out->strides[od++];
    ++nk;
  }
  int64_t R = 1, C = 1;
  for (int i = 0; i < nk; ++i) R *= ksz[i];
  for (int j = 0; j < nr; ++j) C *= x->sizes[rax[j]];
  const int fast = nr == 1 && rax[0] == nd - 1 && x->strides[nd - 1] == 1;
  if (threads <= 0) threads = 256;
  float* shm = (float*)malloc(sizeof(float) * (size_t)threads);
  for (int64_t r = 0; r < R; ++r) {
    int64_t rem = r, ib = 0, ob = 0;
    for (int i = (int)nk - 1; i >= 0; --i) {
      const int64_t k = rem % ksz[i];
      rem /= ksz[i];
      ib += k * kst[i];
      ob += k * kso[i];
    }
    float acc = 0.f;
    if (fast) {
      for (int t = 0; t < threads; ++t) {
        float s = 0.f;
        for (int64_t c = t; c < C; c += threads) s += ld(x->data, x->dtype, ib + c);
        shm[t] = s;
      }
      for (int step = threads >> 1; step > 0; step >>= 1)
        for (int t = 0; t < step; ++t) shm[t] += shm[t + step];
      acc = shm[0];
    } else {
      for (int64_t rv = 0; rv < C; ++rv) {
        int64_t t = rv, off = 0;
        for (int j = 0; j < nr; ++j) {
          const int64_t sz = x->sizes[rax[j]];
          off += (t % sz) * x->strides[rax[j]];
          t /= sz;
        }
        acc += ld(x->data, x->dtype, ib + off);
      }
    }
    if (mean) acc = acc / (float)C;
    st(out->data, out->dtype, ob, acc);
  }
  free(shm);
  return 0;
}

typedef struct run_ctx {
  const or_req* reqs;
  int n;
  atomic_int next;
} run_ctx;

static void run_one(const or_req* q) {
  if (q->kind == 0)
    oracle_ew(q->variant, q->p0, q->p1, &q->a, q->has_b ? &q->b : 0, &q->out);
  else
    oracle_reduce(q->variant == OR_MEAN, &q->a, &q->out, q->axes, q->naxes, q->keepdim, 256);
}

static void* run_worker(void* arg) {
  run_ctx* c = (run_ctx*)arg;
  for (;;) {
    const int i0 = atomic_fetch_add(&c->next, 4);
    if (i0 >= c->n) break;
    const int i1 = i0 + 4 < c->n ? i0 + 4 : c->n;
    for (int i = i0; i < i1; ++i) run_one(&c->reqs[i]);
  }
  return 0;
}

/* requests are independent: threads pull them four at a time */
int oracle_run(const or_req* reqs, int n, int nthreads) {
  if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
  if (nthreads < 1) nthreads = 1;
  if (nthreads > 256) nthreads = 256;
  run_ctx c;
  c.reqs = reqs;
  c.n = n;
  atomic_init(&c.next, 0);
  if (nthreads == 1) {
    run_worker(&c);
    return 1;
  }
  pthread_t th[256];
  int started = 0;
  for (int t = 0; t < nthreads - 1; ++t)
    if (pthread_create(&th[started], 0, run_worker, &c) == 0) ++started;
  run_worker(&c);
  for (int t = 0; t < started; ++t) pthread_join(th[t], 0);
  return started + 1;
}
