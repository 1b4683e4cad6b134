/* llmq_oracle.c - TEST INFRASTRUCTURE ONLY (see llmq_oracle.h).
 *
 * Compiled with -std=c11 (ISO mode: GCC does not contract a*b+c into FMA) and
 * without -ffast-math, so float reductions stay sequential and every product and
 * sum is rounded on its own, exactly as the reference is built (Makefile:5).
 */
#include "llmq_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* The reference's code rounding: (int)lrintf(v) then clamp to +-127
 * (quant.c:21-23 and quant.c:74-76 use the same three steps). */
static signed char code_of(float v) {
  int c = (int)lrintf(v);
  if (c > 127) c = 127;
  if (c < -127) c = -127;
  return (signed char)c;
}

void orc_quantize_int8_percol(const float *w, int rows, int cols, signed char *q, float *scale) {
  /* quant.c:10-27: column absmax, s = mx/127 (1 if zero), codes use 1/s. */
  for (int j = 0; j < cols; j++) {
    float amax = 0.0f;
    for (int i = 0; i < rows; i++) {
      const float a = fabsf(w[(size_t)i * cols + j]);
      if (a > amax) amax = a;
    }
    const float s = (amax > 0.0f) ? amax / 127.0f : 1.0f;
    const float r = 1.0f / s;
    scale[j] = s;
    for (int i = 0; i < rows; i++) q[(size_t)i * cols + j] = code_of(w[(size_t)i * cols + j] * r);
  }
}

void orc_dequantize_int8_percol(const signed char *q, const float *scale, int rows, int cols, float *w) {
  /* quant.c:29-33 */
  for (int i = 0; i < rows; i++)
    for (int j = 0; j < cols; j++) w[(size_t)i * cols + j] = (float)q[(size_t)i * cols + j] * scale[j];
}

float orc_quantize_row(const float *a, int K, signed char *qa) {
  /* quant.c:69-78 */
  float amax = 0.0f;
  for (int k = 0; k < K; k++) {
    const float t = fabsf(a[k]);
    if (t > amax) amax = t;
  }
  const float as = (amax > 0.0f) ? amax / 127.0f : 1.0f;
  const float r = 1.0f / as;
  for (int k = 0; k < K; k++) qa[k] = code_of(a[k] * r);
  return as;
}

void orc_qacc_columns(const signed char *qa, const signed char *qw, int K, int N, int32_t *acc) {
  /* matrix.c:358-368: integer sums, so the loop order cannot change the result. */
  for (int j = 0; j < N; j++) acc[j] = 0;
  for (int k = 0; k < K; k++) {
    const int32_t av = qa[k];
    const signed char *row = qw + (size_t)k * N;
    for (int j = 0; j < N; j++) acc[j] += av * (int32_t)row[j];
  }
}

void orc_qmatmul(const float *A, int M, int K, const signed char *wq, const float *wscale, int N,
                 float *C) {
  /* quant.c:60-85: per row: quantise, int32 accumulate, c = as * ws[j] * acc. */
  signed char *qa = (signed char *)malloc((size_t)K > 0 ? (size_t)K : 1);
  int32_t *acc = (int32_t *)malloc(((size_t)N > 0 ? (size_t)N : 1) * sizeof(int32_t));
  for (int m = 0; m < M; m++) {
    const float as = orc_quantize_row(A + (size_t)m * K, K, qa);
    orc_qacc_columns(qa, wq, K, N, acc);
    float *c = C + (size_t)m * N;
    for (int j = 0; j < N; j++) c[j] = as * wscale[j] * (float)acc[j];
  }
  free(qa);
  free(acc);
}

void orc_rmsnorm_row(const float *x, const float *gamma, int n, float eps, float *y) {
  /* rmsnorm.c:7-21: sequential sum of squares, times 1/n, r = 1/sqrtf(ms+eps),
   * y = (x*r)*gamma. */
  const float inv_n = 1.0f / (float)n;
  float ms = 0.0f;
  for (int j = 0; j < n; j++) ms += x[j] * x[j];
  ms *= inv_n;
  const float r = 1.0f / sqrtf(ms + eps);
  for (int j = 0; j < n; j++) y[j] = x[j] * r * gamma[j];
}

void orc_rope_heads_pos_row(float *x, int n_heads, int head_dim, float base, int pos) {
  /* rope.c:48-68 (one row): rotate_half pairs (k, k+hd/2) of every head by
   * pos * base^(-2k/hd). */
  const int half = head_dim / 2;
  for (int h = 0; h < n_heads; h++) {
    float *xh = x + (size_t)h * head_dim;
    for (int k = 0; k < half; k++) {
      const float inv_freq = powf(base, -2.0f * (float)k / (float)head_dim);
      const float ang = (float)pos * inv_freq;
      const float c = cosf(ang), s = sinf(ang);
      const float x1 = xh[k], x2 = xh[k + half];
      xh[k] = x1 * c - x2 * s;
      xh[k + half] = x2 * c + x1 * s;
    }
  }
}

int orc_argmax(const float *r, int n) {
  /* sampler.c:8-21: strict '>' keeps the first of equal maxima. */
  int best = 0;
  float bv = r[0];
  for (int j = 1; j < n; j++)
    if (r[j] > bv) { bv = r[j]; best = j; }
  return best;
}

/* sampler.c:32-39 */
unsigned long long orc_xorshift64(unsigned long long *state) {
  unsigned long long x = *state;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *state = x;
  return x;
}

typedef struct {
  float p;
  int idx;
} OrcCand;

/* p descending, then index ascending: the order glibc's stable qsort leaves
 * the reference's (p, index) array in (sampler.c:54-58, 84), as a total order. */
static int orc_cand_order(const void *a, const void *b) {
  const OrcCand *x = (const OrcCand *)a, *y = (const OrcCand *)b;
  if (x->p > y->p) return -1;
  if (x->p < y->p) return 1;
  return (x->idx > y->idx) - (x->idx < y->idx);
}

int orc_sample_token(const float *l, int V, float temperature, int top_k, float top_p,
                     unsigned long long *state) {
  if (temperature <= 0.0f) return orc_argmax(l, V); /* sampler.c:65-67 */
  float mx = l[0];                                  /* sampler.c:70-71 */
  for (int j = 1; j < V; j++)
    if (l[j] > mx) mx = l[j];
  OrcCand *c = (OrcCand *)malloc((size_t)V * sizeof(OrcCand));
  float sum = 0.0f; /* sampler.c:74-81 */
  for (int j = 0; j < V; j++) {
    const float e = expf((l[j] - mx) / temperature);
    c[j].p = e;
    c[j].idx = j;
    sum += e;
  }
  for (int j = 0; j < V; j++) c[j].p /= sum;
  qsort(c, (size_t)V, sizeof(OrcCand), orc_cand_order);
  int keep = (top_k > 0 && top_k < V) ? top_k : V; /* sampler.c:87-99 */
  if (top_p > 0.0f && top_p < 1.0f) {
    float cum = 0.0f;
    int n = 0;
    while (n < keep) {
      cum += c[n++].p;
      if (cum >= top_p) break;
    }
    keep = n;
  }
  if (keep < 1) keep = 1;
  float z = 0.0f; /* sampler.c:102-111 */
  for (int i = 0; i < keep; i++) z += c[i].p;
  const float u = (float)((double)(orc_xorshift64(state) >> 11) * (1.0 / 9007199254740992.0)) * z;
  int chosen = c[keep - 1].idx;
  float run = 0.0f;
  for (int i = 0; i < keep; i++) {
    run += c[i].p;
    if (u <= run) {
      chosen = c[i].idx;
      break;
    }
  }
  free(c);
  return chosen;
}

LlamaKV orc_kv_create(const QLlamaModel *m) {
  /* llama.c:513-526 */
  LlamaKV kv;
  kv.n_layers = m->n_layers;
  kv.max_seq = m->max_seq;
  kv.kv_dim = m->n_kv * m->head_dim;
  kv.len = 0;
  kv.k = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  kv.v = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  for (int l = 0; l < m->n_layers; l++) {
    kv.k[l] = (float *)calloc((size_t)m->max_seq * kv.kv_dim, sizeof(float));
    kv.v[l] = (float *)calloc((size_t)m->max_seq * kv.kv_dim, sizeof(float));
  }
  return kv;
}

void orc_kv_free(LlamaKV *kv) {
  for (int l = 0; l < kv->n_layers; l++) { free(kv->k[l]); free(kv->v[l]); }
  free(kv->k);
  free(kv->v);
  kv->k = kv->v = NULL;
}

static void qlinear(const float *x, int K, const QTensor *W, float *out) {
  orc_qmatmul(x, 1, K, W->q, W->scale, W->cols, out);
}

/* llama.c:554-576 (and llama.c:326-341, the same code in the fp32 step): per
 * query head, scores over 0..pos, softmax, weighted values; kc / vc hold one
 * layer's cache rows [pos][n_kv * hd]. */
static void orc_attend(const float *q, const float *kc, const float *vc, int n_heads, int n_kv, int hd, int pos,
                       float *sc, float *o) {
  const int kvd = n_kv * hd, group = n_heads / n_kv;
  const float att_scale = 1.0f / sqrtf((float)hd);
  for (int h = 0; h < n_heads; h++) {
    const int kh = h / group;
    const float *qh = q + (size_t)h * hd;
    float mx = -INFINITY;
    for (int p = 0; p <= pos; p++) {
      const float *kp = kc + (size_t)p * kvd + (size_t)kh * hd;
      float dot = 0.0f;
      for (int d = 0; d < hd; d++) dot += qh[d] * kp[d];
      const float s = dot * att_scale;
      sc[p] = s;
      if (s > mx) mx = s;
    }
    float sum = 0.0f;
    for (int p = 0; p <= pos; p++) {
      const float e = expf(sc[p] - mx);
      sc[p] = e;
      sum += e;
    }
    const float inv = 1.0f / sum;
    float *oh = o + (size_t)h * hd;
    for (int d = 0; d < hd; d++) oh[d] = 0.0f;
    for (int p = 0; p <= pos; p++) {
      const float w = sc[p] * inv;
      const float *vp = vc + (size_t)p * kvd + (size_t)kh * hd;
      for (int d = 0; d < hd; d++) oh[d] += w * vp[d];
    }
  }
}

void orc_decode_step(const QLlamaModel *m, LlamaKV *kv, int token, float *logits) {
  /* llama.c:528-600, one token at position kv->len. */
  const int dm = m->d_model, hd = m->head_dim, dff = m->d_ff;
  const int qd = m->n_heads * hd, kvd = m->n_kv * hd;
  const int pos = kv->len;

  float *x = (float *)calloc((size_t)dm, sizeof(float));
  float *xn = (float *)calloc((size_t)dm, sizeof(float));
  float *q = (float *)calloc((size_t)qd, sizeof(float));
  float *k = (float *)calloc((size_t)kvd, sizeof(float));
  float *v = (float *)calloc((size_t)kvd, sizeof(float));
  float *o = (float *)calloc((size_t)qd, sizeof(float));
  float *t = (float *)calloc((size_t)dm, sizeof(float));
  float *g = (float *)calloc((size_t)dff, sizeof(float));
  float *u = (float *)calloc((size_t)dff, sizeof(float));
  float *sc = (float *)calloc((size_t)pos + 1, sizeof(float));

  /* llama.c:535-536: embedding row, dequantised */
  for (int j = 0; j < dm; j++) x[j] = (float)m->wte.q[(size_t)token * dm + j] * m->wte.scale[j];

  for (int l = 0; l < m->n_layers; l++) {
    const QLlamaBlock *b = &m->blocks[l];
    /* llama.c:545-552 */
    orc_rmsnorm_row(x, b->attn_norm.data, dm, m->eps, xn);
    qlinear(xn, dm, &b->Wq, q);
    for (int j = 0; j < qd; j++) q[j] = q[j] + b->b_q.data[j];
    qlinear(xn, dm, &b->Wk, k);
    for (int j = 0; j < kvd; j++) k[j] = k[j] + b->b_k.data[j];
    qlinear(xn, dm, &b->Wv, v);
    for (int j = 0; j < kvd; j++) v[j] = v[j] + b->b_v.data[j];
    orc_rope_heads_pos_row(q, m->n_heads, hd, m->rope_base, pos);
    orc_rope_heads_pos_row(k, m->n_kv, hd, m->rope_base, pos);
    memcpy(kv->k[l] + (size_t)pos * kvd, k, (size_t)kvd * sizeof(float));
    memcpy(kv->v[l] + (size_t)pos * kvd, v, (size_t)kvd * sizeof(float));

    orc_attend(q, kv->k[l], kv->v[l], m->n_heads, m->n_kv, hd, pos, sc, o);  /* llama.c:554-576 */
    /* llama.c:577-578 */
    qlinear(o, qd, &b->Wo, t);
    for (int j = 0; j < dm; j++) x[j] += t[j];
    /* llama.c:580-589 */
    orc_rmsnorm_row(x, b->ffn_norm.data, dm, m->eps, xn);
    qlinear(xn, dm, &b->Wgate, g);
    qlinear(xn, dm, &b->Wup, u);
    for (int j = 0; j < dff; j++) {
      const float z = g[j];
      const float s = 1.0f / (1.0f + expf(-z));
      g[j] = (z * s) * u[j];
    }
    qlinear(g, dff, &b->Wdown, t);
    for (int j = 0; j < dm; j++) x[j] += t[j];
  }
  /* llama.c:592-594 */
  orc_rmsnorm_row(x, m->final_norm.data, dm, m->eps, xn);
  qlinear(xn, dm, &m->lm_head, logits);
  kv->len = pos + 1;

  free(x); free(xn); free(q); free(k); free(v); free(o); free(t); free(g); free(u); free(sc);
}

/* ------------------------------------------------------- fp32 (LLMA) step */

/* matrix.c:178-191 for one row: c[j] = 0, then c[j] += a[k] * W[k][j] for
 * k in order (one rounded product and one rounded sum per term). */
static void flinear(const float *a, int K, const Tensor *W, float *c) {
  const int N = W->shape[1];
  for (int j = 0; j < N; j++) c[j] = 0.0f;
  for (int k = 0; k < K; k++) {
    const float ak = a[k];
    const float *wk = W->data + (size_t)k * N;
    for (int j = 0; j < N; j++) c[j] += ak * wk[j];
  }
}

LlamaKV orc_f32_kv_create(const LlamaModel *m) {
  /* llama.c:275-288 */
  LlamaKV kv;
  kv.n_layers = m->n_layers;
  kv.max_seq = m->max_seq;
  kv.kv_dim = m->n_kv * m->head_dim;
  kv.len = 0;
  kv.k = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  kv.v = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  for (int l = 0; l < m->n_layers; l++) {
    kv.k[l] = (float *)calloc((size_t)m->max_seq * kv.kv_dim, sizeof(float));
    kv.v[l] = (float *)calloc((size_t)m->max_seq * kv.kv_dim, sizeof(float));
  }
  return kv;
}

void orc_f32_decode_step(const LlamaModel *m, LlamaKV *kv, int token, float *logits) {
  /* llama.c:296-362, one token at position kv->len. */
  const int dm = m->d_model, hd = m->head_dim, dff = m->d_ff;
  const int qd = m->n_heads * hd, kvd = m->n_kv * hd;
  const int pos = kv->len;
  float *x = (float *)calloc((size_t)dm, sizeof(float));
  float *xn = (float *)calloc((size_t)dm, sizeof(float));
  float *q = (float *)calloc((size_t)qd, sizeof(float));
  float *k = (float *)calloc((size_t)kvd, sizeof(float));
  float *v = (float *)calloc((size_t)kvd, sizeof(float));
  float *o = (float *)calloc((size_t)qd, sizeof(float));
  float *t = (float *)calloc((size_t)dm, sizeof(float));
  float *g = (float *)calloc((size_t)dff, sizeof(float));
  float *u = (float *)calloc((size_t)dff, sizeof(float));
  float *sc = (float *)calloc((size_t)pos + 1, sizeof(float));

  for (int j = 0; j < dm; j++) x[j] = m->wte.data[(size_t)token * dm + j]; /* llama.c:302-303 */
  for (int l = 0; l < m->n_layers; l++) {
    const LlamaBlock *b = &m->blocks[l];
    /* llama.c:312-322 */
    orc_rmsnorm_row(x, b->attn_norm.data, dm, m->eps, xn);
    flinear(xn, dm, &b->Wq, q);
    for (int j = 0; j < qd; j++) q[j] = q[j] + b->b_q.data[j];
    flinear(xn, dm, &b->Wk, k);
    for (int j = 0; j < kvd; j++) k[j] = k[j] + b->b_k.data[j];
    flinear(xn, dm, &b->Wv, v);
    for (int j = 0; j < kvd; j++) v[j] = v[j] + b->b_v.data[j];
    orc_rope_heads_pos_row(q, m->n_heads, hd, m->rope_base, pos);
    orc_rope_heads_pos_row(k, m->n_kv, hd, m->rope_base, pos);
    memcpy(kv->k[l] + (size_t)pos * kvd, k, (size_t)kvd * sizeof(float));
    memcpy(kv->v[l] + (size_t)pos * kvd, v, (size_t)kvd * sizeof(float));
    orc_attend(q, kv->k[l], kv->v[l], m->n_heads, m->n_kv, hd, pos, sc, o); /* llama.c:324-341 */
    /* llama.c:342-343 */
    flinear(o, qd, &b->Wo, t);
    for (int j = 0; j < dm; j++) x[j] += t[j];
    /* llama.c:346-348 over swiglu.c:33-43 */
    orc_rmsnorm_row(x, b->ffn_norm.data, dm, m->eps, xn);
    flinear(xn, dm, &b->Wgate, g);
    flinear(xn, dm, &b->Wup, u);
    for (int j = 0; j < dff; j++) {
      const float z = g[j];
      const float s = 1.0f / (1.0f + expf(-z)); /* swiglu.c:9-12 */
      const float a = z * s;
      g[j] = a * u[j];
    }
    flinear(g, dff, &b->Wdown, t);
    for (int j = 0; j < dm; j++) x[j] += t[j];
  }
  /* llama.c:351-353 */
  orc_rmsnorm_row(x, m->final_norm.data, dm, m->eps, xn);
  flinear(xn, dm, &m->lm_head, logits);
  kv->len = pos + 1;

  free(x); free(xn); free(q); free(k); free(v); free(o); free(t); free(g); free(u); free(sc);
}

/* ---------------------------------------------------------------- LLMQ I/O */

#define ORC_LLMQ_MAGIC 0x514D4C4Cu /* llama.c:193 */
#define ORC_VERSION 2u             /* llama.c:194 */

static Tensor vec_alloc(int n) {
  Tensor t;
  t.ndim = 1;
  t.shape = (int *)malloc(sizeof(int));
  t.shape[0] = n;
  t.size = (size_t)n;
  t.data = (float *)calloc((size_t)n, sizeof(float));
  t.grad = NULL;
  return t;
}
static void vec_free(Tensor *t) {
  free(t->data);
  free(t->shape);
  t->data = NULL;
  t->shape = NULL;
}
static QTensor qt_alloc(int rows, int cols) {
  QTensor t;
  t.rows = rows;
  t.cols = cols;
  t.q = (signed char *)malloc((size_t)rows * cols);
  t.scale = (float *)malloc((size_t)cols * sizeof(float));
  return t;
}
static void qt_free(QTensor *t) {
  free(t->q);
  free(t->scale);
  t->q = NULL;
  t->scale = NULL;
}

static QLlamaModel model_alloc(const int32_t *c, const float *f) {
  /* llama.c:447-481 shapes */
  QLlamaModel m;
  m.vocab = c[0]; m.d_model = c[1]; m.n_layers = c[2]; m.n_heads = c[3];
  m.n_kv = c[4]; m.head_dim = c[5]; m.d_ff = c[6]; m.max_seq = c[7];
  m.rope_base = f[0]; m.eps = f[1];
  const int qd = m.n_heads * m.head_dim, kvd = m.n_kv * m.head_dim;
  m.wte = qt_alloc(m.vocab, m.d_model);
  m.blocks = (QLlamaBlock *)malloc((size_t)m.n_layers * sizeof(QLlamaBlock));
  for (int l = 0; l < m.n_layers; l++) {
    QLlamaBlock *b = &m.blocks[l];
    b->attn_norm = vec_alloc(m.d_model);
    b->ffn_norm = vec_alloc(m.d_model);
    b->b_q = vec_alloc(qd);
    b->b_k = vec_alloc(kvd);
    b->b_v = vec_alloc(kvd);
    b->Wq = qt_alloc(m.d_model, qd);
    b->Wk = qt_alloc(m.d_model, kvd);
    b->Wv = qt_alloc(m.d_model, kvd);
    b->Wo = qt_alloc(qd, m.d_model);
    b->Wgate = qt_alloc(m.d_model, m.d_ff);
    b->Wup = qt_alloc(m.d_model, m.d_ff);
    b->Wdown = qt_alloc(m.d_ff, m.d_model);
  }
  m.final_norm = vec_alloc(m.d_model);
  m.lm_head = qt_alloc(m.d_model, m.vocab);
  return m;
}

void orc_model_free(QLlamaModel *m) {
  qt_free(&m->wte);
  for (int l = 0; l < m->n_layers; l++) {
    QLlamaBlock *b = &m->blocks[l];
    vec_free(&b->attn_norm); vec_free(&b->ffn_norm);
    vec_free(&b->b_q); vec_free(&b->b_k); vec_free(&b->b_v);
    qt_free(&b->Wq); qt_free(&b->Wk); qt_free(&b->Wv); qt_free(&b->Wo);
    qt_free(&b->Wgate); qt_free(&b->Wup); qt_free(&b->Wdown);
  }
  free(m->blocks);
  m->blocks = NULL;
  vec_free(&m->final_norm);
  qt_free(&m->lm_head);
}

static int rd(FILE *f, void *p, size_t sz, size_t n) { return fread(p, sz, n, f) == n; }
static int rdq(FILE *f, QTensor *t) {
  /* llama.c:603-608: scales then codes */
  return rd(f, t->scale, sizeof(float), (size_t)t->cols) &&
         rd(f, t->q, 1, (size_t)t->rows * t->cols);
}

static int cfg_ok(const int32_t *c) {
  /* llama.c:371-386 */
  for (int i = 0; i < 8; i++)
    if (c[i] <= 0 || c[i] > 1000000) return 0;
  if (c[3] % c[4] != 0) return 0;
  const long long qd = (long long)c[3] * c[5], kvd = (long long)c[4] * c[5];
  if (qd > 1000000 || kvd > 1000000) return 0;
  if ((long long)c[0] * c[1] > 2147483647LL) return 0;
  if ((long long)c[1] * c[6] > 2147483647LL) return 0;
  if (qd * c[1] > 2147483647LL) return 0;
  return 1;
}

int orc_model_load(const char *path, QLlamaModel *out) {
  /* llama.c:610-657 */
  FILE *f = fopen(path, "rb");
  if (!f) return 1;
  uint32_t hdr[2];
  int32_t c[8];
  float fc[2];
  if (!rd(f, hdr, 4, 2) || !rd(f, c, 4, 8) || !rd(f, fc, 4, 2)) { fclose(f); return 1; }
  if (hdr[0] != ORC_LLMQ_MAGIC || hdr[1] != ORC_VERSION || !cfg_ok(c)) { fclose(f); return 1; }
  *out = model_alloc(c, fc);
  const size_t dm = (size_t)out->d_model;
  int ok = rdq(f, &out->wte);
  for (int l = 0; l < out->n_layers && ok; l++) {
    QLlamaBlock *b = &out->blocks[l];
    ok = ok && rd(f, b->attn_norm.data, 4, dm);
    ok = ok && rdq(f, &b->Wq) && rdq(f, &b->Wk) && rdq(f, &b->Wv);
    ok = ok && rd(f, b->b_q.data, 4, b->b_q.size) && rd(f, b->b_k.data, 4, b->b_k.size) &&
         rd(f, b->b_v.data, 4, b->b_v.size);
    ok = ok && rdq(f, &b->Wo);
    ok = ok && rd(f, b->ffn_norm.data, 4, dm);
    ok = ok && rdq(f, &b->Wgate) && rdq(f, &b->Wup) && rdq(f, &b->Wdown);
  }
  ok = ok && rd(f, out->final_norm.data, 4, dm);
  ok = ok && rdq(f, &out->lm_head);
  fclose(f);
  if (!ok) { orc_model_free(out); return 1; }
  return 0;
}

static int wr(FILE *f, const void *p, size_t sz, size_t n) { return fwrite(p, sz, n, f) == n; }
static int wrq(FILE *f, const QTensor *t) {
  return wr(f, t->scale, sizeof(float), (size_t)t->cols) && wr(f, t->q, 1, (size_t)t->rows * t->cols);
}

int orc_model_save(const char *path, const QLlamaModel *m) {
  FILE *f = fopen(path, "wb");
  if (!f) return 1;
  const uint32_t hdr[2] = {ORC_LLMQ_MAGIC, ORC_VERSION};
  const int32_t c[8] = {m->vocab, m->d_model, m->n_layers, m->n_heads,
                        m->n_kv, m->head_dim, m->d_ff, m->max_seq};
  const float fc[2] = {m->rope_base, m->eps};
  int ok = wr(f, hdr, 4, 2) && wr(f, c, 4, 8) && wr(f, fc, 4, 2);
  ok = ok && wrq(f, &m->wte);
  for (int l = 0; l < m->n_layers && ok; l++) {
    const QLlamaBlock *b = &m->blocks[l];
    ok = ok && wr(f, b->attn_norm.data, 4, (size_t)m->d_model);
    ok = ok && wrq(f, &b->Wq) && wrq(f, &b->Wk) && wrq(f, &b->Wv);
    ok = ok && wr(f, b->b_q.data, 4, b->b_q.size) && wr(f, b->b_k.data, 4, b->b_k.size) &&
         wr(f, b->b_v.data, 4, b->b_v.size);
    ok = ok && wrq(f, &b->Wo);
    ok = ok && wr(f, b->ffn_norm.data, 4, (size_t)m->d_model);
    ok = ok && wrq(f, &b->Wgate) && wrq(f, &b->Wup) && wrq(f, &b->Wdown);
  }
  ok = ok && wr(f, m->final_norm.data, 4, (size_t)m->d_model);
  ok = ok && wrq(f, &m->lm_head);
  ok = (fclose(f) == 0) && ok;
  return ok ? 0 : 1;
}

QLlamaModel orc_quantize_from(const LlamaModel *s) {
  /* llama.c:490-511 */
  const int32_t c[8] = {s->vocab, s->d_model, s->n_layers, s->n_heads,
                        s->n_kv, s->head_dim, s->d_ff, s->max_seq};
  const float fc[2] = {s->rope_base, s->eps};
  QLlamaModel m = model_alloc(c, fc);
  const size_t dmb = (size_t)s->d_model * sizeof(float);
#define QT(dst, src) orc_quantize_int8_percol((src).data, (dst).rows, (dst).cols, (dst).q, (dst).scale)
  QT(m.wte, s->wte);
  for (int l = 0; l < s->n_layers; l++) {
    const LlamaBlock *a = &s->blocks[l];
    QLlamaBlock *b = &m.blocks[l];
    memcpy(b->attn_norm.data, a->attn_norm.data, dmb);
    memcpy(b->ffn_norm.data, a->ffn_norm.data, dmb);
    memcpy(b->b_q.data, a->b_q.data, a->b_q.size * sizeof(float));
    memcpy(b->b_k.data, a->b_k.data, a->b_k.size * sizeof(float));
    memcpy(b->b_v.data, a->b_v.data, a->b_v.size * sizeof(float));
    QT(b->Wq, a->Wq); QT(b->Wk, a->Wk); QT(b->Wv, a->Wv); QT(b->Wo, a->Wo);
    QT(b->Wgate, a->Wgate); QT(b->Wup, a->Wup); QT(b->Wdown, a->Wdown);
  }
  memcpy(m.final_norm.data, s->final_norm.data, dmb);
  QT(m.lm_head, s->lm_head);
#undef QT
  return m;
}

/* ------------------------------------------------------------ host expf */
typedef struct {
  uint32_t first;
  uint64_t lo, hi;
  float *out;
} ExpJob;

static void *exp_job(void *arg) {
  ExpJob *j = (ExpJob *)arg;
  for (uint64_t i = j->lo; i < j->hi; i++) {
    const uint32_t u = (uint32_t)(j->first + i);
    float x;
    memcpy(&x, &u, 4);
    j->out[i] = expf(x);
  }
  return NULL;
}

void orc_expf_bits(uint32_t first, uint64_t count, float *out) {
  long nt = sysconf(_SC_NPROCESSORS_ONLN);
  if (nt < 1) nt = 1;
  if (nt > 64) nt = 64;
  pthread_t th[64];
  ExpJob jobs[64];
  for (long t = 0; t < nt; t++) {
    jobs[t].first = first;
    jobs[t].lo = count * (uint64_t)t / (uint64_t)nt;
    jobs[t].hi = count * (uint64_t)(t + 1) / (uint64_t)nt;
    jobs[t].out = out;
    pthread_create(&th[t], NULL, exp_job, &jobs[t]);
  }
  for (long t = 0; t < nt; t++) pthread_join(th[t], NULL);
}
