/* llmq_host.c - C11 host layer of libllmq_cuda.so: the quant.h / llama.h entry
 * points, host allocation with the reference's conventions, the LLMQ v2 reader
 * and writer, error reporting, and the RoPE angle tables.  All arithmetic on
 * the data runs on the GPU through llmq_dev.cu.
 *
 * Built with -std=c11 (no FMA contraction), like the reference.
 */
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "llmq_internal.h"

/* ------------------------------------------------------------------ errors */
static _Thread_local int tl_err = LLMQ_OK;
static _Thread_local char tl_msg[512];

void llmq_set_error(int code, const char *fmt, ...) {
  tl_err = code;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(tl_msg, sizeof tl_msg, fmt, ap);
  va_end(ap);
  fprintf(stderr, "%s\n", tl_msg);
}

LLMQ_API int q_llama_last_error(void) { return tl_err; }
LLMQ_API const char *q_llama_last_error_message(void) { return tl_err == LLMQ_OK ? "" : tl_msg; }
LLMQ_API void q_llama_clear_error(void) {
  tl_err = LLMQ_OK;
  tl_msg[0] = '\0';
}

/* --------------------------------------------------------- host allocation */
/* 64-byte aligned, zero-filled f32 vector with a malloc'd shape, the allocation
 * pattern of tensor.c:33-60 (so tensor_free can release it). */
static Tensor vec_new(int n) {
  Tensor t;
  t.ndim = 1;
  t.shape = (int *)malloc(sizeof(int));
  t.size = (size_t)n;
  size_t bytes = ((size_t)n * sizeof(float) + 63) & ~(size_t)63;
  t.data = (float *)aligned_alloc(64, bytes ? bytes : 64);
  t.grad = NULL;
  if (!t.shape || !t.data) {
    fprintf(stderr, "Error: aligned allocation failed\n");
    exit(EXIT_FAILURE);
  }
  t.shape[0] = n;
  memset(t.data, 0, bytes ? bytes : 64);
  return t;
}
static void vec_del(Tensor *t) {
  free(t->data);
  free(t->shape);
  t->data = NULL;
  t->shape = NULL;
}

/* --------------------------------------------------------------------- RoPE */
void llmq_rope_tables(float base, int head_dim, int max_seq, float *cos_out, float *sin_out) {
  /* The angle of pair k at position pos, evaluated as rope.c:59-61 does. */
  const int half = head_dim / 2;
  for (int pos = 0; pos < max_seq; pos++) {
    for (int k = 0; k < half; k++) {
      const float inv_freq = powf(base, -2.0f * (float)k / (float)head_dim);
      const float ang = (float)pos * inv_freq;
      cos_out[(size_t)pos * half + k] = cosf(ang);
      sin_out[(size_t)pos * half + k] = sinf(ang);
    }
  }
}

/* ------------------------------------------------------------------ quant.h */
LLMQ_API void quantize_int8_percol(const float *w, int rows, int cols, signed char *q, float *scale) {
  if (!llmqd_quantize(w, rows, cols, q, scale))
    fprintf(stderr, "quantize_int8_percol: failed (%s)\n", q_llama_last_error_message());
}

LLMQ_API void dequantize_int8_percol(const signed char *q, const float *scale, int rows, int cols, float *w) {
  if (!llmqd_dequantize(q, scale, rows, cols, w))
    fprintf(stderr, "dequantize_int8_percol: failed (%s)\n", q_llama_last_error_message());
}

LLMQ_API QTensor qtensor_create(int rows, int cols) {
  QTensor t;
  t.rows = rows;
  t.cols = cols;
  const size_t nq = (size_t)rows * (size_t)cols;
  t.q = (signed char *)malloc(nq > 0 ? nq : 1);
  t.scale = (float *)malloc(((size_t)cols ? (size_t)cols : 1) * sizeof(float));
  return t;
}

LLMQ_API void qtensor_free(QTensor *t) {
  free(t->q);
  free(t->scale);
  t->q = NULL;
  t->scale = NULL;
}

LLMQ_API void qtensor_quantize(QTensor *t, const float *w) {
  quantize_int8_percol(w, t->rows, t->cols, t->q, t->scale);
}

LLMQ_API void qmatmul(const Tensor *A, const QTensor *W, Tensor *C) {
  const int M = A->shape[0], K = W->rows, N = W->cols;
  if (A->ndim != 2 || A->shape[1] != K || A->size != (size_t)M * K || C->size < (size_t)M * N) {
    llmq_set_error(LLMQ_ERR_ARG, "qmatmul: bad shapes A(%d,%d) @ W(%d,%d) -> C(%zu elements)", M,
                   A->ndim > 1 ? A->shape[1] : -1, K, N, C->size);
    return;
  }
  if (!llmqd_qmatmul(A->data, M, W, C->data))
    fprintf(stderr, "qmatmul: failed (%s)\n", q_llama_last_error_message());
}

/* ------------------------------------------------------------------ models */
#define LLMQ_MAGIC 0x514D4C4Cu /* 'LLMQ' (llama.c:193) */
#define LLMQ_VERSION 2u        /* llama.c:194 */

static QLlamaModel model_alloc(const int32_t *c, const float *f) {
  /* shapes of llama.c:447-481 */
  QLlamaModel m;
  m.vocab = c[0];
  m.d_model = c[1];
  m.n_layers = c[2];
  m.n_heads = c[3];
  m.n_kv = c[4];
  m.head_dim = c[5];
  m.d_ff = c[6];
  m.max_seq = c[7];
  m.rope_base = f[0];
  m.eps = f[1];
  const int qd = m.n_heads * m.head_dim, kvd = m.n_kv * m.head_dim;
  m.wte = qtensor_create(m.vocab, m.d_model);
  m.blocks = (QLlamaBlock *)malloc((size_t)m.n_layers * sizeof(QLlamaBlock));
  for (int l = 0; l < m.n_layers; l++) {
    QLlamaBlock *b = &m.blocks[l];
    b->attn_norm = vec_new(m.d_model);
    b->ffn_norm = vec_new(m.d_model);
    b->b_q = vec_new(qd);
    b->b_k = vec_new(kvd);
    b->b_v = vec_new(kvd);
    b->Wq = qtensor_create(m.d_model, qd);
    b->Wk = qtensor_create(m.d_model, kvd);
    b->Wv = qtensor_create(m.d_model, kvd);
    b->Wo = qtensor_create(qd, m.d_model);
    b->Wgate = qtensor_create(m.d_model, m.d_ff);
    b->Wup = qtensor_create(m.d_model, m.d_ff);
    b->Wdown = qtensor_create(m.d_ff, m.d_model);
  }
  m.final_norm = vec_new(m.d_model);
  m.lm_head = qtensor_create(m.d_model, m.vocab);
  return m;
}

static void qt_release(QTensor *t) {
  free(t->q);
  free(t->scale);
  t->q = NULL;
  t->scale = NULL;
}

LLMQ_API void q_llama_model_free(QLlamaModel *m) {
  llmqd_model_release(m);
  qt_release(&m->wte);
  for (int l = 0; l < m->n_layers; l++) {
    QLlamaBlock *b = &m->blocks[l];
    vec_del(&b->attn_norm);
    vec_del(&b->ffn_norm);
    vec_del(&b->b_q);
    vec_del(&b->b_k);
    vec_del(&b->b_v);
    qt_release(&b->Wq);
    qt_release(&b->Wk);
    qt_release(&b->Wv);
    qt_release(&b->Wo);
    qt_release(&b->Wgate);
    qt_release(&b->Wup);
    qt_release(&b->Wdown);
  }
  free(m->blocks);
  m->blocks = NULL;
  vec_del(&m->final_norm);
  qt_release(&m->lm_head);
}

/* Header sanity (llama.c:371-386): positive bounded dims, GQA groups that divide,
 * and 2-D element counts that fit an int. */
int llmq_config_valid(const int32_t *c) {
  const int32_t maxd = 1000000;
  for (int i = 0; i < 8; i++)
    if (c[i] <= 0 || c[i] > maxd) return 0;
  if (c[3] % c[4] != 0) return 0;
  const long long qd = (long long)c[3] * c[5], kvd = (long long)c[4] * c[5];
  if (qd > maxd || kvd > maxd) return 0;
  if ((long long)c[0] * c[1] > 2147483647LL) return 0;
  if ((long long)c[1] * c[6] > 2147483647LL) return 0;
  if (qd * c[1] > 2147483647LL) return 0;
  return 1;
}

static int rd(FILE *f, void *p, size_t sz, size_t n) { return fread(p, sz, n, f) == n; }
static int rd_q(FILE *f, QTensor *t) {
  return rd(f, t->scale, sizeof(float), (size_t)t->cols) && rd(f, t->q, 1, (size_t)t->rows * t->cols);
}

LLMQ_API int q_llama_model_load(const char *path, QLlamaModel *out) {
  FILE *f = fopen(path, "rb");
  if (!f) {
    fprintf(stderr, "Error: cannot open '%s' for reading\n", path);
    llmq_set_error(LLMQ_ERR_IO, "q_llama_model_load: cannot open '%s'", path);
    return 1;
  }
  uint32_t hdr[2];
  int32_t cfg[8];
  float fcfg[2];
  if (!rd(f, hdr, sizeof(uint32_t), 2) || !rd(f, cfg, sizeof(int32_t), 8) || !rd(f, fcfg, sizeof(float), 2)) {
    fprintf(stderr, "Error: '%s' is truncated (bad header)\n", path);
    fclose(f);
    return 1;
  }
  if (hdr[0] != LLMQ_MAGIC || hdr[1] != LLMQ_VERSION) {
    fprintf(stderr, "Error: '%s' is not a v%u int8 LLMQ checkpoint\n", path, LLMQ_VERSION);
    fclose(f);
    return 1;
  }
  if (!llmq_config_valid(cfg)) {
    fprintf(stderr, "Error: '%s' has an invalid/unsupported config\n", path);
    fclose(f);
    return 1;
  }
  *out = model_alloc(cfg, fcfg);
  const size_t dm = (size_t)out->d_model;
  int ok = rd_q(f, &out->wte);
  for (int l = 0; l < out->n_layers && ok; l++) {
    QLlamaBlock *b = &out->blocks[l];
    ok = ok && rd(f, b->attn_norm.data, sizeof(float), dm);
    ok = ok && rd_q(f, &b->Wq) && rd_q(f, &b->Wk) && rd_q(f, &b->Wv);
    ok = ok && rd(f, b->b_q.data, sizeof(float), b->b_q.size) && rd(f, b->b_k.data, sizeof(float), b->b_k.size) &&
         rd(f, b->b_v.data, sizeof(float), b->b_v.size);
    ok = ok && rd_q(f, &b->Wo);
    ok = ok && rd(f, b->ffn_norm.data, sizeof(float), dm);
    ok = ok && rd_q(f, &b->Wgate) && rd_q(f, &b->Wup) && rd_q(f, &b->Wdown);
  }
  ok = ok && rd(f, out->final_norm.data, sizeof(float), dm);
  ok = ok && rd_q(f, &out->lm_head);
  fclose(f);
  if (!ok) {
    fprintf(stderr, "Error: '%s' is truncated (bad weights)\n", path);
    q_llama_model_free(out);
    return 1;
  }
  /* with a tensor-parallel group formed the whole model is only read: it is
   * meant to be cut with q_llama_model_shard, and each shard uploads itself */
  if (llmqd_tp_world() <= 1 && !llmqd_model_upload(out)) {
    fprintf(stderr, "Error: '%s' could not be placed on the GPU (%s)\n", path, q_llama_last_error_message());
    q_llama_model_free(out);
    return 1;
  }
  return 0;
}

static int wr(FILE *f, const void *p, size_t sz, size_t n) { return fwrite(p, sz, n, f) == n; }
static int wr_q(FILE *f, const QTensor *t) {
  return wr(f, t->scale, sizeof(float), (size_t)t->cols) && wr(f, t->q, 1, (size_t)t->rows * t->cols);
}

LLMQ_API int q_llama_model_save(const char *path, const QLlamaModel *m) {
  /* Same atomic tmp + rename discipline as llama.c:230-269. */
  const size_t plen = strlen(path);
  char *tmp = (char *)malloc(plen + 5);
  if (!tmp) {
    fprintf(stderr, "Error: out of memory saving '%s'\n", path);
    return 1;
  }
  memcpy(tmp, path, plen);
  memcpy(tmp + plen, ".tmp", 5);
  FILE *f = fopen(tmp, "wb");
  if (!f) {
    fprintf(stderr, "Error: cannot open '%s' for writing\n", tmp);
    free(tmp);
    return 1;
  }
  const uint32_t hdr[2] = {LLMQ_MAGIC, LLMQ_VERSION};
  const int32_t cfg[8] = {m->vocab, m->d_model, m->n_layers, m->n_heads, m->n_kv, m->head_dim, m->d_ff, m->max_seq};
  const float fcfg[2] = {m->rope_base, m->eps};
  int ok = wr(f, hdr, sizeof(uint32_t), 2) && wr(f, cfg, sizeof(int32_t), 8) && wr(f, fcfg, sizeof(float), 2);
  ok = ok && wr_q(f, &m->wte);
  for (int l = 0; l < m->n_layers && ok; l++) {
    const QLlamaBlock *b = &m->blocks[l];
    ok = ok && wr(f, b->attn_norm.data, sizeof(float), (size_t)m->d_model);
    ok = ok && wr_q(f, &b->Wq) && wr_q(f, &b->Wk) && wr_q(f, &b->Wv);
    ok = ok && wr(f, b->b_q.data, sizeof(float), b->b_q.size) && wr(f, b->b_k.data, sizeof(float), b->b_k.size) &&
         wr(f, b->b_v.data, sizeof(float), b->b_v.size);
    ok = ok && wr_q(f, &b->Wo);
    ok = ok && wr(f, b->ffn_norm.data, sizeof(float), (size_t)m->d_model);
    ok = ok && wr_q(f, &b->Wgate) && wr_q(f, &b->Wup) && wr_q(f, &b->Wdown);
  }
  ok = ok && wr(f, m->final_norm.data, sizeof(float), (size_t)m->d_model);
  ok = ok && wr_q(f, &m->lm_head);
  ok = (fflush(f) == 0) && ok;
  ok = (fclose(f) == 0) && ok;
  if (ok && rename(tmp, path) != 0) {
    remove(path);
    ok = rename(tmp, path) == 0;
  }
  if (!ok) {
    remove(tmp);
    fprintf(stderr, "Error: failed while writing '%s'\n", path);
    llmq_set_error(LLMQ_ERR_IO, "q_llama_model_save: failed while writing '%s'", path);
    free(tmp);
    return 1;
  }
  free(tmp);
  return 0;
}

LLMQ_API QLlamaModel q_llama_quantize_from(const LlamaModel *s) {
  const int32_t cfg[8] = {s->vocab, s->d_model, s->n_layers, s->n_heads, s->n_kv, s->head_dim, s->d_ff, s->max_seq};
  const float fcfg[2] = {s->rope_base, s->eps};
  QLlamaModel m = model_alloc(cfg, fcfg);
  const size_t dmb = (size_t)s->d_model * sizeof(float);
#define QT(dst, src) quantize_int8_percol((src).data, (dst).rows, (dst).cols, (dst).q, (dst).scale)
  QT(m.wte, s->wte);
  for (int l = 0; l < s->n_layers; l++) {
    const LlamaBlock *a = &s->blocks[l];
    QLlamaBlock *b = &m.blocks[l];
    memcpy(b->attn_norm.data, a->attn_norm.data, dmb);
    memcpy(b->ffn_norm.data, a->ffn_norm.data, dmb);
    memcpy(b->b_q.data, a->b_q.data, a->b_q.size * sizeof(float));
    memcpy(b->b_k.data, a->b_k.data, a->b_k.size * sizeof(float));
    memcpy(b->b_v.data, a->b_v.data, a->b_v.size * sizeof(float));
    QT(b->Wq, a->Wq);
    QT(b->Wk, a->Wk);
    QT(b->Wv, a->Wv);
    QT(b->Wo, a->Wo);
    QT(b->Wgate, a->Wgate);
    QT(b->Wup, a->Wup);
    QT(b->Wdown, a->Wdown);
  }
  memcpy(m.final_norm.data, s->final_norm.data, dmb);
  QT(m.lm_head, s->lm_head);
#undef QT
  return m;
}

/* ------------------------------------------------------------------- caches */
LLMQ_API LlamaKV q_llama_kv_create(const QLlamaModel *m) {
  LlamaKV kv;
  kv.n_layers = m->n_layers;
  kv.max_seq = m->max_seq;
  kv.kv_dim = m->n_kv * m->head_dim;
  kv.len = 0;
  kv.k = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  kv.v = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  for (int l = 0; l < m->n_layers; l++) {
    /* host mirror: pages are only touched by q_llama_kv_sync_host */
    kv.k[l] = (float *)malloc((size_t)m->max_seq * kv.kv_dim * sizeof(float));
    kv.v[l] = (float *)malloc((size_t)m->max_seq * kv.kv_dim * sizeof(float));
  }
  if (!llmqd_kv_register(m, &kv))
    fprintf(stderr, "q_llama_kv_create: GPU cache not created (%s)\n", q_llama_last_error_message());
  return kv;
}

LLMQ_API void llama_kv_free(LlamaKV *kv) {
  llmqd_kv_release(kv);
  for (int l = 0; l < kv->n_layers; l++) {
    free(kv->k[l]);
    free(kv->v[l]);
  }
  free(kv->k);
  free(kv->v);
  kv->k = kv->v = NULL;
}

LLMQ_API void q_llama_decode_step(const QLlamaModel *m, LlamaKV *kv, int token, Tensor *logits) {
  if (!logits || !logits->data || logits->size < (size_t)m->vocab) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_decode_step: logits tensor must hold %d floats", m->vocab);
    return;
  }
  if (llmqd_decode(m, kv, token, logits->data, NULL)) kv->len = kv->len + 1;
}

LLMQ_API int q_llama_decode_step_argmax(const QLlamaModel *m, LlamaKV *kv, int token, Tensor *logits) {
  if (logits && (!logits->data || logits->size < (size_t)m->vocab)) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_decode_step_argmax: logits tensor must hold %d floats", m->vocab);
    return -1;
  }
  int next = -1;
  if (!llmqd_decode(m, kv, token, logits ? logits->data : NULL, &next)) return -1;
  kv->len = kv->len + 1;
  return next;
}

LLMQ_API int q_llama_generate(const QLlamaModel *m, LlamaKV *kv, int token, int n, int *ids) {
  if (n < 0 || (n > 0 && !ids)) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_generate: bad arguments");
    return LLMQ_ERR_ARG;
  }
  if (!llmqd_generate(m, kv, token, n, ids)) return q_llama_last_error();
  kv->len = kv->len + n;
  return LLMQ_OK;
}

/* ---- sampler.h (sampler.c): the stream on the host, the draw on the GPU ---- */

/* xorshift64 with the reference's shifts and non-zero default seed
 * (sampler.c:26-39): the stream must be the same number for number. */
LLMQ_API Rng rng_create(unsigned long long seed) {
  Rng r;
  r.state = seed ? seed : 0x9E3779B97F4A7C15ULL;
  return r;
}

static unsigned long long rng_next(unsigned long long *s) {
  unsigned long long x = *s;
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  *s = x;
  return x;
}

LLMQ_API float rng_uniform(Rng *r) {
  /* top 53 bits times 2^-53, exact in double, then rounded to float (sampler.c:41-44) */
  return (float)((double)(rng_next(&r->state) >> 11) * (1.0 / 9007199254740992.0));
}

/* The device form of one sampler call: top_k resolved to the number of
 * candidates it keeps (sampler.c:87-88). */
LlmqSample llmq_sample_settings(int vocab, float temperature, int top_k, float top_p, const Rng *rng) {
  LlmqSample s;
  s.temperature = temperature;
  s.k = (top_k > 0 && top_k < vocab) ? top_k : vocab;
  s.top_p = top_p;
  s.pad = 0;
  s.rng = rng ? rng->state : 0;
  return s;
}

static const float *logits_row(const Tensor *logits, int row, const char *who) {
  if (!logits || !logits->data || !logits->shape || logits->ndim < 2 || logits->shape[1] <= 0 || row < 0 ||
      (size_t)(row + 1) * (size_t)logits->shape[1] > logits->size) {
    llmq_set_error(LLMQ_ERR_ARG, "%s: logits row %d out of range", who, row);
    return NULL;
  }
  return logits->data + (size_t)row * (size_t)logits->shape[1];
}

LLMQ_API int sample_argmax(const Tensor *logits, int row) {
  const float *r = logits_row(logits, row, "sample_argmax");
  if (!r) return -1;
  LlmqSample s = llmq_sample_settings(logits->shape[1], 0.0f, 0, 1.0f, NULL);
  int id = -1;
  if (!llmqd_sample_row(r, logits->shape[1], &s, &id)) return -1;
  return id;
}

LLMQ_API int sample_token(const Tensor *logits, int row, float temperature, int top_k, float top_p, Rng *rng) {
  const float *r = logits_row(logits, row, "sample_token");
  if (!r) return -1;
  if (!rng) {
    llmq_set_error(LLMQ_ERR_ARG, "sample_token: rng is NULL");
    return -1;
  }
  LlmqSample s = llmq_sample_settings(logits->shape[1], temperature, top_k, top_p, rng);
  int id = -1;
  if (!llmqd_sample_row(r, logits->shape[1], &s, &id)) return -1;
  rng->state = s.rng;
  return id;
}

LLMQ_API int q_llama_decode_step_sample(const QLlamaModel *m, LlamaKV *kv, int token, float temperature, int top_k,
                                        float top_p, Rng *rng, Tensor *logits) {
  if (!rng || (logits && (!logits->data || logits->size < (size_t)m->vocab))) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_decode_step_sample: bad rng or logits tensor (needs %d floats)",
                   m->vocab);
    return -1;
  }
  int next = -1;
  float *out = logits ? logits->data : NULL;
  if (temperature <= 0.0f) { /* greedy (sampler.c:65-67): the fused argmax, no draw */
    if (!llmqd_decode(m, kv, token, out, &next)) return -1;
  } else {
    LlmqSample s = llmq_sample_settings(m->vocab, temperature, top_k, top_p, rng);
    if (!llmqd_decode_sample(m, kv, token, out, &next, &s)) return -1;
    rng->state = s.rng;
  }
  kv->len = kv->len + 1;
  return next;
}

LLMQ_API int q_llama_generate_sample(const QLlamaModel *m, LlamaKV *kv, int token, int n, float temperature,
                                     int top_k, float top_p, Rng *rng, int *ids) {
  if (n < 0 || (n > 0 && !ids) || !rng) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_generate_sample: bad arguments");
    return LLMQ_ERR_ARG;
  }
  if (temperature <= 0.0f) {
    if (!llmqd_generate(m, kv, token, n, ids)) return q_llama_last_error();
  } else {
    LlmqSample s = llmq_sample_settings(m->vocab, temperature, top_k, top_p, rng);
    if (!llmqd_generate_sample(m, kv, token, n, ids, &s)) return q_llama_last_error();
    rng->state = s.rng;
  }
  kv->len = kv->len + n;
  return LLMQ_OK;
}

LLMQ_API void q_llama_decode_batch(const QLlamaModel *m, LlamaKV **kvs, const int *tokens, int B, Tensor *logits) {
  if (!logits || !logits->data || B <= 0 || logits->size < (size_t)B * (size_t)m->vocab) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_decode_batch: logits tensor must hold B x %d floats", m->vocab);
    return;
  }
  if (llmqd_decode_rows(m, kvs, tokens, B, logits->data, NULL))
    for (int b = 0; b < B; b++) kvs[b]->len = kvs[b]->len + 1;
}

LLMQ_API int q_llama_decode_batch_argmax(const QLlamaModel *m, LlamaKV **kvs, const int *tokens, int B, int *ids) {
  if (B <= 0 || !ids) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_decode_batch_argmax: bad arguments");
    return LLMQ_ERR_ARG;
  }
  if (!llmqd_decode_rows(m, kvs, tokens, B, NULL, ids)) return q_llama_last_error();
  for (int b = 0; b < B; b++) kvs[b]->len = kvs[b]->len + 1;
  return LLMQ_OK;
}

LLMQ_API void q_llama_prefill(const QLlamaModel *m, LlamaKV *kv, const int *ids, int n, Tensor *logits) {
  if (logits && (!logits->data || logits->size < (size_t)m->vocab)) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_prefill: logits tensor must hold %d floats", m->vocab);
    return;
  }
  if (llmqd_prefill(m, kv, ids, n, logits ? logits->data : NULL, NULL)) kv->len = kv->len + n;
}

LLMQ_API int q_llama_prefill_argmax(const QLlamaModel *m, LlamaKV *kv, const int *ids, int n, Tensor *logits) {
  if (logits && (!logits->data || logits->size < (size_t)m->vocab)) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_prefill_argmax: logits tensor must hold %d floats", m->vocab);
    return -1;
  }
  int next = -1;
  if (!llmqd_prefill(m, kv, ids, n, logits ? logits->data : NULL, &next)) return -1;
  kv->len = kv->len + n;
  return next;
}

LLMQ_API int q_llama_kv_sync_host(const QLlamaModel *m, LlamaKV *kv) {
  if (!llmqd_kv_download(m, kv, kv->len)) return q_llama_last_error();
  return LLMQ_OK;
}

LLMQ_API int q_llama_model_upload(const QLlamaModel *m) {
  return llmqd_model_upload(m) ? LLMQ_OK : q_llama_last_error();
}

LLMQ_API float q_llama_last_step_ms(void) { return llmqd_last_ms(); }
