/* llmq_synth.c - seeded synthetic int8 models (the benchmark and test inputs).
 *
 * Element e of tensor t is drawn from N(0, stddev): splitmix64 (Vigna) keyed by
 * (seed, t) gives two uniforms per element pair (e>>1), Box-Muller turns them
 * into two normals (cos half for even e, sin half for odd e).  2-D tensors are
 * then quantised per column with the reference rule of quant.c:10-27.  Work is
 * split over column strips across threads; every value depends only on
 * (seed, t, e), so the model is the same for any thread count.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include "llmq_internal.h"

static uint64_t splitmix64(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static uint64_t tensor_key(uint64_t seed, int tid) {
  return splitmix64(seed ^ (0xD1B54A32D192ED03ull * (uint64_t)(tid + 1)));
}

/* Both normals of pair p. */
static void normal_pair(uint64_t key, uint64_t p, double *z0, double *z1) {
  const uint64_t a = splitmix64(key + 2 * p), b = splitmix64(key + 2 * p + 1);
  const double u1 = ((double)(a >> 11) + 1.0) * 0x1p-53; /* (0, 1] */
  const double u2 = (double)(b >> 11) * 0x1p-53;         /* [0, 1) */
  const double r = sqrt(-2.0 * log(u1));
  const double t = 6.283185307179586476925286766559 * u2;
  *z0 = r * cos(t);
  *z1 = r * sin(t);
}

static float draw(uint64_t key, uint64_t e, float stddev) {
  double z0, z1;
  normal_pair(key, e >> 1, &z0, &z1);
  return (float)((double)stddev * ((e & 1) ? z1 : z0));
}

/* quant.c:21-23 */
static signed char code_of(float v) {
  int c = (int)lrintf(v);
  if (c > 127) c = 127;
  if (c < -127) c = -127;
  return (signed char)c;
}

/* Columns [c0, c0 + t->cols) and rows [r0, r0 + t->rows) of a full (K, N)
 * tensor; the per-column scales are those of the full columns (all K rows). */
typedef struct {
  QTensor *t;
  uint64_t key;
  float stddev;
  int K, N, c0, r0;
  atomic_int next;
} QJob;

enum { STRIP = 64 };

static void *qjob_run(void *arg) {
  QJob *j = (QJob *)arg;
  const int K = j->K, N = j->N, W = j->t->cols, R = j->t->rows;
  const int nstrips = (W + STRIP - 1) / STRIP;
  float *buf = (float *)malloc((size_t)K * STRIP * sizeof(float));
  if (!buf) return NULL;
  for (;;) {
    const int s = atomic_fetch_add(&j->next, 1);
    if (s >= nstrips) break;
    const int l0 = s * STRIP, l1 = l0 + STRIP < W ? l0 + STRIP : W, w = l1 - l0;
    const int j0 = j->c0 + l0; /* full-tensor column of local column l0 */
    for (int i = 0; i < K; i++) {
      const uint64_t e0 = (uint64_t)i * N + j0;
      float *row = buf + (size_t)i * STRIP;
      int c = 0;
      while (c < w) {
        const uint64_t e = e0 + c;
        if ((e & 1) == 0 && c + 1 < w) { /* both halves of the pair land in the strip */
          double z0, z1;
          normal_pair(j->key, e >> 1, &z0, &z1);
          row[c] = (float)((double)j->stddev * z0);
          row[c + 1] = (float)((double)j->stddev * z1);
          c += 2;
        } else {
          row[c] = draw(j->key, e, j->stddev);
          c += 1;
        }
      }
    }
    for (int c = 0; c < w; c++) {
      float amax = 0.0f;
      for (int i = 0; i < K; i++) {
        const float a = fabsf(buf[(size_t)i * STRIP + c]);
        if (a > amax) amax = a;
      }
      const float sc = (amax > 0.0f) ? amax / 127.0f : 1.0f;
      const float inv = 1.0f / sc;
      j->t->scale[l0 + c] = sc;
      for (int i = 0; i < R; i++)
        j->t->q[(size_t)i * W + l0 + c] = code_of(buf[(size_t)(j->r0 + i) * STRIP + c] * inv);
    }
  }
  free(buf);
  return NULL;
}

/* LLMQ_THREADS caps the generator's threads (one process per GPU shares the
 * host cores); default: every online core. */
static int n_threads(void) {
  const char *env = getenv("LLMQ_THREADS");
  long n = (env && atoi(env) > 0) ? atoi(env) : sysconf(_SC_NPROCESSORS_ONLN);
  if (n < 1) n = 1;
  if (n > 128) n = 128;
  return (int)n;
}

/* t (rows x cols, allocated) receives rows [r0, r0 + rows) x columns
 * [c0, c0 + cols) of the full (K, N) tensor `tid`. */
static void synth_qtensor_part(QTensor *t, uint64_t seed, int tid, float stddev, int K, int N, int r0, int c0) {
  QJob j;
  j.t = t;
  j.key = tensor_key(seed, tid);
  j.stddev = stddev;
  j.K = K;
  j.N = N;
  j.c0 = c0;
  j.r0 = r0;
  atomic_init(&j.next, 0);
  const int nt = n_threads();
  pthread_t th[128];
  int started = 0;
  for (int i = 0; i < nt - 1; i++)
    if (pthread_create(&th[started], NULL, qjob_run, &j) == 0) started++;
  qjob_run(&j);
  for (int i = 0; i < started; i++) pthread_join(th[i], NULL);
}

/* The fast benchmark weights: code of element e of tensor tid uniform in
 * [-127, 127] (splitmix64 of (tensor key, e)), scale of column j uniform in
 * [2e-4, 1e-3) (the size of N(0, 0.02) weights quantised per column).  Any
 * slice costs only its own elements. */
typedef struct {
  QTensor *t;
  uint64_t key, skey;
  int N, c0, r0;
  atomic_int next;
} FJob;

static void *fjob_run(void *arg) {
  FJob *j = (FJob *)arg;
  const int W = j->t->cols, R = j->t->rows;
  for (;;) {
    const int i = atomic_fetch_add(&j->next, 1);
    if (i >= R) break;
    const uint64_t e0 = (uint64_t)(j->r0 + i) * j->N + j->c0;
    signed char *q = j->t->q + (size_t)i * W;
    for (int c = 0; c < W; c++) q[c] = (signed char)((int)(splitmix64(j->key + e0 + c) % 255u) - 127);
  }
  return NULL;
}

static void synth_fast_part(QTensor *t, uint64_t seed, int tid, int N, int r0, int c0) {
  FJob j;
  j.t = t;
  j.key = tensor_key(seed, tid);
  j.skey = tensor_key(seed ^ 0x5CA1Eull, tid);
  j.N = N;
  j.c0 = c0;
  j.r0 = r0;
  atomic_init(&j.next, 0);
  for (int c = 0; c < t->cols; c++) {
    const double u = (double)(splitmix64(j.skey + (uint64_t)(c0 + c)) >> 11) * 0x1p-53;
    t->scale[c] = (float)(2e-4 + 8e-4 * u);
  }
  const int nt = n_threads();
  pthread_t th[128];
  int started = 0;
  for (int i = 0; i < nt - 1; i++)
    if (pthread_create(&th[started], NULL, fjob_run, &j) == 0) started++;
  fjob_run(&j);
  for (int i = 0; i < started; i++) pthread_join(th[i], NULL);
}

static void synth_qtensor_normal(QTensor *t, uint64_t seed, int tid, float stddev) {
  synth_qtensor_part(t, seed, tid, stddev, t->rows, t->cols, 0, 0);
}

static void synth_vec_part(Tensor *t, uint64_t seed, int tid, float stddev, size_t e0) {
  const uint64_t key = tensor_key(seed, tid);
  for (size_t e = 0; e < t->size; e++) t->data[e] = draw(key, e0 + e, stddev);
}


static void fill_ones(Tensor *t) {
  for (size_t e = 0; e < t->size; e++) t->data[e] = 1.0f;
}

static void vec_alloc(Tensor *t, int n) {
  t->ndim = 1;
  t->shape = (int *)malloc(sizeof(int));
  t->shape[0] = n;
  t->size = (size_t)n;
  t->grad = NULL;
  const size_t bytes = (((size_t)n * sizeof(float)) + 63) & ~(size_t)63;
  t->data = (float *)aligned_alloc(64, bytes);
  memset(t->data, 0, bytes);
}

/* Whether `world` tensor-parallel shards of config c are well formed: whole
 * query and KV heads, d_ff and vocab columns per rank. */
static int shardable(const LlmqConfig *c, int world) {
  return world >= 1 && c->n_heads % world == 0 && c->n_kv % world == 0 && c->d_ff % world == 0 &&
         c->vocab % world == 0;
}

static void copy_config(const LlmqConfig *c, QLlamaModel *out) {
  out->vocab = c->vocab;
  out->d_model = c->d_model;
  out->n_layers = c->n_layers;
  out->n_heads = c->n_heads;
  out->n_kv = c->n_kv;
  out->head_dim = c->head_dim;
  out->d_ff = c->d_ff;
  out->max_seq = c->max_seq;
  out->rope_base = c->rope_base;
  out->eps = c->eps;
}

/* Tensor ids follow the checkpoint order of llama.c:199-219.  Shard `rank` of
 * `world` keeps the columns of its query heads (Wq, b_q), KV heads (Wk, Wv,
 * b_k, b_v), d_ff slice (Wgate, Wup) and vocab slice (lm_head), and the rows
 * of its query dims (Wo) and d_ff slice (Wdown); per-column scales are those
 * of the full columns.  wte and the norms are whole.  world = 1: the model. */
static int synth_model(const LlmqConfig *c, uint64_t seed, float stddev, int with_bias, int rank, int world, int fast,
                       QLlamaModel *out) {
  if (!c || !out || c->vocab <= 0 || c->d_model <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv <= 0 ||
      c->head_dim <= 0 || c->d_ff <= 0 || c->max_seq <= 0 || c->n_heads % c->n_kv != 0 || !shardable(c, world) ||
      rank < 0 || rank >= world) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_synth_model: invalid configuration");
    return LLMQ_ERR_ARG;
  }
  memset(out, 0, sizeof *out);
  copy_config(c, out);
  const int dm = c->d_model, hd = c->head_dim, qd = c->n_heads * hd, kvd = c->n_kv * hd, dff = c->d_ff;
  const int qd_l = qd / world, kvd_l = kvd / world, dff_l = dff / world, V_l = c->vocab / world;
  out->wte = qtensor_create(c->vocab, dm);
  out->blocks = (QLlamaBlock *)calloc((size_t)c->n_layers, sizeof(QLlamaBlock));
  if (!out->blocks) {
    llmq_set_error(LLMQ_ERR_OOM, "llmq_synth_model: out of host memory");
    return LLMQ_ERR_OOM;
  }
  if (fast)
    synth_fast_part(&out->wte, seed, 0, dm, 0, 0);
  else
    synth_qtensor_normal(&out->wte, seed, 0, stddev);
  for (int l = 0; l < c->n_layers; l++) {
    QLlamaBlock *b = &out->blocks[l];
    const int base = 1 + 12 * l;
    vec_alloc(&b->attn_norm, dm);
    vec_alloc(&b->ffn_norm, dm);
    vec_alloc(&b->b_q, qd_l);
    vec_alloc(&b->b_k, kvd_l);
    vec_alloc(&b->b_v, kvd_l);
    fill_ones(&b->attn_norm);
    fill_ones(&b->ffn_norm);
    if (with_bias) {
      synth_vec_part(&b->b_q, seed, base + 4, stddev, (size_t)rank * qd_l);
      synth_vec_part(&b->b_k, seed, base + 5, stddev, (size_t)rank * kvd_l);
      synth_vec_part(&b->b_v, seed, base + 6, stddev, (size_t)rank * kvd_l);
    }
    b->Wq = qtensor_create(dm, qd_l);
    b->Wk = qtensor_create(dm, kvd_l);
    b->Wv = qtensor_create(dm, kvd_l);
    b->Wo = qtensor_create(qd_l, dm);
    b->Wgate = qtensor_create(dm, dff_l);
    b->Wup = qtensor_create(dm, dff_l);
    b->Wdown = qtensor_create(dff_l, dm);
    if (fast) {
      synth_fast_part(&b->Wq, seed, base + 1, qd, 0, rank * qd_l);
      synth_fast_part(&b->Wk, seed, base + 2, kvd, 0, rank * kvd_l);
      synth_fast_part(&b->Wv, seed, base + 3, kvd, 0, rank * kvd_l);
      synth_fast_part(&b->Wo, seed, base + 7, dm, rank * qd_l, 0);
      synth_fast_part(&b->Wgate, seed, base + 9, dff, 0, rank * dff_l);
      synth_fast_part(&b->Wup, seed, base + 10, dff, 0, rank * dff_l);
      synth_fast_part(&b->Wdown, seed, base + 11, dm, rank * dff_l, 0);
      continue;
    }
    synth_qtensor_part(&b->Wq, seed, base + 1, stddev, dm, qd, 0, rank * qd_l);
    synth_qtensor_part(&b->Wk, seed, base + 2, stddev, dm, kvd, 0, rank * kvd_l);
    synth_qtensor_part(&b->Wv, seed, base + 3, stddev, dm, kvd, 0, rank * kvd_l);
    synth_qtensor_part(&b->Wo, seed, base + 7, stddev, qd, dm, rank * qd_l, 0);
    synth_qtensor_part(&b->Wgate, seed, base + 9, stddev, dm, dff, 0, rank * dff_l);
    synth_qtensor_part(&b->Wup, seed, base + 10, stddev, dm, dff, 0, rank * dff_l);
    synth_qtensor_part(&b->Wdown, seed, base + 11, stddev, dff, dm, rank * dff_l, 0);
  }
  vec_alloc(&out->final_norm, dm);
  fill_ones(&out->final_norm);
  out->lm_head = qtensor_create(dm, V_l);
  if (fast)
    synth_fast_part(&out->lm_head, seed, 2 + 12 * c->n_layers, c->vocab, 0, rank * V_l);
  else
    synth_qtensor_part(&out->lm_head, seed, 2 + 12 * c->n_layers, stddev, dm, c->vocab, 0, rank * V_l);
  return LLMQ_OK;
}

LLMQ_API int llmq_synth_model_shard(const LlmqConfig *c, uint64_t seed, float stddev, int with_bias, int rank,
                                    int world, QLlamaModel *out) {
  return synth_model(c, seed, stddev, with_bias, rank, world, 0, out);
}

LLMQ_API int llmq_synth_model(const LlmqConfig *c, uint64_t seed, float stddev, int with_bias, QLlamaModel *out) {
  return synth_model(c, seed, stddev, with_bias, 0, 1, 0, out);
}

LLMQ_API int llmq_synth_model_fast_shard(const LlmqConfig *c, uint64_t seed, int rank, int world, QLlamaModel *out) {
  return synth_model(c, seed, 0.0f, 0, rank, world, 1, out);
}

/* Copies rows [r0, r0 + rows) x columns [c0, c0 + cols) of a (K, N) QTensor;
 * the scales of those columns come along. */
static QTensor qslice(const QTensor *src, int r0, int rows, int c0, int cols) {
  QTensor t = qtensor_create(rows, cols);
  for (int i = 0; i < rows; i++)
    memcpy(t.q + (size_t)i * cols, src->q + (size_t)(r0 + i) * src->cols + c0, (size_t)cols);
  memcpy(t.scale, src->scale + c0, (size_t)cols * sizeof(float));
  return t;
}

static void vslice(Tensor *dst, const Tensor *src, int e0, int n) {
  vec_alloc(dst, n);
  memcpy(dst->data, src->data + e0, (size_t)n * sizeof(float));
}

LLMQ_API int q_llama_model_shard(const QLlamaModel *m, int rank, int world, QLlamaModel *out) {
  LlmqConfig c = {m->vocab, m->d_model, m->n_layers, m->n_heads, m->n_kv, m->head_dim, m->d_ff, m->max_seq,
                  m->rope_base, m->eps};
  if (!m->blocks || !shardable(&c, world) || rank < 0 || rank >= world ||
      m->blocks[0].Wq.cols != m->n_heads * m->head_dim) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_model_shard: not a whole model, or not divisible into %d shards", world);
    return LLMQ_ERR_ARG;
  }
  memset(out, 0, sizeof *out);
  copy_config(&c, out);
  const int dm = m->d_model, hd = m->head_dim, qd = m->n_heads * hd, kvd = m->n_kv * hd;
  const int qd_l = qd / world, kvd_l = kvd / world, dff_l = m->d_ff / world, V_l = m->vocab / world;
  out->wte = qslice(&m->wte, 0, m->vocab, 0, dm);
  out->blocks = (QLlamaBlock *)calloc((size_t)m->n_layers, sizeof(QLlamaBlock));
  if (!out->blocks) {
    llmq_set_error(LLMQ_ERR_OOM, "q_llama_model_shard: out of host memory");
    return LLMQ_ERR_OOM;
  }
  for (int l = 0; l < m->n_layers; l++) {
    const QLlamaBlock *s = &m->blocks[l];
    QLlamaBlock *b = &out->blocks[l];
    vslice(&b->attn_norm, &s->attn_norm, 0, dm);
    vslice(&b->ffn_norm, &s->ffn_norm, 0, dm);
    vslice(&b->b_q, &s->b_q, rank * qd_l, qd_l);
    vslice(&b->b_k, &s->b_k, rank * kvd_l, kvd_l);
    vslice(&b->b_v, &s->b_v, rank * kvd_l, kvd_l);
    b->Wq = qslice(&s->Wq, 0, dm, rank * qd_l, qd_l);
    b->Wk = qslice(&s->Wk, 0, dm, rank * kvd_l, kvd_l);
    b->Wv = qslice(&s->Wv, 0, dm, rank * kvd_l, kvd_l);
    b->Wo = qslice(&s->Wo, rank * qd_l, qd_l, 0, dm);
    b->Wgate = qslice(&s->Wgate, 0, dm, rank * dff_l, dff_l);
    b->Wup = qslice(&s->Wup, 0, dm, rank * dff_l, dff_l);
    b->Wdown = qslice(&s->Wdown, rank * dff_l, dff_l, 0, dm);
  }
  vslice(&out->final_norm, &m->final_norm, 0, dm);
  out->lm_head = qslice(&m->lm_head, 0, dm, rank * V_l, V_l);
  return LLMQ_OK;
}

LLMQ_API void llmq_synth_qtensor(QTensor *t, uint64_t seed) {
  const uint64_t key = tensor_key(seed, 0x5EED);
  const size_t n = (size_t)t->rows * t->cols;
  for (size_t i = 0; i < n; i++) t->q[i] = (signed char)((int)(splitmix64(key + i) % 255u) - 127);
  const uint64_t skey = tensor_key(seed, 0x5CA1E);
  for (int j = 0; j < t->cols; j++) {
    const double u = (double)(splitmix64(skey + (uint64_t)j) >> 11) * 0x1p-53;
    t->scale[j] = (float)(1e-3 + 9e-3 * u);
  }
}

/* ----------------------------------------------------------- streaming writer */
static int wr_all(FILE *f, const void *p, size_t size, size_t n) { return n == 0 || fwrite(p, size, n, f) == n; }

/* Writes one synthetic 2-D tensor (tensor id tid, full shape K x N) as LLMQ
 * stores it: the per-column scales, then the row-major int8 codes.  Only this
 * tensor is in memory meanwhile. */
static int save_qtensor(FILE *f, uint64_t seed, int tid, float stddev, int fast, int K, int N) {
  QTensor t = qtensor_create(K, N);
  if (!t.q || !t.scale) {
    free(t.q);
    free(t.scale);
    return 0;
  }
  if (fast)
    synth_fast_part(&t, seed, tid, N, 0, 0);
  else
    synth_qtensor_normal(&t, seed, tid, stddev);
  const int ok = wr_all(f, t.scale, sizeof(float), (size_t)N) && wr_all(f, t.q, 1, (size_t)K * N);
  free(t.q);
  free(t.scale);
  return ok;
}

/* Writes one synthetic 1-D tensor: ones (norm gains), or the seeded biases
 * (zero when with_bias is 0). */
static int save_vec(FILE *f, uint64_t seed, int tid, float stddev, int n, int kind) {
  Tensor t;
  vec_alloc(&t, n);
  if (!t.data) return 0;
  if (kind == 1)
    fill_ones(&t);
  else if (kind == 2)
    synth_vec_part(&t, seed, tid, stddev, 0);
  const int ok = wr_all(f, t.data, sizeof(float), (size_t)n);
  free(t.data);
  free(t.shape);
  return ok;
}

/* The model llmq_synth_model (fast = 0) or llmq_synth_model_fast_shard with
 * one shard (fast = 1) builds, written straight to an LLMQ v2 file in the
 * canonical order of llama.c:199-219 (the layout q_llama_model_load reads,
 * llama.c:603-657): header, then each tensor as it is generated, so no more
 * than one tensor is ever in memory (a 70B-shaped file needs ~1 GB, not 70).
 * Written to path.tmp, then renamed over path, like llama.c:230-269.  Returns 0
 * on success, LLMQ_ERR_ARG / LLMQ_ERR_IO / LLMQ_ERR_OOM on failure. */
LLMQ_API int llmq_synth_model_save(const LlmqConfig *c, uint64_t seed, float stddev, int with_bias, int fast,
                                   const char *path) {
  if (!c || !path || c->vocab <= 0 || c->d_model <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv <= 0 ||
      c->head_dim <= 0 || c->d_ff <= 0 || c->max_seq <= 0 || c->n_heads % c->n_kv != 0) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_synth_model_save: invalid configuration");
    return LLMQ_ERR_ARG;
  }
  if (fast) {
    stddev = 0.0f;
    with_bias = 0;
  }
  const size_t plen = strlen(path);
  char *tmp = (char *)malloc(plen + 5);
  if (!tmp) {
    llmq_set_error(LLMQ_ERR_OOM, "llmq_synth_model_save: out of host memory");
    return LLMQ_ERR_OOM;
  }
  memcpy(tmp, path, plen);
  memcpy(tmp + plen, ".tmp", 5);
  FILE *f = fopen(tmp, "wb");
  if (!f) {
    llmq_set_error(LLMQ_ERR_IO, "llmq_synth_model_save: cannot open '%s' for writing", tmp);
    free(tmp);
    return LLMQ_ERR_IO;
  }
  const int dm = c->d_model, qd = c->n_heads * c->head_dim, kvd = c->n_kv * c->head_dim, dff = c->d_ff;
  const uint32_t hdr[2] = {0x514D4C4Cu, 2u}; /* 'LLMQ', version 2 (llama.c:192-194) */
  const int32_t cfg[8] = {c->vocab, dm, c->n_layers, c->n_heads, c->n_kv, c->head_dim, dff, c->max_seq};
  const float fcfg[2] = {c->rope_base, c->eps};
  int ok = wr_all(f, hdr, sizeof(uint32_t), 2) && wr_all(f, cfg, sizeof(int32_t), 8) &&
           wr_all(f, fcfg, sizeof(float), 2);
  ok = ok && save_qtensor(f, seed, 0, stddev, fast, c->vocab, dm);
  const int bias_kind = with_bias ? 2 : 0;
  for (int l = 0; l < c->n_layers && ok; l++) {
    const int base = 1 + 12 * l;
    ok = ok && save_vec(f, seed, base + 0, stddev, dm, 1);               /* attn_norm */
    ok = ok && save_qtensor(f, seed, base + 1, stddev, fast, dm, qd);    /* Wq */
    ok = ok && save_qtensor(f, seed, base + 2, stddev, fast, dm, kvd);   /* Wk */
    ok = ok && save_qtensor(f, seed, base + 3, stddev, fast, dm, kvd);   /* Wv */
    ok = ok && save_vec(f, seed, base + 4, stddev, qd, bias_kind);       /* b_q */
    ok = ok && save_vec(f, seed, base + 5, stddev, kvd, bias_kind);      /* b_k */
    ok = ok && save_vec(f, seed, base + 6, stddev, kvd, bias_kind);      /* b_v */
    ok = ok && save_qtensor(f, seed, base + 7, stddev, fast, qd, dm);    /* Wo */
    ok = ok && save_vec(f, seed, base + 8, stddev, dm, 1);               /* ffn_norm */
    ok = ok && save_qtensor(f, seed, base + 9, stddev, fast, dm, dff);   /* Wgate */
    ok = ok && save_qtensor(f, seed, base + 10, stddev, fast, dm, dff);  /* Wup */
    ok = ok && save_qtensor(f, seed, base + 11, stddev, fast, dff, dm);  /* Wdown */
  }
  ok = ok && save_vec(f, seed, 1 + 12 * c->n_layers, stddev, dm, 1); /* final_norm */
  ok = ok && save_qtensor(f, seed, 2 + 12 * c->n_layers, stddev, fast, dm, c->vocab);
  ok = (fflush(f) == 0) && ok;
  ok = (fclose(f) == 0) && ok;
  if (ok && rename(tmp, path) != 0) {
    remove(path);
    ok = rename(tmp, path) == 0;
  }
  if (!ok) {
    remove(tmp);
    llmq_set_error(LLMQ_ERR_IO, "llmq_synth_model_save: failed while writing '%s'", path);
    free(tmp);
    return LLMQ_ERR_IO;
  }
  free(tmp);
  return LLMQ_OK;
}
