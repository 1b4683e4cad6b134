/* llmq_synth.c - seeded synthetic int8 models (the benchmark and test inputs).
 *
 * Element e of tensor t is drawn from N(0, stddev): splitmix64 (Vigna) keyed by
 * (seed, t) gives two uniforms per element pair (e>>1), Box-Muller turns them
 * into two normals (cos half for even e, sin half for odd e).  2-D tensors are
 * then quantised per column with the reference rule of quant.c:45-62.  Work is
 * split over column strips across threads; every value depends only on
 * (seed, t, e), so the model is the same for any thread count.
 */
#define _GNU_SOURCE
#include <math.h>
#include <pthread.h>
#include <stdatomic.h>
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

/* quant.c:56-58 */
static signed char code_of(float v) {
  int c = (int)lrintf(v);
  if (c > 127) c = 127;
  if (c < -127) c = -127;
  return (signed char)c;
}

typedef struct {
  QTensor *t;
  uint64_t key;
  float stddev;
  int strip;
  atomic_int next;
} QJob;

enum { STRIP = 64 };

static void *qjob_run(void *arg) {
  QJob *j = (QJob *)arg;
  const int K = j->t->rows, N = j->t->cols;
  const int nstrips = (N + STRIP - 1) / STRIP;
  float *buf = (float *)malloc((size_t)K * STRIP * sizeof(float));
  if (!buf) return NULL;
  for (;;) {
    const int s = atomic_fetch_add(&j->next, 1);
    if (s >= nstrips) break;
    const int j0 = s * STRIP, j1 = j0 + STRIP < N ? j0 + STRIP : N, w = j1 - j0;
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
      j->t->scale[j0 + c] = sc;
      for (int i = 0; i < K; i++) j->t->q[(size_t)i * N + j0 + c] = code_of(buf[(size_t)i * STRIP + c] * inv);
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

static void synth_qtensor_normal(QTensor *t, uint64_t seed, int tid, float stddev) {
  QJob j;
  j.t = t;
  j.key = tensor_key(seed, tid);
  j.stddev = stddev;
  atomic_init(&j.next, 0);
  const int nt = n_threads();
  pthread_t th[128];
  int started = 0;
  for (int i = 0; i < nt - 1; i++)
    if (pthread_create(&th[started], NULL, qjob_run, &j) == 0) started++;
  qjob_run(&j);
  for (int i = 0; i < started; i++) pthread_join(th[i], NULL);
}

static void synth_vec(Tensor *t, uint64_t seed, int tid, float stddev) {
  const uint64_t key = tensor_key(seed, tid);
  for (size_t e = 0; e < t->size; e++) t->data[e] = draw(key, e, stddev);
}

static void fill_ones(Tensor *t) {
  for (size_t e = 0; e < t->size; e++) t->data[e] = 1.0f;
}

/* Tensor ids follow the checkpoint order of llama.c:199-219. */
LLMQ_API int llmq_synth_model(const LlmqConfig *c, uint64_t seed, float stddev, int with_bias, QLlamaModel *out) {
  if (!c || !out || c->vocab <= 0 || c->d_model <= 0 || c->n_layers <= 0 || c->n_heads <= 0 || c->n_kv <= 0 ||
      c->head_dim <= 0 || c->d_ff <= 0 || c->max_seq <= 0 || c->n_heads % c->n_kv != 0) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_synth_model: invalid configuration");
    return LLMQ_ERR_ARG;
  }
  memset(out, 0, sizeof *out);
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
  const int dm = c->d_model, qd = c->n_heads * c->head_dim, kvd = c->n_kv * c->head_dim, dff = c->d_ff;
  out->wte = qtensor_create(c->vocab, dm);
  out->blocks = (QLlamaBlock *)calloc((size_t)c->n_layers, sizeof(QLlamaBlock));
  if (!out->blocks) {
    llmq_set_error(LLMQ_ERR_OOM, "llmq_synth_model: out of host memory");
    return LLMQ_ERR_OOM;
  }
  synth_qtensor_normal(&out->wte, seed, 0, stddev);
  for (int l = 0; l < c->n_layers; l++) {
    QLlamaBlock *b = &out->blocks[l];
    const int base = 1 + 12 * l;
    /* vectors: same allocation convention as the loader */
    Tensor *vecs[5] = {&b->attn_norm, &b->ffn_norm, &b->b_q, &b->b_k, &b->b_v};
    const int lens[5] = {dm, dm, qd, kvd, kvd};
    for (int i = 0; i < 5; i++) {
      Tensor *t = vecs[i];
      t->ndim = 1;
      t->shape = (int *)malloc(sizeof(int));
      t->shape[0] = lens[i];
      t->size = (size_t)lens[i];
      t->grad = NULL;
      const size_t bytes = (((size_t)lens[i] * sizeof(float)) + 63) & ~(size_t)63;
      t->data = (float *)aligned_alloc(64, bytes);
      memset(t->data, 0, bytes);
    }
    fill_ones(&b->attn_norm);
    fill_ones(&b->ffn_norm);
    if (with_bias) {
      synth_vec(&b->b_q, seed, base + 4, stddev);
      synth_vec(&b->b_k, seed, base + 5, stddev);
      synth_vec(&b->b_v, seed, base + 6, stddev);
    }
    b->Wq = qtensor_create(dm, qd);
    b->Wk = qtensor_create(dm, kvd);
    b->Wv = qtensor_create(dm, kvd);
    b->Wo = qtensor_create(qd, dm);
    b->Wgate = qtensor_create(dm, dff);
    b->Wup = qtensor_create(dm, dff);
    b->Wdown = qtensor_create(dff, dm);
    synth_qtensor_normal(&b->Wq, seed, base + 1, stddev);
    synth_qtensor_normal(&b->Wk, seed, base + 2, stddev);
    synth_qtensor_normal(&b->Wv, seed, base + 3, stddev);
    synth_qtensor_normal(&b->Wo, seed, base + 7, stddev);
    synth_qtensor_normal(&b->Wgate, seed, base + 9, stddev);
    synth_qtensor_normal(&b->Wup, seed, base + 10, stddev);
    synth_qtensor_normal(&b->Wdown, seed, base + 11, stddev);
  }
  {
    Tensor *t = &out->final_norm;
    t->ndim = 1;
    t->shape = (int *)malloc(sizeof(int));
    t->shape[0] = dm;
    t->size = (size_t)dm;
    t->grad = NULL;
    const size_t bytes = (((size_t)dm * sizeof(float)) + 63) & ~(size_t)63;
    t->data = (float *)aligned_alloc(64, bytes);
    fill_ones(t);
  }
  out->lm_head = qtensor_create(dm, c->vocab);
  synth_qtensor_normal(&out->lm_head, seed, 2 + 12 * c->n_layers, stddev);
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
