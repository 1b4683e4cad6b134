/* llmq_host_f32.c - host layer of the fp32 (LLMA) decode path.
 *
 *   llama_kv_create, llama_decode_step          llama.c:275-288, 296-362 (llama.h:101, 106) on the GPU
 *   llama_decode_step_argmax / _sample,
 *   llama_generate / _sample                    additions, as for the int8 model
 *   llmq_llama_model_load                       llama.c:390-440: an LLMA (f32) or LLMQ (int8,
 *                                               dequantised on load) checkpoint into an fp32 model
 *   llmq_synth_model_f32, llmq_llama_model_free seeded synthetic fp32 models
 *
 * The fp32 model struct is the reference's LlamaModel (llama.h:59-66); the
 * GPU copy is made on first use and kept until llmq_llama_model_release /
 * llmq_llama_model_free. */
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "llmq_internal.h"

#define LLMA_MAGIC 0x414D4C4Cu /* 'LLMA' (llama.c:192) */
#define LLMQ_MAGIC 0x514D4C4Cu /* 'LLMQ' (llama.c:193) */
#define LLMA_VERSION 2u        /* llama.c:194 */

/* 64-byte aligned, zero-filled tensor with a malloc'd shape (tensor.c:33-60):
 * (rows, cols), or a vector of `cols` when rows == 0. */
static Tensor f_new(int rows, int cols) {
  Tensor t;
  t.ndim = rows ? 2 : 1;
  t.shape = (int *)malloc(2 * sizeof(int));
  t.size = (size_t)(rows ? rows : 1) * (size_t)cols;
  const size_t bytes = (t.size * sizeof(float) + 63) & ~(size_t)63;
  t.data = (float *)aligned_alloc(64, bytes ? bytes : 64);
  t.grad = NULL;
  if (!t.shape || !t.data) {
    fprintf(stderr, "Error: aligned allocation failed\n");
    exit(EXIT_FAILURE);
  }
  if (rows) {
    t.shape[0] = rows;
    t.shape[1] = cols;
  } else {
    t.shape[0] = cols;
  }
  memset(t.data, 0, bytes ? bytes : 64);
  return t;
}

static void f_del(Tensor *t) {
  free(t->data);
  free(t->shape);
  t->data = NULL;
  t->shape = NULL;
}

/* The shapes of llama.c:139-158 (model_create_ex). */
static LlamaModel f_model_alloc(const int32_t *c, const float *f) {
  LlamaModel m;
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
  const int dm = m.d_model, qd = m.n_heads * m.head_dim, kvd = m.n_kv * m.head_dim;
  m.wte = f_new(m.vocab, dm);
  m.blocks = (LlamaBlock *)calloc((size_t)m.n_layers, sizeof(LlamaBlock));
  for (int l = 0; l < m.n_layers; l++) {
    LlamaBlock *b = &m.blocks[l];
    b->d_model = dm;
    b->n_heads = m.n_heads;
    b->n_kv = m.n_kv;
    b->head_dim = m.head_dim;
    b->d_ff = m.d_ff;
    b->rope_base = m.rope_base;
    b->eps = m.eps;
    b->attn_norm = f_new(0, dm);
    b->Wq = f_new(dm, qd);
    b->Wk = f_new(dm, kvd);
    b->Wv = f_new(dm, kvd);
    b->b_q = f_new(0, qd);
    b->b_k = f_new(0, kvd);
    b->b_v = f_new(0, kvd);
    b->Wo = f_new(qd, dm);
    b->ffn_norm = f_new(0, dm);
    b->Wgate = f_new(dm, m.d_ff);
    b->Wup = f_new(dm, m.d_ff);
    b->Wdown = f_new(m.d_ff, dm);
  }
  m.final_norm = f_new(0, dm);
  m.lm_head = f_new(dm, m.vocab);
  return m;
}

/* The tensors in checkpoint order (llama.c:199-220). */
static int f_collect(LlamaModel *m, Tensor **list) {
  int n = 0;
  list[n++] = &m->wte;
  for (int l = 0; l < m->n_layers; l++) {
    LlamaBlock *b = &m->blocks[l];
    Tensor *t[12] = {&b->attn_norm, &b->Wq, &b->Wk, &b->Wv, &b->b_q, &b->b_k,
                     &b->b_v,       &b->Wo, &b->ffn_norm, &b->Wgate, &b->Wup, &b->Wdown};
    for (int i = 0; i < 12; i++) list[n++] = t[i];
  }
  list[n++] = &m->final_norm;
  list[n++] = &m->lm_head;
  return n;
}

LLMQ_API void llmq_llama_model_release(const LlamaModel *m) { llmqd_model_release_f32(m); }

LLMQ_API void llmq_llama_model_free(LlamaModel *m) {
  if (!m || !m->blocks) return;
  llmqd_model_release_f32(m);
  Tensor **list = (Tensor **)malloc((size_t)(3 + 12 * m->n_layers) * sizeof(Tensor *));
  const int n = f_collect(m, list);
  for (int i = 0; i < n; i++) f_del(list[i]);
  free(list);
  free(m->blocks);
  m->blocks = NULL;
}

LLMQ_API int llmq_llama_model_upload(const LlamaModel *m) {
  return llmqd_model_upload_f32(m) ? LLMQ_OK : q_llama_last_error();
}

/* ------------------------------------------------------------------ loader */
static int rd(FILE *f, void *p, size_t sz, size_t n) { return fread(p, sz, n, f) == n; }

LLMQ_API int llmq_llama_model_load(const char *path, LlamaModel *out) {
  FILE *f = fopen(path, "rb");
  if (!f) {
    fprintf(stderr, "Error: cannot open '%s' for reading\n", path);
    llmq_set_error(LLMQ_ERR_IO, "llmq_llama_model_load: cannot open '%s'", path);
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
  const int quant = hdr[0] == LLMQ_MAGIC;
  if ((hdr[0] != LLMA_MAGIC && !quant) || hdr[1] != LLMA_VERSION) {
    fprintf(stderr, "Error: '%s' is not a v%u LLMA/LLMQ checkpoint\n", path, LLMA_VERSION);
    fclose(f);
    return 1;
  }
  if (!llmq_config_valid(cfg)) {
    fprintf(stderr, "Error: '%s' has an invalid/unsupported config\n", path);
    fclose(f);
    return 1;
  }
  *out = f_model_alloc(cfg, fcfg);
  Tensor **list = (Tensor **)malloc((size_t)(3 + 12 * out->n_layers) * sizeof(Tensor *));
  const int n = f_collect(out, list);
  int ok = 1;
  for (int i = 0; i < n && ok; i++) {
    Tensor *t = list[i];
    if (quant && t->ndim == 2) {
      /* per-column scales, then the codes, dequantised as quant.c:29-33 does */
      const int rows = t->shape[0], cols = t->shape[1];
      float *scale = (float *)malloc((size_t)cols * sizeof(float));
      signed char *q = (signed char *)malloc((size_t)rows * cols);
      ok = scale && q && rd(f, scale, sizeof(float), (size_t)cols) && rd(f, q, 1, (size_t)rows * cols);
      if (ok)
        for (size_t r = 0; r < (size_t)rows; r++)
          for (size_t c = 0; c < (size_t)cols; c++) t->data[r * cols + c] = (float)q[r * cols + c] * scale[c];
      free(scale);
      free(q);
    } else {
      ok = rd(f, t->data, sizeof(float), t->size);
    }
  }
  free(list);
  fclose(f);
  if (!ok) {
    fprintf(stderr, "Error: '%s' is truncated (bad weights)\n", path);
    llmq_llama_model_free(out);
    return 1;
  }
  return 0; /* the GPU copy is made on first use (or by llmq_llama_model_upload) */
}

/* --------------------------------------------------------------- synthetic */
typedef struct {
  const QTensor *src;
  Tensor *dst;
  int r0, r1;
} DqJob;

static void *dq_run(void *arg) {
  const DqJob *j = (const DqJob *)arg;
  const int cols = j->src->cols;
  for (size_t r = (size_t)j->r0; r < (size_t)j->r1; r++)
    for (size_t c = 0; c < (size_t)cols; c++)
      j->dst->data[r * cols + c] = (float)j->src->q[r * cols + c] * j->src->scale[c];
  return NULL;
}

static void dequant_into(Tensor *dst, const QTensor *src) {
  enum { kMaxJobs = 64 };
  pthread_t th[kMaxJobs];
  DqJob jobs[kMaxJobs];
  int nt = src->rows < 256 ? 1 : 32;
  for (int t = 0; t < nt; t++) {
    jobs[t].src = src;
    jobs[t].dst = dst;
    jobs[t].r0 = (int)((long long)t * src->rows / nt);
    jobs[t].r1 = (int)((long long)(t + 1) * src->rows / nt);
    if (pthread_create(&th[t], NULL, dq_run, &jobs[t]) != 0) {
      dq_run(&jobs[t]);
      th[t] = 0;
    }
  }
  for (int t = 0; t < nt; t++)
    if (th[t]) pthread_join(th[t], NULL);
}

static void vcopy(Tensor *dst, const Tensor *src) {
  if (src->data) memcpy(dst->data, src->data, dst->size * sizeof(float));
}

/* The fp32 model an LLMQ checkpoint of llmq_synth_model(cfg, seed, stddev,
 * with_bias) loads as (llama.c:419-427: every 2-D tensor dequantised). */
LLMQ_API int llmq_synth_model_f32(const LlmqConfig *cfg, uint64_t seed, float stddev, int with_bias,
                                  LlamaModel *out) {
  QLlamaModel q;
  const int rc = llmq_synth_model(cfg, seed, stddev, with_bias, &q);
  if (rc != LLMQ_OK) return rc;
  const int32_t c[8] = {cfg->vocab, cfg->d_model, cfg->n_layers, cfg->n_heads, cfg->n_kv, cfg->head_dim, cfg->d_ff,
                        cfg->max_seq};
  const float fc[2] = {cfg->rope_base, cfg->eps};
  *out = f_model_alloc(c, fc);
  dequant_into(&out->wte, &q.wte);
  for (int l = 0; l < cfg->n_layers; l++) {
    const QLlamaBlock *a = &q.blocks[l];
    LlamaBlock *b = &out->blocks[l];
    vcopy(&b->attn_norm, &a->attn_norm);
    vcopy(&b->ffn_norm, &a->ffn_norm);
    vcopy(&b->b_q, &a->b_q);
    vcopy(&b->b_k, &a->b_k);
    vcopy(&b->b_v, &a->b_v);
    dequant_into(&b->Wq, &a->Wq);
    dequant_into(&b->Wk, &a->Wk);
    dequant_into(&b->Wv, &a->Wv);
    dequant_into(&b->Wo, &a->Wo);
    dequant_into(&b->Wgate, &a->Wgate);
    dequant_into(&b->Wup, &a->Wup);
    dequant_into(&b->Wdown, &a->Wdown);
  }
  vcopy(&out->final_norm, &q.final_norm);
  dequant_into(&out->lm_head, &q.lm_head);
  q_llama_model_free(&q);
  return LLMQ_OK;
}

/* ------------------------------------------------------------ decode steps */
LLMQ_API LlamaKV llama_kv_create(const LlamaModel *m) {
  LlamaKV kv;
  kv.n_layers = m->n_layers;
  kv.max_seq = m->max_seq;
  kv.kv_dim = m->n_kv * m->head_dim;
  kv.len = 0;
  kv.k = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  kv.v = (float **)malloc((size_t)m->n_layers * sizeof(float *));
  for (int l = 0; l < m->n_layers; l++) {
    /* host mirror, as for the int8 model: filled only on request */
    kv.k[l] = (float *)malloc((size_t)m->max_seq * kv.kv_dim * sizeof(float));
    kv.v[l] = (float *)malloc((size_t)m->max_seq * kv.kv_dim * sizeof(float));
  }
  if (!llmqd_kv_register_f32(m, &kv))
    fprintf(stderr, "llama_kv_create: GPU cache not created (%s)\n", q_llama_last_error_message());
  return kv;
}

static int logits_ok(const LlamaModel *m, const Tensor *logits, const char *who) {
  if (logits && (!logits->data || logits->size < (size_t)m->vocab)) {
    llmq_set_error(LLMQ_ERR_ARG, "%s: logits tensor must hold %d floats", who, m->vocab);
    return 0;
  }
  return 1;
}

LLMQ_API void llama_decode_step(const LlamaModel *m, LlamaKV *kv, int token, Tensor *logits) {
  if (!logits || !logits_ok(m, logits, "llama_decode_step")) {
    if (!logits) llmq_set_error(LLMQ_ERR_ARG, "llama_decode_step: logits tensor is NULL");
    return;
  }
  if (llmqd_decode_f32(m, kv, token, logits->data, NULL, NULL)) kv->len = kv->len + 1;
}

LLMQ_API int llama_decode_step_argmax(const LlamaModel *m, LlamaKV *kv, int token, Tensor *logits) {
  if (!logits_ok(m, logits, "llama_decode_step_argmax")) return -1;
  int next = -1;
  if (!llmqd_decode_f32(m, kv, token, logits ? logits->data : NULL, &next, NULL)) return -1;
  kv->len = kv->len + 1;
  return next;
}

LLMQ_API int llama_decode_step_sample(const LlamaModel *m, LlamaKV *kv, int token, float temperature, int top_k,
                                      float top_p, Rng *rng, Tensor *logits) {
  if (!rng || !logits_ok(m, logits, "llama_decode_step_sample")) {
    if (!rng) llmq_set_error(LLMQ_ERR_ARG, "llama_decode_step_sample: rng is NULL");
    return -1;
  }
  int next = -1;
  float *out = logits ? logits->data : NULL;
  if (temperature <= 0.0f) { /* greedy (sampler.c:65-67): the fused argmax, no draw */
    if (!llmqd_decode_f32(m, kv, token, out, &next, NULL)) return -1;
  } else {
    LlmqSample s = llmq_sample_settings(m->vocab, temperature, top_k, top_p, rng);
    if (!llmqd_decode_f32(m, kv, token, out, &next, &s)) return -1;
    rng->state = s.rng;
  }
  kv->len = kv->len + 1;
  return next;
}

LLMQ_API int llama_generate(const LlamaModel *m, LlamaKV *kv, int token, int n, int *ids) {
  if (n < 0 || (n > 0 && !ids)) {
    llmq_set_error(LLMQ_ERR_ARG, "llama_generate: bad arguments");
    return LLMQ_ERR_ARG;
  }
  if (!llmqd_generate_f32(m, kv, token, n, ids, NULL)) return q_llama_last_error();
  kv->len = kv->len + n;
  return LLMQ_OK;
}

LLMQ_API int llama_generate_sample(const LlamaModel *m, LlamaKV *kv, int token, int n, float temperature, int top_k,
                                   float top_p, Rng *rng, int *ids) {
  if (n < 0 || (n > 0 && !ids) || !rng) {
    llmq_set_error(LLMQ_ERR_ARG, "llama_generate_sample: bad arguments");
    return LLMQ_ERR_ARG;
  }
  if (temperature <= 0.0f) {
    if (!llmqd_generate_f32(m, kv, token, n, ids, NULL)) return q_llama_last_error();
  } else {
    LlmqSample s = llmq_sample_settings(m->vocab, temperature, top_k, top_p, rng);
    if (!llmqd_generate_f32(m, kv, token, n, ids, &s)) return q_llama_last_error();
    rng->state = s.rng;
  }
  kv->len = kv->len + n;
  return LLMQ_OK;
}

/* ------------------------------------------------------- LLMA v1 -> v2 upgrade */
/* Copies n f32 values from src to dst in 4 MiB pieces; 0 when src runs short. */
static int copy_floats(FILE *src, FILE *dst, size_t n, char *buf) {
  size_t left = n * sizeof(float);
  while (left) {
    const size_t take = left < ((size_t)1 << 22) ? left : ((size_t)1 << 22);
    if (fread(buf, 1, take, src) != take) return 0;
    if (fwrite(buf, 1, take, dst) != take) return -1;
    left -= take;
  }
  return 1;
}

/* The reference's tools/upgrade_llma.py in C: an LLMA v1 checkpoint (no q/k/v
 * biases) becomes v2 by copying every tensor across and inserting three zero
 * bias vectors after each layer's Wv (the v2 canonical order, llama.c:199-219).
 * Streams the file in 4 MiB pieces, so a checkpoint of any size needs no more
 * memory than that.  Refuses files that are not LLMA, are already v2 or later,
 * are truncated or have trailing bytes, with the tool's messages on stderr;
 * returns 0 on success, 1 on error (dst then holds no partial file). */
LLMQ_API int llmq_llma_upgrade_v1(const char *src_path, const char *dst_path) {
  FILE *f = fopen(src_path, "rb");
  if (!f) {
    fprintf(stderr, "error: cannot open '%s'\n", src_path);
    llmq_set_error(LLMQ_ERR_IO, "llmq_llma_upgrade_v1: cannot open '%s'", src_path);
    return 1;
  }
  uint32_t hdr[2];
  int32_t cfg[8];
  float fcfg[2];
  if (fread(hdr, 4, 2, f) != 2 || fread(cfg, 4, 8, f) != 8 || fread(fcfg, 4, 2, f) != 2) {
    fprintf(stderr, "error: '%s' is too small to be an LLMA checkpoint\n", src_path);
    llmq_set_error(LLMQ_ERR_IO, "llmq_llma_upgrade_v1: '%s' is too small", src_path);
    fclose(f);
    return 1;
  }
  if (hdr[0] != 0x414D4C4Cu) {
    fprintf(stderr, "error: '%s' is not an LLMA checkpoint (magic %#x)\n", src_path, hdr[0]);
    llmq_set_error(LLMQ_ERR_ARG, "llmq_llma_upgrade_v1: '%s' is not an LLMA checkpoint", src_path);
    fclose(f);
    return 1;
  }
  if (hdr[1] != 1u) {
    fprintf(stderr, "error: '%s' is already version %u, nothing to do\n", src_path, hdr[1]);
    llmq_set_error(LLMQ_ERR_ARG, "llmq_llma_upgrade_v1: '%s' is already version %u", src_path, hdr[1]);
    fclose(f);
    return 1;
  }
  for (int i = 0; i < 8; i++)
    if (cfg[i] <= 0) {
      fprintf(stderr, "error: '%s' has an invalid config\n", src_path);
      llmq_set_error(LLMQ_ERR_ARG, "llmq_llma_upgrade_v1: '%s' has an invalid config", src_path);
      fclose(f);
      return 1;
    }
  const size_t vocab = (size_t)cfg[0], dm = (size_t)cfg[1], qd = (size_t)cfg[3] * cfg[5], kvd = (size_t)cfg[4] * cfg[5];
  const size_t dff = (size_t)cfg[6];
  const int n_layers = cfg[2];
  const size_t plen = strlen(dst_path);
  char *tmp = (char *)malloc(plen + 5);
  char *buf = (char *)malloc((size_t)1 << 22);
  float *zeros = (float *)calloc(qd + 2 * kvd, sizeof(float));
  FILE *g = NULL;
  if (tmp && buf && zeros) {
    memcpy(tmp, dst_path, plen);
    memcpy(tmp + plen, ".tmp", 5);
    g = fopen(tmp, "wb");
  }
  if (!g) {
    fprintf(stderr, "error: cannot open '%s' for writing\n", dst_path);
    llmq_set_error(LLMQ_ERR_IO, "llmq_llma_upgrade_v1: cannot write '%s'", dst_path);
    free(tmp);
    free(buf);
    free(zeros);
    fclose(f);
    return 1;
  }
  const uint32_t hdr2[2] = {0x414D4C4Cu, 2u};
  int st = fwrite(hdr2, 4, 2, g) == 2 && fwrite(cfg, 4, 8, g) == 8 && fwrite(fcfg, 4, 2, g) == 2 ? 1 : -1;
  if (st > 0) st = copy_floats(f, g, vocab * dm, buf); /* wte */
  for (int l = 0; l < n_layers && st > 0; l++) {
    st = copy_floats(f, g, dm, buf);                           /* attn_norm */
    if (st > 0) st = copy_floats(f, g, dm * qd, buf);          /* Wq */
    if (st > 0) st = copy_floats(f, g, dm * kvd, buf);         /* Wk */
    if (st > 0) st = copy_floats(f, g, dm * kvd, buf);         /* Wv */
    if (st > 0 && fwrite(zeros, sizeof(float), qd + 2 * kvd, g) != qd + 2 * kvd) st = -1; /* b_q, b_k, b_v */
    if (st > 0) st = copy_floats(f, g, qd * dm, buf);          /* Wo */
    if (st > 0) st = copy_floats(f, g, dm, buf);               /* ffn_norm */
    if (st > 0) st = copy_floats(f, g, dm * dff, buf);         /* Wgate */
    if (st > 0) st = copy_floats(f, g, dm * dff, buf);         /* Wup */
    if (st > 0) st = copy_floats(f, g, dff * dm, buf);         /* Wdown */
  }
  if (st > 0) st = copy_floats(f, g, dm, buf);                 /* final_norm */
  if (st > 0) st = copy_floats(f, g, dm * vocab, buf);         /* lm_head */
  int trailing = 0;
  if (st > 0) trailing = fgetc(f) != EOF;
  fclose(f);
  int ok = st > 0 && !trailing;
  ok = (fclose(g) == 0) && ok;
  if (ok && rename(tmp, dst_path) != 0) {
    remove(dst_path);
    ok = rename(tmp, dst_path) == 0;
  }
  if (!ok) {
    remove(tmp);
    if (st == 0)
      fprintf(stderr, "error: input '%s' truncated\n", src_path);
    else if (trailing)
      fprintf(stderr, "error: trailing bytes in '%s' — layout assumption wrong\n", src_path);
    else
      fprintf(stderr, "error: failed while writing '%s'\n", dst_path);
    llmq_set_error(LLMQ_ERR_IO, "llmq_llma_upgrade_v1: %s", st == 0 ? "input truncated" : trailing ? "trailing bytes"
                                                                                          : "write failed");
  }
  free(tmp);
  free(buf);
  free(zeros);
  return ok ? 0 : 1;
}
