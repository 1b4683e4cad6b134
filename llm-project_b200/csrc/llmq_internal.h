/* llmq_internal.h - internal C interface between the C11 host layer
 * (llmq_host.c, llmq_synth.c) and the CUDA runtime layer (llmq_dev.cu).
 * Nothing here is exported from libllmq_cuda.so. */
#ifndef LLMQ_INTERNAL_H
#define LLMQ_INTERNAL_H

#include <stddef.h>
#include <stdint.h>

#include "llmq_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

#define LLMQ_API __attribute__((visibility("default")))
#define LLMQ_HIDDEN __attribute__((visibility("hidden")))

/* error state (thread local) */
LLMQ_HIDDEN void llmq_set_error(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));

/* RoPE angle tables for positions [0, max_seq): cos/sin of pos * base^(-2k/hd),
 * evaluated with the host libm exactly as rope.c:59-61 does. */
LLMQ_HIDDEN void llmq_rope_tables(float base, int head_dim, int max_seq, float *cos_out, float *sin_out);

/* ---- device layer (llmq_dev.cu); all return 1 on success, 0 with the error set */
LLMQ_HIDDEN int llmqd_quantize(const float *w, int rows, int cols, signed char *q, float *scale);
LLMQ_HIDDEN int llmqd_dequantize(const signed char *q, const float *scale, int rows, int cols, float *w);
LLMQ_HIDDEN int llmqd_qmatmul(const float *A, int M, const QTensor *W, float *C);

LLMQ_HIDDEN int llmqd_model_upload(const QLlamaModel *m);
LLMQ_HIDDEN void llmqd_model_release(const QLlamaModel *m);
LLMQ_HIDDEN int llmqd_kv_register(const QLlamaModel *m, const LlamaKV *kv);
LLMQ_HIDDEN void llmqd_kv_release(const LlamaKV *kv);
/* One decode step at position kv->len.  logits (may be NULL) receives vocab
 * floats; *next receives the greedy id. */
LLMQ_HIDDEN int llmqd_decode(const QLlamaModel *m, const LlamaKV *kv, int token, float *logits, int *next);
/* n greedy steps chained on the device starting from `token` at kv->len;
 * ids[i] = argmax after step i. */
LLMQ_HIDDEN int llmqd_generate(const QLlamaModel *m, const LlamaKV *kv, int token, int n, int *ids);
LLMQ_HIDDEN int llmqd_kv_download(const QLlamaModel *m, const LlamaKV *kv, int len);
/* Multi-row passes: B sequences one token each (batched decode), or n prompt
 * tokens of one sequence (prefill).  logits/ids may be NULL. */
LLMQ_HIDDEN int llmqd_decode_rows(const QLlamaModel *m, LlamaKV *const *kvs, const int *tokens, int B,
                                  float *logits, int *ids);
LLMQ_HIDDEN int llmqd_prefill(const QLlamaModel *m, const LlamaKV *kv, const int *ids, int n, float *logits,
                              int *next);
LLMQ_HIDDEN float llmqd_last_ms(void);

/* Sampler settings (sampler.c:60-115) as the device keeps them: k is the
 * number of candidates top-k keeps (top_k when 0 < top_k < vocab, else vocab,
 * sampler.c:87-88); rng is Rng.state (sampler.h). */
typedef struct {
  float temperature;
  int k;
  float top_p;
  int pad;
  unsigned long long rng;
} LlmqSample;
/* As llmqd_decode, with the next token drawn by the sampler; smp->rng advances. */
LLMQ_HIDDEN int llmqd_decode_sample(const QLlamaModel *m, const LlamaKV *kv, int token, float *logits, int *next,
                                    LlmqSample *smp);
/* As llmqd_generate, each next token drawn by the sampler. */
LLMQ_HIDDEN int llmqd_generate_sample(const QLlamaModel *m, const LlamaKV *kv, int token, int n, int *ids,
                                      LlmqSample *smp);
/* One host logits row of V floats sampled on the current device. */
LLMQ_HIDDEN int llmqd_sample_row(const float *row, int V, LlmqSample *smp, int *id);
/* The device form of one sampler call: top_k resolved to the number of
 * candidates it keeps (sampler.c:87-88). */
LLMQ_HIDDEN LlmqSample llmq_sample_settings(int vocab, float temperature, int top_k, float top_p, const Rng *rng);
/* LLMA / LLMQ header check (llama.c:371-386). */
LLMQ_HIDDEN int llmq_config_valid(const int32_t *cfg);

/* ---- fp32 (LLMA) models: the same decode step with fp32 products */
LLMQ_HIDDEN int llmqd_model_upload_f32(const LlamaModel *m);
LLMQ_HIDDEN void llmqd_model_release_f32(const LlamaModel *m);
LLMQ_HIDDEN int llmqd_kv_register_f32(const LlamaModel *m, const LlamaKV *kv);
/* One step; logits / next / smp may be NULL (smp: draw the next token). */
LLMQ_HIDDEN int llmqd_decode_f32(const LlamaModel *m, const LlamaKV *kv, int token, float *logits, int *next,
                                 LlmqSample *smp);
/* n device-chained steps (greedy, or drawn when smp is set). */
LLMQ_HIDDEN int llmqd_generate_f32(const LlamaModel *m, const LlamaKV *kv, int token, int n, int *ids,
                                   LlmqSample *smp);
/* Size of this process's tensor-parallel group (1 if none). */
LLMQ_HIDDEN int llmqd_tp_world(void);

#ifdef __cplusplus
}
#endif
#endif
