/* llmq_oracle.h - TEST INFRASTRUCTURE ONLY: the CPU checker for libllmq_cuda.so.
 *
 * A plain-C restatement of the reference's int8 decode path
 * (marjoncajocon/llm-project quant.c, matrix.c qacc_*, rmsnorm.c, rope.c,
 * llama.c q_* section, sampler.c).  Every function names the reference
 * lines it follows and performs the same fp32 operations in the same order,
 * so its results are bit-identical to the reference's (checked against the
 * reference sources compiled into oracle/_ref/ and against tests/golden/).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use
 * this code.  The product library never links or calls it.
 */
#ifndef LLMQ_ORACLE_H
#define LLMQ_ORACLE_H

#include <stdint.h>
#include "llmq_cuda.h"   /* struct layouts only */

#ifdef __cplusplus
extern "C" {
#endif

/* quant.c:10-27 */
void orc_quantize_int8_percol(const float *w, int rows, int cols, signed char *q, float *scale);
/* quant.c:29-33 */
void orc_dequantize_int8_percol(const signed char *q, const float *scale, int rows, int cols, float *w);
/* quant.c:69-78: per-row activation quantisation; returns the row scale. */
float orc_quantize_row(const float *a, int K, signed char *qa);
/* matrix.c:354-374: acc[j] = sum_k qa[k]*qw[k*N+j] (int32). */
void orc_qacc_columns(const signed char *qa, const signed char *qw, int K, int N, int32_t *acc);
/* quant.c:60-85 on raw pointers: A (M,K) f32, W codes (K,N) + scale[N], C (M,N). */
void orc_qmatmul(const float *A, int M, int K, const signed char *wq, const float *wscale, int N,
                 float *C);
/* rmsnorm.c:7-21 for one row. */
void orc_rmsnorm_row(const float *x, const float *gamma, int n, float eps, float *y);
/* rope.c:48-68 for one row (x holds n_heads*head_dim values). */
void orc_rope_heads_pos_row(float *x, int n_heads, int head_dim, float base, int pos);
/* sampler.c:8-21 */
int orc_argmax(const float *r, int n);
/* sampler.c:32-39: one xorshift64 step. */
unsigned long long orc_xorshift64(unsigned long long *state);
/* sampler.c:60-115 on one row of V logits; *state is Rng.state. */
int orc_sample_token(const float *l, int V, float temperature, int top_k, float top_p,
                     unsigned long long *state);

/* llama.c:513-526 / 290-294 */
LlamaKV orc_kv_create(const QLlamaModel *m);
void orc_kv_free(LlamaKV *kv);
/* llama.c:528-600: one decode step; logits has m->vocab floats. */
void orc_decode_step(const QLlamaModel *m, LlamaKV *kv, int token, float *logits);

/* llama.c:275-288 / 296-362: the fp32 (LLMA) model's cache and decode step. */
LlamaKV orc_f32_kv_create(const LlamaModel *m);
void orc_f32_decode_step(const LlamaModel *m, LlamaKV *kv, int token, float *logits);

/* llama.c:603-657: LLMQ v2 reader (0 ok, 1 error). */
int orc_model_load(const char *path, QLlamaModel *out);
void orc_model_free(QLlamaModel *m);
/* LLMQ v2 writer in the order llama.c:603-648 reads (0 ok, 1 error). */
int orc_model_save(const char *path, const QLlamaModel *m);

/* out[i] = expf(x) for the float x whose bit pattern is first + i, i < count:
 * the host C library's expf, threaded (reference for the device expf test). */
void orc_expf_bits(uint32_t first, uint64_t count, float *out);

/* llama.c:490-511: quantise an fp32 model. */
QLlamaModel orc_quantize_from(const LlamaModel *src);

#ifdef __cplusplus
}
#endif
#endif
