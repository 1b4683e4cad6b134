/* llmq_cuda.h - C ABI of libllmq_cuda.so, the B200 (sm_100a) implementation of the
 * int8 (W8A8) LLaMA-family KV-cache decode path of marjoncajocon/llm-project.
 *
 * The library is a link-time drop-in for the int8 half of the reference:
 *   quant.c in full (quant.h:15-33) and the QLlamaModel section of llama.c
 *   (llama.c:443-657, declared at llama.h:114-140) plus llama_kv_free (llama.h:102).
 * Every exported name, argument order, struct layout, ownership rule and return
 * convention below is the reference's, so a caller written against quant.h /
 * llama.h compiles and links unchanged.  All arithmetic runs on the GPU: the
 * results are bit-identical to the reference CPU code (same int8 codes, same
 * int32 accumulators, same fp32 rounding sequence, the same libm expf results).
 *
 * Additions (new names, same C style) carry a comment saying so.  No entry point
 * takes or returns a torch or CUDA type.  Compute functions that return void in the
 * reference keep returning void; their failures are reported by
 * q_llama_last_error() and a one-line message on stderr.
 */
#ifndef LLMQ_CUDA_H
#define LLMQ_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------- */
/* Host structs.  The guards are the reference headers' own include guards, so */
/* this header and tensor.h / quant.h / llama.h may be included in any order.  */
/* ------------------------------------------------------------------------- */
#ifndef TENSOR_H
#define TENSOR_H
/* Same layout as the reference Tensor (tensor.h:10-16): row-major f32 data,
 * optional grad, malloc'd shape array.  Tensors this library allocates use a
 * 64-byte aligned `data` block and a malloc'd `shape`, like tensor.c:33-60, so
 * the reference tensor_free can release them. */
typedef struct {
  float *data;
  float *grad;
  int *shape;
  int ndim;
  size_t size;
} Tensor;
#endif

#ifndef QUANT_H
#define QUANT_H
/* int8 weight, (rows=in, cols=out) row-major, one f32 scale per column
 * (quant.h:22-26).  x(M,rows) @ W -> (M,cols). */
typedef struct {
  int rows, cols;
  signed char *q;
  float *scale;
} QTensor;
#endif

#ifndef LLAMA_H
#define LLAMA_H
/* fp32 block / model (llama.h:19-36, 59-66).  Only read here, by
 * q_llama_quantize_from. */
typedef struct {
  int d_model, n_heads, n_kv, head_dim, d_ff;
  float rope_base, eps;
  Tensor attn_norm, Wq, Wk, Wv, b_q, b_k, b_v, Wo;
  Tensor ffn_norm, Wgate, Wup, Wdown;
} LlamaBlock;

typedef struct {
  int vocab, d_model, n_layers, n_heads, n_kv, head_dim, d_ff, max_seq;
  float rope_base, eps;
  Tensor wte;
  LlamaBlock *blocks;
  Tensor final_norm;
  Tensor lm_head;
} LlamaModel;

/* KV cache handle (llama.h:94-99).  `len` is the number of cached positions and
 * is the source of truth on every call: callers restart a sequence by writing
 * kv.len = 0 (main.c:661).  The cache itself lives on the GPU; the host arrays
 * k/v are allocated with the reference's shapes and are filled only by
 * q_llama_kv_sync_host(). */
typedef struct {
  int n_layers, max_seq, kv_dim;
  int len;
  float **k;
  float **v;
} LlamaKV;

/* int8 block / model (llama.h:114-127). */
typedef struct {
  Tensor attn_norm, ffn_norm;
  Tensor b_q, b_k, b_v;
  QTensor Wq, Wk, Wv, Wo, Wgate, Wup, Wdown;
} QLlamaBlock;

typedef struct {
  int vocab, d_model, n_layers, n_heads, n_kv, head_dim, d_ff, max_seq;
  float rope_base, eps;
  QTensor wte;
  QLlamaBlock *blocks;
  Tensor final_norm;
  QTensor lm_head;
} QLlamaModel;
#endif

#ifndef SAMPLER_H
#define SAMPLER_H
/* xorshift64 stream (sampler.h:13-15). */
typedef struct {
  unsigned long long state;
} Rng;
#endif

/* ========================================================================= */
/* quant.h entry points                                                       */
/* ========================================================================= */

/* Replaces quant.c:10-27 (declared quant.h:15).  Per-column symmetric int8
 * quantisation of a row-major (rows, cols) f32 matrix, computed on the GPU:
 * scale[j] = max_i|w[i,j]|/127 (1 for an all-zero column),
 * q = clamp(lrintf(w * (1/scale[j])), -127, 127).  Bit-identical to the
 * reference.  Host pointers in and out. */
void quantize_int8_percol(const float *w, int rows, int cols, signed char *q, float *scale);

/* Replaces quant.c:29-33 (quant.h:16).  w[i,j] = q[i,j] * scale[j], on the GPU. */
void dequantize_int8_percol(const signed char *q, const float *scale, int rows, int cols, float *w);

/* Replace quant.c:35-50 (quant.h:28-30).  Host allocation, as in the reference. */
QTensor qtensor_create(int rows, int cols);
void qtensor_free(QTensor *t);
void qtensor_quantize(QTensor *t, const float *w);

/* Replaces quant.c:60-85 (quant.h:33).  C(M,N) = W8A8 product of A(M,K) with W:
 * each row of A is quantised to int8 with its own absmax scale, multiplied
 * exactly in int32 against W's codes, and rescaled as a_scale*w_scale[j]*acc.
 * A, W and C are host memory, read and written on every call exactly like the
 * reference: each call copies A and W to the GPU (W is tiled there) and C back,
 * so a QTensor rewritten in place between calls is always seen. */
void qmatmul(const Tensor *A, const QTensor *W, Tensor *C);

/* ========================================================================= */
/* llama.h entry points (int8 model)                                          */
/* ========================================================================= */

/* Replaces llama.c:610-657 (llama.h:136).  Reads an LLMQ v2 checkpoint into
 * host memory exactly like the reference (0 on success, 1 with a message on
 * stderr on any error; the model is freed on failure) and uploads it to the
 * current GPU.  With a tensor-parallel group formed (q_llama_tp_init) it only
 * reads: the whole model is then meant to be cut with q_llama_model_shard. */
int q_llama_model_load(const char *path, QLlamaModel *out);

/* Replaces llama.c:483-488 (llama.h:129).  Frees host arrays and the device copy
 * (weights, every KV cache and CUDA graph made for this model). */
void q_llama_model_free(QLlamaModel *m);

/* Replaces llama.c:490-511 (llama.h:132).  Quantises an fp32 model on the GPU
 * (bit-identical codes and scales). */
QLlamaModel q_llama_quantize_from(const LlamaModel *src);

/* Replaces llama.c:513-526 (llama.h:140).  Creates the GPU KV cache
 * (head-major f32 [n_layers][n_kv][max_seq][head_dim], K and V) plus the reference-shaped host
 * arrays. */
LlamaKV q_llama_kv_create(const QLlamaModel *m);

/* Replaces llama.c:290-294 (llama.h:102) for caches made by q_llama_kv_create. */
void llama_kv_free(LlamaKV *kv);

/* Replaces llama.c:528-600 (llama.h:139).  Decodes `token` at position kv->len:
 * appends its K/V to the GPU cache, attends over 0..kv->len, writes the f32
 * logits (1, vocab) into the caller's host tensor and advances kv->len.  One
 * CUDA graph replay per call. */
void q_llama_decode_step(const QLlamaModel *m, LlamaKV *kv, int token, Tensor *logits);

/* ========================================================================= */
/* llama.h fp32 (LLMA) decode entry points                                   */
/* ========================================================================= */

/* Replaces llama.c:275-288 (llama.h:101): the KV cache of an fp32 model, on
 * the GPU (head-major as for the int8 model) plus the reference-shaped host
 * arrays.  The model's GPU copy is made on first use. */
LlamaKV llama_kv_create(const LlamaModel *m);

/* Replaces llama.c:296-362 (llama.h:106): one decode step of an fp32 model on
 * the GPU, bit-identical to the reference's.  Every product is fp32 with the
 * reference's accumulation order (matrix.c:178-199: one sequential chain per
 * output column, each product and sum rounded on its own); norms, RoPE,
 * attention and SwiGLU are the int8 path's kernels.  The model is
 * snapshotted at its first use: release the GPU copy with
 * llmq_llama_model_release (or llmq_llama_model_free) before editing it. */
void llama_decode_step(const LlamaModel *m, LlamaKV *kv, int token, Tensor *logits);

/* As llama_decode_step; returns the greedy next id (-1 on error); logits may
 * be NULL.  Additive extension. */
int llama_decode_step_argmax(const LlamaModel *m, LlamaKV *kv, int token, Tensor *logits);
/* As q_llama_decode_step_sample, for an fp32 model. */
int llama_decode_step_sample(const LlamaModel *m, LlamaKV *kv, int token, float temperature, int top_k,
                             float top_p, Rng *rng, Tensor *logits);
/* As q_llama_generate / q_llama_generate_sample, for an fp32 model. */
int llama_generate(const LlamaModel *m, LlamaKV *kv, int token, int n, int *ids);
int llama_generate_sample(const LlamaModel *m, LlamaKV *kv, int token, int n, float temperature, int top_k,
                          float top_p, Rng *rng, int *ids);

/* llama.c:390-440 under a name of this library: reads an LLMA (f32) or LLMQ
 * (int8, dequantised on load as quant.c:29-33) checkpoint into an fp32 model
 * in host memory (the GPU copy is made on first use).  Same messages and 0/1
 * return as llama_model_load.  Free with llmq_llama_model_free. */
int llmq_llama_model_load(const char *path, LlamaModel *out);
/* Frees a model made by llmq_llama_model_load / llmq_synth_model_f32 and its
 * GPU copy. */
void llmq_llama_model_free(LlamaModel *m);
/* Uploads / releases the GPU copy of an fp32 model (both otherwise implicit).
 * Returns 0 or an error code. */
int llmq_llama_model_upload(const LlamaModel *m);
void llmq_llama_model_release(const LlamaModel *m);

/* ========================================================================= */
/* sampler.h entry points (sampler.c, the generation loop's token choice)     */
/* ========================================================================= */

/* Replace sampler.c:26-30 and sampler.c:41-44 (host arithmetic, same stream). */
Rng rng_create(unsigned long long seed);
float rng_uniform(Rng *r);

/* Replaces sampler.c:8-21 (sampler.h:10): the first index of the largest
 * logit of row `row`, computed on the GPU. */
int sample_argmax(const Tensor *logits, int row);

/* Replaces sampler.c:60-115 (sampler.h:25-26): temperature, top-k and top-p
 * sampling of row `row` on the GPU, advancing *rng by one draw (none when
 * temperature <= 0).  The returned id equals the reference's for every input,
 * ties included (glibc's stable qsort order: p descending, then index).  The
 * GPU keeps up to 1024 candidates: top_k must be in 1..1024 unless vocab <=
 * 1024; otherwise -1 is returned with q_llama_last_error() set and *rng
 * unchanged. */
int sample_token(const Tensor *logits, int row, float temperature, int top_k, float top_p, Rng *rng);

/* ========================================================================= */
/* Additions (no counterpart in the reference headers)                        */
/* ========================================================================= */

enum {
  LLMQ_OK = 0,
  LLMQ_ERR_ARG = 1,      /* bad shape / id / position / null pointer */
  LLMQ_ERR_CUDA = 2,     /* a CUDA runtime call failed */
  LLMQ_ERR_NO_DEVICE = 3,/* no CUDA device, or not an sm_100 part */
  LLMQ_ERR_IO = 4,       /* checkpoint read / write failure */
  LLMQ_ERR_OOM = 5,      /* host or device allocation failed */
  LLMQ_ERR_STATE = 6     /* model / cache not known to this library */
};

/* Error code of the most recent failing call on this thread (LLMQ_OK if none)
 * and its message.  q_llama_clear_error resets both. */
int q_llama_last_error(void);
const char *q_llama_last_error_message(void);
void q_llama_clear_error(void);

/* As q_llama_decode_step, but also returns the greedy next token (first index
 * of the largest logit, the rule of sampler.c:8-21) computed on the GPU.
 * `logits` may be NULL, in which case no logits are copied to the host (4 bytes
 * cross PCIe per token).  Returns -1 on error. */
int q_llama_decode_step_argmax(const QLlamaModel *m, LlamaKV *kv, int token, Tensor *logits);

/* q_llama_decode_step followed by sample_token on its logits row
 * (main.c:663-668), with the sampler run on the GPU inside the same graph:
 * returns the drawn next token (-1 on error) and advances kv->len and *rng.
 * `logits` may be NULL.  temperature <= 0 takes the greedy id and draws
 * nothing; top_k follows sample_token's limit.  Additive extension. */
int q_llama_decode_step_sample(const QLlamaModel *m, LlamaKV *kv, int token, float temperature, int top_k,
                               float top_p, Rng *rng, Tensor *logits);

/* Sampled generation chained on the GPU: as q_llama_generate, with each next
 * token drawn by the sampler (the reference's loop of q_llama_decode_step and
 * sample_token, main.c:663-668).  ids[i] is the token drawn after step i;
 * kv->len advances by n and *rng by n draws.  Returns 0 or an error code. */
int q_llama_generate_sample(const QLlamaModel *m, LlamaKV *kv, int token, int n, float temperature, int top_k,
                            float top_p, Rng *rng, int *ids);

/* Batched decode: one token for each of B sequences at once.  Sequence b feeds
 * tokens[b] at position kvs[b]->len of its own cache; row b of `logits`
 * (B x vocab floats, caller-owned) receives its logits and every kvs[b]->len
 * advances by one.  Each row equals what q_llama_decode_step (llama.c:528-600)
 * gives for that sequence alone, bit for bit; the caches must be distinct.
 * The reference has no batch entry point: this is the additive
 * `q_llama_decode_batch` extension of the C API. */
void q_llama_decode_batch(const QLlamaModel *m, LlamaKV **kvs, const int *tokens, int B, Tensor *logits);

/* As q_llama_decode_batch, but writes the B greedy ids (first maximum,
 * sampler.c:8-21) to ids[] instead of logits.  Returns 0 or an error code. */
int q_llama_decode_batch_argmax(const QLlamaModel *m, LlamaKV **kvs, const int *tokens, int B, int *ids);

/* Prefill: feeds ids[0..n) at positions kv->len .. kv->len + n - 1 in one pass
 * (the tensor-core GEMMs see n rows).  The cache then equals that of n
 * q_llama_decode_step calls, and `logits` (1 x vocab, may be NULL) receives the
 * logits of the last id, bit for bit those of the n-th step.  kv->len advances
 * by n.  Additive extension (the reference feeds prompts token by token,
 * main.c:650-671). */
void q_llama_prefill(const QLlamaModel *m, LlamaKV *kv, const int *ids, int n, Tensor *logits);

/* As q_llama_prefill; returns the greedy id after the last prompt token, or -1
 * on error. */
int q_llama_prefill_argmax(const QLlamaModel *m, LlamaKV *kv, const int *ids, int n, Tensor *logits);

/* Kernels launched by the last q_llama_decode_batch[_argmax] or
 * q_llama_prefill[_argmax] call (diagnostic; no reference counterpart). */
long long llmq_last_launches(void);

/* ---- Tensor parallelism (the `q_llama_tp_init` extension; the reference is
 * single-process).  One process per GPU: select the device with
 * q_llama_set_device, have rank 0 make an id with q_llama_tp_unique_id and
 * hand its 128 bytes to every rank, then call q_llama_tp_init on all ranks
 * (it returns once all have joined).  A model whose tensors are shard `rank`
 * of `world` (llmq_synth_model_shard, q_llama_model_shard) then decodes as
 * one: Wq/Wk/Wv/Wgate/Wup and the lm-head by columns, Wo/Wdown by rows, with
 * an NCCL max-reduce of the activation absmax and a sum-reduce of the exact
 * int32 partial products per row-parallel product, and a max-reduce of the
 * argmax key.  Logits and greedy ids equal the single-GPU ones bit for bit;
 * q_llama_decode_step returns the whole logits row on every rank, and
 * q_llama_kv_sync_host fills only this rank's KV heads.  All ranks must make
 * the same calls in the same order.  Returns 0 or an error code. */
int q_llama_tp_unique_id(unsigned char *id /* 128 bytes */);
int q_llama_tp_init(int rank, int world, const unsigned char *id);
/* Releases the group's communicator (and the decode graphs that use it). */
void q_llama_tp_shutdown(void);

/* Copies the GPU KV cache rows [0, kv->len) into kv->k / kv->v (the
 * reference-shaped host arrays).  Returns LLMQ_OK or an error code. */
int q_llama_kv_sync_host(const QLlamaModel *m, LlamaKV *kv);

/* Writes an LLMQ v2 checkpoint (the layout q_llama_model_load reads,
 * llama.c:192-220 and llama.c:603-648): atomically, through `path`.tmp and a
 * rename.  Returns 0 on success, 1 with a message on stderr on error. */
int q_llama_model_save(const char *path, const QLlamaModel *m);

/* Replaces tools/upgrade_llma.py: an LLMA v1 checkpoint (no q/k/v biases)
 * becomes v2 with three zero bias vectors per layer inserted after Wv,
 * streamed in 4 MiB pieces.  Refuses non-LLMA, already-v2, truncated and
 * overlong files with the tool's messages; 0 on success, 1 on error. */
int llmq_llma_upgrade_v1(const char *src, const char *dst);

/* Model configuration, in LLMQ header order (llama.c:241-243). */
typedef struct {
  int vocab, d_model, n_layers, n_heads, n_kv, head_dim, d_ff, max_seq;
  float rope_base, eps;
} LlmqConfig;

/* Builds a seeded synthetic int8 model in host memory (not uploaded; the first
 * q_llama_kv_create / decode call uploads it).  Every 2-D weight is drawn
 * f32 N(0, stddev) from splitmix64 + Box-Muller keyed by (seed, tensor index,
 * element index), then quantised per column by the reference rule.  Norm gains
 * are 1; biases are 0, or N(0, stddev) when `with_bias` (the Qwen2 path).
 * Multi-threaded; the result does not depend on the thread count.
 * Returns 0 or an error code. */
int llmq_synth_model(const LlmqConfig *cfg, uint64_t seed, float stddev, int with_bias,
                     QLlamaModel *out);

/* The fp32 model an LLMQ checkpoint of llmq_synth_model(cfg, seed, stddev,
 * with_bias) loads as with llama_model_load (llama.c:419-427: every 2-D
 * tensor dequantised).  Free with llmq_llama_model_free.  Returns 0 or an
 * error code. */
int llmq_synth_model_f32(const LlmqConfig *cfg, uint64_t seed, float stddev, int with_bias, LlamaModel *out);

/* Tensor-parallel shard `rank` of `world` of the same synthetic model (no
 * reference counterpart): Wq/Wk/Wv and b_q/b_k/b_v keep the columns of this
 * rank's query and KV heads, Wgate/Wup its d_ff columns, lm_head its vocab
 * columns; Wo and Wdown keep the rows of its query dims and d_ff slice.  Every
 * kept code and per-column scale equals the whole model's (row shards keep the
 * scale of the whole column).  wte and the norms are whole; the config fields
 * are the whole model's.  Needs n_heads, n_kv, d_ff and vocab divisible by
 * world.  Returns 0 or an error code. */
int llmq_synth_model_shard(const LlmqConfig *cfg, uint64_t seed, float stddev, int with_bias, int rank,
                           int world, QLlamaModel *out);

/* Shard `rank` of `world` of a quickly generated benchmark model: codes uniform
 * in [-127, 127] and per-column scales uniform in [2e-4, 1e-3), seeded per
 * element, so a shard costs only its own elements (a 70B shard in seconds).
 * Same layout and shard rules as llmq_synth_model_shard; no reference
 * counterpart.  Returns 0 or an error code. */
int llmq_synth_model_fast_shard(const LlmqConfig *cfg, uint64_t seed, int rank, int world, QLlamaModel *out);

/* The same shard cut from a whole model held in host memory (for instance one
 * read by q_llama_model_load).  `out` is freed with q_llama_model_free.
 * Returns 0 or an error code. */
int q_llama_model_shard(const QLlamaModel *m, int rank, int world, QLlamaModel *out);

/* Fills an existing QTensor with uniform codes in [-127, 127] and uniform scales
 * in [1e-3, 1e-2), seeded (the isolated matvec sweep's weights). */
void llmq_synth_qtensor(QTensor *t, uint64_t seed);

/* Addition (the writer tools/convert_llama.py:73-97 is for converted models):
 * the model llmq_synth_model (fast = 0) or llmq_synth_model_fast_shard with
 * one shard (fast = 1, stddev and with_bias ignored) builds, written straight
 * to an LLMQ v2 file tensor by tensor, so no more than one tensor is ever in
 * host memory (a 70B-shaped file needs ~1 GB of RAM, not ~70 GB).  Byte for byte
 * what q_llama_model_save writes for that model; atomic like llama.c:230-269.
 * Returns 0 or an error code. */
int llmq_synth_model_save(const LlmqConfig *cfg, uint64_t seed, float stddev, int with_bias, int fast,
                          const char *path);

/* Upload / release the device copy of a model explicitly (both are otherwise
 * implicit).  Returns 0 or an error code. */
int q_llama_model_upload(const QLlamaModel *m);

/* Selects the CUDA device that later uploads, caches and standalone calls on
 * this thread use (one process per GPU: pass the local rank).  A model keeps
 * the device it was uploaded to.  Returns 0 or an error code. */
int q_llama_set_device(int device);

/* Greedy generation chained on the GPU: feeds `token` at position kv->len, then
 * keeps feeding the argmax of each step, for n steps in total (one CUDA graph
 * replay per step, no host round trip in between).  ids[i] receives the argmax
 * after step i; kv->len advances by n.  Returns 0 or an error code. */
int q_llama_generate(const QLlamaModel *m, LlamaKV *kv, int token, int n, int *ids);

/* GPU time in milliseconds of the last q_llama_decode_step[_argmax] (one step,
 * including its small host<->device copies) or q_llama_generate (all n steps),
 * from CUDA events on the model's stream. */
float q_llama_last_step_ms(void);

/* ---- diagnostics for tests and benchmarks ---- */

/* y[i] = expf(x[i]) evaluated on the GPU by the routine the decode kernels use
 * (bit-identical to the host C library's expf).  Returns 0 or an error code. */
int llmq_expf_device(const float *x, float *y, long long n);

/* Times `iters` back-to-back launches of one kernel of an uploaded model
 * (which: 0 fused QKV, 1 Wo, 2 fused W1|W3, 3 W2, 4 lm-head GEMV, 5 attention
 * over the first KV cache at its current position) with CUDA events on the
 * model's stream.  Launch i takes block (layer + i) mod n_layers, so
 * consecutive launches stream different weights; the launches are replayed
 * from one CUDA graph with programmatic dependent launch, as inside a decode
 * step, so the host's launch rate is not timed.  *ms_per_launch receives the mean
 * launch time and *bytes_per_launch the algorithmic bytes of one launch (GEMV:
 * int8 weights + f32 scales + f32 input + f32 output; attention: the K and V
 * rows read plus q and the output).  Returns 0 or an error code. */
int llmq_bench_gemv(const QLlamaModel *m, int which, int layer, int iters, float *ms_per_launch,
                    double *bytes_per_launch);

/* Kernels launched by one decode step: per layer QKV, attention (one fused
 * launch, or two), Wo, W1|W3, W2 (+ 2 absmax exchanges under tensor
 * parallelism); then lm-head and the step's bookkeeping. */
int llmq_kernels_per_step(const QLlamaModel *m);

/* Attention launches per layer of a batch-1 step with these dimensions: 1 (the
 * fused cluster kernel) or 2 (scores, then softmax and values; chosen when the
 * fused kernel's shared memory would not fit, or LLMQ_ATTN_TWO_KERNELS=1);
 * -1 without a suitable GPU. */
int llmq_attention_launches(int n_heads, int n_kv, int head_dim, int max_seq);

/* Times `iters` device-resident products C(M, N) = A(M, K) x W on the path
 * qmatmul uses (int8 GEMV for M <= 8, tcgen05 tensor cores for larger M), with
 * W tiled once and seeded A resident in device memory.  *ms receives the mean
 * time per product.  Returns 0 or an error code. */
int llmq_bench_qmatmul(const QTensor *W, int M, int iters, float *ms);

/* Runs one decode step of `token` at kv->len outside the CUDA graph, kernel by
 * kernel with CUDA events between the launches, writes each kernel's time in
 * milliseconds to ms[0 .. min(max_n, llmq_kernels_per_step(m))) and advances
 * kv->len like a decode step.  For attributing step time to kernels; the
 * kernels do not overlap here.  Returns 0 or an error code. */
int llmq_step_profile(const QLlamaModel *m, LlamaKV *kv, int token, float *ms, int max_n);

/* RMSNorm of the row x[W->rows] with gain gamma and epsilon eps
 * (rmsnorm.c:7-21), then qmatmul of the normalised row by W (quant.c:60-85):
 * out[W->cols], host arrays, computed by the GEMV with the RMSNorm prologue that
 * QKV, W1|W3 and the lm-head use in a decode step (for tests on chosen rows).
 * Returns 0 or an error code. */
int llmq_rmsnorm_qmatmul(const float *x, const float *gamma, float eps, const QTensor *W, float *out);

/* The RMSNorm's sum of squares (rmsnorm.c:15) as the GEMV prologues form it:
 * one thread block sums a row in the loop's order and rounding, its 32
 * segments run in parallel from candidate starts around estimated partial sums
 * and linked exactly.  For each of `rows` rows of
 * n floats (host array v), sums[2r] is the block's sum and sums[2r+1] the
 * one-thread loop's (equal bit for bit), misses[r] the segments whose exact
 * start was not a candidate (summed by one thread), cycles[2r] and
 * cycles[2r+1] the SM cycles of the two.  threads: block size, a multiple of
 * 32 in 64..1024.  Returns 0 or an error code. */
int llmq_spec_sum_check(const float *v, int rows, int n, int threads, float *sums, int *misses, long long *cycles);

/* Failure detection on one GPU (no reference counterpart): runs a two-rank
 * tensor-parallel exchange whose second rank is a local region nothing writes,
 * so the peer-flag waits give up after `polls` polls.  which 0: the absmax
 * exchange kernel; 1: the row-parallel GEMV.  The kernel returns by itself;
 * *err_word receives the device error word (1 = timeout) and *ms its duration.
 * Returns LLMQ_ERR_CUDA when the error word is set (as a decode step does),
 * else 0; frees everything it allocated. */
int llmq_tp_wait_timeout_check(int which, unsigned polls, int *err_word, float *ms);

/* ---- allocation-free entry point ---- */

/* No counterpart in the reference (it has no GPU).  The qmatmul product
 * (quant.c:60-85, bit-identical results) on buffers the caller already holds on
 * the current GPU, for callers that cannot call cudaMalloc where they multiply:
 * a host framework whose own memory pool already owns the GPU's memory, a plugin
 * that must not change the application's device-memory accounting, or a
 * latency-critical loop that cannot afford an allocation and the device
 * synchronisation of the matching cudaFree.
 *   A      device f32 [M][K]          Wq  device int8 [K][N], row-major (QTensor.q layout)
 *   Wscale device f32 [N]             C   device f32 [M][N], written
 *   stream a cudaStream_t (NULL: the default stream); the call only enqueues work.
 * M = 0 or N = 0 enqueue nothing; K = 0 writes zeros (A and Wq may then be NULL).
 * It allocates nothing: its scratch (split-K int32 sums, counters and the row's
 * activation scale) is one fixed __device__ array of 513 KiB inside the library,
 * held by every GPU that loads it until the process exits; hence N <= 131072
 * (larger N is rejected with LLMQ_ERR_ARG, nothing launched).  Every call looks
 * up that array's address (cudaGetSymbolAddress) with the caller's device
 * current; the first call on a device also loads it, so make that first call
 * before any stream capture.  All calls share the array and each clears the
 * words it sums into: calls that overlap on the GPU (other streams, other
 * threads) race and must be serialised by the caller.  Returns 0 or an error
 * code. */
int qmatmul_device_noalloc(const float *A, int M, int K, const signed char *Wq, const float *Wscale, int N,
                           float *C, void *stream);

#ifdef __cplusplus
}
#endif

#endif /* LLMQ_CUDA_H */
