/* llmq_run - the reference CLI's `llama` subcommand (main.c:624-702, LLMQ
 * branch) on the GPU path of libllmq_cuda.so.
 *
 *   llmq_run llama <checkpoint.bin> [n_new=40]
 *   llmq_run upgrade-llma <v1.bin> <v2.bin>
 *
 * Same protocol as `transformer llama`: each stdin line holds space-separated
 * token ids; the sequence restarts (kv.len = 0), the ids are fed, and n_new
 * tokens are sampled with temperature 0.8, top-k 40, top-p 0.95 from one
 * xorshift64 stream seeded 1234 for the whole run (main.c:643-646).  Each
 * sampled id is printed as "t <id>" as soon as it exists, then
 * "gen: <prompt ids> <sampled ids>" (main.c:569-574).  Tools that spawn the
 * reference binary (tools/llama_stream.py:61-65) read the same lines.
 *
 * LLMQ (int8) checkpoints: the prompt goes through q_llama_prefill in one
 * pass (its logits equal those of the token-by-token loop); the first id is
 * drawn by sample_token from those logits, every later one by
 * q_llama_decode_step_sample inside the step graph.  LLMA (f32) checkpoints
 * run the fp32 path: the prompt token by token through
 * llama_decode_step_argmax, the last step's logits sampled, then
 * llama_decode_step_sample.  The ids equal the reference CLI's.  The LLMA
 * text mode (a tokenizer as 4th argument, main.c:584-622) needs the
 * reference's tokenizer and is not provided.
 *
 * `upgrade-llma` is the reference's tools/upgrade_llma.py: an LLMA v1
 * checkpoint rewritten as v2 (zero q/k/v biases inserted), streamed. */
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "llmq_cuda.h"

#define LLMQ_MAGIC 0x514D4C4Cu /* 'LLMQ' */
#define LLMA_MAGIC 0x414D4C4Cu /* 'LLMA' */

/* One stdin line of space-separated ids (main.c:562-572): a UTF-8 byte-order
 * mark is skipped, ids outside [0, vocab) are reported and skipped, at most
 * max_seq ids are kept. */
static int parse_ids(char *line, int *seq, int vocab, int max_seq) {
  char *p = line;
  if ((unsigned char)p[0] == 0xEF && (unsigned char)p[1] == 0xBB && (unsigned char)p[2] == 0xBF) p += 3;
  int n = 0;
  for (char *t = strtok(p, " \t\r\n"); t && n < max_seq; t = strtok(NULL, " \t\r\n")) {
    const int id = atoi(t);
    if (id < 0 || id >= vocab) {
      fprintf(stderr, "skip out-of-range id %d (vocab %d)\n", id, vocab);
      continue;
    }
    seq[n++] = id;
  }
  return n;
}

static void print_gen(const int *seq, int n) {
  printf("gen:");
  for (int i = 0; i < n; i++) printf(" %d", seq[i]);
  printf("\n");
  fflush(stdout);
}

static int fail(const char *what) {
  fprintf(stderr, "Error: %s: %s\n", what, q_llama_last_error_message());
  return 1;
}

/* The LLMA branch of main.c:675-700 on the fp32 GPU path. */
static int run_llama_f32(const char *path, int n_new) {
  const float temperature = 0.8f;
  const int top_k = 40;
  const float top_p = 0.95f;
  Rng rng = rng_create(1234);
  LlamaModel m;
  if (llmq_llama_model_load(path, &m) != 0) return 1;
  fprintf(stderr, "loaded LLMA (f32): vocab %d d_model %d layers %d heads %d kv %d head_dim %d d_ff %d\n", m.vocab,
          m.d_model, m.n_layers, m.n_heads, m.n_kv, m.head_dim, m.d_ff);
  LlamaKV kv = llama_kv_create(&m);
  if (q_llama_last_error()) {
    llmq_llama_model_free(&m);
    return fail("llama_kv_create");
  }
  float *row = (float *)malloc((size_t)m.vocab * sizeof(float));
  int shape[2] = {1, m.vocab};
  Tensor logits = {row, NULL, shape, 2, (size_t)m.vocab};
  int *seq = (int *)malloc((size_t)m.max_seq * sizeof(int));
  static char line[8192];
  int rc = 0;
  while (rc == 0 && fgets(line, sizeof line, stdin)) {
    int n = parse_ids(line, seq, m.vocab, m.max_seq);
    if (n == 0) continue;
    kv.len = 0;
    for (int i = 0; i < n && rc == 0; i++)
      if (llama_decode_step_argmax(&m, &kv, seq[i], i == n - 1 ? &logits : NULL) < 0) rc = fail("llama_decode_step");
    for (int s = 0; s < n_new && n < m.max_seq && rc == 0; s++) {
      const int nxt = s == 0 ? sample_token(&logits, 0, temperature, top_k, top_p, &rng)
                             : llama_decode_step_sample(&m, &kv, seq[n - 1], temperature, top_k, top_p, &rng, NULL);
      if (nxt < 0) {
        rc = fail("sampling");
        break;
      }
      seq[n++] = nxt;
      printf("t %d\n", nxt);
      fflush(stdout);
    }
    if (rc == 0) print_gen(seq, n);
  }
  free(seq);
  free(row);
  llama_kv_free(&kv);
  llmq_llama_model_free(&m);
  return rc;
}

static int run_llama(int argc, char **argv) {
  if (argc < 3) {
    fprintf(stderr, "usage: llmq_run llama <checkpoint.bin> [n_new=40]\n"
                    "  LLMA (f32) or LLMQ (int8) checkpoint, decoded on the GPU;\n"
                    "  reads space-separated token IDs per stdin line; prints 't <id>' per\n"
                    "  sampled token, then 'gen: <ids>'\n");
    return 2;
  }
  const int n_new = (argc > 3) ? atoi(argv[3]) : 40;
  FILE *pf = fopen(argv[2], "rb");
  if (!pf) {
    fprintf(stderr, "Error: cannot open '%s'\n", argv[2]);
    return 1;
  }
  unsigned int magic = 0;
  if (fread(&magic, sizeof magic, 1, pf) != 1) {
    fclose(pf);
    fprintf(stderr, "Error: '%s' too small\n", argv[2]);
    return 1;
  }
  fclose(pf);
  if (magic != LLMQ_MAGIC && magic != LLMA_MAGIC) {
    fprintf(stderr, "Error: '%s' is not an LLMA/LLMQ checkpoint\n", argv[2]);
    return 1;
  }
  if (magic == LLMA_MAGIC) {
    if (argc > 4) {
      fprintf(stderr, "Error: text mode (a tokenizer argument) is not provided; pass token ids\n");
      return 2;
    }
    return run_llama_f32(argv[2], n_new);
  }

  const float temperature = 0.8f;
  const int top_k = 40;
  const float top_p = 0.95f;
  Rng rng = rng_create(1234);

  QLlamaModel m;
  if (q_llama_model_load(argv[2], &m) != 0) return 1;
  fprintf(stderr, "loaded LLMQ (int8, in-memory): vocab %d d_model %d layers %d heads %d kv %d head_dim %d d_ff %d\n",
          m.vocab, m.d_model, m.n_layers, m.n_heads, m.n_kv, m.head_dim, m.d_ff);
  LlamaKV kv = q_llama_kv_create(&m);
  if (q_llama_last_error()) return fail("q_llama_kv_create");
  float *row = (float *)malloc((size_t)m.vocab * sizeof(float));
  int shape[2] = {1, m.vocab};
  Tensor logits = {row, NULL, shape, 2, (size_t)m.vocab};
  int *seq = (int *)malloc((size_t)m.max_seq * sizeof(int));
  static char line[8192];
  int rc = 0;
  while (rc == 0 && fgets(line, sizeof line, stdin)) {
    int n = parse_ids(line, seq, m.vocab, m.max_seq);
    if (n == 0) continue;
    kv.len = 0;
    q_llama_prefill(&m, &kv, seq, n, &logits);
    if (q_llama_last_error()) {
      rc = fail("q_llama_prefill");
      break;
    }
    for (int s = 0; s < n_new && n < m.max_seq; s++) {
      const int nxt = s == 0 ? sample_token(&logits, 0, temperature, top_k, top_p, &rng)
                             : q_llama_decode_step_sample(&m, &kv, seq[n - 1], temperature, top_k, top_p, &rng, NULL);
      if (nxt < 0) {
        rc = fail("sampling");
        break;
      }
      seq[n++] = nxt;
      printf("t %d\n", nxt);
      fflush(stdout);
    }
    if (rc == 0) print_gen(seq, n);
  }
  free(seq);
  free(row);
  llama_kv_free(&kv);
  q_llama_model_free(&m);
  return rc;
}

int main(int argc, char **argv) {
  if (argc > 1 && strcmp(argv[1], "llama") == 0) return run_llama(argc, argv);
  if (argc == 4 && strcmp(argv[1], "upgrade-llma") == 0) return llmq_llma_upgrade_v1(argv[2], argv[3]);
  fprintf(stderr, "usage: llmq_run llama <checkpoint.bin> [n_new=40]\n"
                  "       llmq_run upgrade-llma <v1.bin> <v2.bin>   (tools/upgrade_llma.py)\n");
  return 2;
}
