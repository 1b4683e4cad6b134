/* link_check.c - TEST PROGRAM (not part of the library): the drop-in claim at
 * link level.  It includes the reference's own headers first (tensor.h,
 * quant.h, llama.h, sampler.h, from the reference checkout), then
 * include/llmq_cuda.h, and links against libllmq_cuda.so alone, so every
 * declaration the two headers share must agree and every call below must
 * resolve in this library.  It then runs the int8 half of the reference's
 * selftest part [21] (selftest.c:1215-1250): load the quantised model, create
 * its cache, decode ids {3, 7, 1, 9, 2, 5} one at a time with
 * q_llama_decode_step, and sample_argmax each row.  The six logits rows go to
 * argv[2] as raw f32, the six argmax ids to stdout; the calling test compares
 * them with the rows the reference produced for the same model. */
#include "tensor.h"
#include "quant.h"
#include "llama.h"
#include "sampler.h"

#include "llmq_cuda.h"

#include <stdio.h>
#include <stdlib.h>

int main(int argc, char **argv) {
  if (argc != 3) {
    fprintf(stderr, "usage: link_check <model.llmq> <logits.f32>\n");
    return 2;
  }
  QLlamaModel m;
  if (q_llama_model_load(argv[1], &m) != 0) return 1;
  LlamaKV kv = q_llama_kv_create(&m);
  /* a (1, vocab) logits tensor laid out as tensor.h:10-16 describes */
  int *shape = (int *)malloc(2 * sizeof(int));
  float *data = (float *)calloc((size_t)m.vocab, sizeof(float));
  if (!shape || !data) return 1;
  shape[0] = 1;
  shape[1] = m.vocab;
  Tensor logits = {data, NULL, shape, 2, (size_t)m.vocab};
  FILE *f = fopen(argv[2], "wb");
  if (!f) return 1;
  const int ids[6] = {3, 7, 1, 9, 2, 5};
  for (int i = 0; i < 6; i++) {
    q_llama_decode_step(&m, &kv, ids[i], &logits);
    if (q_llama_last_error() != 0) return 1;
    if (fwrite(logits.data, sizeof(float), (size_t)m.vocab, f) != (size_t)m.vocab) return 1;
    printf("%d\n", sample_argmax(&logits, 0));
  }
  fclose(f);
  printf("len %d\n", kv.len);
  llama_kv_free(&kv);
  q_llama_model_free(&m);
  free(data);
  free(shape);
  return 0;
}
