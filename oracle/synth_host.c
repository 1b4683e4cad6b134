/* synth_host.c - TEST INFRASTRUCTURE ONLY.  The two host helpers the seeded
 * synthetic-model generator (llm-project_b200/csrc/llmq_synth.c) calls, so
 * that generator can also be built into oracle/_build/libsynth.so: the
 * benchmark's reference arm makes its inputs there and then runs the
 * reference's own code on them, without mapping libllmq_cuda.so.
 *
 * qtensor_create allocates as the reference's quant.c:35-41 does (malloc'd
 * codes and scales), so the reference's q_llama_model_free releases the
 * models built here. */
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>

#include "llmq_internal.h"

QTensor qtensor_create(int rows, int cols) {
  QTensor t;
  t.rows = rows;
  t.cols = cols;
  t.q = (signed char *)malloc((size_t)rows * cols > 0 ? (size_t)rows * cols : 1);
  t.scale = (float *)malloc(((size_t)cols > 0 ? (size_t)cols : 1) * sizeof(float));
  return t;
}

void llmq_set_error(int code, const char *fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  fprintf(stderr, "synth (error %d): ", code);
  vfprintf(stderr, fmt, ap);
  fputc('\n', stderr);
  va_end(ap);
}
