/* expf_window_check.c - CPU check of the device expf's fast paths
 * (libm_expf in llmq_kernels.cuh): for a normal float result, the decisions
 * taken from the 29 mantissa bits that the double-to-float rounding drops
 * must equal those of lx_expf_cr (libm_expf.h) for the same y = exp((double)x):
 *   |bits - 2^28| > 2^20          -> far from the midpoint: (float)y, not near;
 *   2^5 < |bits - 2^28| <= 2^20   -> near, decidable by y: the correctly rounded
 *                                    f = (float)y, and the float on the other side
 *                                    of y is one step of f's bit pattern.
 * Inputs whose y is within 2^5 of the midpoint take the general path on the
 * device and are not checked here.
 *   expf_window_check <stride>   checks every stride-th binary32 input
 * Exit status 0 when every checked input agrees. */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "libm_expf.h"

int main(int argc, char **argv) {
  const uint64_t stride = argc > 1 ? strtoull(argv[1], NULL, 10) : 1;
  uint64_t checked = 0, far = 0, nearish = 0, bad = 0;
  for (uint64_t i = 0; i < (1ull << 32); i += stride ? stride : 1) {
    const float x = lx_float((uint32_t)i);
    if (x != x) continue;
    const double y = exp((double)x);
    uint64_t yb;
    memcpy(&yb, &y, 8);
    const int ye = (int)((yb >> 52) & 0x7ffu);
    if (ye < 897 || ye > 1150) continue; /* not a normal float result: general path */
    const int dist = (int)(uint32_t)(yb & 0x1fffffffull) - (1 << 28);
    int near = 0;
    float lo = 0.0f, up = 0.0f;
    const float cr = lx_expf_cr(x, y, &near, &lo, &up);
    const float f = (float)y;
    ++checked;
    if (dist > (1 << 20) || dist < -(1 << 20)) {
      ++far;
      if (near || lx_bits(cr) != lx_bits(f)) {
        if (bad++ < 5) printf("far mismatch: x=%a y=%a\n", (double)x, y);
      }
    } else if (dist > (1 << 5) || dist < -(1 << 5)) {
      ++nearish;
      const uint32_t fb = lx_bits(f);
      const float other = lx_float((double)f < y ? fb + 1u : fb - 1u);
      const float ref_other = (cr == up) ? lo : up;
      if (!near || lx_bits(cr) != lx_bits(f) || lx_bits(other) != lx_bits(ref_other)) {
        if (bad++ < 5) printf("near mismatch: x=%a y=%a\n", (double)x, y);
      }
    }
  }
  printf("checked %llu inputs: %llu far, %llu near and decidable, %llu mismatches\n", (unsigned long long)checked,
         (unsigned long long)far, (unsigned long long)nearish, (unsigned long long)bad);
  return bad ? 1 : 0;
}
