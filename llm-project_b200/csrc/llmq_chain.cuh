// llmq_chain.cuh - the arithmetic of a sequential f32 sum of non-negative
// terms, ((0 + v_0) + v_1) + ... rounded after every add exactly as a C loop
// does, when a thread block evaluates it in windows (the sampler's softmax
// denominator, sampler.c:79, of up to 128K terms; one thread needs ~4.5
// cycles per term):
//  * While the running sum s stays inside one binade, its grid spacing u is
//    fixed, and each rounded add moves s by a whole number of grid steps,
//    round(v / u), which does not depend on s.
//  * Two exceptions depend on s:
//    - v / u ending in exactly one half: the add rounds to even, which
//      depends on the parity of s / u;
//    - an add that may take s into the next binade.
//  * So a window is one block scan of the integer step counts. The half-way
//    cases are resolved in order from the scanned prefix. The first add that
//    may leave the binade is done on its own with one rounded add, and the
//    next window starts after it.
// The result is the loop's, bit for bit. A CPU restatement of this logic is
// checked against the loop in the CPU tests.  (For the 4096-term RMSNorm sum
// the windows do not pay: with a handful of binade crossings per row, each a
// dependent pass of scans and barriers, they were no faster than the loop.)
#pragma once

#include <cstdint>
#include <cuda_runtime.h>


namespace llmq {

constexpr uint32_t kChainSat = 1u << 30;  // step counts saturate here (>= 2^24 ends the binade)

// Grid steps of v >= 0 on the grid of spacing 2^uexp: n = floor(v / u),
// r = v / u rounded to nearest, tie when v / u ends in exactly one half (then
// r = n).  Counts saturate at kChainSat.
struct ChainStep {
  uint32_t n, r;
  bool tie;
};
__device__ __forceinline__ ChainStep chain_step(uint32_t vb, int uexp) {
  const uint32_t ef = vb >> 23;
  const uint32_t me = ef ? ((vb & 0x7fffffu) | 0x800000u) : vb;
  const int d = (ef ? static_cast<int>(ef) - 150 : -149) - uexp;
  ChainStep c{0u, 0u, false};
  if (d >= 0) {
    const unsigned long long n = d >= 40 ? kChainSat : (static_cast<unsigned long long>(me) << d);
    c.n = c.r = n >= kChainSat ? kChainSat : static_cast<uint32_t>(n);
  } else if (d > -32) {
    const int sh = -d;
    const uint32_t rem = me & ((1u << sh) - 1u), half = 1u << (sh - 1);
    c.n = me >> sh;
    c.r = c.n + (rem > half ? 1u : 0u);
    c.tie = rem == half;
  }
  return c;
}

// The same from v and 1/u in float, for grids with 2^-100 <= u <= 1: v / u is
// then exact (a power-of-two scaling) and so are its floor and fraction.
__device__ __forceinline__ ChainStep chain_step_f(uint32_t vb, float inv_u) {
  const float t = __fmul_rn(__uint_as_float(vb), inv_u);
  const float n = floorf(t);
  const float fr = __fsub_rn(t, n);
  ChainStep c;
  c.n = static_cast<uint32_t>(fminf(n, 1073741824.0f));  // kChainSat
  c.r = min(c.n + (fr > 0.5f ? 1u : 0u), kChainSat);
  c.tie = fr == 0.5f;
  return c;
}

__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) { return min(a + b, kChainSat); }

// 2^x as a float, x in [-149, 127]
__device__ __forceinline__ float pow2f(int x) {
  return x >= -126 ? __uint_as_float(static_cast<uint32_t>(x + 127) << 23) : __uint_as_float(1u << (x + 149));
}

__device__ __forceinline__ int warp_min(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace llmq
