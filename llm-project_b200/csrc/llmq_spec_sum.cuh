// llmq_spec_sum.cuh - the sequential f32 sum of a long row, bit for bit, by a
// whole thread block: the RMSNorm's sum of squares (rmsnorm.c:15) without the
// latency of one thread adding 4096 or 8192 terms one after another.
//
// The loop s = acc; for k: s = s + v[k] (each add rounded) depends on the terms
// before k only through the value s holds after them.  The row is cut into 32
// segments.  What segment w adds to a start value x, e_w(x) - x, hardly depends
// on x: while the partial sums stay within one binade they lie on one grid of
// ulps, every add rounds its term to that grid the same way whatever the start
// (ties aside), so e_w(x + d ulps) = e_w(x) + d ulps.  The sum is formed in
// four steps, all in f32:
//  1. every segment's plain sum (an estimate of the partial sums);
//  2. one warp, a lane per segment, runs each segment's loop from its estimated
//     start and takes the shift it produced; a sequential scan of the shifts
//     from acc gives new estimates of the segment starts, exact up to where
//     some segment's rounding depended on its start (a binade crossed at a
//     different place, a tie), and a few ulps off after that;
//  3. C warps, a warp per offset o in [-C/2, C/2), a lane per segment, run each
//     segment's loop from its estimate + o ulps (consecutive bit patterns are
//     consecutive floats for non-negative values); a ballot marks the segments
//     whose end is the next estimate + the same o, and every (o, segment) keeps
//     the first segment at or after it whose end leaves the offset, with that
//     end;
//  4. one thread walks: from acc (offset 0 at segment 0), each jump goes to the
//     end of such a run of segments, which is then the exact start of the next
//     segment (same start bits, same terms, same rounded adds); when an exact
//     start is outside every window the thread sums that segment itself.
// The walk only ever uses loops run from the exact start, so the result is the
// loop's for every input (negative terms, infinities and NaN only make the
// jumps shorter or the fallbacks more frequent); only the time depends on the
// estimates.
#pragma once

#include "llmq_device_common.cuh"

namespace llmq {

constexpr int kSpecMinN = 1024;  // shorter rows: the one-thread loop is as fast
constexpr int kSpecSeg = 32;     // segments
constexpr int kSpecC = 8;        // candidate offsets per segment

// Shared-memory scratch of spec_seq_sum (any block size).
struct SpecScratch {
  float est[kSpecSeg + 1];       // estimated start of each segment (est[0] = acc)
  float segsum[kSpecSeg];
  float jv[kSpecC][kSpecSeg];    // the end after the jump from (offset, segment)
  int jf[kSpecC][kSpecSeg];      // the segment after that jump
  float result;
  int misses;
};
__host__ __device__ constexpr size_t spec_sum_bytes() { return (sizeof(SpecScratch) + 15) & ~size_t(15); }

// Returns acc0 + v[0] + v[1] + ... + v[n-1], every add rounded in index order
// (the C loop's value), to every thread of the block.  All threads of the
// block call it; blockDim.x is a multiple of 32.  v: n floats in shared memory,
// 16-byte aligned, not written until every thread has returned.  scratch:
// spec_sum_bytes() bytes of shared memory, 16-byte aligned; between two calls on
// the same scratch the block passes a barrier.  *misses, if given, receives
// from thread 0 the number of segments that thread summed itself.
__device__ float spec_seq_sum(const float *v, int n, float acc0, void *scratch, int *misses = nullptr) {
  SpecScratch *J = reinterpret_cast<SpecScratch *>(scratch);
  const int W = static_cast<int>(blockDim.x >> 5);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (n < kSpecMinN || W < 4) {
    if (tid == 0) {
      J->result = seq_sum_a16(v, n, acc0);
      J->misses = 0;
    }
    __syncthreads();
    if (misses && tid == 0) *misses = 0;
    return J->result;
  }
  // Segments of L terms: L a multiple of 4 (16-byte aligned starts) with L / 4
  // odd, so the lanes of step 2 and 3, one per segment, load from 8 different
  // 16-byte bank groups.
  int L = ((n + kSpecSeg - 1) / kSpecSeg + 3) & ~3;
  if (((L >> 2) & 1) == 0) L += 4;
  // 1. plain segment sums: half a warp per segment
  for (int seg = 2 * warp + (lane >> 4); seg < kSpecSeg; seg += 2 * W) {  // same trip count in both halves
    const int k0 = min(n, seg * L), k1 = min(n, k0 + L);
    float p = 0.0f;
    for (int k = k0 + (lane & 15); k < k1; k += 16) p += v[k];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    if ((lane & 15) == 0) J->segsum[seg] = p;
  }
  __syncthreads();
  // 2. each segment's shift from its plain estimate; estimates from the shifts
  if (warp == 0) {
    float P = J->segsum[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float u = __shfl_up_sync(0xffffffffu, P, o);
      if (lane >= o) P += u;
    }
    const float prev = __shfl_up_sync(0xffffffffu, P, 1);
    const float b = lane == 0 ? acc0 : __fadd_rn(prev, acc0);
    const int k0 = min(n, lane * L), k1 = min(n, k0 + L);
    const float d = __fsub_rn(seq_sum_a16(v + k0, k1 - k0, b), b);
    float S = acc0;
#pragma unroll
    for (int w = 0; w < kSpecSeg; ++w) {
      const float dw = __shfl_sync(0xffffffffu, d, w);
      if (lane == w) J->est[w] = S;
      S = __fadd_rn(S, dw);
    }
    if (lane == 0) J->est[kSpecSeg] = S;
  }
  __syncthreads();
  // 3. candidates around the estimates; the jump of every (offset, segment)
  for (int c = warp; c < kSpecC; c += W) {
    const int off = c - kSpecC / 2;
    const int k0 = min(n, lane * L), k1 = min(n, k0 + L);
    const uint32_t start = __float_as_uint(J->est[lane]) + static_cast<uint32_t>(off);
    const float e = seq_sum_a16(v + k0, k1 - k0, __uint_as_float(start));
    const bool keeps = lane + 1 < kSpecSeg &&
                       __float_as_uint(e) == __float_as_uint(J->est[lane + 1]) + static_cast<uint32_t>(off);
    const unsigned m = __ballot_sync(0xffffffffu, keeps);  // bit 31 (the last segment) is never set
    const int f = lane + __ffs(~(m >> lane)) - 1;           // first segment >= lane whose end leaves the offset
    J->jf[c][lane] = f + 1;
    J->jv[c][lane] = __shfl_sync(0xffffffffu, e, f);
  }
  __syncthreads();
  // 4. the walk over exact segment starts
  if (tid == 0) {
    float S = acc0;
    int w = 0, miss = 0;
    while (w < kSpecSeg) {
      const int c = static_cast<int>(__float_as_uint(S) - __float_as_uint(J->est[w])) + kSpecC / 2;
      if (c >= 0 && c < kSpecC) {
        S = J->jv[c][w];
        w = J->jf[c][w];
      } else {
        const int k0 = min(n, w * L), k1 = min(n, k0 + L);
        S = seq_sum_a16(v + k0, k1 - k0, S);
        ++miss;
        ++w;
      }
    }
    J->result = S;
    J->misses = miss;
  }
  __syncthreads();
  if (misses && tid == 0) *misses = J->misses;
  return J->result;
}

}  // namespace llmq
