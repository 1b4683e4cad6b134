// llmq_spec_sum.cuh - the sequential f32 sum of a long row, bit for bit, by a
// whole thread block: the RMSNorm's sum of squares (rmsnorm.c:15) without the
// latency of one thread adding 4096 or 8192 terms one after another.
//
// The loop s = acc; for k: s = s + v[k] (each add rounded) depends on the terms
// before k only through the value s holds after them.  The row is cut into one
// segment per warp.  The value at the start of segment w is not known until the
// segments before it are summed, but it lies within a few dozen ulps of the
// exact prefix sum: for non-negative terms the partial sums grow, and the
// loop's rounding errors add up to a slow random walk (measured on Gaussian rows
// with outliers: at most 30 ulps after 3840 terms, 62 after 7680).  So every
// lane of warp w runs the segment's loop from its own candidate start, the
// float whose bit pattern is the estimate's plus a lane offset; for
// non-negative values consecutive bit patterns are consecutive floats, so the
// lanes cover a window of 32 or 64 floats around the estimate.  One thread then
// walks the segments in order: the true start of segment w is the true end of
// segment w-1, and when it equals a candidate bit for bit, that candidate's end
// is the true end of segment w (same start, same terms, same rounded adds).
// When it is not in the window, the thread sums the segment itself.  The result
// is the loop's in every case, for any input (negative terms, infinities and
// NaN only make hits rarer); only the time depends on the estimate.
#pragma once

#include "llmq_device_common.cuh"

namespace llmq {

constexpr int kSpecMinN = 1024;    // shorter rows: the one-thread loop is as fast
constexpr int kSpecWideN = 6144;   // longer rows: 64 candidates per segment, else 32
constexpr int kSpecMaxC = 64;

// Shared-memory scratch of spec_seq_sum for a block of nt threads: the
// candidates' ends [nt/32][64], the segments' double sums, the estimates' bit
// patterns and the result (a multiple of 16 bytes).
__host__ __device__ constexpr size_t spec_sum_bytes(int nt) {
  return (size_t)(nt / 32) * (kSpecMaxC * 4 + 8 + 4) + 16;
}

// acc[q] + v[0] + v[1] + ... + v[n-1] for NC starting values at once, each add
// rounded in index order; the loads are shared.  v is 16-byte aligned.
template <int NC>
__device__ __forceinline__ void seq_sum_multi_a16(const float *v, int n, float (&acc)[NC]) {
  const float4 *v4 = reinterpret_cast<const float4 *>(v);
  auto add4 = [&](const float4 t) {
#pragma unroll
    for (int q = 0; q < NC; ++q) {
      acc[q] = __fadd_rn(acc[q], t.x);
      acc[q] = __fadd_rn(acc[q], t.y);
      acc[q] = __fadd_rn(acc[q], t.z);
      acc[q] = __fadd_rn(acc[q], t.w);
    }
  };
  int i = 0;
  if (n >= 16) {
    float4 c[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) c[u] = v4[u];
    for (i = 16; i + 16 <= n; i += 16) {
      float4 nx[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) nx[u] = v4[(i >> 2) + u];
#pragma unroll
      for (int u = 0; u < 4; ++u) add4(c[u]);
#pragma unroll
      for (int u = 0; u < 4; ++u) c[u] = nx[u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) add4(c[u]);
  }
  for (; i < n; ++i) {
    const float t = v[i];
#pragma unroll
    for (int q = 0; q < NC; ++q) acc[q] = __fadd_rn(acc[q], t);
  }
}

// Returns acc0 + v[0] + v[1] + ... + v[n-1], every add rounded in index order
// (the C loop's value), to every thread of the block.  All threads of the
// block call it; the block has at most MAXT threads, a multiple of 32.  v: n
// floats in shared memory, 16-byte aligned, not written until every thread has
// returned.  scratch: spec_sum_bytes(MAXT) bytes of shared memory, 16-byte
// aligned; between two calls on the same scratch the block passes a barrier.
// *misses, if given, receives from thread 0 the number of segments whose start
// was outside the window (summed again by one thread).
template <int MAXT>
__device__ float spec_seq_sum(const float *v, int n, float acc0, void *scratch, int *misses = nullptr) {
  static_assert(MAXT % 32 == 0 && MAXT <= 1024, "block size");
  const int W = static_cast<int>(blockDim.x >> 5);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float *ends = reinterpret_cast<float *>(scratch);                 // [W][kSpecMaxC]
  double *segsum = reinterpret_cast<double *>(ends + W * kSpecMaxC);  // [W]
  uint32_t *base = reinterpret_cast<uint32_t *>(segsum + W);          // [W]
  float *result = reinterpret_cast<float *>(base + W);
  if (n < kSpecMinN || W < 2) {
    if (tid == 0) {
      *result = seq_sum_a16(v, n, acc0);
      if (misses) *misses = 0;
    }
    __syncthreads();
    return *result;
  }
  // segments of L terms (a multiple of 4: every segment starts 16-byte aligned)
  const int L = ((n + W - 1) / W + 3) & ~3;
  const int k0 = min(n, warp * L), k1 = min(n, k0 + L);
  // each segment's sum in double precision (an estimate only: any order will do)
  double s = 0.0;
  for (int k = k0 + lane; k < k1; k += 32) s += static_cast<double>(v[k]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane == 0) segsum[warp] = s;
  __syncthreads();
  // the estimate of this segment's start: the exact prefix, rounded to f32
  double pre = static_cast<double>(acc0);
  for (int q = 0; q < warp; ++q) pre += segsum[q];
  const uint32_t b = __float_as_uint(__double2float_rn(pre));
  if (lane == 0) base[warp] = b;
  const bool wide = n > kSpecWideN;
  if (wide) {
    float c[2] = {__uint_as_float(b - 32u + lane), __uint_as_float(b + lane)};
    seq_sum_multi_a16<2>(v + k0, k1 - k0, c);
    ends[warp * kSpecMaxC + lane] = c[0];
    ends[warp * kSpecMaxC + 32 + lane] = c[1];
  } else {
    float c[1] = {__uint_as_float(b - 16u + lane)};
    seq_sum_multi_a16<1>(v + k0, k1 - k0, c);
    ends[warp * kSpecMaxC + lane] = c[0];
  }
  __syncthreads();
  if (tid == 0) {
    const uint32_t half = wide ? 32u : 16u;
    float S = acc0;
    int miss = 0;
#pragma unroll 4
    for (int w = 0; w < W; ++w) {
      const uint32_t idx = __float_as_uint(S) - base[w] + half;  // candidate index, if S is one
      if (idx < 2u * half) {
        S = ends[w * kSpecMaxC + idx];
      } else {
        const int a0 = min(n, w * L), a1 = min(n, a0 + L);
        S = seq_sum_a16(v + a0, a1 - a0, S);
        ++miss;
      }
    }
    *result = S;
    if (misses) *misses = miss;
  }
  __syncthreads();
  return *result;
}

}  // namespace llmq
