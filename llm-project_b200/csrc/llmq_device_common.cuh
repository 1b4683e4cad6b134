// llmq_device_common.cuh - device helpers shared by the CUDA translation units
// of libllmq_cuda.so: the reference's activation-code rounding and rescale, and
// block-wide max reductions.  Inline functions only (no globals, no kernels).
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

namespace llmq {

// ------------------------------------------------------- reference arithmetic
// (int)lrintf(v) as the reference's x86-64 build evaluates it (cvtss2si to a
// 64-bit long, then truncation to int), followed by the clamp to +-127
// (quant.c:56-58, quant.c:109-111).
__device__ __forceinline__ int8_t code_of(float v) {
  int c;
  if (fabsf(v) < 2147483648.0f) {
    c = __float2int_rn(v);
  } else if (fabsf(v) < 9.2233720368547758e18f) {  // finite, fits a long
    c = static_cast<int>(static_cast<unsigned long long>(__float2ll_rn(v)) & 0xffffffffull);
  } else {
    c = 0;  // NaN / out of range: integer indefinite 0x8000000000000000, low half 0
  }
  c = c > 127 ? 127 : c;
  c = c < -127 ? -127 : c;
  return static_cast<int8_t>(c);
}
// as * ws[j] * (float)acc, left to right (quant.c:117)
__device__ __forceinline__ float dequant(float as, float ws, int acc) {
  return __fmul_rn(__fmul_rn(as, ws), __int2float_rn(acc));
}

// ------------------------------------------------------------- block helpers
template <int NT>
__device__ __forceinline__ float block_max(float v, float *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < NT / 32 ? red[lane] : v;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

template <int NT>
__device__ __forceinline__ unsigned long long block_max_u64(unsigned long long v, unsigned long long *red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
    v = w > v ? w : v;
  }
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < NT / 32 ? red[lane] : 0ull;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long w = __shfl_xor_sync(0xffffffffu, v, o);
      v = w > v ? w : v;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// Sequential f32 sum acc + v[0] + v[stride] + ... + v[(n-1)*stride], one
// rounded add after another exactly as a C loop does, with the next 8 values
// loaded while the current 8 are added (the adds form the only dependency).
__device__ __forceinline__ float seq_sum(const float *v, int stride, int n, float acc) {
  int i = 0;
  if (n >= 8) {
    float cur[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) cur[u] = v[(size_t)u * stride];
    for (i = 8; i + 8 <= n; i += 8) {
      float nxt[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) nxt[u] = v[(size_t)(i + u) * stride];
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, cur[u]);
#pragma unroll
      for (int u = 0; u < 8; ++u) cur[u] = nxt[u];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, cur[u]);
  }
  for (; i < n; ++i) acc = __fadd_rn(acc, v[(size_t)i * stride]);
  return acc;
}

// Sequential f32 dot product acc + a[0]*b[0] + a[1]*b[sb] + ..., each product
// and each sum rounded on its own in C order; the 8 products of a group are
// formed back to back (independent), then added one after another.
__device__ __forceinline__ float seq_dot(const float *a, const float *b, int sb, int n, float acc) {
  int i = 0;
  for (; i + 8 <= n; i += 8) {
    float p[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) p[u] = __fmul_rn(a[i + u], b[(size_t)(i + u) * sb]);
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, p[u]);
  }
  for (; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(a[i], b[(size_t)i * sb]));
  return acc;
}

}  // namespace llmq
