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
// (quant.c:21-23, quant.c:74-76).
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
// as * ws[j] * (float)acc, left to right (quant.c:82)
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

// seq_sum for a contiguous, 16-byte aligned v: 16 values in flight as four
// 16-byte loads, so a single thread's chain keeps running while the shared
// memory is busy with other traffic (e.g. copies landing).
__device__ __forceinline__ float seq_sum_a16(const float *v, int n, float acc) {
  const float4 *v4 = reinterpret_cast<const float4 *>(v);
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
      for (int u = 0; u < 4; ++u) {
        acc = __fadd_rn(acc, c[u].x);
        acc = __fadd_rn(acc, c[u].y);
        acc = __fadd_rn(acc, c[u].z);
        acc = __fadd_rn(acc, c[u].w);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) c[u] = nx[u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc = __fadd_rn(acc, c[u].x);
      acc = __fadd_rn(acc, c[u].y);
      acc = __fadd_rn(acc, c[u].z);
      acc = __fadd_rn(acc, c[u].w);
    }
  }
  for (; i < n; ++i) acc = __fadd_rn(acc, v[i]);
  return acc;
}

// seq_sum_a16 with 32 values in flight (eight 16-byte loads ahead), for a
// lone thread whose loads would otherwise wait on shared-memory latency.
__device__ __forceinline__ float seq_sum_a32(const float *v, int n, float acc) {
  const float4 *v4 = reinterpret_cast<const float4 *>(v);
  int i = 0;
  if (n >= 32) {
    float4 c[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) c[u] = v4[u];
    for (i = 32; i + 32 <= n; i += 32) {
      float4 nx[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) nx[u] = v4[(i >> 2) + u];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        acc = __fadd_rn(acc, c[u].x);
        acc = __fadd_rn(acc, c[u].y);
        acc = __fadd_rn(acc, c[u].z);
        acc = __fadd_rn(acc, c[u].w);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) c[u] = nx[u];
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      acc = __fadd_rn(acc, c[u].x);
      acc = __fadd_rn(acc, c[u].y);
      acc = __fadd_rn(acc, c[u].z);
      acc = __fadd_rn(acc, c[u].w);
    }
  }
  for (; i < n; ++i) acc = __fadd_rn(acc, v[i]);
  return acc;
}

// Sequential f32 dot product acc + a[0]*b[0] + a[1]*b[sb] + ..., each product
// and each sum rounded on its own in C order.  Software-pipelined: the loads of
// the next group of 8 are issued before the 8 adds of the current group, so
// the chain advances at the add latency; products are independent and formed
// back to back.  The arithmetic is the plain sequential loop's.
__device__ __forceinline__ float seq_dot(const float *a, const float *b, int sb, int n, float acc) {
  int i = 0;
  if (n >= 8) {
    float ca[8], cb[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      ca[u] = a[u];
      cb[u] = b[(size_t)u * sb];
    }
    for (i = 8; i + 8 <= n; i += 8) {
      float na[8], nb[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        na[u] = a[i + u];
        nb[u] = b[(size_t)(i + u) * sb];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(ca[u], cb[u]));
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        ca[u] = na[u];
        cb[u] = nb[u];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(ca[u], cb[u]));
  }
  for (; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(a[i], b[(size_t)i * sb]));
  return acc;
}

// seq_dot with a contiguous and 16-byte aligned (read as float4), b strided:
// 16 terms in flight, so a lone warp's chain is not held up by load latency.
__device__ __forceinline__ float seq_dot_a4(const float *a, const float *b, int sb, int n, float acc) {
  const float4 *a4 = reinterpret_cast<const float4 *>(a);
  int i = 0;
  if (n >= 16) {
    float4 ca[4];
    float cb[16];
#pragma unroll
    for (int u = 0; u < 4; ++u) ca[u] = a4[u];
#pragma unroll
    for (int u = 0; u < 16; ++u) cb[u] = b[(size_t)u * sb];
    for (i = 16; i + 16 <= n; i += 16) {
      float4 na[4];
      float nb[16];
#pragma unroll
      for (int u = 0; u < 4; ++u) na[u] = a4[(i >> 2) + u];
#pragma unroll
      for (int u = 0; u < 16; ++u) nb[u] = b[(size_t)(i + u) * sb];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc = __fadd_rn(acc, __fmul_rn(ca[u].x, cb[4 * u]));
        acc = __fadd_rn(acc, __fmul_rn(ca[u].y, cb[4 * u + 1]));
        acc = __fadd_rn(acc, __fmul_rn(ca[u].z, cb[4 * u + 2]));
        acc = __fadd_rn(acc, __fmul_rn(ca[u].w, cb[4 * u + 3]));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) ca[u] = na[u];
#pragma unroll
      for (int u = 0; u < 16; ++u) cb[u] = nb[u];
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc = __fadd_rn(acc, __fmul_rn(ca[u].x, cb[4 * u]));
      acc = __fadd_rn(acc, __fmul_rn(ca[u].y, cb[4 * u + 1]));
      acc = __fadd_rn(acc, __fmul_rn(ca[u].z, cb[4 * u + 2]));
      acc = __fadd_rn(acc, __fmul_rn(ca[u].w, cb[4 * u + 3]));
    }
  }
  for (; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(a[i], b[(size_t)i * sb]));
  return acc;
}

// As seq_dot with 16-byte shared-memory loads: a and b 16-byte aligned, n a
// multiple of 4.
__device__ __forceinline__ float seq_dot_v4(const float *a, const float *b, int n, float acc) {
  const float4 *a4 = reinterpret_cast<const float4 *>(a), *b4 = reinterpret_cast<const float4 *>(b);
  const int n4 = n >> 2;
  auto add4 = [&](const float4 x, const float4 y) {
    const float p0 = __fmul_rn(x.x, y.x), p1 = __fmul_rn(x.y, y.y), p2 = __fmul_rn(x.z, y.z),
                p3 = __fmul_rn(x.w, y.w);
    acc = __fadd_rn(acc, p0);
    acc = __fadd_rn(acc, p1);
    acc = __fadd_rn(acc, p2);
    acc = __fadd_rn(acc, p3);
  };
  int i = 0;
  if (n4 >= 2) {
    float4 x0 = a4[0], y0 = b4[0], x1 = a4[1], y1 = b4[1];
    for (i = 2; i + 2 <= n4; i += 2) {
      const float4 nx0 = a4[i], ny0 = b4[i], nx1 = a4[i + 1], ny1 = b4[i + 1];
      add4(x0, y0);
      add4(x1, y1);
      x0 = nx0;
      y0 = ny0;
      x1 = nx1;
      y1 = ny1;
    }
    add4(x0, y0);
    add4(x1, y1);
  }
  if (i < n4) add4(a4[i], b4[i]);
  return acc;
}

// Sequential dot product acc + (e[0]*s)*b[0] + (e[1]*s)*b[sb] + ..., each
// product rounded as written, then added in index order (the weights
// w = e * s of a softmax formed on the fly); pipelined as seq_dot.
__device__ __forceinline__ float seq_dot_scaled(const float *e, float sc, const float *b, int sb, int n, float acc) {
  int i = 0;
  if (n >= 8) {
    float cw[8], cb[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      cw[u] = __fmul_rn(e[u], sc);
      cb[u] = b[(size_t)u * sb];
    }
    for (i = 8; i + 8 <= n; i += 8) {
      float ne[8], nb[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        ne[u] = e[i + u];
        nb[u] = b[(size_t)(i + u) * sb];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(cw[u], cb[u]));
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        cw[u] = __fmul_rn(ne[u], sc);
        cb[u] = nb[u];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = __fadd_rn(acc, __fmul_rn(cw[u], cb[u]));
  }
  for (; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(__fmul_rn(e[i], sc), b[(size_t)i * sb]));
  return acc;
}

// ---- packed pairs of independent f32 chains (Blackwell f32x2 arithmetic):
// each lane is rounded exactly as the scalar __fmul_rn / __fadd_rn would, so
// two chains advance with one instruction stream and unchanged results.
__device__ __forceinline__ unsigned long long f2_bits(float2 v) {
  return (static_cast<unsigned long long>(__float_as_uint(v.y)) << 32) | __float_as_uint(v.x);
}
__device__ __forceinline__ float2 f2_from(unsigned long long b) {
  return make_float2(__uint_as_float(static_cast<uint32_t>(b)), __uint_as_float(static_cast<uint32_t>(b >> 32)));
}
__device__ __forceinline__ float2 f2_mul_rn(float2 a, float2 b) {
  unsigned long long r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(r);
}
__device__ __forceinline__ float2 f2_add_rn(float2 a, float2 b) {
  unsigned long long r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(r);
}

// acc + a*b per lane with the product rounded on its own.  ptxas contracts a
// packed mul.rn whose only use is a packed add into a fused multiply-add (so
// the product would not be rounded); the product therefore goes through an
// add of +0.0 first: fused or not, that yields round(a*b) exactly (the sign of
// a zero product can change, which a sum starting from +0 never sees).
__device__ __forceinline__ float2 f2_madd_rn(float2 acc, float2 a, float2 b) {
  return f2_add_rn(acc, f2_add_rn(f2_mul_rn(a, b), make_float2(0.0f, 0.0f)));
}

// Two sequential dot products at once: acc.x + w[0]*b[0].x + w[1]*b[sb].x + ...
// and the same with .y, where w[i] = e[i] * sc if `scaled`, else e[i]; every
// product and sum rounded on its own in index order (the weighted sums of
// values of two adjacent output dimensions).  Pipelined as seq_dot.
template <bool scaled>
__device__ __forceinline__ float2 seq_dot2(const float *e, float sc, const float2 *b, int sb, int n, float2 acc) {
  auto wt = [&](float v) { return scaled ? __fmul_rn(v, sc) : v; };
  int i = 0;
  if (n >= 8) {
    float cw[8];
    float2 cb[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      cw[u] = wt(e[u]);
      cb[u] = b[(size_t)u * sb];
    }
    for (i = 8; i + 8 <= n; i += 8) {
      float ne[8];
      float2 nb[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        ne[u] = e[i + u];
        nb[u] = b[(size_t)(i + u) * sb];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) acc = f2_madd_rn(acc, make_float2(cw[u], cw[u]), cb[u]);
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        cw[u] = wt(ne[u]);
        cb[u] = nb[u];
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) acc = f2_madd_rn(acc, make_float2(cw[u], cw[u]), cb[u]);
  }
  for (; i < n; ++i) {
    const float w = wt(e[i]);
    acc = f2_madd_rn(acc, make_float2(w, w), b[(size_t)i * sb]);
  }
  return acc;
}

}  // namespace llmq
