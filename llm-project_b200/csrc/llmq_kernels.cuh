// llmq_kernels.cuh - sm_100a kernels of the int8 (W8A8) LLaMA decode path.
//
// Arithmetic contract: every fp32 value the reference computes is computed here
// with the same operations in the same order, each rounded on its own
// (__fmul_rn/__fadd_rn/__fdiv_rn/__fsqrt_rn never contract into FMA), integer
// products are summed exactly in int32 (any order gives the same sum), and expf
// is the host-libm-exact routine of libm_expf.h.  The results are therefore
// bit-identical to the reference CPU code.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#include "libm_expf.h"

namespace llmq {

constexpr int kThreads = 256;     // GEMV CTA size (8 warps)
constexpr int kMaxRows = 8;       // rows per GEMV launch (decode uses 1)

// Error bits written to the per-model error word.
enum : int { ERR_TIMEOUT = 1, ERR_BAD_TOKEN = 2, ERR_BAD_POS = 4 };

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// One contiguous global->shared bulk copy completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
// Bounded wait on an mbarrier phase: gives up after ~2 s of wall time (and a hard
// iteration cap), so a lost copy can never hang the GPU.
__device__ __noinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0; it < (1u << 24); ++it) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((it & 255u) == 255u && global_ns() - t0 > 2000000000ull) break;
  }
  return false;
}
// Programmatic dependent launch: let the next kernel in the stream start its
// weight prefetch now / wait until the previous kernel's writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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

// The host-libm-exact expf (libm_expf.h) with the exception set in a hash table.
struct ExpfTable {
  const uint32_t *keys;  // open addressing, 0 = empty
  uint32_t mask;
};
__device__ ExpfTable g_expf_table;

__host__ __device__ __forceinline__ uint32_t expf_hash(uint32_t k) { return (k * 2654435761u) >> 7; }

__device__ __noinline__ bool expf_is_exception(uint32_t key) {
  const ExpfTable t = g_expf_table;
  if (t.keys == nullptr) return false;
  uint32_t i = expf_hash(key) & t.mask;
  for (uint32_t probe = 0; probe <= t.mask; ++probe) {
    const uint32_t v = __ldg(t.keys + i);
    if (v == key) return true;
    if (v == 0u) return false;
    i = (i + 1) & t.mask;
  }
  return false;
}

__device__ __forceinline__ float libm_expf(float x) {
  int near;
  float lo, up;
  const float cr = lx_expf_cr(x, exp(static_cast<double>(x)), &near, &lo, &up);
  if (!near) return cr;
  if (expf_is_exception(lx_bits(x))) return (cr == up) ? lo : up;
  return cr;
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

// Key whose unsigned order is the float order with ties broken towards the
// lower index: the "first maximum wins" rule of sampler.c:8-21.
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  if (v != v) u = 0u;  // NaN never wins
  return (static_cast<unsigned long long>(u) << 32) | static_cast<unsigned long long>(0xffffffffu - idx);
}

// ----------------------------------------------------------- GEMV arguments
enum Prologue : int {
  PRO_ABSMAX = 0,        // rows of `in` quantised as they are (qmatmul, Wo, W2)
  PRO_RMSNORM = 1,       // RMSNorm(in, gamma) first (QKV, W1|W3, lm-head)
  PRO_EMBED_RMSNORM = 2  // x = dequantised embedding row of step->token, then RMSNorm
};
enum Epilogue : int {
  EPI_PLAIN = 0,   // out[r][j] = as*ws*acc                         (qmatmul)
  EPI_QKV = 1,     // + bias, RoPE on q and k, k/v appended to the cache
  EPI_RESID = 2,   // out[j] += as*ws*acc                           (Wo, W2)
  EPI_SWIGLU = 3,  // out[j] = SiLU(gate) * up                      (W1|W3)
  EPI_LOGITS = 4   // logits + device argmax                        (lm-head)
};

struct StepState {
  int token;
  int pos;
};

struct GemvArgs {
  const uint8_t *w;    // tiles [n_slabs][n_ktiles][KT/16][NT][16]
  const float *ws;     // per physical column scale [Npad]
  int K, Kpad, N, Npad, NT, KT, n_slabs, n_ktiles, stages, rows;
  int *acc;            // [rows][Npad] int32, zero before and after
  int *cnt;            // [n_slabs], zero before and after
  int *err;
  // prologue
  const float *in;     // [rows][K]
  const float *gamma;
  float eps;
  const int8_t *wte_q;
  const float *wte_s;
  int vocab;
  const StepState *step;
  float *x_out;        // PRO_EMBED_RMSNORM: the residual stream is written here
  // epilogue
  float *out;          // [rows][N]
  const float *bias;   // EPI_QKV, physical order
  int qd, kvd, hd, max_seq;
  float *kcache, *vcache;  // this layer's [max_seq][kvd]
  const float *rope_cos, *rope_sin;  // [max_seq][hd/2]
  unsigned long long *argmax;
};

// Owner CTA of tile t under the contiguous split [c*T/G, (c+1)*T/G).
__device__ __forceinline__ long long tile_owner(long long t, long long T, long long G) {
  return ((t + 1) * G + T - 1) / T - 1;
}

// ------------------------------------------------------------ the GEMV kernel
// x(rows, K) @ W(K, N) with W pre-tiled so every tile is one contiguous bulk
// copy.  Each CTA owns a contiguous range of tiles (balanced to one tile),
// streams them through a `stages`-deep shared-memory ring, and accumulates
// exact int32 dot products with dp4a.  Partial sums of a column slab are added
// into `acc` with integer atomics; the CTA that completes a slab applies the
// fused epilogue and re-zeroes `acc` and `cnt` for the next launch.
template <int PRO, int EPI, int MR>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const GemvArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ float s_red[32];
  __shared__ unsigned long long s_red64[32];
  __shared__ float s_as[MR];
  __shared__ float s_r;
  __shared__ int s_flag;
  __shared__ int s_abort;

  const int tid = threadIdx.x;
  const int tile_bytes = a.KT * a.NT;
  const int S = a.stages;
  uint8_t *stage0 = sm;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + (size_t)S * tile_bytes);
  int8_t *codes = reinterpret_cast<int8_t *>(sm + (((size_t)S * tile_bytes + 8 * S + 15) & ~size_t(15)));
  float *xs = reinterpret_cast<float *>(codes + (((size_t)a.rows * a.Kpad + 15) & ~size_t(15)));
  float *ebuf = xs;  // epilogue exchange buffer (prologue vector is dead by then)

  const long long T = (long long)a.n_slabs * a.n_ktiles;
  const long long G = gridDim.x;
  const long long t_begin = (long long)blockIdx.x * T / G;
  const long long t_end = (long long)(blockIdx.x + 1) * T / G;
  const int n = static_cast<int>(t_end - t_begin);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  // Weights never depend on the previous kernel: start streaming them now.
  int issued = 0;
  if (tid == 0) {
    const int first = n < S ? n : S;
    for (; issued < first; ++issued) {
      mbar_expect_tx(&bars[issued], tile_bytes);
      bulk_load(stage0 + (size_t)issued * tile_bytes, a.w + (size_t)(t_begin + issued) * tile_bytes,
                tile_bytes, &bars[issued]);
    }
  }
  pdl_launch_dependents();
  pdl_wait();

  // ------------------------------------------------------------ prologue
  if (PRO == PRO_ABSMAX) {
    for (int r = 0; r < a.rows && r < MR; ++r) {
      const float *in = a.in + (size_t)r * a.K;
      float m = 0.0f;
      for (int k = tid; k < a.K; k += kThreads) m = fmaxf(m, fabsf(in[k]));
      m = block_max<kThreads>(m, s_red);
      const float as = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;  // quant.c:106
      const float inv = __fdiv_rn(1.0f, as);                      // quant.c:107
      if (tid == 0) s_as[r] = as;
      int8_t *cr = codes + (size_t)r * a.Kpad;
      for (int k = tid; k < a.Kpad; k += kThreads) cr[k] = k < a.K ? code_of(__fmul_rn(in[k], inv)) : 0;
    }
  } else {
    // RMSNorm of one row (rmsnorm.c:7-21), then activation quantisation.
    const int K = a.K;
    if (PRO == PRO_EMBED_RMSNORM) {
      int token = a.step->token;
      if (token < 0 || token >= a.vocab) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(a.err, ERR_BAD_TOKEN);
        token = 0;
      }
      const int8_t *row = a.wte_q + (size_t)token * K;
      for (int k = tid; k < K; k += kThreads) {
        const float v = __fmul_rn(static_cast<float>(row[k]), a.wte_s[k]);  // llama.c:536
        xs[k] = v;
        if (blockIdx.x == 0) a.x_out[k] = v;
      }
    } else {
      for (int k = tid; k < K; k += kThreads) xs[k] = a.in[k];
    }
    __syncthreads();
    if (tid == 0) {
      // The sequential sum of squares: one dependent chain, like the reference.
      float ms = 0.0f;
      int k = 0;
      for (; k + 4 <= K; k += 4) {
        const float4 v = *reinterpret_cast<const float4 *>(xs + k);
        ms = __fadd_rn(ms, __fmul_rn(v.x, v.x));
        ms = __fadd_rn(ms, __fmul_rn(v.y, v.y));
        ms = __fadd_rn(ms, __fmul_rn(v.z, v.z));
        ms = __fadd_rn(ms, __fmul_rn(v.w, v.w));
      }
      for (; k < K; ++k) ms = __fadd_rn(ms, __fmul_rn(xs[k], xs[k]));
      ms = __fmul_rn(ms, __fdiv_rn(1.0f, static_cast<float>(K)));
      s_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
    }
    __syncthreads();
    const float r = s_r;
    float m = 0.0f;
    for (int k = tid; k < K; k += kThreads) {
      const float y = __fmul_rn(__fmul_rn(xs[k], r), a.gamma[k]);
      xs[k] = y;
      m = fmaxf(m, fabsf(y));
    }
    m = block_max<kThreads>(m, s_red);  // also orders the xs writes before the reads below
    const float as = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
    const float inv = __fdiv_rn(1.0f, as);
    if (tid == 0) s_as[0] = as;
    for (int k = tid; k < a.Kpad; k += kThreads) codes[k] = k < K ? code_of(__fmul_rn(xs[k], inv)) : 0;
  }
  __syncthreads();

  // --------------------------------------------------------------- main loop
  const int NT = a.NT;
  const int P = kThreads / NT;  // threads per column
  const int col = tid % NT;
  const int part = tid / NT;
  const bool active = part < P;
  const int CH = a.KT / 16;
  int acc[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc[r] = 0;

  auto flush = [&](long long slab) {
    // combine the P partial sums of each column
    int *red = reinterpret_cast<int *>(ebuf);
    if (P > 1) {
#pragma unroll
      for (int r = 0; r < MR; ++r) {
        if (r >= a.rows) break;
        __syncthreads();
        red[tid] = active ? acc[r] : 0;
        __syncthreads();
        if (part == 0) {
          int s = 0;
          for (int p = 0; p < P; ++p) s += red[p * NT + col];
          acc[r] = s;
        }
      }
    }
    if (part == 0) {
#pragma unroll
      for (int r = 0; r < MR; ++r)
        if (r < a.rows) atomicAdd(a.acc + (size_t)r * a.Npad + slab * NT + col, acc[r]);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const long long nk = a.n_ktiles;
      const int arrivals =
          static_cast<int>(tile_owner((slab + 1) * nk - 1, T, G) - tile_owner(slab * nk, T, G) + 1);
      const int prev = atomicAdd(a.cnt + slab, 1);
      s_flag = (prev == arrivals - 1);
    }
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
    // ---- fused epilogue for columns [slab*NT, slab*NT + NT)
    const int p0 = static_cast<int>(slab) * NT;
    if (EPI == EPI_PLAIN || EPI == EPI_RESID) {
      for (int r = 0; r < a.rows && r < MR; ++r) {
        const float as = s_as[r];
        for (int c = tid; c < NT; c += kThreads) {
          const int j = p0 + c;
          const int v = atomicExch(a.acc + (size_t)r * a.Npad + j, 0);
          if (j < a.N) {
            const float y = dequant(as, a.ws[j], v);
            float *o = a.out + (size_t)r * a.N + j;
            if (EPI == EPI_RESID)
              *o = __fadd_rn(*o, y);  // llama.c:578 / llama.c:589
            else
              *o = y;
          }
        }
      }
    } else if (EPI == EPI_LOGITS) {
      const float as = s_as[0];
      unsigned long long best = 0ull;
      for (int c = tid; c < NT; c += kThreads) {
        const int j = p0 + c;
        const int v = atomicExch(a.acc + j, 0);
        if (j < a.N) {
          const float y = dequant(as, a.ws[j], v);
          a.out[j] = y;
          const unsigned long long key = argmax_key(y, static_cast<uint32_t>(j));
          best = key > best ? key : best;
        }
      }
      best = block_max_u64<kThreads>(best, s_red64);
      if (tid == 0) atomicMax(a.argmax, best);
    } else if (EPI == EPI_SWIGLU) {
      // slab = NT/2 gate columns followed by the NT/2 matching up columns
      const float as = s_as[0];
      const int half = NT / 2;
      for (int c = tid; c < half; c += kThreads) {
        const int j = static_cast<int>(slab) * half + c;  // d_ff index
        const int vg = atomicExch(a.acc + p0 + c, 0);
        const int vu = atomicExch(a.acc + p0 + half + c, 0);
        if (j < a.N) {
          const float z = dequant(as, a.ws[p0 + c], vg);
          const float u = dequant(as, a.ws[p0 + half + c], vu);
          const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, libm_expf(-z)));  // llama.c:585
          a.out[j] = __fmul_rn(__fmul_rn(z, s), u);                         // llama.c:586
        }
      }
    } else if (EPI == EPI_QKV) {
      const float as = s_as[0];
      const int pos = a.step->pos;
      for (int c = tid; c < NT; c += kThreads) {
        const int j = p0 + c;
        const int v = atomicExch(a.acc + j, 0);
        ebuf[c] = j < a.N ? __fadd_rn(dequant(as, a.ws[j], v), a.bias[j]) : 0.0f;  // llama.c:546-548
      }
      __syncthreads();
      const int half = a.hd / 2;
      const bool pos_ok = pos >= 0 && pos < a.max_seq;
      if (!pos_ok && tid == 0) atomicOr(a.err, ERR_BAD_POS);
      for (int c = tid; c < NT; c += kThreads) {
        const int j = p0 + c;
        if (j >= a.N || !pos_ok) continue;
        float y = ebuf[c];
        if (j < a.qd + a.kvd) {  // RoPE on q and k (rope.c:58-64)
          const int jj = j < a.qd ? j : j - a.qd;
          const int kk = jj % a.hd;
          if (kk < half) {
            const float cs = a.rope_cos[(size_t)pos * half + kk], sn = a.rope_sin[(size_t)pos * half + kk];
            y = __fsub_rn(__fmul_rn(ebuf[c], cs), __fmul_rn(ebuf[c + half], sn));
          } else {
            const int k0 = kk - half;
            const float cs = a.rope_cos[(size_t)pos * half + k0], sn = a.rope_sin[(size_t)pos * half + k0];
            y = __fadd_rn(__fmul_rn(ebuf[c], cs), __fmul_rn(ebuf[c - half], sn));
          }
        }
        if (j < a.qd)
          a.out[j] = y;
        else if (j < a.qd + a.kvd)
          a.kcache[(size_t)pos * a.kvd + (j - a.qd)] = y;  // llama.c:551
        else
          a.vcache[(size_t)pos * a.kvd + (j - a.qd - a.kvd)] = y;  // llama.c:552
      }
    }
    if (tid == 0) a.cnt[slab] = 0;
    __syncthreads();
  };

  long long cur = n > 0 ? t_begin / a.n_ktiles : -1;
  int done = 0;
  for (int i = 0; i < n; ++i) {
    const long long t = t_begin + i;
    const long long slab = t / a.n_ktiles;
    const int kt = static_cast<int>(t - slab * a.n_ktiles);
    if (slab != cur) {
      flush(cur);
#pragma unroll
      for (int r = 0; r < MR; ++r) acc[r] = 0;
      cur = slab;
    }
    const int s = i % S;
    if (!mbar_wait_bounded(&bars[s], static_cast<uint32_t>((i / S) & 1))) s_abort = 1;
    const uint8_t *tile = stage0 + (size_t)s * tile_bytes;
    if (active) {
      const int8_t *cbase = codes + (size_t)kt * a.KT;
      for (int c = part; c < CH; c += P) {
        const int4 w = *reinterpret_cast<const int4 *>(tile + ((size_t)c * NT + col) * 16);
#pragma unroll
        for (int r = 0; r < MR; ++r) {
          if (r < a.rows) {
            const int4 x = *reinterpret_cast<const int4 *>(cbase + (size_t)r * a.Kpad + c * 16);
            acc[r] = __dp4a(w.x, x.x, acc[r]);
            acc[r] = __dp4a(w.y, x.y, acc[r]);
            acc[r] = __dp4a(w.z, x.z, acc[r]);
            acc[r] = __dp4a(w.w, x.w, acc[r]);
          }
        }
      }
    }
    __syncthreads();
    done = i + 1;
    if (s_abort) break;
    if (tid == 0 && issued < n) {
      mbar_expect_tx(&bars[s], tile_bytes);
      bulk_load(stage0 + (size_t)s * tile_bytes, a.w + (size_t)(t_begin + issued) * tile_bytes, tile_bytes,
                &bars[s]);
      ++issued;
    }
  }
  if (s_abort) {
    // Record the failure and wait (bounded) for this CTA's copies still in flight.
    if (tid == 0) {
      atomicOr(a.err, ERR_TIMEOUT);
      for (int i = done; i < issued; ++i) mbar_wait_bounded(&bars[i % S], static_cast<uint32_t>((i / S) & 1));
    }
    return;
  }
  if (n > 0) flush(cur);
}

// --------------------------------------------------------------- attention
struct AttnArgs {
  const float *q;       // [n_heads * hd]
  const float *kcache;  // this layer's [max_seq][kvd]
  const float *vcache;
  float *out;           // [n_heads * hd]
  const StepState *step;
  int n_heads, n_kv, hd, max_seq;
};

constexpr int kAttnThreads = 512;

// One CTA per query head (llama.c:554-576): scores over positions 0..pos, each a
// sequential dot product; max; exp; the sequential sum; then for every d the
// sequential weighted sum over positions.  Needs (max_seq + hd) floats of
// dynamic shared memory.
__global__ void __launch_bounds__(kAttnThreads) k_attention(const AttnArgs a) {
  extern __shared__ __align__(16) float asm_[];
  __shared__ float s_red[32];
  __shared__ float s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int h = blockIdx.x;
  const int group = a.n_heads / a.n_kv;
  const int kvh = h / group;
  const int hd = a.hd, kvd = a.n_kv * hd;
  int pos = a.step->pos;
  if (pos < 0 || pos >= a.max_seq) return;  // flagged by the QKV epilogue
  const int np = pos + 1;
  float *qs = asm_;
  float *sc = asm_ + ((hd + 3) & ~3);
  for (int d = tid; d < hd; d += kAttnThreads) qs[d] = a.q[(size_t)h * hd + d];
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));  // llama.c:532
  float mloc = -INFINITY;
  for (int p = tid; p < np; p += kAttnThreads) {
    const float *kp = a.kcache + (size_t)p * kvd + (size_t)kvh * hd;
    float dot = 0.0f;
    if ((hd & 3) == 0) {
      for (int d = 0; d < hd; d += 4) {
        const float4 k4 = *reinterpret_cast<const float4 *>(kp + d);
        dot = __fadd_rn(dot, __fmul_rn(qs[d], k4.x));
        dot = __fadd_rn(dot, __fmul_rn(qs[d + 1], k4.y));
        dot = __fadd_rn(dot, __fmul_rn(qs[d + 2], k4.z));
        dot = __fadd_rn(dot, __fmul_rn(qs[d + 3], k4.w));
      }
    } else {
      for (int d = 0; d < hd; ++d) dot = __fadd_rn(dot, __fmul_rn(qs[d], kp[d]));
    }
    const float s = __fmul_rn(dot, scale);
    sc[p] = s;
    mloc = fmaxf(mloc, s);
  }
  const float mx = block_max<kAttnThreads>(mloc, s_red);
  for (int p = tid; p < np; p += kAttnThreads) sc[p] = libm_expf(__fsub_rn(sc[p], mx));
  __syncthreads();
  if (tid == 0) {
    float sum = 0.0f;
    for (int p = 0; p < np; ++p) sum = __fadd_rn(sum, sc[p]);
    s_inv = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = s_inv;
  for (int p = tid; p < np; p += kAttnThreads) sc[p] = __fmul_rn(sc[p], inv);
  __syncthreads();
  for (int d = tid; d < hd; d += kAttnThreads) {
    const float *vp = a.vcache + (size_t)kvh * hd + d;
    float o = 0.0f;
    int p = 0;
    for (; p + 8 <= np; p += 8) {
      float v[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) v[u] = vp[(size_t)(p + u) * kvd];
#pragma unroll
      for (int u = 0; u < 8; ++u) o = __fadd_rn(o, __fmul_rn(sc[p + u], v[u]));
    }
    for (; p < np; ++p) o = __fadd_rn(o, __fmul_rn(sc[p], vp[(size_t)p * kvd]));
    a.out[(size_t)h * hd + d] = o;
  }
}

// Final step bookkeeping: publish the argmax and error flags, advance the
// device-side token and position (used when steps are chained on the device),
// record the generated id, and reset the argmax cell and error word.
__global__ void k_step_finish(StepState *step, unsigned long long *argmax, int *err, int *result, int *tokens,
                              int max_seq) {
  pdl_wait();
  const unsigned long long key = *argmax;
  const int idx = static_cast<int>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
  const int pos = step->pos;
  const int e = *err;
  result[0] = idx;
  result[1] = e;
  result[2] = pos;
  result[3] |= e;
  if (pos >= 0 && pos < max_seq) tokens[pos] = idx;
  step->token = idx;
  step->pos = pos + 1;
  *argmax = 0ull;
  *err = 0;
}

// ------------------------------------------------------------ utility kernels
// Column absmax and codes of a row-major (rows, cols) matrix (quant.c:45-62):
// one thread per column walks the rows, so the loads of a warp are coalesced.
__global__ void k_quantize_percol(const float *w, int rows, int cols, int8_t *q, float *scale) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= cols) return;
  float m = 0.0f;
  for (int i = 0; i < rows; ++i) m = fmaxf(m, fabsf(w[(size_t)i * cols + j]));
  const float s = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, s);
  scale[j] = s;
  for (int i = 0; i < rows; ++i) q[(size_t)i * cols + j] = code_of(__fmul_rn(w[(size_t)i * cols + j], inv));
}

__global__ void k_dequantize_percol(const int8_t *q, const float *scale, long long rows, int cols, float *w) {
  const long long n = rows * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    w[i] = __fmul_rn(static_cast<float>(q[i]), scale[i % cols]);
}

// Writes the tiled layout: physical column p of the fused matrix comes from
// source `colsrc[p] >> 24` column `colsrc[p] & 0xffffff` (-1 = zero padding).
struct RepackSrc {
  const int8_t *m[3];
  int ncols[3];
};
__global__ void k_repack(RepackSrc src, const int *colsrc, int K, int Kpad, int Npad, int NT, int KT,
                         uint8_t *dst) {
  const long long chunks = (long long)Kpad / 16 * Npad;  // 16-byte chunks
  const int n_ktiles = Kpad / KT;
  for (long long ci = blockIdx.x * (long long)blockDim.x + threadIdx.x; ci < chunks;
       ci += (long long)gridDim.x * blockDim.x) {
    // chunk order == storage order: [slab][ktile][c][n]
    const int per_tile = (KT / 16) * NT;
    const long long tile = ci / per_tile;
    const int within = static_cast<int>(ci - tile * per_tile);
    const int c = within / NT, nn = within % NT;
    const long long slab = tile / n_ktiles;
    const int kt = static_cast<int>(tile - slab * n_ktiles);
    const int p = static_cast<int>(slab) * NT + nn;
    const int k0 = kt * KT + c * 16;
    const int cs = colsrc[p];
    uint8_t bytes[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      const int k = k0 + b;
      int8_t v = 0;
      if (cs >= 0 && k < K) {
        const int which = cs >> 24, jc = cs & 0xffffff;
        v = src.m[which][(size_t)k * src.ncols[which] + jc];
      }
      bytes[b] = static_cast<uint8_t>(v);
    }
    uint4 o;
    memcpy(&o, bytes, 16);
    reinterpret_cast<uint4 *>(dst)[ci] = o;
  }
}

// Tiles a plain row-major (K, N) matrix: physical column p is column p
// (p >= N: zero padding).  Same chunk order as k_repack.
__global__ void k_repack_plain(const int8_t *src, int K, int N, int Kpad, int Npad, int NT, int KT, uint8_t *dst) {
  const long long chunks = (long long)Kpad / 16 * Npad;
  const int n_ktiles = Kpad / KT;
  const int per_tile = (KT / 16) * NT;
  for (long long ci = blockIdx.x * (long long)blockDim.x + threadIdx.x; ci < chunks;
       ci += (long long)gridDim.x * blockDim.x) {
    const long long tile = ci / per_tile;
    const int within = static_cast<int>(ci - tile * per_tile);
    const int c = within / NT, nn = within % NT;
    const long long slab = tile / n_ktiles;
    const int kt = static_cast<int>(tile - slab * n_ktiles);
    const int p = static_cast<int>(slab) * NT + nn;
    const int k0 = kt * KT + c * 16;
    uint8_t bytes[16];
#pragma unroll
    for (int b = 0; b < 16; ++b) {
      const int k = k0 + b;
      bytes[b] = (p < N && k < K) ? static_cast<uint8_t>(src[(size_t)k * N + p]) : 0;
    }
    uint4 o;
    memcpy(&o, bytes, 16);
    reinterpret_cast<uint4 *>(dst)[ci] = o;
  }
}

// expf of a batch (tests compare this against the host libm over all inputs).
__global__ void k_expf_batch(const float *x, float *y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = libm_expf(x[i]);
}

}  // namespace llmq
