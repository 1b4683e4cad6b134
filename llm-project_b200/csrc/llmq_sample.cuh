// llmq_sample.cuh - the reference's token sampler (sampler.c:60-115) on the
// GPU: one CTA of 1024 threads turns one logits row into one token id and
// advances the xorshift64 stream (sampler.c:26-44) held in device memory.
//
// Every f32 value is formed with the reference's operations, in its order:
//   max_l: l[0], then each larger l[j] (a NaN l[0] stays the max);
//   e_j = expf((l_j - max_l) / T) with the host C library's expf;
//   sum = ((0 + e_0) + e_1) + ...: one thread, the row streaming through a
//   double-buffered shared-memory ring that the other 31 warps fill;
//   p_j = e_j / sum.
// The reference then sorts all V (p, index) pairs by p, descending, with the
// C library's qsort; glibc 2.39's qsort is a stable merge sort, so equal p
// keep index order and the first k of the sorted array are the k largest by
// (p descending, index ascending).  That is what is selected here, without a
// full sort: a 4-pass radix select of the k-th largest p (bit patterns of
// non-negative floats order like the floats), then every token above it plus
// the lowest-index tokens equal to it.  The k candidates are bitonic-sorted by
// (p descending, index ascending), after which one thread runs the reference's
// top-p cut, renormalised mass, draw and scan (sampler.c:86-111) on them.  The
// result is the reference's token for every input, ties included.
//
// Covered: 1 <= k <= kSampleMaxK, where k = top_k when 0 < top_k < V and V
// otherwise (sampler.c:87-88).  temperature <= 0 is the greedy rule
// (sampler.c:65-67 -> sampler.c:8-21) and draws nothing.
#pragma once

#include "llmq_kernels.cuh"

namespace llmq {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;
constexpr int kSampleChunk = 4096;  // e values per ring slot of the sequential sum

// Device-resident sampler settings and stream; the host mirrors it in pinned
// memory and copies it in / out around the steps that sample.
struct SampleState {
  float temperature;
  int k;                    // candidates kept by top-k, already resolved (see above)
  float top_p;
  int pad;
  unsigned long long rng;   // Rng.state (sampler.h)
};

struct SampleArgs {
  const float *logits;           // [V]
  int V;
  SampleState *st;
  float *p;                      // scratch [V]
  unsigned long long *argmax;    // optional: receives the id in the key format k_step_finish reads
  int *out;                      // optional: receives the id
};

// Order-preserving 32-bit key of a float (a larger float has a larger key);
// NaN maps to 0, below every number.
__device__ __forceinline__ uint32_t sample_key(float v) {
  if (v != v) return 0u;
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// One shared-memory histogram increment per distinct digit of the warp
// (every lane of the warp calls this).
__device__ __forceinline__ void sample_hist_add(unsigned *hist, uint32_t digit, bool active) {
  const unsigned act = __ballot_sync(0xffffffffu, active);
  if (active) {
    const unsigned peers = __match_any_sync(act, digit);
    if ((threadIdx.x & 31) == static_cast<unsigned>(__ffs(peers) - 1)) atomicAdd(&hist[digit], __popc(peers));
  }
}

__global__ void __launch_bounds__(kSampleThreads) k_sample(const SampleArgs a) {
  __shared__ __align__(16) float s_ring[2][kSampleChunk];
  __shared__ uint32_t s_key[kSampleMaxK];
  __shared__ int s_idx[kSampleMaxK];
  __shared__ float s_p[kSampleMaxK];
  __shared__ unsigned s_hist[256];
  __shared__ unsigned long long s_red64[32];
  __shared__ float s_red[32];
  __shared__ int s_wcount[32];
  __shared__ float s_sum;
  __shared__ uint32_t s_prefix;
  __shared__ int s_remaining, s_ngt;
  pdl_wait();
  LLMQ_TSTAMP(0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, V = a.V;
  const float T = a.st->temperature;
  const int K = min(max(a.st->k, 1), min(kSampleMaxK, V));  // the host passes 1 <= k <= min(1024, V)
  const float l0 = a.logits[0];

  auto publish = [&](int id) {
    if (a.argmax) *a.argmax = 0xffffffffull - static_cast<unsigned long long>(static_cast<uint32_t>(id));
    if (a.out) *a.out = id;
  };

  if (T <= 0.0f) {  // greedy: the first index of the largest logit (sampler.c:8-21)
    unsigned long long best = 0ull;
    for (int j = tid; j < V; j += kSampleThreads) {
      const float v = a.logits[j];
      if (v == v) {
        const unsigned long long key =
            (static_cast<unsigned long long>(sample_key(v)) << 32) | (0xffffffffu - static_cast<uint32_t>(j));
        best = key > best ? key : best;
      }
    }
    best = block_max_u64<kSampleThreads>(best, s_red64);
    if (tid == 0) publish(l0 != l0 ? 0 : static_cast<int>(0xffffffffu - static_cast<uint32_t>(best)));
    return;
  }

  // ---- max_l (sampler.c:70-71)
  float m = -INFINITY;
  for (int j = tid; j < V; j += kSampleThreads) m = fmaxf(m, a.logits[j]);
  m = block_max<kSampleThreads>(m, s_red);
  const float mx = (l0 != l0) ? l0 : m;
  LLMQ_TSTAMP(1);

  // ---- e_j and their sequential sum (sampler.c:74-80)
  const int n_chunks = (V + kSampleChunk - 1) / kSampleChunk;
  auto fill = [&](int c, float *slot, int t0, int nt) {
    const int base = c * kSampleChunk, n = min(kSampleChunk, V - base);
    for (int j = t0; j < n; j += nt) {
      const float e = libm_expf(__fdiv_rn(__fsub_rn(a.logits[base + j], mx), T));
      slot[j] = e;
      a.p[base + j] = e;
    }
  };
  fill(0, s_ring[0], tid, kSampleThreads);
  float sum = 0.0f;
  for (int c = 0; c < n_chunks; ++c) {
    __syncthreads();  // slot c & 1 is full; slot (c + 1) & 1 was consumed in the previous round
    if (warp == 0) {
      if (lane == 0) sum = seq_sum(s_ring[c & 1], 1, min(kSampleChunk, V - c * kSampleChunk), sum);
    } else if (c + 1 < n_chunks) {
      fill(c + 1, s_ring[(c + 1) & 1], tid - 32, kSampleThreads - 32);
    }
  }
  if (tid == 0) {
    s_sum = sum;
    s_prefix = 0u;
    s_remaining = K;
    s_ngt = 0;
  }
  for (int b = tid; b < 256; b += kSampleThreads) s_hist[b] = 0u;
  __syncthreads();
  LLMQ_TSTAMP(2);

  // ---- p_j = e_j / sum (sampler.c:81), with the histogram of the keys' top byte
  const float total = s_sum;
  for (int j0 = 0; j0 < V; j0 += kSampleThreads) {
    const int j = j0 + tid;
    uint32_t key = 0u;
    if (j < V) {
      const float p = __fdiv_rn(a.p[j], total);
      a.p[j] = p;
      key = sample_key(p);
    }
    sample_hist_add(s_hist, key >> 24, j < V);
  }
  __syncthreads();
  LLMQ_TSTAMP(3);

  // ---- radix select of the k-th largest key, one byte per pass
  uint32_t mask = 0u;
  for (int shift = 24; shift >= 0; shift -= 8) {
    if (shift < 24) {
      for (int b = tid; b < 256; b += kSampleThreads) s_hist[b] = 0u;
      __syncthreads();
      const uint32_t prefix = s_prefix;
      for (int j0 = 0; j0 < V; j0 += kSampleThreads) {
        const int j = j0 + tid;
        const uint32_t key = j < V ? sample_key(a.p[j]) : 0u;
        sample_hist_add(s_hist, (key >> shift) & 255u, j < V && (key & mask) == prefix);
      }
      __syncthreads();
    }
    if (tid == 0) {
      int rem = s_remaining;
      for (int b = 255; b >= 0; --b) {
        const int h = static_cast<int>(s_hist[b]);
        if (h >= rem) {
          s_prefix |= static_cast<uint32_t>(b) << shift;
          break;
        }
        rem -= h;
      }
      s_remaining = rem;
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t kth = s_prefix;
  LLMQ_TSTAMP(4);
  const int n_eq = min(max(s_remaining, 0), K), n_gt = K - n_eq;

  // ---- the k candidates: every key above kth, then the n_eq lowest indices
  // with key == kth (each warp owns one contiguous index range, in order)
  const int span = ((V + 32 * 32 - 1) / (32 * 32)) * 32;
  const int w0 = min(V, warp * span), w1 = min(V, w0 + span);
  int eq_count = 0;
  for (int j0 = w0; j0 < w1; j0 += 32) {
    const int j = j0 + lane;
    const uint32_t key = j < w1 ? sample_key(a.p[j]) : 0u;
    const bool gt = j < w1 && key > kth, eq = j < w1 && key == kth;
    if (gt) {
      const int slot = atomicAdd(&s_ngt, 1);
      if (slot < n_gt) {
        s_key[slot] = key;
        s_idx[slot] = j;
      }
    }
    eq_count += __popc(__ballot_sync(0xffffffffu, eq));
  }
  if (lane == 0) s_wcount[warp] = eq_count;
  __syncthreads();
  int rank0 = lane < warp ? s_wcount[lane] : 0;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) rank0 += __shfl_xor_sync(0xffffffffu, rank0, o);
  for (int j0 = w0; j0 < w1 && rank0 < n_eq; j0 += 32) {
    const int j = j0 + lane;
    const bool eq = j < w1 && sample_key(a.p[j]) == kth;
    const unsigned bal = __ballot_sync(0xffffffffu, eq);
    const int rank = rank0 + __popc(bal & ((1u << lane) - 1u));
    if (eq && rank < n_eq) {
      s_key[n_gt + rank] = kth;
      s_idx[n_gt + rank] = j;
    }
    rank0 += __popc(bal);
  }
  __syncthreads();
  LLMQ_TSTAMP(5);

  // ---- bitonic sort of the candidates by (p descending, index ascending);
  // padding entries (key 0, index INT_MAX) sort last
  int P = 1;
  while (P < K) P <<= 1;
  for (int i = K + tid; i < P; i += kSampleThreads) {
    s_key[i] = 0u;
    s_idx[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int size = 2; size <= P; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P; i += kSampleThreads) {
        const int q = i ^ stride;
        if (q > i) {
          const uint32_t ki = s_key[i], kq = s_key[q];
          const int ii = s_idx[i], iq = s_idx[q];
          const bool i_first = ki > kq || (ki == kq && ii < iq);
          if (i_first != ((i & size) == 0)) {
            s_key[i] = kq;
            s_key[q] = ki;
            s_idx[i] = iq;
            s_idx[q] = ii;
          }
        }
      }
      __syncthreads();
    }
  for (int i = tid; i < K; i += kSampleThreads) s_p[i] = a.p[min(max(s_idx[i], 0), V - 1)];
  __syncthreads();
  LLMQ_TSTAMP(6);

  // ---- top-p, renormalised mass, draw, scan (sampler.c:89-111)
  if (tid == 0) {
    const float top_p = a.st->top_p;
    int keep = K;
    if (top_p > 0.0f && top_p < 1.0f) {
      float cum = 0.0f;
      int kp = 0;
      for (int i = 0; i < keep; ++i) {
        cum = __fadd_rn(cum, s_p[i]);
        ++kp;
        if (cum >= top_p) break;
      }
      keep = kp;
    }
    if (keep < 1) keep = 1;
    float z = 0.0f;
    for (int i = 0; i < keep; ++i) z = __fadd_rn(z, s_p[i]);
    unsigned long long x = a.st->rng;  // xorshift64 (sampler.c:32-39)
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    a.st->rng = x;
    // top 53 bits scaled by 2^-53 (exact in double), then rounded to float (sampler.c:43)
    const float uni = __double2float_rn(__dmul_rn(__ull2double_rn(x >> 11), 1.0 / 9007199254740992.0));
    const float u = __fmul_rn(uni, z);
    int chosen = s_idx[keep - 1];
    float acc = 0.0f;
    for (int i = 0; i < keep; ++i) {
      acc = __fadd_rn(acc, s_p[i]);
      if (u <= acc) {
        chosen = s_idx[i];
        break;
      }
    }
    publish(chosen);
  }
  LLMQ_TSTAMP(7);
}

}  // namespace llmq
