// llmq_sample.cuh - the reference's token sampler (sampler.c:60-115) on the
// GPU, drawing from the same xorshift64 stream (sampler.c:26-44) held in
// device memory.  Two kernels per draw:
//
//  k_sample_exp (all SMs): e_j = expf((l_j - max_l) / T) with the host C
//    library's expf, stored to scratch, plus a histogram of the e_j by their
//    top 11 bits (exponent and 3 mantissa bits) and a flag for NaN.  max_l is
//    read from the row's argmax key (argmax_key format).
//  k_sample (one CTA of 1024 threads): the reference's sum, candidates, top-p
//    cut, draw and scan.
//
// Every f32 value is the reference's, formed by the same rounded operations:
//  * sum = ((0 + e_0) + e_1) + ... (sampler.c:74-80).  While the running sum s
//    stays inside one binade its grid spacing u is fixed and every rounded add
//    moves s by a whole number of grid steps, round(e_j / u), which does not
//    depend on s, except when e_j / u ends in exactly one half (round to
//    even: depends on the parity of s / u) or when s + e_j may reach the next
//    binade.  So the chain is evaluated in windows of 8192 elements: a block
//    scan of the integer step counts, the half-way cases resolved in order
//    from the scanned prefix, and the first element that may leave the binade
//    added on its own with one rounded add; the next window starts after it.
//    The result is the sequential chain's, bit for bit.
//  * p_j = e_j / sum (sampler.c:81).  The reference sorts all (p, index) pairs
//    by p with qsort; glibc 2.39's qsort is a stable merge sort, so its first
//    k entries are the k largest by (p descending, index ascending).  p is
//    monotone in e, and two e that round to the same normal p differ by less
//    than 2^-22 relative, so every token with p >= p_(k) lies in the
//    histogram bin of the k-th largest e or in the bin below (bins are at
//    least 1/16 wide).  Those tokens (at most 4096) are collected while the
//    sum runs, their p formed, and bitonic sorted by (p descending, index
//    ascending).  Rows where that set is larger or its p are subnormal take a
//    radix select over the whole row instead.
//  * top-p, renormalised mass, draw and scan (sampler.c:86-111): one thread,
//    in order.
// A NaN anywhere in e (a NaN logit, or an infinite max) makes the reference's
// sum and every p NaN: nothing passes its comparisons and it returns the k-th
// token in index order after one draw; that case is taken directly.
//
// Covered: 1 <= k <= kSampleMaxK, where k = top_k when 0 < top_k < V and V
// otherwise (sampler.c:87-88).  temperature <= 0 is the greedy rule
// (sampler.c:65-67 -> sampler.c:8-21) and draws nothing.
#pragma once

#include "llmq_chain.cuh"
#include "llmq_kernels.cuh"

namespace llmq {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;
constexpr int kSampleBins = 2048;        // e histogram bins (e >= 0: bits 30..20)
constexpr int kSampleCandCap = 4096;     // candidates the histogram path holds
constexpr int kSumPer = 8;               // chain elements per thread and window
constexpr int kSumWindow = kSampleThreads * kSumPer;
constexpr int kSumHead = 1024;           // leading elements added one by one (from shared memory)
constexpr int kSumTieCap = 512;          // half-way cases resolved per window
constexpr int kSampleExpThreads = 512;
// dynamic shared memory of k_sample: the candidates, then the histogram
constexpr size_t kSampleSmem = ((size_t)kSampleCandCap * 2 + kSampleBins) * 4;

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
  const float *logits;               // [V]
  int V;
  SampleState *st;
  float *e;                          // scratch [V]
  unsigned *hist;                    // [kSampleBins + 1]: histogram, NaN flag; zero between draws
  const unsigned long long *maxkey;  // the row's argmax key
  unsigned long long *argmax;        // optional: receives the id in the key format k_step_finish reads
  int *out;                          // optional: receives the id
};

// The value an argmax key was made from (NaN when the row holds no number).
__device__ __forceinline__ float key_value(unsigned long long key) {
  const uint32_t h = static_cast<uint32_t>(key >> 32);
  if (h == 0u) return __uint_as_float(0x7fc00000u);
  return __uint_as_float((h & 0x80000000u) ? (h & 0x7fffffffu) : ~h);
}

__device__ __forceinline__ uint32_t lane_mask_lt() {
  uint32_t m;
  asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
  return m;
}

// One shared-memory histogram increment per distinct bin of the warp (every
// lane of the warp calls this).
__device__ __forceinline__ void sample_hist_add(unsigned *hist, uint32_t bin, bool active) {
  const unsigned act = __ballot_sync(0xffffffffu, active);
  if (active) {
    const unsigned peers = __match_any_sync(act, bin);
    if ((threadIdx.x & 31) == static_cast<unsigned>(__ffs(peers) - 1)) atomicAdd(&hist[bin], __popc(peers));
  }
}

// ---------------------------------------------------------------- exp pass
__global__ void __launch_bounds__(kSampleExpThreads) k_sample_exp(const SampleArgs a) {
  __shared__ unsigned s_h[kSampleBins];
  pdl_wait();
  const float T = a.st->temperature;
  if (T <= 0.0f) return;  // greedy: nothing to prepare
  const int tid = threadIdx.x, V = a.V;
  for (int b = tid; b < kSampleBins; b += kSampleExpThreads) s_h[b] = 0u;
  __syncthreads();
  const float mx = key_value(*a.maxkey);
  bool nan_seen = false;
  for (int j0 = blockIdx.x * kSampleExpThreads; j0 < V; j0 += gridDim.x * kSampleExpThreads) {
    const int j = j0 + tid;
    float e = 0.0f;
    if (j < V) {
      e = libm_expf(__fdiv_rn(__fsub_rn(a.logits[j], mx), T));
      a.e[j] = e;
      nan_seen |= e != e;
    }
    sample_hist_add(s_h, __float_as_uint(e) >> 20, j < V && e == e);
  }
  if (__syncthreads_or(nan_seen) && tid == 0) atomicOr(a.hist + kSampleBins, 1u);
  for (int b = tid; b < kSampleBins; b += kSampleExpThreads)
    if (s_h[b]) atomicAdd(a.hist + b, s_h[b]);
}

// --------------------------------------------------------- the draw (1 CTA)
__global__ void __launch_bounds__(kSampleThreads) k_sample(const SampleArgs a) {
  extern __shared__ __align__(16) unsigned char s_dyn[];
  uint32_t *c_key = reinterpret_cast<uint32_t *>(s_dyn);          // [kSampleCandCap]
  int *c_idx = reinterpret_cast<int *>(c_key + kSampleCandCap);   // [kSampleCandCap]
  // [kSampleBins]: the e histogram, then the chain's head, then 256 radix bins
  unsigned *s_hist = reinterpret_cast<unsigned *>(c_idx + kSampleCandCap);
  __shared__ uint32_t s_wr[32], s_wP[32], s_wE[32];
  __shared__ int s_wt[32], s_wjc[32];
  __shared__ int s_tie_o[kSumTieCap];
  __shared__ uint32_t s_tie_p[kSumTieCap], s_tie_n[kSumTieCap];
  __shared__ float s_cur;
  __shared__ uint32_t s_prefix;
  __shared__ int s_base, s_cons, s_ncand, s_ccount, s_blo, s_remaining, s_ngt;
  pdl_wait();
  LLMQ_TSTAMP(0);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, V = a.V;
  const float T = a.st->temperature;
  const int K = min(max(a.st->k, 1), min(kSampleMaxK, V));  // the host passes 1 <= k <= min(1024, V)

  auto publish = [&](int id) {
    if (a.argmax) *a.argmax = 0xffffffffull - static_cast<unsigned long long>(static_cast<uint32_t>(id));
    if (a.out) *a.out = id;
  };
  auto draw = [&]() -> float {  // rng_uniform (sampler.c:32-44)
    unsigned long long x = a.st->rng;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    a.st->rng = x;
    // top 53 bits scaled by 2^-53 (exact in double), then rounded to float
    return __double2float_rn(__dmul_rn(__ull2double_rn(x >> 11), 1.0 / 9007199254740992.0));
  };

  if (T <= 0.0f) {  // greedy: the first index of the largest logit (sampler.c:8-21)
    if (tid == 0) {
      const unsigned long long key = *a.maxkey;
      const float l0 = a.logits[0];
      publish((l0 != l0 || (key >> 32) == 0ull) ? 0 : static_cast<int>(0xffffffffu - static_cast<uint32_t>(key)));
    }
    return;
  }

  // ---- the histogram of e to shared memory (and zero for the next draw)
  const bool any_nan = a.hist[kSampleBins] != 0u;
  for (int b = tid; b < kSampleBins; b += kSampleThreads) {
    s_hist[b] = a.hist[b];
    a.hist[b] = 0u;
  }
  if (tid == 0) {
    s_blo = -1;
    s_ccount = kSampleCandCap + 1;
    s_ncand = 0;
  }
  __syncthreads();
  if (tid == 0) a.hist[kSampleBins] = 0u;
  if (any_nan) {  // every p is NaN: the k-th token in index order, after one draw
    if (tid == 0) {
      draw();
      publish(K - 1);
    }
    return;
  }
  {
    // counts from the top bin down; thread t holds bins 2047-2t and 2046-2t
    const int b_hi = kSampleBins - 1 - 2 * tid;
    const uint32_t h0 = s_hist[b_hi], h1 = s_hist[b_hi - 1];
    uint32_t incl = h0 + h1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) s_wr[warp] = incl;
    __syncthreads();
    uint32_t off = 0u;
    for (int w = 0; w < warp; ++w) off += s_wr[w];
    const uint32_t above = off + incl - h0 - h1;             // in bins > b_hi
    const uint32_t at0 = above + h0, at1 = at0 + h1;         // in bins >= b_hi, >= b_hi - 1
    const uint32_t k = static_cast<uint32_t>(K);
    // the bin of the k-th largest e, then one bin of margin below it
    if (above < k && at0 >= k) s_blo = max(b_hi - 1, 0);
    if (at0 < k && at1 >= k) s_blo = max(b_hi - 2, 0);
    __syncthreads();
    const int blo = s_blo;
    if (blo == b_hi) s_ccount = static_cast<int>(at0);
    if (blo == b_hi - 1) s_ccount = static_cast<int>(at1);
    __syncthreads();
  }
  const int blo = s_blo;
  const bool hist_path = blo >= 0 && s_ccount <= kSampleCandCap;
  LLMQ_TSTAMP(1);

  // ---- the sequential sum (sampler.c:74-80), collecting the candidates
  auto record = [&](uint32_t eb, int j, bool want) {  // every lane of the warp calls this
    const unsigned bal = __ballot_sync(0xffffffffu, want);
    if (bal == 0u) return;
    const int leader = __ffs(bal) - 1;
    int slot0 = 0;
    if (lane == leader) slot0 = atomicAdd(&s_ncand, __popc(bal));
    slot0 = __shfl_sync(0xffffffffu, slot0, leader);
    if (want) {
      const int slot = slot0 + __popc(bal & lane_mask_lt());
      if (slot < kSampleCandCap) {
        c_key[slot] = eb;
        c_idx[slot] = j;
      }
    }
  };
  const int head = min(V, kSumHead);
  float *s_head = reinterpret_cast<float *>(s_hist);  // the histogram has been read
  for (int j = tid; j < head; j += kSampleThreads) s_head[j] = a.e[j];
  __syncthreads();
  if (tid == 0) {
    s_cur = seq_sum(s_head, 1, head, 0.0f);
    s_base = head;
  }
  for (int j0 = 0; j0 < kSumHead; j0 += kSampleThreads) {  // the head's candidates
    const int j = j0 + tid;
    const uint32_t eb = j < head ? __float_as_uint(s_head[j]) : 0u;
    record(eb, j, hist_path && j < head && static_cast<int>(eb >> 20) >= blo);
  }
  __syncthreads();
  uint32_t pre[kSumPer];
  int pre_base = -1;
  while (true) {
    const int base = s_base;
    if (base >= V) break;
    const int len = min(kSumWindow, V - base);
    const uint32_t sb = __float_as_uint(s_cur);
    const uint32_t sef = sb >> 23;
    const int uexp = sef ? static_cast<int>(sef) - 150 : -149;  // the grid of s: spacing 2^uexp
    const uint32_t M = sef ? ((sb & 0x7fffffu) | 0x800000u) : sb;  // s = M * 2^uexp
    const int o0 = tid * kSumPer;
    uint32_t eb[kSumPer];
    if (pre_base == base) {
#pragma unroll
      for (int q = 0; q < kSumPer; ++q) eb[q] = pre[q];
    } else {
#pragma unroll
      for (int q = 0; q < kSumPer; ++q) eb[q] = o0 + q < len ? __float_as_uint(a.e[base + o0 + q]) : 0u;
    }
    pre_base = base + len;  // prefetch the following window (used when this one runs to its end)
#pragma unroll
    for (int q = 0; q < kSumPer; ++q) {
      const int j = pre_base + o0 + q;
      pre[q] = j < V ? __float_as_uint(a.e[j]) : 0u;
    }
    uint32_t r[kSumPer], tiebits = 0u, rsum = 0u;
    if (uexp >= -100 && uexp <= 0) {
      const float inv_u = pow2f(-uexp);
#pragma unroll
      for (int q = 0; q < kSumPer; ++q) {
        const ChainStep c = chain_step_f(eb[q], inv_u);
        r[q] = c.r;
        tiebits |= c.tie ? (1u << q) : 0u;
        rsum = sat_add(rsum, c.r);
      }
    } else {
#pragma unroll
      for (int q = 0; q < kSumPer; ++q) {
        const ChainStep c = chain_step(eb[q], uexp);
        r[q] = c.r;
        tiebits |= c.tie ? (1u << q) : 0u;
        rsum = sat_add(rsum, c.r);
      }
    }
    const int tsum = __popc(tiebits);
    // block scan of the step counts and half-way counts
    uint32_t ri = rsum;
    int ti = tsum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t rv = __shfl_up_sync(0xffffffffu, ri, o);
      const int tv = __shfl_up_sync(0xffffffffu, ti, o);
      if (lane >= o) {
        ri = sat_add(ri, rv);
        ti += tv;
      }
    }
    if (lane == 31) {
      s_wr[warp] = ri;
      s_wt[warp] = ti;
    }
    __syncthreads();
    uint32_t wr = s_wr[lane];
    int wt = s_wt[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t rv = __shfl_up_sync(0xffffffffu, wr, o);
      const int tv = __shfl_up_sync(0xffffffffu, wt, o);
      if (lane >= o) {
        wr = sat_add(wr, rv);
        wt += tv;
      }
    }
    const uint32_t total = __shfl_sync(0xffffffffu, wr, 31);
    const int n_ties = __shfl_sync(0xffffffffu, wt, 31);
    const uint32_t woff = __shfl_sync(0xffffffffu, wr, (warp + 31) & 31);
    const int toff = __shfl_sync(0xffffffffu, wt, (warp + 31) & 31);
    // exclusive prefix of this thread: the previous lane's inclusive one (a
    // saturated prefix is exact below kChainSat, and nothing past the first flagged
    // element is used)
    uint32_t ex = __shfl_up_sync(0xffffffffu, ri, 1);
    if (lane == 0) ex = 0u;
    uint32_t P = sat_add(warp ? woff : 0u, ex);
    int Tc = (warp ? toff : 0) + ti - tsum;
    int f_o = kSumWindow;
    uint32_t f_P = 0u, f_E = 0u;
#pragma unroll
    for (int q = 0; q < kSumPer; ++q) {
      const int o = o0 + q;
      if (o < len) {
        const bool tie = (tiebits >> q) & 1u;
        // may this add reach the next binade, whatever the half-way cases before it did?
        bool flag = M + P + static_cast<uint32_t>(Tc) + r[q] + 1u >= (1u << 24);  // < 2^32: P, r <= 2^30
        if (tie) {  // listed in order; the first one past the list ends the window
          if (Tc < kSumTieCap) {
            s_tie_o[Tc] = o;
            s_tie_p[Tc] = P;
            s_tie_n[Tc] = r[q];
          } else if (Tc == kSumTieCap) {
            flag = true;
          }
        }
        if (flag && f_o == kSumWindow) {
          f_o = o;
          f_P = P;
          f_E = eb[q];
        }
        P = sat_add(P, r[q]);
        Tc += tie ? 1 : 0;
      }
    }
    {  // the warp's first flagged element, with its prefix and e
      const int wmin = warp_min(f_o);
      const unsigned who = __ballot_sync(0xffffffffu, f_o == wmin);
      if (lane == __ffs(who) - 1) {
        s_wjc[warp] = wmin;
        s_wP[warp] = f_P;
        s_wE[warp] = f_E;
      }
    }
    __syncthreads();
    if (warp == 0) {  // the window's first flagged element; resolve the half-way cases before it
      const int wj = s_wjc[lane];
      const int jmin = warp_min(wj);
      const int src = __ffs(__ballot_sync(0xffffffffu, wj == jmin)) - 1;
      const uint32_t Pj = __shfl_sync(0xffffffffu, s_wP[lane], src);
      const uint32_t Ej = __shfl_sync(0xffffffffu, s_wE[lane], src);
      if (lane == 0) {
        const int jc = min(jmin, len);
        const int nl = min(n_ties, kSumTieCap);
        uint32_t ups = 0u;
        for (int i = 0; i < nl && s_tie_o[i] < jc; ++i) ups += (M + s_tie_p[i] + ups + s_tie_n[i]) & 1u;  // to even
        const uint32_t Mn = M + (jc < len ? Pj : total) + ups;
        float sn = __fmul_rn(__uint2float_rn(Mn), pow2f(uexp));
        if (jc < len) sn = __fadd_rn(sn, __uint_as_float(Ej));  // the flagged element, one rounded add
        s_cur = sn;
        s_cons = jc < len ? jc + 1 : len;
        s_base = base + s_cons;
      }
    }
    __syncthreads();
    const int cons = s_cons;
#pragma unroll
    for (int q = 0; q < kSumPer; ++q) {
      const int o = o0 + q;
      record(eb[q], base + o, hist_path && o < cons && static_cast<int>(eb[q] >> 20) >= blo);
    }
  }
  __syncthreads();
  const float sum = s_cur;
  LLMQ_TSTAMP(2);

  // ---- the k candidates by (p descending, index ascending) in c_key / c_idx
  // (c_key: the bits of p = e / sum, sampler.c:81; every p here is >= +0)
  bool fast = hist_path && s_ncand == s_ccount;
  if (fast) {  // the one-bin margin holds for normal p
    const float p_lo = __fdiv_rn(__uint_as_float(static_cast<uint32_t>(blo) << 20), sum);
    fast = p_lo >= 2.3509887e-38f;  // 2^-125
  }
  int C;
  if (fast) {
    C = s_ncand;
    for (int i = tid; i < C; i += kSampleThreads) c_key[i] = __float_as_uint(__fdiv_rn(__uint_as_float(c_key[i]), sum));
  } else {
    // radix select of the k-th largest p over the whole row
    unsigned *h256 = s_hist;  // the chain's head is done with
    if (tid == 0) {
      s_prefix = 0u;
      s_remaining = K;
      s_ngt = 0;
    }
    for (int b = tid; b < 256; b += kSampleThreads) h256[b] = 0u;
    __syncthreads();
    for (int j0 = 0; j0 < V; j0 += kSampleThreads) {
      const int j = j0 + tid;
      uint32_t key = 0u;
      if (j < V) {
        const float p = __fdiv_rn(a.e[j], sum);
        a.e[j] = p;
        key = __float_as_uint(p);
      }
      sample_hist_add(h256, key >> 24, j < V);
    }
    __syncthreads();
    uint32_t mask = 0u;
    for (int shift = 24; shift >= 0; shift -= 8) {
      if (shift < 24) {
        for (int b = tid; b < 256; b += kSampleThreads) h256[b] = 0u;
        __syncthreads();
        const uint32_t prefix = s_prefix;
        for (int j0 = 0; j0 < V; j0 += kSampleThreads) {
          const int j = j0 + tid;
          const uint32_t key = j < V ? __float_as_uint(a.e[j]) : 0u;
          sample_hist_add(h256, (key >> shift) & 255u, j < V && (key & mask) == prefix);
        }
        __syncthreads();
      }
      if (tid == 0) {
        int rem = s_remaining;
        for (int b = 255; b >= 0; --b) {
          const int h = static_cast<int>(h256[b]);
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
    const int n_eq = min(max(s_remaining, 0), K), n_gt = K - n_eq;
    // every key above kth, then the n_eq lowest indices with key == kth (each
    // warp owns one contiguous index range, in order)
    const int span = ((V + 32 * 32 - 1) / (32 * 32)) * 32;
    const int w0 = min(V, warp * span), w1 = min(V, w0 + span);
    int eq_count = 0;
    for (int j0 = w0; j0 < w1; j0 += 32) {
      const int j = j0 + lane;
      const uint32_t key = j < w1 ? __float_as_uint(a.e[j]) : 0u;
      const bool gt = j < w1 && key > kth, eq = j < w1 && key == kth;
      if (gt) {
        const int slot = atomicAdd(&s_ngt, 1);
        if (slot < n_gt) {
          c_key[slot] = key;
          c_idx[slot] = j;
        }
      }
      eq_count += __popc(__ballot_sync(0xffffffffu, eq));
    }
    if (lane == 0) s_wt[warp] = eq_count;
    __syncthreads();
    int rank0 = lane < warp ? s_wt[lane] : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) rank0 += __shfl_xor_sync(0xffffffffu, rank0, o);
    for (int j0 = w0; j0 < w1 && rank0 < n_eq; j0 += 32) {
      const int j = j0 + lane;
      const bool eq = j < w1 && __float_as_uint(a.e[j]) == kth;
      const unsigned bal = __ballot_sync(0xffffffffu, eq);
      const int rank = rank0 + __popc(bal & lane_mask_lt());
      if (eq && rank < n_eq) {
        c_key[n_gt + rank] = kth;
        c_idx[n_gt + rank] = j;
      }
      rank0 += __popc(bal);
    }
    C = K;
  }
  // bitonic sort of the C candidates; padding (key 0, index INT_MAX) sorts last
  int P2 = 1;
  while (P2 < C) P2 <<= 1;
  for (int i = C + tid; i < P2; i += kSampleThreads) {
    c_key[i] = 0u;
    c_idx[i] = 0x7fffffff;
  }
  __syncthreads();
  LLMQ_TSTAMP(3);
  for (int size = 2; size <= P2; size <<= 1)
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < P2; i += kSampleThreads) {
        const int q = i ^ stride;
        if (q > i) {
          const uint32_t ki = c_key[i], kq = c_key[q];
          const int ii = c_idx[i], iq = c_idx[q];
          const bool i_first = ki > kq || (ki == kq && ii < iq);
          if (i_first != ((i & size) == 0)) {
            c_key[i] = kq;
            c_key[q] = ki;
            c_idx[i] = iq;
            c_idx[q] = ii;
          }
        }
      }
      __syncthreads();
    }
  LLMQ_TSTAMP(4);

  // ---- top-p, renormalised mass, draw, scan (sampler.c:86-111)
  if (tid == 0) {
    const float top_p = a.st->top_p;
    const float *cp = reinterpret_cast<const float *>(c_key);
    int keep = K;
    if (top_p > 0.0f && top_p < 1.0f) {
      float cum = 0.0f;
      int kp = 0;
      for (int i = 0; i < keep; ++i) {
        cum = __fadd_rn(cum, cp[i]);
        ++kp;
        if (cum >= top_p) break;
      }
      keep = kp;
    }
    if (keep < 1) keep = 1;
    float z = 0.0f;
    for (int i = 0; i < keep; ++i) z = __fadd_rn(z, cp[i]);
    const float u = __fmul_rn(draw(), z);
    int chosen = c_idx[keep - 1];
    float acc = 0.0f;
    for (int i = 0; i < keep; ++i) {
      acc = __fadd_rn(acc, cp[i]);
      if (u <= acc) {
        chosen = c_idx[i];
        break;
      }
    }
    publish(chosen);
  }
  LLMQ_TSTAMP(5);
}

// CTAs of k_sample_exp for a row of V logits (one pass of 512 per CTA, at
// most two CTAs per SM).
inline int sample_exp_grid(int V) {
  const int n = (V + kSampleExpThreads - 1) / kSampleExpThreads;
  return n < 1 ? 1 : (n > 2 * 148 ? 2 * 148 : n);
}

// The row's argmax key (argmax_key format) for the standalone sampler; *key
// must be 0 before the launch.
__global__ void __launch_bounds__(256) k_sample_max(const float *l, int V, unsigned long long *key) {
  __shared__ unsigned long long s_red64[32];
  unsigned long long best = 0ull;
  for (int j = blockIdx.x * 256 + threadIdx.x; j < V; j += gridDim.x * 256) {
    const unsigned long long k = argmax_key(l[j], static_cast<uint32_t>(j));
    best = k > best ? k : best;
  }
  best = block_max_u64<256>(best, s_red64);
  if (threadIdx.x == 0) atomicMax(key, best);
}

}  // namespace llmq
