// llmq_rows.cuh - kernels of the multi-row decode pass: several sequences
// decoding one token each (batched decode), or consecutive prompt tokens of one
// sequence (prefill).  Each row is one reference decode step
// (q_llama_decode_step, llama.c:528-600) with its own cache and position; the
// products run on the tcgen05 GEMM (llmq_tc_gemm.cuh) and every per-row
// reduction keeps the reference's sequential order, so each row's logits equal
// those of the single-token path bit for bit.
#pragma once

#include "llmq_tc_gemm.cuh"

namespace llmq {

// One row of a pass: token `token` at position `pos` of the sequence whose
// head-major device cache (per layer [n_kv][max_seq][hd]) starts at k / v.
struct RowDesc {
  float *k, *v;
  int max_seq, pos, token, pad;
};

constexpr int kRowThreads = 512;

struct RowNormArgs {
  const RowDesc *rd;
  const float *in;        // [rows][K]; null: the embedding rows of rd[r].token
  float *x_out;           // embedding rows are also written here (the residual stream)
  const int8_t *wte_q;
  const float *wte_s;
  int vocab;
  const float *gamma;
  float eps;
  int K, Kpad, KT;
  int8_t *codes;          // tcgen05 A tiles (tc_code_offset)
  float *as;              // [rows]
  int *err;
};

// RMSNorm of one row (rmsnorm.c:7-21, the arithmetic of k_gemv's RMSNorm
// prologue), then its activation codes (quant.c:104-113).  One CTA per row;
// dynamic shared memory 2 * K floats.
__global__ void __launch_bounds__(kRowThreads) k_rows_norm_codes(const RowNormArgs a) {
  extern __shared__ __align__(16) float xs[];
  __shared__ float s_red[32];
  __shared__ float s_r;
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x, tid = threadIdx.x, K = a.K;
  float *sq = xs + ((K + 3) & ~3);
  if (a.in == nullptr) {
    int token = a.rd[r].token;
    if (token < 0 || token >= a.vocab) {
      if (tid == 0) atomicOr(a.err, ERR_BAD_TOKEN);
      token = 0;
    }
    const int8_t *row = a.wte_q + (size_t)token * K;
    for (int k = tid; k < K; k += kRowThreads) {
      const float v = __fmul_rn(static_cast<float>(row[k]), a.wte_s[k]);  // llama.c:536
      xs[k] = v;
      a.x_out[(size_t)r * K + k] = v;
    }
  } else {
    const float *row = a.in + (size_t)r * K;
    for (int k = tid; k < K; k += kRowThreads) xs[k] = row[k];
  }
  __syncthreads();
  for (int k = tid; k < K; k += kRowThreads) sq[k] = __fmul_rn(xs[k], xs[k]);
  __syncthreads();
  if (tid == 0) {
    float ms = seq_sum(sq, 1, K, 0.0f);  // rmsnorm.c:15, in index order
    ms = __fmul_rn(ms, __fdiv_rn(1.0f, static_cast<float>(K)));
    s_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
  }
  __syncthreads();
  const float rr = s_r;
  float m = 0.0f;
  for (int k = tid; k < K; k += kRowThreads) {
    const float y = __fmul_rn(__fmul_rn(xs[k], rr), a.gamma[k]);
    xs[k] = y;
    m = fmaxf(m, fabsf(y));
  }
  m = block_max<kRowThreads>(m, s_red);
  __syncthreads();
  const float as = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;  // quant.c:106
  const float inv = __fdiv_rn(1.0f, as);                      // quant.c:107
  if (tid == 0) a.as[r] = as;
  for (int ch = tid; ch < a.Kpad / 16; ch += kRowThreads)
    *reinterpret_cast<int4 *>(a.codes + tc_code_offset(r, ch, a.Kpad, a.KT)) = tc_pack16(xs, ch * 16, K, inv);
}

struct RowAttnArgs {
  const RowDesc *rd;
  const float *qkv;       // [rows][qd + 2 kvd]: q, k, v of each row (bias added, before RoPE)
  float *qr;              // [rows][qd]: q after RoPE
  float *scores;          // [rows][n_heads][smax]
  float *out;             // [rows][qd]
  const float *rope_cos, *rope_sin;  // [max_seq][hd/2]
  int layer, n_heads, n_kv, hd, smax;
  int *err;
};

__device__ __forceinline__ size_t row_cache_offset(const RowDesc &d, int layer, int n_kv, int kvh, int hd) {
  return (((size_t)layer * n_kv + kvh) * d.max_seq) * hd;
}

// RoPE of q and k (rope.c:48-68) at the row's position; the rotated k and the
// v of the row are appended to its cache (llama.c:551-552).  One CTA per row.
__global__ void __launch_bounds__(256) k_rows_append(const RowAttnArgs a) {
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x, tid = threadIdx.x;
  const RowDesc d = a.rd[r];
  const int hd = a.hd, half = hd / 2, qd = a.n_heads * hd, kvd = a.n_kv * hd;
  if (d.pos < 0 || d.pos >= d.max_seq) {
    if (tid == 0) atomicOr(a.err, ERR_BAD_POS);
    return;
  }
  const float *row = a.qkv + (size_t)r * (qd + 2 * kvd);
  const float *cs = a.rope_cos + (size_t)d.pos * half, *sn = a.rope_sin + (size_t)d.pos * half;
  for (int e = tid; e < qd; e += 256) {
    const int h = e / hd, i = e - h * hd;
    a.qr[(size_t)r * qd + e] = rope_elem(row + (size_t)h * hd, i, half, cs, sn);
  }
  for (int e = tid; e < kvd; e += 256) {
    const int h = e / hd, i = e - h * hd;
    const size_t at = row_cache_offset(d, a.layer, a.n_kv, h, hd) + (size_t)d.pos * hd + i;
    d.k[at] = rope_elem(row + qd + (size_t)h * hd, i, half, cs, sn);
    d.v[at] = row[qd + kvd + e];
  }
}

// Scores of one row's query group (one KV head) over one chunk of key
// positions [p0, min(p0 + 64, pos + 1)) of its cache (llama.c:558-565): each a
// sequential dot product over the head dimension, times 1/sqrt(hd).
// Grid (ceil(smax / 64), n_kv, rows).
__global__ void __launch_bounds__(kScoreThreads) k_rows_scores(const RowAttnArgs a) {
  extern __shared__ __align__(16) float sm_s[];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, kvh = blockIdx.y, r = blockIdx.z;
  const RowDesc d = a.rd[r];
  const int p0 = blockIdx.x * kScoreChunk;
  if (d.pos < 0 || d.pos >= d.max_seq || p0 > d.pos) return;
  const int hd = a.hd, group = a.n_heads / a.n_kv, qd = a.n_heads * hd;
  const int stride = (hd & 3) == 0 ? hd + 4 : hd + 1;
  const int hd4 = (hd + 3) & ~3;
  float *qs = sm_s;                        // [group][hd4]
  float *ks = sm_s + (size_t)group * hd4;  // [kScoreChunk][stride]
  const int p1 = min(p0 + kScoreChunk, d.pos + 1);
  stage_rows(ks, stride, d.k + row_cache_offset(d, a.layer, a.n_kv, kvh, hd), hd, p0, p1, 0, hd, tid,
             kScoreThreads);
  cp_async_commit();
  const float *q = a.qr + (size_t)r * qd + (size_t)kvh * group * hd;
  for (int i = tid; i < group * hd; i += kScoreThreads) {
    const int g = i / hd, e = i - g * hd;
    qs[g * hd4 + e] = q[i];
  }
  cp_async_wait<0>();
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));  // llama.c:532
  float *srow = a.scores + ((size_t)r * a.n_heads + (size_t)kvh * group) * a.smax;
  for (int i = tid; i < group * kScoreChunk; i += kScoreThreads) {
    const int g = i / kScoreChunk, p = i - g * kScoreChunk;
    if (p0 + p >= p1) continue;
    const float dot = seq_dot(qs + (size_t)g * hd4, ks + (size_t)p * stride, 1, hd, 0.0f);  // llama.c:561
    srow[(size_t)g * a.smax + p0 + p] = __fmul_rn(dot, scale);
  }
}

// Softmax and the weighted sum of values for one row, one query head and a
// slice of kPVSlice output dimensions (llama.c:566-575), as k_attn_pv.
// Grid (ceil(hd / 32), n_heads, rows); (smax + kPVRing*kPVChunk*kPVSlice)
// floats of dynamic shared memory.
__global__ void __launch_bounds__(kPVThreads) k_rows_pv(const RowAttnArgs a) {
  extern __shared__ __align__(16) float sm_v[];
  __shared__ float s_red[32];
  __shared__ float s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, h = blockIdx.y, r = blockIdx.z;
  const RowDesc d = a.rd[r];
  if (d.pos < 0 || d.pos >= d.max_seq) return;
  const int d0 = blockIdx.x * kPVSlice;
  const int np = d.pos + 1, hd = a.hd, group = a.n_heads / a.n_kv, kvh = h / group;
  const int w = min(kPVSlice, hd - d0);
  float *wts = sm_v;                                           // [smax]
  float *ring = sm_v + (((size_t)a.smax + 3) & ~size_t(3));  // [kPVRing][kPVChunk][kPVSlice]
  const float *vc = d.v + row_cache_offset(d, a.layer, a.n_kv, kvh, hd);
  const int nchunks = (np + kPVChunk - 1) / kPVChunk;
  for (int c = 0; c < kPVRing; ++c) {
    if (c < nchunks)
      stage_rows(ring + (size_t)c * kPVChunk * kPVSlice, kPVSlice, vc, hd, c * kPVChunk,
                 min((c + 1) * kPVChunk, np), d0, w, tid, kPVThreads);
    cp_async_commit();
  }
  const float *sc = a.scores + ((size_t)r * a.n_heads + h) * a.smax;
  float m = -INFINITY;
  for (int p = tid; p < np; p += kPVThreads) {
    const float s = sc[p];
    wts[p] = s;
    m = fmaxf(m, s);
  }
  m = block_max<kPVThreads>(m, s_red);
  for (int p = tid; p < np; p += kPVThreads) wts[p] = libm_expf(__fsub_rn(wts[p], m));
  __syncthreads();
  if (tid == 0) {
    const float sum = seq_sum(wts, 1, np, 0.0f);  // llama.c:567
    s_inv = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  const float inv = s_inv;
  for (int p = tid; p < np; p += kPVThreads) wts[p] = __fmul_rn(wts[p], inv);
  float o = 0.0f;
  for (int c = 0; c < nchunks; ++c) {
    cp_async_wait<kPVRing - 1>();
    __syncthreads();
    const float *buf = ring + (size_t)(c % kPVRing) * kPVChunk * kPVSlice;
    const int pe = min((c + 1) * kPVChunk, np) - c * kPVChunk;
    if (tid < w) o = seq_dot(wts + (size_t)c * kPVChunk, buf + tid, kPVSlice, pe, o);  // llama.c:574
    __syncthreads();
    const int nc = c + kPVRing;
    if (nc < nchunks)
      stage_rows(ring + (size_t)(nc % kPVRing) * kPVChunk * kPVSlice, kPVSlice, vc, hd, nc * kPVChunk,
                 min((nc + 1) * kPVChunk, np), d0, w, tid, kPVThreads);
    cp_async_commit();
  }
  if (tid < w) a.out[(size_t)r * a.n_heads * hd + (size_t)h * hd + d0 + tid] = o;
}

// Greedy ids of the rows (first maximum: sampler.c:8-21) from the lm-head
// epilogue's keys; the key cells are re-zeroed for the next pass.
__global__ void k_rows_finish(unsigned long long *argmax, int rows, int *ids) {
  pdl_wait();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const unsigned long long key = argmax[r];
    ids[r] = static_cast<int>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
    argmax[r] = 0ull;
  }
}

}  // namespace llmq
