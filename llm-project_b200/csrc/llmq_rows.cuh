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
// prologue), then its activation codes (quant.c:69-78).  One CTA per row;
// dynamic shared memory 2 * K floats and spec_sum_bytes().
__global__ void __launch_bounds__(kRowThreads) k_rows_norm_codes(const RowNormArgs a) {
  LLMQ_LAUNCH_SPAN(10);
  extern __shared__ __align__(16) float xs[];
  __shared__ float s_red[32];
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
  float ms = spec_seq_sum(sq, K, 0.0f, sq + ((K + 3) & ~3));  // rmsnorm.c:15, in index order
  ms = __fmul_rn(ms, __fdiv_rn(1.0f, static_cast<float>(K)));
  const float rr = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
  float m = 0.0f;
  for (int k = tid; k < K; k += kRowThreads) {
    const float y = __fmul_rn(__fmul_rn(xs[k], rr), a.gamma[k]);
    xs[k] = y;
    m = fmaxf(m, fabsf(y));
  }
  m = block_max<kRowThreads>(m, s_red);
  __syncthreads();
  const float as = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;  // quant.c:71
  const float inv = __fdiv_rn(1.0f, as);                      // quant.c:72
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
  int layer, n_heads, n_kv, hd, smax;  // smax: the model's max_seq (score row stride)
  int *err;
};

__device__ __forceinline__ size_t row_cache_offset(const RowDesc &d, int layer, int n_kv, int kvh, int hd) {
  return (((size_t)layer * n_kv + kvh) * d.max_seq) * hd;
}

// RoPE of q and k (rope.c:48-68) at the row's position; the rotated k and the
// v of the row are appended to its cache (llama.c:551-552).  One CTA per row.
__global__ void __launch_bounds__(256) k_rows_append(const RowAttnArgs a) {
  LLMQ_LAUNCH_SPAN(11);
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
// sequential dot product over the head dimension, times 1/sqrt(hd).  The keys
// are staged in rows padded to hd + 4 floats, so the 16-byte loads of the 8
// threads of a load phase (8 consecutive keys) hit distinct banks.
// Grid (ceil(smax / 64), n_kv, rows), 256 threads; head_dim % 4 == 0.
constexpr int kRowScoreKeys = 64;
constexpr int kRowScoreThreads = 256;
__host__ __device__ inline size_t rows_scores_smem(int group, int hd) {
  return ((size_t)group * hd + (size_t)kRowScoreKeys * (hd + 4)) * sizeof(float);
}
__global__ void __launch_bounds__(kRowScoreThreads) k_rows_scores(const RowAttnArgs a) {
  LLMQ_LAUNCH_SPAN(12);
  extern __shared__ __align__(16) float sm_s[];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, kvh = blockIdx.y, r = blockIdx.z;
  const RowDesc d = a.rd[r];
  const int p0 = blockIdx.x * kRowScoreKeys;
  if (d.pos < 0 || d.pos >= d.max_seq || p0 > d.pos) return;
  const int hd = a.hd, group = a.n_heads / a.n_kv, qd = a.n_heads * hd, ks = hd + 4;
  float *qs = sm_s;                        // [group][hd]
  float *kst = sm_s + (size_t)group * hd;  // [64][hd + 4]
  const int p1 = min(p0 + kRowScoreKeys, d.pos + 1);
  stage_rows(kst, ks, d.k + row_cache_offset(d, a.layer, a.n_kv, kvh, hd), hd, p0, p1, 0, hd, tid,
             kRowScoreThreads);
  cp_async_commit();
  const float4 *q4 = reinterpret_cast<const float4 *>(a.qr + (size_t)r * qd + (size_t)kvh * group * hd);
  for (int i = tid; i < group * hd / 4; i += kRowScoreThreads) reinterpret_cast<float4 *>(qs)[i] = q4[i];
  cp_async_wait<0>();
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));  // llama.c:532
  float *srow = a.scores + ((size_t)r * a.n_heads + (size_t)kvh * group) * a.smax;
  for (int t = tid; t < group * kRowScoreKeys; t += kRowScoreThreads) {
    const int g = t / kRowScoreKeys, p = t - g * kRowScoreKeys;
    if (p0 + p >= p1) continue;
    const float dot = seq_dot_v4(qs + (size_t)g * hd, kst + (size_t)p * ks, hd, 0.0f);  // llama.c:561
    srow[(size_t)g * a.smax + p0 + p] = __fmul_rn(dot, scale);
  }
}

// Scores of a prefill pass (every row one position of the same sequence and
// cache): a CTA takes a block of consecutive rows, one KV head and 64 key
// positions, so each key chunk is staged once for the block's whole query
// group instead of once per row.  64 query vectors (rows x the group's heads)
// times 64 keys; thread (i, j) forms the 4 x 4 scores of query vectors
// 4 i .. 4 i + 3 and keys 4 j .. 4 j + 3, each the sequential dot product over
// the head dimension in index order (llama.c:561), times 1/sqrt(hd); keys past
// a row's position are skipped (llama.c:558).  q and k are staged transposed
// ([hd][64]) so every step is two 16-byte shared loads.  Grid
// (ceil(smax / 64), n_kv, row blocks of pf_rows_per_block(group) rows); 256
// threads; head_dim % 4 == 0.
constexpr int kPfVecs = 64;  // query vectors and keys per CTA
__host__ __device__ inline int pf_rows_per_block(int group) { return kPfVecs / group; }
__host__ __device__ inline size_t pf_scores_smem(int hd) { return (size_t)2 * hd * kPfVecs * sizeof(float); }
__global__ void __launch_bounds__(256) k_pf_scores(const RowAttnArgs a, int rows) {
  LLMQ_LAUNCH_SPAN(15);
  extern __shared__ __align__(16) float sm_p[];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, kvh = blockIdx.y;
  const int hd = a.hd, group = a.n_heads / a.n_kv, qd = a.n_heads * hd;
  const int rpb = pf_rows_per_block(group), r0 = blockIdx.z * rpb, r1 = min(r0 + rpb, rows);
  const int k0 = blockIdx.x * kPfVecs;
  const RowDesc d0 = a.rd[r0];
  const int pos_hi = a.rd[r1 - 1].pos;  // rows are consecutive positions
  if (d0.pos < 0 || pos_hi >= d0.max_seq || k0 > pos_hi) return;  // bad positions: flagged by k_rows_append
  float *qT = sm_p;                          // [hd][64]
  float *kT = sm_p + (size_t)hd * kPfVecs;   // [hd][64]
  const int nv = (r1 - r0) * group;          // query vectors in use
  const int hd4 = hd / 4;
  // consecutive threads take consecutive vectors: conflict-free transposed stores
  for (int t = tid; t < kPfVecs * hd4; t += 256) {
    const int v = t & (kPfVecs - 1), e = 4 * (t / kPfVecs);
    float4 q = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (v < nv) {
      const int r = r0 + v / group, g = v - (v / group) * group;
      q = *reinterpret_cast<const float4 *>(a.qr + (size_t)r * qd + (size_t)(kvh * group + g) * hd + e);
    }
    qT[(size_t)(e + 0) * kPfVecs + v] = q.x;
    qT[(size_t)(e + 1) * kPfVecs + v] = q.y;
    qT[(size_t)(e + 2) * kPfVecs + v] = q.z;
    qT[(size_t)(e + 3) * kPfVecs + v] = q.w;
  }
  const float *kc = d0.k + row_cache_offset(d0, a.layer, a.n_kv, kvh, hd);
  for (int t = tid; t < kPfVecs * hd4; t += 256) {
    const int j = t & (kPfVecs - 1), e = 4 * (t / kPfVecs);
    float4 k = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (k0 + j <= pos_hi) k = *reinterpret_cast<const float4 *>(kc + (size_t)(k0 + j) * hd + e);
    kT[(size_t)(e + 0) * kPfVecs + j] = k.x;
    kT[(size_t)(e + 1) * kPfVecs + j] = k.y;
    kT[(size_t)(e + 2) * kPfVecs + j] = k.z;
    kT[(size_t)(e + 3) * kPfVecs + j] = k.w;
  }
  __syncthreads();
  const int ti = tid >> 4, tj = tid & 15;
  float2 acc[4][2];  // query vector i, key pairs (4 tj, 4 tj + 1) and (4 tj + 2, 4 tj + 3)
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i][0] = acc[i][1] = make_float2(0.0f, 0.0f);
  const float4 *q4 = reinterpret_cast<const float4 *>(qT) + ti;
  const float4 *k4 = reinterpret_cast<const float4 *>(kT) + tj;
#pragma unroll 4
  for (int e = 0; e < hd; ++e) {
    const float4 qv = q4[(size_t)e * (kPfVecs / 4)], kv = k4[(size_t)e * (kPfVecs / 4)];
    const float qa[4] = {qv.x, qv.y, qv.z, qv.w};
    const float2 k01 = make_float2(kv.x, kv.y), k23 = make_float2(kv.z, kv.w);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 q2 = make_float2(qa[i], qa[i]);
      acc[i][0] = f2_madd_rn(acc[i][0], q2, k01);  // llama.c:561
      acc[i][1] = f2_madd_rn(acc[i][1], q2, k23);
    }
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));  // llama.c:532
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = 4 * ti + i;
    if (v >= nv) continue;
    const int r = r0 + v / group, g = v - (v / group) * group;
    const int pos = a.rd[r].pos;
    float *srow = a.scores + ((size_t)r * a.n_heads + (size_t)kvh * group + g) * a.smax;
    const float dots[4] = {acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int p = k0 + 4 * tj + j;
      if (p <= pos) srow[p] = __fmul_rn(dots[j], scale);
    }
  }
}

// Softmax and values of one row for one KV head and its whole query group
// (llama.c:566-575), in one CTA of group * hd / 2 threads (rounded up to a warp):
// the group's scores come into shared memory; per head the max, expf(s - max),
// the sequential sum of the exponentials (one thread per head) and
// w = e * (1/sum); then the values [0, pos] stream through a ring
// (kPvStages stages of kPvKeys positions, one bulk copy each) and thread (g, e2)
// forms out[g][e] = sum_p w[g][p] * v[p][e] for e = 2 e2, 2 e2 + 1, each
// sequentially in position order (two chains in packed f32x2 lanes).
// Each value row is read once for the whole group.  Grid (n_kv, rows); dynamic
// shared memory rows_pv_smem().
constexpr int kPvKeys = 64;
constexpr int kPvStages = 2;
constexpr int kAttnMaxGroup = 16;
__host__ __device__ inline size_t rows_pv_smem(int group, int hd, int smax) {
  return ((size_t)kPvStages * kPvKeys * hd + (size_t)group * ((smax + 3) & ~3)) * sizeof(float);
}

__global__ void __launch_bounds__(1024) k_rows_pv(const RowAttnArgs a) {
  LLMQ_LAUNCH_SPAN(13);
  extern __shared__ __align__(16) float sm_a[];
  __shared__ __align__(8) uint64_t full[kPvStages];
  __shared__ float s_max[kAttnMaxGroup][32];
  __shared__ float s_inv[kAttnMaxGroup];
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x;
  const int kvh = blockIdx.x, r = blockIdx.y;
  const int hd = a.hd, group = a.n_heads / a.n_kv, qd = a.n_heads * hd, smax4 = (a.smax + 3) & ~3;
  float *ring = sm_a;                                     // [S][kPvKeys][hd]
  float *wts = ring + (size_t)kPvStages * kPvKeys * hd;  // [group][smax4]
  if (tid == 0) {
    for (int i = 0; i < kPvStages; ++i) mbar_init(&full[i], 1);
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  const RowDesc d = a.rd[r];  // written by the host before the pass: no wait needed
  if (d.pos < 0 || d.pos >= d.max_seq) return;  // flagged by k_rows_append
  const int np = d.pos + 1, nch = (np + kPvKeys - 1) / kPvKeys;
  const float *vc = d.v + row_cache_offset(d, a.layer, a.n_kv, kvh, hd);
  const uint32_t row_bytes = (uint32_t)hd * 4u;
  auto issue = [&](int c) {  // thread 0
    const int st = c % kPvStages, c0 = c * kPvKeys, cnt = min(kPvKeys, np - c0);
    mbar_expect_tx(&full[st], (uint32_t)cnt * row_bytes);
    bulk_load(ring + (size_t)st * kPvKeys * hd, vc + (size_t)c0 * hd, (uint32_t)cnt * row_bytes, &full[st]);
  };
  pdl_launch_dependents();
  pdl_wait();  // the values of this step's rows and the scores come from the previous kernels
  int issued = 0;
  if (tid == 0)
    for (; issued < kPvStages && issued < nch; ++issued) issue(issued);
  // ---- softmax per head (llama.c:566-572)
  const float *sc = a.scores + ((size_t)r * a.n_heads + (size_t)kvh * group) * a.smax;
  float mloc[kAttnMaxGroup];
  for (int g = 0; g < group; ++g) {
    float m = -INFINITY;
    for (int p = tid; p < np; p += nthr) {
      const float v = sc[(size_t)g * a.smax + p];
      wts[(size_t)g * smax4 + p] = v;
      m = fmaxf(m, v);
    }
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    mloc[g] = m;
  }
  if (lane == 0)
    for (int g = 0; g < group; ++g) s_max[g][warp] = mloc[g];
  __syncthreads();
  if (tid < group) {
    float m = -INFINITY;
    for (int w = 0; w < (nthr + 31) / 32; ++w) m = fmaxf(m, s_max[tid][w]);
    s_max[tid][0] = m;
  }
  __syncthreads();
  for (int t = tid; t < group * np; t += nthr) {
    const int g = t / np, p = t - g * np;
    float *e = wts + (size_t)g * smax4 + p;
    *e = libm_expf(__fsub_rn(*e, s_max[g][0]));
  }
  __syncthreads();
  if (tid < group) s_inv[tid] = __fdiv_rn(1.0f, seq_sum(wts + (size_t)tid * smax4, 1, np, 0.0f));  // llama.c:567
  __syncthreads();
  for (int t = tid; t < group * np; t += nthr) {
    const int g = t / np, p = t - g * np;
    wts[(size_t)g * smax4 + p] = __fmul_rn(wts[(size_t)g * smax4 + p], s_inv[g]);
  }
  __syncthreads();
  // ---- weighted sum of the values (llama.c:573-575): thread (g, e2) carries
  // dims 2 e2 and 2 e2 + 1 as two chains in packed lanes
  const int hd2 = hd / 2;
  const int g = tid / hd2, e = 2 * (tid - g * hd2);
  const float *wg = wts + (size_t)min(g, group - 1) * smax4;
  float2 o = make_float2(0.0f, 0.0f);
  int c = 0;
  for (; c < nch; ++c) {
    const int st = c % kPvStages;
    const bool got = mbar_wait_bounded(&full[st], (uint32_t)(c / kPvStages) & 1u);
    if (!got) s_abort = 1;
    const float *buf = ring + (size_t)st * kPvKeys * hd + e;
    const int c0 = c * kPvKeys, cnt = min(kPvKeys, np - c0);
    if (g < group && got)
      o = seq_dot2<false>(wg + c0, 0.0f, reinterpret_cast<const float2 *>(buf), hd2, cnt, o);  // llama.c:574
    __syncthreads();
    if (s_abort) break;  // chunk c stays counted as outstanding
    if (tid == 0 && issued < nch) issue(issued++);
  }
  if (s_abort) {
    if (tid == 0) {
      atomicOr(a.err, ERR_TIMEOUT);
      for (int t = c; t < issued; ++t) mbar_wait_bounded(&full[t % kPvStages], (uint32_t)(t / kPvStages) & 1u);
    }
    return;
  }
  if (g < group) *reinterpret_cast<float2 *>(a.out + (size_t)r * qd + (size_t)(kvh * group + g) * hd + e) = o;
}

// Softmax of one prefill row and one KV head's query group (llama.c:566-572)
// in place: for each of the group's heads the scores [0, pos] become
// w = expf(s - max) * (1 / sum), the sum of the exponentials taken
// sequentially in position order (one thread per head, the group's sums side
// by side).  Grid (rows, n_kv), 256 threads, dynamic shared memory
// group * smax4 floats.
__global__ void __launch_bounds__(256) k_pf_softmax(const RowAttnArgs a) {
  LLMQ_LAUNCH_SPAN(16);
  extern __shared__ __align__(16) float ex[];
  __shared__ float s_max[kAttnMaxGroup][8];
  __shared__ float s_inv[kAttnMaxGroup];
  pdl_launch_dependents();
  pdl_wait();
  const int r = blockIdx.x, kvh = blockIdx.y, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const RowDesc d = a.rd[r];
  if (d.pos < 0 || d.pos >= d.max_seq) return;  // flagged by k_rows_append
  const int np = d.pos + 1, group = a.n_heads / a.n_kv, smax4 = (a.smax + 3) & ~3;
  float *sc = a.scores + ((size_t)r * a.n_heads + (size_t)kvh * group) * a.smax;
  for (int g = 0; g < group; ++g) {
    float m = -INFINITY;
    for (int p = tid; p < np; p += 256) {
      const float v = sc[(size_t)g * a.smax + p];
      ex[(size_t)g * smax4 + p] = v;
      m = fmaxf(m, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) s_max[g][warp] = m;
  }
  __syncthreads();
  if (tid < group) {
    float m = s_max[tid][0];
    for (int w = 1; w < 8; ++w) m = fmaxf(m, s_max[tid][w]);
    s_max[tid][0] = m;
  }
  __syncthreads();
  for (int t = tid; t < group * np; t += 256) {
    const int g = t / np, p = t - g * np;
    float *e = ex + (size_t)g * smax4 + p;
    *e = libm_expf(__fsub_rn(*e, s_max[g][0]));  // llama.c:566
  }
  __syncthreads();
  if (tid < group) s_inv[tid] = __fdiv_rn(1.0f, seq_sum_a16(ex + (size_t)tid * smax4, np, 0.0f));  // llama.c:567
  __syncthreads();
  for (int t = tid; t < group * np; t += 256) {
    const int g = t / np, p = t - g * np;
    sc[(size_t)g * a.smax + p] = __fmul_rn(ex[(size_t)g * smax4 + p], s_inv[g]);  // llama.c:571
  }
}

// Weighted values of a prefill pass (llama.c:573-575): a CTA takes a block of
// consecutive rows and one KV head, and streams the head's value rows
// [0, last row's position] once through a two-chunk ring for the block's whole
// query group (64 query vectors).  Thread (i, j) carries query vectors
// 4 i .. 4 i + 3 and dims {4 j .. 4 j + 3, 64 + 4 j .. 64 + 4 j + 3}: 32
// chains, each out[v][d] = sum of w[v][p] * v[p][d] over p = 0 .. pos(v) in
// position order, every product rounded on its own.  The weights come from
// k_pf_softmax.  Grid (n_kv, row blocks of pf_rows_per_block(group) rows); 256
// threads; head_dim 128; dynamic shared memory pf_pv_smem(hd).
constexpr int kPfKeys = 32;
__host__ __device__ inline size_t pf_pv_smem(int hd) {
  return (size_t)2 * kPfKeys * (hd + kPfVecs) * sizeof(float);
}
__global__ void __launch_bounds__(256) k_pf_pv(const RowAttnArgs a, int rows) {
  LLMQ_LAUNCH_SPAN(17);
  extern __shared__ __align__(16) float sm_pv[];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x, kvh = blockIdx.x;
  const int hd = a.hd, group = a.n_heads / a.n_kv, qd = a.n_heads * hd;
  const int rpb = pf_rows_per_block(group), r0 = blockIdx.y * rpb, r1 = min(r0 + rpb, rows);
  const RowDesc d0 = a.rd[r0];
  const int pos_hi = a.rd[r1 - 1].pos;
  if (d0.pos < 0 || pos_hi >= d0.max_seq) return;  // flagged by k_rows_append
  const int nv = (r1 - r0) * group;
  float *Vs = sm_pv;                               // [2][kPfKeys][hd]
  float *Ws = sm_pv + (size_t)2 * kPfKeys * hd;    // [2][kPfKeys][64]
  const float *vc = d0.v + row_cache_offset(d0, a.layer, a.n_kv, kvh, hd);
  const int nch = (pos_hi + kPfKeys) / kPfKeys;
  auto stage = [&](int c) {
    const int b = c & 1, p0 = c * kPfKeys, rows_in = min(kPfKeys, pos_hi + 1 - p0);
    stage_rows(Vs + (size_t)b * kPfKeys * hd, hd, vc, hd, p0, p0 + rows_in, 0, hd, tid, 256);
    cp_async_commit();
    float *w = Ws + (size_t)b * kPfKeys * kPfVecs;
    for (int t = tid; t < kPfVecs * kPfKeys; t += 256) {
      const int v = t / kPfKeys, j = t - v * kPfKeys, p = p0 + j;
      float x = 0.0f;
      if (v < nv) {
        const int r = r0 + v / group, g = v - (v / group) * group;
        if (p <= a.rd[r].pos) x = a.scores[((size_t)r * a.n_heads + (size_t)kvh * group + g) * a.smax + p];
      }
      w[(size_t)j * kPfVecs + v] = x;
    }
  };
  const int ti = tid >> 4, tj = tid & 15;
  int lim[4];  // the last position each of the thread's vectors adds
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = 4 * ti + i;
    lim[i] = v < nv ? a.rd[r0 + v / group].pos : -1;
  }
  float2 acc[4][4];  // dims pairs (4 tj, 4 tj + 1), (4 tj + 2, + 3), (64 + 4 tj, ..), (64 + 4 tj + 2, ..)
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[i][k] = make_float2(0.0f, 0.0f);
  const int lim_lo = min(min(lim[0], lim[1]), min(lim[2], lim[3]));
  stage(0);
  for (int c = 0; c < nch; ++c) {
    if (c + 1 < nch) {
      stage(c + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const int b = c & 1, p0 = c * kPfKeys, cnt = min(kPfKeys, pos_hi + 1 - p0);
    const float *vb = Vs + (size_t)b * kPfKeys * hd;
    const float *wb = Ws + (size_t)b * kPfKeys * kPfVecs;
    // keys every vector of the thread adds, then the ones past some vector's position
    const int full = max(0, min(cnt, lim_lo - p0 + 1));
    auto step = [&](int j, bool masked) {
      const float4 w4 = reinterpret_cast<const float4 *>(wb + (size_t)j * kPfVecs)[ti];
      const float4 va = reinterpret_cast<const float4 *>(vb + (size_t)j * hd)[tj];
      const float4 vb4 = reinterpret_cast<const float4 *>(vb + (size_t)j * hd + 64)[tj];
      const float wv[4] = {w4.x, w4.y, w4.z, w4.w};
      const float2 vv[4] = {make_float2(va.x, va.y), make_float2(va.z, va.w), make_float2(vb4.x, vb4.y),
                            make_float2(vb4.z, vb4.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (masked && p0 + j > lim[i]) continue;
        const float2 w2 = make_float2(wv[i], wv[i]);
#pragma unroll
        for (int k = 0; k < 4; ++k) acc[i][k] = f2_madd_rn(acc[i][k], w2, vv[k]);  // llama.c:574
      }
    };
    for (int j = 0; j < full; ++j) step(j, false);
    for (int j = full; j < cnt; ++j) step(j, true);
    __syncthreads();  // the buffer is free for chunk c + 2
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int v = 4 * ti + i;
    if (v >= nv) continue;
    const int r = r0 + v / group, g = v - (v / group) * group;
    float *o = a.out + (size_t)r * qd + (size_t)(kvh * group + g) * hd;
    *reinterpret_cast<float4 *>(o + 4 * tj) = make_float4(acc[i][0].x, acc[i][0].y, acc[i][1].x, acc[i][1].y);
    *reinterpret_cast<float4 *>(o + 64 + 4 * tj) = make_float4(acc[i][2].x, acc[i][2].y, acc[i][3].x, acc[i][3].y);
  }
}

// Greedy ids of the rows (first maximum: sampler.c:8-21) from the lm-head
// epilogue's keys; the key cells are re-zeroed for the next pass.
__global__ void k_rows_finish(unsigned long long *argmax, int rows, int *ids) {
  LLMQ_LAUNCH_SPAN(14);
  pdl_wait();
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    const unsigned long long key = argmax[r];
    ids[r] = static_cast<int>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffull));
    argmax[r] = 0ull;
  }
}

}  // namespace llmq
