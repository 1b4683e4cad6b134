// llmq_f32.cuh - the fp32 (LLMA) decode path's matrix-vector products
// (llama.c:296-362 over matrix.c:178-199).
//
// The reference's matmul forms every output column as one sequential chain,
// C[j] = ((0 + a_0 w_0j) + a_1 w_1j) + ..., each product and each sum rounded
// on its own (no contraction under -std=c11).  The chain of a column cannot be
// split, so the parallelism is across columns: one thread per column, whole K.
// Columns are grouped in units of 8; CTA c owns a contiguous range of units
// and its weights are stored as its own region, row k holding the 8 floats of
// each of its units in turn.  Row blocks of a region are contiguous, so the
// region streams through a shared-memory ring in 1-D bulk copies, and the
// threads of a warp read 32 consecutive floats of a row (conflict-free) while
// the input row is a broadcast.  The fused prologues and epilogues are the
// int8 path's: RMSNorm (+ embedding row), SiLU(g)*u for the down projection,
// bias and q/k/v routing, residual add, logits with the first-maximum argmax.
#pragma once

#include "llmq_kernels.cuh"

namespace llmq {

constexpr int kF32Unit = 8;             // output columns per unit
constexpr int kF32MaxThreads = 1024;    // one thread per column of a CTA's range
constexpr int kF32MaxStages = 12;

enum F32Pro : int {
  F32_PRO_PLAIN = 0,          // the input row as it is (Wo)
  F32_PRO_RMSNORM = 1,        // RMSNorm(in, gamma) (QKV, W1|W3, lm-head)
  F32_PRO_EMBED_RMSNORM = 2,  // x = wte row of step->token, then RMSNorm (first QKV)
  F32_PRO_SWIGLU = 3          // h_j = SiLU(g_j) * u_j from in = [g | u] (W2)
};
enum F32Epi : int {
  F32_EPI_PLAIN = 0,   // out[j] = y (W1|W3: g and u)
  F32_EPI_QKV = 1,     // + bias; q and k to out, v appended to the cache
  F32_EPI_RESID = 2,   // out[j] += y (Wo, W2)
  F32_EPI_LOGITS = 3   // logits + device argmax
};

struct F32Args {
  const float *w;           // tiled regions (see the file comment)
  const long long *cta_off; // [G + 1]: float offset of CTA c's region
  const int *cta_u0;        // [G + 1]: first unit of CTA c
  int K, N;
  int KC;                   // rows per ring stage
  int stages;
  int stage_floats;         // ring slot size: KC * (most units of a CTA) * 8
  int *err;
  // prologue
  const float *in;
  const float *gamma;
  float eps;
  const StepState *step;
  const float *wte;         // F32_PRO_EMBED_RMSNORM: [vocab][K]
  int vocab;
  float *x_out;             // F32_PRO_EMBED_RMSNORM: receives the embedding row
  int dff;                  // F32_PRO_SWIGLU: in holds g[dff] then u[dff]
  // epilogue
  float *out;
  const float *bias;
  int qd, kvd, hd, max_seq;
  float *vcache;
  unsigned long long *argmax;
  int idx_offset;
};

template <int PRO, int EPI>
__global__ void __launch_bounds__(kF32MaxThreads, 1) k_gemv_f32(const F32Args a) {
  extern __shared__ __align__(128) uint8_t sm_f32[];
  __shared__ uint64_t s_bar[2 * kF32MaxStages];  // full[S], then empty[S]
  __shared__ float s_red[32];
  __shared__ unsigned long long s_red64[32];
  __shared__ float s_r;
  __shared__ int s_abort;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nwarps = nthr >> 5;
  const int S = a.stages;
  float *ring = reinterpret_cast<float *>(sm_f32);
  float *xs = ring + (size_t)S * a.stage_floats;  // the input row [K]
  uint64_t *full = s_bar, *empty = s_bar + kF32MaxStages;
  const int u0 = a.cta_u0[blockIdx.x];
  const int nc8 = (a.cta_u0[blockIdx.x + 1] - u0) * kF32Unit;  // floats per row of this region
  const float *region = a.w + a.cta_off[blockIdx.x];
  const int n_st = (a.K + a.KC - 1) / a.KC;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], nwarps);
    }
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  auto issue = [&](int i) {  // thread 0: rows [i*KC, i*KC + KC) of the region into slot i % S
    const int rows = min(a.KC, a.K - i * a.KC);
    const uint32_t bytes = static_cast<uint32_t>(rows * nc8 * 4);
    uint64_t *bar = &full[i % S];
    mbar_expect_tx(bar, bytes);
    bulk_load(ring + (size_t)(i % S) * a.stage_floats, region + (size_t)i * a.KC * nc8, bytes, bar);
  };
  // the weights never depend on the previous kernel: fill the ring now
  int issued = 0, done = 0;  // stages copied / consumed (thread 0's count)
  if (tid == 0 && nc8 > 0)
    for (; issued < S && issued < n_st; ++issued) issue(issued);
  pdl_launch_dependents();
  pdl_wait();

  // ------------------------------------------------------------ prologue
  const int K = a.K;
  if (PRO == F32_PRO_PLAIN) {
    for (int k = tid; k < K; k += nthr) xs[k] = a.in[k];
  } else if (PRO == F32_PRO_SWIGLU) {
    for (int k = tid; k < K; k += nthr) {  // swiglu.c:9-12, 36-41 (llama.c:357)
      const float z = a.in[k];
      const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, libm_expf(-z)));
      xs[k] = __fmul_rn(__fmul_rn(z, s), a.in[a.dff + k]);
    }
  } else {
    if (PRO == F32_PRO_EMBED_RMSNORM) {  // llama.c:302-303
      int token = a.step->token;
      if (token < 0 || token >= a.vocab) {
        if (tid == 0 && blockIdx.x == 0) atomicOr(a.err, ERR_BAD_TOKEN);
        token = 0;
      }
      const float *row = a.wte + (size_t)token * K;
      for (int k = tid; k < K; k += nthr) {
        const float v = row[k];
        xs[k] = v;
        if (blockIdx.x == 0) a.x_out[k] = v;
      }
    } else {
      for (int k = tid; k < K; k += nthr) xs[k] = a.in[k];
    }
    // rmsnorm.c:14-19: the sum of squares is one sequential chain
    float *sq = xs + ((K + 3) & ~3);
    for (int k = tid; k < K; k += nthr) sq[k] = __fmul_rn(xs[k], xs[k]);
    __syncthreads();
    if (tid == 0) {
      float ms = seq_sum(sq, 1, K, 0.0f);
      ms = __fmul_rn(ms, __fdiv_rn(1.0f, static_cast<float>(K)));
      s_r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
    }
    __syncthreads();
    const float r = s_r;
    for (int k = tid; k < K; k += nthr) xs[k] = __fmul_rn(__fmul_rn(xs[k], r), a.gamma[k]);
  }
  __syncthreads();

  // --------------------------------------------------------------- chains
  const bool active = tid < nc8;
  float acc = 0.0f;  // matrix.c:183
  for (int i = 0; i < n_st && nc8 > 0; ++i) {
    const int slot = i % S;
    if (!mbar_wait_bounded(&full[slot], static_cast<uint32_t>((i / S) & 1))) {
      if (tid == 0) atomicOr(a.err, ERR_TIMEOUT);
      s_abort = 1;
    }
    if (*reinterpret_cast<volatile int *>(&s_abort)) break;
    const int rows = min(a.KC, K - i * a.KC);
    if (active) {
      const float *t = ring + (size_t)slot * a.stage_floats + tid;
      const float *xk = xs + i * a.KC;
      int kk = 0;
      for (; kk + 4 <= rows; kk += 4) {  // matrix.c:185-188, in k order
        const float w0 = t[(kk + 0) * nc8], w1 = t[(kk + 1) * nc8], w2 = t[(kk + 2) * nc8], w3 = t[(kk + 3) * nc8];
        acc = __fadd_rn(acc, __fmul_rn(xk[kk + 0], w0));
        acc = __fadd_rn(acc, __fmul_rn(xk[kk + 1], w1));
        acc = __fadd_rn(acc, __fmul_rn(xk[kk + 2], w2));
        acc = __fadd_rn(acc, __fmul_rn(xk[kk + 3], w3));
      }
      for (; kk < rows; ++kk) acc = __fadd_rn(acc, __fmul_rn(xk[kk], t[kk * nc8]));
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    done = i + 1;
    // refill the slot of the previous stage, which every warp has most likely left
    if (tid == 0 && i >= 1 && issued < n_st) {
      const int ps = (i - 1) % S;
      if (!mbar_wait_bounded(&empty[ps], static_cast<uint32_t>(((i - 1) / S) & 1))) {
        atomicOr(a.err, ERR_TIMEOUT);
        s_abort = 1;
      } else {
        issue(issued++);
      }
    }
  }
  // after a failed wait, the copies still in flight must land before the CTA leaves
  if (tid == 0 && *reinterpret_cast<volatile int *>(&s_abort)) {
    for (int i = done; i < issued; ++i) mbar_wait_bounded(&full[i % S], static_cast<uint32_t>((i / S) & 1));
  }
  __syncthreads();
  if (s_abort) return;

  // ------------------------------------------------------------- epilogue
  const int j = u0 * kF32Unit + tid;
  const bool has = active && j < a.N;
  if (EPI == F32_EPI_PLAIN) {
    if (has) a.out[j] = acc;
  } else if (EPI == F32_EPI_RESID) {
    if (has) a.out[j] = __fadd_rn(a.out[j], acc);  // llama.c:343 / 348
  } else if (EPI == F32_EPI_QKV) {
    const int pos = a.step->pos;
    const bool pos_ok = pos >= 0 && pos < a.max_seq;
    if (!pos_ok && tid == 0) atomicOr(a.err, ERR_BAD_POS);
    if (has && pos_ok) {
      const float y = __fadd_rn(acc, a.bias[j]);  // llama.c:316-318
      if (j < a.qd + a.kvd) {
        a.out[j] = y;
      } else {
        const int jv = j - a.qd - a.kvd, vh = jv / a.hd;
        a.vcache[((size_t)vh * a.max_seq + pos) * a.hd + (jv - vh * a.hd)] = y;  // llama.c:322
      }
    }
  } else if (EPI == F32_EPI_LOGITS) {
    unsigned long long key = 0ull;
    if (has) {
      a.out[j] = acc;
      key = argmax_key(acc, static_cast<uint32_t>(j + a.idx_offset));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long w = __shfl_xor_sync(0xffffffffu, key, o);
      key = w > key ? w : key;
    }
    if (lane == 0) s_red64[warp] = key;
    __syncthreads();
    if (tid == 0) {
      unsigned long long best = 0ull;
      for (int w = 0; w < nwarps; ++w) best = s_red64[w] > best ? s_red64[w] : best;
      atomicMax(a.argmax, best);
    }
  }
  (void)s_red;
}

}  // namespace llmq
