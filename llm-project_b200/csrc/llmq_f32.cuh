// llmq_f32.cuh - the fp32 (LLMA) decode path's matrix-vector products
// (llama.c:296-362 over matrix.c:178-199).
//
// The reference's matmul forms every output column as one sequential chain,
// C[j] = ((0 + a_0 w_0j) + a_1 w_1j) + ..., each product and each sum rounded
// on its own (no contraction under -std=c11).  The chain of a column cannot be
// split, so the parallelism is across columns: one lane per column, whole K.
//
// Columns are grouped in tiles of 32, one per warp.  A tile is stored as its
// own contiguous [K][32] block, and each warp streams its tile through a
// private shared-memory ring of bulk copies: lane 0 refills a slot right after
// the warp has read it, so no warp ever waits for another.  CTA c owns a
// contiguous range of tiles (one warp each), so the weights stream from all
// SMs.  The input row is staged once per CTA and read as a broadcast.
//
// Fused around the products, as on the int8 path: RMSNorm (+ embedding row)
// before, and bias with q/k/v routing, residual add, SiLU(g)*u (gate and up
// columns interleaved in fours, so a shuffle pairs them), or logits with the
// first-maximum argmax after.
#pragma once

#include "llmq_kernels.cuh"

namespace llmq {

constexpr int kF32Tile = 32;            // output columns per warp
constexpr int kF32MaxThreads = 1024;
constexpr int kF32MaxSlots = 8;         // ring slots per warp

enum F32Pro : int {
  F32_PRO_PLAIN = 0,          // the input row as it is (Wo, W2)
  F32_PRO_RMSNORM = 1,        // RMSNorm(in, gamma) (QKV, W1|W3, lm-head)
  F32_PRO_EMBED_RMSNORM = 2   // x = wte row of step->token, then RMSNorm (first QKV)
};
enum F32Epi : int {
  F32_EPI_PLAIN = 0,   // out[j] = y
  F32_EPI_QKV = 1,     // + bias; q and k to out, v appended to the cache
  F32_EPI_RESID = 2,   // out[j] += y (Wo, W2)
  F32_EPI_LOGITS = 3,  // logits + device argmax
  F32_EPI_SWIGLU = 4   // columns [g0..g3 u0..u3 g4..]: out[i] = SiLU(g_i) * u_i (W1|W3)
};

struct F32Args {
  const float *w;           // tiles: tile t at w + t * K * 32
  const int *cta_t0;        // [G + 1]: first tile of CTA c
  int K, N;
  int rows;                 // rows per ring slot
  int slots;                // ring slots per warp
  int *err;
  // prologue
  const float *in;
  const float *gamma;
  float eps;
  const StepState *step;
  const float *wte;         // F32_PRO_EMBED_RMSNORM: [vocab][K]
  int vocab;
  float *x_out;             // F32_PRO_EMBED_RMSNORM: receives the embedding row
  // epilogue
  float *out;
  const float *bias;
  int qd, kvd, hd, max_seq;
  float *vcache;
  unsigned long long *argmax;
  int idx_offset;
  int n_out;                // F32_EPI_SWIGLU: d_ff
};

// MAXT: the launch's thread bound (256 for CTAs of a few warps, which gives
// the compiler more registers to schedule with; 1024 for the widest).
template <int PRO, int EPI, int MAXT>
__global__ void __launch_bounds__(MAXT, 1) k_gemv_f32(const F32Args a) {
  extern __shared__ __align__(128) uint8_t sm_f32[];
  __shared__ unsigned long long s_red64[32];
  __shared__ float s_r;
  __shared__ uint64_t s_xbar;  // the input row's bulk copy
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nwarps = nthr >> 5;
  const int K = a.K, R = a.rows, S = a.slots;
  const int slot_floats = R * kF32Tile;
  // per warp: S slots of R rows x 32 floats, then S mbarriers; then the input row
  float *ring = reinterpret_cast<float *>(sm_f32) + (size_t)warp * S * slot_floats;
  uint64_t *bars = reinterpret_cast<uint64_t *>(reinterpret_cast<float *>(sm_f32) + (size_t)nwarps * S * slot_floats) +
                   (size_t)warp * S;
  float *xs = reinterpret_cast<float *>(reinterpret_cast<uint64_t *>(reinterpret_cast<float *>(sm_f32) +
                                                                     (size_t)nwarps * S * slot_floats) +
                                        (((size_t)nwarps * S + 1) & ~size_t(1)));  // 16-byte aligned
  const int t0 = a.cta_t0[blockIdx.x], t1 = a.cta_t0[blockIdx.x + 1];
  const int tile = t0 + warp;
  const bool has_tile = tile < t1;
  const float *src = a.w + (size_t)(has_tile ? tile : 0) * K * kF32Tile;
  const int n_chunks = (K + R - 1) / R;
  if (lane == 0)
    for (int s = 0; s < S; ++s) mbar_init(&bars[s], 1);
  if (tid == 0) mbar_init(&s_xbar, 1);
  fence_mbar_init();
  __syncthreads();
  auto issue = [&](int i) {  // lane 0: rows [i*R, i*R + R) of this warp's tile into slot i % S
    const int rows = min(R, K - i * R);
    const uint32_t bytes = static_cast<uint32_t>(rows * kF32Tile * 4);
    uint64_t *bar = &bars[i % S];
    mbar_expect_tx(bar, bytes);
    bulk_load(ring + (size_t)(i % S) * slot_floats, src + (size_t)i * R * kF32Tile, bytes, bar);
  };
  // the weights never depend on the previous kernel: fill the ring now
  int issued = 0;
  if (lane == 0 && has_tile)
    for (; issued < S && issued < n_chunks; ++issued) issue(issued);
  pdl_launch_dependents();
  pdl_wait();

  // ------------------------------------------------------------ prologue
  // The input row (or embedding row) arrives with one bulk copy: a CTA of few
  // warps would otherwise spend hundreds of dependent load round trips on it.
  const float *row = a.in;
  if (PRO == F32_PRO_EMBED_RMSNORM) {  // llama.c:302-303
    int token = a.step->token;
    if (token < 0 || token >= a.vocab) {
      if (tid == 0 && blockIdx.x == 0) atomicOr(a.err, ERR_BAD_TOKEN);
      token = 0;
    }
    row = a.wte + (size_t)token * K;
  }
  const bool bulk_row = (K & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  if (bulk_row) {
    if (tid == 0) {
      asm volatile("fence.proxy.async.global;" ::: "memory");  // the previous kernel's writes, to the copy engine
      mbar_expect_tx(&s_xbar, static_cast<uint32_t>(K * 4));
      bulk_load(xs, row, static_cast<uint32_t>(K * 4), &s_xbar);
    }
    const bool landed = mbar_wait_bounded(&s_xbar, 0u);
    if (!landed && tid == 0) atomicOr(a.err, ERR_TIMEOUT);  // the step reports it; xs holds what landed
  } else {
    for (int k = tid; k < K; k += nthr) xs[k] = row[k];
  }
  __syncthreads();
  if (PRO != F32_PRO_PLAIN) {
    if (PRO == F32_PRO_EMBED_RMSNORM && blockIdx.x == 0)
      for (int k = tid; k < K; k += nthr) a.x_out[k] = xs[k];
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
  float acc = 0.0f;  // matrix.c:183
  bool ok = true;
  int done = 0;
  for (int i = 0; i < n_chunks && has_tile; ++i) {
    const int slot = i % S;
    const bool landed = mbar_wait_bounded(&bars[slot], static_cast<uint32_t>((i / S) & 1));
    if (!__all_sync(0xffffffffu, landed)) {
      ok = false;
      break;
    }
    const int rows = min(R, K - i * R);
    const float *t = ring + (size_t)slot * slot_floats + lane;
    const float *xk = xs + i * R;
    // matrix.c:185-188, in k order, in blocks of 8 rows.  The block loop is
    // unrolled so the compiler can hoist loads and products of later blocks
    // into the latency of the rounded adds (the only dependency).  (Explicit
    // software pipelines with rotating registers measured slower.)
    const int nb = rows >> 3;
#pragma unroll 4
    for (int b = 0; b < nb; ++b) {
      const int r0 = b * 8;
      float w[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) w[u] = t[(r0 + u) * kF32Tile];
      const float4 xa = *reinterpret_cast<const float4 *>(xk + r0);
      const float4 xb = *reinterpret_cast<const float4 *>(xk + r0 + 4);
      acc = __fadd_rn(acc, __fmul_rn(xa.x, w[0]));
      acc = __fadd_rn(acc, __fmul_rn(xa.y, w[1]));
      acc = __fadd_rn(acc, __fmul_rn(xa.z, w[2]));
      acc = __fadd_rn(acc, __fmul_rn(xa.w, w[3]));
      acc = __fadd_rn(acc, __fmul_rn(xb.x, w[4]));
      acc = __fadd_rn(acc, __fmul_rn(xb.y, w[5]));
      acc = __fadd_rn(acc, __fmul_rn(xb.z, w[6]));
      acc = __fadd_rn(acc, __fmul_rn(xb.w, w[7]));
    }
    for (int kk = nb * 8; kk < rows; ++kk) acc = __fadd_rn(acc, __fmul_rn(xk[kk], t[kk * kF32Tile]));
    done = i + 1;
    __syncwarp();  // every lane is done with the slot: refill it
    if (lane == 0 && issued < n_chunks) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the reads above before the copy's writes
      issue(issued++);
    }
  }
  if (!ok && lane == 0) {
    // record the failure and let this warp's copies still in flight land
    atomicOr(a.err, ERR_TIMEOUT);
    for (int i = done; i < issued; ++i) mbar_wait_bounded(&bars[i % S], static_cast<uint32_t>((i / S) & 1));
  }

  // ------------------------------------------------------------- epilogue
  const int j = tile * kF32Tile + lane;
  const bool has = ok && has_tile && j < a.N;
  if (EPI == F32_EPI_PLAIN) {
    if (has) a.out[j] = acc;
  } else if (EPI == F32_EPI_RESID) {
    if (has) a.out[j] = __fadd_rn(a.out[j], acc);  // llama.c:343 / 348
  } else if (EPI == F32_EPI_SWIGLU) {
    // lane l (l % 8 < 4) holds gate i, lane l + 4 the matching up (swiglu.c:9-12, 36-41)
    const float u = __shfl_down_sync(0xffffffffu, acc, 4);
    const int i = (j / 8) * 4 + (j % 8);
    if (has && (j % 8) < 4 && i < a.n_out) {
      const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, libm_expf(-acc)));
      a.out[i] = __fmul_rn(__fmul_rn(acc, s), u);
    }
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
}

}  // namespace llmq
