// llmq_f32.cuh - the fp32 (LLMA) decode path's matrix-vector products
// (llama.c:296-362 over matrix.c:178-199).
//
// The reference's matmul forms every output column as one sequential chain,
// C[j] = ((0 + a_0 w_0j) + a_1 w_1j) + ..., each product and each sum rounded
// on its own (no contraction under -std=c11).  The chain of a column cannot be
// split, so the parallelism is across columns: one lane per column, whole K.
//
// Columns are grouped in tiles, one per warp, of 32 columns (one per lane)
// for the narrow products, whose time is one warp's chain latency per row, or
// of 64 (two adjacent columns per lane: two independent chains and shared
// input loads, half the warps) for the wide ones (W1|W3, lm-head), which are
// bandwidth-bound.  A tile is stored as its own contiguous block, and each
// warp streams its tile through a private shared-memory ring of bulk copies,
// refilled by a producer warp (32-column tiles) or by the warp itself, so no
// warp ever waits for another.  CTA c owns a contiguous range of tiles, so
// the weights stream from all SMs.  The input row is staged once per CTA and
// read as a broadcast.
//
// Fused around the products, as on the int8 path: RMSNorm (+ embedding row)
// before, and bias with q/k/v routing, residual add, SiLU(g)*u (gate and up
// columns interleaved in fours, so a shuffle pairs them), or logits with the
// first-maximum argmax after.
#pragma once

#include "llmq_kernels.cuh"

namespace llmq {

// columns per lane: two for the wide products' epilogues, one otherwise
__host__ __device__ constexpr int f32_cpl(int epi) { return epi == 3 || epi == 4 ? 2 : 1; }
// a producer warp issues the copies (32-column tiles)
__host__ __device__ constexpr bool f32_producer(int epi) { return f32_cpl(epi) == 1; }
// Rows stored per tile.  A 64-column tile is [K][64] (lane l reads the float2
// of columns 2l, 2l+1 of a row).  A 32-column tile is [K/4][32][4]: the four
// consecutive rows of one column sit side by side, so a lane reads 4 rows of
// its column with one 16-byte load; K is padded to a multiple of 4 with zeros
// that are stored, copied and never read.
__host__ __device__ constexpr int f32_tile_rows(int K, int cpl) { return cpl == 1 ? (K + 3) & ~3 : K; }
constexpr int kF32MaxThreads = 1024;
constexpr int kF32MaxSlots = 8;         // ring slots per warp
constexpr int kF32RowsFull = 256;      // rows per slot of the unrolled 32-column path

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
  const float *w;           // tiles: tile t at w + t * f32_tile_rows(K, cpl) * 32 * cpl
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

// Shared memory of a CTA with nc consumer warps (plus the producer warp):
// nc rings of S slots of R rows x tile floats, the slots' "full" and "empty"
// mbarriers, then the input row (and, for RMSNorm, its squares).
__host__ __device__ constexpr size_t f32_ring_floats(int nc, int S, int R, int tile) {
  return (size_t)nc * S * R * tile;
}
__host__ __device__ constexpr size_t f32_bars(int nc, int S) { return ((size_t)2 * nc * S + 1) & ~size_t(1); }

// Chain of `rows` rows of a 32-column tile slot (CPL 1): rows in groups of 4
// per lane (one 16-byte load), matrix.c:185-188 in k order.  RC > 0: a full
// slot of RC rows, fully unrolled, so loads and products of later rows fill the
// latency of the rounded adds (the only dependency) with no loop overhead.
template <int RC>
__device__ __forceinline__ float chain32(float acc, const float4 *t, const float *xk, int rows) {
  auto blk8 = [&](int r0) {
    const float4 wa = t[(r0 >> 2) * 32], wb = t[((r0 >> 2) + 1) * 32];
    const float4 xa = *reinterpret_cast<const float4 *>(xk + r0);
    const float4 xb = *reinterpret_cast<const float4 *>(xk + r0 + 4);
    acc = __fadd_rn(acc, __fmul_rn(xa.x, wa.x));
    acc = __fadd_rn(acc, __fmul_rn(xa.y, wa.y));
    acc = __fadd_rn(acc, __fmul_rn(xa.z, wa.z));
    acc = __fadd_rn(acc, __fmul_rn(xa.w, wa.w));
    acc = __fadd_rn(acc, __fmul_rn(xb.x, wb.x));
    acc = __fadd_rn(acc, __fmul_rn(xb.y, wb.y));
    acc = __fadd_rn(acc, __fmul_rn(xb.z, wb.z));
    acc = __fadd_rn(acc, __fmul_rn(xb.w, wb.w));
  };
  if (RC > 0 && rows == RC) {
    // software-pipelined: the products of the next 8 rows are formed between
    // the adds of the current 8, in the order the warp issues them, so the
    // multiplies and loads sit in the adds' latency (5.8 instead of 7.4 cycles
    // per row when measured on its own)
    float p[8];
    {
      const float4 wa = t[0], wb = t[32];
      const float4 xa = *reinterpret_cast<const float4 *>(xk);
      const float4 xb = *reinterpret_cast<const float4 *>(xk + 4);
      p[0] = __fmul_rn(xa.x, wa.x);
      p[1] = __fmul_rn(xa.y, wa.y);
      p[2] = __fmul_rn(xa.z, wa.z);
      p[3] = __fmul_rn(xa.w, wa.w);
      p[4] = __fmul_rn(xb.x, wb.x);
      p[5] = __fmul_rn(xb.y, wb.y);
      p[6] = __fmul_rn(xb.z, wb.z);
      p[7] = __fmul_rn(xb.w, wb.w);
    }
    constexpr int NB = RC > 0 ? RC / 8 : 1;
#pragma unroll
    for (int b = 0; b < NB; ++b) {
      const int rn = (b + 1 < NB ? b + 1 : b) * 8;  // the last block reloads itself (unused)
      const float4 wa = t[(rn >> 2) * 32], wb = t[((rn >> 2) + 1) * 32];
      const float4 xa = *reinterpret_cast<const float4 *>(xk + rn);
      const float4 xb = *reinterpret_cast<const float4 *>(xk + rn + 4);
      float q[8];
      acc = __fadd_rn(acc, p[0]);
      q[0] = __fmul_rn(xa.x, wa.x);
      acc = __fadd_rn(acc, p[1]);
      q[1] = __fmul_rn(xa.y, wa.y);
      acc = __fadd_rn(acc, p[2]);
      q[2] = __fmul_rn(xa.z, wa.z);
      acc = __fadd_rn(acc, p[3]);
      q[3] = __fmul_rn(xa.w, wa.w);
      acc = __fadd_rn(acc, p[4]);
      q[4] = __fmul_rn(xb.x, wb.x);
      acc = __fadd_rn(acc, p[5]);
      q[5] = __fmul_rn(xb.y, wb.y);
      acc = __fadd_rn(acc, p[6]);
      q[6] = __fmul_rn(xb.z, wb.z);
      acc = __fadd_rn(acc, p[7]);
      q[7] = __fmul_rn(xb.w, wb.w);
#pragma unroll
      for (int u = 0; u < 8; ++u) p[u] = q[u];
    }
    return acc;
  }
  const int nb = rows >> 3;
#pragma unroll 4
  for (int b = 0; b < nb; ++b) blk8(b * 8);
  const float *tf = reinterpret_cast<const float *>(t);
  for (int kk = nb * 8; kk < rows; ++kk) acc = __fadd_rn(acc, __fmul_rn(xk[kk], tf[(kk >> 2) * 128 + (kk & 3)]));
  return acc;
}

// The same for a 64-column tile slot (CPL 2): float2 of columns 2l, 2l+1 per row.
__device__ __forceinline__ void chain64(float &acc0, float &acc1, const float2 *t, const float *xk, int rows) {
  const int nb = rows >> 3;
#pragma unroll 4
  for (int b = 0; b < nb; ++b) {
    const int r0 = b * 8;
    float2 w[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) w[u] = t[(r0 + u) * 32];
    const float4 xa = *reinterpret_cast<const float4 *>(xk + r0);
    const float4 xb = *reinterpret_cast<const float4 *>(xk + r0 + 4);
    const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      acc0 = __fadd_rn(acc0, __fmul_rn(xv[u], w[u].x));
      acc1 = __fadd_rn(acc1, __fmul_rn(xv[u], w[u].y));
    }
  }
  for (int kk = nb * 8; kk < rows; ++kk) {
    const float2 w = t[kk * 32];
    acc0 = __fadd_rn(acc0, __fmul_rn(xk[kk], w.x));
    acc1 = __fadd_rn(acc1, __fmul_rn(xk[kk], w.y));
  }
}

// MAXT: the launch's thread bound (256 for CTAs of a few warps, which gives
// the compiler more registers to schedule with; 1024 for the widest).  RC:
// rows per ring slot fixed at compile time (0: a.rows).
//
// Warps 0 .. nc-1 each own one tile.  32-column tiles (chain-latency-bound
// warps, one or two per CTA): the warps only compute - they wait for a slot's
// "full" barrier, run the chains over it and arrive on its "empty" barrier -
// and one more warp is the producer: its lane w issues every bulk copy of
// warp w's ring, the first S before the PDL wait, then each refill as soon as
// the slot's "empty" phase completes.  Taking the copy issue off the
// consumers shortens the gap between slots, which a latency-bound warp pays
// per slot.  64-column tiles (bandwidth-bound, many warps with small slots,
// faster than one producer can refill): lane 0 of each warp refills its own
// slot right after the warp has read it.
template <int PRO, int EPI, int MAXT, int RC>
__global__ void __launch_bounds__(MAXT, 1) k_gemv_f32(const F32Args a) {
  constexpr int CPL = f32_cpl(EPI), kF32Tile = 32 * CPL;
  constexpr bool kProd = f32_producer(EPI);
  extern __shared__ __align__(128) uint8_t sm_f32[];
  __shared__ unsigned long long s_red64[32];
  __shared__ uint64_t s_xbar;  // the input row's bulk copy
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = blockDim.x, nwarps = nthr >> 5;
  const int nc = kProd ? nwarps - 1 : nwarps;  // consumer warps; warp nc is the producer
  const int K = a.K, R = RC > 0 ? RC : a.rows, S = a.slots;
  const int slot_floats = R * kF32Tile;
  float *rings = reinterpret_cast<float *>(sm_f32);
  uint64_t *full = reinterpret_cast<uint64_t *>(rings + f32_ring_floats(nc, S, R, kF32Tile));
  uint64_t *empty = full + (size_t)nc * S;
  float *xs = reinterpret_cast<float *>(full + f32_bars(nc, S));  // 16-byte aligned
  const int t0 = a.cta_t0[blockIdx.x], t1 = a.cta_t0[blockIdx.x + 1];
  const int tile = t0 + warp;
  const bool has_tile = warp < nc && tile < t1;
  const int n_chunks = (K + R - 1) / R;
  for (int i = tid; i < nc * S; i += nthr) {
    mbar_init(&full[i], 1);
    mbar_init(&empty[i], 1);
  }
  if (tid == 0) mbar_init(&s_xbar, 1);
  fence_mbar_init();
  __syncthreads();
  // the issuing lane (the producer's lane pw, or lane 0 of warp pw): rows
  // [i*R, i*R + R) of warp pw's tile into its slot i % S
  const int pw = kProd ? lane : warp;
  const bool producing = kProd ? (warp == nc && pw < nc && t0 + pw < t1) : (lane == 0 && has_tile);
  const float *src = a.w + (size_t)(producing ? t0 + pw : 0) * f32_tile_rows(K, CPL) * kF32Tile;
  auto issue = [&](int i) {
    const int rows = min(R, f32_tile_rows(K, CPL) - i * R);  // R is a multiple of 8
    const uint32_t bytes = static_cast<uint32_t>(rows * kF32Tile * 4);
    uint64_t *bar = &full[pw * S + i % S];
    mbar_expect_tx(bar, bytes);
    bulk_load(rings + ((size_t)pw * S + i % S) * slot_floats, src + (size_t)i * R * kF32Tile, bytes, bar);
  };
  // the weights never depend on the previous kernel: fill the rings now
  int issued = 0;
  if (producing)
    for (; issued < S && issued < n_chunks; ++issued) issue(issued);
  pdl_wait();
  // The next kernel may start once every CTA is past its wait (the attention
  // kernel reads the step state and earlier cache rows before its own wait).
  pdl_launch_dependents();

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
    // rmsnorm.c:14-19: the sum of squares is one sequential chain, formed by
    // the block in the loop's order and rounding (spec_seq_sum)
    float *sq = xs + ((K + 3) & ~3);
    for (int k = tid; k < K; k += nthr) sq[k] = __fmul_rn(xs[k], xs[k]);
    __syncthreads();
    float ms = spec_seq_sum(sq, K, 0.0f, sq + ((K + 3) & ~3));  // sq is 16-byte aligned
    ms = __fmul_rn(ms, __fdiv_rn(1.0f, static_cast<float>(K)));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
    for (int k = tid; k < K; k += nthr) xs[k] = __fmul_rn(__fmul_rn(xs[k], r), a.gamma[k]);
  }
  __syncthreads();

  // --------------------------------------------------------------- chains
  float acc0 = 0.0f, acc1 = 0.0f;  // matrix.c:183: this lane's column(s)
  bool ok = true;
  if (kProd && warp == nc) {
    // producer: refill each slot once its consumer is done with it (the
    // consumer's arrive orders its reads before the copy's writes).  The loop
    // is bounded: 2^32 SM cycles in all, then the error flag.
    bool fail = false;
    const long long start = clock64();
    uint32_t polls = 0;
    while (__any_sync(0xffffffffu, producing && issued < n_chunks && !fail)) {
      bool progressed = false;
      if (producing && issued < n_chunks && !fail) {
        if (mbar_test_wait(&empty[pw * S + issued % S], static_cast<uint32_t>((issued / S - 1) & 1))) {
          issue(issued++);
          progressed = true;
        } else if ((++polls & 63u) == 0u && clock64() - start > (1ll << 32)) {
          fail = true;
        }
      }
      // nothing to refill yet: yield the issue slots to the consumers
      if (nc > 1 && !__any_sync(0xffffffffu, progressed)) __nanosleep(32);
    }
    // the last copy into each slot lands before the CTA may exit
    if (producing)
      for (int j = max(0, issued - S); j < issued; ++j)
        if (!mbar_wait_bounded(&full[pw * S + j % S], static_cast<uint32_t>((j / S) & 1))) fail = true;
    if (fail) atomicOr(a.err, ERR_TIMEOUT);
  } else if (has_tile) {
    float *ring = rings + (size_t)warp * S * slot_floats;
    for (int i = 0; i < n_chunks; ++i) {
      const int slot = i % S;
      const bool landed = mbar_wait_bounded(&full[warp * S + slot], static_cast<uint32_t>((i / S) & 1));
      if (!__all_sync(0xffffffffu, landed)) {
        ok = false;
        if (lane == 0) {
          atomicOr(a.err, ERR_TIMEOUT);
          // the copies still in flight land before the CTA may exit (the
          // producer drains its own)
          if (!kProd)
            for (int j = i; j < issued; ++j)
              mbar_wait_bounded(&full[warp * S + j % S], static_cast<uint32_t>((j / S) & 1));
        }
        break;
      }
      const int rows = min(R, K - i * R);
      const float *xk = xs + i * R;
      if constexpr (CPL == 2) {
        chain64(acc0, acc1, reinterpret_cast<const float2 *>(ring + (size_t)slot * slot_floats) + lane, xk, rows);
      } else {
        acc0 = chain32<RC>(acc0, reinterpret_cast<const float4 *>(ring + (size_t)slot * slot_floats) + lane, xk, rows);
      }
      __syncwarp();  // every lane is done with the slot
      if (kProd) {
        if (lane == 0) mbar_arrive(&empty[warp * S + slot]);
      } else if (lane == 0 && issued < n_chunks) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the reads above before the copy's writes
        issue(issued++);
      }
    }
  }

  // ------------------------------------------------------------- epilogue
  const int j0 = tile * kF32Tile + CPL * lane;  // this lane's column(s) j0 (, j0 + 1)
  const bool live = ok && has_tile;
  auto each = [&](auto &&fn) {
    if (live && j0 < a.N) fn(j0, acc0);
    if (CPL == 2 && live && j0 + 1 < a.N) fn(j0 + 1, acc1);
  };
  if (EPI == F32_EPI_PLAIN) {
    each([&](int j, float y) { a.out[j] = y; });
  } else if (EPI == F32_EPI_RESID) {
    each([&](int j, float y) { a.out[j] = __fadd_rn(a.out[j], y); });  // llama.c:343 / 348
  } else if (EPI == F32_EPI_SWIGLU) {
    // columns in eights [g g g g u u u u]: lanes 4m, 4m+1 hold gates, lanes
    // 4m+2, 4m+3 the matching ups (swiglu.c:9-12, 36-41)
    const float u0 = __shfl_down_sync(0xffffffffu, acc0, 2);
    const float u1 = __shfl_down_sync(0xffffffffu, acc1, 2);
    if (live && (lane & 3) < 2) {
      const int i0 = (j0 / 8) * 4 + (j0 % 8);
      const float g[2] = {acc0, acc1}, uu[2] = {u0, u1};
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        if (j0 + q < a.N && i0 + q < a.n_out) {
          const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, libm_expf(-g[q])));
          a.out[i0 + q] = __fmul_rn(__fmul_rn(g[q], s), uu[q]);
        }
      }
    }
  } else if (EPI == F32_EPI_QKV) {
    const int pos = a.step->pos;
    const bool pos_ok = pos >= 0 && pos < a.max_seq;
    if (!pos_ok && tid == 0) atomicOr(a.err, ERR_BAD_POS);
    if (pos_ok)
      each([&](int j, float acc) {
        const float y = __fadd_rn(acc, a.bias[j]);  // llama.c:316-318
        if (j < a.qd + a.kvd) {
          a.out[j] = y;
        } else {
          const int jv = j - a.qd - a.kvd, vh = jv / a.hd;
          a.vcache[((size_t)vh * a.max_seq + pos) * a.hd + (jv - vh * a.hd)] = y;  // llama.c:322
        }
      });
  } else if (EPI == F32_EPI_LOGITS) {
    unsigned long long key = 0ull;
    each([&](int j, float y) {
      a.out[j] = y;
      const unsigned long long k = argmax_key(y, static_cast<uint32_t>(j + a.idx_offset));
      key = k > key ? k : key;
    });
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
