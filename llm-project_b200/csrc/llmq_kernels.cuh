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
#include "llmq_device_common.cuh"
#include "llmq_spec_sum.cuh"

#include <cooperative_groups.h>

namespace llmq {

namespace cg = cooperative_groups;

// Phase timestamps for profiling builds (-DLLMQ_PHASE_TIMING): thread 0 of the
// first 64 CTAs records %globaltimer at numbered points.  Compiled out otherwise.
#ifdef LLMQ_PHASE_TIMING
__device__ unsigned long long g_phase_ts[64][16];
__device__ unsigned long long g_phase_grid;  // record only this launch (%gridid; 0: every launch)
#define LLMQ_TSTAMP(i)                                                  \
  do {                                                                  \
    if (threadIdx.x == 0 && blockIdx.x < 64 && blockIdx.y == 0) {       \
      unsigned long long t_, g_;                                        \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));           \
      asm volatile("mov.u64 %0, %%gridid;" : "=l"(g_));                \
      if (g_phase_grid == 0 || g_phase_grid == g_) g_phase_ts[blockIdx.x][i] = t_; \
    }                                                                   \
  } while (0)
// Launch spans: per grid launch (%gridid), the earliest CTA start and the
// latest CTA end, so a graph replay's kernels can be laid out in time.
__device__ unsigned long long g_launch_tab[4096][4];  // gridid, first start, last end, kernel tag
__device__ __forceinline__ unsigned long long llmq_now() {
  unsigned long long t_;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));
  return t_;
}
__device__ __forceinline__ unsigned long long llmq_gridid() {
  unsigned long long g_;
  asm volatile("mov.u64 %0, %%gridid;" : "=l"(g_));
  return g_;
}
#define LLMQ_LAUNCH_ENTER_TAG(tag)                                       \
  do {                                                                   \
    if (threadIdx.x == 0) {                                              \
      const unsigned long long g_ = llmq_gridid();                       \
      unsigned long long *e_ = g_launch_tab[g_ & 4095];                  \
      e_[0] = g_;                                                        \
      e_[3] = (tag);                                                     \
      atomicMin(&e_[1], llmq_now());                                     \
    }                                                                    \
  } while (0)
#define LLMQ_LAUNCH_ENTER() LLMQ_LAUNCH_ENTER_TAG(0)
#define LLMQ_LAUNCH_EXIT()                                               \
  do {                                                                   \
    if (threadIdx.x == 0) atomicMax(&g_launch_tab[llmq_gridid() & 4095][2], llmq_now()); \
  } while (0)
// Both ends of a launch span around a whole kernel body (every return path).
struct LaunchSpanGuard {
  __device__ explicit LaunchSpanGuard(int tag) { LLMQ_LAUNCH_ENTER_TAG(tag); }
  __device__ ~LaunchSpanGuard() { LLMQ_LAUNCH_EXIT(); }
};
#define LLMQ_LAUNCH_SPAN(tag) LaunchSpanGuard llmq_span_guard_(tag)
#else
#define LLMQ_TSTAMP(i) \
  do {               \
  } while (0)
#define LLMQ_LAUNCH_ENTER() \
  do {                    \
  } while (0)
#define LLMQ_LAUNCH_ENTER_TAG(tag) \
  do {                           \
  } while (0)
#define LLMQ_LAUNCH_EXIT() \
  do {                   \
  } while (0)
#define LLMQ_LAUNCH_SPAN(tag) \
  do {                      \
  } while (0)
#endif

constexpr int kThreads = 512;     // GEMV CTA size (16 warps)
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
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
// One contiguous global->shared bulk copy into this CTA's own shared memory, completing on `bar`.
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
// Non-blocking test of an mbarrier phase (for a lane that polls several).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}
// Bounded wait on an mbarrier phase: gives up after 2^32 SM cycles (about 2 s
// at boost clock; the SM-local counter is cheap to read, unlike %globaltimer)
// or 2^26 polls, so a lost copy can never hang the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase) {
  if (mbar_try_wait(bar, phase)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 0; it < (1u << 26); ++it) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((it & 63u) == 63u && clock64() - t0 > (1ll << 32)) break;
  }
  return false;
}
// Programmatic dependent launch: let the next kernel in the stream start its
// weight prefetch now / wait until the previous kernel's writes are visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

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
  const double y = exp(static_cast<double>(x));
  // Fast paths, the same decisions as lx_expf_cr's tests: when y lies in the
  // normal float range (biased double exponent 897..1150), the 29 low mantissa
  // bits of y are its position inside one float ulp, with the rounding
  // midpoint at 2^28.  y is more than LX_WINDOW (2^-9) ulp from the midpoint
  // exactly when they differ from 2^28 by more than 2^20: (float)y is the
  // result.  Within the window but more than LX_AMBIG (2^-24) ulp away, y
  // decides the correct rounding f, and the result is f unless the input is
  // one of the host library's exceptions, which round to the float on the other
  // side of y (f's neighbour: exp is positive, so one step of the bit pattern).
  const unsigned long long yb = static_cast<unsigned long long>(__double_as_longlong(y));
  const int ye = static_cast<int>((yb >> 52) & 0x7ffu);
  if (ye >= 897 && ye <= 1150) {
    const int dist = static_cast<int>(static_cast<uint32_t>(yb & 0x1fffffffull)) - (1 << 28);
    if (dist > (1 << 20) || dist < -(1 << 20)) return __double2float_rn(y);
    if (dist > (1 << 5) || dist < -(1 << 5)) {
      const float f = __double2float_rn(y);
      const uint32_t fb = __float_as_uint(f);
      const float other = __uint_as_float(static_cast<double>(f) < y ? fb + 1u : fb - 1u);
      return expf_is_exception(__float_as_uint(x)) ? other : f;
    }
  }
  int near;
  float lo, up;
  const float cr = lx_expf_cr(x, y, &near, &lo, &up);
  if (!near) return cr;
  if (expf_is_exception(lx_bits(x))) return (cr == up) ? lo : up;
  return cr;
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
  EPI_QKV = 1,     // + bias; q and k to `out`, v appended to the cache
  EPI_RESID = 2,   // out[j] += as*ws*acc                           (Wo, W2)
  EPI_SWIGLU = 3,  // out[j] = SiLU(gate) * up                      (W1|W3)
  EPI_LOGITS = 4,  // logits + device argmax                        (lm-head)
  EPI_TP_RESID = 5 // row-parallel shard: exchange the slab's partial sums with the peers over
                   // NVLink peer memory, add them, then out[j] += as*ws*sum (tp_exchange.h)
};

// ------------------------------------------- tensor-parallel peer exchange
// Every rank of a tensor-parallel group holds one exchange region, mapped into
// the other ranks' address spaces (CUDA IPC).  Layout, for world W, d_model dm
// and ns slabs of 256 columns:
//   int      data[2][W][dm]   partial sums of a row-parallel product, by the
//                             product's parity and the source rank
//   float    amax[2][W]       the source rank's absmax of the product's input
//   unsigned flag_slab[ns][W] epoch of the last slab partials received from W
//   unsigned flag_amax[W]     epoch of the last absmax received
// (ns = ceil(dm / 256)).  A rank stores into every region (its own
// included), fences system-wide, then raises its flag in every region;
// readers wait for the flags of all ranks to reach the product's epoch.
// Epochs increase by one per product and never repeat; a rank is at most one
// product ahead of another (its next push needs the others' pushes of the
// current product), so two data buffers suffice.
struct TpExchange {
  char *const *peers;      // [W] region base of every rank, this rank's own included
  const unsigned *seq;     // products completed before this step
  int rank, world, dm, pidx;  // pidx: the product's index within the step (epoch = *seq + pidx + 1)
  unsigned poll_limit;     // polls before a flag wait gives up (0: kFlagPolls)
};
__host__ __device__ inline size_t tpx_data_off() { return 0; }
__host__ __device__ inline size_t tpx_amax_off(int W, int dm) { return (size_t)2 * W * dm * 4; }
__host__ __device__ inline size_t tpx_fslab_off(int W, int dm) {
  return (tpx_amax_off(W, dm) + (size_t)2 * W * 4 + 15) & ~size_t(15);
}
__host__ __device__ inline size_t tpx_famax_off(int W, int dm) {
  return tpx_fslab_off(W, dm) + (size_t)((dm + 255) / 256) * W * 4;
}
__host__ __device__ inline size_t tpx_bytes(int W, int dm) { return tpx_famax_off(W, dm) + (size_t)W * 4; }

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *p >= epoch; false after `limit` polls (0: kFlagPolls,
// 2^24 polls of ~32 ns sleep each, about a second).  A wait that gives up
// leaves the kernel to record ERR_TIMEOUT and return.
constexpr uint32_t kFlagPolls = 1u << 24;
__device__ __forceinline__ bool wait_flag(const unsigned *p, unsigned epoch, uint32_t limit) {
  const uint32_t n = limit ? limit : kFlagPolls;
  for (uint32_t it = 0; it < n; ++it) {
    if (ld_acquire_u32(p) >= epoch) return true;
    __nanosleep(32);
  }
  return false;
}

// Tile geometry: a tile is KT rows of k by kNT columns, stored as
// [KT/16][kNT][16 bytes] so that one column's 16 consecutive k values form one
// 16-byte chunk (four dp4a operands) and a warp reads 512 contiguous bytes.
// KT is 64 (16 KB tiles, finer load balance for small matrices) or 128 (32 KB
// tiles, half the per-tile overhead for large ones).
constexpr int kNT = 256;
constexpr int kParts = kThreads / kNT;  // threads per column
static_assert(kParts * kNT == kThreads, "tile geometry");

// Shared memory of a GEMV's mbarriers: full[S] and empty[S] of the ring and
// the input row's, rounded to 16 bytes.
__host__ __device__ inline size_t gemv_bar_bytes(int S) { return ((size_t)(2 * S + 1) * 8 + 15) & ~size_t(15); }

struct StepState {
  int token;
  int pos;
};

struct GemvArgs {
  const uint8_t *w;    // tiles [n_slabs][n_ktiles][KT/16][kNT][16]
  const float *ws;     // per physical column scale [Npad]
  int K, Kpad, N, Npad, n_slabs, n_ktiles, stages, rows;
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
  float *out;          // [rows][N]; EPI_QKV: q then k of this step (qd + kvd)
  const float *bias;   // EPI_QKV, physical order
  int qd, kvd, hd, max_seq;
  float *vcache;       // EPI_QKV: this layer's [n_kv][max_seq][hd]
  unsigned long long *argmax;
  int idx_offset;      // EPI_LOGITS: global index of column 0 (vocab shard)
  const float *absmax_in;  // PRO_ABSMAX, one row: the row's absmax, published by the producer (else computed
                           // here); only the CTA's own k-tiles of the row are then loaded and quantised
  float *amax_out;         // EPI_SWIGLU: max |out| is folded in here (the next product's absmax_in)
  TpExchange tp;           // EPI_TP_RESID
};

// Folds max |v| over this warp's values into *dst (a non-negative float kept
// as its bit pattern, which orders like the float).  NaN values are left out,
// as the reference's absmax loop leaves them out (quant.c:70).
__device__ __forceinline__ void warp_amax_publish(float v, float *dst) {
  float m = v == v ? fabsf(v) : 0.0f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m > 0.0f) atomicMax(reinterpret_cast<unsigned *>(dst), __float_as_uint(m));
}

// Owner CTA of tile t under the contiguous split [c*T/G, (c+1)*T/G).
__device__ __forceinline__ long long tile_owner(long long t, long long T, long long G) {
  return ((t + 1) * G + T - 1) / T - 1;
}

__device__ __forceinline__ int dot16(const int4 w, const int4 x, int acc) {
  acc = __dp4a(w.x, x.x, acc);
  acc = __dp4a(w.y, x.y, acc);
  acc = __dp4a(w.z, x.z, acc);
  return __dp4a(w.w, x.w, acc);
}

// ------------------------------------------------------------ the GEMV kernel
// x(rows, K) @ W(K, N) with W pre-tiled so every tile is one contiguous bulk
// copy.  Each CTA owns a contiguous range of tiles (balanced to one tile),
// streams them through a `stages`-deep shared-memory ring, and accumulates
// exact int32 dot products with dp4a (two threads per column, each with two
// independent accumulators).  Partial sums of a column slab are added into
// `acc` with integer atomics; the CTA that completes a slab applies the fused
// epilogue and re-zeroes `acc` and `cnt` for the next launch.
template <int PRO, int EPI, int MR, int KT>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const GemvArgs a) {
  constexpr int kTileBytes = kNT * KT;
  constexpr int kChunksPerPart = (KT / 16) / kParts;
  static_assert(kChunksPerPart * kParts * 16 == KT && kChunksPerPart % 2 == 0, "tile depth");
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ float s_red[32];
  __shared__ unsigned long long s_red64[32];
  __shared__ float s_as[MR];
  __shared__ int s_flag;
  __shared__ int s_abort;

  LLMQ_TSTAMP(0);
  LLMQ_LAUNCH_ENTER_TAG(1);
  const int tid = threadIdx.x;
  const int S = a.stages;
  uint8_t *stage0 = sm;
  uint64_t *bars = reinterpret_cast<uint64_t *>(sm + (size_t)S * kTileBytes);  // full[S], empty[S], row
  uint64_t *empty = bars + S;
  uint64_t *rowbar = bars + 2 * S;  // the input row's bulk copy
  int8_t *codes = reinterpret_cast<int8_t *>(sm + (size_t)S * kTileBytes + gemv_bar_bytes(S));
  float *xs = reinterpret_cast<float *>(codes + (((size_t)a.rows * a.Kpad + 15) & ~size_t(15)));
  float *ebuf = xs;  // epilogue exchange buffer (prologue vector is dead by then)

  const long long T = (long long)a.n_slabs * a.n_ktiles;
  const long long G = gridDim.x;
  const long long t_begin = (long long)blockIdx.x * T / G;
  const long long t_end = (long long)(blockIdx.x + 1) * T / G;
  const int n = static_cast<int>(t_end - t_begin);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&bars[s], 1);               // the stage's copy landed
      mbar_init(&empty[s], kThreads / 32);  // every warp has read the stage
    }
    mbar_init(rowbar, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  __syncthreads();
  // Weights never depend on the previous kernel: start streaming them now.
  // Only the first two stages go out before the wait: the input row is on the
  // critical path (the RMSNorm chain needs all of it), so its loads must not
  // queue behind the whole ring's copies.  The rest of the ring is issued
  // right after the row's loads.
  int issued = 0;
  auto issue_to = [&](int upto) {
    if (tid == 0) {
      const int first = n < upto ? n : upto;
      for (; issued < first; ++issued) {
        mbar_expect_tx(&bars[issued], kTileBytes);
        bulk_load(stage0 + (size_t)issued * kTileBytes, a.w + (size_t)(t_begin + issued) * kTileBytes,
                  kTileBytes, &bars[issued]);
      }
    }
  };
  issue_to(2);
  LLMQ_TSTAMP(1);
  pdl_wait();
  // The next kernel may start once every CTA is past its wait: whatever it
  // reads before its own wait was then written by kernels already complete.
  pdl_launch_dependents();
  LLMQ_TSTAMP(2);

  // ------------------------------------------------------------ prologue
  // The input rows come from the previous kernel: copied into xs with one bulk
  // copy per row once that kernel's writes are visible, ahead of the rest of
  // the ring (plain loads when the row is not 16-byte sized and aligned).
  const bool vec_in = (a.K & 3) == 0 && (reinterpret_cast<uintptr_t>(a.in) & 15) == 0;
  uint32_t row_phase = 0;
  auto load_row = [&](const float *src) {
    if (vec_in) {
      if (tid == 0) {
        mbar_expect_tx(rowbar, static_cast<uint32_t>(a.K) * 4u);
        bulk_load(xs, src, static_cast<uint32_t>(a.K) * 4u, rowbar);
      }
      issue_to(S);
      if (!mbar_wait_bounded(rowbar, row_phase)) s_abort = 1;
      row_phase ^= 1u;
    } else {
      for (int k = tid; k < a.K; k += kThreads) xs[k] = src[k];
      issue_to(S);
    }
    __syncthreads();
  };
  if (PRO == PRO_ABSMAX && a.absmax_in && a.rows == 1 && vec_in) {
    // The absmax comes from the producer: only the k-tiles of this CTA's tiles
    // are loaded and quantised (its range spans one slab, two, or whole ones).
    const long long nk = a.n_ktiles, s0 = t_begin / nk, s1 = (t_end - 1) / nk;
    int ra0 = 0, ra1 = a.n_ktiles, rb0 = 0, rb1 = 0;  // k-tiles [ra0, ra1) and [rb0, rb1)
    if (s0 == s1) {
      ra0 = static_cast<int>(t_begin - s0 * nk);
      ra1 = static_cast<int>(t_end - s0 * nk);
    } else if (s1 == s0 + 1 && t_end - s1 * nk < t_begin - s0 * nk) {
      ra0 = static_cast<int>(t_begin - s0 * nk);
      rb1 = static_cast<int>(t_end - s1 * nk);
    }
    auto bytes_of = [&](int t0, int t1) -> uint32_t {
      const int k0 = t0 * KT, k1 = min(t1 * KT, a.K);
      return k1 > k0 ? static_cast<uint32_t>(k1 - k0) * 4u : 0u;
    };
    if (tid == 0) {
      const uint32_t ba = bytes_of(ra0, ra1), bb = bytes_of(rb0, rb1);
      mbar_expect_tx(rowbar, ba + bb);
      if (ba) bulk_load(xs + (size_t)ra0 * KT, a.in + (size_t)ra0 * KT, ba, rowbar);
      if (bb) bulk_load(xs + (size_t)rb0 * KT, a.in + (size_t)rb0 * KT, bb, rowbar);
    }
    issue_to(S);
    if (!mbar_wait_bounded(rowbar, 0)) s_abort = 1;
    __syncthreads();
    const float m = *a.absmax_in;
    const float as = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;  // quant.c:71
    const float inv = __fdiv_rn(1.0f, as);                      // quant.c:72
    if (tid == 0) s_as[0] = as;
    for (int k = ra0 * KT + tid; k < ra1 * KT; k += kThreads) codes[k] = k < a.K ? code_of(__fmul_rn(xs[k], inv)) : 0;
    for (int k = rb0 * KT + tid; k < rb1 * KT; k += kThreads) codes[k] = k < a.K ? code_of(__fmul_rn(xs[k], inv)) : 0;
  } else if (PRO == PRO_ABSMAX) {
    for (int r = 0; r < a.rows && r < MR; ++r) {
      load_row(a.in + (size_t)r * a.K);
      float m = 0.0f;
      if (a.absmax_in) {
        m = a.absmax_in[r];
      } else {
        for (int k = tid; k < a.K; k += kThreads) m = fmaxf(m, fabsf(xs[k]));
        m = block_max<kThreads>(m, s_red);
      }
      const float as = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;  // quant.c:71
      const float inv = __fdiv_rn(1.0f, as);                      // quant.c:72
      if (tid == 0) s_as[r] = as;
      int8_t *cr = codes + (size_t)r * a.Kpad;
      for (int k = tid; k < a.Kpad; k += kThreads) cr[k] = k < a.K ? code_of(__fmul_rn(xs[k], inv)) : 0;
      __syncthreads();  // xs is reloaded for the next row
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
      issue_to(S);
      __syncthreads();
    } else {
      load_row(a.in);
    }
    LLMQ_TSTAMP(3);
    // The sum of squares (rmsnorm.c:15): the products are independent, so all
    // threads form them; the adds keep the loop's order and rounding
    // (spec_seq_sum: segments run in parallel from candidate starts, linked
    // exactly).
    float *sq = xs + ((K + 3) & ~3);
    for (int k = tid; k < K; k += kThreads) sq[k] = __fmul_rn(xs[k], xs[k]);
    __syncthreads();
    float ms = spec_seq_sum(sq, K, 0.0f, sq + ((K + 3) & ~3));  // sq is 16-byte aligned
    ms = __fmul_rn(ms, __fdiv_rn(1.0f, static_cast<float>(K)));
    const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, a.eps)));
    LLMQ_TSTAMP(4);
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

  LLMQ_TSTAMP(5);
  // --------------------------------------------------------------- main loop
  const int col = tid % kNT;
  const int part = tid / kNT;
  int acc0[MR], acc1[MR];
#pragma unroll
  for (int r = 0; r < MR; ++r) acc0[r] = acc1[r] = 0;

  auto flush = [&](long long slab) {
    // combine the two accumulators, then the kParts threads of each column
    int *red = reinterpret_cast<int *>(ebuf);
#pragma unroll
    for (int r = 0; r < MR; ++r) {
      if (r >= a.rows) break;
      __syncthreads();
      red[tid] = acc0[r] + acc1[r];
      __syncthreads();
      if (part == 0) {
        int s = 0;
#pragma unroll
        for (int p = 0; p < kParts; ++p) s += red[p * kNT + col];
        atomicAdd(a.acc + (size_t)r * a.Npad + slab * kNT + col, s);
      }
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
    // ---- fused epilogue for columns [slab*kNT, slab*kNT + kNT)
    const int p0 = static_cast<int>(slab) * kNT;
    if (EPI == EPI_TP_RESID) {
      // This slab's partial sums go to every rank; once every rank's have
      // arrived, their (exact, integer) sum feeds the residual update.
      const TpExchange &x = a.tp;
      const unsigned epoch = *x.seq + x.pidx + 1;
      const int par = epoch & 1u;
      const size_t fs = tpx_fslab_off(x.world, x.dm);
      for (int c = tid; c < kNT; c += kThreads) {
        const int j = p0 + c;
        const int v = atomicExch(a.acc + j, 0);
        if (j < a.N)
          for (int q = 0; q < x.world; ++q)
            reinterpret_cast<int *>(x.peers[q] + tpx_data_off())[((size_t)par * x.world + x.rank) * x.dm + j] = v;
      }
      __threadfence_system();
      __syncthreads();
      if (tid < x.world) {
        st_release_u32(reinterpret_cast<unsigned *>(x.peers[tid] + fs) + (size_t)slab * x.world + x.rank, epoch);
        const unsigned *own = reinterpret_cast<const unsigned *>(x.peers[x.rank] + fs) + (size_t)slab * x.world + tid;
        if (!wait_flag(own, epoch, x.poll_limit)) {
          atomicOr(a.err, ERR_TIMEOUT);
          s_abort = 1;
        }
      }
      __syncthreads();
      if (!s_abort) {
        const int *data = reinterpret_cast<const int *>(x.peers[x.rank] + tpx_data_off());
        const float as = s_as[0];
        for (int c = tid; c < kNT; c += kThreads) {
          const int j = p0 + c;
          if (j >= a.N) continue;
          int sum = 0;
          for (int q = 0; q < x.world; ++q) sum += __ldcv(data + ((size_t)par * x.world + q) * x.dm + j);
          a.out[j] = __fadd_rn(a.out[j], dequant(as, a.ws[j], sum));  // llama.c:578 / 589
        }
      }
    } else if (EPI == EPI_PLAIN || EPI == EPI_RESID) {
      for (int r = 0; r < a.rows && r < MR; ++r) {
        const float as = s_as[r];
        for (int c = tid; c < kNT; c += kThreads) {
          const int j = p0 + c;
          float *o = a.out + (size_t)r * a.N + j;
          // the scale and the residual are read before the sum, so the three round trips overlap
          const float wsj = j < a.N ? a.ws[j] : 0.0f;
          const float res = EPI == EPI_RESID && j < a.N ? *o : 0.0f;
          const int v = atomicExch(a.acc + (size_t)r * a.Npad + j, 0);
          if (j < a.N) {
            const float y = dequant(as, wsj, v);
            if (EPI == EPI_RESID)
              *o = __fadd_rn(res, y);  // llama.c:578 / llama.c:589
            else
              *o = y;
          }
        }
      }
    } else if (EPI == EPI_LOGITS) {
      const float as = s_as[0];
      unsigned long long best = 0ull;
      for (int c = tid; c < kNT; c += kThreads) {
        const int j = p0 + c;
        const float wsj = j < a.N ? a.ws[j] : 0.0f;
        const int v = atomicExch(a.acc + j, 0);
        if (j < a.N) {
          const float y = dequant(as, wsj, v);
          a.out[j] = y;
          const unsigned long long key = argmax_key(y, static_cast<uint32_t>(j + a.idx_offset));
          best = key > best ? key : best;
        }
      }
      best = block_max_u64<kThreads>(best, s_red64);
      if (tid == 0) atomicMax(a.argmax, best);
    } else if (EPI == EPI_SWIGLU) {
      // slab = kNT/2 gate columns followed by the kNT/2 matching up columns
      const float as = s_as[0];
      constexpr int half = kNT / 2;
      for (int c = tid; c < half; c += kThreads) {
        const int j = static_cast<int>(slab) * half + c;  // d_ff index
        const float wg = j < a.N ? a.ws[p0 + c] : 0.0f, wu = j < a.N ? a.ws[p0 + half + c] : 0.0f;
        const int vg = atomicExch(a.acc + p0 + c, 0);
        const int vu = atomicExch(a.acc + p0 + half + c, 0);
        float h = 0.0f;
        if (j < a.N) {
          const float z = dequant(as, wg, vg);
          const float u = dequant(as, wu, vu);
          const float s = __fdiv_rn(1.0f, __fadd_rn(1.0f, libm_expf(-z)));  // llama.c:585
          h = __fmul_rn(__fmul_rn(z, s), u);                                // llama.c:586
          a.out[j] = h;
        }
        if (a.amax_out) warp_amax_publish(h, a.amax_out);  // the W2 product's row absmax
      }
    } else if (EPI == EPI_QKV) {
      // q, k (before RoPE, which the attention kernel applies) and v of this step
      const float as = s_as[0];
      const int pos = a.step->pos;
      const bool pos_ok = pos >= 0 && pos < a.max_seq;
      if (!pos_ok && tid == 0) atomicOr(a.err, ERR_BAD_POS);
      for (int c = tid; c < kNT; c += kThreads) {
        const int j = p0 + c;
        const float wsj = j < a.N ? a.ws[j] : 0.0f, bj = j < a.N ? a.bias[j] : 0.0f;
        const int v = atomicExch(a.acc + j, 0);
        if (j >= a.N || !pos_ok) continue;
        const float y = __fadd_rn(dequant(as, wsj, v), bj);  // llama.c:546-548
        if (j < a.qd + a.kvd) {
          a.out[j] = y;
        } else {
          const int jv = j - a.qd - a.kvd, vh = jv / a.hd;
          a.vcache[((size_t)vh * a.max_seq + pos) * a.hd + (jv - vh * a.hd)] = y;  // llama.c:552
        }
      }
    }
    if (tid == 0) a.cnt[slab] = 0;
    __syncthreads();
  };

  // (slab, kt) of tile t_begin + i and its ring stage / phase, advanced
  // incrementally (no division in the loop)
  long long slab = t_begin / a.n_ktiles;
  int kt = static_cast<int>(t_begin - slab * a.n_ktiles);
  long long cur = n > 0 ? slab : -1;
  int done = 0, s = 0, ps = 0;
  uint32_t phase = 0, pphase = 0;  // ring position of tile i and of tile i - 1
  const uint8_t *tile_base = stage0 + ((size_t)part * kChunksPerPart * kNT + col) * 16;
  const int8_t *code_base = codes + part * (kChunksPerPart * 16);
  for (int i = 0; i < n; ++i) {
    if (*reinterpret_cast<volatile int *>(&s_abort)) break;  // thread 0 gave up refilling
    if (i > 0 && ++kt == a.n_ktiles) {
      kt = 0;
      ++slab;
    }
    if (slab != cur) {
      flush(cur);
#pragma unroll
      for (int r = 0; r < MR; ++r) acc0[r] = acc1[r] = 0;
      cur = slab;
    }
    if (!mbar_wait_bounded(&bars[s], phase)) s_abort = 1;
    const uint8_t *tile = tile_base + (size_t)s * kTileBytes;
    int4 wv[kChunksPerPart];
#pragma unroll
    for (int c = 0; c < kChunksPerPart; ++c) wv[c] = *reinterpret_cast<const int4 *>(tile + (size_t)c * kNT * 16);
    const int8_t *cb = code_base + (size_t)kt * KT;
#pragma unroll
    for (int r = 0; r < MR; ++r) {
      if (r < a.rows) {
#pragma unroll
        for (int c = 0; c < kChunksPerPart; c += 2) {
          const int4 x0 = *reinterpret_cast<const int4 *>(cb + (size_t)r * a.Kpad + c * 16);
          const int4 x1 = *reinterpret_cast<const int4 *>(cb + (size_t)r * a.Kpad + c * 16 + 16);
          acc0[r] = dot16(wv[c], x0, acc0[r]);
          acc1[r] = dot16(wv[c + 1], x1, acc1[r]);
        }
      }
    }
    // This warp is done with stage s.  Thread 0 then refills the stage of the
    // previous tile (read by all warps by now, or soon: it waits on that
    // stage's empty barrier) with tile i - 1 + S; no warp waits for another
    // at a block barrier.
    __syncwarp();
    if ((tid & 31) == 0) mbar_arrive(&empty[s]);
    done = i + 1;
    if (s_abort) break;
    if (tid == 0 && i > 0 && issued < n) {
      if (!mbar_wait_bounded(&empty[ps], pphase)) {
        s_abort = 1;
        break;
      }
      mbar_expect_tx(&bars[ps], kTileBytes);
      bulk_load(stage0 + (size_t)ps * kTileBytes, a.w + (size_t)(t_begin + issued) * kTileBytes, kTileBytes,
                &bars[ps]);
      ++issued;
    }
    ps = s;
    pphase = phase;
    if (++s == S) {
      s = 0;
      phase ^= 1u;
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
  LLMQ_TSTAMP(6);
  if (n > 0) flush(cur);
  LLMQ_TSTAMP(7);
  LLMQ_LAUNCH_EXIT();
}

// --------------------------------------------------------------- attention
// Device KV cache layout, per layer: [n_kv][max_seq][hd] (head-major), so the
// rows of one KV head are contiguous and can be staged with asynchronous copies.
struct AttnArgs {
  const float *q;       // [n_heads * hd] q, then [kvd] k of this step, before RoPE
  float *kcache;        // this layer's [n_kv][max_seq][hd]
  const float *vcache;
  float *scores;        // [n_heads][max_seq] scratch
  float *out;           // [n_heads * hd]
  const StepState *step;
  const float *rope_cos, *rope_sin;  // [max_seq][hd/2]
  int n_heads, n_kv, hd, max_seq;
  int pv_whole;  // k_attn_pv stages the whole value slice at once (it fits in shared memory)
  int fused_chunk;  // > 0: k_attn_fused with key chunks of this many rows (0: the two-kernel path)
  float *amax_out;  // if set, max |out| is folded in here (the Wo product's absmax_in)
};

constexpr int kScoreChunk = 32;    // key positions per scores CTA
constexpr int kScoreThreads = 128;
constexpr int kPVSlice = 32;       // output dims per softmax-V CTA
constexpr int kPVThreads = 256;
constexpr int kPVChunk = 128;      // value positions per staged chunk
constexpr int kPVRing = 4;         // staged chunks in flight

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// RoPE (rope.c:58-64) of element d of one head: pairs (k, k + hd/2).
__device__ __forceinline__ float rope_elem(const float *x, int d, int half, const float *cs, const float *sn) {
  if (d < half) return __fsub_rn(__fmul_rn(x[d], cs[d]), __fmul_rn(x[d + half], sn[d]));
  const int k = d - half;
  return __fadd_rn(__fmul_rn(x[d], cs[k]), __fmul_rn(x[k], sn[k]));
}

// Copies rows [r0, r1) x cols [c0, c0 + w) of a row-major f32 matrix (row
// stride `ld`) into shared memory rows of stride `sld`, with 16-byte
// asynchronous copies when alignment allows, else plain loads.
__device__ __forceinline__ void stage_rows(float *dst, int sld, const float *src, int ld, int r0, int r1, int c0,
                                           int w, int tid, int nthreads) {
  if (((ld | c0 | w | sld) & 3) == 0) {
    // 16-byte pieces i = r * q + j; the (r, j) of a thread's next piece follow
    // from one division up front (no division per copy: the issue loop is on
    // the critical path of the attention kernels)
    const int q = w >> 2;
    if (q <= 0 || r1 <= r0) return;
    const int dr = nthreads / q, dj = nthreads - dr * q;
    int r = tid / q, j = tid - r * q;
    const float *s = src + (size_t)(r0 + r) * ld + c0;
    float *d = dst + (size_t)r * sld;
    while (r < r1 - r0) {
      cp_async16(d + 4 * j, s + 4 * j);
      r += dr;
      s += (size_t)dr * ld;
      d += (size_t)dr * sld;
      j += dj;
      if (j >= q) {
        j -= q;
        ++r;
        s += ld;
        d += sld;
      }
    }
  } else {
    for (int i = tid; i < (r1 - r0) * w; i += nthreads) {
      const int r = i / w, c = i - r * w;
      dst[(size_t)r * sld + c] = src[(size_t)(r0 + r) * ld + c0 + c];
    }
  }
}

// Scores of one KV head's query group over one chunk of key positions
// (llama.c:558-565): q and the new k get RoPE here (the chunk holding `pos`
// appends the rotated k to the cache), each score is a sequential dot product
// over the head dimension, times 1/sqrt(hd).  Grid (ceil(max_seq/64), n_kv).
__global__ void __launch_bounds__(kScoreThreads) k_attn_scores(const AttnArgs a) {
  extern __shared__ __align__(16) float sm_s[];
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int kvh = blockIdx.y;
  const int p0 = blockIdx.x * kScoreChunk;
  const int pos = a.step->pos;
  if (pos < 0 || pos >= a.max_seq || p0 > pos) return;  // bad positions are flagged by the QKV epilogue
  const int hd = a.hd, half = hd / 2, group = a.n_heads / a.n_kv;
  const int stride = (hd & 3) == 0 ? hd + 4 : hd + 1;  // padded rows: conflict-free column reads
  const int hd4 = (hd + 3) & ~3;
  float *qs = sm_s;                                  // [group][hd4]
  float *ks = sm_s + (size_t)group * hd4;            // [kScoreChunk][stride]
  const int p1 = min(p0 + kScoreChunk, pos + 1);     // positions [p0, p1)
  const float *kc = a.kcache + (size_t)kvh * a.max_seq * hd;
  // cached keys [p0, min(p1, pos)); the key at `pos` is this step's, rotated below
  stage_rows(ks, stride, kc, hd, p0, min(p1, pos), 0, hd, tid, kScoreThreads);
  cp_async_commit();
  const float *cs = a.rope_cos + (size_t)pos * half, *sn = a.rope_sin + (size_t)pos * half;
  for (int i = tid; i < group * hd; i += kScoreThreads) {
    const int g = i / hd, d = i - g * hd;
    qs[g * hd4 + d] = rope_elem(a.q + (size_t)(kvh * group + g) * hd, d, half, cs, sn);
  }
  if (pos < p1) {
    const float *kn = a.q + (size_t)a.n_heads * hd + (size_t)kvh * hd;
    for (int d = tid; d < hd; d += kScoreThreads) {
      const float kr = rope_elem(kn, d, half, cs, sn);
      ks[(size_t)(pos - p0) * stride + d] = kr;
      a.kcache[((size_t)kvh * a.max_seq + pos) * hd + d] = kr;  // llama.c:551
    }
  }
  cp_async_wait<0>();
  __syncthreads();
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));  // llama.c:532
  for (int i = tid; i < group * kScoreChunk; i += kScoreThreads) {
    const int g = i / kScoreChunk, p = i - g * kScoreChunk;
    if (p0 + p >= p1) continue;
    const float *kr = ks + (size_t)p * stride;
    const float *qr = qs + (size_t)g * hd4;
    // 16-byte loads when the rows allow (rows of hd + 4 floats: the 8 threads
    // of a load phase, 8 consecutive keys, hit distinct banks)
    const float dot = (hd & 3) == 0 ? seq_dot_v4(qr, kr, hd, 0.0f) : seq_dot(qr, kr, 1, hd, 0.0f);  // llama.c:561
    a.scores[(size_t)(kvh * group + g) * a.max_seq + p0 + p] = __fmul_rn(dot, scale);
  }
}

// Softmax and the weighted sum of values for one query head and a slice of
// kPVSlice output dimensions (llama.c:566-575): max; exp; the sequential sum of
// the exponentials; w = e/sum; then for every d the sequential sum over
// positions of w*v.  Value rows stream through a ring of staged chunks.
// Grid (ceil(hd/32), n_heads); needs (max_seq + kPVRing*kPVChunk*kPVSlice)
// floats of dynamic shared memory.
__global__ void __launch_bounds__(kPVThreads) k_attn_pv(const AttnArgs a) {
  extern __shared__ __align__(16) float sm_v[];
  __shared__ float s_red[32];
  __shared__ float s_inv;
  pdl_launch_dependents();
  pdl_wait();
  const int tid = threadIdx.x;
  const int h = blockIdx.y;
  const int d0 = blockIdx.x * kPVSlice;
  const int pos = a.step->pos;
  if (pos < 0 || pos >= a.max_seq) return;
  LLMQ_TSTAMP(0);
  const int np = pos + 1, hd = a.hd, group = a.n_heads / a.n_kv, kvh = h / group;
  const int w = min(kPVSlice, hd - d0);
  float *wts = sm_v;                                          // [max_seq]
  float *ring = sm_v + (((size_t)a.max_seq + 3) & ~size_t(3));  // [kPVRing][kPVChunk][kPVSlice]
  const float *vc = a.vcache + (size_t)kvh * a.max_seq * hd;
  const int nchunks = (np + kPVChunk - 1) / kPVChunk;
  if (a.pv_whole) {
    // The whole slice [0, np) x [d0, d0 + w) is staged while the softmax runs;
    // then w = e * (1/sum) for every position, and one uninterrupted chain per
    // output dimension (one lane each).
    float *vs = ring;  // [np][kPVSlice]
    stage_rows(vs, kPVSlice, vc, hd, 0, np, d0, w, tid, kPVThreads);
    cp_async_commit();
    const float *sc = a.scores + (size_t)h * a.max_seq;
    float m = -INFINITY;
    for (int p = tid; p < np; p += kPVThreads) {
      const float sv = sc[p];
      wts[p] = sv;
      m = fmaxf(m, sv);
    }
    m = block_max<kPVThreads>(m, s_red);
    LLMQ_TSTAMP(1);
    for (int p = tid; p < np; p += kPVThreads) wts[p] = libm_expf(__fsub_rn(wts[p], m));
    __syncthreads();
    LLMQ_TSTAMP(2);
    if (tid == 0) s_inv = __fdiv_rn(1.0f, seq_sum_a16(wts, np, 0.0f));  // llama.c:567
    LLMQ_TSTAMP(3);
    __syncthreads();
    const float inv = s_inv;
    for (int p = tid; p < np; p += kPVThreads) wts[p] = __fmul_rn(wts[p], inv);
    cp_async_wait<0>();
    __syncthreads();
    LLMQ_TSTAMP(4);
    const float o = tid < w ? seq_dot(wts, vs + tid, kPVSlice, np, 0.0f) : 0.0f;  // llama.c:574
    if (tid < w) a.out[(size_t)h * hd + d0 + tid] = o;
    if (a.amax_out && tid < 32) warp_amax_publish(o, a.amax_out);
    LLMQ_TSTAMP(5);
    return;
  }
  // start streaming the value rows while the softmax runs
  for (int c = 0; c < kPVRing; ++c) {
    if (c < nchunks)
      stage_rows(ring + (size_t)c * kPVChunk * kPVSlice, kPVSlice, vc, hd, c * kPVChunk,
                 min((c + 1) * kPVChunk, np), d0, w, tid, kPVThreads);
    cp_async_commit();
  }
  const float *sc = a.scores + (size_t)h * a.max_seq;
  float m = -INFINITY;
  for (int p = tid; p < np; p += kPVThreads) {
    const float s = sc[p];
    wts[p] = s;
    m = fmaxf(m, s);
  }
  m = block_max<kPVThreads>(m, s_red);
  LLMQ_TSTAMP(1);
  for (int p = tid; p < np; p += kPVThreads) wts[p] = libm_expf(__fsub_rn(wts[p], m));
  __syncthreads();
  LLMQ_TSTAMP(2);
  if (tid == 0) {
    const float sum = seq_sum_a16(wts, np, 0.0f);  // llama.c:567
    s_inv = __fdiv_rn(1.0f, sum);
  }
  __syncthreads();
  LLMQ_TSTAMP(3);
  const float inv = s_inv;
  for (int p = tid; p < np; p += kPVThreads) wts[p] = __fmul_rn(wts[p], inv);
  float o = 0.0f;
  for (int c = 0; c < nchunks; ++c) {
    cp_async_wait<kPVRing - 1>();
    __syncthreads();
    const float *buf = ring + (size_t)(c % kPVRing) * kPVChunk * kPVSlice;
    const int pe = min((c + 1) * kPVChunk, np) - c * kPVChunk;
    const float *wc = wts + (size_t)c * kPVChunk;
    if (tid < w) o = seq_dot(wc, buf + tid, kPVSlice, pe, o);  // llama.c:574, in position order
    __syncthreads();
    const int nc = c + kPVRing;
    if (nc < nchunks)
      stage_rows(ring + (size_t)(nc % kPVRing) * kPVChunk * kPVSlice, kPVSlice, vc, hd, nc * kPVChunk,
                 min((nc + 1) * kPVChunk, np), d0, w, tid, kPVThreads);
    cp_async_commit();
  }
  LLMQ_TSTAMP(4);
  if (tid < w) a.out[(size_t)h * hd + d0 + tid] = o;
  if (a.amax_out && tid < 32) warp_amax_publish(tid < w ? o : 0.0f, a.amax_out);
}

// Attention of one query head in one launch (llama.c:558-575), for batch-1
// decode: a cluster of nsl = ceil(hd / 32) CTAs per head, CTA r owning the
// output dimensions [32 r, 32 r + 32) and the key positions [pa, pb) of the
// r-th part of [0, pos].
//  1. The value slice [0, pos) x [32 r, 32 r + 32) and the part's first key
//     chunk are staged before the wait on the QKV product; then q (and, in the
//     part holding `pos`, this step's k) get RoPE, the part's keys stream
//     through a two-chunk ring and each score is the sequential dot product
//     over hd, times 1/sqrt(hd), into e[p] (own shared memory).
//  2. The cluster's maximum: each CTA stores its part's maximum into every
//     CTA (distributed shared memory); after a cluster barrier each takes the
//     maximum, exponentiates its own part and stores it into every CTA's e.
//  3. After a second barrier every CTA holds e[0 .. pos]: the sequential sum,
//     w = e * (1/sum), and one chain per output dimension over the positions.
// The arithmetic and its order are the two-kernel path's (k_attn_scores,
// k_attn_pv), so the outputs are the same bits.
// Shared memory: q and rotated k (2 hd4), e (max_seq, rounded to 4), the value
// slice (max_seq x 32), the key chunks (one or two slots of a.fused_chunk rows
// of hd + 4 (or + 1) floats).
constexpr int kFusedThreads = 256;
__global__ void __launch_bounds__(kFusedThreads) k_attn_fused(const AttnArgs a) {
  extern __shared__ __align__(16) float sm_f[];
  __shared__ float s_red[32];
  __shared__ float s_part_max[8];  // [rank]: stored by that CTA
  __shared__ float s_inv;
  cg::cluster_group cluster = cg::this_cluster();
  LLMQ_TSTAMP(0);
  LLMQ_LAUNCH_ENTER_TAG(2);
  pdl_launch_dependents();
  // Before the wait: the previous kernel (this layer's QKV product) starts its
  // dependents only once all its CTAs are past their own wait, so the step
  // state and the cache rows [0, pos) (written by earlier steps) are final
  // here; only this step's value row `pos` (the QKV epilogue) is read after.
  const int tid = threadIdx.x;
  const int h = blockIdx.y;
  const int nsl = gridDim.x, r = blockIdx.x;  // the cluster spans gridDim.x: rank r = blockIdx.x
  const int pos = a.step->pos;
  if (pos < 0 || pos >= a.max_seq) return;  // same for every CTA of the cluster; flagged by the QKV epilogue
  const int np = pos + 1, hd = a.hd, half = hd / 2, group = a.n_heads / a.n_kv, kvh = h / group;
  const int hd4 = (hd + 3) & ~3, stride = (hd & 3) == 0 ? hd + 4 : hd + 1;
  const int d0 = r * kPVSlice, w = max(0, min(kPVSlice, hd - d0));
  const int pa = (int)((long long)r * np / nsl), pb = (int)((long long)(r + 1) * np / nsl);
  float *qs = sm_f;                                                 // [hd4]
  float *kn = qs + hd4;                                             // [hd4] this step's rotated k
  float *e = kn + hd4;                                              // [max_seq] scores, then exps, then weights
  float *vs = e + (((size_t)a.max_seq + 3) & ~size_t(3));           // [max_seq][32]
  float *kring = vs + (size_t)a.max_seq * kPVSlice;                 // [1 or 2][KC][stride]
  const int KC = a.fused_chunk;
  const float *kc = a.kcache + (size_t)kvh * a.max_seq * hd;
  const float *vc = a.vcache + (size_t)kvh * a.max_seq * hd;
  const int nchunks = (pb - pa + KC - 1) / KC;  // one slot when a part fits in one chunk, else two
  auto stage_keys = [&](int c) {  // cached keys of chunk c (not the row `pos`, rotated below)
    const int r0 = pa + c * KC, r1 = min(pa + (c + 1) * KC, pb);
    stage_rows(kring + (size_t)(c & 1) * KC * stride, stride, kc, hd, r0, min(r1, pos), 0, hd, tid, kFusedThreads);
  };
  // Copy groups: the first key chunk, then the value slice rows [0, pos) (row
  // `pos` is this step's: loaded after the wait), so the scores start once
  // their keys are in; the values keep landing until the weighted sums.
  if (nchunks > 0) stage_keys(0);
  cp_async_commit();
  if (w > 0) stage_rows(vs, kPVSlice, vc, hd, 0, pos, d0, w, tid, kFusedThreads);
  cp_async_commit();
  pdl_wait();
  LLMQ_TSTAMP(1);
  if (tid < w) vs[(size_t)pos * kPVSlice + tid] = vc[(size_t)pos * hd + d0 + tid];  // llama.c:552, this step's v
  const float *cs = a.rope_cos + (size_t)pos * half, *sn = a.rope_sin + (size_t)pos * half;
  const bool own_pos = pos >= pa && pos < pb;
  for (int d = tid; d < hd; d += kFusedThreads) {
    qs[d] = rope_elem(a.q + (size_t)h * hd, d, half, cs, sn);
    if (own_pos) {
      const float kr = rope_elem(a.q + (size_t)a.n_heads * hd + (size_t)kvh * hd, d, half, cs, sn);
      kn[d] = kr;
      if (h % group == 0) a.kcache[((size_t)kvh * a.max_seq + pos) * hd + d] = kr;  // llama.c:551
    }
  }
  const float scale = __fdiv_rn(1.0f, __fsqrt_rn(static_cast<float>(hd)));  // llama.c:532
  float m = -INFINITY;
  for (int c = 0; c < nchunks; ++c) {
    if (c + 1 < nchunks) stage_keys(c + 1);
    cp_async_commit();
    if (c == 0)
      cp_async_wait<2>();  // chunk 0 has landed (the value slice and chunk 1 may still be in flight)
    else
      cp_async_wait<1>();  // chunk c has landed (and everything committed before it)
    __syncthreads();
    const float *ring = kring + (size_t)(c & 1) * KC * stride;
    const int r0 = pa + c * KC, rows = min(KC, pb - r0);
    for (int i = tid; i < rows; i += kFusedThreads) {
      const int p = r0 + i;
      const float *kr = p == pos ? kn : ring + (size_t)i * stride;
      const float dot = (hd & 3) == 0 ? seq_dot_v4(qs, kr, hd, 0.0f) : seq_dot(qs, kr, 1, hd, 0.0f);  // llama.c:561
      const float sv = __fmul_rn(dot, scale);
      e[p] = sv;
      m = fmaxf(m, sv);
    }
    __syncthreads();  // the slot is free for chunk c + 2
  }
  m = block_max<kFusedThreads>(m, s_red);
  LLMQ_TSTAMP(2);
  if (tid < nsl) *cluster.map_shared_rank(&s_part_max[r], tid) = m;  // this part's maximum, into CTA tid
  cluster.sync();  // every part's maximum is in every CTA
  LLMQ_TSTAMP(3);
  for (int q = 0; q < nsl; ++q) m = fmaxf(m, s_part_max[q]);
  for (int p = pa + tid; p < pb; p += kFusedThreads) {
    const float ex = libm_expf(__fsub_rn(e[p], m));  // llama.c:566
    for (int q = 0; q < nsl; ++q) *cluster.map_shared_rank(&e[p], q) = ex;  // into every CTA's e
  }
  cluster.sync();  // every part's exponentials are in every CTA; no remote accesses after this point
  LLMQ_TSTAMP(4);
  if (tid == 0) s_inv = __fdiv_rn(1.0f, seq_sum_a32(e, np, 0.0f));  // llama.c:567
  __syncthreads();
  LLMQ_TSTAMP(5);
  const float inv = s_inv;
  for (int p = tid; p < np; p += kFusedThreads) e[p] = __fmul_rn(e[p], inv);
  cp_async_wait<0>();
  __syncthreads();
  LLMQ_TSTAMP(6);
  const float o = tid < w ? seq_dot_a4(e, vs + tid, kPVSlice, np, 0.0f) : 0.0f;  // llama.c:574
  if (tid < w) a.out[(size_t)h * hd + d0 + tid] = o;
  if (a.amax_out && tid < 32) warp_amax_publish(o, a.amax_out);  // the Wo product's row absmax
  __syncwarp();
  LLMQ_TSTAMP(7);
  LLMQ_LAUNCH_EXIT();
}

// Final step bookkeeping: publish the argmax and error flags, advance the
// device-side token and position (used when steps are chained on the device),
// record the generated id, and reset the argmax cell and error word.
__global__ void k_step_finish(StepState *step, unsigned long long *argmax, int *err, int *result, int *tokens,
                              int max_seq, unsigned *tp_seq, unsigned tp_products, float *amax, int n_amax) {
  LLMQ_LAUNCH_ENTER_TAG(3);
  pdl_wait();
  if (tp_seq) *tp_seq += tp_products;  // the step's row-parallel products are done on this rank
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
  for (int i = 0; i < n_amax; ++i) amax[i] = 0.0f;  // the step's published absmax cells, for the next step
  LLMQ_LAUNCH_EXIT();
}

// ------------------------------------------------------------ utility kernels
// Column absmax and codes of a row-major (rows, cols) matrix (quant.c:10-27):
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

// ---------------------------------------------------- tensor parallelism
// Absmax of a row-parallel product's input over the whole group: this rank's
// absmax (quant.c:69-71) goes to every rank's region, the group maximum of
// all ranks' values to *out.  One CTA.
__global__ void __launch_bounds__(kThreads) k_tp_absmax(const float *x, int n, float *out, TpExchange t, int *err) {
  __shared__ float s_red[32];
  __shared__ int s_bad;
  pdl_launch_dependents();
  pdl_wait();
  float m = 0.0f;
  for (int k = threadIdx.x; k < n; k += kThreads) m = fmaxf(m, fabsf(x[k]));
  m = block_max<kThreads>(m, s_red);
  const unsigned epoch = *t.seq + t.pidx + 1;
  const int par = epoch & 1u;
  const size_t ao = tpx_amax_off(t.world, t.dm), fo = tpx_famax_off(t.world, t.dm);
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  if (threadIdx.x < t.world) {
    char *peer = t.peers[threadIdx.x];
    reinterpret_cast<float *>(peer + ao)[par * t.world + t.rank] = m;
    __threadfence_system();
    st_release_u32(reinterpret_cast<unsigned *>(peer + fo) + t.rank, epoch);
    if (!wait_flag(reinterpret_cast<const unsigned *>(t.peers[t.rank] + fo) + threadIdx.x, epoch, t.poll_limit))
      s_bad = 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    if (s_bad) {
      atomicOr(err, ERR_TIMEOUT);
      return;
    }
    const float *am = reinterpret_cast<const float *>(t.peers[t.rank] + ao) + par * t.world;
    float g = 0.0f;
    for (int q = 0; q < t.world; ++q) g = fmaxf(g, __ldcv(am + q));
    *out = g;
  }
}

// expf of a batch (tests compare this against the host libm over all inputs).
__global__ void k_expf_batch(const float *x, float *y, long long n) {
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x)
    y[i] = libm_expf(x[i]);
}

}  // namespace llmq
