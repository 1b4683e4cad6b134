// llmq_tc_gemm.cuh - the W8A8 product for 64..128 activation rows per launch
// on the 5th-generation tensor cores: tcgen05.mma.kind::i8, int8 x int8 with
// int32 accumulators in tensor memory (TMEM).  Integer sums are exact, so the
// result equals the reference's qmatmul (quant.c:95-120) bit for bit.
//
// Operands, both K-major without swizzle (the canonical core-matrix layout:
// 8 rows x 16 bytes per 128-byte core matrix):
//   B, the weights: the same tiles as k_gemv, [KT/16][256 columns][16 B], so
//     8-column groups are 128 B apart (SBO) and 16-k chunks 4096 B apart (LBO);
//   A, the activation codes: written by k_act_codes as [ktile][KT/16][128 rows][16 B],
//     so 8-row groups are 128 B apart and 16-k chunks 2048 B apart.
// One tcgen05.mma covers M=128 rows, N=256 columns (one slab), K=32.
#pragma once

#include "llmq_kernels.cuh"

namespace llmq {

constexpr int kTcRows = 128;     // MMA M; activation rows are zero-padded to it
constexpr int kTcThreads = 128;  // 4 warps, one per 32 TMEM lanes (rows)
constexpr int kTcMaxStages = 8;
constexpr uint32_t kTcTmemCols = 256;  // one 128 x 256 int32 accumulator

// Instruction descriptor: D int32 (2 << 4), A and B signed int8 (1 << 7, 1 << 10),
// both K-major, N = 256 (N >> 3 at bit 17), M = 128 (M >> 4 at bit 24).
constexpr uint32_t kIdescS8 = (2u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((128u >> 4) << 24);

// Shared-memory matrix descriptor, K-major, no swizzle: start address, leading
// byte offset (between the two 16-byte k chunks of one MMA), stride byte
// offset (between 8-row core-matrix groups), version 1 (bit 46).
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

__device__ __forceinline__ void umma_s8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %3, 0;\n"
      " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %4, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(accumulate), "r"(kIdescS8), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}
// Arrives on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive int32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, int v[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = static_cast<int>(r[i]);
}

// ---------------------------------------------------------------- act codes
// Per-row activation quantisation (quant.c:104-113) for rows [0, rows), written
// as tcgen05 A tiles; rows [rows, 128) get zero codes.  One CTA per row.
__global__ void __launch_bounds__(256) k_act_codes(const float *a, int rows, int K, int Kpad, int KT, int8_t *codes,
                                                   float *as_out) {
  __shared__ float s_red[32];
  const int m = blockIdx.x;
  const int tid = threadIdx.x;
  float as = 1.0f, inv = 1.0f;
  const float *row = a + (size_t)m * K;
  if (m < rows) {
    float mx = 0.0f;
    for (int k = tid; k < K; k += 256) mx = fmaxf(mx, fabsf(row[k]));
    mx = block_max<256>(mx, s_red);
    as = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    inv = __fdiv_rn(1.0f, as);
    if (tid == 0) as_out[m] = as;
  }
  const int chunks_per_tile = KT / 16;
  for (int k = tid; k < Kpad; k += 256) {
    const int8_t c = (m < rows && k < K) ? code_of(__fmul_rn(row[k], inv)) : 0;
    const int kt = k / KT, kc = (k % KT) / 16, kb = k % 16;
    codes[(((size_t)kt * chunks_per_tile + kc) * kTcRows + m) * 16 + kb] = c;
  }
}

// ------------------------------------------------------------------- GEMM
struct TcArgs {
  const uint8_t *w;       // weight tiles, as for k_gemv
  const int8_t *acodes;   // [n_ktiles][KT/16][128][16]
  const float *as;        // per-row activation scales [rows]
  const float *ws;        // per physical column scale [Npad]
  int N, Npad, n_slabs, n_ktiles, stages, rows;
  int *part;              // [gridDim.x][2][128][256] int32 partial sums of split slabs
  int *cnt;               // [n_slabs], zero before and after
  int *err;
  float *out;             // [rows][N]
};

// Which of CTA c's two partial-sum slots holds slab s: 0 if s is the slab of
// the CTA's first tile, else 1.
__device__ __forceinline__ int tc_slot(long long c, long long s, long long T, long long G, long long nk) {
  return ((c * T / G) / nk) == s ? 0 : 1;
}

template <int KT>
__global__ void __launch_bounds__(kTcThreads, 1) k_tc_gemm(const TcArgs a) {
  constexpr int WB = kNT * KT;       // weight tile bytes
  constexpr int AB = kTcRows * KT;   // activation tile bytes
  constexpr int SB = WB + AB;
  constexpr int kMma = KT / 32;      // MMAs per tile
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[kTcMaxStages];
  __shared__ __align__(8) uint64_t empty[kTcMaxStages];
  __shared__ __align__(8) uint64_t accb;
  __shared__ uint32_t s_tmem;
  __shared__ int s_flag, s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = a.stages;
  const long long T = (long long)a.n_slabs * a.n_ktiles;
  const long long G = gridDim.x;
  const long long t_begin = (long long)blockIdx.x * T / G;
  const long long t_end = (long long)(blockIdx.x + 1) * T / G;
  const int n = static_cast<int>(t_end - t_begin);
  const long long nk = a.n_ktiles;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accb, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 0) {  // one warp allocates (and later frees) the accumulator columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  auto issue = [&](int idx, int s, bool weights, bool acts) {
    const long long t = t_begin + idx;
    const long long kt = t % nk;
    uint8_t *dst = sm + (size_t)s * SB;
    if (weights) bulk_load(dst, a.w + (size_t)t * WB, WB, &full[s]);
    if (acts) bulk_load(dst + WB, a.acodes + (size_t)kt * AB, AB, &full[s]);
  };
  int issued = 0;
  if (tid == 0) {  // weights do not depend on the previous kernel: start them now
    for (; issued < n && issued < S; ++issued) {
      mbar_expect_tx(&full[issued], SB);
      issue(issued, issued, true, false);
    }
  }
  pdl_launch_dependents();
  pdl_wait();
  if (tid == 0)
    for (int i = 0; i < issued; ++i) issue(i, i, false, true);

  uint32_t acc_phase = 0;
  bool fresh = true;  // the next MMA overwrites the accumulator

  auto flush = [&](long long slab) {
    if (tid == 0) umma_commit(&accb);
    if (!mbar_wait_bounded(&accb, acc_phase)) s_abort = 1;
    acc_phase ^= 1u;
    tc_fence_after();
    const long long c_first = tile_owner(slab * nk, T, G), c_last = tile_owner((slab + 1) * nk - 1, T, G);
    const bool whole = c_first == c_last;
    const int m = warp * 32 + lane;  // this thread's TMEM lane = output row
    const int p0 = static_cast<int>(slab) * kNT;
    int *slot = a.part + (((size_t)blockIdx.x * 2 + tc_slot(blockIdx.x, slab, T, G, nk)) * kTcRows + m) * kNT;
    for (int cb = 0; cb < kNT / 32; ++cb) {
      int v[32];
      tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(cb * 32), v);
      if (m >= a.rows) continue;
      if (whole) {
        const float as = a.as[m];
#pragma unroll
        for (int q = 0; q < 32; ++q) {
          const int j = p0 + cb * 32 + q;
          if (j < a.N) a.out[(size_t)m * a.N + j] = dequant(as, a.ws[j], v[q]);
        }
      } else {
#pragma unroll
        for (int q = 0; q < 32; q += 4)
          *reinterpret_cast<int4 *>(slot + cb * 32 + q) = make_int4(v[q], v[q + 1], v[q + 2], v[q + 3]);
      }
    }
    tc_fence_before();
    __syncthreads();
    fresh = true;
    if (whole) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) s_flag = atomicAdd(a.cnt + slab, 1) == static_cast<int>(c_last - c_first);
    __syncthreads();
    if (!s_flag) return;
    __threadfence();
    // last of the slab's CTAs: add the partial sums (exact in any order) and rescale
    if (m < a.rows) {
      const float as = a.as[m];
      for (int j0 = 0; j0 < kNT; j0 += 4) {
        int4 sum = make_int4(0, 0, 0, 0);
        for (long long c = c_first; c <= c_last; ++c) {
          const int4 p = *reinterpret_cast<const int4 *>(
              a.part + (((size_t)c * 2 + tc_slot(c, slab, T, G, nk)) * kTcRows + m) * kNT + j0);
          sum.x += p.x;
          sum.y += p.y;
          sum.z += p.z;
          sum.w += p.w;
        }
        const int vv[4] = {sum.x, sum.y, sum.z, sum.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int j = p0 + j0 + q;
          if (j < a.N) a.out[(size_t)m * a.N + j] = dequant(as, a.ws[j], vv[q]);
        }
      }
    }
    if (tid == 0) a.cnt[slab] = 0;
    __syncthreads();
  };

  long long slab = t_begin / nk;
  int kt = static_cast<int>(t_begin - slab * nk);
  long long cur = n > 0 ? slab : -1;
  int s = 0, sp = 0;
  uint32_t phase = 0, phase_p = 0;
  for (int i = 0; i < n; ++i) {
    if (i > 0 && ++kt == a.n_ktiles) {
      kt = 0;
      ++slab;
    }
    if (slab != cur) {
      flush(cur);
      cur = slab;
    }
    if (tid == 0 && !s_abort) {
      if (!mbar_wait_bounded(&full[s], phase)) {
        s_abort = 1;
      } else {
        tc_fence_after();
        const uint32_t wbase = smem_addr(sm + (size_t)s * SB), abase = wbase + WB;
#pragma unroll
        for (int j = 0; j < kMma; ++j) {
          const uint64_t ad = umma_desc(abase + j * 2 * (kTcRows * 16), kTcRows * 16, 128);
          const uint64_t bd = umma_desc(wbase + j * 2 * (kNT * 16), kNT * 16, 128);
          umma_s8(tmem, ad, bd, (fresh && j == 0) ? 0u : 1u);
        }
        fresh = false;
        umma_commit(&empty[s]);
        // refill the stage of the previous tile once its MMAs have read it
        if (i > 0 && issued < n) {
          if (!mbar_wait_bounded(&empty[sp], phase_p)) {
            s_abort = 1;
          } else {
            mbar_expect_tx(&full[sp], SB);
            issue(issued, sp, true, true);
            ++issued;
          }
        }
      }
    }
    fresh = false;
    if (i > 0 && ++sp == S) {
      sp = 0;
      phase_p ^= 1u;
    }
    if (++s == S) {
      s = 0;
      phase ^= 1u;
    }
    if (((i + 1) & 15) == 0 || i + 1 == n) {  // keep all threads in step with thread 0
      __syncthreads();
      if (s_abort) break;
    }
  }
  if (!s_abort && n > 0) flush(cur);
  // drain: every MMA this CTA issued must be finished before the columns go back
  if (tid == 0) {
    umma_commit(&accb);
    mbar_wait_bounded(&accb, acc_phase);
    if (s_abort) atomicOr(a.err, ERR_TIMEOUT);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
}

}  // namespace llmq
