// llmq_tc_gemm.cuh - the W8A8 product for 64..128 activation rows per launch
// on the 5th-generation tensor cores: tcgen05.mma.kind::i8, int8 x int8 with
// int32 accumulators in tensor memory (TMEM).  Integer sums are exact, so the
// result equals the reference's qmatmul (quant.c:60-85) bit for bit.
//
// Operands, both K-major without swizzle (the canonical core-matrix layout:
// 8 rows x 16 bytes per 128-byte core matrix):
//   B, the weights: the same tiles as k_gemv, [KT/16][256 columns][16 B], so
//     8-column groups are 128 B apart (SBO) and 16-k chunks 4096 B apart (LBO);
//   A, the activation codes: written by k_act_codes as [row block][ktile][KT/16][128 rows][16 B],
//     so 8-row groups are 128 B apart and 16-k chunks 2048 B apart.
// One tcgen05.mma covers M=128 rows, N=256 columns (one slab), K=32.
#pragma once

#include "llmq_kernels.cuh"

namespace llmq {

constexpr int kTcRows = 128;     // MMA M; activation rows are zero-padded to it
constexpr int kTcThreads = 128;  // 4 warps, one per 32 TMEM lanes (rows)
constexpr int kTcMaxStages = 8;
constexpr int kTcRingBytes = 98304;  // ring per CTA: two CTAs (and 2 x 256 TMEM columns) per SM
constexpr int kTcStageBytes = 64 * (256 + 1) * 4;  // the epilogue stages 64 accumulator rows in the ring
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
// Activation codes of row m live in 128-row block m / 128, laid out as tcgen05
// A tiles: [block][ktile][KT/16][128 rows][16 B] (block stride 128 * Kpad).
__device__ __forceinline__ size_t tc_code_offset(int m, int chunk, int Kpad, int KT) {
  const int rb = m / kTcRows, mm = m - rb * kTcRows;
  const int per_tile = KT / 16;
  const int kt = chunk / per_tile, kc = chunk - kt * per_tile;
  return (size_t)rb * kTcRows * Kpad + (((size_t)kt * per_tile + kc) * kTcRows + mm) * 16;
}

// Codes of 16 consecutive values x[0..16) (k >= K gives 0) times `inv`
// (quant.c:73-77), packed little-endian into one 16-byte chunk.
__device__ __forceinline__ int4 tc_pack16(const float *x, int k0, int K, float inv) {
  uint32_t w[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint32_t v = 0;
#pragma unroll
    for (int b = 0; b < 4; ++b) {
      const int k = k0 + q * 4 + b;
      const int8_t c = k < K ? code_of(__fmul_rn(x[k], inv)) : 0;
      v |= (uint32_t)(uint8_t)c << (8 * b);
    }
    w[q] = v;
  }
  return make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
}

// Per-row activation quantisation (quant.c:69-78) of rows [0, rows) of a
// (row stride K), written as tcgen05 A tiles; the row's absmax comes from
// absmax_in when given.  One CTA per row.
__global__ void __launch_bounds__(256) k_act_codes(const float *a, int rows, int K, int Kpad, int KT, int8_t *codes,
                                                   float *as_out, const float *absmax_in) {
  LLMQ_LAUNCH_SPAN(20);
  __shared__ float s_red[32];
  pdl_launch_dependents();
  pdl_wait();
  const int m = blockIdx.x;
  const int tid = threadIdx.x;
  const float *row = a + (size_t)m * K;
  float mx = 0.0f;
  if (absmax_in) {  // a row-parallel shard: the absmax of the whole row, reduced over the ranks
    mx = absmax_in[m];
  } else {
    for (int k = tid; k < K; k += 256) mx = fmaxf(mx, fabsf(row[k]));
    mx = block_max<256>(mx, s_red);
  }
  const float as = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  const float inv = __fdiv_rn(1.0f, as);
  if (tid == 0) as_out[m] = as;
  for (int ch = tid; ch < Kpad / 16; ch += 256)
    *reinterpret_cast<int4 *>(codes + tc_code_offset(m, ch, Kpad, KT)) = tc_pack16(row, ch * 16, K, inv);
}

// Absmax of each row of a (row stride K), the local part of a row-parallel
// product's activation scale (quant.c:69-71).  One CTA per row.
__global__ void __launch_bounds__(256) k_rows_absmax(const float *a, int K, float *out) {
  LLMQ_LAUNCH_SPAN(21);
  __shared__ float s_red[32];
  pdl_launch_dependents();
  pdl_wait();
  const float *row = a + (size_t)blockIdx.x * K;
  float mx = 0.0f;
  for (int k = threadIdx.x; k < K; k += 256) mx = fmaxf(mx, fabsf(row[k]));
  mx = block_max<256>(mx, s_red);
  if (threadIdx.x == 0) out[blockIdx.x] = mx;
}

// ------------------------------------------------------------------- GEMM
// Epilogues applied to y = a_scale[m] * w_scale[p] * acc (quant.c:82) of
// physical column p of the tiled matrix.
enum TcEpilogue : int {
  TC_PLAIN = 0,   // out[m][p] = y                                  (qmatmul)
  TC_BIAS = 1,    // out[m][p] = y + bias[p]                        (q/k/v, llama.c:546-548)
  TC_RESID = 2,   // out[m][p] += y                                 (Wo, W2: llama.c:578, 589)
  TC_SWIGLU = 3,  // slab = 128 gate + 128 up columns: out[m][slab*128 + c] = SiLU(gate) * up (llama.c:583-587)
  TC_LOGITS = 4   // TC_PLAIN plus the first maximum of each row into argmax[m]   (sampler.c:8-21)
};

struct TcArgs {
  const uint8_t *w;       // weight tiles, as for k_gemv
  const int8_t *acodes;   // see tc_code_offset
  const float *as;        // per-row activation scales [rows]
  const float *ws;        // per physical column scale [Npad]
  const float *bias;      // TC_BIAS, physical order
  int N;                  // valid physical columns (TC_SWIGLU: output columns)
  int Npad, n_slabs, n_ktiles, n_rb, splits, stages, rows, epi;
  int *acc;               // splits > 1: [rows][Npad] int32, zero before and after (k_tc_epilogue)
  int *err;
  unsigned long long *argmax;  // TC_LOGITS: [rows] keys, zero before the launch
  int idx_offset;         // TC_LOGITS: global index of column 0 (vocab shard)
  int acc_only;           // leave the int32 sums in `acc` (a row-parallel shard's partials)
  float *out;             // [rows][ld]
  int ld;                 // row stride of out
};

// Epilogue of row m for columns lane + 32 i (i < 8) of one slab; v[i] is the
// exact int32 dot product of that column.
__device__ __forceinline__ void tc_epilogue_lane(const TcArgs &a, int m, int slab, int lane, const int v[8]) {
  const int p0 = slab * kNT;
  const float as = a.as[m];
  float *orow = a.out + (size_t)m * a.ld;
  if (a.epi == TC_SWIGLU) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = lane + 32 * i, j = slab * (kNT / 2) + c;
      if (j < a.N) {
        const float z = dequant(as, a.ws[p0 + c], v[i]);
        const float u = dequant(as, a.ws[p0 + kNT / 2 + c], v[i + 4]);
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, libm_expf(-z)));  // llama.c:585
        orow[j] = __fmul_rn(__fmul_rn(z, sg), u);                          // llama.c:586
      }
    }
    return;
  }
  unsigned long long best = 0ull;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int j = p0 + lane + 32 * i;
    if (j < a.N) {
      const float y = dequant(as, a.ws[j], v[i]);
      if (a.epi == TC_BIAS) {
        orow[j] = __fadd_rn(y, a.bias[j]);
      } else if (a.epi == TC_RESID) {
        orow[j] = __fadd_rn(orow[j], y);
      } else {
        orow[j] = y;
        if (a.epi == TC_LOGITS) {
          const unsigned long long key = argmax_key(y, static_cast<uint32_t>(j + a.idx_offset));
          best = key > best ? key : best;
        }
      }
    }
  }
  if (a.epi == TC_LOGITS) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
      best = other > best ? other : best;
    }
    if (lane == 0) atomicMax(a.argmax + m, best);
  }
}

__device__ __forceinline__ void red_add_s32(int *p, int v) {
  asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// CTA (slab, row block, split) computes the 128 x 256 block of one 256-column
// slab and 128-row block over k tiles [split*nk/splits, (split+1)*nk/splits).
// Thread 0 streams (weight, activation) tile pairs through a ring and issues
// the MMAs.  The accumulator then goes TMEM -> shared memory (64 rows at a
// time) so that every warp works on whole rows: with one split it applies the
// epilogue directly; otherwise it adds the block into `acc` (integer adds: the
// order does not matter) and k_tc_epilogue, the next launch, applies it.
template <int KT>
__global__ void __launch_bounds__(kTcThreads) k_tc_gemm(const TcArgs a) {
  LLMQ_LAUNCH_SPAN(22);
  constexpr int WB = kNT * KT;       // weight tile bytes
  constexpr int AB = kTcRows * KT;   // activation tile bytes
  constexpr int SB = WB + AB;
  constexpr int kMma = KT / 32;      // MMAs per tile
  constexpr int kLd = kNT + 1;       // staged accumulator row stride (words): conflict-free
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ __align__(8) uint64_t full[kTcMaxStages];
  __shared__ __align__(8) uint64_t empty[kTcMaxStages];
  __shared__ __align__(8) uint64_t accb;
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = a.stages;
  const int split = blockIdx.x % a.splits;
  const int tile = blockIdx.x / a.splits;  // row blocks of one slab are neighbours: the slab is read once
  const int rb = tile % a.n_rb, slab = tile / a.n_rb;
  const int row0 = rb * kTcRows, rows_here = min(kTcRows, a.rows - row0);
  const int kt0 = (int)((long long)split * a.n_ktiles / a.splits);
  const int kt1 = (int)((long long)(split + 1) * a.n_ktiles / a.splits);
  const int n = kt1 - kt0;

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accb, 1);
    fence_mbar_init();
    s_abort = 0;
  }
  if (warp == 0) {  // one warp allocates (and at the end frees) the accumulator columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(&s_tmem)),
                 "r"(kTcTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  const uint8_t *wsrc = a.w + ((size_t)slab * a.n_ktiles + kt0) * WB;
  const int8_t *asrc = a.acodes + (size_t)rb * kTcRows * a.n_ktiles * KT + (size_t)kt0 * AB;
  if (tid == 0) {  // weights do not depend on the previous kernel: start them now
    for (int i = 0; i < n && i < S; ++i) {
      mbar_expect_tx(&full[i], SB);
      bulk_load(sm + (size_t)i * SB, wsrc + (size_t)i * WB, WB, &full[i]);
    }
  }
  pdl_launch_dependents();
  pdl_wait();
  if (tid == 0) {
    for (int i = 0; i < n && i < S; ++i) bulk_load(sm + (size_t)i * SB + WB, asrc + (size_t)i * AB, AB, &full[i]);
    int issued = min(n, S), i = 0, s = 0, ps = S - 1;
    uint32_t phase = 0, pphase = 1;  // ring position of tile i and of tile i - 1
    for (; i < n; ++i) {
      if (!mbar_wait_bounded(&full[s], phase)) {
        s_abort = 1;
        break;
      }
      tc_fence_after();
      const uint32_t wbase = smem_addr(sm + (size_t)s * SB), abase = wbase + WB;
#pragma unroll
      for (int j = 0; j < kMma; ++j) {
        const uint64_t ad = umma_desc(abase + j * 2 * (kTcRows * 16), kTcRows * 16, 128);
        const uint64_t bd = umma_desc(wbase + j * 2 * (kNT * 16), kNT * 16, 128);
        umma_s8(tmem, ad, bd, (i > 0 || j > 0) ? 1u : 0u);
      }
      umma_commit(&empty[s]);
      // Refill the stage of tile i - 1 (whose MMAs ran while these were issued)
      // with tile i - 1 + S.
      if (i > 0 && i - 1 + S < n) {
        if (!mbar_wait_bounded(&empty[ps], pphase)) {
          s_abort = 1;
          ++i;
          break;
        }
        mbar_expect_tx(&full[ps], SB);
        bulk_load(sm + (size_t)ps * SB, wsrc + (size_t)(i - 1 + S) * WB, WB, &full[ps]);
        bulk_load(sm + (size_t)ps * SB + WB, asrc + (size_t)(i - 1 + S) * AB, AB, &full[ps]);
        ++issued;
      }
      ps = s;
      pphase = phase;
      if (++s == S) {
        s = 0;
        phase ^= 1u;
      }
    }
    // After a timeout, wait (bounded) for the copies still landing in the ring.
    for (int t = i; t < issued; ++t) mbar_wait_bounded(&full[t % S], (uint32_t)(t / S) & 1u);
    umma_commit(&accb);  // arrives when every MMA above is done
  }
  if (!mbar_wait_bounded(&accb, 0)) s_abort = 1;
  tc_fence_after();
  __syncthreads();  // s_abort is final; the ring is free for staging
  const bool ok = !s_abort;
  const bool direct = a.splits == 1 && !a.acc_only;
  int *stg = reinterpret_cast<int *>(sm);  // [64][kLd]
  const int p0 = slab * kNT;
  for (int g = 0; g < 2 && g * 64 < rows_here; ++g) {
    if ((warp >> 1) == g) {  // warps 2g, 2g+1 own TMEM lanes (rows) [64g, 64g + 64)
      const int lr = (warp & 1) * 32 + lane;
#pragma unroll 1
      for (int cb = 0; cb < kNT / 32; ++cb) {
        int v[32];
        tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(cb * 32), v);
#pragma unroll
        for (int q = 0; q < 32; ++q) stg[lr * kLd + cb * 32 + q] = v[q];
      }
    }
    __syncthreads();
    const int nr = min(64, rows_here - g * 64);
    if (ok) {
      for (int r = warp; r < nr; r += kTcThreads / 32) {
        const int m = row0 + g * 64 + r;
        const int *vr = stg + r * kLd;
        if (direct) {
          int v[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = vr[lane + 32 * i];
          tc_epilogue_lane(a, m, slab, lane, v);
        } else {
          int *accr = a.acc + (size_t)m * a.Npad + p0;
#pragma unroll
          for (int i = 0; i < 8; ++i) red_add_s32(accr + lane + 32 * i, vr[lane + 32 * i]);
        }
      }
    }
    __syncthreads();
  }
  if (tid == 0 && !ok) atomicOr(a.err, ERR_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
}

// Epilogue of a split-K product: one warp per (row, slab) takes the summed
// int32 block from `acc`, re-zeroes it and applies the epilogue.
// Grid ceil(rows * n_slabs / 4) x 128 threads.
__global__ void __launch_bounds__(128) k_tc_epilogue(const TcArgs a) {
  LLMQ_LAUNCH_SPAN(23);
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int gw = blockIdx.x * 4 + (threadIdx.x >> 5);
  if (gw >= a.rows * a.n_slabs) return;
  const int m = gw % a.rows, slab = gw / a.rows;
  int *accr = a.acc + (size_t)m * a.Npad + slab * kNT;
  int v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __ldcg(accr + lane + 32 * i);
#pragma unroll
  for (int i = 0; i < 8; ++i) __stcg(accr + lane + 32 * i, 0);
  tc_epilogue_lane(a, m, slab, lane, v);
}

}  // namespace llmq
