// llmq_noalloc.cu - qmatmul_device_noalloc: the W8A8 product on buffers the
// caller already holds on the GPU, with no device allocation at all.
//
// Who needs it: callers that cannot call cudaMalloc where they multiply, such
// as a host framework whose own memory pool already owns the GPU's memory (a
// further cudaMalloc fails or fragments it), a plugin that must not change the
// host application's device-memory accounting, or a latency-critical loop where
// an allocation, and the device synchronisation of the matching cudaFree, cannot
// be afforded.  The caller passes device pointers for A, W (the reference's
// (in, out) row-major int8 codes plus per-column scales) and C; the only
// scratch, the split-K int32 partial sums, the per-slab arrival counters and
// the row's activation scale, lives in one file-scope __device__ array of
// fixed size.
//
// Arithmetic is the reference's qmatmul (quant.c:60-85): per-row absmax
// activation codes, exact int32 products, c = a_scale * w_scale[j] * (float)acc.
#include <cuda_runtime.h>

#include "llmq_device_common.cuh"
#include "llmq_internal.h"

namespace {

constexpr int kNaMaxN = 131072;              // largest N (covers a 128256 vocab)
constexpr int kNaSlab = 256;                 // output columns per CTA
constexpr int kNaMaxSlabs = kNaMaxN / kNaSlab;
constexpr int kNaKChunk = 256;               // k rows per CTA (split-K)
constexpr int kNaThreads = 256;
constexpr int kNaScaleWord = kNaMaxN + kNaMaxSlabs;  // the row's activation scale (f32 bits)

// acc[kNaMaxN], cnt[kNaMaxSlabs], then one word for the row's activation
// scale: 513 KiB, held by every GPU that loads the library until the process
// exits.  Host code must not pass this name to a kernel (on the host it is only
// a stand-in); it passes the address cudaGetSymbolAddress returns.
static __device__ __align__(256) int g_noalloc_scratch[kNaMaxN + kNaMaxSlabs + 64];

// Four rows w0..w3 of four int8 columns each -> four words, word c holding the
// column c values of rows 0..3 (dp4a operand order).
__device__ __forceinline__ void transpose4x4(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3, uint32_t c[4]) {
  const uint32_t lo01 = __byte_perm(w0, w1, 0x5140), hi01 = __byte_perm(w0, w1, 0x7362);
  const uint32_t lo23 = __byte_perm(w2, w3, 0x5140), hi23 = __byte_perm(w2, w3, 0x7362);
  c[0] = __byte_perm(lo01, lo23, 0x5410);
  c[1] = __byte_perm(lo01, lo23, 0x7632);
  c[2] = __byte_perm(hi01, hi23, 0x5410);
  c[3] = __byte_perm(hi01, hi23, 0x7632);
}

__device__ __forceinline__ uint32_t load4(const int8_t *w, long long K, int N, long long k, int j, bool aligned) {
  if (k >= K) return 0u;
  const int8_t *p = w + k * N + j;
  if (aligned && j + 3 < N) return *reinterpret_cast<const uint32_t *>(p);
  uint32_t v = 0;
  for (int b = 0; b < 4; ++b)
    if (j + b < N) v |= (uint32_t)(uint8_t)p[b] << (8 * b);
  return v;
}

// The activation scale of one row (quant.c:69-71), computed once per row by one
// CTA so that the product's CTAs each read only their own k rows of A.
__global__ void __launch_bounds__(kNaThreads) k_qmm_row_scale(const float *__restrict__ a, int K, int *scratch) {
  __shared__ float s_red[32];
  float m = 0.0f;
  for (int k = threadIdx.x; k < K; k += kNaThreads) m = fmaxf(m, fabsf(a[k]));
  m = llmq::block_max<kNaThreads>(m, s_red);
  if (threadIdx.x == 0) scratch[kNaScaleWord] = __float_as_int(m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f);
}

// One row of C.  Grid (ceil(N/256), ceil(K/256)): CTA (slab, split) multiplies
// k rows [split*256, +256) of columns [slab*256, +256); the CTA that completes a
// slab's splits applies the epilogue and re-zeroes the slab's scratch.
__global__ void __launch_bounds__(kNaThreads) k_qmm_noalloc(const float *__restrict__ a, const int8_t *__restrict__ w,
                                                             const float *__restrict__ ws, float *__restrict__ c,
                                                             int K, int N, int *scratch) {
  __shared__ __align__(16) int8_t codes[kNaKChunk];
  __shared__ int red[kNaThreads * 4];
  __shared__ int s_last;
  int *acc = scratch;
  int *cnt = scratch + kNaMaxN;
  const int tid = threadIdx.x;
  const int slab = blockIdx.x;
  const long long k0 = (long long)blockIdx.y * kNaKChunk;
  // codes of this CTA's k rows with the row's scale (quant.c:72-78)
  const float as = __int_as_float(scratch[kNaScaleWord]);
  const float inv = __fdiv_rn(1.0f, as);
  for (int i = tid; i < kNaKChunk; i += kNaThreads) {
    const long long k = k0 + i;
    codes[i] = k < K ? llmq::code_of(__fmul_rn(a[k], inv)) : 0;
  }
  __syncthreads();
  // thread -> 4 adjacent columns, and every 4th group of 4 k rows
  const int cq = tid & 63, kg0 = tid >> 6;
  const int j = slab * kNaSlab + 4 * cq;
  const bool aligned = (N & 3) == 0 && (reinterpret_cast<uintptr_t>(w) & 3) == 0;
  int s[4] = {0, 0, 0, 0};
  if (j < N) {
    for (int kg = kg0; kg < kNaKChunk / 4; kg += 4) {
      const long long k = k0 + 4LL * kg;
      if (k >= K) break;
      uint32_t col[4];
      transpose4x4(load4(w, K, N, k, j, aligned), load4(w, K, N, k + 1, j, aligned),
                   load4(w, K, N, k + 2, j, aligned), load4(w, K, N, k + 3, j, aligned), col);
      const int act = *reinterpret_cast<const int *>(codes + 4 * kg);
#pragma unroll
      for (int q = 0; q < 4; ++q) s[q] = __dp4a(static_cast<int>(col[q]), act, s[q]);
    }
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) red[tid * 4 + q] = s[q];
  __syncthreads();
  if (kg0 == 0 && j < N) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int v = red[tid * 4 + q] + red[(tid + 64) * 4 + q] + red[(tid + 128) * 4 + q] + red[(tid + 192) * 4 + q];
      if (j + q < N) atomicAdd(acc + j + q, v);
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = atomicAdd(cnt + slab, 1) == static_cast<int>(gridDim.y) - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int jj = slab * kNaSlab + tid; jj < min(N, (slab + 1) * kNaSlab); jj += kNaThreads)
    c[jj] = llmq::dequant(as, ws[jj], atomicExch(acc + jj, 0));  // quant.c:82
  if (tid == 0) cnt[slab] = 0;
}

}  // namespace

extern "C" LLMQ_API int qmatmul_device_noalloc(const float *A, int M, int K, const signed char *Wq,
                                               const float *Wscale, int N, float *C, void *stream) {
  if (M < 0 || K < 0 || N < 0) {
    llmq_set_error(LLMQ_ERR_ARG, "qmatmul_device_noalloc: negative size (M=%d K=%d N=%d)", M, K, N);
    return LLMQ_ERR_ARG;
  }
  if (N > kNaMaxN) {
    llmq_set_error(LLMQ_ERR_ARG, "qmatmul_device_noalloc: N=%d exceeds the static scratch limit of %d columns", N,
                   kNaMaxN);
    return LLMQ_ERR_ARG;
  }
  if (M == 0 || N == 0) return LLMQ_OK;
  if (!C || !Wscale || (K > 0 && (!A || !Wq))) {
    llmq_set_error(LLMQ_ERR_ARG, "qmatmul_device_noalloc: null device pointer");
    return LLMQ_ERR_ARG;
  }
  // The array's device address, looked up on every call with the caller's
  // device and context current (the host-side symbol is only a stand-in).  No
  // copy of it is kept: one taken earlier would be stale after a
  // cudaDeviceReset or under another context, and a per-device table would be
  // shared by the caller's threads.
  int *scratch = nullptr;
  cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void **>(&scratch), g_noalloc_scratch);
  if (e != cudaSuccess || !scratch) {
    llmq_set_error(e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? LLMQ_ERR_NO_DEVICE : LLMQ_ERR_CUDA,
                   "qmatmul_device_noalloc: cudaGetSymbolAddress failed (%s)", cudaGetErrorString(e));
    return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver ? LLMQ_ERR_NO_DEVICE : LLMQ_ERR_CUDA;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int slabs = (N + kNaSlab - 1) / kNaSlab;
  // The array keeps the last call's contents: clear the words this call sums into.
  e = cudaMemsetAsync(scratch, 0, (size_t)slabs * kNaSlab * sizeof(int), st);
  if (e == cudaSuccess) e = cudaMemsetAsync(scratch + kNaMaxN, 0, (size_t)slabs * sizeof(int), st);
  const dim3 grid(slabs, K > 0 ? (K + kNaKChunk - 1) / kNaKChunk : 1);
  for (int r = 0; r < M && e == cudaSuccess; ++r) {
    const float *ar = K > 0 ? A + (size_t)r * K : A;
    k_qmm_row_scale<<<1, kNaThreads, 0, st>>>(ar, K, scratch);
    e = cudaGetLastError();
    if (e != cudaSuccess) break;
    k_qmm_noalloc<<<grid, kNaThreads, 0, st>>>(ar, reinterpret_cast<const int8_t *>(Wq), Wscale, C + (size_t)r * N, K,
                                                N, scratch);
    e = cudaGetLastError();
  }
  if (e != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "qmatmul_device_noalloc: launch failed (%s)", cudaGetErrorString(e));
    return LLMQ_ERR_CUDA;
  }
  return LLMQ_OK;
}
