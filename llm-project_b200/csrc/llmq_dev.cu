// llmq_dev.cu - CUDA runtime layer of libllmq_cuda.so: device contexts, weight
// upload and tiling, the per-(model, cache) decode graphs, and the launchers of
// the kernels in llmq_kernels.cuh.  Called only through llmq_internal.h.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <unordered_map>
#include <thread>
#include <vector>

#include "llmq_internal.h"
#include "llmq_kernels.cuh"
#include "llmq_tc_gemm.cuh"
#include "llmq_rows.cuh"
#include "llmq_sample.cuh"
#include "llmq_f32.cuh"

using namespace llmq;

extern "C" const uint32_t llmq_expf_exceptions[];
extern "C" const uint32_t llmq_expf_exceptions_count;

#define CK(call)                                                                                       \
  do {                                                                                                 \
    cudaError_t e_ = (call);                                                                           \
    if (e_ != cudaSuccess) {                                                                           \
      llmq_set_error(LLMQ_ERR_CUDA, "%s: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
      return 0;                                                                                        \
    }                                                                                                  \
  } while (0)

namespace {

constexpr int kMaxDevices = 64;

size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

// Zeroes device memory and waits until it is done.  cudaMemset runs on the
// legacy default stream, which the library's non-blocking streams do not wait
// for: without the wait, a kernel on a model or context stream could run
// before (or during) the zeroing.
cudaError_t zero_sync(void *p, size_t bytes) {
  const cudaError_t e = cudaMemset(p, 0, bytes);
  return e != cudaSuccess ? e : cudaStreamSynchronize(nullptr);
}
// Host -> device copy that has landed on return.  A cudaMemcpy from pageable
// host memory may return before its last DMA completes, on the legacy stream,
// which the library's non-blocking streams do not wait for.
cudaError_t upload_sync(void *dst, const void *src, size_t bytes) {
  const cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
  return e != cudaSuccess ? e : cudaStreamSynchronize(nullptr);
}
int roundup(int v, int m) { return (v + m - 1) / m * m; }

// Tile depth: 32 KB tiles (KT 128) once a matrix spans at least 16 of them per
// SM, else 16 KB tiles (KT 64) so the contiguous split stays balanced.
// Tile depth: 32 KB tiles (KT 128) whenever a GEMV of `rows` rows still fits
// two of them in shared memory next to its codes and input row, else 16 KB
// tiles (KT 64).  Deeper tiles halve the per-tile costs of the ring.
int choose_kt(int K, int rows) {
  if (K < 128) return 64;
  const size_t need = (size_t)rows * roundup(K, 128) + 8 * (size_t)roundup(K, 4) + 2 * (32768 + 16) + 4096;
  return need <= 220 * 1024 ? 128 : 64;
}

// ------------------------------------------------------------------ context
struct Mat {
  uint8_t *w = nullptr;
  float *ws = nullptr;
  int K = 0, Kpad = 0, N = 0, Npad = 0, NT = 0, KT = 64, n_slabs = 0, n_ktiles = 0;
  size_t bytes() const { return (size_t)Kpad * Npad; }
};

struct DevCtx {
  bool ready = false;
  int device = -1;
  int num_sms = 0;
  int max_smem = 0;  // dynamic shared memory available to one CTA
  cudaStream_t stream = nullptr;
  uint32_t *expf_keys = nullptr;
  // qmatmul scratch (grow-only; acc/cnt kept zero between launches)
  float *dA = nullptr, *dC = nullptr;
  size_t dA_n = 0, dC_n = 0;
  int *acc = nullptr, *cnt = nullptr, *err = nullptr;
  size_t acc_n = 0, cnt_n = 0;
  uint8_t *wraw = nullptr, *wtile = nullptr;
  float *wscale = nullptr;
  size_t wraw_n = 0, wtile_n = 0, wscale_n = 0;
  // tensor-core path scratch: activation codes, row scales, split-K sums (kept
  // zero between launches)
  int8_t *tc_codes = nullptr;
  float *tc_as = nullptr;
  int *tc_acc = nullptr;
  size_t tc_codes_n = 0, tc_as_n = 0, tc_acc_n = 0;
  // standalone sampler: state, id, row and scratch
  char *sample_buf = nullptr;
  size_t sample_n = 0;
};

DevCtx g_ctx[kMaxDevices];
std::recursive_mutex g_mu;
// Programmatic dependent launch between the kernels of a step (LLMQ_NO_PDL=1
// turns it off, for measurements).
bool pdl_enabled() {
  static const bool on = [] {
    const char *e = getenv("LLMQ_NO_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}

void free_mat(Mat &m) {
  cudaFree(m.w);
  cudaFree(m.ws);
  m = Mat{};
}

// An fp32 matrix of the LLMA path: tiles of 32 columns, each a contiguous
// [K][32] block (llmq_f32.cuh), split over a grid of `grid` CTAs.
struct MatF {
  float *w = nullptr;
  int *cta_t0 = nullptr;
  int K = 0, N = 0, grid = 0, threads = 0, rows = 0, slots = 0;
  int tw = 32;  // tile width: output columns per warp
  size_t smem = 0;
};

void free_matf(MatF &m) {
  cudaFree(m.w);
  cudaFree(m.cta_t0);
  m = MatF{};
}

// Every kernel asks for the largest shared-memory carveout, so consecutive
// launches with different shared-memory needs never make an SM repartition
// its L1 / shared memory between them.
// The dynamic limit is `smem`, or less where the kernel's static shared memory
// leaves less of the per-block maximum `optin`.
int g_smem_optin = 0;
long long g_launches = 0;       // kernels launched by the running multi-row call
long long g_last_launches = 0;  // ... by the last completed one

// ------------------------------------------------------ tensor parallelism
// One process per GPU; the ranks of a tensor-parallel group share an NCCL
// communicator.  NCCL is loaded when the group is formed, so single-GPU use
// never needs it.
struct NcclApi {
  void *h = nullptr;
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
} g_nccl;

struct TpGroup {
  int rank = 0, world = 1, device = -1;
  ncclComm_t comm = nullptr;
} g_tp;

int load_nccl() {
  if (g_nccl.h) return 1;
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) {
    llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: tensor parallelism needs libnccl.so.2 (%s)", dlerror());
    return 0;
  }
#define LLMQ_NCCL_SYM(field, name)                                                        \
  g_nccl.field = reinterpret_cast<decltype(g_nccl.field)>(dlsym(h, name));              \
  if (!g_nccl.field) {                                                                  \
    llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: libnccl.so.2 lacks %s", name);         \
    return 0;                                                                           \
  }
  LLMQ_NCCL_SYM(GetUniqueId, "ncclGetUniqueId")
  LLMQ_NCCL_SYM(CommInitRank, "ncclCommInitRank")
  LLMQ_NCCL_SYM(AllReduce, "ncclAllReduce")
  LLMQ_NCCL_SYM(AllGather, "ncclAllGather")
  LLMQ_NCCL_SYM(CommDestroy, "ncclCommDestroy")
  LLMQ_NCCL_SYM(GetErrorString, "ncclGetErrorString")
#undef LLMQ_NCCL_SYM
  g_nccl.h = h;
  return 1;
}

#define NK(call)                                                                                      \
  do {                                                                                                \
    const ncclResult_t r_ = (call);                                                                   \
    if (r_ != ncclSuccess) {                                                                          \
      llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: NCCL error %s at %s:%d", g_nccl.GetErrorString(r_), \
                     __FILE__, __LINE__);                                                             \
      return 0;                                                                                       \
    }                                                                                                 \
  } while (0)
template <typename K>
cudaError_t set_attr(K *fn, int smem) {
  cudaFuncAttributes fa{};
  cudaError_t e = cudaFuncGetAttributes(&fa, fn);
  if (e != cudaSuccess) return e;
  smem = std::min(smem, g_smem_optin - static_cast<int>(fa.sharedSizeBytes));
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
}

template <int PRO, int EPI, int MR>
cudaError_t set_gemv_attr(int smem) {
  cudaError_t e = set_attr(k_gemv<PRO, EPI, MR, 64>, smem);
  if (e != cudaSuccess) return e;
  return set_attr(k_gemv<PRO, EPI, MR, 128>, smem);
}

template <int PRO, int EPI>
cudaError_t set_f32_attr(int smem) {
  cudaError_t e = set_attr(k_gemv_f32<PRO, EPI, 256, 0>, smem);
  if constexpr (f32_cpl(EPI) == 1)
    if (e == cudaSuccess) e = set_attr(k_gemv_f32<PRO, EPI, 256, kF32RowsFull>, smem);
  if (e != cudaSuccess) return e;
  return set_attr(k_gemv_f32<PRO, EPI, kF32MaxThreads, 0>, smem);
}

int init_expf_table(DevCtx &c) {
  const uint32_t n = llmq_expf_exceptions_count;
  uint32_t cap = 1;
  while (cap < 3 * n + 1) cap <<= 1;
  std::vector<uint32_t> table(cap, 0u);
  for (uint32_t i = 0; i < n; ++i) {
    const uint32_t key = llmq_expf_exceptions[i];
    uint32_t h = expf_hash(key) & (cap - 1);
    while (table[h] != 0u) h = (h + 1) & (cap - 1);
    table[h] = key;
  }
  CK(cudaMalloc(&c.expf_keys, cap * sizeof(uint32_t)));
  CK(upload_sync(c.expf_keys, table.data(), cap * sizeof(uint32_t)));
  ExpfTable t{c.expf_keys, cap - 1};
  CK(cudaMemcpyToSymbol(g_expf_table, &t, sizeof(t)));
  return 1;
}

DevCtx *get_ctx() {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    llmq_set_error(LLMQ_ERR_NO_DEVICE, "libllmq_cuda: no CUDA device available (%s)", cudaGetErrorString(e));
    return nullptr;
  }
  DevCtx &c = g_ctx[dev];
  if (c.ready) return &c;
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, dev);
  if (e != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_NO_DEVICE, "libllmq_cuda: cannot query device %d (%s)", dev, cudaGetErrorString(e));
    return nullptr;
  }
  if (prop.major != 10) {
    llmq_set_error(LLMQ_ERR_NO_DEVICE, "libllmq_cuda: device %d is sm_%d%d; this build targets sm_100a (B200)", dev,
                   prop.major, prop.minor);
    return nullptr;
  }
  c.device = dev;
  c.num_sms = prop.multiProcessorCount;
  c.max_smem = static_cast<int>(prop.sharedMemPerBlockOptin) - 2048;  // room for static shared memory
  g_smem_optin = static_cast<int>(prop.sharedMemPerBlockOptin);
  if (cudaStreamCreateWithFlags(&c.stream, cudaStreamNonBlocking) != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: cudaStreamCreate failed");
    return nullptr;
  }
  if (!init_expf_table(c)) return nullptr;
  const int sm = c.max_smem;
  cudaError_t ea = cudaSuccess;
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_ABSMAX, EPI_PLAIN, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_ABSMAX, EPI_PLAIN, 8>(sm);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_RMSNORM, EPI_PLAIN, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_EMBED_RMSNORM, EPI_QKV, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_RMSNORM, EPI_QKV, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_ABSMAX, EPI_RESID, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_ABSMAX, EPI_TP_RESID, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_tp_absmax, 0);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_RMSNORM, EPI_SWIGLU, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_gemv_attr<PRO_RMSNORM, EPI_LOGITS, 1>(sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_attn_scores, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_attn_pv, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_attn_fused, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_tc_gemm<64>, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_tc_gemm<128>, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_act_codes, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_rows_absmax, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_tc_epilogue, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_rows_norm_codes, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_rows_append, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_rows_scores, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_pf_scores, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_pf_softmax, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_pf_pv, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_rows_pv, sm);
  ea = ea != cudaSuccess ? ea : set_attr(k_rows_finish, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_step_finish, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_sample_exp, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_sample_max, 0);
  ea = ea != cudaSuccess ? ea : set_attr(k_sample, static_cast<int>(kSampleSmem));
  ea = ea != cudaSuccess ? ea : set_f32_attr<F32_PRO_PLAIN, F32_EPI_RESID>(sm);
  ea = ea != cudaSuccess ? ea : set_f32_attr<F32_PRO_RMSNORM, F32_EPI_QKV>(sm);
  ea = ea != cudaSuccess ? ea : set_f32_attr<F32_PRO_EMBED_RMSNORM, F32_EPI_QKV>(sm);
  ea = ea != cudaSuccess ? ea : set_f32_attr<F32_PRO_RMSNORM, F32_EPI_SWIGLU>(sm);
  ea = ea != cudaSuccess ? ea : set_f32_attr<F32_PRO_RMSNORM, F32_EPI_LOGITS>(sm);
  if (ea != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: cudaFuncSetAttribute failed (%s)", cudaGetErrorString(ea));
    return nullptr;
  }
  if (cudaMalloc(&c.err, 16) != cudaSuccess || zero_sync(c.err, 16) != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_OOM, "libllmq_cuda: device allocation failed");
    return nullptr;
  }
  c.ready = true;
  return &c;
}

// Grow-only device buffer (contents not preserved).
template <typename T>
int ensure(T **p, size_t *have, size_t need, bool zero) {
  if (*have >= need && *p) return 1;
  cudaFree(*p);
  *p = nullptr;
  *have = 0;
  const size_t n = std::max<size_t>(need, 1);
  CK(cudaMalloc(p, n * sizeof(T)));
  if (zero) CK(zero_sync(*p, n * sizeof(T)));
  *have = n;
  return 1;
}

// -------------------------------------------------------------- weight tiling
// Builds the tiled copy of a (K, N) matrix whose physical column p is column
// colsrc[p] & 0xffffff of source colsrc[p] >> 24 (-1 = zero padding).
int build_mat(Mat &out, int K, int Nlog, int NT, const std::vector<int> &colsrc, const signed char *const src[3],
              const int srcN[3], const float *const srcScale[3], int rows = 1) {
  out = Mat{};
  out.K = K;
  out.N = Nlog;
  out.NT = NT;
  out.KT = choose_kt(K, rows);
  out.Kpad = std::max(roundup(K, out.KT), out.KT);
  out.Npad = static_cast<int>(colsrc.size());
  out.n_slabs = out.Npad / NT;
  out.n_ktiles = out.Kpad / out.KT;
  CK(cudaMalloc(&out.w, std::max<size_t>(out.bytes(), 16)));
  CK(cudaMalloc(&out.ws, (size_t)out.Npad * sizeof(float)));
  RepackSrc rs{};
  int8_t *tmp[3] = {nullptr, nullptr, nullptr};
  for (int i = 0; i < 3; ++i) {
    rs.ncols[i] = srcN[i];
    if (!src[i] || K == 0 || srcN[i] == 0) continue;
    const size_t bytes = (size_t)K * srcN[i];
    CK(cudaMalloc(&tmp[i], bytes));
    CK(upload_sync(tmp[i], src[i], bytes));
    rs.m[i] = tmp[i];
  }
  int *dcol = nullptr;
  CK(cudaMalloc(&dcol, colsrc.size() * sizeof(int)));
  CK(upload_sync(dcol, colsrc.data(), colsrc.size() * sizeof(int)));
  const long long chunks = (long long)out.Kpad / 16 * out.Npad;
  const int blocks = static_cast<int>(std::min<long long>((chunks + 255) / 256, 148LL * 64));
  k_repack<<<std::max(blocks, 1), 256>>>(rs, dcol, K, out.Kpad, out.Npad, NT, out.KT, out.w);
  CK(cudaGetLastError());
  std::vector<float> ws(out.Npad, 0.0f);
  for (int p = 0; p < out.Npad; ++p) {
    const int cs = colsrc[p];
    if (cs >= 0) ws[p] = srcScale[cs >> 24][cs & 0xffffff];
  }
  CK(upload_sync(out.ws, ws.data(), ws.size() * sizeof(float)));
  CK(cudaDeviceSynchronize());
  for (int i = 0; i < 3; ++i) cudaFree(tmp[i]);
  cudaFree(dcol);
  return 1;
}

int build_plain(Mat &out, const QTensor &W, int rows = 1) {
  const int NT = 256;
  const int Npad = std::max(roundup(W.cols, NT), NT);
  std::vector<int> colsrc(Npad, -1);
  for (int j = 0; j < W.cols; ++j) colsrc[j] = j;
  const signed char *src[3] = {W.q, nullptr, nullptr};
  const int srcN[3] = {W.cols, 0, 0};
  const float *sc[3] = {W.scale, nullptr, nullptr};
  return build_mat(out, W.rows, W.cols, NT, colsrc, src, srcN, sc, rows);
}

// --------------------------------------------------------------- GEMV launch
struct GemvPlan {
  int kt = 64;
  int stages = 0;
  int grid = 0;
  size_t smem = 0;
};


int plan_gemv(const DevCtx &c, const Mat &m, int pro, int rows, GemvPlan &p) {
  const size_t tile = (size_t)kNT * m.KT;
  const size_t codes = align16((size_t)rows * m.Kpad);
  // xs holds one input row (both prologues) and later the epilogue exchange
  // (RMSNorm prologues also keep the K squares after the row, then the sum's
  // scratch)
  size_t xs = std::max<size_t>((size_t)kNT * 4, (size_t)kThreads * 4);
  xs = std::max<size_t>(xs, pro == PRO_ABSMAX ? (((size_t)m.K + 3) & ~size_t(3)) * 4
                                              : 2 * (((size_t)m.K + 3) & ~size_t(3)) * 4 + spec_sum_bytes());
  const size_t fixed = codes + align16(xs);
  const size_t budget = (size_t)c.max_smem;
  if (fixed + 2 * (tile + 16) + 32 > budget) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: GEMV K=%d x %d rows does not fit in shared memory", m.K, rows);
    return 0;
  }
  int S = static_cast<int>((budget - fixed - 32) / (tile + 16));
  S = std::min(S, 12);
  const long long T = (long long)m.n_slabs * m.n_ktiles;
  p.kt = m.KT;
  p.stages = S;
  p.smem = (size_t)S * tile + gemv_bar_bytes(S) + codes + align16(xs);
  p.grid = static_cast<int>(std::max<long long>(1, std::min<long long>(T, c.num_sms)));
  return 1;
}

GemvArgs base_args(const Mat &m, const GemvPlan &p, int *acc, int *cnt, int *err) {
  GemvArgs a{};
  a.w = m.w;
  a.ws = m.ws;
  a.K = m.K;
  a.Kpad = m.Kpad;
  a.N = m.N;
  a.Npad = m.Npad;


  a.n_slabs = m.n_slabs;
  a.n_ktiles = m.n_ktiles;
  a.stages = p.stages;
  a.rows = 1;
  a.acc = acc;
  a.cnt = cnt;
  a.err = err;
  return a;
}

template <int PRO, int EPI, int MR>
cudaError_t launch_gemv(const GemvArgs &a, const GemvPlan &p, cudaStream_t st, bool pdl) {
  if (p.kt != 64 && p.kt != 128) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.grid);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
  return p.kt == 128 ? cudaLaunchKernelEx(&cfg, k_gemv<PRO, EPI, MR, 128>, a)
                     : cudaLaunchKernelEx(&cfg, k_gemv<PRO, EPI, MR, 64>, a);
}

// ---------------------------------------------------- tensor-core GEMM launch
// Activation codes of `rows` rows of dA (row stride m.K) for the tiled matrix m.
int launch_act_codes(DevCtx &c, const Mat &m, const float *dA, int rows, cudaStream_t st) {
  const int n_rb = (rows + kTcRows - 1) / kTcRows;
  if (!ensure(&c.tc_codes, &c.tc_codes_n, (size_t)m.Kpad * kTcRows * n_rb, false) ||
      !ensure(&c.tc_as, &c.tc_as_n, (size_t)n_rb * kTcRows, false))
    return 0;
  k_act_codes<<<rows, 256, 0, st>>>(dA, rows, m.K, m.Kpad, m.KT, c.tc_codes, c.tc_as, nullptr);
  CK(cudaGetLastError());
  return 1;
}

// Fills a TcArgs for `rows` activation rows (codes and scales as written by
// launch_act_codes) times the tiled matrix m; the split count keeps the grid
// within two CTAs per SM.
int plan_tc(DevCtx &c, const Mat &m, int rows, TcArgs &a, bool acc_only = false) {
  const size_t SB = (size_t)(kNT + kTcRows) * m.KT;
  const int n_rb = (rows + kTcRows - 1) / kTcRows;
  const int tiles = m.n_slabs * n_rb;
  const int splits = std::max(1, std::min(m.n_ktiles, (2 * c.num_sms) / tiles));
  a = TcArgs{};
  a.w = m.w;
  a.acodes = c.tc_codes;
  a.as = c.tc_as;
  a.ws = m.ws;
  a.N = m.N;
  a.Npad = m.Npad;
  a.n_slabs = m.n_slabs;
  a.n_ktiles = m.n_ktiles;
  a.n_rb = n_rb;
  a.splits = splits;
  a.stages = (int)std::max<size_t>((kTcStageBytes + SB - 1) / SB, std::min<size_t>(kTcMaxStages, kTcRingBytes / SB));
  a.rows = rows;
  a.err = c.err;
  a.acc_only = acc_only ? 1 : 0;
  if ((splits > 1 || acc_only) && !ensure(&c.tc_acc, &c.tc_acc_n, (size_t)rows * m.Npad, true)) return 0;
  a.acc = c.tc_acc;
  return 1;
}

// The epilogue of a product whose int32 sums are in a.acc (k_tc_epilogue).
int launch_tc_epilogue(const TcArgs &a, cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3((a.rows * a.n_slabs + 3) / 4);
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  ++g_launches;
  CK(cudaLaunchKernelEx(&cfg, k_tc_epilogue, a));
  return 1;
}

int launch_tc_gemm(const TcArgs &a, int KT, cudaStream_t st, bool pdl) {
  const size_t smem = (size_t)a.stages * (kNT + kTcRows) * KT;
  const dim3 grid(a.n_slabs * a.n_rb * a.splits);
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  CK(KT == 128 ? cudaLaunchKernelEx(&cfg, k_tc_gemm<128>, a) : cudaLaunchKernelEx(&cfg, k_tc_gemm<64>, a));
  ++g_launches;
  if (a.splits > 1 && !a.acc_only) return launch_tc_epilogue(a, st);
  return 1;
}

// rows rows of dA (row stride m.K) times the tiled matrix m, epilogue `epi`
// into out (row stride ld).
int launch_tc(DevCtx &c, const Mat &m, const float *dA, int rows, float *out, int ld, int epi, const float *bias,
              cudaStream_t st) {
  if (!launch_act_codes(c, m, dA, rows, st)) return 0;
  TcArgs a;
  if (!plan_tc(c, m, rows, a)) return 0;
  a.epi = epi;
  a.bias = bias;
  a.out = out;
  a.ld = ld;
  return launch_tc_gemm(a, m.KT, st, false);
}

size_t scores_smem(const AttnArgs &a) {
  const int hd4 = (a.hd + 3) & ~3, stride = (a.hd & 3) == 0 ? a.hd + 4 : a.hd + 1;
  return ((size_t)(a.n_heads / a.n_kv) * hd4 + (size_t)kScoreChunk * stride) * sizeof(float);
}
// Shared memory of k_attn_pv: the weights, then the value ring or, when the
// whole value slice fits in kPVWholeLimit, the whole slice.
constexpr size_t kPVWholeLimit = 200 * 1024;
size_t pv_whole_bytes(int max_seq) {
  return ((((size_t)max_seq + 3) & ~size_t(3)) + (size_t)max_seq * kPVSlice) * sizeof(float);
}
size_t pv_smem(const AttnArgs &a) {
  if (a.pv_whole) return pv_whole_bytes(a.max_seq);
  return ((((size_t)a.max_seq + 3) & ~size_t(3)) + (size_t)kPVRing * kPVChunk * kPVSlice) * sizeof(float);
}

// Shared memory of k_attn_fused with key chunks of kc rows: q and the rotated
// k, the weights, the value slice, the key chunk slots (one when a part of the
// positions always fits in one chunk, else two).
size_t fused_smem(const AttnArgs &a, int kc) {
  const int hd4 = (a.hd + 3) & ~3, stride = (a.hd & 3) == 0 ? a.hd + 4 : a.hd + 1;
  const int nsl = (a.hd + kPVSlice - 1) / kPVSlice;
  const int part = (a.max_seq + nsl - 1) / nsl;
  const int slots = kc >= part ? 1 : 2;
  return (2 * (size_t)hd4 + (((size_t)a.max_seq + 3) & ~size_t(3)) + (size_t)a.max_seq * kPVSlice +
          (size_t)slots * kc * stride) *
         sizeof(float);
}
// Key chunk for the fused attention: a whole part of the positions when it
// fits in shared memory, else the largest multiple of 32 rows (at least 32)
// that does; 0 (the two-kernel path) when not even that fits or a head spans
// more than 8 slices (the portable cluster size).
int fused_chunk_rows(const AttnArgs &a, size_t max_smem) {
  const int nsl = (a.hd + kPVSlice - 1) / kPVSlice;
  if (nsl > 8) return 0;
  const int part = (a.max_seq + nsl - 1) / nsl;
  if (fused_smem(a, part) <= max_smem) return part;
  for (int kc = ((part - 1) / 32) * 32; kc >= 32; kc -= 32)
    if (fused_smem(a, kc) <= max_smem) return kc;
  return 0;
}

// LLMQ_ATTN_TWO_KERNELS=1 selects the two-kernel attention everywhere (the
// same arithmetic; for comparisons).
bool attn_two_kernels_forced() {
  static const bool on = [] {
    const char *e = getenv("LLMQ_ATTN_TWO_KERNELS");
    return e && e[0] == '1';
  }();
  return on;
}
// The batch-1 attention arguments' choice between the two paths.
void choose_attention(AttnArgs &a) {
  a.pv_whole = pv_whole_bytes(a.max_seq) <= kPVWholeLimit;
  // the limit is the kernels' dynamic shared memory attribute (DevCtx::max_smem)
  a.fused_chunk = attn_two_kernels_forced() ? 0 : fused_chunk_rows(a, (size_t)g_smem_optin - 2048);
}

// The attention of one layer: k_attn_fused when a.fused_chunk > 0 (part 0;
// part 1 launches nothing), else the scores (part 0), then softmax and values
// (part 1).
cudaError_t launch_attention(const AttnArgs &a, cudaStream_t st, bool pdl, int part) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.stream = st;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
  if (a.fused_chunk > 0) {
    if (part != 0) return cudaSuccess;
    const int nsl = (a.hd + kPVSlice - 1) / kPVSlice;
    cudaLaunchAttribute fat[2];
    fat[0] = attr[0];
    fat[1].id = cudaLaunchAttributeClusterDimension;
    fat[1].val.clusterDim.x = nsl;
    fat[1].val.clusterDim.y = 1;
    fat[1].val.clusterDim.z = 1;
    cfg.attrs = fat;
    cfg.numAttrs = (pdl && pdl_enabled()) ? 2 : 1;
    if (cfg.numAttrs == 1) fat[0] = fat[1];
    cfg.gridDim = dim3(nsl, a.n_heads);
    cfg.blockDim = dim3(kFusedThreads);
    cfg.dynamicSmemBytes = fused_smem(a, a.fused_chunk);
    return cudaLaunchKernelEx(&cfg, k_attn_fused, a);
  }
  if (part == 0) {
    cfg.gridDim = dim3((a.max_seq + kScoreChunk - 1) / kScoreChunk, a.n_kv);
    cfg.blockDim = dim3(kScoreThreads);
    cfg.dynamicSmemBytes = scores_smem(a);
    return cudaLaunchKernelEx(&cfg, k_attn_scores, a);
  }
  cfg.gridDim = dim3((a.hd + kPVSlice - 1) / kPVSlice, a.n_heads);
  cfg.blockDim = dim3(kPVThreads);
  cfg.dynamicSmemBytes = pv_smem(a);
  return cudaLaunchKernelEx(&cfg, k_attn_pv, a);
}

cudaError_t launch_finish(StepState *step, unsigned long long *argmax, int *err, int *result, int *tokens,
                          int max_seq, cudaStream_t st, unsigned *tp_seq, unsigned tp_products, float *amax,
                          int n_amax) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1);
  cfg.blockDim = dim3(1);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_step_finish, step, argmax, err, result, tokens, max_seq, tp_seq, tp_products,
                            amax, n_amax);
}

// Launches `kern` with programmatic dependent launch (the kernel itself waits
// for its predecessor with griddepcontrol.wait before touching shared data).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  ++g_launches;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

// ------------------------------------------------------------------- models
struct DevModel;

struct DevKV {
  const void *key = nullptr;
  DevModel *model = nullptr;
  int max_seq = 0;
  float *k = nullptr, *v = nullptr;  // [n_layers][max_seq][kvd]
  // greedy: device-chained, host io, host io + logits; sampled: the same three
  cudaGraphExec_t graph[6] = {nullptr, nullptr, nullptr, nullptr, nullptr, nullptr};
};

struct DevModel {
  const void *key = nullptr;
  int device = -1;
  LlmqConfig cfg{};
  int qd = 0, kvd = 0;
  std::vector<Mat> qkv, wo, w13, w2;
  Mat lm;
  // fp32 (LLMA) model: the same step with fp32 products
  bool f32 = false;
  std::vector<MatF> fqkv, fwo, fw13, fw2;
  MatF flm;
  float *wte_f = nullptr;  // [vocab][d_model]
  std::vector<float *> attn_norm, ffn_norm, bias_qkv;
  float *final_norm = nullptr;
  int8_t *wte_q = nullptr;
  float *wte_s = nullptr;
  float *rope_cos = nullptr, *rope_sin = nullptr;
  // activations and scratch
  float *x = nullptr, *q = nullptr, *o = nullptr, *h = nullptr, *logits = nullptr, *scores = nullptr;
  int *acc = nullptr, *cnt = nullptr, *err = nullptr, *result = nullptr, *tokens = nullptr;
  unsigned long long *argmax = nullptr;
  StepState *step = nullptr;
  SampleState *sample = nullptr;  // sampler settings and xorshift64 state
  float *sample_e = nullptr;      // [vocab_full] sampler scratch
  unsigned *sample_hist = nullptr;  // [kSampleBins + 1], zero between draws
  // pinned host staging
  StepState *h_step = nullptr;
  SampleState *h_sample = nullptr;
  int *h_result = nullptr;
  int *h_tokens = nullptr;
  float *h_logits = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  // launch plans
  GemvPlan p_qkv, p_wo, p_w13, p_w2, p_lm;
  size_t attn_smem = 0;
  int max_npad = 0, max_slabs = 0;
  // tensor parallelism: this model is shard tp_rank of tp_world (cfg holds the
  // shard's head, d_ff and vocab counts; these keep the whole model's)
  int tp_rank = 0, tp_world = 1, vocab_full = 0, kvd_full = 0;
  float *tp_max = nullptr;      // reduced activation absmax of a row-parallel product
  float *amax = nullptr;        // [n_layers][2]: absmax of Wo's and W2's inputs, published by their producers
  int *tp_acc = nullptr;        // [d_model] partial / reduced int32 sums
  float *logits_full = nullptr; // [vocab_full] gathered logits
  // peer-memory exchange of the single-sequence step (see TpExchange)
  char *tpx = nullptr;               // this rank's region
  std::vector<char *> tpx_peer;      // every rank's region, mapped here (own included)
  char **tpx_peers_dev = nullptr;    // the same, in device memory
  unsigned *tp_seq = nullptr;        // row-parallel products completed
  std::vector<DevKV *> kvs;
  // per-kernel events while llmq_step_profile records a step outside a graph
  std::vector<cudaEvent_t> *prof = nullptr;
  // multi-row passes (batched decode, prefill): grow-only scratch
  struct Rows {
    int cap = 0, lm_cap = 0;
    float *x = nullptr, *qkv = nullptr, *qr = nullptr, *ao = nullptr, *h = nullptr, *scores = nullptr;
    float *logits = nullptr, *logits_all = nullptr;  // logits_all: gathered shards (tensor parallel)
    float *tp_max = nullptr;                         // [rows] reduced absmax (tensor parallel)
    RowDesc *rd = nullptr;
    int *ids = nullptr;
    unsigned long long *argmax = nullptr;
    RowDesc *h_rd = nullptr;  // pinned
    int *h_ids = nullptr;     // pinned
    int *h_err = nullptr;     // pinned
  } rows;
};

std::unordered_map<const void *, DevModel *> g_models;
std::unordered_map<const void *, DevKV *> g_kvs;
float g_last_ms = 0.0f;

void release_kv(DevKV *K) {
  for (auto &g : K->graph)
    if (g) cudaGraphExecDestroy(g);
  cudaFree(K->k);
  cudaFree(K->v);
  delete K;
}

void release_model(DevModel *M) {
  int cur = -1;
  cudaGetDevice(&cur);
  if (M->device >= 0) cudaSetDevice(M->device);
  if (M->stream) cudaStreamSynchronize(M->stream);
  for (DevKV *K : M->kvs) {
    g_kvs.erase(K->key);
    release_kv(K);
  }
  for (auto *v : {&M->qkv, &M->wo, &M->w13, &M->w2})
    for (Mat &m : *v) free_mat(m);
  free_mat(M->lm);
  for (auto *v : {&M->fqkv, &M->fwo, &M->fw13, &M->fw2})
    for (MatF &m : *v) free_matf(m);
  free_matf(M->flm);
  cudaFree(M->wte_f);
  for (auto *v : {&M->attn_norm, &M->ffn_norm, &M->bias_qkv})
    for (float *p : *v) cudaFree(p);
  for (int q = 0; q < (int)M->tpx_peer.size(); ++q)
    if (q != M->tp_rank && M->tpx_peer[q]) cudaIpcCloseMemHandle(M->tpx_peer[q]);
  cudaFree(M->amax);
  void *tp_ptrs[] = {M->tp_max, M->tp_acc, M->logits_full, M->tpx, M->tpx_peers_dev, M->tp_seq};
  for (void *p : tp_ptrs) cudaFree(p);
  void *dev_ptrs[] = {M->final_norm, M->wte_q, M->wte_s, M->rope_cos, M->rope_sin, M->x, M->q, M->o, M->scores,
                      M->h, M->logits, M->acc, M->cnt, M->err, M->result, M->tokens, M->argmax, M->step,
                      M->sample, M->sample_e, M->sample_hist};
  for (void *p : dev_ptrs) cudaFree(p);
  {
    auto &R = M->rows;
    void *rp[] = {R.x, R.qkv, R.qr, R.ao, R.h, R.scores, R.logits, R.logits_all, R.tp_max, R.rd, R.ids, R.argmax};
    for (void *p : rp) cudaFree(p);
    cudaFreeHost(R.h_rd);
    cudaFreeHost(R.h_ids);
    cudaFreeHost(R.h_err);
  }
  cudaFreeHost(M->h_step);
  cudaFreeHost(M->h_sample);
  cudaFreeHost(M->h_result);
  cudaFreeHost(M->h_tokens);
  cudaFreeHost(M->h_logits);
  if (M->ev0) cudaEventDestroy(M->ev0);
  if (M->ev1) cudaEventDestroy(M->ev1);
  if (M->stream) cudaStreamDestroy(M->stream);
  delete M;
  if (cur >= 0) cudaSetDevice(cur);
}

template <typename T>
int dev_upload(T **dst, const T *src, size_t n) {
  CK(cudaMalloc(dst, std::max<size_t>(n, 1) * sizeof(T)));
  if (n) CK(upload_sync(*dst, src, n * sizeof(T)));
  return 1;
}
template <typename T>
int dev_zeros(T **dst, size_t n) {
  CK(cudaMalloc(dst, std::max<size_t>(n, 1) * sizeof(T)));
  CK(zero_sync(*dst, std::max<size_t>(n, 1) * sizeof(T)));
  return 1;
}

// The peer-memory exchange region of a shard (TpExchange): allocated here,
// shared with the other ranks through CUDA IPC handles that the ranks
// all-gather over NCCL (every rank uploads its shard in the same order).
int tp_map_peers(DevModel *M) {
  const int W = M->tp_world, dm = M->cfg.d_model;
  if (!dev_zeros(&M->tpx, tpx_bytes(W, dm)) || !dev_zeros(&M->tp_seq, 1)) return 0;
  cudaIpcMemHandle_t mine;
  CK(cudaIpcGetMemHandle(&mine, M->tpx));
  std::vector<cudaIpcMemHandle_t> all(W);
  unsigned char *dh = nullptr;
  CK(cudaMalloc(&dh, sizeof(cudaIpcMemHandle_t) * (size_t)(W + 1)));
  CK(upload_sync(dh, &mine, sizeof(mine)));
  const ncclResult_t r = g_nccl.AllGather(dh, dh + sizeof(mine), sizeof(mine), ncclUint8, g_tp.comm, M->stream);
  const cudaError_t es = cudaStreamSynchronize(M->stream);
  const cudaError_t ec = cudaMemcpy(all.data(), dh + sizeof(mine), sizeof(mine) * (size_t)W, cudaMemcpyDeviceToHost);
  cudaFree(dh);
  if (r != ncclSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: NCCL all-gather of exchange handles: %s", g_nccl.GetErrorString(r));
    return 0;
  }
  CK(es);
  CK(ec);
  M->tpx_peer.assign(W, nullptr);
  for (int q = 0; q < W; ++q) {
    if (q == M->tp_rank) {
      M->tpx_peer[q] = M->tpx;
      continue;
    }
    void *p = nullptr;
    CK(cudaIpcOpenMemHandle(&p, all[q], cudaIpcMemLazyEnablePeerAccess));
    M->tpx_peer[q] = static_cast<char *>(p);
  }
  CK(cudaMalloc(&M->tpx_peers_dev, sizeof(char *) * (size_t)W));
  CK(upload_sync(M->tpx_peers_dev, M->tpx_peer.data(), sizeof(char *) * (size_t)W));
  return 1;
}

int upload_model(DevCtx &c, const QLlamaModel *m, DevModel *M) {
  LlmqConfig &cfg = M->cfg;
  cfg.vocab = m->vocab;
  cfg.d_model = m->d_model;
  cfg.n_layers = m->n_layers;
  cfg.n_heads = m->n_heads;
  cfg.n_kv = m->n_kv;
  cfg.head_dim = m->head_dim;
  cfg.d_ff = m->d_ff;
  cfg.max_seq = m->max_seq;
  cfg.rope_base = m->rope_base;
  cfg.eps = m->eps;
  M->vocab_full = m->vocab;
  M->kvd_full = m->n_kv * m->head_dim;
  {
    // A shard of the tensor-parallel group (llmq_synth_model_shard,
    // q_llama_model_shard) holds 1/world of the heads, d_ff and vocab columns.
    const int Wsh = g_tp.world;
    const bool shard = Wsh > 1 && m->n_heads % Wsh == 0 && m->blocks[0].Wq.cols == m->n_heads * m->head_dim / Wsh;
    if (!shard && m->blocks[0].Wq.cols != m->n_heads * m->head_dim) {
      llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: Wq has %d columns: neither the whole model nor a shard of the "
                     "tensor-parallel group of %d", m->blocks[0].Wq.cols, Wsh);
      return 0;
    }
    if (shard) {
      if (g_tp.device != c.device) {
        llmq_set_error(LLMQ_ERR_STATE, "libllmq_cuda: shard uploaded on device %d, group formed on %d", c.device,
                       g_tp.device);
        return 0;
      }
      M->tp_rank = g_tp.rank;
      M->tp_world = Wsh;
      cfg.n_heads /= Wsh;
      cfg.n_kv /= Wsh;
      cfg.d_ff /= Wsh;
      cfg.vocab /= Wsh;
    }
  }
  const int dm = cfg.d_model, hd = cfg.head_dim, dff = cfg.d_ff, L = cfg.n_layers;
  M->qd = cfg.n_heads * hd;
  M->kvd = cfg.n_kv * hd;
  const int qd = M->qd, kvd = M->kvd;
  if (hd % 2 != 0 || hd > 256) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: head_dim %d unsupported (even, <= 256)", hd);
    return 0;
  }
  M->device = c.device;
  CK(cudaStreamCreateWithFlags(&M->stream, cudaStreamNonBlocking));
  CK(cudaEventCreate(&M->ev0));
  CK(cudaEventCreate(&M->ev1));
  // fused QKV: [Wq | Wk | Wv], slabs of whole heads
  const int nt_qkv = kNT;  // RoPE happens in the attention kernel, so slabs need not align with heads
  const int n_qkv = qd + 2 * kvd;
  for (int l = 0; l < L; ++l) {
    const QLlamaBlock &b = m->blocks[l];
    {
      const int Npad = roundup(n_qkv, nt_qkv);
      std::vector<int> cs(Npad, -1);
      for (int p = 0; p < n_qkv; ++p)
        cs[p] = p < qd ? p : (p < qd + kvd ? ((1 << 24) | (p - qd)) : ((2 << 24) | (p - qd - kvd)));
      const signed char *src[3] = {b.Wq.q, b.Wk.q, b.Wv.q};
      const int sn[3] = {qd, kvd, kvd};
      const float *ss[3] = {b.Wq.scale, b.Wk.scale, b.Wv.scale};
      M->qkv.emplace_back();
      if (!build_mat(M->qkv.back(), dm, n_qkv, nt_qkv, cs, src, sn, ss)) return 0;
      std::vector<float> bias(Npad, 0.0f);
      std::memcpy(bias.data(), b.b_q.data, qd * sizeof(float));
      std::memcpy(bias.data() + qd, b.b_k.data, kvd * sizeof(float));
      std::memcpy(bias.data() + qd + kvd, b.b_v.data, kvd * sizeof(float));
      float *db = nullptr;
      if (!dev_upload(&db, bias.data(), bias.size())) return 0;
      M->bias_qkv.push_back(db);
    }
    M->wo.emplace_back();
    if (!build_plain(M->wo.back(), b.Wo)) return 0;
    {
      // W1|W3 interleaved per slab: 128 gate columns, then the same 128 up columns
      const int half = 128, NT = 2 * half;
      const int slabs = (dff + half - 1) / half;
      std::vector<int> cs((size_t)slabs * NT, -1);
      for (int s = 0; s < slabs; ++s)
        for (int c2 = 0; c2 < half; ++c2) {
          const int j = s * half + c2;
          if (j < dff) {
            cs[(size_t)s * NT + c2] = j;
            cs[(size_t)s * NT + half + c2] = (1 << 24) | j;
          }
        }
      const signed char *src[3] = {b.Wgate.q, b.Wup.q, nullptr};
      const int sn[3] = {dff, dff, 0};
      const float *ss[3] = {b.Wgate.scale, b.Wup.scale, nullptr};
      M->w13.emplace_back();
      if (!build_mat(M->w13.back(), dm, dff, NT, cs, src, sn, ss)) return 0;
    }
    M->w2.emplace_back();
    if (!build_plain(M->w2.back(), b.Wdown)) return 0;
    float *an = nullptr, *fn = nullptr;
    if (!dev_upload(&an, b.attn_norm.data, dm) || !dev_upload(&fn, b.ffn_norm.data, dm)) return 0;
    M->attn_norm.push_back(an);
    M->ffn_norm.push_back(fn);
  }
  if (!build_plain(M->lm, m->lm_head)) return 0;
  if (!dev_upload(&M->final_norm, m->final_norm.data, dm)) return 0;
  if (!dev_upload(&M->wte_q, reinterpret_cast<const int8_t *>(m->wte.q), (size_t)m->vocab * dm)) return 0;
  if (!dev_upload(&M->wte_s, m->wte.scale, dm)) return 0;
  {
    const size_t n = (size_t)cfg.max_seq * (hd / 2);
    std::vector<float> cs(n), sn(n);
    llmq_rope_tables(cfg.rope_base, hd, cfg.max_seq, cs.data(), sn.data());
    if (!dev_upload(&M->rope_cos, cs.data(), n) || !dev_upload(&M->rope_sin, sn.data(), n)) return 0;
  }
  // plans and scratch
  if (!plan_gemv(c, M->qkv[0], PRO_RMSNORM, 1, M->p_qkv) || !plan_gemv(c, M->wo[0], PRO_ABSMAX, 1, M->p_wo) ||
      !plan_gemv(c, M->w13[0], PRO_RMSNORM, 1, M->p_w13) || !plan_gemv(c, M->w2[0], PRO_ABSMAX, 1, M->p_w2) ||
      !plan_gemv(c, M->lm, PRO_RMSNORM, 1, M->p_lm))
    return 0;
  {
    AttnArgs probe{};
    probe.n_heads = cfg.n_heads;
    probe.n_kv = cfg.n_kv;
    probe.hd = hd;
    probe.max_seq = cfg.max_seq;
    probe.pv_whole = pv_whole_bytes(cfg.max_seq) <= kPVWholeLimit;
    M->attn_smem = std::max(scores_smem(probe), pv_smem(probe));
  }
  if (!dev_zeros(&M->scores, (size_t)cfg.n_heads * cfg.max_seq)) return 0;
  if (M->attn_smem > (size_t)c.max_smem) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: max_seq %d too long for the attention kernel", cfg.max_seq);
    return 0;
  }
  int max_npad = 0, max_slabs = 0;
  for (auto *v : {&M->qkv, &M->wo, &M->w13, &M->w2})
    for (Mat &mm : *v) {
      max_npad = std::max(max_npad, mm.Npad);
      max_slabs = std::max(max_slabs, mm.n_slabs);
    }
  max_npad = std::max(max_npad, M->lm.Npad);
  max_slabs = std::max(max_slabs, M->lm.n_slabs);
  M->max_npad = max_npad;
  M->max_slabs = max_slabs;
  if (!dev_zeros(&M->x, dm) || !dev_zeros(&M->q, (size_t)qd + kvd) || !dev_zeros(&M->o, qd) || !dev_zeros(&M->h, dff) ||
      !dev_zeros(&M->logits, std::max(cfg.vocab, max_npad)) || !dev_zeros(&M->acc, max_npad) ||
      !dev_zeros(&M->cnt, max_slabs) || !dev_zeros(&M->err, 4) || !dev_zeros(&M->result, 4) ||
      !dev_zeros(&M->tokens, cfg.max_seq) || !dev_zeros(&M->argmax, 1) || !dev_zeros(&M->step, 1) ||
      !dev_zeros(&M->sample, 1) || !dev_zeros(&M->sample_e, M->vocab_full) ||
      !dev_zeros(&M->sample_hist, kSampleBins + 1))
    return 0;
  CK(cudaMallocHost(&M->h_step, sizeof(StepState)));
  CK(cudaMallocHost(&M->h_sample, sizeof(SampleState)));
  CK(cudaMallocHost(&M->h_result, 4 * sizeof(int)));
  CK(cudaMallocHost(&M->h_tokens, (size_t)cfg.max_seq * sizeof(int)));
  CK(cudaMallocHost(&M->h_logits, (size_t)M->vocab_full * sizeof(float)));
  if (M->tp_world > 1 && (!dev_zeros(&M->tp_max, 1) || !dev_zeros(&M->tp_acc, dm) ||
                          !dev_zeros(&M->logits_full, M->vocab_full)))
    return 0;
  if (M->tp_world == 1 && !dev_zeros(&M->amax, 2 * (size_t)L)) return 0;
  if (M->tp_world > 1 && !tp_map_peers(M)) return 0;
  CK(cudaDeviceSynchronize());
  return 1;
}

// ------------------------------------------------------------ fp32 models
// Lays out the N columns of a fused matrix as tiles of kF32Tile (32 or 64, the
// width the consuming epilogue's kernel reads: 32 * f32_cpl(epi)) columns,
// each a contiguous block of f32_tile_rows(K) rows in the order the kernel
// reads them ([K][64], or [K/4][32][4]); fused column p is column
// colsrc[p] & 0xffffff of source colsrc[p] >> 24 (row-major [K][ns[src]]), or
// zero when colsrc[p] < 0.  Splits the tiles over `grid` CTAs (one consumer
// warp per tile, plus the producer warp for 32-column tiles) and plans the
// per-warp rings.
int build_matf(DevCtx &c, MatF &out, int K, const std::vector<int> &colsrc, const float *const src[3],
               const int ns[3], int grid, int pro, int epi) {
  const int kF32Tile = 32 * f32_cpl(epi);
  const int N = static_cast<int>(colsrc.size());
  const int T = (N + kF32Tile - 1) / kF32Tile;
  std::vector<int> t0(grid + 1);
  int per_cta = 0;
  for (int g = 0; g <= grid; ++g) {
    t0[g] = static_cast<int>((long long)g * T / grid);
    if (g > 0) per_cta = std::max(per_cta, t0[g] - t0[g - 1]);
  }
  const int nc = std::max(1, per_cta);  // consumer warps, one per tile
  const int threads = (nc + (f32_producer(epi) ? 1 : 0)) * 32;
  if (threads > kF32MaxThreads) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: fp32 product with %d columns is wider than this build handles", N);
    return 0;
  }
  const int Kp = f32_tile_rows(K, f32_cpl(epi));
  // position of (row k, column q) inside a tile
  auto at = [kF32Tile](int k, int q) -> size_t {
    return kF32Tile == 64 ? (size_t)k * 64 + q : ((size_t)(k >> 2) * 32 + q) * 4 + (k & 3);
  };
  std::vector<float> buf((size_t)T * Kp * kF32Tile, 0.0f);
  auto fill = [&](int ta, int tb) {
    for (int t = ta; t < tb; ++t) {
      float *blk = buf.data() + (size_t)t * Kp * kF32Tile;
      // a tile whose columns are consecutive columns of one source is copied row by row
      const int p0 = t * kF32Tile;
      bool run = p0 + kF32Tile <= N && colsrc[p0] >= 0;
      for (int q = 1; run && q < kF32Tile; ++q) run = colsrc[p0 + q] == colsrc[p0] + q;
      if (run) {
        const int sidx = colsrc[p0] >> 24, col = colsrc[p0] & 0xffffff;
        for (int k = 0; k < K; ++k) {
          const float *rowp = src[sidx] + (size_t)k * ns[sidx] + col;
          if (kF32Tile == 64) {
            std::memcpy(blk + (size_t)k * 64, rowp, 64 * sizeof(float));
          } else {
            for (int q = 0; q < 32; ++q) blk[at(k, q)] = rowp[q];
          }
        }
        continue;
      }
      for (int q = 0; q < kF32Tile && p0 + q < N; ++q) {
        const int cs = colsrc[p0 + q];
        if (cs < 0) continue;
        const float *sp = src[cs >> 24] + (cs & 0xffffff);
        const int ld = ns[cs >> 24];
        for (int k = 0; k < K; ++k) blk[at(k, q)] = sp[(size_t)k * ld];
      }
    }
  };
  {
    const int nt = std::max(1, std::min(32, static_cast<int>(std::thread::hardware_concurrency())));
    std::vector<std::thread> pool;
    for (int t = 0; t < nt; ++t) pool.emplace_back(fill, (int)((long long)t * T / nt), (int)((long long)(t + 1) * T / nt));
    for (auto &th : pool) th.join();
  }
  if (!dev_upload(&out.w, buf.data(), buf.size()) || !dev_upload(&out.cta_t0, t0.data(), t0.size())) return 0;
  out.K = K;
  out.N = N;
  out.grid = grid;
  out.threads = threads;
  out.tw = kF32Tile;
  // each consumer warp's share of shared memory beside the input row (and, for
  // RMSNorm, its squares and the sum's scratch).  32-column tiles: slots of 256 rows (the kernel's
  // unrolled full-slot path) when two or more fit; otherwise, and for 64-column
  // tiles, slots of up to 128 rows (16 or 32 KB), as many as fit, at most 8.
  const long long xs_bytes = ((pro == F32_PRO_PLAIN ? 1LL : 2LL) * roundup(K, 4) + 8) * 4 +
                             (pro == F32_PRO_PLAIN ? 0LL : (long long)spec_sum_bytes());
  const long long per_warp = ((long long)c.max_smem - 1024 - xs_bytes) / nc - 2LL * 2 * kF32MaxSlots * 8;
  int rows = 0, slots = 0;
  if (kF32Tile == 32 && per_warp / (kF32RowsFull * 128LL) >= 2) {
    rows = kF32RowsFull;
    slots = static_cast<int>(std::min<long long>(kF32MaxSlots, per_warp / (kF32RowsFull * 128LL)));
  } else {
    rows = static_cast<int>(std::min<long long>(128, per_warp / 4 / (kF32Tile * 4))) & ~7;
    if (rows < 8) rows = 8;
    slots = static_cast<int>(std::min<long long>(kF32MaxSlots, per_warp / ((long long)rows * kF32Tile * 4)));
  }
  if (slots < 2) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: fp32 product (K %d, %d columns) does not fit in shared memory", K, N);
    return 0;
  }
  out.rows = rows;
  out.slots = slots;
  out.smem = f32_ring_floats(nc, slots, rows, kF32Tile) * 4 + f32_bars(nc, slots) * 8 + (size_t)xs_bytes;
  return 1;
}

// Column maps: sources side by side, or gate / up interleaved in fours.
std::vector<int> cols_concat(const int ns[3]) {
  std::vector<int> cs;
  for (int i = 0; i < 3; ++i)
    for (int j = 0; j < ns[i]; ++j) cs.push_back((i << 24) | j);
  return cs;
}
std::vector<int> cols_interleave4(int n) {
  std::vector<int> cs((size_t)8 * ((n + 3) / 4), -1);
  for (size_t p = 0; p < cs.size(); ++p) {
    const int g = static_cast<int>(p / 8), w = static_cast<int>(p % 8);
    const int j = g * 4 + (w & 3);
    if (j < n) cs[p] = ((w < 4 ? 0 : 1) << 24) | j;
  }
  return cs;
}

template <int PRO, int EPI>
cudaError_t launch_f32(const MatF &m, F32Args a, cudaStream_t st, bool pdl = true) {
  if (m.tw != 32 * f32_cpl(EPI)) return cudaErrorInvalidValue;  // laid out for another epilogue
  a.w = m.w;
  a.cta_t0 = m.cta_t0;
  a.K = m.K;
  a.N = m.N;
  a.rows = m.rows;
  a.slots = m.slots;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(m.grid);
  cfg.blockDim = dim3(m.threads);
  cfg.dynamicSmemBytes = m.smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = (pdl && pdl_enabled()) ? 1 : 0;
  ++g_launches;
  if constexpr (f32_cpl(EPI) == 1) {
    if (m.rows == kF32RowsFull && m.threads <= 256)
      return cudaLaunchKernelEx(&cfg, k_gemv_f32<PRO, EPI, 256, kF32RowsFull>, a);
  }
  if (m.threads <= 256) return cudaLaunchKernelEx(&cfg, k_gemv_f32<PRO, EPI, 256, 0>, a);
  return cudaLaunchKernelEx(&cfg, k_gemv_f32<PRO, EPI, kF32MaxThreads, 0>, a);
}

int upload_model_f32(DevCtx &c, const LlamaModel *m, DevModel *M) {
  if (g_tp.world > 1) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: fp32 models decode on one GPU (no tensor-parallel group)");
    return 0;
  }
  LlmqConfig &cfg = M->cfg;
  cfg.vocab = m->vocab;
  cfg.d_model = m->d_model;
  cfg.n_layers = m->n_layers;
  cfg.n_heads = m->n_heads;
  cfg.n_kv = m->n_kv;
  cfg.head_dim = m->head_dim;
  cfg.d_ff = m->d_ff;
  cfg.max_seq = m->max_seq;
  cfg.rope_base = m->rope_base;
  cfg.eps = m->eps;
  M->f32 = true;
  M->vocab_full = m->vocab;
  M->kvd_full = m->n_kv * m->head_dim;
  const int dm = cfg.d_model, hd = cfg.head_dim, dff = cfg.d_ff, L = cfg.n_layers;
  M->qd = cfg.n_heads * hd;
  M->kvd = cfg.n_kv * hd;
  const int qd = M->qd, kvd = M->kvd;
  if (hd % 2 != 0 || hd > 256) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: head_dim %d unsupported (even, <= 256)", hd);
    return 0;
  }
  auto shape_ok = [](const Tensor &t, int r, int cc) {
    return t.data && t.ndim == 2 && t.shape && t.shape[0] == r && t.shape[1] == cc;
  };
  M->device = c.device;
  CK(cudaStreamCreateWithFlags(&M->stream, cudaStreamNonBlocking));
  CK(cudaEventCreate(&M->ev0));
  CK(cudaEventCreate(&M->ev1));
  const int grid = c.num_sms;
  for (int l = 0; l < L; ++l) {
    const LlamaBlock &b = m->blocks[l];
    if (!shape_ok(b.Wq, dm, qd) || !shape_ok(b.Wk, dm, kvd) || !shape_ok(b.Wv, dm, kvd) || !shape_ok(b.Wo, qd, dm) ||
        !shape_ok(b.Wgate, dm, dff) || !shape_ok(b.Wup, dm, dff) || !shape_ok(b.Wdown, dff, dm)) {
      llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: layer %d weights do not match the model config", l);
      return 0;
    }
    {
      const float *src[3] = {b.Wq.data, b.Wk.data, b.Wv.data};
      const int ns[3] = {qd, kvd, kvd};
      M->fqkv.emplace_back();
      if (!build_matf(c, M->fqkv.back(), dm, cols_concat(ns), src, ns, grid, F32_PRO_RMSNORM, F32_EPI_QKV)) return 0;
      std::vector<float> bias((size_t)qd + 2 * kvd, 0.0f);  // llama.c:316-318 (absent biases are zero)
      if (b.b_q.data) std::memcpy(bias.data(), b.b_q.data, qd * sizeof(float));
      if (b.b_k.data) std::memcpy(bias.data() + qd, b.b_k.data, kvd * sizeof(float));
      if (b.b_v.data) std::memcpy(bias.data() + qd + kvd, b.b_v.data, kvd * sizeof(float));
      float *db = nullptr;
      if (!dev_upload(&db, bias.data(), bias.size())) return 0;
      M->bias_qkv.push_back(db);
    }
    {
      const float *src[3] = {b.Wo.data, nullptr, nullptr};
      const int ns[3] = {dm, 0, 0};
      M->fwo.emplace_back();
      if (!build_matf(c, M->fwo.back(), qd, cols_concat(ns), src, ns, grid, F32_PRO_PLAIN, F32_EPI_RESID)) return 0;
    }
    {
      const float *src[3] = {b.Wgate.data, b.Wup.data, nullptr};
      const int ns[3] = {dff, dff, 0};
      M->fw13.emplace_back();
      if (!build_matf(c, M->fw13.back(), dm, cols_interleave4(dff), src, ns, grid, F32_PRO_RMSNORM, F32_EPI_SWIGLU)) return 0;
    }
    {
      const float *src[3] = {b.Wdown.data, nullptr, nullptr};
      const int ns[3] = {dm, 0, 0};
      M->fw2.emplace_back();
      if (!build_matf(c, M->fw2.back(), dff, cols_concat(ns), src, ns, grid, F32_PRO_PLAIN, F32_EPI_RESID)) return 0;
    }
    float *an = nullptr, *fn = nullptr;
    if (!dev_upload(&an, b.attn_norm.data, dm) || !dev_upload(&fn, b.ffn_norm.data, dm)) return 0;
    M->attn_norm.push_back(an);
    M->ffn_norm.push_back(fn);
  }
  if (!shape_ok(m->lm_head, dm, cfg.vocab) || !shape_ok(m->wte, cfg.vocab, dm) || !m->final_norm.data) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: embedding / lm-head shapes do not match the model config");
    return 0;
  }
  {
    const float *src[3] = {m->lm_head.data, nullptr, nullptr};
    const int ns[3] = {cfg.vocab, 0, 0};
    if (!build_matf(c, M->flm, dm, cols_concat(ns), src, ns, grid, F32_PRO_RMSNORM, F32_EPI_LOGITS)) return 0;
  }
  if (!dev_upload(&M->final_norm, m->final_norm.data, dm)) return 0;
  if (!dev_upload(&M->wte_f, m->wte.data, (size_t)cfg.vocab * dm)) return 0;
  {
    const size_t n = (size_t)cfg.max_seq * (hd / 2);
    std::vector<float> cs(n), sn(n);
    llmq_rope_tables(cfg.rope_base, hd, cfg.max_seq, cs.data(), sn.data());
    if (!dev_upload(&M->rope_cos, cs.data(), n) || !dev_upload(&M->rope_sin, sn.data(), n)) return 0;
  }
  {
    AttnArgs probe{};
    probe.n_heads = cfg.n_heads;
    probe.n_kv = cfg.n_kv;
    probe.hd = hd;
    probe.max_seq = cfg.max_seq;
    probe.pv_whole = pv_whole_bytes(cfg.max_seq) <= kPVWholeLimit;
    M->attn_smem = std::max(scores_smem(probe), pv_smem(probe));
  }
  if (M->attn_smem > (size_t)c.max_smem) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: max_seq %d too long for the attention kernel", cfg.max_seq);
    return 0;
  }
  if (!dev_zeros(&M->scores, (size_t)cfg.n_heads * cfg.max_seq) || !dev_zeros(&M->x, dm) ||
      !dev_zeros(&M->q, (size_t)qd + kvd) || !dev_zeros(&M->o, qd) || !dev_zeros(&M->h, dff) ||
      !dev_zeros(&M->logits, cfg.vocab) || !dev_zeros(&M->err, 4) || !dev_zeros(&M->result, 4) ||
      !dev_zeros(&M->tokens, cfg.max_seq) || !dev_zeros(&M->argmax, 1) || !dev_zeros(&M->step, 1) ||
      !dev_zeros(&M->sample, 1) || !dev_zeros(&M->sample_e, M->vocab_full) ||
      !dev_zeros(&M->sample_hist, kSampleBins + 1))
    return 0;
  CK(cudaMallocHost(&M->h_step, sizeof(StepState)));
  CK(cudaMallocHost(&M->h_sample, sizeof(SampleState)));
  CK(cudaMallocHost(&M->h_result, 4 * sizeof(int)));
  CK(cudaMallocHost(&M->h_tokens, (size_t)cfg.max_seq * sizeof(int)));
  CK(cudaMallocHost(&M->h_logits, (size_t)M->vocab_full * sizeof(float)));
  CK(cudaDeviceSynchronize());
  return 1;
}

DevModel *get_model_f32(const LlamaModel *m) {
  if (!m || !m->blocks) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: null model");
    return nullptr;
  }
  auto it = g_models.find(m->blocks);
  if (it != g_models.end()) {
    DevModel *M = it->second;
    if (!M->f32) {
      llmq_set_error(LLMQ_ERR_STATE, "libllmq_cuda: these blocks belong to an int8 model");
      return nullptr;
    }
    if (cudaSetDevice(M->device) != cudaSuccess) {
      llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: cannot select device %d", M->device);
      return nullptr;
    }
    return M;
  }
  DevCtx *c = get_ctx();
  if (!c) return nullptr;
  DevModel *M = new DevModel();
  M->key = m->blocks;
  if (!upload_model_f32(*c, m, M)) {
    release_model(M);
    return nullptr;
  }
  g_models[M->key] = M;
  return M;
}

DevModel *find_model(const QLlamaModel *m) {
  auto it = g_models.find(m->blocks);
  return it == g_models.end() ? nullptr : it->second;
}

DevModel *get_model(const QLlamaModel *m) {
  if (!m || !m->blocks) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: null model");
    return nullptr;
  }
  if (DevModel *M = find_model(m)) {
    if (M->f32) {
      llmq_set_error(LLMQ_ERR_STATE, "libllmq_cuda: these blocks belong to an fp32 model");
      return nullptr;
    }
    if (cudaSetDevice(M->device) != cudaSuccess) {
      llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: cannot select device %d", M->device);
      return nullptr;
    }
    return M;
  }
  DevCtx *c = get_ctx();
  if (!c) return nullptr;
  DevModel *M = new DevModel();
  M->key = m->blocks;
  if (!upload_model(*c, m, M)) {
    release_model(M);
    return nullptr;
  }
  g_models[M->key] = M;
  return M;
}

// Copies cache rows [0, len) between the reference's host layout
// (per layer [max_seq][n_kv*hd]) and the head-major device layout
// (per layer [n_kv][max_seq][hd]).
int kv_transfer(DevModel *M, DevKV *K, const LlamaKV *kv, int len, cudaMemcpyKind dir) {
  const int hd = M->cfg.head_dim, nkv = M->cfg.n_kv;  // this rank's KV heads
  const size_t per_layer = (size_t)K->max_seq * M->kvd;
  const int h0 = M->tp_rank * nkv;                     // their first head in the host layout
  for (int l = 0; l < M->cfg.n_layers; ++l)
    for (int h = 0; h < nkv; ++h) {
      float *dk = K->k + l * per_layer + (size_t)h * K->max_seq * hd;
      float *dv = K->v + l * per_layer + (size_t)h * K->max_seq * hd;
      float *hk = kv->k[l] + (size_t)(h0 + h) * hd, *hv = kv->v[l] + (size_t)(h0 + h) * hd;
      const size_t hp = (size_t)M->kvd_full * sizeof(float), dp = (size_t)hd * sizeof(float);
      if (dir == cudaMemcpyHostToDevice) {
        CK(cudaMemcpy2D(dk, dp, hk, hp, dp, len, dir));
        CK(cudaMemcpy2D(dv, dp, hv, hp, dp, len, dir));
      } else {
        CK(cudaMemcpy2D(hk, hp, dk, dp, dp, len, dir));
        CK(cudaMemcpy2D(hv, hp, dv, dp, dp, len, dir));
      }
    }
  return 1;
}

DevKV *get_kv(DevModel *M, const LlamaKV *kv) {
  if (!kv || !kv->k || !kv->v) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: null KV cache");
    return nullptr;
  }
  auto it = g_kvs.find(kv->k);
  if (it != g_kvs.end()) {
    if (it->second->model != M) {
      llmq_set_error(LLMQ_ERR_STATE, "libllmq_cuda: this KV cache belongs to another model");
      return nullptr;
    }
    return it->second;
  }
  const LlmqConfig &cfg = M->cfg;
  if (kv->n_layers != cfg.n_layers || kv->kv_dim != M->kvd_full || kv->max_seq <= 0 || kv->max_seq > cfg.max_seq) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: KV cache shape (%d layers, kv_dim %d, max_seq %d) does not match the model",
                   kv->n_layers, kv->kv_dim, kv->max_seq);
    return nullptr;
  }
  DevKV *K = new DevKV();
  K->key = kv->k;
  K->model = M;
  K->max_seq = kv->max_seq;
  const size_t per_layer = (size_t)kv->max_seq * M->kvd;
  if (!dev_zeros(&K->k, per_layer * cfg.n_layers) || !dev_zeros(&K->v, per_layer * cfg.n_layers)) {
    release_kv(K);
    return nullptr;
  }
  // A cache that already holds positions (filled elsewhere): adopt its rows.
  const int len = std::min(std::max(kv->len, 0), kv->max_seq);
  if (len > 0 && !kv_transfer(M, K, kv, len, cudaMemcpyHostToDevice)) {
    release_kv(K);
    return nullptr;
  }
  M->kvs.push_back(K);
  g_kvs[K->key] = K;
  return K;
}

// A row-parallel product of one decode step (Wo or W2 shard, this rank's rows
// of K), as two kernels over NVLink peer memory: k_tp_absmax forms the group's
// absmax of the input (the reference quantises with the whole row's absmax,
// quant.c:69-71); the GEMV then forms this rank's exact int32 partial sums
// and, per slab, exchanges them with the other ranks and applies
// as * ws * sum + residual itself (quant.c:82, llama.c:578 / 589).  Integer
// sums: bit-identical to one GPU.  pidx numbers the step's products.
int row_parallel(DevModel *M, const Mat &w, const GemvPlan &p, const float *in, int pidx, cudaStream_t st) {
  TpExchange t{};
  t.peers = M->tpx_peers_dev;
  t.seq = M->tp_seq;
  t.rank = M->tp_rank;
  t.world = M->tp_world;
  t.dm = M->cfg.d_model;
  t.pidx = pidx;
  CK(launch_pdl(k_tp_absmax, dim3(1), dim3(kThreads), 0, st, in, w.K, M->tp_max, t, M->err));
  GemvArgs a = base_args(w, p, M->acc, M->cnt, M->err);
  a.in = in;
  a.absmax_in = M->tp_max;
  a.out = M->x;
  a.tp = t;
  CK((launch_gemv<PRO_ABSMAX, EPI_TP_RESID, 1>(a, p, st, true)));
  return 1;
}

// Records one decode step into the model stream.  mode 0: token/pos come from
// the device state (chained steps); 1: copied from h_step, result copied back;
// 2: as 1, plus the logits.  Modes 3-5 are modes 0-2 with the next token drawn
// by k_sample (sampler.c:60-115) instead of the greedy argmax; in modes 4 and 5
// the sampler settings and stream are copied in from h_sample and back out.
int record_step(DevModel *M, DevKV *K, int mode) {
  if (M->tp_world > 1 && (!g_tp.comm || g_tp.world != M->tp_world)) {
    llmq_set_error(LLMQ_ERR_STATE, "libllmq_cuda: the tensor-parallel group of this shard is gone");
    return 0;
  }
#define PROF_MARK()                                                     \
  do {                                                                  \
    if (M->prof) {                                                      \
      M->prof->emplace_back();                                          \
      cudaEventCreate(&M->prof->back());                                \
      cudaEventRecord(M->prof->back(), st);                             \
    }                                                                   \
  } while (0)
  cudaStream_t st = M->stream;
  const LlmqConfig &cfg = M->cfg;
  const size_t per_layer = (size_t)K->max_seq * M->kvd;
  const bool sampled = mode >= 3, host_io = mode % 3 != 0, want_logits = mode % 3 == 2;
  if (host_io) CK(cudaMemcpyAsync(M->step, M->h_step, sizeof(StepState), cudaMemcpyHostToDevice, st));
  if (host_io && sampled)
    CK(cudaMemcpyAsync(M->sample, M->h_sample, sizeof(SampleState), cudaMemcpyHostToDevice, st));
  auto f32_args = [&]() {
    F32Args a{};
    a.err = M->err;
    a.eps = cfg.eps;
    a.step = M->step;
    return a;
  };
  for (int l = 0; l < cfg.n_layers; ++l) {
    if (M->f32) {
      F32Args a = f32_args();
      a.in = M->x;
      a.gamma = M->attn_norm[l];
      a.out = M->q;
      a.bias = M->bias_qkv[l];
      a.qd = M->qd;
      a.kvd = M->kvd;
      a.hd = cfg.head_dim;
      a.max_seq = K->max_seq;
      a.vcache = K->v + l * per_layer;
      if (l == 0) {
        a.wte = M->wte_f;
        a.vocab = M->vocab_full;
        a.x_out = M->x;
        CK((launch_f32<F32_PRO_EMBED_RMSNORM, F32_EPI_QKV>(M->fqkv[l], a, st, false)));
      } else {
        CK((launch_f32<F32_PRO_RMSNORM, F32_EPI_QKV>(M->fqkv[l], a, st)));
      }
      PROF_MARK();
    } else {
      GemvArgs a = base_args(M->qkv[l], M->p_qkv, M->acc, M->cnt, M->err);
      a.in = M->x;
      a.gamma = M->attn_norm[l];
      a.eps = cfg.eps;
      a.step = M->step;
      a.out = M->q;
      a.bias = M->bias_qkv[l];
      a.qd = M->qd;
      a.kvd = M->kvd;
      a.hd = cfg.head_dim;
      a.max_seq = K->max_seq;
      a.vcache = K->v + l * per_layer;
      if (l == 0) {
        a.wte_q = M->wte_q;
        a.wte_s = M->wte_s;
        a.vocab = M->vocab_full;
        a.x_out = M->x;
        CK((launch_gemv<PRO_EMBED_RMSNORM, EPI_QKV, 1>(a, M->p_qkv, st, false)));
      PROF_MARK();
      } else {
        CK((launch_gemv<PRO_RMSNORM, EPI_QKV, 1>(a, M->p_qkv, st, true)));
      PROF_MARK();
      }
    }
    {
      AttnArgs a{};
      a.q = M->q;
      a.kcache = K->k + l * per_layer;
      a.vcache = K->v + l * per_layer;
      a.scores = M->scores;
      a.out = M->o;
      a.step = M->step;
      a.rope_cos = M->rope_cos;
      a.rope_sin = M->rope_sin;
      a.n_heads = cfg.n_heads;
      a.n_kv = cfg.n_kv;
      a.hd = cfg.head_dim;
      a.max_seq = K->max_seq;
      a.amax_out = M->amax ? M->amax + 2 * l : nullptr;  // Wo's absmax_in
      choose_attention(a);
      CK(launch_attention(a, st, true, 0));
      PROF_MARK();
      if (a.fused_chunk == 0) {
        CK(launch_attention(a, st, true, 1));
        PROF_MARK();
      }
    }
    if (M->f32) {
      F32Args a = f32_args();
      a.in = M->o;
      a.out = M->x;
      CK((launch_f32<F32_PRO_PLAIN, F32_EPI_RESID>(M->fwo[l], a, st)));
      PROF_MARK();
    } else if (M->tp_world > 1) {
      if (!row_parallel(M, M->wo[l], M->p_wo, M->o, 2 * l, st)) return 0;
    } else {
      GemvArgs a = base_args(M->wo[l], M->p_wo, M->acc, M->cnt, M->err);
      a.in = M->o;
      a.out = M->x;
      a.absmax_in = M->amax + 2 * l;
      CK((launch_gemv<PRO_ABSMAX, EPI_RESID, 1>(a, M->p_wo, st, true)));
      PROF_MARK();
    }
    if (M->f32) {
      F32Args a = f32_args();
      a.in = M->x;
      a.gamma = M->ffn_norm[l];
      a.out = M->h;
      a.n_out = cfg.d_ff;
      CK((launch_f32<F32_PRO_RMSNORM, F32_EPI_SWIGLU>(M->fw13[l], a, st)));
      PROF_MARK();
    } else {
      GemvArgs a = base_args(M->w13[l], M->p_w13, M->acc, M->cnt, M->err);
      a.in = M->x;
      a.gamma = M->ffn_norm[l];
      a.eps = cfg.eps;
      a.out = M->h;
      a.amax_out = M->amax ? M->amax + 2 * l + 1 : nullptr;  // W2's absmax_in
      CK((launch_gemv<PRO_RMSNORM, EPI_SWIGLU, 1>(a, M->p_w13, st, true)));
      PROF_MARK();
    }
    if (M->f32) {
      F32Args a = f32_args();
      a.in = M->h;
      a.out = M->x;
      CK((launch_f32<F32_PRO_PLAIN, F32_EPI_RESID>(M->fw2[l], a, st)));
      PROF_MARK();
    } else if (M->tp_world > 1) {
      if (!row_parallel(M, M->w2[l], M->p_w2, M->h, 2 * l + 1, st)) return 0;
    } else {
      GemvArgs a = base_args(M->w2[l], M->p_w2, M->acc, M->cnt, M->err);
      a.in = M->h;
      a.out = M->x;
      a.absmax_in = M->amax + 2 * l + 1;
      CK((launch_gemv<PRO_ABSMAX, EPI_RESID, 1>(a, M->p_w2, st, true)));
      PROF_MARK();
    }
  }
  if (M->f32) {
    F32Args a = f32_args();
    a.in = M->x;
    a.gamma = M->final_norm;
    a.out = M->logits;
    a.argmax = M->argmax;
    CK((launch_f32<F32_PRO_RMSNORM, F32_EPI_LOGITS>(M->flm, a, st)));
    PROF_MARK();
  } else {
    GemvArgs a = base_args(M->lm, M->p_lm, M->acc, M->cnt, M->err);
    a.in = M->x;
    a.gamma = M->final_norm;
    a.eps = cfg.eps;
    a.out = M->logits;
    a.argmax = M->argmax;
    a.idx_offset = M->tp_rank * cfg.vocab;
    CK((launch_gemv<PRO_RMSNORM, EPI_LOGITS, 1>(a, M->p_lm, st, true)));
      PROF_MARK();
  }
  if (M->tp_world > 1) {  // the first maximum over every shard's vocab slice (sampler.c:8-21)
    NK(g_nccl.AllReduce(M->argmax, M->argmax, 1, ncclUint64, ncclMax, g_tp.comm, st));
    if (want_logits || sampled)
      NK(g_nccl.AllGather(M->logits, M->logits_full, (size_t)cfg.vocab, ncclFloat32, g_tp.comm, st));
  }
  if (sampled) {  // every rank draws from the same whole row with the same stream
    SampleArgs a{};
    a.logits = M->tp_world > 1 ? M->logits_full : M->logits;
    a.V = M->vocab_full;
    a.st = M->sample;
    a.e = M->sample_e;
    a.hist = M->sample_hist;
    a.maxkey = M->argmax;  // the row's max comes with its argmax key
    a.argmax = M->argmax;  // and the drawn id replaces it
    CK(launch_pdl(k_sample_exp, dim3(sample_exp_grid(a.V)), dim3(kSampleExpThreads), 0, st, a));
    PROF_MARK();
    CK(launch_pdl(k_sample, dim3(1), dim3(kSampleThreads), kSampleSmem, st, a));
    PROF_MARK();
  }
  CK(launch_finish(M->step, M->argmax, M->err, M->result, M->tokens, K->max_seq, st,
                   M->tp_world > 1 ? M->tp_seq : nullptr, 2u * (unsigned)cfg.n_layers, M->amax,
                   M->amax ? 2 * cfg.n_layers : 0));
      PROF_MARK();
  if (host_io) CK(cudaMemcpyAsync(M->h_result, M->result, 4 * sizeof(int), cudaMemcpyDeviceToHost, st));
  if (host_io && sampled)
    CK(cudaMemcpyAsync(M->h_sample, M->sample, sizeof(SampleState), cudaMemcpyDeviceToHost, st));
  if (want_logits)
    CK(cudaMemcpyAsync(M->h_logits, M->tp_world > 1 ? M->logits_full : M->logits,
                       (size_t)M->vocab_full * sizeof(float), cudaMemcpyDeviceToHost, st));
#undef PROF_MARK
  return 1;
}

int get_graph(DevModel *M, DevKV *K, int mode, cudaGraphExec_t *out) {
  if (K->graph[mode]) {
    *out = K->graph[mode];
    return 1;
  }
  cudaGraph_t g = nullptr;
  CK(cudaStreamBeginCapture(M->stream, cudaStreamCaptureModeThreadLocal));
  const int ok = record_step(M, K, mode);
  const cudaError_t e = cudaStreamEndCapture(M->stream, &g);
  if (!ok) {
    if (g) cudaGraphDestroy(g);
    return 0;
  }
  CK(e);
  const cudaError_t ei = cudaGraphInstantiate(&K->graph[mode], g, 0);
  cudaGraphDestroy(g);
  CK(ei);
  *out = K->graph[mode];
  return 1;
}

int check_step_inputs(DevModel *M, const LlamaKV *kv, int token, int n) {
  if (token < 0 || token >= M->vocab_full) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: token id %d outside [0, %d)", token, M->vocab_full);
    return 0;
  }
  if (kv->len < 0 || kv->len + n > kv->max_seq) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: position %d + %d steps exceeds max_seq %d", kv->len, n, kv->max_seq);
    return 0;
  }
  return 1;
}

int reset_after_device_error(DevModel *M, int flags) {
  // A failed launch may leave partial sums behind: clear the scratch words.
  cudaMemsetAsync(M->acc, 0, (size_t)M->max_npad * sizeof(int), M->stream);
  cudaMemsetAsync(M->cnt, 0, (size_t)M->max_slabs * sizeof(int), M->stream);
  cudaMemsetAsync(M->argmax, 0, sizeof(unsigned long long), M->stream);
  cudaMemsetAsync(M->err, 0, 4 * sizeof(int), M->stream);
  if (M->amax) cudaMemsetAsync(M->amax, 0, 2 * (size_t)M->cfg.n_layers * sizeof(float), M->stream);
  cudaStreamSynchronize(M->stream);
  llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: device reported error flags 0x%x (%s%s%s)", flags,
                 (flags & ERR_TIMEOUT) ? "copy timeout " : "", (flags & ERR_BAD_TOKEN) ? "bad token " : "",
                 (flags & ERR_BAD_POS) ? "bad position" : "");
  return 0;
}

// ------------------------------------------------------- multi-row passes
constexpr int kRowsPerPass = 1024;  // rows of one pass (longer prompts run in several)

int ensure_rows(DevModel *M, int rows, int lm_rows) {
  auto &R = M->rows;
  const LlmqConfig &cfg = M->cfg;
  if (rows > R.cap) {
    void *old[] = {R.x, R.qkv, R.qr, R.ao, R.h, R.scores, R.rd, R.tp_max};
    for (void *p : old) cudaFree(p);
    cudaFreeHost(R.h_rd);
    R.x = R.qkv = R.qr = R.ao = R.h = R.scores = R.tp_max = nullptr;
    R.rd = nullptr;
    R.h_rd = nullptr;
    R.cap = 0;
    const size_t n = (size_t)rows;
    CK(cudaMalloc(&R.x, n * cfg.d_model * sizeof(float)));
    CK(cudaMalloc(&R.qkv, n * (M->qd + 2 * M->kvd) * sizeof(float)));
    CK(cudaMalloc(&R.qr, n * M->qd * sizeof(float)));
    CK(cudaMalloc(&R.ao, n * M->qd * sizeof(float)));
    CK(cudaMalloc(&R.h, n * cfg.d_ff * sizeof(float)));
    CK(cudaMalloc(&R.scores, n * cfg.n_heads * cfg.max_seq * sizeof(float)));
    CK(cudaMalloc(&R.rd, n * sizeof(RowDesc)));
    CK(cudaMalloc(&R.tp_max, n * sizeof(float)));
    CK(cudaMallocHost(&R.h_rd, n * sizeof(RowDesc)));
    R.cap = rows;
  }
  if (lm_rows > R.lm_cap) {
    cudaFree(R.logits);
    cudaFree(R.logits_all);
    R.logits_all = nullptr;
    cudaFree(R.ids);
    cudaFree(R.argmax);
    cudaFreeHost(R.h_ids);
    R.logits = nullptr;
    R.ids = nullptr;
    R.argmax = nullptr;
    R.h_ids = nullptr;
    R.lm_cap = 0;
    CK(cudaMalloc(&R.logits, (size_t)lm_rows * cfg.vocab * sizeof(float)));
    if (M->tp_world > 1) CK(cudaMalloc(&R.logits_all, (size_t)lm_rows * M->vocab_full * sizeof(float)));
    CK(cudaMalloc(&R.ids, (size_t)lm_rows * sizeof(int)));
    if (!dev_zeros(&R.argmax, (size_t)lm_rows)) return 0;
    CK(cudaMallocHost(&R.h_ids, (size_t)lm_rows * sizeof(int)));
    R.lm_cap = lm_rows;
  }
  if (!R.h_err) CK(cudaMallocHost(&R.h_err, 4 * sizeof(int)));
  return 1;
}

// One pass over `rows` rows (each one decode step of its own sequence, at its
// own position).  All layers run for every row; the final norm, lm-head and
// greedy id run for rows [lm0, rows) only: their ids go to ids_h and, if
// logits_h is given, their logits (row-major, vocab per row) as well.
int run_rows(DevCtx &c, DevModel *M, const RowDesc *rows_h, int rows, int lm0, float *logits_h, int *ids_h) {
  const LlmqConfig &cfg = M->cfg;
  cudaStream_t st = M->stream;

  const int dm = cfg.d_model, qd = M->qd, kvd = M->kvd, hd = cfg.head_dim, dff = cfg.d_ff;
  const int lm_rows = rows - lm0;
  if (!ensure_rows(M, rows, lm_rows)) return 0;
  auto &R = M->rows;
  int max_kpad = M->lm.Kpad;
  for (int l = 0; l < cfg.n_layers; ++l)
    max_kpad = std::max({max_kpad, M->qkv[l].Kpad, M->wo[l].Kpad, M->w13[l].Kpad, M->w2[l].Kpad});
  const int n_rb = (rows + kTcRows - 1) / kTcRows;
  if (!ensure(&c.tc_codes, &c.tc_codes_n, (size_t)n_rb * kTcRows * max_kpad, false) ||
      !ensure(&c.tc_as, &c.tc_as_n, (size_t)n_rb * kTcRows, false))
    return 0;
  std::memcpy(R.h_rd, rows_h, (size_t)rows * sizeof(RowDesc));
  CK(cudaMemcpyAsync(R.rd, R.h_rd, (size_t)rows * sizeof(RowDesc), cudaMemcpyHostToDevice, st));

  RowNormArgs na{};
  na.rd = R.rd;
  na.x_out = R.x;
  na.wte_q = M->wte_q;
  na.wte_s = M->wte_s;
  na.vocab = M->vocab_full;  // token ids index the whole embedding
  na.eps = cfg.eps;
  na.K = dm;
  na.codes = c.tc_codes;
  na.as = c.tc_as;
  na.err = M->err;
  const size_t norm_smem = 2 * (size_t)((dm + 3) & ~3) * sizeof(float) + spec_sum_bytes();
  RowAttnArgs aa{};
  aa.rd = R.rd;
  aa.qkv = R.qkv;
  aa.qr = R.qr;
  aa.scores = R.scores;
  aa.out = R.ao;
  aa.rope_cos = M->rope_cos;
  aa.rope_sin = M->rope_sin;
  aa.n_heads = cfg.n_heads;
  aa.n_kv = cfg.n_kv;
  aa.hd = hd;
  aa.smax = cfg.max_seq;
  aa.err = M->err;
  const int group = cfg.n_heads / cfg.n_kv;
  const size_t sc_sm = rows_scores_smem(group, hd), pv_sm = rows_pv_smem(group, hd, cfg.max_seq);
  // A prefill (every row the next position of one sequence's cache) takes the
  // row-block tiled scores kernel.
  bool pf_tiled = group <= kPfVecs && pf_scores_smem(hd) + 1024 <= (size_t)g_smem_optin;
  for (int r = 1; r < rows && pf_tiled; ++r)
    pf_tiled = rows_h[r].k == rows_h[0].k && rows_h[r].v == rows_h[0].v && rows_h[r].pos == rows_h[0].pos + r;
  const int pf_rpb = pf_rows_per_block(group);
  const size_t pf_sm = pf_scores_smem(hd);
  const int attn_threads = (group * hd / 2 + 31) / 32 * 32;  // k_rows_pv: two output dims per thread
  if (hd % 4 != 0 || group > kAttnMaxGroup || attn_threads > 1024 || pv_sm + 4096 > (size_t)g_smem_optin) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: batched attention needs head_dim %% 4 == 0, group <= %d, "
                   "group*head_dim <= 1024 and max_seq %d short enough for shared memory", kAttnMaxGroup,
                   cfg.max_seq);
    return 0;
  }
  auto norm = [&](const float *in, const float *gamma, const Mat &m, int nrows) {
    na.in = in;
    na.gamma = gamma;
    na.Kpad = m.Kpad;
    na.KT = m.KT;
    return launch_pdl(k_rows_norm_codes, dim3(nrows), dim3(kRowThreads), norm_smem, st, na);
  };
  auto codes = [&](const float *in, int K, const Mat &m) {
    return launch_pdl(k_act_codes, dim3(rows), dim3(256), 0, st, in, rows, K, m.Kpad, m.KT, c.tc_codes, c.tc_as,
                      static_cast<const float *>(nullptr));
  };
  auto gemm = [&](const Mat &m, int nrows, int epi, const float *bias, float *out, int ld,
                  unsigned long long *am) -> int {
    TcArgs t;
    if (!plan_tc(c, m, nrows, t)) return 0;
    t.epi = epi;
    t.bias = bias;
    t.out = out;
    t.ld = ld;
    t.err = M->err;
    t.argmax = am;
    t.idx_offset = M->tp_rank * cfg.vocab;  // vocab shard of the lm-head
    return launch_tc_gemm(t, m.KT, st, pdl_enabled());
  };
  // A row-parallel product of a tensor-parallel shard (Wo, W2: this rank's
  // rows of K), with residual epilogue into x: the rows' absmax max-reduced
  // over the ranks, codes with that scale, the exact int32 partial sums
  // sum-reduced, then as * ws * acc + x (quant.c:69-82, llama.c:578 / 589).
  auto row_parallel_rows = [&](const Mat &m, const float *in) -> int {
    CK(launch_pdl(k_rows_absmax, dim3(rows), dim3(256), 0, st, in, m.K, R.tp_max));
    NK(g_nccl.AllReduce(R.tp_max, R.tp_max, (size_t)rows, ncclFloat32, ncclMax, g_tp.comm, st));
    CK(launch_pdl(k_act_codes, dim3(rows), dim3(256), 0, st, in, rows, m.K, m.Kpad, m.KT, c.tc_codes, c.tc_as,
                  static_cast<const float *>(R.tp_max)));
    TcArgs t;
    if (!plan_tc(c, m, rows, t, true)) return 0;
    t.epi = TC_RESID;
    t.out = R.x;
    t.ld = dm;
    t.err = M->err;
    if (!launch_tc_gemm(t, m.KT, st, pdl_enabled())) return 0;
    NK(g_nccl.AllReduce(t.acc, t.acc, (size_t)rows * m.Npad, ncclInt32, ncclSum, g_tp.comm, st));
    return launch_tc_epilogue(t, st);
  };
  for (int l = 0; l < cfg.n_layers; ++l) {
    CK(norm(l == 0 ? nullptr : R.x, M->attn_norm[l], M->qkv[l], rows));
    if (!gemm(M->qkv[l], rows, TC_BIAS, M->bias_qkv[l], R.qkv, qd + 2 * kvd, nullptr)) return 0;
    aa.layer = l;
    CK(launch_pdl(k_rows_append, dim3(rows), dim3(256), 0, st, aa));
    if (pf_tiled)  // a prefill: each key chunk staged once per block of rows
      CK(launch_pdl(k_pf_scores, dim3((cfg.max_seq + kPfVecs - 1) / kPfVecs, cfg.n_kv, (rows + pf_rpb - 1) / pf_rpb),
                    dim3(256), pf_sm, st, aa, rows));
    else
      CK(launch_pdl(k_rows_scores, dim3((cfg.max_seq + kRowScoreKeys - 1) / kRowScoreKeys, cfg.n_kv, rows),
                    dim3(kRowScoreThreads), sc_sm, st, aa));
    if (pf_tiled && hd == 128 && (size_t)group * ((cfg.max_seq + 3) & ~3) * 4 + 4096 <= (size_t)g_smem_optin) {
      // softmax in place, then the row-block tiled values
      CK(launch_pdl(k_pf_softmax, dim3(rows, cfg.n_kv), dim3(256), (size_t)group * ((cfg.max_seq + 3) & ~3) * 4, st,
                    aa));
      CK(launch_pdl(k_pf_pv, dim3(cfg.n_kv, (rows + pf_rpb - 1) / pf_rpb), dim3(256), pf_pv_smem(hd), st, aa, rows));
    } else {
      CK(launch_pdl(k_rows_pv, dim3(cfg.n_kv, rows), dim3(attn_threads), pv_sm, st, aa));
    }
    if (M->tp_world > 1) {
      if (!row_parallel_rows(M->wo[l], R.ao)) return 0;
    } else {
      CK(codes(R.ao, qd, M->wo[l]));
      if (!gemm(M->wo[l], rows, TC_RESID, nullptr, R.x, dm, nullptr)) return 0;
    }
    CK(norm(R.x, M->ffn_norm[l], M->w13[l], rows));
    if (!gemm(M->w13[l], rows, TC_SWIGLU, nullptr, R.h, dff, nullptr)) return 0;
    if (M->tp_world > 1) {
      if (!row_parallel_rows(M->w2[l], R.h)) return 0;
    } else {
      CK(codes(R.h, dff, M->w2[l]));
      if (!gemm(M->w2[l], rows, TC_RESID, nullptr, R.x, dm, nullptr)) return 0;
    }
  }
  if (lm_rows > 0) {
    CK(norm(R.x + (size_t)lm0 * dm, M->final_norm, M->lm, lm_rows));
    if (!gemm(M->lm, lm_rows, TC_LOGITS, nullptr, R.logits, cfg.vocab, R.argmax)) return 0;
    if (M->tp_world > 1)  // the first maximum over every shard's vocab slice (sampler.c:8-21)
      NK(g_nccl.AllReduce(R.argmax, R.argmax, (size_t)lm_rows, ncclUint64, ncclMax, g_tp.comm, st));
    CK(launch_pdl(k_rows_finish, dim3(1), dim3(256), 0, st, R.argmax, lm_rows, R.ids));
    CK(cudaMemcpyAsync(R.h_ids, R.ids, (size_t)lm_rows * sizeof(int), cudaMemcpyDeviceToHost, st));
    if (logits_h && M->tp_world > 1) {
      // gathered as [rank][rows][vocab slice]: each rank's block lands in its
      // columns of the caller's [rows][vocab] rows
      const size_t blk = (size_t)lm_rows * cfg.vocab;
      NK(g_nccl.AllGather(R.logits, R.logits_all, blk, ncclFloat32, g_tp.comm, st));
      for (int r = 0; r < M->tp_world; ++r)
        CK(cudaMemcpy2DAsync(logits_h + (size_t)r * cfg.vocab, (size_t)M->vocab_full * sizeof(float),
                             R.logits_all + r * blk, (size_t)cfg.vocab * sizeof(float), (size_t)cfg.vocab * sizeof(float),
                             lm_rows, cudaMemcpyDeviceToHost, st));
    } else if (logits_h) {
      CK(cudaMemcpyAsync(logits_h, R.logits, (size_t)lm_rows * cfg.vocab * sizeof(float), cudaMemcpyDeviceToHost,
                         st));
    }
  }
  CK(cudaMemcpyAsync(R.h_err, M->err, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (R.h_err[0]) {
    if (c.tc_acc) cudaMemsetAsync(c.tc_acc, 0, c.tc_acc_n * sizeof(int), st);
    cudaMemsetAsync(R.argmax, 0, (size_t)R.lm_cap * sizeof(unsigned long long), st);
    return reset_after_device_error(M, R.h_err[0]);
  }
  if (lm_rows > 0 && ids_h) std::memcpy(ids_h, R.h_ids, (size_t)lm_rows * sizeof(int));
  return 1;
}

}  // namespace

// ======================================================================== API
extern "C" {

int llmqd_quantize(const float *w, int rows, int cols, signed char *q, float *scale) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (rows < 0 || cols < 0) {
    llmq_set_error(LLMQ_ERR_ARG, "quantize_int8_percol: negative shape");
    return 0;
  }
  if (cols == 0) return 1;
  DevCtx *c = get_ctx();
  if (!c) return 0;
  const size_t n = (size_t)rows * cols;
  float *dw = nullptr, *ds = nullptr;
  int8_t *dq = nullptr;
  int ok = 1;
  if (cudaMalloc(&dw, std::max<size_t>(n, 1) * 4) != cudaSuccess || cudaMalloc(&dq, std::max<size_t>(n, 1)) != cudaSuccess ||
      cudaMalloc(&ds, (size_t)cols * 4) != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_OOM, "quantize_int8_percol: device allocation of %zu bytes failed", n * 5);
    ok = 0;
  }
  if (ok && n && upload_sync(dw, w, n * 4) != cudaSuccess) ok = 0;
  if (ok) {
    k_quantize_percol<<<(cols + 127) / 128, 128, 0, c->stream>>>(dw, rows, cols, dq, ds);
    if (cudaGetLastError() != cudaSuccess || cudaStreamSynchronize(c->stream) != cudaSuccess) ok = 0;
  }
  if (ok && n && cudaMemcpy(q, dq, n, cudaMemcpyDeviceToHost) != cudaSuccess) ok = 0;
  if (ok && cudaMemcpy(scale, ds, (size_t)cols * 4, cudaMemcpyDeviceToHost) != cudaSuccess) ok = 0;
  if (!ok && q_llama_last_error() == LLMQ_OK)
    llmq_set_error(LLMQ_ERR_CUDA, "quantize_int8_percol: CUDA failure (%s)", cudaGetErrorString(cudaGetLastError()));
  cudaFree(dw);
  cudaFree(dq);
  cudaFree(ds);
  return ok;
}

int llmqd_dequantize(const signed char *q, const float *scale, int rows, int cols, float *w) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (rows < 0 || cols < 0) {
    llmq_set_error(LLMQ_ERR_ARG, "dequantize_int8_percol: negative shape");
    return 0;
  }
  const size_t n = (size_t)rows * cols;
  if (n == 0) return 1;
  DevCtx *c = get_ctx();
  if (!c) return 0;
  float *dw = nullptr, *ds = nullptr;
  int8_t *dq = nullptr;
  int ok = cudaMalloc(&dw, n * 4) == cudaSuccess && cudaMalloc(&dq, n) == cudaSuccess &&
           cudaMalloc(&ds, (size_t)cols * 4) == cudaSuccess;
  ok = ok && upload_sync(dq, q, n) == cudaSuccess &&
       upload_sync(ds, scale, (size_t)cols * 4) == cudaSuccess;
  if (ok) {
    k_dequantize_percol<<<std::min<long long>((n + 255) / 256, 148 * 32), 256, 0, c->stream>>>(dq, ds, rows, cols, dw);
    ok = cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(c->stream) == cudaSuccess;
  }
  ok = ok && cudaMemcpy(w, dw, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
  if (!ok) llmq_set_error(LLMQ_ERR_CUDA, "dequantize_int8_percol: CUDA failure");
  cudaFree(dw);
  cudaFree(dq);
  cudaFree(ds);
  return ok;
}

int llmqd_qmatmul(const float *A, int M, const QTensor *W, float *C) {
  // The reference reads W from host memory on every call, and callers may
  // rewrite a QTensor in place, so W is uploaded and tiled on every call
  // (into grow-only scratch); nothing is cached across calls.
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (M == 0 || W->cols == 0) return 1;
  DevCtx *c = get_ctx();
  if (!c) return 0;
  const int K = W->rows, N = W->cols;
  Mat m;
  m.K = K;
  m.N = N;
  m.NT = 256;
  m.KT = choose_kt(K, M > 8 ? 1 : M);
  m.Kpad = std::max(roundup(K, m.KT), m.KT);
  m.Npad = std::max(roundup(N, m.NT), m.NT);
  m.n_slabs = m.Npad / m.NT;
  m.n_ktiles = m.Kpad / m.KT;
  const bool many = M > 1;
  GemvPlan plan;
  int rows_per = many ? 8 : 1;
  while (true) {
    if (plan_gemv(*c, m, PRO_ABSMAX, rows_per, plan)) break;
    if (rows_per == 1) return 0;
    q_llama_clear_error();
    rows_per /= 2;
  }
  if (!ensure(&c->dA, &c->dA_n, (size_t)M * K, false) || !ensure(&c->dC, &c->dC_n, (size_t)M * N, false) ||
      !ensure(&c->acc, &c->acc_n, (size_t)8 * m.Npad, true) || !ensure(&c->cnt, &c->cnt_n, (size_t)m.n_slabs, true) ||
      !ensure(&c->wraw, &c->wraw_n, (size_t)K * N, false) || !ensure(&c->wtile, &c->wtile_n, m.bytes(), false) ||
      !ensure(&c->wscale, &c->wscale_n, (size_t)m.Npad, false))
    return 0;
  m.w = c->wtile;
  m.ws = c->wscale;
  cudaStream_t st = c->stream;
  if (K > 0) {
    CK(cudaMemcpyAsync(c->wraw, W->q, (size_t)K * N, cudaMemcpyHostToDevice, st));
    CK(cudaMemcpyAsync(c->dA, A, (size_t)M * K * sizeof(float), cudaMemcpyHostToDevice, st));
  }
  CK(cudaMemcpyAsync(c->wscale, W->scale, (size_t)N * sizeof(float), cudaMemcpyHostToDevice, st));
  CK(cudaMemsetAsync(c->wscale + N, 0, (size_t)(m.Npad - N) * sizeof(float), st));
  {
    const long long chunks = (long long)m.Kpad / 16 * m.Npad;
    const int blocks = static_cast<int>(std::min<long long>((chunks + 255) / 256, 148LL * 64));
    k_repack_plain<<<std::max(blocks, 1), 256, 0, st>>>(reinterpret_cast<const int8_t *>(c->wraw), K, N, m.Kpad,
                                                         m.Npad, kNT, m.KT, c->wtile);
    CK(cudaGetLastError());
  }
  if (M > 8) {  // tensor cores
    if (!launch_tc(*c, m, c->dA, M, c->dC, N, TC_PLAIN, nullptr, st)) return 0;
  } else {
    for (int r0 = 0; r0 < M; r0 += rows_per) {
      GemvArgs a = base_args(m, plan, c->acc, c->cnt, c->err);
      a.rows = std::min(rows_per, M - r0);
      a.in = c->dA + (size_t)r0 * K;
      a.out = c->dC + (size_t)r0 * N;
      if (many)
        CK((launch_gemv<PRO_ABSMAX, EPI_PLAIN, 8>(a, plan, st, false)));
      else
        CK((launch_gemv<PRO_ABSMAX, EPI_PLAIN, 1>(a, plan, st, false)));
    }
  }
  CK(cudaMemcpyAsync(C, c->dC, (size_t)M * N * sizeof(float), cudaMemcpyDeviceToHost, st));
  int flags = 0;
  CK(cudaMemcpyAsync(&flags, c->err, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  if (flags) {
    zero_sync(c->err, 16);
    zero_sync(c->acc, c->acc_n * sizeof(int));
    zero_sync(c->cnt, c->cnt_n * sizeof(int));
    llmq_set_error(LLMQ_ERR_CUDA, "qmatmul: device reported error flags 0x%x", flags);
    return 0;
  }
  return 1;
}

int llmqd_model_upload(const QLlamaModel *m) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return get_model(m) != nullptr;
}

void llmqd_model_release(const QLlamaModel *m) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!m || !m->blocks) return;
  auto it = g_models.find(m->blocks);
  if (it == g_models.end()) return;
  DevModel *M = it->second;
  g_models.erase(it);
  release_model(M);
}

int llmqd_kv_register(const QLlamaModel *m, const LlamaKV *kv) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevModel *M = get_model(m);
  return M && get_kv(M, kv) != nullptr;
}

void llmqd_kv_release(const LlamaKV *kv) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!kv || !kv->k) return;
  auto it = g_kvs.find(kv->k);
  if (it == g_kvs.end()) return;
  DevKV *K = it->second;
  g_kvs.erase(it);
  DevModel *M = K->model;
  auto &v = M->kvs;
  v.erase(std::remove(v.begin(), v.end(), K), v.end());
  int cur = -1;
  cudaGetDevice(&cur);
  cudaSetDevice(M->device);
  cudaStreamSynchronize(M->stream);
  release_kv(K);
  if (cur >= 0) cudaSetDevice(cur);
}

static_assert(sizeof(SampleState) == sizeof(LlmqSample) && offsetof(SampleState, rng) == offsetof(LlmqSample, rng),
              "LlmqSample mirrors SampleState");

int check_sample(const LlmqSample *s, int V) {
  if (!(s->temperature <= 0.0f) && (s->k < 1 || s->k > kSampleMaxK || s->k > V)) {
    llmq_set_error(LLMQ_ERR_ARG,
                   "libllmq_cuda: device sampling keeps 1..%d candidates; top-k resolves to %d of vocab %d "
                   "(sample on the host from the logits instead)",
                   kSampleMaxK, s->k, V);
    return 0;
  }
  return 1;
}

// One step of model M (the caller holds g_mu).
int decode_one(DevModel *M, const LlamaKV *kv, int token, float *logits, int *next, LlmqSample *smp) {
  if (!M) return 0;
  DevKV *K = get_kv(M, kv);
  if (!K || !check_step_inputs(M, kv, token, 1)) return 0;
  if (smp && !check_sample(smp, M->vocab_full)) return 0;
  const int mode = (logits ? 2 : 1) + (smp ? 3 : 0);
  cudaGraphExec_t g = nullptr;
  if (!get_graph(M, K, mode, &g)) return 0;
  M->h_step->token = token;
  M->h_step->pos = kv->len;
  if (smp) std::memcpy(M->h_sample, smp, sizeof(SampleState));
  CK(cudaEventRecord(M->ev0, M->stream));
  CK(cudaGraphLaunch(g, M->stream));
  CK(cudaEventRecord(M->ev1, M->stream));
  CK(cudaStreamSynchronize(M->stream));
  cudaEventElapsedTime(&g_last_ms, M->ev0, M->ev1);
  if (M->h_result[1]) return reset_after_device_error(M, M->h_result[1]);
  if (logits) std::memcpy(logits, M->h_logits, (size_t)M->vocab_full * sizeof(float));
  if (next) *next = M->h_result[0];
  if (smp) smp->rng = M->h_sample->rng;
  return 1;
}

// n device-chained steps of model M (the caller holds g_mu).
int generate_n(DevModel *M, const LlamaKV *kv, int token, int n, int *ids, LlmqSample *smp) {
  if (!M) return 0;
  DevKV *K = get_kv(M, kv);
  if (!K || n < 0 || !check_step_inputs(M, kv, token, n)) return 0;
  if (smp && !check_sample(smp, M->vocab_full)) return 0;
  if (n == 0) return 1;
  cudaGraphExec_t g = nullptr;
  if (!get_graph(M, K, smp ? 3 : 0, &g)) return 0;
  M->h_step->token = token;
  M->h_step->pos = kv->len;
  cudaStream_t st = M->stream;
  CK(cudaMemcpyAsync(M->step, M->h_step, sizeof(StepState), cudaMemcpyHostToDevice, st));
  CK(cudaMemsetAsync(M->result, 0, 4 * sizeof(int), st));
  if (smp) {
    std::memcpy(M->h_sample, smp, sizeof(SampleState));
    CK(cudaMemcpyAsync(M->sample, M->h_sample, sizeof(SampleState), cudaMemcpyHostToDevice, st));
  }
  CK(cudaEventRecord(M->ev0, st));
  for (int i = 0; i < n; ++i) CK(cudaGraphLaunch(g, st));
  CK(cudaEventRecord(M->ev1, st));
  CK(cudaMemcpyAsync(M->h_result, M->result, 4 * sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(M->h_tokens, M->tokens + kv->len, (size_t)n * sizeof(int), cudaMemcpyDeviceToHost, st));
  if (smp) CK(cudaMemcpyAsync(M->h_sample, M->sample, sizeof(SampleState), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  cudaEventElapsedTime(&g_last_ms, M->ev0, M->ev1);
  if (M->h_result[3]) return reset_after_device_error(M, M->h_result[3]);
  std::memcpy(ids, M->h_tokens, (size_t)n * sizeof(int));
  if (smp) smp->rng = M->h_sample->rng;
  return 1;
}

int llmqd_decode(const QLlamaModel *m, const LlamaKV *kv, int token, float *logits, int *next) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return decode_one(get_model(m), kv, token, logits, next, nullptr);
}

int llmqd_decode_sample(const QLlamaModel *m, const LlamaKV *kv, int token, float *logits, int *next,
                        LlmqSample *smp) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return decode_one(get_model(m), kv, token, logits, next, smp);
}

int llmqd_generate(const QLlamaModel *m, const LlamaKV *kv, int token, int n, int *ids) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return generate_n(get_model(m), kv, token, n, ids, nullptr);
}

int llmqd_generate_sample(const QLlamaModel *m, const LlamaKV *kv, int token, int n, int *ids, LlmqSample *smp) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return generate_n(get_model(m), kv, token, n, ids, smp);
}

// ---- the fp32 (LLMA) model: the same steps with fp32 products
int llmqd_model_upload_f32(const LlamaModel *m) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return get_model_f32(m) != nullptr;
}

void llmqd_model_release_f32(const LlamaModel *m) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!m || !m->blocks) return;
  auto it = g_models.find(m->blocks);
  if (it == g_models.end() || !it->second->f32) return;
  DevModel *M = it->second;
  g_models.erase(it);
  release_model(M);
}

int llmqd_kv_register_f32(const LlamaModel *m, const LlamaKV *kv) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevModel *M = get_model_f32(m);
  return M && get_kv(M, kv) != nullptr;
}

int llmqd_decode_f32(const LlamaModel *m, const LlamaKV *kv, int token, float *logits, int *next, LlmqSample *smp) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return decode_one(get_model_f32(m), kv, token, logits, next, smp);
}

int llmqd_generate_f32(const LlamaModel *m, const LlamaKV *kv, int token, int n, int *ids, LlmqSample *smp) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  return generate_n(get_model_f32(m), kv, token, n, ids, smp);
}

// One logits row in host memory, sampled on the current device (the
// standalone sample_token / sample_argmax).
int llmqd_sample_row(const float *row, int V, LlmqSample *smp, int *id) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!row || V <= 0 || !smp || !id) {
    llmq_set_error(LLMQ_ERR_ARG, "libllmq_cuda: bad sampler arguments");
    return 0;
  }
  if (!check_sample(smp, V)) return 0;
  DevCtx *c = get_ctx();
  if (!c) return 0;
  cudaStream_t st = c->stream;
  // the state (32 B), the id and the argmax key (32 B), the histogram, then
  // [V] logits and [V] scratch
  const size_t hist_bytes = roundup((kSampleBins + 1) * 4, 256);
  const size_t head = 64 + hist_bytes;
  const size_t need = head + 2 * (size_t)roundup(V, 64) * sizeof(float);
  if (c->sample_n < need) {
    cudaFree(c->sample_buf);
    c->sample_buf = nullptr;
    c->sample_n = 0;
    CK(cudaMalloc(&c->sample_buf, need));
    CK(zero_sync(c->sample_buf, head));
    c->sample_n = need;
  }
  SampleState *d_st = reinterpret_cast<SampleState *>(c->sample_buf);
  int *d_id = reinterpret_cast<int *>(c->sample_buf + 32);
  unsigned long long *d_key = reinterpret_cast<unsigned long long *>(c->sample_buf + 48);
  unsigned *d_hist = reinterpret_cast<unsigned *>(c->sample_buf + 64);
  float *d_row = reinterpret_cast<float *>(c->sample_buf + head);
  SampleArgs a{};
  a.logits = d_row;
  a.V = V;
  a.st = d_st;
  a.e = d_row + roundup(V, 64);
  a.hist = d_hist;
  a.maxkey = d_key;
  a.out = d_id;
  CK(cudaMemcpyAsync(d_st, smp, sizeof(SampleState), cudaMemcpyHostToDevice, st));
  CK(cudaMemcpyAsync(d_row, row, (size_t)V * sizeof(float), cudaMemcpyHostToDevice, st));
  CK(cudaMemsetAsync(d_key, 0, sizeof(unsigned long long), st));
  k_sample_max<<<std::min(c->num_sms, (V + 255) / 256), 256, 0, st>>>(d_row, V, d_key);
  k_sample_exp<<<sample_exp_grid(V), kSampleExpThreads, 0, st>>>(a);
  k_sample<<<1, kSampleThreads, kSampleSmem, st>>>(a);
  CK(cudaGetLastError());
  LlmqSample back{};
  CK(cudaMemcpyAsync(&back, d_st, sizeof(SampleState), cudaMemcpyDeviceToHost, st));
  CK(cudaMemcpyAsync(id, d_id, sizeof(int), cudaMemcpyDeviceToHost, st));
  CK(cudaStreamSynchronize(st));
  smp->rng = back.rng;
  return 1;
}

int llmqd_decode_rows(const QLlamaModel *m, LlamaKV *const *kvs, const int *tokens, int B, float *logits,
                      int *ids) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (B <= 0 || !kvs || !tokens) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_decode_batch: bad arguments");
    return 0;
  }
  DevModel *M = get_model(m);
  if (!M) return 0;
  DevCtx *c = get_ctx();
  if (!c) return 0;
  std::vector<RowDesc> rows((size_t)B);
  for (int b = 0; b < B; ++b) {
    const LlamaKV *kv = kvs[b];
    DevKV *K = get_kv(M, kv);
    if (!K || !check_step_inputs(M, kv, tokens[b], 1)) return 0;
    for (int e = 0; e < b; ++e)
      if (rows[e].k == K->k) {
        llmq_set_error(LLMQ_ERR_ARG, "q_llama_decode_batch: sequence %d and %d share one KV cache", e, b);
        return 0;
      }
    rows[b] = RowDesc{K->k, K->v, K->max_seq, kv->len, tokens[b], 0};
  }
  std::vector<int> tmp;
  if (!ids) {
    tmp.resize((size_t)B);
    ids = tmp.data();
  }
  g_launches = 0;
  CK(cudaEventRecord(M->ev0, M->stream));
  for (int off = 0; off < B; off += kRowsPerPass) {
    const int n = std::min(kRowsPerPass, B - off);
    if (!run_rows(*c, M, rows.data() + off, n, 0, logits ? logits + (size_t)off * M->vocab_full : nullptr, ids + off))
      return 0;
  }
  CK(cudaEventRecord(M->ev1, M->stream));
  CK(cudaEventSynchronize(M->ev1));
  cudaEventElapsedTime(&g_last_ms, M->ev0, M->ev1);
  g_last_launches = g_launches;
  return 1;
}

int llmqd_prefill(const QLlamaModel *m, const LlamaKV *kv, const int *ids, int n, float *logits, int *next) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (n <= 0 || !ids) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_prefill: bad arguments");
    return 0;
  }
  DevModel *M = get_model(m);
  if (!M) return 0;
  DevCtx *c = get_ctx();
  if (!c) return 0;
  DevKV *K = get_kv(M, kv);
  if (!K || !check_step_inputs(M, kv, 0, n)) return 0;
  for (int i = 0; i < n; ++i)
    if (ids[i] < 0 || ids[i] >= M->vocab_full) {
      llmq_set_error(LLMQ_ERR_ARG, "q_llama_prefill: token id %d at %d outside [0, %d)", ids[i], i, M->vocab_full);
      return 0;
    }
  std::vector<RowDesc> rows((size_t)std::min(n, kRowsPerPass));
  int last = -1;
  g_launches = 0;
  CK(cudaEventRecord(M->ev0, M->stream));
  for (int off = 0; off < n; off += kRowsPerPass) {
    const int cnt = std::min(kRowsPerPass, n - off);
    for (int r = 0; r < cnt; ++r) rows[r] = RowDesc{K->k, K->v, K->max_seq, kv->len + off + r, ids[off + r], 0};
    const bool final_pass = off + cnt == n;
    if (!run_rows(*c, M, rows.data(), cnt, final_pass ? cnt - 1 : cnt, final_pass ? logits : nullptr, &last))
      return 0;
  }
  CK(cudaEventRecord(M->ev1, M->stream));
  CK(cudaEventSynchronize(M->ev1));
  cudaEventElapsedTime(&g_last_ms, M->ev0, M->ev1);
  g_last_launches = g_launches;
  if (next) *next = last;
  return 1;
}

int llmqd_kv_download(const QLlamaModel *m, const LlamaKV *kv, int len) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevModel *M = get_model(m);
  if (!M) return 0;
  DevKV *K = get_kv(M, kv);
  if (!K) return 0;
  const size_t per_layer = (size_t)K->max_seq * M->kvd;
  CK(cudaStreamSynchronize(M->stream));
  (void)per_layer;
  return len > 0 ? kv_transfer(M, K, kv, len, cudaMemcpyDeviceToHost) : 1;
}

float llmqd_last_ms(void) { return g_last_ms; }

int llmqd_tp_world(void) { return g_tp.world; }

// ---- diagnostics exported for tests and the benchmark (declared in llmq_cuda.h)
LLMQ_API long long llmq_last_launches(void) { return g_last_launches; }

LLMQ_API int llmq_expf_device(const float *x, float *y, long long n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (n <= 0) return LLMQ_OK;
  DevCtx *c = get_ctx();
  if (!c) return q_llama_last_error();
  float *dx = nullptr, *dy = nullptr;
  int ok = cudaMalloc(&dx, n * 4) == cudaSuccess && cudaMalloc(&dy, n * 4) == cudaSuccess &&
           upload_sync(dx, x, n * 4) == cudaSuccess;
  if (ok) {
    k_expf_batch<<<148 * 8, 256, 0, c->stream>>>(dx, dy, n);
    ok = cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(c->stream) == cudaSuccess &&
         cudaMemcpy(y, dy, n * 4, cudaMemcpyDeviceToHost) == cudaSuccess;
  }
  cudaFree(dx);
  cudaFree(dy);
  if (!ok) {
    llmq_set_error(LLMQ_ERR_CUDA, "llmq_expf_device: CUDA failure");
    return LLMQ_ERR_CUDA;
  }
  return LLMQ_OK;
}

// Times `iters` back-to-back launches of one of the model's GEMVs on the model
// stream (which: 0 QKV, 1 Wo, 2 W1|W3, 3 W2, 4 lm-head; 5 the batch-1
// attention) with CUDA events, using the activations left by the last step.
// The launches go through the layers in turn, starting at `layer`, and run
// from one captured CUDA graph with programmatic dependent launch, as in a
// decode step.  Reports the mean time per launch and the algorithmic bytes of
// one launch (int8 weights + scales + input + output).
LLMQ_API int llmq_bench_gemv(const QLlamaModel *m, int which, int layer, int iters, float *ms_per_launch,
                             double *bytes_per_launch) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevModel *M = get_model(m);
  if (!M) return q_llama_last_error();
  if (layer < 0 || layer >= M->cfg.n_layers || which < 0 || which > 5 || iters <= 0 ||
      (which == 5 && M->kvs.empty())) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_bench_gemv: bad arguments");
    return LLMQ_ERR_ARG;
  }
  cudaStream_t st = M->stream;
  std::function<cudaError_t()> launch;
  GemvArgs a{};
  AttnArgs at{};
  int next = layer;  // the layer of the next launch
  if (which == 5) {  // attention over the first cache at its current position
    DevKV *K = M->kvs.front();
    const size_t per_layer = (size_t)K->max_seq * M->kvd;
    at.q = M->q;
    at.kcache = K->k + layer * per_layer;
    at.vcache = K->v + layer * per_layer;
    at.scores = M->scores;
    at.out = M->o;
    at.step = M->step;
    at.rope_cos = M->rope_cos;
    at.rope_sin = M->rope_sin;
    at.n_heads = M->cfg.n_heads;
    at.n_kv = M->cfg.n_kv;
    at.hd = M->cfg.head_dim;
    at.max_seq = K->max_seq;
    choose_attention(at);
    launch = [&at, &next, M, K, per_layer, st]() {
      const int l = next++ % M->cfg.n_layers;
      at.kcache = K->k + l * per_layer;
      at.vcache = K->v + l * per_layer;
      const cudaError_t e = launch_attention(at, st, true, 0);
      return e != cudaSuccess ? e : launch_attention(at, st, true, 1);
    };
  } else {
    // Launch i takes layer (layer + i) mod n_layers, so consecutive launches
    // stream different weights (a layer's QKV, Wo or W2 alone fits in L2).
    const GemvPlan *pl[5] = {&M->p_qkv, &M->p_wo, &M->p_w13, &M->p_w2, &M->p_lm};
    const bool rms[5] = {true, false, true, false, true};
    float *const ins[5] = {M->x, M->o, M->x, M->h, M->x};
    const GemvPlan *p = pl[which];
    float *in = ins[which];
    const int L = M->cfg.n_layers;
    auto mat_of = [M, which, L](int l) -> const Mat & {
      const int ll = l % L;
      return which == 0 ? M->qkv[ll] : which == 1 ? M->wo[ll] : which == 2 ? M->w13[ll] : which == 3 ? M->w2[ll]
                                                                                                   : M->lm;
    };
    const Mat &mm = mat_of(layer);
    const bool r = rms[which];
    launch = [&a, &next, mat_of, p, in, M, st, r]() {
      a = base_args(mat_of(next++), *p, M->acc, M->cnt, M->err);
      a.in = in;
      if (!r) a.absmax_in = M->amax;  // Wo / W2 take their absmax from the producer, as in a step
      a.gamma = M->final_norm;
      a.eps = M->cfg.eps;
      a.out = M->logits;
      return r ? launch_gemv<PRO_RMSNORM, EPI_PLAIN, 1>(a, *p, st, true)
               : launch_gemv<PRO_ABSMAX, EPI_PLAIN, 1>(a, *p, st, true);
    };
    const int logical_n = which == 2 ? 2 * mm.N : mm.N;
    *bytes_per_launch = (double)mm.K * logical_n + 4.0 * logical_n + 4.0 * mm.K + 4.0 * mm.N;
  }
  // The `iters` launches are captured into one CUDA graph, back to back with
  // programmatic dependent launch as inside a decode step's graph, so the
  // timing is the kernels' own and not the host's launch rate; the graph is
  // replayed once to warm up, then once between the two events.
  cudaGraph_t g = nullptr;
  cudaGraphExec_t ge = nullptr;
  cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  for (int i = 0; i < iters && e == cudaSuccess; ++i) e = launch();
  const cudaError_t ee = cudaStreamEndCapture(st, &g);
  if (e == cudaSuccess) e = ee;
  if (e == cudaSuccess) e = cudaGraphInstantiate(&ge, g, 0);
  if (g) cudaGraphDestroy(g);
  if (e == cudaSuccess) e = cudaGraphLaunch(ge, st);
  if (e == cudaSuccess) e = cudaEventRecord(M->ev0, st);
  if (e == cudaSuccess) e = cudaGraphLaunch(ge, st);
  if (e == cudaSuccess) e = cudaEventRecord(M->ev1, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (ge) cudaGraphExecDestroy(ge);
  if (e != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "llmq_bench_gemv: %s", cudaGetErrorString(e));
    return LLMQ_ERR_CUDA;
  }
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, M->ev0, M->ev1);
  *ms_per_launch = ms / iters;
  if (which == 5) {
    int pos = 0;
    cudaMemcpy(&pos, &M->step->pos, sizeof(int), cudaMemcpyDeviceToHost);
    // K and V rows of one layer read for every query head (the group shares them in L2)
    *bytes_per_launch = 2.0 * (pos + 1) * M->kvd * 4.0 + 8.0 * M->qd;
  }
  return LLMQ_OK;
}

// Attention launches per layer of a batch-1 step for these dimensions: 1 (the
// fused kernel) or 2.
LLMQ_API int llmq_attention_launches(int n_heads, int n_kv, int head_dim, int max_seq) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!get_ctx()) return -1;
  AttnArgs probe{};
  probe.n_heads = n_heads;
  probe.n_kv = n_kv;
  probe.hd = head_dim;
  probe.max_seq = max_seq;
  choose_attention(probe);
  return probe.fused_chunk > 0 ? 1 : 2;
}

// Number of kernels one decode step launches (for the benchmark's gpu_launches).
LLMQ_API int llmq_kernels_per_step(const QLlamaModel *m) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  const DevModel *M = find_model(m);
  if (!M) return 0;
  AttnArgs probe{};
  probe.n_heads = M->cfg.n_heads;
  probe.n_kv = M->cfg.n_kv;
  probe.hd = M->cfg.head_dim;
  probe.max_seq = M->cfg.max_seq;
  choose_attention(probe);
  const int attn = probe.fused_chunk > 0 ? 1 : 2;
  // QKV, attention, Wo, W1|W3, W2 (+ the absmax exchange per row-parallel product); lm-head, finish
  return (4 + attn + (M->tp_world > 1 ? 2 : 0)) * m->n_layers + 2;
}

// ------------------------------------------------- tensor-parallel group API
LLMQ_API int q_llama_tp_unique_id(unsigned char *id) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (!id) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_tp_unique_id: null buffer");
    return LLMQ_ERR_ARG;
  }
  if (!load_nccl()) return q_llama_last_error();
  ncclUniqueId u;
  const ncclResult_t r = g_nccl.GetUniqueId(&u);
  if (r != ncclSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "q_llama_tp_unique_id: %s", g_nccl.GetErrorString(r));
    return LLMQ_ERR_CUDA;
  }
  static_assert(sizeof(u) == NCCL_UNIQUE_ID_BYTES, "NCCL id size");
  std::memcpy(id, &u, sizeof(u));
  return LLMQ_OK;
}

LLMQ_API int q_llama_tp_init(int rank, int world, const unsigned char *id) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  if (world < 1 || rank < 0 || rank >= world || (world > 1 && !id)) {
    llmq_set_error(LLMQ_ERR_ARG, "q_llama_tp_init: bad rank %d / world %d", rank, world);
    return LLMQ_ERR_ARG;
  }
  if (g_tp.comm) {
    llmq_set_error(LLMQ_ERR_STATE, "q_llama_tp_init: a tensor-parallel group is already formed");
    return LLMQ_ERR_STATE;
  }
  DevCtx *c = get_ctx();
  if (!c) return q_llama_last_error();
  if (world == 1) {
    g_tp = TpGroup{0, 1, c->device, nullptr};
    return LLMQ_OK;
  }
  if (!load_nccl()) return q_llama_last_error();
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclComm_t comm = nullptr;
  ncclResult_t r = g_nccl.CommInitRank(&comm, world, u, rank);
  if (r == ncclSuccess) {  // first collective outside any graph capture
    int *one = nullptr;
    if (cudaMalloc(&one, sizeof(int)) == cudaSuccess) {
      r = g_nccl.AllReduce(one, one, 1, ncclInt32, ncclSum, comm, c->stream);
      cudaStreamSynchronize(c->stream);
      cudaFree(one);
    }
  }
  if (r != ncclSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "q_llama_tp_init: %s", g_nccl.GetErrorString(r));
    if (comm) g_nccl.CommDestroy(comm);
    return LLMQ_ERR_CUDA;
  }
  g_tp = TpGroup{rank, world, c->device, comm};
  return LLMQ_OK;
}

LLMQ_API void q_llama_tp_shutdown(void) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  // graphs that hold collectives of this communicator go first
  for (auto &kv : g_models)
    if (kv.second->tp_world > 1) {
      cudaStreamSynchronize(kv.second->stream);
      for (DevKV *K : kv.second->kvs)
        for (auto &g : K->graph)
          if (g) {
            cudaGraphExecDestroy(g);
            g = nullptr;
          }
    }
  if (g_tp.comm) g_nccl.CommDestroy(g_tp.comm);
  g_tp = TpGroup{};
}

}  // extern "C"

extern "C" LLMQ_API int q_llama_set_device(int device) {
  const cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_NO_DEVICE, "q_llama_set_device(%d): %s", device, cudaGetErrorString(e));
    return LLMQ_ERR_NO_DEVICE;
  }
  return LLMQ_OK;
}

// Runs one decode step of `token` at kv->len outside the graph, kernel by
// kernel with CUDA events between launches, and writes each kernel's time in
// milliseconds to ms[0 .. llmq_kernels_per_step(m)).  Advances kv->len by one
// like a decode step.  For attribution only: no overlap between kernels.
extern "C" LLMQ_API int llmq_step_profile(const QLlamaModel *m, LlamaKV *kv, int token, float *ms, int max_n) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevModel *M = get_model(m);
  if (!M) return q_llama_last_error();
  DevKV *K = get_kv(M, kv);
  if (!K || !check_step_inputs(M, kv, token, 1)) return q_llama_last_error();
  M->h_step->token = token;
  M->h_step->pos = kv->len;
  std::vector<cudaEvent_t> evs;
  cudaEvent_t e0;
  cudaEventCreate(&e0);
  M->prof = &evs;
  cudaEventRecord(e0, M->stream);
  const int ok = record_step(M, K, 1);
  M->prof = nullptr;
  cudaStreamSynchronize(M->stream);
  int rc = ok ? LLMQ_OK : q_llama_last_error();
  cudaEvent_t prev = e0;
  for (size_t i = 0; i < evs.size(); ++i) {
    float t = 0.0f;
    cudaEventElapsedTime(&t, prev, evs[i]);
    if ((int)i < max_n) ms[i] = t;
    prev = evs[i];
  }
  for (cudaEvent_t e : evs) cudaEventDestroy(e);
  cudaEventDestroy(e0);
  if (rc == LLMQ_OK) {
    if (M->h_result[1]) return reset_after_device_error(M, M->h_result[1]), LLMQ_ERR_CUDA;
    kv->len += 1;
  }
  return rc;
}

#ifdef LLMQ_PHASE_TIMING
// Profiling builds only: copies the phase timestamps (64 CTAs x 16 points).
extern "C" LLMQ_API int llmq_phase_ts(unsigned long long *out) {
  return cudaMemcpyFromSymbol(out, g_phase_ts, sizeof(unsigned long long) * 64 * 16) == cudaSuccess ? 0 : 2;
}
// Profiling builds only: phase timestamps from launch `grid` (%gridid) only (0: all).
extern "C" LLMQ_API int llmq_phase_grid(unsigned long long grid) {
  static const unsigned long long zero[64][16] = {};
  if (cudaMemcpyToSymbol(g_phase_ts, zero, sizeof(zero)) != cudaSuccess) return 2;
  return cudaMemcpyToSymbol(g_phase_grid, &grid, sizeof(grid)) == cudaSuccess ? 0 : 2;
}
// Profiling builds only: copies the launch spans (4096 x {gridid, first start,
// last end, kernel tag}) to out (when given), then resets them.
extern "C" LLMQ_API int llmq_launch_spans(unsigned long long *out) {
  static unsigned long long tab[4096][4];
  if (cudaDeviceSynchronize() != cudaSuccess) return 2;
  if (out && cudaMemcpyFromSymbol(out, g_launch_tab, sizeof(tab)) != cudaSuccess) return 2;
  for (auto &e : tab) {
    e[0] = 0;
    e[1] = ~0ull;
    e[2] = 0;
    e[3] = 0;
  }
  return cudaMemcpyToSymbol(g_launch_tab, tab, sizeof(tab)) == cudaSuccess ? 0 : 2;
}
#endif

// Times `iters` device-resident products C(M, N) = A(M, K) x W on the path
// qmatmul takes (GEMV for M <= 8, tensor cores above), with W tiled once and A,
// C resident; random A.  *ms receives the mean time per product.
extern "C" LLMQ_API int llmq_bench_qmatmul(const QTensor *W, int M, int iters, float *ms) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevCtx *c = get_ctx();
  if (!c) return q_llama_last_error();
  if (M <= 0 || iters <= 0 || !W || W->rows <= 0 || W->cols <= 0) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_bench_qmatmul: bad arguments");
    return LLMQ_ERR_ARG;
  }
  Mat m;
  if (!build_plain(m, *W, M > 8 ? 1 : M)) return q_llama_last_error();
  const int K = W->rows, N = W->cols;
  std::vector<float> hA((size_t)M * K);
  uint64_t st64 = 0x9E3779B97F4A7C15ull;
  for (float &v : hA) {
    st64 ^= st64 << 13;
    st64 ^= st64 >> 7;
    st64 ^= st64 << 17;
    v = (float)((int64_t)(st64 >> 11) - (1ll << 52)) * 0x1p-52f;
  }
  float *dA = nullptr, *dC = nullptr;
  int rc = LLMQ_OK;
  if (cudaMalloc(&dA, hA.size() * 4) != cudaSuccess || cudaMalloc(&dC, (size_t)M * N * 4) != cudaSuccess ||
      upload_sync(dA, hA.data(), hA.size() * 4) != cudaSuccess ||
      !ensure(&c->acc, &c->acc_n, (size_t)8 * m.Npad, true) || !ensure(&c->cnt, &c->cnt_n, (size_t)m.n_slabs, true)) {
    llmq_set_error(LLMQ_ERR_OOM, "llmq_bench_qmatmul: allocation failed");
    rc = LLMQ_ERR_OOM;
  }
  GemvPlan plan;
  if (rc == LLMQ_OK && M <= 8 && !plan_gemv(*c, m, PRO_ABSMAX, M == 1 ? 1 : 8, plan)) rc = q_llama_last_error();
  cudaStream_t st = c->stream;
  auto once = [&]() -> int {
    if (M > 8) {
      return launch_tc(*c, m, dA, M, dC, N, TC_PLAIN, nullptr, st);
    }
    GemvArgs a = base_args(m, plan, c->acc, c->cnt, c->err);
    a.rows = M;
    a.in = dA;
    a.out = dC;
    return (M == 1 ? launch_gemv<PRO_ABSMAX, EPI_PLAIN, 1>(a, plan, st, false)
                   : launch_gemv<PRO_ABSMAX, EPI_PLAIN, 8>(a, plan, st, false)) == cudaSuccess;
  };
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  if (rc == LLMQ_OK) {
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    for (int i = 0; i < 3 && rc == LLMQ_OK; ++i)
      if (!once()) rc = LLMQ_ERR_CUDA;
    cudaEventRecord(e0, st);
    for (int i = 0; i < iters && rc == LLMQ_OK; ++i)
      if (!once()) rc = LLMQ_ERR_CUDA;
    cudaEventRecord(e1, st);
    if (cudaStreamSynchronize(st) != cudaSuccess) rc = LLMQ_ERR_CUDA;
    float t = 0.0f;
    cudaEventElapsedTime(&t, e0, e1);
    *ms = t / iters;
    int flags = 0;
    cudaMemcpy(&flags, c->err, sizeof(int), cudaMemcpyDeviceToHost);
    if (flags) {
      zero_sync(c->err, 16);
      llmq_set_error(LLMQ_ERR_CUDA, "llmq_bench_qmatmul: device error flags 0x%x", flags);
      rc = LLMQ_ERR_CUDA;
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  cudaFree(dA);
  cudaFree(dC);
  free_mat(m);
  return rc;
}

namespace {
// One row per CTA: the row's sequential sum by spec_seq_sum and by the
// one-thread loop, the segments that missed their window, and the SM cycles of
// each (clock64 on thread 0, barrier to barrier).
__global__ void __launch_bounds__(1024) k_spec_sum_check(const float *v, int n, float *sums, int *misses,
                                                         long long *cycles) {
  extern __shared__ __align__(16) float row[];
  __shared__ float s_loop;
  const int r = blockIdx.x, n4 = (n + 3) & ~3;
  void *scratch = row + n4;
  for (int k = threadIdx.x; k < n; k += blockDim.x) row[k] = v[(size_t)r * n + k];
  __syncthreads();
  const long long t0 = clock64();
  int miss = 0;
  const float s = spec_seq_sum(row, n, 0.0f, scratch, &miss);
  const long long t1 = clock64();
  if (threadIdx.x == 0) s_loop = seq_sum_a16(row, n, 0.0f);
  __syncthreads();
  const long long t2 = clock64();
  if (threadIdx.x == 0) {
    sums[2 * r] = s;
    sums[2 * r + 1] = s_loop;
    misses[r] = miss;
    cycles[2 * r] = t1 - t0;
    cycles[2 * r + 1] = t2 - t1;
  }
}
}  // namespace

// The block-wide sequential sum of the RMSNorm prologues, checked on given
// rows: for each of `rows` rows of n floats (host memory), sums[2r] is the
// block's result, sums[2r+1] the one-thread loop's, misses[r] the segments that
// were summed again, cycles[2r] / cycles[2r+1] the two methods' SM cycles.
// threads: the block size (a multiple of 32, 64..1024).
extern "C" LLMQ_API int llmq_spec_sum_check(const float *v, int rows, int n, int threads, float *sums, int *misses,
                                            long long *cycles) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevCtx *c = get_ctx();
  if (!c) return q_llama_last_error();
  const size_t smem = (size_t)((n + 3) & ~3) * 4 + spec_sum_bytes();
  if (!v || !sums || !misses || !cycles || rows <= 0 || n < 0 || threads < 64 || threads > 1024 || threads % 32 ||
      smem > (size_t)c->max_smem) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_spec_sum_check: bad arguments");
    return LLMQ_ERR_ARG;
  }
  float *dv = nullptr, *ds = nullptr;
  int *dm = nullptr;
  long long *dc = nullptr;
  int rc = LLMQ_OK;
  const size_t vb = (size_t)rows * n * sizeof(float);
  cudaError_t e = cudaMalloc(&dv, vb ? vb : 4);
  if (e == cudaSuccess) e = cudaMalloc(&ds, (size_t)rows * 2 * sizeof(float));
  if (e == cudaSuccess) e = cudaMalloc(&dm, (size_t)rows * sizeof(int));
  if (e == cudaSuccess) e = cudaMalloc(&dc, (size_t)rows * 2 * sizeof(long long));
  if (e == cudaSuccess && vb) e = upload_sync(dv, v, vb);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(k_spec_sum_check, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 static_cast<int>(smem));
  if (e == cudaSuccess) {
    k_spec_sum_check<<<rows, threads, smem, c->stream>>>(dv, n, ds, dm, dc);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(sums, ds, (size_t)rows * 2 * sizeof(float), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(misses, dm, (size_t)rows * sizeof(int), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(cycles, dc, (size_t)rows * 2 * sizeof(long long), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) {
    llmq_set_error(LLMQ_ERR_CUDA, "llmq_spec_sum_check: %s", cudaGetErrorString(e));
    rc = LLMQ_ERR_CUDA;
  }
  cudaFree(dv);
  cudaFree(ds);
  cudaFree(dm);
  cudaFree(dc);
  return rc;
}

// Failure detection on one GPU: drives the tensor-parallel peer-flag waits to
// their limit.  A two-rank exchange is set up whose second "rank" is a local
// region that nothing writes, so every wait on that rank's flag gives up after
// `polls` polls (0 would be the production bound of about a second; the test
// passes a few thousand).  which 0: k_tp_absmax (the absmax exchange); 1: the
// row-parallel GEMV (EPI_TP_RESID) on a 512 x 512 matrix, whose slab-completing
// CTAs wait for the missing rank's partial sums.  The kernel must return by
// itself: *err_word receives the device error word (ERR_TIMEOUT expected) and
// *ms the kernel's duration.  Returns LLMQ_ERR_CUDA when the error word is set,
// as the decode path does, LLMQ_OK when it is not; everything the check
// allocated is freed, and the device stays usable.
extern "C" LLMQ_API int llmq_tp_wait_timeout_check(int which, unsigned polls, int *err_word, float *ms) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevCtx *c = get_ctx();
  if (!c) return q_llama_last_error();
  if ((which != 0 && which != 1) || polls == 0 || !err_word || !ms) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_tp_wait_timeout_check: bad arguments");
    return LLMQ_ERR_ARG;
  }
  constexpr int kW = 2, kDm = 512, kK = 512;
  const size_t rb = tpx_bytes(kW, kDm);
  char *region[kW] = {nullptr, nullptr};
  char **peers = nullptr;
  unsigned *seq = nullptr;
  int *err = nullptr, *acc = nullptr, *cnt = nullptr;
  float *x = nullptr, *out = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
  Mat m;
  int rc = LLMQ_OK;
  std::vector<float> hx(kK);
  for (int k = 0; k < kK; ++k) hx[k] = (float)((k * 37) % 101 - 50) * 0.03125f;
  std::vector<signed char> hq((size_t)kK * kDm);
  for (size_t i = 0; i < hq.size(); ++i) hq[i] = (signed char)((int)((i * 2654435761u) >> 24) % 255 - 127);
  std::vector<float> hs(kDm, 0.004f);
  QTensor W{kK, kDm, hq.data(), hs.data()};
  bool ok = cudaMalloc(&region[0], rb) == cudaSuccess && cudaMalloc(&region[1], rb) == cudaSuccess &&
            zero_sync(region[0], rb) == cudaSuccess && zero_sync(region[1], rb) == cudaSuccess &&
            cudaMalloc(&peers, sizeof(region)) == cudaSuccess &&
            upload_sync(peers, region, sizeof(region)) == cudaSuccess &&
            cudaMalloc(&seq, sizeof(unsigned)) == cudaSuccess && zero_sync(seq, sizeof(unsigned)) == cudaSuccess &&
            cudaMalloc(&err, sizeof(int)) == cudaSuccess && zero_sync(err, sizeof(int)) == cudaSuccess &&
            cudaMalloc(&x, kK * sizeof(float)) == cudaSuccess &&
            upload_sync(x, hx.data(), kK * sizeof(float)) == cudaSuccess &&
            cudaMalloc(&out, kDm * sizeof(float)) == cudaSuccess && zero_sync(out, kDm * sizeof(float)) == cudaSuccess;
  ok = ok && build_plain(m, W, 1);
  GemvPlan plan;
  ok = ok && plan_gemv(*c, m, PRO_ABSMAX, 1, plan);
  ok = ok && cudaMalloc(&acc, (size_t)m.Npad * sizeof(int)) == cudaSuccess &&
       zero_sync(acc, (size_t)m.Npad * sizeof(int)) == cudaSuccess &&
       cudaMalloc(&cnt, (size_t)m.n_slabs * sizeof(int)) == cudaSuccess &&
       zero_sync(cnt, (size_t)m.n_slabs * sizeof(int)) == cudaSuccess;
  if (!ok) {
    if (q_llama_last_error() == LLMQ_OK) llmq_set_error(LLMQ_ERR_OOM, "llmq_tp_wait_timeout_check: set-up failed");
    rc = q_llama_last_error();
  } else {
    TpExchange t{};
    t.peers = peers;
    t.seq = seq;
    t.rank = 0;
    t.world = kW;
    t.dm = kDm;
    t.pidx = 0;
    t.poll_limit = polls;
    cudaStream_t st = c->stream;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, st);
    cudaError_t e;
    if (which == 0) {
      k_tp_absmax<<<1, kThreads, 0, st>>>(x, kK, out, t, err);
      e = cudaGetLastError();
    } else {
      GemvArgs a = base_args(m, plan, acc, cnt, err);
      a.in = x;
      a.out = out;
      a.tp = t;
      e = launch_gemv<PRO_ABSMAX, EPI_TP_RESID, 1>(a, plan, st, false);
    }
    cudaEventRecord(e1, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
      llmq_set_error(LLMQ_ERR_CUDA, "llmq_tp_wait_timeout_check: %s", cudaGetErrorString(e));
      rc = LLMQ_ERR_CUDA;
    } else {
      cudaEventElapsedTime(ms, e0, e1);
      cudaMemcpy(err_word, err, sizeof(int), cudaMemcpyDeviceToHost);
      if (*err_word) {
        llmq_set_error(LLMQ_ERR_CUDA, "libllmq_cuda: device reported error flags 0x%x (peer flag wait gave up)",
                       *err_word);
        rc = LLMQ_ERR_CUDA;
      }
    }
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
  }
  cudaFree(region[0]);
  cudaFree(region[1]);
  cudaFree(peers);
  cudaFree(seq);
  cudaFree(err);
  cudaFree(x);
  cudaFree(out);
  cudaFree(acc);
  cudaFree(cnt);
  free_mat(m);
  return rc;
}

// RMSNorm of one row (rmsnorm.c:7-21) followed by qmatmul of the normalised
// row (quant.c:60-85), as the GEMV with the RMSNorm prologue computes it for
// QKV, W1|W3 and the lm-head inside a decode step: out[N] = qmatmul(rmsnorm(x,
// gamma, eps), W).  For tests of that prologue on chosen rows.
extern "C" LLMQ_API int llmq_rmsnorm_qmatmul(const float *x, const float *gamma, float eps, const QTensor *W,
                                             float *out) {
  std::lock_guard<std::recursive_mutex> lk(g_mu);
  DevCtx *c = get_ctx();
  if (!c) return q_llama_last_error();
  if (!x || !gamma || !W || !out || W->rows <= 0 || W->cols <= 0) {
    llmq_set_error(LLMQ_ERR_ARG, "llmq_rmsnorm_qmatmul: bad arguments");
    return LLMQ_ERR_ARG;
  }
  const int K = W->rows, N = W->cols;
  Mat m;
  if (!build_plain(m, *W, 1)) return q_llama_last_error();
  GemvPlan plan;
  float *dx = nullptr, *dg = nullptr, *dout = nullptr;
  int rc = LLMQ_OK;
  if (!plan_gemv(*c, m, PRO_RMSNORM, 1, plan)) {
    rc = q_llama_last_error();
  } else if (cudaMalloc(&dx, (size_t)K * 4) != cudaSuccess || cudaMalloc(&dg, (size_t)K * 4) != cudaSuccess ||
             cudaMalloc(&dout, (size_t)N * 4) != cudaSuccess ||
             !ensure(&c->acc, &c->acc_n, (size_t)8 * m.Npad, true) ||
             !ensure(&c->cnt, &c->cnt_n, (size_t)m.n_slabs, true)) {
    llmq_set_error(LLMQ_ERR_OOM, "llmq_rmsnorm_qmatmul: allocation failed");
    rc = LLMQ_ERR_OOM;
  } else {
    cudaStream_t st = c->stream;
    GemvArgs a = base_args(m, plan, c->acc, c->cnt, c->err);
    a.in = dx;
    a.gamma = dg;
    a.eps = eps;
    a.out = dout;
    int flags = 0;
    cudaError_t e = cudaMemcpyAsync(dx, x, (size_t)K * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(dg, gamma, (size_t)K * 4, cudaMemcpyHostToDevice, st);
    if (e == cudaSuccess) e = launch_gemv<PRO_RMSNORM, EPI_PLAIN, 1>(a, plan, st, false);
    if (e == cudaSuccess) e = cudaMemcpyAsync(out, dout, (size_t)N * 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaMemcpyAsync(&flags, c->err, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) {
      llmq_set_error(LLMQ_ERR_CUDA, "llmq_rmsnorm_qmatmul: %s", cudaGetErrorString(e));
      rc = LLMQ_ERR_CUDA;
    } else if (flags) {
      zero_sync(c->err, 16);
      llmq_set_error(LLMQ_ERR_CUDA, "llmq_rmsnorm_qmatmul: device error flags 0x%x", flags);
      rc = LLMQ_ERR_CUDA;
    }
  }
  cudaFree(dx);
  cudaFree(dg);
  cudaFree(dout);
  free_mat(m);
  return rc;
}
