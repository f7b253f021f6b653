// C ABI of the B200 quantized-matmul hot path (include/llmq.h).
#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/llmq.h"
#include "attention.cuh"
#include "batch.cuh"
#include "dense.cuh"
#include "gemv_a16.cuh"
#include "gemv_float.cuh"
#include "mega.cuh"
#include "cluster.cuh"
#include "prefill_a16.cuh"
#include "sample.cuh"
#include "tc_gemm.cuh"
#include "tcl_gemm.cuh"

using namespace llmq;

struct llmq_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t own = nullptr;
  cudaStream_t stream = nullptr;
  std::string err;
  // scratch owned by the context (grown on demand)
  void *scratch = nullptr;
  size_t scratch_bytes = 0;
  DecodeState *state = nullptr;  // device, for llmq_head_argmax
  int dense_parts = 4;           // gemv's parts: the reference team of 4 threads (gpt2t.mojo:281 on 4 cores)
  int prefill_kernel = LLMQ_PREFILL_AUTO;
  long long wait_cycles = 4000000000LL;  // limit of a persistent kernel's or a row GEMV's device-side wait
  int *tc_err = nullptr;         // device error code of the tcgen05 GEMM (a wait that gave up)
  bool tc_used = false;          // a tcgen05 GEMM ran since the last check
  // sampling scratch (device, grown on demand): sort keys, chunk candidates,
  // the Rng state of llmq_generate_sampled
  unsigned long long *samp_keys = nullptr;
  unsigned long long *samp_cand = nullptr;
  unsigned long long *samp_rng = nullptr;
  int *samp_done = nullptr;  // set by topk_fast_kernel when it finished the draw
  int samp_n = 0;
};

enum { WK_AFFINE = 0, WK_GGUF = 1, WK_DENSE = 2 };

struct llmq_weight {
  llmq_ctx *ctx;
  int kind = WK_AFFINE;
  int bits = 0, group = 0, sym = 0, a16 = 0, blocked = 0;
  int rows = 0, cols = 0;
  uint8_t *codes = nullptr;  // affine codes; GGUF blocks; dense values
  uint16_t *scale = nullptr;
  uint8_t *zp = nullptr;
  int rtype = 0;             // GGUF / dense: the RT_* row type
  long long row_bytes = 0;
  long long nbytes = 0;
  mutable uint8_t *tc_b = nullptr;  // split-int8 GEMM tiles of the codes, built on first several-token use
  mutable int tc_tn = 0;            // their output tile width
  mutable uint8_t *tc_w = nullptr;  // the transposed GEMM's 128-row weight tiles (first use)
  mutable int *tc_wsum = nullptr;   // and the rows' per-segment sums of the weight values
  mutable uint8_t *tcl_a = nullptr; // the lane-mode GEMM's weight tiles (batched decode)
  WeightView view() const { return WeightView{codes, scale, zp, rows, cols, group, bits, blocked}; }
  RowMat rowmat() const { return RowMat{codes, rows, cols, rtype, row_bytes}; }
};

struct llmq_kv {
  llmq_ctx *ctx;
  int kind;
  int n_layer, max_t, n_head, head_dim;
  KV8View v8{};  // LLMQ_KV_QUANT8
  IAView ia{};   // LLMQ_KV_INTATTN
};

struct llmq_model {
  llmq_ctx *ctx;
  int n_layer, C, V, max_t, n_head;
  std::vector<const llmq_weight *> mats;
  const llmq_weight *head;
  const llmq_weight *embed = nullptr;  // token embeddings when they are not the head (an untied GGUF output.weight)
  llmq_kv *kv;
  float *small;  // device copy of the float32 parameters
  float *x, *xn, *qkv, *att, *fc, *logits;
  int *tokens;
  int *ids;
  int max_ids;
  float *part_val;
  int *part_idx;
  DecodeState *state;
  DecodeState *state_host;  // pinned staging
  int *ids_host;            // pinned staging
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int mode = LLMQ_MODE_GRAPH;
  // persistent decode kernel (mega.cuh)
  bool mega_ok = false;
  int mega_grid = 0, mega_nchunks = 0;
  uint8_t *mega_stream = nullptr;
  long long *mega_base = nullptr;
  MkChunk *mega_chunks = nullptr;
  unsigned long long *mega_ll = nullptr;
  int *mega_err = nullptr;
  unsigned mega_flag = 1;
  // cluster decode kernel (cluster.cuh); shares mega_err
  bool cd_ok = false;
  int cd_grid = 0, cd_nhcta = 0;
  uint8_t *cd_lstream = nullptr, *cd_hstream = nullptr;
  long long *cd_lbase = nullptr, *cd_lbytes = nullptr, *cd_hbase = nullptr;
  CdChunk *cd_lchunks = nullptr;
  int *cd_lnch = nullptr;
  unsigned long long *cd_ll = nullptr;
  unsigned cd_flag = 1;
  bool float_only = false;  // float-activation formats: the generic eager decode
  std::vector<llmq_weight *> owned;  // weights a loader created for this model
  long long *prof = nullptr;  // [2][MK_PROF] when profiling
  const float *vec(int l, int which) const {
    static const int mult[8] = {0, 1, 2, 5, 6, 7, 8, 12};
    return small + (size_t)l * 13 * C + (size_t)mult[which] * C;
  }
  const float *wpe() const { return small + (size_t)n_layer * 13 * C; }
  const float *lnf_w() const { return wpe() + (size_t)1024 * C; }
  const float *lnf_b() const { return lnf_w() + C; }
};

namespace {

llmq_status fail(llmq_ctx *ctx, llmq_status st, const std::string &msg) {
  if (ctx) ctx->err = msg;
  return st;
}

#define CK(call)                                                                                 \
  do {                                                                                           \
    cudaError_t e_ = (call);                                                                     \
    if (e_ != cudaSuccess)                                                                       \
      return fail(ctx, LLMQ_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));     \
  } while (0)

#define CKL()                                                                                    \
  do {                                                                                           \
    cudaError_t e_ = cudaGetLastError();                                                         \
    if (e_ != cudaSuccess) return fail(ctx, LLMQ_ERR_CUDA, std::string("launch: ") + cudaGetErrorString(e_)); \
  } while (0)

constexpr int kMaxPrefillSmem = 225 * 1024;  // the several-token attention's staging limit
constexpr int kBgemvSmem = 200 * 1024;       // the batched GEMV's shared memory limit
constexpr int kR = 16, kP = 3;
constexpr int kThreads = kR * kP * 4;

// Matrices with fewer rows than this use tiles of 4 rows x 12 parts (the
// same 192 threads), so that the grid still covers every SM.
constexpr int kR2 = 4, kP2 = 12;
constexpr int kShortRows = 2048;
static_assert(kR2 * kP2 == kR * kP, "both tile shapes launch kThreads threads");
bool use_short(const WeightView &w) { return w.rows < kShortRows; }

template <int FMT>
int smem_bytes_r(const WeightView &w, int R) {
  SmemPlan<FMT> pl(w.cols, w.group, R);
  return pl.total;
}
template <int FMT>
int smem_bytes(const WeightView &w) {
  return smem_bytes_r<FMT>(w, use_short(w) ? kR2 : kR);
}

constexpr int kMaxSmem = 200 * 1024;

// From this many rows on, the whole-row kernel (4 threads per row, no split
// along the row) has enough rows to fill the GPU and wins.
constexpr int kTallRows = 8192;
bool use_tall(const WeightView &w) { return w.rows >= kTallRows; }
// The head formats with whole 256-column slabs stream through per-warp
// cp.async rings instead of register slabs.
bool use_ring(const WeightView &w) {
  if (!use_tall(w) || w.cols % 256) return false;
  if (w.blocked) return ring_smem<FMT_BLK4>(w.cols, w.group) <= kMaxSmem;
  return w.bits == 8 && w.group == w.cols && ring_smem<FMT_GEN8>(w.cols, w.group) <= kMaxSmem;
}

template <int FMT, int PRO, bool ARG>
cudaError_t launch_gemv_t(const GemvArgs &a, int grid, cudaStream_t s) {
  if ((FMT == FMT_BLK4 || FMT == FMT_GEN8) && use_ring(a.w))
    gemv_ring_kernel<FMT == FMT_BLK4 ? FMT_BLK4 : FMT_GEN8, PRO, ARG>
        <<<grid, kRingWarps * 32, ring_smem<FMT == FMT_BLK4 ? FMT_BLK4 : FMT_GEN8>(a.w.cols, a.w.group), s>>>(a);
  else if (use_tall(a.w))
    gemv_tall_kernel<FMT, PRO, ARG><<<grid, kTallWarps * 32, SmemPlan<FMT>(a.w.cols, a.w.group, 0).total, s>>>(a);
  else if (use_short(a.w))
    gemv_a16_kernel<FMT, PRO, kR2, kP2, ARG><<<grid, kThreads, smem_bytes<FMT>(a.w), s>>>(a);
  else
    gemv_a16_kernel<FMT, PRO, kR, kP, ARG><<<grid, kThreads, smem_bytes<FMT>(a.w), s>>>(a);
  return cudaGetLastError();
}

template <int FMT>
cudaError_t configure_fmt() {
  cudaError_t e = cudaSuccess;
  auto set = [&](const void *k) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  };
  set((const void *)gemv_a16_kernel<FMT, PRO_LN, kR, kP, true>);
  set((const void *)gemv_a16_kernel<FMT, PRO_LN, kR, kP, false>);
  set((const void *)gemv_a16_kernel<FMT, PRO_QUANT, kR, kP, true>);
  set((const void *)gemv_a16_kernel<FMT, PRO_QUANT, kR, kP, false>);
  set((const void *)gemv_a16_kernel<FMT, PRO_LN, kR2, kP2, true>);
  set((const void *)gemv_a16_kernel<FMT, PRO_LN, kR2, kP2, false>);
  set((const void *)gemv_a16_kernel<FMT, PRO_QUANT, kR2, kP2, true>);
  set((const void *)gemv_a16_kernel<FMT, PRO_QUANT, kR2, kP2, false>);
  set((const void *)gemv_tall_kernel<FMT, PRO_LN, true>);
  set((const void *)gemv_tall_kernel<FMT, PRO_LN, false>);
  set((const void *)gemv_tall_kernel<FMT, PRO_QUANT, true>);
  set((const void *)gemv_tall_kernel<FMT, PRO_QUANT, false>);
  if (FMT != FMT_GEN4) {
    constexpr int RF = FMT == FMT_BLK4 ? FMT_BLK4 : FMT_GEN8;
    set((const void *)gemv_ring_kernel<RF, PRO_LN, true>);
    set((const void *)gemv_ring_kernel<RF, PRO_LN, false>);
    set((const void *)gemv_ring_kernel<RF, PRO_QUANT, true>);
    set((const void *)gemv_ring_kernel<RF, PRO_QUANT, false>);
  }
  if (FMT == FMT_BLK4) {  // once: the dense strips
    auto set_ds = [&](const void *k) {
      if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, DS_SMEM);
    };
    set_ds((const void *)dense_strip_kernel<0>);
    set_ds((const void *)dense_strip_kernel<1>);
    set_ds((const void *)dense_strip_kernel<2>);
  }
  return e;
}

int fmt_of(const WeightView &w) { return w.blocked ? FMT_BLK4 : (w.bits == 4 ? FMT_GEN4 : FMT_GEN8); }

int gemv_grid(const llmq_ctx *ctx, const WeightView &w) {
  if (use_ring(w)) return ctx->num_sms * kRingBlocks;
  if (use_tall(w)) {
    const int ctas = ((w.rows + 7) / 8 + kTallWarps - 1) / kTallWarps;
    return std::min(ctas, ctx->num_sms * kTallMinBlocks);
  }
  const int r = use_short(w) ? kR2 : kR;
  int tiles = (w.rows + r - 1) / r;
  int cap = ctx->num_sms * 8;
  return tiles < cap ? tiles : cap;
}

cudaError_t launch_gemv(const llmq_ctx *ctx, const GemvArgs &a, int pro, bool argmax, cudaStream_t s) {
  int grid = gemv_grid(ctx, a.w);
  int fmt = fmt_of(a.w);
#define DISPATCH(F)                                                             \
  if (fmt == F) {                                                               \
    if (pro == PRO_LN)                                                          \
      return argmax ? launch_gemv_t<F, PRO_LN, true>(a, grid, s) : launch_gemv_t<F, PRO_LN, false>(a, grid, s); \
    return argmax ? launch_gemv_t<F, PRO_QUANT, true>(a, grid, s) : launch_gemv_t<F, PRO_QUANT, false>(a, grid, s); \
  }
  DISPATCH(FMT_BLK4)
  DISPATCH(FMT_GEN4)
  DISPATCH(FMT_GEN8)
#undef DISPATCH
  return cudaErrorInvalidValue;
}

bool smem_ok(const WeightView &w) {
  int fmt = fmt_of(w);
  int b = fmt == FMT_BLK4 ? smem_bytes_r<FMT_BLK4>(w, kR)
                          : (fmt == FMT_GEN4 ? smem_bytes_r<FMT_GEN4>(w, kR) : smem_bytes_r<FMT_GEN8>(w, kR));
  return b <= kMaxSmem;
}

// Reads (and clears) the tcgen05 GEMM's error code once a GEMM ran; call
// after the stream was synchronised.
llmq_status tc_check(llmq_ctx *ctx) {
  if (!ctx->tc_used) return LLMQ_OK;
  ctx->tc_used = false;
  int code = 0;
  CK(cudaMemcpy(&code, ctx->tc_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code == 0) return LLMQ_OK;
  CK(cudaMemset(ctx->tc_err, 0, sizeof(int)));
  return fail(ctx, LLMQ_ERR_TIMEOUT, "a tcgen05 GEMM wait gave up (code " + std::to_string(code) + ")");
}

llmq_status ensure_scratch(llmq_ctx *ctx, size_t bytes) {
  if (ctx->scratch_bytes >= bytes) return LLMQ_OK;
  if (ctx->scratch) cudaFree(ctx->scratch);
  ctx->scratch = nullptr;
  ctx->scratch_bytes = 0;
  CK(cudaMalloc(&ctx->scratch, bytes));
  ctx->scratch_bytes = bytes;
  return LLMQ_OK;
}

}  // namespace

template <int FMT>
__global__ void __launch_bounds__(kThreads) lane_sums_kernel(GemvArgs a, int32_t *lanes_out);

namespace {
// Raises the dynamic shared-memory limit of every kernel once, outside any
// stream capture.
cudaError_t configure_kernels() {
  cudaError_t e = configure_fmt<FMT_BLK4>();
  if (e == cudaSuccess) e = configure_fmt<FMT_GEN4>();
  if (e == cudaSuccess) e = configure_fmt<FMT_GEN8>();
  if (e == cudaSuccess) e = cudaFuncSetAttribute((const void *)lane_sums_kernel<FMT_BLK4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute((const void *)lane_sums_kernel<FMT_GEN4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute((const void *)lane_sums_kernel<FMT_GEN8>, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void *)mega_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(MkSmem));
  const int rsm = 4096 * 4 + 128 + RF_STAGES * RF_TILE_BYTES;
  auto rs = [&](const void *k) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, rsm);
  };
  rs((const void *)row_gemv_kernel<RT_F32>);
  rs((const void *)row_gemv_kernel<RT_F16>);
  rs((const void *)row_gemv_kernel<RT_BF16>);
  rs((const void *)row_gemv_kernel<RT_Q4_0>);
  rs((const void *)row_gemv_kernel<RT_Q4_1>);
  rs((const void *)row_gemv_kernel<RT_Q8_0>);
  rs((const void *)row_gemv_kernel<RT_Q4_K>);
  rs((const void *)row_gemv_kernel<RT_Q5_K>);
  rs((const void *)row_gemv_kernel<RT_Q6_K>);
  for (const void *k : {(const void *)kv_prefill_kernel<0>, (const void *)kv_prefill_kernel<1>,
                        (const void *)kv_prefill_kernel<2>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxPrefillSmem);
  for (const void *k : {(const void *)kv8_attend_kernel<false, 0>, (const void *)kv8_attend_kernel<true, 0>,
                        (const void *)kv8_attend_kernel<true, 64>})
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  auto tcs = [&](const void *k) {
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(TcSmem) + 1024);
  };
  tcs((const void *)tc_gemm_a16_kernel<true, 64>);
  tcs((const void *)tc_gemm_a16_kernel<true, 32>);
  tcs((const void *)tc_gemm_a16_kernel<false, 64>);
  tcs((const void *)tc_gemm_a16_kernel<false, 32>);
  auto tct = [&](const void *k, size_t n) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)n + 1024);
  };
  tct((const void *)tct_gemm_kernel<true, 32>, sizeof(TcSmemT<32>));
  tct((const void *)tct_gemm_kernel<false, 32>, sizeof(TcSmemT<32>));
  tct((const void *)tct_gemm_kernel<true, 64>, sizeof(TcSmemT<64>));
  tct((const void *)tct_gemm_kernel<false, 64>, sizeof(TcSmemT<64>));
  tct((const void *)tcp_gemm_kernel, sizeof(TcpSmem));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void *)merge_draw_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)merge_smem(kMergeCap));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute((const void *)topk_fast_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)fast_smem());
  return e;
}
}  // namespace

// Debug: lane sums of one row range. Runs the PRO_QUANT prologue and the
// integer phase, then copies the lane sums (zero point applied for the
// grouped layouts) to lanes_out[rows][units][16].
template <int FMT>
__global__ void __launch_bounds__(kThreads) lane_sums_kernel(GemvArgs a, int32_t *lanes_out) {
  extern __shared__ __align__(16) unsigned char smem[];
  SmemPlan<FMT> pl(a.w.cols, a.w.group, kR);
  prologue<FMT, PRO_QUANT>(a, smem, pl);
  const int units = FMT == FMT_BLK4 ? a.w.cols >> 8 : a.w.cols / a.w.group;
  int *lanes_all = (int *)(smem + pl.lanes);
  const int *xp32 = (const int *)(smem + pl.xq);
  const int *xsum = (const int *)(smem + pl.xs);
  const int t = threadIdx.x, q = t & 3, p = (t >> 2) % kP, r = (t >> 2) / kP;
  for (int row0 = blockIdx.x * kR; row0 < a.w.rows; row0 += gridDim.x * kR) {
    for (int i = t; i < kR * units * 16; i += blockDim.x) lanes_all[i] = 0;
    __syncthreads();
    const int row = row0 + r;
    if (row < a.w.rows) int_phase<FMT, kP>(a.w, row, q, p, xp32, lanes_all + r * units * 16);
    __syncthreads();
    for (int i = t; i < kR * units * 16; i += blockDim.x) {
      int rr = row0 + i / (units * 16), u = (i / 16) % units, L = i % 16;
      if (rr >= a.w.rows) continue;
      int v = lanes_all[i];
      if (FMT != FMT_BLK4) {
        int zp = a.w.zp[(size_t)rr * units + u];
        v = (int)((unsigned)v - (unsigned)(zp * xsum[u * 16 + L]));
      }
      lanes_out[(size_t)rr * units * 16 + u * 16 + L] = v;
    }
    __syncthreads();
  }
}

namespace {
// Contexts alive per device, and the device address of the no-allocation
// entry point's scratch array (g_head_argmax_scratch) on each device, looked
// up by its first call there. The address belongs to the device's context:
// when the last llmq context of a device is destroyed it is dropped, so a
// context created after cudaDeviceReset looks it up again.
constexpr int kNoallocMaxDevices = 64;
std::mutex g_noalloc_mu;
int g_dev_contexts[kNoallocMaxDevices] = {};
void *g_noalloc_ptr[kNoallocMaxDevices] = {};
}  // namespace

extern "C" {

llmq_status llmq_init(int device, llmq_ctx **out) {
  if (!out) return LLMQ_ERR_INVALID;
  *out = nullptr;
  llmq_ctx *ctx = new llmq_ctx();
  ctx->device = device;
  cudaError_t e = cudaSetDevice(device);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&ctx->num_sms, cudaDevAttrMultiProcessorCount, device);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->own, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaMalloc(&ctx->state, sizeof(DecodeState));
  if (e == cudaSuccess) e = cudaMemset(ctx->state, 0, sizeof(DecodeState));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->tc_err, sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(ctx->tc_err, 0, sizeof(int));
  if (e == cudaSuccess) e = configure_kernels();
  if (e != cudaSuccess) {
    delete ctx;
    return LLMQ_ERR_CUDA;
  }
  ctx->stream = ctx->own;
  if (device >= 0 && device < kNoallocMaxDevices) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    g_dev_contexts[device]++;
  }
  *out = ctx;
  return LLMQ_OK;
}

llmq_status llmq_destroy(llmq_ctx *ctx) {
  if (!ctx) return LLMQ_ERR_INVALID;
  if (ctx->device >= 0 && ctx->device < kNoallocMaxDevices) {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (--g_dev_contexts[ctx->device] == 0) g_noalloc_ptr[ctx->device] = nullptr;
  }
  cudaSetDevice(ctx->device);
  if (ctx->own) cudaStreamSynchronize(ctx->own);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->state) cudaFree(ctx->state);
  if (ctx->tc_err) cudaFree(ctx->tc_err);
  for (void *q : {(void *)ctx->samp_keys, (void *)ctx->samp_cand, (void *)ctx->samp_rng, (void *)ctx->samp_done})
    if (q) cudaFree(q);
  if (ctx->own) cudaStreamDestroy(ctx->own);
  delete ctx;
  return LLMQ_OK;
}

const char *llmq_last_error(const llmq_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

llmq_status llmq_set_stream(llmq_ctx *ctx, void *s) {
  if (!ctx) return LLMQ_ERR_INVALID;
  ctx->stream = s ? (cudaStream_t)s : ctx->own;
  return LLMQ_OK;
}

void *llmq_stream(const llmq_ctx *ctx) { return ctx ? (void *)ctx->stream : nullptr; }

llmq_status llmq_sync(llmq_ctx *ctx) {
  if (!ctx) return LLMQ_ERR_INVALID;
  CK(cudaStreamSynchronize(ctx->stream));
  return tc_check(ctx);
}

llmq_status llmq_set_wait_limit(llmq_ctx *ctx, long long cycles) {
  if (!ctx || cycles < 0) return fail(ctx, LLMQ_ERR_INVALID, "bad wait limit");
  ctx->wait_cycles = cycles == 0 ? 4000000000LL : cycles;
  return LLMQ_OK;
}

llmq_status llmq_set_prefill_kernel(llmq_ctx *ctx, int kind) {
  if (!ctx || kind < LLMQ_PREFILL_AUTO || kind > LLMQ_PREFILL_TCGEN05) return fail(ctx, LLMQ_ERR_INVALID, "bad kind");
  ctx->prefill_kernel = kind;
  return LLMQ_OK;
}

llmq_status llmq_weight_create_affine(llmq_ctx *ctx, int bits, int group, int sym, int a16, int rows, int cols,
                                      const uint8_t *codes, const uint16_t *scale, const uint8_t *zp,
                                      llmq_weight **out) {
  if (!ctx || !out || !codes || !scale || !zp) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  *out = nullptr;
  int g = group == 0 ? cols : group;
  if ((bits != 4 && bits != 8) || rows <= 0 || cols <= 0 || group < 0 || cols % g != 0 || g % 32 != 0)
    return fail(ctx, LLMQ_ERR_INVALID, "group size must divide the reduction axis and be a multiple of 32");
  int blocked = a16 && bits == 4 && group == 32;
  if (blocked && cols % 256 != 0) return fail(ctx, LLMQ_ERR_INVALID, "the BLOCKED layout needs cols % 256 == 0");
  CK(cudaSetDevice(ctx->device));
  llmq_weight *w = new llmq_weight();
  w->ctx = ctx;
  w->bits = bits;
  w->group = g;
  w->sym = sym;
  w->a16 = a16;
  w->blocked = blocked;
  w->rows = rows;
  w->cols = cols;
  size_t nc = (size_t)rows * cols * bits / 8, ng = (size_t)rows * (cols / g);
  w->nbytes = (long long)(nc + 3 * ng);
  cudaError_t e = cudaMalloc(&w->codes, nc);
  if (e == cudaSuccess) e = cudaMalloc(&w->scale, ng * 2);
  if (e == cudaSuccess) e = cudaMalloc(&w->zp, ng);
  if (e == cudaSuccess) e = cudaMemcpy(w->codes, codes, nc, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(w->scale, scale, ng * 2, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMemcpy(w->zp, zp, ng, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    llmq_weight_free(w);
    return fail(ctx, LLMQ_ERR_CUDA, std::string("weight upload: ") + cudaGetErrorString(e));
  }
  if (!smem_ok(w->view())) {
    llmq_weight_free(w);
    return fail(ctx, LLMQ_ERR_UNSUPPORTED, "matrix too wide for the one-token kernel's shared memory");
  }
  *out = w;
  return LLMQ_OK;
}

llmq_status llmq_weight_create_gguf(llmq_ctx *ctx, int ggml_type, const void *blocks, int rows, int cols,
                                    llmq_weight **out) {
  if (!ctx || !out || !blocks || rows <= 0 || cols <= 0) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  *out = nullptr;
  static const int types[] = {RT_F32, RT_F16, RT_Q4_0, RT_Q4_1, RT_Q8_0, RT_Q4_K, RT_Q5_K, RT_Q6_K};
  bool known = false;
  for (int t : types) known |= t == ggml_type;
  if (!known) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "GGUF type " + std::to_string(ggml_type) + " not supported");
  const int bs = (ggml_type == RT_F32 || ggml_type == RT_F16) ? 1 : rt_block_size(ggml_type);
  const int bb = (ggml_type == RT_F32) ? 4 : (ggml_type == RT_F16) ? 2 : rt_block_bytes(ggml_type);
  if (cols % 16 != 0 || cols % bs != 0 || cols > 4096)
    return fail(ctx, LLMQ_ERR_INVALID, "columns must be a multiple of the block size (and of 16, at most 4096)");
  CK(cudaSetDevice(ctx->device));
  llmq_weight *w = new llmq_weight();
  w->ctx = ctx;
  w->kind = WK_GGUF;
  w->rtype = ggml_type;
  w->rows = rows;
  w->cols = cols;
  w->row_bytes = (long long)(cols / bs) * bb;
  w->nbytes = w->row_bytes * rows;
  cudaError_t e = cudaMalloc(&w->codes, w->nbytes + 32);  // padding: tiles are copied as 16-byte aligned supersets
  if (e == cudaSuccess) e = cudaMemset(w->codes + w->nbytes, 0, 32);
  if (e == cudaSuccess) e = cudaMemcpy(w->codes, blocks, w->nbytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    llmq_weight_free(w);
    return fail(ctx, LLMQ_ERR_CUDA, std::string("weight upload: ") + cudaGetErrorString(e));
  }
  *out = w;
  return LLMQ_OK;
}

llmq_status llmq_weight_create_dense(llmq_ctx *ctx, int dtype, const void *data, int rows, int cols,
                                     llmq_weight **out) {
  if (!ctx || !out || !data || rows <= 0 || cols <= 0) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  if (dtype != LLMQ_DENSE_F32 && dtype != LLMQ_DENSE_F16 && dtype != LLMQ_DENSE_BF16)
    return fail(ctx, LLMQ_ERR_INVALID, "dtype must be LLMQ_DENSE_F32, _F16 or _BF16");
  *out = nullptr;
  CK(cudaSetDevice(ctx->device));
  llmq_weight *w = new llmq_weight();
  w->ctx = ctx;
  w->kind = WK_DENSE;
  w->rtype = dtype == LLMQ_DENSE_F32 ? RT_F32 : dtype == LLMQ_DENSE_F16 ? RT_F16 : RT_BF16;
  w->rows = rows;
  w->cols = cols;
  w->row_bytes = (long long)cols * (dtype == LLMQ_DENSE_F32 ? 4 : 2);
  w->nbytes = w->row_bytes * rows;
  cudaError_t e = cudaMalloc(&w->codes, w->nbytes + 32);
  if (e == cudaSuccess) e = cudaMemset(w->codes + w->nbytes, 0, 32);
  if (e == cudaSuccess) e = cudaMemcpy(w->codes, data, w->nbytes, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    llmq_weight_free(w);
    return fail(ctx, LLMQ_ERR_CUDA, std::string("weight upload: ") + cudaGetErrorString(e));
  }
  *out = w;
  return LLMQ_OK;
}

llmq_status llmq_weight_free(llmq_weight *w) {
  if (!w) return LLMQ_ERR_INVALID;
  if (w->codes) cudaFree(w->codes);
  if (w->scale) cudaFree(w->scale);
  if (w->zp) cudaFree(w->zp);
  if (w->tc_b) cudaFree(w->tc_b);
  if (w->tc_w) cudaFree(w->tc_w);
  if (w->tc_wsum) cudaFree(w->tc_wsum);
  if (w->tcl_a) cudaFree(w->tcl_a);
  delete w;
  return LLMQ_OK;
}

long long llmq_weight_nbytes(const llmq_weight *w) { return w ? w->nbytes : -1; }

}  // extern "C"

namespace {
template <int T>
cudaError_t launch_row_gemv(const llmq_ctx *ctx, const RowGemvArgs &a) {  // a.err / a.timeout set by row_gemv
  const int rb = (int)a.w.row_bytes;
  const int R = rf_rows(rb);
  const int ntiles = (a.w.rows + R - 1) / R;
  const int grid = std::min(ntiles, ctx->num_sms * 2);
  const int sm = a.w.cols * 4 + 128 + RF_STAGES * RF_TILE_BYTES;
  row_gemv_kernel<T><<<grid, RF_THREADS, sm, ctx->stream>>>(a);
  return cudaGetLastError();
}

// Launches the row GEMV with the context's wait limit and error word; a wait
// that gives up is reported by the next tc_check (llmq_sync and the calls
// that synchronise).
cudaError_t row_gemv(llmq_ctx *ctx, RowGemvArgs a) {
  a.err = ctx->tc_err;
  a.timeout = ctx->wait_cycles;
  ctx->tc_used = true;
  switch (a.w.type) {
    case RT_F32: return launch_row_gemv<RT_F32>(ctx, a);
    case RT_F16: return launch_row_gemv<RT_F16>(ctx, a);
    case RT_BF16: return launch_row_gemv<RT_BF16>(ctx, a);
    case RT_Q4_0: return launch_row_gemv<RT_Q4_0>(ctx, a);
    case RT_Q4_1: return launch_row_gemv<RT_Q4_1>(ctx, a);
    case RT_Q8_0: return launch_row_gemv<RT_Q8_0>(ctx, a);
    case RT_Q4_K: return launch_row_gemv<RT_Q4_K>(ctx, a);
    case RT_Q5_K: return launch_row_gemv<RT_Q5_K>(ctx, a);
    case RT_Q6_K: return launch_row_gemv<RT_Q6_K>(ctx, a);
  }
  return cudaErrorInvalidValue;
}
}  // namespace

extern "C" {

llmq_status llmq_set_dense_parts(llmq_ctx *ctx, int nparts) {
  if (!ctx || nparts <= 0 || nparts > 256) return fail(ctx, LLMQ_ERR_INVALID, "parts must be in [1, 256]");
  ctx->dense_parts = nparts;
  return LLMQ_OK;
}

}  // extern "C"

namespace {

// Whether the several-token A16 matmul of w runs on the tcgen05 GEMM: K in
// whole 128-byte blocks and segments, at most TC_MAX_GROUPS groups per row,
// and (AUTO) at least 16 tokens.
bool tc_eligible(const llmq_ctx *ctx, const llmq_weight *w, int T) {
  if (ctx->prefill_kernel == LLMQ_PREFILL_CUDA_CORE) return false;
  if (ctx->prefill_kernel == LLMQ_PREFILL_AUTO && T < 16) return false;
  const int K = w->cols, G = w->group, seg = std::min(G, 256);
  return w->kind == WK_AFFINE && w->a16 && K % TC_KB == 0 && K % seg == 0 && seg % 32 == 0 &&
         K / G <= TC_MAX_GROUPS && K / seg <= TC_MAX_GROUPS * 8 && w->rows >= 32;
}

size_t align256(size_t n) { return (n + 255) / 256 * 256; }

llmq_status dequant_rows(llmq_ctx *ctx, const llmq_weight *w, int r0, int nrows, float *dst) {
  if (w->kind == WK_AFFINE) {
    if (w->a16 || w->blocked) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "dequant_rows takes the natural layouts");
    const size_t bytes = (size_t)nrows * w->cols * w->bits / 8;
    const int grid = (int)std::min<size_t>((bytes + 255) / 256, (size_t)ctx->num_sms * 16);
    affine_dequant_rows_kernel<<<grid, 256, 0, ctx->stream>>>(w->view(), r0, nrows, dst);
    CKL();
    return LLMQ_OK;
  }
  const int grid = (nrows + 15) / 16;
  const RowMat rm = w->rowmat();
#define DQ(T) \
  case T:     \
    gguf_dequant_rows_kernel<T><<<grid, 256, 0, ctx->stream>>>(rm, r0, nrows, dst); \
    break;
  switch (w->rtype) {
    DQ(RT_F32) DQ(RT_F16) DQ(RT_BF16) DQ(RT_Q4_0) DQ(RT_Q4_1) DQ(RT_Q8_0) DQ(RT_Q4_K) DQ(RT_Q5_K) DQ(RT_Q6_K)
    default:
      return fail(ctx, LLMQ_ERR_UNSUPPORTED, "GGUF type");
  }
#undef DQ
  CKL();
  return LLMQ_OK;
}

// matmul_rows for T > 1 (kernels.mojo:325-358) of the OUT_MAJOR formats
// (GGUF rows, affine W4A32 / W8A32): rows of 32 outputs dequantized to
// float32 and run through the mm_tile chain; the OUT % 32 leftover rows
// through rows_dot (:361-397).
llmq_status rows_linear(llmq_ctx *ctx, const llmq_weight *w, const float *x, const float *bias, float *out,
                             int T, int IN, int OUT, int epi) {
  const int full = OUT / 32 * 32;
  llmq_status st = ensure_scratch(ctx, (size_t)OUT * IN * 4);
  if (st != LLMQ_OK) return st;
  float *wd = (float *)ctx->scratch;
  if ((st = dequant_rows(ctx, w, 0, OUT, wd)) != LLMQ_OK) return st;
  if (full > 0) {
    const dim3 grid((full + DM_N - 1) / DM_N, (T + DM_T - 1) / DM_T);
    dense_mm_kernel<0, true><<<grid, 256, 0, ctx->stream>>>(wd, x, bias, out, T, IN, OUT, full, epi);
    CKL();
  }
  if (OUT > full) {
    const int pairs = T * (OUT - full);
    rows_dot_kernel<<<(pairs * 16 + 255) / 256, 256, 0, ctx->stream>>>(wd + (size_t)full * IN, x, bias, out, T, IN,
                                                                       OUT, full, epi);
    CKL();
  }
  return LLMQ_OK;
}

// matmul_rows_a16 for T > 1 on the transposed GEMM (tct_gemm_kernel): the
// weight rows as the MMA's M, both activation planes of TT tokens as its N
// (TT 32 for matrices of at most 1024 outputs, so that more CTAs take part,
// else 64); the OUT % 32 leftover rows on rows_a16_kernel.
llmq_status tct_linear(llmq_ctx *ctx, const llmq_weight *w, const float *x, const float *bias, float *out, int T,
                       int IN, int OUT, int epi) {
  const int K = IN, nkb = K / TC_KB, seg = std::min(w->group, 256), nseg = K / seg;
  // int4 rows with 32-column groups (one K step per segment) take the
  // two-producer kernel on tiles of 32 tokens
  const bool tcp = w->bits == 4 && w->group == 32;
  const int TT = tcp || OUT <= 1024 ? 32 : 64;
  const int ttiles = (T + TT - 1) / TT, t_pad = ttiles * TT;
  const int full = OUT / 32 * 32, ntiles = (full + TC_M - 1) / TC_M;
  const bool zc = w->bits == 8;
  const size_t b_bytes = align256((size_t)ttiles * nkb * 2 * TT * TC_KB), sx_bytes = align256((size_t)t_pad * 4);
  const size_t xs_bytes = zc ? align256((size_t)t_pad * nseg * 4) : 0;
  const size_t xq_bytes = (OUT % 32) ? align256((size_t)T * IN * 2) : 0;
  llmq_status st = ensure_scratch(ctx, b_bytes + sx_bytes + xs_bytes + xq_bytes);
  if (st != LLMQ_OK) return st;
  uint8_t *b = (uint8_t *)ctx->scratch;
  float *sx = (float *)(b + b_bytes);
  int *xsum = zc ? (int *)((char *)sx + sx_bytes) : nullptr;
  int16_t *xq = xq_bytes ? (int16_t *)((char *)sx + sx_bytes + xs_bytes) : nullptr;
  if (!w->tc_w) {
    const int wt = (w->rows + TC_M - 1) / TC_M;
    CK(cudaMalloc(&w->tc_w, (size_t)wt * nkb * TCT_A_BYTES));
    CK(cudaMalloc(&w->tc_wsum, (size_t)w->rows * nseg * 4));
    tc_prep_b_kernel<<<dim3(wt, nkb), 256, 0, ctx->stream>>>(w->view(), w->tc_w, TC_M);
    CKL();
    tct_wsum_kernel<<<(w->rows * nseg + 255) / 256, 256, 0, ctx->stream>>>(w->view(), seg, nseg, w->tc_wsum);
    CKL();
  }
  if (TT == 32)
    tct_split_rows_kernel<32><<<(t_pad + 7) / 8, 256, 0, ctx->stream>>>(x, T, t_pad, K, nseg, seg, b, sx, xsum, xq);
  else
    tct_split_rows_kernel<64><<<(t_pad + 7) / 8, 256, 0, ctx->stream>>>(x, T, t_pad, K, nseg, seg, b, sx, xsum, xq);
  CKL();
  if (ntiles > 0) {
    TcArgsT p{};
    p.a = w->tc_w;
    p.b = b;
    p.sx = sx;
    p.xsum = xsum;
    p.wsum = w->tc_wsum;
    p.w = w->view();
    p.bias = bias;
    p.out = out;
    p.err = ctx->tc_err;
    p.T = T;
    p.OUT = OUT;
    p.n_full = full;
    p.K = K;
    p.nkb = nkb;
    p.nseg = nseg;
    p.seg_ks = seg / 32;
    p.seg = seg;
    p.epi = epi;
    // one CTA per SM: the weight tiles times as many token-tile columns as
    // fit, each CTA looping over its column's token tiles
    const dim3 grid(ntiles, std::min(ttiles, std::max(1, ctx->num_sms / ntiles)));
    if (tcp) {
      tcp_gemm_kernel<<<grid, TCL_THREADS, sizeof(TcpSmem) + 1024, ctx->stream>>>(p);
    } else if (TT == 32) {
      const size_t sm = sizeof(TcSmemT<32>) + 1024;
      if (zc)
        tct_gemm_kernel<true, 32><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
      else
        tct_gemm_kernel<false, 32><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
    } else {
      const size_t sm = sizeof(TcSmemT<64>) + 1024;
      if (zc)
        tct_gemm_kernel<true, 64><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
      else
        tct_gemm_kernel<false, 64><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
    }
    CKL();
    ctx->tc_used = true;
  }
  if (OUT % 32) {
    int n = T * (OUT - full);
    rows_a16_kernel<<<(n + 127) / 128, 128, 0, ctx->stream>>>(w->view(), xq, sx, bias, out, T, OUT, full, epi);
    CKL();
  }
  return LLMQ_OK;
}

// matmul_rows_a16 for T > 1 (kernels.mojo:461-507) with the tile_i16 rows
// (the first OUT / 32 * 32 outputs) on the split-int8 tcgen05 GEMM and the
// leftover rows (rows_i16) on rows_a16_kernel.
llmq_status tc_linear(llmq_ctx *ctx, const llmq_weight *w, const float *x, const float *bias, float *out, int T,
                      int IN, int OUT, int epi) {
  const int K = IN, nkb = K / TC_KB, seg = std::min(w->group, 256), nseg = K / seg;
  if (w->bits == 4 || nseg <= TC_MAX_GROUPS) return tct_linear(ctx, w, x, bias, out, T, IN, OUT, epi);
  const int mtiles = (T + TC_M - 1) / TC_M, m_pad = mtiles * TC_M;
  // 32-wide output tiles for narrow matrices (more CTAs), 64 otherwise; the
  // weight's prepared tiles follow the width chosen on its first use.
  const int tn = w->tc_b ? w->tc_tn : (OUT <= 1024 ? 32 : 64);
  const int full = OUT / 32 * 32, ntiles = (full + tn - 1) / tn;
  const bool zc = w->bits == 8;
  const size_t a_bytes = align256((size_t)mtiles * nkb * TC_A_BYTES), sx_bytes = align256((size_t)m_pad * 4);
  const size_t xs_bytes = zc ? align256((size_t)m_pad * nseg * 4) : 0;
  const size_t xq_bytes = (OUT % 32) ? align256((size_t)T * IN * 2) : 0;
  llmq_status st = ensure_scratch(ctx, a_bytes + sx_bytes + xs_bytes + xq_bytes);
  if (st != LLMQ_OK) return st;
  uint8_t *a = (uint8_t *)ctx->scratch;
  float *sx = (float *)(a + a_bytes);
  int *xsum = zc ? (int *)((char *)sx + sx_bytes) : nullptr;
  int16_t *xq = xq_bytes ? (int16_t *)((char *)sx + sx_bytes + xs_bytes) : nullptr;
  if (!w->tc_b) {
    const int wt = (w->rows + tn - 1) / tn;
    CK(cudaMalloc(&w->tc_b, (size_t)wt * nkb * tn * TC_KB));
    w->tc_tn = tn;
    tc_prep_b_kernel<<<dim3(wt, nkb), 256, 0, ctx->stream>>>(w->view(), w->tc_b, tn);
    CKL();
  }
  tc_split_rows_kernel<<<m_pad, 256, 0, ctx->stream>>>(x, T, K, nseg, seg, a, sx, xsum, xq);
  CKL();
  if (ntiles > 0) {
    TcArgs p{};
    p.a = a;
    p.b = w->tc_b;
    p.sx = sx;
    p.xsum = xsum;
    p.w = w->view();
    p.bias = bias;
    p.out = out;
    p.err = ctx->tc_err;
    p.T = T;
    p.OUT = OUT;
    p.n_full = full;
    p.K = K;
    p.nkb = nkb;
    p.nseg = nseg;
    p.seg_ks = seg / 32;
    p.seg = seg;
    p.epi = epi;
    dim3 grid(ntiles, mtiles);
    const size_t sm = sizeof(TcSmem) + 1024;
    if (zc && tn == 64)
      tc_gemm_a16_kernel<true, 64><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
    else if (zc)
      tc_gemm_a16_kernel<true, 32><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
    else if (tn == 64)
      tc_gemm_a16_kernel<false, 64><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
    else
      tc_gemm_a16_kernel<false, 32><<<grid, TC_THREADS, sm, ctx->stream>>>(p);
    CKL();
    ctx->tc_used = true;
  }
  if (OUT % 32) {
    int n = T * (OUT - full);
    rows_a16_kernel<<<(n + 127) / 128, 128, 0, ctx->stream>>>(w->view(), xq, sx, bias, out, T, OUT, full, epi);
    CKL();
  }
  return LLMQ_OK;
}

}  // namespace

extern "C" {

llmq_status llmq_linear(llmq_ctx *ctx, const llmq_weight *w, const float *x, const float *bias, float *out, int T,
                        int IN, int OUT, int flags) {
  if (!ctx || !w || !x || !out || T <= 0) return fail(ctx, LLMQ_ERR_INVALID, "null argument or T <= 0");
  if ((flags & LLMQ_BIAS) && !bias) return fail(ctx, LLMQ_ERR_INVALID, "LLMQ_BIAS without a bias");
  CK(cudaSetDevice(ctx->device));
  int epi = (flags & LLMQ_BIAS ? EPI_BIAS : 0) | (flags & LLMQ_GELU ? EPI_GELU : 0) |
            (flags & LLMQ_RESID ? EPI_RESID : 0);
  if (w->kind == WK_DENSE) {
    // DenseMatrix layer matrices are [IN, OUT] (tensor.mojo:150-227).
    if (IN != w->rows || OUT != w->cols) return fail(ctx, LLMQ_ERR_INVALID, "IN/OUT do not match the [IN, OUT] matrix");
    if (T > 1) {
      // matmul / mm_tile (kernels.mojo:51-129): one fma chain per output
      const dim3 grid((OUT + DM_N - 1) / DM_N, (T + DM_T - 1) / DM_T);
      if (w->rtype == RT_F32)
        dense_mm_kernel<0, false><<<grid, 256, 0, ctx->stream>>>(w->codes, x, bias, out, T, IN, OUT, OUT, epi);
      else if (w->rtype == RT_BF16)
        dense_mm_kernel<1, false><<<grid, 256, 0, ctx->stream>>>(w->codes, x, bias, out, T, IN, OUT, OUT, epi);
      else
        return fail(ctx, LLMQ_ERR_UNSUPPORTED, "several-token dense matmuls take float32 or bfloat16");
      CKL();
      return LLMQ_OK;
    }
    const int np = ctx->dense_parts;
    llmq_status st = ensure_scratch(ctx, (size_t)np * OUT * 4);
    if (st != LLMQ_OK) return st;
    float *scratch = (float *)ctx->scratch;
    const int es = w->rtype == RT_F32 ? 4 : 2;
    if ((OUT * es) % 16 == 0 && ds_smem(IN, np, es) <= DS_SMEM) {
      const dim3 sgrid((OUT + 31) / 32, np);
      const int sm = ds_smem(IN, np, es);
      if (w->rtype == RT_F32)
        dense_strip_kernel<0><<<sgrid, DS_THREADS, sm, ctx->stream>>>(w->codes, x, IN, OUT, np, scratch);
      else if (w->rtype == RT_F16)
        dense_strip_kernel<1><<<sgrid, DS_THREADS, sm, ctx->stream>>>(w->codes, x, IN, OUT, np, scratch);
      else
        dense_strip_kernel<2><<<sgrid, DS_THREADS, sm, ctx->stream>>>(w->codes, x, IN, OUT, np, scratch);
      CKL();
      dense_gemv_combine_kernel<<<(OUT + 255) / 256, 256, 0, ctx->stream>>>(scratch, bias, out, OUT, np, epi);
      CKL();
      return LLMQ_OK;
    }
    dim3 grid((OUT + 255) / 256, np);
    if (w->rtype == RT_F32) dense_gemv_parts_kernel<0><<<grid, 256, 0, ctx->stream>>>(w->codes, x, IN, OUT, np, scratch);
    else if (w->rtype == RT_F16) dense_gemv_parts_kernel<1><<<grid, 256, 0, ctx->stream>>>(w->codes, x, IN, OUT, np, scratch);
    else dense_gemv_parts_kernel<2><<<grid, 256, 0, ctx->stream>>>(w->codes, x, IN, OUT, np, scratch);
    CKL();
    dense_gemv_combine_kernel<<<(OUT + 255) / 256, 256, 0, ctx->stream>>>(scratch, bias, out, OUT, np, epi);
    CKL();
    return LLMQ_OK;
  }
  if (IN != w->cols || OUT != w->rows) return fail(ctx, LLMQ_ERR_INVALID, "IN/OUT do not match the matrix");
  if (w->kind == WK_GGUF || (w->kind == WK_AFFINE && !w->a16)) {
    if (T > 1) return rows_linear(ctx, w, x, bias, out, T, IN, OUT, epi);
    // matmul_rows (kernels.mojo:285-349) for one token: dot_row per output.
    if (w->kind == WK_GGUF) {
      RowGemvArgs a{w->rowmat(), x, bias, out, epi, nullptr, 0};
      CK(row_gemv(ctx, a));
    } else {
      AffFloatArgs a{w->view(), x, bias, out, epi};
      const bool tall = w->rows >= 8192;
      const int rpc = tall ? 16 : 4;
      const size_t sm = afg_smem(w->cols, w->cols / w->group, rpc);
      if (w->group <= 128 && sm <= (size_t)kMaxSmem) {
        // grouped rows: the group sums in parallel, the folds per row
        const int grid = std::min((w->rows + rpc - 1) / rpc, ctx->num_sms * 8);
        const void *k = w->bits == 4 ? (tall ? (const void *)affine_float_group_kernel<4, 16>
                                             : (const void *)affine_float_group_kernel<4, 4>)
                                     : (tall ? (const void *)affine_float_group_kernel<8, 16>
                                             : (const void *)affine_float_group_kernel<8, 4>);
        if (sm > 48 * 1024) CK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm));
        if (w->bits == 4 && tall)
          affine_float_group_kernel<4, 16><<<grid, 256, sm, ctx->stream>>>(a);
        else if (w->bits == 4)
          affine_float_group_kernel<4, 4><<<grid, 256, sm, ctx->stream>>>(a);
        else if (tall)
          affine_float_group_kernel<8, 16><<<grid, 256, sm, ctx->stream>>>(a);
        else
          affine_float_group_kernel<8, 4><<<grid, 256, sm, ctx->stream>>>(a);
      } else {
        const int grid = std::min((w->rows + 15) / 16, ctx->num_sms * 4);
        if (w->bits == 4)
          affine_float_gemv_kernel<4><<<grid, 256, w->cols * 4, ctx->stream>>>(a);
        else
          affine_float_gemv_kernel<8><<<grid, 256, w->cols * 4, ctx->stream>>>(a);
      }
      CKL();
    }
    return LLMQ_OK;
  }
  if (T == 1) {
    GemvArgs a{};
    a.w = w->view();
    a.x = x;
    a.bias = bias;
    a.out = out;
    a.epi = epi;
    CK(launch_gemv(ctx, a, PRO_QUANT, false, ctx->stream));
    return LLMQ_OK;
  }
  if (tc_eligible(ctx, w, T)) return tc_linear(ctx, w, x, bias, out, T, IN, OUT, epi);
  size_t need = (size_t)T * IN * 2 + (size_t)T * 4 + 256;
  llmq_status st = ensure_scratch(ctx, need);
  if (st != LLMQ_OK) return st;
  int16_t *xq = (int16_t *)ctx->scratch;
  float *sx = (float *)((char *)ctx->scratch + (((size_t)T * IN * 2 + 255) / 256) * 256);
  quantize_rows_kernel<<<T, 256, 0, ctx->stream>>>(x, IN, xq, sx);
  CKL();
  int full = OUT / 32;
  if (full > 0) {
    dim3 grid(full, (T + 31) / 32);
    tile_a16_kernel<<<grid, 256, 0, ctx->stream>>>(w->view(), xq, sx, bias, out, T, OUT, epi);
    CKL();
  }
  if (OUT % 32) {
    int n = T * (OUT - full * 32);
    rows_a16_kernel<<<(n + 127) / 128, 128, 0, ctx->stream>>>(w->view(), xq, sx, bias, out, T, OUT, full * 32, epi);
    CKL();
  }
  return LLMQ_OK;
}

llmq_status llmq_head(llmq_ctx *ctx, const llmq_weight *w, const float *h, float *logits, int T, int C, int V) {
  if (!ctx || !w || !h || !logits || T <= 0) return fail(ctx, LLMQ_ERR_INVALID, "null argument or T <= 0");
  if (w->rows != V || w->cols != C) return fail(ctx, LLMQ_ERR_INVALID, "the head must be [V, C]");
  if (w->kind == WK_DENSE && (C % 16 != 0 || C > 4096))
    return fail(ctx, LLMQ_ERR_INVALID, "a dense head needs C a multiple of 16, at most 4096");
  CK(cudaSetDevice(ctx->device));
  if (w->kind == WK_GGUF && (w->rtype == RT_Q8_0 || w->rtype == RT_Q6_K)) {
    // head_i16: the same arithmetic for one token and for several.
    const dim3 grid(std::min((V + 15) / 16, T > 1 ? ctx->num_sms : ctx->num_sms * 4), T);
    if (w->rtype == RT_Q8_0)
      gguf_head_i16_kernel<RT_Q8_0><<<grid, 256, 0, ctx->stream>>>(w->rowmat(), h, logits);
    else
      gguf_head_i16_kernel<RT_Q6_K><<<grid, 256, 0, ctx->stream>>>(w->rowmat(), h, logits);
    CKL();
    return LLMQ_OK;
  }
  if (w->kind == WK_AFFINE && w->a16) return llmq_linear(ctx, w, h, nullptr, logits, T, C, V, 0);
  // head (kernels.mojo:677-689): an OUT_MAJOR head (GGUF rows without the
  // integer kernel, affine W4A32 / W8A32) runs matmul_rows for all T tokens,
  // so T > 1 takes the dequantized tiles, not T one-token dots
  if (T > 1 && (w->kind == WK_GGUF || w->kind == WK_AFFINE)) return llmq_linear(ctx, w, h, nullptr, logits, T, C, V, 0);
  if (w->kind == WK_DENSE && T > 1 && (w->rtype == RT_F32 || w->rtype == RT_BF16)) {
    // lm_head_rows (kernels.mojo:230-271): the 16 lane chains of lm_head, per token
    const dim3 grid((V + 15) / 16, (T + 15) / 16);
    if (w->rtype == RT_F32)
      dense_head_rows_kernel<0><<<grid, 256, 0, ctx->stream>>>(w->codes, h, logits, T, V, C);
    else
      dense_head_rows_kernel<1><<<grid, 256, 0, ctx->stream>>>(w->codes, h, logits, T, V, C);
    CKL();
    return LLMQ_OK;
  }
  // lm_head / lm_head_rows (dense, kernels.mojo:213-271) and matmul_rows
  // (OUT_MAJOR formats) for one token: a 16-lane dot per vocabulary row;
  // lm_head_rows gives every token the same arithmetic as lm_head.
  for (int t = 0; t < T; t++) {
    if (w->kind == WK_DENSE) {
      RowGemvArgs a{w->rowmat(), h + (size_t)t * C, nullptr, logits + (size_t)t * V, 0, nullptr, 0};
      CK(row_gemv(ctx, a));
    } else {
      llmq_status st = llmq_linear(ctx, w, h + (size_t)t * C, nullptr, logits + (size_t)t * V, 1, C, V, 0);
      if (st != LLMQ_OK) return st;
    }
  }
  return LLMQ_OK;
}

llmq_status llmq_head_argmax(llmq_ctx *ctx, const llmq_weight *w, const float *h, float *logits, int *argmax) {
  if (!ctx || !w || !h || !argmax) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  if (!w->a16) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "llmq_head_argmax takes A16 formats");
  CK(cudaSetDevice(ctx->device));
  int grid = gemv_grid(ctx, w->view());
  llmq_status st = ensure_scratch(ctx, (size_t)grid * 8 + 256);
  if (st != LLMQ_OK) return st;
  GemvArgs a{};
  a.w = w->view();
  a.x = h;
  a.out = logits;
  a.part_val = (float *)ctx->scratch;
  a.part_idx = (int *)((char *)ctx->scratch + (size_t)grid * 4);
  a.state = ctx->state;
  a.ids = argmax;  // written at state->step, kept at 0 here
  CK(cudaMemsetAsync(ctx->state, 0, sizeof(DecodeState), ctx->stream));
  CK(launch_gemv(ctx, a, PRO_QUANT, true, ctx->stream));
  return LLMQ_OK;
}

// ---------------------------------------------------------------------------
// llmq_head_argmax_noalloc: the head GEMV + greedy argmax of llmq_head_argmax
// with its scratch in a fixed device array instead of the context's
// cudaMalloc'd buffer. It is for callers that cannot allocate device memory
// while they run: a serving process whose memory pool has reserved the
// device's HBM up front, and hosts that must not meet the device-wide
// synchronisation of cudaMalloc / cudaFree between two launches. The
// existing entry point grows ctx->scratch on demand and is unchanged.
//
// The array holds one DecodeState (the CTA ticket and the id slot, which must
// start at zero and are cleared by a cudaMemsetAsync before every launch) and
// one (value, index) partial per CTA of the gemv grid, at most
// LLMQ_NOALLOC_MAX_PARTS of them (16 KiB in all). One array exists per device:
// calls on the same device that overlap in time (two streams, two contexts,
// two host threads) race on it and must be ordered by the caller.
// ---------------------------------------------------------------------------
constexpr int kNoallocMaxParts = 1920;
constexpr size_t kNoallocStateBytes = 256;
constexpr size_t kNoallocBytes = kNoallocStateBytes + (size_t)kNoallocMaxParts * 8;  // 15,616 B
static_assert(sizeof(DecodeState) <= kNoallocStateBytes, "DecodeState fits its slot");
static_assert(LLMQ_NOALLOC_MAX_PARTS == kNoallocMaxParts, "header limit matches the array");

static __device__ __align__(256) unsigned char g_head_argmax_scratch[kNoallocBytes];

namespace {
// The device address of g_head_argmax_scratch on ctx's device, looked up once
// per device (again after the device's last context was destroyed) with that
// device current. The lookup may load the module on the device, so the first
// call should come before any stream capture.
llmq_status noalloc_scratch(llmq_ctx *ctx, unsigned char **out) {
  if (ctx->device < 0 || ctx->device >= kNoallocMaxDevices)
    return fail(ctx, LLMQ_ERR_INVALID, "llmq_head_argmax_noalloc: device index beyond 63");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_ptr[ctx->device]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_head_argmax_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(ctx, LLMQ_ERR_CUDA,
                  std::string("llmq_head_argmax_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
    g_noalloc_ptr[ctx->device] = ptr;
  }
  *out = (unsigned char *)g_noalloc_ptr[ctx->device];
  return LLMQ_OK;
}
}  // namespace

llmq_status llmq_head_argmax_noalloc(llmq_ctx *ctx, const llmq_weight *w, const float *h, float *logits,
                                     int *argmax) {
  if (!ctx || !w || !h || !argmax) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  if (w->kind != WK_AFFINE || !w->a16)
    return fail(ctx, LLMQ_ERR_UNSUPPORTED, "llmq_head_argmax_noalloc takes A16 formats");
  CK(cudaSetDevice(ctx->device));
  int grid = gemv_grid(ctx, w->view());
  if (grid > kNoallocMaxParts)
    return fail(ctx, LLMQ_ERR_INVALID,
                "llmq_head_argmax_noalloc: the gemv grid needs " + std::to_string(grid) +
                    " partials, beyond the fixed scratch's " + std::to_string(kNoallocMaxParts));
  unsigned char *scratch = nullptr;
  llmq_status st = noalloc_scratch(ctx, &scratch);
  if (st != LLMQ_OK) return st;
  GemvArgs a{};
  a.w = w->view();
  a.x = h;
  a.out = logits;
  a.state = (DecodeState *)scratch;
  a.part_val = (float *)(scratch + kNoallocStateBytes);
  a.part_idx = (int *)(scratch + kNoallocStateBytes + (size_t)kNoallocMaxParts * 4);
  a.ids = argmax;  // written at state->step, which the memset sets to 0
  CK(cudaMemsetAsync(scratch, 0, sizeof(DecodeState), ctx->stream));
  CK(launch_gemv(ctx, a, PRO_QUANT, true, ctx->stream));
  return LLMQ_OK;
}

llmq_status llmq_layernorm(llmq_ctx *ctx, float *out, const float *x, const float *w, const float *b, int T, int C) {
  if (!ctx || !out || !x || !w || !b || T <= 0 || C <= 0 || C % 16) return fail(ctx, LLMQ_ERR_INVALID, "bad argument");
  CK(cudaSetDevice(ctx->device));
  launch_layernorm(out, x, w, b, T, C, ctx->stream);
  CKL();
  return LLMQ_OK;
}

llmq_status llmq_quantize_rows(llmq_ctx *ctx, const float *x, int T, int IN, int16_t *xq, float *sx) {
  if (!ctx || !x || !xq || !sx || T <= 0 || IN <= 0) return fail(ctx, LLMQ_ERR_INVALID, "bad argument");
  CK(cudaSetDevice(ctx->device));
  quantize_rows_kernel<<<T, 256, 0, ctx->stream>>>(x, IN, xq, sx);
  CKL();
  return LLMQ_OK;
}

llmq_status llmq_debug_lane_sums(llmq_ctx *ctx, const llmq_weight *w, const float *x, int32_t *lanes) {
  if (!ctx || !w || !x || !lanes) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  CK(cudaSetDevice(ctx->device));
  GemvArgs a{};
  a.w = w->view();
  a.x = x;
  int grid = gemv_grid(ctx, a.w);
  int fmt = fmt_of(a.w);
  if (fmt == FMT_BLK4) {
    lane_sums_kernel<FMT_BLK4><<<grid, kThreads, smem_bytes_r<FMT_BLK4>(a.w, kR), ctx->stream>>>(a, lanes);
  } else if (fmt == FMT_GEN4) {
    lane_sums_kernel<FMT_GEN4><<<grid, kThreads, smem_bytes_r<FMT_GEN4>(a.w, kR), ctx->stream>>>(a, lanes);
  } else {
    lane_sums_kernel<FMT_GEN8><<<grid, kThreads, smem_bytes_r<FMT_GEN8>(a.w, kR), ctx->stream>>>(a, lanes);
  }
  CKL();
  return LLMQ_OK;
}

// ---- KV cache --------------------------------------------------------------

llmq_status llmq_kv_create(llmq_ctx *ctx, int kind, int n_layer, int max_t, int n_head, int head_dim,
                           llmq_kv **out) {
  if (!ctx || !out || n_layer <= 0 || max_t <= 0 || n_head <= 0 || head_dim <= 0 || head_dim % 16 || head_dim > 128)
    return fail(ctx, LLMQ_ERR_INVALID, "bad cache shape");
  if (kind != LLMQ_KV_QUANT8 && kind != LLMQ_KV_INTATTN && kind != LLMQ_KV_F32 && kind != LLMQ_KV_BF16)
    return fail(ctx, LLMQ_ERR_UNSUPPORTED, "unknown cache kind");
  // IntAttnKV keeps keys in blocks of 16 positions and pairs of dimensions
  // (int_attention.mojo:283-284 aborts on other shapes).
  if (kind == LLMQ_KV_INTATTN && (max_t % IA_PB || head_dim % 32))
    return fail(ctx, LLMQ_ERR_INVALID, "IntAttnKV needs max_t % 16 == 0 and head_dim % 32 == 0");
  *out = nullptr;
  CK(cudaSetDevice(ctx->device));
  llmq_kv *c = new llmq_kv();
  c->ctx = ctx;
  c->kind = kind;
  c->n_layer = n_layer;
  c->max_t = max_t;
  c->n_head = n_head;
  c->head_dim = head_dim;
  size_t n = (size_t)n_layer * max_t * n_head * head_dim, ns = (size_t)n_layer * max_t * n_head;
  const size_t el = kind == LLMQ_KV_F32 ? 4 : kind == LLMQ_KV_BF16 ? 2 : 1;  // bytes per key or value element
  const bool dense = el > 1;
  void *k = nullptr, *v = nullptr, *ks = nullptr, *vs = nullptr;
  cudaError_t e = cudaMalloc(&k, n * el);
  if (e == cudaSuccess) e = cudaMalloc(&v, n * el);
  if (e == cudaSuccess && !dense) e = cudaMalloc(&ks, ns * 4);
  if (e == cudaSuccess && !dense) e = cudaMalloc(&vs, ns * 4);
  if (e == cudaSuccess) e = cudaMemset(k, 0, n * el);
  if (e == cudaSuccess) e = cudaMemset(v, 0, n * el);
  if (e == cudaSuccess && !dense) e = cudaMemset(ks, 0, ns * 4);
  if (e == cudaSuccess && !dense) e = cudaMemset(vs, 0, ns * 4);
  if (kind == LLMQ_KV_QUANT8 || dense)
    c->v8 = KV8View{(int8_t *)k, (int8_t *)v, (float *)ks, (float *)vs, n_layer, max_t, n_head, head_dim};
  else
    c->ia = IAView{(int8_t *)k, (int8_t *)v, (int32_t *)ks, (int32_t *)vs, n_layer, max_t, n_head, head_dim};
  if (e != cudaSuccess) {
    llmq_kv_free(c);
    return fail(ctx, LLMQ_ERR_CUDA, std::string("kv alloc: ") + cudaGetErrorString(e));
  }
  *out = c;
  return LLMQ_OK;
}

llmq_status llmq_kv_free(llmq_kv *c) {
  if (!c) return LLMQ_ERR_INVALID;
  void *bufs[8] = {c->v8.k, c->v8.v, c->v8.ks, c->v8.vs, c->ia.k, c->ia.v, c->ia.kq, c->ia.vq};
  for (void *b : bufs)
    if (b) cudaFree(b);
  delete c;
  return LLMQ_OK;
}

namespace {
// exp_multiplier (intmath.mojo:48-50) of the score scale 2^-16.
long long ia_mult() { return (long long)(1.0 / (double)(1 << IA_SF) * 1.4426950408889634 * (double)(1LL << 40) + 0.5); }

size_t ia_attend_smem(const llmq_kv *kv) { return (size_t)kv->max_t * 4 + (size_t)(kv->max_t + 2) * 2; }
}  // namespace

llmq_status llmq_kv_store(llmq_ctx *ctx, llmq_kv *kv, int layer, int pos0, int T, const float *qkv) {
  if (!ctx || !kv || !qkv || T <= 0 || layer < 0 || layer >= kv->n_layer || pos0 < 0 || pos0 + T > kv->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad layer or positions");
  CK(cudaSetDevice(ctx->device));
  if (kv->kind == LLMQ_KV_QUANT8)
    kv8_store_kernel<<<(kv->n_head * T * 2 + 7) / 8, 256, 0, ctx->stream>>>(kv->v8, qkv, layer, pos0, nullptr, T, 1);
  else if (kv->kind == LLMQ_KV_F32)
    dkv_store_kernel<1><<<T, 256, 0, ctx->stream>>>(kv->v8, qkv, layer, pos0);
  else if (kv->kind == LLMQ_KV_BF16)
    dkv_store_kernel<2><<<T, 256, 0, ctx->stream>>>(kv->v8, qkv, layer, pos0);
  else
    ia_store_kernel<<<dim3(kv->n_head, T, 2), 128, 0, ctx->stream>>>(kv->ia, qkv, layer, pos0);
  CKL();
  return LLMQ_OK;
}

// kv8_attend_kernel with the key codes staged in shared memory where they
// fit beside the values (the launch's queries see at most cap positions).
llmq_status kv8_attend(llmq_ctx *ctx, const KV8View &v, float *out, const float *qkv, int layer, int pos0,
                       const int *pos_dev, int store, int cap, dim3 grid, cudaStream_t s) {
  const int HS = v.head_dim;
  if (HS == 64 && kv8_attend_smem(cap, HS, true) <= (size_t)kMaxSmem)
    kv8_attend_kernel<true, 64><<<grid, 128, kv8_attend_smem(cap, HS, true), s>>>(v, out, qkv, layer, pos0, pos_dev,
                                                                                  store, cap);
  else if (kv8_attend_smem(cap, HS, true) <= (size_t)kMaxSmem)
    kv8_attend_kernel<true, 0><<<grid, 128, kv8_attend_smem(cap, HS, true), s>>>(v, out, qkv, layer, pos0, pos_dev,
                                                                                 store, cap);
  else if (kv8_attend_smem(cap, HS, false) <= (size_t)kMaxSmem)
    kv8_attend_kernel<false, 0><<<grid, 128, kv8_attend_smem(cap, HS, false), s>>>(v, out, qkv, layer, pos0,
                                                                                   pos_dev, store, cap);
  else
    return fail(ctx, LLMQ_ERR_UNSUPPORTED, "context too long for the int8 cache kernel");
  CKL();
  return LLMQ_OK;
}

llmq_status llmq_kv_attend(llmq_ctx *ctx, llmq_kv *kv, float *out, const float *qkv, int layer, int T, int pos0) {
  if (!ctx || !kv || !qkv || !out || T <= 0 || layer < 0 || layer >= kv->n_layer || pos0 < 0 ||
      pos0 + T > kv->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad layer or positions");
  CK(cudaSetDevice(ctx->device));
  dim3 grid(kv->n_head, T);
  if (kv->kind == LLMQ_KV_F32 || kv->kind == LLMQ_KV_BF16) {
    // attend_float_one through DenseKV, every token count
    const size_t sm = kv8_prefill_smem(pos0 + T, kv->head_dim);
    if (sm > (size_t)kMaxPrefillSmem) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "context too long for the dense cache kernel");
    const dim3 g(kv->n_head, (T + KV_QB - 1) / KV_QB);
    if (kv->kind == LLMQ_KV_F32)
      kv_prefill_kernel<1><<<g, 256, sm, ctx->stream>>>(kv->v8, out, qkv, layer, pos0, T);
    else
      kv_prefill_kernel<2><<<g, 256, sm, ctx->stream>>>(kv->v8, out, qkv, layer, pos0, T);
  } else if (kv->kind == LLMQ_KV_QUANT8 && T > 1 && kv8_prefill_smem(pos0 + T, kv->head_dim) <= (size_t)kMaxPrefillSmem) {
    const size_t sm = kv8_prefill_smem(pos0 + T, kv->head_dim);
    kv_prefill_kernel<0><<<dim3(kv->n_head, (T + KV_QB - 1) / KV_QB), 256, sm, ctx->stream>>>(kv->v8, out, qkv, layer,
                                                                                            pos0, T);
  } else if (kv->kind == LLMQ_KV_QUANT8) {
    // the last query sees pos0 + T positions
    const llmq_status st = kv8_attend(ctx, kv->v8, out, qkv, layer, pos0, nullptr, 0, pos0 + T, grid, ctx->stream);
    if (st) return st;
  } else {
    ia_attend_kernel<<<grid, 256, ia_attend_smem(kv), ctx->stream>>>(kv->ia, out, qkv, layer, pos0, nullptr, 0,
                                                                     ia_mult());
  }
  CKL();
  return LLMQ_OK;
}

llmq_status llmq_kv_read(llmq_ctx *ctx, const llmq_kv *kv, void *k, void *v, void *ks, void *vs) {
  if (!ctx || !kv) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->stream));
  size_t n = (size_t)kv->n_layer * kv->max_t * kv->n_head * kv->head_dim;
  size_t ns = (size_t)kv->n_layer * kv->max_t * kv->n_head;
  const bool q8 = kv->kind != LLMQ_KV_INTATTN;  // the int8 and dense caches live in v8
  const size_t el = kv->kind == LLMQ_KV_F32 ? 4 : kv->kind == LLMQ_KV_BF16 ? 2 : 1;
  const void *src[4] = {q8 ? (const void *)kv->v8.k : kv->ia.k, q8 ? (const void *)kv->v8.v : kv->ia.v,
                        q8 ? (const void *)kv->v8.ks : kv->ia.kq, q8 ? (const void *)kv->v8.vs : kv->ia.vq};
  void *dst[4] = {k, v, ks, vs};
  size_t bytes[4] = {n * el, n * el, ns * 4, ns * 4};
  for (int i = 0; i < 4; i++)
    if (dst[i] && src[i]) CK(cudaMemcpy(dst[i], src[i], bytes[i], cudaMemcpyDeviceToHost));
  return LLMQ_OK;
}

}  // extern "C"

// ---- model -----------------------------------------------------------------

namespace {

struct CopyDesc {
  const uint8_t *src;
  long long dst;
  long long bytes;
};

// Byte gather used once per model to build the per-CTA weight streams.
__global__ void gather_kernel(const CopyDesc *d, uint8_t *dst) {
  const CopyDesc c = d[blockIdx.x];
  for (long long i = threadIdx.x; i < c.bytes; i += blockDim.x) dst[c.dst + i] = c.src[i];
}

inline long long align16(long long x) { return (x + 15) & ~15LL; }

// Builds the persistent kernel's per-CTA weight streams (mega.cuh): CTA c
// gets rows [rows*c/G, rows*(c+1)/G) of every layer matrix, in use order,
// then its share of the head in 32-row tiles. Returns LLMQ_OK without
// enabling the kernel when the formats are not the ones it runs.
llmq_status mega_setup(llmq_model *m) {
  llmq_ctx *ctx = m->ctx;
  m->mega_ok = false;
  if (m->n_head != 12 || m->C != 768) return LLMQ_OK;
  if (!(m->kv->kind == LLMQ_KV_QUANT8 && m->kv->v8.head_dim == 64) &&
      !(m->kv->kind == LLMQ_KV_INTATTN && m->kv->ia.head_dim == 64 && m->kv->max_t <= 1024))
    return LLMQ_OK;
  for (const llmq_weight *w : m->mats)
    if (!w->blocked) return LLMQ_OK;
  const llmq_weight *hd = m->head;
  if (hd->bits != 8 || hd->group != hd->cols || hd->blocked || !hd->a16) return LLMQ_OK;
  int occ = 0;
  CK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, mega_decode_kernel, MK_THREADS, sizeof(MkSmem)));
  if (occ < 1) return LLMQ_OK;
  const int G = ctx->num_sms;
  int max_tiles = 0;
  for (int c = 0; c < G; c++) {
    int h0 = (int)((long long)m->V * c / G), h1 = (int)((long long)m->V * (c + 1) / G);
    int t = (h1 - h0 + MK_HEAD_TILE - 1) / MK_HEAD_TILE;
    if (t > max_tiles) max_tiles = t;
  }
  const int nch = 4 * m->n_layer + max_tiles;
  if (nch > MK_MAX_CHUNKS) return LLMQ_OK;
  std::vector<MkChunk> chunks((size_t)G * nch);
  std::vector<long long> base(G);
  std::vector<CopyDesc> copies;
  long long total = 0;
  for (int c = 0; c < G; c++) {
    base[c] = total;
    long long off = 0;
    int k = 0;
    auto add = [&](int kind, int layer, const llmq_weight *w, int r0, int r1) -> bool {
      int n = r1 - r0, gpr = w->cols / w->group;
      long long row_bytes = (long long)w->cols * w->bits / 8;
      long long codes = n * row_bytes, sc = (long long)n * gpr * 2, zpb = (long long)n * gpr;
      MkChunk ch{};
      ch.kind = kind;
      ch.layer = layer;
      ch.r0 = r0;
      ch.r1 = r1;
      ch.off = (int)off;
      ch.scale_off = (int)align16(codes);
      ch.zp_off = (int)(ch.scale_off + align16(sc));
      ch.bytes = (int)(ch.zp_off + align16(zpb));
      if (ch.bytes == 0) ch.bytes = 16;
      if (ch.bytes > MK_SLOT || (kind != PH_HEAD && n > 64)) return false;
      if (n > 0) {
        copies.push_back({w->codes + r0 * row_bytes, total + off, codes});
        copies.push_back({(const uint8_t *)w->scale + (long long)r0 * gpr * 2, total + off + ch.scale_off, sc});
        copies.push_back({w->zp + (long long)r0 * gpr, total + off + ch.zp_off, zpb});
      }
      chunks[(size_t)c * nch + k++] = ch;
      off += ch.bytes;
      return true;
    };
    // The QKV and PROJ rows go to the CTAs without an attention head: the
    // attention CTAs start their head as soon as its q, k, v arrive and
    // poll the heads' outputs without a PROJ share of their own.
    const int nh = m->n_head;
    for (int l = 0; l < m->n_layer; l++)
      for (int j = 0; j < 4; j++) {
        const llmq_weight *w = m->mats[4 * l + j];
        int r0, r1;
        if (j <= 1) {
          r0 = c < nh ? 0 : (int)((long long)w->rows * (c - nh) / (G - nh));
          r1 = c < nh ? 0 : (int)((long long)w->rows * (c + 1 - nh) / (G - nh));
        } else {
          r0 = (int)((long long)w->rows * c / G);
          r1 = (int)((long long)w->rows * (c + 1) / G);
        }
        if (!add(j, l, w, r0, r1)) return LLMQ_OK;
      }
    int h0 = (int)((long long)m->V * c / G), h1 = (int)((long long)m->V * (c + 1) / G);
    for (int t = 0; t < max_tiles; t++) {
      int r0 = h0 + t * MK_HEAD_TILE;
      if (r0 > h1) r0 = h1;
      int r1 = r0 + MK_HEAD_TILE < h1 ? r0 + MK_HEAD_TILE : h1;
      if (!add(PH_HEAD, -1, hd, r0, r1)) return LLMQ_OK;
    }
    total += align16(off);
  }
  CK(cudaMalloc(&m->mega_stream, total + 16));
  CK(cudaMalloc(&m->mega_base, sizeof(long long) * G));
  CK(cudaMalloc(&m->mega_chunks, sizeof(MkChunk) * chunks.size()));
  CK(cudaMemcpy(m->mega_base, base.data(), sizeof(long long) * G, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(m->mega_chunks, chunks.data(), sizeof(MkChunk) * chunks.size(), cudaMemcpyHostToDevice));
  CopyDesc *dd = nullptr;
  CK(cudaMalloc(&dd, sizeof(CopyDesc) * copies.size()));
  CK(cudaMemcpy(dd, copies.data(), sizeof(CopyDesc) * copies.size(), cudaMemcpyHostToDevice));
  gather_kernel<<<(unsigned)copies.size(), 256, 0, ctx->stream>>>(dd, m->mega_stream);
  CKL();
  CK(cudaStreamSynchronize(ctx->stream));
  cudaFree(dd);
  MkLL ll(m->C, m->n_layer, G);
  CK(cudaMalloc(&m->mega_ll, sizeof(unsigned long long) * ll.total()));
  CK(cudaMemset(m->mega_ll, 0, sizeof(unsigned long long) * ll.total()));
  CK(cudaMalloc(&m->mega_err, sizeof(int)));
  CK(cudaMemset(m->mega_err, 0, sizeof(int)));
  m->mega_grid = G;
  m->mega_nchunks = nch;
  m->mega_flag = 1;
  m->mega_ok = true;
  m->mode = LLMQ_MODE_PERSISTENT;
  return LLMQ_OK;
}

// Builds the cluster decode kernel's streams (cluster.cuh) when the model's
// formats are the ones it runs (those of the persistent kernel with the
// QuantKV[8] cache) and the device holds at least two 16-CTA clusters:
//   layer rank r (cluster 0): per layer, [q, k, v rows of head r (r < 12)],
//   PROJ rows [48r, 48r + 48), FC rows [192r, 192r + 192) in three chunks,
//   FCPROJ rows [48r, 48r + 48) in four chunks of three 256-column blocks;
//   head CTA j (clusters 1..): head rows [V j / H, V (j + 1) / H) in 32-row
//   chunks. Chunk layouts are in cluster.cuh. Returns LLMQ_OK without
//   enabling the kernel otherwise.
llmq_status cd_setup(llmq_model *m) {
  llmq_ctx *ctx = m->ctx;
  m->cd_ok = false;
  if (!m->mega_ok || m->kv->kind != LLMQ_KV_QUANT8 || m->C != 768 || m->n_head != 12) return LLMQ_OK;
  const size_t smem = cd_smem_bytes();
  CK(cudaFuncSetAttribute((const void *)cluster_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  CK(cudaFuncSetAttribute((const void *)cluster_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CD_CLUSTER;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeCooperative;
  at[1].val.cooperative = 1;
  cfg.gridDim = dim3(CD_CLUSTER * 2);
  cfg.blockDim = dim3(CD_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  int ncl = 0;
  if (cudaOccupancyMaxActiveClusters(&ncl, (const void *)cluster_decode_kernel, &cfg) != cudaSuccess || ncl < 2) {
    cudaGetLastError();
    return LLMQ_OK;
  }
  const int C = m->C, L = m->n_layer, V = m->V;
  const int grid = ncl * CD_CLUSTER, nh = grid - CD_CLUSTER;
  // the weights as stored, on the host
  auto fetch = [&](const llmq_weight *w, std::vector<uint8_t> &codes, std::vector<uint16_t> &sc,
                   std::vector<uint8_t> &zp) -> cudaError_t {
    const size_t gpr = (size_t)w->cols / w->group;
    codes.resize((size_t)w->rows * w->cols * w->bits / 8);
    sc.resize((size_t)w->rows * gpr);
    zp.resize((size_t)w->rows * gpr);
    cudaError_t e = cudaMemcpy(codes.data(), w->codes, codes.size(), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(sc.data(), w->scale, sc.size() * 2, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(zp.data(), w->zp, zp.size(), cudaMemcpyDeviceToHost);
    return e;
  };
  // per-layer chunk templates of each rank
  std::vector<CdChunk> tmpl((size_t)CD_CLUSTER * CD_MAX_CHUNKS);
  std::vector<int> nch(CD_CLUSTER);
  std::vector<long long> lbytes(CD_CLUSTER), lbase(CD_CLUSTER);
  long long ltotal = 0;
  for (int r = 0; r < CD_CLUSTER; r++) {
    int k = 0, off = 0;
    auto add = [&](int kind, int r0, int n, int b0, int nb) {
      CdChunk c{};
      c.kind = kind;
      c.r0 = r0;
      c.n = n;
      c.rp = (n + 7) & ~7;
      c.b0 = b0;
      c.nb = nb;
      c.off = off;
      c.scale_off = nb * c.rp * 128;
      c.zp_off = c.scale_off + nb * c.rp * 16;
      c.bytes = c.zp_off + nb * c.rp * 8;
      off += c.bytes;
      tmpl[(size_t)r * CD_MAX_CHUNKS + k++] = c;
    };
    if (r < m->n_head)
      for (int c = 0; c < 3; c++) add(CD_QKV, c * C + 64 * r, 64, 0, 3);
    add(CD_PROJ, 48 * r, 48, 0, 3);
    for (int c = 0; c < 3; c++) add(CD_FC, 192 * r + 64 * c, 64, 0, 3);
    for (int c = 0; c < 4; c++) add(CD_FCPROJ, 48 * r, 48, 3 * c, 3);
    nch[r] = k;
    lbytes[r] = off;
    lbase[r] = ltotal;
    ltotal += (long long)off * L;
  }
  for (const CdChunk &c : tmpl)
    if (c.bytes > CD_SLOT) return fail(ctx, LLMQ_ERR_INVALID, "cluster decode: a chunk exceeds its ring slot");
  std::vector<uint8_t> lh((size_t)ltotal, 0);
  std::vector<uint8_t> codes, zp;
  std::vector<uint16_t> sc;
  for (int l = 0; l < L; l++)
    for (int kind = 0; kind < 4; kind++) {
      const llmq_weight *w = m->mats[4 * l + kind];
      CK(fetch(w, codes, sc, zp));
      const long long rb = (long long)w->cols / 2, gpr = w->cols / w->group;
      for (int r = 0; r < CD_CLUSTER; r++)
        for (int k = 0; k < nch[r]; k++) {
          const CdChunk &c = tmpl[(size_t)r * CD_MAX_CHUNKS + k];
          if (c.kind != kind) continue;
          uint8_t *dst = lh.data() + lbase[r] + (long long)l * lbytes[r] + c.off;
          for (int bb = 0; bb < c.nb; bb++)
            for (int i = 0; i < c.n; i++) {
              const long long row = c.r0 + i;
              const int b = c.b0 + bb;
              for (int h = 0; h < 2; h++)
                for (int q = 0; q < 4; q++)
                  for (int j = 0; j < 4; j++)
                    std::memcpy(dst + ((size_t)(bb * 2 + h) * c.rp + i) * 64 + q * 16 + j * 4,
                                codes.data() + row * rb + b * 128 + (4 * h + j) * 16 + q * 4, 4);
              for (int g = 0; g < 8; g++) {
                std::memcpy(dst + c.scale_off + ((size_t)(bb * c.rp + i) * 8 + g) * 2, &sc[row * gpr + b * 8 + g], 2);
                dst[c.zp_off + (size_t)(bb * c.rp + i) * 8 + g] = zp[row * gpr + b * 8 + g];
              }
            }
        }
    }
  // head CTAs
  const llmq_weight *hd = m->head;
  CK(fetch(hd, codes, sc, zp));
  std::vector<long long> hbase(nh);
  long long htotal = 0;
  for (int j = 0; j < nh; j++) {
    hbase[j] = htotal;
    const int r0 = (int)((long long)V * j / nh), r1 = (int)((long long)V * (j + 1) / nh);
    htotal += (long long)((r1 - r0 + CD_HROWS - 1) / CD_HROWS) * CD_HSLOT;
  }
  std::vector<uint8_t> hh((size_t)htotal, 0);
  for (int j = 0; j < nh; j++) {
    const int r0 = (int)((long long)V * j / nh), r1 = (int)((long long)V * (j + 1) / nh);
    for (int row = r0; row < r1; row++) {
      const int ck = (row - r0) / CD_HROWS, r = (row - r0) % CD_HROWS;
      uint8_t *dst = hh.data() + hbase[j] + (long long)ck * CD_HSLOT;
      for (int c = 0; c < 24; c++)
        for (int q = 0; q < 4; q++)
          std::memcpy(dst + ((size_t)(c * 32 + r) * 4 + q) * 8, codes.data() + (size_t)row * C + c * 32 + q * 8, 8);
      std::memcpy(dst + CD_HROWS * 768 + r * 2, &sc[row], 2);
      dst[CD_HROWS * 768 + CD_HROWS * 2 + r] = zp[row];
    }
  }
  CK(cudaMalloc(&m->cd_lstream, lh.size()));
  CK(cudaMemcpy(m->cd_lstream, lh.data(), lh.size(), cudaMemcpyHostToDevice));
  CK(cudaMalloc(&m->cd_hstream, hh.size()));
  CK(cudaMemcpy(m->cd_hstream, hh.data(), hh.size(), cudaMemcpyHostToDevice));
  CK(cudaMalloc(&m->cd_lbase, sizeof(long long) * CD_CLUSTER));
  CK(cudaMemcpy(m->cd_lbase, lbase.data(), sizeof(long long) * CD_CLUSTER, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&m->cd_lbytes, sizeof(long long) * CD_CLUSTER));
  CK(cudaMemcpy(m->cd_lbytes, lbytes.data(), sizeof(long long) * CD_CLUSTER, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&m->cd_lnch, sizeof(int) * CD_CLUSTER));
  CK(cudaMemcpy(m->cd_lnch, nch.data(), sizeof(int) * CD_CLUSTER, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&m->cd_lchunks, sizeof(CdChunk) * tmpl.size()));
  CK(cudaMemcpy(m->cd_lchunks, tmpl.data(), sizeof(CdChunk) * tmpl.size(), cudaMemcpyHostToDevice));
  CK(cudaMalloc(&m->cd_hbase, sizeof(long long) * nh));
  CK(cudaMemcpy(m->cd_hbase, hbase.data(), sizeof(long long) * nh, cudaMemcpyHostToDevice));
  CK(cudaMalloc(&m->cd_ll, sizeof(unsigned long long) * (C + 2 * nh)));
  CK(cudaMemset(m->cd_ll, 0, sizeof(unsigned long long) * (C + 2 * nh)));
  m->cd_grid = grid;
  m->cd_nhcta = nh;
  m->cd_flag = 1;
  m->cd_ok = true;  // selectable; the persistent kernel stays the default (it is faster on B200)
  return LLMQ_OK;
}

// One cooperative launch of the cluster decode kernel: `steps` greedy steps
// from *first_token at pos0.
llmq_status run_cluster(llmq_model *m, const int *first_token, int pos0, int steps, int *ids, float *logits) {
  llmq_ctx *ctx = m->ctx;
  CdArgs a{};
  a.lstream = m->cd_lstream;
  a.lbase = m->cd_lbase;
  a.lchunks = m->cd_lchunks;
  a.lnch = m->cd_lnch;
  a.lbytes = m->cd_lbytes;
  a.hstream = m->cd_hstream;
  a.hbase = m->cd_hbase;
  a.n_hcta = m->cd_nhcta;
  a.n_layer = m->n_layer;
  a.C = m->C;
  a.V = m->V;
  a.n_head = m->n_head;
  a.small = m->small;
  a.head = m->head->view();
  a.kv = m->kv->v8;
  a.ll = m->cd_ll;
  a.logits = logits;
  a.ids = ids;
  a.first_token = first_token;
  a.pos0 = pos0;
  a.steps = steps;
  a.flag0 = m->cd_flag;
  a.err = m->mega_err;
  a.timeout_cycles = ctx->wait_cycles;
  a.prof = m->prof;
  m->cd_flag += (unsigned)steps;
  cudaLaunchConfig_t cfg{};
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CD_CLUSTER;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeCooperative;
  at[1].val.cooperative = 1;
  cfg.gridDim = dim3(m->cd_grid);
  cfg.blockDim = dim3(CD_THREADS);
  cfg.dynamicSmemBytes = cd_smem_bytes();
  cfg.stream = ctx->stream;
  cfg.attrs = at;
  cfg.numAttrs = 2;
  CK(cudaLaunchKernelEx(&cfg, cluster_decode_kernel, a));
  return LLMQ_OK;
}

// One cooperative launch: `steps` greedy steps from *first_token at pos0.
llmq_status run_mega(llmq_model *m, const int *first_token, int pos0, int steps, int *ids, float *logits) {
  if (m->mode == LLMQ_MODE_CLUSTER && m->cd_ok) return run_cluster(m, first_token, pos0, steps, ids, logits);
  llmq_ctx *ctx = m->ctx;
  MegaArgs a{};
  a.stream = m->mega_stream;
  a.stream_base = m->mega_base;
  a.chunks = m->mega_chunks;
  a.nchunks = m->mega_nchunks;
  a.n_layer = m->n_layer;
  a.C = m->C;
  a.V = m->V;
  a.n_head = m->n_head;
  a.small = m->small;
  a.head = m->head->view();
  a.kv = m->kv->v8;
  a.ia = m->kv->ia;
  a.intattn = m->kv->kind == LLMQ_KV_INTATTN;
  a.ia_mult = ia_mult();
  a.ll = m->mega_ll;
  a.logits = logits;
  a.ids = ids;
  a.first_token = first_token;
  a.pos0 = pos0;
  a.steps = steps;
  a.flag0 = m->mega_flag;
  a.err = m->mega_err;
  a.timeout_cycles = ctx->wait_cycles;
  a.prof = m->prof;
  m->mega_flag += (unsigned)steps;
  void *args[] = {&a};
  CK(cudaLaunchCooperativeKernel((const void *)mega_decode_kernel, m->mega_grid, MK_THREADS, args, sizeof(MkSmem),
                                 ctx->stream));
  return LLMQ_OK;
}

// After a synchronisation: turns a recorded device-side timeout into a status.
llmq_status mega_check(llmq_model *m) {
  llmq_ctx *ctx = m->ctx;
  if (!m->mega_ok) return LLMQ_OK;
  int code = 0;
  CK(cudaMemcpy(&code, m->mega_err, sizeof(int), cudaMemcpyDeviceToHost));
  if (code) {
    cudaMemset(m->mega_err, 0, sizeof(int));
    return fail(ctx, LLMQ_ERR_TIMEOUT, "persistent decode kernel: a bounded wait gave up (code " +
                                           std::to_string(code) + ")");
  }
  return LLMQ_OK;
}

// One decode step (gpt2t.mojo:350-447): embedding, 12 x (LN1 + QKV, KV store
// + attention, PROJ + residual, LN2 + FC + GELU, FCPROJ + residual), LN_f +
// head + argmax. Token, position and step index come from m->state.
llmq_status enqueue_decode_step(llmq_model *m, cudaStream_t s) {
  llmq_ctx *ctx = m->ctx;
  embed_kernel<<<3, 256, 0, s>>>(m->head->view(), m->wpe(), m->x, m->state);
  CKL();
  for (int l = 0; l < m->n_layer; l++) {
    const llmq_weight *const *w = &m->mats[4 * l];
    GemvArgs a{};
    a.w = w[0]->view();
    a.x = m->x;
    a.ln_w = m->vec(l, 0);
    a.ln_b = m->vec(l, 1);
    a.bias = m->vec(l, 2);
    a.out = m->qkv;
    a.epi = EPI_BIAS;
    CK(launch_gemv(ctx, a, PRO_LN, false, s));
    if (m->kv->kind == LLMQ_KV_QUANT8) {
      const llmq_status st = kv8_attend(ctx, m->kv->v8, m->att, m->qkv, l, 0, &m->state->pos, 1, m->max_t,
                                        dim3(m->n_head, 1), s);
      if (st) return st;
    } else
      ia_attend_kernel<<<dim3(m->n_head, 1), 256, ia_attend_smem(m->kv), s>>>(m->kv->ia, m->att, m->qkv, l, 0,
                                                                               &m->state->pos, 1, ia_mult());
    CKL();
    a = GemvArgs{};
    a.w = w[1]->view();
    a.x = m->att;
    a.bias = m->vec(l, 3);
    a.out = m->x;
    a.epi = EPI_BIAS | EPI_RESID;
    CK(launch_gemv(ctx, a, PRO_QUANT, false, s));
    a = GemvArgs{};
    a.w = w[2]->view();
    a.x = m->x;
    a.ln_w = m->vec(l, 4);
    a.ln_b = m->vec(l, 5);
    a.bias = m->vec(l, 6);
    a.out = m->fc;
    a.epi = EPI_BIAS | EPI_GELU;
    CK(launch_gemv(ctx, a, PRO_LN, false, s));
    a = GemvArgs{};
    a.w = w[3]->view();
    a.x = m->fc;
    a.bias = m->vec(l, 7);
    a.out = m->x;
    a.epi = EPI_BIAS | EPI_RESID;
    CK(launch_gemv(ctx, a, PRO_QUANT, false, s));
  }
  GemvArgs a{};
  a.w = m->head->view();
  a.x = m->x;
  a.ln_w = m->lnf_w();
  a.ln_b = m->lnf_b();
  a.out = m->logits;
  a.part_val = m->part_val;
  a.part_idx = m->part_idx;
  a.state = m->state;
  a.ids = m->ids;
  CK(launch_gemv(ctx, a, PRO_LN, true, s));
  return LLMQ_OK;
}

// Several tokens at positions pos0.. through all layers (gpt2t.mojo:485-571);
// leaves the hidden states in m->x.
llmq_status enqueue_blocks(llmq_model *m, int T, int pos0, cudaStream_t s) {
  llmq_ctx *ctx = m->ctx;
  const int C = m->C;
  const llmq_weight *hd = m->embed ? m->embed : m->head;
  if (hd->kind == WK_AFFINE) {
    embed_rows_kernel<<<T, 256, 0, s>>>(hd->view(), m->wpe(), m->x, m->tokens, pos0);
  } else if (hd->kind == WK_DENSE) {
    if (hd->rtype == RT_F32)
      embed_dense_kernel<0><<<T, 256, 0, s>>>(hd->codes, C, hd->rows, m->wpe(), m->x, m->tokens, pos0);
    else if (hd->rtype == RT_BF16)
      embed_dense_kernel<1><<<T, 256, 0, s>>>(hd->codes, C, hd->rows, m->wpe(), m->x, m->tokens, pos0);
    else
      return fail(ctx, LLMQ_ERR_UNSUPPORTED, "dense embeddings take float32 or bfloat16");
  } else {
    const RowMat rm = hd->rowmat();
#define EG(T) \
  case T:     \
    embed_gguf_kernel<T><<<T_, 256, 0, s>>>(rm, m->wpe(), m->x, m->tokens, pos0); \
    break;
    const int T_ = T;
    switch (hd->rtype) {
      EG(RT_F32) EG(RT_F16) EG(RT_BF16) EG(RT_Q4_0) EG(RT_Q4_1) EG(RT_Q8_0) EG(RT_Q4_K) EG(RT_Q5_K) EG(RT_Q6_K)
      default:
        return fail(ctx, LLMQ_ERR_UNSUPPORTED, "GGUF type");
    }
#undef EG
  }
  CKL();
  llmq_status st;
  for (int l = 0; l < m->n_layer; l++) {
    const llmq_weight *const *w = &m->mats[4 * l];
    launch_layernorm(m->xn, m->x, m->vec(l, 0), m->vec(l, 1), T, C, s);
    CKL();
    if ((st = llmq_linear(ctx, w[0], m->xn, m->vec(l, 2), m->qkv, T, C, 3 * C, LLMQ_BIAS)) != LLMQ_OK) return st;
    if ((st = llmq_kv_store(ctx, m->kv, l, pos0, T, m->qkv)) != LLMQ_OK) return st;
    if ((st = llmq_kv_attend(ctx, m->kv, m->att, m->qkv, l, T, pos0)) != LLMQ_OK) return st;
    if ((st = llmq_linear(ctx, w[1], m->att, m->vec(l, 3), m->x, T, C, C, LLMQ_BIAS | LLMQ_RESID)) != LLMQ_OK) return st;
    launch_layernorm(m->xn, m->x, m->vec(l, 4), m->vec(l, 5), T, C, s);
    CKL();
    if ((st = llmq_linear(ctx, w[2], m->xn, m->vec(l, 6), m->fc, T, C, 4 * C, LLMQ_BIAS | LLMQ_GELU)) != LLMQ_OK) return st;
    if ((st = llmq_linear(ctx, w[3], m->fc, m->vec(l, 7), m->x, T, 4 * C, C, LLMQ_BIAS | LLMQ_RESID)) != LLMQ_OK) return st;
  }
  return LLMQ_OK;
}

}  // namespace

extern "C" {

llmq_status llmq_model_create(llmq_ctx *ctx, int n_layer, llmq_weight *const *mats, const llmq_weight *head,
                              const float *small_host, int kv_kind, int max_t, llmq_model **out) {
  if (!ctx || !mats || !head || !small_host || !out || n_layer <= 0 || max_t <= 0 || max_t > 1024)
    return fail(ctx, LLMQ_ERR_INVALID, "bad model arguments");
  const int C = 768;
  bool a16 = head->kind == WK_AFFINE && head->a16;
  for (int i = 0; i < 4 * n_layer; i++) {
    static const int ins[4] = {C, C, C, 4 * C}, outs[4] = {3 * C, C, 4 * C, C};
    const llmq_weight *w = mats[i];
    // dense layers are [IN, OUT] (Conv1D); the others [OUT, IN]
    const bool shape_ok = w && (w->kind == WK_DENSE ? (w->rows == ins[i % 4] && w->cols == outs[i % 4])
                                                    : (w->cols == ins[i % 4] && w->rows == outs[i % 4]));
    const bool fmt_ok = w && (w->kind == WK_DENSE || w->kind == WK_GGUF || w->kind == WK_AFFINE);
    if (!shape_ok || !fmt_ok)
      return fail(ctx, LLMQ_ERR_INVALID, "layer matrix " + std::to_string(i) + " has an unexpected shape or format");
    a16 = a16 && w->kind == WK_AFFINE && w->a16;
  }
  if (head->cols != C) return fail(ctx, LLMQ_ERR_INVALID, "head must be a [V, 768] matrix");
  if (!a16 && kv_kind == LLMQ_KV_INTATTN)
    return fail(ctx, LLMQ_ERR_UNSUPPORTED, "float-format models take the int8 or a dense cache");
  *out = nullptr;
  CK(cudaSetDevice(ctx->device));
  llmq_model *m = new llmq_model();
  m->ctx = ctx;
  m->n_layer = n_layer;
  m->C = C;
  m->V = head->rows;
  m->max_t = max_t;
  m->n_head = 12;
  m->mats.assign(mats, mats + 4 * n_layer);
  m->head = head;
  m->float_only = !a16;
  m->max_ids = 4096;
  llmq_status st = llmq_kv_create(ctx, kv_kind, n_layer, max_t, m->n_head, C / m->n_head, &m->kv);
  if (st != LLMQ_OK) {
    delete m;
    return st;
  }
  size_t small_n = (size_t)n_layer * 13 * C + (size_t)1024 * C + 2 * C;
  int grid = a16 ? gemv_grid(ctx, head->view()) : 1;
  cudaError_t e = cudaMalloc(&m->small, small_n * 4);
  if (e == cudaSuccess) e = cudaMemcpy(m->small, small_host, small_n * 4, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) e = cudaMalloc(&m->x, (size_t)max_t * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->xn, (size_t)max_t * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->qkv, (size_t)max_t * 3 * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->att, (size_t)max_t * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->fc, (size_t)max_t * 4 * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->logits, (size_t)m->V * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->tokens, (size_t)max_t * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->ids, (size_t)m->max_ids * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->part_val, (size_t)grid * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->part_idx, (size_t)grid * 4);
  if (e == cudaSuccess) e = cudaMalloc(&m->state, sizeof(DecodeState));
  if (e == cudaSuccess) e = cudaMemset(m->state, 0, sizeof(DecodeState));
  if (e == cudaSuccess) e = cudaMallocHost(&m->state_host, sizeof(DecodeState));
  if (e == cudaSuccess) e = cudaMallocHost(&m->ids_host, (size_t)m->max_ids * 4);
  if (e != cudaSuccess) {
    llmq_model_free(m);
    return fail(ctx, LLMQ_ERR_CUDA, std::string("model alloc: ") + cudaGetErrorString(e));
  }
  if ((st = mega_setup(m)) != LLMQ_OK || (st = cd_setup(m)) != LLMQ_OK) {
    llmq_model_free(m);
    return st;
  }
  *out = m;
  return LLMQ_OK;
}

llmq_status llmq_model_free(llmq_model *m) {
  if (!m) return LLMQ_ERR_INVALID;
  cudaSetDevice(m->ctx->device);
  if (m->exec) cudaGraphExecDestroy(m->exec);
  if (m->graph) cudaGraphDestroy(m->graph);
  if (m->kv) llmq_kv_free(m->kv);
  float *fs[] = {m->small, m->x, m->xn, m->qkv, m->att, m->fc, m->logits, m->part_val};
  for (float *p : fs)
    if (p) cudaFree(p);
  if (m->tokens) cudaFree(m->tokens);
  if (m->ids) cudaFree(m->ids);
  if (m->part_idx) cudaFree(m->part_idx);
  if (m->state) cudaFree(m->state);
  if (m->state_host) cudaFreeHost(m->state_host);
  if (m->ids_host) cudaFreeHost(m->ids_host);
  if (m->mega_stream) cudaFree(m->mega_stream);
  if (m->mega_base) cudaFree(m->mega_base);
  if (m->mega_chunks) cudaFree(m->mega_chunks);
  if (m->mega_ll) cudaFree(m->mega_ll);
  if (m->mega_err) cudaFree(m->mega_err);
  void *cds[] = {m->cd_lstream, m->cd_hstream, m->cd_lbase, m->cd_lbytes, m->cd_hbase, m->cd_lchunks, m->cd_lnch,
                 m->cd_ll};
  for (void *p : cds)
    if (p) cudaFree(p);
  if (m->prof) cudaFree(m->prof);
  for (llmq_weight *w : m->owned) llmq_weight_free(w);
  delete m;
  return LLMQ_OK;
}

llmq_status llmq_model_set_mode(llmq_model *m, int mode) {
  if (!m) return LLMQ_ERR_INVALID;
  if (mode != LLMQ_MODE_EAGER && mode != LLMQ_MODE_GRAPH && mode != LLMQ_MODE_PERSISTENT && mode != LLMQ_MODE_CLUSTER)
    return fail(m->ctx, LLMQ_ERR_INVALID, "unknown mode");
  if (mode == LLMQ_MODE_PERSISTENT && !m->mega_ok)
    return fail(m->ctx, LLMQ_ERR_UNSUPPORTED, "the persistent decode kernel runs int4-g32 A16 layers, a per-channel "
                                              "int8 A16 head and the QuantKV[8] or IntAttnKV cache");
  if (mode == LLMQ_MODE_CLUSTER && !m->cd_ok)
    return fail(m->ctx, LLMQ_ERR_UNSUPPORTED, "the cluster decode kernel runs int4-g32 A16 layers, a per-channel int8 "
                                              "A16 head and the QuantKV[8] cache of a 768-wide, 12-head model, on a "
                                              "device with room for two 16-CTA clusters");
  m->mode = mode;
  return LLMQ_OK;
}

int llmq_model_mode(const llmq_model *m) { return m ? m->mode : -1; }

// ---- sampling (gpt2t.mojo:775-834) ----

static int pow2_at_least(int v) {
  int n = 1;
  while (n < v) n <<= 1;
  return n;
}

constexpr int kSampleMaxV = 1 << 24;

static llmq_status sample_scratch(llmq_ctx *ctx, int V) {
  const int n = std::max(pow2_at_least(V), kSortChunk);
  if (!ctx->samp_cand) CK(cudaMalloc(&ctx->samp_cand, sizeof(unsigned long long) * kMergeCap));
  if (!ctx->samp_rng) CK(cudaMalloc(&ctx->samp_rng, sizeof(unsigned long long)));
  if (!ctx->samp_done) CK(cudaMalloc(&ctx->samp_done, sizeof(int)));
  if (n <= ctx->samp_n) return LLMQ_OK;
  CK(cudaStreamSynchronize(ctx->stream));
  if (ctx->samp_keys) cudaFree(ctx->samp_keys);
  ctx->samp_keys = nullptr;
  ctx->samp_n = 0;
  CK(cudaMalloc(&ctx->samp_keys, sizeof(unsigned long long) * n));
  ctx->samp_n = n;
  return LLMQ_OK;
}

// A draw from logits[0, V) into `o` (topk_ids == nullptr), or the top-k ids
// into topk_ids. k <= 0 or k >= V means all V (sample: `k if k > 0 else V`;
// top_k stops at V). The scratch must hold V keys (sample_scratch).
static llmq_status enqueue_sample(llmq_ctx *ctx, const float *logits, int V, float temperature, int k,
                                  unsigned long long *rng, SampleOut o, int *topk_ids, cudaStream_t s) {
  const int kk = (k > 0 && k < V) ? k : V;
  const int chunks = (V + kSortChunk - 1) / kSortChunk;
  if (kk <= kTopkSmall && (long long)chunks * kk <= kMergeCap) {
    const int n_cand = chunks * kk, n_pad = std::max(pow2_at_least(n_cand), 2);
    int *done = ctx->samp_done;
    topk_fast_kernel<<<1, kSortThreads, fast_smem(), s>>>(logits, V, kk, temperature, rng, o, topk_ids, done);
    CKL();
    sort_chunk_kernel<<<chunks, kSortThreads, 0, s>>>(logits, V, nullptr, 2, kSortChunk, 1, ctx->samp_cand, kk, done);
    CKL();
    merge_draw_kernel<<<1, kSortThreads, merge_smem(n_pad), s>>>(ctx->samp_cand, n_cand, n_pad, kk, logits,
                                                                   temperature, rng, o, topk_ids, done);
    CKL();
    return LLMQ_OK;
  }
  const int n = std::max(pow2_at_least(V), kSortChunk);
  unsigned long long *keys = ctx->samp_keys;
  sort_chunk_kernel<<<n / kSortChunk, kSortThreads, 0, s>>>(logits, V, keys, 2, kSortChunk, 0, nullptr, 0);
  CKL();
  for (int sz = 2 * kSortChunk; sz <= n; sz <<= 1) {
    for (int j = sz / 2; j >= kSortChunk; j >>= 1) {
      bitonic_global_kernel<<<std::min(n / 512, 4 * ctx->num_sms), 256, 0, s>>>(keys, n, sz, j);
      CKL();
    }
    sort_chunk_kernel<<<n / kSortChunk, kSortThreads, 0, s>>>(nullptr, V, keys, sz, sz, 0, nullptr, 0);
    CKL();
  }
  sorted_draw_kernel<<<1, kSortThreads, 0, s>>>(keys, kk, logits, temperature, rng, o, topk_ids);
  CKL();
  return LLMQ_OK;
}

// What generate_sampled draws with: temperature > 0, k, the device Rng state.
struct SampleSpec {
  float temperature;
  int k;
  unsigned long long *rng;
};

static llmq_status run_decode_step(llmq_model *m) {
  llmq_ctx *ctx = m->ctx;
  cudaStream_t s = ctx->stream;
  if (m->mode == LLMQ_MODE_EAGER) return enqueue_decode_step(m, s);
  if (!m->exec) {
    CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    llmq_status st = enqueue_decode_step(m, s);
    cudaGraph_t g = nullptr;
    cudaError_t e = cudaStreamEndCapture(s, &g);
    if (st != LLMQ_OK) {
      if (g) cudaGraphDestroy(g);
      return st;
    }
    CK(e);
    m->graph = g;
    CK(cudaGraphInstantiate(&m->exec, g, 0));
  }
  CK(cudaGraphLaunch(m->exec, s));
  return LLMQ_OK;
}

__global__ void init_state_kernel(DecodeState *st, const int *tokens, int pos0) {
  st->token = tokens[0];
  st->pos = pos0;
  st->step = 0;
  st->ticket = 0;
}

// Prefill of the T tokens in m->tokens at positions pos0.., then the head's
// argmax: ids[0], state = {token: ids[0], pos: pos0 + T, step: 1}.
static llmq_status run_prompt_tail(llmq_model *m, int T, int pos0) {
  llmq_ctx *ctx = m->ctx;
  cudaStream_t s = ctx->stream;
  llmq_status st = enqueue_blocks(m, T, pos0, s);
  if (st != LLMQ_OK) return st;
  *m->state_host = DecodeState{};
  m->state_host->pos = pos0 + T - 1;
  CK(cudaMemcpyAsync(m->state, m->state_host, sizeof(DecodeState), cudaMemcpyHostToDevice, s));
  GemvArgs a{};
  a.w = m->head->view();
  a.x = m->x + (size_t)(T - 1) * m->C;
  a.ln_w = m->lnf_w();
  a.ln_b = m->lnf_b();
  a.out = m->logits;
  a.part_val = m->part_val;
  a.part_idx = m->part_idx;
  a.state = m->state;
  a.ids = m->ids;
  CK(launch_gemv(ctx, a, PRO_LN, true, s));
  return LLMQ_OK;
}

// `steps` greedy steps from the T tokens in m->tokens at positions pos0..:
// ids into m->ids[0, steps), the last step's logits into m->logits (always
// in the graph and eager modes; with want_logits in the persistent mode).
// Asynchronous on the context's stream.
// forward + greedy decode for the float-activation formats (generate,
// gpt2t.mojo:942-980): the blocks for the T prompt tokens, the final
// LayerNorm of the last row, the head for it and the argmax, then one token
// at a time through the same one-token paths (dense gemv, GGUF dot_row).
static llmq_status float_generation(llmq_model *m, int T, int pos0, int steps, const SampleSpec *sp) {
  llmq_ctx *ctx = m->ctx;
  cudaStream_t s = ctx->stream;
  const int C = m->C;
  llmq_status st;
  for (int i = 0; i < steps; i++) {
    const int n = i == 0 ? T : 1, p = i == 0 ? pos0 : pos0 + T + i - 1;
    if ((st = enqueue_blocks(m, n, p, s)) != LLMQ_OK) return st;
    layernorm_kernel<<<1, 256, C * 4, s>>>(m->xn, m->x + (size_t)(n - 1) * C, m->lnf_w(), m->lnf_b(), C);
    CKL();
    if ((st = llmq_head(ctx, m->head, m->xn, m->logits, 1, C, m->V)) != LLMQ_OK) return st;
    if (sp) {
      st = enqueue_sample(ctx, m->logits, m->V, sp->temperature, sp->k, sp->rng,
                          SampleOut{m->ids + i, m->tokens, nullptr, nullptr, nullptr}, nullptr, s);
      if (st != LLMQ_OK) return st;
      continue;
    }
    argmax_rows_kernel<<<1, 256, 0, s>>>(m->logits, m->V, m->ids + i, 0, m->tokens, nullptr);
    CKL();
  }
  return LLMQ_OK;
}

// With a SampleSpec every head's argmax is replaced by a draw: the head
// still writes the logits, the draw overwrites the id and the next token. In
// the persistent mode the kernel then runs one token per launch (it writes
// the logits, the draw writes the token the next launch embeds).
// Whether decode steps run as one launch of a persistent kernel per generation.
static bool persistent_mode(const llmq_model *m) {
  return (m->mode == LLMQ_MODE_PERSISTENT && m->mega_ok) || (m->mode == LLMQ_MODE_CLUSTER && m->cd_ok);
}

static llmq_status run_generation(llmq_model *m, int T, int pos0, int steps, bool want_logits,
                                  const SampleSpec *sp = nullptr) {
  llmq_ctx *ctx = m->ctx;
  cudaStream_t s = ctx->stream;
  if (m->float_only) return float_generation(m, T, pos0, steps, sp);
  if (sp && persistent_mode(m)) {
    llmq_status st;
    int pos = pos0, i = 0;
    if (T > 1) {
      if ((st = run_prompt_tail(m, T, pos0)) != LLMQ_OK) return st;
      st = enqueue_sample(ctx, m->logits, m->V, sp->temperature, sp->k, sp->rng,
                          SampleOut{m->ids, m->tokens, nullptr, nullptr, nullptr}, nullptr, s);
      if (st != LLMQ_OK) return st;
      pos = pos0 + T;
      i = 1;
    }
    for (; i < steps; i++, pos++) {
      if ((st = run_mega(m, m->tokens, pos, 1, m->ids + i, m->logits)) != LLMQ_OK) return st;
      st = enqueue_sample(ctx, m->logits, m->V, sp->temperature, sp->k, sp->rng,
                          SampleOut{m->ids + i, m->tokens, nullptr, nullptr, nullptr}, nullptr, s);
      if (st != LLMQ_OK) return st;
    }
    return LLMQ_OK;
  }
  const bool pers = persistent_mode(m) && !sp;
  const SampleOut so{nullptr, nullptr, &m->state->token, &m->state->step, m->ids};
  auto draw = [&]() -> llmq_status {
    return sp ? enqueue_sample(ctx, m->logits, m->V, sp->temperature, sp->k, sp->rng, so, nullptr, s) : LLMQ_OK;
  };
  llmq_status st;
  if (T == 1) {
    if (pers) return run_mega(m, m->tokens, pos0, steps, m->ids, want_logits ? m->logits : nullptr);
    init_state_kernel<<<1, 1, 0, s>>>(m->state, m->tokens, pos0);
    CKL();
    for (int i = 0; i < steps; i++) {
      if ((st = run_decode_step(m)) != LLMQ_OK) return st;
      if ((st = draw()) != LLMQ_OK) return st;
    }
    return LLMQ_OK;
  }
  if ((st = run_prompt_tail(m, T, pos0)) != LLMQ_OK) return st;
  if ((st = draw()) != LLMQ_OK) return st;
  if (steps == 1) return LLMQ_OK;
  if (pers) return run_mega(m, &m->state->token, pos0 + T, steps - 1, m->ids + 1, want_logits ? m->logits : nullptr);
  for (int i = 1; i < steps; i++) {
    if ((st = run_decode_step(m)) != LLMQ_OK) return st;
    if ((st = draw()) != LLMQ_OK) return st;
  }
  return LLMQ_OK;
}

static llmq_status check_tokens(llmq_ctx *ctx, llmq_model *m, const int *tokens, int T) {
  for (int i = 0; i < T; i++)
    if (tokens[i] < 0 || tokens[i] >= m->V) return fail(ctx, LLMQ_ERR_INVALID, "token id out of range");
  return LLMQ_OK;
}

llmq_status llmq_model_forward(llmq_ctx *ctx, llmq_model *m, const int *tokens, int T, int pos0, float *logits_dev,
                               int *argmax_host) {
  if (!ctx || !m || !tokens || T <= 0 || pos0 < 0 || pos0 + T > m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad tokens or positions");
  llmq_status st = check_tokens(ctx, m, tokens, T);
  if (st != LLMQ_OK) return st;
  CK(cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->stream;
  CK(cudaStreamSynchronize(s));
  CK(cudaMemcpyAsync(m->tokens, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, s));
  if ((st = run_generation(m, T, pos0, 1, logits_dev != nullptr)) != LLMQ_OK) return st;
  if (logits_dev) CK(cudaMemcpyAsync(logits_dev, m->logits, (size_t)m->V * 4, cudaMemcpyDeviceToDevice, s));
  CK(cudaMemcpyAsync(m->ids_host, m->ids, 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if ((st = mega_check(m)) != LLMQ_OK) return st;
  if (argmax_host) *argmax_host = m->ids_host[0];
  return LLMQ_OK;
}

llmq_status llmq_model_forward_all(llmq_ctx *ctx, llmq_model *m, const int *tokens, int T, float *logits_dev) {
  if (!ctx || !m || !tokens || !logits_dev || T <= 0 || T > m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad tokens");
  for (int i = 0; i < T; i++)
    if (tokens[i] < 0 || tokens[i] >= m->V) return fail(ctx, LLMQ_ERR_INVALID, "token id out of range");
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->stream));
  cudaStream_t s = ctx->stream;
  CK(cudaMemcpyAsync(m->tokens, tokens, (size_t)T * 4, cudaMemcpyHostToDevice, s));
  llmq_status st = enqueue_blocks(m, T, 0, s);
  if (st == LLMQ_OK) {
    launch_layernorm(m->xn, m->x, m->lnf_w(), m->lnf_b(), T, m->C, s);
    st = llmq_head(ctx, m->head, m->xn, logits_dev, T, m->C, m->V);
  }
  if (st != LLMQ_OK) return st;
  CK(cudaStreamSynchronize(s));
  return LLMQ_OK;
}

llmq_status llmq_generate(llmq_ctx *ctx, llmq_model *m, const int *prompt, int n_prompt, int steps, int *out_ids) {
  if (!ctx || !m || !prompt || !out_ids || n_prompt <= 0 || steps <= 0 || steps > m->max_ids ||
      n_prompt + steps - 1 > m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad prompt or step count");
  llmq_status st = check_tokens(ctx, m, prompt, n_prompt);
  if (st != LLMQ_OK) return st;
  CK(cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->stream;
  CK(cudaStreamSynchronize(s));
  CK(cudaMemcpyAsync(m->tokens, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, s));
  if ((st = run_generation(m, n_prompt, 0, steps, false)) != LLMQ_OK) return st;
  CK(cudaMemcpyAsync(m->ids_host, m->ids, (size_t)steps * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if ((st = mega_check(m)) != LLMQ_OK) return st;
  std::memcpy(out_ids, m->ids_host, (size_t)steps * 4);
  return LLMQ_OK;
}

llmq_status llmq_generate_async(llmq_ctx *ctx, llmq_model *m, const int *prompt_dev, int n_prompt, int steps,
                                int *ids_dev) {
  if (!ctx || !m || !prompt_dev || !ids_dev || n_prompt <= 0 || steps <= 0 || steps > m->max_ids ||
      n_prompt + steps - 1 > m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad prompt or step count");
  CK(cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->stream;
  CK(cudaMemcpyAsync(m->tokens, prompt_dev, (size_t)n_prompt * 4, cudaMemcpyDeviceToDevice, s));
  llmq_status st = run_generation(m, n_prompt, 0, steps, false);
  if (st != LLMQ_OK) return st;
  CK(cudaMemcpyAsync(ids_dev, m->ids, (size_t)steps * 4, cudaMemcpyDeviceToDevice, s));
  return LLMQ_OK;
}

unsigned long long llmq_rng_init(long long seed) { return (unsigned long long)seed * 0x9E3779B97F4A7C15ull + 1ull; }

llmq_status llmq_top_k(llmq_ctx *ctx, const float *logits_dev, int V, int k, int *ids_dev) {
  if (!ctx || !logits_dev || !ids_dev || V <= 0 || V > kSampleMaxV) return fail(ctx, LLMQ_ERR_INVALID, "bad top_k");
  CK(cudaSetDevice(ctx->device));
  llmq_status st = sample_scratch(ctx, V);
  if (st != LLMQ_OK) return st;
  return enqueue_sample(ctx, logits_dev, V, 1.0f, k, nullptr, SampleOut{}, ids_dev, ctx->stream);
}

llmq_status llmq_sample(llmq_ctx *ctx, const float *logits_dev, int V, float temperature, int k,
                        unsigned long long *rng_dev, int *id_dev) {
  if (!ctx || !logits_dev || !rng_dev || !id_dev || V <= 0 || V > kSampleMaxV)
    return fail(ctx, LLMQ_ERR_INVALID, "bad sample arguments");
  CK(cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->stream;
  if (temperature <= 0) {
    argmax_rows_kernel<<<1, 256, 0, s>>>(logits_dev, V, id_dev, 0, id_dev, nullptr);
    CKL();
    return LLMQ_OK;
  }
  llmq_status st = sample_scratch(ctx, V);
  if (st != LLMQ_OK) return st;
  return enqueue_sample(ctx, logits_dev, V, temperature, k, rng_dev, SampleOut{id_dev, nullptr, nullptr, nullptr,
                                                                              nullptr}, nullptr, s);
}

llmq_status llmq_generate_sampled(llmq_ctx *ctx, llmq_model *m, const int *prompt, int n_prompt, int steps,
                                  float temperature, int k, unsigned long long *rng_state, int *out_ids) {
  if (!rng_state) return fail(ctx, LLMQ_ERR_INVALID, "null rng state");
  if (temperature <= 0) return llmq_generate(ctx, m, prompt, n_prompt, steps, out_ids);
  if (!ctx || !m || !prompt || !out_ids || n_prompt <= 0 || steps <= 0 || steps > m->max_ids ||
      n_prompt + steps - 1 > m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad prompt or step count");
  llmq_status st = check_tokens(ctx, m, prompt, n_prompt);
  if (st != LLMQ_OK) return st;
  CK(cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->stream;
  CK(cudaStreamSynchronize(s));
  if ((st = sample_scratch(ctx, m->V)) != LLMQ_OK) return st;
  CK(cudaMemcpyAsync(ctx->samp_rng, rng_state, sizeof(unsigned long long), cudaMemcpyHostToDevice, s));
  CK(cudaMemcpyAsync(m->tokens, prompt, (size_t)n_prompt * 4, cudaMemcpyHostToDevice, s));
  const SampleSpec sp{temperature, k, ctx->samp_rng};
  if ((st = run_generation(m, n_prompt, 0, steps, false, &sp)) != LLMQ_OK) return st;
  CK(cudaMemcpyAsync(m->ids_host, m->ids, (size_t)steps * 4, cudaMemcpyDeviceToHost, s));
  CK(cudaMemcpyAsync(rng_state, ctx->samp_rng, sizeof(unsigned long long), cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if ((st = mega_check(m)) != LLMQ_OK) return st;
  std::memcpy(out_ids, m->ids_host, (size_t)steps * 4);
  return LLMQ_OK;
}

llmq_status llmq_model_profile(llmq_ctx *ctx, llmq_model *m, int enable) {
  if (!ctx || !m) return LLMQ_ERR_INVALID;
  CK(cudaSetDevice(ctx->device));
  if (enable && !m->prof) {
    CK(cudaMalloc(&m->prof, sizeof(long long) * 2 * MK_PROF));
    CK(cudaMemset(m->prof, 0, sizeof(long long) * 2 * MK_PROF));
  } else if (!enable && m->prof) {
    CK(cudaStreamSynchronize(ctx->stream));
    cudaFree(m->prof);
    m->prof = nullptr;
  }
  return LLMQ_OK;
}

llmq_status llmq_model_profile_read(llmq_ctx *ctx, llmq_model *m, long long *cycles_host, int n, int reset) {
  if (!ctx || !m || !cycles_host || n < 2 * MK_PROF) return fail(ctx, LLMQ_ERR_INVALID, "need 40 entries");
  if (!m->prof) return fail(ctx, LLMQ_ERR_INVALID, "profiling is off");
  CK(cudaStreamSynchronize(ctx->stream));
  CK(cudaMemcpy(cycles_host, m->prof, sizeof(long long) * 2 * MK_PROF, cudaMemcpyDeviceToHost));
  if (reset) CK(cudaMemset(m->prof, 0, sizeof(long long) * 2 * MK_PROF));
  return LLMQ_OK;
}

llmq_status llmq_model_check(llmq_ctx *ctx, llmq_model *m) {
  if (!ctx || !m) return LLMQ_ERR_INVALID;
  CK(cudaStreamSynchronize(ctx->stream));
  return mega_check(m);
}

}  // extern "C"

// ---- batched greedy decode of independent sequences ----------------------

struct llmq_batch {
  float *part_val = nullptr;  // [max_seqs][head row tiles] argmax partials
  int *part_idx = nullptr;
  llmq_ctx *ctx;
  llmq_model *m;
  int max_seqs, max_prompt;
  KV8View kv{};            // [max_seqs] QuantKV[8] caches of m->max_t positions
  float *x = nullptr, *xn = nullptr, *qkv = nullptr, *att = nullptr, *fc = nullptr;  // [max_seqs * max_prompt] rows
  float *logits = nullptr; // [max_seqs][V]
  int16_t *xq = nullptr;   // [max_seqs][3072]
  float *xsf = nullptr;    // [max_seqs][3072 / 16]
  int *xsi = nullptr;      // [max_seqs][units * 16] (units of the widest matrix)
  float *sx = nullptr;     // [max_seqs]
  int *tokens = nullptr;   // [max_seqs * max_prompt]
  int *ids = nullptr;      // [max_seqs][max_t]
  int *state = nullptr;    // [0] position, [1] step
  int *ids_host = nullptr; // pinned [max_seqs][max_t]
  int *prompt_host = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t exec = nullptr;
  int graph_B = 0, graph_steps = 0;
  int graph_kernel = -1;      // the kernel choice the decode-step graph was captured with
  int graph_cap = 0;          // and the attention context it was sized for
  uint8_t *tcl_b = nullptr;  // the lane-mode GEMM's sequence tiles [max_seqs padded to TCL_TT][widest K x 4]
  int kernel = LLMQ_BATCH_AUTO;
};

namespace {

int fmt_code(const llmq_weight *w) { return fmt_of(w->view()); }

constexpr int TCL_TT = 16;          // sequences per lane-mode GEMM tile
constexpr int TCL_MIN_SEQS = 16;    // AUTO: the lane-mode GEMM from this many sequences

// Whether batch_linear runs w for B sequences as the lane-mode tcgen05 GEMM.
bool batch_uses_tcl(const llmq_batch *bt, const llmq_weight *w, int B) {
  if (!w->tcl_a || bt->kernel == LLMQ_BATCH_CUDA_CORE) return false;
  return bt->kernel == LLMQ_BATCH_TCGEN05 || B >= TCL_MIN_SEQS;
}

// The argmax partials per sequence of the batched head (row tiles of the
// kernel that runs it).
int batch_head_parts(const llmq_batch *bt, int B) {
  const llmq_model *m = bt->m;
  return batch_uses_tcl(bt, m->head, B) ? 4 * ((m->V + TC_M - 1) / TC_M) : (m->V + BG_ROWS - 1) / BG_ROWS;
}

// The lane-mode GEMM of B rows: up to TCL_PACK_K columns each CTA quantizes
// (+ LayerNorm) its sequences' rows into shared memory itself; wider rows
// are quantized into the sequence tiles first (tcl_quant_pack_kernel, with
// sx and, for the int8 head, the lane sums of x).
llmq_status batch_linear_tcl(llmq_batch *bt, const llmq_weight *w, const float *x, const float *ln_w,
                             const float *ln_b, const float *bias, float *out, int B, int epi, cudaStream_t s) {
  llmq_ctx *ctx = bt->ctx;
  const WeightView v = w->view();
  const int K = v.cols, mode = v.bits == 4 ? TCL_BLK4 : TCL_CH8;
  const int bpad = (B + TCL_TT - 1) / TCL_TT * TCL_TT;
  TcArgsL a{};
  a.a = w->tcl_a;
  a.res = K <= TCL_PACK_K && K / TC_KB <= TCL_STAGES;
  if (a.res) {
    a.x = x;
    a.ln_w = ln_w;
    a.ln_b = ln_b;
  } else {
    const size_t qsm = (size_t)K * 4;
    if (ln_w)
      tcl_quant_pack_kernel<TCL_TT, PRO_LN><<<bpad, 256, qsm, s>>>(x, ln_w, ln_b, B, bpad, K, mode, bt->tcl_b,
                                                                   bt->sx, bt->xsi);
    else
      tcl_quant_pack_kernel<TCL_TT, PRO_QUANT><<<bpad, 256, qsm, s>>>(x, nullptr, nullptr, B, bpad, K, mode,
                                                                      bt->tcl_b, bt->sx, bt->xsi);
    CKL();
    a.b = bt->tcl_b;
    a.sx = bt->sx;
    a.xsl = bt->xsi;
  }
  a.w = v;
  a.bias = bias;
  a.out = out;
  a.part_val = out ? nullptr : bt->part_val;
  a.part_idx = out ? nullptr : bt->part_idx;
  a.err = ctx->tc_err;
  a.B = B;
  a.OUT = v.rows;
  a.K = K;
  a.nkb = K / TC_KB;
  a.nseg = K / 32;
  a.epi = epi;
  a.ntiles = (v.rows + TC_M - 1) / TC_M;
  a.nparts = 4 * a.ntiles;
  // one CTA per SM: the sequence tiles times as many row-tile columns as
  // fit, each CTA looping over its column's row tiles
  const int stiles = bpad / TCL_TT;
  const dim3 grid(stiles, std::min(a.ntiles, std::max(1, ctx->num_sms / stiles)));
  const size_t sm = sizeof(TcSmemL<TCL_TT>) + 1024;
  if (mode == TCL_BLK4)
    tcl_gemm_kernel<TCL_BLK4, TCL_TT><<<grid, TCL_THREADS, sm, s>>>(a);
  else
    tcl_gemm_kernel<TCL_CH8, TCL_TT><<<grid, TCL_THREADS, sm, s>>>(a);
  CKL();
  return LLMQ_OK;
}

// The lane-mode GEMM's weight tiles of every matrix it takes (the layers'
// and the head), built once per weight.
llmq_status batch_prepare_tcl(llmq_batch *bt) {
  llmq_ctx *ctx = bt->ctx;
  std::vector<const llmq_weight *> ws(bt->m->mats.begin(), bt->m->mats.end());
  ws.push_back(bt->m->head);
  for (const llmq_weight *w : ws) {
    const WeightView v = w->view();
    if (w->tcl_a || w->kind != WK_AFFINE || !w->a16 || !tcl_supported(v)) continue;
    const int nt = (v.rows + TC_M - 1) / TC_M, nkb = v.cols / TC_KB;
    CK(cudaMalloc(&w->tcl_a, (size_t)nt * nkb * TCT_A_BYTES));
    tcl_prep_a_kernel<<<dim3(nt, nkb), 256, 0, ctx->stream>>>(v, v.bits == 4 ? TCL_BLK4 : TCL_CH8, w->tcl_a);
    CKL();
  }
  CK(cudaStreamSynchronize(ctx->stream));
  return LLMQ_OK;
}

// bquant + bgemv for B rows: out[B][rows] (+)= act(quantize(ln?(x)) . w).
llmq_status batch_linear(llmq_batch *bt, const llmq_weight *w, const float *x, const float *ln_w, const float *ln_b,
                         const float *bias, float *out, int B, int epi, cudaStream_t s) {
  if (batch_uses_tcl(bt, w, B)) return batch_linear_tcl(bt, w, x, ln_w, ln_b, bias, out, B, epi, s);
  llmq_ctx *ctx = bt->ctx;
  const WeightView v = w->view();
  const int fmt = fmt_code(w), K = v.cols;
  BQuantArgs q{x, ln_w, ln_b, bt->xq, bt->xsf, bt->xsi, bt->sx, v};
  const size_t qsm = SmemPlan<FMT_BLK4>(K, v.group, 0).total > SmemPlan<FMT_GEN8>(K, v.group, 0).total
                         ? SmemPlan<FMT_BLK4>(K, v.group, 0).total
                         : SmemPlan<FMT_GEN8>(K, v.group, 0).total;
  const bool ln = ln_w != nullptr;
#define BQ(F)                                                                   \
  if (fmt == F) {                                                               \
    if (ln)                                                                     \
      bquant_kernel<F, PRO_LN><<<B, 256, qsm, s>>>(q);                          \
    else                                                                        \
      bquant_kernel<F, PRO_QUANT><<<B, 256, qsm, s>>>(q);                       \
  }
  BQ(FMT_BLK4) else BQ(FMT_GEN4) else BQ(FMT_GEN8)
#undef BQ
  CKL();
  // out == nullptr: the greedy head, whose argmax partials replace the logits
  BGemvArgs g{v, bt->xq, bt->xsf, bt->xsi, bt->sx, bias, out, B, epi, out ? nullptr : bt->part_val,
              out ? nullptr : bt->part_idx, ctx->tc_err};
  const int gx = (v.rows + BG_ROWS - 1) / BG_ROWS;
  // 8 sequences per CTA (registers and shared memory for 2-3 CTAs per SM);
  // the weight rows staged in shared memory where they fit beside the
  // activations
  const int sb = 8;
  const bool stage = bgemv_smem(fmt, K, v.group, sb, true) <= (size_t)kBgemvSmem;
  const size_t sm = bgemv_smem(fmt, K, v.group, sb, stage);
  const dim3 grid(gx, (B + sb - 1) / sb);
  // the row-major kernel for the BLOCKED int4 and per-channel int8 formats
  if (stage && (fmt == FMT_BLK4 || (fmt == FMT_GEN8 && v.group == K && K % 256 == 0))) {
    // two passes of 8 sequences over the staged rows where their activations
    // fit beside them (four passes measured slower: too few CTAs)
    int np = 2;
    while (np > 1 && bgemv_smem(fmt, K, v.group, 8 * np, true) > (size_t)kBgemvSmem) np >>= 1;
    const size_t sm2 = bgemv_smem(fmt, K, v.group, 8 * np, true);
    const dim3 grid2(gx, (B + 8 * np - 1) / (8 * np));
#define BR(F)                                                              \
  if (np == 4)                                                             \
    bgemv_rows_kernel<F, 4><<<grid2, 256, sm2, s>>>(g);                    \
  else if (np == 2)                                                        \
    bgemv_rows_kernel<F, 2><<<grid2, 256, sm2, s>>>(g);                    \
  else                                                                     \
    bgemv_rows_kernel<F, 1><<<grid2, 256, sm2, s>>>(g);
    if (fmt == FMT_BLK4) {
      BR(FMT_BLK4)
    } else {
      BR(FMT_GEN8)
    }
#undef BR
    CKL();
    return LLMQ_OK;
  }
#define BG(F, SB, ST) bgemv_a16_kernel<F, SB, ST><<<grid, 256, sm, s>>>(g)
#define BG2(F)                       \
  if (sb == 16 && stage) BG(F, 16, true); \
  else if (sb == 16) BG(F, 16, false);    \
  else if (stage) BG(F, 8, true);         \
  else BG(F, 8, false);
  if (fmt == FMT_BLK4) {
    BG2(FMT_BLK4)
  } else if (fmt == FMT_GEN4) {
    BG2(FMT_GEN4)
  } else {
    BG2(FMT_GEN8)
  }
#undef BG2
#undef BG
  CKL();
  return LLMQ_OK;
}

// One decode step of B sequences at position state[0], writing ids[b][state[1]]
// and advancing both.
__global__ void batch_advance_kernel(int *state) {
  state[0] += 1;
  state[1] += 1;
}

// cap: the positions the step's attention may see (its shared memory).
llmq_status batch_decode_step(llmq_batch *bt, int B, int cap, cudaStream_t s) {
  llmq_model *m = bt->m;
  llmq_ctx *ctx = bt->ctx;
  embed_batch_kernel<<<B, 256, 0, s>>>(m->head->view(), m->wpe(), bt->x, bt->tokens, bt->state);
  CKL();
  llmq_status st;
  for (int l = 0; l < m->n_layer; l++) {
    const llmq_weight *const *w = &m->mats[4 * l];
    if ((st = batch_linear(bt, w[0], bt->x, m->vec(l, 0), m->vec(l, 1), m->vec(l, 2), bt->qkv, B, EPI_BIAS, s)))
      return st;
    if ((st = kv8_attend(ctx, bt->kv, bt->att, bt->qkv, l, 0, bt->state, 1, cap, dim3(m->n_head, 1, B), s)))
      return st;
    if ((st = batch_linear(bt, w[1], bt->att, nullptr, nullptr, m->vec(l, 3), bt->x, B, EPI_BIAS | EPI_RESID, s)))
      return st;
    if ((st = batch_linear(bt, w[2], bt->x, m->vec(l, 4), m->vec(l, 5), m->vec(l, 6), bt->fc, B, EPI_BIAS | EPI_GELU, s)))
      return st;
    if ((st = batch_linear(bt, w[3], bt->fc, nullptr, nullptr, m->vec(l, 7), bt->x, B, EPI_BIAS | EPI_RESID, s)))
      return st;
  }
  if ((st = batch_linear(bt, m->head, bt->x, m->lnf_w(), m->lnf_b(), nullptr, nullptr, B, 0, s))) return st;
  return LLMQ_OK;
}

__global__ void embed_prompts_kernel(WeightView head, const float *wpe, float *x, const int *tokens, int P) {
  const int r = blockIdx.x, C = head.cols, gpr = head.cols / head.group;
  const int token = min(max(tokens[r], 0), head.rows - 1), p = r % P;  // ids were checked on the host
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    const size_t gi = (size_t)token * gpr + i / head.group;
    const float sc = half_bits_to_float(head.scale[gi]);
    const float v = (float)(code_at(head, token, i) - (int)head.zp[gi]) * sc;
    x[(size_t)r * C + i] = v + wpe[(size_t)p * C + i];
  }
}

__global__ void gather_last_rows_kernel(const float *x, float *dst, int P, int C) {
  const int b = blockIdx.x;
  for (int i = threadIdx.x; i < C; i += blockDim.x) dst[(size_t)b * C + i] = x[((size_t)b * P + P - 1) * C + i];
}

__global__ void batch_init_state_kernel(int *state, int pos, int step) {
  state[0] = pos;
  state[1] = step;
}

// The prompts of B sequences (P tokens each, ids in bt->tokens), all rows at
// once through the several-token path; the last row of each through the
// one-token head; ids[b][0] and tokens[b] from its argmax.
llmq_status batch_prompt(llmq_batch *bt, int B, int P, cudaStream_t s) {
  llmq_model *m = bt->m;
  llmq_ctx *ctx = bt->ctx;
  const int C = m->C, T = B * P;
  embed_prompts_kernel<<<T, 256, 0, s>>>(m->head->view(), m->wpe(), bt->x, bt->tokens, P);
  CKL();
  llmq_status st;
  for (int l = 0; l < m->n_layer; l++) {
    const llmq_weight *const *w = &m->mats[4 * l];
    launch_layernorm(bt->xn, bt->x, m->vec(l, 0), m->vec(l, 1), T, C, s);
    CKL();
    if ((st = llmq_linear(ctx, w[0], bt->xn, m->vec(l, 2), bt->qkv, T, C, 3 * C, LLMQ_BIAS)) != LLMQ_OK) return st;
    kv8_store_kernel<<<(m->n_head * P * 2 * B + 7) / 8, 256, 0, s>>>(bt->kv, bt->qkv, l, 0, nullptr, P, B);
    CKL();
    const size_t sm = kv8_prefill_smem(P, C / m->n_head);
    kv_prefill_kernel<0><<<dim3(m->n_head, (P + KV_QB - 1) / KV_QB, B), 256, sm, s>>>(bt->kv, bt->att, bt->qkv, l, 0, P);
    CKL();
    if ((st = llmq_linear(ctx, w[1], bt->att, m->vec(l, 3), bt->x, T, C, C, LLMQ_BIAS | LLMQ_RESID)) != LLMQ_OK)
      return st;
    launch_layernorm(bt->xn, bt->x, m->vec(l, 4), m->vec(l, 5), T, C, s);
    CKL();
    if ((st = llmq_linear(ctx, w[2], bt->xn, m->vec(l, 6), bt->fc, T, C, 4 * C, LLMQ_BIAS | LLMQ_GELU)) != LLMQ_OK)
      return st;
    if ((st = llmq_linear(ctx, w[3], bt->fc, m->vec(l, 7), bt->x, T, 4 * C, C, LLMQ_BIAS | LLMQ_RESID)) != LLMQ_OK)
      return st;
  }
  gather_last_rows_kernel<<<B, 256, 0, s>>>(bt->x, bt->xn, P, C);
  CKL();
  if ((st = batch_linear(bt, m->head, bt->xn, m->lnf_w(), m->lnf_b(), nullptr, nullptr, B, 0, s))) return st;
  return LLMQ_OK;
}

// generate for B sequences whose prompts are in bt->tokens ([B][P]): ids
// into bt->ids ([B][max_t], columns 0..steps-1), and also into ids_dev
// ([B][steps]) when given.
llmq_status batch_run(llmq_batch *bt, int B, int P, int steps, int *ids_dev) {
  llmq_ctx *ctx = bt->ctx;
  llmq_model *m = bt->m;
  cudaStream_t s = ctx->stream;
  llmq_status st = batch_prompt(bt, B, P, s);
  if (st != LLMQ_OK) return st;
  ctx->tc_used = true;  // the GEMVs' copy waits report through the same flag
  // decode step i (1..steps-1) embeds the token of column i-1 at position P+i-1
  batch_init_state_kernel<<<1, 1, 0, s>>>(bt->state, P - 1, 0);
  CKL();
  const int nparts = batch_head_parts(bt, B);
  argmax_parts_kernel<<<B, 256, 0, s>>>(bt->part_val, bt->part_idx, nparts, bt->ids, m->max_t, bt->tokens, nullptr);
  CKL();
  if (steps > 1) {
    // decode steps as one CUDA graph, captured for this batch size, kernel
    // choice and attention context: the last step's queries see P + steps - 1
    // positions; the shared memory is sized for that, rounded up to 64
    const int cap = std::min(m->max_t, (P + steps - 1 + 63) / 64 * 64);
    if (!bt->exec || bt->graph_B != B || bt->graph_kernel != bt->kernel || bt->graph_cap != cap) {
      if (bt->exec) cudaGraphExecDestroy(bt->exec);
      if (bt->graph) cudaGraphDestroy(bt->graph);
      bt->exec = nullptr;
      bt->graph = nullptr;
      CK(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
      batch_advance_kernel<<<1, 1, 0, s>>>(bt->state);
      llmq_status cst = batch_decode_step(bt, B, cap, s);
      if (cst == LLMQ_OK)
        argmax_parts_kernel<<<B, 256, 0, s>>>(bt->part_val, bt->part_idx, nparts, bt->ids, m->max_t, bt->tokens,
                                              bt->state + 1);
      cudaGraph_t g = nullptr;
      cudaError_t e = cudaStreamEndCapture(s, &g);
      if (cst != LLMQ_OK) {
        if (g) cudaGraphDestroy(g);
        return cst;
      }
      CK(e);
      bt->graph = g;
      CK(cudaGraphInstantiate(&bt->exec, g, 0));
      bt->graph_B = B;
      bt->graph_kernel = bt->kernel;
      bt->graph_cap = cap;
    }
    for (int i = 1; i < steps; i++) CK(cudaGraphLaunch(bt->exec, s));
  }
  if (ids_dev)
    CK(cudaMemcpy2DAsync(ids_dev, (size_t)steps * 4, bt->ids, (size_t)m->max_t * 4, (size_t)steps * 4, B,
                         cudaMemcpyDeviceToDevice, s));
  return LLMQ_OK;
}

}  // namespace

extern "C" {

llmq_status llmq_batch_create(llmq_ctx *ctx, llmq_model *m, int max_seqs, int max_prompt, llmq_batch **out) {
  if (m && m->float_only)
    return fail(ctx, LLMQ_ERR_UNSUPPORTED, "batched decode runs the A16 formats");
  if (!ctx || !m || !out || max_seqs <= 0 || max_prompt <= 0 || max_prompt > m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad batch arguments");
  if (m->kv->kind != LLMQ_KV_QUANT8) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "batched decode takes the QuantKV[8] cache");
  *out = nullptr;
  CK(cudaSetDevice(ctx->device));
  llmq_batch *bt = new llmq_batch();
  bt->ctx = ctx;
  bt->m = m;
  bt->max_seqs = max_seqs;
  bt->max_prompt = max_prompt;
  const int C = m->C, HS = C / m->n_head;
  const size_t seq = (size_t)m->n_layer * m->max_t * m->n_head * HS, rows = (size_t)max_seqs * max_prompt;
  KV8View &v = bt->kv;
  v.n_layer = m->n_layer;
  v.max_t = m->max_t;
  v.n_head = m->n_head;
  v.head_dim = HS;
  v.seq = seq;
  int maxu = 0;
  for (const llmq_weight *w : m->mats) maxu = std::max(maxu, w->cols / w->group);
  maxu = std::max(maxu, m->head->cols / m->head->group);
  cudaError_t e = cudaMalloc(&v.k, seq * max_seqs);
  if (e == cudaSuccess) e = cudaMalloc(&v.v, seq * max_seqs);
  if (e == cudaSuccess) e = cudaMalloc(&v.ks, seq / HS * max_seqs * 4);
  if (e == cudaSuccess) e = cudaMalloc(&v.vs, seq / HS * max_seqs * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->x, rows * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->xn, rows * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->qkv, rows * 3 * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->att, rows * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->fc, rows * 4 * C * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->logits, (size_t)max_seqs * m->V * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->xq, (size_t)max_seqs * 4 * C * 2);
  if (e == cudaSuccess) e = cudaMalloc(&bt->xsf, (size_t)max_seqs * 4 * C / 16 * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->xsi, (size_t)max_seqs * maxu * 16 * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->sx, (size_t)max_seqs * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->tokens, rows * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->ids, (size_t)max_seqs * m->max_t * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->state, 2 * sizeof(int));
  // argmax partials per sequence: the CUDA-core head's row tiles or the
  // lane-mode GEMM's four lane quarters per row tile
  const size_t nparts = std::max((size_t)(m->V + BG_ROWS - 1) / BG_ROWS, (size_t)4 * ((m->V + TC_M - 1) / TC_M));
  if (e == cudaSuccess) e = cudaMalloc(&bt->part_val, (size_t)max_seqs * nparts * 4);
  if (e == cudaSuccess) e = cudaMalloc(&bt->part_idx, (size_t)max_seqs * nparts * 4);
  if (e == cudaSuccess) e = cudaMemset(v.k, 0, seq * max_seqs);
  if (e == cudaSuccess) e = cudaMemset(v.v, 0, seq * max_seqs);
  if (e == cudaSuccess) e = cudaMemset(v.ks, 0, seq / HS * max_seqs * 4);
  if (e == cudaSuccess) e = cudaMemset(v.vs, 0, seq / HS * max_seqs * 4);
  if (e == cudaSuccess) e = cudaMallocHost(&bt->ids_host, (size_t)max_seqs * m->max_t * 4);
  if (e == cudaSuccess) e = cudaMallocHost(&bt->prompt_host, rows * 4);
  const int tcl_seqs = (max_seqs + TCL_TT - 1) / TCL_TT * TCL_TT;
  if (e == cudaSuccess) e = cudaMalloc(&bt->tcl_b, (size_t)tcl_seqs * 4 * C * 4);
  if (e != cudaSuccess) {
    llmq_batch_free(bt);
    return fail(ctx, LLMQ_ERR_NOMEM, std::string("batch alloc: ") + cudaGetErrorString(e));
  }
  // the bgemv and several-token attention kernels' shared memory
  auto attr = [&](const void *k, size_t n) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)n);
  };
#define BA(F)                                                           \
  attr((const void *)bgemv_a16_kernel<F, 16, true>, kBgemvSmem);        \
  attr((const void *)bgemv_a16_kernel<F, 16, false>, kBgemvSmem);       \
  attr((const void *)bgemv_a16_kernel<F, 8, true>, kBgemvSmem);         \
  attr((const void *)bgemv_a16_kernel<F, 8, false>, kBgemvSmem);
  BA(FMT_BLK4)
  BA(FMT_GEN4)
  BA(FMT_GEN8)
#undef BA
  for (const void *k : {(const void *)bgemv_rows_kernel<FMT_BLK4, 1>, (const void *)bgemv_rows_kernel<FMT_BLK4, 2>,
                        (const void *)bgemv_rows_kernel<FMT_BLK4, 4>, (const void *)bgemv_rows_kernel<FMT_GEN8, 1>,
                        (const void *)bgemv_rows_kernel<FMT_GEN8, 2>, (const void *)bgemv_rows_kernel<FMT_GEN8, 4>})
    attr(k, kBgemvSmem);
  attr((const void *)tcl_gemm_kernel<TCL_BLK4, TCL_TT>, sizeof(TcSmemL<TCL_TT>) + 1024);
  attr((const void *)tcl_gemm_kernel<TCL_CH8, TCL_TT>, sizeof(TcSmemL<TCL_TT>) + 1024);
  attr((const void *)tcl_quant_pack_kernel<TCL_TT, PRO_LN>, 4096 * 4);
  attr((const void *)tcl_quant_pack_kernel<TCL_TT, PRO_QUANT>, 4096 * 4);
  if (e != cudaSuccess) {
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, ctx->device);
    llmq_batch_free(bt);
    return fail(ctx, LLMQ_ERR_CUDA, std::string("batch attributes: ") + cudaGetErrorString(e) +
                                        " (shared memory per block up to " + std::to_string(optin) + ")");
  }
  llmq_status pst = batch_prepare_tcl(bt);
  if (pst != LLMQ_OK) {
    llmq_batch_free(bt);
    return pst;
  }
  *out = bt;
  return LLMQ_OK;
}

llmq_status llmq_batch_set_kernel(llmq_batch *bt, int kind) {
  if (!bt || kind < LLMQ_BATCH_AUTO || kind > LLMQ_BATCH_TCGEN05) return LLMQ_ERR_INVALID;
  bt->kernel = kind;
  return LLMQ_OK;
}

llmq_status llmq_batch_free(llmq_batch *bt) {
  if (!bt) return LLMQ_ERR_INVALID;
  cudaSetDevice(bt->ctx->device);
  if (bt->exec) cudaGraphExecDestroy(bt->exec);
  if (bt->graph) cudaGraphDestroy(bt->graph);
  void *ps[] = {bt->kv.k, bt->kv.v, bt->kv.ks, bt->kv.vs, bt->x, bt->xn, bt->qkv, bt->att, bt->fc, bt->logits,
                bt->xq, bt->xsf, bt->xsi, bt->sx, bt->tokens, bt->ids, bt->state, bt->part_val, bt->part_idx,
                bt->tcl_b};
  for (void *p : ps)
    if (p) cudaFree(p);
  if (bt->ids_host) cudaFreeHost(bt->ids_host);
  if (bt->prompt_host) cudaFreeHost(bt->prompt_host);
  delete bt;
  return LLMQ_OK;
}

llmq_status llmq_batch_generate_async(llmq_ctx *ctx, llmq_batch *bt, const int *prompts_dev, int B, int n_prompt,
                                      int steps, int *ids_dev) {
  if (!ctx || !bt || !prompts_dev || !ids_dev || B <= 0 || B > bt->max_seqs || n_prompt <= 0 ||
      n_prompt > bt->max_prompt || steps <= 0 || n_prompt + steps - 1 > bt->m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad batch size, prompt length or steps");
  CK(cudaSetDevice(ctx->device));
  CK(cudaMemcpyAsync(bt->tokens, prompts_dev, (size_t)B * n_prompt * 4, cudaMemcpyDeviceToDevice, ctx->stream));
  return batch_run(bt, B, n_prompt, steps, ids_dev);
}

llmq_status llmq_batch_generate(llmq_ctx *ctx, llmq_batch *bt, const int *prompts, int B, int n_prompt, int steps,
                                int *out_ids) {
  if (!ctx || !bt || !prompts || !out_ids || B <= 0 || B > bt->max_seqs || n_prompt <= 0 ||
      n_prompt > bt->max_prompt || steps <= 0 || n_prompt + steps - 1 > bt->m->max_t)
    return fail(ctx, LLMQ_ERR_INVALID, "bad batch size, prompt length or steps");
  for (long i = 0; i < (long)B * n_prompt; i++)
    if (prompts[i] < 0 || prompts[i] >= bt->m->V) return fail(ctx, LLMQ_ERR_INVALID, "token id out of range");
  CK(cudaSetDevice(ctx->device));
  cudaStream_t s = ctx->stream;
  CK(cudaStreamSynchronize(s));
  std::memcpy(bt->prompt_host, prompts, (size_t)B * n_prompt * 4);
  CK(cudaMemcpyAsync(bt->tokens, bt->prompt_host, (size_t)B * n_prompt * 4, cudaMemcpyHostToDevice, s));
  llmq_status st = batch_run(bt, B, n_prompt, steps, nullptr);
  if (st != LLMQ_OK) return st;
  CK(cudaMemcpy2DAsync(bt->ids_host, (size_t)steps * 4, bt->ids, (size_t)bt->m->max_t * 4, (size_t)steps * 4, B,
                       cudaMemcpyDeviceToHost, s));
  CK(cudaStreamSynchronize(s));
  if ((st = tc_check(ctx)) != LLMQ_OK) return st;
  std::memcpy(out_ids, bt->ids_host, (size_t)B * steps * 4);
  return LLMQ_OK;
}

}  // extern "C"

extern "C" {

llmq_status llmq_score_rows(llmq_ctx *ctx, const float *logits_dev, const float *base_dev, const int *targets_dev, int V,
                            int r0, int r1, double *stats_dev, int stride) {
  if (!ctx || !logits_dev || !targets_dev || !stats_dev || V <= 0 || r0 < 0 || r1 < r0 || stride < r1 - r0)
    return fail(ctx, LLMQ_ERR_INVALID, "bad score arguments");
  if (r1 == r0) return LLMQ_OK;
  CK(cudaSetDevice(ctx->device));
  score_rows_kernel<<<r1 - r0, 256, 0, ctx->stream>>>(logits_dev, base_dev, targets_dev, V, r0, stats_dev, stride);
  CKL();
  return LLMQ_OK;
}

}  // extern "C"

// ---- saved weights (.llmm) and GGUF files --------------------------------

namespace {

const char kSavedMagic[] = "llm_mojo GPT-2 124M weights";  // gpt2t.mojo:621
constexpr long long kSavedVersion = 1;
constexpr int kSavedLayers = 12;  // the reference's N_LAYER

// The reference's --dtype names of the affine formats (gpt2t.mojo:1313-1346,
// QuantMatrix.name at tensor.mojo:325-331): int{4,8}-{ch,g32,g64,g128}
// [-sym][-a16]. group 0 = per channel.
bool parse_affine_name(const std::string &n, int &bits, int &group, int &sym, int &a16) {
  size_t p = 0;
  auto next = [&](std::string &tok) {
    if (p > n.size()) return false;
    size_t q = n.find('-', p);
    tok = n.substr(p, q == std::string::npos ? std::string::npos : q - p);
    p = q == std::string::npos ? n.size() + 1 : q + 1;
    return true;
  };
  std::string t;
  if (!next(t) || (t != "int4" && t != "int8")) return false;
  bits = t == "int4" ? 4 : 8;
  if (!next(t)) return false;
  if (t == "ch")
    group = 0;
  else if (t == "g32" || t == "g64" || t == "g128")
    group = std::stoi(t.substr(1));
  else
    return false;
  sym = a16 = 0;
  while (p <= n.size() && next(t)) {
    if (t == "sym")
      sym = 1;
    else if (t == "a16")
      a16 = 1;
    else
      return false;
  }
  return true;
}

std::string affine_name(const llmq_weight *w) {
  std::string n = std::string(w->bits == 4 ? "int4" : "int8") + "-" +
                  (w->group == w->cols ? std::string("ch") : "g" + std::to_string(w->group));
  if (w->sym) n += "-sym";
  if (w->a16) n += "-a16";
  return n;
}

int dense_code(const std::string &n) { return n == "f32" ? LLMQ_DENSE_F32 : n == "f16" ? LLMQ_DENSE_F16 : n == "bf16" ? LLMQ_DENSE_BF16 : -1; }

struct ByteOut {
  FILE *f;
  bool ok = true;
  void bytes(const void *p, size_t n) { ok = ok && (n == 0 || fwrite(p, 1, n, f) == n); }
  void i64(long long v) {
    unsigned char b[8];
    for (int i = 0; i < 8; i++) b[i] = (unsigned char)((unsigned long long)v >> (8 * i));
    bytes(b, 8);
  }
  void str(const std::string &s) {
    i64((long long)s.size());
    bytes(s.data(), s.size());
  }
};

struct ByteIn {
  FILE *f;
  bool ok = true;
  void bytes(void *p, size_t n) { ok = ok && (n == 0 || fread(p, 1, n, f) == n); }
  long long i64() {
    unsigned char b[8] = {0};
    bytes(b, 8);
    unsigned long long v = 0;
    for (int i = 0; i < 8; i++) v |= (unsigned long long)b[i] << (8 * i);
    return (long long)v;
  }
  std::string str() {
    long long n = i64();
    if (!ok || n < 0 || n > (1 << 20)) {
      ok = false;
      return "";
    }
    std::string s((size_t)n, '\0');
    bytes(&s[0], (size_t)n);
    return s;
  }
};

// WeightMatrix.save (tensor.mojo:634-643 affine, :215-218 dense) of one device weight.
llmq_status save_weight(llmq_ctx *ctx, ByteOut &o, const llmq_weight *w) {
  if (w->kind == WK_AFFINE) {
    const size_t nc = (size_t)w->rows * w->cols * w->bits / 8, ng = (size_t)w->rows * (w->cols / w->group);
    std::vector<uint8_t> codes(nc), zp(ng);
    std::vector<uint16_t> scale(ng);
    CK(cudaMemcpy(codes.data(), w->codes, nc, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(scale.data(), w->scale, ng * 2, cudaMemcpyDeviceToHost));
    CK(cudaMemcpy(zp.data(), w->zp, ng, cudaMemcpyDeviceToHost));
    o.i64(w->rows);
    o.i64(w->cols);
    o.i64(w->group);
    o.bytes(codes.data(), nc);
    o.bytes(scale.data(), ng * 2);
    o.bytes(zp.data(), ng);
  } else if (w->kind == WK_DENSE) {
    const size_t n = (size_t)w->rows * w->row_bytes;
    std::vector<uint8_t> data(n);
    CK(cudaMemcpy(data.data(), w->codes, n, cudaMemcpyDeviceToHost));
    o.i64(w->rows);
    o.i64(w->cols);
    o.bytes(data.data(), n);
  } else {
    return fail(ctx, LLMQ_ERR_UNSUPPORTED, "GGUF matrices are saved as GGUF files already");
  }
  return LLMQ_OK;
}

// WeightMatrix.restore of the format called `name`, created on the device.
llmq_status restore_weight(llmq_ctx *ctx, ByteIn &in, const std::string &name, llmq_weight **out) {
  int bits, group, sym, a16;
  const long long rows = in.i64(), cols = in.i64();
  if (!in.ok || rows <= 0 || cols <= 0 || rows > (1 << 24) || cols > (1 << 24))
    return fail(ctx, LLMQ_ERR_INVALID, "bad matrix shape in saved file");
  if (parse_affine_name(name, bits, group, sym, a16)) {
    const long long g = in.i64();
    if (!in.ok || g != (group == 0 ? cols : group)) return fail(ctx, LLMQ_ERR_INVALID, "group size does not match " + name);
    const size_t nc = (size_t)rows * cols * bits / 8, ng = (size_t)rows * (cols / g);
    std::vector<uint8_t> codes(nc), zp(ng);
    std::vector<uint16_t> scale(ng);
    in.bytes(codes.data(), nc);
    in.bytes(scale.data(), ng * 2);
    in.bytes(zp.data(), ng);
    if (!in.ok) return fail(ctx, LLMQ_ERR_INVALID, "unexpected end of saved file");
    return llmq_weight_create_affine(ctx, bits, group, sym, a16, (int)rows, (int)cols, codes.data(), scale.data(),
                                     zp.data(), out);
  }
  const int dt = dense_code(name);
  if (dt < 0) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "unknown saved format " + name);
  const size_t n = (size_t)rows * cols * (dt == LLMQ_DENSE_F32 ? 4 : 2);
  std::vector<uint8_t> data(n);
  in.bytes(data.data(), n);
  if (!in.ok) return fail(ctx, LLMQ_ERR_INVALID, "unexpected end of saved file");
  return llmq_weight_create_dense(ctx, dt, data.data(), (int)rows, (int)cols, out);
}

std::string weight_name(const llmq_weight *w) {
  if (w->kind == WK_AFFINE) return affine_name(w);
  if (w->kind == WK_DENSE) return w->rtype == RT_F32 ? "f32" : w->rtype == RT_F16 ? "f16" : "bf16";
  return "gguf";
}

// The GGUF file (gguf.mojo:519-636): header, metadata (skipped but for
// general.alignment), tensor index, data section.
struct GgufTensor {
  int type;
  long long cols, rows, offset;
};

struct GgufFile {
  std::vector<uint8_t> buf;
  size_t data_start = 0;
  std::map<std::string, GgufTensor> tensors;
  std::string err;

  uint32_t u32(size_t p) const { uint32_t v; std::memcpy(&v, &buf[p], 4); return v; }
  uint64_t u64(size_t p) const { uint64_t v; std::memcpy(&v, &buf[p], 8); return v; }
  bool has(size_t p, size_t n) const { return p <= buf.size() && n <= buf.size() - p; }

  bool skip_value(uint32_t vt, size_t &p, int depth) {
    static const int sizes[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (depth > 4 || vt > 12) return false;
    if (vt == 8) {  // string
      if (!has(p, 8)) return false;
      const uint64_t n = u64(p);
      if (!has(p + 8, n)) return false;
      p += 8 + n;
      return true;
    }
    if (vt == 9) {  // array: element type, count, elements
      if (!has(p, 12)) return false;
      const uint32_t et = u32(p);
      const uint64_t count = u64(p + 4);
      p += 12;
      for (uint64_t i = 0; i < count; i++)
        if (!skip_value(et, p, depth + 1)) return false;
      return true;
    }
    if (!has(p, sizes[vt])) return false;
    p += sizes[vt];
    return true;
  }

  bool read(const char *path) {
    FILE *f = fopen(path, "rb");
    if (!f) return err = std::string("cannot open ") + path, false;
    fseek(f, 0, SEEK_END);
    const long size = ftell(f);
    fseek(f, 0, SEEK_SET);
    buf.resize(size > 0 ? (size_t)size : 0);
    const bool got = size > 0 && fread(buf.data(), 1, buf.size(), f) == buf.size();
    fclose(f);
    if (!got || !has(0, 24)) return err = "short read", false;
    if (u32(0) != 0x46554747u) return err = std::string(path) + " is not a GGUF file", false;
    if (u32(4) < 2) return err = "GGUF version below 2", false;
    const uint64_t n_tensors = u64(8), n_kv = u64(16);
    size_t p = 24;
    uint64_t alignment = 32;
    for (uint64_t i = 0; i < n_kv; i++) {
      if (!has(p, 8)) return err = "truncated metadata", false;
      const uint64_t kn = u64(p);
      if (!has(p + 8, kn + 4)) return err = "truncated metadata", false;
      const std::string key((const char *)&buf[p + 8], kn);
      p += 8 + kn;
      const uint32_t vt = u32(p);
      p += 4;
      if (key == "general.alignment" && vt == 4 && has(p, 4)) alignment = u32(p);
      if (!skip_value(vt, p, 0)) return err = "bad metadata value", false;
    }
    for (uint64_t i = 0; i < n_tensors; i++) {
      if (!has(p, 8)) return err = "truncated tensor index", false;
      const uint64_t nn = u64(p);
      if (!has(p + 8, nn + 4)) return err = "truncated tensor index", false;
      const std::string name((const char *)&buf[p + 8], nn);
      p += 8 + nn;
      const uint32_t nd = u32(p);
      p += 4;
      if (nd < 1 || nd > 4 || !has(p, 8 * nd + 12)) return err = "bad tensor dims", false;
      long long cols = (long long)u64(p), rows = 1;
      for (uint32_t d = 1; d < nd; d++) rows *= (long long)u64(p + 8 * d);
      p += 8 * nd;
      tensors[name] = GgufTensor{(int)u32(p), cols, rows, (long long)u64(p + 4)};
      p += 12;
    }
    if (alignment == 0) alignment = 32;
    data_start = (p + alignment - 1) / alignment * alignment;
    return true;
  }

  // bytes of tensor t, or nullptr when it lies outside the file
  const uint8_t *data(const GgufTensor &t, size_t bytes) const {
    const size_t off = data_start + (size_t)t.offset;
    return has(off, bytes) ? &buf[off] : nullptr;
  }
};

size_t gguf_tensor_bytes(const GgufTensor &t) {
  const int bs = rt_block_size(t.type), bb = rt_block_bytes(t.type);
  if (bs <= 0 || bb <= 0 || t.cols % bs) return 0;
  return (size_t)t.rows * (size_t)(t.cols / bs) * bb;
}

}  // namespace

extern "C" {

llmq_status llmq_model_save(llmq_ctx *ctx, const llmq_model *m, const char *path) {
  if (!ctx || !m || !path) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  if (m->n_layer != kSavedLayers) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "saved models have 12 layers");
  if (m->embed) return fail(ctx, LLMQ_ERR_UNSUPPORTED, "the saved format holds one tied embedding / head matrix");
  CK(cudaSetDevice(ctx->device));
  CK(cudaStreamSynchronize(ctx->stream));
  FILE *f = fopen(path, "wb");
  if (!f) return fail(ctx, LLMQ_ERR_INVALID, std::string("cannot write ") + path);
  ByteOut o{f};
  o.str(kSavedMagic);
  o.i64(kSavedVersion);
  o.str(weight_name(m->mats[0]));
  o.str(weight_name(m->head));
  llmq_status st = save_weight(ctx, o, m->head);
  for (size_t i = 0; st == LLMQ_OK && i < m->mats.size(); i++) st = save_weight(ctx, o, m->mats[i]);
  if (st == LLMQ_OK) {
    const size_t n = (size_t)m->n_layer * 13 * m->C + (size_t)1024 * m->C + 2 * m->C;
    std::vector<float> small(n);
    cudaError_t e = cudaMemcpy(small.data(), m->small, n * 4, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) st = fail(ctx, LLMQ_ERR_CUDA, cudaGetErrorString(e));
    o.i64((long long)n);
    o.bytes(small.data(), n * 4);
  }
  if (fclose(f) != 0) o.ok = false;
  if (st == LLMQ_OK && !o.ok) st = fail(ctx, LLMQ_ERR_INVALID, std::string("write to ") + path + " failed");
  return st;
}

llmq_status llmq_model_load(llmq_ctx *ctx, const char *path, int kv_kind, int max_t, llmq_model **out) {
  if (!ctx || !path || !out) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  *out = nullptr;
  FILE *f = fopen(path, "rb");
  if (!f) return fail(ctx, LLMQ_ERR_INVALID, std::string("cannot open ") + path);
  ByteIn in{f};
  std::vector<llmq_weight *> ws;
  auto cleanup = [&](llmq_status st) {
    fclose(f);
    for (llmq_weight *w : ws) llmq_weight_free(w);
    return st;
  };
  const std::string magic = in.str();
  if (!in.ok || magic != kSavedMagic) return cleanup(fail(ctx, LLMQ_ERR_INVALID, std::string(path) + " is not a saved llm_mojo model"));
  if (in.i64() != kSavedVersion) return cleanup(fail(ctx, LLMQ_ERR_UNSUPPORTED, "unsupported saved-model version"));
  const std::string wname = in.str(), hname = in.str();
  if (!in.ok) return cleanup(fail(ctx, LLMQ_ERR_INVALID, "truncated header"));
  llmq_weight *w = nullptr;
  llmq_status st = restore_weight(ctx, in, hname, &w);
  if (st != LLMQ_OK) return cleanup(st);
  ws.push_back(w);
  for (int i = 0; i < 4 * kSavedLayers; i++) {
    if ((st = restore_weight(ctx, in, wname, &w)) != LLMQ_OK) return cleanup(st);
    ws.push_back(w);
  }
  const long long n = in.i64();
  const long long want = (long long)kSavedLayers * 13 * 768 + 1024LL * 768 + 2 * 768;
  if (!in.ok || n != want) return cleanup(fail(ctx, LLMQ_ERR_INVALID, "unexpected size of the float32 tensors"));
  std::vector<float> small((size_t)n);
  in.bytes(small.data(), (size_t)n * 4);
  if (!in.ok) return cleanup(fail(ctx, LLMQ_ERR_INVALID, "unexpected end of saved file"));
  llmq_model *m = nullptr;
  if ((st = llmq_model_create(ctx, kSavedLayers, ws.data() + 1, ws[0], small.data(), kv_kind, max_t, &m)) != LLMQ_OK)
    return cleanup(st);
  fclose(f);
  m->owned = ws;
  *out = m;
  return LLMQ_OK;
}

llmq_status llmq_model_load_gguf(llmq_ctx *ctx, const char *path, int kv_kind, int max_t, llmq_model **out) {
  if (!ctx || !path || !out) return fail(ctx, LLMQ_ERR_INVALID, "null argument");
  *out = nullptr;
  GgufFile g;
  if (!g.read(path)) return fail(ctx, LLMQ_ERR_INVALID, g.err);
  std::vector<llmq_weight *> ws;
  auto cleanup = [&](llmq_status st) {
    for (llmq_weight *w : ws) llmq_weight_free(w);
    return st;
  };
  auto matrix = [&](const std::string &name, long long rows, long long cols, llmq_weight **w) -> llmq_status {
    auto it = g.tensors.find(name);
    if (it == g.tensors.end()) return fail(ctx, LLMQ_ERR_INVALID, "tensor not in GGUF file: " + name);
    const GgufTensor &t = it->second;
    if (t.rows != rows || t.cols != cols) return fail(ctx, LLMQ_ERR_INVALID, name + " has an unexpected shape");
    const size_t bytes = gguf_tensor_bytes(t);
    const uint8_t *d = bytes ? g.data(t, bytes) : nullptr;
    if (!d) return fail(ctx, LLMQ_ERR_UNSUPPORTED, name + ": unsupported format or outside the file");
    return llmq_weight_create_gguf(ctx, t.type, d, (int)rows, (int)cols, w);
  };
  auto f32 = [&](const std::string &name, size_t n, float *dst) -> llmq_status {
    auto it = g.tensors.find(name);
    if (it == g.tensors.end()) return fail(ctx, LLMQ_ERR_INVALID, "tensor not in GGUF file: " + name);
    const GgufTensor &t = it->second;
    const uint8_t *d = g.data(t, n * 4);
    if (t.type != RT_F32 || (size_t)(t.rows * t.cols) != n || !d)
      return fail(ctx, LLMQ_ERR_INVALID, name + " is not the expected float32 tensor");
    std::memcpy(dst, d, n * 4);
    return LLMQ_OK;
  };
  const int C = 768, L = 12;
  static const char *mat_names[4] = {"attn_qkv.weight", "attn_output.weight", "ffn_up.weight", "ffn_down.weight"};
  static const char *vec_names[8] = {"attn_norm.weight", "attn_norm.bias", "attn_qkv.bias", "attn_output.bias",
                                     "ffn_norm.weight", "ffn_norm.bias", "ffn_up.bias", "ffn_down.bias"};
  static const int vec_lens[8] = {1, 1, 3, 1, 1, 1, 4, 1};
  static const long long outs[4] = {3 * C, C, 4 * C, C}, ins[4] = {C, C, C, 4 * C};
  // ws[0] the head (output.weight, else the tied token_embd.weight), ws[1..48]
  // the layer matrices, ws[49] token_embd.weight when the head is untied
  const bool tied = g.tensors.count("output.weight") == 0;
  llmq_weight *w = nullptr;
  llmq_status st = matrix(tied ? "token_embd.weight" : "output.weight", 50257, C, &w);
  if (st != LLMQ_OK) return cleanup(st);
  ws.push_back(w);
  std::vector<float> small((size_t)L * 13 * C + 1024 * C + 2 * C);
  size_t off = 0;
  for (int l = 0; l < L; l++) {
    const std::string pre = "blk." + std::to_string(l) + ".";
    for (int i = 0; i < 4; i++) {
      if ((st = matrix(pre + mat_names[i], outs[i], ins[i], &w)) != LLMQ_OK) return cleanup(st);
      ws.push_back(w);
    }
    for (int i = 0; i < 8; i++) {
      if ((st = f32(pre + vec_names[i], (size_t)vec_lens[i] * C, small.data() + off)) != LLMQ_OK) return cleanup(st);
      off += (size_t)vec_lens[i] * C;
    }
  }
  if ((st = f32("position_embd.weight", (size_t)1024 * C, small.data() + off)) != LLMQ_OK) return cleanup(st);
  off += (size_t)1024 * C;
  if ((st = f32("output_norm.weight", C, small.data() + off)) != LLMQ_OK) return cleanup(st);
  if ((st = f32("output_norm.bias", C, small.data() + off + C)) != LLMQ_OK) return cleanup(st);
  if (!tied) {
    if ((st = matrix("token_embd.weight", 50257, C, &w)) != LLMQ_OK) return cleanup(st);
    ws.push_back(w);
  }
  llmq_model *m = nullptr;
  if ((st = llmq_model_create(ctx, L, ws.data() + 1, ws[0], small.data(), kv_kind, max_t, &m)) != LLMQ_OK)
    return cleanup(st);
  if (!tied) m->embed = ws.back();
  m->owned = ws;
  *out = m;
  return LLMQ_OK;
}

}  // extern "C"

