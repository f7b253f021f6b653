// Persistent decode kernel: a whole greedy generation (many tokens) in one
// cooperative launch on sm_100a, one CTA per SM.
//
// Why: a decode step is ~60 dependent operations (per layer: LayerNorm +
// QKV GEMV, KV store + attention, PROJ GEMV, LayerNorm + FC GEMV, FCPROJ
// GEMV; then LN_f + head GEMV + argmax), each of which needs the whole
// previous activation vector (LayerNorm and the int16 quantization of every
// matmul input take a max or sums over all of it). Launched one by one, each
// costs a launch and a cold start; here every CTA stays resident and
//   - streams its own slice of every weight matrix, in the order it will use
//     them, from a per-CTA packed copy in HBM into a shared-memory ring with
//     cp.async.bulk (mbarrier completion): the thread that releases a slot
//     issues the copy of the chunk MK_NSLOT ahead into it, so the ring runs
//     ahead of the computation across layers and tokens and weights never sit
//     on the critical path;
//   - exchanges activations through global buffers of 8-byte words that
//     hold a float and a 32-bit flag (the step's sequence number): a writer
//     publishes a value and its flag with one single-copy-atomic store, and a
//     reader spins on the words it needs until their flags match. This is
//     both the data transfer and the synchronisation; there is no separate
//     grid barrier.
// Every spin (ring slots, flags) is bounded by a cycle budget; on timeout
// the kernel records an error code, waits (bounded) for its own copies in
// flight, and returns.
//
// The phase helpers are deliberately not inlined: one copy of each keeps
// the kernel's code small enough to stay in the SMs' instruction caches
// while it loops over layers and tokens.
//
// The arithmetic of each phase is that of the one-token kernels
// (gemv_a16.cuh, attention.cuh): bit-identical to the reference's.
#pragma once

#include "attention.cuh"
#include "gemv_a16.cuh"
#include "gemv_float.cuh"

namespace llmq {

constexpr int MK_THREADS = 256;
constexpr int MK_NSLOT = 7;
constexpr int MK_SLOT = 18512;     // bytes per ring slot: one chunk (largest: 24 head rows)
constexpr int MK_HEAD_TILE = 24;
constexpr int MK_KV_STAGE = 256;   // cache positions an attention CTA stages in shared memory
constexpr int MK_LANES = 4096;     // int32 lane sums held at once
constexpr int MK_MAX_CHUNKS = 64;  // chunks per CTA per token
constexpr int MK_POLL = 12;        // exchange words a thread polls at once (n <= 3072)
#ifndef MK_BACKOFF_NS
#define MK_BACKOFF_NS 0             // pause between unsuccessful poll rounds (0: none; 64 and 200 ns measured slower)
#endif

enum { PH_QKV = 0, PH_PROJ = 1, PH_FC = 2, PH_FCPROJ = 3, PH_HEAD = 4 };

// One chunk of a CTA's weight stream: rows [r0, r1) of one matrix, as codes
// (rows * row_bytes), then float16 scales, then zero points, each padded to
// 16 bytes.
struct MkChunk {
  int kind, layer, r0, r1;
  int off, bytes, scale_off, zp_off;
};

struct MegaArgs {
  const uint8_t *stream;         // packed weight streams of all CTAs
  const long long *stream_base;  // [grid] offset of CTA c's stream
  const MkChunk *chunks;         // [grid][nchunks]
  int nchunks;                   // chunks per CTA per token
  int n_layer, C, V, n_head;
  const float *small;            // float32 parameters in Model.small order
  WeightView head;               // the tied wte / head in its stored layout (embedding lookups)
  KV8View kv;                    // QuantKV[8] cache (intattn == 0)
  IAView ia;                     // IntAttnKV cache (intattn != 0)
  int intattn;
  long long ia_mult;             // exp2_neg's multiplier (2^40 log2(e) / 2^16)
  unsigned long long *ll;        // exchange buffers (see MkLL)
  float *logits;                 // [V] last step's logits, or null
  int *ids;                      // [steps] produced ids
  const int *first_token;        // device: the token of the first step
  int pos0;                      // its position
  int steps;
  unsigned flag0;                // flag of the first step (steps use flag0, flag0 + 1, ...)
  int *err;                      // device error word (0 = ok)
  long long timeout_cycles;
  long long *prof;               // [2][MK_PROF] cycles per category (CTA 0 and CTA grid/2), or null
};

// Profiling categories (the reference's --profile timers, gpt2t.mojo:121-142,
// split into the time spent waiting for the previous phase's activations and
// the time spent computing).
enum {
  PF_EMBED = 0, PF_QKV_WAIT, PF_QKV, PF_ATTN, PF_PROJ_WAIT, PF_PROJ, PF_FC_WAIT, PF_FC, PF_FCPROJ_WAIT, PF_FCPROJ,
  PF_HEAD_WAIT, PF_HEAD, PF_ARGMAX, PF_RING_WAIT, PF_STEPS,
  // sub-phase timers (also counted in the phases above)
  PF_LN, PF_QUANT, PF_INT, PF_FLOAT, MK_PROF = 20
};

// Adds the cycles since t to acc[k] and restarts t (when acc is not null).
__device__ __forceinline__ void sub_tick(long long *acc, int k, long long &t) {
  if (acc) {
    long long n = clock64();
    acc[k] += n - t;
    t = n;
  }
}

// Offsets (in 8-byte words) of the exchange buffers inside MegaArgs::ll.
struct MkLL {
  int C, L, grid;
  __host__ __device__ MkLL(int c, int l, int g) : C(c), L(l), grid(g) {}
  __host__ __device__ long long qkv(int l) const { return (long long)l * 9 * C; }          // 3C
  __host__ __device__ long long att(int l) const { return (long long)l * 9 * C + 3 * C; }  // C
  __host__ __device__ long long xmid(int l) const { return (long long)l * 9 * C + 4 * C; } // C
  __host__ __device__ long long fc(int l) const { return (long long)l * 9 * C + 5 * C; }   // 4C
  __host__ __device__ long long xout(int l) const { return (long long)L * 9 * C + (long long)l * C; }
  __host__ __device__ long long part() const { return (long long)L * 10 * C; }           // 2 * grid
  __host__ __device__ long long total() const { return part() + 2LL * grid; }
};

// --- PTX helpers -------------------------------------------------------------

__device__ __forceinline__ unsigned smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(unsigned long long *b, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(b)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(unsigned long long *b, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(unsigned long long *b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, unsigned long long *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
__device__ __forceinline__ void cta_sync() { asm volatile("bar.sync 1, %0;" ::"n"(MK_THREADS) : "memory"); }

__device__ __forceinline__ unsigned long long ll_pack(float v, unsigned flag) {
  return ((unsigned long long)flag << 32) | (unsigned long long)__float_as_uint(v);
}

// --- shared memory ---------------------------------------------------------

struct MkSmem {
  unsigned long long full[MK_NSLOT];
  volatile int abort;               // set by a thread whose wait timed out
  int token;
  alignas(16) float red[64];
  alignas(16) float xfull[768];     // the residual stream x of this token (all 768)
  alignas(16) float xf[3072];       // the current matmul input (after LayerNorm)
  alignas(16) int16_t xq[3072];     // its int16 codes (permuted for BLOCKED)
  alignas(16) int xs[192];          // BLOCKED lane sums (as float) / per-channel pair sums (int)
  alignas(16) int lanes[MK_LANES];  // int32 lane sums of the current rows
  alignas(16) float lnw[768];       // the next LayerNorm's weight and bias
  alignas(16) float lnb[768];
  alignas(16) float bias[64];       // the current phase's biases for this CTA's rows
  alignas(16) float att_sc[1024];   // attention scores / exponentials
  alignas(16) float att_ps[1024];   // p * vs
  alignas(16) float att_q[64];
  alignas(16) int8_t att_k[64];
  alignas(16) int8_t att_v[64];
  alignas(16) int8_t kst[MK_KV_STAGE][64];  // staged key codes of positions [0, pos)
  alignas(16) int8_t vst[MK_KV_STAGE][64];  // staged value codes
  alignas(16) float kss[MK_KV_STAGE];       // their scales
  alignas(16) float vss[MK_KV_STAGE];
  alignas(16) float best_v[8];
  alignas(16) int best_i[8];
  alignas(16) float thr_v[MK_THREADS];  // per-thread argmax candidates of the head phase
  alignas(16) int thr_i[MK_THREADS];
  alignas(16) MkChunk chunks[MK_MAX_CHUNKS];
  alignas(128) uint8_t ring[MK_NSLOT][MK_SLOT];
};

// Bounded spin helper: false (and the error recorded) once the budget is
// spent or another thread has given up.
__device__ __forceinline__ bool mk_alive(const MegaArgs &a, MkSmem &sm, long long t0, int code) {
  if (sm.abort) return false;
  if (clock64() - t0 > a.timeout_cycles) {
    sm.abort = 1;
    atomicCAS(a.err, 0, code);
    return false;
  }
  return true;
}

// Reads n <= MK_POLL * MK_THREADS exchange words with flag `flag` into dst
// (all threads). Each round issues every pending load of the thread before
// checking any, so a round costs one memory round trip.
__device__ __noinline__ bool mk_poll(const MegaArgs &a, MkSmem &sm, const unsigned long long *src, int n,
                                     unsigned flag, float *dst, int code) {
  long long t0 = clock64();
  const int tid = threadIdx.x;
  unsigned pending = 0;
#pragma unroll
  for (int k = 0; k < MK_POLL; k++)
    if (tid + k * MK_THREADS < n) pending |= 1u << k;
  while (pending) {
    unsigned long long v[MK_POLL];
#pragma unroll
    for (int k = 0; k < MK_POLL; k++)
      if (pending & (1u << k)) v[k] = ld_relaxed_u64(src + tid + k * MK_THREADS);
#pragma unroll
    for (int k = 0; k < MK_POLL; k++)
      if ((pending & (1u << k)) && (unsigned)(v[k] >> 32) == flag) {
        dst[tid + k * MK_THREADS] = __uint_as_float((unsigned)v[k]);
        pending &= ~(1u << k);
      }
    if (pending) {
      if (!mk_alive(a, sm, t0, code)) break;
      if (MK_BACKOFF_NS > 0) __nanosleep(MK_BACKOFF_NS);
    }
  }
  cp_async_wait_all();  // parameters prefetched before the wait are then visible after the barrier
  cta_sync();
  return !sm.abort;
}

// Starts copying a LayerNorm's weight and bias (768 each) and this CTA's
// biases of rows [r0, r0 + n) into shared memory; waited for before use
// (cp_async_wait_all). Issued before the wait for the activations.
__device__ __forceinline__ void mk_params_load(MkSmem &sm, const float *lnw, const float *lnb, const float *bias,
                                               int r0, int n) {
  const int tid = threadIdx.x;
  if (lnw && tid < 192) {
    cp_async16(&sm.lnw[tid * 4], lnw + tid * 4);
    cp_async16(&sm.lnb[tid * 4], lnb + tid * 4);
  }
  if (bias && tid < n) cp_async4(&sm.bias[tid], bias + r0 + tid);
  cp_async_commit();
}

// LayerNorm of src[0..768) into sm.xf with sm.lnw / sm.lnb
// (kernels.mojo:179-197): 16 lane sums, each sequential over the row's
// 16-float chunks, reduced by the halving tree. The parameters were
// prefetched and the row published by the preceding mk_poll barrier.
// Returns this thread's max |output| (for mk_quantize).
__device__ __noinline__ float mk_layernorm(MkSmem &sm, const float *src) {
  const int C = 768;
  if (threadIdx.x < 32) {
    const int l = threadIdx.x & 15;
    float s = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < 48; k0 += 16) {
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; k++) v[k] = src[16 * (k0 + k) + l];
#pragma unroll
      for (int k = 0; k < 16; k++) s = s + v[k];
    }
    float mean = tree16_warp(s) / (float)C;
    float sq = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < 48; k0 += 16) {
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; k++) v[k] = src[16 * (k0 + k) + l];
#pragma unroll
      for (int k = 0; k < 16; k++) {
        float d = v[k] - mean;
        sq = sq + d * d;
      }
    }
    float var = tree16_warp(sq) / (float)C;
    if (threadIdx.x == 0) {
      sm.red[40] = mean;
      sm.red[41] = 1.0f / sqrtf(var + 1e-5f);
    }
  }
  cta_sync();
  const float mean = sm.red[40], rstd = sm.red[41];
  float mx = 0.0f;
  for (int i = threadIdx.x; i < C; i += MK_THREADS) {
    float n = (src[i] - mean) * rstd;
    float o = n * sm.lnw[i] + sm.lnb[i];
    sm.xf[i] = o;
    mx = fmaxf(mx, fabsf(o));
  }
  return mx;
}

// This thread's max |sm.xf[i]| over its elements of [0, IN).
template <int IN>
__device__ __forceinline__ float mk_local_max(const MkSmem &sm) {
  float mx = 0.0f;
#pragma unroll
  for (int i = threadIdx.x; i < IN; i += MK_THREADS) mx = fmaxf(mx, fabsf(sm.xf[i]));
  return mx;
}

// Largest of the threads' maxima (each >= 0 and not NaN, so their bit
// patterns order like the values): one redux per warp, 8 words in shared
// memory. Ends with the barrier that makes sm.xf's writes visible.
__device__ __forceinline__ float mk_block_max(MkSmem &sm, float mx) {
  const unsigned m = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
  if ((threadIdx.x & 31) == 0) ((unsigned *)sm.red)[threadIdx.x >> 5] = m;
  cta_sync();
  const uint4 a = *(const uint4 *)&sm.red[0], b = *(const uint4 *)&sm.red[4];
  const unsigned r = max(max(max(a.x, a.y), max(a.z, a.w)), max(max(b.x, b.y), max(b.z, b.w)));
  return __uint_as_float(r);
}

// quantize_rows of sm.xf[0..IN) into sm.xq (kernels.mojo:400-416), given
// each thread's max |x| of its elements (mk_local_max or mk_layernorm): the
// BLOCKED lane order and lane sums when BLOCKED (permute_x_i16,
// tensor.mojo:498-516), natural order and per-lane pair sums otherwise.
// Thread t takes columns 4t.. 4t+3 (+ 1024 k) as one float4, so the reads are
// conflict-free; the integer sums are exact in any order. Returns sx.
template <int IN, bool BLOCKED>
__device__ __noinline__ float mk_quantize(MkSmem &sm, float mx) {
  static_assert(IN % 128 == 0 && IN <= 3072, "whole warps of 4 columns per thread");
  float s = mk_block_max(sm, mx) / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  const float inv = 1.0f / s;
  int *xp32 = (int *)sm.xq;
  constexpr int ITER = (IN + 4 * MK_THREADS - 1) / (4 * MK_THREADS);
  if (BLOCKED) {
    // Column col = blk*256 + g*32 + h*16 + e is element e of lane L = g + 8h
    // of block blk: word blk*128 + (e/2)*16 + L, half e%2. A thread's four
    // columns are e = 4j..4j+3 of one lane; four threads make the lane sum.
    float *xsf = (float *)sm.xs;
#pragma unroll
    for (int k = 0; k < ITER; k++) {
      const int c = 4 * threadIdx.x + 4 * MK_THREADS * k;
      if (c < IN) {
        const float4 v = *(const float4 *)(sm.xf + c);
        const int c0 = round_away(v.x * inv), c1 = round_away(v.y * inv);
        const int c2 = round_away(v.z * inv), c3 = round_away(v.w * inv);
        const int blk = c >> 8, w = c & 255, L = ((w >> 5) & 7) + 8 * ((w >> 4) & 1), st = (w & 15) >> 1;
        int *dst = xp32 + blk * 128 + st * 16 + L;
        dst[0] = (c0 & 0xFFFF) | (c1 << 16);
        dst[16] = (c2 & 0xFFFF) | (c3 << 16);
        int sum = (c0 + c1) + (c2 + c3);
        sum += __shfl_xor_sync(0xffffffffu, sum, 1);
        sum += __shfl_xor_sync(0xffffffffu, sum, 2);
        if ((threadIdx.x & 3) == 0) xsf[blk * 16 + L] = (float)sum;
      }
    }
    cta_sync();
  } else {
    // Natural order; xs[L] = sum over the 32-column groups of columns 2L and
    // 2L+1: within a warp the threads t, t^8, t^16, t^24 hold the same
    // pairs, then one partial per warp in sm.lanes and 16 threads add them.
    int *part = sm.lanes;
    int p0 = 0, p1 = 0;
#pragma unroll
    for (int k = 0; k < ITER; k++) {
      const int c = 4 * threadIdx.x + 4 * MK_THREADS * k;
      if (c < IN) {
        const float4 v = *(const float4 *)(sm.xf + c);
        const int c0 = round_away(v.x * inv), c1 = round_away(v.y * inv);
        const int c2 = round_away(v.z * inv), c3 = round_away(v.w * inv);
        xp32[c >> 1] = (c0 & 0xFFFF) | (c1 << 16);
        xp32[(c >> 1) + 1] = (c2 & 0xFFFF) | (c3 << 16);
        p0 += c0 + c1;
        p1 += c2 + c3;
      }
    }
    p0 += __shfl_xor_sync(0xffffffffu, p0, 8);
    p1 += __shfl_xor_sync(0xffffffffu, p1, 8);
    p0 += __shfl_xor_sync(0xffffffffu, p0, 16);
    p1 += __shfl_xor_sync(0xffffffffu, p1, 16);
    const int lane = threadIdx.x & 31;
    if (lane < 8) {
      part[(threadIdx.x >> 5) * 16 + 2 * lane] = p0;
      part[(threadIdx.x >> 5) * 16 + 2 * lane + 1] = p1;
    }
    cta_sync();
    if (threadIdx.x < 16) {
      int sum = 0;
#pragma unroll
      for (int w = 0; w < MK_THREADS / 32; w++) sum += part[w * 16 + threadIdx.x];
      sm.xs[threadIdx.x] = sum;
    }
    cta_sync();
  }
  return s;
}

// Epilogue flags of mk_gemv_blk4 (store_out, kernels.mojo:38-48).
enum { MK_GELU = 1, MK_RESID = 2 };

// The float phase of mk_gemv_blk4 for rows [rbase, rbase + rows) of the
// chunk: thread j of a row's TPR threads carries the chains of lanes j,
// j+TPR, ... over the row's blocks (lane L uses group L & 7 of each block:
// (lane - zp * lane sum of x) * scale, fused, in block order), then the 16
// lanes add as the halving tree (i and i+8, i+4, i+2, i+1): the levels whose
// partner is in the same thread first, then shuffles. The row's value
// dot * sx + bias (+ GELU) (+ residual) is published as an exchange word.
template <int TPR, int NBLK>
__device__ __forceinline__ void mk_float_rows(MkSmem &sm, const MkChunk &ch, const uint8_t *zpp, const uint16_t *scl,
                                              int rbase, int rows, float sx, int epi, unsigned long long *out,
                                              unsigned flag) {
  constexpr int M = 16 / TPR, gpr = NBLK * 8;
  const int j = threadIdx.x % TPR, r = threadIdx.x / TPR;
  const int rr = r < rows ? r : 0;
  const uint8_t *zrow = zpp + (rbase + rr) * gpr;
  const uint16_t *srow = scl + (rbase + rr) * gpr;
  const int *lrow = sm.lanes + rr * NBLK * 16;
  const float *xs = (const float *)sm.xs;
  float f[M];
#pragma unroll
  for (int m = 0; m < M; m++) f[m] = 0.0f;
#pragma unroll
  for (int b = 0; b < NBLK; b++) {
#pragma unroll
    for (int m = 0; m < M; m++) {
      const int L = j + TPR * m, g = b * 8 + (L & 7);
      const float zp = (float)zrow[g];
      const float sc = __half2float(__ushort_as_half(srow[g]));
      f[m] = fmaf((float)lrow[b * 16 + L] - zp * xs[b * 16 + L], sc, f[m]);
    }
  }
  float v;
  if (M == 4) {
    v = (f[0] + f[2]) + (f[1] + f[3]);  // lanes j, j+4, j+8, j+12
  } else if (M == 2) {
    v = f[0] + f[1];  // lanes j, j+8
  } else {
    v = f[0];
  }
#pragma unroll
  for (int o = TPR / 2; o > 0; o >>= 1) v = v + __shfl_xor_sync(0xffffffffu, v, o);
  if (j == 0 && r < rows) {
    const int rl = rbase + r, o = ch.r0 + rl;
    float y = v * sx + sm.bias[rl];
    if (epi & MK_GELU) y = gelu(y);
    if (epi & MK_RESID) y += sm.xfull[o];
    st_relaxed_u64(out + o, ll_pack(y, flag));
  }
}

// BLOCKED int4-g32 rows of the chunk in `slot` against sm.xq (dot_row_i16,
// tensor.mojo:522-540), then v = dot * sx + bias (+ GELU) (+ sm.xfull[o]),
// published as exchange words out[o] with `flag`.
template <int IN>
__device__ __noinline__ void mk_gemv_blk4(MkSmem &sm, const uint8_t *slot, const MkChunk &ch, float sx, int epi,
                                          unsigned long long *out, unsigned flag, long long *pacc) {
  long long t0 = clock64();
  constexpr int nblk = IN >> 8, row_bytes = IN >> 1;
  const int R = ch.r1 - ch.r0;
  const int *xp32 = (const int *)sm.xq;
  const uint16_t *scl = (const uint16_t *)(slot + ch.scale_off);
  const uint8_t *zpp = slot + ch.zp_off;
  constexpr int pass = MK_LANES / (nblk * 16) < 64 ? MK_LANES / (nblk * 16) : 64;
  static_assert(pass <= 64, "one float pass: at least four threads per row");
  for (int rbase = 0; rbase < R; rbase += pass) {
    const int rows = R - rbase < pass ? R - rbase : pass;
    // integer phase: items (row, block, q); the steps of a block are visited
    // in an order rotated by the item so that a warp's shared-memory reads
    // fall in different banks.
    const int items = rows * nblk * 4;
    for (int it = threadIdx.x; it < items; it += MK_THREADS) {
      int q = it & 3, rb = it >> 2, b = rb % nblk, r = rb / nblk;
      const uint32_t *wp = (const uint32_t *)(slot + (size_t)(rbase + r) * row_bytes + b * 128) + q;
      int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
      const int rot = rb & 7;
#pragma unroll
      for (int j = 0; j < 8; j++) {
        int s = (j + rot) & 7;
        uint32_t wv = wp[4 * s];
        uint32_t lo = wv & 0x0F0F0F0Fu, hi = (wv >> 4) & 0x0F0F0F0Fu;
        const int *xv = xp32 + b * 128 + s * 16;
        int2 x01 = *(const int2 *)(xv + 2 * q);
        int2 x89 = *(const int2 *)(xv + 2 * q + 8);
        a0 = dp2a_lo_su(x01.x, lo, a0);
        a1 = dp2a_hi_su(x01.y, lo, a1);
        a2 = dp2a_lo_su(x89.x, hi, a2);
        a3 = dp2a_hi_su(x89.y, hi, a3);
      }
      int *ln = sm.lanes + (r * nblk + b) * 16;
      ln[2 * q] = a0;
      ln[2 * q + 1] = a1;
      ln[2 * q + 8] = a2;
      ln[2 * q + 9] = a3;
    }
    cta_sync();
    sub_tick(pacc, PF_INT, t0);
    // float phase, one pass: TPR threads per row (16 for up to 16 rows, 8 up
    // to 32, 4 up to 64)
    if (rows <= 16)
      mk_float_rows<16, nblk>(sm, ch, zpp, scl, rbase, rows, sx, epi, out, flag);
    else if (rows <= 32)
      mk_float_rows<8, nblk>(sm, ch, zpp, scl, rbase, rows, sx, epi, out, flag);
    else
      mk_float_rows<4, nblk>(sm, ch, zpp, scl, rbase, rows, sx, epi, out, flag);
    cta_sync();
    sub_tick(pacc, PF_FLOAT, t0);
  }
}

// Per-channel int8 head rows of one or two chunks (dot_row_i16 per channel,
// tensor.mojo:541-566): threads 0-127 take the chunk in slot0, threads
// 128-255 the one in slot1 (if any). Thread (r, q) accumulates lanes
// 4q..4q+3 of row r over all the row's 32-column chunks (the int32 sums are
// exact in any order), converts them, and the row's four threads add the 16
// lanes as the halving tree. logit = dot * sx goes to logits (if any) and
// into this thread's argmax candidate (sm.thr_v / thr_i). No barrier: the
// caller's barrier ends the use of the slots.
template <int IN>
__device__ __noinline__ void mk_head_pair(MkSmem &sm, const uint8_t *slot0, const MkChunk &ch0, const uint8_t *slot1,
                                          const MkChunk *ch1, float sx, float *logits) {
  constexpr int nch = IN >> 5;
  const int half = threadIdx.x >> 7;
  if (half == 1 && !ch1) return;  // whole warps
  const uint8_t *slot = half ? slot1 : slot0;
  const MkChunk &ch = half ? *ch1 : ch0;
  const int R = ch.r1 - ch.r0;
  const int *xp32 = (const int *)sm.xq;
  const int q = threadIdx.x & 3, r = (threadIdx.x >> 2) & 31;
  const int rr = r < R ? r : 0;  // rows past R repeat row 0 (their results are dropped)
  const uint8_t *rp = slot + (size_t)rr * IN;
  // a row visits its chunks in an order rotated by the row, so that the
  // rows of a warp read different banks
  const int rot = rr % nch;
  int acc[4] = {0, 0, 0, 0};
#pragma unroll 8
  for (int cc = 0; cc < nch; cc++) {
    int c = cc + rot;
    c = c >= nch ? c - nch : c;
    const uint2 v = *(const uint2 *)(rp + c * 32 + 8 * q);
    const int4 xv = *(const int4 *)(xp32 + c * 16 + 4 * q);
    acc[0] = dp2a_lo_su(xv.x, v.x, acc[0]);
    acc[1] = dp2a_hi_su(xv.y, v.x, acc[1]);
    acc[2] = dp2a_lo_su(xv.z, v.y, acc[2]);
    acc[3] = dp2a_hi_su(xv.w, v.y, acc[3]);
  }
  const int zp = (slot + ch.zp_off)[rr];
  const float sc = __half2float(__ushort_as_half(((const uint16_t *)(slot + ch.scale_off))[rr]));
  float f[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int a = (int)((unsigned)acc[j] - (unsigned)(zp * sm.xs[4 * q + j]));
    f[j] = fmaf((float)a, sc, 0.0f);
  }
  // halving tree: lanes i and i+8 from thread q^2, i and i+4 from q^1
  float b[4];
#pragma unroll
  for (int j = 0; j < 4; j++) b[j] = f[j] + __shfl_xor_sync(0xffffffffu, f[j], 2);
#pragma unroll
  for (int j = 0; j < 4; j++) b[j] = b[j] + __shfl_xor_sync(0xffffffffu, b[j], 1);
  const float dot = (b[0] + b[2]) + (b[1] + b[3]);
  if (q == 0 && r < R) {
    const int o = ch.r0 + r;
    const float v = dot * sx;
    if (logits) logits[o] = v;
    const int t = threadIdx.x;
    if (better(v, o, sm.thr_v[t], sm.thr_i[t])) {
      sm.thr_v[t] = v;
      sm.thr_i[t] = o;
    }
  }
}

// Starts copying this head's cached keys, values and their scales for
// positions [0, pos) into shared memory (pos <= MK_KV_STAGE); mk_attention
// waits for them. Issued early so that the copies overlap the QKV phase.
__device__ __noinline__ void mk_kv_prefetch(const MegaArgs &a, MkSmem &sm, int l, int h, int pos) {
  if (pos > MK_KV_STAGE) return;
  const size_t row0 = ((size_t)l * a.kv.max_t) * a.kv.n_head + h;  // slot of position 0
  const size_t stride = a.kv.n_head;
  for (int i = threadIdx.x; i < pos * 8; i += MK_THREADS) {
    int s = i >> 3, part = i & 7;  // parts 0-3: key, 4-7: value (16 bytes each)
    size_t slot = row0 + s * stride;
    if (part < 4)
      cp_async16(&sm.kst[s][part * 16], a.kv.k + slot * 64 + part * 16);
    else
      cp_async16(&sm.vst[s][(part - 4) * 16], a.kv.v + slot * 64 + (part - 4) * 16);
  }
  for (int i = threadIdx.x; i < pos * 2; i += MK_THREADS) {
    int s = i >> 1;
    size_t slot = row0 + s * stride;
    if (i & 1)
      cp_async4(&sm.vss[s], a.kv.vs + slot);
    else
      cp_async4(&sm.kss[s], a.kv.ks + slot);
  }
  cp_async_commit();
}

// Order-preserving 32-bit keys of floats (not NaN): unsigned comparison of
// the keys is float comparison of the values.
__device__ __forceinline__ unsigned f2key(float f) {
  const unsigned u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(unsigned k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

// Byte k of w (a signed 8-bit code) as a float, exactly, without an
// int-to-float conversion: the code + 128 becomes the low byte of the float
// 2^23 + (code + 128), from which 2^23 + 128 is subtracted.
__device__ __forceinline__ float s8_byte_to_f(unsigned w_biased, int k) {
  return __uint_as_float(__byte_perm(w_biased, 0x4B000000u, 0x7540u + k)) - 8388736.0f;
}
__device__ __forceinline__ float s8_to_f(int8_t c) {
  return __uint_as_float(0x4B000000u | ((unsigned)(uint8_t)c ^ 0x80u)) - 8388736.0f;
}

// Score of one cached position: the 16-lane dot of q with the 64 key codes,
// reduced by the halving tree, times the key scale and 1/sqrt(64).
__device__ __forceinline__ float mk_score(const MkSmem &sm, const int8_t *kp, float ksc) {
  float d[16];
#pragma unroll
  for (int k = 0; k < 16; k++) d[k] = 0.0f;
#pragma unroll
  for (int i = 0; i < 64; i += 16) {
    const uint4 kv4 = *(const uint4 *)(kp + i);
    const unsigned w[4] = {kv4.x ^ 0x80808080u, kv4.y ^ 0x80808080u, kv4.z ^ 0x80808080u, kv4.w ^ 0x80808080u};
#pragma unroll
    for (int k = 0; k < 16; k++) d[k] = d[k] + sm.att_q[i + k] * s8_byte_to_f(w[k >> 2], k & 3);
  }
#pragma unroll
  for (int k = 0; k < 8; k++) d[k] = d[k] + d[k + 8];
#pragma unroll
  for (int k = 0; k < 4; k++) d[k] = d[k] + d[k + 4];
  d[0] = d[0] + d[2];
  d[1] = d[1] + d[3];
  return ((d[0] + d[1]) * ksc) * 0.125f;
}

// Attention phase of head h (QuantKV[8]): store the token's key and value
// (QuantKV.store, kvcache.mojo:333-342), then attend over positions 0..pos
// (attend_float_one, kvcache.mojo:113-150) and publish att[h*64 .. +64).
// Warps 0 and 1 quantize the key and the value (two elements per lane, one
// redux for the max) while warps 2-7 score the cached positions; the
// softmax sum and the value chains run in position order as in the
// reference. Returns false on timeout.
__device__ __noinline__ bool mk_attention(const MegaArgs &a, MkSmem &sm, const MkLL &ll, int l, int h, int pos,
                                          unsigned flag) {
  const int C = a.C, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // poll q, k, v of head h (3 x 64 words); the staged cache copies complete
  {
    long long t0 = clock64();
    if (tid < 192) {
      const int which = tid >> 6, d = tid & 63;
      const unsigned long long *src = a.ll + ll.qkv(l) + which * C + h * 64 + d;
      unsigned long long v;
      while (true) {
        v = ld_relaxed_u64(src);
        if ((unsigned)(v >> 32) == flag) break;
        if (!mk_alive(a, sm, t0, 2)) break;
        if (MK_BACKOFF_NS > 0) __nanosleep(MK_BACKOFF_NS);
      }
      const float x = __uint_as_float((unsigned)v);
      if (which == 0)
        sm.att_q[d] = x;
      else
        sm.xf[(which - 1) * 64 + d] = x;
    }
    cp_async_wait_all();
    cta_sync();
    if (sm.abort) return false;
  }
  const size_t stride_h = a.kv.n_head, base = (size_t)l * a.kv.max_t * stride_h + h;  // slot of position 0
  const size_t sl = base + (size_t)pos * stride_h;
  const bool staged = pos <= MK_KV_STAGE;
  const int npos = pos + 1;
  float mx = -__int_as_float(0x7f800000);
  if (warp < 2) {
    // store: per-head int8 quantization (QuantKV.quantize); warp 0 the key,
    // warp 1 the value
    const float x0 = sm.xf[warp * 64 + lane], x1 = sm.xf[warp * 64 + lane + 32];
    const unsigned m = __reduce_max_sync(0xffffffffu, max(__float_as_uint(fabsf(x0)), __float_as_uint(fabsf(x1))));
    float s = __uint_as_float(m) / 127.0f;
    if (s == 0.0f) s = 1.0f;
    const float inv = 1.0f / s;
    const int8_t q0 = (int8_t)round_away(x0 * inv), q1 = (int8_t)round_away(x1 * inv);
    int8_t *g = (warp == 0 ? a.kv.k : a.kv.v) + sl * 64;
    int8_t *sh = warp == 0 ? sm.att_k : sm.att_v;
    g[lane] = q0;
    g[lane + 32] = q1;
    sh[lane] = q0;
    sh[lane + 32] = q1;
    if (lane == 0) {
      (warp == 0 ? a.kv.ks : a.kv.vs)[sl] = s;
      sm.red[50 + warp] = s;
    }
    if (warp == 0) {
      // the new position's score across the warp: lane k < 16 carries lane
      // k's chain over elements k, 16+k, 32+k, 48+k (lane k + 16 holds the
      // 16+k and 48+k codes), then the halving tree by shuffles
      const float c0 = (float)q0, c1 = (float)q1;
      const float c16 = __shfl_down_sync(0xffffffffu, c0, 16), c48 = __shfl_down_sync(0xffffffffu, c1, 16);
      const int k = lane & 15;
      float d = 0.0f + sm.att_q[k] * c0;
      d = d + sm.att_q[16 + k] * c16;
      d = d + sm.att_q[32 + k] * c1;
      d = d + sm.att_q[48 + k] * c48;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) d = d + __shfl_xor_sync(0xffffffffu, d, o);
      if (lane == 0) {
        const float v = (d * s) * 0.125f;
        sm.att_sc[pos] = v;
        mx = v;
      }
    }
  }
  // scores of the cached positions: warps 2-7 take positions 0..191 first
  for (int s = (tid + 192) & 255; s < pos; s += MK_THREADS) {
    const size_t ss = base + (size_t)s * stride_h;
    const float v = staged ? mk_score(sm, sm.kst[s], sm.kss[s]) : mk_score(sm, a.kv.k + ss * 64, a.kv.ks[ss]);
    sm.att_sc[s] = v;
    mx = fmaxf(mx, v);
  }
  {
    const unsigned k = __reduce_max_sync(0xffffffffu, f2key(mx));
    if (lane == 0) ((unsigned *)sm.red)[warp] = k;
  }
  cta_sync();
  {
    const uint4 ka = *(const uint4 *)&sm.red[0], kb = *(const uint4 *)&sm.red[4];
    mx = key2f(max(max(max(ka.x, ka.y), max(ka.z, ka.w)), max(max(kb.x, kb.y), max(kb.z, kb.w))));
  }
  for (int s = tid; s < npos; s += MK_THREADS) sm.att_sc[s] = lm_expf(sm.att_sc[s] - mx);
  cta_sync();
  if (tid == 0) {
    // sequential sum in position order; the next 16 values load while the
    // current 16 add
    const float4 *e4 = reinterpret_cast<const float4 *>(sm.att_sc);
    float total = 0.0f;
    int s = 0;
    if (npos >= 16) {
      float4 e[4];
#pragma unroll
      for (int k = 0; k < 4; k++) e[k] = e4[k];
      for (; s + 32 <= npos; s += 16) {
        float4 nx[4];
#pragma unroll
        for (int k = 0; k < 4; k++) nx[k] = e4[(s >> 2) + 4 + k];
#pragma unroll
        for (int k = 0; k < 4; k++) total = (((total + e[k].x) + e[k].y) + e[k].z) + e[k].w;
#pragma unroll
        for (int k = 0; k < 4; k++) e[k] = nx[k];
      }
#pragma unroll
      for (int k = 0; k < 4; k++) total = (((total + e[k].x) + e[k].y) + e[k].z) + e[k].w;
      s += 16;
    }
    for (; s < npos; s++) total += sm.att_sc[s];
    sm.red[36] = total;
  }
  cta_sync();
  const float total = sm.red[36];
  for (int s = tid; s < npos; s += MK_THREADS) {
    const float vsc = s == pos ? sm.red[51] : (staged ? sm.vss[s] : a.kv.vs[base + (size_t)s * stride_h]);
    sm.att_ps[s] = (sm.att_sc[s] / total) * vsc;
  }
  cta_sync();
  if (tid < 64) {
    // acc = fma(p * vs, v, acc) over positions in order
    const int d = tid;
    float acc = 0.0f;
    if (staged) {
      // 16 positions at a time; the next 16 load while the current 16 add
      int s = 0;
      if (pos >= 16) {
        const float4 *p4 = reinterpret_cast<const float4 *>(sm.att_ps);
        float pv[16], vv[16];
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float4 q = p4[k];
          pv[4 * k] = q.x;
          pv[4 * k + 1] = q.y;
          pv[4 * k + 2] = q.z;
          pv[4 * k + 3] = q.w;
        }
#pragma unroll
        for (int k = 0; k < 16; k++) vv[k] = s8_to_f(sm.vst[k][d]);
        for (; s + 32 <= pos; s += 16) {
          float np[16], nv[16];
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const float4 q = p4[(s >> 2) + 4 + k];
            np[4 * k] = q.x;
            np[4 * k + 1] = q.y;
            np[4 * k + 2] = q.z;
            np[4 * k + 3] = q.w;
          }
#pragma unroll
          for (int k = 0; k < 16; k++) nv[k] = s8_to_f(sm.vst[s + 16 + k][d]);
#pragma unroll
          for (int k = 0; k < 16; k++) acc = fmaf(pv[k], vv[k], acc);
#pragma unroll
          for (int k = 0; k < 16; k++) {
            pv[k] = np[k];
            vv[k] = nv[k];
          }
        }
#pragma unroll
        for (int k = 0; k < 16; k++) acc = fmaf(pv[k], vv[k], acc);
        s += 16;
      }
      for (; s < pos; s++) acc = fmaf(sm.att_ps[s], s8_to_f(sm.vst[s][d]), acc);
    } else {
      const int8_t *vp = a.kv.v + base * 64 + d;
      for (int s = 0; s < pos; s++) acc = fmaf(sm.att_ps[s], (float)vp[(size_t)s * stride_h * 64], acc);
    }
    acc = fmaf(sm.att_ps[pos], (float)sm.att_v[d], acc);
    st_relaxed_u64(a.ll + ll.att(l) + h * 64 + d, ll_pack(acc, flag));
  }
  return true;
}

// Attention phase of head h with IntAttnKV (int_attention.mojo:119-269): the
// token's key and value quantized into the cache (quantize_head), then
// attend_one over positions 0..pos, published as att[h*64 .. +64). The
// arithmetic is ia_attend_kernel's: integer scores and softmax, value sums
// flushed to float per 128 pairs of positions in order. The K/V staging
// buffers (unused by this cache) hold the reductions' scratch. Returns false
// on timeout.
__device__ __noinline__ bool mk_ia_attention(const MegaArgs &a, MkSmem &sm, const MkLL &ll, int l, int h, int pos,
                                             unsigned flag) {
  const IAView &c = a.ia;
  const int HS = 64, C = a.C, tid = threadIdx.x;
  {
    long long t0 = clock64();
    if (tid < 192) {
      const int which = tid >> 6, d = tid & 63;
      const unsigned long long *src = a.ll + ll.qkv(l) + which * C + h * 64 + d;
      unsigned long long v;
      while (true) {
        v = ld_relaxed_u64(src);
        if ((unsigned)(v >> 32) == flag) break;
        if (!mk_alive(a, sm, t0, 2)) break;
        if (MK_BACKOFF_NS > 0) __nanosleep(MK_BACKOFF_NS);
      }
      const float x = __uint_as_float((unsigned)v);
      if (which == 0)
        sm.att_q[d] = x;
      else
        sm.xf[(which - 1) * 64 + d] = x;
    }
    cta_sync();
    if (sm.abort) return false;
  }
  long long *redl = reinterpret_cast<long long *>(&sm.kst[0][0]);  // 32 slots
  int32_t *qpair = reinterpret_cast<int32_t *>(&sm.kst[4][0]);     // 32 pairs
  int32_t *part = reinterpret_cast<int32_t *>(&sm.kst[8][0]);      // [4][64]
  float *redf = sm.red;
  int32_t *sc = reinterpret_cast<int32_t *>(sm.att_sc);            // [max_t]
  int16_t *w = reinterpret_cast<int16_t *>(sm.att_ps);             // [max_t + 2]
  // store (quantize_head) of the key and the value
  for (int which = 0; which < 2; which++) {
    const bool act = tid < HS;
    ia_quantize_head(c, act ? sm.xf[which * 64 + tid] : 0.0f, act, l, h, pos, which, redf);
  }
  __syncthreads();  // the cache writes of this CTA are visible to it
  const int npos = pos + 1;
  const int nr = (npos + IA_PB - 1) / IA_PB * IA_PB;
  // 1. the query as int16
  const float qv = tid < HS ? sm.att_q[tid] : 0.0f;
  const float mq = ia_block_max_f(fabsf(qv), redf);
  float sq = mq / 32767.0f;
  if (sq == 0.0f) sq = 1.0f;
  const float invq = 1.0f / sq;
  const int16_t qi = (int16_t)roundf(qv * invq);
  const int16_t qi_next = (int16_t)__shfl_down_sync(0xffffffffu, (int)qi, 1);
  if (tid < HS && (tid & 1) == 0) qpair[tid / 2] = (int32_t)(uint16_t)qi | ((int32_t)qi_next << 16);
  const long long qm = llround((double)sq / sqrt((double)HS) * (double)(1LL << (IA_SF + IA_KS)));
  __syncthreads();
  // 2. scores of positions [0, nr)
  const int32_t *ks = c.kq + ia_lh(c, l, h) * c.max_t;
  long long smax = LLONG_MIN;
  for (int p = tid; p < nr; p += MK_THREADS) {
    const uint16_t *kp = (const uint16_t *)(c.k + ia_k_at(c, l, h, p, 0));
    int acc = 0;
    for (int j = 0; j < HS / 2; j++) acc = __dp2a_lo(qpair[j], (int)kp[(size_t)j * IA_PB], acc);
    const long long t1 = ((long long)acc * (long long)ks[p] + (1LL << (IA_KS - 1))) >> IA_KS;
    const long long sfix = (t1 * qm + (1LL << (IA_KS - 1))) >> IA_KS;
    sc[p] = (int32_t)sfix;
    if (p < npos && (long long)(int32_t)sfix > smax) smax = (int32_t)sfix;
  }
  const long long m = ia_block_max_ll(smax, redl);
  // 3. masked_exp: e in Q30 over the valid positions, total in int64
  long long part_total = 0;
  for (int p = tid; p < nr; p += MK_THREADS) {
    const long long ev = p < npos ? ia_exp2_neg(m - (long long)sc[p], a.ia_mult) : 0;
    sc[p] = (int32_t)ev;
    part_total += ev;
  }
  const long long total = ia_block_sum_ll(part_total, redl);
  // 4. value weights and sums
  const int32_t *vs = c.vq + ia_lh(c, l, h) * c.max_t;
  long long vm = 0;
  for (int p = tid; p < npos; p += MK_THREADS) vm = (long long)vs[p] > vm ? (long long)vs[p] : vm;
  const long long vmax = ia_block_max_ll(vm, redl);
  unsigned long long *o = a.ll + ll.att(l) + h * HS;
  if (vmax == 0 || total == 0) {
    if (tid < HS) st_relaxed_u64(o + tid, ll_pack(0.0f, flag));
    return true;
  }
  const long long inv47 = (1LL << 47) / vmax;
  for (int p = tid; p < nr + 2; p += MK_THREADS) {
    long long ww = 0;
    if (p < nr) {
      const long long ee = sc[p];
      const long long r16 = p < npos ? ((long long)vs[p] * inv47) >> 31 : 0;
      ww = (ee * r16 + (1LL << 30)) >> 31;
      if (ww > 32767) ww = 32767;
      if (ee == 0) ww = 0;
    }
    w[p] = (int16_t)ww;
  }
  __syncthreads();
  constexpr int nparts = MK_THREADS / 64;  // threads per dimension
  const int d = tid % HS, pidx = tid / HS;
  const int npairs = (npos + 1) / 2;
  float accf = 0.0f;
  const uint16_t *vbase = (const uint16_t *)(c.v + ia_v_at(c, l, h, 0, 0));
  for (int sg = 0; sg < npairs; sg += 128) {
    const int end = npairs < sg + 128 ? npairs : sg + 128;
    int acc = 0;
    for (int pp = sg + pidx; pp < end; pp += nparts) {
      const int wp = (int)(uint16_t)w[2 * pp] | ((int)w[2 * pp + 1] << 16);
      acc = __dp2a_lo(wp, (int)vbase[(size_t)pp * HS + d], acc);
    }
    part[pidx * HS + d] = acc;
    __syncthreads();
    if (pidx == 0) {
      unsigned sum = 0;
      for (int q = 0; q < nparts; q++) sum += (unsigned)part[q * HS + d];
      accf += (float)(int32_t)sum;
    }
    __syncthreads();
  }
  if (pidx == 0) {
    const float fs = (float)((double)vmax * (double)(1 << 15) / ((double)(1 << IA_KS) * (double)total));
    st_relaxed_u64(o + d, ll_pack(accf * fs, flag));
  }
  return true;
}

// Embedding of `token` at `pos` (gpt2t.mojo:378-385) into sm.xfull.
__device__ __noinline__ void mk_embed(const MegaArgs &a, MkSmem &sm, int token, int pos) {
  const int C = a.C, gpr = a.head.cols / a.head.group;
  const float *wpe = a.small + (size_t)a.n_layer * 13 * C;
  for (int i = threadIdx.x; i < C; i += MK_THREADS) {
    size_t gi = (size_t)token * gpr + i / a.head.group;
    float s = __half2float(__ushort_as_half(a.head.scale[gi]));
    float v = (float)(code_at(a.head, token, i) - (int)a.head.zp[gi]) * s;
    sm.xfull[i] = v + wpe[(size_t)pos * C + i];
  }
  cta_sync();
}

// The greedy argmax over all CTAs' candidates (gpt2t.mojo:792-797) after
// the head phase; the winner goes to sm.token (and ids[step] from CTA 0).
// Returns false on timeout.
__device__ __noinline__ bool mk_argmax(const MegaArgs &a, MkSmem &sm, const MkLL &ll, unsigned flag, int step) {
  const int tid = threadIdx.x, cta = blockIdx.x, grid = gridDim.x;
  float bv = sm.thr_v[tid];
  int bi = sm.thr_i[tid];
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((tid & 31) == 0) {
    sm.best_v[tid >> 5] = bv;
    sm.best_i[tid >> 5] = bi;
  }
  cta_sync();
  if (tid == 0) {
    for (int w = 1; w < MK_THREADS / 32; w++)
      if (better(sm.best_v[w], sm.best_i[w], bv, bi)) {
        bv = sm.best_v[w];
        bi = sm.best_i[w];
      }
    st_relaxed_u64(a.ll + ll.part() + 2 * cta, ll_pack(bv, flag));
    st_relaxed_u64(a.ll + ll.part() + 2 * cta + 1, ((unsigned long long)flag << 32) | (unsigned)bi);
  }
  if (!mk_poll(a, sm, a.ll + ll.part(), 2 * grid, flag, sm.xf, 8)) return false;
  if (tid < 32) {
    float v = -__int_as_float(0x7f800000);
    int i = 0x7fffffff;
    for (int c = tid; c < grid; c += 32) {
      float cv = sm.xf[2 * c];
      int cidx = __float_as_int(sm.xf[2 * c + 1]);
      if (better(cv, cidx, v, i)) {
        v = cv;
        i = cidx;
      }
    }
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, v, o);
      int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (better(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (tid == 0) {
      if (i == 0x7fffffff) i = 0;  // every logit NaN: the scan keeps index 0
      sm.token = i;
      if (cta == 0) a.ids[step] = i;
    }
  }
  cta_sync();
  return true;
}

__global__ void __launch_bounds__(MK_THREADS, 1) mega_decode_kernel(MegaArgs a) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  MkSmem &sm = *reinterpret_cast<MkSmem *>(smem_raw);
  const int tid = threadIdx.x;
  const int cta = blockIdx.x, grid = gridDim.x;
  const MkLL ll(a.C, a.n_layer, grid);
  const uint8_t *stream = a.stream + a.stream_base[cta];
  const int total_chunks = a.nchunks * a.steps;  // <= 64 x 4096
  const int C = a.C, C4 = 4 * C;

  for (int i = tid; i < a.nchunks; i += MK_THREADS) sm.chunks[i] = a.chunks[(size_t)cta * a.nchunks + i];
  if (tid == 0) {
    for (int i = 0; i < MK_NSLOT; i++) mbar_init(&sm.full[i], 1);
    sm.abort = 0;
    int t0 = *a.first_token;
    if (t0 < 0 || t0 >= a.V) {
      atomicCAS(a.err, 0, 9);
      t0 = 0;
    }
    sm.token = t0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  // The ring: chunk q of the whole generation goes to slot q % MK_NSLOT
  // with mbarrier phase parity (q / MK_NSLOT) & 1. The indices advance by one
  // per chunk (no divisions on the way).
  int seq = 0, rslot = 0, rpar = 0;  // chunks consumed; slot and parity of chunk seq
  int iss = 0, iss_slot = 0, iss_ci = 0;  // thread 0: chunks issued; slot and token chunk index of the next
  auto issue = [&]() {  // the next chunk into its slot (thread 0)
    const MkChunk &ch = sm.chunks[iss_ci];
    mbar_expect_tx(&sm.full[iss_slot], (unsigned)ch.bytes);
    bulk_g2s(sm.ring[iss_slot], stream + ch.off, (unsigned)ch.bytes, &sm.full[iss_slot]);
    iss++;
    iss_slot = iss_slot + 1 == MK_NSLOT ? 0 : iss_slot + 1;
    iss_ci = iss_ci + 1 == a.nchunks ? 0 : iss_ci + 1;
  };
  if (tid == 0)
    while (iss < MK_NSLOT && iss < total_chunks) issue();

  // profiling (thread 0 of CTAs 0 and grid/2)
  const bool prof_on = a.prof && tid == 0 && (cta == 0 || cta == grid / 2);
  long long pacc[MK_PROF];
  for (int k = 0; k < MK_PROF; k++) pacc[k] = 0;
  long long *pp = prof_on ? pacc : nullptr;
  long long tlast = clock64();
  auto tick = [&](int k) {
    if (prof_on) {
      long long t = clock64();
      pacc[k] += t - tlast;
      tlast = t;
    }
  };
  // Slot of chunk `seq + ahead` (ahead 0 or 1), or -1 on timeout. Every
  // thread waits; the answer is the CTA's, read after a barrier, so that no
  // thread leaves for the exit path while others enter a phase's barriers.
  auto slot_wait = [&](int ahead = 0) -> int {
    int slot = rslot + ahead;
    unsigned par = (unsigned)rpar;
    if (slot >= MK_NSLOT) {
      slot -= MK_NSLOT;
      par ^= 1u;
    }
    long long t0 = clock64();
    while (!mbar_try_wait(&sm.full[slot], par)) {
      if (!mk_alive(a, sm, t0, 1)) break;
    }
    if (prof_on) pacc[PF_RING_WAIT] += clock64() - t0;
    cta_sync();
    return sm.abort ? -1 : slot;
  };
  // Called after the barrier that ends the use of the slot (the last one in
  // mk_gemv_blk4, or the one after mk_head_pair).
  auto slot_release = [&]() {
    if (tid == 0 && iss < total_chunks) issue();  // chunk seq + MK_NSLOT
    seq++;
    if (++rslot == MK_NSLOT) {
      rslot = 0;
      rpar ^= 1;
    }
  };
  // One GEMV phase: wait for its weights, compute, publish, release.
  auto gemv = [&](const MkChunk &ch, int IN, float sx, int epi, unsigned long long *out, unsigned flag) -> bool {
    const int slot = slot_wait();
    if (slot < 0) return false;
    if (IN == 768)
      mk_gemv_blk4<768>(sm, sm.ring[slot], ch, sx, epi, out, flag, pp);
    else
      mk_gemv_blk4<3072>(sm, sm.ring[slot], ch, sx, epi, out, flag, pp);
    slot_release();
    return true;
  };

  // A chunk without rows (the attention CTAs have no QKV and PROJ rows): its
  // ring slot is taken and handed back, the phase is skipped.
  auto skip_chunk = [&]() -> bool {
    const int slot = slot_wait();
    if (slot < 0) return false;
    cta_sync();
    slot_release();
    return true;
  };

  const float *lnf = a.small + (size_t)a.n_layer * 13 * C + (size_t)1024 * C;
  bool ok = true;
  for (int step = 0; ok && step < a.steps; step++) {
    const unsigned flag = a.flag0 + (unsigned)step;
    const int pos = a.pos0 + step;
    mk_embed(a, sm, sm.token, pos);
    tick(PF_EMBED);
    int ci = 0;  // chunk index within the token
    for (int l = 0; ok && l < a.n_layer; l++) {
      const float *vec = a.small + (size_t)l * 13 * C;
      // ---- A: LN1 + QKV ----
      {
        if (cta < a.n_head && !a.intattn) mk_kv_prefetch(a, sm, l, cta, pos);
        const MkChunk &ch = sm.chunks[ci++];
        if (ch.r1 == ch.r0) {
          if (!(ok = skip_chunk())) break;
          tick(PF_QKV_WAIT);
          tick(PF_QKV);
        } else {
          mk_params_load(sm, vec, vec + C, vec + 2 * C, ch.r0, ch.r1 - ch.r0);
          if (l == 0) {  // x is this CTA's embedding; only the parameters to wait for
            cp_async_wait_all();
            cta_sync();
          } else if (!mk_poll(a, sm, a.ll + ll.xout(l - 1), C, flag, sm.xfull, 3)) {
            ok = false;
            break;
          }
          tick(PF_QKV_WAIT);
          long long t0 = clock64();
          const float lmx = mk_layernorm(sm, sm.xfull);
          sub_tick(pp, PF_LN, t0);
          const float sx = mk_quantize<768, true>(sm, lmx);
          sub_tick(pp, PF_QUANT, t0);
          if (!(ok = gemv(ch, C, sx, 0, a.ll + ll.qkv(l), flag))) break;
          tick(PF_QKV);
        }
      }
      // ---- B: KV store + attention (CTA h for head h) ----
      if (cta < a.n_head) {
        ok = a.intattn ? mk_ia_attention(a, sm, ll, l, cta, pos, flag) : mk_attention(a, sm, ll, l, cta, pos, flag);
        if (!ok) break;
        tick(PF_ATTN);
      }
      // ---- C: PROJ + residual ----
      {
        const MkChunk &ch = sm.chunks[ci++];
        if (ch.r1 == ch.r0) {
          if (!(ok = skip_chunk())) break;
          tick(PF_PROJ_WAIT);
          tick(PF_PROJ);
        } else {
          mk_params_load(sm, nullptr, nullptr, vec + 5 * C, ch.r0, ch.r1 - ch.r0);
          if (!(ok = mk_poll(a, sm, a.ll + ll.att(l), C, flag, sm.xf, 4))) break;
          tick(PF_PROJ_WAIT);
          long long t0 = clock64();
          const float sx = mk_quantize<768, true>(sm, mk_local_max<768>(sm));
          sub_tick(pp, PF_QUANT, t0);
          if (!(ok = gemv(ch, C, sx, MK_RESID, a.ll + ll.xmid(l), flag))) break;
          tick(PF_PROJ);
        }
      }
      // ---- D: LN2 + FC + GELU ----
      {
        const MkChunk &ch = sm.chunks[ci++];
        mk_params_load(sm, vec + 6 * C, vec + 7 * C, vec + 8 * C, ch.r0, ch.r1 - ch.r0);
        if (!(ok = mk_poll(a, sm, a.ll + ll.xmid(l), C, flag, sm.xfull, 5))) break;
        tick(PF_FC_WAIT);
        long long t0 = clock64();
        const float lmx = mk_layernorm(sm, sm.xfull);
        sub_tick(pp, PF_LN, t0);
        const float sx = mk_quantize<768, true>(sm, lmx);
        sub_tick(pp, PF_QUANT, t0);
        if (!(ok = gemv(ch, C, sx, MK_GELU, a.ll + ll.fc(l), flag))) break;
        tick(PF_FC);
      }
      // ---- E: FCPROJ + residual ----
      {
        const MkChunk &ch = sm.chunks[ci++];
        mk_params_load(sm, nullptr, nullptr, vec + 12 * C, ch.r0, ch.r1 - ch.r0);
        if (!(ok = mk_poll(a, sm, a.ll + ll.fc(l), C4, flag, sm.xf, 6))) break;
        tick(PF_FCPROJ_WAIT);
        long long t0 = clock64();
        const float sx = mk_quantize<3072, true>(sm, mk_local_max<3072>(sm));
        sub_tick(pp, PF_QUANT, t0);
        if (!(ok = gemv(ch, C4, sx, MK_RESID, a.ll + ll.xout(l), flag))) break;
        tick(PF_FCPROJ);
      }
    }
    if (!ok) break;
    // ---- H: LN_f + head + argmax ----
    mk_params_load(sm, lnf, lnf + C, nullptr, 0, 0);
    if (!(ok = mk_poll(a, sm, a.ll + ll.xout(a.n_layer - 1), C, flag, sm.xf, 7))) break;
    tick(PF_HEAD_WAIT);
    const float sx = mk_quantize<768, false>(sm, mk_layernorm(sm, sm.xf));
    sm.thr_v[tid] = -__int_as_float(0x7f800000);
    sm.thr_i[tid] = 0x7fffffff;
    for (; ci < a.nchunks; ci += 2) {  // two chunks per round
      const bool two = ci + 1 < a.nchunks;
      const int s0 = slot_wait(), s1 = two ? slot_wait(1) : 0;
      if (s0 < 0 || s1 < 0) {
        ok = false;
        break;
      }
      mk_head_pair<768>(sm, sm.ring[s0], sm.chunks[ci], sm.ring[s1], two ? &sm.chunks[ci + 1] : nullptr, sx,
                        a.logits);
      cta_sync();
      slot_release();
      if (two) slot_release();
    }
    if (!ok) break;
    tick(PF_HEAD);
    // ---- I: global argmax (every CTA) ----
    if (!(ok = mk_argmax(a, sm, ll, flag, step))) break;
    tick(PF_ARGMAX);
    if (prof_on) pacc[PF_STEPS] += 1;
  }

  if (!ok) {
    // On a timeout every thread leaves; first each waits for its own
    // cp.async copies, and thread 0 (bounded) for the ring's bulk copies in
    // flight.
    cp_async_wait_all();
    if (tid == 0) {
      int slot = rslot;
      unsigned par = (unsigned)rpar;
      for (int q = seq; q < seq + MK_NSLOT && q < total_chunks; q++) {
        long long t1 = clock64();
        while (!mbar_try_wait(&sm.full[slot], par) && clock64() - t1 < kDrainCycles) {
        }
        if (++slot == MK_NSLOT) {
          slot = 0;
          par ^= 1u;
        }
      }
    }
    return;
  }
  if (prof_on) {
    long long *dst = a.prof + (cta == 0 ? 0 : MK_PROF);
    for (int k = 0; k < MK_PROF; k++) dst[k] += pacc[k];
  }
}

}  // namespace llmq
