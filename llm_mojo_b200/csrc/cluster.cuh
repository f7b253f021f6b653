// Cluster decode kernel: a whole greedy generation in one cooperative launch
// of thread-block clusters of 16 CTAs on sm_100a.
//
// Why a cluster. A decode token is a chain of ~50 dependent steps (per
// layer: LayerNorm + QKV, attention, PROJ, LayerNorm + FC, FCPROJ), each of
// which needs the whole output of the step before (LayerNorm statistics and
// the int16 quantization scale of every matmul input are reductions over the
// full vector). On B200 an exchange of a vector between CTAs through global
// memory costs 1.2-2.2 us (a store and a polling load both cross L2), while
// an all-gather between the 16 CTAs of a cluster through distributed shared
// memory (st.async with mbarrier completion) costs ~0.4 us. So:
//   - cluster 0 ("layer ranks" 0..15) runs all the layers. Rank h < 12 owns
//     attention head h: it computes that head's 192 QKV rows itself and runs
//     its attention, so q, k and v never leave the CTA. PROJ, FC and FCPROJ
//     rows are split evenly over the 16 ranks. After each of attention,
//     PROJ, FC and FCPROJ every rank pushes its slice of the output vector
//     into the matching receive buffer of all 16 ranks; the buffer's
//     mbarrier completes when all bytes have arrived. LayerNorm and the
//     int16 quantization of each matmul input run redundantly in every rank.
//   - clusters 1.. ("head CTAs") run the output head: each owns a slice of
//     the 50257 rows, streamed through its own shared-memory ring (prefetched
//     while the layers run), and publishes an argmax candidate. The hidden
//     state goes from cluster 0 to the head CTAs, and the candidates back,
//     through global memory as (value, flag) words: two global exchanges per
//     token instead of one per step.
// Each CTA streams its weights from a per-CTA packed copy in HBM in the order
// it uses them, with cp.async.bulk into a ring of shared-memory slots; the
// thread that releases a slot issues the copy of the chunk NSLOT ahead.
//
// Every wait (ring slots, receive buffers, global flags) is bounded; on a
// timeout the CTA records an error code, stops, waits (bounded) for its own
// copies and for the pushes it expects, and meets the other ranks at the
// final cluster barrier.
//
// The arithmetic of every step is that of the one-token kernels and of the
// persistent kernel (mega.cuh): bit-identical to the reference's.
#pragma once

#include "mega.cuh"

namespace llmq {

constexpr int CD_THREADS = 256;
constexpr int CD_CLUSTER = 16;
constexpr int CD_NSLOT = 5;         // layer ring slots
constexpr int CD_SLOT = 29184;      // 64 rows x 3 blocks of int4-g32 (codes, f16 scales, zero points)
constexpr int CD_KV_STAGE = 128;    // cache positions an attention rank stages in shared memory
constexpr int CD_MAX_CHUNKS = 12;   // layer chunks per rank per layer
constexpr int CD_HROWS = 32;        // head rows per chunk
constexpr int CD_HSLOT = CD_HROWS * 768 + CD_HROWS * 2 + CD_HROWS;  // 24672
constexpr int CD_HNSLOT = 8;        // head ring slots

enum { CD_QKV = 0, CD_PROJ = 1, CD_FC = 2, CD_FCPROJ = 3 };
enum { RB_ATT = 0, RB_XMID = 1, RB_FC = 2, RB_XOUT = 3 };

// One chunk of a layer rank's stream: output rows [r0, r0 + n) of one
// matrix, padded to rp rows (a multiple of 8), 256-column blocks
// [b0, b0 + nb). Layout inside the chunk (bytes):
//   codes  [nb][2 halves][rp][4 words q][4 steps] x 4 B  (word q of steps 4h..4h+3)
//   scales [nb][rp][8 groups] float16                    at scale_off
//   zps    [nb][rp][8 groups] u8                         at zp_off
// so that 8 consecutive rows x 4 words are 512 contiguous bytes (one
// conflict-free 16-byte load per thread).
struct CdChunk {
  int kind, r0, n, rp;
  int b0, nb;
  int off, bytes;  // within one layer of the rank's stream
  int scale_off, zp_off;
};

struct CdArgs {
  const uint8_t *lstream;    // layer ranks' streams
  const long long *lbase;    // [16] start of rank r's stream
  const CdChunk *lchunks;    // [16][CD_MAX_CHUNKS] chunk templates of one layer
  const int *lnch;           // [16] chunks per layer
  const long long *lbytes;   // [16] stream bytes per layer
  const uint8_t *hstream;    // head CTAs' streams (CD_HSLOT bytes per 32-row chunk)
  const long long *hbase;    // [n_hcta] start of head CTA j's stream
  int n_hcta;                // head CTAs (CTAs of clusters 1..)
  int n_layer, C, V, n_head;
  const float *small;        // float32 parameters in Model.small order
  WeightView head;           // the tied wte / head in its stored layout (embedding lookups)
  KV8View kv;                // QuantKV[8] cache
  unsigned long long *ll;    // [C] final hidden state words, then [2 * n_hcta] argmax candidates
  float *logits;             // [V] last step's logits, or null
  int *ids;                  // [steps] produced ids
  const int *first_token;    // device: the token of the first step
  int pos0, steps;
  unsigned flag0;            // flag of the first step (steps use flag0, flag0 + 1, ...)
  int *err;
  long long timeout_cycles;
  long long *prof;           // [2][MK_PROF] cycles per category (layer rank 0, head CTA 0), or null
};

// Profiling categories of this kernel (layer rank 0: CP_*; head CTA 0: CH_*).
enum {
  CP_EMBED = 0, CP_LN1, CP_QKV, CP_ATTN, CP_HOP_ATT, CP_PROJ, CP_HOP_XMID, CP_LN2, CP_FC, CP_HOP_FC, CP_FCPROJ,
  CP_HOP_XOUT, CP_ARGMAX_WAIT, CP_RING_WAIT, CP_STEPS,
  // sub-phase timers (also counted in the phases above)
  CP_GEMV, CP_QUANT, CP_PUSH, CP_ATTN_INNER
};
enum { CH_X_WAIT = 0, CH_LN = 1, CH_ROWS = 2, CH_RING_WAIT = 3, CH_STEPS = 4 };

// --- PTX helpers (cluster) ------------------------------------------------------

__device__ __forceinline__ unsigned cd_rank() {
  unsigned r;
  asm("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ unsigned cd_cluster_id() {
  unsigned r;
  asm("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ unsigned cd_mapa(unsigned a, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
__device__ __forceinline__ void cd_cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ bool cd_try_wait_cluster(unsigned long long *b, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, "
      "p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(b)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void cp_async_wait_group1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cd_st_async_v4(unsigned dst, float4 v, unsigned bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(dst),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar)
               : "memory");
}

// --- shared memory ------------------------------------------------------------

struct CdLSmem {  // a layer rank
  unsigned long long full[CD_NSLOT];  // ring slots
  unsigned long long rbar[4];         // receive buffers: att, xmid, fc, xout
  volatile int abort;
  int token;
  unsigned rph_left;                  // parities of the receive phases open when the rank gave up
  alignas(16) float red[64];
  alignas(16) float b_att[768];       // attention output (all heads), pushed by ranks 0..11
  alignas(16) float b_xmid[768];      // x after attention + PROJ + residual
  alignas(16) float b_fc[3072];       // GELU(FC)
  alignas(16) float b_xout[768];      // x after the block (the residual stream)
  alignas(16) float xf[768];          // LayerNorm output
  alignas(16) int xq[1536];           // int16 codes of the current matmul input in the kernel's lane order
  alignas(16) int xs[192];            // their lane sums: [block][q][4 lanes 2q, 2q+1, 2q+8, 2q+9]
  alignas(16) float lnw[768];
  alignas(16) float lnb[768];
  alignas(16) float bias[192];        // the current phase's biases of this rank's rows
  alignas(16) float outv[192];        // this rank's outputs of the current phase
  alignas(16) float att_o[64];        // this rank's head output
  alignas(16) float att_sc[1024];     // attention scores / exponentials
  alignas(16) float att_ps[1024];     // p * vs
  alignas(16) int8_t att_k[64];
  alignas(16) int8_t att_v[64];
  alignas(16) int8_t kst[CD_KV_STAGE][64];
  alignas(16) int8_t vst[CD_KV_STAGE][64];
  alignas(16) float kss[CD_KV_STAGE];
  alignas(16) float vss[CD_KV_STAGE];
  alignas(16) float best_v[8];
  alignas(16) int best_i[8];
  alignas(16) CdChunk chunks[CD_MAX_CHUNKS];
  alignas(128) uint8_t ring[CD_NSLOT][CD_SLOT];
};

struct CdHSmem {  // a head CTA
  unsigned long long full[CD_HNSLOT];
  volatile int abort;
  alignas(16) float red[64];
  alignas(16) float xin[768];         // the final hidden state
  alignas(16) float xf[768];          // LN_f output
  alignas(16) int xq[384];            // int16 codes, natural order
  alignas(16) int xs[16];             // per-lane pair sums
  alignas(16) float lnw[768];
  alignas(16) float lnb[768];
  alignas(16) float best_v[8];
  alignas(16) int best_i[8];
  alignas(128) uint8_t ring[CD_HNSLOT][CD_HSLOT];
};

constexpr size_t cd_smem_bytes() { return sizeof(CdLSmem) > sizeof(CdHSmem) ? sizeof(CdLSmem) : sizeof(CdHSmem); }

// --- small helpers (either role) -----------------------------------------------

// Bounded spin helper: false (and the error recorded) once the budget is
// spent or another thread of the CTA has given up.
template <class SM>
__device__ __forceinline__ bool cd_alive(const CdArgs &a, SM &sm, long long t0, int code) {
  if (sm.abort) return false;
  if (clock64() - t0 > a.timeout_cycles) {
    sm.abort = 1;
    atomicCAS(a.err, 0, code);
    return false;
  }
  return true;
}

// Largest of the threads' maxima (each >= 0, not NaN): one redux per warp.
// Ends with the barrier that makes earlier shared-memory writes visible.
template <class SM>
__device__ __forceinline__ float cd_block_max(SM &sm, float mx) {
  const unsigned m = __reduce_max_sync(0xffffffffu, __float_as_uint(mx));
  if ((threadIdx.x & 31) == 0) ((unsigned *)sm.red)[threadIdx.x >> 5] = m;
  __syncthreads();
  const uint4 a = *(const uint4 *)&sm.red[0], b = *(const uint4 *)&sm.red[4];
  const unsigned r = max(max(max(a.x, a.y), max(a.z, a.w)), max(max(b.x, b.y), max(b.z, b.w)));
  __syncthreads();  // sm.red is reused by the next reduction
  return __uint_as_float(r);
}

// LayerNorm of src[0..768) into sm.xf with sm.lnw / sm.lnb (kernels.mojo:179-197):
// 16 lane sums, each sequential over the row's 16-float chunks, reduced by
// the halving tree; returns this thread's max |output|.
template <class SM>
__device__ __noinline__ float cd_layernorm(SM &sm, const float *src) {
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
    const float mean = tree16_warp(s) / (float)C;
    float sq = 0.0f;
#pragma unroll
    for (int k0 = 0; k0 < 48; k0 += 16) {
      float v[16];
#pragma unroll
      for (int k = 0; k < 16; k++) v[k] = src[16 * (k0 + k) + l];
#pragma unroll
      for (int k = 0; k < 16; k++) {
        const float d = v[k] - mean;
        sq = sq + d * d;
      }
    }
    const float var = tree16_warp(sq) / (float)C;
    if (threadIdx.x == 0) {
      sm.red[40] = mean;
      sm.red[41] = 1.0f / sqrtf(var + 1e-5f);
    }
  }
  __syncthreads();
  const float mean = sm.red[40], rstd = sm.red[41];
  float mx = 0.0f;
  for (int i = threadIdx.x; i < C; i += CD_THREADS) {
    const float n = (src[i] - mean) * rstd;
    const float o = n * sm.lnw[i] + sm.lnb[i];
    sm.xf[i] = o;
    mx = fmaxf(mx, fabsf(o));
  }
  return mx;
}

template <int IN>
__device__ __forceinline__ float cd_local_max(const float *src) {
  float mx = 0.0f;
#pragma unroll
  for (int i = threadIdx.x; i < IN; i += CD_THREADS) mx = fmaxf(mx, fabsf(src[i]));
  return mx;
}

// quantize_rows of src[0..IN) (kernels.mojo:400-416) into sm.xq in the
// layer ranks' lane order, given each thread's max |x| (of the elements it
// read or wrote): the int16 codes of column col = blk*256 + g*32 + h*16 + e
// (lane L = g + 8h of block blk, element e; permute_x_i16, tensor.mojo:
// 498-516) go to word ((blk*8 + e/2)*4 + q)*4 + t, half e%2, where
// L = 2q + (t & 1) + 8 (t >> 1); the lane sums to sm.xs[(blk*4 + q)*4 + t].
// Thread t takes columns 4t..4t+3 (+ 1024 k): one lane's elements, so four
// threads make a lane sum. Returns sx.
template <int IN>
__device__ __noinline__ float cd_quantize_blk(CdLSmem &sm, const float *src, float mx) {
  static_assert(IN % 256 == 0 && IN <= 3072, "whole blocks");
  float s = cd_block_max(sm, mx) / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  const float inv = 1.0f / s;
  constexpr int ITER = (IN + 4 * CD_THREADS - 1) / (4 * CD_THREADS);
#pragma unroll
  for (int k = 0; k < ITER; k++) {
    const int c = 4 * threadIdx.x + 4 * CD_THREADS * k;
    if (c < IN) {  // whole warps: IN is a multiple of 256 = 2 warps x 128 columns
      const float4 v = *(const float4 *)(src + c);
      const int c0 = round_away(v.x * inv), c1 = round_away(v.y * inv);
      const int c2 = round_away(v.z * inv), c3 = round_away(v.w * inv);
      const int blk = c >> 8, w = c & 255, L = ((w >> 5) & 7) + 8 * ((w >> 4) & 1), st = (w & 15) >> 1;
      const int q = (L & 7) >> 1, t = (L & 1) + 2 * (L >> 3);
      int *dst = sm.xq + ((blk * 8 + st) * 4 + q) * 4 + t;
      dst[0] = (c0 & 0xFFFF) | (c1 << 16);
      dst[16] = (c2 & 0xFFFF) | (c3 << 16);  // step st + 1
      int sum = (c0 + c1) + (c2 + c3);
      sum += __shfl_xor_sync(0xffffffffu, sum, 1);
      sum += __shfl_xor_sync(0xffffffffu, sum, 2);
      if ((threadIdx.x & 3) == 0) sm.xs[(blk * 4 + q) * 4 + t] = sum;
    }
  }
  __syncthreads();
  return s;
}

// quantize_rows of sm.xf[0..768) into sm.xq in natural order, with the
// per-channel pair sums xs[L] = sum over the 32-column groups of columns 2L
// and 2L+1 (the head's per-channel int8 dot, tensor.mojo:541-566).
__device__ __noinline__ float cd_quantize_nat(CdHSmem &sm, float mx) {
  float s = cd_block_max(sm, mx) / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  const float inv = 1.0f / s;
  int *part = reinterpret_cast<int *>(sm.xin);  // the hidden state was read already
  int p0 = 0, p1 = 0;
  const int c = 4 * threadIdx.x;
  if (c < 768) {
    const float4 v = *(const float4 *)(sm.xf + c);
    const int c0 = round_away(v.x * inv), c1 = round_away(v.y * inv);
    const int c2 = round_away(v.z * inv), c3 = round_away(v.w * inv);
    sm.xq[c >> 1] = (c0 & 0xFFFF) | (c1 << 16);
    sm.xq[(c >> 1) + 1] = (c2 & 0xFFFF) | (c3 << 16);
    p0 = c0 + c1;
    p1 = c2 + c3;
  }
  // within a warp the threads t, t^8, t^16, t^24 hold the same pairs
  p0 += __shfl_xor_sync(0xffffffffu, p0, 8);
  p1 += __shfl_xor_sync(0xffffffffu, p1, 8);
  p0 += __shfl_xor_sync(0xffffffffu, p0, 16);
  p1 += __shfl_xor_sync(0xffffffffu, p1, 16);
  const int lane = threadIdx.x & 31;
  if (lane < 8) {
    part[(threadIdx.x >> 5) * 16 + 2 * lane] = p0;
    part[(threadIdx.x >> 5) * 16 + 2 * lane + 1] = p1;
  }
  __syncthreads();
  if (threadIdx.x < 16) {
    int sum = 0;
#pragma unroll
    for (int w = 0; w < CD_THREADS / 32; w++) sum += part[w * 16 + threadIdx.x];
    sm.xs[threadIdx.x] = sum;
  }
  __syncthreads();
  return s;
}

// --- layer ranks ------------------------------------------------------------------

// The BLOCKED int4-g32 rows of one phase against sm.xq (dot_row_i16,
// tensor.mojo:522-540), for `nsets` sets of rows of `cps` chunks each (a
// set's chunks hold the same rows and consecutive block ranges; slot[k] is
// the ring slot of chunk k). Thread item (set, row, q) keeps lanes 2q, 2q+1,
// 2q+8, 2q+9 of its row: per block the 8 steps of int32 pair products, then
// (lane - zp * lane sum of x) * scale fused into the lane's float chain in
// block order; the four threads of a row add the 16 lanes as the halving
// tree (i and i+8 in the thread, i+4 and i+2 by shuffles, i+1 in the
// thread). Row value v = dot * sx + bias (+ GELU) (+ resid[row]) goes to
// sm.outv[set * rp + row].
template <int EPI>
__device__ __noinline__ void cd_gemv(CdLSmem &sm, const int *slot, const CdChunk *ch, int nsets, int cps, float sx,
                                     const float *resid) {
  const int rp = ch[0].rp;
  const int items = nsets * rp * 4;
  for (int it = threadIdx.x; it < ((items + 31) & ~31); it += CD_THREADS) {  // whole warps (shuffles)
    const bool live = it < items;
    const int iv = live ? it : 0;
    const int set = iv / (rp * 4), r = (iv % (rp * 4)) >> 2, q = iv & 3;
    float f0 = 0.0f, f1 = 0.0f, f2 = 0.0f, f3 = 0.0f;  // lanes 2q, 2q+1, 2q+8, 2q+9
    for (int k = 0; k < cps; k++) {
      const CdChunk &c = ch[set * cps + k];
      const uint8_t *base = sm.ring[slot[set * cps + k]];
      for (int bb = 0; bb < c.nb; bb++) {
        const int b = c.b0 + bb;
        const uint4 w0 = *(const uint4 *)(base + ((bb * 2 + 0) * rp + r) * 64 + q * 16);
        const uint4 w1 = *(const uint4 *)(base + ((bb * 2 + 1) * rp + r) * 64 + q * 16);
        const unsigned wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const int4 *xv = reinterpret_cast<const int4 *>(sm.xq) + (b * 8) * 4 + q;
        int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
        for (int s = 0; s < 8; s++) {
          const unsigned lo = wv[s] & 0x0F0F0F0Fu, hi = (wv[s] >> 4) & 0x0F0F0F0Fu;
          const int4 x = xv[s * 4];
          a0 = dp2a_lo_su(x.x, lo, a0);
          a1 = dp2a_hi_su(x.y, lo, a1);
          a2 = dp2a_lo_su(x.z, hi, a2);
          a3 = dp2a_hi_su(x.w, hi, a3);
        }
        const unsigned zp2 = *(const uint16_t *)(base + c.zp_off + (bb * rp + r) * 8 + 2 * q);
        const unsigned sc2 = *(const uint32_t *)(base + c.scale_off + ((bb * rp + r) * 8 + 2 * q) * 2);
        const int za = (int)(zp2 & 0xFFu), zb = (int)(zp2 >> 8);  // groups 2q (lanes 2q, 2q+8) and 2q+1
        const float sa = __half2float(__ushort_as_half((unsigned short)(sc2 & 0xFFFFu)));
        const float sb = __half2float(__ushort_as_half((unsigned short)(sc2 >> 16)));
        const int4 xs = *reinterpret_cast<const int4 *>(sm.xs + (b * 4 + q) * 4);
        // f32(lane) - zp * f32(lane sum) is exact here (all terms below 2^24)
        f0 = fmaf((float)(a0 - za * xs.x), sa, f0);
        f1 = fmaf((float)(a1 - zb * xs.y), sb, f1);
        f2 = fmaf((float)(a2 - za * xs.z), sa, f2);
        f3 = fmaf((float)(a3 - zb * xs.w), sb, f3);
      }
    }
    const float s8a = f0 + f2, s8b = f1 + f3;  // s8[2q], s8[2q+1]
    const float s4a = s8a + __shfl_xor_sync(0xffffffffu, s8a, 2);
    const float s4b = s8b + __shfl_xor_sync(0xffffffffu, s8b, 2);  // q < 2: s4[2q], s4[2q+1]
    const float s2a = s4a + __shfl_xor_sync(0xffffffffu, s4a, 1);
    const float s2b = s4b + __shfl_xor_sync(0xffffffffu, s4b, 1);  // q == 0: s2[0], s2[1]
    const float dot = s2a + s2b;
    if (live && q == 0 && r < ch[set * cps].n) {
      const int o = set * rp + r;
      float y = dot * sx + sm.bias[o];
      if (EPI & MK_GELU) y = gelu(y);
      if (EPI & MK_RESID) y += resid[r];
      sm.outv[o] = y;
    }
  }
  __syncthreads();
}

// Pushes src[0..n) (n a multiple of 4) into dst[0..n) of every rank of the
// cluster (dst is this CTA's copy of the buffer; the same offset in each
// peer), completing bytes on each rank's barrier `bar`.
__device__ __forceinline__ void cd_push(const float *src, int n, float *dst, unsigned long long *bar) {
  const int nv = n >> 2;
  for (int i = threadIdx.x; i < nv * CD_CLUSTER; i += CD_THREADS) {
    const int p = i / nv, k = i - p * nv;
    const unsigned d = cd_mapa(smem_u32(dst + 4 * k), (unsigned)p);
    const unsigned b = cd_mapa(smem_u32(bar), (unsigned)p);
    cd_st_async_v4(d, *(const float4 *)(src + 4 * k), b);
  }
}

// Starts copying this head's cached keys, values and their scales for
// positions [0, pos) into shared memory (pos <= CD_KV_STAGE); waited for by
// cp_async_wait_all before the attention.
// Always commits one group (empty when pos > CD_KV_STAGE): the caller waits
// for the group before it with cp.async.wait_group 1.
__device__ __noinline__ void cd_kv_prefetch(const CdArgs &a, CdLSmem &sm, int l, int h, int pos) {
  if (pos > CD_KV_STAGE) {
    cp_async_commit();
    return;
  }
  const size_t row0 = ((size_t)l * a.kv.max_t) * a.kv.n_head + h;
  const size_t stride = a.kv.n_head;
  for (int i = threadIdx.x; i < pos * 8; i += CD_THREADS) {
    const int s = i >> 3, part = i & 7;
    const size_t slot = row0 + s * stride;
    if (part < 4)
      cp_async16(&sm.kst[s][part * 16], a.kv.k + slot * 64 + part * 16);
    else
      cp_async16(&sm.vst[s][(part - 4) * 16], a.kv.v + slot * 64 + (part - 4) * 16);
  }
  for (int i = threadIdx.x; i < pos * 2; i += CD_THREADS) {
    const int s = i >> 1;
    const size_t slot = row0 + s * stride;
    if (i & 1)
      cp_async4(&sm.vss[s], a.kv.vs + slot);
    else
      cp_async4(&sm.kss[s], a.kv.ks + slot);
  }
  cp_async_commit();
}

// Score of one cached position (kvcache.mojo:346-354): the 16-lane dot of q
// with the 64 key codes, the halving tree, times the key scale and 1/8.
__device__ __forceinline__ float cd_score(const float *q, const int8_t *kp, float ksc) {
  float d[16];
#pragma unroll
  for (int k = 0; k < 16; k++) d[k] = 0.0f;
#pragma unroll
  for (int i = 0; i < 64; i += 16) {
    const uint4 kv4 = *(const uint4 *)(kp + i);
    const unsigned w[4] = {kv4.x ^ 0x80808080u, kv4.y ^ 0x80808080u, kv4.z ^ 0x80808080u, kv4.w ^ 0x80808080u};
#pragma unroll
    for (int k = 0; k < 16; k++) d[k] = d[k] + q[i + k] * s8_byte_to_f(w[k >> 2], k & 3);
  }
#pragma unroll
  for (int k = 0; k < 8; k++) d[k] = d[k] + d[k + 8];
#pragma unroll
  for (int k = 0; k < 4; k++) d[k] = d[k] + d[k + 4];
  d[0] = d[0] + d[2];
  d[1] = d[1] + d[3];
  return ((d[0] + d[1]) * ksc) * 0.125f;
}

// Attention of head h (QuantKV[8]) with q, k, v in sm.outv[0..192): store
// the token's key and value (QuantKV.store, kvcache.mojo:333-342), attend
// over positions 0..pos (attend_float_one, kvcache.mojo:113-150) into
// sm.att_o. Warps 0 and 1 quantize the key and the value while warps 2-7
// score the cached positions; the softmax sum and the value chains run in
// position order as in the reference.
__device__ __noinline__ void cd_attention(const CdArgs &a, CdLSmem &sm, int l, int h, int pos) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float *q = sm.outv;
  const size_t stride_h = a.kv.n_head, base = (size_t)l * a.kv.max_t * stride_h + h;
  const size_t sl = base + (size_t)pos * stride_h;
  const bool staged = pos <= CD_KV_STAGE;
  const int npos = pos + 1;
  cp_async_wait_all();  // the staged cache
  __syncthreads();
  float mx = -__int_as_float(0x7f800000);
  if (warp < 2) {
    const float x0 = sm.outv[64 + warp * 64 + lane], x1 = sm.outv[64 + warp * 64 + lane + 32];
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
    __threadfence();  // the next token's cache staging (cp.async, L2) reads these
    if (warp == 0) {
      // the new position's score: lane k < 16 carries lane k's chain over
      // elements k, 16+k, 32+k, 48+k, then the halving tree by shuffles
      const float c0 = (float)q0, c1 = (float)q1;
      const float c16 = __shfl_down_sync(0xffffffffu, c0, 16), c48 = __shfl_down_sync(0xffffffffu, c1, 16);
      const int k = lane & 15;
      float d = 0.0f + q[k] * c0;
      d = d + q[16 + k] * c16;
      d = d + q[32 + k] * c1;
      d = d + q[48 + k] * c48;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) d = d + __shfl_xor_sync(0xffffffffu, d, o);
      if (lane == 0) {
        const float v = (d * s) * 0.125f;
        sm.att_sc[pos] = v;
        mx = v;
      }
    }
  }
  for (int s = (tid + 192) & 255; s < pos; s += CD_THREADS) {
    const size_t ss = base + (size_t)s * stride_h;
    const float v = staged ? cd_score(q, sm.kst[s], sm.kss[s]) : cd_score(q, a.kv.k + ss * 64, a.kv.ks[ss]);
    sm.att_sc[s] = v;
    mx = fmaxf(mx, v);
  }
  {
    const unsigned k = __reduce_max_sync(0xffffffffu, f2key(mx));
    if (lane == 0) ((unsigned *)sm.red)[warp] = k;
  }
  __syncthreads();
  {
    const uint4 ka = *(const uint4 *)&sm.red[0], kb = *(const uint4 *)&sm.red[4];
    mx = key2f(max(max(max(ka.x, ka.y), max(ka.z, ka.w)), max(max(kb.x, kb.y), max(kb.z, kb.w))));
  }
  for (int s = tid; s < npos; s += CD_THREADS) sm.att_sc[s] = lm_expf(sm.att_sc[s] - mx);
  __syncthreads();
  if (tid == 0) {
    // sequential sum in position order
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
  __syncthreads();
  const float total = sm.red[36];
  for (int s = tid; s < npos; s += CD_THREADS) {
    const float vsc = s == pos ? sm.red[51] : (staged ? sm.vss[s] : a.kv.vs[base + (size_t)s * stride_h]);
    sm.att_ps[s] = (sm.att_sc[s] / total) * vsc;
  }
  __syncthreads();
  if (tid < 64) {
    // acc = fma(p * vs, v, acc) over positions in order
    const int d = tid;
    float acc = 0.0f;
    if (staged) {
      int s = 0;
      if (pos >= 16) {
        const float4 *p4 = reinterpret_cast<const float4 *>(sm.att_ps);
        float pv[16], vv[16];
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float4 t = p4[k];
          pv[4 * k] = t.x;
          pv[4 * k + 1] = t.y;
          pv[4 * k + 2] = t.z;
          pv[4 * k + 3] = t.w;
        }
#pragma unroll
        for (int k = 0; k < 16; k++) vv[k] = s8_to_f(sm.vst[k][d]);
        for (; s + 32 <= pos; s += 16) {
          float np[16], nv[16];
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const float4 t = p4[(s >> 2) + 4 + k];
            np[4 * k] = t.x;
            np[4 * k + 1] = t.y;
            np[4 * k + 2] = t.z;
            np[4 * k + 3] = t.w;
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
    sm.att_o[d] = acc;
  }
  __syncthreads();
}

// Embedding of `token` at `pos` (gpt2t.mojo:378-385) into sm.b_xout.
__device__ __noinline__ void cd_embed(const CdArgs &a, CdLSmem &sm, int token, int pos) {
  const int C = a.C, gpr = a.head.cols / a.head.group;
  const float *wpe = a.small + (size_t)a.n_layer * 13 * C;
  for (int i = threadIdx.x; i < C; i += CD_THREADS) {
    const size_t gi = (size_t)token * gpr + i / a.head.group;
    const float s = __half2float(__ushort_as_half(a.head.scale[gi]));
    const float v = (float)(code_at(a.head, token, i) - (int)a.head.zp[gi]) * s;
    sm.b_xout[i] = v + wpe[(size_t)pos * C + i];
  }
  __syncthreads();
}

// Starts copying a LayerNorm's weight and bias (768 each, when given) and n
// biases into shared memory; waited for by cp_async_wait_all.
template <class SM>
__device__ __forceinline__ void cd_params(SM &sm, const float *lnw, const float *lnb) {
  if (lnw && threadIdx.x < 192) {
    cp_async16(&sm.lnw[threadIdx.x * 4], lnw + threadIdx.x * 4);
    cp_async16(&sm.lnb[threadIdx.x * 4], lnb + threadIdx.x * 4);
  }
}
__device__ __forceinline__ void cd_bias(CdLSmem &sm, int dst, const float *src, int n) {
  for (int i = threadIdx.x; i < n / 4; i += CD_THREADS) cp_async16(&sm.bias[dst + 4 * i], src + 4 * i);
}

// Reads n exchange words with flag `flag` into dst (all threads; bounded).
// With `gate`, thread 0 first waits alone for word 0, pausing between reads,
// so that CTAs which wait long (the head CTAs, for a whole token's layers)
// do not flood the L2 slices that hold the words.
template <class SM>
__device__ __noinline__ bool cd_poll(const CdArgs &a, SM &sm, const unsigned long long *src, int n, unsigned flag,
                                     float *dst, int code, bool gate = false) {
  constexpr int P = 4;  // words per thread per round (n <= P * CD_THREADS)
  long long t0 = clock64();
  const int tid = threadIdx.x;
  if (gate) {
    if (tid == 0)
      while ((unsigned)(ld_relaxed_u64(src) >> 32) != flag) {
        if (!cd_alive(a, sm, t0, code)) break;
        __nanosleep(128);
      }
    __syncthreads();
  }
  unsigned pending = 0;
#pragma unroll
  for (int k = 0; k < P; k++)
    if (tid + k * CD_THREADS < n) pending |= 1u << k;
  while (pending) {
    unsigned long long v[P];
#pragma unroll
    for (int k = 0; k < P; k++)
      if (pending & (1u << k)) v[k] = ld_relaxed_u64(src + tid + k * CD_THREADS);
#pragma unroll
    for (int k = 0; k < P; k++)
      if ((pending & (1u << k)) && (unsigned)(v[k] >> 32) == flag) {
        dst[tid + k * CD_THREADS] = __uint_as_float((unsigned)v[k]);
        pending &= ~(1u << k);
      }
    if (pending && !cd_alive(a, sm, t0, code)) break;
  }
  cp_async_wait_all();
  __syncthreads();
  return !sm.abort;
}

__device__ __noinline__ void cd_layer_rank(const CdArgs &a, CdLSmem &sm, const int rank) {
  const int tid = threadIdx.x;
  const int C = a.C, C4 = 4 * C;
  const int nch = a.lnch[rank];
  const uint8_t *stream = a.lstream + a.lbase[rank];
  const long long lbytes = a.lbytes[rank];
  const int total_chunks = nch * a.n_layer * a.steps;
  const bool head_rank = rank < a.n_head;
  const int hc = a.n_hcta;

  if (tid < nch) sm.chunks[tid] = a.lchunks[rank * CD_MAX_CHUNKS + tid];
  if (tid == 0) {
    for (int i = 0; i < CD_NSLOT; i++) mbar_init(&sm.full[i], 1);
    for (int i = 0; i < 4; i++) mbar_init(&sm.rbar[i], 1);
    sm.abort = 0;
    sm.rph_left = 0;
    int t0 = *a.first_token;
    if (t0 < 0 || t0 >= a.V) {
      atomicCAS(a.err, 0, 9);
      t0 = 0;
    }
    sm.token = t0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // bytes each receive buffer expects per phase
  const unsigned rb_bytes[4] = {(unsigned)C * 4u, (unsigned)C * 4u, (unsigned)C4 * 4u, (unsigned)C * 4u};
  if (tid == 0)
    for (int i = 0; i < 4; i++) mbar_expect_tx(&sm.rbar[i], rb_bytes[i]);
  unsigned rph = 0;  // bit i: parity of receive buffer i's current phase
  // every rank's barriers are initialised and armed before anyone pushes
  cd_cluster_sync();

  // the ring (as in mega.cuh): chunk q of the generation goes to slot
  // q % CD_NSLOT with parity (q / CD_NSLOT) & 1
  int seq = 0, rslot = 0, rpar = 0;
  int iss = 0, iss_slot = 0, iss_ci = 0, iss_layer = 0;
  auto issue = [&]() {
    const CdChunk &ch = sm.chunks[iss_ci];
    mbar_expect_tx(&sm.full[iss_slot], (unsigned)ch.bytes);
    bulk_g2s(sm.ring[iss_slot], stream + (long long)iss_layer * lbytes + ch.off, (unsigned)ch.bytes,
             &sm.full[iss_slot]);
    iss++;
    iss_slot = iss_slot + 1 == CD_NSLOT ? 0 : iss_slot + 1;
    if (++iss_ci == nch) {
      iss_ci = 0;
      iss_layer = iss_layer + 1 == a.n_layer ? 0 : iss_layer + 1;
    }
  };
  if (tid == 0)
    while (iss < CD_NSLOT && iss < total_chunks) issue();

  const bool prof_on = a.prof && rank == 0 && tid == 0;
  long long pacc[MK_PROF];
  for (int k = 0; k < MK_PROF; k++) pacc[k] = 0;
  long long tlast = clock64();
  auto tick = [&](int k) {
    if (prof_on) {
      const long long t = clock64();
      pacc[k] += t - tlast;
      tlast = t;
    }
  };
  long long tsub = 0;
  auto sub0 = [&]() {
    if (prof_on) tsub = clock64();
  };
  auto sub1 = [&](int k) {
    if (prof_on) pacc[k] += clock64() - tsub;
  };
  // waits for the next n chunks; their slots in slots[0..n)
  // (every thread waits; the result is the CTA's, after a barrier)
  auto take = [&](int n, int *slots) -> bool {
    int slot = rslot;
    unsigned par = (unsigned)rpar;
    bool good = true;
    for (int k = 0; k < n && good; k++) {
      const long long t0 = clock64();
      while (good && !mbar_try_wait(&sm.full[slot], par)) good = cd_alive(a, sm, t0, 1);
      if (prof_on) pacc[CP_RING_WAIT] += clock64() - t0;
      slots[k] = slot;
      if (++slot == CD_NSLOT) {
        slot = 0;
        par ^= 1u;
      }
    }
    __syncthreads();
    return !sm.abort;
  };
  // after the barrier that ends the use of the n slots: hand them back
  auto give = [&](int n) {
    for (int k = 0; k < n; k++) {
      if (tid == 0 && iss < total_chunks) issue();
      seq++;
      if (++rslot == CD_NSLOT) {
        rslot = 0;
        rpar ^= 1;
      }
    }
  };
  // waits for receive buffer i's current phase, then (thread 0) arms the next
  auto recv = [&](int i, int code) -> bool {
    const long long t0 = clock64();
    bool good = true;
    while (good && !cd_try_wait_cluster(&sm.rbar[i], (rph >> i) & 1u)) good = cd_alive(a, sm, t0, code);
    if (good) {
      rph ^= 1u << i;
      if (tid == 0) mbar_expect_tx(&sm.rbar[i], rb_bytes[i]);
    }
    __syncthreads();
    return !sm.abort;
  };

  bool ok = true;
  int ci = 0;  // chunk index within the layer
  int slots[4];
  const unsigned long long *part = a.ll + C;
  for (int step = 0; ok && step < a.steps; step++) {
    const unsigned flag = a.flag0 + (unsigned)step;
    const int pos = a.pos0 + step;
    cd_embed(a, sm, sm.token, pos);
    tick(CP_EMBED);
    for (int l = 0; ok && l < a.n_layer; l++) {
      const float *vec = a.small + (size_t)l * 13 * C;
      ci = 0;
      // ---- LN1 + QKV + attention (ranks 0..n_head-1) ----
      if (head_rank) {
        cd_params(sm, vec, vec + C);
        cd_bias(sm, 0, vec + 2 * C + 64 * rank, 64);
        cd_bias(sm, 64, vec + 2 * C + C + 64 * rank, 64);
        cd_bias(sm, 128, vec + 2 * C + 2 * C + 64 * rank, 64);
        cp_async_commit();
        cd_kv_prefetch(a, sm, l, rank, pos);  // its own group, waited for by the attention
        cp_async_wait_group1();
        __syncthreads();
        sub0();
        const float sx = cd_quantize_blk<768>(sm, sm.xf, cd_layernorm(sm, sm.b_xout));
        sub1(CP_QUANT);
        tick(CP_LN1);
        if (!(ok = take(3, slots))) break;
        sub0();
        cd_gemv<0>(sm, slots, sm.chunks + ci, 3, 1, sx, nullptr);
        sub1(CP_GEMV);
        give(3);
        ci += 3;
        tick(CP_QKV);
        sub0();
        cd_attention(a, sm, l, rank, pos);
        sub1(CP_ATTN_INNER);
        cd_push(sm.att_o, 64, sm.b_att + 64 * rank, &sm.rbar[RB_ATT]);
        tick(CP_ATTN);
      }
      // ---- PROJ + residual ----
      cd_bias(sm, 0, vec + 5 * C + 48 * rank, 48);
      cp_async_commit();
      if (!(ok = recv(RB_ATT, 4))) break;
      cp_async_wait_all();
      __syncthreads();
      tick(CP_HOP_ATT);
      {
        sub0();
        const float sx = cd_quantize_blk<768>(sm, sm.b_att, cd_local_max<768>(sm.b_att));
        sub1(CP_QUANT);
        if (!(ok = take(1, slots))) break;
        sub0();
        cd_gemv<MK_RESID>(sm, slots, sm.chunks + ci, 1, 1, sx, sm.b_xout + 48 * rank);
        sub1(CP_GEMV);
        give(1);
        ci += 1;
        sub0();
        cd_push(sm.outv, 48, sm.b_xmid + 48 * rank, &sm.rbar[RB_XMID]);
        sub1(CP_PUSH);
      }
      tick(CP_PROJ);
      // ---- LN2 + FC + GELU ----
      cd_params(sm, vec + 6 * C, vec + 7 * C);
      cd_bias(sm, 0, vec + 8 * C + 192 * rank, 192);
      cp_async_commit();
      if (!(ok = recv(RB_XMID, 5))) break;
      cp_async_wait_all();
      __syncthreads();
      tick(CP_HOP_XMID);
      {
        sub0();
        const float sx = cd_quantize_blk<768>(sm, sm.xf, cd_layernorm(sm, sm.b_xmid));
        sub1(CP_QUANT);
        tick(CP_LN2);
        if (!(ok = take(3, slots))) break;
        sub0();
        cd_gemv<MK_GELU>(sm, slots, sm.chunks + ci, 3, 1, sx, nullptr);
        sub1(CP_GEMV);
        give(3);
        ci += 3;
        sub0();
        cd_push(sm.outv, 192, sm.b_fc + 192 * rank, &sm.rbar[RB_FC]);
        sub1(CP_PUSH);
      }
      tick(CP_FC);
      // ---- FCPROJ + residual ----
      cd_bias(sm, 0, vec + 12 * C + 48 * rank, 48);
      cp_async_commit();
      if (!(ok = recv(RB_FC, 6))) break;
      cp_async_wait_all();
      __syncthreads();
      tick(CP_HOP_FC);
      {
        sub0();
        const float sx = cd_quantize_blk<3072>(sm, sm.b_fc, cd_local_max<3072>(sm.b_fc));
        sub1(CP_QUANT);
        if (!(ok = take(4, slots))) break;
        sub0();
        cd_gemv<MK_RESID>(sm, slots, sm.chunks + ci, 1, 4, sx, sm.b_xmid + 48 * rank);
        sub1(CP_GEMV);
        give(4);
        ci += 4;
        if (l == a.n_layer - 1 && tid < 48)  // the final hidden state for the head CTAs
          st_relaxed_u64(a.ll + 48 * rank + tid, ll_pack(sm.outv[tid], flag));
        sub0();
        cd_push(sm.outv, 48, sm.b_xout + 48 * rank, &sm.rbar[RB_XOUT]);
        sub1(CP_PUSH);
      }
      tick(CP_FCPROJ);
      if (!(ok = recv(RB_XOUT, 7))) break;
      __syncthreads();
      tick(CP_HOP_XOUT);
    }
    if (!ok) break;
    // ---- the greedy argmax over the head CTAs' candidates (gpt2t.mojo:792-797) ----
    if (!(ok = cd_poll(a, sm, part, 2 * hc, flag, sm.att_sc, 8))) break;
    tick(CP_ARGMAX_WAIT);
    if (tid < 32) {
      float v = -__int_as_float(0x7f800000);
      int i = 0x7fffffff;
      for (int c = tid; c < hc; c += 32) {
        const float cv = sm.att_sc[2 * c];
        const int cidx = __float_as_int(sm.att_sc[2 * c + 1]);
        if (better(cv, cidx, v, i)) {
          v = cv;
          i = cidx;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
          v = ov;
          i = oi;
        }
      }
      if (tid == 0) {
        if (i == 0x7fffffff) i = 0;  // every logit NaN: the scan keeps index 0
        sm.token = i;
        if (rank == 0) a.ids[step] = i;
      }
    }
    __syncthreads();
    if (prof_on) pacc[CP_STEPS] += 1;
  }

  if (!ok) {
    // give up: own copies (bounded), then the pushes this rank still expects
    cp_async_wait_all();
    if (tid == 0) {
      int slot = rslot;
      unsigned par = (unsigned)rpar;
      for (int q = seq; q < iss; q++) {
        const long long t1 = clock64();
        while (!mbar_try_wait(&sm.full[slot], par) && clock64() - t1 < kDrainCycles) {
        }
        if (++slot == CD_NSLOT) {
          slot = 0;
          par ^= 1u;
        }
      }
    }
    sm.rph_left = rph;  // the receive phases still open, drained at the kernel's end
  } else if (prof_on) {
    for (int k = 0; k < MK_PROF; k++) a.prof[k] += pacc[k];
  }
}

// --- head CTAs ----------------------------------------------------------------------

// Per-channel int8 head rows of one or two 32-row chunks (dot_row_i16 per
// channel, tensor.mojo:541-566): threads 0-127 the chunk in slot0, 128-255
// the one in slot1 (if any). Thread (r, q) accumulates lanes 4q..4q+3 of row
// r over the row's 24 column chunks; the row's four threads add the 16
// lanes as the halving tree. Chunk layout: codes [24][32 rows][4 q] x 8 B,
// then 32 float16 scales, then 32 zero points.
__device__ __noinline__ void cd_head_pair(CdHSmem &sm, const uint8_t *slot0, int r0a, int na, const uint8_t *slot1,
                                          int r0b, int nb, float sx, float *logits, float &bv, int &bi) {
  const int half = threadIdx.x >> 7;
  if (half == 1 && !slot1) return;  // whole warps
  const uint8_t *slot = half ? slot1 : slot0;
  const int R = half ? nb : na, rbase = half ? r0b : r0a;
  const int i = threadIdx.x & 127, q = i & 3, r = i >> 2;
  int acc[4] = {0, 0, 0, 0};
#pragma unroll 8
  for (int c = 0; c < 24; c++) {
    const uint2 v = *(const uint2 *)(slot + ((c * 32 + r) * 4 + q) * 8);
    const int4 xv = *(const int4 *)(sm.xq + c * 16 + 4 * q);
    acc[0] = dp2a_lo_su(xv.x, v.x, acc[0]);
    acc[1] = dp2a_hi_su(xv.y, v.x, acc[1]);
    acc[2] = dp2a_lo_su(xv.z, v.y, acc[2]);
    acc[3] = dp2a_hi_su(xv.w, v.y, acc[3]);
  }
  const int zp = slot[CD_HROWS * 768 + CD_HROWS * 2 + r];
  const float sc = __half2float(__ushort_as_half(((const uint16_t *)(slot + CD_HROWS * 768))[r]));
  float f[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int d = (int)((unsigned)acc[j] - (unsigned)(zp * sm.xs[4 * q + j]));
    f[j] = fmaf((float)d, sc, 0.0f);
  }
  float b[4];
#pragma unroll
  for (int j = 0; j < 4; j++) b[j] = f[j] + __shfl_xor_sync(0xffffffffu, f[j], 2);
#pragma unroll
  for (int j = 0; j < 4; j++) b[j] = b[j] + __shfl_xor_sync(0xffffffffu, b[j], 1);
  const float dot = (b[0] + b[2]) + (b[1] + b[3]);
  if (q == 0 && r < R) {
    const int o = rbase + r;
    const float v = dot * sx;
    if (logits) logits[o] = v;
    if (better(v, o, bv, bi)) {
      bv = v;
      bi = o;
    }
  }
}

__device__ __noinline__ void cd_head_cta(const CdArgs &a, CdHSmem &sm, const int j) {
  const int tid = threadIdx.x;
  const int C = a.C;
  const int r0 = (int)((long long)a.V * j / a.n_hcta), r1 = (int)((long long)a.V * (j + 1) / a.n_hcta);
  const int nch = (r1 - r0 + CD_HROWS - 1) / CD_HROWS;
  const uint8_t *stream = a.hstream + a.hbase[j];
  const int total_chunks = nch * a.steps;
  if (tid == 0) {
    for (int i = 0; i < CD_HNSLOT; i++) mbar_init(&sm.full[i], 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  int seq = 0, rslot = 0, rpar = 0;
  int iss = 0, iss_slot = 0, iss_ci = 0;
  auto issue = [&]() {
    mbar_expect_tx(&sm.full[iss_slot], (unsigned)CD_HSLOT);
    bulk_g2s(sm.ring[iss_slot], stream + (long long)iss_ci * CD_HSLOT, (unsigned)CD_HSLOT, &sm.full[iss_slot]);
    iss++;
    iss_slot = iss_slot + 1 == CD_HNSLOT ? 0 : iss_slot + 1;
    iss_ci = iss_ci + 1 == nch ? 0 : iss_ci + 1;
  };
  if (tid == 0)
    while (iss < CD_HNSLOT && iss < total_chunks) issue();
  const bool prof_on = a.prof && j == 0 && tid == 0;
  long long pacc[MK_PROF];
  for (int k = 0; k < MK_PROF; k++) pacc[k] = 0;
  long long tlast = clock64();
  auto tick = [&](int k) {
    if (prof_on) {
      const long long t = clock64();
      pacc[k] += t - tlast;
      tlast = t;
    }
  };
  auto slot_wait = [&](int ahead) -> int {
    int slot = rslot + ahead;
    unsigned par = (unsigned)rpar;
    if (slot >= CD_HNSLOT) {
      slot -= CD_HNSLOT;
      par ^= 1u;
    }
    const long long t0 = clock64();
    bool good = true;
    while (good && !mbar_try_wait(&sm.full[slot], par)) good = cd_alive(a, sm, t0, 1);
    if (prof_on) pacc[CH_RING_WAIT] += clock64() - t0;
    return slot;
  };
  auto slot_release = [&]() {
    if (tid == 0 && iss < total_chunks) issue();
    seq++;
    if (++rslot == CD_HNSLOT) {
      rslot = 0;
      rpar ^= 1;
    }
  };
  const float *lnf = a.small + (size_t)a.n_layer * 13 * C + (size_t)1024 * C;
  bool ok = true;
  for (int step = 0; ok && step < a.steps; step++) {
    const unsigned flag = a.flag0 + (unsigned)step;
    cd_params(sm, lnf, lnf + C);
    cp_async_commit();
    if (!(ok = cd_poll(a, sm, a.ll, C, flag, sm.xin, 3, true))) break;
    tick(CH_X_WAIT);
    const float sx = cd_quantize_nat(sm, cd_layernorm(sm, sm.xin));
    tick(CH_LN);
    float bv = -__int_as_float(0x7f800000);
    int bi = 0x7fffffff;
    for (int ci = 0; ci < nch; ci += 2) {
      const bool two = ci + 1 < nch;
      const int s0 = slot_wait(0), s1 = two ? slot_wait(1) : 0;
      __syncthreads();
      if (sm.abort) {  // read after the barrier: the same decision in every thread
        ok = false;
        break;
      }
      const int ra = r0 + ci * CD_HROWS, rb = ra + CD_HROWS;
      cd_head_pair(sm, sm.ring[s0], ra, min(CD_HROWS, r1 - ra), two ? sm.ring[s1] : nullptr, rb,
                   two ? min(CD_HROWS, r1 - rb) : 0, sx, a.logits, bv, bi);
      __syncthreads();
      slot_release();
      if (two) slot_release();
    }
    if (!ok) break;
    tick(CH_ROWS);
    // this CTA's candidate
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    if ((tid & 31) == 0) {
      sm.best_v[tid >> 5] = bv;
      sm.best_i[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < CD_THREADS / 32; w++)
        if (better(sm.best_v[w], sm.best_i[w], bv, bi)) {
          bv = sm.best_v[w];
          bi = sm.best_i[w];
        }
      st_relaxed_u64(a.ll + C + 2 * j, ll_pack(bv, flag));
      st_relaxed_u64(a.ll + C + 2 * j + 1, ((unsigned long long)flag << 32) | (unsigned)bi);
    }
    __syncthreads();
    if (prof_on) pacc[CH_STEPS] += 1;
  }
  if (!ok) {
    cp_async_wait_all();
    if (tid == 0) {
      int slot = rslot;
      unsigned par = (unsigned)rpar;
      for (int q = seq; q < iss; q++) {
        const long long t1 = clock64();
        while (!mbar_try_wait(&sm.full[slot], par) && clock64() - t1 < kDrainCycles) {
        }
        if (++slot == CD_HNSLOT) {
          slot = 0;
          par ^= 1u;
        }
      }
    }
  } else if (prof_on) {
    for (int k = 0; k < MK_PROF; k++) a.prof[MK_PROF + k] += pacc[k];
  }
}

__global__ void __launch_bounds__(CD_THREADS, 1) cluster_decode_kernel(CdArgs a) {
  extern __shared__ __align__(128) unsigned char cd_smem_raw[];
  const unsigned cl = cd_cluster_id(), rank = cd_rank();
  if (cl == 0)
    cd_layer_rank(a, *reinterpret_cast<CdLSmem *>(cd_smem_raw), (int)rank);
  else
    cd_head_cta(a, *reinterpret_cast<CdHSmem *>(cd_smem_raw), (int)((cl - 1) * CD_CLUSTER + rank));
  __syncthreads();
  // every CTA of the cluster has stopped pushing ...
  cd_cluster_sync();
  if (cl == 0) {
    // ... a layer rank that gave up waits (bounded) for the pushes it was
    // expecting that were already in flight (after a normal run every push
    // has been waited for) ...
    CdLSmem &sm = *reinterpret_cast<CdLSmem *>(cd_smem_raw);
    if (sm.abort && threadIdx.x == 0)
      for (int i = 0; i < 4; i++) {
        const long long t1 = clock64();
        while (!cd_try_wait_cluster(&sm.rbar[i], (sm.rph_left >> i) & 1u) && clock64() - t1 < kDrainCycles / 16) {
        }
      }
    __syncthreads();
  }
  // ... and no CTA leaves while a peer may still write into its shared memory
  cd_cluster_sync();
}

}  // namespace llmq
