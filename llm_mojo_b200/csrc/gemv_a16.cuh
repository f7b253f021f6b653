// W4A16 / W8A16 one-token matmul (decode GEMV) on sm_100a.
//
// Computes out[o] = act(dot_row_i16(o, x) * sx + b[o]) for the reference's
// affine formats (tensor.mojo:518-577 dot_row_i16, kernels.mojo:774-816
// linear_team / :419-458 matmul_rows_a16 T == 1):
//   - FMT_BLK4: int4, 32-weight groups, the BLOCKED layout (each 256 weights
//     are 8 steps of 16 bytes; lane i of a step holds a pair of codes of
//     group i % 8, tensor.mojo:277-288);
//   - FMT_GEN4 / FMT_GEN8: int4 (Q4_0-style nibbles) or int8 codes in
//     natural order, any group size that is a multiple of 32 (incl. per
//     channel).
// Each CTA first rebuilds the int16 activations in shared memory (optional
// LayerNorm, then quantize_rows, kernels.mojo:400-416, and for BLOCKED the
// lane order and lane sums of permute_x_i16, tensor.mojo:498-516), so no
// extra launch or global round trip is needed for them.
//
// Integer part: the int32 lane sums of the reference's 16 VPDPWSSD lanes are
// exact in any order, so 4 threads per row (thread q owns 4 of the 16
// lanes) and P threads along the row accumulate them with dp2a (s16 x u8)
// into shared memory. Float part: per row, the 16 lane chains
// accf = fma(f32(acc) [- zp * xs], scale, accf) run over the groups (or
// 256-blocks) in the reference's order, then the 16 lanes are added as a
// halving tree (SIMD.reduce_add), so every output is bit-identical to the
// reference's float32 arithmetic.
#pragma once

#include "common.cuh"

namespace llmq {

enum { FMT_BLK4 = 0, FMT_GEN4 = 1, FMT_GEN8 = 2 };
enum { PRO_QUANT = 0, PRO_LN = 1 };
enum { EPI_BIAS = 1, EPI_GELU = 2, EPI_RESID = 4 };

struct WeightView {
  const uint8_t *codes;
  const uint16_t *scale;  // float16 bits, [rows][cols / group]
  const uint8_t *zp;      // [rows][cols / group]
  int rows, cols, group;  // stored [rows = OUT, cols = IN]
  int bits, blocked;      // 4 or 8; BLOCKED int4-g32 decode layout
};

// One code of a stored matrix (QuantMatrix.code, tensor.mojo:419-429 with
// nibble_at, :385-404).
__device__ __forceinline__ int code_at(const WeightView &w, int row, int col) {
  const uint8_t *p = w.codes + (size_t)row * w.cols * w.bits / 8;
  if (w.bits == 8) return p[col];
  int j, chunk;
  if (w.blocked) {
    int ww = col & 255, e = ww & 31, pp = e >> 1;
    int lane = (ww >> 5) + 8 * (pp >> 3);
    chunk = (col >> 8) * 8 + (pp & 7);
    j = 2 * lane + (e & 1);
  } else {
    chunk = col >> 5;
    j = col & 31;
  }
  int b = p[chunk * 16 + (j & 15)];
  return j >= 16 ? (b >> 4) : (b & 0xF);
}

// Decode-step state kept on the device, so a captured graph replays with
// the token and position of the step it runs.
struct DecodeState {
  int token;        // token to embed at this step
  int pos;          // its position
  int step;         // index of the id this step produces
  int _pad;
  unsigned ticket;  // CTAs done with the head (last one reduces the argmax)
  unsigned _pad2[3];
};

struct GemvArgs {
  WeightView w;
  const float *x;            // [IN] input activations (device)
  const float *ln_w, *ln_b;  // LayerNorm parameters (PRO_LN)
  const float *bias;         // [OUT] or null
  float *out;                // [OUT] (null allowed with argmax: logits not kept)
  int epi;                   // EPI_* flags
  // argmax over the outputs (the greedy head), fused:
  float *part_val;
  int *part_idx;
  DecodeState *state;
  int *ids;                  // [steps] ids written at state->step
};

// ---------------------------------------------------------------------------
// Shared-memory layout of the activation prologue
// ---------------------------------------------------------------------------

template <int FMT>
struct SmemPlan {
  int IN;
  // offsets in bytes
  int xf, xq, xs, red, lanes, total;
  __host__ __device__ SmemPlan(int in, int group, int R) : IN(in) {
    int units = FMT == FMT_BLK4 ? in / 256 : in / group;
    xf = 0;                                // float[IN]
    xq = xf + in * 4;                      // int16[IN] (as int32 pairs)
    xs = xq + in * 2;                      // BLK4: float[IN/16]; GEN: int32[units][16]
    int xs_bytes = FMT == FMT_BLK4 ? (in / 16) * 4 : units * 16 * 4;
    red = xs + xs_bytes;                   // 64 floats of scratch
    lanes = red + 64 * 4;                  // int32[R][units][16]
    total = lanes + R * units * 16 * 4;
  }
};

// Block-wide max of non-negative floats (exact in any order).
__device__ __forceinline__ float block_max(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  __syncthreads();
  if (l == 0) red[w] = v;
  __syncthreads();
  if (w == 0) {
    v = (l < (int)(blockDim.x >> 5)) ? red[l] : 0.0f;
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (l == 0) red[32] = v;
  }
  __syncthreads();
  return red[32];
}

// 16-lane halving-tree sum, lanes 0..15 of warp 0 hold one value each; the
// result is valid in lane 0 (and, by commutativity, in every lane).
__device__ __forceinline__ float tree16_warp(float v) {
  v = v + __shfl_xor_sync(0xffffffffu, v, 8);
  v = v + __shfl_xor_sync(0xffffffffu, v, 4);
  v = v + __shfl_xor_sync(0xffffffffu, v, 2);
  v = v + __shfl_xor_sync(0xffffffffu, v, 1);
  return v;
}

// LayerNorm of one row in place (kernels.mojo:179-197): 16 lane sums, each
// sequential over the row's 16-float chunks, reduced by the halving tree.
__device__ void ln_inplace(float *xf, int C, const float *w, const float *b, float *red) {
  if (threadIdx.x < 32) {
    int l = threadIdx.x & 15;
    float s = 0.0f;
    for (int i = 0; i < C; i += 16) s = s + xf[i + l];
    float mean = tree16_warp(s) / (float)C;
    float sq = 0.0f;
    for (int i = 0; i < C; i += 16) {
      float d = xf[i + l] - mean;
      sq = sq + d * d;
    }
    float var = tree16_warp(sq) / (float)C;
    if (threadIdx.x == 0) {
      red[40] = mean;
      red[41] = 1.0f / sqrtf(var + 1e-5f);
    }
  }
  __syncthreads();
  float mean = red[40], rstd = red[41];
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    float n = (xf[i] - mean) * rstd;
    xf[i] = n * w[i] + b[i];
  }
  __syncthreads();
}

// Rebuilds the quantized activations in shared memory. Returns sx.
template <int FMT, int PRO>
__device__ float prologue(const GemvArgs &a, unsigned char *smem, const SmemPlan<FMT> &pl) {
  const int IN = pl.IN;
  float *xf = (float *)(smem + pl.xf);
  int16_t *xq = (int16_t *)(smem + pl.xq);
  float *red = (float *)(smem + pl.red);
  for (int i = threadIdx.x; i < IN; i += blockDim.x) xf[i] = a.x[i];
  __syncthreads();
  if (PRO == PRO_LN) ln_inplace(xf, IN, a.ln_w, a.ln_b, red);
  float mx = 0.0f;
  for (int i = threadIdx.x; i < IN; i += blockDim.x) mx = fmaxf(mx, fabsf(xf[i]));
  mx = block_max(mx, red);
  float s = mx / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  float inv = 1.0f / s;
  if (FMT == FMT_BLK4) {
    // permute_x_i16: column k goes to blk*256 + step*32 + 2*lane + e%2.
    for (int col = threadIdx.x; col < IN; col += blockDim.x) {
      int blk = col >> 8, w = col & 255, e = w & 31, p = e >> 1;
      int lane = (w >> 5) + 8 * (p >> 3);
      xq[blk * 256 + (p & 7) * 32 + 2 * lane + (e & 1)] = (int16_t)roundf(xf[col] * inv);
    }
    __syncthreads();
    // lane sums: lane L of block blk covers group L%8, half L/8: 16 columns.
    float *xs = (float *)(smem + pl.xs);
    for (int i = threadIdx.x; i < IN / 16; i += blockDim.x) {
      int blk = i >> 4, lane = i & 15;
      int base = blk * 256 + (lane & 7) * 32 + (lane >> 3) * 16;
      int sum = 0;
      for (int e = 0; e < 16; e++) sum += (int)roundf(xf[base + e] * inv);
      xs[i] = (float)sum;
    }
  } else {
    for (int i = threadIdx.x; i < IN; i += blockDim.x) xq[i] = (int16_t)roundf(xf[i] * inv);
    __syncthreads();
    // per (group, lane) sums of the lane's activation pairs, for the zero point.
    int G = a.w.group, units = IN / G;
    int *xsum = (int *)(smem + pl.xs);
    for (int i = threadIdx.x; i < units * 16; i += blockDim.x) {
      int g = i >> 4, L = i & 15, sum = 0;
      for (int k0 = g * G; k0 < (g + 1) * G; k0 += 32) sum += (int)xq[k0 + 2 * L] + (int)xq[k0 + 2 * L + 1];
      xsum[i] = sum;
    }
  }
  __syncthreads();
  return s;
}

// Lanes owned by thread q (0..3) of a row.
template <int FMT>
__device__ __forceinline__ int lane_of(int q, int j) {
  if (FMT == FMT_GEN8) return 4 * q + j;                      // bytes 8q..8q+7
  return (j < 2) ? (2 * q + j) : (2 * q + 8 + (j - 2));       // int4: low / high nibbles of word q
}

// Integer phase for one row and part: adds this thread's 4 lane sums per
// unit (256-block or group) into lanes[unit][16].
template <int FMT, int P>
__device__ __forceinline__ void int_phase(const WeightView &w, int row, int q, int p, const int *xp32,
                                          int *lanes) {
  if (FMT == FMT_BLK4) {
    const int nblk = w.cols >> 8;
    const uint8_t *rp = w.codes + (size_t)row * (w.cols >> 1);
    for (int b = p; b < nblk; b += P) {
      int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
      const uint32_t *wp = (const uint32_t *)(rp + b * 128) + q;
      uint32_t wv[8];
#pragma unroll
      for (int s = 0; s < 8; s++) wv[s] = __ldg(wp + 4 * s);
#pragma unroll
      for (int s = 0; s < 8; s++) {
        uint32_t lo = wv[s] & 0x0F0F0F0Fu, hi = (wv[s] >> 4) & 0x0F0F0F0Fu;
        const int *xs = xp32 + b * 128 + s * 16;
        a0 = dp2a_lo_su(xs[2 * q], lo, a0);
        a1 = dp2a_hi_su(xs[2 * q + 1], lo, a1);
        a2 = dp2a_lo_su(xs[2 * q + 8], hi, a2);
        a3 = dp2a_hi_su(xs[2 * q + 9], hi, a3);
      }
      int *ln = lanes + b * 16;
      ln[2 * q] = a0;
      ln[2 * q + 1] = a1;
      ln[2 * q + 8] = a2;
      ln[2 * q + 9] = a3;
    }
  } else if (FMT == FMT_GEN8 && w.group == w.cols) {
    // per-channel int8: one group, so the part's chunks are read 8 at a
    // time with all loads in flight, then accumulated
    const int nch = w.cols >> 5;
    const uint8_t *rp = w.codes + (size_t)row * w.cols;
    const int c0 = (nch * p) / P, c1 = (nch * (p + 1)) / P;
    int a[4] = {0, 0, 0, 0};
    for (int cb = c0; cb < c1; cb += 8) {
      uint2 v[8];
#pragma unroll
      for (int k = 0; k < 8; k++)
        if (cb + k < c1) v[k] = __ldg((const uint2 *)(rp + (cb + k) * 32) + q);
#pragma unroll
      for (int k = 0; k < 8; k++) {
        if (cb + k < c1) {
          const int *xs = xp32 + (cb + k) * 16;
          a[0] = dp2a_lo_su(xs[4 * q], v[k].x, a[0]);
          a[1] = dp2a_hi_su(xs[4 * q + 1], v[k].x, a[1]);
          a[2] = dp2a_lo_su(xs[4 * q + 2], v[k].y, a[2]);
          a[3] = dp2a_hi_su(xs[4 * q + 3], v[k].y, a[3]);
        }
      }
    }
    if (c0 < c1) {
#pragma unroll
      for (int j = 0; j < 4; j++) atomicAdd(&lanes[lane_of<FMT>(q, j)], a[j]);
    }
  } else {
    const int G = w.group, nch = w.cols >> 5;
    const int bits = FMT == FMT_GEN8 ? 8 : 4;
    const uint8_t *rp = w.codes + (size_t)row * w.cols * bits / 8;
    int c0 = (nch * p) / P, c1 = (nch * (p + 1)) / P;
    int a[4] = {0, 0, 0, 0};
    int g_cur = (c0 * 32) / G;
    for (int c = c0; c < c1; c++) {
      int g = (c * 32) / G;
      if (g != g_cur) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          atomicAdd(&lanes[g_cur * 16 + lane_of<FMT>(q, j)], a[j]);
          a[j] = 0;
        }
        g_cur = g;
      }
      const int *xs = xp32 + c * 16;
      if (FMT == FMT_GEN8) {
        uint2 v = __ldg((const uint2 *)(rp + c * 32) + q);
        a[0] = dp2a_lo_su(xs[4 * q], v.x, a[0]);
        a[1] = dp2a_hi_su(xs[4 * q + 1], v.x, a[1]);
        a[2] = dp2a_lo_su(xs[4 * q + 2], v.y, a[2]);
        a[3] = dp2a_hi_su(xs[4 * q + 3], v.y, a[3]);
      } else {
        uint32_t v = __ldg((const uint32_t *)(rp + c * 16) + q);
        uint32_t lo = v & 0x0F0F0F0Fu, hi = (v >> 4) & 0x0F0F0F0Fu;
        a[0] = dp2a_lo_su(xs[2 * q], lo, a[0]);
        a[1] = dp2a_hi_su(xs[2 * q + 1], lo, a[1]);
        a[2] = dp2a_lo_su(xs[2 * q + 8], hi, a[2]);
        a[3] = dp2a_hi_su(xs[2 * q + 9], hi, a[3]);
      }
    }
    if (c0 < c1) {
#pragma unroll
      for (int j = 0; j < 4; j++) atomicAdd(&lanes[g_cur * 16 + lane_of<FMT>(q, j)], a[j]);
    }
  }
}

template <int FMT>
__device__ __forceinline__ float tree_lanes(const float f[4]);

// Float phase: the 4 lane chains of thread q over the row's units, then the
// halving tree across the 4 threads of the row. Returns dot_row_i16.
template <int FMT>
__device__ __forceinline__ float float_phase(const WeightView &w, int row, int q, const int *lanes,
                                             const unsigned char *smem, const SmemPlan<FMT> &pl) {
  float f[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (FMT == FMT_BLK4) {
    const int nblk = w.cols >> 8, gpr = w.cols >> 5;
    const float *xs = (const float *)(smem + pl.xs);
    for (int b = 0; b < nblk; b++) {
      size_t g0 = (size_t)row * gpr + b * 8;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        int L = lane_of<FMT>(q, j);
        float zp = (float)w.zp[g0 + (L & 7)];
        float sc = half_bits_to_float(w.scale[g0 + (L & 7)]);
        f[j] = fmaf((float)lanes[b * 16 + L] - zp * xs[b * 16 + L], sc, f[j]);
      }
    }
  } else {
    const int G = w.group, gpr = w.cols / G;
    const int *xsum = (const int *)(smem + pl.xs);
    for (int g = 0; g < gpr; g++) {
      size_t gi = (size_t)row * gpr + g;
      int zp = w.zp[gi];
      float sc = half_bits_to_float(w.scale[gi]);
#pragma unroll
      for (int j = 0; j < 4; j++) {
        int L = lane_of<FMT>(q, j);
        int acc = (int)((unsigned)lanes[g * 16 + L] - (unsigned)(zp * xsum[g * 16 + L]));
        f[j] = fmaf((float)acc, sc, f[j]);
      }
    }
  }
  return tree_lanes<FMT>(f);
}

// Halving tree over a row's 16 lane chains, 4 per thread in 4 consecutive
// threads (thread q holds lanes lane_of(q, 0..3)).
template <int FMT>
__device__ __forceinline__ float tree_lanes(const float f[4]) {
  if (FMT == FMT_GEN8) {
    // lanes 4q..4q+3: level 1 pairs thread q with q^2, level 2 q with q^1.
    float a[4];
#pragma unroll
    for (int j = 0; j < 4; j++) a[j] = f[j] + __shfl_xor_sync(0xffffffffu, f[j], 2);
#pragma unroll
    for (int j = 0; j < 4; j++) a[j] = a[j] + __shfl_xor_sync(0xffffffffu, a[j], 1);
    float c0 = a[0] + a[2], c1 = a[1] + a[3];
    return c0 + c1;
  } else {
    // lanes 2q, 2q+1, 2q+8, 2q+9: level 1 inside the thread, then q^2, q^1.
    float a0 = f[0] + f[2], a1 = f[1] + f[3];
    a0 = a0 + __shfl_xor_sync(0xffffffffu, a0, 2);
    a1 = a1 + __shfl_xor_sync(0xffffffffu, a1, 2);
    float c0 = a0 + __shfl_xor_sync(0xffffffffu, a0, 1);
    float c1 = a1 + __shfl_xor_sync(0xffffffffu, a1, 1);
    return c0 + c1;
  }
}

// argmax candidate order: larger value wins, equal values go to the lower
// index (the reference's strict > scan, gpt2t.mojo:792-797); NaN never wins.
__device__ __forceinline__ bool better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

__device__ __forceinline__ void block_argmax_finish(const GemvArgs &a, float best_v, int best_i, float *red);

// One-token GEMV. CTA = R rows x P parts x 4 threads; the CTA loops over
// row tiles with a grid stride.
template <int FMT, int PRO, int R, int P, bool ARGMAX>
__global__ void __launch_bounds__(R * P * 4) gemv_a16_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  SmemPlan<FMT> pl(a.w.cols, a.w.group, R);
  const float sx = prologue<FMT, PRO>(a, smem, pl);
  const int units = FMT == FMT_BLK4 ? a.w.cols >> 8 : a.w.cols / a.w.group;
  int *lanes_all = (int *)(smem + pl.lanes);
  const int *xp32 = (const int *)(smem + pl.xq);
  const int t = threadIdx.x, q = t & 3, p = (t >> 2) % P, r = (t >> 2) / P;
  float best_v = -__int_as_float(0x7f800000);
  int best_i = 0x7fffffff;

  for (int row0 = blockIdx.x * R; row0 < a.w.rows; row0 += gridDim.x * R) {
    for (int i = t; i < R * units * 16; i += blockDim.x) lanes_all[i] = 0;
    __syncthreads();
    const int row = row0 + r;
    int *lanes = lanes_all + r * units * 16;
    if (row < a.w.rows) int_phase<FMT, P>(a.w, row, q, p, xp32, lanes);
    __syncthreads();
    const int rr = row < a.w.rows ? row : a.w.rows - 1;
    float dot = float_phase<FMT>(a.w, rr, q, lanes, smem, pl);
    if (row < a.w.rows && q == 0 && p == 0) {
      float v = dot * sx;
      if (a.epi & EPI_BIAS) v += a.bias[row];
      if (a.epi & EPI_GELU) v = gelu(v);
      if (a.epi & EPI_RESID) v += a.out[row];
      if (a.out) a.out[row] = v;
      if (ARGMAX && better(v, row, best_v, best_i)) {
        best_v = v;
        best_i = row;
      }
    }
    __syncthreads();
  }

  if (ARGMAX) block_argmax_finish(a, best_v, best_i, (float *)(smem + pl.red));
}

// ---------------------------------------------------------------------------
// Tall matrices (the vocabulary head): whole rows per 4 threads
// ---------------------------------------------------------------------------
// Thread q of a row holds lanes lane_of(q, 0..3) over the WHOLE row, so the
// integer lane sums, the float chains over the row's units (groups or
// 256-blocks, in the reference's order) and the halving tree all stay in
// registers and no warp waits for another after the prologue. A warp takes
// 8 rows at a time. Rows are read in slabs of 256 columns (8 chunks of 32):
// the next slab's codes, scales and zero points are in flight while the
// current slab is summed, and the first slab is requested before the
// prologue so that its latency hides behind it. Group ends are tracked by a
// cursor (no division per chunk). Same sums in the same order as
// gemv_a16_kernel, so the outputs are identical.

constexpr int kTallWarps = 8;
constexpr int kTallMinBlocks = 3;

template <int FMT>
struct TallSlab {
  uint32_t c[FMT == FMT_GEN8 ? 16 : 8];  // codes: chunk k in c[2k], c[2k+1] (int8) or c[k] (int4)
  uint32_t sc[4];                        // f16 bits of entry k at bits 16 * (k % 2) of sc[k / 2]
  uint32_t zp[2];                        // zero point of entry k at bits 8 * (k % 4) of zp[k / 4]
  uint32_t ends;                         // GEN: bit k set when chunk k of the slab ends a group
  int g;                                 // GEN: group of the slab's first chunk
};
// Entries: BLK4, the groups 2q and 2q + 1 of the 256-block; GEN, the group
// that ends at chunk k of the slab (if one does).

struct TallGeo {
  int nch, cpg, gpr;  // 32-column chunks per row, chunks per group, groups per row
};

// Loads slab s of a row; cg / crem: the loader's group cursor (group index
// and chunks of it seen so far), reset at the row's first slab.
template <int FMT>
__device__ __forceinline__ void tall_load(const WeightView &w, const TallGeo &geo, int row, int s, int q, int &cg,
                                          int &crem, TallSlab<FMT> &d) {
  if (FMT == FMT_BLK4) {
    const uint32_t *wp = (const uint32_t *)(w.codes + (size_t)row * (w.cols >> 1) + s * 128) + q;
#pragma unroll
    for (int k = 0; k < 8; k++) d.c[k] = __ldg(wp + 4 * k);
    const size_t g0 = (size_t)row * geo.gpr + s * 8 + 2 * q;
    d.sc[0] = __ldg((const uint32_t *)(w.scale + g0));
    d.zp[0] = __ldg((const uint16_t *)(w.zp + g0));
  } else {
    const int cb = FMT == FMT_GEN8 ? 32 : 16;
    const uint8_t *rp = w.codes + ((size_t)row * geo.nch + s * 8) * cb;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      if (s * 8 + k < geo.nch) {
        if (FMT == FMT_GEN8) {
          const uint2 v = __ldg((const uint2 *)(rp + k * 32) + q);
          d.c[2 * k] = v.x;
          d.c[2 * k + 1] = v.y;
        } else {
          d.c[k] = __ldg((const uint32_t *)(rp + k * 16) + q);
        }
      }
    }
    if (s == 0) {
      cg = 0;
      crem = 0;
    }
    d.g = cg;
    d.ends = 0;
#pragma unroll
    for (int k = 0; k < 4; k++) d.sc[k] = 0;
    d.zp[0] = d.zp[1] = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      if (s * 8 + k < geo.nch && ++crem == geo.cpg) {
        const size_t gi = (size_t)row * geo.gpr + cg;
        d.sc[k >> 1] |= (uint32_t)__ldg(w.scale + gi) << (16 * (k & 1));
        d.zp[k >> 2] |= (uint32_t)__ldg(w.zp + gi) << (8 * (k & 3));
        d.ends |= 1u << k;
        cg++;
        crem = 0;
      }
    }
  }
}

// Sums slab s of this thread's row into the integer lanes acc (GEN: the open
// group) and folds finished units into the float chains f.
template <int FMT>
__device__ __forceinline__ void tall_sum(const TallGeo &geo, int s, int q, const TallSlab<FMT> &d, const int *xp32,
                                         const unsigned char *smem, const SmemPlan<FMT> &pl, int acc[4], float f[4]) {
  if (FMT == FMT_BLK4) {
    int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const uint32_t lo = d.c[k] & 0x0F0F0F0Fu, hi = (d.c[k] >> 4) & 0x0F0F0F0Fu;
      const int2 xa = *(const int2 *)(xp32 + s * 128 + k * 16 + 2 * q);
      const int2 xb = *(const int2 *)(xp32 + s * 128 + k * 16 + 2 * q + 8);
      a0 = dp2a_lo_su(xa.x, lo, a0);
      a1 = dp2a_hi_su(xa.y, lo, a1);
      a2 = dp2a_lo_su(xb.x, hi, a2);
      a3 = dp2a_hi_su(xb.y, hi, a3);
    }
    // lanes 2q, 2q + 1, 2q + 8, 2q + 9 belong to groups 2q, 2q + 1, 2q, 2q + 1
    const float *xsf = (const float *)(smem + pl.xs) + s * 16;
    const float zp0 = (float)(d.zp[0] & 0xFFu), zp1 = (float)((d.zp[0] >> 8) & 0xFFu);
    const float sc0 = half_bits_to_float((uint16_t)(d.sc[0] & 0xFFFFu));
    const float sc1 = half_bits_to_float((uint16_t)(d.sc[0] >> 16));
    f[0] = fmaf((float)a0 - zp0 * xsf[2 * q], sc0, f[0]);
    f[1] = fmaf((float)a1 - zp1 * xsf[2 * q + 1], sc1, f[1]);
    f[2] = fmaf((float)a2 - zp0 * xsf[2 * q + 8], sc0, f[2]);
    f[3] = fmaf((float)a3 - zp1 * xsf[2 * q + 9], sc1, f[3]);
  } else {
    const int *xsum = (const int *)(smem + pl.xs);
    int g = d.g;
#pragma unroll
    for (int k = 0; k < 8; k++) {
      const int c = s * 8 + k;
      if (c < geo.nch) {
        if (FMT == FMT_GEN8) {
          const int4 xv = *(const int4 *)(xp32 + c * 16 + 4 * q);
          acc[0] = dp2a_lo_su(xv.x, d.c[2 * k], acc[0]);
          acc[1] = dp2a_hi_su(xv.y, d.c[2 * k], acc[1]);
          acc[2] = dp2a_lo_su(xv.z, d.c[2 * k + 1], acc[2]);
          acc[3] = dp2a_hi_su(xv.w, d.c[2 * k + 1], acc[3]);
        } else {
          const uint32_t lo = d.c[k] & 0x0F0F0F0Fu, hi = (d.c[k] >> 4) & 0x0F0F0F0Fu;
          const int2 xa = *(const int2 *)(xp32 + c * 16 + 2 * q);
          const int2 xb = *(const int2 *)(xp32 + c * 16 + 2 * q + 8);
          acc[0] = dp2a_lo_su(xa.x, lo, acc[0]);
          acc[1] = dp2a_hi_su(xa.y, lo, acc[1]);
          acc[2] = dp2a_lo_su(xb.x, hi, acc[2]);
          acc[3] = dp2a_hi_su(xb.y, hi, acc[3]);
        }
        if ((d.ends >> k) & 1u) {  // the group ends with this chunk: fold it into the lane chains
          const int zp = (int)((d.zp[k >> 2] >> (8 * (k & 3))) & 0xFFu);
          const float sc = half_bits_to_float((uint16_t)((d.sc[k >> 1] >> (16 * (k & 1))) & 0xFFFFu));
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int v = (int)((unsigned)acc[j] - (unsigned)(zp * xsum[g * 16 + lane_of<FMT>(q, j)]));
            f[j] = fmaf((float)v, sc, f[j]);
            acc[j] = 0;
          }
          g++;
        }
      }
    }
  }
}

template <int FMT, int PRO, bool ARGMAX>
__global__ void __launch_bounds__(kTallWarps * 32, kTallMinBlocks) gemv_tall_kernel(GemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  SmemPlan<FMT> pl(a.w.cols, a.w.group, 0);
  const int t = threadIdx.x, q = t & 3, rw = (t & 31) >> 2;
  const int rows = a.w.rows;
  TallGeo geo;
  geo.nch = a.w.cols >> 5;
  geo.cpg = FMT == FMT_BLK4 ? 1 : a.w.group >> 5;
  geo.gpr = FMT == FMT_BLK4 ? a.w.cols >> 5 : a.w.cols / a.w.group;
  const int nslab = FMT == FMT_BLK4 ? a.w.cols >> 8 : (geo.nch + 7) >> 3;
  const int n8 = (rows + 7) >> 3, stride = gridDim.x * kTallWarps;
  int rg = blockIdx.x * kTallWarps + (t >> 5), s = 0, cg = 0, crem = 0;
  TallSlab<FMT> A, B;
  if (rg < n8) tall_load<FMT>(a.w, geo, min(rg * 8 + rw, rows - 1), 0, q, cg, crem, A);
  const float sx = prologue<FMT, PRO>(a, smem, pl);
  const int *xp32 = (const int *)(smem + pl.xq);
  float best_v = -__int_as_float(0x7f800000);
  int best_i = 0x7fffffff;
  float f[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int acc[4] = {0, 0, 0, 0};
  // one slab: request the next position's slab into nx, sum cur, finish the
  // row after its last slab
  auto step = [&](const TallSlab<FMT> &cur, TallSlab<FMT> &nx) {
    int ns = s + 1, nrg = rg;
    if (ns == nslab) {
      ns = 0;
      nrg += stride;
    }
    if (nrg < n8) tall_load<FMT>(a.w, geo, min(nrg * 8 + rw, rows - 1), ns, q, cg, crem, nx);
    tall_sum<FMT>(geo, s, q, cur, xp32, smem, pl, acc, f);
    if (ns == 0) {
      const float dot = tree_lanes<FMT>(f);
      const int row = rg * 8 + rw;
      if (q == 0 && row < rows) {
        float v = dot * sx;
        if (a.epi & EPI_BIAS) v += a.bias[row];
        if (a.epi & EPI_GELU) v = gelu(v);
        if (a.epi & EPI_RESID) v += a.out[row];
        if (a.out) a.out[row] = v;
        if (ARGMAX && better(v, row, best_v, best_i)) {
          best_v = v;
          best_i = row;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        f[j] = 0.0f;
        acc[j] = 0;
      }
    }
    s = ns;
    rg = nrg;
  };
  while (rg < n8) {
    step(A, B);
    if (rg >= n8) break;
    step(B, A);
  }
  if (ARGMAX) block_argmax_finish(a, best_v, best_i, (float *)(smem + pl.red));
}

// ---------------------------------------------------------------------------
// Tall matrices in the head formats: per-warp cp.async rings
// ---------------------------------------------------------------------------
// For per-channel int8 (the head of config 0) and BLOCKED int4-g32 with
// whole 256-column slabs: the same whole-row threads as gemv_tall_kernel,
// but each warp streams its units (8 rows x one slab) through a private
// ring of NSTG shared-memory stages filled by 16-byte cp.async copies, so
// NSTG - 1 units are in flight per warp without holding registers. Each
// warp waits only for its own copies (cp.async.wait_group + __syncwarp);
// there are no mbarriers and no block-wide waits after the prologue. Rows
// in a stage are padded so that a warp's 8 rows fall in different banks.
// Same sums in the same order as gemv_a16_kernel.

constexpr int kRingWarps = 8;
constexpr int kRingBlocks = 2;  // CTAs per SM that the rings are sized for

template <int FMT>
struct Ring {
  static constexpr int RB = FMT == FMT_GEN8 ? 256 : 128;            // code bytes per row and slab
  static constexpr int RS = RB + (FMT == FMT_GEN8 ? 32 : 16);       // padded row stride in a stage
  static constexpr int SCO = 8 * RS;                                // scales: BLK4 16 B per row; int8-ch 8 halves
  static constexpr int ZPO = SCO + (FMT == FMT_BLK4 ? 8 * 16 : 16);  // zero points: BLK4 8 B per row; int8-ch 8 B
  static constexpr int STAGE = (ZPO + (FMT == FMT_BLK4 ? 8 * 8 : 8) + 15) & ~15;
  static constexpr int NSTG = FMT == FMT_GEN8 ? 5 : 8;
};

template <int FMT>
__host__ __device__ inline int ring_smem(int in, int group) {
  return ((SmemPlan<FMT>(in, group, 0).total + 15) & ~15) + kRingWarps * Ring<FMT>::NSTG * Ring<FMT>::STAGE;
}

__device__ __forceinline__ void cp16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp8(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

template <int FMT, int PRO, bool ARGMAX>
__global__ void __launch_bounds__(kRingWarps * 32, kRingBlocks) gemv_ring_kernel(GemvArgs a) {
  using R = Ring<FMT>;
  extern __shared__ __align__(16) unsigned char smem[];
  SmemPlan<FMT> pl(a.w.cols, a.w.group, 0);
  const int t = threadIdx.x, q = t & 3, rw = (t & 31) >> 2, lane = t & 31, warp = t >> 5;
  const int rows = a.w.rows, in = a.w.cols, gpr = in >> 5;
  const int nslab = in >> 8, n8 = (rows + 7) >> 3;
  const int gw = blockIdx.x * kRingWarps + warp, nw = gridDim.x * kRingWarps;
  const int units = gw < n8 ? ((n8 - 1 - gw) / nw + 1) * nslab : 0;
  uint8_t *ring = smem + ((pl.total + 15) & ~15) + (size_t)warp * R::NSTG * R::STAGE;

  // copies unit (row group rg, slab s) into stage st
  auto issue = [&](int rg, int s, uint8_t *st) {
    const int row0 = rg * 8;
    if (FMT == FMT_GEN8) {
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int pc = lane + 32 * i, r = pc >> 4, c = pc & 15;
        const int row = min(row0 + r, rows - 1);
        cp16(st + r * R::RS + c * 16, a.w.codes + (size_t)row * in + s * 256 + c * 16);
      }
      if (row0 + 8 <= rows) {
        if (lane == 0) cp16(st + R::SCO, a.w.scale + row0);
        if (lane == 1) cp8(st + R::ZPO, a.w.zp + row0);
      } else if (lane < 8) {  // the last, partial row group: plain loads of the rows that exist
        const int row = min(row0 + lane, rows - 1);
        ((uint16_t *)(st + R::SCO))[lane] = a.w.scale[row];
        st[R::ZPO + lane] = a.w.zp[row];
      }
    } else {
#pragma unroll
      for (int i = 0; i < 2; i++) {
        const int pc = lane + 32 * i, r = pc >> 3, c = pc & 7;
        const int row = min(row0 + r, rows - 1);
        cp16(st + r * R::RS + c * 16, a.w.codes + (size_t)row * (in >> 1) + s * 128 + c * 16);
      }
      if (lane < 16) {
        const int r = lane & 7, row = min(row0 + r, rows - 1);
        const size_t g0 = (size_t)row * gpr + s * 8;
        if (lane < 8)
          cp16(st + R::SCO + r * 16, a.w.scale + g0);
        else
          cp8(st + R::ZPO + r * 8, a.w.zp + g0);
      }
    }
  };
  int irg = gw, is = 0;  // next unit to issue
  auto issue_next = [&](int k) {
    if (k < units) {
      issue(irg, is, ring + (k % R::NSTG) * R::STAGE);
      if (++is == nslab) {
        is = 0;
        irg += nw;
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  for (int k = 0; k < R::NSTG - 1; k++) issue_next(k);
  const float sx = prologue<FMT, PRO>(a, smem, pl);
  const int *xp32 = (const int *)(smem + pl.xq);
  float best_v = -__int_as_float(0x7f800000);
  int best_i = 0x7fffffff;
  float f[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  int acc[4] = {0, 0, 0, 0};
  int rg = gw, s = 0;
  for (int u = 0; u < units; u++) {
    issue_next(u + R::NSTG - 1);
    asm volatile("cp.async.wait_group %0;" ::"n"(R::NSTG - 1) : "memory");
    __syncwarp();
    const uint8_t *st = ring + (u % R::NSTG) * R::STAGE;
    const uint8_t *rp = st + rw * R::RS;
    if (FMT == FMT_GEN8) {
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const uint2 v = *(const uint2 *)(rp + k * 32 + q * 8);
        const int4 xv = *(const int4 *)(xp32 + (s * 8 + k) * 16 + 4 * q);
        acc[0] = dp2a_lo_su(xv.x, v.x, acc[0]);
        acc[1] = dp2a_hi_su(xv.y, v.x, acc[1]);
        acc[2] = dp2a_lo_su(xv.z, v.y, acc[2]);
        acc[3] = dp2a_hi_su(xv.w, v.y, acc[3]);
      }
      if (s == nslab - 1) {  // one group per row: fold it
        const int *xsum = (const int *)(smem + pl.xs);
        const int zp = (int)st[R::ZPO + rw];
        const float sc = half_bits_to_float(((const uint16_t *)(st + R::SCO))[rw]);
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int v = (int)((unsigned)acc[j] - (unsigned)(zp * xsum[lane_of<FMT>(q, j)]));
          f[j] = fmaf((float)v, sc, f[j]);
        }
      }
    } else {
      int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
      for (int k = 0; k < 8; k++) {
        const uint32_t v = *(const uint32_t *)(rp + k * 16 + q * 4);
        const uint32_t lo = v & 0x0F0F0F0Fu, hi = (v >> 4) & 0x0F0F0F0Fu;
        const int2 xa = *(const int2 *)(xp32 + s * 128 + k * 16 + 2 * q);
        const int2 xb = *(const int2 *)(xp32 + s * 128 + k * 16 + 2 * q + 8);
        a0 = dp2a_lo_su(xa.x, lo, a0);
        a1 = dp2a_hi_su(xa.y, lo, a1);
        a2 = dp2a_lo_su(xb.x, hi, a2);
        a3 = dp2a_hi_su(xb.y, hi, a3);
      }
      // lanes 2q, 2q + 1, 2q + 8, 2q + 9 belong to groups 2q, 2q + 1, 2q, 2q + 1
      const uint32_t scw = *(const uint32_t *)(st + R::SCO + rw * 16 + 4 * q);
      const uint32_t zpw = *(const uint16_t *)(st + R::ZPO + rw * 8 + 2 * q);
      const float zp0 = (float)(zpw & 0xFFu), zp1 = (float)(zpw >> 8);
      const float sc0 = half_bits_to_float((uint16_t)(scw & 0xFFFFu)), sc1 = half_bits_to_float((uint16_t)(scw >> 16));
      const float *xs = (const float *)(smem + pl.xs) + s * 16;
      f[0] = fmaf((float)a0 - zp0 * xs[2 * q], sc0, f[0]);
      f[1] = fmaf((float)a1 - zp1 * xs[2 * q + 1], sc1, f[1]);
      f[2] = fmaf((float)a2 - zp0 * xs[2 * q + 8], sc0, f[2]);
      f[3] = fmaf((float)a3 - zp1 * xs[2 * q + 9], sc1, f[3]);
    }
    if (s == nslab - 1) {
      const float dot = tree_lanes<FMT>(f);
      const int row = rg * 8 + rw;
      if (q == 0 && row < rows) {
        float v = dot * sx;
        if (a.epi & EPI_BIAS) v += a.bias[row];
        if (a.epi & EPI_GELU) v = gelu(v);
        if (a.epi & EPI_RESID) v += a.out[row];
        if (a.out) a.out[row] = v;
        if (ARGMAX && better(v, row, best_v, best_i)) {
          best_v = v;
          best_i = row;
        }
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        f[j] = 0.0f;
        acc[j] = 0;
      }
      s = 0;
      rg += nw;
    } else {
      s++;
    }
    __syncwarp();  // the stage is read: it may be refilled
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  if (ARGMAX) block_argmax_finish(a, best_v, best_i, (float *)(smem + pl.red));
}

// The fused greedy head's argmax: block reduction of the threads'
// candidates, one partial per CTA, and the last CTA to finish reduces the
// partials in CTA order and advances the decode state.
__device__ __forceinline__ void block_argmax_finish(const GemvArgs &a, float best_v, int best_i, float *red) {
  const int t = threadIdx.x;
  {
    int *redi = (int *)(red + 32);
    // warp reduce
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
      int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
      if (better(ov, oi, best_v, best_i)) {
        best_v = ov;
        best_i = oi;
      }
    }
    if ((t & 31) == 0) {
      red[t >> 5] = best_v;
      redi[t >> 5] = best_i;
    }
    __syncthreads();
    if (t == 0) {
      for (int w = 1; w < (int)(blockDim.x >> 5); w++)
        if (better(red[w], redi[w], best_v, best_i)) {
          best_v = red[w];
          best_i = redi[w];
        }
      a.part_val[blockIdx.x] = best_v;
      a.part_idx[blockIdx.x] = best_i;
      __threadfence();
      unsigned done = atomicAdd(&a.state->ticket, 1u);
      if (done == gridDim.x - 1) {
        __threadfence();
        float bv = -__int_as_float(0x7f800000);
        int bi = 0x7fffffff;
        for (int c = 0; c < (int)gridDim.x; c++) {
          float v = ((volatile float *)a.part_val)[c];
          int i = ((volatile int *)a.part_idx)[c];
          if (better(v, i, bv, bi)) {
            bv = v;
            bi = i;
          }
        }
        if (bi == 0x7fffffff) bi = 0;  // every logit NaN: the scan keeps index 0
        DecodeState *st = a.state;
        if (a.ids) a.ids[st->step] = bi;
        st->token = bi;
        st->step += 1;
        st->pos += 1;
        st->ticket = 0;
        __threadfence();
      }
    }
  }
}

// Embedding of the step's token (gpt2t.mojo:378-385): dequant_row of the
// per-channel int8 head row (tensor.mojo:453-473) plus wpe[pos].
__global__ void embed_kernel(WeightView head, const float *wpe, float *x, const DecodeState *st) {
  int token = st->token, pos = st->pos, C = head.cols;
  int gpr = head.cols / head.group;
  for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < C; i += blockDim.x * gridDim.x) {
    size_t gi = (size_t)token * gpr + i / head.group;
    float s = half_bits_to_float(head.scale[gi]);
    float v = (float)(code_at(head, token, i) - (int)head.zp[gi]) * s;
    x[i] = v + wpe[(size_t)pos * C + i];
  }
}

}  // namespace llmq
