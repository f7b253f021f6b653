// Lane-mode tcgen05 GEMM: the one-token dot products (dot_row_i16,
// tensor.mojo:522-566) of many independent sequences at once, for batched
// decode on sm_100a.
//
// The one-token dot keeps 16 int32 lanes per output row: for BLOCKED
// int4-g32 rows (tensor.mojo:522-540) lane L of each 256-column block is the
// 16 columns of group L % 8, half L / 8, folded per block as
//   accf_L = fma(f32(lane) - zp * f32(lane sum of x), scale_g, accf_L),
// for per-channel int8 rows (the head, tensor.mojo:541-566) lane L is columns
// 2L, 2L+1 of every 32-column chunk, converted once as
//   f_L = fma(f32(lane - zp * lane sum of x), scale, 0);
// then the 16 lanes add as the halving tree (i + i+8, + i+4, + i+2, + i+1).
// The sums of a lane are what an MMA must produce, exactly, for every
// (row, sequence).
//
// The weights are the MMA's M (128 rows per tile, int4 as int8 u - zp, int8
// as its u8 code), the sequences its N. Its K order is permuted so that each
// 32-column K step holds exactly two lanes, 16 columns each:
//   int4-g32 rows: lane pairs (g, g + 8) in the tree's order g = 0, 4, 2, 6,
//     1, 5, 3, 7, and inside each pair the row's blocks in order; a K step
//     is block b's columns g*32 .. g*32 + 31 (lane g, then lane g + 8);
//   int8 rows: the same pair order; lane g's 48 columns, then lane g + 8's,
//     in column order: three K steps per pair, each 16-column half one lane.
// Each sequence's int16 activation x = 256 xh + xl (xh signed, xl unsigned)
// appears as four rows of the N operand: (low, half 0), (low, half 1),
// (high, half 0), (high, half 1), each row zero in the other half of every
// K step. Two kind::i8 MMAs per K step (the low rows as u8, the high rows as
// s8) give, per row and sequence, each of its two lanes' sums: 256 D_h + D_l,
// int32 modulo 2^32 like the reference's accumulator, for the int8 rows minus
// zp * sum(x). The folds keep the reference's order, so each sequence's
// outputs equal its one-token outputs bit for bit.
//
// The kernel is persistent over row tiles: CTA (sequence tile, column c)
// takes row tiles c, c + gridDim.y, ... and streams their K blocks as units
// of 4 K steps. Two producer warps (16, 17) take alternate units: each
// copies its units' [A: 128 rows x 128 B][B: 4 TT rows x 128 B] tiles (the
// 128-byte swizzle layout) through its own 3 stages, issues the unit's 8 MMAs
// into its own tensor-memory buffer (4 K steps x 4 TT columns) and commits
// once per unit, so one producer's waits and issue latency overlap the
// other's. Warps 0-15 fold (warp w: tensor-memory lanes = weight rows
// 32 * (w % 4) + lane, sequences (w / 4) * TT / 4 .. + TT / 4). The int4
// rows' lane sums become floats through a float-magic bias (an integer add and
// a float subtraction), and the pair arithmetic runs on f32x2.
#pragma once

#include "tc_gemm.cuh"

namespace llmq {

enum { TCL_BLK4 = 0, TCL_CH8 = 1 };

// Lane g of the halving tree's pair gp (g = 0, 4, 2, 6, 1, 5, 3, 7): pairs 2i
// and 2i + 1 make s4[i'], pairs 0-3 make s2[0] and pairs 4-7 s2[1].
__host__ __device__ __forceinline__ int tcl_pair_lane(int gp) {
  return 4 * (gp & 1) + 2 * ((gp >> 1) & 1) + (gp >> 2);
}

// The natural column of position k of the permuted K order.
__host__ __device__ __forceinline__ int tcl_col(int mode, int k, int K) {
  if (mode == TCL_BLK4) {
    const int nblk = K >> 8, s = k >> 5, gp = s / nblk, b = s - gp * nblk;
    return b * 256 + tcl_pair_lane(gp) * 32 + (k & 31);
  }
  const int lw = K >> 4, pair = k / (2 * lw), w = k - pair * 2 * lw, g = tcl_pair_lane(pair);
  const int lane = w < lw ? g : g + 8, j = w < lw ? w : w - lw;
  return (j >> 1) * 32 + 2 * lane + (j & 1);
}

// Whether the lane-mode GEMM takes the matrix: BLOCKED int4-g32 A16 rows or
// per-channel int8 A16 rows, 256-column multiples.
__host__ __device__ inline bool tcl_supported(const WeightView &w) {
  if (w.cols % 256 != 0 || w.cols > 4096) return false;
  if (w.bits == 4 && w.blocked && w.group == 32) return true;
  return w.bits == 8 && w.group == w.cols;
}

// A tiles of a weight: grid (row tiles, K blocks), 256 threads. Row n, K
// position k holds the value of column tcl_col(k): u - zp for int4, the u8
// code for int8; rows past the matrix are zero.
__global__ void tcl_prep_a_kernel(WeightView w, int mode, uint8_t *a) {
  const int nt = blockIdx.x, kb = blockIdx.y, nkb = gridDim.y, K = w.cols, gpr = K / w.group;
  uint8_t *dst = a + ((size_t)nt * nkb + kb) * TCT_A_BYTES;
  for (int ci = threadIdx.x; ci < 8 * TC_M; ci += blockDim.x) {
    const int chunk = ci / TC_M, r = ci % TC_M, n = nt * TC_M + r, k0 = kb * TC_KB + chunk * 16;
    uint32_t v[4] = {0, 0, 0, 0};
    if (n < w.rows) {
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int col = tcl_col(mode, k0 + i, K);
        const int code = code_at(w, n, col);
        const int e = mode == TCL_BLK4 ? code - (int)w.zp[(size_t)n * gpr + col / w.group] : code;
        v[i >> 2] |= (uint32_t)(e & 0xFF) << (8 * (i & 3));
      }
    }
    *(uint4 *)(dst + tc_sw128_off(r, chunk)) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// quantize_rows (+ LayerNorm) of each sequence's row (kernels.mojo:179-197,
// 400-416: the one-token prologue's arithmetic, in natural column order)
// into the B tiles [sequence tile][K block][4 TT rows x 128 B]: row (plane
// p, half h) of sequence t at p * 2 TT + 2 t + h holds, in the K step's half
// h, the low byte xl (p = 0) or the high byte xh (p = 1) of x at column
// tcl_col(k), and zero in the other half. Also sx[m] and, for the int8 rows,
// the 16 lane sums of x (columns 2L, 2L + 1 of every 32-column chunk). One
// CTA of 256 threads per sequence of the padded count, the row staged in
// shared memory: warp 0 takes the LayerNorm sums (16 lane sums, each
// sequential over the row's 16-float chunks, then the halving tree), every
// thread a share of the columns for the max of |x| (exact in any order), the
// integer lane sums and the packing; padding sequences get zero tiles.
template <int TT, int PRO>
__global__ void __launch_bounds__(256) tcl_quant_pack_kernel(const float *x, const float *ln_w, const float *ln_b,
                                                             int B, int bpad, int K, int mode, uint8_t *b, float *sx,
                                                             int *xsl) {
  extern __shared__ __align__(16) float xf[];  // [K]
  __shared__ float red[8], stat[2];
  __shared__ int lsum[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
  const int m = blockIdx.x;
  const bool valid = m < B;
  const int nkb = K / TC_KB, r = m % TT;
  uint8_t *tile = b + (size_t)(m / TT) * nkb * (4 * TT * TC_KB);
  if (tid < 16) lsum[tid] = 0;
  float inv = 0.0f;
  if (valid) {
    const float *row = x + (size_t)m * K;
    for (int i = tid * 4; i < K; i += 1024) *(float4 *)(xf + i) = *(const float4 *)(row + i);
    __syncthreads();
    if (PRO == PRO_LN) {
      if (warp == 0) {
        const int l = lane & 15;
        float s = 0.0f;
        for (int i = 0; i < K; i += 16) s = s + xf[i + l];
        const float mean = tree16_warp(s) / (float)K;
        float sq = 0.0f;
        for (int i = 0; i < K; i += 16) {
          const float d = xf[i + l] - mean;
          sq = sq + d * d;
        }
        const float var = tree16_warp(sq) / (float)K;
        if (lane == 0) {
          stat[0] = mean;
          stat[1] = 1.0f / sqrtf(var + 1e-5f);
        }
      }
      __syncthreads();
      const float mean = stat[0], rstd = stat[1];
      for (int i = tid; i < K; i += 256) {
        const float n = (xf[i] - mean) * rstd;
        xf[i] = n * ln_w[i] + ln_b[i];
      }
      __syncthreads();
    }
    float mx = 0.0f;
    for (int i = tid; i < K; i += 256) mx = fmaxf(mx, fabsf(xf[i]));
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp] = mx;
    __syncthreads();
    mx = red[0];
    for (int w = 1; w < 8; w++) mx = fmaxf(mx, red[w]);
    float s = mx / 32767.0f;
    if (s == 0.0f) s = 1.0f;
    inv = 1.0f / s;
    if (tid == 0) sx[m] = s;
    if (mode == TCL_CH8) {
      // lane L's sum over the 32-column chunks: thread tid takes lane tid % 16
      // of chunks tid / 16, tid / 16 + 16, ...
      const int L = tid & 15;
      int acc = 0;
      for (int c = tid >> 4; c < K / 32; c += 16)
        acc += (int)roundf(xf[c * 32 + 2 * L] * inv) + (int)roundf(xf[c * 32 + 2 * L + 1] * inv);
      atomicAdd(&lsum[L], acc);
    }
  }
  __syncthreads();
  if (mode == TCL_CH8 && tid < 16) xsl[(size_t)m * 16 + tid] = valid ? lsum[tid] : 0;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int ci = tid; ci < K / 16; ci += 256) {
    const int k0 = ci * 16, kb = k0 / TC_KB, chunk = (k0 % TC_KB) / 16, half = (k0 >> 4) & 1;
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    if (valid) {
      // the chunk's 16 columns: contiguous for int4 rows; for int8 rows the
      // column pairs (2L, 2L + 1) of 8 consecutive 32-column chunks
      const int c0 = tcl_col(mode, k0, K);
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int col = mode == TCL_BLK4 ? c0 + i : c0 + (i >> 1) * 32 + (i & 1);
        const unsigned q = (uint16_t)(int16_t)roundf(xf[col] * inv);
        lo[i >> 2] |= (q & 0xFFu) << (8 * (i & 3));
        hi[i >> 2] |= ((q >> 8) & 0xFFu) << (8 * (i & 3));
      }
    }
    uint8_t *kbase = tile + (size_t)kb * (4 * TT * TC_KB);
    *(uint4 *)(kbase + tc_sw128_off(2 * r + half, chunk)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *(uint4 *)(kbase + tc_sw128_off(2 * TT + 2 * r + half, chunk)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *(uint4 *)(kbase + tc_sw128_off(2 * r + 1 - half, chunk)) = zero;
    *(uint4 *)(kbase + tc_sw128_off(2 * TT + 2 * r + 1 - half, chunk)) = zero;
  }
}

// Registers per lane of a row in tcl_pack_seq: lane L holds columns L + 32 j.
constexpr int TCL_PJ = 24;
constexpr int TCL_PACK_K = 32 * TCL_PJ;  // the widest row packed inside the GEMM

// tcl_quant_pack_kernel's arithmetic for one sequence of a K <= TCL_PACK_K
// row, by one warp, into B tiles in shared memory (K block kb at tiles + kb
// * kbs): the codes' positions only (the other halves are zeroed by the
// caller). Returns sx; for the int8 rows also writes the 16 lane sums of x
// to xsl. Lane L holds columns L + 32 j in registers (one coalesced read).
// The LayerNorm sums keep their order: lane sum l adds columns l + 16 i for
// i = 0, 1, ..., i.e. the registers j of lanes l and l + 16 in turn, which
// every lane reads with two shuffles (no divergence). Each lane stores the
// two bytes of its own codes. With ln_stage, the nthr threads 0 ... nthr - 1
// (each packing one sequence) first copy the LayerNorm weights there
// together. A padding sequence (valid false) stores zero codes.
template <int TT>
__device__ float tcl_pack_seq(const float *row, const float *ln_w, const float *ln_b, int K, int mode, bool valid,
                              int t, uint8_t *tiles, int kbs, int *xsl, float *ln_stage, int nthr, int lane) {
  constexpr unsigned HI = (2 * TT / 8) * 1024;  // tc_sw128_off(r + 2 TT, c) - tc_sw128_off(r, c)
  const bool ln = ln_w != nullptr;
  const int n = K >> 5, l = lane & 15;
  float xr[TCL_PJ];
#pragma unroll
  for (int j = 0; j < TCL_PJ; j++) xr[j] = (valid && j < n) ? __ldg(row + lane + 32 * j) : 0.0f;
  if (ln && ln_stage) {
    for (int i = threadIdx.x; i < K; i += nthr) {
      ln_stage[i] = __ldg(ln_w + i);
      ln_stage[K + i] = __ldg(ln_b + i);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(nthr) : "memory");
    ln_w = ln_stage;
    ln_b = ln_stage + K;
  }
  if (ln && valid) {
    float a = 0.0f;
#pragma unroll
    for (int j = 0; j < TCL_PJ; j++)
      if (j < n) {
        const float u0 = __shfl_sync(0xffffffffu, xr[j], l), u1 = __shfl_sync(0xffffffffu, xr[j], l + 16);
        a = a + u0;
        a = a + u1;
      }
    const float mean = tree16_warp(a) / (float)K;
    float sq = 0.0f;
#pragma unroll
    for (int j = 0; j < TCL_PJ; j++)
      if (j < n) {
        const float d0 = __shfl_sync(0xffffffffu, xr[j], l) - mean;
        const float d1 = __shfl_sync(0xffffffffu, xr[j], l + 16) - mean;
        sq = sq + d0 * d0;
        sq = sq + d1 * d1;
      }
    const float rstd = 1.0f / sqrtf(tree16_warp(sq) / (float)K + 1e-5f);
#pragma unroll
    for (int j = 0; j < TCL_PJ; j++)
      if (j < n) {
        const int c = lane + 32 * j;
        const float v = (xr[j] - mean) * rstd;
        xr[j] = v * ln_w[c] + ln_b[c];
      }
  }
  float mx = 0.0f;
#pragma unroll
  for (int j = 0; j < TCL_PJ; j++) mx = fmaxf(mx, fabsf(xr[j]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = mx / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  const float inv = valid ? 1.0f / s : 0.0f;
  int qsum = 0;
  if (mode == TCL_BLK4) {
    // register j: the 32-column group j (block b = j / 8, lane group g =
    // j % 8) is K step st = gp * nblk + b with tcl_pair_lane(gp) = g; lane
    // L is its byte L % 16 of half L / 16
    const int nblk = K >> 8, half = lane >> 4;
    uint8_t *base = tiles + (lane & 15);
#pragma unroll
    for (int j = 0; j < TCL_PJ; j++)
      if (j < n) {
        const unsigned q = (uint16_t)(int16_t)roundf(xr[j] * inv);
        const int st = tcl_pair_lane(j & 7) * nblk + (j >> 3);
        uint8_t *dst = base + (size_t)(st >> 2) * kbs + tc_sw128_off(2 * t + half, (st & 3) * 2 + half);
        dst[0] = (uint8_t)q;
        dst[HI] = (uint8_t)(q >> 8);
      }
  } else {
    // lane L = 2 lp + e holds, in register j, position 2 j + e of lane
    // position lp (columns 2 lp, 2 lp + 1 of every 32-column chunk), i.e. K
    // position gp * 2 lw + (lp >= 8 ? lw : 0) + 2 j + e, tcl_pair_lane(gp) = lp % 8
    const int lw = K >> 4, lp = lane >> 1;
    const int k00 = tcl_pair_lane(lp & 7) * 2 * lw + (lp >= 8 ? lw : 0) + (lane & 1);
#pragma unroll
    for (int j = 0; j < TCL_PJ; j++)
      if (j < n) {
        const float f = roundf(xr[j] * inv);
        const unsigned q = (uint16_t)(int16_t)f;
        qsum += (int)f;
        const int k = k00 + 2 * j, half = (k >> 4) & 1;
        uint8_t *dst = tiles + (size_t)(k >> 7) * kbs + tc_sw128_off(2 * t + half, (k & 127) >> 4) + (k & 15);
        dst[0] = (uint8_t)q;
        dst[HI] = (uint8_t)(q >> 8);
      }
    // lane 2L's and lane 2L + 1's sums of their codes: columns 2L, 2L + 1
    qsum += __shfl_xor_sync(0xffffffffu, qsum, 1);
    if ((lane & 1) == 0) xsl[lane >> 1] = qsum;
  }
  return s;
}

struct TcArgsL {
  const uint8_t *a;   // weight tiles (tcl_prep_a_kernel)
  const float *x;     // K <= TCL_PACK_K: [sequences][K] rows, packed by the CTA (tcl_pack_seq)
  const float *ln_w;  //   LayerNorm applied first when non-null
  const float *ln_b;
  const uint8_t *b;   // else: sequence tiles (tcl_quant_pack_kernel)
  const float *sx;    //   [sequences] activation scales
  const int *xsl;     //   int8 rows: [sequences][16] lane sums of x
  WeightView w;
  const float *bias;  // int4 rows: [rows] or null
  float *out;         // int4 rows: [sequences][rows]
  float *part_val;    // int8 rows: [sequences][nparts] argmax candidates, 4 per row tile
  int *part_idx;
  int *err;
  int B, OUT, K, nkb, nseg, epi, ntiles, nparts;
  int res;            // x given: B tile kb stays in stage kb's B slot (nkb <= TCL_STAGES)
};

// A CTA's units: K blocks (4 segments, one 128-byte K block of the A and B
// tiles) of its row tiles blockIdx.y, blockIdx.y + gridDim.y, ... in order.
// Unit u's accumulators fill tensor-memory buffer u % 2 (4 segments x 4 TT
// columns); producer warp u % 2 issues its copies, MMAs and commits, so the
// two producers' instruction latencies overlap and each buffer has its own
// producer. Its copies use the producer's own stages (TCL_SPP of them).
constexpr int TCL_NPROD = 2;
constexpr int TCL_SPP = 3;                                       // copy stages per producer
constexpr int TCL_STAGES = TCL_NPROD * TCL_SPP;
constexpr int TCL_EPI = 16;                                      // epilogue warps: 4 per lane quarter
constexpr int TCL_CG = TCL_EPI / 4;                              // sequence groups among them
constexpr int TCL_THREADS = (TCL_EPI + TCL_NPROD) * 32;          // 192
constexpr int TCL_MAX_SEG = 128;                                 // K steps per row: K <= 4096

// What the epilogue does at K step s of a row, packed once per CTA so that
// the loop needs no divisions: int4 rows: the scale column b * 8 + g (bits
// 0-6), whether the pair closes (bit 7), the pair gp (bits 8-10); int8 rows:
// the lane g (bits 0-2), whether the pair closes (bit 7), gp (bits 8-10),
// whether each half belongs to lane g (bits 11, 12; else to lane g + 8).
__device__ __forceinline__ int tcl_seg_entry(int mode, int s, int K) {
  if (mode == TCL_BLK4) {
    const int nblk = K >> 8, gp = s / nblk, b = s - gp * nblk;
    return (b * 8 + tcl_pair_lane(gp)) | ((b == nblk - 1) << 7) | (gp << 8);
  }
  const int spp = K >> 8, gp = s / spp, s3 = s - gp * spp, h0 = 2 * s3;
  return tcl_pair_lane(gp) | ((s3 == spp - 1) << 7) | (gp << 8) | ((h0 < spp) << 11) | ((h0 + 1 < spp) << 12);
}

template <int TT>
struct TcSmemL {
  alignas(1024) uint8_t stage[TCL_STAGES][TCT_A_BYTES + 4 * TT * TC_KB];
  int xsl[TT][16];
  float sx[TT];                               // the sequences' activation scales
  alignas(16) int seg[TCL_MAX_SEG];           // the K steps' schedule (tcl_seg_entry)
  float tree[3][TT / TCL_CG][TCL_EPI * 32];  // the epilogue's halving-tree partial sums
  alignas(8) unsigned long long full[TCL_STAGES], empty[TCL_STAGES], accfull[TCL_NPROD], accempty[TCL_NPROD],
      drain[TCL_NPROD], packed;
  unsigned tmem;
  int abort;
};


// The halving tree is fed one lane pair at a time in tcl_pair_lane order:
// s8 = lane g + lane g + 8; pairs (0, 4), (2, 6), (1, 5), (3, 7) make
// s4[0], s4[2], s4[1], s4[3]; s2[0] = s4[0] + s4[2], s2[1] = s4[1] + s4[3],
// dot = s2[0] + s2[1].

// A lane's exact int32 sum v (|v| < 2^16 per K step) becomes a float without
// the conversion unit: the bits of TCL_MAGIC + v (TCL_MAGIC = the bits of
// 1.5 * 2^23) read as the float 1.5 * 2^23 + v, and one float subtraction
// (paired as f32x2) gives f32(v) exactly.
constexpr int TCL_MAGIC = 0x4B400000;
constexpr float TCL_MAGIC_F = 12582912.0f;


// Warps 0-15: per segment g of the CTA's units (u = g / 4, K step g % 4),
// the accumulators of this thread's weight row and CW sequences. Column
// 2t + h of a plane holds sequence t's half h, so one 2 CW-column load per
// plane gives each sequence's two lanes as an adjacent pair, and the pair's
// arithmetic runs as f32x2. int4 rows fold lanes g and g + 8 of block b
// into their chains and close the pair after the row's last block; int8
// rows add the halves into the pair's two int32 lane sums and close the pair
// after its third K step. The tree's partial sums wait in shared memory
// (touched once per pair). After a row tile's last segment its values go to
// out (int4) or to the argmax candidates of its four lane quarters (int8).
// The next segment's tensor-memory loads (and int4 scale) are in flight
// while this one folds.
template <int MODE, int TT>
__device__ __forceinline__ void tcl_epilogue(const TcArgsL &p, TcSmemL<TT> &sm, unsigned tmem, int warp, int lane,
                                             int t0, int nunits) {
  constexpr int N = 4 * TT, KBN = 4 * N, CW = TT / TCL_CG, W = 2 * CW;
  const int q = warp & 3, cg = warp >> 2, rl = 32 * q + lane, tid = threadIdx.x;
  const unsigned tbase = tmem + ((unsigned)(32 * q) << 16) + cg * W;  // low plane; the high plane at + 2 TT
  const int nkb = p.nkb, gpr = p.K / p.w.group;
  unsigned long long cab[CW];  // int4 rows: the pair's two lane chains
  int ia[CW], ib[CW];          // int8 rows: the pair's two lane sums
#pragma unroll
  for (int c = 0; c < CW; c++) {
    cab[c] = 0ull;
    ia[c] = ib[c] = 0;
  }
  float sc8 = 0.0f;  // int8 rows: the row's scale and zero point
  int zp8 = 0;
  const unsigned long long neg_magic = f2_pair(-TCL_MAGIC_F, -TCL_MAGIC_F), k256 = f2_pair(256.0f, 256.0f);
  auto row_of = [&](int it) {
    const int n = (blockIdx.y + it * gridDim.y) * TC_M + rl;
    return n < p.w.rows ? n : p.w.rows - 1;
  };
  // int4 rows: the scales of the next unit's four K steps, loaded a unit ahead
  unsigned scn[4] = {0, 0, 0, 0};
  auto fetch_scales = [&](int it, int kb) {
    const int4 e = *reinterpret_cast<const int4 *>(&sm.seg[kb * 4]);
    const uint16_t *rs = p.w.scale + (size_t)row_of(it) * gpr;
    scn[0] = rs[e.x & 127];
    scn[1] = rs[e.y & 127];
    scn[2] = rs[e.z & 127];
    scn[3] = rs[e.w & 127];
  };
  // the halving tree of sequence c (the order above), its partial sums in
  // shared memory: tree[0] the pending s8, tree[1] the pending s4, tree[2]
  // s2[0] and then the dot
  auto tree = [&](int gp, int c, float s8) {
    if ((gp & 1) == 0) {
      sm.tree[0][c][tid] = s8;
      return;
    }
    const float s4 = sm.tree[0][c][tid] + s8;
    if (gp == 1 || gp == 5) {
      sm.tree[1][c][tid] = s4;
      return;
    }
    const float s2 = sm.tree[1][c][tid] + s4;
    if (gp == 3) {
      sm.tree[2][c][tid] = s2;
      return;
    }
    sm.tree[2][c][tid] = sm.tree[2][c][tid] + s2;
  };
  // the row tile's values (its last K step folded)
  auto emit = [&](int it) {
    const int nt = blockIdx.y + it * gridDim.y, n = nt * TC_M + rl;
    if (MODE == TCL_BLK4) {
      if (n >= p.OUT) return;
      const float bn = (p.epi & EPI_BIAS) ? p.bias[n] : 0.0f;
#pragma unroll
      for (int c = 0; c < CW; c++) {
        const int m = t0 + cg * CW + c;
        if (m >= p.B) break;
        float *dst = p.out + (size_t)m * p.OUT + n;
        float r = sm.tree[2][c][tid] * sm.sx[cg * CW + c];
        if (p.epi & EPI_BIAS) r += bn;
        if (p.epi & EPI_GELU) r = gelu(r);
        if (p.epi & EPI_RESID) r += *dst;
        *dst = r;
      }
    } else {
      // the best of the warp's 32 rows per sequence, one candidate per lane
      // quarter and row tile
#pragma unroll
      for (int c = 0; c < CW; c++) {
        const int m = t0 + cg * CW + c;
        float bv = -__int_as_float(0x7f800000);
        int bi = 0x7fffffff;
        if (n < p.w.rows && m < p.B) {
          bv = sm.tree[2][c][tid] * sm.sx[cg * CW + c];
          bi = n;
        }
        for (int o = 16; o > 0; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
          }
        }
        if (lane == 0 && m < p.B) {
          p.part_val[(size_t)m * p.nparts + nt * 4 + q] = bv;
          p.part_idx[(size_t)m * p.nparts + nt * 4 + q] = bi;
        }
      }
    }
  };
  // one K step: its accumulators (dl, dh) and schedule entry e
  auto step = [&](const int (&dl)[W], const int (&dh)[W], int e, unsigned sc16) {
    const int gp = e >> 8;
    if (MODE == TCL_BLK4) {
      const float sc = half_bits_to_float((uint16_t)sc16);
      const unsigned long long sc2 = f2_pair(sc, sc);
#pragma unroll
      for (int c = 0; c < CW; c++) {
        // |high| < 2^15, |low| < 2^16: exact floats, one rounding in the fma,
        // as the reference's f32(lane) - zp * f32(lane sum of x)
        const unsigned long long lo =
            f2_add(f2_bits(dl[2 * c] + TCL_MAGIC, dl[2 * c + 1] + TCL_MAGIC), neg_magic);
        const unsigned long long hi =
            f2_add(f2_bits(dh[2 * c] + TCL_MAGIC, dh[2 * c + 1] + TCL_MAGIC), neg_magic);
        cab[c] = f2_fma(f2_fma(k256, hi, lo), sc2, cab[c]);
      }
      if (e & 128) {
#pragma unroll
        for (int c = 0; c < CW; c++) {
          float ca, cb;
          f2_split(cab[c], ca, cb);
          tree(gp, c, ca + cb);
          cab[c] = 0ull;
        }
      }
    } else {
      const bool a_lo = (e >> 11) & 1, b_lo = (e >> 12) & 1;  // each half's lane: g (true) or g + 8
#pragma unroll
      for (int c = 0; c < CW; c++) {
        const unsigned ua = ((unsigned)dh[2 * c] << 8) + (unsigned)dl[2 * c];
        const unsigned ub = ((unsigned)dh[2 * c + 1] << 8) + (unsigned)dl[2 * c + 1];
        if (a_lo) ia[c] = (int)((unsigned)ia[c] + ua);
        else ib[c] = (int)((unsigned)ib[c] + ua);
        if (b_lo) ia[c] = (int)((unsigned)ia[c] + ub);
        else ib[c] = (int)((unsigned)ib[c] + ub);
      }
      if (e & 128) {
        const int gg = e & 7;
#pragma unroll
        for (int c = 0; c < CW; c++) {
          const int t = cg * CW + c;
          const int a0 = (int)((unsigned)ia[c] - (unsigned)(zp8 * sm.xsl[t][gg]));
          const int a1 = (int)((unsigned)ib[c] - (unsigned)(zp8 * sm.xsl[t][gg + 8]));
          const float fx = fmaf((float)a0, sc8, 0.0f), fy = fmaf((float)a1, sc8, 0.0f);
          tree(gp, c, fx + fy);
          ia[c] = ib[c] = 0;
        }
      }
    }
  };
  int it = 0, kb = 0;  // the unit's row-tile iteration and K block
  if (MODE == TCL_BLK4 && nunits > 0) fetch_scales(0, 0);
  for (int u = 0; u < nunits; u++) {
    const int buf = u & 1;
    bool ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accfull[buf]), (u >> 1) & 1, p.err, TC_ERR_ACC);
    ok = __all_sync(0xffffffffu, ok);  // the tensor-memory loads are warp-wide
    if (!ok) return;
    tc_fence_after();
    // the unit's K steps in two halves of two (32 registers of loads in
    // flight, no spills); the buffer is released once the second half's
    // loads have landed and its columns are refilled
    int dla[W], dha[W], dlb[W], dhb[W];
    const unsigned tb = tbase + buf * KBN;
    tc_ld(tb, dla);
    tc_ld(tb + 2 * TT, dha);
    tc_ld(tb + N, dlb);
    tc_ld(tb + N + 2 * TT, dhb);
    const int4 e = *reinterpret_cast<const int4 *>(&sm.seg[kb * 4]);
    const unsigned s0 = scn[0], s1 = scn[1], s2 = scn[2], s3 = scn[3];
    if (MODE == TCL_CH8 && kb == 0) {
      const int nr = row_of(it);
      sc8 = half_bits_to_float(p.w.scale[nr]);
      zp8 = p.w.zp[nr];
    }
    // the next unit's cursor and (int4 rows) its scales
    int it2 = it, kb2 = kb + 1;
    if (kb2 == nkb) {
      kb2 = 0;
      ++it2;
    }
    if (MODE == TCL_BLK4 && u + 1 < nunits) fetch_scales(it2, kb2);
    tc_ld_wait();
    tc_ld_done(dla);
    tc_ld_done(dha);
    tc_ld_done(dlb);
    tc_ld_done(dhb);
    step(dla, dha, e.x, s0);
    step(dlb, dhb, e.y, s1);
    tc_ld(tb + 2 * N, dla);
    tc_ld(tb + 2 * N + 2 * TT, dha);
    tc_ld(tb + 3 * N, dlb);
    tc_ld(tb + 3 * N + 2 * TT, dhb);
    tc_ld_wait();
    tc_ld_done(dla);
    tc_ld_done(dha);
    tc_ld_done(dlb);
    tc_ld_done(dhb);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) tc_mbar_arrive(tc_u32(&sm.accempty[buf]));
    step(dla, dha, e.z, s2);
    step(dlb, dhb, e.w, s3);
    if (kb == nkb - 1) emit(it);
    it = it2;
    kb = kb2;
  }
}

// Producer warp pr (lane 0 issues): its units u = pr, pr + 2, ... (local
// index k = u / 2): the copies of unit k into stage pr * TCL_SPP + k %
// TCL_SPP, then, once buffer pr is free again and the copies landed, the
// unit's 8 MMAs (4 K steps x the low and high rows) into buffer pr, one
// commit for the epilogue and one for the stage; then the stage of unit k - 1
// is refilled with unit k - 1 + TCL_SPP.
template <int MODE, int TT>
__device__ __forceinline__ void tcl_producer(const TcArgsL &p, TcSmemL<TT> &sm, unsigned tmem, int pr, int lane,
                                             int nunits) {
  constexpr int N = 4 * TT, KBN = 4 * N, BB = N * TC_KB, STAGE = TCT_A_BYTES + BB;
  constexpr unsigned ACC = 0u;  // every K step into fresh accumulators
  const bool leader = lane == 0;
  // low rows (u8) and high rows (s8), N = 2 TT each
  const unsigned idesc_l = tc_idesc(MODE == TCL_BLK4 ? 1 : 0, 0, 2 * TT);
  const unsigned idesc_h = tc_idesc(MODE == TCL_BLK4 ? 1 : 0, 1, 2 * TT);
  constexpr unsigned long long HIGH = (2 * TT * TC_KB) >> 4;  // descriptor start of the high rows
  const unsigned long long desc_a0 = tc_desc_sw128(tc_u32(sm.stage[0]));
  const unsigned long long desc_b0 = tc_desc_sw128(tc_u32(sm.stage[0]) + TCT_A_BYTES);
  const int nk = nunits > pr ? (nunits - pr + 1) / 2 : 0;
  const uint8_t *gb = p.b + (size_t)blockIdx.x * p.nkb * BB;
  auto stage_of = [&](int k) { return pr * TCL_SPP + k % TCL_SPP; };
  // the copies of unit k (2 k + pr overall): its weight tile (wa) and its
  // B tile (wb); one expected-bytes count covers both
  auto load = [&](int k, bool wa, bool wb) {
    const int u = 2 * k + pr, it = u / p.nkb, kb = u - it * p.nkb, nt = blockIdx.y + it * gridDim.y;
    const int st = stage_of(k);
    const unsigned dst = tc_u32(sm.stage[st]), bar = tc_u32(&sm.full[st]);
    if (leader) {
      if (wa) {
        tc_mbar_expect_tx(bar, p.res ? TCT_A_BYTES : STAGE);
        tc_bulk_g2s(dst, p.a + ((size_t)nt * p.nkb + kb) * TCT_A_BYTES, TCT_A_BYTES, bar);
      }
      if (wb && !p.res) tc_bulk_g2s(dst + TCT_A_BYTES, gb + (size_t)kb * BB, BB, bar);
    }
    __syncwarp();
  };
  // the first stages' weight tiles while the epilogue warps pack B (or copy
  // sx), then their B tiles (issued even after a failed wait, so that every
  // stage's count completes before the drain)
  int issued = 0, waited = 0;
  for (; issued < nk && issued < TCL_SPP; issued++) load(issued, true, false);
  bool ok = tc_wait_flag(&sm.abort, tc_u32(&sm.packed), 0, p.err, TC_ERR_FULL);
  ok = __all_sync(0xffffffffu, ok);
  for (int k = 0; k < issued; k++) load(k, false, true);
  for (int k = 0; k < nk && ok; k++) {
    const int st = stage_of(k);
    if (k >= 1) ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accempty[pr]), (k - 1) & 1, p.err, TC_ERR_ACCEMPTY);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    ok = tc_wait_flag(&sm.abort, tc_u32(&sm.full[st]), (k / TCL_SPP) & 1, p.err, TC_ERR_FULL);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    waited = k + 1;
    tc_fence_after();
    if (leader) {
      const unsigned long long off = (unsigned long long)((st * STAGE) >> 4);
      const int u = 2 * k + pr, kb = u - (u / p.nkb) * p.nkb;
      const unsigned long long offb = p.res ? (unsigned long long)((kb * STAGE) >> 4) : off;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const unsigned long long da = desc_a0 + off + (unsigned long long)(2 * j);
        const unsigned long long db = desc_b0 + offb + (unsigned long long)(2 * j);
        const unsigned d = tmem + pr * KBN + j * N;
        tc_mma(d, da, db, idesc_l, ACC);
        tc_mma(d + 2 * TT, da, db + HIGH, idesc_h, ACC);
      }
      tc_commit(tc_u32(&sm.accfull[pr]));
      tc_commit(tc_u32(&sm.empty[st]));
    }
    __syncwarp();
    // refill the stage of unit k - 1, whose MMAs were queued ahead of these
    if (k >= 1 && issued < nk) {
      ok = tc_wait_flag(&sm.abort, tc_u32(&sm.empty[stage_of(k - 1)]), ((k - 1) / TCL_SPP) & 1, p.err,
                        TC_ERR_EMPTY);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      load(issued++, true, true);
    }
  }
  if (!ok) {
    // drain: copies issued but not yet waited for, then every MMA issued
    for (int k = waited; k < issued; k++) tc_drain_wait(tc_u32(&sm.full[stage_of(k)]), (k / TCL_SPP) & 1);
    if (leader) tc_commit(tc_u32(&sm.drain[pr]));
    __syncwarp();
    tc_drain_wait(tc_u32(&sm.drain[pr]), 0);
  }
}

template <int MODE, int TT>
__global__ void __launch_bounds__(TCL_THREADS, 1) tcl_gemm_kernel(TcArgsL p) {
  constexpr int N = 4 * TT, KBN = 4 * N, CW = TT / TCL_CG;
  static_assert(TCL_NPROD * KBN <= TC_TMEM_COLS, "two unit buffers of tensor memory");
  static_assert(CW == 4 || CW == 8 || CW == 16, "tc_ld widths");
  extern __shared__ __align__(128) unsigned char tc_raw[];
  TcSmemL<TT> &sm = *reinterpret_cast<TcSmemL<TT> *>(tc_raw + ((1024u - (tc_u32(tc_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.x * TT;
  const int iters = (int)blockIdx.y < p.ntiles ? (p.ntiles - 1 - (int)blockIdx.y) / (int)gridDim.y + 1 : 0;
  const int nunits = iters * p.nkb;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TCL_STAGES; s++) {
      tc_mbar_init(tc_u32(&sm.full[s]), 1);
      tc_mbar_init(tc_u32(&sm.empty[s]), 1);
    }
    for (int b = 0; b < TCL_NPROD; b++) {
      tc_mbar_init(tc_u32(&sm.accfull[b]), 1);
      tc_mbar_init(tc_u32(&sm.accempty[b]), TCL_EPI);
      tc_mbar_init(tc_u32(&sm.drain[b]), 1);
    }
    tc_mbar_init(tc_u32(&sm.packed), TCL_EPI * 32);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == TCL_EPI) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_u32(&sm.tmem)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  } else if (warp < TCL_EPI) {
    if (threadIdx.x < p.nseg) sm.seg[threadIdx.x] = tcl_seg_entry(MODE, threadIdx.x, p.K);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = sm.tmem;
  if (warp >= TCL_EPI) {
    tcl_producer<MODE, TT>(p, sm, tmem, warp - TCL_EPI, lane, nunits);
  } else {
    // the CTA's sequences into its B tiles (the producers copy their first
    // weight tiles meanwhile), made visible to the MMAs (async proxy) before
    // each thread's arrival on sm.packed; or their scales and lane sums
    static_assert(TT == TCL_EPI, "one sequence per epilogue warp");
    const int m = t0 + warp;
    if (p.res) {
      constexpr int STAGE = TCT_A_BYTES + 4 * TT * TC_KB;
      uint8_t *tiles = &sm.stage[0][TCT_A_BYTES];
      // the other halves of the warp's rows (row 2 t + h holds codes in
      // chunks of parity h only): zero
      for (int i = lane; i < 16 * p.nkb; i += 32) {
        const int kb = i >> 4, rr = (i >> 2) & 3, row = (rr & 2) * TT + 2 * warp + (rr & 1);
        const int chunk = 2 * (i & 3) + 1 - (rr & 1);
        *(uint4 *)(tiles + (size_t)kb * STAGE + tc_sw128_off(row, chunk)) = make_uint4(0, 0, 0, 0);
      }
      const bool stage_ln = p.ln_w != nullptr && (size_t)p.K * 8 <= sizeof(sm.tree);
      const float sxm = tcl_pack_seq<TT>(p.x + (size_t)m * p.K, p.ln_w, p.ln_b, p.K, MODE, m < p.B, warp, tiles,
                                         STAGE, sm.xsl[warp], stage_ln ? &sm.tree[0][0][0] : nullptr, TCL_EPI * 32,
                                         lane);
      if (lane == 0) sm.sx[warp] = sxm;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    } else {
      if (lane == 0) sm.sx[warp] = m < p.B ? p.sx[m] : 1.0f;
      if (MODE == TCL_CH8 && lane < 16) sm.xsl[warp][lane] = m < p.B ? p.xsl[(size_t)m * 16 + lane] : 0;
    }
    tc_mbar_arrive(tc_u32(&sm.packed));
    // sm.sx and sm.xsl of every sequence before the epilogue reads them
    asm volatile("bar.sync 1, %0;" ::"r"(TCL_EPI * 32) : "memory");
    tcl_epilogue<MODE, TT>(p, sm, tmem, warp, lane, t0, nunits);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == TCL_EPI) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

// ---------------------------------------------------------------------------
// The prefill GEMM (tile_i16, kernels.mojo:512-573) for int4 rows with
// 32-column groups: every segment is one 32-column K step, so a K block holds
// 4 segments. The arithmetic is tct_gemm_kernel's (weights as the MMA's M,
// both activation planes of TT = 32 tokens in one N = 64 operand, the
// segment sum 256 D_h + D_l + 128 W, the float folds in order); the
// pipeline is the lane-mode GEMM's: units of one K block alternate between
// two producer warps, each with its own copy stages and a tensor-memory
// buffer of 4 segments, one commit per unit; 16 epilogue warps (8 tokens
// each) read a unit in two halves and fold token pairs as f32x2. Persistent
// over token tiles.
// ---------------------------------------------------------------------------
constexpr int TCP_TT = 32;

struct TcpSmem {
  alignas(1024) uint8_t stage[TCL_STAGES][TCT_A_BYTES + 2 * TCP_TT * TC_KB];
  alignas(8) unsigned long long full[TCL_STAGES], empty[TCL_STAGES], accfull[TCL_NPROD], accempty[TCL_NPROD],
      drain[TCL_NPROD];
  unsigned tmem;
  int abort;
};

// Producer warp pr: its units u = pr, pr + 2, ... (local index k), as
// tcl_producer: copies through its own stages, 4 MMAs into buffer pr, one
// commit for the epilogue and one for the stage.
__device__ __forceinline__ void tcp_producer(const TcArgsT &p, TcpSmem &sm, unsigned tmem, int pr, int lane,
                                             int nunits) {
  constexpr int TT = TCP_TT, N = 2 * TT, KBN = 4 * N, BB = 2 * TT * TC_KB, STAGE = TCT_A_BYTES + BB;
  const bool leader = lane == 0;
  const unsigned idesc = tc_idesc(1, 1, N);
  const unsigned long long desc_a0 = tc_desc_sw128(tc_u32(sm.stage[0]));
  const unsigned long long desc_b0 = tc_desc_sw128(tc_u32(sm.stage[0]) + TCT_A_BYTES);
  const int nk = nunits > pr ? (nunits - pr + 1) / 2 : 0;
  const uint8_t *ga = p.a + (size_t)blockIdx.x * p.nkb * TCT_A_BYTES;
  auto stage_of = [&](int k) { return pr * TCL_SPP + k % TCL_SPP; };
  int it_ld = 0, kb_ld = pr;  // the next load's unit as (token-tile iteration, K block)
  auto load = [&](int k) {
    const int tt = blockIdx.y + it_ld * gridDim.y, kb = kb_ld;
    kb_ld += 2;
    while (kb_ld >= p.nkb) {
      kb_ld -= p.nkb;
      ++it_ld;
    }
    const int st = stage_of(k);
    const unsigned dst = tc_u32(sm.stage[st]), bar = tc_u32(&sm.full[st]);
    if (leader) {
      tc_mbar_expect_tx(bar, STAGE);
      tc_bulk_g2s(dst, ga + (size_t)kb * TCT_A_BYTES, TCT_A_BYTES, bar);
      tc_bulk_g2s(dst + TCT_A_BYTES, p.b + ((size_t)tt * p.nkb + kb) * BB, BB, bar);
    }
    __syncwarp();
  };
  int issued = 0, waited = 0;
  for (; issued < nk && issued < TCL_SPP; issued++) load(issued);
  bool ok = true;
  for (int k = 0; k < nk && ok; k++) {
    const int st = stage_of(k);
    if (k >= 1) ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accempty[pr]), (k - 1) & 1, p.err, TC_ERR_ACCEMPTY);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    ok = tc_wait_flag(&sm.abort, tc_u32(&sm.full[st]), (k / TCL_SPP) & 1, p.err, TC_ERR_FULL);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) break;
    waited = k + 1;
    tc_fence_after();
    if (leader) {
      const unsigned long long off = (unsigned long long)((st * STAGE) >> 4);
#pragma unroll
      for (int j = 0; j < 4; j++)
        tc_mma(tmem + pr * KBN + j * N, desc_a0 + off + (unsigned long long)(2 * j),
               desc_b0 + off + (unsigned long long)(2 * j), idesc, 0);
      tc_commit(tc_u32(&sm.accfull[pr]));
      tc_commit(tc_u32(&sm.empty[st]));
    }
    __syncwarp();
    if (k >= 1 && issued < nk) {
      ok = tc_wait_flag(&sm.abort, tc_u32(&sm.empty[stage_of(k - 1)]), ((k - 1) / TCL_SPP) & 1, p.err,
                        TC_ERR_EMPTY);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      load(issued++);
    }
  }
  if (!ok) {
    for (int k = waited; k < issued; k++) tc_drain_wait(tc_u32(&sm.full[stage_of(k)]), (k / TCL_SPP) & 1);
    if (leader) tc_commit(tc_u32(&sm.drain[pr]));
    __syncwarp();
    tc_drain_wait(tc_u32(&sm.drain[pr]), 0);
  }
}

// Epilogue warp (lane quarter q, token group cg): row n0 + 32 q + lane, tokens
// cg * 8 .. + 8 of each token tile; segment s of a row is group s.
__device__ __forceinline__ void tcp_epilogue(const TcArgsT &p, TcpSmem &sm, unsigned tmem, int warp, int lane,
                                             int nunits) {
  constexpr int TT = TCP_TT, N = 2 * TT, KBN = 4 * N, CW = TT / 4;
  const int q = warp & 3, cg = warp >> 2;
  const int n = blockIdx.x * TC_M + 32 * q + lane;
  const int nr = n < p.w.rows ? n : p.w.rows - 1;
  const unsigned tbase = tmem + ((unsigned)(32 * q) << 16) + cg * CW;  // low plane; the high plane at + TT
  const int nkb = p.nkb, gpr = p.w.cols / p.w.group;
  const unsigned long long neg_magic = f2_pair(-TCL_MAGIC_F, -TCL_MAGIC_F), k256 = f2_pair(256.0f, 256.0f);
  unsigned long long acc[CW / 2];  // token pairs' float chains
#pragma unroll
  for (int c = 0; c < CW / 2; c++) acc[c] = 0ull;
  // the next unit's 4 scales (float16 bits) and weight sums, loaded a unit ahead
  uint2 scn = make_uint2(0, 0);
  int4 wsn = make_int4(0, 0, 0, 0);
  auto fetch = [&](int kb) {
    scn = *reinterpret_cast<const uint2 *>(p.w.scale + (size_t)nr * gpr + kb * 4);
    wsn = *reinterpret_cast<const int4 *>(p.wsum + (size_t)nr * p.nseg + kb * 4);
  };
  auto step = [&](const int (&l)[CW], const int (&h)[CW], unsigned sc16, int ws) {
    const float sc = half_bits_to_float((uint16_t)sc16);
    const unsigned long long sc2 = f2_pair(sc, sc);
    const int lb = ws * 128 + TCL_MAGIC;  // 128 W, with the float magic
#pragma unroll
    for (int c = 0; c < CW / 2; c++) {
      // |h|, |l + 128 W| < 2^22: exact floats, one rounding in the fma, as
      // the conversion of the int32 sum 256 h + l + 128 W
      const unsigned long long lo = f2_add(f2_bits(l[2 * c] + lb, l[2 * c + 1] + lb), neg_magic);
      const unsigned long long hi = f2_add(f2_bits(h[2 * c] + TCL_MAGIC, h[2 * c + 1] + TCL_MAGIC), neg_magic);
      acc[c] = f2_fma(f2_fma(k256, hi, lo), sc2, acc[c]);
    }
  };
  auto emit = [&](int it) {
    if (n >= p.n_full) return;
    const float bn = (p.epi & EPI_BIAS) ? p.bias[n] : 0.0f;
    const int t0 = (blockIdx.y + it * gridDim.y) * TT + cg * CW;
#pragma unroll
    for (int c = 0; c < CW; c++) {
      const int m = t0 + c;
      if (m >= p.T) break;
      float a0, a1;
      f2_split(acc[c / 2], a0, a1);
      float *dst = p.out + (size_t)m * p.OUT + n;
      float r = ((c & 1) ? a1 : a0) * p.sx[m];
      if (p.epi & EPI_BIAS) r += bn;
      if (p.epi & EPI_GELU) r = gelu(r);
      if (p.epi & EPI_RESID) r += *dst;
      *dst = r;
    }
  };
  int it = 0, kb = 0;
  if (nunits > 0) fetch(0);
  for (int u = 0; u < nunits; u++) {
    const int buf = u & 1;
    bool ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accfull[buf]), (u >> 1) & 1, p.err, TC_ERR_ACC);
    ok = __all_sync(0xffffffffu, ok);
    if (!ok) return;
    tc_fence_after();
    int la[CW], ha[CW], lb[CW], hb[CW];
    const unsigned tb = tbase + buf * KBN;
    tc_ld(tb, la);
    tc_ld(tb + TT, ha);
    tc_ld(tb + N, lb);
    tc_ld(tb + N + TT, hb);
    const uint2 sc = scn;
    const int4 ws = wsn;
    int it2 = it, kb2 = kb + 1;
    if (kb2 == nkb) {
      kb2 = 0;
      ++it2;
    }
    if (u + 1 < nunits) fetch(kb2);
    tc_ld_wait();
    tc_ld_done(la);
    tc_ld_done(ha);
    tc_ld_done(lb);
    tc_ld_done(hb);
    step(la, ha, sc.x & 0xFFFFu, ws.x);
    step(lb, hb, sc.x >> 16, ws.y);
    tc_ld(tb + 2 * N, la);
    tc_ld(tb + 2 * N + TT, ha);
    tc_ld(tb + 3 * N, lb);
    tc_ld(tb + 3 * N + TT, hb);
    tc_ld_wait();
    tc_ld_done(la);
    tc_ld_done(ha);
    tc_ld_done(lb);
    tc_ld_done(hb);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) tc_mbar_arrive(tc_u32(&sm.accempty[buf]));
    step(la, ha, sc.y & 0xFFFFu, ws.z);
    step(lb, hb, sc.y >> 16, ws.w);
    if (kb == nkb - 1) {
      if (!*(volatile int *)&sm.abort) emit(it);
#pragma unroll
      for (int c = 0; c < CW / 2; c++) acc[c] = 0ull;
    }
    it = it2;
    kb = kb2;
  }
}

__global__ void __launch_bounds__(TCL_THREADS, 1) tcp_gemm_kernel(TcArgsT p) {
  constexpr int KBN = 4 * 2 * TCP_TT;
  static_assert(TCL_NPROD * KBN <= TC_TMEM_COLS, "two unit buffers of tensor memory");
  static_assert(TCL_EPI == 16, "4 token groups of 8 per lane quarter");
  extern __shared__ __align__(128) unsigned char tc_raw[];
  TcpSmem &sm = *reinterpret_cast<TcpSmem *>(tc_raw + ((1024u - (tc_u32(tc_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ttiles = (p.T + TCP_TT - 1) / TCP_TT;
  const int iters = (int)blockIdx.y < ttiles ? (ttiles - 1 - (int)blockIdx.y) / (int)gridDim.y + 1 : 0;
  const int nunits = iters * p.nkb;
  if (threadIdx.x == 0) {
    for (int s = 0; s < TCL_STAGES; s++) {
      tc_mbar_init(tc_u32(&sm.full[s]), 1);
      tc_mbar_init(tc_u32(&sm.empty[s]), 1);
    }
    for (int b = 0; b < TCL_NPROD; b++) {
      tc_mbar_init(tc_u32(&sm.accfull[b]), 1);
      tc_mbar_init(tc_u32(&sm.accempty[b]), TCL_EPI);
      tc_mbar_init(tc_u32(&sm.drain[b]), 1);
    }
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == TCL_EPI) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_u32(&sm.tmem)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = sm.tmem;
  if (warp >= TCL_EPI) tcp_producer(p, sm, tmem, warp - TCL_EPI, lane, nunits);
  else tcp_epilogue(p, sm, tmem, warp, lane, nunits);
  tc_fence_before();
  __syncthreads();
  if (warp == TCL_EPI) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

}  // namespace llmq
