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
// The pipeline is the transposed GEMM's (tc_gemm.cuh): 4 stages of
// [A: 128 rows x 128 B][B: 4 TT rows x 128 B] in the 128-byte swizzle
// layout, warp 16 issuing copies, MMAs and commits, warps 0-15 folding (warp
// w: tensor-memory lanes = weight rows 32 * (w % 4) + lane, sequences
// (w / 4) * TT / 4 .. + TT / 4), accumulators in rotating buffers of 4 TT
// columns. The epilogue keeps 5 floats per (row, sequence): the pair's two
// lane chains and the tree's partial sums.
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
  if (w.cols % 256 != 0) return false;
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

// quantize_rows (+ LayerNorm) of each sequence's row (kernels.mojo:400-416,
// the one-token prologue's arithmetic in natural column order) into the B
// tiles [sequence tile][K block][4 TT rows x 128 B]: row (plane p, half h)
// at (2p + h) * TT + t holds, in the K step's half h, the low byte xl (p = 0)
// or the high byte xh (p = 1) of x at column tcl_col(k), and zero in the
// other half. Also sx[m] and, for the int8 rows, the 16 lane sums of x
// (columns 2L, 2L + 1 of every 32-column chunk). One CTA per sequence of the
// padded count; padding sequences get zero tiles.
template <int TT, int PRO>
__global__ void __launch_bounds__(256) tcl_quant_pack_kernel(const float *x, const float *ln_w, const float *ln_b,
                                                             int B, int K, int mode, uint8_t *b, float *sx,
                                                             int *xsl) {
  extern __shared__ __align__(16) unsigned char qsm[];
  const int m = blockIdx.x, nkb = K / TC_KB, tt = m / TT, r = m % TT;
  const bool valid = m < B;
  SmemPlan<FMT_GEN8> pl(K, K, 0);
  const int16_t *xq = (const int16_t *)(qsm + pl.xq);
  if (valid) {
    GemvArgs g{};
    g.w.cols = K;
    g.w.group = K;
    g.w.bits = 8;
    g.x = x + (size_t)m * K;
    g.ln_w = ln_w;
    g.ln_b = ln_b;
    const float s = prologue<FMT_GEN8, PRO>(g, qsm, pl);
    if (threadIdx.x == 0) sx[m] = s;
    if (mode == TCL_CH8 && threadIdx.x < 16) xsl[(size_t)m * 16 + threadIdx.x] = ((const int *)(qsm + pl.xs))[threadIdx.x];
  }
  uint8_t *tile = b + (size_t)tt * nkb * (4 * TT * TC_KB);
  for (int ci = threadIdx.x; ci < K / 16; ci += blockDim.x) {
    const int k0 = ci * 16, kb = k0 / TC_KB, chunk = (k0 % TC_KB) / 16, half = (k0 >> 4) & 1;
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    if (valid) {
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const unsigned q = (uint16_t)xq[tcl_col(mode, k0 + i, K)];
        lo[i >> 2] |= (q & 0xFFu) << (8 * (i & 3));
        hi[i >> 2] |= ((q >> 8) & 0xFFu) << (8 * (i & 3));
      }
    }
    uint8_t *kbase = tile + (size_t)kb * (4 * TT * TC_KB);
    const uint4 zero = make_uint4(0, 0, 0, 0);
    *(uint4 *)(kbase + tc_sw128_off(half * TT + r, chunk)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *(uint4 *)(kbase + tc_sw128_off(2 * TT + half * TT + r, chunk)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
    *(uint4 *)(kbase + tc_sw128_off((1 - half) * TT + r, chunk)) = zero;
    *(uint4 *)(kbase + tc_sw128_off(2 * TT + (1 - half) * TT + r, chunk)) = zero;
  }
}

struct TcArgsL {
  const uint8_t *a;   // weight tiles (tcl_prep_a_kernel)
  const uint8_t *b;   // sequence tiles (tcl_quant_pack_kernel)
  const float *sx;    // [sequences] activation scales
  const int *xsl;     // int8 rows: [sequences][16] lane sums of x
  WeightView w;
  const float *bias;  // int4 rows: [rows] or null
  float *out;         // int4 rows: [sequences][rows]
  float *part_val;    // int8 rows: [sequences][row tiles] argmax candidates
  int *part_idx;
  int *err;
  int B, OUT, K, nkb, nseg, epi;
};

template <int TT>
struct TcSmemL {
  alignas(1024) uint8_t stage[TC_STAGES][TCT_A_BYTES + 4 * TT * TC_KB];
  int xsl[TT][16];
  uint16_t scl[TC_MAX_GROUPS][TC_M];  // int4 rows: the tile's float16 scales, [group][row]
  float cand_v[4][TT];
  int cand_i[4][TT];
  alignas(8) unsigned long long full[TC_STAGES], empty[TC_STAGES], accfull[TC_NBUF_MAX], accempty[TC_NBUF_MAX],
      drain;
  unsigned tmem;
  int abort;
};

// The halving tree, fed one lane pair at a time in tcl_pair_lane order:
// s8 = lane g + lane g + 8; pairs (0, 4), (2, 6), (1, 5), (3, 7) make
// s4[0], s4[2], s4[1], s4[3]; s2[0] = s4[0] + s4[2], s2[1] = s4[1] + s4[3],
// dot = s2[0] + s2[1], left in r2 after the last pair (returns true then).
__device__ __forceinline__ bool tcl_tree(int gp, float s8, float &p8, float &q4, float &r2) {
  if ((gp & 1) == 0) {
    p8 = s8;
    return false;
  }
  const float s4 = p8 + s8;
  if (gp == 1 || gp == 5) {
    q4 = s4;
    return false;
  }
  const float s2 = q4 + s4;
  if (gp == 3) {
    r2 = s2;
    return false;
  }
  r2 = r2 + s2;
  return true;
}

// Warps 0-15: per K step (segment) of the permuted order, the accumulators of
// this thread's weight row and CW sequences: groups (plane p, half h) at
// columns (2p + h) * TT. int4 rows fold lanes g and g + 8 of block b into
// their chains and close the pair after the row's last block; int8 rows add
// the halves into the pair's two int32 lane sums and close the pair after its
// third K step. The row value then goes to out (int4) or to the tile's
// argmax candidates (int8). The next segment's tensor-memory loads are in
// flight while this one folds.
template <int MODE, int TT>
__device__ __forceinline__ void tcl_epilogue(const TcArgsL &p, TcSmemL<TT> &sm, unsigned tmem, int warp, int lane,
                                             int n0, int t0) {
  constexpr int N = 4 * TT, NBUF = TC_TMEM_COLS / N, CW = TT / 4;
  const int q = warp & 3, cg = warp >> 2, rl = 32 * q + lane;
  const int n = n0 + rl;  // this thread's weight row
  const int nr = n < p.w.rows ? n : p.w.rows - 1;
  const unsigned tbase = tmem + ((unsigned)(32 * q) << 16) + cg * CW;
  float ca[CW], cb[CW], p8[CW], q4[CW], r2[CW];  // r2 ends as the row's dot
  int ia[CW], ib[CW];  // int8 rows: the pair's lane sums
#pragma unroll
  for (int c = 0; c < CW; c++) {
    ca[c] = cb[c] = p8[c] = q4[c] = r2[c] = 0.0f;
    ia[c] = ib[c] = 0;
  }
  const int nblk = p.K >> 8;  // int4 rows: K steps per lane pair
  const int spp = p.K / 256;  // int8 rows: K steps per lane pair (3 for 768 columns: 2 lanes x 48)
  float sc8 = 0.0f;
  int zp8 = 0;
  if (MODE == TCL_CH8) {
    sc8 = half_bits_to_float(p.w.scale[nr]);
    zp8 = p.w.zp[nr];
  }
  int d[4][CW];  // the next segment's accumulators, loads in flight while this one folds
  // the segment being folded, its halves combined: int4 rows as floats
  // (256 high + low), int8 rows as unsigned lane-sum increments
  float fa[CW], fb[CW];
  unsigned ua[CW], ub[CW];
  auto start = [&](int seg) -> bool {
    const int buf = seg % NBUF;
    bool ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accfull[buf]), (seg / NBUF) & 1, p.err, TC_ERR_ACC);
    ok = __all_sync(0xffffffffu, ok);  // the tensor-memory loads are warp-wide
    if (!ok) return false;
    tc_fence_after();
#pragma unroll
    for (int g4 = 0; g4 < 4; g4++) tc_ld(tbase + buf * N + g4 * TT, d[g4]);
    return true;
  };
  auto finish = [&](int seg) {
    tc_ld_wait();
#pragma unroll
    for (int g4 = 0; g4 < 4; g4++) tc_ld_done(d[g4]);
    tc_fence_before();
    __syncwarp();
    if (lane == 0) tc_mbar_arrive(tc_u32(&sm.accempty[seg % NBUF]));
#pragma unroll
    for (int c = 0; c < CW; c++) {
      if (MODE == TCL_BLK4) {
        // |high| < 2^15, |low| < 2^16: exact floats, one rounding in the fma,
        // as the reference's f32(lane) - zp * f32(lane sum of x)
        fa[c] = fmaf(256.0f, tc_small_to_float(d[2][c]), tc_small_to_float(d[0][c]));
        fb[c] = fmaf(256.0f, tc_small_to_float(d[3][c]), tc_small_to_float(d[1][c]));
      } else {
        ua[c] = ((unsigned)d[2][c] << 8) + (unsigned)d[0][c];
        ub[c] = ((unsigned)d[3][c] << 8) + (unsigned)d[1][c];
      }
    }
  };
  auto fold = [&](int seg) {
    if (MODE == TCL_BLK4) {
      const int gp = seg / nblk, b = seg - gp * nblk, g = tcl_pair_lane(gp);
      const float sc = half_bits_to_float(sm.scl[b * 8 + g][rl]);
#pragma unroll
      for (int c = 0; c < CW; c++) {
        ca[c] = fmaf(fa[c], sc, ca[c]);
        cb[c] = fmaf(fb[c], sc, cb[c]);
      }
      if (b == nblk - 1) {
#pragma unroll
        for (int c = 0; c < CW; c++) {
          tcl_tree(gp, ca[c] + cb[c], p8[c], q4[c], r2[c]);
          ca[c] = cb[c] = 0.0f;
        }
      }
    } else {
      const int gp = seg / spp, s3 = seg - gp * spp, g = tcl_pair_lane(gp);
      const int h0 = 2 * s3;  // halves [0, spp) are lane g, [spp, 2 spp) lane g + 8
#pragma unroll
      for (int c = 0; c < CW; c++) {
        if (h0 < spp) ia[c] = (int)((unsigned)ia[c] + ua[c]);
        else ib[c] = (int)((unsigned)ib[c] + ua[c]);
        if (h0 + 1 < spp) ia[c] = (int)((unsigned)ia[c] + ub[c]);
        else ib[c] = (int)((unsigned)ib[c] + ub[c]);
      }
      if (s3 == spp - 1) {
#pragma unroll
        for (int c = 0; c < CW; c++) {
          const int t = cg * CW + c;
          const int a0 = (int)((unsigned)ia[c] - (unsigned)(zp8 * sm.xsl[t][g]));
          const int a1 = (int)((unsigned)ib[c] - (unsigned)(zp8 * sm.xsl[t][g + 8]));
          const float fx = fmaf((float)a0, sc8, 0.0f), fy = fmaf((float)a1, sc8, 0.0f);
          tcl_tree(gp, fx + fy, p8[c], q4[c], r2[c]);
          ia[c] = ib[c] = 0;
        }
      }
    }
  };
  bool ok = start(0);
  if (ok) finish(0);
  for (int seg = 0; ok && seg < p.nseg; seg++) {
    const bool more = seg + 1 < p.nseg;
    if (more) ok = start(seg + 1);
    fold(seg);
    if (!ok || !more) break;
    finish(seg + 1);
  }
  if (!ok || *(volatile int *)&sm.abort) return;
  if (MODE == TCL_BLK4) {
    if (n >= p.OUT) return;
    const float bn = (p.epi & EPI_BIAS) ? p.bias[n] : 0.0f;
#pragma unroll
    for (int c = 0; c < CW; c++) {
      const int m = t0 + cg * CW + c;
      if (m >= p.B) break;
      float *dst = p.out + (size_t)m * p.OUT + n;
      float r = r2[c] * p.sx[m];
      if (p.epi & EPI_BIAS) r += bn;
      if (p.epi & EPI_GELU) r = gelu(r);
      if (p.epi & EPI_RESID) r += *dst;
      *dst = r;
    }
  } else {
    // the tile's argmax candidate per sequence: the best of the warp's 32
    // rows by shuffles, then of the four warps of the sequence group
#pragma unroll
    for (int c = 0; c < CW; c++) {
      const int m = t0 + cg * CW + c;
      float bv = -__int_as_float(0x7f800000);
      int bi = 0x7fffffff;
      if (n < p.w.rows && m < p.B) {
        const float v = r2[c] * p.sx[m];
        if (better(v, n, bv, bi)) {
          bv = v;
          bi = n;
        }
      }
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if (lane == 0) {
        sm.cand_v[q][cg * CW + c] = bv;
        sm.cand_i[q][cg * CW + c] = bi;
      }
    }
  }
}

// The int8 rows' candidates of the four lane quarters, per sequence, to
// part_val / part_idx[sequence][row tile] (after the epilogue's barrier).
template <int TT>
__device__ __forceinline__ void tcl_store_candidates(const TcArgsL &p, TcSmemL<TT> &sm, int t0, int nt, int ntiles) {
  const int t = threadIdx.x;
  if (t >= TT || t0 + t >= p.B || *(volatile int *)&sm.abort) return;
  float bv = sm.cand_v[0][t];
  int bi = sm.cand_i[0][t];
  for (int k = 1; k < 4; k++)
    if (better(sm.cand_v[k][t], sm.cand_i[k][t], bv, bi)) {
      bv = sm.cand_v[k][t];
      bi = sm.cand_i[k][t];
    }
  p.part_val[(size_t)(t0 + t) * ntiles + nt] = bv;
  p.part_idx[(size_t)(t0 + t) * ntiles + nt] = bi;
}

template <int MODE, int TT>
__global__ void __launch_bounds__(TC_THREADS, 1) tcl_gemm_kernel(TcArgsL p) {
  constexpr int N = 4 * TT;                  // MMA N: 4 rows per sequence
  constexpr int NBUF = TC_TMEM_COLS / N;     // accumulator buffers in tensor memory
  constexpr int CW = TT / 4;                 // sequences per epilogue warp
  constexpr int BB = N * TC_KB;              // sequence-tile bytes per K block
  constexpr int STAGE = TCT_A_BYTES + BB;
  static_assert(CW == 8 || CW == 16, "tc_ld widths");
  extern __shared__ __align__(128) unsigned char tc_raw[];
  TcSmemL<TT> &sm = *reinterpret_cast<TcSmemL<TT> *>(tc_raw + ((1024u - (tc_u32(tc_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.y, tt = blockIdx.x, n0 = nt * TC_M, t0 = tt * TT;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; s++) {
      tc_mbar_init(tc_u32(&sm.full[s]), 1);
      tc_mbar_init(tc_u32(&sm.empty[s]), 1);
    }
    for (int b = 0; b < NBUF; b++) {
      tc_mbar_init(tc_u32(&sm.accfull[b]), 1);
      tc_mbar_init(tc_u32(&sm.accempty[b]), TC_EPI_WARPS);
    }
    tc_mbar_init(tc_u32(&sm.drain), 1);
    sm.abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == TC_EPI_WARPS) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(tc_u32(&sm.tmem)),
                 "r"(TC_TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  } else if (MODE == TCL_CH8) {
    for (int i = threadIdx.x; i < TT * 16; i += TC_EPI_WARPS * 32) {
      const int t = t0 + i / 16;
      sm.xsl[i / 16][i % 16] = t < p.B ? p.xsl[(size_t)t * 16 + i % 16] : 0;
    }
  } else {
    // the tile's scales as [group][row] (rows past the matrix: 0)
    const int gpr = p.K / p.w.group;
    for (int i = threadIdx.x; i < gpr * TC_M; i += TC_EPI_WARPS * 32) {
      const int r = i / gpr, g = i - r * gpr, row = n0 + r;
      sm.scl[g][r] = row < p.w.rows ? p.w.scale[(size_t)row * gpr + g] : (uint16_t)0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = sm.tmem;

  if (warp == TC_EPI_WARPS) {
    // the whole warp runs the loop (waits included); lane 0 issues the
    // copies, MMAs and commits. One MMA per K step: each K step is a whole
    // segment (two lanes), its accumulators a fresh buffer.
    const bool leader = lane == 0;
    // low rows (u8) and high rows (s8), N = 2 TT each
    const unsigned idesc_l = tc_idesc(MODE == TCL_BLK4 ? 1 : 0, 0, 2 * TT);
    const unsigned idesc_h = tc_idesc(MODE == TCL_BLK4 ? 1 : 0, 1, 2 * TT);
    constexpr unsigned long long HIGH = (2 * TT * TC_KB) >> 4;  // descriptor start of the high rows
    const unsigned long long desc_a0 = tc_desc_sw128(tc_u32(sm.stage[0]));
    const unsigned long long desc_b0 = tc_desc_sw128(tc_u32(sm.stage[0]) + TCT_A_BYTES);
    const uint8_t *ga = p.a + (size_t)nt * p.nkb * TCT_A_BYTES;
    const uint8_t *gb = p.b + (size_t)tt * p.nkb * BB;
    int issued = 0, waited = 0;
    auto issue = [&](int kb) {
      const int st = kb % TC_STAGES;
      const unsigned dst = tc_u32(sm.stage[st]), bar = tc_u32(&sm.full[st]);
      if (leader) {
        tc_mbar_expect_tx(bar, STAGE);
        tc_bulk_g2s(dst, ga + (size_t)kb * TCT_A_BYTES, TCT_A_BYTES, bar);
        tc_bulk_g2s(dst + TCT_A_BYTES, gb + (size_t)kb * BB, BB, bar);
      }
      __syncwarp();
    };
    for (; issued < p.nkb && issued < TC_STAGES; issued++) issue(issued);
    bool ok = true;
    for (int seg = 0; seg < p.nseg && ok; seg++) {
      const int buf = seg % NBUF, kb = seg >> 2, j = seg & 3, st = kb % TC_STAGES;
      if (seg >= NBUF)
        ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accempty[buf]), ((seg / NBUF) - 1) & 1, p.err, TC_ERR_ACCEMPTY);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      if (j == 0) {
        ok = tc_wait_flag(&sm.abort, tc_u32(&sm.full[st]), (kb / TC_STAGES) & 1, p.err, TC_ERR_FULL);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        waited = kb + 1;
      }
      tc_fence_after();
      const unsigned long long off = (unsigned long long)((st * STAGE) >> 4);
      if (leader) {
        const unsigned long long da = desc_a0 + off + (unsigned long long)(2 * j);
        const unsigned long long db = desc_b0 + off + (unsigned long long)(2 * j);
        tc_mma(tmem + buf * N, da, db, idesc_l, 0);
        tc_mma(tmem + buf * N + 2 * TT, da, db + HIGH, idesc_h, 0);
        tc_commit(tc_u32(&sm.accfull[buf]));
      }
      __syncwarp();
      if (j == 3) {
        if (leader) tc_commit(tc_u32(&sm.empty[st]));
        __syncwarp();
        // refill the stage of the previous K block, whose MMAs were queued
        // ahead of these
        if (kb >= 1 && issued < p.nkb) {
          const int pkb = kb - 1;
          ok = tc_wait_flag(&sm.abort, tc_u32(&sm.empty[pkb % TC_STAGES]), (pkb / TC_STAGES) & 1, p.err,
                            TC_ERR_EMPTY);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          issue(issued++);
        }
      }
    }
    if (!ok) {
      // drain: copies issued but not yet waited for, then every MMA issued
      for (int kb = waited; kb < issued; kb++) tc_drain_wait(tc_u32(&sm.full[kb % TC_STAGES]), (kb / TC_STAGES) & 1);
      if (leader) tc_commit(tc_u32(&sm.drain));
      __syncwarp();
      tc_drain_wait(tc_u32(&sm.drain), 0);
    }
  } else {
    tcl_epilogue<MODE, TT>(p, sm, tmem, warp, lane, n0, t0);
  }
  tc_fence_before();
  __syncthreads();
  if (MODE == TCL_CH8) tcl_store_candidates<TT>(p, sm, t0, nt, gridDim.y);
  if (warp == TC_EPI_WARPS) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

}  // namespace llmq
