// Batched greedy decode of independent sequences on sm_100a.
//
// The reference decodes one sequence at a time (generate, gpt2t.mojo:942-980):
// its prompt runs through the several-token path (tile_i16) and every later
// token through the one-token path (dot_row_i16 per output). Here B
// sequences advance together, each with its own KV cache; the decode steps
// keep the one-token arithmetic of every sequence, so each sequence's ids
// are those of its own single-sequence decode.
//
// bquant_kernel      quantize_rows (+ LayerNorm) of B rows into the GEMV's
//                    activation layout (BLOCKED permutation and lane sums for
//                    int4-g32, (group, lane) pair sums otherwise).
// bgemv_a16_kernel   the one-token GEMV for B rows: each thread keeps one
//                    output row's weight words in registers for a unit and
//                    applies them to SB sequences (weights read once per CTA).
// argmax_rows_kernel the first index of the largest logit, per row.
// embed_batch_kernel embeddings of B tokens at one position.
#pragma once

#include "gemv_a16.cuh"
#include "tc_gemm.cuh"

namespace llmq {

struct BQuantArgs {
  const float *x;        // [B][K]
  const float *ln_w, *ln_b;
  int16_t *xq;           // [B][K] (BLOCKED: permuted)
  float *xsf;            // BLOCKED: [B][K / 16] lane sums
  int *xsi;              // other formats: [B][units][16] pair sums
  float *sx;             // [B]
  WeightView w;          // the matrix the rows feed (format, group)
};

// One CTA per row: the same prologue as the one-token GEMV, written out.
template <int FMT, int PRO>
__global__ void __launch_bounds__(256) bquant_kernel(BQuantArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int b = blockIdx.x, K = a.w.cols;
  SmemPlan<FMT> pl(K, a.w.group, 0);
  GemvArgs g{};
  g.w = a.w;
  g.x = a.x + (size_t)b * K;
  g.ln_w = a.ln_w;
  g.ln_b = a.ln_b;
  const float s = prologue<FMT, PRO>(g, smem, pl);
  const int4 *src = (const int4 *)(smem + pl.xq);
  int4 *dst = (int4 *)(a.xq + (size_t)b * K);
  for (int i = threadIdx.x; i < K / 8; i += blockDim.x) dst[i] = src[i];
  if (FMT == FMT_BLK4) {
    const float *xs = (const float *)(smem + pl.xs);
    for (int i = threadIdx.x; i < K / 16; i += blockDim.x) a.xsf[(size_t)b * (K / 16) + i] = xs[i];
  } else {
    const int n = (K / a.w.group) * 16;
    const int *xs = (const int *)(smem + pl.xs);
    for (int i = threadIdx.x; i < n; i += blockDim.x) a.xsi[(size_t)b * n + i] = xs[i];
  }
  if (threadIdx.x == 0) a.sx[b] = s;
}

struct BGemvArgs {
  WeightView w;
  const int16_t *xq;
  const float *xsf;
  const int *xsi;
  const float *sx;
  const float *bias;
  float *out;            // [B][OUT], or null with part_val (the greedy head keeps no logits)
  int B, epi;
  float *part_val;       // with the argmax: [B][gridDim.x] best value of each row tile
  int *part_idx;         //                  and its row
  int *err;              // set when the weight-tile copy wait gave up
};

constexpr int BG_ROWS = 64;  // output rows per CTA (4 threads each)

// Bytes of one weight row of the tile in shared memory: the row padded by 16
// bytes so that the 8 rows a warp reads fall in different banks.
__host__ __device__ inline int bgemv_wstride(int fmt, int K) { return (fmt == FMT_GEN8 ? K : K / 2) + 16; }

// The batched GEMVs' shared-memory prologue: the CTA's weight rows staged by
// bulk copies (STAGE), the SB sequences' activations regrouped so that the
// four pairs thread q multiplies per 16-pair step are 16 contiguous bytes
// (the int8 format's pairs 4q..4q+3 already are), their sums, and a bounded
// wait for the rows. Returns false (every thread) when the wait gave up.
template <int FMT, int SB, bool STAGE>
__device__ __forceinline__ bool bgemv_prologue(const BGemvArgs &a, unsigned char *smem, unsigned long long &wbar,
                                               int row0, int nrows, int b0, int nb) {
  const int K = a.w.cols;
  const int units = FMT == FMT_BLK4 ? K >> 8 : K / a.w.group;
  const int nxs = FMT == FMT_BLK4 ? K / 16 : units * 16;
  const int wstride = bgemv_wstride(FMT, K), rbytes = FMT == FMT_GEN8 ? K : K / 2;
  uint8_t *wt = smem;
  int *xq = (int *)(smem + (STAGE ? (size_t)BG_ROWS * wstride : 0));
  int *xs = xq + (size_t)SB * (K / 2);
  if (STAGE && threadIdx.x == 0) {
    tc_mbar_init(tc_u32(&wbar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc_mbar_expect_tx(tc_u32(&wbar), (unsigned)(nrows * rbytes));
  }
  {
    // The activations, 16 ints (one 16-pair step) per item, read as four
    // int4 and regrouped in registers: each 16-pair step of the int4 formats
    // is regrouped so that the 4 pairs thread q multiplies (2q, 2q+1, 2q+8,
    // 2q+9) are 16 contiguous bytes; the int8 format's pairs 4q..4q+3
    // already are.
    const int4 *src = (const int4 *)(a.xq + (size_t)b0 * K);
    int4 *dst = (int4 *)xq;
    const int items = nb * (K / 32);
    for (int i = threadIdx.x; i < items; i += blockDim.x) {
      int v[16];
#pragma unroll
      for (int k = 0; k < 4; k++) *(int4 *)(v + 4 * k) = src[4 * i + k];
      int w[16];
#pragma unroll
      for (int e = 0; e < 16; e++) w[e] = v[FMT == FMT_GEN8 ? e : (e >> 2) * 2 + (e & 1) + ((e & 2) << 2)];
#pragma unroll
      for (int k = 0; k < 4; k++) dst[4 * i + k] = *(const int4 *)(w + 4 * k);
    }
    const int *s2 = FMT == FMT_BLK4 ? (const int *)(a.xsf + (size_t)b0 * nxs) : a.xsi + (size_t)b0 * nxs;
    for (int i = threadIdx.x; i < nb * nxs; i += blockDim.x) xs[i] = s2[i];
  }
  // the weight rows, one bulk copy per row issued by thread r, after the
  // barrier that publishes the initialised mbarrier
  __syncthreads();
  if (STAGE && threadIdx.x < nrows)
    tc_bulk_g2s(tc_u32(wt + (size_t)threadIdx.x * wstride), a.w.codes + (size_t)(row0 + threadIdx.x) * rbytes, rbytes,
                tc_u32(&wbar));
  // the weight rows' arrival: a bounded wait (all threads), after which a
  // CTA that gave up records the error and computes nothing
  __syncthreads();
  bool ok = true;
  if (STAGE) {
    const long long t0 = clock64();
    while (!tc_mbar_try(tc_u32(&wbar), 0)) {
      if (clock64() - t0 > TC_TIMEOUT) {
        ok = false;
        break;
      }
    }
  }
  if (!__syncthreads_and(ok)) {
    if (threadIdx.x == 0) {
      atomicExch(a.err, 5);
      if (STAGE) tc_drain_wait(tc_u32(&wbar), 0);
    }
    return false;
  }
  return true;
}

// grid (ceil(rows / 64), ceil(B / SB)), 256 threads. Shared memory: the CTA's
// 64 weight rows (STAGE: one bulk copy per row; otherwise they are read from
// global memory), the SB rows' activations and their sums.
template <int FMT, int SB, bool STAGE>
__global__ void __launch_bounds__(256) bgemv_a16_kernel(BGemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ alignas(8) unsigned long long wbar;
  const int K = a.w.cols, G = a.w.group;
  const int units = FMT == FMT_BLK4 ? K >> 8 : K / G;
  const int nxs = FMT == FMT_BLK4 ? K / 16 : units * 16;
  const int b0 = blockIdx.y * SB, nb = min(SB, a.B - b0);
  const int wstride = bgemv_wstride(FMT, K), rbytes = FMT == FMT_GEN8 ? K : K / 2;
  const int row0 = blockIdx.x * BG_ROWS, nrows = min(BG_ROWS, a.w.rows - row0);
  uint8_t *wt = smem;                                        // [64][wstride] weight rows (STAGE)
  int *xq = (int *)(smem + (STAGE ? (size_t)BG_ROWS * wstride : 0));  // [SB][K / 2] int16 pairs, regrouped
  int *xs = xq + (size_t)SB * (K / 2);                       // [SB][nxs] (float bits for BLOCKED)
  if (!bgemv_prologue<FMT, SB, STAGE>(a, smem, wbar, row0, nrows, b0, nb)) return;
  const int q = threadIdx.x & 3, row = blockIdx.x * BG_ROWS + (threadIdx.x >> 2);
  const bool live = row < a.w.rows;
  const int rr = live ? row : a.w.rows - 1;
  const uint8_t *wrow = STAGE ? wt + (size_t)(live ? (threadIdx.x >> 2) : 0) * wstride : a.w.codes + (size_t)rr * rbytes;
  float f[SB][4];
#pragma unroll
  for (int s = 0; s < SB; s++)
#pragma unroll
    for (int j = 0; j < 4; j++) f[s][j] = 0.0f;

  if (FMT == FMT_BLK4) {
    const int gpr = K >> 5;
    for (int u = 0; u < units; u++) {
      uint32_t lo[8], hi[8];
      const uint32_t *wp = (const uint32_t *)(wrow + u * 128) + q;
#pragma unroll
      for (int st = 0; st < 8; st++) {
        const uint32_t v = wp[4 * st];
        lo[st] = v & 0x0F0F0F0Fu;
        hi[st] = (v >> 4) & 0x0F0F0F0Fu;
      }
      float zp[4], sc[4];
      int L[4];
#pragma unroll
      for (int j = 0; j < 4; j++) {
        L[j] = lane_of<FMT_BLK4>(q, j);
        const size_t gi = (size_t)rr * gpr + u * 8 + (L[j] & 7);
        zp[j] = (float)a.w.zp[gi];
        sc[j] = half_bits_to_float(a.w.scale[gi]);
      }
#pragma unroll
      for (int s = 0; s < SB; s++) {
        if (s < nb) {
          const int *x = xq + (size_t)s * (K / 2) + u * 128;
          int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
          for (int st = 0; st < 8; st++) {
            const int4 xx = *(const int4 *)(x + st * 16 + 4 * q);  // pairs 2q, 2q+1, 2q+8, 2q+9
            a0 = dp2a_lo_su(xx.x, lo[st], a0);
            a1 = dp2a_hi_su(xx.y, lo[st], a1);
            a2 = dp2a_lo_su(xx.z, hi[st], a2);
            a3 = dp2a_hi_su(xx.w, hi[st], a3);
          }
          const float *xsum = (const float *)xs + (size_t)s * nxs + u * 16;
          const int acc[4] = {a0, a1, a2, a3};
#pragma unroll
          for (int j = 0; j < 4; j++) f[s][j] = fmaf((float)acc[j] - zp[j] * xsum[L[j]], sc[j], f[s][j]);
        }
      }
    }
  } else {
    const uint8_t *rp = wrow;
    const int cpg = G >> 5;  // 32-chunks per group
    for (int g = 0; g < units; g++) {
      int acc[SB][4];
#pragma unroll
      for (int s = 0; s < SB; s++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[s][j] = 0;
      for (int c = g * cpg; c < (g + 1) * cpg; c++) {
        uint32_t w0, w1;
        if (FMT == FMT_GEN8) {
          const uint2 v = ((const uint2 *)(rp + c * 32))[q];
          w0 = v.x;
          w1 = v.y;
        } else {
          const uint32_t v = ((const uint32_t *)(rp + c * 16))[q];
          w0 = v & 0x0F0F0F0Fu;
          w1 = (v >> 4) & 0x0F0F0F0Fu;
        }
#pragma unroll
        for (int s = 0; s < SB; s++) {
          if (s < nb) {
            const int4 xx = *(const int4 *)(xq + (size_t)s * (K / 2) + c * 16 + 4 * q);
            acc[s][0] = dp2a_lo_su(xx.x, w0, acc[s][0]);
            acc[s][1] = dp2a_hi_su(xx.y, w0, acc[s][1]);
            acc[s][2] = dp2a_lo_su(xx.z, w1, acc[s][2]);
            acc[s][3] = dp2a_hi_su(xx.w, w1, acc[s][3]);
          }
        }
      }
      const size_t gi = (size_t)rr * units + g;
      const int zpv = a.w.zp[gi];
      const float scv = half_bits_to_float(a.w.scale[gi]);
#pragma unroll
      for (int s = 0; s < SB; s++) {
        const int *xsum = xs + (size_t)s * nxs + g * 16;
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const int L = lane_of<FMT>(q, j);
          const int v = (int)((unsigned)acc[s][j] - (unsigned)(zpv * xsum[L]));
          f[s][j] = fmaf((float)v, scv, f[s][j]);
        }
      }
    }
  }
  // halving tree over the 16 lanes of each sequence (as float_phase)
#pragma unroll
  for (int s = 0; s < SB; s++) {
    float dot;
    if (FMT == FMT_GEN8) {
      float t[4];
#pragma unroll
      for (int j = 0; j < 4; j++) t[j] = f[s][j] + __shfl_xor_sync(0xffffffffu, f[s][j], 2);
#pragma unroll
      for (int j = 0; j < 4; j++) t[j] = t[j] + __shfl_xor_sync(0xffffffffu, t[j], 1);
      const float c0 = t[0] + t[2], c1 = t[1] + t[3];
      dot = c0 + c1;
    } else {
      float a0 = f[s][0] + f[s][2], a1 = f[s][1] + f[s][3];
      a0 = a0 + __shfl_xor_sync(0xffffffffu, a0, 2);
      a1 = a1 + __shfl_xor_sync(0xffffffffu, a1, 2);
      const float c0 = a0 + __shfl_xor_sync(0xffffffffu, a0, 1);
      const float c1 = a1 + __shfl_xor_sync(0xffffffffu, a1, 1);
      dot = c0 + c1;
    }
    float v = 0.0f;
    if (live && s < nb) {
      const int b = b0 + s;
      float *dst = a.out ? a.out + (size_t)b * a.w.rows + row : nullptr;
      v = dot * a.sx[b];
      if (a.epi & EPI_BIAS) v += a.bias[row];
      if (a.epi & EPI_GELU) v = gelu(v);
      if ((a.epi & EPI_RESID) && dst) v += *dst;
      if (dst && q == 0) *dst = v;
    }
    if (a.part_val) {
      // this row tile's best row for sequence s: warp, then CTA
      __shared__ float pv[8];
      __shared__ int pi[8];
      float bv = (live && s < nb) ? v : -__int_as_float(0x7f800000);
      int bi = (live && s < nb) ? row : 0x7fffffff;
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      if ((threadIdx.x & 31) == 0) {
        pv[threadIdx.x >> 5] = bv;
        pi[threadIdx.x >> 5] = bi;
      }
      __syncthreads();
      if (threadIdx.x == 0 && s < nb) {
        for (int w = 1; w < 8; w++)
          if (better(pv[w], pi[w], bv, bi)) {
            bv = pv[w];
            bi = pi[w];
          }
        a.part_val[(size_t)(b0 + s) * gridDim.x + blockIdx.x] = bv;
        a.part_idx[(size_t)(b0 + s) * gridDim.x + blockIdx.x] = bi;
      }
      __syncthreads();
    }
  }
}

// The batched GEMV with the roles of weights and activations swapped, for
// the BLOCKED int4-g32 and per-channel int8 formats: grid (ceil(rows / 64),
// ceil(B / 8)), 256 threads; warp w takes rows 8w..8w+7 of the CTA's 64 staged
// rows for the CTA's 8 sequences, lane = (sequence s, q). A thread keeps its
// sequence's activations of one unit (BLOCKED: a 256-block; int8: 8 chunks of
// 32) in registers and applies them to the warp's rows, whose weight words it
// reads from shared memory as broadcasts (all 8 sequences of a warp read the
// same 4 words). The arithmetic per (row, sequence) is bgemv_a16_kernel's:
// the same int32 lane sums, float lane chains in unit order and halving tree.
template <int FMT, int NP>
__global__ void __launch_bounds__(256) bgemv_rows_kernel(BGemvArgs a) {
  constexpr int SB = 8 * NP, RW = BG_ROWS / 8;  // NP passes of 8 sequences over the staged rows
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ alignas(8) unsigned long long wbar;
  __shared__ float pbv[8][SB];
  __shared__ int pbi[8][SB];
  const int K = a.w.cols;
  const int nxs = FMT == FMT_BLK4 ? K / 16 : 16;
  const int b0 = blockIdx.y * SB, nb = min(SB, a.B - b0);
  const int wstride = bgemv_wstride(FMT, K);
  const int row0 = blockIdx.x * BG_ROWS, nrows = min(BG_ROWS, a.w.rows - row0);
  const uint8_t *wt = smem;
  const int *xq = (const int *)(smem + (size_t)BG_ROWS * wstride);
  const int *xs = xq + (size_t)SB * (K / 2);
  if (!bgemv_prologue<FMT, SB, true>(a, smem, wbar, row0, nrows, b0, nb)) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, sq = lane >> 2, q = lane & 3;
  const int rbase = warp * RW;              // this warp's rows in the CTA's tile
  const int nr = max(0, min(RW, nrows - rbase));
  for (int pass = 0; pass < NP; pass++) {
    const int sp = sq + 8 * pass;             // this lane's sequence in the CTA's SB
    const bool sv = sp < nb;
    const int se = sv ? sp : 0;               // an absent sequence computes sequence 0's values, dropped
    float f[RW][4];
#pragma unroll
    for (int r = 0; r < RW; r++)
#pragma unroll
      for (int j = 0; j < 4; j++) f[r][j] = 0.0f;
    if (FMT == FMT_BLK4) {
      const int units = K >> 8, gpr = K >> 5;
      int L[4];
#pragma unroll
      for (int j = 0; j < 4; j++) L[j] = lane_of<FMT_BLK4>(q, j);
      for (int u = 0; u < units; u++) {
        int4 xr[8];
#pragma unroll
        for (int st = 0; st < 8; st++) xr[st] = *(const int4 *)(xq + (size_t)se * (K / 2) + u * 128 + st * 16 + 4 * q);
        float xsum[4];
#pragma unroll
        for (int j = 0; j < 4; j++) xsum[j] = ((const float *)xs)[(size_t)se * nxs + u * 16 + L[j]];
#pragma unroll
        for (int r = 0; r < RW; r++) {
          if (r < nr) {
            const int row = row0 + rbase + r;
            const uint32_t *wp = (const uint32_t *)(wt + (size_t)(rbase + r) * wstride + u * 128) + q;
            int a0 = 0, a1 = 0, a2 = 0, a3 = 0;
#pragma unroll
            for (int st = 0; st < 8; st++) {
              const uint32_t v = wp[4 * st];
              const uint32_t lo = v & 0x0F0F0F0Fu, hi = (v >> 4) & 0x0F0F0F0Fu;
              a0 = dp2a_lo_su(xr[st].x, lo, a0);
              a1 = dp2a_hi_su(xr[st].y, lo, a1);
              a2 = dp2a_lo_su(xr[st].z, hi, a2);
              a3 = dp2a_hi_su(xr[st].w, hi, a3);
            }
            const size_t g0 = (size_t)row * gpr + u * 8 + 2 * q;  // groups of lanes 2q(+8) and 2q+1(+9)
            const float zp0 = (float)a.w.zp[g0], zp1 = (float)a.w.zp[g0 + 1];
            const float sc0 = half_bits_to_float(a.w.scale[g0]), sc1 = half_bits_to_float(a.w.scale[g0 + 1]);
            f[r][0] = fmaf((float)a0 - zp0 * xsum[0], sc0, f[r][0]);
            f[r][1] = fmaf((float)a1 - zp1 * xsum[1], sc1, f[r][1]);
            f[r][2] = fmaf((float)a2 - zp0 * xsum[2], sc0, f[r][2]);
            f[r][3] = fmaf((float)a3 - zp1 * xsum[3], sc1, f[r][3]);
          }
        }
      }
    } else {
      // per-channel int8: one group per row; int32 lane sums over all chunks,
      // one conversion at the end
      int acc[RW][4];
#pragma unroll
      for (int r = 0; r < RW; r++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[r][j] = 0;
      for (int cb = 0; cb < K / 32; cb += 8) {
        int4 xr[8];
#pragma unroll
        for (int c = 0; c < 8; c++) xr[c] = *(const int4 *)(xq + (size_t)se * (K / 2) + (cb + c) * 16 + 4 * q);
#pragma unroll
        for (int r = 0; r < RW; r++) {
          if (r < nr) {
            const uint8_t *rp = wt + (size_t)(rbase + r) * wstride + cb * 32 + 8 * q;
#pragma unroll
            for (int c = 0; c < 8; c++) {
              const uint2 v = *(const uint2 *)(rp + c * 32);
              acc[r][0] = dp2a_lo_su(xr[c].x, v.x, acc[r][0]);
              acc[r][1] = dp2a_hi_su(xr[c].y, v.x, acc[r][1]);
              acc[r][2] = dp2a_lo_su(xr[c].z, v.y, acc[r][2]);
              acc[r][3] = dp2a_hi_su(xr[c].w, v.y, acc[r][3]);
            }
          }
        }
      }
#pragma unroll
      for (int r = 0; r < RW; r++) {
        if (r < nr) {
          const int row = row0 + rbase + r;
          const int zpv = a.w.zp[row];
          const float scv = half_bits_to_float(a.w.scale[row]);
#pragma unroll
          for (int j = 0; j < 4; j++) {
            const int v = (int)((unsigned)acc[r][j] - (unsigned)(zpv * xs[(size_t)se * nxs + 4 * q + j]));
            f[r][j] = fmaf((float)v, scv, f[r][j]);
          }
        }
      }
    }
    // halving tree over each row's 16 lanes (the four threads of a sequence),
    // epilogue, and for the head the best row per sequence
    float bv = -__int_as_float(0x7f800000);
    int bi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < RW; r++) {
      float dot;
      if (FMT == FMT_GEN8) {
        float t[4];
#pragma unroll
        for (int j = 0; j < 4; j++) t[j] = f[r][j] + __shfl_xor_sync(0xffffffffu, f[r][j], 2);
#pragma unroll
        for (int j = 0; j < 4; j++) t[j] = t[j] + __shfl_xor_sync(0xffffffffu, t[j], 1);
        dot = (t[0] + t[2]) + (t[1] + t[3]);
      } else {
        float a0 = f[r][0] + f[r][2], a1 = f[r][1] + f[r][3];
        a0 = a0 + __shfl_xor_sync(0xffffffffu, a0, 2);
        a1 = a1 + __shfl_xor_sync(0xffffffffu, a1, 2);
        const float c0 = a0 + __shfl_xor_sync(0xffffffffu, a0, 1);
        const float c1 = a1 + __shfl_xor_sync(0xffffffffu, a1, 1);
        dot = c0 + c1;
      }
      if (r < nr && sv) {
        const int row = row0 + rbase + r, b = b0 + sp;
        float *dst = a.out ? a.out + (size_t)b * a.w.rows + row : nullptr;
        float v = dot * a.sx[b];
        if (a.epi & EPI_BIAS) v += a.bias[row];
        if (a.epi & EPI_GELU) v = gelu(v);
        if ((a.epi & EPI_RESID) && dst) v += *dst;
        if (dst && q == 0) *dst = v;
        if (better(v, row, bv, bi)) {
          bv = v;
          bi = row;
        }
      }
    }
    if (a.part_val) {
      if (q == 0) {
        pbv[warp][sq] = bv;
        pbi[warp][sq] = bi;
      }
      __syncthreads();
      if (threadIdx.x < 8 && threadIdx.x + 8 * pass < nb) {
        const int s = threadIdx.x;
        float v = pbv[0][s];
        int i = pbi[0][s];
        for (int w = 1; w < 8; w++)
          if (better(pbv[w][s], pbi[w][s], v, i)) {
            v = pbv[w][s];
            i = pbi[w][s];
          }
        a.part_val[(size_t)(b0 + s + 8 * pass) * gridDim.x + blockIdx.x] = v;
        a.part_idx[(size_t)(b0 + s + 8 * pass) * gridDim.x + blockIdx.x] = i;
      }
      __syncthreads();
    }
  }
}

// The argmax of each sequence from the row tiles' partials (first index of
// the largest value; every value NaN keeps index 0, as the reference's scan).
__global__ void argmax_parts_kernel(const float *part_val, const int *part_idx, int nparts, int *ids, int stride,
                                    int *tokens, const int *col) {
  __shared__ float rv[32];
  __shared__ int ri[32];
  const float *pv = part_val + (size_t)blockIdx.x * nparts;
  const int *pi = part_idx + (size_t)blockIdx.x * nparts;
  float bv = -__int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < nparts; i += blockDim.x)
    if (better(pv[i], pi[i], bv, bi)) {
      bv = pv[i];
      bi = pi[i];
    }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    rv[threadIdx.x >> 5] = bv;
    ri[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (better(rv[w], ri[w], bv, bi)) {
        bv = rv[w];
        bi = ri[w];
      }
    if (bi == 0x7fffffff) bi = 0;
    ids[(size_t)blockIdx.x * stride + (col ? *col : 0)] = bi;
    tokens[blockIdx.x] = bi;
  }
}

__host__ __device__ inline size_t bgemv_smem(int fmt, int K, int G, int SB, bool stage) {
  const int nxs = fmt == FMT_BLK4 ? K / 16 : (K / G) * 16;
  return (stage ? (size_t)BG_ROWS * bgemv_wstride(fmt, K) : 0) + (size_t)SB * (K / 2) * 4 + (size_t)SB * nxs * 4;
}

// First index of the largest value of each row (argmax, gpt2t.mojo:792-797);
// one CTA per row. ids[row * stride + *col] (column 0 without col) receives
// it, and tokens[row] too.
__global__ void __launch_bounds__(256) argmax_rows_kernel(const float *logits, int V, int *ids, int stride,
                                                          int *tokens, const int *col) {
  __shared__ float rv[32];
  __shared__ int ri[32];
  const float *row = logits + (size_t)blockIdx.x * V;
  float bv = -__int_as_float(0x7f800000);
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x)
    if (better(row[i], i, bv, bi)) {
      bv = row[i];
      bi = i;
    }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    rv[threadIdx.x >> 5] = bv;
    ri[threadIdx.x >> 5] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); w++)
      if (better(rv[w], ri[w], bv, bi)) {
        bv = rv[w];
        bi = ri[w];
      }
    if (bi == 0x7fffffff) bi = 0;  // every logit NaN: the scan keeps index 0
    ids[(size_t)blockIdx.x * stride + (col ? *col : 0)] = bi;
    tokens[blockIdx.x] = bi;
  }
}

// Embeddings of B tokens at position *pos (gpt2t.mojo:378-385); one CTA per row.
__global__ void embed_batch_kernel(WeightView head, const float *wpe, float *x, const int *tokens, const int *pos) {
  const int b = blockIdx.x, C = head.cols, gpr = head.cols / head.group;
  const int token = min(max(tokens[b], 0), head.rows - 1), p = *pos;  // ids were checked on the host
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    const size_t gi = (size_t)token * gpr + i / head.group;
    const float s = half_bits_to_float(head.scale[gi]);
    const float v = (float)(code_at(head, token, i) - (int)head.zp[gi]) * s;
    x[(size_t)b * C + i] = v + wpe[(size_t)p * C + i];
  }
}

}  // namespace llmq
