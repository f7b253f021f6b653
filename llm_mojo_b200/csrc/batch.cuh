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
  if (STAGE && threadIdx.x == 0) {
    tc_mbar_init(tc_u32(&wbar), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc_mbar_expect_tx(tc_u32(&wbar), (unsigned)(nrows * rbytes));
    for (int r = 0; r < nrows; r++)
      tc_bulk_g2s(tc_u32(wt + (size_t)r * wstride), a.w.codes + (size_t)(row0 + r) * rbytes, rbytes, tc_u32(&wbar));
  }
  {
    // Each 16-pair step of the int4 formats is regrouped so that the 4 pairs
    // thread q multiplies (2q, 2q+1, 2q+8, 2q+9) are 16 contiguous bytes; the
    // int8 format's pairs 4q..4q+3 already are.
    const int *src = (const int *)(a.xq + (size_t)b0 * K);
    for (int i = threadIdx.x; i < nb * (K / 2); i += blockDim.x) {
      const int e = i & 15;
      const int from = FMT == FMT_GEN8 ? e : (e >> 2) * 2 + (e & 1) + ((e & 2) << 2);
      xq[i] = src[(i & ~15) + from];
    }
    const int *s2 = FMT == FMT_BLK4 ? (const int *)(a.xsf + (size_t)b0 * nxs) : a.xsi + (size_t)b0 * nxs;
    for (int i = threadIdx.x; i < nb * nxs; i += blockDim.x) xs[i] = s2[i];
  }
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
    return;
  }
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
