// Float-activation several-token paths on sm_100a: the dense matmul tile
// (mm_tile / matmul, kernels.mojo:51-129), the tied head for every position
// (lm_head_rows, kernels.mojo:230-271), GGUF rows for several tokens
// (matmul_rows / rows_dot, kernels.mojo:285-397), float embeddings, and the
// per-row scores of the perplexity harness (score_rows, gpt2t.mojo:1042-1097).
//
// The float orders are the reference's, so results are bit-identical:
//   mm_tile:      out[t][j] = chain over i of fma(x[t][i], w(i, j), acc),
//                 then + b[j], store_out;
//   lm_head_rows: 16 lane chains fma(h[i+l], w[v][i+l], d[l]) over i in
//                 steps of 16, then the halving tree;
//   rows_dot:     the same 16-lane chains over a dequantized row, + bias.
#pragma once

#include "gemv_a16.cuh"
#include "gemv_float.cuh"

namespace llmq {

template <int WT>
__device__ __forceinline__ float wload(const void *w, size_t i) {
  if (WT == 0) return ((const float *)w)[i];
  return __uint_as_float((unsigned)((const uint16_t *)w)[i] << 16);  // bfloat16 widened
}

constexpr int DM_T = 64, DM_N = 64, DM_K = 16;

// out[T][OUT] (+)= act(x[T][IN] @ w + b): w is [IN][OUT] (the Conv1D layout
// of DenseMatrix layers, NK = false) or [OUT][IN] (rows, NK = true: GGUF
// rows dequantized to float32). WT: 0 float32, 1 bfloat16. Columns
// >= n_end are left alone. 64 x 64 tiles, 256 threads of 4 x 4 outputs;
// every output is one fma chain over i in order.
template <int WT, bool NK>
__global__ void __launch_bounds__(256) dense_mm_kernel(const void *w, const float *x, const float *bias, float *out,
                                                       int T, int IN, int OUT, int n_end, int epi) {
  __shared__ float xs[DM_K][DM_T + 1];
  __shared__ float ws[DM_K][DM_N + 1];
  const int t0 = blockIdx.y * DM_T, n0 = blockIdx.x * DM_N;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) acc[a][b] = 0.0f;
  for (int k0 = 0; k0 < IN; k0 += DM_K) {
    for (int i = threadIdx.x; i < DM_K * DM_T; i += 256) {
      const int kk = i % DM_K, r = i / DM_K, t = t0 + r, k = k0 + kk;
      xs[kk][r] = (t < T && k < IN) ? x[(size_t)t * IN + k] : 0.0f;
    }
    for (int i = threadIdx.x; i < DM_K * DM_N; i += 256) {
      int kk, c;
      if (NK) {
        kk = i % DM_K;
        c = i / DM_K;
      } else {
        c = i % DM_N;
        kk = i / DM_N;
      }
      const int n = n0 + c, k = k0 + kk;
      float v = 0.0f;
      if (n < n_end && k < IN) v = NK ? wload<WT>(w, (size_t)n * IN + k) : wload<WT>(w, (size_t)k * OUT + n);
      ws[kk][c] = v;
    }
    __syncthreads();
    const int kn = min(DM_K, IN - k0);
    for (int kk = 0; kk < kn; kk++) {
      float a[4], b[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        a[u] = xs[kk][ty + 16 * u];
        b[u] = ws[kk][tx + 16 * u];
      }
#pragma unroll
      for (int u = 0; u < 4; u++)
#pragma unroll
        for (int v = 0; v < 4; v++) acc[u][v] = fmaf(a[u], b[v], acc[u][v]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; u++) {
    const int t = t0 + ty + 16 * u;
    if (t >= T) continue;
#pragma unroll
    for (int v = 0; v < 4; v++) {
      const int n = n0 + tx + 16 * v;
      if (n >= n_end) continue;
      float r = acc[u][v];
      if (epi & EPI_BIAS) r += bias[n];
      if (epi & EPI_GELU) r = gelu(r);
      float *dst = out + (size_t)t * OUT + n;
      if (epi & EPI_RESID) r += *dst;
      *dst = r;
    }
  }
}

// logits[T][V] = h[T][C] @ wte[V][C]^T, lm_head_rows' order. CTA = 16 lanes x
// 16 groups; group g covers 4 tokens x 4 rows of a 16 x 16 tile; lane l runs
// the chains of elements l, l + 16, ...; the halving tree across the lanes.
template <int WT>
__global__ void __launch_bounds__(256) dense_head_rows_kernel(const void *w, const float *h, float *logits, int T,
                                                              int V, int C) {
  __shared__ float hs[16][17];
  __shared__ float wsm[16][17];
  const int l = threadIdx.x & 15, g = threadIdx.x >> 4, gt = g >> 2, gv = g & 3;
  const int t0 = blockIdx.y * 16, v0 = blockIdx.x * 16;
  float d[4][4];
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) d[a][b] = 0.0f;
  for (int i0 = 0; i0 < C; i0 += 16) {
    {
      const int r = threadIdx.x >> 4, c = threadIdx.x & 15;
      const int t = t0 + r, v = v0 + r;
      hs[r][c] = t < T ? h[(size_t)t * C + i0 + c] : 0.0f;
      wsm[r][c] = v < V ? wload<WT>(w, (size_t)v * C + i0 + c) : 0.0f;
    }
    __syncthreads();
#pragma unroll
    for (int a = 0; a < 4; a++)
#pragma unroll
      for (int b = 0; b < 4; b++) d[a][b] = fmaf(hs[gt * 4 + a][l], wsm[gv * 4 + b][l], d[a][b]);
    __syncthreads();
  }
#pragma unroll
  for (int a = 0; a < 4; a++)
#pragma unroll
    for (int b = 0; b < 4; b++) {
      float e = d[a][b];
      e = e + __shfl_xor_sync(0xffffffffu, e, 8);
      e = e + __shfl_xor_sync(0xffffffffu, e, 4);
      e = e + __shfl_xor_sync(0xffffffffu, e, 2);
      e = e + __shfl_xor_sync(0xffffffffu, e, 1);
      const int t = t0 + gt * 4 + a, v = v0 + gv * 4 + b;
      if (l == 0 && t < T && v < V) logits[(size_t)t * V + v] = e;
    }
}

// Rows [r0, r0 + gridDim.x * 16) of a GGUF matrix dequantized to float32
// (dequant_row, gguf.mojo:395-434): dst[row - r0][cols]. 256 threads = 16
// rows x 16 lanes.
template <int T>
__global__ void __launch_bounds__(256) gguf_dequant_rows_kernel(RowMat w, int r0, int nrows, float *dst) {
  const int L = threadIdx.x & 15, rr = blockIdx.x * 16 + (threadIdx.x >> 4);
  if (rr >= nrows) return;
  const int row = r0 + rr, bs = rt_block_size(T), bb = rt_block_bytes(T);
  const uint8_t *p = w.data + (size_t)row * w.row_bytes;
  float *o = dst + (size_t)rr * w.cols;
  if (T == RT_F32 || T == RT_F16 || T == RT_BF16) {
    for (int i0 = 0; i0 < w.cols; i0 += 16)
      block_values<T>(p + (size_t)i0 * bb, L, [&](float v, int i) { o[i0 + i] = v; });
  } else {
    for (int blk = 0; blk < w.cols / bs; blk++)
      block_values<T>(p + (size_t)blk * bb, L, [&](float v, int i) { o[blk * bs + i] = v; });
  }
}

// QuantMatrix.dequant_row (tensor.mojo:431-479, the natural layout of the
// W4A32 / W8A32 formats): value k of row r0 + rr is (u - zp) * scale, the
// code and the zero point as exact floats, one rounding in the product.
// One thread per pair of bytes' worth of values (two int4 codes of a byte
// for 4 bits, one code for 8), rows [r0, r0 + nrows) into dst[rr][cols].
__global__ void __launch_bounds__(256) affine_dequant_rows_kernel(WeightView w, int r0, int nrows, float *dst) {
  const int gpr = w.cols / w.group;
  const size_t per_row = (size_t)w.cols * w.bits / 8;  // bytes
  const size_t total = per_row * nrows;
  for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int rr = (int)(i / per_row), j = (int)(i - (size_t)rr * per_row), row = r0 + rr;
    const uint8_t b = w.codes[(size_t)row * per_row + j];
    float *o = dst + (size_t)rr * w.cols;
    if (w.bits == 8) {
      const int g = j / w.group;
      const float s = __half2float(__ushort_as_half(w.scale[(size_t)row * gpr + g]));
      const float zp = (float)w.zp[(size_t)row * gpr + g];
      o[j] = ((float)b - zp) * s;
    } else {
      // byte j of a 32-code run: code (j % 16) low nibble, code (j % 16) + 16 high
      const int k0 = (j >> 4) * 32 + (j & 15), g = k0 / w.group;
      const float s = __half2float(__ushort_as_half(w.scale[(size_t)row * gpr + g]));
      const float zp = (float)w.zp[(size_t)row * gpr + g];
      o[k0] = ((float)(b & 0xF) - zp) * s;
      o[k0 + 16] = ((float)(b >> 4) - zp) * s;
    }
  }
}

// rows_dot (kernels.mojo:361-397): output rows [o_start, OUT) from float32
// rows wd[o - o_start][IN]: 16-lane chains, the halving tree, + bias, finish.
// One warp per (token, row) pair half: lanes 0-15 and 16-31 take two pairs.
__global__ void rows_dot_kernel(const float *wd, const float *x, const float *bias, float *out, int T, int IN, int OUT,
                                int o_start, int epi) {
  const int pair = (blockIdx.x * blockDim.x + threadIdx.x) >> 4, l = threadIdx.x & 15;
  const int nrows = OUT - o_start;
  const bool live = pair < T * nrows;
  const int t = live ? pair / nrows : 0, o = o_start + (live ? pair % nrows : 0);
  float d = 0.0f;
  if (live)
    for (int i = l; i < IN; i += 16) d = fmaf(x[(size_t)t * IN + i], wd[(size_t)(o - o_start) * IN + i], d);
  d = d + __shfl_xor_sync(0xffffffffu, d, 8);
  d = d + __shfl_xor_sync(0xffffffffu, d, 4);
  d = d + __shfl_xor_sync(0xffffffffu, d, 2);
  d = d + __shfl_xor_sync(0xffffffffu, d, 1);
  if (live && l == 0) {
    float r = d + ((epi & EPI_BIAS) ? bias[o] : 0.0f);
    if (epi & EPI_GELU) r = gelu(r);
    float *dst = out + (size_t)t * OUT + o;
    if (epi & EPI_RESID) r += *dst;
    *dst = r;
  }
}

// Embeddings of T tokens at positions pos0.. from a dense ([V][C], WT) or
// GGUF (dequantized rows) head: x[t] = row(token) + wpe[pos0 + t].
template <int WT>
__global__ void embed_dense_kernel(const void *w, int C, int V, const float *wpe, float *x, const int *tokens,
                                   int pos0) {
  const int t = blockIdx.x, token = min(max(tokens[t], 0), V - 1);
  for (int i = threadIdx.x; i < C; i += blockDim.x)
    x[(size_t)t * C + i] = wload<WT>(w, (size_t)token * C + i) + wpe[(size_t)(pos0 + t) * C + i];
}

template <int T>
__global__ void __launch_bounds__(256) embed_gguf_kernel(RowMat w, const float *wpe, float *x, const int *tokens,
                                                          int pos0) {
  // one CTA per token: 16 groups of 16 lanes, a block (or 16 plain values) each
  const int t = blockIdx.x, token = min(max(tokens[t], 0), w.rows - 1);
  const int L = threadIdx.x & 15, grp = threadIdx.x >> 4, bs = rt_block_size(T), bb = rt_block_bytes(T);
  const uint8_t *p = w.data + (size_t)token * w.row_bytes;
  float *o = x + (size_t)t * w.cols;
  if (bs == 1) {
    for (int i0 = grp * 16; i0 < w.cols; i0 += 256)
      block_values<T>(p + (size_t)i0 * bb, L, [&](float v, int i) { o[i0 + i] = v; });
  } else {
    for (int blk = grp; blk < w.cols / bs; blk += 16)
      block_values<T>(p + (size_t)blk * bb, L, [&](float v, int i) { o[blk * bs + i] = v; });
  }
  __syncthreads();
  for (int i = threadIdx.x; i < w.cols; i += blockDim.x) o[i] = o[i] + wpe[(size_t)(pos0 + t) * w.cols + i];
}

// score_rows (gpt2t.mojo:1042-1097) for rows [r0, r1) of a window: stats
// [6][rows] in float64: NLL, NLL under the base (f32) logits, top-1
// agreement, KL(base || model), max and sum of |logit differences|. log_sum_exp
// (gpt2t.mojo:1030-1039): the row's float32 max, then sum of the float32
// exp(v - max) in float64, mx + log(s). One CTA per row.
__global__ void __launch_bounds__(256) score_rows_kernel(const float *logits, const float *base, const int *targets,
                                                         int V, int r0, double *stats, int stride) {
  __shared__ double sd[32];
  __shared__ float sf[32];
  __shared__ int si[32];
  const int r = r0 + blockIdx.x, tid = threadIdx.x, lane = tid & 31, wp = tid >> 5, nw = blockDim.x >> 5;
  const float *lm = logits + (size_t)r * V;
  const float *lb = base ? base + (size_t)r * V : nullptr;
  // block reductions
  auto fmax_all = [&](float v) {
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) sf[wp] = v;
    __syncthreads();
    float m = sf[0];
    for (int i = 1; i < nw; i++) m = fmaxf(m, sf[i]);
    return m;
  };
  auto dsum_all = [&](double v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if (lane == 0) sd[wp] = v;
    __syncthreads();
    double s = 0.0;
    for (int i = 0; i < nw; i++) s += sd[i];
    return s;
  };
  auto dmax_all = [&](double v) {
    for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) sd[wp] = v;
    __syncthreads();
    double m = sd[0];
    for (int i = 1; i < nw; i++) m = fmax(m, sd[i]);
    return m;
  };
  // argmax: first index of the largest (the reference's strict > scan)
  auto argmax_all = [&](const float *row) {
    float bv = -__int_as_float(0x7f800000);
    int bi = 0x7fffffff;
    for (int v = tid; v < V; v += blockDim.x)
      if (better(row[v], v, bv, bi)) {
        bv = row[v];
        bi = v;
      }
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ov, oi, bv, bi)) {
        bv = ov;
        bi = oi;
      }
    }
    __syncthreads();
    if (lane == 0) {
      sf[wp] = bv;
      si[wp] = bi;
    }
    __syncthreads();
    bv = sf[0];
    bi = si[0];
    for (int i = 1; i < nw; i++)
      if (better(sf[i], si[i], bv, bi)) {
        bv = sf[i];
        bi = si[i];
      }
    return bi == 0x7fffffff ? 0 : bi;
  };
  auto lse_of = [&](const float *row) {
    float mx = -__int_as_float(0x7f800000);
    for (int v = tid; v < V; v += blockDim.x) mx = fmaxf(mx, row[v]);
    mx = fmax_all(mx);
    double s = 0.0;
    for (int v = tid; v < V; v += blockDim.x) s += (double)lm_expf(row[v] - mx);
    s = dsum_all(s);
    return (double)mx + log(s);
  };
  const int target = min(max(targets[r], 0), V - 1);  // next-token ids are in range; clamped for safety
  const double lse = lse_of(lm);
  double nll = lse - (double)lm[target];
  double nll_b = 0.0, agree = 0.0, kl = 0.0, dmax = 0.0, dsum = 0.0;
  if (lb) {
    const double lse_b = lse_of(lb);
    nll_b = lse_b - (double)lb[target];
    double k = 0.0, dm = 0.0, ds = 0.0;
    for (int v = tid; v < V; v += blockDim.x) {
      const double m = (double)lm[v], b = (double)lb[v];
      const double lpb = b - lse_b;
      k += exp(lpb) * (lpb - (m - lse));
      const double d = fabs(m - b);
      dm = fmax(dm, d);
      ds += d;
    }
    kl = dsum_all(k);
    dmax = dmax_all(dm);
    dsum = dsum_all(ds);
    agree = argmax_all(lm) == argmax_all(lb) ? 1.0 : 0.0;
  }
  if (tid == 0) {
    const double vals[6] = {nll, nll_b, agree, kl, dmax, dsum};
    for (int k = 0; k < 6; k++) stats[(size_t)k * stride + (r - r0)] = vals[k];
  }
}

}  // namespace llmq
