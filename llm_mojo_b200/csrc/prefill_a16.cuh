// W4A16 / W8A16 several-token matmul (prefill) on CUDA cores, sm_100a.
//
// matmul_rows_a16 for T > 1 (kernels.mojo:461-507): x quantized to int16 per
// row (quantize_rows, :400-416); outputs in 32-row tiles follow tile_i16
// (:512-573): per (token, output) the int32 sum of x * (u - zp) over each
// segment of min(G, 256) inputs (exact), then accf = fma(f32(acc), scale_g,
// accf) over the segments in order, r = accf * sx (+ b), store_out. The
// OUT % 32 leftover rows follow rows_i16 / dot1_i16 (:576-628): 16 lane sums
// per group, fma per group, halving tree, d * sx + bias.
#pragma once

#include "gemv_a16.cuh"

namespace llmq {

// quantize_rows: one CTA per row. xq [T][IN] int16, sx [T].
__global__ void quantize_rows_kernel(const float *x, int IN, int16_t *xq, float *sx) {
  __shared__ float red[64];
  const float *row = x + (size_t)blockIdx.x * IN;
  float mx = 0.0f;
  for (int i = threadIdx.x; i < IN; i += blockDim.x) mx = fmaxf(mx, fabsf(row[i]));
  mx = block_max(mx, red);
  float s = mx / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  float inv = 1.0f / s;
  for (int i = threadIdx.x; i < IN; i += blockDim.x) xq[(size_t)blockIdx.x * IN + i] = (int16_t)roundf(row[i] * inv);
  if (threadIdx.x == 0) sx[blockIdx.x] = s;
}

// LayerNorm of T rows, one CTA per row (kernels.mojo:179-197).
__global__ void layernorm_kernel(float *out, const float *x, const float *w, const float *b, int C) {
  extern __shared__ __align__(16) float xf[];
  __shared__ float red[64];
  const float *xr = x + (size_t)blockIdx.x * C;
  for (int i = threadIdx.x; i < C; i += blockDim.x) xf[i] = xr[i];
  __syncthreads();
  ln_inplace(xf, C, w, b, red);
  for (int i = threadIdx.x; i < C; i += blockDim.x) out[(size_t)blockIdx.x * C + i] = xf[i];
}

// layernorm_kernel's arithmetic with one warp per row (8 rows per CTA of 256
// threads), for C % 32 == 0 and C <= 1024: lane L holds columns L + 32 j in
// registers; lane sum l adds columns l + 16 i for i = 0, 1, ... in turn,
// i.e. the registers j of lanes l and l + 16 alternately, read through two
// shuffles per step, so the sums, the tree and every result equal
// ln_inplace's. out may alias x.
__global__ void __launch_bounds__(256) layernorm_rows_kernel(float *out, const float *x, const float *w,
                                                             const float *b, int T, int C) {
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31, l = lane & 15;
  if (row >= T) return;
  const int n = C >> 5;
  const float *xr = x + (size_t)row * C;
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; j++) v[j] = j < n ? xr[lane + 32 * j] : 0.0f;
  float a = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j++)
    if (j < n) {
      const float u0 = __shfl_sync(0xffffffffu, v[j], l), u1 = __shfl_sync(0xffffffffu, v[j], l + 16);
      a = a + u0;
      a = a + u1;
    }
  const float mean = tree16_warp(a) / (float)C;
  float sq = 0.0f;
#pragma unroll
  for (int j = 0; j < 32; j++)
    if (j < n) {
      const float d0 = __shfl_sync(0xffffffffu, v[j], l) - mean, d1 = __shfl_sync(0xffffffffu, v[j], l + 16) - mean;
      sq = sq + d0 * d0;
      sq = sq + d1 * d1;
    }
  const float rstd = 1.0f / sqrtf(tree16_warp(sq) / (float)C + 1e-5f);
  float *orow = out + (size_t)row * C;
#pragma unroll
  for (int j = 0; j < 32; j++)
    if (j < n) {
      const int c = lane + 32 * j;
      const float t = (v[j] - mean) * rstd;
      orow[c] = t * w[c] + b[c];
    }
}

// LayerNorm of T rows of C: one warp per row where the row fits in registers
// and there are enough rows to fill the GPU many times over (for a prompt of
// a few hundred tokens the CTA per row is faster: measured 2.69 vs 2.46 ms
// per 476-token config 2 prompt).
inline void launch_layernorm(float *out, const float *x, const float *w, const float *b, int T, int C,
                             cudaStream_t s) {
  if (C % 32 == 0 && C <= 1024 && T >= 4096)
    layernorm_rows_kernel<<<(T + 7) / 8, 256, 0, s>>>(out, x, w, b, T, C);
  else
    layernorm_kernel<<<T, 256, C * 4, s>>>(out, x, w, b, C);
}

// Tile kernel: 32 tokens x 32 outputs per CTA, 256 threads, each thread 2
// tokens x 2 outputs. Only output rows below full = OUT / 32 * 32.
__global__ void __launch_bounds__(256) tile_a16_kernel(WeightView w, const int16_t *xq, const float *sx,
                                                       const float *bias, float *out, int T, int OUT, int epi) {
  __shared__ int16_t xs[32][34];
  __shared__ int16_t ws[32][34];
  const int IN = w.cols, G = w.group, seg = G < 256 ? G : 256, gpr = IN / G;
  const int t0 = blockIdx.y * 32, o0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  int acc[2][2] = {{0, 0}, {0, 0}};
  float accf[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
  for (int k0 = 0; k0 < IN; k0 += 32) {
    // load 32x32 activations and 32x32 weights (code - zp) as int16
    for (int i = threadIdx.x; i < 32 * 32; i += 256) {
      int r = i >> 5, kk = i & 31;
      int t = t0 + r;
      xs[r][kk] = t < T ? xq[(size_t)t * IN + k0 + kk] : (int16_t)0;
      int o = o0 + r;
      int g = (k0 + kk) / G;
      ws[r][kk] = (int16_t)(code_at(w, o, k0 + kk) - (int)w.zp[(size_t)o * gpr + g]);
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; kk++) {
#pragma unroll
      for (int i = 0; i < 2; i++)
#pragma unroll
        for (int j = 0; j < 2; j++) acc[i][j] += (int)xs[ty + 16 * i][kk] * (int)ws[tx + 16 * j][kk];
    }
    __syncthreads();
    if ((k0 + 32) % seg == 0) {
      int g = k0 / G;
#pragma unroll
      for (int j = 0; j < 2; j++) {
        float s = half_bits_to_float(w.scale[(size_t)(o0 + tx + 16 * j) * gpr + g]);
#pragma unroll
        for (int i = 0; i < 2; i++) {
          accf[i][j] = fmaf((float)acc[i][j], s, accf[i][j]);
          acc[i][j] = 0;
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 2; i++) {
    int t = t0 + ty + 16 * i;
    if (t >= T) continue;
#pragma unroll
    for (int j = 0; j < 2; j++) {
      int o = o0 + tx + 16 * j;
      float r = accf[i][j] * sx[t];
      if (epi & EPI_BIAS) r += bias[o];
      if (epi & EPI_GELU) r = gelu(r);
      float *dst = out + (size_t)t * OUT + o;
      if (epi & EPI_RESID) r += *dst;
      *dst = r;
    }
  }
}

// Leftover rows o in [o_start, OUT): one thread per (token, output).
__global__ void rows_a16_kernel(WeightView w, const int16_t *xq, const float *sx, const float *bias, float *out,
                                int T, int OUT, int o_start, int epi) {
  int idx = blockIdx.x * blockDim.x + threadIdx.x;
  int nrows = OUT - o_start;
  if (idx >= T * nrows) return;
  int t = idx / nrows, o = o_start + idx % nrows;
  const int IN = w.cols, G = w.group, gpr = IN / G;
  const int16_t *xt = xq + (size_t)t * IN;
  float accf[16];
#pragma unroll
  for (int l = 0; l < 16; l++) accf[l] = 0.0f;
  for (int g = 0; g < gpr; g++) {
    int zp = w.zp[(size_t)o * gpr + g];
    float s = half_bits_to_float(w.scale[(size_t)o * gpr + g]);
    int acc[16];
#pragma unroll
    for (int l = 0; l < 16; l++) acc[l] = 0;
    for (int k = g * G; k < (g + 1) * G; k += 32) {
#pragma unroll
      for (int l = 0; l < 16; l++) {
        int w0 = code_at(w, o, k + 2 * l) - zp, w1 = code_at(w, o, k + 2 * l + 1) - zp;
        acc[l] += (int)xt[k + 2 * l] * w0 + (int)xt[k + 2 * l + 1] * w1;
      }
    }
#pragma unroll
    for (int l = 0; l < 16; l++) accf[l] = fmaf((float)acc[l], s, accf[l]);
  }
#pragma unroll
  for (int l = 0; l < 8; l++) accf[l] = accf[l] + accf[l + 8];
#pragma unroll
  for (int l = 0; l < 4; l++) accf[l] = accf[l] + accf[l + 4];
  accf[0] = accf[0] + accf[2];
  accf[1] = accf[1] + accf[3];
  float d = accf[0] + accf[1];
  float b = (epi & EPI_BIAS) ? bias[o] : 0.0f;
  float r = d * sx[t] + b;
  if (epi & EPI_GELU) r = gelu(r);
  float *dst = out + (size_t)t * OUT + o;
  if (epi & EPI_RESID) r += *dst;
  *dst = r;
}

// Embeddings of T tokens at positions pos0.. (gpt2t.mojo:495-502).
__global__ void embed_rows_kernel(WeightView head, const float *wpe, float *x, const int *tokens, int pos0) {
  int t = blockIdx.x, C = head.cols, gpr = head.cols / head.group;
  int token = tokens[t];
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    size_t gi = (size_t)token * gpr + i / head.group;
    float s = half_bits_to_float(head.scale[gi]);
    float v = (float)(code_at(head, token, i) - (int)head.zp[gi]) * s;
    x[(size_t)t * C + i] = v + wpe[(size_t)(pos0 + t) * C + i];
  }
}

}  // namespace llmq
