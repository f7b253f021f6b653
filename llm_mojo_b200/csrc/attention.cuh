// KV caches and attention (kvcache.mojo, int_attention.mojo) on sm_100a.
//
// QuantKV[8] (kvcache.mojo:248-385): int8 codes [layer][pos][head][64] with a
// float32 scale per (layer, pos, head) for keys and for values; attention in
// float32 through score/add_value (attend_float_one, kvcache.mojo:113-150).
// One CTA per (token, head): scores in parallel over positions, then the
// softmax total and the value sums in the reference's sequential order over
// positions (one chain per output dimension), so outputs are bit-identical.
#pragma once

#include "common.cuh"

namespace llmq {

struct KV8View {
  int8_t *k, *v;
  float *ks, *vs;
  int n_layer, max_t, n_head, head_dim;
};

// QuantKV.quantize (kvcache.mojo:319-331) of one head's 64 values by one
// warp... any block of >= head_dim threads: threads [0, head_dim) hold x.
__device__ __forceinline__ float quant_i8_head(float x, bool active, float *red, int8_t *dst, int d) {
  float a = active ? fabsf(x) : 0.0f;
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
  __syncthreads();
  float mx = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) mx = fmaxf(mx, red[w]);
  __syncthreads();
  float s = mx / 127.0f;
  if (s == 0.0f) s = 1.0f;
  float inv = 1.0f / s;
  if (active) dst[d] = (int8_t)roundf(x * inv);
  return s;
}

// Stores the keys and values of T tokens at positions pos0.. of `layer`
// (QuantKV.store, kvcache.mojo:333-342). grid (n_head, T, 2), block >= 64.
__global__ void kv8_store_kernel(KV8View c, const float *qkv, int layer, int pos0, const int *pos_dev) {
  __shared__ float red[32];
  int h = blockIdx.x, t = blockIdx.y, which = blockIdx.z;  // 0 = key, 1 = value
  int pos = (pos_dev ? *pos_dev : pos0) + t;
  int HS = c.head_dim, C = c.n_head * HS;
  int d = threadIdx.x;
  bool act = d < HS;
  float x = act ? qkv[(size_t)t * 3 * C + (1 + which) * C + h * HS + d] : 0.0f;
  size_t sl = ((size_t)layer * c.max_t + pos) * c.n_head + h;
  int8_t *dst = (which == 0 ? c.k : c.v) + sl * HS;
  float s = quant_i8_head(x, act, red, dst, d);
  if (threadIdx.x == 0) (which == 0 ? c.ks : c.vs)[sl] = s;
}

// attend_float_one for token t (position pos0 + t), head h. grid (n_head, T).
// With store != 0 (decode, T == 1) the CTA first stores this token's key and
// value for its head, which is all its own attention reads of this step.
// Shared memory: 3 * max_t floats.
__global__ void __launch_bounds__(128) kv8_attend_kernel(KV8View c, float *out, const float *qkv, int layer,
                                                         int pos0, const int *pos_dev, int store) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[40];
  const int h = blockIdx.x, t = blockIdx.y;
  const int HS = c.head_dim, C = c.n_head * HS;
  const int P0 = pos_dev ? *pos_dev : pos0;
  const int npos = P0 + t + 1;
  const float *q = qkv + (size_t)t * 3 * C + h * HS;
  float *sc = sm;               // [npos] scores, then exponentials
  float *ps = sm + c.max_t;     // [npos] p * vs
  float *qs = sm + 2 * c.max_t; // [HS] query

  if (store) {
    int d = threadIdx.x;
    size_t sl = ((size_t)layer * c.max_t + (P0 + t)) * c.n_head + h;
    for (int which = 0; which < 2; which++) {
      bool act = d < HS;
      float x = act ? qkv[(size_t)t * 3 * C + (1 + which) * C + h * HS + d] : 0.0f;
      float s = quant_i8_head(x, act, red, (which == 0 ? c.k : c.v) + sl * HS, d);
      if (threadIdx.x == 0) (which == 0 ? c.ks : c.vs)[sl] = s;
    }
    __syncthreads();
  }
  for (int i = threadIdx.x; i < HS; i += blockDim.x) qs[i] = q[i];
  __syncthreads();

  // scores: 16 lanes of q*k, 4 chunks each, halving tree, * ks, * scale.
  const float scale = 1.0f / sqrtf((float)HS);
  float mx = -__int_as_float(0x7f800000);
  for (int s = threadIdx.x; s < npos; s += blockDim.x) {
    size_t sl = ((size_t)layer * c.max_t + s) * c.n_head + h;
    const int8_t *kp = c.k + sl * HS;
    float d[16];
#pragma unroll
    for (int l = 0; l < 16; l++) d[l] = 0.0f;
    for (int i = 0; i < HS; i += 16) {
      int4 kv = *(const int4 *)(kp + i);
      const int8_t *kb = (const int8_t *)&kv;
#pragma unroll
      for (int l = 0; l < 16; l++) d[l] = d[l] + qs[i + l] * (float)kb[l];
    }
#pragma unroll
    for (int l = 0; l < 8; l++) d[l] = d[l] + d[l + 8];
#pragma unroll
    for (int l = 0; l < 4; l++) d[l] = d[l] + d[l + 4];
    d[0] = d[0] + d[2];
    d[1] = d[1] + d[3];
    float v = ((d[0] + d[1]) * c.ks[sl]) * scale;
    sc[s] = v;
    mx = fmaxf(mx, v);
  }
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); w++) mx = fmaxf(mx, red[w]);
  for (int s = threadIdx.x; s < npos; s += blockDim.x) sc[s] = lm_expf(sc[s] - mx);
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.0f;
    for (int s = 0; s < npos; s++) total += sc[s];
    red[36] = total;
  }
  __syncthreads();
  const float total = red[36];
  for (int s = threadIdx.x; s < npos; s += blockDim.x) {
    size_t sl = ((size_t)layer * c.max_t + s) * c.n_head + h;
    float p = sc[s] / total;
    ps[s] = p * c.vs[sl];
  }
  __syncthreads();
  // acc[d] = fma(p * vs, v[s][d], acc[d]) over positions in order.
  for (int d = threadIdx.x; d < HS; d += blockDim.x) {
    float acc = 0.0f;
    const int8_t *vp = c.v + ((size_t)layer * c.max_t * c.n_head + h) * HS + d;
    const size_t stride = (size_t)c.n_head * HS;
    int s = 0;
    for (; s + 4 <= npos; s += 4) {
      float v0 = (float)vp[(size_t)s * stride], v1 = (float)vp[(size_t)(s + 1) * stride];
      float v2 = (float)vp[(size_t)(s + 2) * stride], v3 = (float)vp[(size_t)(s + 3) * stride];
      acc = fmaf(ps[s], v0, acc);
      acc = fmaf(ps[s + 1], v1, acc);
      acc = fmaf(ps[s + 2], v2, acc);
      acc = fmaf(ps[s + 3], v3, acc);
    }
    for (; s < npos; s++) acc = fmaf(ps[s], (float)vp[(size_t)s * stride], acc);
    out[(size_t)t * C + h * HS + d] = acc;
  }
}

}  // namespace llmq
