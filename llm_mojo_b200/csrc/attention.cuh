// KV caches and attention (kvcache.mojo, int_attention.mojo) on sm_100a.
//
// IntAttnKV (int_attention.mojo:62-280): int8 K in [layer*head][pos/16]
// [d/2][16][2] and V in [layer*head][pos/2][d][2] with int32 Q24 scales;
// scores, softmax and value sums in integer fixed point (see ia_attend_kernel).
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
  size_t seq;  // codes per sequence when the view holds several caches (blockIdx.z), else 0

  // The view of sequence b's cache.
  __device__ KV8View of(int b) const {
    KV8View c = *this;
    c.k += b * seq;
    c.v += b * seq;
    c.ks += b * (seq / head_dim);
    c.vs += b * (seq / head_dim);
    return c;
  }
};

// The exact float of an int8 code without the conversion unit (the bits of
// 1.5 * 2^23 + v, minus 1.5 * 2^23; exact for |v| < 2^22).
__device__ __forceinline__ float i8_to_float(int v) { return __int_as_float(0x4B400000 + v) - 12582912.0f; }

__device__ __forceinline__ void kv_cp_async16(void *dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void kv_cp_async4(void *dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"((unsigned)__cvta_generic_to_shared(dst)), "l"(src)
               : "memory");
}

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
// (QuantKV.store, kvcache.mojo:333-342) for nseq sequences, sequence b's T
// rows of qkv after sequence b - 1's. One warp per (sequence, token, head,
// key or value): lane L holds elements L + 32 j (head_dim <= 128); the
// maximum of |x| (exact in any order), s = max / 127 (1 when 0) and the codes
// round(x / s) are quant_i8_head's. grid ceil(warps / 8), 256 threads.
__global__ void __launch_bounds__(256) kv8_store_kernel(KV8View c0, const float *qkv, int layer, int pos0,
                                                        const int *pos_dev, int T, int nseq) {
  const int gw = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int nh = c0.n_head;
  if (gw >= nseq * T * nh * 2) return;
  const int which = gw & 1, h = (gw >> 1) % nh, rest = (gw >> 1) / nh, t = rest % T, sb = rest / T;
  const KV8View c = c0.of(sb);
  const int HS = c.head_dim, C = nh * HS;
  const float *src = qkv + ((size_t)sb * T + t) * 3 * C + (1 + which) * C + h * HS;
  const size_t sl = ((size_t)layer * c.max_t + (pos_dev ? *pos_dev : pos0) + t) * nh + h;
  int8_t *dst = (which == 0 ? c.k : c.v) + sl * HS;
  float xv[4];
  float a = 0.0f;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int d = lane + 32 * j;
    xv[j] = d < HS ? src[d] : 0.0f;
    a = fmaxf(a, fabsf(xv[j]));
  }
  for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  float sv = a / 127.0f;
  if (sv == 0.0f) sv = 1.0f;
  const float inv = 1.0f / sv;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int d = lane + 32 * j;
    if (d < HS) dst[d] = (int8_t)roundf(xv[j] * inv);
  }
  if (lane == 0) (which == 0 ? c.ks : c.vs)[sl] = sv;
}

// DenseKV.store (kvcache.mojo:204-208): the keys and values of T tokens at
// positions pos0.. of `layer`, as float32 (KVT 1) or bfloat16 (KVT 2, round
// to nearest even). grid (T), block 256.
template <int KVT>
__global__ void dkv_store_kernel(KV8View c, const float *qkv, int layer, int pos0) {
  const int t = blockIdx.x, C = c.n_head * c.head_dim;
  const size_t o = ((size_t)layer * c.max_t + pos0 + t) * C;
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    const float k = qkv[(size_t)t * 3 * C + C + i], v = qkv[(size_t)t * 3 * C + 2 * C + i];
    if (KVT == 1) {
      ((float *)c.k)[o + i] = k;
      ((float *)c.v)[o + i] = v;
    } else {
      ((uint16_t *)c.k)[o + i] = __bfloat16_as_ushort(__float2bfloat16_rn(k));
      ((uint16_t *)c.v)[o + i] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
  }
}

// attend_float_one for token t (position pos0 + t), head h. grid (n_head, T).
// With store != 0 (decode, T == 1) the CTA first stores this token's key and
// value for its head, which is all its own attention reads of this step.
// Every read the CTA makes of the cache is issued at its start: the value
// codes, both scale columns, the query and (KST) the key codes are copied
// into shared memory (cp.async) while the token's key and value are
// quantized, and this token's codes and scales are written to the shared
// copies as well as to the cache, so the CTA waits for memory once. The
// arithmetic and its order are attend_float_one's: 16 score lanes of q * k
// over 4 chunks, halving tree, * ks, * scale; exp of (score - max); the total
// summed in position order; acc[d] = fma(p * vs, v[s][d], acc) in position
// order. Key rows in shared memory hold their 16-byte chunks in the order ch
// ^ ((s >> 1) & 3), so that the 8 rows of each quarter warp's 16-byte loads
// fall in distinct banks. HSC: the head size when fixed at compile time (64),
// else 0. Shared memory: kv8_attend_smem(cap, head_dim, KST), cap >= the
// positions any query of the launch sees (at most max_t).
template <bool KST, int HSC>
__global__ void __launch_bounds__(128) kv8_attend_kernel(KV8View c0, float *out, const float *qkv, int layer,
                                                         int pos0, const int *pos_dev, int store, int cap) {
  extern __shared__ __align__(16) float sm[];
  __shared__ float red[40];
  const int h = blockIdx.x, t = blockIdx.y;
  const KV8View c = c0.of(blockIdx.z);  // grid z: sequences, each with gridDim.y rows
  const int HS = HSC ? HSC : c.head_dim, C = c.n_head * HS, cpr = HS / 16;
  cap = (cap + 3) & ~3;
  qkv += (size_t)blockIdx.z * gridDim.y * 3 * C;
  out += (size_t)blockIdx.z * gridDim.y * C;
  const int P0 = pos_dev ? *pos_dev : pos0;
  const int npos = P0 + t + 1;
  const float *q = qkv + (size_t)t * 3 * C + h * HS;
  float *qs = sm;              // [HS] query
  float *sc = sm + HS;         // [cap] scores, then exponentials
  float *ps = sc + cap;        // [cap] p * vs
  float *kss = ps + cap;       // [cap] key scales
  float *vss = kss + cap;      // [cap] value scales
  int8_t *vst = (int8_t *)(((uintptr_t)(vss + cap) + 15) & ~(uintptr_t)15);  // [cap][HS] value codes
  int8_t *kst = vst + (size_t)cap * HS;                                   // [cap][HS] key codes (KST)
  const size_t slot0 = (size_t)layer * c.max_t * c.n_head + h;  // cache slot of position s: slot0 + s * n_head
  const int8_t *vb = c.v + slot0 * HS, *kb = c.k + slot0 * HS;
  const size_t rs = (size_t)c.n_head * HS;
  const int npre = store ? npos - 1 : npos;
  for (int i = threadIdx.x; i < npre * cpr; i += blockDim.x) {
    const int s = i / cpr, ch = i - s * cpr;
    kv_cp_async16(vst + (size_t)s * HS + ch * 16, vb + (size_t)s * rs + ch * 16);
    if (KST) kv_cp_async16(kst + (size_t)s * HS + ((ch ^ ((s >> 1) & 3)) * 16), kb + (size_t)s * rs + ch * 16);
  }
  for (int s = threadIdx.x; s < npre; s += blockDim.x) {
    kv_cp_async4(kss + s, c.ks + slot0 + (size_t)s * c.n_head);
    kv_cp_async4(vss + s, c.vs + slot0 + (size_t)s * c.n_head);
  }
  if (((uintptr_t)q & 15) == 0)
    for (int i = threadIdx.x; i < HS / 4; i += blockDim.x) kv_cp_async16(qs + 4 * i, q + 4 * i);
  else
    for (int i = threadIdx.x; i < HS; i += blockDim.x) qs[i] = q[i];
  asm volatile("cp.async.commit_group;" ::: "memory");

  if (store) {
    // QuantKV.quantize of this token's key and value (quant_i8_head's
    // arithmetic), into the cache and the shared copies
    const int d = threadIdx.x, s = npos - 1;
    const size_t sl = slot0 + (size_t)(P0 + t) * c.n_head;
    for (int which = 0; which < 2; which++) {
      const bool act = d < HS;
      const float x = act ? qkv[(size_t)t * 3 * C + (1 + which) * C + h * HS + d] : 0.0f;
      float a = act ? fabsf(x) : 0.0f;
      for (int o = 16; o > 0; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
      if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = a;
      __syncthreads();
      float mx = 0.0f;
      for (int w = 0; w < (int)(blockDim.x >> 5); w++) mx = fmaxf(mx, red[w]);
      __syncthreads();
      float sv = mx / 127.0f;
      if (sv == 0.0f) sv = 1.0f;
      const float inv = 1.0f / sv;
      if (act) {
        const int8_t code = (int8_t)roundf(x * inv);
        (which == 0 ? c.k : c.v)[sl * HS + d] = code;
        if (which == 1)
          vst[(size_t)s * HS + d] = code;
        else if (KST)
          kst[(size_t)s * HS + (((d >> 4) ^ ((s >> 1) & 3)) << 4) + (d & 15)] = code;
      }
      if (threadIdx.x == 0) {
        (which == 0 ? c.ks : c.vs)[sl] = sv;
        (which == 0 ? kss : vss)[s] = sv;
      }
    }
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();

  const float scale = 1.0f / sqrtf((float)HS);
  float mx = -__int_as_float(0x7f800000);
  for (int s = threadIdx.x; s < npos; s += blockDim.x) {
    const int8_t *kp = KST ? kst + (size_t)s * HS : c.k + (slot0 + (size_t)s * c.n_head) * HS;
    const int sw = KST ? ((s >> 1) & 3) : 0;
    float d[16];
#pragma unroll
    for (int l = 0; l < 16; l++) d[l] = 0.0f;
#pragma unroll
    for (int i = 0; i < HS; i += 16) {
      // code b as a float: the byte b + 128 in the low mantissa bits of
      // 1.5 * 2^23 (one byte permute), minus 1.5 * 2^23 + 128; exact
      const int4 kv = *(const int4 *)(kp + (((i >> 4) ^ sw) << 4));
      const unsigned w[4] = {(unsigned)kv.x ^ 0x80808080u, (unsigned)kv.y ^ 0x80808080u,
                             (unsigned)kv.z ^ 0x80808080u, (unsigned)kv.w ^ 0x80808080u};
#pragma unroll
      for (int l = 0; l < 16; l++) {
        const float kf = __int_as_float((int)__byte_perm(w[l >> 2], 0x4B400000u, 0x7640u | (l & 3))) - 12583040.0f;
        d[l] = d[l] + qs[i + l] * kf;
      }
    }
#pragma unroll
    for (int l = 0; l < 8; l++) d[l] = d[l] + d[l + 8];
#pragma unroll
    for (int l = 0; l < 4; l++) d[l] = d[l] + d[l + 4];
    d[0] = d[0] + d[2];
    d[1] = d[1] + d[3];
    const float v = ((d[0] + d[1]) * kss[s]) * scale;
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
  for (int s = threadIdx.x; s < npos; s += blockDim.x) ps[s] = (sc[s] / total) * vss[s];
  __syncthreads();
  // acc[d] = fma(p * vs, v[s][d], acc[d]) over positions in order.
  for (int d = threadIdx.x; d < HS; d += blockDim.x) {
    float acc = 0.0f;
    const int8_t *vp = vst + d;
    int s = 0;
    for (; s + 4 <= npos; s += 4, vp += 4 * HS) {
      const float4 p4 = *(const float4 *)(ps + s);
      const float v0 = i8_to_float(vp[0]), v1 = i8_to_float(vp[HS]);
      const float v2 = i8_to_float(vp[2 * HS]), v3 = i8_to_float(vp[3 * HS]);
      acc = fmaf(p4.x, v0, acc);
      acc = fmaf(p4.y, v1, acc);
      acc = fmaf(p4.z, v2, acc);
      acc = fmaf(p4.w, v3, acc);
    }
    for (; s < npos; s++, vp += HS) acc = fmaf(ps[s], i8_to_float(vp[0]), acc);
    out[(size_t)t * C + h * HS + d] = acc;
  }
}

// Dynamic shared memory of kv8_attend_kernel<kst, *> for queries that see at
// most cap positions.
__host__ __device__ inline size_t kv8_attend_smem(int cap, int HS, bool kst) {
  cap = (cap + 3) & ~3;
  return (size_t)(4 * cap + HS) * 4 + 16 + (size_t)cap * HS * (kst ? 2 : 1);
}

// attend_float_one for QB consecutive query tokens of one head at once (the
// several-token path, prefill). Keys, then values, are staged in tiles of 128
// positions converted once to float (each converted value then serves all
// QB queries); the scores of every query stay in shared memory for the
// softmax. Per query the arithmetic is attend_float_one's, in the same
// order: score lanes + halving tree, * ks, * scale; exp of (score - max); the
// total summed in position order; acc[d] = fma(p * vs, v[d], acc) in
// position order. grid (n_head, ceil(T / QB)), 256 threads; shared memory
// kv8_prefill_smem(P, head_dim), P the positions the block's last query sees.
// Tile rows are HS + 4 floats (16-byte loads along a row, and the 8 rows of
// a quarter warp's loads in distinct banks); score rows are padded to a
// multiple of 4 positions (16-byte loads of 4 consecutive positions).
constexpr int KV_QB = 16;
constexpr int KV_TILE = 128;

__host__ __device__ inline size_t kv8_prefill_smem(int P, int HS) {
  // tile [128][HS + 4] floats, its scales [128], q [QB][HS], scores [QB][P padded], totals [QB]
  const int Pp = (P + 3) & ~3;
  return (size_t)KV_TILE * (HS + 4) * 4 + KV_TILE * 4 + (size_t)KV_QB * HS * 4 + (size_t)KV_QB * Pp * 4 + KV_QB * 4;
}

// KVT: 0 QuantKV[8] (int8 codes and per-head scales), 1 DenseKV[float32],
// 2 DenseKV[bfloat16] (kvcache.mojo:153-246: the values widened to float32,
// no scales: score = tree * scale, p = e / total).
template <int KVT>
__global__ void __launch_bounds__(256) kv_prefill_kernel(KV8View c0, float *out, const float *qkv, int layer, int pos0,
                                                         int T) {
  extern __shared__ __align__(16) float kvp_sm[];
  // the query blocks that see the most positions first (grid y reversed),
  // so the longest CTAs start in the first wave
  const int h = blockIdx.x, t0 = (gridDim.y - 1 - blockIdx.y) * KV_QB;
  const int nq = min(KV_QB, T - t0);
  const KV8View c = c0.of(blockIdx.z);  // grid z: sequences, each with T rows
  const int HS = c.head_dim, C = c.n_head * HS, HP = HS + 4;
  qkv += (size_t)blockIdx.z * T * 3 * C;
  out += (size_t)blockIdx.z * T * C;
  const int P = pos0 + t0 + nq;  // positions the last query of the block sees
  const int Pp = (P + 3) & ~3;   // score row stride
  float *tile = kvp_sm;                        // [128][HS + 4]
  float *tsc = tile + KV_TILE * HP;            // [128]
  float *qs = tsc + KV_TILE;                   // [QB][HS]
  float *sc = qs + KV_QB * HS;                 // [QB][Pp]
  float *tot = sc + (size_t)KV_QB * Pp;        // [QB]
  const int tid = threadIdx.x;
  const size_t head_stride = (size_t)c.n_head * HS;
  const int8_t *kbase = c.k + ((size_t)layer * c.max_t * c.n_head + h) * HS;
  const int8_t *vbase = c.v + ((size_t)layer * c.max_t * c.n_head + h) * HS;
  const size_t sbase = (size_t)layer * c.max_t * c.n_head + h;

  for (int i = tid; i < KV_QB * HS; i += blockDim.x) {
    const int qi = i / HS, d = i % HS;
    qs[i] = qi < nq ? qkv[(size_t)(t0 + qi) * 3 * C + h * HS + d] : 0.0f;
  }
  // a tile of 128 positions of keys (which 0) or values (1) as floats, and
  // their scales
  auto stage = [&](int s0, int which) {
    const int n = min(KV_TILE, P - s0);
    if (KVT == 0) {
      const int8_t *src = which == 0 ? kbase : vbase;
      const float *scl = which == 0 ? c.ks : c.vs;
      const int cpr = HS / 16;
      for (int i = tid; i < n * cpr; i += blockDim.x) {
        const int r = i / cpr, ch = i % cpr;
        int4 raw = *(const int4 *)(src + (size_t)(s0 + r) * head_stride + ch * 16);
        const int8_t *b = (const int8_t *)&raw;
        float4 *dst = (float4 *)(tile + r * HP + ch * 16);
#pragma unroll
        for (int l = 0; l < 4; l++)
          dst[l] = make_float4((float)b[4 * l], (float)b[4 * l + 1], (float)b[4 * l + 2], (float)b[4 * l + 3]);
      }
      for (int r = tid; r < n; r += blockDim.x) tsc[r] = scl[(sbase + (size_t)(s0 + r) * c.n_head)];
    } else {
      // dense caches: element offsets like the int8 codes', 4 or 2 bytes each
      const size_t base = ((size_t)layer * c.max_t * c.n_head + h) * HS;
      const void *src = which == 0 ? (const void *)c.k : (const void *)c.v;
      for (int i = tid; i < n * HS; i += blockDim.x) {
        const int r = i / HS, d = i % HS;
        const size_t e = base + (size_t)(s0 + r) * head_stride + d;
        tile[r * HP + d] = KVT == 1 ? ((const float *)src)[e]
                                    : __uint_as_float((unsigned)((const uint16_t *)src)[e] << 16);
      }
      for (int r = tid; r < n; r += blockDim.x) tsc[r] = 1.0f;
    }
  };

  // 1. scores, a tile of keys at a time; a thread takes one position for 4
  // queries, so each key value it loads serves 4 dot products
  const float scale = 1.0f / sqrtf((float)HS);
  const int ngroups = (nq + 3) / 4;
  for (int s0 = 0; s0 < P; s0 += KV_TILE) {
    __syncthreads();
    stage(s0, 0);
    __syncthreads();
    const int n = min(KV_TILE, P - s0);
    for (int i = tid; i < n * ngroups; i += blockDim.x) {
      const int r = i % n, g = i / n, s = s0 + r, q0 = g * 4;
      const float *kr = tile + r * HP;
      float d[4][16];
#pragma unroll
      for (int j = 0; j < 4; j++)
#pragma unroll
        for (int l = 0; l < 16; l++) d[j][l] = 0.0f;
      for (int i0 = 0; i0 < HS; i0 += 16) {
        float kf[16];
#pragma unroll
        for (int l = 0; l < 4; l++) {
          const float4 k4 = *(const float4 *)(kr + i0 + 4 * l);
          kf[4 * l] = k4.x;
          kf[4 * l + 1] = k4.y;
          kf[4 * l + 2] = k4.z;
          kf[4 * l + 3] = k4.w;
        }
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float4 *q4 = (const float4 *)(qs + (q0 + j) * HS + i0);
#pragma unroll
          for (int l = 0; l < 4; l++) {
            const float4 q = q4[l];
            d[j][4 * l] = d[j][4 * l] + q.x * kf[4 * l];
            d[j][4 * l + 1] = d[j][4 * l + 1] + q.y * kf[4 * l + 1];
            d[j][4 * l + 2] = d[j][4 * l + 2] + q.z * kf[4 * l + 2];
            d[j][4 * l + 3] = d[j][4 * l + 3] + q.w * kf[4 * l + 3];
          }
        }
      }
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int qi = q0 + j;
        if (qi >= nq || s >= pos0 + t0 + qi + 1) continue;
        float *e = d[j];
#pragma unroll
        for (int l = 0; l < 8; l++) e[l] = e[l] + e[l + 8];
#pragma unroll
        for (int l = 0; l < 4; l++) e[l] = e[l] + e[l + 4];
        e[0] = e[0] + e[2];
        e[1] = e[1] + e[3];
        sc[(size_t)qi * Pp + s] = KVT == 0 ? ((e[0] + e[1]) * tsc[r]) * scale : (e[0] + e[1]) * scale;
      }
    }
  }
  __syncthreads();

  // 2. per query: max and exponentials (a warp per query), the totals in
  // position order (a thread per query), then p * vs
  const int warp = tid >> 5, lane = tid & 31, nwarps = blockDim.x >> 5;
  for (int qi = warp; qi < nq; qi += nwarps) {
    const int np = pos0 + t0 + qi + 1;
    float *row = sc + (size_t)qi * Pp;
    float mx = -__int_as_float(0x7f800000);
    for (int s = lane; s < np; s += 32) mx = fmaxf(mx, row[s]);
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    for (int s = lane; s < np; s += 32) row[s] = lm_expf(row[s] - mx);
  }
  __syncthreads();
  if (tid < nq) {
    const int np = pos0 + t0 + tid + 1;
    const float *row = sc + (size_t)tid * Pp;
    float total = 0.0f;
    int s = 0;
    for (; s + 8 <= np; s += 8) {
      float e[8];
#pragma unroll
      for (int j = 0; j < 8; j++) e[j] = row[s + j];
#pragma unroll
      for (int j = 0; j < 8; j++) total += e[j];
    }
    for (; s < np; s++) total += row[s];
    tot[tid] = total;
  }
  __syncthreads();

  // 3. values, a tile at a time: one chain per (query, dimension) in position
  // order; a thread runs the chains of 4 consecutive queries for one dimension
  const int nchains = ngroups * HS;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};  // chains of thread tid (nchains <= blockDim)
  const int g = tid / HS, dd = tid % HS, q0 = g * 4;
  for (int s0 = 0; s0 < P; s0 += KV_TILE) {
    __syncthreads();
    stage(s0, 1);
    __syncthreads();
    // p * vs for this tile's positions
    const int n = min(KV_TILE, P - s0);
    for (int qi = warp; qi < nq; qi += nwarps) {
      float *row = sc + (size_t)qi * Pp;
      const int end = min(n, pos0 + t0 + qi + 1 - s0);
      for (int r = lane; r < end; r += 32)
        row[s0 + r] = KVT == 0 ? (row[s0 + r] / tot[qi]) * tsc[r] : row[s0 + r] / tot[qi];
    }
    __syncthreads();
    if (tid < nchains) {
      // the 4 queries' chains advance together (each in position order), so
      // that each value read serves all 4 and the chains' latencies overlap
      int npj[4];
      int send = s0;
#pragma unroll
      for (int j = 0; j < 4; j++) {
        const int qi = q0 + j;
        npj[j] = qi < nq ? min(pos0 + t0 + qi + 1, s0 + n) : s0;  // this query's positions within the tile
        send = max(send, npj[j]);
      }
      // positions every one of the 4 queries sees (4 at a time, no
      // compares), then the ragged end
      const int lo = min(min(npj[0], npj[1]), min(npj[2], npj[3]));
      const float *vp = tile + dd;
      const float *sr0 = sc + (size_t)q0 * Pp, *sr1 = sr0 + Pp, *sr2 = sr1 + Pp, *sr3 = sr2 + Pp;
      int s = s0;
      for (; s + 4 <= lo; s += 4, vp += 4 * HP) {
        const float v0 = vp[0], v1 = vp[HP], v2 = vp[2 * HP], v3 = vp[3 * HP];
        const float4 p0 = *(const float4 *)(sr0 + s), p1 = *(const float4 *)(sr1 + s);
        const float4 p2 = *(const float4 *)(sr2 + s), p3 = *(const float4 *)(sr3 + s);
        acc[0] = fmaf(p0.x, v0, acc[0]);
        acc[1] = fmaf(p1.x, v0, acc[1]);
        acc[2] = fmaf(p2.x, v0, acc[2]);
        acc[3] = fmaf(p3.x, v0, acc[3]);
        acc[0] = fmaf(p0.y, v1, acc[0]);
        acc[1] = fmaf(p1.y, v1, acc[1]);
        acc[2] = fmaf(p2.y, v1, acc[2]);
        acc[3] = fmaf(p3.y, v1, acc[3]);
        acc[0] = fmaf(p0.z, v2, acc[0]);
        acc[1] = fmaf(p1.z, v2, acc[1]);
        acc[2] = fmaf(p2.z, v2, acc[2]);
        acc[3] = fmaf(p3.z, v2, acc[3]);
        acc[0] = fmaf(p0.w, v3, acc[0]);
        acc[1] = fmaf(p1.w, v3, acc[1]);
        acc[2] = fmaf(p2.w, v3, acc[2]);
        acc[3] = fmaf(p3.w, v3, acc[3]);
      }
      for (; s < send; s++, vp += HP) {
        const float v = vp[0];
        if (s < npj[0]) acc[0] = fmaf(sr0[s], v, acc[0]);
        if (s < npj[1]) acc[1] = fmaf(sr1[s], v, acc[1]);
        if (s < npj[2]) acc[2] = fmaf(sr2[s], v, acc[2]);
        if (s < npj[3]) acc[3] = fmaf(sr3[s], v, acc[3]);
      }
    }
  }
  if (tid < nchains)
    for (int j = 0; j < 4 && q0 + j < nq; j++) out[(size_t)(t0 + q0 + j) * C + h * HS + dd] = acc[j];
}

// ---------------------------------------------------------------------------
// IntAttnKV (int_attention.mojo:62-280, intmath.mojo:48-123)
// ---------------------------------------------------------------------------

constexpr int IA_KS = 24;  // K/V scale fraction bits
constexpr int IA_SF = 16;  // score fraction bits
constexpr int IA_PB = 16;  // positions per K block

struct IAView {
  int8_t *k, *v;
  int32_t *kq, *vq;  // [layer][head][max_t] scales in Q24
  int n_layer, max_t, n_head, head_dim;
};

__device__ __forceinline__ size_t ia_lh(const IAView &c, int layer, int head) {
  return (size_t)layer * c.n_head + head;
}

// Byte offset of key (pos, d): blocks of 16 positions, d in pairs, the 16
// positions of a block interleaved per pair (the VNNI layout of the reference).
__device__ __forceinline__ size_t ia_k_at(const IAView &c, int layer, int head, int pos, int d) {
  size_t blk = ia_lh(c, layer, head) * (c.max_t / IA_PB) + pos / IA_PB;
  return ((blk * (c.head_dim / 2) + d / 2) * IA_PB + pos % IA_PB) * 2 + d % 2;
}

// Byte offset of value (pos, d): positions in pairs, the pair's two values of
// dimension d adjacent.
__device__ __forceinline__ size_t ia_v_at(const IAView &c, int layer, int head, int pos, int d) {
  size_t pair = ia_lh(c, layer, head) * (c.max_t / 2) + pos / 2;
  return (pair * c.head_dim + d) * 2 + pos % 2;
}

// Block-wide reductions over blockDim.x threads (a multiple of 32); red holds
// 32 slots. Every thread gets the result.
__device__ __forceinline__ float ia_block_max_f(float v, float *red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = fmaxf(m, red[w]);
  return m;
}

__device__ __forceinline__ long long ia_block_max_ll(long long v, long long *red) {
  for (int o = 16; o > 0; o >>= 1) {
    long long u = __shfl_xor_sync(0xffffffffu, v, o);
    v = u > v ? u : v;
  }
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  long long m = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); w++) m = red[w] > m ? red[w] : m;
  return m;
}

__device__ __forceinline__ long long ia_block_sum_ll(long long v, long long *red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  long long t = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); w++) t += red[w];
  return t;
}

// quantize_head (int_attention.mojo:140-168) of one head's key or value by
// the block's threads [0, head_dim): int8 codes round(x / s), s = max|x| / 127
// (1 if zero), the scale kept as round(s * 2^24).
__device__ __forceinline__ void ia_quantize_head(const IAView &c, float x, bool act, int layer, int h, int pos,
                                                 int which, float *red) {
  float mx = ia_block_max_f(act ? fabsf(x) : 0.0f, red);
  float s = mx / 127.0f;
  if (s == 0.0f) s = 1.0f;
  float inv = 1.0f / s;
  int d = threadIdx.x;
  if (act) {
    int8_t code = (int8_t)roundf(x * inv);
    if (which == 0)
      c.k[ia_k_at(c, layer, h, pos, d)] = code;
    else
      c.v[ia_v_at(c, layer, h, pos, d)] = code;
  }
  if (threadIdx.x == 0) {
    int32_t q = (int32_t)llround((double)s * (double)(1 << IA_KS));
    (which == 0 ? c.kq : c.vq)[ia_lh(c, layer, h) * c.max_t + pos] = q;
  }
}

// IntAttnKV.store of T tokens at pos0.. (int_attention.mojo:119-138).
// grid (n_head, T, 2), block >= head_dim.
__global__ void ia_store_kernel(IAView c, const float *qkv, int layer, int pos0) {
  __shared__ float red[32];
  int h = blockIdx.x, t = blockIdx.y, which = blockIdx.z;
  int HS = c.head_dim, C = c.n_head * HS;
  int d = threadIdx.x;
  bool act = d < HS;
  float x = act ? qkv[(size_t)t * 3 * C + (1 + which) * C + h * HS + d] : 0.0f;
  ia_quantize_head(c, x, act, layer, h, pos0 + t, which, red);
}

// exp2_neg (intmath.mojo:53-65): 2^(-d * mult / 2^40) in Q30 by a cubic in
// the fraction and a shift by the integer part.
__device__ __forceinline__ long long ia_exp2_neg(long long d, long long mult) {
  const long long DCAP = 1LL << 31;
  long long y = ((d < DCAP ? d : DCAP) * mult) >> 24;
  long long q = y >> 16;
  long long r = y & ((1 << 16) - 1);
  long long p = -42480028LL;
  p = ((p * r) >> 16) + 248207216LL;
  p = ((p * r) >> 16) + (-742598100LL);
  p = ((p * r) >> 16) + 1073741824LL;
  return q >= 31 ? 0 : p >> (q < 63 ? q : 63);
}

// IntAttnKV.attend_one (int_attention.mojo:170-269) for token t (position
// pos0 + t, or *pos_dev + t) and head h; grid (n_head, T), 256 threads.
//   1. q as int16: sq = max|q| / 32767, qi = round(q / sq); qm = round(sq /
//      sqrt(hd) * 2^40).
//   2. scores over the 16-rounded positions: int32 dot of qi with the int8 key
//      (dp2a), t = (dot * kq + 2^23) >> 24, S = (t * qm + 2^23) >> 24.
//   3. masked_exp over the npos valid scores: e in Q30, total in int64.
//   4. weights w = min((e * r16 + 2^30) >> 31, 32767), r16 = (vq * (2^47 /
//      vmax)) >> 31; values summed as int32 per 128 pairs of positions and
//      flushed to float in order; out = acc * vmax * 2^15 / (2^24 * total).
// Integer sums are exact (mod 2^32 as the reference's), so their order is
// free; the float flushes keep the reference's order. With store != 0 the CTA
// first stores this token's key and value for its head (decode, T == 1).
// Shared memory: max_t * 4 (scores, then e) + (max_t + 2) * 2 (weights) bytes.
__global__ void __launch_bounds__(256) ia_attend_kernel(IAView c, float *out, const float *qkv, int layer, int pos0,
                                                        const int *pos_dev, int store, long long mult) {
  extern __shared__ __align__(16) unsigned char ia_sm[];
  __shared__ long long redl[32];
  __shared__ float redf[32];
  __shared__ int32_t qpair[64];       // qi as int16 pairs (head_dim <= 128)
  __shared__ int32_t part[4 * 128];   // value partials [part][d]
  const int h = blockIdx.x, t = blockIdx.y;
  const int HS = c.head_dim, C = c.n_head * HS;
  const int P0 = pos_dev ? *pos_dev : pos0;
  const int npos = P0 + t + 1;
  const int nr = (npos + IA_PB - 1) / IA_PB * IA_PB;
  int32_t *sc = (int32_t *)ia_sm;                          // [max_t]
  int16_t *w = (int16_t *)(ia_sm + (size_t)c.max_t * 4);   // [max_t + 2]
  const int tid = threadIdx.x;

  if (store) {
    int pos = P0 + t;
    for (int which = 0; which < 2; which++) {
      bool act = tid < HS;
      float x = act ? qkv[(size_t)t * 3 * C + (1 + which) * C + h * HS + tid] : 0.0f;
      ia_quantize_head(c, x, act, layer, h, pos, which, redf);
    }
    __syncthreads();
  }

  // 1. the query as int16
  const float *q = qkv + (size_t)t * 3 * C + h * HS;
  float qv = tid < HS ? q[tid] : 0.0f;
  float mq = ia_block_max_f(fabsf(qv), redf);
  float sq = mq / 32767.0f;
  if (sq == 0.0f) sq = 1.0f;
  float invq = 1.0f / sq;
  int16_t qi = (int16_t)roundf(qv * invq);
  int16_t qi_next = (int16_t)__shfl_down_sync(0xffffffffu, (int)qi, 1);
  if (tid < HS && (tid & 1) == 0) qpair[tid / 2] = (int32_t)(uint16_t)qi | ((int32_t)qi_next << 16);
  const long long qm = llround((double)sq / sqrt((double)HS) * (double)(1LL << (IA_SF + IA_KS)));
  __syncthreads();

  // 2. scores of positions [0, nr)
  const int32_t *ks = c.kq + ia_lh(c, layer, h) * c.max_t;
  long long smax = LLONG_MIN;
  for (int pos = tid; pos < nr; pos += blockDim.x) {
    const uint16_t *kp = (const uint16_t *)(c.k + ia_k_at(c, layer, h, pos, 0));
    int acc = 0;
    for (int j = 0; j < HS / 2; j++) acc = __dp2a_lo(qpair[j], (int)kp[(size_t)j * IA_PB], acc);
    long long t1 = ((long long)acc * (long long)ks[pos] + (1LL << (IA_KS - 1))) >> IA_KS;
    long long sfix = (t1 * qm + (1LL << (IA_KS - 1))) >> IA_KS;
    sc[pos] = (int32_t)sfix;
    if (pos < npos && (long long)(int32_t)sfix > smax) smax = (int32_t)sfix;
  }
  const long long m = ia_block_max_ll(smax, redl);

  // 3. masked_exp: e in Q30 over the valid positions, total in int64
  long long part_total = 0;
  for (int pos = tid; pos < nr; pos += blockDim.x) {
    long long ev = pos < npos ? ia_exp2_neg(m - (long long)sc[pos], mult) : 0;
    sc[pos] = (int32_t)ev;
    part_total += ev;
  }
  const long long total = ia_block_sum_ll(part_total, redl);

  // 4. value weights and sums
  const int32_t *vs = c.vq + ia_lh(c, layer, h) * c.max_t;
  long long vm = 0;
  for (int pos = tid; pos < npos; pos += blockDim.x) vm = (long long)vs[pos] > vm ? (long long)vs[pos] : vm;
  const long long vmax = ia_block_max_ll(vm, redl);
  float *o = out + (size_t)t * C + h * HS;
  if (vmax == 0 || total == 0) {
    for (int d = tid; d < HS; d += blockDim.x) o[d] = 0.0f;
    return;
  }
  const long long inv47 = (1LL << 47) / vmax;
  for (int pos = tid; pos < nr + 2; pos += blockDim.x) {
    long long ww = 0;
    if (pos < nr) {
      long long ee = sc[pos];
      long long r16 = pos < npos ? ((long long)vs[pos] * inv47) >> 31 : 0;
      ww = (ee * r16 + (1LL << 30)) >> 31;
      if (ww > 32767) ww = 32767;
      if (ee == 0) ww = 0;
    }
    w[pos] = (int16_t)ww;
  }
  __syncthreads();
  const int nparts = blockDim.x / HS;  // threads per dimension
  const int d = tid % HS, pidx = tid / HS;
  const int npairs = (npos + 1) / 2;
  float accf = 0.0f;
  const uint16_t *vbase = (const uint16_t *)(c.v + ia_v_at(c, layer, h, 0, 0));
  for (int seg = 0; seg < npairs; seg += 128) {
    int end = npairs < seg + 128 ? npairs : seg + 128;
    int acc = 0;
    if (pidx < nparts)
      for (int pp = seg + pidx; pp < end; pp += nparts) {
        int wp = (int)(uint16_t)w[2 * pp] | ((int)w[2 * pp + 1] << 16);
        acc = __dp2a_lo(wp, (int)vbase[(size_t)pp * HS + d], acc);
      }
    if (pidx < nparts) part[pidx * HS + d] = acc;
    __syncthreads();
    if (pidx == 0) {
      unsigned sum = 0;
      for (int p = 0; p < nparts; p++) sum += (unsigned)part[p * HS + d];
      accf += (float)(int32_t)sum;
    }
    __syncthreads();
  }
  if (pidx == 0) {
    float fs = (float)((double)vmax * (double)(1 << 15) / ((double)(1 << IA_KS) * (double)total));
    o[d] = accf * fs;
  }
}

}  // namespace llmq
