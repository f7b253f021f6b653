// One-token matmuls with float32 arithmetic (sm_100a): dequantize-and-dot
// for the GGUF block formats and dense rows, the affine W4A32 / W8A32 path,
// and the dense [IN, OUT] split-K GEMV; plus the integer GGUF head.
//
// Reference order: every output is the reference's 16 float32 lane chains,
// acc[l] = fma(w, x, acc[l]) over the row in its put order (gguf.mojo:
// 166-297 each_block/dequant_q*, tensor.mojo:431-476 row_op,
// tensor.mojo:206-210 DenseMatrix.dot_row), added by the halving tree. Here
// 16 threads share a row, thread l carrying lane l's chain; the tree is four
// xor shuffles. Rows of the GGUF and dense-row formats are staged through
// shared memory: a tile of rows (contiguous bytes) per cp.async.bulk copy,
// two stages, mbarrier completion.
#pragma once

#include "common.cuh"
#include "gemv_a16.cuh"

namespace llmq {

enum {
  RT_F32 = 0, RT_F16 = 1, RT_Q4_0 = 2, RT_Q4_1 = 3, RT_Q8_0 = 8, RT_Q4_K = 12, RT_Q5_K = 13, RT_Q6_K = 14,
  RT_BF16 = 30  // dense bfloat16 rows (not a GGUF type)
};

__host__ __device__ inline int rt_block_size(int t) {
  return (t == RT_F32 || t == RT_F16 || t == RT_BF16) ? 16 : (t == RT_Q4_0 || t == RT_Q4_1 || t == RT_Q8_0) ? 32 : 256;
}
__host__ __device__ inline int rt_block_bytes(int t) {
  switch (t) {
    case RT_F32: return 64;
    case RT_F16: return 32;
    case RT_BF16: return 32;
    case RT_Q4_0: return 18;
    case RT_Q4_1: return 20;
    case RT_Q8_0: return 34;
    case RT_Q4_K: return 144;
    case RT_Q5_K: return 176;
    case RT_Q6_K: return 210;
  }
  return 0;
}

struct RowMat {
  const uint8_t *data;  // rows * row_bytes
  int rows, cols, type;
  long long row_bytes;
};

__device__ __forceinline__ float ld_f16(const uint8_t *p) {
  return __half2float(__ushort_as_half((unsigned short)(p[0] | (p[1] << 8))));
}

// k_scale_min (gguf.mojo:205-221).
__device__ __forceinline__ void k_sm(const uint8_t *q, int j, int &sc, int &m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// The dequantized values of lane L of one block of type T at b
// (dequant_q4_0 .. dequant_q6_k, gguf.mojo:178-297), in the reference's put
// order: f(value, index in the block) for each. The dot (block_lane) and the
// plain dequantization (gguf_dequant_rows_kernel) both use it.
template <int T, class F>
__device__ __forceinline__ void block_values(const uint8_t *b, int L, F &&f) {
  if (T == RT_Q4_0) {
    const float d = ld_f16(b);
    const int q = b[2 + L];
    f(((float)(q & 0xF) - 8.0f) * d, L);
    f(((float)(q >> 4) - 8.0f) * d, 16 + L);
  } else if (T == RT_Q4_1) {
    const float d = ld_f16(b), m = ld_f16(b + 2);
    const int q = b[4 + L];
    f(d * (float)(q & 0xF) + m, L);
    f(d * (float)(q >> 4) + m, 16 + L);
  } else if (T == RT_Q8_0) {
    const float d = ld_f16(b);
    f(d * (float)(int8_t)b[2 + L], L);
    f(d * (float)(int8_t)b[18 + L], 16 + L);
  } else if (T == RT_Q4_K || T == RT_Q5_K) {
    const float d = ld_f16(b), dmin = ld_f16(b + 2);
    const uint8_t *sc = b + 4;
#pragma unroll
    for (int j = 0; j < 4; j++) {
      int s1, m1i, s2, m2i;
      k_sm(sc, 2 * j, s1, m1i);
      k_sm(sc, 2 * j + 1, s2, m2i);
      const float d1 = d * (float)s1, m1 = dmin * (float)m1i, d2 = d * (float)s2, m2 = dmin * (float)m2i;
#pragma unroll
      for (int h = 0; h < 2; h++) {
        int lo, hi;
        if (T == RT_Q4_K) {
          const int q = b[16 + 32 * j + 16 * h + L];
          lo = q & 0xF;
          hi = q >> 4;
        } else {
          const int qh = b[16 + 16 * h + L], q = b[48 + 32 * j + 16 * h + L];
          lo = (q & 0xF) | (((qh >> (2 * j)) & 1) << 4);
          hi = (q >> 4) | (((qh >> (2 * j + 1)) & 1) << 4);
        }
        f(d1 * (float)lo - m1, 64 * j + 16 * h + L);
        f(d2 * (float)hi - m2, 64 * j + 32 + 16 * h + L);
      }
    }
  } else if (T == RT_Q6_K) {
    const float d = ld_f16(b + 208);
#pragma unroll
    for (int n = 0; n < 2; n++) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int lo0 = b[64 * n + 16 * h + L], lo1 = b[64 * n + 32 + 16 * h + L], hi = b[128 + 32 * n + 16 * h + L];
        const int base = 128 * n + 16 * h;
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const float ds = d * (float)(int8_t)b[192 + 8 * n + h + 2 * k];
          int q;
          if (k == 0) q = (lo0 & 0xF) | ((hi & 3) << 4);
          else if (k == 1) q = (lo1 & 0xF) | (((hi >> 2) & 3) << 4);
          else if (k == 2) q = (lo0 >> 4) | (((hi >> 4) & 3) << 4);
          else q = (lo1 >> 4) | (((hi >> 6) & 3) << 4);
          f(ds * ((float)q - 32.0f), base + 32 * k + L);
        }
      }
    }
  } else if (T == RT_F32) {
    f(((const float *)b)[L], L);
  } else if (T == RT_F16) {
    f(__half2float(((const __half *)b)[L]), L);
  } else if (T == RT_BF16) {
    f(__uint_as_float((unsigned)((const uint16_t *)b)[L] << 16), L);
  }
}

// Lane L's chain over one block of type T at b (in shared memory); x is the
// block's slice of the input.
template <int T>
__device__ __forceinline__ float block_lane(const uint8_t *b, const float *x, int L, float acc) {
  block_values<T>(b, L, [&](float v, int i) { acc = fmaf(v, x[i], acc); });
  return acc;
}

constexpr int RF_THREADS = 256;
constexpr int RF_TILE_BYTES = 32 * 1024;  // bytes of rows per stage
constexpr int RF_STAGES = 2;              // stages per CTA (4 stages of 24 KB measured no faster)
constexpr int RF_MAX_ROWS = 16;           // rows per tile: one per half-warp

// Rows per tile for rows of rb bytes (the copied span is 16-byte rounded
// at both ends, hence the 32 bytes of slack).
__host__ __device__ inline int rf_rows(int rb) {
  const int r = (RF_TILE_BYTES - 32) / rb;
  return r < 1 ? 1 : (r > RF_MAX_ROWS ? RF_MAX_ROWS : r);
}

struct RowGemvArgs {
  RowMat w;
  const float *x;     // [cols]
  const float *bias;  // [rows] or null
  float *out;         // [rows]
  int epi;            // EPI_BIAS / EPI_GELU / EPI_RESID
  int *err;           // device error word: set to 6 when a tile's copy wait gives up
  long long timeout;  // cycles a tile's copy wait may take
};

// Bound of the waits for copies still in flight when a kernel gives up
// (independent of the settable wait limit, so that no CTA leaves while a
// copy may still write its shared memory).
constexpr long long kDrainCycles = 4000000000LL;

__device__ __forceinline__ unsigned rf_smem_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

// Row-major float GEMV: CTA tiles of R rows (R * row_bytes <= RF_TILE_BYTES,
// R <= RF_MAX_ROWS), RF_STAGES shared-memory stages filled by
// cp.async.bulk: thread 0 arms a stage's mbarrier and issues the tile's one
// contiguous copy; tile it + RF_STAGES - 1 is requested as tile it is summed.
template <int T>
__global__ void __launch_bounds__(RF_THREADS) row_gemv_kernel(RowGemvArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  const int cols = a.w.cols, rb = (int)a.w.row_bytes;
  const int R = rf_rows(rb);
  float *xs = (float *)smem;                                         // [cols]
  unsigned long long *bar = (unsigned long long *)(smem + cols * 4);  // [RF_STAGES]
  uint8_t *stages = smem + cols * 4 + 128;                            // [RF_STAGES][RF_TILE_BYTES]
  const int ntiles = (a.w.rows + R - 1) / R;
  for (int i = threadIdx.x; i < cols; i += RF_THREADS) xs[i] = a.x[i];
  if (threadIdx.x == 0) {
    for (int k = 0; k < RF_STAGES; k++) asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(rf_smem_u32(&bar[k])));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  // Rows [r0, r0 + n) start at byte r0 * rb, which need not be 16-byte
  // aligned (Q6_K rows are 630 bytes for 768 columns): copy the aligned
  // superset [floor16(r0 * rb), ceil16((r0 + n) * rb)) and read the rows at
  // the offset. The matrix buffer has 32 bytes of padding after its end.
  auto issue = [&](int tile, int s) {
    const int r0 = tile * R, n = min(R, a.w.rows - r0);
    const long long start = (long long)r0 * rb, lo = start & ~15LL, hi = (start + (long long)n * rb + 15) & ~15LL;
    const unsigned bytes = (unsigned)(hi - lo);
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(rf_smem_u32(&bar[s])), "r"(bytes)
                 : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            rf_smem_u32(stages + (size_t)s * RF_TILE_BYTES)),
        "l"(a.w.data + lo), "r"(bytes), "r"(rf_smem_u32(&bar[s]))
        : "memory");
  };
  if (threadIdx.x == 0)
    for (int k = 0; k < RF_STAGES - 1; k++) {
      const int tile = blockIdx.x + k * gridDim.x;
      if (tile < ntiles) issue(tile, k);
    }
  int it = 0;
  for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, it++) {
    const int s = it % RF_STAGES;
    const int ahead = tile + (RF_STAGES - 1) * gridDim.x;
    if (threadIdx.x == 0 && ahead < ntiles) issue(ahead, (it + RF_STAGES - 1) % RF_STAGES);
    // wait for this tile (phase it / RF_STAGES of stage s); the decision to
    // give up is taken by the whole CTA, so every thread meets the same barriers
    auto wait_stage = [&](int k, long long limit) {
      const unsigned par = (unsigned)((k / RF_STAGES) & 1);
      unsigned ok = 0;
      const long long t0 = clock64();
      while (!ok && clock64() - t0 < limit)
        asm volatile(
            "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
            : "=r"(ok)
            : "r"(rf_smem_u32(&bar[k % RF_STAGES])), "r"(par)
            : "memory");
      return ok != 0;
    };
    if (__syncthreads_or(!wait_stage(it, a.timeout))) {
      // a copy did not land in time: record it, wait (bounded) for this
      // tile's copy and the ones issued after it, then give up
      if (threadIdx.x == 0) {
        atomicCAS(a.err, 0, 6);
        for (int k = it; k < it + RF_STAGES && tile + (k - it) * gridDim.x < ntiles; k++) wait_stage(k, kDrainCycles);
      }
      __syncthreads();
      return;
    }
    const int r0 = tile * R, n = min(R, a.w.rows - r0);
    const int shift = (int)(((long long)r0 * rb) & 15);
    const uint8_t *stage = stages + (size_t)s * RF_TILE_BYTES;
    const int L = threadIdx.x & 15, g = threadIdx.x >> 4;
    // rows of the tile handled by this half-warp: every half-warp runs the
    // same number of rounds (the shuffles below take the full warp)
    for (int rr0 = 0; rr0 < R; rr0 += RF_THREADS / 16) {
      const int rr = rr0 + g;
      const bool live = rr < n;
      const uint8_t *row = stage + shift + (size_t)(live ? rr : 0) * rb;
      float acc = 0.0f;
      const int bs = rt_block_size(T), bb = rt_block_bytes(T);
      for (int blk = 0; blk < cols / bs; blk++) acc = block_lane<T>(row + blk * bb, xs + blk * bs, L, acc);
      acc = acc + __shfl_xor_sync(0xffffffffu, acc, 8);
      acc = acc + __shfl_xor_sync(0xffffffffu, acc, 4);
      acc = acc + __shfl_xor_sync(0xffffffffu, acc, 2);
      acc = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
      if (live && L == 0) {
        const int o = r0 + rr;
        float v = acc;
        if (a.epi & EPI_BIAS) v += a.bias[o];
        if (a.epi & EPI_GELU) v = gelu(v);
        if (a.epi & EPI_RESID) v += a.out[o];
        a.out[o] = v;
      }
    }
    __syncthreads();  // the stage is free for the tile RF_STAGES - 1 ahead
  }
}

// Affine W4A32 / W8A32 rows (QuantMatrix.dot_row, tensor.mojo:431-482, natural
// layout): per group, lane chains accg = fma(u - zp, x, accg) over the group's
// 32-chunks (low half, then high half of each), then acc = fma(accg, s, acc).
struct AffFloatArgs {
  WeightView w;
  const float *x;
  const float *bias;
  float *out;
  int epi;
};

template <int BITS>
__global__ void __launch_bounds__(256) affine_float_gemv_kernel(AffFloatArgs a) {
  extern __shared__ __align__(16) float xsh[];
  const int cols = a.w.cols, G = a.w.group, gpr = cols / G;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) xsh[i] = a.x[i];
  __syncthreads();
  const int L = threadIdx.x & 15;
  // the loop bound is the CTA's: every half-warp runs every round, so the
  // full-warp shuffles below always have the whole warp
  for (int base = blockIdx.x * 16; base < a.w.rows; base += gridDim.x * 16) {
    const bool live = base + (threadIdx.x >> 4) < a.w.rows;
    const int row = live ? base + (threadIdx.x >> 4) : a.w.rows - 1;
    const uint8_t *p = a.w.codes + (size_t)row * cols * BITS / 8;
    float acc = 0.0f;
    for (int g = 0; g < gpr; g++) {
      const float s = __half2float(__ushort_as_half(a.w.scale[(size_t)row * gpr + g]));
      const float zp = (float)a.w.zp[(size_t)row * gpr + g];
      float accg = 0.0f;
      for (int c = 0; c < G / 32; c++) {
        const int k0 = g * G + 32 * c;
        float v0, v1;
        if (BITS == 4) {
          const int b = __ldg(p + k0 / 2 + L);
          v0 = (float)(b & 0xF) - zp;
          v1 = (float)(b >> 4) - zp;
        } else {
          v0 = (float)__ldg(p + k0 + L) - zp;
          v1 = (float)__ldg(p + k0 + 16 + L) - zp;
        }
        accg = fmaf(v0, xsh[k0 + L], accg);
        accg = fmaf(v1, xsh[k0 + 16 + L], accg);
      }
      acc = fmaf(accg, s, acc);
    }
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 8);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 4);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 2);
    acc = acc + __shfl_xor_sync(0xffffffffu, acc, 1);
    if (live && L == 0) {
      float v = acc;
      if (a.epi & EPI_BIAS) v += a.bias[row];
      if (a.epi & EPI_GELU) v = gelu(v);
      if (a.epi & EPI_RESID) v += a.out[row];
      a.out[row] = v;
    }
  }
}

// The same rows for group sizes 32, 64 and 128, with the work split so that
// small matrices still fill the GPU: a row's group sums accg[g][L] (lane L's
// chain over the group's 32-chunks) are independent of each other, and only
// the fold acc = fma(accg, s, acc) is sequential over the groups. Phase 1:
// thread (row, g) computes the 16 lane sums of one group from one 16-byte (int4)
// or two (int8) loads per 32-chunk, into shared memory; phase 2: one thread per
// (row, lanes L, L + 8) folds them over the groups in order, and one thread per
// row adds the halving tree. AFG_ROWS rows per CTA (more CTAs than the
// 16-lanes-per-row kernel for layer shapes). x sits in shared memory padded by
// one float per 32, so threads of different groups read different banks.
__host__ __device__ inline size_t afg_smem(int cols, int gpr, int rows_per_cta) {
  return (size_t)(cols + cols / 32) * 4 + (size_t)16 * (gpr * rows_per_cta + 1) * 4 + (size_t)gpr * rows_per_cta * 4 +
         8 * rows_per_cta * 4;
}

template <int BITS, int AFG_ROWS>
__global__ void __launch_bounds__(256) affine_float_group_kernel(AffFloatArgs a) {
  extern __shared__ __align__(16) float afg[];
  const int cols = a.w.cols, G = a.w.group, gpr = cols / G, cpg = G / 32, LS = gpr * AFG_ROWS + 1;
  float *xsh = afg;                              // [cols + cols / 32], x[k] at k + k / 32
  float *acc_s = xsh + cols + cols / 32;         // [16][LS]: lane L, group g, row r at L * LS + g * ROWS + r
  float *scl = acc_s + 16 * LS;                  // [gpr][ROWS]
  float *tsum = scl + gpr * AFG_ROWS;            // [8][ROWS]: the tree's first level
  const int tid = threadIdx.x;
  for (int i = tid; i < cols; i += blockDim.x) xsh[i + (i >> 5)] = a.x[i];
  for (int base = blockIdx.x * AFG_ROWS; base < a.w.rows; base += gridDim.x * AFG_ROWS) {
    __syncthreads();  // x staged; the previous rows' sums consumed
    // phase 1: thread (row r, group g) for items i = r + ROWS * g
    for (int i = tid; i < gpr * AFG_ROWS; i += blockDim.x) {
      const int r = i % AFG_ROWS, g = i / AFG_ROWS;
      const int row = min(base + r, a.w.rows - 1);
      const uint8_t *p = a.w.codes + (size_t)row * cols * BITS / 8;
      const float zp = (float)a.w.zp[(size_t)row * gpr + g];
      scl[g * AFG_ROWS + r] = __half2float(__ushort_as_half(a.w.scale[(size_t)row * gpr + g]));
      float acc[16];
#pragma unroll
      for (int L = 0; L < 16; L++) acc[L] = 0.0f;
      for (int c = 0; c < cpg; c++) {
        const int k0 = g * G + 32 * c;
        const float *x0 = xsh + k0 + (k0 >> 5), *x1 = x0 + 16;  // columns k0 .. k0 + 31 (one 32-chunk)
        uint32_t wlo[4], whi[4];
        if (BITS == 4) {
          const uint4 w = __ldg((const uint4 *)(p + k0 / 2));
          wlo[0] = w.x, wlo[1] = w.y, wlo[2] = w.z, wlo[3] = w.w;
        } else {
          const uint4 w0 = __ldg((const uint4 *)(p + k0)), w1 = __ldg((const uint4 *)(p + k0 + 16));
          wlo[0] = w0.x, wlo[1] = w0.y, wlo[2] = w0.z, wlo[3] = w0.w;
          whi[0] = w1.x, whi[1] = w1.y, whi[2] = w1.z, whi[3] = w1.w;
        }
#pragma unroll
        for (int L = 0; L < 16; L++) {
          const unsigned b = (wlo[L >> 2] >> (8 * (L & 3))) & 0xFFu;
          float v0, v1;
          if (BITS == 4) {
            v0 = (float)(b & 0xFu) - zp;
            v1 = (float)(b >> 4) - zp;
          } else {
            v0 = (float)b - zp;
            v1 = (float)((whi[L >> 2] >> (8 * (L & 3))) & 0xFFu) - zp;
          }
          acc[L] = fmaf(v0, x0[L], acc[L]);
          acc[L] = fmaf(v1, x1[L], acc[L]);
        }
      }
#pragma unroll
      for (int L = 0; L < 16; L++) acc_s[L * LS + g * AFG_ROWS + r] = acc[L];
    }
    __syncthreads();
    // phase 2: thread (row r, lanes L and L + 8): acc = fma(accg, s, acc) over
    // the groups in order, then the tree's first level acc_L + acc_{L+8}
    if (tid < 8 * AFG_ROWS) {
      const int r = tid % AFG_ROWS, L = tid / AFG_ROWS;
      const float *a0 = acc_s + L * LS + r, *a1 = acc_s + (L + 8) * LS + r;
      float c0 = 0.0f, c1 = 0.0f;
#pragma unroll 8
      for (int g = 0; g < gpr; g++) {
        const float s = scl[g * AFG_ROWS + r];
        c0 = fmaf(a0[g * AFG_ROWS], s, c0);
        c1 = fmaf(a1[g * AFG_ROWS], s, c1);
      }
      tsum[L * AFG_ROWS + r] = c0 + c1;
    }
    __syncthreads();
    if (tid < AFG_ROWS && base + tid < a.w.rows) {
      const int r = tid, row = base + r;
      const float *t = tsum + r;  // t[i * ROWS] = acc_i + acc_{i+8}
      const float u0 = t[0] + t[4 * AFG_ROWS], u1 = t[1 * AFG_ROWS] + t[5 * AFG_ROWS];
      const float u2 = t[2 * AFG_ROWS] + t[6 * AFG_ROWS], u3 = t[3 * AFG_ROWS] + t[7 * AFG_ROWS];
      float v = (u0 + u2) + (u1 + u3);
      if (a.epi & EPI_BIAS) v += a.bias[row];
      if (a.epi & EPI_GELU) v = gelu(v);
      if (a.epi & EPI_RESID) v += a.out[row];
      a.out[row] = v;
    }
  }
}

// Dense [IN, OUT] split-K GEMV (kernels.mojo:132-176 gemv, :828-865
// linear_team): part p accumulates rows [p*rows, min(IN, (p+1)*rows)),
// rows = ceil(IN / nparts), as one sequential fma chain per output; the
// parts are added in order after the bias. Stage 1: thread per (part,
// output) into scratch; stage 2: thread per output.
template <int DT>
__global__ void dense_gemv_parts_kernel(const void *w, const float *x, int IN, int OUT, int nparts, float *scratch) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, p = blockIdx.y;
  if (j >= OUT) return;
  const int rows = (IN + nparts - 1) / nparts;
  const int i0 = p * rows, i1 = min(IN, i0 + rows);
  float acc = 0.0f;
  for (int i = i0; i < i1; i++) {
    float wv;
    if (DT == 0) wv = __ldg((const float *)w + (size_t)i * OUT + j);
    else if (DT == 1) wv = __half2float(((const __half *)w)[(size_t)i * OUT + j]);
    else wv = __uint_as_float((unsigned)__ldg((const uint16_t *)w + (size_t)i * OUT + j) << 16);
    acc = fmaf(x[i], wv, acc);
  }
  scratch[(size_t)p * OUT + j] = acc;
}

// The same parts, staged: a CTA takes one part x 32 columns. Its threads
// copy the strip (the part's rows x 32 columns, 128 or 64 bytes a row) into
// shared memory with 16-byte cp.async copies, all of them in flight at
// once; warp 0 then runs the 32 chains in row order from shared memory.
// Needs OUT * element size to be a multiple of 16 bytes.
constexpr int DS_THREADS = 256;
constexpr int DS_SMEM = 200 * 1024;

__host__ __device__ inline int ds_rows(int IN, int nparts) { return (IN + nparts - 1) / nparts; }
__host__ __device__ inline int ds_smem(int IN, int nparts, int es) {
  const int rows = ds_rows(IN, nparts);
  return ((rows * 4 + 15) & ~15) + rows * 32 * es;
}

template <int DT>
__global__ void __launch_bounds__(DS_THREADS) dense_strip_kernel(const void *w, const float *x, int IN, int OUT,
                                                                int nparts, float *scratch) {
  extern __shared__ __align__(16) unsigned char smem[];
  constexpr int es = DT == 0 ? 4 : 2;
  const int j0 = blockIdx.x * 32, p = blockIdx.y;
  const int rows = ds_rows(IN, nparts);
  const int i0 = p * rows, n = max(0, min(IN, i0 + rows) - i0);
  float *xs = (float *)smem;
  uint8_t *tiles = smem + ((rows * 4 + 15) & ~15);
  const int ppr = min(32, OUT - j0) * es / 16;  // 16-byte pieces per row
  const uint8_t *src = (const uint8_t *)w + ((size_t)i0 * OUT + j0) * es;
  const size_t rstride = (size_t)OUT * es;
  for (int k = threadIdx.x; k < n * ppr; k += DS_THREADS) {
    const int r = k / ppr, c = k - r * ppr;
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(rf_smem_u32(tiles + r * 32 * es + c * 16)),
                 "l"(src + r * rstride + c * 16)
                 : "memory");
  }
  asm volatile("cp.async.commit_group;" ::: "memory");
  for (int k = threadIdx.x; k < n; k += DS_THREADS) xs[k] = x[i0 + k];
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  __syncthreads();
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  auto wv = [&](int r) {
    if (DT == 0) return ((const float *)tiles)[r * 32 + lane];
    const uint16_t h = ((const uint16_t *)tiles)[r * 32 + lane];
    if (DT == 1) return __half2float(__ushort_as_half(h));
    return __uint_as_float((unsigned)h << 16);
  };
  float acc = 0.0f;
  int r = 0;
  for (; r + 8 <= n; r += 8) {
#pragma unroll
    for (int k = 0; k < 8; k++) acc = fmaf(xs[r + k], wv(r + k), acc);
  }
  for (; r < n; r++) acc = fmaf(xs[r], wv(r), acc);
  if (j0 + lane < OUT) scratch[(size_t)p * OUT + j0 + lane] = acc;
}

__global__ void dense_gemv_combine_kernel(const float *scratch, const float *bias, float *out, int OUT, int nparts,
                                          int epi) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= OUT) return;
  float r = (epi & EPI_BIAS) ? bias[j] : 0.0f;
  for (int p = 0; p < nparts; p++) r += scratch[(size_t)p * OUT + j];
  if (epi & EPI_GELU) r = gelu(r);
  if (epi & EPI_RESID) r += out[j];
  out[j] = r;
}

// The GGUF integer head (gguf.mojo:456-505, kernels.mojo:693-736) for one
// token: x quantized to int16 (quantize_rows), weights as int16
// ((q - 32) * scale for Q6_K, q for Q8_0), int32 lane sums (lane i: pair
// 2i, 2i+1 of each 32 weights) per block (Q8_0) or superblock (Q6_K), then
// accf = fma(f32(acc), d, accf) and the halving tree; logit = dot * sx.
template <int T>
__global__ void __launch_bounds__(256) gguf_head_i16_kernel(RowMat w, const float *h, float *logits) {
  __shared__ __align__(16) int16_t xq[4096];
  __shared__ float red[64];
  const int cols = w.cols;
  h += (size_t)blockIdx.y * cols;  // grid y: the tokens
  logits += (size_t)blockIdx.y * w.rows;
  float mx = 0.0f;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) mx = fmaxf(mx, fabsf(h[i]));
  mx = block_max(mx, red);
  float s = mx / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  const float inv = 1.0f / s;
  for (int i = threadIdx.x; i < cols; i += blockDim.x) xq[i] = (int16_t)round_away(h[i] * inv);
  __syncthreads();
  const int L = threadIdx.x & 15;
  // CTA-uniform rounds: the full-warp shuffles below always have the whole warp
  for (int base = blockIdx.x * 16; base < w.rows; base += gridDim.x * 16) {
    const bool live = base + (threadIdx.x >> 4) < w.rows;
    const int row = live ? base + (threadIdx.x >> 4) : w.rows - 1;
    const uint8_t *p = w.data + (size_t)row * w.row_bytes;
    float accf = 0.0f;
    if (T == RT_Q8_0) {
      for (int blk = 0; blk < cols / 32; blk++) {
        const uint8_t *b = p + blk * 34;
        const int acc = (int)xq[blk * 32 + 2 * L] * (int)(int8_t)b[2 + 2 * L] +
                        (int)xq[blk * 32 + 2 * L + 1] * (int)(int8_t)b[3 + 2 * L];
        accf = fmaf((float)acc, ld_f16(b), accf);
      }
    } else {
      for (int sb = 0; sb < cols / 256; sb++) {
        const uint8_t *b = p + sb * 210;
        int acc = 0;
#pragma unroll
        for (int n = 0; n < 2; n++)
#pragma unroll
          for (int k = 0; k < 4; k++) {
            const uint8_t *Lb = b + 64 * n + ((k & 1) ? 32 : 0);
            const uint8_t *Hb = b + 128 + 32 * n;
            const int sc = (int8_t)b[192 + 8 * n + 2 * k + (L >= 8 ? 1 : 0)];
#pragma unroll
            for (int e = 0; e < 2; e++) {
              const int j = 2 * L + e;
              const int q = ((k >= 2) ? (Lb[j] >> 4) : (Lb[j] & 0xF)) | (((Hb[j] >> (2 * k)) & 3) << 4);
              acc += (int)xq[sb * 256 + 128 * n + 32 * k + j] * ((q - 32) * sc);
            }
          }
        accf = fmaf((float)acc, ld_f16(b + 208), accf);
      }
    }
    accf = accf + __shfl_xor_sync(0xffffffffu, accf, 8);
    accf = accf + __shfl_xor_sync(0xffffffffu, accf, 4);
    accf = accf + __shfl_xor_sync(0xffffffffu, accf, 2);
    accf = accf + __shfl_xor_sync(0xffffffffu, accf, 1);
    if (live && L == 0) logits[row] = accf * s;
  }
}

}  // namespace llmq
