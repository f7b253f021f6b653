// Split-int8 tcgen05 GEMM for the W4A16 / W8A16 several-token matmul
// (tile_i16, kernels.mojo:512-573) on sm_100a.
//
// The reference computes, per (token m, output n), an int32 sum of
// x[m,k] * (u[n,k] - zp[n,g]) over each segment of min(G, 256) inputs and
// folds it into accf = fma(f32(acc), s[n,g], accf), segment by segment, then
// r = accf * sx[m] (+ b[n]) and store_out. The int16 activation is split as
// x = 256 * xh + xl (xh signed, xl unsigned, both 8-bit), so every segment sum
// is 256 * D_h + D_l (- zp * sum(x) for int8 weights), with D_h and D_l from
// two tcgen05 kind::i8 MMAs into int32 tensor-memory accumulators. The int32
// arithmetic is exact modulo 2^32, as the reference's accumulator is, so each
// segment sum equals the reference's bit for bit; the float folds keep its
// order, so outputs are bit-identical.
//
// Operands are staged as tiles that one bulk copy each brings into shared
// memory, already in the MMA's no-swizzle K-major layout (8-row x 16-byte core
// matrices): for each 128-byte K block, 8 columns of 16 bytes, each column
// the tile's rows one after the other.
//   A (activations, prepared per call by tc_split_rows_kernel):
//     [m_tile][k_block][plane l,h][chunk 8][128 rows][16 B]
//   B (weights, prepared once per weight by tc_prep_b_kernel):
//     [n_tile][k_block][chunk 8][64 rows][16 B], int4 as int8 (u - zp), int8
//     as its u8 code (zero point applied in the epilogue).
//
// One CTA per 128 x 64 output tile: warp 8 issues the bulk copies and the
// MMAs (one thread), warps 0-7 read the accumulators segment by segment
// (warp w: tensor-memory lanes 32 * (w % 4), columns 32 * (w / 4)), while
// the MMAs of the next segments run into 4 rotating accumulator pairs.
#pragma once

#include "gemv_a16.cuh"

namespace llmq {

constexpr int TC_M = 128;                                  // tokens per tile (MMA M)
constexpr int TC_N = 64;                                   // outputs per tile (MMA N)
constexpr int TC_KB = 128;                                 // K bytes per pipeline stage
constexpr int TC_STAGES = 4;
constexpr int TC_NBUF = 4;                                 // accumulator pairs: 4 * 2 * 64 = 512 columns
constexpr int TC_A_PLANE = TC_M * TC_KB;                   // 16 KB
constexpr int TC_A_BYTES = 2 * TC_A_PLANE;                 // 32 KB, planes l and h
constexpr int TC_B_BYTES = TC_N * TC_KB;                   // 8 KB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_BYTES;    // 40 KB
constexpr int TC_EPI_WARPS = 8;
constexpr int TC_THREADS = (TC_EPI_WARPS + 1) * 32;        // 288
constexpr int TC_MAX_GROUPS = 96;                          // groups per row in the scale table
constexpr int TC_TMEM_COLS = 512;
constexpr long long TC_TIMEOUT = 4000000000LL;             // cycles a wait may take (~2 s)

enum { TC_ERR_FULL = 1, TC_ERR_EMPTY = 2, TC_ERR_ACC = 3, TC_ERR_ACCEMPTY = 4 };

struct TcSmem {
  alignas(128) uint8_t stage[TC_STAGES][TC_STAGE_BYTES];
  float scale[TC_MAX_GROUPS][TC_N];
  uint8_t zc[TC_MAX_GROUPS][TC_N];
  alignas(8) unsigned long long full[TC_STAGES], empty[TC_STAGES], accfull[TC_NBUF], accempty[TC_NBUF], drain;
  unsigned tmem;
  int abort;
};

struct TcArgs {
  const uint8_t *a;   // prepared activations
  const uint8_t *b;   // prepared weights
  const float *sx;    // [m_pad] activation scales
  const int *xsum;    // [m_pad][nseg] segment sums of x (int8 weights)
  WeightView w;       // scales and zero points
  const float *bias;
  float *out;
  int *err;
  int T, OUT, n_full, K, nkb, nseg, seg_ks, seg, epi;
};

// --- PTX wrappers -----------------------------------------------------------

__device__ __forceinline__ unsigned tc_u32(const void *p) { return (unsigned)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void tc_mbar_init(unsigned bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void tc_mbar_arrive(unsigned bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mbar_expect_tx(unsigned bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool tc_mbar_try(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ void tc_bulk_g2s(unsigned dst, const void *src, unsigned bytes, unsigned bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor, no swizzle, K-major: start, LBO (between
// the two 16-byte K columns of one MMA), SBO (between 8-row core matrices).
__device__ __forceinline__ unsigned long long tc_desc(unsigned addr, unsigned lbo, unsigned sbo) {
  return (unsigned long long)((addr >> 4) & 0x3FFF) | ((unsigned long long)((lbo >> 4) & 0x3FFF) << 16) |
         ((unsigned long long)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);  // version 1, base 0, no swizzle
}

// Instruction descriptor of kind::i8: D s32, A/B u8 (0) or s8 (1), both
// K-major, N = 64, M = 128.
__host__ __device__ constexpr unsigned tc_idesc(int a_signed, int b_signed) {
  return (2u << 4) | ((unsigned)a_signed << 7) | ((unsigned)b_signed << 10) | ((unsigned)(TC_N >> 3) << 17) |
         ((unsigned)(TC_M >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(unsigned d, unsigned long long a, unsigned long long b, unsigned idesc,
                                       unsigned accumulate) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(unsigned bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_ld32(unsigned addr, int (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
}
__device__ __forceinline__ void tc_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Bounded wait: false once the CTA aborted or after TC_TIMEOUT cycles (then
// the CTA aborts and the error code is recorded).
__device__ __forceinline__ bool tc_wait(TcSmem &sm, unsigned bar, unsigned parity, int *err, int code) {
  long long t0 = clock64();
  while (!tc_mbar_try(bar, parity)) {
    if (*(volatile int *)&sm.abort) return false;
    if (clock64() - t0 > TC_TIMEOUT) {
      *(volatile int *)&sm.abort = 1;
      atomicExch(err, code);
      return false;
    }
  }
  return true;
}

// A wait that ignores the abort flag, for draining one's own copies and MMAs.
__device__ __forceinline__ void tc_drain_wait(unsigned bar, unsigned parity) {
  long long t0 = clock64();
  while (!tc_mbar_try(bar, parity) && clock64() - t0 < TC_TIMEOUT) {
  }
}

// --- operand preparation ----------------------------------------------------

// quantize_rows (kernels.mojo:400-416) of rows [0, T) into the split-int8 A
// tiles, one CTA per row of the padded M (rows >= T are zero). Also writes
// sx[m], the per-segment sums of x (xsum, when non-null) and the plain int16
// rows (xq, when non-null, for the leftover output rows).
__global__ void __launch_bounds__(256) tc_split_rows_kernel(const float *x, int T, int K, int nseg, int seg,
                                                            uint8_t *a, float *sx, int *xsum, int16_t *xq) {
  __shared__ float red[64];
  __shared__ int ssum[TC_MAX_GROUPS * 8];
  const int m = blockIdx.x, nkb = K / TC_KB;
  const bool valid = m < T;
  const float *row = x + (size_t)m * K;
  for (int i = threadIdx.x; i < nseg; i += blockDim.x) ssum[i] = 0;
  float mx = 0.0f;
  if (valid)
    for (int i = threadIdx.x; i < K; i += blockDim.x) mx = fmaxf(mx, fabsf(row[i]));
  mx = block_max(mx, red);
  float s = mx / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  const float inv = 1.0f / s;
  const int mt = m / TC_M, r = m % TC_M;
  for (int ci = threadIdx.x; ci < K / 16; ci += blockDim.x) {
    const int k0 = ci * 16, kb = k0 / TC_KB, chunk = (k0 % TC_KB) / 16;
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    int part = 0;
    if (valid) {
      uint32_t qw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int16_t q = (int16_t)roundf(row[k0 + i] * inv);
        part += q;
        qw[i >> 1] |= (uint32_t)(uint16_t)q << (16 * (i & 1));
        lo[i >> 2] |= (uint32_t)((uint16_t)q & 0xFF) << (8 * (i & 3));
        hi[i >> 2] |= (uint32_t)(((uint16_t)q >> 8) & 0xFF) << (8 * (i & 3));
      }
      if (xq) {
        uint4 *dq = (uint4 *)(xq + (size_t)m * K + k0);
        dq[0] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
        dq[1] = make_uint4(qw[4], qw[5], qw[6], qw[7]);
      }
      if (xsum) atomicAdd(&ssum[k0 / seg], part);
    }
    uint8_t *base = a + ((size_t)mt * nkb + kb) * TC_A_BYTES + ((size_t)chunk * TC_M + r) * 16;
    *(uint4 *)base = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *(uint4 *)(base + TC_A_PLANE) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0) sx[m] = valid ? s : 0.0f;
  if (xsum)
    for (int i = threadIdx.x; i < nseg; i += blockDim.x) xsum[(size_t)m * nseg + i] = ssum[i];
}

// B tiles of a weight: grid (n_tiles, nkb), 256 threads; int4 codes become
// int8 (u - zp), int8 codes stay u8. Rows >= rows are zero.
__global__ void tc_prep_b_kernel(WeightView w, uint8_t *b) {
  const int nt = blockIdx.x, kb = blockIdx.y, nkb = gridDim.y;
  const int gpr = w.cols / w.group;
  uint8_t *dst = b + ((size_t)nt * nkb + kb) * TC_B_BYTES;
  for (int ci = threadIdx.x; ci < 8 * TC_N; ci += blockDim.x) {
    const int chunk = ci / TC_N, r = ci % TC_N, n = nt * TC_N + r, k0 = kb * TC_KB + chunk * 16;
    uint32_t v[4] = {0, 0, 0, 0};
    if (n < w.rows) {
#pragma unroll
      for (int i = 0; i < 16; i++) {
        int code = code_at(w, n, k0 + i);
        int e = w.bits == 4 ? code - (int)w.zp[(size_t)n * gpr + (k0 + i) / w.group] : code;
        v[i >> 2] |= (uint32_t)(e & 0xFF) << (8 * (i & 3));
      }
    }
    *(uint4 *)(dst + ((size_t)chunk * TC_N + r) * 16) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// --- the GEMM -----------------------------------------------------------------

template <bool ZC>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_a16_kernel(TcArgs p) {
  extern __shared__ __align__(128) unsigned char tc_raw[];
  TcSmem &sm = *reinterpret_cast<TcSmem *>(tc_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y, n0 = nt * TC_N, m0 = mt * TC_M;
  const int G = p.w.group, gpr = p.w.cols / G;

  if (threadIdx.x == 0) {
    for (int s = 0; s < TC_STAGES; s++) {
      tc_mbar_init(tc_u32(&sm.full[s]), 1);
      tc_mbar_init(tc_u32(&sm.empty[s]), 1);
    }
    for (int b = 0; b < TC_NBUF; b++) {
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
  } else {
    // this tile's scales (and zero points) as [group][output]
    for (int i = threadIdx.x; i < gpr * TC_N; i += TC_EPI_WARPS * 32) {
      const int g = i / TC_N, c = i % TC_N, n = n0 + c;
      const bool ok = n < p.w.rows;
      sm.scale[g][c] = ok ? half_bits_to_float(p.w.scale[(size_t)n * gpr + g]) : 0.0f;
      sm.zc[g][c] = ok ? p.w.zp[(size_t)n * gpr + g] : 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = sm.tmem;

  if (warp == TC_EPI_WARPS) {
    if (lane == 0) {
      const unsigned idesc_l = tc_idesc(0, ZC ? 0 : 1), idesc_h = tc_idesc(1, ZC ? 0 : 1);
      const uint8_t *ga = p.a + (size_t)mt * p.nkb * TC_A_BYTES;
      const uint8_t *gb = p.b + (size_t)nt * p.nkb * TC_B_BYTES;
      int issued = 0, waited = 0, kstep = 0;
      auto issue = [&](int kb) {
        const int st = kb % TC_STAGES;
        const unsigned dst = tc_u32(sm.stage[st]), bar = tc_u32(&sm.full[st]);
        tc_mbar_expect_tx(bar, TC_STAGE_BYTES);
        tc_bulk_g2s(dst, ga + (size_t)kb * TC_A_BYTES, TC_A_BYTES, bar);
        tc_bulk_g2s(dst + TC_A_BYTES, gb + (size_t)kb * TC_B_BYTES, TC_B_BYTES, bar);
      };
      for (; issued < p.nkb && issued < TC_STAGES; issued++) issue(issued);
      bool ok = true;
      for (int seg = 0; seg < p.nseg && ok; seg++) {
        const int buf = seg % TC_NBUF;
        if (seg >= TC_NBUF)
          ok = tc_wait(sm, tc_u32(&sm.accempty[buf]), ((seg / TC_NBUF) - 1) & 1, p.err, TC_ERR_ACCEMPTY);
        if (!ok) break;
        tc_fence_after();
        const unsigned dl = tmem + buf * 2 * TC_N, dh = dl + TC_N;
        for (int ks = 0; ks < p.seg_ks && ok; ks++, kstep++) {
          const int kb = kstep >> 2, j = kstep & 3, st = kb % TC_STAGES;
          if (j == 0) {
            ok = tc_wait(sm, tc_u32(&sm.full[st]), (kb / TC_STAGES) & 1, p.err, TC_ERR_FULL);
            if (!ok) break;
            waited = kb + 1;
            tc_fence_after();
          }
          const unsigned sa = tc_u32(sm.stage[st]), sb = sa + TC_A_BYTES;
          const unsigned long long db = tc_desc(sb + j * 2 * TC_N * 16, TC_N * 16, 128);
          tc_mma(dl, tc_desc(sa + j * 2 * TC_M * 16, TC_M * 16, 128), db, idesc_l, ks > 0);
          tc_mma(dh, tc_desc(sa + TC_A_PLANE + j * 2 * TC_M * 16, TC_M * 16, 128), db, idesc_h, ks > 0);
          if (j == 3) {
            tc_commit(tc_u32(&sm.empty[st]));
            // refill the stage of the previous k block, whose MMAs were queued
            // ahead of these
            if (kb >= 1 && issued < p.nkb) {
              const int pkb = kb - 1;
              ok = tc_wait(sm, tc_u32(&sm.empty[pkb % TC_STAGES]), (pkb / TC_STAGES) & 1, p.err, TC_ERR_EMPTY);
              if (!ok) break;
              issue(issued++);
            }
          }
        }
        if (ok) tc_commit(tc_u32(&sm.accfull[buf]));
      }
      if (!ok) {
        // drain: copies issued but not yet waited for, then every MMA issued
        for (int kb = waited; kb < issued; kb++)
          tc_drain_wait(tc_u32(&sm.full[kb % TC_STAGES]), (kb / TC_STAGES) & 1);
        tc_commit(tc_u32(&sm.drain));
        tc_drain_wait(tc_u32(&sm.drain), 0);
      }
    }
  } else {
    const int q = warp & 3, hf = warp >> 2;
    const int mrow = m0 + 32 * q + lane;
    float accf[32];
#pragma unroll
    for (int c = 0; c < 32; c++) accf[c] = 0.0f;
    bool ok = true;
    for (int seg = 0; seg < p.nseg; seg++) {
      const int buf = seg % TC_NBUF;
      ok = tc_wait(sm, tc_u32(&sm.accfull[buf]), (seg / TC_NBUF) & 1, p.err, TC_ERR_ACC);
      ok = __all_sync(0xffffffffu, ok);  // the tensor-memory loads below are warp-wide
      if (!ok) break;
      tc_fence_after();
      const unsigned base = tmem + ((unsigned)(32 * q) << 16) + buf * 2 * TC_N + hf * 32;
      int l[32], h[32];
      tc_ld32(base, l);
      tc_ld32(base + TC_N, h);
      tc_ld_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) tc_mbar_arrive(tc_u32(&sm.accempty[buf]));
      const int g = seg * p.seg / G;
      const float *sc = &sm.scale[g][hf * 32];
      const uint8_t *zc = &sm.zc[g][hf * 32];
      const unsigned xs = ZC ? (unsigned)p.xsum[(size_t)mrow * p.nseg + seg] : 0u;
#pragma unroll
      for (int c = 0; c < 32; c++) {
        unsigned a = ((unsigned)h[c] << 8) + (unsigned)l[c];
        if (ZC) a -= (unsigned)zc[c] * xs;
        accf[c] = fmaf((float)(int)a, sc[c], accf[c]);
      }
    }
    if (ok && !*(volatile int *)&sm.abort && mrow < p.T) {
      const float sxm = p.sx[mrow];
      const int nb = n0 + hf * 32;
      float *dst = p.out + (size_t)mrow * p.OUT + nb;
#pragma unroll
      for (int c = 0; c < 32; c++) {
        if (nb + c >= p.n_full) break;
        float r = accf[c] * sxm;
        if (p.epi & EPI_BIAS) r += p.bias[nb + c];
        if (p.epi & EPI_GELU) r = gelu(r);
        if (p.epi & EPI_RESID) r += dst[c];
        dst[c] = r;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == TC_EPI_WARPS) {
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TC_TMEM_COLS));
  }
}

}  // namespace llmq
