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
// memory, already in the MMA's K-major 128-byte swizzle layout (rows of one
// 128-byte K block, 8-row atoms with the 16-byte chunks permuted by row, which
// keeps the tensor core's shared-memory reads free of bank conflicts):
//   A (activations, prepared per call by tc_split_rows_kernel):
//     [m_tile][k_block][plane l,h][128 rows x 128 B, swizzled]
//   B (weights, prepared once per weight by tc_prep_b_kernel):
//     [n_tile][k_block][TN rows x 128 B, swizzled], int4 as int8 (u - zp),
//     int8 as its u8 code (zero point applied in the epilogue).
//
// One CTA per 128 x TN output tile (TN 64, or 32 for narrow matrices, so
// that more SMs take part): warp 16 issues the bulk copies and the MMAs (one
// thread), warps 0-15 read the accumulators segment by segment (warp w:
// tensor-memory lanes 32 * (w % 4), TN / 4 columns at (w / 4) * TN / 4),
// loading the next segment while folding this one, while the MMAs of the
// following segments run into rotating accumulator pairs (512 columns).
#pragma once

#include "gemv_a16.cuh"

namespace llmq {

constexpr int TC_M = 128;                                  // tokens per tile (MMA M)
constexpr int TC_KB = 128;                                 // K bytes per pipeline stage
constexpr int TC_STAGES = 4;
constexpr int TC_A_PLANE = TC_M * TC_KB;                   // 16 KB
constexpr int TC_A_BYTES = 2 * TC_A_PLANE;                 // 32 KB, planes l and h
constexpr int TC_NMAX = 64;                                // outputs per tile (MMA N): 64, or 32 for narrow matrices
constexpr int TC_B_MAX = TC_NMAX * TC_KB;                  // 8 KB
constexpr int TC_STAGE_BYTES = TC_A_BYTES + TC_B_MAX;      // 40 KB
constexpr int TC_EPI_WARPS = 16;                           // 4 lane quarters x 4 column groups
constexpr int TC_THREADS = (TC_EPI_WARPS + 1) * 32;        // 544
constexpr int TC_MAX_GROUPS = 96;                          // groups per row in the scale table
constexpr int TC_TMEM_COLS = 512;
constexpr long long TC_TIMEOUT = 4000000000LL;             // cycles a wait may take (~2 s)

enum { TC_ERR_FULL = 1, TC_ERR_EMPTY = 2, TC_ERR_ACC = 3, TC_ERR_ACCEMPTY = 4 };

constexpr int TC_NBUF_MAX = 8;

struct TcSmem {
  alignas(1024) uint8_t stage[TC_STAGES][TC_STAGE_BYTES];
  float scale[TC_MAX_GROUPS][TC_NMAX];
  uint8_t zc[TC_MAX_GROUPS][TC_NMAX];
  alignas(8) unsigned long long full[TC_STAGES], empty[TC_STAGES], accfull[TC_NBUF_MAX], accempty[TC_NBUF_MAX],
      drain;
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
// try_wait with a suspend-time hint: the warp sleeps in hardware until the
// phase completes (or ~0.1 ms pass) instead of spinning on the issue slots
// that the working warps need.
__device__ __forceinline__ bool tc_mbar_try(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n.reg .pred p;\nmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\nselp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(100000u)
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

// Shared-memory matrix descriptor of a K-major operand in the 128-byte
// swizzle layout: rows of 128 bytes (one K block), 8-row atoms of 1024 bytes
// (SBO), the 16-byte chunk c of row r stored at chunk c ^ (r % 8). LBO is
// unused for this layout (1). The start address steps by 32 bytes per MMA K
// step inside the row; the swizzle applies to the final addresses, so atoms
// must be 1024-byte aligned.
__device__ __forceinline__ unsigned long long tc_desc_sw128(unsigned addr) {
  return (unsigned long long)((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}

// Byte offset of the 16-byte chunk c of row r in a 128-byte-swizzled tile.
__host__ __device__ __forceinline__ unsigned tc_sw128_off(int r, int c) {
  return (unsigned)((r >> 3) * 1024 + (r & 7) * 128 + ((c ^ (r & 7)) << 4));
}

// Instruction descriptor of kind::i8: D s32, A/B u8 (0) or s8 (1), both
// K-major, N = n, M = 128.
__host__ __device__ constexpr unsigned tc_idesc(int a_signed, int b_signed, int n) {
  return (2u << 4) | ((unsigned)a_signed << 7) | ((unsigned)b_signed << 10) | ((unsigned)(n >> 3) << 17) |
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

// Tensor-memory loads of 32, 16 or 8 consecutive columns of the warp's 32 lanes
// (asynchronous until tc_ld_wait; tc_ld_done then ties later uses to it).
__device__ __forceinline__ void tc_ld(unsigned addr, int (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(addr));
}
__device__ __forceinline__ void tc_ld(unsigned addr, int (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(addr));
}
__device__ __forceinline__ void tc_ld(unsigned addr, int (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(addr));
}
template <int N>
__device__ __forceinline__ void tc_ld_done(int (&r)[N]) {
#pragma unroll
  for (int i = 0; i < N; i++) asm volatile("" : "+r"(r[i]));
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
    uint8_t *base = a + ((size_t)mt * nkb + kb) * TC_A_BYTES + tc_sw128_off(r, chunk);
    *(uint4 *)base = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *(uint4 *)(base + TC_A_PLANE) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  }
  __syncthreads();
  if (threadIdx.x == 0) sx[m] = valid ? s : 0.0f;
  if (xsum)
    for (int i = threadIdx.x; i < nseg; i += blockDim.x) xsum[(size_t)m * nseg + i] = ssum[i];
}

// B tiles of a weight for an output tile width tn (64 or 32): grid
// (n_tiles, nkb), 256 threads; int4 codes become int8 (u - zp), int8 codes
// stay u8. Rows >= rows are zero.
__global__ void tc_prep_b_kernel(WeightView w, uint8_t *b, int tn) {
  const int nt = blockIdx.x, kb = blockIdx.y, nkb = gridDim.y;
  const int gpr = w.cols / w.group;
  uint8_t *dst = b + ((size_t)nt * nkb + kb) * tn * TC_KB;
  for (int ci = threadIdx.x; ci < 8 * tn; ci += blockDim.x) {
    const int chunk = ci / tn, r = ci % tn, n = nt * tn + r, k0 = kb * TC_KB + chunk * 16;
    uint32_t v[4] = {0, 0, 0, 0};
    if (n < w.rows) {
#pragma unroll
      for (int i = 0; i < 16; i++) {
        int code = code_at(w, n, k0 + i);
        int e = w.bits == 4 ? code - (int)w.zp[(size_t)n * gpr + (k0 + i) / w.group] : code;
        v[i >> 2] |= (uint32_t)(e & 0xFF) << (8 * (i & 3));
      }
    }
    *(uint4 *)(dst + tc_sw128_off(r, chunk)) = make_uint4(v[0], v[1], v[2], v[3]);
  }
}

// --- the GEMM -----------------------------------------------------------------

// Exact float of an int32 |v| < 2^22 without the conversion unit: the bits
// of 1.5 * 2^23 + v, minus 1.5 * 2^23.
__device__ __forceinline__ float tc_small_to_float(int v) { return __int_as_float(0x4B400000 + v) - 12582912.0f; }

// Folds one segment's accumulators into the float chains of CW columns:
// accf = fma(f32(256 * h + l - zp * sum x), s, accf). Without a zero-point
// term (int4 weights, whose |h|, |l| < 2^22 for every segment length) the
// float of 256 * h + l is fma(256, f32(h), f32(l)): both exact, one rounding,
// the same as the conversion of the int32 sum; the conversions then use the
// FMA and ALU pipes instead of the slower conversion unit.
template <bool ZC, int CW>
__device__ __forceinline__ void tc_fold(float (&accf)[CW], const int (&l)[CW], const int (&h)[CW], const float *sc,
                                        const uint8_t *zc, unsigned xs) {
#pragma unroll
  for (int c = 0; c < CW; c++) {
    float v;
    if (ZC) {
      unsigned a = ((unsigned)h[c] << 8) + (unsigned)l[c] - (unsigned)zc[c] * xs;
      v = (float)(int)a;
    } else {
      v = fmaf(256.0f, tc_small_to_float(h[c]), tc_small_to_float(l[c]));
    }
    accf[c] = fmaf(v, sc[c], accf[c]);
  }
}

template <bool ZC, int TN>
__global__ void __launch_bounds__(TC_THREADS, 1) tc_gemm_a16_kernel(TcArgs p) {
  constexpr int NBUF = TC_TMEM_COLS / (2 * TN);  // accumulator pairs in tensor memory
  constexpr int CW = TN / 4;                     // columns per epilogue warp
  constexpr int BBYTES = TN * TC_KB;
  extern __shared__ __align__(128) unsigned char tc_raw[];
  // the swizzle atoms need 1024-byte aligned stages (the launch adds 1 KB)
  TcSmem &sm = *reinterpret_cast<TcSmem *>(tc_raw + ((1024u - (tc_u32(tc_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nt = blockIdx.x, mt = blockIdx.y, n0 = nt * TN, m0 = mt * TC_M;
  const int G = p.w.group, gpr = p.w.cols / G;

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
  } else {
    // this tile's scales (and zero points) as [group][output]
    for (int i = threadIdx.x; i < gpr * TN; i += TC_EPI_WARPS * 32) {
      const int g = i / TN, c = i % TN, n = n0 + c;
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
    // The whole warp runs the loop (waits included) and lane 0 issues the
    // copies, MMAs and commits: tcgen05 issue from a converged warp.
    const bool leader = lane == 0;
    {
      const unsigned idesc_l = tc_idesc(0, ZC ? 0 : 1, TN), idesc_h = tc_idesc(1, ZC ? 0 : 1, TN);
      const unsigned long long desc_a0 = tc_desc_sw128(tc_u32(sm.stage[0]));
      const unsigned long long desc_b0 = tc_desc_sw128(tc_u32(sm.stage[0]) + TC_A_BYTES);
      const uint8_t *ga = p.a + (size_t)mt * p.nkb * TC_A_BYTES;
      const uint8_t *gb = p.b + (size_t)nt * p.nkb * BBYTES;
      int issued = 0, waited = 0, kstep = 0;
      auto issue = [&](int kb) {
        const int st = kb % TC_STAGES;
        const unsigned dst = tc_u32(sm.stage[st]), bar = tc_u32(&sm.full[st]);
        if (leader) {
          tc_mbar_expect_tx(bar, TC_A_BYTES + BBYTES);
          tc_bulk_g2s(dst, ga + (size_t)kb * TC_A_BYTES, TC_A_BYTES, bar);
          tc_bulk_g2s(dst + TC_A_BYTES, gb + (size_t)kb * BBYTES, BBYTES, bar);
        }
        __syncwarp();
      };
      for (; issued < p.nkb && issued < TC_STAGES; issued++) issue(issued);
      bool ok = true;
      for (int seg = 0; seg < p.nseg && ok; seg++) {
        const int buf = seg % NBUF;
        if (seg >= NBUF) ok = tc_wait(sm, tc_u32(&sm.accempty[buf]), ((seg / NBUF) - 1) & 1, p.err, TC_ERR_ACCEMPTY);
        ok = __all_sync(0xffffffffu, ok);
        if (!ok) break;
        tc_fence_after();
        const unsigned dl = tmem + buf * 2 * TN, dh = dl + TN;
        for (int ks = 0; ks < p.seg_ks && ok; ks++, kstep++) {
          const int kb = kstep >> 2, j = kstep & 3, st = kb % TC_STAGES;
          if (j == 0) {
            ok = tc_wait(sm, tc_u32(&sm.full[st]), (kb / TC_STAGES) & 1, p.err, TC_ERR_FULL);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            waited = kb + 1;
            tc_fence_after();
          }
          // descriptors: the stage-0, j-0 ones plus the start-address offset
          const unsigned long long off = (unsigned long long)((st * TC_STAGE_BYTES) >> 4);
          const unsigned long long db = desc_b0 + off + (unsigned long long)(2 * j);
          const unsigned long long da = desc_a0 + off + (unsigned long long)(2 * j);
          if (leader) {
            tc_mma(dl, da, db, idesc_l, ks > 0);
            tc_mma(dh, da + (TC_A_PLANE >> 4), db, idesc_h, ks > 0);
          }
          __syncwarp();
          if (j == 3) {
            if (leader) tc_commit(tc_u32(&sm.empty[st]));
            __syncwarp();
            // refill the stage of the previous k block, whose MMAs were queued
            // ahead of these
            if (kb >= 1 && issued < p.nkb) {
              const int pkb = kb - 1;
              ok = tc_wait(sm, tc_u32(&sm.empty[pkb % TC_STAGES]), (pkb / TC_STAGES) & 1, p.err, TC_ERR_EMPTY);
              ok = __all_sync(0xffffffffu, ok);
              if (!ok) break;
              issue(issued++);
            }
          }
        }
        if (ok && leader) tc_commit(tc_u32(&sm.accfull[buf]));
        __syncwarp();
      }
      if (!ok) {
        // drain: copies issued but not yet waited for, then every MMA issued
        for (int kb = waited; kb < issued; kb++)
          tc_drain_wait(tc_u32(&sm.full[kb % TC_STAGES]), (kb / TC_STAGES) & 1);
        if (leader) tc_commit(tc_u32(&sm.drain));
        __syncwarp();
        tc_drain_wait(tc_u32(&sm.drain), 0);
      }
    }
  } else {
    const int q = warp & 3, cg = warp >> 2;
    const int mrow = m0 + 32 * q + lane;
    const unsigned tbase = tmem + ((unsigned)(32 * q) << 16) + cg * CW;
    float accf[CW];
#pragma unroll
    for (int c = 0; c < CW; c++) accf[c] = 0.0f;
    int la[CW], ha[CW], lb[CW], hb[CW];
    // Waits for segment seg's accumulators and starts loading them.
    auto start = [&](int seg, int (&l)[CW], int (&h)[CW]) -> bool {
      const int buf = seg % NBUF;
      bool ok = tc_wait(sm, tc_u32(&sm.accfull[buf]), (seg / NBUF) & 1, p.err, TC_ERR_ACC);
      ok = __all_sync(0xffffffffu, ok);  // the tensor-memory loads are warp-wide
      if (!ok) return false;
      tc_fence_after();
      tc_ld(tbase + buf * 2 * TN, l);
      tc_ld(tbase + buf * 2 * TN + TN, h);
      return true;
    };
    // Completes the loads and hands the accumulator pair back to the MMAs.
    auto finish = [&](int seg, int (&l)[CW], int (&h)[CW]) {
      tc_ld_wait();
      tc_ld_done(l);
      tc_ld_done(h);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) tc_mbar_arrive(tc_u32(&sm.accempty[seg % NBUF]));
    };
    auto fold = [&](int seg, const int (&l)[CW], const int (&h)[CW]) {
      const int g = seg * p.seg / G;
      const unsigned xs = ZC ? (unsigned)p.xsum[(size_t)mrow * p.nseg + seg] : 0u;
      tc_fold<ZC, CW>(accf, l, h, &sm.scale[g][cg * CW], &sm.zc[g][cg * CW], xs);
    };
    bool ok = start(0, la, ha);
    if (ok) finish(0, la, ha);
    // two segments per trip: fold one while the next one's loads are in flight
    for (int seg = 0; ok && seg < p.nseg; seg += 2) {
      if (seg + 1 < p.nseg) ok = start(seg + 1, lb, hb);
      fold(seg, la, ha);
      if (!ok || seg + 1 >= p.nseg) break;
      finish(seg + 1, lb, hb);
      if (seg + 2 < p.nseg) ok = start(seg + 2, la, ha);
      fold(seg + 1, lb, hb);
      if (ok && seg + 2 < p.nseg) finish(seg + 2, la, ha);
    }
    if (ok && !*(volatile int *)&sm.abort && mrow < p.T) {
      const float sxm = p.sx[mrow];
      const int nb = n0 + cg * CW;
      float *dst = p.out + (size_t)mrow * p.OUT + nb;
#pragma unroll
      for (int c = 0; c < CW; c++) {
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


// --- the transposed GEMM: weights as A, both activation planes as one B -----
//
// The weight rows are the MMA's M (128 per tile), the tokens its N: B holds
// the tile's TT tokens twice, as the low plane xl' = xl - 128 and the high
// plane xh, both signed bytes (x = 256 xh + xl' + 128), so ONE kind::i8 MMA
// per 32-element K step gives both planes' sums: D[n][t] (low) and
// D[n][TT + t] (high). The segment sum is 256 D_h + D_l + 128 W (W: the
// segment's sum of the weight values, u - zp for int4, u for int8), minus
// zp * sum(x) for int8, all modulo 2^32 like the reference's int32
// accumulator; the float folds keep the reference's order: bit-identical.
//
// Shared memory: 4 stages of [A: 128 rows x 128 B][B: 2 TT rows x 128 B],
// both in the 128-byte swizzle layout. Warp 16 issues copies, MMAs and
// commits; warps 0-15 fold (warp w: tensor-memory lanes = weight rows
// 32 * (w % 4) + lane, tokens (w / 4) * TT / 4 .. + TT / 4).

constexpr int TCT_A_BYTES = TC_M * TC_KB;  // 16 KB of weight rows per K block

template <int TT>
struct TcSmemT {
  alignas(1024) uint8_t stage[TC_STAGES][TCT_A_BYTES + 2 * TT * TC_KB];
  alignas(8) unsigned long long full[TC_STAGES], empty[TC_STAGES], accfull[TC_NBUF_MAX], accempty[TC_NBUF_MAX],
      drain;
  unsigned tmem;
  int abort;
};

// The bounded wait of tc_wait on a given abort flag.
__device__ __forceinline__ bool tc_wait_flag(int *abort, unsigned bar, unsigned parity, int *err, int code) {
  long long t0 = clock64();
  while (!tc_mbar_try(bar, parity)) {
    if (*(volatile int *)abort) return false;
    if (clock64() - t0 > TC_TIMEOUT) {
      *(volatile int *)abort = 1;
      atomicExch(err, code);
      return false;
    }
  }
  return true;
}

// quantize_rows of rows [0, T) into the transposed B tiles
// [t_tile][kb][plane l' (TT rows), plane h (TT rows)], sx[m], the
// per-segment sums of x (xsum, when non-null) and the plain int16 rows (xq,
// when non-null). One warp per row of the padded token count t_pad (8 per
// CTA; the max of |x| is exact in any order, the codes and segment sums are
// integers); rows >= T hold codes 0 (their outputs are not stored).
template <int TT>
__global__ void __launch_bounds__(256) tct_split_rows_kernel(const float *x, int T, int t_pad, int K, int nseg,
                                                             int seg, uint8_t *b, float *sx, int *xsum, int16_t *xq) {
  __shared__ int ssum[8][TC_MAX_GROUPS * 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m = blockIdx.x * 8 + warp, nkb = K / TC_KB;
  if (m >= t_pad) return;
  const bool valid = m < T;
  const float *row = x + (size_t)m * K;
  const bool vec = ((uintptr_t)row & 15) == 0;
  int *ss = ssum[warp];
  if (xsum)
    for (int i = lane; i < nseg; i += 32) ss[i] = 0;
  __syncwarp();
  float mx = 0.0f;
  if (valid)
    for (int i = lane; i < K; i += 32) mx = fmaxf(mx, fabsf(row[i]));
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float s = mx / 32767.0f;
  if (s == 0.0f) s = 1.0f;
  const float inv = 1.0f / s;
  const int tt = m / TT, r = m % TT;
  for (int ci = lane; ci < K / 16; ci += 32) {
    const int k0 = ci * 16, kb = k0 / TC_KB, chunk = (k0 % TC_KB) / 16;
    uint32_t lo[4] = {0, 0, 0, 0}, hi[4] = {0, 0, 0, 0};
    int part = 0;
    if (valid) {
      float v[16];
      if (vec) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
          const float4 f = *(const float4 *)(row + k0 + 4 * j);
          v[4 * j] = f.x;
          v[4 * j + 1] = f.y;
          v[4 * j + 2] = f.z;
          v[4 * j + 3] = f.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; i++) v[i] = row[k0 + i];
      }
      uint32_t qw[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
      for (int i = 0; i < 16; i++) {
        const int16_t q = (int16_t)roundf(v[i] * inv);
        part += q;
        qw[i >> 1] |= (uint32_t)(uint16_t)q << (16 * (i & 1));
        lo[i >> 2] |= (uint32_t)(((uint16_t)q & 0xFF) ^ 0x80) << (8 * (i & 3));  // xl - 128
        hi[i >> 2] |= (uint32_t)(((uint16_t)q >> 8) & 0xFF) << (8 * (i & 3));
      }
      if (xq) {
        uint4 *dq = (uint4 *)(xq + (size_t)m * K + k0);
        dq[0] = make_uint4(qw[0], qw[1], qw[2], qw[3]);
        dq[1] = make_uint4(qw[4], qw[5], qw[6], qw[7]);
      }
      if (xsum) atomicAdd(&ss[k0 / seg], part);
    }
    uint8_t *base = b + ((size_t)tt * nkb + kb) * (2 * TT * TC_KB) + tc_sw128_off(r, chunk);
    *(uint4 *)base = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    *(uint4 *)(base + TT * TC_KB) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  }
  __syncwarp();
  if (lane == 0) sx[m] = valid ? s : 0.0f;
  if (xsum)
    for (int i = lane; i < nseg; i += 32) xsum[(size_t)m * nseg + i] = ss[i];
}

// W[n][s]: the sum over segment s of row n's weight values (u - zp for int4,
// the u8 code for int8). One thread per (row, segment).
__global__ void tct_wsum_kernel(WeightView w, int seg, int nseg, int *wsum) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= w.rows * nseg) return;
  const int n = i / nseg, sg = i % nseg, gpr = w.cols / w.group;
  int t = 0;
  for (int k = sg * seg; k < (sg + 1) * seg; k++) {
    const int code = code_at(w, n, k);
    t += w.bits == 4 ? code - (int)w.zp[(size_t)n * gpr + k / w.group] : code;
  }
  wsum[i] = t;
}

struct TcArgsT {
  const uint8_t *a;   // weight tiles [n_tile][kb][128 rows x 128 B] (tc_prep_b_kernel, 128 rows)
  const uint8_t *b;   // activation tiles [t_tile][kb][2 TT rows x 128 B]
  const float *sx;    // [t_pad]
  const int *xsum;    // [t_pad][nseg] (int8 weights)
  const int *wsum;    // [rows][nseg]
  WeightView w;
  const float *bias;
  float *out;
  int *err;
  int T, OUT, n_full, K, nkb, nseg, seg_ks, seg, epi;
};

template <bool ZC, int TT>
__global__ void __launch_bounds__(TC_THREADS, 1) tct_gemm_kernel(TcArgsT p) {
  constexpr int NBUF = TC_TMEM_COLS / (2 * TT);  // accumulators of 2 TT columns in tensor memory
  constexpr int CW = TT / 4;                     // tokens per epilogue warp
  constexpr int BB = 2 * TT * TC_KB;             // activation bytes per K block
  constexpr int STAGE = TCT_A_BYTES + BB;
  static_assert(CW == 16 || CW == 8, "tc_ld widths");
  extern __shared__ __align__(128) unsigned char tc_raw[];
  TcSmemT<TT> &sm = *reinterpret_cast<TcSmemT<TT> *>(tc_raw + ((1024u - (tc_u32(tc_raw) & 1023u)) & 1023u));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // persistent over token tiles: CTA (nt, c) takes token tiles c, c + gridDim.y, ...;
  // the copy pipeline and the accumulator rotation run on across them
  const int nt = blockIdx.x, n0 = nt * TC_M;
  const int ttiles = (p.T + TT - 1) / TT;
  const int iters = (int)blockIdx.y < ttiles ? (ttiles - 1 - (int)blockIdx.y) / (int)gridDim.y + 1 : 0;
  const int G = p.w.group, gpr = p.w.cols / G;

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
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const unsigned tmem = sm.tmem;

  if (warp == TC_EPI_WARPS) {
    // the whole warp runs the loop (waits included); lane 0 issues the
    // copies, MMAs and commits. K blocks and segments are counted across
    // the CTA's token tiles: K block kg = it * nkb + kb, segment sg.
    const bool leader = lane == 0;
    const unsigned idesc = tc_idesc(ZC ? 0 : 1, 1, 2 * TT);
    const unsigned long long desc_a0 = tc_desc_sw128(tc_u32(sm.stage[0]));
    const unsigned long long desc_b0 = tc_desc_sw128(tc_u32(sm.stage[0]) + TCT_A_BYTES);
    const uint8_t *ga = p.a + (size_t)nt * p.nkb * TCT_A_BYTES;
    const int nkg = iters * p.nkb, nsg = iters * p.nseg;
    int issued = 0, waited = 0, kstep = 0;
    auto issue = [&](int kg) {
      const int st = kg % TC_STAGES, it = kg / p.nkb, kb = kg - it * p.nkb;
      const int tt = blockIdx.y + it * gridDim.y;
      const unsigned dst = tc_u32(sm.stage[st]), bar = tc_u32(&sm.full[st]);
      if (leader) {
        tc_mbar_expect_tx(bar, STAGE);
        tc_bulk_g2s(dst, ga + (size_t)kb * TCT_A_BYTES, TCT_A_BYTES, bar);
        tc_bulk_g2s(dst + TCT_A_BYTES, p.b + ((size_t)tt * p.nkb + kb) * BB, BB, bar);
      }
      __syncwarp();
    };
    for (; issued < nkg && issued < TC_STAGES; issued++) issue(issued);
    bool ok = true;
    for (int sg = 0; sg < nsg && ok; sg++) {
      const int buf = sg % NBUF;
      if (sg >= NBUF)
        ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accempty[buf]), ((sg / NBUF) - 1) & 1, p.err, TC_ERR_ACCEMPTY);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const unsigned d = tmem + buf * 2 * TT;
      for (int ks = 0; ks < p.seg_ks && ok; ks++, kstep++) {
        const int kg = kstep >> 2, j = kstep & 3, st = kg % TC_STAGES;
        if (j == 0) {
          ok = tc_wait_flag(&sm.abort, tc_u32(&sm.full[st]), (kg / TC_STAGES) & 1, p.err, TC_ERR_FULL);
          ok = __all_sync(0xffffffffu, ok);
          if (!ok) break;
          waited = kg + 1;
          tc_fence_after();
        }
        const unsigned long long off = (unsigned long long)((st * STAGE) >> 4);
        if (leader) tc_mma(d, desc_a0 + off + (unsigned long long)(2 * j), desc_b0 + off + (unsigned long long)(2 * j),
                           idesc, ks > 0);
        __syncwarp();
        if (j == 3) {
          if (leader) tc_commit(tc_u32(&sm.empty[st]));
          __syncwarp();
          // refill the stage of the previous K block, whose MMA was queued
          // ahead of these
          if (kg >= 1 && issued < nkg) {
            const int pkg = kg - 1;
            ok = tc_wait_flag(&sm.abort, tc_u32(&sm.empty[pkg % TC_STAGES]), (pkg / TC_STAGES) & 1, p.err,
                              TC_ERR_EMPTY);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) break;
            issue(issued++);
          }
        }
      }
      if (ok && leader) tc_commit(tc_u32(&sm.accfull[buf]));
      __syncwarp();
    }
    if (!ok) {
      // drain: copies issued but not yet waited for, then every MMA issued
      for (int kg = waited; kg < issued; kg++) tc_drain_wait(tc_u32(&sm.full[kg % TC_STAGES]), (kg / TC_STAGES) & 1);
      if (leader) tc_commit(tc_u32(&sm.drain));
      __syncwarp();
      tc_drain_wait(tc_u32(&sm.drain), 0);
    }
  } else {
    const int q = warp & 3, cg = warp >> 2;
    const int n = n0 + 32 * q + lane;            // this thread's weight row
    const int nr = n < p.w.rows ? n : p.w.rows - 1;
    const unsigned tbase = tmem + ((unsigned)(32 * q) << 16) + cg * CW;
    const int nseg = p.nseg, nsg = iters * nseg;
    float accf[CW];
#pragma unroll
    for (int c = 0; c < CW; c++) accf[c] = 0.0f;
    // one segment's loads in flight (l, h) while the previous one, already
    // converted to its CW floats v, folds into the chains
    int l[CW], h[CW];
    float v[CW];
    unsigned short sc_nxt = 0;  // the next segment's scale, weight sum and zero point,
    int ws_nxt = 0, zp_nxt = 0;  // loaded with its accumulators
    float sc_cur = 0.0f;
    int seg_l = 0, it_l = 0;  // the loads' (segment, token-tile iteration); the fold's below
    auto start = [&](int sg) -> bool {
      const int buf = sg % NBUF;
      bool ok = tc_wait_flag(&sm.abort, tc_u32(&sm.accfull[buf]), (sg / NBUF) & 1, p.err, TC_ERR_ACC);
      ok = __all_sync(0xffffffffu, ok);  // the tensor-memory loads are warp-wide
      if (!ok) return false;
      tc_fence_after();
      tc_ld(tbase + buf * 2 * TT, l);
      tc_ld(tbase + buf * 2 * TT + TT, h);
      const int g = seg_l * p.seg / G;
      sc_nxt = p.w.scale[(size_t)nr * gpr + g];
      ws_nxt = p.wsum[(size_t)nr * nseg + seg_l];
      if (ZC) zp_nxt = p.w.zp[(size_t)nr * gpr + g];
      return true;
    };
    // completes the loads, hands the accumulators back to the MMAs and
    // converts the segment's sums: f32(256 h + l + 128 W - zp sum(x))
    auto finish = [&](int sg) {
      tc_ld_wait();
      tc_ld_done(l);
      tc_ld_done(h);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) tc_mbar_arrive(tc_u32(&sm.accempty[sg % NBUF]));
      const int w128 = ws_nxt * 128;
      const int t0 = (blockIdx.y + it_l * gridDim.y) * TT + cg * CW;
#pragma unroll
      for (int c = 0; c < CW; c++) {
        if (ZC) {
          const unsigned xs = (unsigned)p.xsum[(size_t)(t0 + c) * nseg + seg_l];
          const unsigned a = ((unsigned)h[c] << 8) + (unsigned)l[c] + (unsigned)w128 - (unsigned)zp_nxt * xs;
          v[c] = (float)(int)a;
        } else {
          // |h|, |l + 128 W| < 2^22 for int4 weights: both exact as floats,
          // one rounding in the fma, as the conversion of the int32 sum
          v[c] = fmaf(256.0f, tc_small_to_float(h[c]), tc_small_to_float(l[c] + w128));
        }
      }
      sc_cur = half_bits_to_float(sc_nxt);
      if (++seg_l == nseg) {
        seg_l = 0;
        ++it_l;
      }
    };
    // the outputs of token tile it (its last segment folded)
    auto emit = [&](int it) {
      if (n >= p.n_full) return;
      const float bn = (p.epi & EPI_BIAS) ? p.bias[n] : 0.0f;
      const int t0 = (blockIdx.y + it * gridDim.y) * TT + cg * CW;
#pragma unroll
      for (int c = 0; c < CW; c++) {
        const int m = t0 + c;
        if (m >= p.T) break;
        float *dst = p.out + (size_t)m * p.OUT + n;
        float r = accf[c] * p.sx[m];
        if (p.epi & EPI_BIAS) r += bn;
        if (p.epi & EPI_GELU) r = gelu(r);
        if (p.epi & EPI_RESID) r += *dst;
        *dst = r;
      }
    };
    bool ok = nsg > 0 && start(0);
    if (ok) finish(0);
    int seg_f = 0, it_f = 0;  // the fold's segment and token-tile iteration
    for (int sg = 0; ok && sg < nsg; sg++) {
      const bool more = sg + 1 < nsg;
      if (more) ok = start(sg + 1);
#pragma unroll
      for (int c = 0; c < CW; c++) accf[c] = fmaf(v[c], sc_cur, accf[c]);
      if (++seg_f == nseg) {
        if (!*(volatile int *)&sm.abort) emit(it_f);
#pragma unroll
        for (int c = 0; c < CW; c++) accf[c] = 0.0f;
        seg_f = 0;
        ++it_f;
      }
      if (!ok || !more) break;
      finish(sg + 1);
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
