/*
 * oracle.c -- TEST INFRASTRUCTURE ONLY. A CPU restatement of llm_mojo's
 * quantized-weight matmul hot path, used by tests/, __graft_entry__.smoke()
 * and bench.py's CPU baseline as the checker. Nothing in the llm_mojo_b200
 * package links, loads or calls this file.
 *
 * Every function follows the reference's Mojo code (file:line cited) in its
 * integer arithmetic exactly and in its float32 operation order:
 *   - NW = 16 float lanes (tensor.mojo:26 on AVX-512), lane sums reduced by a
 *     halving tree (SIMD.reduce_add: lanes i and i+8, then i and i+4, ...);
 *   - Mojo `round` is round-half-away-from-zero (roundf);
 *   - float16 scales are IEEE binary16, round to nearest even;
 *   - `.fma` is a fused multiply-add; every other a*b+c is two roundings
 *     (compiled with -ffp-contract=off).
 * The float transcendental functions of the reference (Mojo stdlib exp, tanh)
 * are not in the reference tree; this build defines exp and tanh once
 * (lm_expf, lm_tanhf below: Cody-Waite reduction plus Taylor polynomials,
 * from IEEE add/mul/fma/div only) and uses the same definition on the GPU.
 */
#include <immintrin.h>
#include <math.h>
#include <pthread.h>
#include <sched.h>
#include <stdatomic.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#define OQ_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* float helpers                                                             */
/* ------------------------------------------------------------------------ */

static inline uint16_t f32_to_f16(float f) {
  _Float16 h = (_Float16)f;
  uint16_t u;
  memcpy(&u, &h, 2);
  return u;
}

static inline float f16_to_f32(uint16_t u) {
  _Float16 h;
  memcpy(&h, &u, 2);
  return (float)h;
}

/* SIMD.reduce_add over 16 lanes as a halving tree. */
static inline float tree16(const float *v) {
  float a[8], b[4], c[2];
  for (int i = 0; i < 8; i++) a[i] = v[i] + v[i + 8];
  for (int i = 0; i < 4; i++) b[i] = a[i] + a[i + 4];
  for (int i = 0; i < 2; i++) c[i] = b[i] + b[i + 2];
  return c[0] + c[1];
}

static inline float pow2i(int k) { /* 2^k for -126 <= k <= 127 */
  uint32_t bits = (uint32_t)(k + 127) << 23;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* e^x: k = rint(x log2 e), r = x - k ln2 (Cody-Waite two-part ln2),
 * e^r by its Taylor series through r^7, times 2^k. */
OQ_EXPORT float lm_expf(float x) {
  if (x != x) return x;
  if (x > 88.7228394f) return INFINITY;
  if (x < -103.972084f) return 0.0f;
  float k = rintf(x * 1.44269502f);
  float r = fmaf(-k, 0.693145751953125f, x);
  r = fmaf(-k, 1.42860677e-06f, r);
  float p = (float)(1.0 / 5040.0);
  p = fmaf(p, r, (float)(1.0 / 720.0));
  p = fmaf(p, r, (float)(1.0 / 120.0));
  p = fmaf(p, r, (float)(1.0 / 24.0));
  p = fmaf(p, r, (float)(1.0 / 6.0));
  p = fmaf(p, r, 0.5f);
  p = fmaf(p, r, 1.0f);
  p = fmaf(p, r, 1.0f);
  int ki = (int)k;
  if (ki > 127) return (p * pow2i(127)) * 2.0f;
  if (ki < -125) return (p * pow2i(ki + 24)) * pow2i(-24);
  return p * pow2i(ki);
}

/* tanh: odd Taylor polynomial through a^15 for |a| < 0.5, else
 * 1 - 2 / (e^(2a) + 1); 1 beyond 9. */
OQ_EXPORT float lm_tanhf(float x) {
  float a = fabsf(x);
  float t;
  if (a != a) return x;
  if (a < 0.5f) {
    float z = a * a;
    float p = (float)(-929569.0 / 638512875.0);
    p = fmaf(p, z, (float)(21844.0 / 6081075.0));
    p = fmaf(p, z, (float)(-1382.0 / 155925.0));
    p = fmaf(p, z, (float)(62.0 / 2835.0));
    p = fmaf(p, z, (float)(-17.0 / 315.0));
    p = fmaf(p, z, (float)(2.0 / 15.0));
    p = fmaf(p, z, (float)(-1.0 / 3.0));
    t = fmaf(a * z, p, a);
  } else if (a > 9.0f) {
    t = 1.0f;
  } else {
    float e = lm_expf(2.0f * a);
    t = 1.0f - 2.0f / (e + 1.0f);
  }
  return copysignf(t, x);
}

/* GELU-tanh as store_out / finish write it (kernels.mojo:43-45, :277-279). */
OQ_EXPORT float oq_gelu(float r) {
  const float s = 0.7978845608028654f;
  float inner = r + ((0.044715f * r) * r) * r;
  return (0.5f * r) * (1.0f + lm_tanhf(s * inner));
}

/* finish (kernels.mojo:274-282): optional GELU, residual add, store. */
static inline void finish(float *o, int i, float r, int resid, int gelu) {
  if (gelu) r = oq_gelu(r);
  if (resid) r += o[i];
  o[i] = r;
}

/* ------------------------------------------------------------------------ */
/* Affine quantized matrices (tensor.mojo:230-667)                           */
/* ------------------------------------------------------------------------ */

typedef struct {
  int bits, group, sym, a16, blocked; /* group: weights per group (cols when per-channel) */
  int rows, cols;                     /* stored [rows = OUT, cols = IN] */
  const uint8_t *codes;
  const uint16_t *scale; /* float16 bits, one per group */
  const uint8_t *zp;     /* one per group */
} oq_qmat;

/* nibble_at (tensor.mojo:385-404): byte within the row and high-nibble flag. */
static inline void nibble_at(int blocked, int col, int *byte, int *high) {
  int j, chunk;
  if (blocked) {
    int w = col % 256, e = w % 32, p = e / 2;
    int lane = w / 32 + 8 * (p / 8);
    chunk = (col / 256) * 8 + p % 8;
    j = 2 * lane + e % 2;
  } else {
    chunk = col / 32;
    j = col % 32;
  }
  *byte = chunk * 16 + j % 16;
  *high = j >= 16;
}

static inline int clamp_code(int u, int levels) { return u < 0 ? 0 : (u > levels ? levels : u); }

/* QuantMatrix.from_f32 (tensor.mojo:333-383). src is [rows, cols] row-major;
 * reduce_rows=1 stores the transpose ([cols, rows], layer matrices),
 * reduce_rows=0 stores src as is (wte). group 0 = per channel.
 * codes: n*k*bits/8 bytes, scale/zp: n*(k/group) each. Returns 0 or -1. */
OQ_EXPORT int oq_quant_affine(const float *src, int rows, int cols, int reduce_rows, int bits, int group,
                              int sym, int a16, uint8_t *codes, uint16_t *scale, uint8_t *zp) {
  int n = reduce_rows ? cols : rows;
  int k = reduce_rows ? rows : cols;
  int g = group == 0 ? k : group;
  if ((bits != 4 && bits != 8) || k % g != 0 || g % 32 != 0) return -1;
  int blocked = a16 && bits == 4 && group == 32;
  if (blocked && k % 256 != 0) return -1;
  int gpr = k / g;
  int levels = (1 << bits) - 1, half = 1 << (bits - 1);
  long row_bytes = (long)k * bits / 8;
  memset(codes, 0, (size_t)n * row_bytes);
  float *vals = (float *)malloc(sizeof(float) * g);
  for (int r = 0; r < n; r++) {
    uint8_t *p = codes + (long)r * row_bytes;
    for (int gi = 0; gi < gpr; gi++) {
      float lo = 0.0f, hi = 0.0f;
      for (int j = 0; j < g; j++) {
        int c = gi * g + j;
        float v = reduce_rows ? src[(long)c * cols + r] : src[(long)r * cols + c];
        vals[j] = v;
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
      }
      float s = sym ? fmaxf(-lo, hi) / (float)(half - 1) : (hi - lo) / (float)levels;
      if (s == 0.0f) s = 1.0f;
      uint16_t s16 = f32_to_f16(s);
      float sf = f16_to_f32(s16);
      int z = sym ? half : clamp_code((int)roundf(-lo / sf), levels);
      scale[(long)r * gpr + gi] = s16;
      zp[(long)r * gpr + gi] = (uint8_t)z;
      for (int j = 0; j < g; j++) {
        int u = clamp_code((int)roundf(vals[j] / sf) + z, levels);
        int col = gi * g + j;
        if (bits == 8) {
          p[col] = (uint8_t)u;
        } else {
          int byte, high;
          nibble_at(blocked, col, &byte, &high);
          p[byte] = high ? (uint8_t)((p[byte] & 0x0F) | (u << 4)) : (uint8_t)((p[byte] & 0xF0) | u);
        }
      }
    }
  }
  free(vals);
  return 0;
}

/* QuantMatrix.code (tensor.mojo:419-429). */
static inline int qcode(const oq_qmat *w, int row, int col) {
  const uint8_t *p = w->codes + (long)row * w->cols * w->bits / 8;
  if (w->bits == 8) return p[col];
  int byte, high;
  nibble_at(w->blocked, col, &byte, &high);
  return high ? p[byte] >> 4 : p[byte] & 0xF;
}

/* row_op (tensor.mojo:431-476): dequantize (dot = 0) or the 16 partial sums
 * of a float dot product with x (dot = 1), returned in acc[16]. */
static void row_op(const oq_qmat *w, int row, float *dst, const float *x, int dot, float *acc) {
  int gpr = w->cols / w->group;
  for (int l = 0; l < 16; l++) acc[l] = 0.0f;
  if (w->blocked) { /* scalar path */
    float d = 0.0f;
    for (int k = 0; k < w->cols; k++) {
      int g = row * gpr + k / w->group;
      float v = (float)(qcode(w, row, k) - (int)w->zp[g]) * f16_to_f32(w->scale[g]);
      if (dot)
        d += v * x[k];
      else
        dst[k] = v;
    }
    acc[0] = d;
    return;
  }
  const uint8_t *p = w->codes + (long)row * w->cols * w->bits / 8;
  for (int g = 0; g < gpr; g++) {
    float s = f16_to_f32(w->scale[(long)row * gpr + g]);
    float zp = (float)w->zp[(long)row * gpr + g];
    float accg[16];
    for (int l = 0; l < 16; l++) accg[l] = 0.0f;
    for (int c = 0; c < w->group / 32; c++) {
      int k0 = g * w->group + 32 * c;
      float v0[16], v1[16];
      for (int l = 0; l < 16; l++) {
        if (w->bits == 4) {
          uint8_t b = p[k0 / 2 + l];
          v0[l] = (float)(b & 0xF) - zp;
          v1[l] = (float)(b >> 4) - zp;
        } else {
          v0[l] = (float)p[k0 + l] - zp;
          v1[l] = (float)p[k0 + 16 + l] - zp;
        }
      }
      for (int l = 0; l < 16; l++) {
        if (dot) {
          accg[l] = fmaf(v0[l], x[k0 + l], accg[l]);
          accg[l] = fmaf(v1[l], x[k0 + 16 + l], accg[l]);
        } else {
          dst[k0 + l] = v0[l] * s;
          dst[k0 + 16 + l] = v1[l] * s;
        }
      }
    }
    if (dot)
      for (int l = 0; l < 16; l++) acc[l] = fmaf(accg[l], s, acc[l]);
  }
}

OQ_EXPORT void oq_dequant_row(const oq_qmat *w, int row, float *dst) {
  float acc[16];
  row_op(w, row, dst, dst, 0, acc);
}

/* QuantMatrix.dot_row (tensor.mojo:481-482): W4A32 / W8A32 float dot. */
OQ_EXPORT float oq_dot_row(const oq_qmat *w, int row, const float *x) {
  float acc[16];
  row_op(w, row, NULL, x, 1, acc);
  return tree16(acc);
}

/* ------------------------------------------------------------------------ */
/* Integer (A16) path                                                        */
/* ------------------------------------------------------------------------ */

/* quantize_rows (kernels.mojo:400-416). */
OQ_EXPORT void oq_quantize_rows(const float *x, int T, int IN, int16_t *xq, float *sx) {
  for (int t = 0; t < T; t++) {
    const float *row = x + (long)t * IN;
    float mx = 0.0f;
    for (int i = 0; i < IN; i++) mx = fmaxf(mx, fabsf(row[i]));
    float s = mx / 32767.0f;
    if (s == 0.0f) s = 1.0f;
    sx[t] = s;
    float inv = 1.0f / s;
    for (int i = 0; i < IN; i++) xq[(long)t * IN + i] = (int16_t)roundf(row[i] * inv);
  }
}

/* permute_x_i16 BLOCKED (tensor.mojo:498-516). */
OQ_EXPORT void oq_permute_x_i16(const int16_t *xq, int n, int16_t *dst, float *sums) {
  for (int blk = 0; blk < n / 256; blk++) {
    for (int lane = 0; lane < 16; lane++) sums[blk * 16 + lane] = 0.0f;
    for (int w = 0; w < 256; w++) {
      int col = blk * 256 + w, e = w % 32, p = e / 2;
      int lane = w / 32 + 8 * (p / 8);
      int16_t v = xq[col];
      dst[blk * 256 + (p % 8) * 32 + 2 * lane + e % 2] = v;
      sums[blk * 16 + lane] += (float)v;
    }
  }
}

/* 32 codes of 16-byte step b as int16 ((b & 0xF).join(b >> 4)), or 32 int8
 * codes; dot_pairs (tensor.mojo:34-46) adds lanes i of a[2i]b[2i]+a[2i+1]b[2i+1]. */
static inline void dot_pairs(int32_t *acc, const int16_t *a, const int16_t *b) {
  for (int i = 0; i < 16; i++)
    acc[i] = (int32_t)((uint32_t)acc[i] + (uint32_t)((int32_t)a[2 * i] * b[2 * i]) +
                       (uint32_t)((int32_t)a[2 * i + 1] * b[2 * i + 1]));
}

static inline void codes_i16(const oq_qmat *w, const uint8_t *p, int k0, int zp, int16_t *u) {
  if (w->bits == 4) {
    for (int j = 0; j < 16; j++) {
      u[j] = (int16_t)((p[k0 / 2 + j] & 0xF) - zp);
      u[j + 16] = (int16_t)((p[k0 / 2 + j] >> 4) - zp);
    }
  } else {
    for (int j = 0; j < 32; j++) u[j] = (int16_t)(p[k0 + j] - zp);
  }
}

/* ------------------------------------------------------------------------ */
/* The thread team (team.mojo:36-82): persistent workers meeting at a       */
/* spin-then-yield barrier; work split into contiguous ranges (split).      */
/* Results never depend on the split: every output is computed whole by     */
/* one thread.                                                               */
/* ------------------------------------------------------------------------ */

typedef void (*oq_range_fn)(void *arg, int begin, int end);

static struct {
  int nt;
  pthread_t th[256];
  _Atomic long gen;
  _Atomic int done;
  oq_range_fn fn;
  void *arg;
  int n;
} team;

static void team_wait_gen(long g) {
  int spins = 0;
  while (atomic_load_explicit(&team.gen, memory_order_acquire) == g) {
    if (spins < 1000) {
      _mm_pause();
      spins++;
    } else {
      sched_yield();
    }
  }
}

static void *team_worker(void *p) {
  int tid = (int)(long)p;
  long g = 0;
  for (;;) {
    team_wait_gen(g);
    g = atomic_load_explicit(&team.gen, memory_order_acquire);
    int per = (team.n + team.nt - 1) / team.nt;
    int b = tid * per < team.n ? tid * per : team.n, e = (tid + 1) * per < team.n ? (tid + 1) * per : team.n;
    if (b < e) team.fn(team.arg, b, e);
    atomic_fetch_add_explicit(&team.done, 1, memory_order_acq_rel);
  }
  return NULL;
}

/* Hardware threads per core, from cpu0's sibling list ("0,8" or "0-1"). */
static int threads_per_core(void) {
  FILE *f = fopen("/sys/devices/system/cpu/cpu0/topology/thread_siblings_list", "r");
  if (!f) return 2;
  char buf[64] = {0};
  int n = 1;
  if (fgets(buf, sizeof(buf), f)) {
    int a, b;
    if (sscanf(buf, "%d-%d", &a, &b) == 2)
      n = b - a + 1;
    else
      for (const char *c = buf; *c; c++) n += *c == ',';
  }
  fclose(f);
  return n < 1 ? 1 : n;
}

/* Threads: OQ_THREADS, else one per physical core (gpt2t.mojo:281 takes half
 * the logical CPUs, i.e. one per core on a two-way SMT machine), at most
 * 256. */
OQ_EXPORT int oq_threads(void) {
  if (team.nt) return team.nt;
  const char *env = getenv("OQ_THREADS");
  int n = env ? atoi(env) : (int)(sysconf(_SC_NPROCESSORS_ONLN) / threads_per_core());
  if (n < 1) n = 1;
  if (n > 256) n = 256;
  team.nt = n;
  for (int i = 1; i < n; i++) pthread_create(&team.th[i], NULL, team_worker, (void *)(long)i);
  return n;
}

/* Runs fn over [0, n) split into nt contiguous ranges; thread 0 is the
 * caller. */
static void parallel_for(int n, oq_range_fn fn, void *arg) {
  int nt = oq_threads();
  if (nt == 1 || n < 2) {
    fn(arg, 0, n);
    return;
  }
  team.fn = fn;
  team.arg = arg;
  team.n = n;
  atomic_store_explicit(&team.done, 0, memory_order_release);
  atomic_fetch_add_explicit(&team.gen, 1, memory_order_acq_rel);
  int per = (n + nt - 1) / nt;
  fn(arg, 0, per < n ? per : n);
  int spins = 0;
  while (atomic_load_explicit(&team.done, memory_order_acquire) != nt - 1) {
    if (spins < 1000) {
      _mm_pause();
      spins++;
    } else {
      sched_yield();
    }
  }
}

/* VPDPWSSD (tensor.mojo:34-46 dot_pairs with AVX-512 VNNI): the BLOCKED and
 * per-channel int8 integer dots, selected at run time. */
static int vnni_state = -1;

static int have_vnni(void) {
  if (vnni_state < 0) vnni_state = __builtin_cpu_supports("avx512vnni") && __builtin_cpu_supports("avx512bw") ? 1 : 0;
  return vnni_state;
}

/* Enables (1) or disables (0) the VNNI dots where the CPU has them; returns
 * whether they are in use afterwards. Lets a test compare both paths. */
OQ_EXPORT int oq_set_vnni(int on) {
  vnni_state = -1;
  if (on && have_vnni()) return 1;
  vnni_state = 0;
  return 0;
}

__attribute__((target("avx512f,avx512bw,avx512vnni"))) static void blk4_lanes_vnni(const uint8_t *p, const int16_t *xq,
                                                                                   int nblk, int32_t *lanes) {
  const __m128i mask = _mm_set1_epi8(0x0F);
  for (int blk = 0; blk < nblk; blk++) {
    __m512i acc = _mm512_setzero_si512();
    for (int step = 0; step < 8; step++) {
      __m128i b = _mm_loadu_si128((const __m128i *)(p + blk * 128 + step * 16));
      __m128i lo = _mm_and_si128(b, mask), hi = _mm_and_si128(_mm_srli_epi16(b, 4), mask);
      __m512i u = _mm512_cvtepu8_epi16(_mm256_set_m128i(hi, lo));
      __m512i x = _mm512_loadu_si512((const void *)(xq + blk * 256 + step * 32));
      acc = _mm512_dpwssd_epi32(acc, x, u);
    }
    _mm512_storeu_si512((void *)(lanes + blk * 16), acc);
  }
}

__attribute__((target("avx512f,avx512bw,avx512vnni"))) static void ch8_lanes_vnni(const uint8_t *p, const int16_t *xq,
                                                                                  int cols, int zp, int32_t *lanes) {
  __m512i acc = _mm512_setzero_si512();
  const __m512i z = _mm512_set1_epi16((short)zp);
  for (int k = 0; k < cols; k += 32) {
    __m512i u = _mm512_sub_epi16(_mm512_cvtepu8_epi16(_mm256_loadu_si256((const __m256i *)(p + k))), z);
    acc = _mm512_dpwssd_epi32(acc, _mm512_loadu_si512((const void *)(xq + k)), u);
  }
  _mm512_storeu_si512((void *)lanes, acc);
}

/* dot_row_i16 (tensor.mojo:518-577). If lanes != NULL it also receives the
 * int32 lane sums: BLOCKED [cols/256][16] (before the zero point), otherwise
 * [groups][16]. */
OQ_EXPORT float oq_dot_row_i16_lanes(const oq_qmat *w, int row, const int16_t *xq, const float *xsums,
                                     int32_t *lanes) {
  const uint8_t *p = w->codes + (long)row * w->cols * w->bits / 8;
  int gpr = w->cols / w->group;
  float accf[16];
  for (int l = 0; l < 16; l++) accf[l] = 0.0f;
  if (w->blocked) {
    int32_t vl[12 * 16];
    const int vnni = have_vnni() && w->cols / 256 <= 12;
    if (vnni) blk4_lanes_vnni(p, xq, w->cols / 256, vl);
    for (int blk = 0; blk < w->cols / 256; blk++) {
      int32_t acc[16] = {0};
      if (vnni) {
        memcpy(acc, vl + blk * 16, sizeof(acc));
      } else {
        for (int step = 0; step < 8; step++) {
          const uint8_t *b = p + blk * 128 + step * 16;
          int16_t u[32];
          for (int j = 0; j < 16; j++) {
            u[j] = b[j] & 0xF;
            u[j + 16] = b[j] >> 4;
          }
          dot_pairs(acc, xq + blk * 256 + step * 32, u);
        }
      }
      long g0 = (long)row * gpr + blk * 8;
      for (int l = 0; l < 16; l++) {
        float zp = (float)w->zp[g0 + l % 8];
        float sc = f16_to_f32(w->scale[g0 + l % 8]);
        float xs = xsums[blk * 16 + l];
        accf[l] = fmaf((float)acc[l] - zp * xs, sc, accf[l]);
        if (lanes) lanes[blk * 16 + l] = acc[l];
      }
    }
    return tree16(accf);
  }
  for (int g = 0; g < gpr; g++) {
    int zp = w->zp[(long)row * gpr + g];
    int32_t acc[16] = {0};
    if (w->bits == 8 && gpr == 1 && have_vnni()) {
      ch8_lanes_vnni(p, xq, w->cols, zp, acc);
    } else {
      for (int c = 0; c < w->group / 32; c++) {
        int k0 = g * w->group + 32 * c;
        int16_t u[32];
        codes_i16(w, p, k0, zp, u);
        dot_pairs(acc, xq + k0, u);
      }
    }
    float s = f16_to_f32(w->scale[(long)row * gpr + g]);
    for (int l = 0; l < 16; l++) {
      accf[l] = fmaf((float)acc[l], s, accf[l]);
      if (lanes) lanes[g * 16 + l] = acc[l];
    }
  }
  return tree16(accf);
}

OQ_EXPORT float oq_dot_row_i16(const oq_qmat *w, int row, const int16_t *xq, const float *xsums) {
  return oq_dot_row_i16_lanes(w, row, xq, xsums, NULL);
}

/* unpack_row_i16 (tensor.mojo:579-615): codes minus zero point in natural
 * order, and the group scales as float32. */
OQ_EXPORT void oq_unpack_row_i16(const oq_qmat *w, int row, int16_t *dst, float *scales) {
  int gpr = w->cols / w->group;
  for (int g = 0; g < gpr; g++) {
    int zp = w->zp[(long)row * gpr + g];
    scales[g] = f16_to_f32(w->scale[(long)row * gpr + g]);
    for (int j = 0; j < w->group; j++) {
      int col = g * w->group + j;
      dst[col] = (int16_t)(qcode(w, row, col) - zp);
    }
  }
}

/* dot1_i16 (kernels.mojo:617-628). */
static float dot1_i16(const int16_t *wq, const float *ws, const int16_t *xq, int IN, int G) {
  float accf[16];
  for (int l = 0; l < 16; l++) accf[l] = 0.0f;
  for (int g = 0; g < IN / G; g++) {
    int32_t acc[16] = {0};
    for (int k = g * G; k < (g + 1) * G; k += 32) dot_pairs(acc, xq + k, wq + k);
    for (int l = 0; l < 16; l++) accf[l] = fmaf((float)acc[l], ws[g], accf[l]);
  }
  return tree16(accf);
}

/* Rows [o0, o1) of the one-token path: dot_row_i16 * sx + b, finish. */
static void rows_i16_range(void *arg, int o0, int o1) {
  struct {
    const oq_qmat *w;
    const int16_t *x1;
    const float *xs, *b;
    float *out, s;
    int resid, gelu;
  } *j = arg;
  for (int o = o0; o < o1; o++) {
    float r = oq_dot_row_i16(j->w, o, j->x1, j->xs) * j->s;
    if (j->b) r += j->b[o];
    finish(j->out, o, r, j->resid, j->gelu);
  }
}

/* matmul_rows_a16 (kernels.mojo:419-509) with tile_i16 (:512-573) and
 * rows_i16 (:576-614). b may be NULL (BIAS=False). out[T, OUT]. */
OQ_EXPORT void oq_matmul_rows_a16(float *out, const float *x, const oq_qmat *w, const float *b, int T, int IN,
                                  int OUT, int resid, int gelu) {
  int16_t *xq = (int16_t *)malloc(sizeof(int16_t) * (size_t)T * IN);
  float *sx = (float *)malloc(sizeof(float) * T);
  oq_quantize_rows(x, T, IN, xq, sx);
  if (T == 1) {
    int16_t *xp = (int16_t *)malloc(sizeof(int16_t) * IN);
    float *xs = (float *)malloc(sizeof(float) * (IN / 16 + 1));
    const int16_t *x1 = xq;
    if (w->blocked) {
      oq_permute_x_i16(xq, IN, xp, xs);
      x1 = xp;
    }
    struct {
      const oq_qmat *w;
      const int16_t *x1;
      const float *xs, *b;
      float *out, s;
      int resid, gelu;
    } job = {w, x1, xs, b, out, sx[0], resid, gelu};
    parallel_for(OUT, (oq_range_fn)rows_i16_range, &job);
    free(xp);
    free(xs);
  } else {
    int G = w->group, seg = G < 256 ? G : 256;
    int full = OUT / 32;
    int16_t *wq = (int16_t *)malloc(sizeof(int16_t) * IN);
    float *ws = (float *)malloc(sizeof(float) * (IN / G));
    for (int o = 0; o < OUT; o++) {
      oq_unpack_row_i16(w, o, wq, ws);
      float bias = b ? b[o] : 0.0f;
      for (int t = 0; t < T; t++) {
        const int16_t *xt = xq + (long)t * IN;
        if (o < full * 32) { /* tile_i16: one scalar chain per output */
          float accf = 0.0f;
          for (int k0 = 0; k0 < IN; k0 += seg) {
            uint32_t acc = 0;
            for (int k = k0; k < k0 + seg; k++) acc += (uint32_t)((int32_t)xt[k] * wq[k]);
            accf = fmaf((float)(int32_t)acc, ws[k0 / G], accf);
          }
          float r = accf * sx[t];
          if (b) r += b[o];
          finish(out + (long)t * OUT, o, r, resid, gelu);
        } else { /* rows_i16 / dot1_i16 / dot4_i16 */
          float d = dot1_i16(wq, ws, xt, IN, G);
          finish(out + (long)t * OUT, o, d * sx[t] + bias, resid, gelu);
        }
      }
    }
    free(wq);
    free(ws);
  }
  free(xq);
  free(sx);
}

/* The int32 per-segment sums of the prefill tile path for output o and
 * token t: seg_sums[IN / seg]. Exposes what tile_i16 accumulates. */
OQ_EXPORT void oq_tile_segment_sums(const oq_qmat *w, const int16_t *xq_row, int o, int32_t *seg_sums) {
  int IN = w->cols, G = w->group, seg = G < 256 ? G : 256;
  int16_t *wq = (int16_t *)malloc(sizeof(int16_t) * IN);
  float *ws = (float *)malloc(sizeof(float) * (IN / G));
  oq_unpack_row_i16(w, o, wq, ws);
  for (int k0 = 0; k0 < IN; k0 += seg) {
    uint32_t acc = 0;
    for (int k = k0; k < k0 + seg; k++) acc += (uint32_t)((int32_t)xq_row[k] * wq[k]);
    seg_sums[k0 / seg] = (int32_t)acc;
  }
  free(wq);
  free(ws);
}

/* ------------------------------------------------------------------------ */
/* LayerNorm, KV caches, attention                                           */
/* ------------------------------------------------------------------------ */

/* layernorm (kernels.mojo:179-197). */
OQ_EXPORT void oq_layernorm(float *out, const float *x, const float *w, const float *b, int T, int C) {
  for (int t = 0; t < T; t++) {
    const float *xr = x + (long)t * C;
    float *o = out + (long)t * C;
    float s[16], sq[16];
    for (int l = 0; l < 16; l++) s[l] = sq[l] = 0.0f;
    for (int i = 0; i < C; i += 16)
      for (int l = 0; l < 16; l++) s[l] = s[l] + xr[i + l];
    float mean = tree16(s) / (float)C;
    for (int i = 0; i < C; i += 16)
      for (int l = 0; l < 16; l++) {
        float d = xr[i + l] - mean;
        sq[l] = sq[l] + d * d;
      }
    float rstd = 1.0f / sqrtf(tree16(sq) / (float)C + 1e-5f);
    for (int i = 0; i < C; i++) {
      float n = (xr[i] - mean) * rstd;
      o[i] = n * w[i] + b[i];
    }
  }
}

/* QuantKV[8] (kvcache.mojo:248-385): int8 codes [layer][pos][head][hd] and a
 * float32 scale per (layer, pos, head) for keys and for values. */
typedef struct {
  int n_layer, max_t, n_head, head_dim;
  int8_t *k, *v;
  float *ks, *vs;
} oq_qkv8;

OQ_EXPORT oq_qkv8 *oq_qkv8_new(int n_layer, int max_t, int n_head, int head_dim) {
  oq_qkv8 *c = (oq_qkv8 *)calloc(1, sizeof(oq_qkv8));
  size_t n = (size_t)n_layer * max_t * n_head * head_dim, ns = (size_t)n_layer * max_t * n_head;
  c->n_layer = n_layer;
  c->max_t = max_t;
  c->n_head = n_head;
  c->head_dim = head_dim;
  c->k = (int8_t *)calloc(n, 1);
  c->v = (int8_t *)calloc(n, 1);
  c->ks = (float *)calloc(ns, 4);
  c->vs = (float *)calloc(ns, 4);
  return c;
}

OQ_EXPORT void oq_qkv8_free(oq_qkv8 *c) {
  if (!c) return;
  free(c->k);
  free(c->v);
  free(c->ks);
  free(c->vs);
  free(c);
}

OQ_EXPORT int8_t *oq_qkv8_k(oq_qkv8 *c) { return c->k; }
OQ_EXPORT int8_t *oq_qkv8_v(oq_qkv8 *c) { return c->v; }
OQ_EXPORT float *oq_qkv8_ks(oq_qkv8 *c) { return c->ks; }
OQ_EXPORT float *oq_qkv8_vs(oq_qkv8 *c) { return c->vs; }

/* QuantKV.quantize (kvcache.mojo:319-331) with QMAX = 127. */
static float quantize_i8(const float *x, int n, int8_t *dst) {
  float mx = 0.0f;
  for (int i = 0; i < n; i++) mx = fmaxf(mx, fabsf(x[i]));
  float s = mx / 127.0f;
  if (s == 0.0f) s = 1.0f;
  float inv = 1.0f / s;
  for (int i = 0; i < n; i++) dst[i] = (int8_t)roundf(x[i] * inv);
  return s;
}

OQ_EXPORT void oq_qkv8_store(oq_qkv8 *c, int layer, int pos, const float *k, const float *v) {
  for (int h = 0; h < c->n_head; h++) {
    long sl = ((long)layer * c->max_t + pos) * c->n_head + h;
    c->ks[sl] = quantize_i8(k + h * c->head_dim, c->head_dim, c->k + sl * c->head_dim);
    c->vs[sl] = quantize_i8(v + h * c->head_dim, c->head_dim, c->v + sl * c->head_dim);
  }
}

/* attend_float_one (kvcache.mojo:113-150) through QuantKV.score / add_value
 * (:344-370). out row t ([T, C]), query from qkv row t ([T, 3C]). */
OQ_EXPORT void oq_qkv8_attend_one(const oq_qkv8 *c, float *out, const float *qkv, int layer, int t, int h,
                                  int pos0) {
  int HS = c->head_dim, C = c->n_head * HS;
  float scale = 1.0f / sqrtf((float)HS);
  int npos = pos0 + t + 1;
  const float *q = qkv + (long)t * 3 * C + h * HS;
  float *scores = (float *)malloc(sizeof(float) * npos);
  float mx = -INFINITY; /* Float32.MIN is minus infinity */
  for (int s = 0; s < npos; s++) {
    long sl = ((long)layer * c->max_t + s) * c->n_head + h;
    const int8_t *kp = c->k + sl * HS;
    float d[16];
    for (int l = 0; l < 16; l++) d[l] = 0.0f;
    for (int i = 0; i < HS; i += 16)
      for (int l = 0; l < 16; l++) d[l] = d[l] + q[i + l] * (float)kp[i + l];
    float sc = (tree16(d) * c->ks[sl]) * scale;
    scores[s] = sc;
    mx = fmaxf(mx, sc);
  }
  for (int s = 0; s < npos; s++) scores[s] = lm_expf(scores[s] - mx);
  float total = 0.0f;
  for (int s = 0; s < npos; s++) total += scores[s];
  float *o = out + (long)t * C + h * HS;
  float *acc = (float *)calloc(HS, sizeof(float));
  for (int s = 0; s < npos; s++) {
    long sl = ((long)layer * c->max_t + s) * c->n_head + h;
    const int8_t *vp = c->v + sl * HS;
    float p = scores[s] / total;
    float ps = p * c->vs[sl];
    for (int i = 0; i < HS; i++) acc[i] = fmaf(ps, (float)vp[i], acc[i]);
  }
  for (int i = 0; i < HS; i++) o[i] = acc[i];
  free(acc);
  free(scores);
}

/* ------------------------------------------------------------------------ */
/* Integer softmax (intmath.mojo) and integer attention (int_attention.mojo) */
/* ------------------------------------------------------------------------ */

#define IM_FB 16
#define IM_MB 24
#define IM_MASKED INT32_MIN
#define IM_DCAP (1LL << 31)
#define IM_C0 1073741824LL
#define IM_C1 (-742598100LL)
#define IM_C2 248207216LL
#define IM_C3 (-42480028LL)

/* exp_multiplier (intmath.mojo:48-50). */
OQ_EXPORT int64_t oq_exp_multiplier(double scale) {
  return (int64_t)(scale * 1.4426950408889634 * (double)(1LL << (IM_FB + IM_MB)) + 0.5);
}

/* exp2_neg (intmath.mojo:53-65) for one value. */
static inline int64_t exp2_neg(int64_t d, int64_t mult) {
  int64_t y = ((d < IM_DCAP ? d : IM_DCAP) * mult) >> IM_MB;
  int64_t q = y >> IM_FB;
  int64_t r = y & ((1 << IM_FB) - 1);
  int64_t p = IM_C3;
  p = ((p * r) >> IM_FB) + IM_C2;
  p = ((p * r) >> IM_FB) + IM_C1;
  p = ((p * r) >> IM_FB) + IM_C0;
  return q >= 31 ? 0 : p >> (q < 63 ? q : 63);
}

/* masked_exp (intmath.mojo:93-123): e in Q30, returns the int64 sum. mask
 * may be NULL (HAS_MASK=False). x, mask, e have room for n rounded up to 16. */
OQ_EXPORT int64_t oq_masked_exp(const int32_t *x, const int32_t *mask, int n, int64_t mult, int32_t *e) {
  int nr = (n + 15) / 16 * 16;
  int64_t m = INT64_MIN;
  for (int i = 0; i < nr; i++) {
    int64_t v = x[i];
    int off = i >= n;
    if (mask) {
      off = off || mask[i] == IM_MASKED;
      v += mask[i];
    }
    if (!off && v > m) m = v;
  }
  int64_t total = 0;
  for (int i = 0; i < nr; i++) {
    int64_t v = x[i];
    int off = i >= n;
    if (mask) {
      off = off || mask[i] == IM_MASKED;
      v += mask[i];
    }
    int64_t ev = off ? 0 : exp2_neg(m - v, mult);
    e[i] = (int32_t)ev;
    total += ev;
  }
  return total;
}

/* masked_softmax (intmath.mojo:126-140): Q15 probabilities. */
OQ_EXPORT void oq_masked_softmax(const int32_t *x, const int32_t *mask, int n, int64_t mult, int32_t *e,
                                 uint16_t *probs) {
  int nr = (n + 15) / 16 * 16;
  int64_t t = oq_masked_exp(x, mask, n, mult, e);
  int64_t inv = t > 0 ? (1LL << 61) / t : 0;
  for (int i = 0; i < nr; i++) probs[i] = (uint16_t)(((int64_t)e[i] * inv + (1LL << 45)) >> 46);
}

/* IntAttnKV (int_attention.mojo:62-280). */
#define IA_KS 24
#define IA_SF 16
#define IA_PB 16

typedef struct {
  int n_layer, max_t, n_head, head_dim;
  int8_t *k, *v;
  int32_t *kq, *vq;
} oq_intkv;

OQ_EXPORT oq_intkv *oq_intkv_new(int n_layer, int max_t, int n_head, int head_dim) {
  if (max_t % IA_PB != 0 || head_dim % 32 != 0) return NULL;
  oq_intkv *c = (oq_intkv *)calloc(1, sizeof(oq_intkv));
  size_t n = (size_t)n_layer * n_head * max_t * head_dim, ns = (size_t)n_layer * n_head * max_t;
  c->n_layer = n_layer;
  c->max_t = max_t;
  c->n_head = n_head;
  c->head_dim = head_dim;
  c->k = (int8_t *)calloc(n, 1);
  c->v = (int8_t *)calloc(n, 1);
  c->kq = (int32_t *)calloc(ns, 4);
  c->vq = (int32_t *)calloc(ns, 4);
  return c;
}

OQ_EXPORT void oq_intkv_free(oq_intkv *c) {
  if (!c) return;
  free(c->k);
  free(c->v);
  free(c->kq);
  free(c->vq);
  free(c);
}

OQ_EXPORT int8_t *oq_intkv_k(oq_intkv *c) { return c->k; }
OQ_EXPORT int8_t *oq_intkv_v(oq_intkv *c) { return c->v; }
OQ_EXPORT int32_t *oq_intkv_kq(oq_intkv *c) { return c->kq; }
OQ_EXPORT int32_t *oq_intkv_vq(oq_intkv *c) { return c->vq; }

static inline long ia_lh(const oq_intkv *c, int layer, int head) { return (long)layer * c->n_head + head; }

static inline long ia_k_at(const oq_intkv *c, int layer, int head, int pos, int d) {
  long blk = ia_lh(c, layer, head) * (c->max_t / IA_PB) + pos / IA_PB;
  return ((blk * (c->head_dim / 2) + d / 2) * IA_PB + pos % IA_PB) * 2 + d % 2;
}

static inline long ia_v_at(const oq_intkv *c, int layer, int head, int pos, int d) {
  long pair = ia_lh(c, layer, head) * (c->max_t / 2) + pos / 2;
  return (pair * c->head_dim + d) * 2 + pos % 2;
}

/* quantize_head (int_attention.mojo:140-168). */
static int32_t ia_quantize_head(oq_intkv *c, const float *x, int layer, int h, int pos, int key) {
  float mx = 0.0f;
  for (int d = 0; d < c->head_dim; d++) mx = fmaxf(mx, fabsf(x[d]));
  float s = mx / 127.0f;
  if (s == 0.0f) s = 1.0f;
  float inv = 1.0f / s;
  for (int d = 0; d < c->head_dim; d++) {
    int8_t code = (int8_t)roundf(x[d] * inv);
    if (key)
      c->k[ia_k_at(c, layer, h, pos, d)] = code;
    else
      c->v[ia_v_at(c, layer, h, pos, d)] = code;
  }
  return (int32_t)llround((double)s * (double)(1 << IA_KS));
}

OQ_EXPORT void oq_intkv_store(oq_intkv *c, int layer, int pos, const float *k, const float *v) {
  for (int h = 0; h < c->n_head; h++) {
    long sl = ia_lh(c, layer, h) * c->max_t + pos;
    c->kq[sl] = ia_quantize_head(c, k + h * c->head_dim, layer, h, pos, 1);
    c->vq[sl] = ia_quantize_head(c, v + h * c->head_dim, layer, h, pos, 0);
  }
}

/* attend_one (int_attention.mojo:170-269). */
OQ_EXPORT void oq_intkv_attend_one(const oq_intkv *c, float *out, const float *qkv, int layer, int t, int h,
                                   int pos0) {
  int HS = c->head_dim, C = c->n_head * HS;
  int64_t mult = oq_exp_multiplier(1.0 / (double)(1 << IA_SF));
  int npos = pos0 + t + 1;
  int nr = (npos + IA_PB - 1) / IA_PB * IA_PB;
  const float *q = qkv + (long)t * 3 * C + h * HS;
  int16_t *qi = (int16_t *)malloc(sizeof(int16_t) * HS);
  int32_t *scores = (int32_t *)calloc(nr, 4);
  int32_t *e = (int32_t *)calloc(nr, 4);
  int16_t *w = (int16_t *)calloc(nr + 2, 2);

  float mq = 0.0f;
  for (int d = 0; d < HS; d++) mq = fmaxf(mq, fabsf(q[d]));
  float sq = mq / 32767.0f;
  if (sq == 0.0f) sq = 1.0f;
  float invq = 1.0f / sq;
  for (int d = 0; d < HS; d++) qi[d] = (int16_t)roundf(q[d] * invq);
  int64_t qm = llround((double)sq / sqrt((double)HS) * (double)(1LL << (IA_SF + IA_KS)));

  const int32_t *ks = c->kq + ia_lh(c, layer, h) * c->max_t;
  for (int b = 0; b < nr / IA_PB; b++) {
    for (int p = 0; p < IA_PB; p++) {
      int pos = b * IA_PB + p;
      uint32_t acc = 0;
      for (int d = 0; d < HS; d++) acc += (uint32_t)((int32_t)qi[d] * (int32_t)c->k[ia_k_at(c, layer, h, pos, d)]);
      int64_t t1 = ((int64_t)(int32_t)acc * (int64_t)ks[pos] + (1LL << (IA_KS - 1))) >> IA_KS;
      int64_t sfix = (t1 * qm + (1LL << (IA_KS - 1))) >> IA_KS;
      scores[pos] = (int32_t)sfix;
    }
  }
  int64_t total = oq_masked_exp(scores, NULL, npos, mult, e);

  const int32_t *vs = c->vq + ia_lh(c, layer, h) * c->max_t;
  int64_t vmax = 0;
  for (int s = 0; s < npos; s++)
    if (vs[s] > vmax) vmax = vs[s];
  float *o = out + (long)t * C + h * HS;
  if (vmax == 0 || total == 0) {
    for (int d = 0; d < HS; d++) o[d] = 0.0f;
  } else {
    int64_t inv47 = (1LL << 47) / vmax;
    for (int pos = 0; pos < nr; pos++) {
      /* positions >= npos have e = 0 and weight 0 whatever their scale */
      int64_t ee = e[pos];
      int64_t r16 = pos < npos ? ((int64_t)vs[pos] * inv47) >> 31 : 0;
      int64_t ww = (ee * r16 + (1LL << 30)) >> 31;
      if (ww > 32767) ww = 32767;
      w[pos] = ee == 0 ? 0 : (int16_t)ww;
    }
    w[nr] = 0;
    w[nr + 1] = 0;
    float *accf = (float *)calloc(HS, 4);
    int npairs = (npos + 1) / 2;
    for (int seg = 0; seg < npairs; seg += 128) {
      int32_t *accv = (int32_t *)calloc(HS, 4);
      int end = npairs < seg + 128 ? npairs : seg + 128;
      for (int pp = seg; pp < end; pp++) {
        for (int d = 0; d < HS; d++) {
          int32_t v0 = c->v[ia_v_at(c, layer, h, 2 * pp, d)];
          int32_t v1 = c->v[ia_v_at(c, layer, h, 2 * pp + 1, d)];
          accv[d] = (int32_t)((uint32_t)accv[d] + (uint32_t)(w[2 * pp] * v0) + (uint32_t)(w[2 * pp + 1] * v1));
        }
      }
      for (int d = 0; d < HS; d++) accf[d] += (float)accv[d];
      free(accv);
    }
    float fs = (float)((double)vmax * (double)(1 << 15) / ((double)(1 << IA_KS) * (double)total));
    for (int d = 0; d < HS; d++) o[d] = accf[d] * fs;
    free(accf);
  }
  free(qi);
  free(scores);
  free(e);
  free(w);
}

/* ------------------------------------------------------------------------ */
/* The model step (gpt2t.mojo:198-572) for A16 formats                       */
/* ------------------------------------------------------------------------ */

enum { OQ_QKV = 0, OQ_PROJ = 1, OQ_FC = 2, OQ_FCPROJ = 3 };
enum { OQ_KV_QUANT8 = 0, OQ_KV_INTATTN = 1 };

typedef struct {
  int n_layer, n_head, C, V, max_t, kv_kind;
  oq_qmat mats[4 * 48];
  oq_qmat head; /* tied wte: embedding and output head */
  const float *small;
  const float *wpe, *lnf_w, *lnf_b;
  oq_qkv8 *kv8;
  oq_intkv *ikv;
  float *x, *xn, *qkv, *att, *fc;
} oq_model;

/* Offsets of a layer's vectors in the small-float buffer (gpt2t.mojo:98-119). */
static const float *layer_vec(const oq_model *m, int l, int which) {
  int C = m->C;
  static const int off_mult[8] = {0, 1, 2, 5, 6, 7, 8, 12}; /* ln1w ln1b qkvb projb ln2w ln2b fcb fcprojb */
  return m->small + (long)l * 13 * C + (long)off_mult[which] * C;
}

OQ_EXPORT oq_model *oq_model_new(int n_layer, const oq_qmat *mats, const oq_qmat *head, const float *small,
                                 int kv_kind, int max_t) {
  if (n_layer > 48) return NULL;
  oq_model *m = (oq_model *)calloc(1, sizeof(oq_model));
  m->n_layer = n_layer;
  m->n_head = 12;
  m->C = 768;
  m->V = head->rows;
  m->max_t = max_t;
  m->kv_kind = kv_kind;
  memcpy(m->mats, mats, sizeof(oq_qmat) * 4 * n_layer);
  m->head = *head;
  m->small = small;
  m->wpe = small + (long)n_layer * 13 * m->C;
  m->lnf_w = m->wpe + (long)1024 * m->C;
  m->lnf_b = m->lnf_w + m->C;
  if (kv_kind == OQ_KV_QUANT8)
    m->kv8 = oq_qkv8_new(n_layer, max_t, m->n_head, m->C / m->n_head);
  else
    m->ikv = oq_intkv_new(n_layer, max_t, m->n_head, m->C / m->n_head);
  m->x = (float *)calloc((size_t)max_t * m->C, 4);
  m->xn = (float *)calloc((size_t)max_t * m->C, 4);
  m->qkv = (float *)calloc((size_t)max_t * 3 * m->C, 4);
  m->att = (float *)calloc((size_t)max_t * m->C, 4);
  m->fc = (float *)calloc((size_t)max_t * 4 * m->C, 4);
  return m;
}

OQ_EXPORT void oq_model_free(oq_model *m) {
  if (!m) return;
  oq_qkv8_free(m->kv8);
  oq_intkv_free(m->ikv);
  free(m->x);
  free(m->xn);
  free(m->qkv);
  free(m->att);
  free(m->fc);
  free(m);
}

static void kv_store(oq_model *m, int l, int pos, const float *row) {
  if (m->kv_kind == OQ_KV_QUANT8)
    oq_qkv8_store(m->kv8, l, pos, row + m->C, row + 2 * m->C);
  else
    oq_intkv_store(m->ikv, l, pos, row + m->C, row + 2 * m->C);
}

struct attend_job {
  oq_model *m;
  int l, pos0;
};

/* (t, h) pairs [i0, i1): each writes its own head slice of att. */
static void attend_range(void *arg, int i0, int i1) {
  struct attend_job *j = arg;
  oq_model *m = j->m;
  for (int i = i0; i < i1; i++) {
    int t = i / m->n_head, h = i % m->n_head;
    if (m->kv_kind == OQ_KV_QUANT8)
      oq_qkv8_attend_one(m->kv8, m->att, m->qkv, j->l, t, h, j->pos0);
    else
      oq_intkv_attend_one(m->ikv, m->att, m->qkv, j->l, t, h, j->pos0);
  }
}

/* The (token, head) attention units split over the team, as
 * gpt2t.mojo:395-420 splits heads over threads. */
static void attend(oq_model *m, int l, int T, int pos0) {
  struct attend_job j = {m, l, pos0};
  parallel_for(m->n_head * T, attend_range, &j);
}

/* blocks (gpt2t.mojo:485-571): embeddings of tokens at pos0.., all layers;
 * leaves the result in m->x. With T == 1 this is the arithmetic of decode
 * (gpt2t.mojo:350-447), whose per-thread partitioning does not change any
 * value. */
static void blocks(oq_model *m, const int32_t *tokens, int T, int pos0) {
  int C = m->C;
  for (int t = 0; t < T; t++) {
    float *xt = m->x + (long)t * C;
    const float *p = m->wpe + (long)(pos0 + t) * C;
    oq_dequant_row(&m->head, tokens[t], xt);
    for (int i = 0; i < C; i++) xt[i] = xt[i] + p[i];
  }
  for (int l = 0; l < m->n_layer; l++) {
    const oq_qmat *w = m->mats + 4 * l;
    oq_layernorm(m->xn, m->x, layer_vec(m, l, 0), layer_vec(m, l, 1), T, C);
    oq_matmul_rows_a16(m->qkv, m->xn, &w[OQ_QKV], layer_vec(m, l, 2), T, C, 3 * C, 0, 0);
    for (int t = 0; t < T; t++) kv_store(m, l, pos0 + t, m->qkv + (long)t * 3 * C);
    attend(m, l, T, pos0);
    oq_matmul_rows_a16(m->x, m->att, &w[OQ_PROJ], layer_vec(m, l, 3), T, C, C, 1, 0);
    oq_layernorm(m->xn, m->x, layer_vec(m, l, 4), layer_vec(m, l, 5), T, C);
    oq_matmul_rows_a16(m->fc, m->xn, &w[OQ_FC], layer_vec(m, l, 6), T, C, 4 * C, 0, 1);
    oq_matmul_rows_a16(m->x, m->fc, &w[OQ_FCPROJ], layer_vec(m, l, 7), T, 4 * C, C, 1, 0);
  }
}

/* forward (gpt2t.mojo:329-342): logits[V] of the last token. */
OQ_EXPORT void oq_model_forward(oq_model *m, const int32_t *tokens, int T, int pos0, float *logits) {
  blocks(m, tokens, T, pos0);
  oq_layernorm(m->xn, m->x + (long)(T - 1) * m->C, m->lnf_w, m->lnf_b, 1, m->C);
  oq_matmul_rows_a16(logits, m->xn, &m->head, NULL, 1, m->C, m->V, 0, 0);
}

/* forward_all (gpt2t.mojo:449-459): logits[T, V] for every position. */
OQ_EXPORT void oq_model_forward_all(oq_model *m, const int32_t *tokens, int T, float *logits) {
  blocks(m, tokens, T, 0);
  oq_layernorm(m->xn, m->x, m->lnf_w, m->lnf_b, T, m->C);
  oq_matmul_rows_a16(logits, m->xn, &m->head, NULL, T, m->C, m->V, 0, 0);
}

/* argmax (gpt2t.mojo:792-797): first index of the largest logit. */
OQ_EXPORT int oq_argmax(const float *logits, int V) {
  int best = 0;
  for (int v = 1; v < V; v++)
    if (logits[v] > logits[best]) best = v;
  return best;
}

/* Greedy generation as generate (gpt2t.mojo:942-980) without the stop on
 * EOT: forward the prompt, then `steps` argmaxes with a forward between
 * consecutive ones. out_ids[steps]. */
OQ_EXPORT void oq_generate(oq_model *m, const int32_t *prompt, int n_prompt, int steps, int32_t *out_ids) {
  float *logits = (float *)malloc(sizeof(float) * m->V);
  oq_model_forward(m, prompt, n_prompt, 0, logits);
  int pos = n_prompt;
  for (int i = 0; i < steps; i++) {
    int next = oq_argmax(logits, m->V);
    out_ids[i] = next;
    if (i == steps - 1) break;
    int32_t one = next;
    oq_model_forward(m, &one, 1, pos, logits);
    pos++;
  }
  free(logits);
}

/* Rng (gpt2t.mojo:775-789): xorshift64* seeded with seed * 0x9E3779B97F4A7C15
 * + 1 (wrapping); uniform() takes the top 24 bits of state * 0x2545F4914F6CDD1D. */
OQ_EXPORT uint64_t oq_rng_init(int64_t seed) { return (uint64_t)seed * 0x9E3779B97F4A7C15ull + 1ull; }

OQ_EXPORT float oq_rng_uniform(uint64_t *state) {
  uint64_t s = *state;
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  *state = s;
  return (float)((s * 0x2545F4914F6CDD1Dull) >> 40) / (float)(1 << 24);
}

/* top_k (gpt2t.mojo:800-815): ids of the k largest logits in descending
 * order, kept by insertion into a sorted list (an equal later logit never
 * passes an earlier one). Returns the number written (min(k, V)). */
OQ_EXPORT int oq_top_k(const float *logits, int V, int k, int32_t *ids) {
  int n = 0;
  for (int v = 0; v < V; v++) {
    float lv = logits[v];
    if (n == k && lv <= logits[ids[k - 1]]) continue;
    /* append at slot n (slot k is the one the reference pops again) */
    int pos = n;
    while (pos > 0 && logits[ids[pos - 1]] < lv) {
      if (pos < k) ids[pos] = ids[pos - 1];
      pos--;
    }
    if (pos < k) ids[pos] = v;
    if (n < k) n++;
  }
  return n;
}

/* sample (gpt2t.mojo:818-834): argmax when temperature <= 0 (the state is
 * not advanced); else the top k (k <= 0: all V) with weights
 * exp((logit - max) / temperature), summed in order in float32, and the first
 * candidate at which r = uniform() * total minus the running weights reaches
 * <= 0 (the last candidate if none does). */
OQ_EXPORT int oq_sample(const float *logits, int V, float temperature, int k, uint64_t *state) {
  if (temperature <= 0) return oq_argmax(logits, V);
  int kk = k > 0 ? (k < V ? k : V) : V;
  int32_t *cand = (int32_t *)malloc(sizeof(int32_t) * kk);
  float *p = (float *)malloc(sizeof(float) * kk);
  int n = oq_top_k(logits, V, kk, cand);
  float mx = logits[cand[0]], total = 0.0f;
  for (int i = 0; i < n; i++) {
    p[i] = lm_expf((logits[cand[i]] - mx) / temperature);
    total += p[i];
  }
  float r = oq_rng_uniform(state) * total;
  int pick = cand[n - 1];
  for (int i = 0; i < n; i++) {
    r -= p[i];
    if (r <= 0) {
      pick = cand[i];
      break;
    }
  }
  free(cand);
  free(p);
  return pick;
}

/* generate (gpt2t.mojo:965-980) with sample() in place of argmax, without
 * the stop on EOT; *state is the Rng state, advanced in place. */
OQ_EXPORT void oq_generate_sampled(oq_model *m, const int32_t *prompt, int n_prompt, int steps, float temperature,
                                   int k, uint64_t *state, int32_t *out_ids) {
  float *logits = (float *)malloc(sizeof(float) * m->V);
  oq_model_forward(m, prompt, n_prompt, 0, logits);
  int pos = n_prompt;
  for (int i = 0; i < steps; i++) {
    int next = oq_sample(logits, m->V, temperature, k, state);
    out_ids[i] = next;
    if (i == steps - 1) break;
    int32_t one = next;
    oq_model_forward(m, &one, 1, pos, logits);
    pos++;
  }
  free(logits);
}

/* ------------------------------------------------------------------------ */
/* GGUF block formats (gguf.mojo:139-512)                                    */
/* ------------------------------------------------------------------------ */

enum { GG_F32 = 0, GG_F16 = 1, GG_Q4_0 = 2, GG_Q4_1 = 3, GG_Q8_0 = 8, GG_Q4_K = 12, GG_Q5_K = 13, GG_Q6_K = 14 };

OQ_EXPORT int oq_gguf_block_size(int t) {
  if (t == GG_F32 || t == GG_F16) return 1;
  if (t == GG_Q4_0 || t == GG_Q4_1 || t == GG_Q8_0) return 32;
  return 256;
}

OQ_EXPORT int oq_gguf_block_bytes(int t) {
  switch (t) {
    case GG_F32: return 4;
    case GG_F16: return 2;
    case GG_Q4_0: return 18;
    case GG_Q4_1: return 20;
    case GG_Q8_0: return 34;
    case GG_Q4_K: return 144;
    case GG_Q5_K: return 176;
    case GG_Q6_K: return 210;
  }
  return 0;
}

static inline float f16_at(const uint8_t *p) { return f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* `put` (gguf.mojo:166-175): store v[16] at dst+off, or with dot fold
 * acc[l] = fma(v[l], x[off+l], acc[l]). */
static inline void put(int dot, float *dst, const float *x, float *acc, int off, const float *v) {
  for (int l = 0; l < 16; l++) {
    if (dot)
      acc[l] = fmaf(v[l], x[off + l], acc[l]);
    else
      dst[off + l] = v[l];
  }
}

/* k_scale_min (gguf.mojo:205-221). */
static inline void k_scale_min(const uint8_t *q, int j, int *sc, int *m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

/* One block at b of type t (dequant_q* in gguf.mojo:178-297), dot or store. */
static void gguf_block(int t, const uint8_t *b, float *dst, const float *x, float *acc, int dot) {
  float v[16];
  if (t == GG_Q4_0) {
    float d = f16_at(b);
    const uint8_t *q = b + 2;
    for (int l = 0; l < 16; l++) v[l] = ((float)(q[l] & 0xF) - 8.0f) * d;
    put(dot, dst, x, acc, 0, v);
    for (int l = 0; l < 16; l++) v[l] = ((float)(q[l] >> 4) - 8.0f) * d;
    put(dot, dst, x, acc, 16, v);
  } else if (t == GG_Q4_1) {
    float d = f16_at(b), m = f16_at(b + 2);
    const uint8_t *q = b + 4;
    for (int l = 0; l < 16; l++) v[l] = d * (float)(q[l] & 0xF) + m;
    put(dot, dst, x, acc, 0, v);
    for (int l = 0; l < 16; l++) v[l] = d * (float)(q[l] >> 4) + m;
    put(dot, dst, x, acc, 16, v);
  } else if (t == GG_Q8_0) {
    float d = f16_at(b);
    for (int h = 0; h < 2; h++) {
      for (int l = 0; l < 16; l++) v[l] = d * (float)(int8_t)b[2 + 16 * h + l];
      put(dot, dst, x, acc, 16 * h, v);
    }
  } else if (t == GG_Q4_K || t == GG_Q5_K) {
    float d = f16_at(b), dmin = f16_at(b + 2);
    const uint8_t *scales = b + 4;
    for (int j = 0; j < 4; j++) {
      int sc1, m1i, sc2, m2i;
      k_scale_min(scales, 2 * j, &sc1, &m1i);
      k_scale_min(scales, 2 * j + 1, &sc2, &m2i);
      float d1 = d * (float)sc1, m1 = dmin * (float)m1i;
      float d2 = d * (float)sc2, m2 = dmin * (float)m2i;
      for (int h = 0; h < 2; h++) {
        if (t == GG_Q4_K) {
          const uint8_t *q = b + 16 + 32 * j + 16 * h;
          for (int l = 0; l < 16; l++) v[l] = d1 * (float)(q[l] & 0xF) - m1;
          put(dot, dst, x, acc, 64 * j + 16 * h, v);
          for (int l = 0; l < 16; l++) v[l] = d2 * (float)(q[l] >> 4) - m2;
          put(dot, dst, x, acc, 64 * j + 32 + 16 * h, v);
        } else {
          const uint8_t *qh = b + 16 + 16 * h;
          const uint8_t *q = b + 48 + 32 * j + 16 * h;
          for (int l = 0; l < 16; l++) {
            int lo = (q[l] & 0xF) | (((qh[l] >> (2 * j)) & 1) << 4);
            v[l] = d1 * (float)lo - m1;
          }
          put(dot, dst, x, acc, 64 * j + 16 * h, v);
          for (int l = 0; l < 16; l++) {
            int hi = (q[l] >> 4) | (((qh[l] >> (2 * j + 1)) & 1) << 4);
            v[l] = d2 * (float)hi - m2;
          }
          put(dot, dst, x, acc, 64 * j + 32 + 16 * h, v);
        }
      }
    }
  } else if (t == GG_Q6_K) {
    float d = f16_at(b + 208);
    for (int n = 0; n < 2; n++) {
      int ql = 64 * n, qhoff = 128 + 32 * n, sc = 192 + 8 * n;
      for (int h = 0; h < 2; h++) {
        const uint8_t *lo0 = b + ql + 16 * h, *lo1 = b + ql + 32 + 16 * h, *hi = b + qhoff + 16 * h;
        int base = 128 * n + 16 * h;
        for (int k = 0; k < 4; k++) {
          float s = (float)(int8_t)b[sc + h + 2 * k];
          float ds = d * s;
          for (int l = 0; l < 16; l++) {
            int q;
            if (k == 0) q = (lo0[l] & 0xF) | ((hi[l] & 3) << 4);
            else if (k == 1) q = (lo1[l] & 0xF) | (((hi[l] >> 2) & 3) << 4);
            else if (k == 2) q = (lo0[l] >> 4) | (((hi[l] >> 4) & 3) << 4);
            else q = (lo1[l] >> 4) | (((hi[l] >> 6) & 3) << 4);
            v[l] = ds * ((float)q - 32.0f);
          }
          put(dot, dst, x, acc, base + 32 * k, v);
        }
      }
    }
  }
}

/* GGUFMatrix.each_block (gguf.mojo:388-417) over one row. */
static void gguf_row(int t, const uint8_t *row, int cols, float *dst, const float *x, float *acc, int dot) {
  for (int l = 0; l < 16; l++) acc[l] = 0.0f;
  if (t == GG_F32 || t == GG_F16) {
    float v[16];
    for (int i = 0; i < cols; i += 16) {
      for (int l = 0; l < 16; l++) {
        float w;
        if (t == GG_F32)
          memcpy(&w, row + 4 * (i + l), 4);
        else
          w = f16_at(row + 2 * (i + l));
        v[l] = w;
      }
      put(dot, dst + i, x + i, acc, 0, v);
    }
    return;
  }
  int bs = oq_gguf_block_size(t), bb = oq_gguf_block_bytes(t);
  for (int blk = 0; blk < cols / bs; blk++)
    gguf_block(t, row + (long)blk * bb, dst ? dst + blk * bs : NULL, x ? x + blk * bs : NULL, acc, dot);
}

OQ_EXPORT void oq_gguf_dequant_row(int t, const uint8_t *row, int cols, float *dst) {
  float acc[16];
  gguf_row(t, row, cols, dst, NULL, acc, 0);
}

/* GGUFMatrix.dot_row (gguf.mojo:384-386). */
OQ_EXPORT float oq_gguf_dot_row(int t, const uint8_t *row, int cols, const float *x) {
  float acc[16];
  gguf_row(t, row, cols, NULL, x, acc, 1);
  return tree16(acc);
}

/* Q6_K weights of superblock b as int16 (q - 32) * scale, 32 at a time
 * (q6_k_i16, gguf.mojo:322-336): weights 128n + 32k + j. */
static void q6k_i16(const uint8_t *b, int n, int k, int16_t *out) {
  const uint8_t *L = b + 64 * n + ((k & 1) ? 32 : 0);
  const uint8_t *H = b + 128 + 32 * n;
  for (int j = 0; j < 32; j++) {
    int q = ((k >= 2) ? (L[j] >> 4) : (L[j] & 0xF)) | (((H[j] >> (2 * k)) & 3) << 4);
    int s = (int8_t)b[192 + 8 * n + 2 * k + (j >= 16 ? 1 : 0)];
    out[j] = (int16_t)((q - 32) * s);
  }
}

/* GGUFMatrix.dot_row_i16 (gguf.mojo:462-487) for Q8_0 and Q6_K. */
OQ_EXPORT float oq_gguf_dot_row_i16(int t, const uint8_t *row, int cols, const int16_t *xq) {
  float accf[16];
  for (int l = 0; l < 16; l++) accf[l] = 0.0f;
  if (t == GG_Q8_0) {
    for (int blk = 0; blk < cols / 32; blk++) {
      const uint8_t *b = row + blk * 34;
      int16_t w[32];
      for (int j = 0; j < 32; j++) w[j] = (int8_t)b[2 + j];
      int32_t acc[16] = {0};
      dot_pairs(acc, xq + blk * 32, w);
      float d = f16_at(b);
      for (int l = 0; l < 16; l++) accf[l] = fmaf((float)acc[l], d, accf[l]);
    }
    return tree16(accf);
  }
  for (int sb = 0; sb < cols / 256; sb++) {
    const uint8_t *b = row + sb * 210;
    int32_t acc[16] = {0};
    for (int n = 0; n < 2; n++)
      for (int k = 0; k < 4; k++) {
        int16_t w[32];
        q6k_i16(b, n, k, w);
        dot_pairs(acc, xq + sb * 256 + 128 * n + 32 * k, w);
      }
    float d = f16_at(b + 208);
    for (int l = 0; l < 16; l++) accf[l] = fmaf((float)acc[l], d, accf[l]);
  }
  return tree16(accf);
}

/* head_i16 for one token (kernels.mojo:693-736, T == 1): logits[v] =
 * dot_row_i16(v, xq) * sx. */
OQ_EXPORT void oq_gguf_head_i16(int t, const uint8_t *w, int V, int C, const float *h, float *logits) {
  int16_t *xq = (int16_t *)malloc(sizeof(int16_t) * C);
  float sx;
  oq_quantize_rows(h, 1, C, xq, &sx);
  long rb = (long)(C / oq_gguf_block_size(t)) * oq_gguf_block_bytes(t);
  for (int v = 0; v < V; v++) logits[v] = oq_gguf_dot_row_i16(t, w + v * rb, C, xq) * sx;
  free(xq);
}

/* ------------------------------------------------------------------------ */
/* Dense float formats (tensor.mojo:150-227, kernels.mojo:132-176, 213-227)  */
/* ------------------------------------------------------------------------ */

enum { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

static inline float dense_at(int dt, const void *w, long i) {
  if (dt == DT_F32) return ((const float *)w)[i];
  uint16_t u = ((const uint16_t *)w)[i];
  if (dt == DT_F16) return f16_to_f32(u);
  uint32_t b = (uint32_t)u << 16;
  float f;
  memcpy(&f, &b, 4);
  return f;
}

/* DenseMatrix.dot_row / lm_head (tensor.mojo:206-210, kernels.mojo:213-227):
 * 16 lane fma chains over the row, halving tree. w is [rows, cols]. */
OQ_EXPORT float oq_dense_dot_row(int dt, const void *w, int row, int cols, const float *x) {
  float d[16];
  for (int l = 0; l < 16; l++) d[l] = 0.0f;
  for (int i = 0; i < cols; i += 16)
    for (int l = 0; l < 16; l++) d[l] = fmaf(x[i + l], dense_at(dt, w, (long)row * cols + i + l), d[l]);
  return tree16(d);
}

/* gemv (kernels.mojo:132-176) with `nparts` parts: out[OUT] (+)= act(x[IN]
 * @ w[IN, OUT] + b). Part p accumulates rows [p*rows, min(IN, (p+1)*rows)),
 * rows = ceil(IN / nparts), each output a sequential fma chain; the parts
 * are then added in order after the bias. */
OQ_EXPORT void oq_dense_gemv(int dt, const void *w, const float *x, const float *b, float *out, int IN, int OUT,
                             int nparts, int resid, int gelu) {
  int rows = (IN + nparts - 1) / nparts;
  float *scratch = (float *)calloc((size_t)nparts * OUT, sizeof(float));
  for (int p = 0; p < nparts; p++) {
    float *acc = scratch + (size_t)p * OUT;
    int end = (p + 1) * rows < IN ? (p + 1) * rows : IN;
    for (int i = p * rows; i < end; i++)
      for (int j = 0; j < OUT; j++) acc[j] = fmaf(x[i], dense_at(dt, w, (long)i * OUT + j), acc[j]);
  }
  for (int j = 0; j < OUT; j++) {
    float r = b ? b[j] : 0.0f;
    for (int p = 0; p < nparts; p++) r += scratch[(size_t)p * OUT + j];
    finish(out, j, r, resid, gelu);
  }
  free(scratch);
}

/* ------------------------------------------------------------------------ */
/* Several-token float paths and the perplexity scores                      */
/* ------------------------------------------------------------------------ */

/* matmul for T > 1 (kernels.mojo:96-129) through mm_tile (:51-93): out[T,
 * OUT] (+)= act(x[T, IN] @ w[IN, OUT] + b), each output one fma chain over i. */
OQ_EXPORT void oq_dense_mm(int dt, const void *w, const float *x, const float *b, float *out, int T, int IN, int OUT,
                           int resid, int gelu) {
  for (int t = 0; t < T; t++)
    for (int j = 0; j < OUT; j++) {
      float acc = 0.0f;
      for (int i = 0; i < IN; i++) acc = fmaf(x[(long)t * IN + i], dense_at(dt, w, (long)i * OUT + j), acc);
      if (b) acc += b[j];
      finish(out + (long)t * OUT, j, acc, resid, gelu);
    }
}

/* lm_head_rows (kernels.mojo:230-271): logits[T, V] = h[T, C] @ w[V, C]^T, each
 * the 16-lane dot of lm_head. */
OQ_EXPORT void oq_dense_head_rows(int dt, const void *w, const float *h, float *logits, int T, int V, int C) {
  for (int t = 0; t < T; t++)
    for (int v = 0; v < V; v++) logits[(long)t * V + v] = oq_dense_dot_row(dt, w, v, C, h + (long)t * C);
}

/* matmul_rows for T > 1 (kernels.mojo:325-358) of a GGUF matrix [OUT rows of
 * row_bytes]: rows of 32 outputs dequantized and run through mm_tile's
 * chain; the OUT % 32 leftover rows through rows_dot (:361-397). */
typedef void (*oq_row_dequant)(const void *w, int row, int IN, float *dst);
typedef float (*oq_row_dot)(const void *w, int row, int IN, const float *x);

static void rows_matmul(oq_row_dequant deq, oq_row_dot dot, const void *w, const float *x, const float *b, float *out,
                        int T, int IN, int OUT, int resid, int gelu);

struct gguf_rows {
  int type;
  const uint8_t *rows;
  long row_bytes;
};

static void gguf_row_deq(const void *w, int row, int IN, float *dst) {
  const struct gguf_rows *g = (const struct gguf_rows *)w;
  oq_gguf_dequant_row(g->type, g->rows + (long)row * g->row_bytes, IN, dst);
}

static float gguf_row_dot(const void *w, int row, int IN, const float *x) {
  const struct gguf_rows *g = (const struct gguf_rows *)w;
  return oq_gguf_dot_row(g->type, g->rows + (long)row * g->row_bytes, IN, x);
}

static void affine_row_deq(const void *w, int row, int IN, float *dst) {
  (void)IN;
  oq_dequant_row((const oq_qmat *)w, row, dst);
}

static float affine_row_dot(const void *w, int row, int IN, const float *x) {
  (void)IN;
  return oq_dot_row((const oq_qmat *)w, row, x);
}

OQ_EXPORT void oq_gguf_matmul_rows(int type, const uint8_t *rows, long row_bytes, const float *x, const float *b,
                                   float *out, int T, int IN, int OUT, int resid, int gelu) {
  struct gguf_rows g = {type, rows, row_bytes};
  rows_matmul(gguf_row_deq, gguf_row_dot, &g, x, b, out, T, IN, OUT, resid, gelu);
}

/* matmul_rows for T > 1 (kernels.mojo:325-358) of an affine W4A32 / W8A32
 * QuantMatrix (OUT_MAJOR, not A16): each row dequantized by dequant_row
 * (tensor.mojo:431-479, (u - zp) * scale per value), then the same mm_tile
 * chain and rows_dot leftovers as the GGUF matrices. The output head of such
 * a model for T > 1 (kernels.mojo:677-689 head) is this with no bias. */
OQ_EXPORT void oq_affine_matmul_rows(const oq_qmat *w, const float *x, const float *b, float *out, int T, int IN,
                                     int OUT, int resid, int gelu) {
  rows_matmul(affine_row_deq, affine_row_dot, w, x, b, out, T, IN, OUT, resid, gelu);
}

/* matmul_rows (kernels.mojo:285-358): one token takes each row's dot_row
 * (+ bias); several take the dequantized rows through mm_tile's chain, the
 * OUT % 32 leftover rows through rows_dot. */
static void rows_matmul(oq_row_dequant deq, oq_row_dot dot, const void *w, const float *x, const float *b, float *out,
                        int T, int IN, int OUT, int resid, int gelu) {
  if (T == 1) {
    for (int o = 0; o < OUT; o++) {
      float r = dot(w, o, IN, x);
      if (b) r += b[o];
      finish(out, o, r, resid, gelu);
    }
    return;
  }
  float *wd = (float *)malloc(sizeof(float) * IN);
  int full = OUT / 32 * 32;
  for (int o = 0; o < OUT; o++) {
    deq(w, o, IN, wd);
    for (int t = 0; t < T; t++) {
      const float *xt = x + (long)t * IN;
      float r;
      if (o < full) {
        float acc = 0.0f;
        for (int i = 0; i < IN; i++) acc = fmaf(xt[i], wd[i], acc);
        r = acc;
        if (b) r += b[o];
      } else {
        float d[16];
        for (int l = 0; l < 16; l++) d[l] = 0.0f;
        for (int i = 0; i < IN; i += 16)
          for (int l = 0; l < 16; l++) d[l] = fmaf(xt[i + l], wd[i + l], d[l]);
        r = tree16(d) + (b ? b[o] : 0.0f);
      }
      finish(out + (long)t * OUT, o, r, resid, gelu);
    }
  }
  free(wd);
}

/* DenseKV (kvcache.mojo:153-246) attend_float_one for token t of qkv ([T,
 * 3C]) at position pos0 + t, head h; k and v are [max_t][C] of one layer as
 * float32 (dt 0) or bfloat16 (dt 2) values. */
OQ_EXPORT void oq_dkv_attend_one(int dt, const void *k, const void *v, int n_head, int HS, float *out,
                                 const float *qkv, int t, int h, int pos0) {
  int C = n_head * HS, npos = pos0 + t + 1;
  float scale = 1.0f / sqrtf((float)HS);
  const float *q = qkv + (long)t * 3 * C + h * HS;
  float *sc = (float *)malloc(sizeof(float) * npos);
  float mx = -INFINITY;
  for (int s = 0; s < npos; s++) {
    float d[16];
    for (int l = 0; l < 16; l++) d[l] = 0.0f;
    for (int i = 0; i < HS; i += 16)
      for (int l = 0; l < 16; l++) d[l] = d[l] + q[i + l] * dense_at(dt, k, (long)s * C + h * HS + i + l);
    sc[s] = tree16(d) * scale;
    mx = fmaxf(mx, sc[s]);
  }
  for (int s = 0; s < npos; s++) sc[s] = lm_expf(sc[s] - mx);
  float total = 0.0f;
  for (int s = 0; s < npos; s++) total += sc[s];
  float *o = out + (long)t * C + h * HS;
  for (int i = 0; i < HS; i++) o[i] = 0.0f;
  for (int s = 0; s < npos; s++) {
    float p = sc[s] / total;
    for (int i = 0; i < HS; i++) o[i] = fmaf(p, dense_at(dt, v, (long)s * C + h * HS + i), o[i]);
  }
  free(sc);
}

/* log_sum_exp (gpt2t.mojo:1030-1039). */
static double oq_lse(const float *row, int V) {
  float mx = row[0];
  for (int v = 1; v < V; v++) mx = fmaxf(mx, row[v]);
  double s = 0.0;
  for (int v = 0; v < V; v++) s += (double)lm_expf(row[v] - mx);
  return (double)mx + log(s);
}

/* score_rows (gpt2t.mojo:1042-1097) of rows [r0, r1): stats[k * stride +
 * (r - r0)] for k = NLL, NLL_BASE, AGREE, KL, DIFF_MAX, DIFF_SUM. base may be
 * NULL (the last five are then 0). */
OQ_EXPORT void oq_score_rows(const float *logits, const float *base, const int *targets, int V, int r0, int r1,
                             double *stats, int stride) {
  for (int r = r0; r < r1; r++) {
    const float *lm = logits + (long)r * V;
    double lse = oq_lse(lm, V);
    double vals[6] = {lse - (double)lm[targets[r]], 0, 0, 0, 0, 0};
    if (base) {
      const float *lb = base + (long)r * V;
      double lse_b = oq_lse(lb, V), kl = 0.0, dmax = 0.0, dsum = 0.0;
      int best = 0, best_b = 0;
      for (int v = 0; v < V; v++) {
        double m = lm[v], b = lb[v], lpb = b - lse_b;
        kl += exp(lpb) * (lpb - (m - lse));
        double d = fabs(m - b);
        if (d > dmax) dmax = d;
        dsum += d;
        if (lm[v] > lm[best]) best = v;
        if (lb[v] > lb[best_b]) best_b = v;
      }
      vals[1] = lse_b - (double)lb[targets[r]];
      vals[2] = best == best_b;
      vals[3] = kl;
      vals[4] = dmax;
      vals[5] = dsum;
    }
    for (int k = 0; k < 6; k++) stats[(long)k * stride + (r - r0)] = vals[k];
  }
}
