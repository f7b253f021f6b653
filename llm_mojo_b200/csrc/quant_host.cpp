// Host-side affine quantizer: QuantMatrix.from_f32 (tensor.mojo:333-383),
// with the int4 packing and BLOCKED decode layout of nibble_at
// (tensor.mojo:385-404). Runs once at load time, split over host threads by
// output row (rows are independent, so the result does not depend on the
// thread count).
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/llmq.h"

namespace {

// float32 -> IEEE binary16 bits, round to nearest even (as Mojo's
// .cast[float16]() converts).
uint16_t f32_to_f16_rne(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0u));
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    int s = 126 - (int)exp;  // value = (2^23 | man) * 2^(exp-150); subnormal unit 2^-24
    if (exp == 0) return (uint16_t)sign;  // float subnormals are far below half's range
    if (s > 25) return (uint16_t)sign;
    uint32_t m24 = 0x800000u | man;
    uint32_t m = m24 >> s, rem = m24 & ((1u << s) - 1u), halfway = 1u << (s - 1);
    if (rem > halfway || (rem == halfway && (m & 1u))) m++;
    return (uint16_t)(sign | m);
  }
  uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
  uint32_t rem = man & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)h;
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
  if (exp == 0x1F) {
    bits = sign | 0x7F800000u | (man << 13);
  } else if (exp == 0) {
    float f = (float)man * 5.9604644775390625e-08f;  // 2^-24
    return sign ? -f : f;
  } else {
    bits = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

inline int clamp_code(int u, int levels) { return u < 0 ? 0 : (u > levels ? levels : u); }

inline void nibble_at(bool blocked, int col, int *byte, bool *high) {
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

}  // namespace

extern "C" llmq_status llmq_quantize_affine(const float *src, int rows, int cols, int reduce_rows, int bits,
                                            int group, int sym, int a16, uint8_t *codes, uint16_t *scale,
                                            uint8_t *zp) {
  if (!src || !codes || !scale || !zp || rows <= 0 || cols <= 0) return LLMQ_ERR_INVALID;
  const int n = reduce_rows ? cols : rows;
  const int k = reduce_rows ? rows : cols;
  const int g = group == 0 ? k : group;
  if ((bits != 4 && bits != 8) || group < 0 || k % g != 0 || g % 32 != 0) return LLMQ_ERR_INVALID;
  const bool blocked = a16 && bits == 4 && group == 32;
  if (blocked && k % 256 != 0) return LLMQ_ERR_INVALID;
  const int gpr = k / g, levels = (1 << bits) - 1, half = 1 << (bits - 1);
  const size_t row_bytes = (size_t)k * bits / 8;
  std::memset(codes, 0, (size_t)n * row_bytes);

  auto work = [&](int r0, int r1) {
    std::vector<float> vals(g);
    for (int r = r0; r < r1; r++) {
      uint8_t *p = codes + (size_t)r * row_bytes;
      for (int gi = 0; gi < gpr; gi++) {
        float lo = 0.0f, hi = 0.0f;  // the range always includes 0
        for (int j = 0; j < g; j++) {
          int c = gi * g + j;
          float v = reduce_rows ? src[(size_t)c * cols + r] : src[(size_t)r * cols + c];
          vals[j] = v;
          lo = std::fmin(lo, v);
          hi = std::fmax(hi, v);
        }
        float s = sym ? std::fmax(-lo, hi) / (float)(half - 1) : (hi - lo) / (float)levels;
        if (s == 0.0f) s = 1.0f;
        uint16_t s16 = f32_to_f16_rne(s);  // quantize against the stored scale
        float sf = f16_to_f32(s16);
        int z = sym ? half : clamp_code((int)std::round(-lo / sf), levels);
        scale[(size_t)r * gpr + gi] = s16;
        zp[(size_t)r * gpr + gi] = (uint8_t)z;
        for (int j = 0; j < g; j++) {
          int u = clamp_code((int)std::round(vals[j] / sf) + z, levels);
          int col = gi * g + j;
          if (bits == 8) {
            p[col] = (uint8_t)u;
          } else {
            int byte;
            bool high;
            nibble_at(blocked, col, &byte, &high);
            p[byte] = high ? (uint8_t)((p[byte] & 0x0F) | (u << 4)) : (uint8_t)((p[byte] & 0xF0) | u);
          }
        }
      }
    }
  };
  unsigned nt = std::thread::hardware_concurrency();
  if (nt == 0) nt = 1;
  if (nt > 32) nt = 32;
  if ((size_t)n * k < (1u << 20)) nt = 1;
  std::vector<std::thread> th;
  for (unsigned i = 0; i < nt; i++) {
    int r0 = (int)((long long)n * i / nt), r1 = (int)((long long)n * (i + 1) / nt);
    th.emplace_back(work, r0, r1);
  }
  for (auto &t : th) t.join();
  return LLMQ_OK;
}
