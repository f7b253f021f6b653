// sample.cuh -- top-k / temperature sampling on the device (gpt2t.mojo:775-834).
//
// The reference keeps the k largest logits in descending order (an equal
// later logit never passes an earlier one), weights them by
// exp((logit - max) / temperature), sums the weights in that order in
// float32, draws r = uniform() * total from a xorshift64* state and walks the
// list subtracting weights until r <= 0.
//
// Here every logit becomes one 64-bit key, (descending order of the value)
// << 32 | id, so the ascending order of the keys is the reference's order of
// candidates and all keys differ. Sorting is a bitonic network: chunks of
// kSortChunk keys sort in shared memory, the levels above a chunk take one
// global compare-exchange launch per stride plus a shared-memory pass for the
// strides inside a chunk.
//   k <= kTopkSmall and (chunks x k) <= kMergeCap: topk_fast_kernel (one CTA:
//     a threshold from per-thread maxima, the logits above it sorted); when
//     too many logits tie at the threshold, every chunk keeps its first k
//     keys and one CTA sorts those candidates and draws (two more launches,
//     which return at once when the first kernel succeeded);
//   otherwise: the whole padded key array is sorted, one CTA draws.
// The draw is one thread: the float32 sum and the subtraction walk are
// sequential chains in the reference's order (the weights are computed by the
// whole CTA first).
#pragma once

#include "common.cuh"

namespace llmq {

constexpr int kSortChunk = 4096;    // keys one CTA sorts in shared memory (32 KB)
constexpr int kSortThreads = 1024;
constexpr int kTopkSmall = 1024;    // largest k of the two-launch path
constexpr int kMergeCap = 16384;    // candidates the merging CTA sorts (128 KB)

typedef unsigned long long u64;

// Where a drawn id goes: *id, *id2, and with a decode state ids[step - 1] and
// the state's next token (the head's fused argmax already advanced step).
struct SampleOut {
  int *id;
  int *id2;
  int *state_token;
  const int *state_step;
  int *ids;
};

__device__ __forceinline__ u64 sample_key(float v, int id) {
  unsigned u = __float_as_uint(v);
  if ((u & 0x7fffffffu) == 0) u = 0;  // -0 and +0 compare equal in the reference
  const unsigned asc = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((u64)(~asc) << 32) | (unsigned)id;
}

__device__ __forceinline__ int key_id(u64 k) { return (int)(unsigned)(k & 0xffffffffull); }

// Bitonic levels s = s_lo, 2 s_lo, ..., s_hi over the n keys in shared memory
// whose first key has global index base; strides from min(s, n) / 2 down to 1.
// Direction of a pair: ascending when (global index & s) == 0; with all_asc
// every level s >= n sorts ascending (each chunk sorted on its own).
__device__ void bitonic_levels(u64 *k, int n, int base, int s_lo, int s_hi, bool all_asc) {
  for (int s = s_lo; s <= s_hi; s <<= 1) {
    for (int j = min(s, n) >> 1; j > 0; j >>= 1) {
      for (int p = threadIdx.x; p < n / 2; p += blockDim.x) {
        const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1)), l = i + j;
        const bool asc = (((base + i) & s) == 0) || (all_asc && s >= n);
        const u64 a = k[i], b = k[l];
        if ((a > b) == asc) {
          k[i] = b;
          k[l] = a;
        }
      }
      __syncthreads();
    }
  }
}

// Ascending bitonic sort of 64 keys held by one warp, key lane + 32 h in
// a[h]: strides below 32 pair lanes (shuffles), stride 32 pairs a[0] with
// a[1] in the same lane.
__device__ __forceinline__ void warp_sort64(u64 a[2]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 2; s <= 64; s <<= 1) {
#pragma unroll
    for (int j = s >> 1; j > 0; j >>= 1) {
      if (j == 32) {
        // e = lane vs lane + 32; level s = 64 is ascending
        const u64 lo = min(a[0], a[1]), hi = max(a[0], a[1]);
        a[0] = lo;
        a[1] = hi;
      } else {
#pragma unroll
        for (int h = 0; h < 2; h++) {
          const int e = lane + 32 * h;
          const u64 o = __shfl_xor_sync(0xffffffffu, a[h], j);
          const bool lower = (e & j) == 0, asc = (e & s) == 0;
          a[h] = (lower == asc) ? min(a[h], o) : max(a[h], o);
        }
      }
    }
  }
}

// One chunk of kSortChunk keys: built from the logits (logits != nullptr,
// keys past V are all ones) or read from keys; levels [s_lo, s_hi]; written
// back to keys, or its first kk keys to cand[chunk * kk ..].
__global__ void __launch_bounds__(kSortThreads)
    sort_chunk_kernel(const float *logits, int V, u64 *keys, int s_lo, int s_hi, int all_asc, u64 *cand, int kk,
                      const int *done = nullptr) {
  if (done && *done) return;  // topk_fast_kernel finished the draw
  __shared__ u64 sk[kSortChunk];
  const int base = blockIdx.x * kSortChunk;
#pragma unroll
  for (int u = 0; u < kSortChunk / kSortThreads; u++) {
    const int i = threadIdx.x + u * kSortThreads, g = base + i;
    sk[i] = logits ? (g < V ? sample_key(logits[g], g) : ~0ull) : keys[g];
  }
  __syncthreads();
  bitonic_levels(sk, kSortChunk, base, s_lo, s_hi, all_asc != 0);
  if (cand) {
    for (int i = threadIdx.x; i < kk; i += blockDim.x) cand[(size_t)blockIdx.x * kk + i] = sk[i];
  } else {
    for (int i = threadIdx.x; i < kSortChunk; i += blockDim.x) keys[base + i] = sk[i];
  }
}

// One stride j >= kSortChunk of level s over the n global keys.
__global__ void bitonic_global_kernel(u64 *keys, int n, int s, int j) {
  for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n / 2; p += gridDim.x * blockDim.x) {
    const int i = ((p & ~(j - 1)) << 1) | (p & (j - 1)), l = i + j;
    const bool asc = (i & s) == 0;
    const u64 a = keys[i], b = keys[l];
    if ((a > b) == asc) {
      keys[i] = b;
      keys[l] = a;
    }
  }
}

__device__ __forceinline__ float rng_uniform(u64 *state) {
  u64 s = *state;
  s ^= s >> 12;
  s ^= s << 25;
  s ^= s >> 27;
  *state = s;
  return (float)((s * 0x2545F4914F6CDD1Dull) >> 40) / (float)(1 << 24);
}

// The draw over the first k sorted keys; p holds k floats in shared memory.
__device__ void draw_sorted(const u64 *sorted, int k, const float *logits, float temperature, float *p, u64 *rng,
                            SampleOut o) {
  const float mx = logits[key_id(sorted[0])];
  for (int i = threadIdx.x; i < k; i += blockDim.x) p[i] = lm_expf((logits[key_id(sorted[i])] - mx) / temperature);
  __syncthreads();
  if (threadIdx.x != 0) return;
  float total = 0.0f;
  int i = 0;
  for (; i + 8 <= k; i += 8) {
    float v[8];
#pragma unroll
    for (int u = 0; u < 8; u++) v[u] = p[i + u];
#pragma unroll
    for (int u = 0; u < 8; u++) total += v[u];
  }
  for (; i < k; i++) total += p[i];
  float r = rng_uniform(rng) * total;
  int pick = k - 1;
  for (i = 0; i < k; i++) {
    r -= p[i];
    if (r <= 0.0f) {
      pick = i;
      break;
    }
  }
  const int id = key_id(sorted[pick]);
  if (o.id) *o.id = id;
  if (o.id2) *o.id2 = id;
  if (o.ids) o.ids[*o.state_step - 1] = id;
  if (o.state_token) *o.state_token = id;
}

// n_cand chunk candidates (padded to n_pad, a power of two <= kMergeCap):
// sort, then draw from the first k.
__global__ void __launch_bounds__(kSortThreads)
    merge_draw_kernel(const u64 *cand, int n_cand, int n_pad, int k, const float *logits, float temperature, u64 *rng,
                      SampleOut o, int *topk_ids, const int *done = nullptr) {
  if (done && *done) return;  // topk_fast_kernel finished the draw
  extern __shared__ __align__(16) unsigned char smem[];
  u64 *sk = reinterpret_cast<u64 *>(smem);
  float *p = reinterpret_cast<float *>(sk + n_pad);
  for (int i = threadIdx.x; i < n_pad; i += blockDim.x) sk[i] = i < n_cand ? cand[i] : ~0ull;
  __syncthreads();
  bitonic_levels(sk, n_pad, 0, 2, n_pad, false);
  if (topk_ids) {
    for (int i = threadIdx.x; i < k; i += blockDim.x) topk_ids[i] = key_id(sk[i]);
    return;
  }
  draw_sorted(sk, k, logits, temperature, p, rng, o);
}

// One-CTA top-k for k <= kTopkSmall, the usual case. Each thread takes its
// share of the logits (for_each_logit) and keeps their largest value; the k-th largest
// maximum of disjoint groups of them, T, has at least k logits >= T (k groups
// each own one), so the top k are among the logits >= T. The groups are 16
// threads for k <= 64 (a one-warp sort of 64 maxima), single threads above. Those are gathered (typically a
// few times k of them) and sorted as 64-bit keys. When more than kFastCap
// logits reach T (large ties), the kernel leaves *done = 0 and the two
// chunk-sort kernels queued after it do the work; otherwise it draws (or
// writes the ids), sets *done = 1, and they return at once.
constexpr int kFastCap = 8192;

inline size_t fast_smem() { return (size_t)kSortThreads * 8 + (size_t)kFastCap * 8 + (size_t)kTopkSmall * 4; }

__device__ __forceinline__ unsigned value_key(float v) {
  unsigned u = __float_as_uint(v);
  if ((u & 0x7fffffffu) == 0) u = 0;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Calls f(value, index) for every logit, the elements of thread t being
// t, t + 1024, ... in units of float4 when the array is 16-byte aligned (8
// loads in flight per thread), single floats otherwise.
template <class F>
__device__ __forceinline__ void for_each_logit(const float *logits, int V, F f) {
  const int t = threadIdx.x;
  constexpr int U = 8;
  if ((reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
    const float4 *l4 = reinterpret_cast<const float4 *>(logits);
    const int V4 = V >> 2;
    for (int i0 = t; i0 < V4; i0 += U * kSortThreads) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; u++) v[u] = i0 + u * kSortThreads < V4 ? l4[i0 + u * kSortThreads] : float4{};
#pragma unroll
      for (int u = 0; u < U; u++)
        if (i0 + u * kSortThreads < V4) {
          const int b = 4 * (i0 + u * kSortThreads);
          f(v[u].x, b);
          f(v[u].y, b + 1);
          f(v[u].z, b + 2);
          f(v[u].w, b + 3);
        }
    }
    for (int i = 4 * V4 + t; i < V; i += kSortThreads) f(logits[i], i);
  } else {
    for (int i0 = t; i0 < V; i0 += U * kSortThreads) {
      float v[U];
#pragma unroll
      for (int u = 0; u < U; u++) v[u] = i0 + u * kSortThreads < V ? logits[i0 + u * kSortThreads] : 0.0f;
#pragma unroll
      for (int u = 0; u < U; u++)
        if (i0 + u * kSortThreads < V) f(v[u], i0 + u * kSortThreads);
    }
  }
}

__global__ void __launch_bounds__(kSortThreads)
    topk_fast_kernel(const float *logits, int V, int k, float temperature, u64 *rng, SampleOut o, int *topk_ids,
                     int *done) {
  extern __shared__ __align__(16) unsigned char smem[];
  u64 *tmax = reinterpret_cast<u64 *>(smem);             // [1024] (~max key) << 32 | group
  u64 *cand = tmax + kSortThreads;                       // [kFastCap]
  float *p = reinterpret_cast<float *>(cand + kFastCap);  // [kTopkSmall]
  __shared__ int cnt;
  __shared__ unsigned thr;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  unsigned mk = 0;
  for_each_logit(logits, V, [&](float v, int) { mk = max(mk, value_key(v)); });
  if (t == 0) cnt = 0;
  if (k <= 64) {
    // groups of 16 threads: 64 group maxima, the k-th largest by one warp
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) mk = max(mk, __shfl_xor_sync(0xffffffffu, mk, off));
    if ((lane & 15) == 0) tmax[warp * 2 + (lane >> 4)] = ((u64)(~mk) << 32) | (unsigned)(warp * 2 + (lane >> 4));
    __syncthreads();
    if (warp == 0) {
      u64 a[2] = {tmax[lane], tmax[lane + 32]};
      warp_sort64(a);
      const u64 kth = __shfl_sync(0xffffffffu, (k - 1) >= 32 ? a[1] : a[0], (k - 1) & 31);
      if (lane == 0) thr = ~(unsigned)(kth >> 32);
    }
  } else {
    tmax[t] = ((u64)(~mk) << 32) | (unsigned)t;
    __syncthreads();
    bitonic_levels(tmax, kSortThreads, 0, 2, kSortThreads, false);
    if (t == 0) thr = ~(unsigned)(tmax[k - 1] >> 32);
  }
  __syncthreads();
  const unsigned T = thr;
  for_each_logit(logits, V, [&](float v, int i) {
    const unsigned key = value_key(v);
    if (key >= T) {
      const int j = atomicAdd(&cnt, 1);
      if (j < kFastCap) cand[j] = ((u64)(~key) << 32) | (unsigned)i;
    }
  });
  __syncthreads();
  const int n = cnt;
  if (n > kFastCap) {
    if (t == 0) *done = 0;
    return;
  }
  if (n <= 64) {
    if (warp == 0) {
      u64 a[2] = {lane < n ? cand[lane] : ~0ull, lane + 32 < n ? cand[lane + 32] : ~0ull};
      warp_sort64(a);
      cand[lane] = a[0];
      cand[lane + 32] = a[1];
    }
    __syncthreads();
  } else {
    int n_pad = 128;
    while (n_pad < n) n_pad <<= 1;
    for (int i = n + t; i < n_pad; i += kSortThreads) cand[i] = ~0ull;
    __syncthreads();
    bitonic_levels(cand, n_pad, 0, 2, n_pad, false);
  }
  if (t == 0) *done = 1;
  if (topk_ids) {
    for (int i = t; i < k; i += kSortThreads) topk_ids[i] = key_id(cand[i]);
    return;
  }
  draw_sorted(cand, k, logits, temperature, p, rng, o);
}

constexpr int kDrawStage = 8192;  // weights of the global-key draw staged per round

// The draw (or the top-k ids) from a fully sorted global key array. The
// weights are computed a stage at a time into shared memory (twice: for the
// sum, then for the walk) so that thread 0's sequential chains read shared
// memory.
__global__ void __launch_bounds__(kSortThreads)
    sorted_draw_kernel(const u64 *keys, int k, const float *logits, float temperature, u64 *rng, SampleOut o,
                       int *topk_ids) {
  if (topk_ids) {
    for (int i = threadIdx.x; i < k; i += blockDim.x) topk_ids[i] = key_id(keys[i]);
    return;
  }
  __shared__ float st[kDrawStage];
  __shared__ float r_sh;
  __shared__ int pick_sh;
  const float mx = logits[key_id(keys[0])];
  float total = 0.0f;
  for (int c0 = 0; c0 < k; c0 += kDrawStage) {
    const int n = min(kDrawStage, k - c0);
    for (int i = threadIdx.x; i < n; i += blockDim.x)
      st[i] = lm_expf((logits[key_id(keys[c0 + i])] - mx) / temperature);
    __syncthreads();
    if (threadIdx.x == 0) {
      int i = 0;
      for (; i + 8 <= n; i += 8) {
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; u++) v[u] = st[i + u];
#pragma unroll
        for (int u = 0; u < 8; u++) total += v[u];
      }
      for (; i < n; i++) total += st[i];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    r_sh = rng_uniform(rng) * total;
    pick_sh = -1;
  }
  __syncthreads();
  for (int c0 = 0; c0 < k; c0 += kDrawStage) {
    const int n = min(kDrawStage, k - c0);
    for (int i = threadIdx.x; i < n; i += blockDim.x)
      st[i] = lm_expf((logits[key_id(keys[c0 + i])] - mx) / temperature);
    __syncthreads();
    if (threadIdx.x == 0) {
      float r = r_sh;
      for (int i = 0; i < n; i++) {
        r -= st[i];
        if (r <= 0.0f) {
          pick_sh = c0 + i;
          break;
        }
      }
      r_sh = r;
    }
    __syncthreads();
    if (pick_sh >= 0) break;
  }
  if (threadIdx.x == 0) {
    const int id = key_id(keys[pick_sh >= 0 ? pick_sh : k - 1]);
    if (o.id) *o.id = id;
    if (o.id2) *o.id2 = id;
    if (o.ids) o.ids[*o.state_step - 1] = id;
    if (o.state_token) *o.state_token = id;
  }
}

inline size_t merge_smem(int n_pad) { return (size_t)n_pad * 8 + (size_t)kTopkSmall * 4; }

}  // namespace llmq
