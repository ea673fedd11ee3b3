// Token sampling after the lm_head: temperature, top-k, top-p, one draw.
//
// The reference exposes these knobs per sequence (top_k, top_p, temperature,
// main.py:57-61 and prepare_sampling_params main.py:197-205) and samples on
// the device through NxDI's OnDeviceSamplingConfig (main.py:129-130; NxDI
// is not part of the reference sources). The published order is followed:
// logits / temperature, keep the top_k largest, softmax over them, keep the
// smallest prefix (by descending probability) whose mass reaches top_p, draw
// from it. top_k == 1 or temperature <= 0 is greedy: the lowest index among
// the maxima, as the decode kernel's own argmax.
//
// One CTA of kSampleThreads per sequence:
//  1. radix select (4 passes of 8-bit digits over order-preserving keys) finds
//     the key of the top_k-th largest logit;
//  2. logits above it, and those equal to it, are appended to a candidate
//     list (kSampleCand entries) and bitonic-sorted by (logit desc, index
//     asc), so ties at the threshold keep the lowest indices; a list that
//     overflows (more than kSampleCand - top_k logits tie at the threshold)
//     is reported as an error instead of guessed;
//  3. p_i = exp((l_i - l_max) / T) over the first top_k, inclusive prefix
//     sums, the top-p cut m = the first prefix reaching top_p of the total,
//     then u in [0, 1) (24 bits from a splitmix64 hash of seed, step and the
//     sequence) selects the first candidate j < m with prefix_j > u *
//     prefix_{m-1}.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mk {

constexpr int kSampleThreads = 1024;
constexpr int kSampleMaxK = 1024;   // top_k is clamped to this (0 or negative: this)
constexpr int kSampleCand = 2048;   // candidate list (top_k plus ties at the threshold)
constexpr int kSampleMaxBatch = 64;

struct SampleParams {
  const float* logits;  // [batch][ld]
  long long ld;
  int V;
  int top_k[kSampleMaxBatch];
  float top_p[kSampleMaxBatch];
  float temperature[kSampleMaxBatch];
  unsigned long long seed, step;
  int* out;        // [batch] drawn ids
  int* tokens;     // optional: the draw is also written here ...
  int* positions;  // ... and the position advanced (device-side feedback)
  int* error;      // [1]: 0, or 1 when a candidate list overflowed
};

__host__ __device__ inline unsigned long long splitmix64(unsigned long long x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

// The draw's uniform in [0, 1): 24 bits, exactly representable in fp32.
__host__ __device__ inline float sample_uniform(unsigned long long seed, unsigned long long step,
                                               int seq) {
  const unsigned long long h =
      splitmix64(seed ^ splitmix64(step * 0xD1B54A32D192ED03ull + (unsigned long long)seq));
  return (float)(h >> 40) * (1.0f / 16777216.0f);
}

__device__ __forceinline__ uint32_t sample_key(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__global__ void __launch_bounds__(kSampleThreads, 1) sample_kernel(const __grid_constant__ SampleParams p) {
  __shared__ unsigned int hist[256];
  __shared__ unsigned long long cand[kSampleCand];
  __shared__ float prob[kSampleMaxK];
  __shared__ float wsum[kSampleThreads / 32];
  __shared__ unsigned int s_prefix, s_need, s_count;
  __shared__ unsigned long long s_best;
  const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* lg = p.logits + (long long)b * p.ld;
  const float T = p.temperature[b];
  int K = p.top_k[b];
  if (K <= 0 || K > kSampleMaxK) K = kSampleMaxK;
  if (K > p.V) K = p.V;

  if (K == 1 || !(T > 0.f)) {
    // greedy: packed (key, ~index) max = highest logit, lowest index
    unsigned long long best = 0;
    for (int i = tid; i < p.V; i += kSampleThreads) {
      const unsigned long long k = ((unsigned long long)sample_key(lg[i]) << 32) | (0xFFFFFFFFu - (uint32_t)i);
      best = k > best ? k : best;
    }
    for (int o = 16; o; o >>= 1) {
      const unsigned long long t = __shfl_xor_sync(0xffffffffu, best, o);
      best = t > best ? t : best;
    }
    if (tid == 0) s_best = 0;
    __syncthreads();
    if (lane == 0) atomicMax(&s_best, best);
    __syncthreads();
    if (tid == 0) {
      const int id = (int)(0xFFFFFFFFu - (uint32_t)(s_best & 0xFFFFFFFFull));
      p.out[b] = id;
      if (p.tokens) {
        p.tokens[b] = id;
        p.positions[b] += 1;
      }
    }
    return;
  }

  // ---- 1. radix select of the K-th largest key
  if (tid == 0) {
    s_prefix = 0;
    s_need = (unsigned)K;
  }
  uint32_t mask = 0;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = tid; i < 256; i += kSampleThreads) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix;
    for (int i = tid; i < p.V; i += kSampleThreads) {
      const uint32_t k = sample_key(lg[i]);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      unsigned int cum = 0, need = s_need;
      int bin = 255;
      for (; bin > 0; --bin) {
        if (cum + hist[bin] >= need) break;
        cum += hist[bin];
      }
      s_need = need - cum;  // keys equal to the final prefix still to take
      s_prefix = prefix | ((uint32_t)bin << shift);
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  const uint32_t thr = s_prefix;

  // ---- 2. candidates: all keys above the threshold, and the ties at it
  if (tid == 0) s_count = 0;
  for (int i = tid; i < kSampleCand; i += kSampleThreads) cand[i] = 0;
  __syncthreads();
  for (int i = tid; i < p.V; i += kSampleThreads) {
    const uint32_t k = sample_key(lg[i]);
    if (k >= thr) {
      const unsigned int slot = atomicAdd(&s_count, 1u);
      if (slot < (unsigned)kSampleCand)
        cand[slot] = ((unsigned long long)k << 32) | (0xFFFFFFFFu - (uint32_t)i);
    }
  }
  __syncthreads();
  if (s_count > (unsigned)kSampleCand) {
    if (tid == 0) {
      atomicExch(p.error, 1);
      p.out[b] = -1;
    }
    return;
  }
  // bitonic sort, descending
  for (int size = 2; size <= kSampleCand; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int i = tid; i < kSampleCand / 2; i += kSampleThreads) {
        const int lo = 2 * i - (i & (stride - 1));
        const int hi = lo + stride;
        const bool desc = ((lo & size) == 0);
        const unsigned long long a = cand[lo], c = cand[hi];
        if ((a < c) == desc) {
          cand[lo] = c;
          cand[hi] = a;
        }
      }
      __syncthreads();
    }
  }

  // ---- 3. probabilities of the first K, prefix sums, top-p cut, draw
  auto value = [&](int j) { return lg[0xFFFFFFFFu - (uint32_t)(cand[j] & 0xFFFFFFFFull)]; };
  const float vmax = value(0);
  float e = 0.f;
  if (tid < K) e = expf((value(tid) - vmax) / T);
  // inclusive scan over the K probabilities (tid order = descending logit)
  float x = e;
  for (int o = 1; o < 32; o <<= 1) {
    const float y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[warp] = x;
  __syncthreads();
  if (warp == 0) {
    float w = wsum[lane];
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    wsum[lane] = w;  // inclusive warp totals
  }
  __syncthreads();
  if (warp > 0) x += wsum[warp - 1];
  if (tid < K) prob[tid] = x;
  __syncthreads();
  if (tid == 0) {
    const float total = prob[K - 1];
    const float P = p.top_p[b];
    int m = K;
    if (P < 1.f) {
      const float cut = P * total;
      m = 1;
      while (m < K && prob[m - 1] < cut) ++m;
    }
    const float r = sample_uniform(p.seed, p.step, b) * prob[m - 1];
    int j = 0;
    while (j < m - 1 && !(prob[j] > r)) ++j;
    const int id = (int)(0xFFFFFFFFu - (uint32_t)(cand[j] & 0xFFFFFFFFull));
    p.out[b] = id;
    if (p.tokens) {
      p.tokens[b] = id;
      p.positions[b] += 1;
    }
  }
}

}  // namespace mk
