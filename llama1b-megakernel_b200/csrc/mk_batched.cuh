// Fused elementwise steps of the batched decode path (batched.py).
//
// Between the projections of a batched step, HF's decode layer does RMSNorm,
// RoPE on q and k, the K/V cache write, and SiLU(gate) * up, each a handful
// of small tensor ops. These kernels do each step in one launch with HF's
// rounding (the same formulas as the persistent kernel's epilogues):
//   rmsnorm:  y = bf16(bf16(x * 1/sqrt(mean(x^2) + eps)) * gamma), sums in fp32
//   rope:     y0 = bf16(bf16(x0 c0) + bf16(-x1 s0)), y1 = bf16(bf16(x1 c1) + bf16(x0 s1))
//             for the pair (d, d + 32) of every q and k head, from the bf16
//             cos/sin table rows of the step's positions
//   swiglu:   a = bf16(bf16(g / (1 + exp(-g))) * u)
//   argmax:   the greedy id of each row of fp32 logits (lowest index on ties)
// and, for the tensor-parallel batched step:
//   add + rmsnorm: x = bf16(x + bf16(partial sum)), then rmsnorm(x)
//   argmax keys:   (order-preserving float bits << 32 | ~global id) per row,
//                  so the ranks' keys combine by an integer max
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "mk_device.cuh"

namespace mk {

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One CTA of 256 threads per row; H a multiple of 8.
__global__ void __launch_bounds__(256) rmsnorm_rows_kernel(const __nv_bfloat16* x, const __nv_bfloat16* gamma,
                                                           float eps, int H, __nv_bfloat16* y) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const int b = blockIdx.x, tid = threadIdx.x;
  const uint4* xr = reinterpret_cast<const uint4*>(x + (size_t)b * H);
  float ss = 0.f;
  for (int i = tid; i < H / 8; i += 256) {
    const uint4 u = xr[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = __uint_as_float(w[e] << 16), c = __uint_as_float(w[e] & 0xFFFF0000u);
      ss = fmaf(a, a, ss);
      ss = fmaf(c, c, ss);
    }
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w];
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)H), eps)));
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)b * H);
  for (int i = tid; i < H / 8; i += 256) {
    const uint4 u = xr[i], g = gr[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bfr(bfr(__uint_as_float(w[e] << 16) * r) * __uint_as_float(gw[e] << 16));
      const float hi = bfr(bfr(__uint_as_float(w[e] & 0xFFFF0000u) * r) * __uint_as_float(gw[e] & 0xFFFF0000u));
      __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
      o[e] = *reinterpret_cast<uint32_t*>(&pr);
    }
    yr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// qkv: [B][(NQ + 2 NKV) * 64] GEMM output in the packed RoPE-pair order
// (column head * 64 + 2 d + pair holds dim d + 32 pair of the head). Writes q
// [B][NQ][64] (rotated) and the rotated k / plain v rows into the layer's page
// pools at the step's positions. One thread per (sequence, head, d < 32).
__global__ void __launch_bounds__(256) rope_scatter_kernel(
    const __nv_bfloat16* qkv, const __nv_bfloat16* cos_t, const __nv_bfloat16* sin_t,
    const int* positions, const int* block_tables, int max_blocks, int num_pages, int ps, int NQ,
    int NKV, int B, __nv_bfloat16* q_out, __nv_bfloat16* k_pages, __nv_bfloat16* v_pages, int* error) {
  pdl_trigger();
  pdl_wait();
  const int nh = NQ + 2 * NKV;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B * nh * 32) return;
  const int d = i & 31, hd = (i >> 5) % nh, b = (i >> 5) / nh;
  const __nv_bfloat16* src = qkv + ((size_t)b * nh + hd) * 64 + 2 * d;
  float x0 = __bfloat162float(src[0]), x1 = __bfloat162float(src[1]);
  const int pos = positions[b];
  if (hd < NQ + NKV) {
    const __nv_bfloat16* cr = cos_t + (size_t)pos * 64;
    const __nv_bfloat16* sr = sin_t + (size_t)pos * 64;
    const float c0 = __bfloat162float(cr[d]), c1 = __bfloat162float(cr[d + 32]);
    const float s0 = __bfloat162float(sr[d]), s1 = __bfloat162float(sr[d + 32]);
    const float y0 = bfr(bfr(x0 * c0) + bfr(-x1 * s0));
    const float y1 = bfr(bfr(x1 * c1) + bfr(x0 * s1));
    x0 = y0;
    x1 = y1;
  }
  if (hd < NQ) {
    __nv_bfloat16* qr = q_out + ((size_t)b * NQ + hd) * 64;
    qr[d] = __float2bfloat16_rn(x0);
    qr[d + 32] = __float2bfloat16_rn(x1);
    return;
  }
  const bool is_k = hd < NQ + NKV;
  const int g = is_k ? hd - NQ : hd - NQ - NKV;
  const int page = block_tables[(size_t)b * max_blocks + pos / ps];
  if (page < 0 || page >= num_pages) {
    atomicExch(error, 1);
    return;
  }
  __nv_bfloat16* dst = (is_k ? k_pages : v_pages) + (((size_t)page * NKV + g) * ps + pos % ps) * 64;
  dst[d] = __float2bfloat16_rn(x0);
  dst[d + 32] = __float2bfloat16_rn(x1);
}

// gu: [B][I][2] (gate, up interleaved, the packed w_gate_up order) -> a [B][I].
__global__ void __launch_bounds__(256) swiglu_kernel(const __nv_bfloat16* gu, int n, __nv_bfloat16* a) {
  pdl_trigger();
  pdl_wait();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const __nv_bfloat162 p = reinterpret_cast<const __nv_bfloat162*>(gu)[i];
  const float g = __bfloat162float(p.x), u = __bfloat162float(p.y);
  const float s = bfr(__fdiv_rn(g, 1.0f + expf(-g)));
  a[i] = __float2bfloat16_rn(s * u);
}

// One CTA of 1024 threads per row of `cols` fp32 values: each thread scans
// columns in order (128-bit loads when cols is a multiple of 4 and x 16-byte
// aligned) and keeps its first maximum; the CTA keeps the largest value, then
// the lowest index.
__global__ void __launch_bounds__(1024) argmax_rows_kernel(const float* x, int cols, bool vec,
                                                           int64_t* ids) {
  pdl_trigger();
  pdl_wait();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const float* rowf = x + (size_t)blockIdx.x * cols;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  if (vec) {
    const float4* row = reinterpret_cast<const float4*>(rowf);
    for (int i = threadIdx.x; i < cols / 4; i += 1024) {
      const float4 v = __ldg(row + i);
      const float e[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (e[k] > best) {
          best = e[k];
          idx = 4 * i + k;
        }
      }
    }
  } else {
    for (int i = threadIdx.x; i < cols; i += 1024) {
      const float v = __ldg(rowf + i);
      if (v > best) {
        best = v;
        idx = i;
      }
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    best = bv[lane];
    idx = bi[lane];
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) {
        best = ov;
        idx = oi;
      }
    }
    if (lane == 0) ids[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
  }
}

// Tensor parallelism, after the o_proj / down partial sums of every rank
// were summed into `sum` ([B][H] fp32): x = bf16(x + bf16(sum)) in place (the
// residual add of HF's decoder layer on the all-reduced projection), then
// y = rmsnorm(x) with gamma. One CTA of 256 threads per row; H a multiple of 8.
__global__ void __launch_bounds__(256) add_rmsnorm_rows_kernel(__nv_bfloat16* x, const float* sum,
                                                               const __nv_bfloat16* gamma,
                                                               float eps, int H,
                                                               __nv_bfloat16* y) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const int b = blockIdx.x, tid = threadIdx.x;
  uint4* xr = reinterpret_cast<uint4*>(x + (size_t)b * H);
  const float4* sr = reinterpret_cast<const float4*>(sum + (size_t)b * H);
  float ss = 0.f;
  for (int i = tid; i < H / 8; i += 256) {
    const uint4 u = xr[i];
    const float4 s0 = sr[2 * i], s1 = sr[2 * i + 1];
    const float sv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bfr(__uint_as_float(w[e] << 16) + bfr(sv[2 * e]));
      const float hi = bfr(__uint_as_float(w[e] & 0xFFFF0000u) + bfr(sv[2 * e + 1]));
      ss = fmaf(lo, lo, ss);
      ss = fmaf(hi, hi, ss);
      __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
      o[e] = *reinterpret_cast<uint32_t*>(&pr);
    }
    xr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w];
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)H), eps)));
  const uint4* gr = reinterpret_cast<const uint4*>(gamma);
  uint4* yr = reinterpret_cast<uint4*>(y + (size_t)b * H);
  for (int i = tid; i < H / 8; i += 256) {
    const uint4 u = xr[i], g = gr[i];  // this thread's own x words, written above
    const uint32_t w[4] = {u.x, u.y, u.z, u.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bfr(bfr(__uint_as_float(w[e] << 16) * r) * __uint_as_float(gw[e] << 16));
      const float hi = bfr(bfr(__uint_as_float(w[e] & 0xFFFF0000u) * r) * __uint_as_float(gw[e] & 0xFFFF0000u));
      __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
      o[e] = *reinterpret_cast<uint32_t*>(&pr);
    }
    yr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// ---------------------------------------------------------------- peer exchange
//
// Tensor parallelism of the batched step without NCCL on the data path. Every
// rank owns one exchange buffer (plain device memory, mapped on the other
// GPUs through CUDA IPC): two partial-sum slots of [rows][H] fp32 and a block
// of 64-bit flag words [2][kMaxTp], flag (slot, src) written by rank src.
// Exchange e of a step uses slot e % 2: the rank's o_proj or down GEMM writes
// its fp32 partial into its own slot, then xreduce_add_rmsnorm_kernel posts a
// tag on every rank's flag (slot, rank), waits (bounded) until every rank's
// flag in its own buffer carries the tag, and reads the W partials of its rows
// straight from the owners' memory over NVLink (plain loads, no multicast).
// Tags grow by step (an epoch word advanced once per step) and exchange, so a
// flag left by an earlier exchange never passes. Two slots suffice: a rank
// writes slot e % 2 again only at exchange e + 2, after its exchange e + 1,
// which waited for every rank's flag e + 1, posted after that rank had
// finished reading exchange e.
constexpr int kXchgSlots = 2;
constexpr int kXchgPerStep = 64;  // exchanges per step at most (2 per decoder layer)

__host__ __device__ inline size_t xchg_slot_floats(int rows, int H) { return (size_t)rows * H; }
__host__ __device__ inline size_t xchg_flags_offset(int rows, int H) {  // bytes
  return ((size_t)kXchgSlots * xchg_slot_floats(rows, H) * 4 + 255) & ~(size_t)255;
}
__host__ __device__ inline size_t xchg_bytes(int rows, int H) {
  return xchg_flags_offset(rows, H) + (size_t)kXchgSlots * kMaxTp * 8;
}

struct XchgParams {
  const unsigned long long* peers;  // [W] every rank's buffer as mapped here (peers[rank] = own)
  int rank, W, rows, H, exchange;
  const uint32_t* epoch;            // the step's epoch (mk_step_epoch)
  __nv_bfloat16* x;                 // [B][H] residual, updated in place
  const __nv_bfloat16* gamma;
  float eps;
  __nv_bfloat16* y;                 // [B][H] RMSNorm output
  int* error;
  unsigned long long timeout_ns;
};

__global__ void epoch_advance_kernel(uint32_t* epoch) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x == 0) epoch[0] += 1u;
}

// Sum of every rank's partial for this exchange (rank order, the same on every
// rank), then the add + RMSNorm of add_rmsnorm_rows_kernel. One CTA of 256
// threads per row.
__global__ void __launch_bounds__(256) xreduce_add_rmsnorm_kernel(const __grid_constant__ XchgParams p) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[8];
  const int b = blockIdx.x, tid = threadIdx.x, H = p.H, W = p.W;
  const int slot = p.exchange % kXchgSlots;
  const unsigned long long tag =
      (unsigned long long)p.epoch[0] * kXchgPerStep + (unsigned long long)p.exchange + 1ull;
  const size_t foff = xchg_flags_offset(p.rows, H) / 8 + (size_t)slot * kMaxTp;  // in u64 words
  int timed_out = 0;
  // Block 0 posts this rank's flag on every rank (the GEMM that wrote the
  // partial finished before this grid started).
  if (b == 0 && tid < W) {
    __threadfence_system();
    unsigned long long* f = reinterpret_cast<unsigned long long*>(p.peers[tid]) + foff + p.rank;
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(f), "l"(tag) : "memory");
  }
  if (tid < W) {
    const unsigned long long* f = reinterpret_cast<const unsigned long long*>(p.peers[p.rank]) + foff + tid;
    uint64_t t0 = 0;
    for (uint32_t it = 0;; ++it) {
      unsigned long long v;
      asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(f) : "memory");
      if (v >= tag) break;
      if ((it & 63) == 63) {
        uint64_t now;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
        if (!t0) {
          t0 = now;
        } else if (now - t0 > p.timeout_ns) {
          atomicCAS(p.error, 0, 3);
          timed_out = 1;
          break;
        }
      }
    }
  }
  if (__syncthreads_or(timed_out)) return;
  uint4* xr = reinterpret_cast<uint4*>(p.x + (size_t)b * H);
  float ss = 0.f;
  for (int i = tid; i < H / 8; i += 256) {
    float sv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < W; ++r) {
      const float4* src = reinterpret_cast<const float4*>(
          reinterpret_cast<const float*>(p.peers[r]) + (size_t)slot * xchg_slot_floats(p.rows, H) +
          (size_t)b * H) + 2 * i;
      const float4 s0 = __ldcv(src), s1 = __ldcv(src + 1);
      sv[0] += s0.x; sv[1] += s0.y; sv[2] += s0.z; sv[3] += s0.w;
      sv[4] += s1.x; sv[5] += s1.y; sv[6] += s1.z; sv[7] += s1.w;
    }
    const uint4 u = xr[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bfr(__uint_as_float(w[e] << 16) + bfr(sv[2 * e]));
      const float hi = bfr(__uint_as_float(w[e] & 0xFFFF0000u) + bfr(sv[2 * e + 1]));
      ss = fmaf(lo, lo, ss);
      ss = fmaf(hi, hi, ss);
      __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
      o[e] = *reinterpret_cast<uint32_t*>(&pr);
    }
    xr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) t += red[w];
  const float rn = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)H), p.eps)));
  const uint4* gr = reinterpret_cast<const uint4*>(p.gamma);
  uint4* yr = reinterpret_cast<uint4*>(p.y + (size_t)b * H);
  for (int i = tid; i < H / 8; i += 256) {
    const uint4 u = xr[i], g = gr[i];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w}, gw[4] = {g.x, g.y, g.z, g.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float lo = bfr(bfr(__uint_as_float(w[e] << 16) * rn) * __uint_as_float(gw[e] << 16));
      const float hi = bfr(bfr(__uint_as_float(w[e] & 0xFFFF0000u) * rn) * __uint_as_float(gw[e] & 0xFFFF0000u));
      __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
      o[e] = *reinterpret_cast<uint32_t*>(&pr);
    }
    yr[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The packed greedy key of each row of fp32 logits (`cols` of them, vocabulary
// ids id0 .. id0 + cols - 1 on this rank): float_key(max) << 32 | (2^32 - 1 -
// id of the first maximum). The largest key over the ranks is the row's
// greedy id with the lowest index on ties. One CTA of 1024 threads per row.
__global__ void __launch_bounds__(1024) argmax_keys_kernel(const float* x, int cols, int id0,
                                                           unsigned long long* keys) {
  pdl_trigger();
  pdl_wait();
  __shared__ float bv[32];
  __shared__ int bi[32];
  const float* rowf = x + (size_t)blockIdx.x * cols;
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < cols; i += 1024) {
    const float v = __ldg(rowf + i);
    if (v > best) {
      best = v;
      idx = i;
    }
  }
  for (int o = 16; o; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > best || (ov == best && oi < idx)) {
      best = ov;
      idx = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    best = bv[lane];
    idx = bi[lane];
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > best || (ov == best && oi < idx)) {
        best = ov;
        idx = oi;
      }
    }
    if (lane == 0) {
      const uint32_t id = (uint32_t)id0 + (uint32_t)(idx == 0x7fffffff ? 0 : idx);
      keys[blockIdx.x] =
          ((unsigned long long)float_key(best) << 32) | (unsigned long long)(0xFFFFFFFFu - id);
    }
  }
}

// keys [W][B] (every rank's argmax_keys) -> ids [B]: the largest key of each
// row, unpacked. One thread per row.
__global__ void keys_to_ids_kernel(const unsigned long long* keys, int W, int B, int64_t* ids) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  unsigned long long k = keys[b];
  for (int r = 1; r < W; ++r) k = max(k, keys[(size_t)r * B + b]);
  ids[b] = (int64_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull));
}

}  // namespace mk
