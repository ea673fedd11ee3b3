// Batched decode attention over the paged KV cache (GQA group of 4, head_dim 64).
//
// The reference's decode attention (nki_kernels/attention.py:270-399) for one
// sequence: per kv head g, scores s = q_h . K[:len] / 8 for its 4 q heads,
// softmax, o_h = P . V. The batched decode path (many
// sequences of ~1024 cached positions) reads B x 2 KB x len of K/V per layer,
// as much as the weights at bs 64, so this kernel is built to stream it:
//
//  * grid (splits, kv heads, sequences); CTA (s, g, b) covers positions
//    [s * split_len, (s+1) * split_len) of sequence b for the 4 q heads of kv
//    head g; its 4 warps take turns at the 32-position chunks of the split;
//  * each warp pipelines its chunks: cp.async copies the next chunk's K and V
//    rows (16-byte pieces, zero-filled past the end) into the other of two
//    shared buffers while it computes the current one, whose pieces are
//    XOR-swizzled by row so both products read shared memory without bank
//    conflicts;
//  * scores: lane (r, h) dots q head h (packed bf16 in registers,
//    fma.rn.f32.bf16) with rows r, r+8, r+16, r+24; P . V: lane j owns dims
//    2j, 2j+1 of all 32 rows for the 4 heads;
//  * online softmax in fp32 per head; the CTA's warps are merged in shared
//    memory, and the CTA writes one (m, l, o[64]) partial per head;
//  * a merge kernel (one CTA per sequence and kv head) combines the splits and
//    writes o as bf16, the rounding of the attention output the single-GPU
//    kernel uses.
// Positions index pages through the block table; a page id outside the pool
// sets the error word and the position is skipped (never dereferenced).
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace mk {

constexpr int kAttnCtaWarps = 4;
constexpr int kAttnPartial = 2 + 64;  // m, l, o[64]
constexpr int kAttnChunkBytes = 32 * 128;  // 32 rows of K (or V)
// Shared memory per CTA: per warp two chunk buffers of K and V.
constexpr int kAttnSmem = kAttnCtaWarps * 2 * 2 * kAttnChunkBytes;

struct PagedAttnParams {
  const __nv_bfloat16* q;      // [B][NQ][64]
  const __nv_bfloat16* k;      // layer base: [num_pages][NKV][ps][64]
  const __nv_bfloat16* v;
  const int* block_tables;     // [B][max_blocks]
  const int* lengths;          // [B]: positions [0, len) are attended
  int NQ, NKV, ps, max_blocks, num_pages, splits, split_len;
  float scale;
  float* work;                 // [B][NKV][splits][4][kAttnPartial]
  __nv_bfloat16* out;          // [B][NQ][64]
  int* error;
};

__device__ __forceinline__ float2 bf2x2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// c0 += lo(a) lo(b), c1 += hi(a) hi(b) on packed bf16 pairs, in fp32 (the
// products of two bf16 values are exact in fp32).
__device__ __forceinline__ void attn_fma2(uint32_t a, uint32_t b, float& c0, float& c1) {
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %2;\n\t"
      "mov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.bf16 %1, ah, bh, %1;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "r"(a), "r"(b));
}

// 16-byte asynchronous copy global -> shared; src_bytes 0 fills zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}

// Row r's 16-byte piece c of a chunk buffer sits at piece c ^ (r & 7): the 8
// rows a score instruction reads, and the 8 pieces a P . V instruction reads,
// fall in different banks.
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

__global__ void __launch_bounds__(kAttnCtaWarps * 32) paged_attn_kernel(const __grid_constant__ PagedAttnParams p) {
  extern __shared__ __align__(128) uint8_t asmem[];
  __shared__ float pw[kAttnCtaWarps][4][32];               // probabilities of a chunk
  __shared__ float st[kAttnCtaWarps][4][kAttnPartial];     // per-warp states
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // scores: lane = (position r8 of each 8, head h); P . V: lane = dims 2 lane, 2 lane + 1
  const int h = lane & 3, r8 = lane >> 2;
  const int len = p.lengths[b];
  const int p0 = s * p.split_len, p1 = min(len, p0 + p.split_len);
  const uint32_t wbuf = (uint32_t)__cvta_generic_to_shared(asmem) + warp * 4 * kAttnChunkBytes;
  // buffer j (0, 1): K at wbuf + j * 2 * kAttnChunkBytes, V right after it
  const int* table = p.block_tables + (size_t)b * p.max_blocks;
  const int nchunks = p1 > p0 ? (p1 - p0 + 31) / 32 : 0;
  // this warp takes chunks warp, warp + 4, ... of the split
  auto issue = [&](int ci, int j) {
    const int c0 = p0 + ci * 32;
    const uint32_t kb = wbuf + j * 2 * kAttnChunkBytes, vb = kb + kAttnChunkBytes;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = k * 4 + (lane >> 3), piece = lane & 7, pos = c0 + row;
      const __nv_bfloat16* ks = p.k;
      const __nv_bfloat16* vs = p.v;
      uint32_t bytes = 0;
      if (pos < p1) {
        const int page = table[pos / p.ps];
        if (page >= 0 && page < p.num_pages) {
          const size_t off = (((size_t)page * p.NKV + g) * p.ps + pos % p.ps) * 64 + piece * 8;
          ks += off;
          vs += off;
          bytes = 16;
        } else {
          atomicExch(p.error, 1);
        }
      }
      cp_async16(kb + swz(row, piece), ks, bytes);
      cp_async16(vb + swz(row, piece), vs, bytes);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  // q head h as packed bf16 (the scale is applied to the fp32 score)
  uint32_t q[32];
  {
    const uint4* qp = reinterpret_cast<const uint4*>(p.q + ((size_t)b * p.NQ + g * 4 + h) * 64);
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 u = __ldg(qp + c);
      q[c * 4 + 0] = u.x;
      q[c * 4 + 1] = u.y;
      q[c * 4 + 2] = u.z;
      q[c * 4 + 3] = u.w;
    }
  }
  float m = -INFINITY, l = 0.f;  // head h's running max and sum (same in its 8 lanes)
  float o[4][2];
#pragma unroll
  for (int hh = 0; hh < 4; ++hh) o[hh][0] = o[hh][1] = 0.f;

  int j = 0;
  if (warp < nchunks) issue(warp, 0);
  for (int ci = warp; ci < nchunks; ci += kAttnCtaWarps, j ^= 1) {
    if (ci + kAttnCtaWarps < nchunks) {
      issue(ci + kAttnCtaWarps, j ^ 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncwarp();
    const int c0 = p0 + ci * 32;
    const uint32_t kb = wbuf + j * 2 * kAttnChunkBytes, vb = kb + kAttnChunkBytes;
    // ---- scores from shared memory
    float sc[4];
    float cm = -INFINITY;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int row = r * 8 + r8;
      float a0 = 0.f, a1 = 0.f, a2 = 0.f, a3 = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint4 u;
        asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                     : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                     : "r"(kb + swz(row, c)));
        attn_fma2(u.x, q[c * 4 + 0], a0, a1);
        attn_fma2(u.y, q[c * 4 + 1], a2, a3);
        attn_fma2(u.z, q[c * 4 + 2], a0, a1);
        attn_fma2(u.w, q[c * 4 + 3], a2, a3);
      }
      const int pos = c0 + row;
      sc[r] = pos < p1 ? ((a0 + a1) + (a2 + a3)) * p.scale : -INFINITY;
      cm = fmaxf(cm, sc[r]);
    }
    // head h's max and sum over the chunk: its 8 lanes differ in lane bits 2..4
#pragma unroll
    for (int d = 4; d < 32; d <<= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, d));
    const float mn = fmaxf(m, cm);
    const float alpha = (mn == -INFINITY) ? 1.f : __expf(m - mn);
    float sum = 0.f;
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const float e = (sc[r] == -INFINITY) ? 0.f : __expf(sc[r] - mn);
      pw[warp][h][r * 8 + r8] = e;
      sum += e;
    }
#pragma unroll
    for (int d = 4; d < 32; d <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
    l = l * alpha + sum;
    m = mn;
    __syncwarp();
    // ---- P . V from shared memory
#pragma unroll
    for (int hh = 0; hh < 4; ++hh) {
      const float a = __shfl_sync(0xffffffffu, alpha, hh);  // lane hh holds head hh
      o[hh][0] *= a;
      o[hh][1] *= a;
    }
    const int n = min(32, p1 - c0);
    for (int jj = 0; jj < n; ++jj) {
      uint32_t vw;
      asm volatile("ld.shared.u32 %0, [%1];"
                   : "=r"(vw)
                   : "r"(vb + swz(jj, lane >> 2) + (lane & 3) * 4));
      const float2 f = bf2x2(vw);
#pragma unroll
      for (int hh = 0; hh < 4; ++hh) {
        const float pr = pw[warp][hh][jj];
        o[hh][0] = fmaf(pr, f.x, o[hh][0]);
        o[hh][1] = fmaf(pr, f.y, o[hh][1]);
      }
    }
    __syncwarp();
  }
  // ---- merge the warps, write the CTA's partial per head
  if (lane < 4) {
    st[warp][h][0] = m;
    st[warp][h][1] = l;
  }
#pragma unroll
  for (int hh = 0; hh < 4; ++hh) {
    st[warp][hh][2 + 2 * lane] = o[hh][0];
    st[warp][hh][3 + 2 * lane] = o[hh][1];
  }
  __syncthreads();
  float* dst = p.work + ((((size_t)b * p.NKV + g) * p.splits + s) * 4) * kAttnPartial;
  for (int i = threadIdx.x; i < 4 * 64; i += kAttnCtaWarps * 32) {
    const int hh = i >> 6, d = i & 63;
    float M = -INFINITY;
    for (int w = 0; w < kAttnCtaWarps; ++w) M = fmaxf(M, st[w][hh][0]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kAttnCtaWarps; ++w) {
      const float a = (st[w][hh][0] == -INFINITY) ? 0.f : __expf(st[w][hh][0] - M);
      L += st[w][hh][1] * a;
      O += st[w][hh][2 + d] * a;
    }
    if (d == 0) {
      dst[hh * kAttnPartial + 0] = M;
      dst[hh * kAttnPartial + 1] = L;
    }
    dst[hh * kAttnPartial + 2 + d] = O;
  }
}

__global__ void __launch_bounds__(256) paged_attn_merge_kernel(const __grid_constant__ PagedAttnParams p) {
  const int g = blockIdx.x, b = blockIdx.y;
  const int h = threadIdx.x >> 6, d = threadIdx.x & 63;
  const float* src = p.work + (((size_t)b * p.NKV + g) * p.splits * 4) * kAttnPartial;
  float M = -INFINITY;
  for (int s = 0; s < p.splits; ++s) M = fmaxf(M, src[(s * 4 + h) * kAttnPartial]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < p.splits; ++s) {
    const float* q = src + (s * 4 + h) * kAttnPartial;
    const float a = (q[0] == -INFINITY) ? 0.f : __expf(q[0] - M);
    L += q[1] * a;
    O += q[2 + d] * a;
  }
  p.out[((size_t)b * p.NQ + g * 4 + h) * 64 + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
}

}  // namespace mk
