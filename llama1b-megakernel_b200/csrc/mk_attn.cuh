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
//  * both products on the tensor cores (mma.sync m16n8k16, bf16 inputs, fp32
//    accumulation): scores with the 4 q heads as the rows of the A tile and
//    K from ldmatrix, P . V with P (rounded to bf16, as flash attention does)
//    taken straight from the score accumulators and V from ldmatrix.trans;
//  * online softmax in fp32 per head; the CTA's warps are merged in shared
//    memory, and the CTA writes one (m, l, o[64]) partial per head;
//  * a merge kernel (one CTA per sequence and kv head) combines the splits and
//    writes o as bf16, the rounding of the attention output the single-GPU
//    kernel uses; with a single split the CTA writes o itself and the merge
//    kernel is not launched.
// Positions index pages through the block table; a page id outside the pool
// sets the error word and the position is skipped (never dereferenced).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "mk_device.cuh"

namespace mk {

constexpr int kAttnCtaWarps = 4;
constexpr int kAttnPartial = 2 + 64;  // m, l, o[64]
constexpr int kAttnChunkBytes = 32 * 128;  // 32 rows of K (or V)
constexpr int kAttnPageCache = 128;        // page ids of a split kept in shared memory
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

// 16-byte asynchronous copy global -> shared; src_bytes 0 fills zeros.
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}

// Row r's 16-byte piece c of a chunk buffer sits at piece c ^ (r & 7): the 8
// rows a score instruction reads, and the 8 pieces a P . V instruction reads,
// fall in different banks.
__device__ __forceinline__ uint32_t swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

// One 32-position chunk of the online softmax on the tensor cores: K rows at
// shared address kb, V rows at vb (32 rows of 128 bytes each, 16-byte pieces
// XOR-swizzled by row, see swz), positions c0 .. c0 + 31 of which those at or
// past p1 are masked. Updates the warp's running (m, l, o) of head g8 = lane / 4.
__device__ __forceinline__ void attn_chunk_mma(uint32_t kb, uint32_t vb, int c0, int p1, float scale,
                                               const uint32_t (&qa)[4][2], float& m, float& l,
                                               float (&o)[8][4], int lane) {
  const int t4 = lane & 3;
    // ---- scores: four blocks of 8 positions
    float sc[4][4];
    float cm = -INFINITY;
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      sc[nb][0] = sc[nb][1] = sc[nb][2] = sc[nb][3] = 0.f;
#pragma unroll
      for (int half = 0; half < 2; ++half) {  // pieces 4 half .. 4 half + 3 = k steps 2 half, 2 half + 1
        uint32_t kf[4];
        const uint32_t addr = kb + swz(nb * 8 + (lane & 7), half * 4 + (lane >> 3));
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(kf[0]), "=r"(kf[1]), "=r"(kf[2]), "=r"(kf[3])
                     : "r"(addr));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int kk = half * 2 + u;
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
              "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
              : "+f"(sc[nb][0]), "+f"(sc[nb][1]), "+f"(sc[nb][2]), "+f"(sc[nb][3])
              : "r"(qa[kk][0]), "r"(0u), "r"(qa[kk][1]), "r"(0u), "r"(kf[2 * u]), "r"(kf[2 * u + 1]));
        }
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int pos = c0 + nb * 8 + 2 * t4 + e;
        sc[nb][e] = pos < p1 ? sc[nb][e] * scale : -INFINITY;
        cm = fmaxf(cm, sc[nb][e]);
      }
    }
    // head g8's max and sum over the chunk: its 4 lanes differ in lane bits 0..1
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
    const float mn = fmaxf(m, cm);
    const float alpha = (mn == -INFINITY) ? 1.f : __expf(m - mn);
    float sum = 0.f;
    uint32_t pa[4];  // P as bf16 pairs: block nb, positions 8 nb + 2 t4, + 1
#pragma unroll
    for (int nb = 0; nb < 4; ++nb) {
      const float e0 = (sc[nb][0] == -INFINITY) ? 0.f : __expf(sc[nb][0] - mn);
      const float e1 = (sc[nb][1] == -INFINITY) ? 0.f : __expf(sc[nb][1] - mn);
      sum += e0 + e1;
      __nv_bfloat162 pr = __floats2bfloat162_rn(e0, e1);
      pa[nb] = *reinterpret_cast<uint32_t*>(&pr);
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    l = l * alpha + sum;
    m = mn;
#pragma unroll
    for (int db = 0; db < 8; ++db) {
      o[db][0] *= alpha;
      o[db][1] *= alpha;
    }
    // ---- P . V: two k steps of 16 positions, eight blocks of 8 dims
#pragma unroll
    for (int ks = 0; ks < 2; ++ks) {
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {  // dim pieces 2 dp, 2 dp + 1
        uint32_t vf[4];
        const int row = ks * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
        const uint32_t addr = vb + swz(row, dp * 2 + (lane >> 4));
        asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                     : "=r"(vf[0]), "=r"(vf[1]), "=r"(vf[2]), "=r"(vf[3])
                     : "r"(addr));
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int db = dp * 2 + u;
          asm volatile(
              "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, "
              "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
              : "+f"(o[db][0]), "+f"(o[db][1]), "+f"(o[db][2]), "+f"(o[db][3])
              : "r"(pa[2 * ks]), "r"(0u), "r"(pa[2 * ks + 1]), "r"(0u), "r"(vf[2 * u]), "r"(vf[2 * u + 1]));
        }
      }
    }
}

// Merge the CTA's kAttnCtaWarps warp states (per head: m, l, o[64]) and write
// the CTA's partial for split s of (sequence b, kv head g). The `nthreads`
// threads starting at thread 0 take part; bar_id 0 syncs the whole CTA, any
// other value is a named barrier over those threads.
__device__ __forceinline__ void attn_write_partial(const PagedAttnParams& p,
                                                   float (&st)[kAttnCtaWarps][4][kAttnPartial],
                                                   int warp, int lane, int s, int g, int b, float m,
                                                   float l, const float (&o)[8][4], int nthreads,
                                                   int bar_id) {
  const int g8 = lane >> 2, t4 = lane & 3;
  // ---- merge the warps, write the CTA's partial per head
  if (g8 < 4) {
    if (t4 == 0) {
      st[warp][g8][0] = m;
      st[warp][g8][1] = l;
    }
#pragma unroll
    for (int db = 0; db < 8; ++db) {
      st[warp][g8][2 + db * 8 + 2 * t4] = o[db][0];
      st[warp][g8][3 + db * 8 + 2 * t4] = o[db][1];
    }
  }
  if (bar_id == 0) {
    __syncthreads();
  } else {
    asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(nthreads) : "memory");
  }
  float* dst = p.work + ((((size_t)b * p.NKV + g) * p.splits + s) * 4) * kAttnPartial;
  for (int i = threadIdx.x; i < 4 * 64; i += nthreads) {
    const int hh = i >> 6, d = i & 63;
    float M = -INFINITY;
    for (int w = 0; w < kAttnCtaWarps; ++w) M = fmaxf(M, st[w][hh][0]);
    float L = 0.f, O = 0.f;
    for (int w = 0; w < kAttnCtaWarps; ++w) {
      const float a = (st[w][hh][0] == -INFINITY) ? 0.f : __expf(st[w][hh][0] - M);
      L += st[w][hh][1] * a;
      O += st[w][hh][2 + d] * a;
    }
    if (p.splits == 1) {
      // the only split: the merge kernel would scale by exp(0) = 1, so write
      // the normalised output here and skip it
      p.out[((size_t)b * p.NQ + g * 4 + hh) * 64 + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
      continue;
    }
    if (d == 0) {
      dst[hh * kAttnPartial + 0] = M;
      dst[hh * kAttnPartial + 1] = L;
    }
    dst[hh * kAttnPartial + 2 + d] = O;
  }
}

__global__ void __launch_bounds__(kAttnCtaWarps * 32) paged_attn_kernel(const __grid_constant__ PagedAttnParams p) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ __align__(128) uint8_t asmem[];
  __shared__ float st[kAttnCtaWarps][4][kAttnPartial];     // per-warp states
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int len = p.lengths[b];
  const int p0 = s * p.split_len, p1 = min(len, p0 + p.split_len);
  const uint32_t wbuf = (uint32_t)__cvta_generic_to_shared(asmem) + warp * 4 * kAttnChunkBytes;
  // buffer j (0, 1): K at wbuf + j * 2 * kAttnChunkBytes, V right after it
  const int* table = p.block_tables + (size_t)b * p.max_blocks;
  const int nchunks = p1 > p0 ? (p1 - p0 + 31) / 32 : 0;
  // The split's page ids, staged in shared memory once (when they fit), so
  // issuing a chunk's copies waits on no global load.
  __shared__ int pages_s[kAttnPageCache];
  const int blk0 = p0 / p.ps;
  const int nblk = p1 > p0 ? (p1 - 1) / p.ps - blk0 + 1 : 0;
  const bool staged = nblk <= kAttnPageCache;
  if (staged)
    for (int i = threadIdx.x; i < nblk; i += kAttnCtaWarps * 32) pages_s[i] = table[blk0 + i];
  __syncthreads();
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
        const int page = staged ? pages_s[pos / p.ps - blk0] : table[pos / p.ps];
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

  // Tensor cores (mma.m16n8k16, bf16 in, fp32 accumulate). Scores: S = Q K^T
  // with Q as the A tile (rows 0..3 the group's q heads, rows 4..15 zero)
  // and 8 positions of K per B tile, loaded from the swizzled rows with
  // ldmatrix; lane (g = lane / 4, t = lane % 4) then holds the scores of head
  // g (if g < 4) at positions 8 nb + 2 t, + 1. P . V: the scores' accumulator
  // layout is the A layout of P (16 positions per k step, P rounded to bf16)
  // and V comes in with ldmatrix.trans; O rows 0..3 are the heads, lane
  // (g, t) holds dims 8 db + 2 t, + 1 of head g in o[db].
  const int g8 = lane >> 2, t4 = lane & 3;
  uint32_t qa[4][2];  // k step kk: dims 16 kk + 2 t4 (+1) and 16 kk + 8 + 2 t4 (+1) of head g8
  {
    const __nv_bfloat16* qh = p.q + ((size_t)b * p.NQ + g * 4 + (g8 & 3)) * 64;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t lo = __ldg(reinterpret_cast<const uint32_t*>(qh + 16 * kk + 2 * t4));
      const uint32_t hi = __ldg(reinterpret_cast<const uint32_t*>(qh + 16 * kk + 8 + 2 * t4));
      qa[kk][0] = g8 < 4 ? lo : 0u;
      qa[kk][1] = g8 < 4 ? hi : 0u;
    }
  }
  float m = -INFINITY, l = 0.f;  // head g8's running max and sum (same in its 4 lanes)
  float o[8][4];
#pragma unroll
  for (int db = 0; db < 8; ++db) o[db][0] = o[db][1] = o[db][2] = o[db][3] = 0.f;

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
    attn_chunk_mma(wbuf + j * 2 * kAttnChunkBytes, wbuf + j * 2 * kAttnChunkBytes + kAttnChunkBytes,
                   p0 + ci * 32, p1, p.scale, qa, m, l, o, lane);
    __syncwarp();
  }
  attn_write_partial(p, st, warp, lane, s, g, b, m, l, o, kAttnCtaWarps * 32, 0);
}

// ---------------------------------------------------------------- TMA pipeline
//
// The same split-K attention for page sizes that are multiples of 32 (every
// 32-position chunk lies inside one page, so its K rows and its V rows are
// each one contiguous 4 KB run of the pool). A fifth warp streams the chunks
// of the split with 2-D TMA boxes of 32 rows x 128 bytes into a ring of
// kAttnStages stages (K box then V box per stage, 128-byte swizzle: the same
// XOR layout as swz), each stage guarded by a full / empty mbarrier pair, and
// runs ahead of the four consumer warps by the ring's depth instead of one
// chunk per warp; the consumers take chunks warp, warp + 4, ... as before.
constexpr int kAttnStages = 8;  // a multiple of kAttnCtaWarps: a stage is always reused by the same warp
constexpr int kAttnStageBytes = 2 * kAttnChunkBytes;
constexpr int kAttnTmaSmem = kAttnStages * kAttnStageBytes + 1024;  // + alignment to the 1 KB swizzle atom
static_assert(kAttnStages % kAttnCtaWarps == 0, "a stage is reused by the warp that last read it");

struct alignas(64) PagedAttnTmaParams {
  CUtensorMap tm_k;  // the layer's K pool as rows of 64 bf16: dims {64, pages * NKV * ps}, box {64, 32}
  CUtensorMap tm_v;
  PagedAttnParams p;
};

__device__ __forceinline__ bool attn_bar_wait(uint32_t bar, uint32_t parity, unsigned long long limit_ns,
                                              const int* error) {
  uint32_t ok;
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    asm volatile(
        "{\n\t.reg .pred q;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 q, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    if (ok) return true;
    if ((it & 15) == 15) {
      if (*reinterpret_cast<const volatile int*>(error)) return false;
      uint64_t now;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(now));
      if (!t0) {
        t0 = now;
      } else if (now - t0 > limit_ns) {
        return false;
      }
    }
  }
}

__global__ void __launch_bounds__((kAttnCtaWarps + 1) * 32)
    paged_attn_tma_kernel(const __grid_constant__ PagedAttnTmaParams tp) {
  const PagedAttnParams& p = tp.p;
  pdl_trigger();
  extern __shared__ __align__(1024) uint8_t tsmem[];
  __shared__ float st[kAttnCtaWarps][4][kAttnPartial];
  __shared__ __align__(8) uint64_t full[kAttnStages], empty[kAttnStages];
  __shared__ int pages_s[kAttnPageCache];
  const int s = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ring = ((uint32_t)__cvta_generic_to_shared(tsmem) + 1023) & ~1023u;
  auto sa = [](uint64_t* x) { return (uint32_t)__cvta_generic_to_shared(x); };
  if (threadIdx.x == 0) {
    for (int i = 0; i < kAttnStages; ++i) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&full[i])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&empty[i])));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  pdl_wait();
  const int len = p.lengths[b];
  const int p0 = s * p.split_len, p1 = min(len, p0 + p.split_len);
  const int nchunks = p1 > p0 ? (p1 - p0 + 31) / 32 : 0;
  const int* table = p.block_tables + (size_t)b * p.max_blocks;
  const int blk0 = p0 / p.ps;
  const int nblk = p1 > p0 ? (p1 - 1) / p.ps - blk0 + 1 : 0;
  const bool staged = nblk <= kAttnPageCache;
  if (staged)
    for (int i = threadIdx.x; i < nblk; i += blockDim.x) pages_s[i] = table[blk0 + i];
  __syncthreads();
  const unsigned long long limit = 2000000000ull;

  if (warp == kAttnCtaWarps) {
    // ---- producer: one lane issues the split's chunks into the ring
    if (lane == 0) {
      int issued = 0;
      for (int ci = 0; ci < nchunks; ++ci) {
        const int st_i = ci % kAttnStages;
        if (ci >= kAttnStages &&
            !attn_bar_wait(sa(&empty[st_i]), ((ci / kAttnStages) + 1) & 1, limit, p.error)) {
          atomicCAS(p.error, 0, 2);
          break;
        }
        const int pos = p0 + ci * 32;
        const int page = staged ? pages_s[pos / p.ps - blk0] : table[pos / p.ps];
        const uint32_t kdst = ring + st_i * kAttnStageBytes, vdst = kdst + kAttnChunkBytes;
        if (page < 0 || page >= p.num_pages) {
          // never read outside the pool: complete the stage without data
          atomicExch(p.error, 1);
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(&full[st_i])) : "memory");
          ++issued;
          continue;
        }
        const int row = (page * p.NKV + g) * p.ps + pos % p.ps;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(&full[st_i])),
                     "r"(kAttnStageBytes)
                     : "memory");
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4}], [%2];" ::"r"(kdst),
            "l"(&tp.tm_k), "r"(sa(&full[st_i])), "r"(0), "r"(row)
            : "memory");
        asm volatile(
            "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
            " [%0], [%1, {%3, %4}], [%2];" ::"r"(vdst),
            "l"(&tp.tm_v), "r"(sa(&full[st_i])), "r"(0), "r"(row)
            : "memory");
        ++issued;
      }
      // every box issued lands before the CTA may exit (bounded)
      for (int ci = (issued > kAttnStages ? issued - kAttnStages : 0); ci < issued; ++ci)
        attn_bar_wait(sa(&full[ci % kAttnStages]), (ci / kAttnStages) & 1, 2 * limit, p.error);
    }
    return;
  }

  // ---- consumers (4 warps), as paged_attn_kernel
  const int g8 = lane >> 2, t4 = lane & 3;
  uint32_t qa[4][2];
  {
    const __nv_bfloat16* qh = p.q + ((size_t)b * p.NQ + g * 4 + (g8 & 3)) * 64;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const uint32_t lo = __ldg(reinterpret_cast<const uint32_t*>(qh + 16 * kk + 2 * t4));
      const uint32_t hi = __ldg(reinterpret_cast<const uint32_t*>(qh + 16 * kk + 8 + 2 * t4));
      qa[kk][0] = g8 < 4 ? lo : 0u;
      qa[kk][1] = g8 < 4 ? hi : 0u;
    }
  }
  float m = -INFINITY, l = 0.f;
  float o[8][4];
#pragma unroll
  for (int db = 0; db < 8; ++db) o[db][0] = o[db][1] = o[db][2] = o[db][3] = 0.f;
  for (int ci = warp; ci < nchunks; ci += kAttnCtaWarps) {
    const int st_i = ci % kAttnStages;
    if (!attn_bar_wait(sa(&full[st_i]), (ci / kAttnStages) & 1, limit, p.error)) {
      atomicCAS(p.error, 0, 2);
      break;
    }
    const uint32_t kb = ring + st_i * kAttnStageBytes;
    attn_chunk_mma(kb, kb + kAttnChunkBytes, p0 + ci * 32, p1, p.scale, qa, m, l, o, lane);
    __syncwarp();
    if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sa(&empty[st_i])) : "memory");
  }
  attn_write_partial(p, st, warp, lane, s, g, b, m, l, o, kAttnCtaWarps * 32, 1);
}

__global__ void __launch_bounds__(256) paged_attn_merge_kernel(const __grid_constant__ PagedAttnParams p) {
  pdl_trigger();
  pdl_wait();
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
