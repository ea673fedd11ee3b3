// Skinny GEMM on the 5th-generation tensor cores for the batched decode path:
//   Y[B][N] = X[B][K] . W[N][K]^T (+ R[B][N]),  bf16 in, fp32 accumulate.
//
// At bs 8-64 the decode projections are "skinny" GEMMs: W (the weights, N x
// K, K contiguous) is large and read once, X (the activations) has 8-64 rows.
// One CTA computes a 128-row tile of W against all of X:
//  * A = the W tile (128 rows; past N the TMA fills zeros), B = X (BP rows:
//    the batch padded to 16, 32 or 64 with zero rows), both K-major with the
//    128-byte swizzle (BP = 128 for prompt prefill: 128 token rows), loaded by 2-D
//    TMA boxes of 64 columns (no multicast) into a ring of kGemmStages stages
//    (kGemmStagesDeep when the launch puts at most one CTA on each SM)
//    with full/empty mbarriers;
//  * one lane issues tcgen05.mma (kind::f16, bf16 x bf16 -> fp32, M = 128,
//    N = BP, K = 16; four per 64-column stage) into a TMEM accumulator of BP
//    columns; tcgen05.commit frees each stage and finally signals the
//    epilogue;
//  * four warps read the accumulator back 32 columns at a time
//    (tcgen05.ld.32x32b: warp w owns TMEM lanes = W rows 32w..32w+31) and
//    write Y[b][n] (coalesced along n);
//  * narrow W (16-24 tiles for 148 SMs) is split along K over the CTAs of a
//    thread-block cluster (at most 8, one cluster per tile): each CTA stages
//    its fp32 accumulator in its (then idle) ring memory, and after a cluster
//    barrier rank r adds slice r of the tile over all ranks' stages through
//    distributed shared memory, in split order, adds the residual and rounds
//    once to bf16 — no partial sums in global memory, no second kernel.
// Every mbarrier wait is time-bounded (flag + early exit), and a CTA waits for
// its own in-flight copies and MMAs before it releases shared memory and TMEM.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "mk_device.cuh"

namespace mk {

constexpr int kGemmStages = 4;      // 96 KB at 64 rows: two CTAs per SM overlap one tile's epilogue with the next's loads
constexpr int kGemmStagesDeep = 8;  // a launch of at most one CTA per SM: twice the bytes in flight
constexpr int kGemmTileN = 128;  // W rows per CTA (the MMA's M)
constexpr int kGemmTileK = 64;   // columns per stage: one 128-byte swizzle atom per row
constexpr int kGemmThreads = 128;

struct GemmParams {
  CUtensorMap tm_w;  // W [N][K] bf16: dims {K, N}, box {64, 128}, 128B swizzle
  CUtensorMap tm_x;  // X [BP][K] bf16: dims {K, BP}, box {64, BP}, 128B swizzle
  int N, K, B;       // B: real rows of X (<= BP)
  int kblocks_per_split;
  int splits;                     // CTAs along K = the cluster size (1: no split)
  const __nv_bfloat16* residual;  // [B][N] or null
  __nv_bfloat16* out;             // [B][N] bf16 (no split)
  float* out_f32;                 // [B][N] fp32 (e.g. logits)
  int* error;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void g_tma_load_2d(uint32_t dst, const CUtensorMap* tm, int c0, int c1,
                                              uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(tm), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ bool g_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t g_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait; false (and the error flag = `where`: 101 producer, 102 MMA
// issuer, 103 epilogue) when it runs out.
__device__ __noinline__ bool g_wait(const GemmParams& p, uint32_t bar, uint32_t parity, int where) {
  if (g_try_wait(bar, parity)) return true;
  const uint64_t t0 = g_now();
  for (uint32_t it = 0;; ++it) {
    if (g_try_wait(bar, parity)) return true;
    if ((it & 15) == 15) {
      if (*reinterpret_cast<volatile int*>(p.error)) return false;
      if (g_now() - t0 > p.timeout_ns) {
        atomicCAS(p.error, 0, where);
        return false;
      }
    }
  }
}

// Shared-memory descriptor of a K-major, 128-byte-swizzled operand tile:
// rows 128 bytes apart, 8-row groups 1024 bytes apart (SBO), version 1,
// layout SWIZZLE_128B (2). The K step inside the atom adds 32 bytes.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFF) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

template <int BP>
__device__ __forceinline__ constexpr uint32_t gemm_idesc() {
  // c_format f32 (bit 4), a/b format bf16 (bits 7, 10), K-major A and B,
  // N >> 3 at bit 17, M >> 4 at bit 24
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BP >> 3) << 17) |
         ((uint32_t)(kGemmTileN >> 4) << 24);
}

// CB (16 or 32) consecutive fp32 accumulator columns of this thread's TMEM lane.
template <int CB>
__device__ __forceinline__ void tmem_ld_chunk(uint32_t taddr, float (&v)[CB]) {
  uint32_t r[CB];
  if constexpr (CB == 16) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
  } else {
    static_assert(CB == 32, "chunks of 16 or 32 columns");
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
        "%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
  }
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < CB; ++i) v[i] = __uint_as_float(r[i]);
}

// One output element: fp32 as is, or rounded to bf16 and, with a residual,
// added to it and rounded again (HF's decoder layer: h = bf16(h + bf16(W a))).
__device__ __forceinline__ void g_store(const GemmParams& p, size_t o, float y) {
  if (p.out_f32) {
    p.out_f32[o] = y;
    return;
  }
  if (p.residual) y = __bfloat162float(__float2bfloat16_rn(y)) + __bfloat162float(p.residual[o]);
  p.out[o] = __float2bfloat16_rn(y);
}

template <int BP, int kStages>
__global__ void __launch_bounds__(kGemmThreads) gemm_kernel(const __grid_constant__ GemmParams p) {
  extern __shared__ __align__(1024) uint8_t gsm[];
  constexpr uint32_t kA = kGemmTileN * kGemmTileK * 2;  // 16 KB
  constexpr uint32_t kB = BP * kGemmTileK * 2;
  constexpr uint32_t kStage = kA + kB;
  static_assert(kStage % 1024 == 0, "stage buffers keep the 1024-byte swizzle alignment");
  const uint32_t base = (uint32_t)__cvta_generic_to_shared(gsm);
  const uint32_t ring = (base + 1023) & ~1023u;
  __shared__ __align__(8) uint64_t full[kStages], empty[kStages], done;
  __shared__ uint32_t tmem_base;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int kb0 = split * p.kblocks_per_split;
  const int kb1 = min(p.K / kGemmTileK, kb0 + p.kblocks_per_split);
  const int nk = kb1 - kb0;
  auto sa = [](uint64_t* b) { return (uint32_t)__cvta_generic_to_shared(b); };
  pdl_trigger();  // barrier init and TMEM allocation below overlap the previous kernel

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&full[s])));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&empty[s])));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sa(&done)));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // TMEM: BP fp32 columns (at least 32)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     (uint32_t)__cvta_generic_to_shared(&tmem_base)),
                 "r"((uint32_t)(BP < 32 ? 32 : BP))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = tmem_base;
  pdl_wait();  // X (and the residual) come from the previous kernel

  if (warp == 0 && lane == 0) {
    // ---- producer: TMA boxes of W rows [tile*128, +128) and all X rows
    int issued = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % kStages;
      if (i >= kStages && !g_wait(p, sa(&empty[s]), ((i / kStages) + 1) & 1, 101)) break;
      const uint32_t a = ring + s * kStage, b = a + kA;
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sa(&full[s])),
                   "r"(kStage)
                   : "memory");
      g_tma_load_2d(a, &p.tm_w, (kb0 + i) * kGemmTileK, tile * kGemmTileN, sa(&full[s]));
      g_tma_load_2d(b, &p.tm_x, (kb0 + i) * kGemmTileK, 0, sa(&full[s]));
      ++issued;
    }
    // every box issued lands before the CTA may exit (bounded)
    for (int i = (issued > kStages ? issued - kStages : 0); i < issued; ++i) {
      const int s = i % kStages;
      const uint32_t par = (i / kStages) & 1;
      const uint64_t t0 = g_now();
      while (!g_try_wait(sa(&full[s]), par) && g_now() - t0 < 2 * p.timeout_ns) {
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer
    constexpr uint32_t idesc = gemm_idesc<BP>();
    bool ok = true;
    for (int i = 0; i < nk && ok; ++i) {
      const int s = i % kStages;
      if (!g_wait(p, sa(&full[s]), (i / kStages) & 1, 102)) {
        ok = false;
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const uint32_t a = ring + s * kStage, b = a + kA;
#pragma unroll
      for (int kk = 0; kk < kGemmTileK / 16; ++kk) {
        const uint64_t da = sw128_desc(a + kk * 32), db = sw128_desc(b + kk * 32);
        const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "setp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
            ::"r"(tmem), "l"(da), "l"(db), "r"(idesc), "r"(acc)
            : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       sa(&empty[s]))
                   : "memory");
    }
    // the accumulator is complete when every MMA issued so far is
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     sa(&done))
                 : "memory");
  }
  __syncwarp();

  // ---- epilogue: warp w reads TMEM lanes 32w..32w+31 = W rows of the tile
  const bool good = g_wait(p, sa(&done), 0, 103) && nk > 0;
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  constexpr int CB = BP < 32 ? BP : 32;  // accumulator columns read per tcgen05.ld
  const uint32_t tlane = tmem + ((uint32_t)(warp * 32) << 16);
  if (p.splits == 1) {
    const int n = tile * kGemmTileN + warp * 32 + lane;
    for (int c0 = 0; c0 < BP && c0 < p.B; c0 += CB) {  // warp-uniform: the loads stay aligned
      float v[CB];
      tmem_ld_chunk<CB>(tlane + c0, v);
      if (good && n < p.N) {  // rows past N (the last tile's) were zero-filled by TMA
#pragma unroll
        for (int b = 0; b < CB; ++b) {
          if (c0 + b >= p.B) break;
          g_store(p, (size_t)(c0 + b) * p.N + n, v[b]);
        }
      }
    }
  } else {
    // Stage the accumulator as [b][row] (consecutive threads, consecutive
    // words), then rank `split` sums its slice of the B x 128 outputs over
    // the cluster's stages in split order. Both cluster barriers are reached
    // by every thread on every path, so no CTA waits for one that left.
    const int r = warp * 32 + lane;
    for (int c0 = 0; c0 < BP; c0 += CB) {
      float v[CB];
      tmem_ld_chunk<CB>(tlane + c0, v);
#pragma unroll
      for (int b = 0; b < CB; ++b)
        asm volatile("st.shared.f32 [%0], %1;" ::"r"(ring + (uint32_t)((c0 + b) * kGemmTileN + r) * 4),
                     "f"(good ? v[b] : 0.f)
                     : "memory");
    }
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
    const int E = p.B * kGemmTileN;
    const int e1 = (split + 1) * E / p.splits;
    for (int i = split * E / p.splits + threadIdx.x; i < e1; i += kGemmThreads) {
      const uint32_t local = ring + (uint32_t)i * 4;
      float y = 0.f;
      for (int q = 0; q < p.splits; ++q) {
        uint32_t remote;
        float t;
        asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local), "r"(q));
        asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(t) : "r"(remote) : "memory");
        y += t;
      }
      const int n = tile * kGemmTileN + (i % kGemmTileN);
      if (good && n < p.N) g_store(p, (size_t)(i / kGemmTileN) * p.N + n, y);
    }
    __syncwarp();
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                     : "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0) {
    // The issuer committed `done` before this barrier; it arrives once its
    // MMAs have finished, so TMEM is released only after them (bounded).
    if (!good) {
      const uint64_t t0 = g_now();
      while (!g_try_wait(sa(&done), 0) && g_now() - t0 < 2 * p.timeout_ns) {
      }
    }
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"((uint32_t)(BP < 32 ? 32 : BP))
                 : "memory");
  }
}

}  // namespace mk
