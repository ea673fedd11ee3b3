// mk_device.cuh — device helpers for the decode megakernel (sm_100a).
//
// mbarrier + bulk-copy (TMA, non-tensor) primitives written as inline PTX,
// acquire/release global atomics for the cross-CTA counters, bf16
// conversion helpers and a time-bounded wait policy. Nothing here spins
// without a limit: every wait checks the global timer and a shared abort word.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

namespace mk {

constexpr int kHeadDim = 64;
constexpr int kGroup = 4;                  // q heads per kv head
constexpr int kSlotBytes = 16384;          // one ring slot
// 14 consumer + 2 producer warps: 16 warps keep 128 registers per thread
// (the register file is split over four schedulers, 16K registers each).
constexpr int kConsumerWarps = 14;
constexpr int kConsumerThreads = kConsumerWarps * 32;
constexpr int kAttnWarps = 8;              // warp states kept for the attention merge
// Ring copies are issued by kProducers lanes (lane 0 of warps kConsumerWarps
// .. + kProducers - 1), producer k taking the fills f with f % kProducers == k:
// one lane issues at most ~50 GB/s of 16 KB bulk copies.
constexpr int kProducers = 2;
// Full barriers of the ring, used round-robin by the fills, so a barrier is
// reused only every kFullBars fills; a producer issues fill f only once the
// other has walked past fill f - kProducerSlack (see the Ring comment in
// mk_kernel.cuh for why both bound a consumer warp's gap between waits).
constexpr int kFullBars = 64;
constexpr int kProducerSlack = 8;
// Tensor parallelism: at most this many GPUs share one decode step.
constexpr int kMaxTp = 8;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kThreads = kConsumerThreads + kProducers * 32;
constexpr int kSegCols = 2048;             // max columns of one piece (a row segment)
// Cached positions per attention slot: four per consumer warp, so every warp
// takes one round of a full chunk (K rows in the slot's first 8 KB, V in its second).
constexpr int kAttnChunk = 4 * kConsumerWarps;
static_assert(kAttnChunk * kHeadDim * 2 <= kSlotBytes / 2, "a chunk's K rows must fit half a slot");
constexpr int kMaxSplit = 32;              // split-K pieces per (sequence, kv head)
constexpr int kSplitMinPositions = 128;    // no split shorter than this (~3 chunks)
constexpr int kPartialStride = kHeadDim + 2;  // o[64], m, l per q head

// Device error codes (error word [0]).
enum DevErr : int {
  kErrNone = 0,
  kErrBarrierTimeout = 1,
  kErrRingTimeout = 2,
  kErrPosition = 3,
  kErrPage = 4,
  kErrToken = 5,
};

// Counters in the scratch counter block.
enum Counter : int {
  kCntDone = 2,  // CTAs finished with the step (the last publishes the argmax)
  kCounters = 4,  // words in the counter block
};

// Programmatic dependent launch (the batched path's kernels, launched with
// the programmatic-serialization attribute): pdl_trigger lets the next kernel
// of the stream start its prologue; pdl_wait blocks until the kernels this one
// depends on have finished and their writes are visible (without the
// attribute both are no-ops). A kernel touches no global memory before
// pdl_wait.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 64-bit words exchanged with the other GPUs of a tensor-parallel group
// (peer memory mapped through CUDA IPC, carried by NVLink): system scope.
__device__ __forceinline__ void st_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Shared-memory word handed between threads of the CTA with release/acquire order.
__device__ __forceinline__ void st_release_shared(uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_addr(p)), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_shared(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_addr(p)) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// ---------------------------------------------------------------- bulk copy

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// global -> shared bulk copy (TMA engine, no tensor map), completion counted
// in bytes on `bar`. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_g2s_nohint(void* dst, const void* src, uint32_t bytes,
                                                uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// 128-bit shared-memory load at a shared-window address. volatile: it must stay
// after the mbarrier wait that made the bulk-copied bytes visible.
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// mbarrier arrive counting `count` arrivals at once.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count)
               : "memory");
}

// ---------------------------------------------------------------- global sync

__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_add_u32(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Atomic add with acquire+release semantics at GPU scope (arrival counters
// whose last arriver reads what the others wrote).
__device__ __forceinline__ uint32_t atom_add_acq_rel_u32(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ int ld_volatile_i32(const int* p) {
  return *reinterpret_cast<const volatile int*>(p);
}

// Named barrier over the consumer warps only (the producer warp never joins).
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kConsumerThreads) : "memory");
}

// Named barrier over the consumer warps that also ORs a predicate across them:
// every consumer thread gets the same answer, so failure exits stay
// collective and no warp is left waiting at a later barrier.
__device__ __forceinline__ bool consumer_any(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, 1, %2, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)v), "n"(kConsumerThreads)
      : "memory");
  return r != 0;
}

// ---------------------------------------------------------------- bf16 math

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ float bf2f(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ __nv_bfloat16 f2bf(float v) { return __float2bfloat16_rn(v); }
// Round to bf16 and back: the value a bf16 tensor op would store.
__device__ __forceinline__ float rbf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

// c0 += lo(a) * lo(b), c1 += hi(a) * hi(b) for packed bf16 pairs, in fp32:
// the products of two bf16 values are exact in fp32, so this equals an fp32
// FMA of the widened operands.
__device__ __forceinline__ void fma2_bf16(uint32_t a, uint32_t b, float& c0, float& c1) {
  asm("{\n\t.reg .b16 al, ah, bl, bh;\n\t"
      "mov.b32 {al, ah}, %2;\n\t"
      "mov.b32 {bl, bh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, al, bl, %0;\n\t"
      "fma.rn.f32.bf16 %1, ah, bh, %1;\n\t}"
      : "+f"(c0), "+f"(c1)
      : "r"(a), "r"(b));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Order-preserving map of an fp32 value to uint32 (for packed argmax keys).
__device__ __forceinline__ uint32_t float_key(float v) {
  uint32_t b = __float_as_uint(v);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

}  // namespace mk
