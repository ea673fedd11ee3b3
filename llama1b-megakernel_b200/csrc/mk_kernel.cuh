// mk_kernel.cuh — the persistent decode megakernel (sm_100a).
//
// One cooperative launch, one CTA per SM, decodes a token for each of B
// sequences through every decoder layer, then the final norm, the tied
// lm_head and a greedy argmax.
//
// CTA = 8 consumer warps + 1 producer warp.
//
// * The producer (one lane) walks the CTA's whole schedule of HBM reads for
//   the step — its slice of every weight matrix of every layer, its KV-cache
//   chunks, its lm_head rows — and streams them with bulk copies
//   (cp.async.bulk, the TMA engine without a tensor map) into a ring of 16 KB
//   shared-memory slots, each guarded by a full/empty mbarrier pair. Weights
//   and cached K/V do not depend on activations, so the producer never waits
//   for a grid barrier: it runs ahead by the ring's depth (~190 KB per SM) and
//   keeps HBM busy while the consumers sit in phase barriers.
// * The consumers walk the same schedule. Each phase starts by reading the
//   activation vector it needs (bf16 residual, q/k/v, attention output or the
//   SwiGLU product, all L2-resident) into shared memory, RMS-normalising it
//   where the layer does, then reduces each streamed weight row against it
//   (one warp per row or row pair, fp32 accumulation, warp-shuffle reduction)
//   and writes the phase output.
//
// Phases per layer (grid barrier = acquire/release counter, time-bounded):
//   QKV    RMSNorm(h), q/k/v rows in RoPE pairs (d, d+32), llama3 RoPE from a
//          bf16 cos/sin table, K/V row scattered into the paged cache.
//   ATTN   split-K GQA flash-decode: item (seq, kv head, position range) per
//          CTA, online softmax per warp, CTA merge, then the last CTA to
//          finish a (seq, kv head) merges the splits plus the new token's own
//          K/V and publishes the head (counter, no full barrier).
//   O      o_proj rows + residual add into h.
//   GU     RMSNorm(h), gate/up row pairs, SiLU(gate) * up.
//   DOWN   down rows + residual add into h.
// then LM: final RMSNorm, lm_head rows, fp32 logits, packed 64-bit atomicMax
// argmax; the last CTA to finish publishes the ids and resets the counters.
//
// Rounding mirrors HF Llama in bf16 (the reference's PyTorch path): every
// linear output, RMSNorm output, RoPE product/sum, SiLU output, SwiGLU product
// and residual sum is rounded to bf16 where the torch graph stores bf16;
// reductions accumulate in fp32. Logits stay fp32.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "mk_device.cuh"

namespace mk {

using bf16 = __nv_bfloat16;

struct Params {
  // geometry
  int L, H, I, NQ, NKV, V;
  float eps;
  int B;
  int page_size, num_pages, max_blocks, rope_len;
  int num_slots;
  int kmax;  // max(H, I, NQ*64): stride of the activation rows in shared memory
  int mode;  // 0: full step (embedding .. argmax); 1: decoder layers only
  int flags;
  // weights (packed, see mk.h)
  const bf16* embed;
  const bf16* w_qkv;
  const bf16* w_o;
  const bf16* w_gu;
  const bf16* w_down;
  const bf16* norm_attn;
  const bf16* norm_mlp;
  const bf16* norm_final;
  const bf16* rope_cos;
  const bf16* rope_sin;
  // KV cache
  bf16* k_pages;
  bf16* v_pages;
  const int* block_tables;
  // step I/O
  int* tokens;
  int* positions;
  const bf16* hidden_in;
  bf16* hidden_out;
  float* logits;
  int* next_ids;
  // scratch (owned by the model handle)
  bf16* h;         // [B][H]
  bf16* qkv;       // [B][NQ + 2 NKV][64]
  bf16* attn;      // [B][NQ * 64]
  bf16* act;       // [B][I]
  float* partials; // [B][NKV][kMaxSplit][kGroup][kPartialStride]
  uint32_t* counters;
  unsigned long long* keys;  // [B]
  int* error;                // [4] code, detail, cta, thread (device)
  int* host_error;           // [4] mapped pinned host mirror of `error`
  unsigned long long timeout_ns;
  int debug_skip_cta;
  // optional phase trace ([grid][trace_per_cta] u64, see kTrace*); nullptr = off
  unsigned long long* trace;
  int trace_per_cta;
};

// Phase trace. Phase index: layer * 5 + {0 QKV, 1 ATTN, 2 O, 3 GU, 4 DOWN},
// num_layers * 5 = LM head. Per (CTA, phase) kTraceKinds u64 entries:
enum TraceKind : int {
  kTrWaitStart = 0,    // consumers reach the phase's grid wait (globaltimer ns)
  kTrWaitDone = 1,     // wait passed
  kTrRowsLoaded = 2,   // activation rows in shared memory (normalised)
  kTrDone = 3,         // consumers finished the phase
  kTrConsStall = 4,    // cumulative ns warp 0 waited for ring data, at phase end
  kTrProdStart = 5,    // producer issues the phase's first copy
  kTrProdStall = 6,    // cumulative ns the producer waited for a free slot
  kTrProdEnd = 7,      // producer issued the phase's last copy
  kTraceKinds = 8,
};

__device__ __forceinline__ void trace_put(const Params& p, int phase, int kind,
                                          unsigned long long v) {
  if (p.trace) p.trace[(size_t)blockIdx.x * p.trace_per_cta + phase * kTraceKinds + kind] = v;
}

struct SmemState {
  int tok[4];
  int pos[4];
  int n_split;
  int flag;
  int pad[6];
  float red[kConsumerWarps * 4];
  float am_val[kConsumerWarps * 4];
  int am_idx[kConsumerWarps * 4];
};

// Shared-memory layout (dynamic): [ring S x 16 KB][x rows B x kmax bf16]
// [attention scratch][mbarriers 2 x S][SmemState]
constexpr int kAttnScratchBytes =
    kConsumerWarps * kGroup * kPartialStride * 4 + kGroup * kHeadDim * 2 + 2 * kHeadDim * 4;

__host__ __device__ inline int smem_bytes_for(int num_slots, int B, int kmax) {
  int x = B * kmax * 2;
  x = (x + 127) & ~127;
  return num_slots * kSlotBytes + x + kAttnScratchBytes + 2 * num_slots * 8 +
         (int)sizeof(SmemState) + 128;
}

// ---------------------------------------------------------------- errors

__device__ __noinline__ void raise_error(const Params& p, int code, int where) {
  if (atomicCAS(p.error, 0, code) == 0) {
    p.error[1] = where;
    p.error[2] = blockIdx.x;
    p.error[3] = threadIdx.x;
    volatile int* he = p.host_error;
    he[1] = where;
    he[2] = blockIdx.x;
    he[3] = threadIdx.x;
    __threadfence_system();
    he[0] = code;
  }
}

__device__ __forceinline__ bool aborted(const Params& p) { return ld_volatile_i32(p.error) != 0; }

// Spin until *c >= target (wrap-safe). false on timeout or abort.
__device__ __noinline__ bool counter_wait(const Params& p, const uint32_t* c, uint32_t target,
                                          int where) {
  uint64_t t0 = 0;
  for (uint32_t it = 0;; ++it) {
    if ((int32_t)(ld_acquire_u32(c) - target) >= 0) return true;
    if ((it & 15) == 15) {
      if (aborted(p)) return false;
      const uint64_t now = global_ns();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > p.timeout_ns) {
        raise_error(p, kErrBarrierTimeout, where);
        return false;
      }
    }
  }
}

__device__ __noinline__ bool mbar_wait(const Params& p, uint64_t* bar, uint32_t parity, int where,
                                       unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 0;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 7) == 7) {
      if (where >= 0 && aborted(p)) return false;
      if (global_ns() - t0 > limit_ns) {
        if (where >= 0) raise_error(p, kErrRingTimeout, where);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------- schedule

// Units [u0, u1) of a phase with U units for CTA c of G. CTAs in the cyclic
// interval [rot, rot + U % G) take one extra unit; the next phase starts its
// interval where this one ended, so every CTA's running total of streamed
// bytes stays within one unit of every other's.
struct Split {
  int u0, u1;
};

__device__ __forceinline__ Split split_units(int U, int G, int c, int rot) {
  const int base = U / G, rem = U % G;
  const int end = rot + rem;
  int before;
  if (end <= G) {
    before = min(max(c - rot, 0), rem);
  } else {
    before = min(c, end - G) + min(max(c - rot, 0), G - rot);
  }
  const bool extra = ((c - rot + G) % G) < rem;
  const int u0 = c * base + before;
  return {u0, u0 + base + (extra ? 1 : 0)};
}

struct Sched {
  int rot = 0;
  __device__ __forceinline__ Split next(int U) {
    const Split s = split_units(U, gridDim.x, blockIdx.x, rot);
    rot = (rot + U % (int)gridDim.x) % (int)gridDim.x;
    return s;
  }
};

__device__ __forceinline__ int units_per_slot(int unit_bytes) {
  return max(1, kSlotBytes / unit_bytes);
}

// Item -> (seq, kv head, split) and its cached-position range [p0, p1).
struct AttnItem {
  int b, g, s, p0, p1;
};

__device__ __forceinline__ AttnItem attn_item(const Params& p, const SmemState& st, int it) {
  AttnItem a;
  const int ns = st.n_split;
  a.b = it / (p.NKV * ns);
  a.g = (it / ns) % p.NKV;
  a.s = it % ns;
  const long long pos = st.pos[a.b];
  a.p0 = (int)(pos * a.s / ns);
  a.p1 = (int)(pos * (a.s + 1) / ns);
  return a;
}

// ---------------------------------------------------------------- ring

struct Ring {
  uint8_t* slots;
  uint64_t* full;
  uint64_t* empty;
  int S;
  uint32_t n = 0;  // fills seen so far (same count on both sides)
  unsigned long long stall_ns = 0;  // time spent waiting (traced runs only)
};

// Consumer warp: wait for fill n; nullptr on abort/timeout. Every lane waits
// on the mbarrier itself; lane 0 alone decides to give up and the decision is
// broadcast, so the result is uniform across the warp.
__device__ __noinline__ const uint8_t* ring_wait(const Params& p, Ring& r, int where) {
  const int slot = r.n % r.S;
  const uint32_t parity = (r.n / r.S) & 1;
  uint64_t* bar = &r.full[slot];
  bool done = mbar_try_wait(bar, parity);
  uint64_t t0 = 0;
  const uint64_t ts = (p.trace && !__all_sync(0xffffffffu, done)) ? global_ns() : 0;
  for (uint32_t it = 0; !__all_sync(0xffffffffu, done); ++it) {
    if (!done) done = mbar_try_wait(bar, parity);
    int give_up = 0;
    if ((it & 7) == 7 && (threadIdx.x & 31) == 0) {
      const uint64_t now = global_ns();
      if (t0 == 0) t0 = now;
      if (aborted(p)) {
        give_up = 1;
      } else if (now - t0 > p.timeout_ns) {
        raise_error(p, kErrRingTimeout, where);
        give_up = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, give_up, 0)) return nullptr;
  }
  if (ts) r.stall_ns += global_ns() - ts;
  return r.slots + (size_t)slot * kSlotBytes;
}

__device__ __forceinline__ void ring_release(Ring& r) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&r.empty[r.n % r.S]);
  r.n++;
}

// ---------------------------------------------------------------- producer

struct Producer {
  const Params& p;
  Ring& r;
  uint64_t pol;
  bool ok = true;

  // Claim the next slot for `bytes` of transfers; nullptr when aborting.
  __device__ uint8_t* begin(uint32_t bytes) {
    if (!ok) return nullptr;
    const int slot = r.n % r.S;
    if (r.n >= (uint32_t)r.S) {
      const uint32_t parity = ((r.n / r.S) + 1) & 1;
      const uint64_t ts = p.trace ? global_ns() : 0;
      if (!mbar_wait(p, &r.empty[slot], parity, 100, p.timeout_ns)) {
        ok = false;
        return nullptr;
      }
      if (ts) r.stall_ns += global_ns() - ts;
    }
    mbar_arrive_expect_tx(&r.full[slot], bytes);
    return r.slots + (size_t)slot * kSlotBytes;
  }
  __device__ uint64_t* bar() { return &r.full[r.n % r.S]; }
  __device__ void end() { r.n++; }

  // Stream units [u0, u1) of `unit_bytes` each from `base`, packed per slot.
  __device__ void units(const bf16* base, int unit_bytes, Split sp) {
    const int ups = units_per_slot(unit_bytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(base);
    for (int u = sp.u0; u < sp.u1 && ok; u += ups) {
      const int n = min(ups, sp.u1 - u);
      const uint32_t bytes = (uint32_t)n * unit_bytes;
      uint8_t* dst = begin(bytes);
      if (!dst) return;
      bulk_g2s(dst, src + (size_t)u * unit_bytes, bytes, bar(), pol);
      end();
    }
  }

  // Stream cached K and V rows [c0, c0 + n) of (seq b, kv head g), n <= 64,
  // K into the slot's first 8 KB and V into its second.
  __device__ void kv_chunk(int layer, int b, int g, int c0, int n) {
    uint8_t* dst = begin((uint32_t)n * 2 * kHeadDim * 2);
    if (!dst) return;
    const int ps = p.page_size;
    const size_t layer_off = (size_t)layer * p.num_pages * p.NKV * ps * kHeadDim;
    for (int q = c0; q < c0 + n;) {
      const int blk = q / ps;
      const int off = q % ps;
      const int run = min(c0 + n - q, ps - off);
      const int page = __ldg(p.block_tables + b * p.max_blocks + blk);
      if (page < 0 || page >= p.num_pages) {
        // Never copy from an invalid page. The slot's transaction count stays
        // short, so its consumers see the abort; count the fill so drain()
        // waits for the pieces already issued into it.
        raise_error(p, kErrPage, layer);
        ok = false;
        end();
        return;
      }
      const size_t src_off = layer_off + (((size_t)page * p.NKV + g) * ps + off) * kHeadDim;
      const uint32_t bytes = (uint32_t)run * kHeadDim * 2;
      bulk_g2s_nohint(dst + (q - c0) * kHeadDim * 2, p.k_pages + src_off, bytes, bar());
      bulk_g2s_nohint(dst + 8192 + (q - c0) * kHeadDim * 2, p.v_pages + src_off, bytes, bar());
      q += run;
    }
    end();
  }

  // After an abort: wait (bounded) until every issued transfer has landed,
  // so no bulk copy is still writing shared memory when the CTA exits.
  __device__ void drain() {
    const uint32_t first = r.n > (uint32_t)r.S ? r.n - r.S : 0;
    for (uint32_t k = first; k < r.n; ++k) {
      mbar_wait(p, &r.full[k % r.S], (k / r.S) & 1, -1, 2 * p.timeout_ns);
    }
  }
};

template <int B>
__device__ void run_producer(const Params& p, const SmemState& st, Ring& ring) {
  Producer pr{p, ring, policy_evict_first()};
  Sched sch;
  const int NQKV = p.NQ + 2 * p.NKV;
  const int H = p.H, I = p.I, QD = p.NQ * kHeadDim;
  const int T = B * p.NKV * st.n_split;
  auto mark = [&](int ph, bool start) {
    if (!p.trace) return;
    if (start) {
      trace_put(p, ph, kTrProdStart, global_ns());
    } else {
      trace_put(p, ph, kTrProdEnd, global_ns());
      trace_put(p, ph, kTrProdStall, ring.stall_ns);
    }
  };
  for (int l = 0; l < p.L && pr.ok; ++l) {
    mark(l * 5 + 0, true);
    pr.units(p.w_qkv + (size_t)l * NQKV * 32 * 2 * H, 4 * H, sch.next(NQKV * 32));
    mark(l * 5 + 0, false);
    mark(l * 5 + 1, true);
    for (int it = blockIdx.x; it < T && pr.ok; it += gridDim.x) {
      const AttnItem a = attn_item(p, st, it);
      for (int c0 = a.p0; c0 < a.p1 && pr.ok; c0 += kAttnChunk) {
        pr.kv_chunk(l, a.b, a.g, c0, min(kAttnChunk, a.p1 - c0));
      }
    }
    mark(l * 5 + 1, false);
    mark(l * 5 + 2, true);
    pr.units(p.w_o + (size_t)l * H * QD, 2 * QD, sch.next(H));
    mark(l * 5 + 2, false);
    mark(l * 5 + 3, true);
    pr.units(p.w_gu + (size_t)l * I * 2 * H, 4 * H, sch.next(I));
    mark(l * 5 + 3, false);
    mark(l * 5 + 4, true);
    pr.units(p.w_down + (size_t)l * H * I, 2 * I, sch.next(H));
    mark(l * 5 + 4, false);
  }
  if (p.mode == 0 && pr.ok) {
    mark(p.L * 5, true);
    pr.units(p.embed, 2 * H, sch.next(p.V));
    mark(p.L * 5, false);
  }
  if (!pr.ok) pr.drain();
}

// ---------------------------------------------------------------- consumers

// Read B activation rows (global, L2) into shared memory; optionally apply
// HF RMSNorm: y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * gamma).
template <int B>
__device__ void load_rows(const bf16* const (&src)[B], int K, const bf16* gamma, float eps,
                          bf16* xs, int kmax, SmemState& st) {
  const int tid = threadIdx.x;
  const int kv = K >> 3;
  float ss[B];
#pragma unroll
  for (int b = 0; b < B; ++b) ss[b] = 0.f;
  for (int v = tid; v < kv; v += kConsumerThreads) {
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const uint4 u = __ldcg(reinterpret_cast<const uint4*>(src[b]) + v);
      reinterpret_cast<uint4*>(xs + b * kmax)[v] = u;
      if (gamma) {
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float a = bf_lo(w[e]), c = bf_hi(w[e]);
          ss[b] += a * a;
          ss[b] += c * c;
        }
      }
    }
  }
  if (gamma) {
    const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      const float t = warp_sum(ss[b]);
      if (lane == 0) st.red[warp * B + b] = t;
    }
    consumer_sync();
    float r[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      float t = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) t += st.red[w * B + b];
      const float var = __fdiv_rn(t, (float)K);
      r[b] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
    for (int v = tid; v < kv; v += kConsumerThreads) {
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gamma) + v);
      const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int b = 0; b < B; ++b) {
        uint4* px = reinterpret_cast<uint4*>(xs + b * kmax) + v;
        uint4 u = *px;
        uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = rbf(rbf(bf_lo(w[e]) * r[b]) * bf_lo(gw[e]));
          const float hi = rbf(rbf(bf_hi(w[e]) * r[b]) * bf_hi(gw[e]));
          __nv_bfloat162 pr = __floats2bfloat162_rn(lo, hi);
          w[e] = *reinterpret_cast<uint32_t*>(&pr);
        }
        *px = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  consumer_sync();
}

__device__ __forceinline__ void unpack8(const uint4& u, float (&f)[8]) {
  f[0] = bf_lo(u.x); f[1] = bf_hi(u.x);
  f[2] = bf_lo(u.y); f[3] = bf_hi(u.y);
  f[4] = bf_lo(u.z); f[5] = bf_hi(u.z);
  f[6] = bf_lo(u.w); f[7] = bf_hi(u.w);
}

__device__ __forceinline__ float dot8(const uint4& w, const float (&x)[8], float acc) {
  acc = fmaf(bf_lo(w.x), x[0], acc);
  acc = fmaf(bf_hi(w.x), x[1], acc);
  acc = fmaf(bf_lo(w.y), x[2], acc);
  acc = fmaf(bf_hi(w.y), x[3], acc);
  acc = fmaf(bf_lo(w.z), x[4], acc);
  acc = fmaf(bf_hi(w.z), x[5], acc);
  acc = fmaf(bf_lo(w.w), x[6], acc);
  acc = fmaf(bf_hi(w.w), x[7], acc);
  return acc;
}

// One phase of row reductions: every streamed unit is ROWS rows of K bf16;
// the warp (unit index mod 8) reduces it against the B activation rows in xs
// and hands the fp32 sums (valid in every lane) to `epi(unit, acc)`.
template <int B, int ROWS, class Epi>
__device__ bool rows_phase(const Params& p, Ring& ring, const bf16* xs, int K, Split sp,
                           int where, Epi&& epi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit_bytes = ROWS * K * 2;
  const int ups = units_per_slot(unit_bytes);
  const int kv = K >> 3;
  for (int s0 = sp.u0; s0 < sp.u1; s0 += ups) {
    const int n = min(ups, sp.u1 - s0);
    const uint8_t* slot = ring_wait(p, ring, where);
    if (!slot) return false;
    for (int i = 0; i < n; ++i) {
      if (((s0 - sp.u0 + i) & (kConsumerWarps - 1)) != warp) continue;
      const uint4* w = reinterpret_cast<const uint4*>(slot + i * unit_bytes);
      float acc[ROWS][B];
#pragma unroll
      for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int b = 0; b < B; ++b) acc[r][b] = 0.f;
#pragma unroll 4
      for (int v = lane; v < kv; v += 32) {
        uint4 wr[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; ++r) wr[r] = w[r * kv + v];
#pragma unroll
        for (int b = 0; b < B; ++b) {
          float xf[8];
          unpack8(reinterpret_cast<const uint4*>(xs + b * p.kmax)[v], xf);
#pragma unroll
          for (int r = 0; r < ROWS; ++r) acc[r][b] = dot8(wr[r], xf, acc[r][b]);
        }
      }
#pragma unroll
      for (int r = 0; r < ROWS; ++r)
#pragma unroll
        for (int b = 0; b < B; ++b) acc[r][b] = warp_sum(acc[r][b]);
      epi(s0 + i, acc, lane);
    }
    ring_release(ring);
  }
  return true;
}

// End of a phase: agree across the consumer warps whether every warp
// finished it (`ok`), then arrive at the grid barrier. false = abort (all
// consumer threads see the same answer).
__device__ __forceinline__ bool grid_arrive(const Params& p, bool ok, bool skip) {
  if (consumer_any(!ok)) return false;
  if (threadIdx.x == 0 && !skip) {
    __threadfence();
    red_release_add_u32(p.counters + kCntBarrier, 1u);
  }
  return true;
}

// Wait until *counter >= target: thread 0 spins (time-bounded), the other
// consumer threads park on the named barrier. false = abort, for everyone.
__device__ __forceinline__ bool grid_wait(const Params& p, uint32_t* counter, uint32_t target,
                                          int where) {
  const bool ok = (threadIdx.x == 0) ? counter_wait(p, counter, target, where) : true;
  return !consumer_any(!ok);
}

template <int B>
__device__ bool attention_phase(const Params& p, Ring& ring, SmemState& st, int layer,
                                float* comb, bf16* qs, float* kvn) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NQKV = p.NQ + 2 * p.NKV;
  const int T = B * p.NKV * st.n_split;
  const float scale = 0.125f;  // head_dim ** -0.5
  const int h = lane >> 3, j = lane & 7;
  for (int it = blockIdx.x; it < T; it += gridDim.x) {
    const AttnItem a = attn_item(p, st, it);
    consumer_sync();
    if (tid < kGroup * kHeadDim / 8) {
      reinterpret_cast<uint4*>(qs)[tid] =
          __ldcg(reinterpret_cast<const uint4*>(p.qkv + ((size_t)a.b * NQKV + a.g * kGroup) * kHeadDim) + tid);
    }
    consumer_sync();
    float m = -INFINITY, l = 0.f, o[8];
    bool fail = false;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
    const uint4* q4 = reinterpret_cast<const uint4*>(qs + h * kHeadDim);
    for (int c0 = a.p0; c0 < a.p1; c0 += kAttnChunk) {
      const int n = min(kAttnChunk, a.p1 - c0);
      const uint8_t* slot = ring_wait(p, ring, 200 + layer);
      if (!slot) {
        fail = true;
        break;
      }
      const int pc = warp * 8 + j;
      const bool valid = pc < n;
      float sc = -INFINITY;
      if (valid) {
        const uint4* k4 = reinterpret_cast<const uint4*>(slot + pc * kHeadDim * 2);
        float acc = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int c = (e + j) & 7;
          float qf[8];
          unpack8(q4[c], qf);
          acc = dot8(k4[c], qf, acc);
        }
        sc = acc * scale;
      }
      float cmax = sc;
      cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 1));
      cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 2));
      cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 4));
      // Warp-uniform: does this warp own any position of the chunk?
      if (warp * 8 < n) {
        const float m_new = fmaxf(m, cmax);
        const float alpha = (m == -INFINITY) ? 0.f : __expf(m - m_new);
        const float pe = (valid && m_new > -INFINITY) ? __expf(sc - m_new) : 0.f;
        float ps = pe;
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        l = l * alpha + ps;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= alpha;
        const uint8_t* vbase = slot + 8192;
#pragma unroll
        for (int pp = 0; pp < 8; ++pp) {
          const float pv = __shfl_sync(0xffffffffu, pe, (lane & ~7) | pp);
          if (warp * 8 + pp < n) {
            const uint4 vv =
                reinterpret_cast<const uint4*>(vbase + (warp * 8 + pp) * kHeadDim * 2)[j];
            float vf[8];
            unpack8(vv, vf);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = fmaf(pv, vf[e], o[e]);
          }
        }
        m = m_new;
      }
      ring_release(ring);
    }
    // Merge the 8 warps' (m, l, o) for each q head of the group.
    float* cw = comb + (warp * kGroup + h) * kPartialStride;
#pragma unroll
    for (int e = 0; e < 8; ++e) cw[j * 8 + e] = o[e];
    if (j == 0) {
      cw[kHeadDim] = m;
      cw[kHeadDim + 1] = l;
    }
    if (consumer_any(fail)) return false;
    {
      const int hh = tid >> 6, d = tid & 63;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w)
        M = fmaxf(M, comb[(w * kGroup + hh) * kPartialStride + kHeadDim]);
      float L = 0.f, O = 0.f;
      if (M > -INFINITY) {
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float* cwp = comb + (w * kGroup + hh) * kPartialStride;
          const float mw = cwp[kHeadDim];
          if (mw > -INFINITY) {
            const float f = __expf(mw - M);
            L += f * cwp[kHeadDim + 1];
            O += f * cwp[d];
          }
        }
      }
      float* pp = p.partials +
                  ((((size_t)a.b * p.NKV + a.g) * kMaxSplit + a.s) * kGroup + hh) * kPartialStride;
      pp[d] = O;
      if (d == 0) {
        pp[kHeadDim] = M;
        pp[kHeadDim + 1] = L;
      }
    }
    consumer_sync();
    if (tid == 0) {
      __threadfence();
      uint32_t* arr = p.counters + kCntArrive + a.b * p.NKV + a.g;
      const uint32_t old = atomicAdd(arr, 1u);
      const int last = (old == (uint32_t)(st.n_split - 1)) ? 1 : 0;
      if (last) {
        atomicExch(arr, 0u);
        __threadfence();
      }
      st.flag = last;
    }
    consumer_sync();
    if (st.flag) {
      // Last split of this (seq, kv head): merge all splits plus the new
      // token's own K/V (the "active slot"), then publish the heads.
      const bf16* kn = p.qkv + ((size_t)a.b * NQKV + p.NQ + a.g) * kHeadDim;
      const bf16* vn = p.qkv + ((size_t)a.b * NQKV + p.NQ + p.NKV + a.g) * kHeadDim;
      if (tid < kHeadDim) {
        kvn[tid] = bf2f(__ldcg(kn + tid));
        kvn[kHeadDim + tid] = bf2f(__ldcg(vn + tid));
      }
      consumer_sync();
      const int hh = tid >> 6, d = tid & 63;
      float sa = 0.f;
      for (int e = 0; e < kHeadDim; ++e) sa = fmaf(bf2f(qs[hh * kHeadDim + e]), kvn[e], sa);
      sa *= scale;
      float M = sa;
      const float* base =
          p.partials + (((size_t)a.b * p.NKV + a.g) * kMaxSplit * kGroup + hh) * kPartialStride;
      for (int s = 0; s < st.n_split; ++s)
        M = fmaxf(M, __ldcg(base + (size_t)s * kGroup * kPartialStride + kHeadDim));
      float L = __expf(sa - M);
      float O = L * kvn[kHeadDim + d];
      for (int s = 0; s < st.n_split; ++s) {
        const float* ps = base + (size_t)s * kGroup * kPartialStride;
        const float ms = __ldcg(ps + kHeadDim);
        if (ms > -INFINITY) {
          const float f = __expf(ms - M);
          L += f * __ldcg(ps + kHeadDim + 1);
          O += f * __ldcg(ps + d);
        }
      }
      p.attn[(size_t)a.b * p.NQ * kHeadDim + (a.g * kGroup + hh) * kHeadDim + d] = f2bf(O / L);
      consumer_sync();
      if (tid == 0) {
        __threadfence();
        red_release_add_u32(p.counters + kCntHeadsDone, 1u);
      }
    }
  }
  return true;
}

template <int B>
__device__ void run_consumers(const Params& p, SmemState& st, Ring& ring, bf16* xs,
                              float* comb, bf16* qs, float* kvn) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int H = p.H, I = p.I, QD = p.NQ * kHeadDim, NQKV = p.NQ + 2 * p.NKV;
  Sched sch;
  uint32_t barriers = 0;  // grid barriers passed so far
  const int G = gridDim.x;
  (void)warp;
  auto mark = [&](int ph, int kind) {
    if (p.trace && threadIdx.x == 0) trace_put(p, ph, kind, global_ns());
  };
  auto mark_done = [&](int ph) {
    if (p.trace && threadIdx.x == 0) {
      trace_put(p, ph, kTrDone, global_ns());
      trace_put(p, ph, kTrConsStall, ring.stall_ns);
    }
  };

  for (int l = 0; l < p.L; ++l) {
    // ------------------------------------------------------------- QKV
    mark(l * 5 + 0, kTrWaitStart);
    if (l > 0) {
      if (!grid_wait(p, p.counters + kCntBarrier, barriers * G, 1000 + l)) return;
    }
    mark(l * 5 + 0, kTrWaitDone);
    {
      const bf16* src[B];
#pragma unroll
      for (int b = 0; b < B; ++b) {
        src[b] = (l > 0) ? p.h + (size_t)b * H
                 : (p.mode == 0 ? p.embed + (size_t)st.tok[b] * H : p.hidden_in + (size_t)b * H);
      }
      load_rows<B>(src, H, p.norm_attn + (size_t)l * H, p.eps, xs, p.kmax, st);
    }
    mark(l * 5 + 0, kTrRowsLoaded);
    const Split sq = sch.next(NQKV * 32);
    const size_t kv_layer = (size_t)l * p.num_pages * p.NKV * p.page_size * kHeadDim;
    bool ok = rows_phase<B, 2>(p, ring, xs, H, sq, 2000 + l, [&](int u, float (&acc)[2][B], int lane) {
      const int hh = u >> 5, d = u & 31;
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (lane != b) continue;
        float x0 = rbf(acc[0][b]), x1 = rbf(acc[1][b]);
        const int pos = st.pos[b];
        if (hh < p.NQ + p.NKV) {
          const bf16* cr = p.rope_cos + (size_t)pos * kHeadDim;
          const bf16* sr = p.rope_sin + (size_t)pos * kHeadDim;
          const float c0 = bf2f(cr[d]), c1 = bf2f(cr[d + 32]);
          const float s0 = bf2f(sr[d]), s1 = bf2f(sr[d + 32]);
          const float y0 = rbf(rbf(x0 * c0) + rbf(-x1 * s0));
          const float y1 = rbf(rbf(x1 * c1) + rbf(x0 * s1));
          x0 = y0;
          x1 = y1;
        }
        bf16* qrow = p.qkv + ((size_t)b * NQKV + hh) * kHeadDim;
        qrow[d] = f2bf(x0);
        qrow[d + 32] = f2bf(x1);
        if (hh >= p.NQ) {
          const bool is_k = hh < p.NQ + p.NKV;
          const int g = is_k ? hh - p.NQ : hh - p.NQ - p.NKV;
          const int page = p.block_tables[b * p.max_blocks + pos / p.page_size];
          if (page < 0 || page >= p.num_pages) {
            raise_error(p, kErrPage, 300 + l);
          } else {
            bf16* dst = (is_k ? p.k_pages : p.v_pages) + kv_layer +
                        (((size_t)page * p.NKV + g) * p.page_size + pos % p.page_size) * kHeadDim;
            dst[d] = f2bf(x0);
            dst[d + 32] = f2bf(x1);
          }
        }
      }
    });
    mark_done(l * 5 + 0);
    if (!grid_arrive(p, ok, l == 0 && (int)blockIdx.x == p.debug_skip_cta)) return;
    ++barriers;

    // ------------------------------------------------------------- ATTN
    mark(l * 5 + 1, kTrWaitStart);
    if (!grid_wait(p, p.counters + kCntBarrier, barriers * G, 3000 + l)) return;
    mark(l * 5 + 1, kTrWaitDone);
    if (!attention_phase<B>(p, ring, st, l, comb, qs, kvn)) return;
    mark_done(l * 5 + 1);

    // ------------------------------------------------------------- O
    mark(l * 5 + 2, kTrWaitStart);
    if (!grid_wait(p, p.counters + kCntHeadsDone, (uint32_t)((l + 1) * B * p.NKV), 4000 + l))
      return;
    mark(l * 5 + 2, kTrWaitDone);
    {
      const bf16* src[B];
#pragma unroll
      for (int b = 0; b < B; ++b) src[b] = p.attn + (size_t)b * QD;
      load_rows<B>(src, QD, nullptr, 0.f, xs, p.kmax, st);
    }
    mark(l * 5 + 2, kTrRowsLoaded);
    ok = rows_phase<B, 1>(p, ring, xs, QD, sch.next(H), 5000 + l, [&](int u, float (&acc)[1][B], int lane) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (lane != b) continue;
        const bf16* res = (l > 0) ? p.h + (size_t)b * H
                          : (p.mode == 0 ? p.embed + (size_t)st.tok[b] * H : p.hidden_in + (size_t)b * H);
        const float r = bf2f(__ldcg(res + u));
        p.h[(size_t)b * H + u] = f2bf(r + rbf(acc[0][b]));
      }
    });
    mark_done(l * 5 + 2);
    if (!grid_arrive(p, ok, false)) return;
    ++barriers;

    // ------------------------------------------------------------- GU
    mark(l * 5 + 3, kTrWaitStart);
    if (!grid_wait(p, p.counters + kCntBarrier, barriers * G, 6000 + l)) return;
    mark(l * 5 + 3, kTrWaitDone);
    {
      const bf16* src[B];
#pragma unroll
      for (int b = 0; b < B; ++b) src[b] = p.h + (size_t)b * H;
      load_rows<B>(src, H, p.norm_mlp + (size_t)l * H, p.eps, xs, p.kmax, st);
    }
    mark(l * 5 + 3, kTrRowsLoaded);
    ok = rows_phase<B, 2>(p, ring, xs, H, sch.next(I), 7000 + l, [&](int u, float (&acc)[2][B], int lane) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (lane != b) continue;
        const float g = rbf(acc[0][b]);
        const float up = rbf(acc[1][b]);
        const float s = rbf(__fdiv_rn(g, 1.0f + expf(-g)));
        p.act[(size_t)b * I + u] = f2bf(s * up);
      }
    });
    mark_done(l * 5 + 3);
    if (!grid_arrive(p, ok, false)) return;
    ++barriers;

    // ------------------------------------------------------------- DOWN
    mark(l * 5 + 4, kTrWaitStart);
    if (!grid_wait(p, p.counters + kCntBarrier, barriers * G, 8000 + l)) return;
    mark(l * 5 + 4, kTrWaitDone);
    {
      const bf16* src[B];
#pragma unroll
      for (int b = 0; b < B; ++b) src[b] = p.act + (size_t)b * I;
      load_rows<B>(src, I, nullptr, 0.f, xs, p.kmax, st);
    }
    mark(l * 5 + 4, kTrRowsLoaded);
    const bool last_layer = (l == p.L - 1);
    ok = rows_phase<B, 1>(p, ring, xs, I, sch.next(H), 9000 + l, [&](int u, float (&acc)[1][B], int lane) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        if (lane != b) continue;
        const float r = bf2f(__ldcg(p.h + (size_t)b * H + u));
        const bf16 y = f2bf(r + rbf(acc[0][b]));
        p.h[(size_t)b * H + u] = y;
        if (last_layer && p.mode == 1) p.hidden_out[(size_t)b * H + u] = y;
      }
    });
    mark_done(l * 5 + 4);
    if (last_layer && p.mode == 1) {
      if (consumer_any(!ok)) return;
    } else {
      if (!grid_arrive(p, ok, false)) return;
      ++barriers;
    }
  }

  // --------------------------------------------------------------- LM head
  if (p.mode == 0) {
    mark(p.L * 5, kTrWaitStart);
    if (!grid_wait(p, p.counters + kCntBarrier, barriers * G, 10000)) return;
    mark(p.L * 5, kTrWaitDone);
    {
      const bf16* src[B];
#pragma unroll
      for (int b = 0; b < B; ++b) src[b] = p.h + (size_t)b * H;
      load_rows<B>(src, H, p.norm_final, p.eps, xs, p.kmax, st);
    }
    mark(p.L * 5, kTrRowsLoaded);
    float best_v[B];
    int best_i[B];
#pragma unroll
    for (int b = 0; b < B; ++b) {
      best_v[b] = -INFINITY;
      best_i[b] = 0x7fffffff;
    }
    const bool ok = rows_phase<B, 1>(p, ring, xs, H, sch.next(p.V), 11000, [&](int u, float (&acc)[1][B], int lane) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        const float v = acc[0][b];
        if (p.logits && lane == b) p.logits[(size_t)b * p.V + u] = v;
        if (v > best_v[b] || (v == best_v[b] && u < best_i[b])) {
          best_v[b] = v;
          best_i[b] = u;
        }
      }
    });
    if (consumer_any(!ok)) return;
    mark_done(p.L * 5);
    const int lane = tid & 31, w = tid >> 5;
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        st.am_val[w * B + b] = best_v[b];
        st.am_idx[w * B + b] = best_i[b];
      }
    }
    consumer_sync();
    if (tid < B) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
      for (int ww = 0; ww < kConsumerWarps; ++ww) {
        const float v = st.am_val[ww * B + tid];
        const int i = st.am_idx[ww * B + tid];
        if (v > bv || (v == bv && i < bi)) {
          bv = v;
          bi = i;
        }
      }
      if (bi != 0x7fffffff) {
        const unsigned long long key =
            ((unsigned long long)float_key(bv) << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)bi);
        atomicMax(p.keys + tid, key);
      }
    }
  }

  // --------------------------------------------------------------- finish
  consumer_sync();
  if (tid == 0) {
    __threadfence();
    const uint32_t t = atomicAdd(p.counters + kCntDone, 1u);
    if (t == (uint32_t)G - 1) {
      __threadfence();
      if (p.mode == 0) {
        for (int b = 0; b < B; ++b) {
          const unsigned long long key = atomicExch(p.keys + b, 0ull);
          const int id = (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
          p.next_ids[b] = id;
          if (p.flags & 1) {
            p.tokens[b] = id;
            p.positions[b] = st.pos[b] + 1;
          }
        }
      }
      atomicExch(p.counters + kCntBarrier, 0u);
      atomicExch(p.counters + kCntHeadsDone, 0u);
      atomicExch(p.counters + kCntDone, 0u);
      __threadfence();
    }
  }
}

template <int B>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int S = p.num_slots;
  uint8_t* ring_mem = smem;
  bf16* xs = reinterpret_cast<bf16*>(smem + (size_t)S * kSlotBytes);
  int xbytes = (B * p.kmax * 2 + 127) & ~127;
  float* comb = reinterpret_cast<float*>(smem + (size_t)S * kSlotBytes + xbytes);
  bf16* qs = reinterpret_cast<bf16*>(comb + kConsumerWarps * kGroup * kPartialStride);
  float* kvn = reinterpret_cast<float*>(qs + kGroup * kHeadDim);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + (size_t)S * kSlotBytes + xbytes + kAttnScratchBytes);
  SmemState* st = reinterpret_cast<SmemState*>(bars + 2 * S);

  Ring ring{ring_mem, bars, bars + S, S};

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&ring.full[s], 1);
      mbar_init(&ring.empty[s], kConsumerWarps);
    }
    fence_mbar_init();
    int pmax = 0;
    bool bad = false;
    for (int b = 0; b < B; ++b) {
      const int pos = p.positions[b];
      const int tok = (p.mode == 0) ? p.tokens[b] : 0;
      st->pos[b] = pos;
      st->tok[b] = tok;
      if (pos < 0 || pos >= p.rope_len || pos / p.page_size >= p.max_blocks) {
        raise_error(p, kErrPosition, pos);
        bad = true;
      }
      if (tok < 0 || tok >= p.V) {
        raise_error(p, kErrToken, tok);
        bad = true;
      }
      pmax = max(pmax, pos);
    }
    // Split-K pieces per (seq, kv head): enough to spread the items over the
    // grid, but no piece shorter than one 64-position chunk.
    int ns = min(kMaxSplit, max(1, (int)gridDim.x / (B * p.NKV)));
    ns = max(1, min(ns, (pmax + kAttnChunk - 1) / kAttnChunk));
    st->n_split = ns;
    st->flag = bad ? 1 : 0;
  }
  __syncthreads();
  if (st->flag) return;

  if (threadIdx.x >= kConsumerThreads) {
    if (threadIdx.x == kConsumerThreads) run_producer<B>(p, *st, ring);
    return;
  }
  run_consumers<B>(p, *st, ring, xs, comb, qs, kvn);
}

}  // namespace mk
