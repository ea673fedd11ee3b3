// mk_kernel.cuh — the persistent decode megakernel (sm_100a).
//
// One cooperative launch, one CTA per SM, decodes a token for each of B
// sequences through every decoder layer, then the final norm, the tied
// lm_head and a greedy argmax.
//
// CTA = 14 consumer warps + 2 producer warps.
//
// * The producers (lane 0 of two warps, alternating fills: one lane issues
//   at most ~50 GB/s of 16 KB bulk copies) walk the CTA's whole schedule of HBM reads for
//   the step — its slice of every weight matrix of every layer, its KV-cache
//   chunks, its lm_head rows — and streams them with bulk copies
//   (cp.async.bulk, the TMA engine without a tensor map) into a ring of 16 KB
//   shared-memory slots, each guarded by a full/empty mbarrier pair. Weights
//   and cached K/V do not depend on activations, so the producer never waits
//   for a grid barrier: it runs ahead by the ring's depth (~190 KB per SM).
// * The consumers walk the same schedule. Every streamed row is cut into
//   pieces of at most 2048 columns (4 KB); piece q of a phase goes to warp
//   q mod 14, so each slot is read by four warps at once, each with 128-bit
//   shared loads. A warp keeps its 2048-column segment of the activation
//   vector in registers as packed bf16 and accumulates with mixed-precision
//   fma.rn.f32.bf16 into four independent fp32 chains, then reduces across
//   the warp and leaves one fp32 partial per piece in shared memory. After
//   the phase the partials of each output are summed in a fixed order and
//   the epilogue (RoPE, KV scatter, SiLU*up, residual add) runs one thread
//   per output, off the streaming loop.
//
// Phases per layer. There is no grid barrier: every activation a phase hands
// to the next is written as tagged words (bf16 << 16 | a tag naming the launch
// and the phase), and a consumer polls exactly the words it needs until they
// carry the producing phase's tag (time-bounded).
//   QKV    RMSNorm(h), q/k/v rows in RoPE pairs (d, d+32), llama3 RoPE from a
//          bf16 cos/sin table, K/V row scattered into the paged cache.
//   ATTN   split-K GQA flash-decode: item (seq, kv head, position range) per
//          CTA, online softmax per warp, CTA merge. A single split writes the
//          heads' tagged output; with several, every split publishes tagged
//          64-bit (o, m, l) partials and split 0, which also holds the new
//          token's own K/V, merges them in split order and publishes.
//   O      o_proj rows + residual add into h.
//   GU     RMSNorm(h), gate/up row pairs, SiLU(gate) * up.
//   DOWN   down rows + residual add into h.
// then LM: final RMSNorm, lm_head rows, fp32 logits, packed 64-bit atomicMax
// argmax; the last CTA to finish (an arrival counter) publishes the ids.
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
  int nseg_h, nseg_qd, nseg_i;  // pieces per row for K = H, NQ*64, I
  int part_cap;                 // floats in the shared partial-sum array
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
  // scratch (owned by the model handle). Activations passed between phases
  // are tagged words: bf16 bits << 16 | a 16-bit tag (see phase_tag).
  uint32_t* h;     // [B][H]
  uint32_t* qkv;   // [B][NQ + 2 NKV][64]
  uint32_t* attn;  // [B][NQ * 64]
  uint32_t* act;   // [B][I]
  // Attention split partials, one block per attention item (< grid when
  // split): [item][kGroup][kPartialStride] words of part_tag << 32 | fp32.
  unsigned long long* partials;
  uint32_t* counters;
  unsigned long long* keys;  // [B]
  int* error;                // [4] code, detail, cta, thread (device)
  int* host_error;           // [4] mapped pinned host mirror of `error`
  unsigned long long timeout_ns;
  int debug_skip_cta;
  // This launch's first activation tag. Tags only grow between two clears of
  // the activation words (the host zeroes them before the counter would pass
  // 65535), so no word left by an earlier launch carries a tag of this one.
  uint32_t tag_base;
  // First 32-bit tag of the tensor-parallel exchange words (peer-written, so
  // never cleared by one rank alone): consecutive launches use disjoint
  // ranges, and a range recurs only after 2^32 / (5 L + 1) launches.
  uint32_t xtag_base;
  uint32_t part_tag0;  // layer 0's partial tag (layer l: + l); never 0, unique until the
                       // host zeroes the partials and restarts the sequence
  // optional phase trace ([grid][trace_per_cta] u64, see kTrace*); nullptr = off
  unsigned long long* trace;
  int trace_per_cta;
  // Tensor parallelism over tp_world GPUs (1: none). This rank holds NQ q
  // heads, NKV kv heads and I MLP rows of the model (the counts above are the
  // local ones) and scores lm_head rows [lm_row0, lm_row0 + lm_rows); V is
  // the whole vocabulary. xpeer[r] is rank r's exchange buffer as mapped on
  // this GPU (xpeer[tp_rank] is this rank's own; see xbuf_* for its layout).
  int tp_rank, tp_world;
  int lm_row0, lm_rows;
  unsigned long long* xpeer[kMaxTp];
};

// Exchange buffer of a tensor-parallel rank, 64-bit words written by every
// rank of the group: o_proj and down partial sums, [2][tp_world][B][H] words
// (tag << 32 | fp32 bits), then the lm_head argmax keys [tp_world][B], then
// one "keys published" flag word per rank (the tag).
__host__ __device__ inline size_t xbuf_partial(int slot, int src, int b, int u, int W, int B, int H) {
  return (((size_t)slot * W + src) * B + b) * H + u;
}
__host__ __device__ inline size_t xbuf_keys(int src, int b, int W, int B, int H) {
  return (size_t)2 * W * B * H + (size_t)src * B + b;
}
__host__ __device__ inline size_t xbuf_flag(int src, int W, int B, int H) {
  return (size_t)2 * W * B * H + (size_t)W * B + src;
}
__host__ __device__ inline size_t xbuf_words(int W, int B, int H) { return xbuf_flag(W, W, B, H); }

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
  kTrAttnQ = 8,        // attention: q / new K,V loaded (last item of the CTA)
  kTrAttnChunks = 9,   // attention: cached chunks reduced
  kTrAttnArrive = 10,  // attention: warp states combined, output or split partials written
  kTrAttnMerged = 11,  // attention: split 0 merged the splits and published (if split)
  kTraceKinds = 12,
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
  uint32_t prod_pos[kProducers];  // fills each producer has walked past
  int pad[4];
  float red[kConsumerWarps * 4];
  float am_val[kConsumerWarps * 4];
  int am_idx[kConsumerWarps * 4];
};

// Shared-memory layout (dynamic): [ring S x 16 KB][x rows B x kmax bf16]
// [partials part_cap fp32][raw residual B x H bf16][RoPE rows B x 128 bf16]
// [attention scratch][mbarriers: kFullBars full, S empty][SmemState]
constexpr int kAttnScratchBytes =
    kAttnWarps * kGroup * kPartialStride * 4 + kGroup * kHeadDim * 2 + 2 * kHeadDim * 4;

__host__ __device__ inline int align128(int x) { return (x + 127) & ~127; }

__host__ __device__ inline int smem_bytes_for(int num_slots, int B, int kmax, int part_cap, int H) {
  return num_slots * kSlotBytes + align128(B * kmax * 2) + align128(part_cap * 4) +
         align128(B * H * 2) + align128(B * 2 * kHeadDim * 2) + kAttnScratchBytes +
         (kFullBars + num_slots) * 8 + (int)sizeof(SmemState) + 128;
}

// Pieces per row of K columns: the fewest equal segments of at most
// kSegCols columns, each a multiple of 256 (32 lanes x 8 bf16).
__host__ __device__ inline int pieces_per_row(int K) {
  for (int n = (K + kSegCols - 1) / kSegCols; n <= K / 256; ++n)
    if (K % n == 0 && (K / n) % 256 == 0) return n;
  return K / 256;
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

// ---------------------------------------------------------------- tagged activations
//
// Every activation one phase hands to the next (q/k/v, attention output, the
// residual h, the SwiGLU product) is written as 32-bit words, bf16 bits << 16
// | a 16-bit tag naming the launch and the phase that wrote it. A reader polls
// the words themselves until each carries the tag it expects, so there is no
// grid barrier and no separate flag round trip between a phase and the next.
// A single buffer per activation is safe: no phase can overwrite a word
// before every CTA has read the previous value, because its own inputs depend
// on all CTAs having done so. Tags are never 0, the value scratch starts at.

__device__ __forceinline__ uint32_t phase_tag(const Params& p, int phase) {
  return 1u + (p.tag_base + (uint32_t)phase) % 65535u;
}

// The exchange-word tag of a phase (tensor parallelism only).
__device__ __forceinline__ uint32_t xchg_tag(const Params& p, int phase) {
  return p.xtag_base + (uint32_t)phase;
}

__device__ __forceinline__ uint32_t tagged(float v, uint32_t tag) {
  return ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v)) << 16) | tag;
}

__device__ __forceinline__ bool tags_ok(const uint4& u, uint32_t tag) {
  return ((u.x & 0xFFFFu) == tag) & ((u.y & 0xFFFFu) == tag) & ((u.z & 0xFFFFu) == tag) &
         ((u.w & 0xFFFFu) == tag);
}

struct Polled {
  uint4 u;
  int ok;
};

// A 64-bit tagged word: tag << 32 | fp32 bits (one single-copy-atomic store).
__device__ __forceinline__ unsigned long long tagged64(float v, uint32_t tag) {
  return ((unsigned long long)tag << 32) | __float_as_uint(v);
}

struct Polled64 {
  unsigned long long v;
  int ok;
};

// Spin (bounded) until the 64-bit word at src carries `tag`.
__device__ __noinline__ Polled64 poll_tagged64_slow(const Params& p, const unsigned long long* src,
                                                    uint32_t tag, int where) {
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    const unsigned long long v = __ldcg(src);
    if ((uint32_t)(v >> 32) == tag) return {v, 1};
    if ((it & 15) == 0) {
      if (aborted(p)) return {v, 0};
      if (global_ns() - t0 > p.timeout_ns) {
        raise_error(p, kErrBarrierTimeout, where);
        return {v, 0};
      }
    }
  }
}

// The fp32 value of a 64-bit word already loaded as v, polled at src until it
// carries `tag` if it did not yet. false on abort or timeout.
__device__ __forceinline__ bool value64(const Params& p, const unsigned long long* src,
                                        unsigned long long v, uint32_t tag, float& out, int where) {
  if ((uint32_t)(v >> 32) != tag) {
    const Polled64 r = poll_tagged64_slow(p, src, tag, where);
    if (!r.ok) return false;
    v = r.v;
  }
  out = __uint_as_float((uint32_t)v);
  return true;
}

// Slow path of poll_tagged: re-read until the tags match (time-bounded). No
// sleep between reads: the wait is on the step's critical path (a 64 ns
// sleep cost 2.5% of the step, measured).
// Returns by value so callers' registers stay out of local memory.
__device__ __noinline__ Polled poll_tagged_slow(const Params& p, const uint32_t* src, uint32_t tag,
                                                int where) {
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    const uint4 u = __ldcg(reinterpret_cast<const uint4*>(src));
    if (tags_ok(u, tag)) return {u, 1};
    if ((it & 15) == 0) {
      if (aborted(p)) return {u, 0};
      if (global_ns() - t0 > p.timeout_ns) {
        raise_error(p, kErrBarrierTimeout, where);
        return {u, 0};
      }
    }
  }
}

// Four tagged words (16-byte aligned) once all carry `tag`. false on abort or
// timeout (the thread's own verdict; callers make it CTA-wide).
__device__ __forceinline__ bool poll_tagged(const Params& p, const uint32_t* src, uint32_t tag,
                                            uint4& out, int where) {
  out = __ldcg(reinterpret_cast<const uint4*>(src));
  if (tags_ok(out, tag)) return true;
  const Polled r = poll_tagged_slow(p, src, tag, where);
  out = r.u;
  return r.ok != 0;
}

// The bf16 values of four tagged words, packed two per word.
__device__ __forceinline__ uint2 untag4(const uint4& u) {
  return make_uint2((u.x >> 16) | (u.y & 0xFFFF0000u), (u.z >> 16) | (u.w & 0xFFFF0000u));
}

// ---------------------------------------------------------------- tensor parallelism
//
// The o_proj and down projections are split over the group by their input
// columns (each rank holds its q heads' o_proj columns and its MLP rows'
// down columns), so every rank has a partial sum of every output row. The
// CTA that owns row u on each rank publishes its fp32 partial, tagged with
// the phase, to every rank's exchange buffer (peer stores over NVLink), then
// reads the tp_world partials of u from its own buffer and adds them in rank
// order, so every rank computes the same residual bit for bit and publishes
// it locally as a tagged activation, as a single GPU does.

__device__ __forceinline__ void tp_publish(const Params& p, int slot, int b, int u, float mine,
                                           uint32_t tag) {
  const unsigned long long w = ((unsigned long long)tag << 32) | __float_as_uint(mine);
  for (int r = 0; r < p.tp_world; ++r)
    st_sys_u64(p.xpeer[r] + xbuf_partial(slot, p.tp_rank, b, u, p.tp_world, p.B, p.H), w);
}

struct Summed {
  float v;
  int ok;
};

// Sum over ranks of row u's partials (time-bounded wait for each).
__device__ __noinline__ Summed tp_sum(const Params& p, int slot, int b, int u, uint32_t tag,
                                      int where) {
  const unsigned long long* own = p.xpeer[p.tp_rank];
  float acc = 0.f;
  uint64_t t0 = 0;
  for (int r = 0; r < p.tp_world; ++r) {
    const unsigned long long* w = own + xbuf_partial(slot, r, b, u, p.tp_world, p.B, p.H);
    unsigned long long v = ld_sys_u64(w);
    for (uint32_t it = 1; (uint32_t)(v >> 32) != tag; ++it) {
      if (!t0) t0 = global_ns();
      v = ld_sys_u64(w);
      if ((it & 15) == 0) {
        if (aborted(p)) return {0.f, 0};
        if (global_ns() - t0 > p.timeout_ns) {
          raise_error(p, kErrBarrierTimeout, where);
          return {0.f, 0};
        }
      }
    }
    acc += __uint_as_float((uint32_t)v);
  }
  return {acc, 1};
}

// The group's argmax: publish this rank's packed keys (B of them) and a flag
// to every rank, wait (bounded) for every rank's flag, and fold the keys into
// `key` (max: highest logit, lowest index). false on abort or timeout.
__device__ __noinline__ bool tp_argmax(const Params& p, unsigned long long* key, uint32_t tag) {
  const int W = p.tp_world, B = p.B, H = p.H;
  for (int r = 0; r < W; ++r)
    for (int b = 0; b < B; ++b) st_sys_u64(p.xpeer[r] + xbuf_keys(p.tp_rank, b, W, B, H), key[b]);
  __threadfence_system();
  for (int r = 0; r < W; ++r) st_release_sys_u64(p.xpeer[r] + xbuf_flag(p.tp_rank, W, B, H), tag);
  const unsigned long long* own = p.xpeer[p.tp_rank];
  const uint64_t t0 = global_ns();
  for (int r = 0; r < W; ++r) {
    for (uint32_t it = 1; ld_acquire_sys_u64(own + xbuf_flag(r, W, B, H)) != tag; ++it) {
      __nanosleep(64);
      if ((it & 15) == 0) {
        if (aborted(p)) return false;
        if (global_ns() - t0 > p.timeout_ns) {
          raise_error(p, kErrBarrierTimeout, 12000 + r);
          return false;
        }
      }
    }
    for (int b = 0; b < B; ++b) {
      const unsigned long long k = ld_sys_u64(own + xbuf_keys(r, b, W, B, H));
      if (k > key[b]) key[b] = k;
    }
  }
  return true;
}

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

__host__ __device__ inline Split split_units(int U, int G, int c, int rot) {
  const int base = U / G, rem = U % G;
  const int end = rot + rem;
  auto mn = [](int a, int b) { return a < b ? a : b; };
  auto mx = [](int a, int b) { return a > b ? a : b; };
  int before;
  if (end <= G) {
    before = mn(mx(c - rot, 0), rem);
  } else {
    before = mn(c, end - G) + mn(mx(c - rot, 0), G - rot);
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

__host__ __device__ inline int units_per_slot(int unit_bytes) {
  return kSlotBytes / unit_bytes > 1 ? kSlotBytes / unit_bytes : 1;
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

// Walk the CTA's streaming schedule for one step, in the order the consumers
// use it: per layer the QKV rows, the KV chunks of its attention items, the
// o_proj rows, the gate/up row pairs, the down rows; then the lm_head rows.
// `ops` is a producer (bulk copies into the ring).
template <int B, class Ops>
__device__ void walk_schedule(const Params& p, const SmemState& st, Ops& ops) {
  Sched sch;
  const int NQKV = p.NQ + 2 * p.NKV;
  const int H = p.H, I = p.I, QD = p.NQ * kHeadDim;
  const int T = B * p.NKV * st.n_split;
  for (int l = 0; l < p.L && ops.ok; ++l) {
    ops.mark(l * 5 + 0, true);
    ops.units(p.w_qkv + (size_t)l * NQKV * 32 * 2 * H, 4 * H, sch.next(NQKV * 32));
    ops.mark(l * 5 + 0, false);
    ops.mark(l * 5 + 1, true);
    for (int it = blockIdx.x; it < T && ops.ok; it += gridDim.x) {
      const AttnItem a = attn_item(p, st, it);
      for (int c0 = a.p0; c0 < a.p1 && ops.ok; c0 += kAttnChunk) {
        ops.kv_chunk(l, a.b, a.g, c0, min(kAttnChunk, a.p1 - c0));
      }
    }
    ops.mark(l * 5 + 1, false);
    ops.mark(l * 5 + 2, true);
    ops.units(p.w_o + (size_t)l * H * QD, 2 * QD, sch.next(H));
    ops.mark(l * 5 + 2, false);
    ops.mark(l * 5 + 3, true);
    ops.units(p.w_gu + (size_t)l * I * 2 * H, 4 * H, sch.next(I));
    ops.mark(l * 5 + 3, false);
    ops.mark(l * 5 + 4, true);
    ops.units(p.w_down + (size_t)l * H * I, 2 * I, sch.next(H));
    ops.mark(l * 5 + 4, false);
  }
  if (p.mode == 0 && ops.ok) {
    ops.mark(p.L * 5, true);
    ops.units(p.embed + (size_t)p.lm_row0 * H, 2 * H, sch.next(p.lm_rows));
    ops.mark(p.L * 5, false);
  }
}

// ---------------------------------------------------------------- ring

// Fill f lands in slot f % S and completes full barrier f % kFullBars; its
// readers release it on empty barrier f % S. An mbarrier wait names a phase
// by parity only, so a consumer warp, which waits only for the fills it reads,
// must never wait on a barrier whose previous phase is still open: it would
// take the phase before that for its own and read a slot still being written.
// Producer k issues fill f only once the other producer has walked past fill
// f - kProducerSlack, so when any fill f' has landed, every fill up to
// f' - kProducerSlack has been issued. A warp that waits for fill f after
// waiting for fill f' with f - f' <= kFullBars - S - kProducerSlack therefore
// knows fill f - kFullBars + S was issued, which its producer could only do
// once the slot's earlier fill f - kFullBars had been read: that fill had
// landed, and the barrier's previous phase is complete. (Fills below
// kFullBars use fresh barriers.) The warp cannot be lapped either: it reads
// fill f, so the slot is not refilled before it releases it. The host checks
// the gap bound for every CTA's schedule before the first launch
// (schedule_gap_ok in mk_api.cu); checking it here would cost the consumer
// loop ~10% (measured).
struct Ring {
  uint8_t* slots;    // generic address of slot 0
  uint32_t slots_s;  // shared-window address of slot 0
  uint64_t* full;    // [kFullBars]
  uint64_t* empty;   // [S]
  int S;
  uint32_t n = 0;  // fills seen so far (the same count on every side)
  unsigned long long stall_ns = 0;  // time spent waiting (traced runs only)
};

// Noinline phase functions take the caller's Ring by reference but work on a
// register copy (a reference into the caller's stack would turn every access
// into a local-memory round trip); this writes the counters back on exit.
struct RingWriteBack {
  Ring& dst;
  const Ring& src;
  __device__ ~RingWriteBack() {
    dst.n = src.n;
    dst.stall_ns = src.stall_ns;
  }
};

// Slow path of a consumer warp's wait for a fill: every lane polls the
// mbarrier; lane 0 alone decides to give up (abort or timeout) and the
// decision is broadcast, so the result is uniform across the warp.
__device__ __noinline__ bool ring_wait_slow(const Params& p, uint64_t* bar, uint32_t parity,
                                            int where) {
  const uint64_t t0 = global_ns();
  bool done = false;
  for (uint32_t it = 0;; ++it) {
    if (!done) done = mbar_try_wait(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    int give_up = 0;
    if ((it & 7) == 7 && (threadIdx.x & 31) == 0) {
      if (aborted(p)) {
        give_up = 1;
      } else if (global_ns() - t0 > p.timeout_ns) {
        raise_error(p, kErrRingTimeout, where);
        give_up = 1;
      }
    }
    if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
  }
}

// Consumer warp: wait until fill `f` has landed. false on abort/timeout.
__device__ __forceinline__ bool ring_wait(const Params& p, Ring& r, uint32_t f, int where) {
  uint64_t* bar = &r.full[f % kFullBars];
  const uint32_t parity = (f / kFullBars) & 1;
  // try_wait may itself suspend the thread for a while, so a traced run
  // times the whole wait.
  const uint64_t ts = p.trace ? global_ns() : 0;
  bool ok = __all_sync(0xffffffffu, mbar_try_wait(bar, parity));
  if (!ok) ok = ring_wait_slow(p, bar, parity, where);
  if (ts) r.stall_ns += global_ns() - ts;
  return ok;
}

// Consumer warp: done with fill `f`; `count` arrivals on its empty barrier
// (the warps that read a fill contribute kConsumerWarps arrivals in total).
__device__ __forceinline__ void ring_release(Ring& r, uint32_t f, uint32_t count) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive_cnt(&r.empty[f % r.S], count);
}

// ---------------------------------------------------------------- producer

struct Producer {
  const Params& p;
  Ring& r;
  SmemState& st;
  uint64_t pol;
  int k;  // this producer takes the fills f with f % kProducers == k
  bool ok = true;

  __device__ bool mine() const { return (int)(r.n % kProducers) == k; }

  // Wait (bounded) until the other producer has walked past fill
  // r.n - kProducerSlack (see the Ring comment). false on abort/timeout.
  __device__ bool couple() {
    const uint32_t* other = &st.prod_pos[k ^ 1];
    if (ld_acquire_shared(other) + kProducerSlack > r.n) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0;; ++it) {
      if (ld_acquire_shared(other) + kProducerSlack > r.n) {
        if (p.trace) r.stall_ns += global_ns() - t0;
        return true;
      }
      if ((it & 7) == 7) {
        if (aborted(p)) return false;
        if (global_ns() - t0 > p.timeout_ns) {
          raise_error(p, kErrRingTimeout, 102);
          return false;
        }
      }
    }
  }

  // Claim the next slot for `bytes` of transfers; nullptr when aborting.
  __device__ uint8_t* begin(uint32_t bytes) {
    if (!ok) return nullptr;
    if (!couple()) {
      ok = false;
      return nullptr;
    }
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
    mbar_arrive_expect_tx(bar(), bytes);
    return r.slots + (size_t)slot * kSlotBytes;
  }
  __device__ uint64_t* bar() { return &r.full[r.n % kFullBars]; }
  // Past fill r.n (issued, or the other producer's): publish the position.
  __device__ void end() {
    r.n++;
    st_release_shared(&st.prod_pos[k], r.n);
  }

  __device__ void mark(int ph, bool start) {
    if (!p.trace || k != 0) return;
    if (start) {
      trace_put(p, ph, kTrProdStart, global_ns());
    } else {
      trace_put(p, ph, kTrProdEnd, global_ns());
      trace_put(p, ph, kTrProdStall, r.stall_ns);
    }
  }

  // Stream units [u0, u1) of `unit_bytes` each from `base`, packed per slot.
  __device__ void units(const bf16* base, int unit_bytes, Split sp) {
    const int ups = units_per_slot(unit_bytes);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(base);
    for (int u = sp.u0; u < sp.u1 && ok; u += ups) {
      if (!mine()) {
        end();
        continue;
      }
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
    if (!mine()) {
      end();
      return;
    }
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
    for (uint32_t f = first; f < r.n; ++f) {
      if ((int)(f % kProducers) == k)
        mbar_wait(p, &r.full[f % kFullBars], (f / kFullBars) & 1, -1, 2 * p.timeout_ns);
    }
  }
};

// ---------------------------------------------------------------- consumers

// Read B activation rows (global, L2) into shared memory; optionally apply
// HF RMSNorm: y = bf16(bf16(x * rsqrt(mean(x^2) + eps)) * gamma).
template <int B>
__device__ void load_rows(const bf16* const (&src)[B], int K, const bf16* gamma, float eps,
                          bf16* xs, int kmax, SmemState& st, bf16* raw = nullptr) {
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
      if (raw) reinterpret_cast<uint4*>(raw + b * K)[v] = u;
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

// load_rows for tagged activations: poll B rows of K (<= 8192) tagged words
// until they carry `tag`, store the bf16 values (and optionally a raw copy)
// and apply the same RMSNorm. A thread issues all its loads, and its gamma
// loads, before waiting on any, so a ready row costs one round trip. false =
// abort, for every consumer thread.
template <int B>
struct RowPtrs {
  const uint32_t* r[B];
};

template <int B>
__device__ __noinline__ bool load_rows_tagged(const Params& p, RowPtrs<B> src, int K, uint32_t tag,
                                              const bf16* gamma, float eps, bf16* xs, int kmax,
                                              SmemState& st, int where, bf16* raw) {
  constexpr int kBatch = 5;   // uint4 of tagged words per thread per row: 2048 / 448 -> 5
  constexpr int kGBatch = 2;  // uint4 of gamma per thread: (hidden <= 4096) / 8 / 448 -> 2
  const int tid = threadIdx.x;
  const int k4 = K >> 2, k8 = K >> 3;
  uint4 gv[kGBatch];
  if (gamma) {
#pragma unroll
    for (int j = 0; j < kGBatch; ++j) {
      const int v = tid + j * kConsumerThreads;
      if (v < k8) gv[j] = __ldg(reinterpret_cast<const uint4*>(gamma) + v);
    }
  }
  float ss[B];
  int ok = 1;
#pragma unroll
  for (int b = 0; b < B; ++b) {
    ss[b] = 0.f;
    uint4 u[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int v = tid + i * kConsumerThreads;
      if (v < k4) u[i] = __ldcg(reinterpret_cast<const uint4*>(src.r[b] + 4 * v));
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int v = tid + i * kConsumerThreads;
      if (v < k4) {
        if (!tags_ok(u[i], tag)) {
          const Polled r = poll_tagged_slow(p, src.r[b] + 4 * v, tag, where);
          u[i] = r.u;
          ok &= r.ok;
        }
        const uint2 w = untag4(u[i]);
        reinterpret_cast<uint2*>(xs + b * kmax)[v] = w;
        if (raw) reinterpret_cast<uint2*>(raw + b * K)[v] = w;
        const float a0 = bf_lo(w.x), a1 = bf_hi(w.x), a2 = bf_lo(w.y), a3 = bf_hi(w.y);
        ss[b] += a0 * a0;
        ss[b] += a1 * a1;
        ss[b] += a2 * a2;
        ss[b] += a3 * a3;
      }
    }
  }
  if (consumer_any(!ok)) return false;
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
#pragma unroll
    for (int j = 0; j < kGBatch; ++j) {
      const int v = tid + j * kConsumerThreads;
      if (v >= k8) continue;
      const uint32_t gw[4] = {gv[j].x, gv[j].y, gv[j].z, gv[j].w};
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
  return true;
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

// One streamed GEMV phase over units [sp.u0, sp.u1): each unit is
// `rows_per_unit` rows of K bf16 columns, cut into pieces of K / nseg
// columns. Work items are groups of `grp` consecutive pieces (1, or a whole
// row when the caller needs full-row sums); item t goes to warp t mod 14.
// The warp reduces its item against the B activation rows in shared memory
// (kept in registers for B == 1) and calls out(t, sums, lane) with the fp32
// sums valid in every lane.
template <int B, class Out>
__device__ __noinline__ bool gemv_phase(const Params& p, Ring& ring_io, uint32_t xs_s, int K,
                                        int nseg, int rows_per_unit, int grp, Split sp, int where,
                                        Out& out_io) {
  constexpr int NC = kConsumerWarps;
  Ring ring = ring_io;  // registers for the loop; written back on every exit
  RingWriteBack wb{ring_io, ring};
  Out out = out_io;  // likewise the output functor's state
  struct OutWriteBack {
    Out& dst;
    const Out& src;
    __device__ ~OutWriteBack() { dst = src; }
  } owb{out_io, out};
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seg = K / nseg;
  const int CH = seg >> 8;
  const int piece_bytes = seg * 2;
  const int unit_bytes = rows_per_unit * K * 2;
  const int ups = units_per_slot(unit_bytes);
  const int ipu = rows_per_unit * nseg / grp;  // items per unit
  uint4 xr[8];
  int cached = -1;
  for (int s0 = sp.u0; s0 < sp.u1; s0 += ups) {
    const int n = min(ups, sp.u1 - s0);
    const int P = n * ipu;                 // items in this fill
    const int t0 = (s0 - sp.u0) * ipu;     // phase-local index of its first item
    const uint32_t f = ring.n++;
    const int lead = t0 % NC;
    const int first = t0 + (warp - lead + NC) % NC;
    if (first >= t0 + P) continue;
    if (!ring_wait(p, ring, f, where)) return false;
    const uint32_t sbase = ring.slots_s + (f % ring.S) * kSlotBytes + lane * 16;
    for (int t = first; t < t0 + P; t += NC) {
      float acc[B][4];
#pragma unroll
      for (int b = 0; b < B; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
      for (int k = 0; k < grp; ++k) {
        const int q = t * grp + k;  // phase-local piece index
        const int j = q % nseg;     // its column segment
        if (B == 1 && j != cached) {
          const uint32_t xa = xs_s + (uint32_t)(j * seg + lane * 8) * 2;
#pragma unroll
          for (int c = 0; c < 8; ++c)
            if (c < CH) xr[c] = lds128(xa + c * 512);
          cached = j;
        }
        const uint32_t wa = sbase + (uint32_t)(q - t0 * grp) * piece_bytes;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          if (c < CH) {
            const uint4 w = lds128(wa + c * 512);
#pragma unroll
            for (int b = 0; b < B; ++b) {
              const uint4 x =
                  (B == 1) ? xr[c]
                           : lds128(xs_s + (uint32_t)(b * p.kmax + j * seg + c * 256 + lane * 8) * 2);
              fma2_bf16(w.x, x.x, acc[b][0], acc[b][1]);
              fma2_bf16(w.y, x.y, acc[b][2], acc[b][3]);
              fma2_bf16(w.z, x.z, acc[b][0], acc[b][1]);
              fma2_bf16(w.w, x.w, acc[b][2], acc[b][3]);
            }
          }
        }
      }
      float v[B];
#pragma unroll
      for (int b = 0; b < B; ++b) v[b] = warp_sum((acc[b][0] + acc[b][1]) + (acc[b][2] + acc[b][3]));
      out(t, v, lane);
    }
    ring_release(ring, f, (P < NC && warp == lead) ? (uint32_t)(NC - P + 1) : 1u);
  }
  return true;
}


static_assert(kConsumerThreads >= kGroup * kHeadDim + kGroup * kMaxSplit,
              "merge_splits needs a thread per (head, dim) plus one per (head, split)");
static_assert(kGroup * kMaxSplit * 2 <= kAttnWarps * kGroup * kPartialStride,
              "merge_splits keeps its (m, l) table in the attention scratch");

// Split 0 of a (seq b, kv head g) merges the tagged (o, m, l) partials of
// all ns splits (blocks base + s * kGroup * kPartialStride; split 0 holds the
// new token's own K/V, so the sum of l is > 0) and writes the group's tagged
// bf16 head outputs to `out`. The merge is
//   M = max_s m_s,  o = sum_s exp(m_s - M) o_s / sum_s exp(m_s - M) l_s
// summed in split order. Every load is issued before any is used; a word
// whose tag is not yet there is polled (bounded). All consumer threads call
// it; false on abort or timeout. Inlined: as a call it made attention_phase
// keep more values in local memory across it (0.3-0.5 % slower per step).
__device__ __forceinline__ bool merge_splits(const Params& p, const unsigned long long* base, int ns,
                                          float* ml, uint32_t ptag, uint32_t* out, uint32_t otag,
                                          int where) {
  constexpr int kChunk = 4;  // o loads in flight per thread
  const int tid = threadIdx.x;
  const bool worker = tid < kGroup * kHeadDim;
  const int hh = (tid >> 6) & (kGroup - 1), d = tid & 63;
  const size_t step = (size_t)kGroup * kPartialStride;
  const unsigned long long* ob = base + hh * kPartialStride + d;  // split s: ob + s * step
  unsigned long long v[kChunk];
  bool ok = true;
  if (worker) {
#pragma unroll
    for (int j = 0; j < kChunk; ++j)
      if (j < ns) v[j] = __ldcg(ob + j * step);
  } else if (tid < kGroup * kHeadDim + kGroup * ns) {
    const int i = tid - kGroup * kHeadDim, h2 = i / ns, s = i % ns;
    const unsigned long long* w = base + s * step + h2 * kPartialStride + kHeadDim;
    const unsigned long long vm = __ldcg(w), vl = __ldcg(w + 1);
    float m = 0.f, l = 0.f;
    ok = value64(p, w, vm, ptag, m, where) && value64(p, w + 1, vl, ptag, l, where);
    ml[(h2 * kMaxSplit + s) * 2] = m;
    ml[(h2 * kMaxSplit + s) * 2 + 1] = l;
  }
  if (consumer_any(!ok)) return false;  // also the barrier before ml is read
  if (worker) {
    const float* mh = ml + hh * kMaxSplit * 2;
    float M = -INFINITY;
    for (int s = 0; s < ns; ++s) M = fmaxf(M, mh[2 * s]);
    float L = 0.f, O = 0.f;
    for (int s0 = 0; s0 < ns && ok; s0 += kChunk) {
      if (s0 > 0) {
#pragma unroll
        for (int j = 0; j < kChunk; ++j)
          if (s0 + j < ns) v[j] = __ldcg(ob + (s0 + j) * step);
      }
#pragma unroll
      for (int j = 0; j < kChunk; ++j) {
        if (s0 + j < ns && ok) {
          float o = 0.f;
          ok = value64(p, ob + (s0 + j) * step, v[j], ptag, o, where);
          const float m = mh[2 * (s0 + j)];
          if (m > -INFINITY) {
            const float f = __expf(m - M);
            L += f * mh[2 * (s0 + j) + 1];
            O += f * o;
          }
        }
      }
    }
    if (ok) out[hh * kHeadDim + d] = tagged(O / L, otag);
  }
  return !consumer_any(!ok);
}

// Online-softmax merge of another (m, l, o[8]) state into this lane's.
__device__ __forceinline__ void softmax_merge(float& m, float& l, float (&o)[8], float m2, float l2,
                                              const float (&o2)[8]) {
  const float M = fmaxf(m, m2);
  if (M == -INFINITY) return;
  const float a1 = (m == -INFINITY) ? 0.f : __expf(m - M);
  const float a2 = (m2 == -INFINITY) ? 0.f : __expf(m2 - M);
  l = l * a1 + l2 * a2;
#pragma unroll
  for (int e = 0; e < 8; ++e) o[e] = o[e] * a1 + o2[e] * a2;
  m = M;
}

// Split-K GQA flash-decode for the CTA's items. A chunk of kAttnChunk
// positions is spread over the consumer warps, four each: lane (h, j) of a warp
// scores position 4w + j/2 against q head h over half of the head dims (the
// other half on lane j^1), with q kept in registers as packed bf16, then
// accumulates dims [8j, 8j + 8) of P.V. Warp states are merged in shared
// memory; a single split writes the heads' output itself, several splits
// publish tagged partials that split 0 merges. Inlined into the consumer
// loop: as a call it cost 2.7 % of the step (registers saved to local memory
// around the call; the result is bit-identical).
template <int B>
__device__ __forceinline__ bool attention_phase(const Params& p, Ring& ring_io, SmemState& st,
                                             int layer, float* comb, bf16* qs, float* kvn) {
  constexpr int NC = kConsumerWarps;
  Ring ring = ring_io;
  RingWriteBack wb{ring_io, ring};
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int NQKV = p.NQ + 2 * p.NKV;
  const int ns = st.n_split;
  const int T = B * p.NKV * ns;
  const float scale = 0.125f;  // head_dim ** -0.5
  const int h = lane >> 3, j = lane & 7;
  const int pp = j >> 1, half = j & 1;
  for (int it = blockIdx.x; it < T; it += gridDim.x) {
    const AttnItem a = attn_item(p, st, it);
    consumer_sync();
    // q of the group's heads, and the new token's own K and V row, polled
    // until the QKV phase's tag is on them (one round trip when ready).
    bool qfail = false;
    {
      const uint32_t tag = phase_tag(p, layer * 5 + 0);
      constexpr int kQ4 = kGroup * kHeadDim / 4;  // q words in uint4s
      if (tid < kQ4 + 2 * kHeadDim / 4) {
        const bool is_q = tid < kQ4;
        const int r = is_q ? tid : tid - kQ4;  // uint4 index within q, or within K|V
        const int head = is_q ? a.g * kGroup : (r < kHeadDim / 4 ? p.NQ + a.g : p.NQ + p.NKV + a.g);
        const int off = is_q ? r * 4 : (r % (kHeadDim / 4)) * 4;
        uint4 u;
        if (!poll_tagged(p, p.qkv + ((size_t)a.b * NQKV + head) * kHeadDim + off, tag, u, 3000 + layer)) {
          qfail = true;
        } else if (is_q) {
          reinterpret_cast<uint2*>(qs)[r] = untag4(u);
        } else {
          float* dst = kvn + (r / (kHeadDim / 4)) * kHeadDim + off;
          dst[0] = __uint_as_float(u.x & 0xFFFF0000u);
          dst[1] = __uint_as_float(u.y & 0xFFFF0000u);
          dst[2] = __uint_as_float(u.z & 0xFFFF0000u);
          dst[3] = __uint_as_float(u.w & 0xFFFF0000u);
        }
      }
    }
    if (consumer_any(qfail)) return false;
    if (p.trace && tid == 0) trace_put(p, layer * 5 + 1, kTrAttnQ, global_ns());
    uint4 qh[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) qh[c] = reinterpret_cast<const uint4*>(qs + h * kHeadDim + half * 32)[c];
    float m = -INFINITY, l = 0.f, o[8];
    bool fail = false;
#pragma unroll
    for (int e = 0; e < 8; ++e) o[e] = 0.f;
    for (int c0 = a.p0; c0 < a.p1; c0 += kAttnChunk) {
      const int n = min(kAttnChunk, a.p1 - c0);
      const int nw = min(NC, (n + 3) >> 2);  // warps with positions in this chunk
      const uint32_t f = ring.n++;
      if (fail || warp >= nw) continue;
      if (!ring_wait(p, ring, f, 200 + layer)) {
        fail = true;
        continue;
      }
      const uint8_t* slot = ring.slots + (size_t)(f % ring.S) * kSlotBytes;
      const uint8_t* vbase = slot + 8192;
      for (int base = warp * 4; base < n; base += NC * 4) {
        const int pc = base + pp;
        const bool valid = pc < n;
        float sc = -INFINITY;
        if (valid) {
          const uint4* k4 = reinterpret_cast<const uint4*>(slot + pc * kHeadDim * 2 + half * 64);
          float s0 = 0.f, s1 = 0.f;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 kw = k4[c];
            fma2_bf16(kw.x, qh[c].x, s0, s1);
            fma2_bf16(kw.y, qh[c].y, s0, s1);
            fma2_bf16(kw.z, qh[c].z, s0, s1);
            fma2_bf16(kw.w, qh[c].w, s0, s1);
          }
          sc = s0 + s1;
        }
        sc += __shfl_xor_sync(0xffffffffu, sc, 1);  // the two halves of the dot
        sc *= scale;
        float cmax = fmaxf(sc, __shfl_xor_sync(0xffffffffu, sc, 2));
        cmax = fmaxf(cmax, __shfl_xor_sync(0xffffffffu, cmax, 4));
        const float m_new = fmaxf(m, cmax);
        const float alpha = (m == -INFINITY) ? 0.f : __expf(m - m_new);
        const float pe = valid ? __expf(sc - m_new) : 0.f;
        float ps = half == 0 ? pe : 0.f;
        ps += __shfl_xor_sync(0xffffffffu, ps, 1);
        ps += __shfl_xor_sync(0xffffffffu, ps, 2);
        ps += __shfl_xor_sync(0xffffffffu, ps, 4);
        l = l * alpha + ps;
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] *= alpha;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float pv = __shfl_sync(0xffffffffu, pe, (lane & ~7) | (q * 2));
          if (base + q < n) {
            const uint4 vv = reinterpret_cast<const uint4*>(vbase + (base + q) * kHeadDim * 2)[j];
            float vf[8];
            unpack8(vv, vf);
#pragma unroll
            for (int e = 0; e < 8; ++e) o[e] = fmaf(pv, vf[e], o[e]);
          }
        }
        m = m_new;
      }
      ring_release(ring, f, warp == 0 ? (uint32_t)(NC - nw + 1) : 1u);
    }
    // Split 0 also takes the new token's own K/V (the "active slot"), on
    // warp 0: lane (h, j) adds dims [8j, 8j + 8) of q_h . k_new, reduced
    // over the head's eight lanes.
    if (a.s == 0 && warp == 0) {
      float qf[8];
      unpack8(reinterpret_cast<const uint4*>(qs + h * kHeadDim)[j], qf);
      float sa = 0.f;
#pragma unroll
      for (int e = 0; e < 8; ++e) sa = fmaf(qf[e], kvn[j * 8 + e], sa);
      sa += __shfl_xor_sync(0xffffffffu, sa, 1);
      sa += __shfl_xor_sync(0xffffffffu, sa, 2);
      sa += __shfl_xor_sync(0xffffffffu, sa, 4);
      sa *= scale;
      const float m_new = fmaxf(m, sa);
      const float alpha = (m == -INFINITY) ? 0.f : __expf(m - m_new);
      const float pe = __expf(sa - m_new);
      l = l * alpha + pe;
#pragma unroll
      for (int e = 0; e < 8; ++e) o[e] = o[e] * alpha + pe * kvn[kHeadDim + j * 8 + e];
      m = m_new;
    }
    if (p.trace && tid == 0) trace_put(p, layer * 5 + 1, kTrAttnChunks, global_ns());
    if (consumer_any(fail)) return false;
    // Merge the warps' states: warps 8.. into 0.. through shared memory,
    // then 0..7 into one state per (head, dim).
    auto put = [&](int w) {
      float* cw = comb + (w * kGroup + h) * kPartialStride;
#pragma unroll
      for (int e = 0; e < 8; ++e) cw[j * 8 + e] = o[e];
      if (j == 0) {
        cw[kHeadDim] = m;
        cw[kHeadDim + 1] = l;
      }
    };
    if (warp >= kAttnWarps) put(warp - kAttnWarps);
    consumer_sync();
    if (warp + kAttnWarps < NC) {
      const float* cw = comb + (warp * kGroup + h) * kPartialStride;
      float o2[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) o2[e] = cw[j * 8 + e];
      softmax_merge(m, l, o, cw[kHeadDim], cw[kHeadDim + 1], o2);
    }
    consumer_sync();
    if (warp < kAttnWarps) put(warp);
    consumer_sync();
    static_assert(kConsumerWarps >= kAttnWarps && kConsumerWarps <= 2 * kAttnWarps,
                  "attention merge assumes kAttnWarps <= warps <= 2 * kAttnWarps");
    if (tid < kGroup * kHeadDim) {
      const int hh = tid >> 6, d = tid & 63;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kAttnWarps; ++w)
        M = fmaxf(M, comb[(w * kGroup + hh) * kPartialStride + kHeadDim]);
      float L = 0.f, O = 0.f;
      if (M > -INFINITY) {
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
          const float* cwp = comb + (w * kGroup + hh) * kPartialStride;
          const float mw = cwp[kHeadDim];
          if (mw > -INFINITY) {
            const float f = __expf(mw - M);
            L += f * cwp[kHeadDim + 1];
            O += f * cwp[d];
          }
        }
      }
      if (ns == 1) {
        // The only split (it holds the active slot, so L > 0): final output.
        p.attn[(size_t)a.b * p.NQ * kHeadDim + (a.g * kGroup + hh) * kHeadDim + d] =
            tagged(O / L, phase_tag(p, layer * 5 + 1));
      } else {
        // Publish this split's partial state; split 0 merges.
        unsigned long long* pp2 = p.partials + ((size_t)it * kGroup + hh) * kPartialStride;
        const uint32_t ptag = p.part_tag0 + (uint32_t)layer;
        pp2[d] = tagged64(O, ptag);
        if (d == 0) {
          pp2[kHeadDim] = tagged64(M, ptag);
          pp2[kHeadDim + 1] = tagged64(L, ptag);
        }
      }
    }
    if (p.trace && tid == 0) trace_put(p, layer * 5 + 1, kTrAttnArrive, global_ns());
    if (ns == 1 || a.s != 0) continue;  // the tagged words written above are the publication
    consumer_sync();  // comb is free again; split 0's own partials are written
    if (!merge_splits(p, p.partials + (size_t)it * kGroup * kPartialStride, ns, comb,
                      p.part_tag0 + (uint32_t)layer,
                      p.attn + (size_t)a.b * p.NQ * kHeadDim + a.g * kGroup * kHeadDim,
                      phase_tag(p, layer * 5 + 1), 3100 + layer))
      return false;
    if (p.trace && tid == 0) trace_put(p, layer * 5 + 1, kTrAttnMerged, global_ns());
    break;  // with ns > 1 a CTA has one item at most (T <= grid)
  }
  return true;
}

// GEMV phase output: one fp32 partial per piece, into shared memory.
template <int B>
struct ToPart {
  float* part;
  __device__ void operator()(int q, const float (&v)[B], int lane) const {
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b) part[q * B + b] = v[b];
    }
  }
};

// lm_head output: optional fp32 logits and this warp's running greedy
// argmax (lowest index on ties), kept by lane 0.
template <int B>
struct LmOut {
  float* logits;  // [B][rows]: this rank's lm_head rows
  int rows, u0, row0;  // row u of the slice is vocabulary id row0 + u
  float best_v[B];
  int best_i[B];
  __device__ void operator()(int t, const float (&v)[B], int lane) {
    if (lane != 0) return;
    const int u = u0 + t, id = row0 + u;
#pragma unroll
    for (int b = 0; b < B; ++b) {
      if (logits) logits[(size_t)b * rows + u] = v[b];
      if (v[b] > best_v[b] || (v[b] == best_v[b] && id < best_i[b])) {
        best_v[b] = v[b];
        best_i[b] = id;
      }
    }
  }
};

template <int B>
__device__ void run_consumers(const Params& p, SmemState& st, Ring& ring, bf16* xs, float* part,
                              float* comb, bf16* qs, float* kvn, bf16* raw, bf16* rope) {
  const int tid = threadIdx.x;
  // This step's RoPE rows (cos, sin per sequence), used by every layer.
  if (tid < B * 2 * kHeadDim / 8) {
    const int b = tid / (2 * kHeadDim / 8), r = tid % (2 * kHeadDim / 8);
    const bf16* tab = (r < kHeadDim / 8) ? p.rope_cos : p.rope_sin;
    reinterpret_cast<uint4*>(rope + b * 2 * kHeadDim)[r] =
        __ldg(reinterpret_cast<const uint4*>(tab + (size_t)st.pos[b] * kHeadDim) + (r % (kHeadDim / 8)));
  }
  const int H = p.H, I = p.I, QD = p.NQ * kHeadDim, NQKV = p.NQ + 2 * p.NKV;
  const uint32_t xs_s = smem_addr(xs);
  Sched sch;
  auto mark = [&](int ph, int kind) {
    if (p.trace && threadIdx.x == 0) trace_put(p, ph, kind, global_ns());
  };
  auto mark_done = [&](int ph) {
    if (p.trace && threadIdx.x == 0) {
      trace_put(p, ph, kTrDone, global_ns());
      trace_put(p, ph, kTrConsStall, ring.stall_ns);
    }
  };
  // Phase-local partial sums: part[piece * B + b].
  ToPart<B> to_part{part};
  // Sum of a row's nseg pieces (fixed order).
  auto row_sum = [&](int q0, int nseg, int b) {
    float s = part[q0 * B + b];
    for (int k = 1; k < nseg; ++k) s += part[(q0 + k) * B + b];
    return s;
  };

  for (int l = 0; l < p.L; ++l) {
    // ------------------------------------------------------------- QKV
    mark(l * 5 + 0, kTrWaitStart);
    mark(l * 5 + 0, kTrWaitDone);
    if (l == 0) {
      const bf16* src[B];
#pragma unroll
      for (int b = 0; b < B; ++b)
        src[b] = p.mode == 0 ? p.embed + (size_t)st.tok[b] * H : p.hidden_in + (size_t)b * H;
      load_rows<B>(src, H, p.norm_attn, p.eps, xs, p.kmax, st, raw);
    } else {
      RowPtrs<B> src;
#pragma unroll
      for (int b = 0; b < B; ++b) src.r[b] = p.h + (size_t)b * H;
      if (!load_rows_tagged<B>(p, src, H, phase_tag(p, (l - 1) * 5 + 4), p.norm_attn + (size_t)l * H,
                               p.eps, xs, p.kmax, st, 1000 + l, raw))
        return;
    }
    mark(l * 5 + 0, kTrRowsLoaded);
    const Split sq = sch.next(NQKV * 32);
    bool ok = gemv_phase<B>(p, ring, xs_s, H, p.nseg_h, 2, 1, sq, 2000 + l, to_part);
    if (consumer_any(!ok)) return;
    // The failure-detection knob: one CTA withholds its layer-0 q/k/v rows,
    // so the attention reads that poll for them run out of time.
    if (!(l == 0 && (int)blockIdx.x == p.debug_skip_cta)) {
      const size_t kv_layer = (size_t)l * p.num_pages * p.NKV * p.page_size * kHeadDim;
      const uint32_t tag = phase_tag(p, l * 5 + 0);
      const int nu = sq.u1 - sq.u0, ns = p.nseg_h;
      for (int i = tid; i < nu * B; i += kConsumerThreads) {
        const int ul = i / B, b = i % B, u = sq.u0 + ul;
        const int hh = u >> 5, d = u & 31;
        float x0 = rbf(row_sum(ul * 2 * ns, ns, b));
        float x1 = rbf(row_sum(ul * 2 * ns + ns, ns, b));
        const int pos = st.pos[b];
        if (hh < p.NQ + p.NKV) {
          const bf16* cr = rope + b * 2 * kHeadDim;
          const bf16* sr = cr + kHeadDim;
          const float c0 = bf2f(cr[d]), c1 = bf2f(cr[d + 32]);
          const float s0 = bf2f(sr[d]), s1 = bf2f(sr[d + 32]);
          const float y0 = rbf(rbf(x0 * c0) + rbf(-x1 * s0));
          const float y1 = rbf(rbf(x1 * c1) + rbf(x0 * s1));
          x0 = y0;
          x1 = y1;
        }
        uint32_t* qrow = p.qkv + ((size_t)b * NQKV + hh) * kHeadDim;
        qrow[d] = tagged(x0, tag);
        qrow[d + 32] = tagged(x1, tag);
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
    }
    mark_done(l * 5 + 0);

    // ------------------------------------------------------------- ATTN
    mark(l * 5 + 1, kTrWaitStart);
    mark(l * 5 + 1, kTrWaitDone);
    if (!attention_phase<B>(p, ring, st, l, comb, qs, kvn)) return;
    mark_done(l * 5 + 1);

    // ------------------------------------------------------------- O
    mark(l * 5 + 2, kTrWaitStart);
    mark(l * 5 + 2, kTrWaitDone);
    {
      RowPtrs<B> src;
#pragma unroll
      for (int b = 0; b < B; ++b) src.r[b] = p.attn + (size_t)b * QD;
      if (!load_rows_tagged<B>(p, src, QD, phase_tag(p, l * 5 + 1), nullptr, 0.f, xs, p.kmax, st,
                               4000 + l, nullptr))
        return;
    }
    mark(l * 5 + 2, kTrRowsLoaded);
    {
      const Split so = sch.next(H);
      ok = gemv_phase<B>(p, ring, xs_s, QD, p.nseg_qd, 1, 1, so, 5000 + l, to_part);
      if (consumer_any(!ok)) return;
      const int nu = so.u1 - so.u0, ns = p.nseg_qd;
      const uint32_t tag = phase_tag(p, l * 5 + 2);
      if (p.tp_world > 1) {
        const uint32_t xtag = xchg_tag(p, l * 5 + 2);
        for (int i = tid; i < nu * B; i += kConsumerThreads)
          tp_publish(p, 0, i % B, so.u0 + i / B, row_sum((i / B) * ns, ns, i % B), xtag);
        int good = 1;
        for (int i = tid; i < nu * B && good; i += kConsumerThreads) {
          const int b = i % B, u = so.u0 + i / B;
          const Summed o = tp_sum(p, 0, b, u, xtag, 4500 + l);
          good = o.ok;
          p.h[(size_t)b * H + u] = tagged(bf2f(raw[b * H + u]) + rbf(o.v), tag);
        }
        if (consumer_any(!good)) return;
      } else {
        for (int i = tid; i < nu * B; i += kConsumerThreads) {
          const int ul = i / B, b = i % B, u = so.u0 + ul;
          // residual: the layer input, kept raw by the QKV phase's row load
          const float r = bf2f(raw[b * H + u]);
          p.h[(size_t)b * H + u] = tagged(r + rbf(row_sum(ul * ns, ns, b)), tag);
        }
      }
    }
    mark_done(l * 5 + 2);

    // ------------------------------------------------------------- GU
    mark(l * 5 + 3, kTrWaitStart);
    mark(l * 5 + 3, kTrWaitDone);
    {
      RowPtrs<B> src;
#pragma unroll
      for (int b = 0; b < B; ++b) src.r[b] = p.h + (size_t)b * H;
      if (!load_rows_tagged<B>(p, src, H, phase_tag(p, l * 5 + 2), p.norm_mlp + (size_t)l * H, p.eps,
                               xs, p.kmax, st, 6000 + l, raw))
        return;
    }
    mark(l * 5 + 3, kTrRowsLoaded);
    {
      const Split sg = sch.next(I);
      ok = gemv_phase<B>(p, ring, xs_s, H, p.nseg_h, 2, 1, sg, 7000 + l, to_part);
      if (consumer_any(!ok)) return;
      const int nu = sg.u1 - sg.u0, ns = p.nseg_h;
      for (int i = tid; i < nu * B; i += kConsumerThreads) {
        const int ul = i / B, b = i % B, u = sg.u0 + ul;
        const float g = rbf(row_sum(ul * 2 * ns, ns, b));
        const float up = rbf(row_sum(ul * 2 * ns + ns, ns, b));
        const float s = rbf(__fdiv_rn(g, 1.0f + expf(-g)));
        p.act[(size_t)b * I + u] = tagged(s * up, phase_tag(p, l * 5 + 3));
      }
    }
    mark_done(l * 5 + 3);

    // ------------------------------------------------------------- DOWN
    mark(l * 5 + 4, kTrWaitStart);
    mark(l * 5 + 4, kTrWaitDone);
    {
      RowPtrs<B> src;
#pragma unroll
      for (int b = 0; b < B; ++b) src.r[b] = p.act + (size_t)b * I;
      if (!load_rows_tagged<B>(p, src, I, phase_tag(p, l * 5 + 3), nullptr, 0.f, xs, p.kmax, st,
                               8000 + l, nullptr))
        return;
    }
    mark(l * 5 + 4, kTrRowsLoaded);
    const bool last_layer = (l == p.L - 1);
    {
      const Split sd = sch.next(H);
      ok = gemv_phase<B>(p, ring, xs_s, I, p.nseg_i, 1, 1, sd, 9000 + l, to_part);
      if (consumer_any(!ok)) return;
      const int nu = sd.u1 - sd.u0, ns = p.nseg_i;
      const uint32_t tag = phase_tag(p, l * 5 + 4);
      if (p.tp_world > 1) {
        const uint32_t xtag = xchg_tag(p, l * 5 + 4);
        for (int i = tid; i < nu * B; i += kConsumerThreads)
          tp_publish(p, 1, i % B, sd.u0 + i / B, row_sum((i / B) * ns, ns, i % B), xtag);
        int good = 1;
        for (int i = tid; i < nu * B && good; i += kConsumerThreads) {
          const int b = i % B, u = sd.u0 + i / B;
          const Summed d = tp_sum(p, 1, b, u, xtag, 8500 + l);
          good = d.ok;
          const float y = bf2f(raw[b * H + u]) + rbf(d.v);
          p.h[(size_t)b * H + u] = tagged(y, tag);
          if (last_layer && p.mode == 1) p.hidden_out[(size_t)b * H + u] = f2bf(y);
        }
        if (consumer_any(!good)) return;
      } else {
        for (int i = tid; i < nu * B; i += kConsumerThreads) {
          const int ul = i / B, b = i % B, u = sd.u0 + ul;
          // residual: h after o_proj, kept raw by the GU phase's row load
          const float r = bf2f(raw[b * H + u]);
          const float y = r + rbf(row_sum(ul * ns, ns, b));
          p.h[(size_t)b * H + u] = tagged(y, tag);
          if (last_layer && p.mode == 1) p.hidden_out[(size_t)b * H + u] = f2bf(y);
        }
      }
    }
    mark_done(l * 5 + 4);
  }

  // --------------------------------------------------------------- LM head
  if (p.mode == 0) {
    mark(p.L * 5, kTrWaitStart);
    mark(p.L * 5, kTrWaitDone);
    {
      RowPtrs<B> src;
#pragma unroll
      for (int b = 0; b < B; ++b) src.r[b] = p.h + (size_t)b * H;
      if (!load_rows_tagged<B>(p, src, H, phase_tag(p, (p.L - 1) * 5 + 4), p.norm_final, p.eps, xs,
                               p.kmax, st, 10000, nullptr))
        return;
    }
    mark(p.L * 5, kTrRowsLoaded);
    const Split sl = sch.next(p.lm_rows);
    LmOut<B> lm{p.logits, p.lm_rows, sl.u0, p.lm_row0};
#pragma unroll
    for (int b = 0; b < B; ++b) {
      lm.best_v[b] = -INFINITY;
      lm.best_i[b] = 0x7fffffff;
    }
    // One item per lm_head row (all its pieces), so the warp has the logit.
    const bool ok = gemv_phase<B>(p, ring, xs_s, H, p.nseg_h, 1, p.nseg_h, sl, 11000, lm);
    if (consumer_any(!ok)) return;
    mark_done(p.L * 5);
    const int lane = tid & 31, w = tid >> 5;
    if (lane == 0) {
#pragma unroll
      for (int b = 0; b < B; ++b) {
        st.am_val[w * B + b] = lm.best_v[b];
        st.am_idx[w * B + b] = lm.best_i[b];
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
    const uint32_t t = atom_add_acq_rel_u32(p.counters + kCntDone, 1u);
    if (t == gridDim.x - 1) {
      if (p.mode == 0) {
        unsigned long long key[B];
        for (int b = 0; b < B; ++b) key[b] = atomicExch(p.keys + b, 0ull);
        if (p.tp_world == 1 || tp_argmax(p, key, xchg_tag(p, p.L * 5))) {
          for (int b = 0; b < B; ++b) {
            const int id = (int)(0xFFFFFFFFu - (uint32_t)(key[b] & 0xFFFFFFFFull));
            p.next_ids[b] = id;
            if (p.flags & 1) {
              p.tokens[b] = id;
              p.positions[b] = st.pos[b] + 1;
            }
          }
        }
      }
      atomicExch(p.counters + kCntDone, 0u);
      __threadfence();
    }
  }
}

template <int B>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  const int S = p.num_slots;
  uint8_t* cur = smem;
  uint8_t* ring_mem = cur;
  cur += (size_t)S * kSlotBytes;
  bf16* xs = reinterpret_cast<bf16*>(cur);
  cur += align128(B * p.kmax * 2);
  float* part = reinterpret_cast<float*>(cur);
  cur += align128(p.part_cap * 4);
  bf16* raw = reinterpret_cast<bf16*>(cur);
  cur += align128(B * p.H * 2);
  bf16* rope = reinterpret_cast<bf16*>(cur);
  cur += align128(B * 2 * kHeadDim * 2);
  float* comb = reinterpret_cast<float*>(cur);
  bf16* qs = reinterpret_cast<bf16*>(comb + kAttnWarps * kGroup * kPartialStride);
  float* kvn = reinterpret_cast<float*>(qs + kGroup * kHeadDim);
  cur += kAttnScratchBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(cur);
  SmemState* st = reinterpret_cast<SmemState*>(bars + kFullBars + S);

  Ring ring{ring_mem, smem_addr(ring_mem), bars, bars + kFullBars, S};

  if (threadIdx.x == 0) {
    for (int s = 0; s < kFullBars; ++s) mbar_init(&ring.full[s], 1);
    for (int s = 0; s < S; ++s) mbar_init(&ring.empty[s], kConsumerWarps);
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
    // Split-K pieces per (seq, kv head): at most one item per CTA, and no
    // piece shorter than kSplitMinPositions (fewer partials to merge).
    int ns = min(kMaxSplit, max(1, (int)gridDim.x / (B * p.NKV)));
    ns = max(1, min(ns, (pmax + kSplitMinPositions - 1) / kSplitMinPositions));
    st->n_split = ns;
    st->flag = bad ? 1 : 0;
    for (int k = 0; k < kProducers; ++k) st->prod_pos[k] = 0;
  }
  __syncthreads();
  if (st->flag) return;

  const int warp = threadIdx.x >> 5;
  if (warp >= kProducerWarp && warp < kProducerWarp + kProducers) {
    if ((threadIdx.x & 31) == 0) {
      Producer pr{p, ring, *st, policy_evict_first(), warp - kProducerWarp};
      walk_schedule<B>(p, *st, pr);
      if (!pr.ok) pr.drain();
    }
    return;
  }
  run_consumers<B>(p, *st, ring, xs, part, comb, qs, kvn, raw, rope);
}

}  // namespace mk
