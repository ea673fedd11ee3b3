// mk_api.cu — C ABI (include/mk.h) around the persistent decode megakernel.
//
// The handle owns the inter-phase scratch (residual, q/k/v, attention
// partials, barrier counters, argmax keys, the device error word); everything
// else is borrowed from the caller per call. Launches are cooperative so all
// CTAs (one per SM) are co-resident, which the kernel's cross-CTA waits need.
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/mk.h"
#include "mk_kernel.cuh"
#include "mk_sample.cuh"
#include "mk_attn.cuh"
#include "mk_batched.cuh"
#include "mk_gemm.cuh"

namespace {

thread_local std::string g_last_error;

constexpr uint64_t kPartTagLimit = 0xFFFFFFFFull;  // attention partial tags stay below this

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define MK_CUDA(call)                                                                    \
  do {                                                                                   \
    cudaError_t e_ = (call);                                                             \
    if (e_ != cudaSuccess) return fail(MK_ECUDA, "%s: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

struct MkModel {
  MkConfig cfg;
  int device = 0;
  int num_sms = 0;
  int grid = 0;
  int num_slots = 0;
  int smem = 0;
  int kmax = 0;
  int part_cap = 0;
  bool has_weights = false;
  MkWeights w{};
  unsigned long long timeout_ns = 2000000000ull;
  int debug_skip_cta = -1;
  // scratch
  void* scratch = nullptr;
  uint32_t* h = nullptr;     // tagged activation words (see mk_kernel.cuh)
  uint32_t* qkv = nullptr;
  uint32_t* attn = nullptr;
  uint32_t* act = nullptr;
  // Activation tags: the next launch's first tag, and the tagged words
  // (h, qkv, attn, act: one contiguous range) zeroed before it would wrap.
  uint32_t tag_next = 0;
  void* act_words = nullptr;
  size_t act_bytes = 0;
  uint64_t xtag_next = 1;    // tensor-parallel exchange tags (32-bit, never 0)
  unsigned long long* partials = nullptr;  // attention split partials (tagged 64-bit words)
  size_t partials_bytes = 0;
  uint64_t part_tag_next = 0;  // partial tags used so far in the current tag sequence
  uint32_t* counters = nullptr;
  unsigned long long* keys = nullptr;
  int* error = nullptr;
  int* host_error = nullptr;      // mapped pinned mirror, read by mk_sync
  int* host_error_dev = nullptr;  // its device address
  // mk_decode_host staging: tokens, positions, next ids ([3][max_batch] int32)
  int32_t* io_dev = nullptr;   // in the scratch allocation
  int32_t* io_host = nullptr;  // pinned
  size_t counters_bytes = 0;
  unsigned long long* trace = nullptr;  // borrowed, see mk_set_trace
  // tensor parallelism (mk_tp_setup / mk_tp_connect)
  int tp_rank = 0, tp_world = 1;
  int lm_row0 = 0, lm_rows = -1;  // -1: the whole vocabulary
  unsigned long long* xbuf = nullptr;  // this rank's exchange buffer
  unsigned long long* xpeer[mk::kMaxTp] = {};
  bool xpeer_ipc[mk::kMaxTp] = {};  // opened with cudaIpcOpenMemHandle (closed on destroy)
  bool tp_connected = false;
};

namespace {
int64_t trace_entries(const MkModel* m) {
  return (int64_t)m->grid * (m->cfg.num_layers * 5 + 1) * mk::kTraceKinds;
}
}  // namespace

namespace {

// The consumer warps' ring waits are safe while a warp never goes more than
// kFullBars - S - kProducerSlack fills between two waits, and its first wait
// is on a fill below kFullBars (see the Ring comment in mk_kernel.cuh). This
// walks every CTA's fill schedule as the kernel does (walk_schedule and
// gemv_phase's item -> warp map) and returns the largest such gap. Attention
// chunks are read by every warp except the last, partial chunk of an item, so
// each attention item of the CTA counts as one fill no warp reads; the item
// count is its maximum over positions.
int max_consumer_gap(const MkConfig* c, int B, int G, int lm_rows) {
  constexpr int NC = mk::kConsumerWarps;
  const int H = c->hidden, I = c->intermediate, QD = c->num_q_heads * 64;
  const int NQKV = c->num_q_heads + 2 * c->num_kv_heads;
  const int nh = mk::pieces_per_row(H), nqd = mk::pieces_per_row(QD), ni = mk::pieces_per_row(I);
  const int ns = std::min(mk::kMaxSplit, std::max(1, G / (B * c->num_kv_heads)));
  const int T = B * c->num_kv_heads * ns;
  int worst = 0;
  for (int cta = 0; cta < G; ++cta) {
    int rot = 0;
    long long f = 0;
    long long last[NC];
    for (int w = 0; w < NC; ++w) last[w] = -1;
    auto gemv = [&](int U, int unit_bytes, int ipu) {
      const mk::Split sp = mk::split_units(U, G, cta, rot);
      rot = (rot + U % G) % G;
      const int ups = mk::units_per_slot(unit_bytes);
      for (int u = sp.u0; u < sp.u1; u += ups, ++f) {
        const int P = std::min(ups, sp.u1 - u) * ipu, t0 = (u - sp.u0) * ipu;
        for (int w = 0; w < NC; ++w) {
          if (t0 + (w - t0 % NC + NC) % NC >= t0 + P) continue;  // no item for warp w
          if (f >= mk::kFullBars)
            worst = std::max(worst, last[w] < 0 ? INT32_MAX : (int)std::min<long long>(f - last[w], INT32_MAX));
          last[w] = f;
        }
      }
    };
    const int items = cta < T ? (T - 1 - cta) / G + 1 : 0;
    for (int l = 0; l < c->num_layers; ++l) {
      gemv(NQKV * 32, 4 * H, 2 * nh);
      f += items;
      gemv(H, 2 * QD, nqd);
      gemv(I, 4 * H, 2 * nh);
      gemv(H, 2 * I, ni);
    }
    gemv(lm_rows, 2 * H, 1);
  }
  return worst;
}

// Every batch a launch may use (1 .. max_batch) has its own schedule.
int check_schedule(const MkConfig* c, int max_batch, int G, int S, int lm_rows = -1) {
  const int bound = mk::kFullBars - S - mk::kProducerSlack;
  for (int B = 1; B <= max_batch; ++B) {
    const int gap = max_consumer_gap(c, B, G, lm_rows < 0 ? c->vocab : lm_rows);
    if (gap > bound)
      return fail(MK_EINVAL, "fill schedule at batch %d: a consumer warp would go %d fills between "
                  "ring waits (at most %d are safe with %d slots)", B,
                  gap == INT32_MAX ? -1 : gap, bound, S);
  }
  return MK_OK;
}

// check_schedule for the allocation-free entry point, which sets up on every
// call: geometries already checked are remembered.
int check_schedule_cached(const MkConfig* c, int B, int G, int S) {
  static std::mutex mu;
  static std::vector<std::array<int, 9>> ok;
  const std::array<int, 9> key = {c->num_layers, c->hidden, c->intermediate, c->num_q_heads,
                                  c->num_kv_heads, c->vocab, B, G, S};
  std::lock_guard<std::mutex> lock(mu);
  for (const auto& k : ok)
    if (k == key) return MK_OK;
  const int rc = check_schedule(c, B, G, S);
  if (rc == MK_OK) ok.push_back(key);
  return rc;
}

int validate_config(const MkConfig* c) {
  if (!c) return fail(MK_EINVAL, "config is NULL");
  if (c->num_layers <= 0 || c->num_layers > 1024)
    return fail(MK_EINVAL, "num_layers must be in [1, 1024] (got %d)", c->num_layers);
  if (c->head_dim != 64) return fail(MK_EINVAL, "head_dim must be 64 (got %d)", c->head_dim);
  if (c->num_kv_heads <= 0 || c->num_q_heads != 4 * c->num_kv_heads)
    return fail(MK_EINVAL, "num_q_heads must be 4 * num_kv_heads (got %d, %d)", c->num_q_heads,
                c->num_kv_heads);
  if (c->hidden <= 0 || c->hidden % 256 || c->hidden > 4096)
    return fail(MK_EINVAL, "hidden must be a multiple of 256 in [256, 4096] (got %d)", c->hidden);
  if (c->intermediate <= 0 || c->intermediate % 256 || c->intermediate > 8192)
    return fail(MK_EINVAL, "intermediate must be a multiple of 256 in [256, 8192] (got %d)",
                c->intermediate);
  if ((c->num_q_heads * 64) % 256 || c->num_q_heads * 64 > 8192)
    return fail(MK_EINVAL, "num_q_heads * 64 must be a multiple of 256, <= 8192");
  if (c->vocab <= 0) return fail(MK_EINVAL, "vocab must be > 0");
  if (!(c->rms_eps > 0.f)) return fail(MK_EINVAL, "rms_eps must be > 0");
  if (c->max_batch < 1 || c->max_batch > 4)
    return fail(MK_EINVAL, "max_batch must be in [1, 4] (got %d)", c->max_batch);
  if (c->page_size < 8 || c->page_size % 8)
    return fail(MK_EINVAL, "page_size must be a positive multiple of 8 (got %d)", c->page_size);
  if (c->num_pages <= 0 || c->max_blocks_per_seq <= 0)
    return fail(MK_EINVAL, "num_pages and max_blocks_per_seq must be > 0");
  if (c->rope_len <= 0) return fail(MK_EINVAL, "rope_len must be > 0");
  return MK_OK;
}

template <int B>
cudaError_t launch_b(const mk::Params& p, int grid, int smem, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(mk::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, mk::decode_kernel<B>, p);
}

template <int B>
cudaError_t set_smem_b(int smem) {
  return cudaFuncSetAttribute(mk::decode_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              smem);
}

template <int B>
cudaError_t occupancy_b(int* blocks, int smem) {
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, mk::decode_kernel<B>, mk::kThreads,
                                                       smem);
}

cudaError_t dispatch_launch(int B, const mk::Params& p, int grid, int smem, cudaStream_t s) {
  switch (B) {
    case 1: return launch_b<1>(p, grid, smem, s);
    case 2: return launch_b<2>(p, grid, smem, s);
    case 3: return launch_b<3>(p, grid, smem, s);
    case 4: return launch_b<4>(p, grid, smem, s);
  }
  return cudaErrorInvalidValue;
}

int enqueue(MkModel* m, int mode, const int32_t* tokens, const int32_t* positions, int32_t batch,
            const MkKVCache* kv, const void* hidden_in, void* hidden_out, float* logits,
            int32_t* next_ids, int32_t flags, void* stream) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  if (!m->has_weights) return fail(MK_ESTATE, "mk_load_weights has not been called");
  if (m->tp_world > 1 && !m->tp_connected)
    return fail(MK_ESTATE, "tensor-parallel rank: mk_tp_connect has not been called");
  if (batch < 1 || batch > m->cfg.max_batch)
    return fail(MK_EINVAL, "batch %d outside [1, max_batch=%d]", batch, m->cfg.max_batch);
  if (!positions) return fail(MK_EINVAL, "positions is NULL");
  if (!kv || !kv->k_pages || !kv->v_pages || !kv->block_tables)
    return fail(MK_EINVAL, "KV cache pointers must be non-NULL");
  if (!aligned16(kv->k_pages) || !aligned16(kv->v_pages))
    return fail(MK_EINVAL, "KV page pools must be 16-byte aligned");
  if (mode == 0) {
    if (!tokens || !next_ids) return fail(MK_EINVAL, "tokens and next_ids must be non-NULL");
  } else {
    if (!hidden_in || !hidden_out) return fail(MK_EINVAL, "hidden_in and hidden_out must be non-NULL");
    if (!aligned16(hidden_in)) return fail(MK_EINVAL, "hidden_in must be 16-byte aligned");
  }
  MK_CUDA(cudaSetDevice(m->device));
  const MkConfig& c = m->cfg;
  mk::Params p{};
  p.L = c.num_layers;
  p.H = c.hidden;
  p.I = c.intermediate;
  p.NQ = c.num_q_heads;
  p.NKV = c.num_kv_heads;
  p.V = c.vocab;
  p.eps = c.rms_eps;
  p.B = batch;
  p.page_size = c.page_size;
  p.num_pages = c.num_pages;
  p.max_blocks = c.max_blocks_per_seq;
  p.rope_len = c.rope_len;
  p.num_slots = m->num_slots;
  p.kmax = m->kmax;
  p.nseg_h = mk::pieces_per_row(c.hidden);
  p.nseg_qd = mk::pieces_per_row(c.num_q_heads * 64);
  p.nseg_i = mk::pieces_per_row(c.intermediate);
  p.part_cap = m->part_cap;
  p.mode = mode;
  p.flags = flags;
  p.embed = static_cast<const mk::bf16*>(m->w.embed);
  p.w_qkv = static_cast<const mk::bf16*>(m->w.w_qkv);
  p.w_o = static_cast<const mk::bf16*>(m->w.w_o);
  p.w_gu = static_cast<const mk::bf16*>(m->w.w_gate_up);
  p.w_down = static_cast<const mk::bf16*>(m->w.w_down);
  p.norm_attn = static_cast<const mk::bf16*>(m->w.norm_attn);
  p.norm_mlp = static_cast<const mk::bf16*>(m->w.norm_mlp);
  p.norm_final = static_cast<const mk::bf16*>(m->w.norm_final);
  p.rope_cos = static_cast<const mk::bf16*>(m->w.rope_cos);
  p.rope_sin = static_cast<const mk::bf16*>(m->w.rope_sin);
  p.k_pages = static_cast<mk::bf16*>(kv->k_pages);
  p.v_pages = static_cast<mk::bf16*>(kv->v_pages);
  p.block_tables = kv->block_tables;
  p.tokens = const_cast<int*>(tokens);
  p.positions = const_cast<int*>(positions);
  p.hidden_in = static_cast<const mk::bf16*>(hidden_in);
  p.hidden_out = static_cast<mk::bf16*>(hidden_out);
  p.logits = logits;
  p.next_ids = next_ids;
  p.h = m->h;
  p.qkv = m->qkv;
  p.attn = m->attn;
  p.act = m->act;
  p.partials = m->partials;
  p.counters = m->counters;
  p.keys = m->keys;
  p.error = m->error;
  p.host_error = m->host_error_dev;
  p.timeout_ns = m->timeout_ns;
  p.debug_skip_cta = m->debug_skip_cta;
  // 5 tagged phases per layer plus the lm_head. A launch takes the next
  // 5 L + 1 tags; before the counter would pass 65535 the tagged words are
  // zeroed (0 is never a tag) and it restarts, so no word an earlier launch
  // left behind, in rows this batch did not write then, can carry a tag of
  // this launch.
  const uint32_t span = (uint32_t)(5 * c.num_layers + 1);
  if (m->tag_next + span > 65535u) {
    MK_CUDA(cudaMemsetAsync(m->act_words, 0, m->act_bytes, static_cast<cudaStream_t>(stream)));
    m->tag_next = 0;
  }
  p.tag_base = m->tag_next;
  m->tag_next += span;
  if (m->xtag_next + span >= 0xFFFFFFFFull) m->xtag_next = 1;
  p.xtag_base = (uint32_t)m->xtag_next;
  m->xtag_next += span;
  // Attention partials carry 32-bit tags of their own, one per layer and
  // launch, so a partial block that no split wrote this launch (the split
  // count follows the context) never matches: tags restart only after the
  // buffer is zeroed, and 0 is never a tag.
  if (m->part_tag_next + c.num_layers >= kPartTagLimit) {
    MK_CUDA(cudaMemsetAsync(m->partials, 0, m->partials_bytes, static_cast<cudaStream_t>(stream)));
    m->part_tag_next = 0;
  }
  p.part_tag0 = (uint32_t)(1 + m->part_tag_next);
  m->part_tag_next += c.num_layers;
  p.trace = m->trace;
  p.trace_per_cta = (c.num_layers * 5 + 1) * mk::kTraceKinds;
  p.tp_rank = m->tp_rank;
  p.tp_world = m->tp_world;
  p.lm_row0 = m->lm_row0;
  p.lm_rows = m->lm_rows < 0 ? c.vocab : m->lm_rows;
  for (int r = 0; r < mk::kMaxTp; ++r) p.xpeer[r] = m->xpeer[r];
  MK_CUDA(dispatch_launch(batch, p, m->grid, m->smem, static_cast<cudaStream_t>(stream)));
  return MK_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
// mk_decode_static: the decode step without a handle and without allocating.
//
// Its scratch (residual, q/k/v, attention partials, counters, argmax keys,
// error words) lives in this file-scope device array instead of a cudaMalloc
// made by mk_init. Every GPU that loads the library holds one copy until the
// process exits, and every call on that GPU shares it.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kStaticScratchBytes = 512 * 1024;  // enough for Llama-3.2-1B at max_batch 1
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

constexpr int kStaticMaxDevices = 64;
std::mutex g_static_mu;
void* g_static_ptr[kStaticMaxDevices] = {};  // device address of g_static_scratch, per device
uint32_t g_static_tag[kStaticMaxDevices] = {};   // next activation tag per device (see enqueue)
uint64_t g_static_part[kStaticMaxDevices] = {};  // partial tags used per device (see enqueue)
// The geometry of the last call on each device: calls may alternate between
// models, and a call whose layout differs from the last one's would find that
// call's tagged words at other offsets, so it starts from zeroed words.
std::array<int, 8> g_static_geom[kStaticMaxDevices] = {};

// Once per device, with that device current: the array's device address (the
// host-side name g_static_scratch is only a stand-in and must never reach a
// kernel) and the kernels' shared-memory limit.
int static_setup(int device, void** out) {
  std::lock_guard<std::mutex> lock(g_static_mu);
  if (device < 0 || device >= kStaticMaxDevices)
    return fail(MK_EINVAL, "device %d beyond the %d devices mk_decode_static supports", device,
                kStaticMaxDevices);
  if (!g_static_ptr[device]) {
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(MK_ECUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
    int cap = 0;
    MK_CUDA(cudaDeviceGetAttribute(&cap, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    MK_CUDA(set_smem_b<1>(cap));
    MK_CUDA(set_smem_b<2>(cap));
    MK_CUDA(set_smem_b<3>(cap));
    MK_CUDA(set_smem_b<4>(cap));
    g_static_ptr[device] = ptr;
  }
  *out = g_static_ptr[device];
  return MK_OK;
}

}  // namespace

namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// A 2-D bf16 tensor map [rows][cols] (cols contiguous), box {64 cols, box_rows},
// 128-byte swizzle: the K-major operand layout of the tcgen05 GEMM.
int encode_sw128(CUtensorMap* out, const void* base, long long rows, long long cols, int box_rows) {
  static EncodeTiledFn enc = nullptr;
  if (!enc) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
      return fail(MK_ECUDA, "cuTensorMapEncodeTiled unavailable");
    enc = reinterpret_cast<EncodeTiledFn>(fn);
  }
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {(cuuint32_t)mk::kGemmTileK, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = enc(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides,
                   box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MK_ECUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return MK_OK;
}

// K blocks per split for an n x k GEMM: narrow W is split along K so the
// grid covers the SMs.
// Launch with programmatic stream serialization: the kernel (which calls
// pdl_trigger / pdl_wait) may start while the previous one in the stream ends.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

constexpr int kGemmMaxCluster = 8;  // portable thread-block cluster size
int gemm_kblocks_per_split(int n, int k, int sms) {
  const int tiles = (n + mk::kGemmTileN - 1) / mk::kGemmTileN, kblocks = k / mk::kGemmTileK;
  int splits = tiles >= sms / 2 ? 1 : (sms + tiles - 1) / tiles;
  if (splits > kGemmMaxCluster) splits = kGemmMaxCluster;  // one cluster per tile
  if (splits > kblocks) splits = kblocks;
  return (kblocks + splits - 1) / splits;
}

template <int BP, int kStages>
cudaError_t launch_gemm_st(const mk::GemmParams& gp, int tiles, int splits, cudaStream_t st) {
  const int smem = kStages * (mk::kGemmTileN + BP) * mk::kGemmTileK * 2 + 1024;
  static bool attr = false;
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(mk::gemm_kernel<BP, kStages>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    attr = true;
  }
  if (splits == 1)
    return launch_pdl(mk::gemm_kernel<BP, kStages>, dim3(tiles, 1), dim3(mk::kGemmThreads), smem, st, gp);
  // the K splits of a tile form one cluster (their sums meet in shared memory)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(tiles, splits);
  cfg.blockDim = dim3(mk::kGemmThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr_c[2];
  attr_c[0].id = cudaLaunchAttributeClusterDimension;
  attr_c[0].val.clusterDim.x = 1;
  attr_c[0].val.clusterDim.y = splits;
  attr_c[0].val.clusterDim.z = 1;
  attr_c[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr_c[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr_c;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, mk::gemm_kernel<BP, kStages>, gp);
}

// An unsplit launch of at most one CTA per SM, each with more than
// kGemmStages K blocks, gets the deeper ring (8 stages, up to 193 KB at 64
// padded rows; at 128 rows 8 stages do not fit, so those launches keep 4).
// Split-K clusters keep 4 stages: with the deep ring the down projection's
// clusters of 8 ran 22.5 -> 32.8 us at 64 rows (measured).
template <int BP>
cudaError_t launch_gemm(const mk::GemmParams& gp, int tiles, int splits, int sms, cudaStream_t st) {
  if constexpr (BP <= 64) {
    if (splits == 1 && tiles <= sms && gp.kblocks_per_split > mk::kGemmStages)
      return launch_gemm_st<BP, mk::kGemmStagesDeep>(gp, tiles, splits, st);
  }
  return launch_gemm_st<BP, mk::kGemmStages>(gp, tiles, splits, st);
}
}  // namespace

namespace {
// Positions per attention CTA (a multiple of 32, at least 128 so each of the
// 4 warps gets a chunk or more). The grid is batch x kv heads x splits CTAs
// over 3 resident CTAs per SM, so the step takes about ceil(CTAs / (3 SMs))
// waves of one split each: pick the length that minimises waves x (length +
// the fixed cost of a CTA, in positions), the longer one on ties. The fixed
// cost is what a CTA pays before its chunks stream: ~64 positions' worth for
// the cp.async kernel (one chunk in flight per warp), ~512 for the TMA kernel
// (measured: its 8-stage ring makes one long split per sequence and kv head
// the fastest at bs 32 and 64; bs 64 1.94 -> 1.86 ms per step).
constexpr int kAttnFixedCostCpAsync = 64;
constexpr int kAttnFixedCostTma = 512;
int attn_split_len(int batch, int num_kv_heads, int max_len, int sms, int fixed_cost) {
  const long long pairs = (long long)batch * num_kv_heads;
  const long long slots = 3LL * sms;
  const int hi = ((max_len + 31) / 32) * 32;
  int best = hi;
  long long best_cost = -1;
  for (int len = hi; len >= 128; len -= 32) {
    const long long splits = (max_len + len - 1) / len;
    const long long waves = (pairs * splits + slots - 1) / slots;
    const long long cost = waves * (len + fixed_cost);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = len;
    }
    if (len == 128) break;
  }
  return best < 128 ? 128 : best;
}
int device_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}
}  // namespace

extern "C" {

int mk_init(const MkConfig* cfg, int device, MkModel** out) {
  if (!out) return fail(MK_EINVAL, "out is NULL");
  *out = nullptr;
  int rc = validate_config(cfg);
  if (rc) return rc;
  MK_CUDA(cudaSetDevice(device));
  cudaDeviceProp prop;
  MK_CUDA(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(MK_EINVAL, "device %d is sm_%d%d; this library is built for sm_100a", device,
                prop.major, prop.minor);
  if (!prop.cooperativeLaunch) return fail(MK_EINVAL, "device lacks cooperative launch");
  MkModel* m = new MkModel();
  m->cfg = *cfg;
  m->device = device;
  m->num_sms = prop.multiProcessorCount;
  m->kmax = cfg->hidden;
  if (cfg->intermediate > m->kmax) m->kmax = cfg->intermediate;
  if (cfg->num_q_heads * 64 > m->kmax) m->kmax = cfg->num_q_heads * 64;
  const int B = cfg->max_batch;
  const int smem_cap = (int)prop.sharedMemPerBlockOptin;
  {
    // Partial sums one CTA keeps per phase: its most units x pieces per unit.
    const int G = prop.multiProcessorCount;
    auto per_cta = [G](int units) { return (units + G - 1) / G; };
    const int nh = mk::pieces_per_row(cfg->hidden), nqd = mk::pieces_per_row(cfg->num_q_heads * 64),
              ni = mk::pieces_per_row(cfg->intermediate);
    int cap = per_cta((cfg->num_q_heads + 2 * cfg->num_kv_heads) * 32) * 2 * nh;
    cap = std::max(cap, per_cta(cfg->hidden) * nqd);
    cap = std::max(cap, per_cta(cfg->intermediate) * 2 * nh);
    cap = std::max(cap, per_cta(cfg->hidden) * ni);
    m->part_cap = cap * B;
  }
  // An even slot count: producer k alone fills the slots s with s % 2 == k,
  // so it sees every phase of their empty barriers.
  int slots = 0;
  for (int s = 16; s >= 4; s -= mk::kProducers) {
    if (mk::smem_bytes_for(s, B, m->kmax, m->part_cap, cfg->hidden) <= smem_cap) {
      slots = s;
      break;
    }
  }
  if (!slots) {
    delete m;
    return fail(MK_EINVAL, "activation rows (%d x %d) leave no room for the ring", B, m->kmax);
  }
  m->num_slots = slots;
  m->smem = mk::smem_bytes_for(slots, B, m->kmax, m->part_cap, cfg->hidden);
  if (int src = check_schedule(cfg, B, m->num_sms, slots)) {
    delete m;
    return src;
  }
  // The attribute is per kernel, not per handle: allow the device maximum so
  // handles with different geometries can be used in any order.
  for (int b = 1; b <= 4; ++b) {
    cudaError_t e = cudaSuccess;
    switch (b) {
      case 1: e = set_smem_b<1>(smem_cap); break;
      case 2: e = set_smem_b<2>(smem_cap); break;
      case 3: e = set_smem_b<3>(smem_cap); break;
      case 4: e = set_smem_b<4>(smem_cap); break;
    }
    if (e != cudaSuccess) {
      delete m;
      return fail(MK_ECUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    }
  }
  int blocks = 0;
  cudaError_t e = occupancy_b<1>(&blocks, m->smem);
  if (e != cudaSuccess || blocks < 1) {
    delete m;
    return fail(MK_ECUDA, "kernel does not fit one CTA per SM (%s)", cudaGetErrorString(e));
  }
  m->grid = m->num_sms;

  // Scratch: one allocation, 256-byte aligned sub-buffers.
  const size_t H = cfg->hidden, I = cfg->intermediate, NQ = cfg->num_q_heads,
               NKV = cfg->num_kv_heads;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_h = take(B * H * 4);
  const size_t o_qkv = take(B * (NQ + 2 * NKV) * 64 * 4);
  const size_t o_attn = take(B * NQ * 64 * 4);
  const size_t o_act = take(B * I * 4);
  const size_t part_bytes = (size_t)m->grid * mk::kGroup * mk::kPartialStride * 8;
  const size_t o_part = take(part_bytes);
  const size_t o_cnt = take(mk::kCounters * 4);
  const size_t o_keys = take(B * 8);
  const size_t o_err = take(16);
  m->counters_bytes = o_err + 256 - o_cnt;  // counters, keys and error word
  const size_t o_io = take((size_t)3 * B * 4);
  void* base = nullptr;
  e = cudaMalloc(&base, off);
  if (e != cudaSuccess) {
    delete m;
    return fail(MK_ENOMEM, "cudaMalloc(%zu): %s", off, cudaGetErrorString(e));
  }
  m->scratch = base;
  char* cb = static_cast<char*>(base);
  m->h = reinterpret_cast<uint32_t*>(cb + o_h);
  m->qkv = reinterpret_cast<uint32_t*>(cb + o_qkv);
  m->attn = reinterpret_cast<uint32_t*>(cb + o_attn);
  m->act = reinterpret_cast<uint32_t*>(cb + o_act);
  m->act_words = cb + o_h;
  m->act_bytes = o_part - o_h;
  m->partials = reinterpret_cast<unsigned long long*>(cb + o_part);
  m->partials_bytes = part_bytes;
  m->counters = reinterpret_cast<uint32_t*>(cb + o_cnt);
  m->keys = reinterpret_cast<unsigned long long*>(cb + o_keys);
  m->error = reinterpret_cast<int*>(cb + o_err);
  m->io_dev = reinterpret_cast<int32_t*>(cb + o_io);
  e = cudaMemset(base, 0, off);
  if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&m->io_host), (size_t)3 * B * 4, cudaHostAllocDefault);
  if (e == cudaSuccess) e = cudaHostAlloc(reinterpret_cast<void**>(&m->host_error), 16, cudaHostAllocMapped);
  if (e == cudaSuccess) {
    memset(m->host_error, 0, 16);
    e = cudaHostGetDevicePointer(reinterpret_cast<void**>(&m->host_error_dev), m->host_error, 0);
  }
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (m->host_error) cudaFreeHost(m->host_error);
    if (m->io_host) cudaFreeHost(m->io_host);
    cudaFree(base);
    delete m;
    return fail(MK_ECUDA, "scratch init: %s", cudaGetErrorString(e));
  }
  *out = m;
  return MK_OK;
}

int mk_load_weights(MkModel* m, const MkWeights* w) {
  if (!m || !w) return fail(MK_EINVAL, "NULL argument");
  const void* ptrs[] = {w->embed, w->w_qkv, w->w_o, w->w_gate_up, w->w_down,
                        w->norm_attn, w->norm_mlp, w->norm_final, w->rope_cos, w->rope_sin};
  const char* names[] = {"embed", "w_qkv", "w_o", "w_gate_up", "w_down",
                         "norm_attn", "norm_mlp", "norm_final", "rope_cos", "rope_sin"};
  for (int i = 0; i < 10; ++i) {
    if (!ptrs[i]) return fail(MK_EINVAL, "weight pointer %s is NULL", names[i]);
    if (!aligned16(ptrs[i])) return fail(MK_EINVAL, "weight pointer %s is not 16-byte aligned", names[i]);
  }
  m->w = *w;
  m->has_weights = true;
  return MK_OK;
}

int mk_decode(MkModel* m, const int32_t* tokens, const int32_t* positions, int32_t batch,
              const MkKVCache* kv, float* logits, int32_t* next_ids, int32_t flags, void* stream) {
  return enqueue(m, 0, tokens, positions, batch, kv, nullptr, nullptr, logits, next_ids, flags,
                 stream);
}

int mk_decode_host(MkModel* m, const int32_t* tokens, const int32_t* positions, int32_t batch,
                   const MkKVCache* kv, float* logits, int32_t* next_ids, void* stream) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  if (!tokens || !positions || !next_ids) return fail(MK_EINVAL, "tokens, positions and next_ids are required");
  if (batch < 1 || batch > m->cfg.max_batch)
    return fail(MK_EINVAL, "batch %d outside [1, max_batch=%d]", batch, m->cfg.max_batch);
  MK_CUDA(cudaSetDevice(m->device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int32_t* in_h = m->io_host;
  memcpy(in_h, tokens, (size_t)batch * 4);
  memcpy(in_h + batch, positions, (size_t)batch * 4);
  MK_CUDA(cudaMemcpyAsync(m->io_dev, in_h, (size_t)2 * batch * 4, cudaMemcpyHostToDevice, st));
  if (int rc = enqueue(m, 0, m->io_dev, m->io_dev + batch, batch, kv, nullptr, nullptr, logits,
                       m->io_dev + 2 * batch, 0, stream))
    return rc;
  MK_CUDA(cudaMemcpyAsync(in_h + 2 * batch, m->io_dev + 2 * batch, (size_t)batch * 4,
                          cudaMemcpyDeviceToHost, st));
  if (int rc = mk_sync(m, stream)) return rc;
  memcpy(next_ids, in_h + 2 * batch, (size_t)batch * 4);
  return MK_OK;
}

int mk_decode_static(const MkConfig* cfg, const MkWeights* w, const int32_t* tokens,
                     const int32_t* positions, int32_t batch, const MkKVCache* kv, float* logits,
                     int32_t* next_ids, int32_t flags, int32_t* error_out, void* stream) {
  int rc = validate_config(cfg);
  if (rc) return rc;
  if (!w) return fail(MK_EINVAL, "weights are NULL");
  int device = 0;
  MK_CUDA(cudaGetDevice(&device));
  int major = 0, coop = 0, sms = 0, cap = 0;
  MK_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  MK_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device));
  MK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device));
  MK_CUDA(cudaDeviceGetAttribute(&cap, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
  if (major != 10) return fail(MK_EINVAL, "device %d is not sm_100a", device);
  if (!coop) return fail(MK_EINVAL, "device lacks cooperative launch");

  // The launch plan, computed like mk_init's, in a handle on the stack.
  MkModel m;
  m.cfg = *cfg;
  m.device = device;
  m.num_sms = sms;
  m.grid = sms;
  m.kmax = std::max(std::max(cfg->hidden, cfg->intermediate), cfg->num_q_heads * 64);
  const int B = cfg->max_batch;
  {
    auto per_cta = [sms](int units) { return (units + sms - 1) / sms; };
    const int nh = mk::pieces_per_row(cfg->hidden), nqd = mk::pieces_per_row(cfg->num_q_heads * 64),
              ni = mk::pieces_per_row(cfg->intermediate);
    int pc = per_cta((cfg->num_q_heads + 2 * cfg->num_kv_heads) * 32) * 2 * nh;
    pc = std::max(pc, per_cta(cfg->hidden) * nqd);
    pc = std::max(pc, per_cta(cfg->intermediate) * 2 * nh);
    pc = std::max(pc, per_cta(cfg->hidden) * ni);
    m.part_cap = pc * B;
  }
  for (int s = 16; s >= 4 && !m.num_slots; s -= mk::kProducers)
    if (mk::smem_bytes_for(s, B, m.kmax, m.part_cap, cfg->hidden) <= cap) m.num_slots = s;
  if (!m.num_slots) return fail(MK_EINVAL, "activation rows (%d x %d) leave no room for the ring", B, m.kmax);
  m.smem = mk::smem_bytes_for(m.num_slots, B, m.kmax, m.part_cap, cfg->hidden);
  if (int src = check_schedule_cached(cfg, B, sms, m.num_slots)) return src;

  // Scratch layout (as mk_init's), checked against the static array's size.
  const size_t H = cfg->hidden, I = cfg->intermediate, NQ = cfg->num_q_heads,
               NKV = cfg->num_kv_heads;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_h = take(B * H * 4);
  const size_t o_qkv = take(B * (NQ + 2 * NKV) * 64 * 4);
  const size_t o_attn = take(B * NQ * 64 * 4);
  const size_t o_act = take(B * I * 4);
  const size_t part_bytes = (size_t)sms * mk::kGroup * mk::kPartialStride * 8;
  const size_t o_part = take(part_bytes);
  const size_t o_cnt = take(mk::kCounters * 4);
  const size_t o_keys = take(B * 8);
  const size_t o_err = take(16);
  const size_t o_mirror = take(16);
  if (off > kStaticScratchBytes)
    return fail(MK_EINVAL,
                "mk_decode_static: this geometry needs %zu bytes of scratch, the static array "
                "holds %zu (use mk_init / mk_decode instead)",
                off, kStaticScratchBytes);

  void* base = nullptr;
  rc = static_setup(device, &base);
  if (rc) return rc;
  char* cb = static_cast<char*>(base);
  m.h = reinterpret_cast<uint32_t*>(cb + o_h);
  m.qkv = reinterpret_cast<uint32_t*>(cb + o_qkv);
  m.attn = reinterpret_cast<uint32_t*>(cb + o_attn);
  m.act = reinterpret_cast<uint32_t*>(cb + o_act);
  m.act_words = cb + o_h;
  m.act_bytes = o_part - o_h;
  m.partials = reinterpret_cast<unsigned long long*>(cb + o_part);
  m.partials_bytes = part_bytes;
  m.counters = reinterpret_cast<uint32_t*>(cb + o_cnt);
  m.keys = reinterpret_cast<unsigned long long*>(cb + o_keys);
  m.error = reinterpret_cast<int*>(cb + o_err);
  // Device-side failures are reported in error_out (or a slot of the static
  // array when the caller passes none) instead of a mapped host mirror.
  m.host_error_dev = error_out ? reinterpret_cast<int*>(error_out) : reinterpret_cast<int*>(cb + o_mirror);
  rc = mk_load_weights(&m, w);
  if (rc) return rc;
  bool restart = false, clear_words = false;
  const uint32_t span = (uint32_t)(5 * cfg->num_layers + 1);
  const std::array<int, 8> geom = {cfg->num_layers, cfg->hidden, cfg->intermediate,
                                   cfg->num_q_heads, cfg->num_kv_heads, cfg->vocab, B, sms};
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    // The activation tags of this call follow the last call's on this device;
    // the words start from zero when the geometry changed or the tags wrap.
    if (g_static_geom[device] != geom || g_static_tag[device] + span > 65535u) {
      clear_words = true;
      g_static_tag[device] = 0;
      g_static_geom[device] = geom;
    }
    m.tag_next = g_static_tag[device];
    g_static_tag[device] += span;
    m.part_tag_next = g_static_part[device];
    if (m.part_tag_next + cfg->num_layers >= kPartTagLimit) {
      m.part_tag_next = 0;
      restart = true;
    }
    g_static_part[device] = m.part_tag_next + cfg->num_layers;
  }

  // What must start at zero: barrier counters, argmax keys and error words
  // (a previous call that failed on the device leaves them set), the tagged
  // activation words when the geometry changed or their tags wrap, and the
  // partials when their tag sequence restarts.
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (clear_words) MK_CUDA(cudaMemsetAsync(cb + o_h, 0, o_part - o_h, st));
  if (restart) MK_CUDA(cudaMemsetAsync(m.partials, 0, m.partials_bytes, st));
  MK_CUDA(cudaMemsetAsync(cb + o_cnt, 0, o_mirror + 16 - o_cnt, st));
  if (error_out) MK_CUDA(cudaMemsetAsync(error_out, 0, 4 * sizeof(int32_t), st));
  return enqueue(&m, 0, tokens, positions, batch, kv, nullptr, nullptr, logits, next_ids, flags,
                 stream);
}

int mk_decode_hidden(MkModel* m, const void* hidden_in, const int32_t* positions, int32_t batch,
                     const MkKVCache* kv, void* hidden_out, void* stream) {
  return enqueue(m, 1, nullptr, positions, batch, kv, hidden_in, hidden_out, nullptr, nullptr, 0,
                 stream);
}

int mk_sync(MkModel* m, void* stream) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  MK_CUDA(cudaSetDevice(m->device));
  MK_CUDA(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
  volatile int* he = m->host_error;
  if (he[0] == 0) return MK_OK;
  int err[4] = {he[0], he[1], he[2], he[3]};
  // Reset the counters, argmax keys and error words so the next launch starts clean.
  MK_CUDA(cudaMemset(m->counters, 0, m->counters_bytes));
  MK_CUDA(cudaDeviceSynchronize());
  he[0] = he[1] = he[2] = he[3] = 0;
  const char* what = "unknown";
  int code = MK_EDEVICE;
  switch (err[0]) {
    case mk::kErrBarrierTimeout: what = "grid barrier wait timed out"; code = MK_ETIMEOUT; break;
    case mk::kErrRingTimeout: what = "weight-stream wait timed out"; code = MK_ETIMEOUT; break;
    case mk::kErrPosition: what = "position out of range (rope table or block table)"; break;
    case mk::kErrPage: what = "block table holds a page id outside the pool"; break;
    case mk::kErrToken: what = "token id outside the vocabulary"; break;
  }
  return fail(code, "device error: %s (code %d, detail %d, cta %d, thread %d)", what, err[0],
              err[1], err[2], err[3]);
}

int mk_set_timeout_ns(MkModel* m, uint64_t ns) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  if (ns == 0) return fail(MK_EINVAL, "timeout must be > 0");
  m->timeout_ns = ns;
  return MK_OK;
}

int mk_debug_skip_arrival(MkModel* m, int32_t cta) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  m->debug_skip_cta = cta;
  return MK_OK;
}

int mk_set_trace(MkModel* m, uint64_t* buffer, int64_t capacity, int64_t* needed) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  const int64_t n = trace_entries(m);
  if (needed) *needed = n;
  if (!buffer) {
    m->trace = nullptr;
    return MK_OK;
  }
  if (capacity < n)
    return fail(MK_EINVAL, "trace buffer holds %lld entries, a launch writes %lld",
                (long long)capacity, (long long)n);
  if (reinterpret_cast<uintptr_t>(buffer) & 7) return fail(MK_EINVAL, "trace buffer must be 8-byte aligned");
  m->trace = reinterpret_cast<unsigned long long*>(buffer);
  return MK_OK;
}

int mk_query(const MkModel* m, int32_t* grid, int32_t* ring_slots, int32_t* smem_bytes) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  if (grid) *grid = m->grid;
  if (ring_slots) *ring_slots = m->num_slots;
  if (smem_bytes) *smem_bytes = m->smem;
  return MK_OK;
}

int mk_schedule_gap(const MkConfig* cfg, int32_t batch, int32_t grid, int32_t* gap) {
  int rc = validate_config(cfg);
  if (rc) return rc;
  if (batch < 1 || batch > cfg->max_batch) return fail(MK_EINVAL, "batch %d outside [1, max_batch]", batch);
  if (grid < 1) return fail(MK_EINVAL, "grid %d < 1", grid);
  if (!gap) return fail(MK_EINVAL, "gap is NULL");
  const int g = max_consumer_gap(cfg, batch, grid, cfg->vocab);
  *gap = g == INT32_MAX ? -1 : g;
  return MK_OK;
}

const char* mk_last_error(void) { return g_last_error.c_str(); }


int64_t mk_paged_attention_workspace(int32_t batch, int32_t num_kv_heads, int32_t max_len) {
  if (batch < 1 || num_kv_heads < 1 || max_len < 1) return 0;
  // the workspace serves either kernel: the cp.async one's shorter splits are the most
  const int sl = attn_split_len(batch, num_kv_heads, max_len, device_sms(), kAttnFixedCostCpAsync);
  const int64_t splits = (max_len + sl - 1) / sl;
  return (int64_t)batch * num_kv_heads * splits * 4 * mk::kAttnPartial * 4;
}

int mk_paged_attention(const void* q, const void* k_pages, const void* v_pages,
                       const int32_t* block_tables, const int32_t* lengths, int32_t batch,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t page_size,
                       int32_t max_blocks, int32_t num_pages, int32_t max_len, float scale,
                       void* workspace, int64_t workspace_bytes, void* out, int32_t* error,
                       void* stream) {
  if (!q || !k_pages || !v_pages || !block_tables || !lengths || !workspace || !out || !error)
    return fail(MK_EINVAL, "NULL argument");
  if (num_kv_heads < 1 || num_q_heads != 4 * num_kv_heads)
    return fail(MK_EINVAL, "num_q_heads must be 4 * num_kv_heads");
  if (batch < 1 || batch > 65535) return fail(MK_EINVAL, "batch %d", batch);
  if (page_size < 1 || max_blocks < 1 || num_pages < 1 || max_len < 1 || max_len > page_size * max_blocks)
    return fail(MK_EINVAL, "cache geometry (page_size %d, max_blocks %d, max_len %d)", page_size,
                max_blocks, max_len);
  if (!aligned16(q) || !aligned16(k_pages) || !aligned16(v_pages))
    return fail(MK_EINVAL, "q and the page pools must be 16-byte aligned");
  const int64_t need = mk_paged_attention_workspace(batch, num_kv_heads, max_len);
  if (workspace_bytes < need) return fail(MK_EINVAL, "workspace %lld < %lld bytes", (long long)workspace_bytes, (long long)need);
  mk::PagedAttnParams ap{};
  ap.q = static_cast<const mk::bf16*>(q);
  ap.k = static_cast<const mk::bf16*>(k_pages);
  ap.v = static_cast<const mk::bf16*>(v_pages);
  ap.block_tables = block_tables;
  ap.lengths = lengths;
  ap.NQ = num_q_heads;
  ap.NKV = num_kv_heads;
  ap.ps = page_size;
  ap.max_blocks = max_blocks;
  ap.num_pages = num_pages;
  ap.split_len = attn_split_len(batch, num_kv_heads, max_len, device_sms(),
                                page_size % 32 == 0 ? kAttnFixedCostTma : kAttnFixedCostCpAsync);
  ap.splits = (max_len + ap.split_len - 1) / ap.split_len;
  ap.scale = scale;
  ap.work = static_cast<float*>(workspace);
  ap.out = static_cast<mk::bf16*>(out);
  ap.error = error;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (page_size % 32 == 0) {
    // every 32-position chunk is one run of a page: TMA boxes into the staged ring
    mk::PagedAttnTmaParams tp{};
    tp.p = ap;
    const long long pool_rows = (long long)num_pages * num_kv_heads * page_size;
    if (pool_rows > 0x7fffffffLL) return fail(MK_EINVAL, "KV pool of %lld rows", pool_rows);
    if (int rc = encode_sw128(&tp.tm_k, k_pages, pool_rows, 64, 32)) return rc;
    if (int rc = encode_sw128(&tp.tm_v, v_pages, pool_rows, 64, 32)) return rc;
    static bool tattr = false;
    if (!tattr) {
      MK_CUDA(cudaFuncSetAttribute(mk::paged_attn_tma_kernel,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, mk::kAttnTmaSmem));
      tattr = true;
    }
    MK_CUDA(launch_pdl(mk::paged_attn_tma_kernel, dim3(ap.splits, num_kv_heads, batch),
                       dim3((mk::kAttnCtaWarps + 1) * 32), mk::kAttnTmaSmem, st, tp));
  } else {
    static bool attr = false;
    if (!attr) {
      MK_CUDA(cudaFuncSetAttribute(mk::paged_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                   mk::kAttnSmem));
      attr = true;
    }
    MK_CUDA(launch_pdl(mk::paged_attn_kernel, dim3(ap.splits, num_kv_heads, batch),
                       dim3(mk::kAttnCtaWarps * 32), mk::kAttnSmem, st, ap));
  }
  // a single split writes its heads' output itself
  if (ap.splits > 1)
    MK_CUDA(launch_pdl(mk::paged_attn_merge_kernel, dim3(num_kv_heads, batch), dim3(256), 0, st, ap));
  return MK_OK;
}

int64_t mk_gemm_workspace(int32_t n, int32_t k, int32_t rows) {
  (void)n;
  (void)k;
  (void)rows;
  return 0;  // split-K sums meet in distributed shared memory, not in a workspace
}

int mk_gemm_bf16(const void* w, int32_t n, int32_t k, const void* x, int32_t rows,
                 int32_t rows_padded, const void* residual, void* out, float* out_f32,
                 void* workspace, int64_t workspace_bytes, int32_t* error, void* stream) {
  if (!w || !x || !error || (!out && !out_f32) || (out && out_f32))
    return fail(MK_EINVAL, "w, x, error and exactly one of out / out_f32 are required");
  if (n < 1 || k < mk::kGemmTileK || k % mk::kGemmTileK)
    return fail(MK_EINVAL, "k must be a positive multiple of 64 and n positive (n %d, k %d)", n, k);
  if (rows_padded != 16 && rows_padded != 32 && rows_padded != 64 && rows_padded != 128)
    return fail(MK_EINVAL, "rows_padded must be 16, 32, 64 or 128 (got %d)", rows_padded);
  if (rows < 1 || rows > rows_padded) return fail(MK_EINVAL, "rows %d outside [1, %d]", rows, rows_padded);
  if (!aligned16(w) || !aligned16(x)) return fail(MK_EINVAL, "w and x must be 16-byte aligned");
  if (residual && out_f32) return fail(MK_EINVAL, "a residual needs the bf16 output");
  int dev = 0, sms = 148;
  MK_CUDA(cudaGetDevice(&dev));
  MK_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  const int tiles = (n + mk::kGemmTileN - 1) / mk::kGemmTileN, kblocks = k / mk::kGemmTileK;
  const int kps = gemm_kblocks_per_split(n, k, sms);
  const int splits = (kblocks + kps - 1) / kps;
  (void)workspace;
  (void)workspace_bytes;
  mk::GemmParams gp{};
  if (int rc = encode_sw128(&gp.tm_w, w, n, k, mk::kGemmTileN)) return rc;
  if (int rc = encode_sw128(&gp.tm_x, x, rows_padded, k, rows_padded)) return rc;
  gp.N = n;
  gp.K = k;
  gp.B = rows;
  gp.kblocks_per_split = kps;
  gp.splits = splits;
  gp.residual = static_cast<const mk::bf16*>(residual);
  gp.out = static_cast<mk::bf16*>(out);
  gp.out_f32 = out_f32;
  gp.error = error;
  gp.timeout_ns = 2000000000ull;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = rows_padded == 16 ? launch_gemm<16>(gp, tiles, splits, sms, st)
                  : rows_padded == 32 ? launch_gemm<32>(gp, tiles, splits, sms, st)
                  : rows_padded == 64 ? launch_gemm<64>(gp, tiles, splits, sms, st)
                                      : launch_gemm<128>(gp, tiles, splits, sms, st);
  if (e != cudaSuccess) return fail(MK_ECUDA, "gemm launch: %s", cudaGetErrorString(e));
  return MK_OK;
}

int mk_rmsnorm_rows(const void* x, const void* gamma, float eps, int32_t rows, int32_t hidden,
                    void* out, void* stream) {
  if (!x || !gamma || !out) return fail(MK_EINVAL, "NULL argument");
  if (rows < 1 || hidden < 8 || hidden % 8) return fail(MK_EINVAL, "rows %d, hidden %d", rows, hidden);
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(out)) return fail(MK_EINVAL, "16-byte alignment");
  MK_CUDA(launch_pdl(mk::rmsnorm_rows_kernel, dim3(rows), dim3(256), 0,
                     static_cast<cudaStream_t>(stream), static_cast<const mk::bf16*>(x),
                     static_cast<const mk::bf16*>(gamma), eps, (int)hidden,
                     static_cast<mk::bf16*>(out)));
  return MK_OK;
}

int mk_rope_scatter(const void* qkv, const void* rope_cos, const void* rope_sin,
                    const int32_t* positions, const int32_t* block_tables, int32_t max_blocks,
                    int32_t num_pages, int32_t page_size, int32_t num_q_heads,
                    int32_t num_kv_heads, int32_t batch, void* q_out, void* k_pages,
                    void* v_pages, int32_t* error, void* stream) {
  if (!qkv || !rope_cos || !rope_sin || !positions || !block_tables || !q_out || !k_pages ||
      !v_pages || !error)
    return fail(MK_EINVAL, "NULL argument");
  if (batch < 1 || num_q_heads < 1 || num_kv_heads < 1 || page_size < 1 || max_blocks < 1)
    return fail(MK_EINVAL, "geometry");
  const int n = batch * (num_q_heads + 2 * num_kv_heads) * 32;
  MK_CUDA(launch_pdl(mk::rope_scatter_kernel, dim3((n + 255) / 256), dim3(256), 0,
                     static_cast<cudaStream_t>(stream), static_cast<const mk::bf16*>(qkv),
                     static_cast<const mk::bf16*>(rope_cos), static_cast<const mk::bf16*>(rope_sin),
                     positions, block_tables, (int)max_blocks, (int)num_pages, (int)page_size,
                     (int)num_q_heads, (int)num_kv_heads, (int)batch, static_cast<mk::bf16*>(q_out),
                     static_cast<mk::bf16*>(k_pages), static_cast<mk::bf16*>(v_pages), error));
  return MK_OK;
}

int mk_argmax_rows(const float* x, int32_t rows, int32_t cols, int64_t* ids, void* stream) {
  if (!x || !ids || rows < 1 || cols < 1)
    return fail(MK_EINVAL, "argmax: x, ids, rows >= 1 and cols >= 1 are required");
  const bool vec = cols % 4 == 0 && aligned16(x);
  MK_CUDA(launch_pdl(mk::argmax_rows_kernel, dim3(rows), dim3(1024), 0,
                     static_cast<cudaStream_t>(stream), x, (int)cols, vec, ids));
  return MK_OK;
}

int mk_add_rmsnorm_rows(void* x, const float* sum, const void* gamma, float eps, int32_t rows,
                        int32_t hidden, void* out, void* stream) {
  if (!x || !sum || !gamma || !out) return fail(MK_EINVAL, "NULL argument");
  if (rows < 1 || hidden < 8 || hidden % 8) return fail(MK_EINVAL, "rows %d, hidden %d", rows, hidden);
  if (!aligned16(x) || !aligned16(sum) || !aligned16(gamma) || !aligned16(out))
    return fail(MK_EINVAL, "16-byte alignment");
  MK_CUDA(launch_pdl(mk::add_rmsnorm_rows_kernel, dim3(rows), dim3(256), 0,
                     static_cast<cudaStream_t>(stream), static_cast<mk::bf16*>(x), sum,
                     static_cast<const mk::bf16*>(gamma), eps, (int)hidden, static_cast<mk::bf16*>(out)));
  return MK_OK;
}

int64_t mk_xbuf_bytes(int32_t rows, int32_t hidden) {
  if (rows < 1 || hidden < 8 || hidden % 8) return 0;
  return (int64_t)mk::xchg_bytes(rows, hidden);
}

int mk_xbuf_alloc(int64_t bytes, MkIpcHandle* handle, void** ptr) {
  if (!handle || !ptr || bytes < 1) return fail(MK_EINVAL, "handle, ptr and bytes >= 1 are required");
  *ptr = nullptr;
  void* buf = nullptr;
  MK_CUDA(cudaMalloc(&buf, (size_t)bytes));
  cudaError_t e = cudaMemset(buf, 0, (size_t)bytes);  // flag 0 is below every tag
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, buf);
  if (e != cudaSuccess) {
    cudaFree(buf);
    return fail(MK_ECUDA, "exchange buffer: %s", cudaGetErrorString(e));
  }
  memcpy(handle, &h, sizeof(h));
  *ptr = buf;
  return MK_OK;
}

int mk_xbuf_open(const MkIpcHandle* handle, void** ptr) {
  if (!handle || !ptr) return fail(MK_EINVAL, "handle and ptr are required");
  *ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  MK_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
  return MK_OK;
}

int mk_xbuf_close(void* ptr) {
  if (!ptr) return MK_OK;
  MK_CUDA(cudaIpcCloseMemHandle(ptr));
  return MK_OK;
}

int mk_xbuf_free(void* ptr) {
  if (!ptr) return MK_OK;
  MK_CUDA(cudaFree(ptr));
  return MK_OK;
}

int mk_step_epoch(uint32_t* epoch, void* stream) {
  if (!epoch) return fail(MK_EINVAL, "epoch is NULL");
  MK_CUDA(launch_pdl(mk::epoch_advance_kernel, dim3(1), dim3(32), 0,
                     static_cast<cudaStream_t>(stream), epoch));
  return MK_OK;
}

int mk_allreduce_add_rmsnorm(const uint64_t* peers, int32_t rank, int32_t world, int32_t rows_cap,
                             int32_t exchange, const uint32_t* epoch, void* x, const void* gamma,
                             float eps, int32_t rows, int32_t hidden, void* out, int32_t* error,
                             uint64_t timeout_ns, void* stream) {
  if (!peers || !epoch || !x || !gamma || !out || !error) return fail(MK_EINVAL, "NULL argument");
  if (world < 2 || world > mk::kMaxTp || rank < 0 || rank >= world)
    return fail(MK_EINVAL, "rank %d of world %d (2 .. %d GPUs)", rank, world, mk::kMaxTp);
  if (rows < 1 || rows > rows_cap || hidden < 8 || hidden % 8)
    return fail(MK_EINVAL, "rows %d (buffer rows %d), hidden %d", rows, rows_cap, hidden);
  if (exchange < 0 || exchange >= mk::kXchgPerStep)
    return fail(MK_EINVAL, "exchange %d outside [0, %d)", exchange, mk::kXchgPerStep);
  if (!aligned16(x) || !aligned16(gamma) || !aligned16(out)) return fail(MK_EINVAL, "16-byte alignment");
  mk::XchgParams xp{};
  xp.peers = reinterpret_cast<const unsigned long long*>(peers);
  xp.rank = rank;
  xp.W = world;
  xp.rows = rows_cap;
  xp.H = hidden;
  xp.exchange = exchange;
  xp.epoch = epoch;
  xp.x = static_cast<mk::bf16*>(x);
  xp.gamma = static_cast<const mk::bf16*>(gamma);
  xp.eps = eps;
  xp.y = static_cast<mk::bf16*>(out);
  xp.error = error;
  xp.timeout_ns = timeout_ns ? timeout_ns : 2000000000ull;
  MK_CUDA(launch_pdl(mk::xreduce_add_rmsnorm_kernel, dim3(rows), dim3(256), 0,
                     static_cast<cudaStream_t>(stream), xp));
  return MK_OK;
}

int mk_argmax_keys(const float* x, int32_t rows, int32_t cols, int32_t id0, uint64_t* keys,
                   void* stream) {
  if (!x || !keys || rows < 1 || cols < 1 || id0 < 0)
    return fail(MK_EINVAL, "argmax keys: x, keys, rows >= 1, cols >= 1 and id0 >= 0 are required");
  MK_CUDA(launch_pdl(mk::argmax_keys_kernel, dim3(rows), dim3(1024), 0,
                     static_cast<cudaStream_t>(stream), x, (int)cols, (int)id0,
                     reinterpret_cast<unsigned long long*>(keys)));
  return MK_OK;
}

int mk_keys_to_ids(const uint64_t* keys, int32_t world, int32_t rows, int64_t* ids, void* stream) {
  if (!keys || !ids || world < 1 || rows < 1) return fail(MK_EINVAL, "keys to ids: arguments");
  MK_CUDA(launch_pdl(mk::keys_to_ids_kernel, dim3((rows + 127) / 128), dim3(128), 0,
                     static_cast<cudaStream_t>(stream),
                     reinterpret_cast<const unsigned long long*>(keys), (int)world, (int)rows, ids));
  return MK_OK;
}

int mk_swiglu(const void* gate_up, int64_t n, void* out, void* stream) {
  if (!gate_up || !out || n < 1 || n > INT32_MAX) return fail(MK_EINVAL, "arguments");
  MK_CUDA(launch_pdl(mk::swiglu_kernel, dim3((int)((n + 255) / 256)), dim3(256), 0,
                     static_cast<cudaStream_t>(stream), static_cast<const mk::bf16*>(gate_up), (int)n,
                     static_cast<mk::bf16*>(out)));
  return MK_OK;
}

int mk_sample(const float* logits, int32_t batch, int32_t vocab, int64_t ld,
              const MkSampling* params, uint64_t seed, uint64_t step, int32_t* out_ids,
              int32_t* tokens, int32_t* positions, int32_t* error, void* stream) {
  if (!logits || !params || !out_ids || !error) return fail(MK_EINVAL, "NULL argument");
  if (batch < 1 || batch > mk::kSampleMaxBatch)
    return fail(MK_EINVAL, "batch %d outside [1, %d]", batch, mk::kSampleMaxBatch);
  if (vocab < 1 || ld < vocab) return fail(MK_EINVAL, "vocab %d / ld %lld", vocab, (long long)ld);
  if ((tokens == nullptr) != (positions == nullptr))
    return fail(MK_EINVAL, "tokens and positions go together");
  mk::SampleParams sp{};
  sp.logits = logits;
  sp.ld = ld;
  sp.V = vocab;
  for (int b = 0; b < batch; ++b) {
    const MkSampling& q = params[b];
    if (!(q.top_p > 0.f) || q.top_p > 1.f) return fail(MK_EINVAL, "top_p %g outside (0, 1]", q.top_p);
    sp.top_k[b] = q.top_k;
    sp.top_p[b] = q.top_p;
    sp.temperature[b] = q.temperature;
  }
  sp.seed = seed;
  sp.step = step;
  sp.out = out_ids;
  sp.tokens = tokens;
  sp.positions = positions;
  sp.error = error;
  mk::sample_kernel<<<batch, mk::kSampleThreads, 0, static_cast<cudaStream_t>(stream)>>>(sp);
  MK_CUDA(cudaGetLastError());
  return MK_OK;
}

int mk_tp_setup(MkModel* m, int32_t rank, int32_t world, int32_t lm_row0, int32_t lm_rows,
                MkIpcHandle* handle, void** buffer) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  if (world < 1 || world > mk::kMaxTp) return fail(MK_EINVAL, "world %d outside [1, %d]", world, mk::kMaxTp);
  if (rank < 0 || rank >= world) return fail(MK_EINVAL, "rank %d outside [0, %d)", rank, world);
  if (lm_row0 < 0 || lm_rows < 1 || (long long)lm_row0 + lm_rows > m->cfg.vocab)
    return fail(MK_EINVAL, "lm_head rows [%d, %d + %d) outside the vocabulary (%d)", lm_row0, lm_row0,
                lm_rows, m->cfg.vocab);
  if (m->xbuf || m->tp_connected) return fail(MK_ESTATE, "mk_tp_setup was already called");
  if (int rc = check_schedule(&m->cfg, m->cfg.max_batch, m->num_sms, m->num_slots, lm_rows)) return rc;
  MK_CUDA(cudaSetDevice(m->device));
  m->tp_rank = rank;
  m->tp_world = world;
  m->lm_row0 = lm_row0;
  m->lm_rows = lm_rows;
  if (world == 1) {
    m->xpeer[0] = nullptr;
    m->tp_connected = true;
    if (buffer) *buffer = nullptr;
    if (handle) memset(handle, 0, sizeof(*handle));
    return MK_OK;
  }
  const size_t bytes = mk::xbuf_words(world, m->cfg.max_batch, m->cfg.hidden) * 8;
  void* buf = nullptr;
  MK_CUDA(cudaMalloc(&buf, bytes));
  m->xbuf = static_cast<unsigned long long*>(buf);
  MK_CUDA(cudaMemset(buf, 0, bytes));  // tag 0 is never a phase tag
  MK_CUDA(cudaDeviceSynchronize());
  if (handle) {
    static_assert(sizeof(cudaIpcMemHandle_t) == sizeof(MkIpcHandle), "IPC handle size");
    cudaIpcMemHandle_t h;
    MK_CUDA(cudaIpcGetMemHandle(&h, buf));
    memcpy(handle, &h, sizeof(h));
  }
  if (buffer) *buffer = buf;
  return MK_OK;
}

int mk_tp_connect(MkModel* m, const MkIpcHandle* handles, void* const* buffers) {
  if (!m) return fail(MK_EINVAL, "model is NULL");
  if (m->tp_world == 1) return m->tp_connected ? MK_OK : fail(MK_ESTATE, "mk_tp_setup has not been called");
  if (!m->xbuf) return fail(MK_ESTATE, "mk_tp_setup has not been called");
  if (m->tp_connected) return fail(MK_ESTATE, "mk_tp_connect was already called");
  if ((handles == nullptr) == (buffers == nullptr))
    return fail(MK_EINVAL, "pass exactly one of handles (one process per GPU) and buffers (one process)");
  MK_CUDA(cudaSetDevice(m->device));
  for (int r = 0; r < m->tp_world; ++r) {
    if (r == m->tp_rank) {
      m->xpeer[r] = m->xbuf;
      continue;
    }
    void* ptr = nullptr;
    if (handles) {
      cudaIpcMemHandle_t h;
      memcpy(&h, &handles[r], sizeof(h));
      MK_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
      m->xpeer_ipc[r] = true;
    } else {
      ptr = buffers[r];
      if (!ptr) return fail(MK_EINVAL, "buffers[%d] is NULL", r);
      cudaPointerAttributes a;
      MK_CUDA(cudaPointerGetAttributes(&a, ptr));
      if (a.device != m->device) {
        const cudaError_t e = cudaDeviceEnablePeerAccess(a.device, 0);
        if (e == cudaErrorPeerAccessAlreadyEnabled) {
          cudaGetLastError();
        } else if (e != cudaSuccess) {
          return fail(MK_ECUDA, "peer access to device %d: %s", a.device, cudaGetErrorString(e));
        }
      }
    }
    m->xpeer[r] = static_cast<unsigned long long*>(ptr);
  }
  m->tp_connected = true;
  return MK_OK;
}

int mk_destroy(MkModel* m) {
  if (!m) return MK_OK;
  cudaSetDevice(m->device);
  for (int r = 0; r < mk::kMaxTp; ++r)
    if (m->xpeer_ipc[r] && m->xpeer[r]) cudaIpcCloseMemHandle(m->xpeer[r]);
  if (m->xbuf) cudaFree(m->xbuf);
  if (m->scratch) cudaFree(m->scratch);
  if (m->host_error) cudaFreeHost(m->host_error);
  if (m->io_host) cudaFreeHost(m->io_host);
  delete m;
  return MK_OK;
}

}  // extern "C"
