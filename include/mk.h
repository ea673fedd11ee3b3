/*
 * mk.h — C ABI of the B200 (sm_100a) Llama decode megakernel.
 *
 * One persistent, cooperative CUDA launch decodes one token for every sequence
 * of a batch: all decoder layers (RMSNorm -> QKV -> llama3 RoPE -> paged KV
 * scatter -> split-K GQA flash-decode -> o_proj + residual -> RMSNorm ->
 * SwiGLU gate/up -> down + residual), then the final RMSNorm, the tied lm_head
 * GEMV and a greedy argmax.
 *
 * Ownership: the caller owns every device buffer passed in (weights, KV pages,
 * block tables, tokens, positions, outputs). The library only borrows the raw
 * pointers for the duration of a call. Scratch the kernel needs between its
 * phases (residual, q/k/v, attention partials, barrier counters) is owned by
 * the MkModel handle and allocated in mk_init.
 *
 * Errors: every entry point returns an MkStatus; mk_last_error() gives the
 * message for the calling thread's last failure. Device-side failures (a
 * barrier or pipeline wait that ran out of time, a position or page id out of
 * range) are recorded in a device error word and reported by mk_sync().
 *
 * Threading: one stream per handle; calls on one handle are not re-entrant.
 * mk_decode is asynchronous with respect to the host.
 *
 * Reference interfaces this replaces (keaganchern/llama1B-megakernel):
 *   - transformer_llama_megakernel_16layers(X, Wq, Wk, Wv, Wo, gpre, Wgu, Wd,
 *     gpost, K_00..K_15, V_00..V_15, cos, sin, position_ids) -> (Y, K.., V..)
 *     transformer_llama.py:196-237, called at llama_with_megakernel.py:165-173
 *     -> mk_decode_hidden (hidden in, hidden out, caches updated in place) and
 *        mk_decode (embedding ... argmax, the whole token-generation step).
 *   - NeuronLlamaForCausalLMMK.convert_hf_to_neuron_state_dict
 *     llama_with_megakernel.py:281-351 (pre-stacked weights bound once)
 *     -> mk_load_weights.
 *   - the shape/TP asserts at llama_with_megakernel.py:145-162 -> MK_EINVAL
 *     from mk_init / mk_load_weights / mk_decode.
 */
#ifndef MK_H_
#define MK_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum MkStatus {
  MK_OK = 0,
  MK_EINVAL = 1,     /* bad argument, shape or configuration */
  MK_ECUDA = 2,      /* a CUDA runtime call failed */
  MK_ETIMEOUT = 3,   /* a device-side wait ran out of time; the kernel returned */
  MK_ENOMEM = 4,     /* device allocation failed */
  MK_ESTATE = 5,     /* call out of order (e.g. decode before load_weights) */
  MK_EDEVICE = 6     /* device reported a bad position, page id or token */
} MkStatus;

/* Model + cache geometry. head_dim must be 64; num_q_heads / num_kv_heads == 4. */
typedef struct MkConfig {
  int32_t num_layers;
  int32_t hidden;
  int32_t intermediate;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t vocab;
  float rms_eps;
  int32_t max_batch;           /* 1..4 */
  int32_t page_size;           /* KV positions per page, multiple of 8 */
  int32_t num_pages;           /* pages per layer in the KV pool */
  int32_t max_blocks_per_seq;  /* columns of the block table */
  int32_t rope_len;            /* rows of the cos/sin tables (max position + 1) */
} MkConfig;

/*
 * Device pointers to the packed bf16 weights (layouts produced by the host
 * packer, llama1b_megakernel_b200/weights.py):
 *   embed      [vocab][hidden]                  (also the tied lm_head)
 *   w_qkv      [L][(nq + 2*nkv) * 32][2][hidden] RoPE pairs: rows (d, d+32) of
 *                                                each q/k/v head, adjacent
 *   w_o        [L][hidden][nq * 64]             (HF o_proj.weight)
 *   w_gate_up  [L][intermediate][2][hidden]     gate row i, up row i adjacent
 *   w_down     [L][hidden][intermediate]        (HF down_proj.weight)
 *   norm_attn  [L][hidden], norm_mlp [L][hidden], norm_final [hidden]
 *   rope_cos, rope_sin [rope_len][64]           bf16 cos/sin per position
 * All pointers must be 16-byte aligned.
 */
typedef struct MkWeights {
  const void* embed;
  const void* w_qkv;
  const void* w_o;
  const void* w_gate_up;
  const void* w_down;
  const void* norm_attn;
  const void* norm_mlp;
  const void* norm_final;
  const void* rope_cos;
  const void* rope_sin;
} MkWeights;

/*
 * Paged bf16 KV cache, updated in place:
 *   k_pages, v_pages  [L][num_pages][nkv][page_size][64]
 *   block_tables      [batch][max_blocks_per_seq] int32 page ids (all layers)
 * Position p of sequence b is slot p % page_size of page
 * block_tables[b][p / page_size].
 */
typedef struct MkKVCache {
  void* k_pages;
  void* v_pages;
  const int32_t* block_tables;
} MkKVCache;

/* mk_decode flags */
#define MK_FLAG_FEEDBACK 1  /* after the step: tokens[b] = next id, positions[b] += 1 */

typedef struct MkModel MkModel;

/* Validate cfg, pick the grid for `device`, allocate scratch. */
int mk_init(const MkConfig* cfg, int device, MkModel** out);

/* Bind (borrow) the packed weight pointers. */
int mk_load_weights(MkModel* m, const MkWeights* w);

/*
 * Enqueue one decode step on `stream` (a cudaStream_t, NULL = legacy default).
 * tokens[batch], positions[batch] (int32, device): the token at `positions[b]`
 * of sequence b; its K/V row is written at that position. logits (device,
 * [batch][vocab] fp32) may be NULL. next_ids (device, [batch] int32) gets the
 * greedy argmax (lowest index on ties).
 */
int mk_decode(MkModel* m, const int32_t* tokens, const int32_t* positions, int32_t batch,
              const MkKVCache* kv, float* logits, int32_t* next_ids, int32_t flags,
              void* stream);

/*
 * mk_decode with HOST buffers, synchronous: copies tokens[batch] and
 * positions[batch] (int32, host) to the device, enqueues the step on
 * `stream`, copies the greedy ids back into next_ids[batch] (int32, host),
 * waits for the stream and reports device errors as mk_sync does. logits is a
 * device pointer as in mk_decode (may be NULL). The staging buffers are the
 * handle's own (allocated by mk_init), so calls on one handle must not
 * overlap. This is one token-generation call of the reference's model
 * forward (`llama_with_megakernel.py:165-173` inside NxDI's decode step) with
 * its host-side inputs and output.
 */
int mk_decode_host(MkModel* m, const int32_t* tokens, const int32_t* positions, int32_t batch,
                   const MkKVCache* kv, float* logits, int32_t* next_ids, void* stream);

/*
 * The decoder layers only, the role of the reference's 16-layer kernel:
 * hidden_in [batch][hidden] bf16 (the embedded token) -> hidden_out
 * [batch][hidden] bf16 (the residual after the last layer, before the final
 * norm); KV rows written at positions like mk_decode.
 */
int mk_decode_hidden(MkModel* m, const void* hidden_in, const int32_t* positions, int32_t batch,
                     const MkKVCache* kv, void* hidden_out, void* stream);

/*
 * mk_decode without a handle and without allocating anything, for callers
 * that cannot call cudaMalloc: a host whose own pool or arena already owns
 * the device memory (a library-side allocation would fail or fragment it), a
 * plugin invoked from inside another runtime's allocator or memory-pressure
 * callback (re-entering the allocator is not allowed there), or a
 * latency-critical loop that cannot afford cudaMalloc's implicit device
 * synchronisation. No counterpart in the reference (its scratch is allocated
 * by the Neuron runtime when the model loads).
 *
 * Same arguments and results as mk_decode, but the geometry and weights are
 * passed in (cfg, w) and the kernel's scratch lives in a 512 KiB array built
 * into the library (one per GPU, held until the process exits): enough for
 * Llama-3.2-1B at cfg->max_batch 1; larger geometries return MK_EINVAL and
 * must use mk_init / mk_decode. Runs on the current device. Its first call on
 * a device looks up the array's device address and sets the kernels'
 * shared-memory limit, so make that call before any stream capture. Each call
 * zeroes the counters it needs first, and the array's activation words too
 * when the geometry differs from the previous call's on that device (calls
 * may alternate between models). All calls on a device share the one array,
 * so calls that overlap on the GPU (other streams, other threads) race:
 * order them on one stream. Device-side failures are not reported by mk_sync:
 * pass error_out (device, 4 int32, zeroed by the call; code, detail, CTA,
 * thread on failure) or NULL.
 */
int mk_decode_static(const MkConfig* cfg, const MkWeights* w, const int32_t* tokens,
                     const int32_t* positions, int32_t batch, const MkKVCache* kv, float* logits,
                     int32_t* next_ids, int32_t flags, int32_t* error_out, void* stream);

/* Wait for `stream`, then report and clear any device-side error. */
int mk_sync(MkModel* m, void* stream);

/* Device-side wait limit in nanoseconds (default 2e9). */
int mk_set_timeout_ns(MkModel* m, uint64_t ns);

/*
 * Test knob for failure detection: CTA `cta` withholds its layer-0 q/k/v rows
 * in the next launches (-1 disables), so the attention reads that wait for
 * them run out of time and the launch ends with MK_ETIMEOUT instead of
 * hanging.
 */
int mk_debug_skip_arrival(MkModel* m, int32_t cta);

/*
 * Phase trace, off by default (no counterpart in the reference; it plays the
 * role of the reference's profiler captures, main.py:377-407). With a device
 * buffer of at least *needed uint64 entries, every later launch records, per
 * CTA and per phase, globaltimer stamps and stall totals:
 *   buffer[(cta * (num_layers * 5 + 1) + phase) * 12 + kind]
 *   phase = layer * 5 + {0 QKV, 1 attention, 2 o_proj, 3 gate/up, 4 down},
 *           num_layers * 5 = lm_head;
 *   kind  = 0 wait start, 1 wait passed, 2 activations loaded, 3 phase done,
 *           4 consumer ns stalled on the weight stream (cumulative),
 *           5 first copy issued, 6 producer ns stalled on a full ring
 *           (cumulative), 7 last copy issued; attention phases also
 *           8 q loaded, 9 cached chunks reduced, 10 warp states combined
 *           and the output (or the split's partials) written, 11 split 0
 *           merged the splits (for the CTA's last item).
 * buffer NULL switches tracing off; *needed (may be NULL) is set either way.
 */
int mk_set_trace(MkModel* m, uint64_t* buffer, int64_t capacity, int64_t* needed);

/* Launch geometry chosen by mk_init: CTAs (one per SM) and ring slots per CTA. */
int mk_query(const MkModel* m, int32_t* grid, int32_t* ring_slots, int32_t* smem_bytes);

/* ---- Sampling after the lm_head -------------------------------------------
 *
 * Per-sequence knobs of the reference's generation (top_k, top_p, temperature:
 * main.py:57-61, prepare_sampling_params main.py:197-205, sampled on device
 * through NxDI's OnDeviceSamplingConfig, main.py:129-130). */
typedef struct MkSampling {
  int32_t top_k;      /* 1: greedy; <= 0 or > 1024: 1024 */
  float top_p;        /* (0, 1] */
  float temperature;  /* <= 0: greedy */
} MkSampling;

/* Draw one token per sequence from fp32 logits [batch][ld] (the first `vocab`
 * columns): divide by the temperature, keep the top_k largest (ties: lowest
 * index first), softmax, keep the smallest prefix whose mass reaches top_p,
 * and draw with a uniform hashed from (seed, step, sequence). Asynchronous
 * on `stream` (launch it after mk_decode wrote the logits). With tokens and
 * positions (device, [batch]) the draw is also written to tokens and the
 * position advanced, as MK_FLAG_FEEDBACK does for the greedy argmax.
 * *error (device int) is set to 1 if a sequence had more than 1024 logits
 * tied at its top_k threshold (its id is then -1). batch <= 64. */
int mk_sample(const float* logits, int32_t batch, int32_t vocab, int64_t ld,
              const MkSampling* params, uint64_t seed, uint64_t step, int32_t* out_ids,
              int32_t* tokens, int32_t* positions, int32_t* error, void* stream);

/* ---- Batched decode attention ---------------------------------------------
 *
 * One layer's decode attention for `batch` sequences over the paged cache:
 * q [batch][num_q_heads][64] bf16 (post-RoPE), k_pages / v_pages the layer's
 * [num_pages][num_kv_heads][page_size][64] bf16 pools, block_tables
 * [batch][max_blocks] and lengths [batch] (device int32; sequence b attends
 * positions [0, lengths[b]), which must already hold the step's own K/V),
 * max_len >= every length; out [batch][num_q_heads][64] bf16 = softmax(q K^T
 * * scale) V per head, GQA group 4 (nki_kernels/attention.py:270-399 for one
 * sequence). Split-K over 256-position pieces, merged in a second launch.
 * *error (device) is set to 1 if a block table names a page outside the
 * pool (that position is skipped). Used by the batched decode path. */
int64_t mk_paged_attention_workspace(int32_t batch, int32_t num_kv_heads, int32_t max_len);
int mk_paged_attention(const void* q, const void* k_pages, const void* v_pages,
                       const int32_t* block_tables, const int32_t* lengths, int32_t batch,
                       int32_t num_q_heads, int32_t num_kv_heads, int32_t page_size,
                       int32_t max_blocks, int32_t num_pages, int32_t max_len, float scale,
                       void* workspace, int64_t workspace_bytes, void* out, int32_t* error,
                       void* stream);

/* Skinny GEMM on the tcgen05 tensor cores for the batched decode path:
 * Y[rows][n] = X[rows][k] . W[n][k]^T (+ residual[rows][n]), bf16 inputs,
 * fp32 accumulation, Y bf16 (out) or fp32 (out_f32, no residual). W is a
 * weight matrix in HF [out][in] layout (any n, k a multiple of 64); X has
 * rows_padded (16, 32, 64, or 128 for prompt prefill) rows of which the first `rows` are real and the
 * rest zero. Narrow W is split along k over the CTAs of a thread-block
 * cluster whose partial sums meet in distributed shared memory, so no
 * workspace is needed: mk_gemm_workspace returns 0 and `workspace` may be
 * NULL (both stay in the interface for callers written against a split-K
 * workspace). *error (device) is set to
 * 101-103 when one of the kernel's (time-bounded) waits ran out. Asynchronous. These
 * are the projections of the reference's decoder (attention.py:95-245,
 * :409-448, mlp.py:60-192, the lm_head llama.py:1208-1227) at batch > 1. */
int64_t mk_gemm_workspace(int32_t n, int32_t k, int32_t rows);
int mk_gemm_bf16(const void* w, int32_t n, int32_t k, const void* x, int32_t rows,
                 int32_t rows_padded, const void* residual, void* out, float* out_f32,
                 void* workspace, int64_t workspace_bytes, int32_t* error, void* stream);

/* Fused elementwise steps of the batched decode path, HF rounding (bf16 with
 * fp32 statistics), asynchronous on `stream`:
 * mk_rmsnorm_rows: out[r] = bf16(bf16(x[r] / sqrt(mean(x[r]^2) + eps)) * gamma)
 *   for `rows` rows of `hidden` bf16 (llama.py:94-145 / HF LlamaRMSNorm);
 * mk_rope_scatter: from qkv [batch][(nq + 2 nkv) * 64], the q/k/v GEMM output
 *   in the packed RoPE-pair order, write q [batch][nq][64] and the K/V rows
 *   into the layer's page pools at positions[b], RoPE (llama3 tables) on q and
 *   k (attention.py:95-245 and the KV scatter, attention.py:450-492); a page id
 *   outside the pool sets *error and the row is not written;
 * mk_swiglu: out[i] = bf16(bf16(silu(g_i)) * u_i) from interleaved (g_i, u_i)
 *   pairs, the packed w_gate_up order (mlp.py:60-192). */
int mk_rmsnorm_rows(const void* x, const void* gamma, float eps, int32_t rows, int32_t hidden,
                    void* out, void* stream);
int mk_rope_scatter(const void* qkv, const void* rope_cos, const void* rope_sin,
                    const int32_t* positions, const int32_t* block_tables, int32_t max_blocks,
                    int32_t num_pages, int32_t page_size, int32_t num_q_heads,
                    int32_t num_kv_heads, int32_t batch, void* q_out, void* k_pages,
                    void* v_pages, int32_t* error, void* stream);
int mk_swiglu(const void* gate_up, int64_t n, void* out, void* stream);

/* Greedy ids of `rows` rows of fp32 logits [rows][cols] (128-bit loads when
 * cols is a multiple of 4 and x 16-byte aligned): ids[r] = the first column
 * holding the row's maximum, as
 * the reference's greedy sampling takes the argmax of the logits
 * (llama.py:1208-1227, torch.argmax). Asynchronous. */
int mk_argmax_rows(const float* x, int32_t rows, int32_t cols, int64_t* ids, void* stream);

/* ---- Tensor-parallel batched step ------------------------------------------
 *
 * The reference's baseline decoder shards o_proj and down by their input
 * columns (RowParallelLinear, llama.py:437-470) and all-reduces their
 * outputs; its lm_head is vocabulary-parallel with the logits gathered for
 * the greedy argmax (llama.py:1208-1227). With the rank's partial sums of
 * o_proj / down all-reduced into `sum` ([rows][hidden] fp32):
 * mk_add_rmsnorm_rows: x = bf16(x + bf16(sum)) in place (the decoder layer's
 *   residual add), out = bf16(bf16(x * 1/sqrt(mean(x^2) + eps)) * gamma).
 * mk_argmax_keys: per row of this rank's fp32 logits [rows][cols] (vocabulary
 *   ids id0 .. id0 + cols - 1), the key (order-preserving float bits of the
 *   maximum << 32 | 2^32 - 1 - the id of its first occurrence), so that the
 *   integer maximum of the ranks' keys names the global greedy id with the
 *   lowest index on ties.
 * mk_keys_to_ids: keys [world][rows] (gathered from every rank) -> ids [rows].
 * All asynchronous on `stream`. */
int mk_add_rmsnorm_rows(void* x, const float* sum, const void* gamma, float eps, int32_t rows,
                        int32_t hidden, void* out, void* stream);
int mk_argmax_keys(const float* x, int32_t rows, int32_t cols, int32_t id0, uint64_t* keys,
                   void* stream);
int mk_keys_to_ids(const uint64_t* keys, int32_t world, int32_t rows, int64_t* ids, void* stream);

/* ---- Tensor parallelism (one decode step over `world` GPUs) --------------
 *
 * Each rank's handle is made with mk_init from the rank's LOCAL geometry:
 * num_q_heads / world q heads, num_kv_heads / world kv heads and
 * intermediate / world MLP rows (vocab stays the whole vocabulary), and its
 * weights are that rank's shard: the q/k/v rows of its heads, the o_proj
 * columns of its q heads, the gate/up rows and down columns of its MLP rows,
 * the whole embedding table (token lookup) of which it scores lm_head rows
 * [lm_row0, lm_row0 + lm_rows). Its KV cache holds only its kv heads. After
 * o_proj and down every rank sends its fp32 partial sums to every other
 * rank's exchange buffer over NVLink inside the kernel and all ranks add them
 * in rank order, so they carry identical residuals; the greedy argmax is
 * exchanged the same way. Logits written by mk_decode are the rank's slice,
 * [batch][lm_rows]. All ranks must make the same sequence of launches.
 * Replaces the all-reduces a tensor-parallel NxDI decoder would issue (the
 * reference's megakernel itself asserts TP = 1, llama_with_megakernel.py:145-149). */
typedef struct MkIpcHandle {
  unsigned char bytes[64]; /* a cudaIpcMemHandle_t */
} MkIpcHandle;

/* Make `m` rank `rank` of `world` scoring lm_head rows [lm_row0, lm_row0 +
 * lm_rows); allocates its exchange buffer (world > 1) and returns its IPC
 * handle and device address (either may be NULL). world == 1 only restricts
 * the lm_head rows. */
int mk_tp_setup(MkModel* m, int32_t rank, int32_t world, int32_t lm_row0, int32_t lm_rows,
                MkIpcHandle* handle, void** buffer);

/* Map the other ranks' exchange buffers: `handles[world]` from their
 * mk_tp_setup when each rank is its own process, or `buffers[world]` when one
 * process drives all GPUs (peer access is enabled); exactly one non-NULL. */
int mk_tp_connect(MkModel* m, const MkIpcHandle* handles, void* const* buffers);

/* ---- Batched tensor-parallel step: the residual all-reduce over peer memory
 *
 * Replaces the all-reduce after the row-parallel o_proj and down of the
 * reference's tensor-parallel decoder (RowParallelLinear, llama.py:437-470)
 * together with the residual add and RMSNorm that follow it (llama.py:1039-1139)
 * in ONE kernel per exchange, with no NCCL on the data path. Each rank owns an
 * exchange buffer of mk_xbuf_bytes(rows, hidden) bytes: two slots of
 * [rows][hidden] fp32 partial sums (slot e % 2 for exchange e of a step, at
 * byte offset (e % 2) * rows * hidden * 4) and a block of flag words.
 * mk_xbuf_alloc allocates and zeroes it on the current device and exports its
 * IPC handle; mk_xbuf_open maps another rank's buffer on the current device
 * (peer access enabled on first use); mk_xbuf_close / mk_xbuf_free undo them
 * (close every mapping on every rank before any owner frees its buffer).
 *
 * mk_step_epoch advances the step counter `epoch` (one device word shared by
 * all exchanges of a step, identical on every rank); launch it once at the
 * start of every step, before the step's first exchange.
 *
 * mk_allreduce_add_rmsnorm, exchange e of the step (0 <= e < 64, each value
 * once per step, the same sequence on every rank): this rank's partial sums
 * for the first `rows` rows must already be in its own slot e % 2 (for
 * instance the fp32 output of mk_gemm_bf16 written there earlier on `stream`).
 * The kernel posts this rank's tag on every rank's flag word, waits (bounded
 * by timeout_ns, 0 = 2 s; on expiry error[0] = 3 and the rows are left
 * unchanged) for every rank's tag, reads the `world` partials of its rows from
 * the owners' buffers over NVLink (plain loads), sums them in rank order (so
 * every rank computes the same bits) and then, as mk_add_rmsnorm_rows,
 * x = bf16(x + bf16(sum)) in place and out = RMSNorm(x) * gamma. `peers` is a
 * device array of `world` buffer addresses as mapped on this GPU (the rank's
 * own at index `rank`); `rows_cap` the rows the buffers were sized for.
 * Asynchronous on `stream`. */
int64_t mk_xbuf_bytes(int32_t rows, int32_t hidden);
int mk_xbuf_alloc(int64_t bytes, MkIpcHandle* handle, void** ptr);
int mk_xbuf_open(const MkIpcHandle* handle, void** ptr);
int mk_xbuf_close(void* ptr);
int mk_xbuf_free(void* ptr);
int mk_step_epoch(uint32_t* epoch, void* stream);
int mk_allreduce_add_rmsnorm(const uint64_t* peers, int32_t rank, int32_t world, int32_t rows_cap,
                             int32_t exchange, const uint32_t* epoch, void* x, const void* gamma,
                             float eps, int32_t rows, int32_t hidden, void* out, int32_t* error,
                             uint64_t timeout_ns, void* stream);

/* The largest number of ring fills a consumer warp goes between two waits in
 * the kernel's schedule for this geometry, batch and grid (-1 if a warp's
 * first wait comes at fill 64 or later). mk_init refuses a geometry whose gap
 * exceeds 64 - ring_slots - 8: the ring's 64 full barriers are told apart by
 * parity, which is safe only within that distance. Host-only; no counterpart
 * in the reference (its kernel has no software ring). */
int mk_schedule_gap(const MkConfig* cfg, int32_t batch, int32_t grid, int32_t* gap);

/* Last error message of the calling thread ("" if none). */
const char* mk_last_error(void);

/* Free scratch and the handle. */
int mk_destroy(MkModel* m);

#ifdef __cplusplus
}
#endif

#endif /* MK_H_ */
