/*
 * sa_b200.h -- C ABI of the B200 (sm_100a) decode-time sparse-KV path.
 *
 * One shared library, libsa_b200.so, exports everything declared here.
 * Signatures use plain pointers, sizes and an opaque stream handle
 * (a cudaStream_t passed as void*; NULL means the handle's own stream for
 * context/backend calls and the legacy default stream for stateless calls).
 * No call throws; every call returns an sa_status and records a message
 * readable with sa_last_error() on the calling thread.
 *
 * The reference interfaces each group replaces are cited by file:line in the
 * reference project (ZjuXxxc/solidattention-repro):
 *
 *  - stateless kernels       cpp/src/attention_reference.cpp:55-96,
 *                            cpp/src/selection.cpp:12-147,
 *                            cpp/src/qwen_layer_main.cpp:224-281
 *  - backend handle          cpp/include/solidattention/backend.hpp:41-58,
 *                            cpp/src/cuda_backend.cpp:171-471
 *  - paged decode context    cpp/src/kv_lifecycle_main.cpp:25-113,
 *                            cpp/src/online_seal_main.cpp:34-47,
 *                            cpp/src/qwen_chain_main.cpp:360-395,
 *                            src/solidattention_lab/kv_lifecycle.py:17-98
 *
 * Data formats (all device buffers unless a name ends in _host):
 *  - token row: FP16 [2][kv_heads][head_dim], K plane then V plane, as the
 *    reference's interleaved buffers (backend.hpp:18-31); 32 tokens form a
 *    block of 32 rows (128 KiB at 8 KV heads x 128 dims).
 *  - query: FP32 [query_heads][head_dim].
 *  - representatives, reference layout: FP32 [query_heads][blocks][head_dim]
 *    (selection.hpp:14-17); the context stores them dimension-major,
 *    [query_heads][head_dim][block capacity], so that block scoring reads
 *    them coalesced.
 */
#ifndef SA_B200_H
#define SA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define SA_API __attribute__((visibility("default")))
#else
#define SA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ status */

typedef int sa_status;
#define SA_OK 0
#define SA_ERR_INVALID_ARG (-1) /* dimensions/pointers the reference rejects */
#define SA_ERR_UNSUPPORTED (-2) /* valid for the reference, not built here   */
#define SA_ERR_CAPACITY (-3)    /* pool, table or workspace too small        */
#define SA_ERR_CUDA (-4)        /* a CUDA runtime/driver call failed         */
#define SA_ERR_DEVICE (-5)      /* a kernel raised a device status bit       */
#define SA_ERR_TIMEOUT (-6)     /* a bounded device wait gave up             */
#define SA_ERR_NO_MEMORY (-7)   /* host or device allocation failed          */

/* Device status bits, OR-ed into a status word by the kernels (never a trap). */
#define SA_DEV_BAD_BLOCK 0x1u    /* block id outside the pool or the table   */
#define SA_DEV_TAIL_FULL 0x2u    /* append into a full tail (no seal ran)    */
#define SA_DEV_POOL_EMPTY 0x4u   /* seal found no free pool block            */
#define SA_DEV_NONFINITE 0x8u    /* a block score was NaN or infinite        */
#define SA_DEV_TIMEOUT 0x10u     /* a bounded barrier wait gave up           */
#define SA_DEV_TABLE_FULL 0x20u  /* seal beyond the block-table capacity     */

SA_API const char* sa_status_string(sa_status status);
/* Message of the last failing call on this host thread ("" if none). */
SA_API const char* sa_last_error(void);
/* Library version string, e.g. "sa_b200 0.1 sm_100a". */
SA_API const char* sa_version(void);

/* ------------------------------------------------------ stateless kernels */

/* GQA decode attention over a packed token-major buffer.
 * Replaces attention_reference (cpp/src/attention_reference.cpp:55-96) and the
 * device kernels sparse_attention / sparse_attention_parallel
 * (cpp/src/cuda_backend.cpp:70-158) and sparse_fp16_attention
 * (cpp/src/qwen_layer_main.cpp:224-268), without their 128/256-token caps.
 * kv: [tokens][2][kv_heads][head_dim] FP16; query: [query_heads][head_dim]
 * FP32; out: [query_heads][head_dim], FP32 (out_fp16 = 0) or FP16 RNE.
 * head_dim must be 128; query_heads/kv_heads in {1,2,4,8}.
 * workspace: device scratch of sa_attention_workspace_size() bytes (split-K
 * partials + arrival counters); it must start zeroed once and is left
 * zeroed by every completed call. */
SA_API size_t sa_attention_workspace_size(size_t tokens, size_t query_heads,
                                          size_t kv_heads);
SA_API sa_status sa_attention_packed(const uint16_t* kv, const float* query,
                                     size_t tokens, size_t query_heads,
                                     size_t kv_heads, size_t head_dim,
                                     float scale, void* out, int out_fp16,
                                     void* workspace, size_t workspace_bytes,
                                     void* stream);

/* The same attention for callers that cannot allocate device memory: a
 * serving process that has already reserved all free HBM for its KV pool, a
 * decode loop that cannot afford the device-wide synchronisation a
 * cudaMalloc brings, or a foreign-language host with no device allocator.
 * It allocates nothing: its split-K scratch is a 2 MiB static device array,
 * held by every GPU that loads this library until the process exits.
 * Problems whose workspace (sa_attention_workspace_size) exceeds 2 MiB are
 * refused with SA_ERR_CAPACITY. Every call made outside a stream capture
 * looks up the array's device address on the current device
 * (cudaGetSymbolAddress), so the address follows a device reset; a call
 * made while its stream is capturing reuses the address of the last such
 * call on that device, so make a first call on each device before any
 * stream capture (a capture with none before it is refused). All calls
 * share the one array, so calls that overlap on the GPU (other streams,
 * other host threads) race; serialise them.
 * This entry point has no counterpart in the reference. */
SA_API sa_status sa_attention_packed_noalloc(const uint16_t* kv,
                                             const float* query, size_t tokens,
                                             size_t query_heads,
                                             size_t kv_heads, size_t head_dim,
                                             float scale, void* out,
                                             int out_fp16, void* stream);

/* InfLLM block scoring + init/local forcing + deterministic top-k.
 * Replaces select_shared_blocks (cpp/src/selection.cpp:96-147,
 * decl cpp/include/solidattention/selection.hpp:25-29), applied to each group
 * of `group` consecutive query heads (group == query_heads is the reference's
 * shared mode; group == query_heads/kv_heads selects per KV head).
 * Scores are computed in the reference's order (per head: sequential
 * head_dim dot, no fused multiply-add, then dot/group added head by head), so
 * they are bit-identical to the reference's; ties go to the lower block id.
 * reps element (h, b, d) lives at reps[h*stride_head + b*stride_block + d*stride_dim].
 * block_ids_out: [query_heads/group][budget] int32, ascending.
 * scores_out (nullable): [query_heads/group][blocks] FP32 (mean_head_scores).
 * Invalid dimensions are rejected as the reference rejects them. */
SA_API size_t sa_select_workspace_size(size_t query_heads, size_t group,
                                       size_t blocks);
SA_API sa_status sa_select_blocks(const float* query, const float* reps,
                                  int64_t stride_head, int64_t stride_block,
                                  int64_t stride_dim, size_t query_heads,
                                  size_t group, size_t blocks, size_t head_dim,
                                  size_t budget_blocks, size_t init_blocks,
                                  size_t local_blocks, int32_t* block_ids_out,
                                  float* scores_out, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* Local-causal received-mass representatives.
 * Replaces build_local_causal_representatives (cpp/src/selection.cpp:12-94).
 * prompt_queries: [query_heads][tokens][head_dim] FP32; kv as above.
 * values_out: [query_heads][tokens/block_tokens][head_dim] FP32;
 * offsets_out: [query_heads][tokens/block_tokens][topk] int32 (rank order).
 * Dot products and sums follow the reference's order; only expf may differ
 * in the last place. head_dim <= 256, block_tokens == 32, local_window <= 128. */
SA_API sa_status sa_build_representatives(
    const float* prompt_queries, const uint16_t* kv, size_t tokens,
    size_t query_heads, size_t kv_heads, size_t head_dim, size_t block_tokens,
    size_t local_window, size_t topk, float* values_out, int32_t* offsets_out,
    void* stream);

/* FP32 -> FP16 (round to nearest even) pack of one token's K and V into row
 * `token` of a packed buffer [rows][K elements | V elements].
 * Replaces append_fp16_kv (cpp/src/qwen_layer_main.cpp:270-281). */
SA_API sa_status sa_pack_kv_fp16(uint16_t* packed, const float* key,
                                 const float* value, size_t token,
                                 size_t elements, void* stream);

/* ---------------------------------------------------------- backend handle */

/* Host-buffer attention calls with the timing split of the reference's
 * AcceleratorBackend (cpp/include/solidattention/backend.hpp:33-58,
 * cpp/src/cuda_backend.cpp:323-415): H2D of KV + query, kernel, optional
 * consumer, optional D2H, then a synchronize. Device buffers grow on demand
 * and persist across calls. One handle per host thread. */
typedef struct sa_backend sa_backend;

typedef struct {
  double h2d_ms;
  double kernel_ms;
  double consumer_ms;
  double d2h_ms;
} sa_timings;

#define SA_ATTN_COPY_OUTPUT 0x1 /* D2H into out_host: the FP32 output, or with
                                   SA_ATTN_CONSUME the checksum (1 float)     */
#define SA_ATTN_CONSUME 0x2     /* run the checksum consumer on the device:
                                   sum(out[i] * (1 + (i % 17) * 1e-3))        */

SA_API sa_status sa_backend_create(int device, sa_backend** out);
SA_API sa_status sa_backend_destroy(sa_backend* backend);
SA_API const char* sa_backend_name(const sa_backend* backend);
SA_API sa_status sa_backend_host_alloc(sa_backend* backend, size_t bytes,
                                       void** out);
SA_API sa_status sa_backend_host_free(sa_backend* backend, void* pointer);
SA_API sa_status sa_backend_attention(sa_backend* backend,
                                      const uint16_t* kv_host,
                                      const float* query_host, size_t tokens,
                                      size_t query_heads, size_t kv_heads,
                                      size_t head_dim, float scale, int flags,
                                      float* out_host, sa_timings* timings);
/* Host-buffer selection with the reference's signature and semantics
 * (select_shared_blocks, cpp/src/selection.cpp:96-147): reps in the reference
 * layout [query_heads][blocks][head_dim]; one shared selection over all query
 * heads. ids_out_host receives budget_blocks ids ascending; scores_out_host
 * (nullable) the blocks' mean_head_scores. Synchronous. */
SA_API sa_status sa_backend_select(sa_backend* backend, const float* query_host,
                                   const float* reps_host, size_t query_heads,
                                   size_t blocks, size_t head_dim,
                                   size_t budget_blocks, size_t init_blocks,
                                   size_t local_blocks, int64_t* ids_out_host,
                                   float* scores_out_host);
/* Host-buffer representative build with the reference's signature and
 * semantics (build_local_causal_representatives, cpp/src/selection.cpp:12-94):
 * values_out_host [query_heads][tokens/block_tokens][head_dim],
 * offsets_out_host [query_heads][tokens/block_tokens][topk]. Synchronous. */
SA_API sa_status sa_backend_build_representatives(
    sa_backend* backend, const float* prompt_queries_host,
    const uint16_t* kv_host, size_t tokens, size_t query_heads,
    size_t kv_heads, size_t head_dim, size_t block_tokens, size_t local_window,
    size_t topk, float* values_out_host, int64_t* offsets_out_host);
/* C0 transport smoke: out = in ^ mask over `bytes`, checksum of the bytes
 * (cpp/src/cuda_backend.cpp:242-280). */
SA_API sa_status sa_backend_execute(sa_backend* backend, void* pinned_input,
                                    size_t bytes, uint8_t mask,
                                    sa_timings* timings,
                                    uint64_t* checksum_out);

/* ---------------------------------------------------- paged decode context */

/* A context owns, on one device: a paged pool of 32-token FP16 blocks, a
 * free list, per-(sequence, layer) block tables, sealed-block counts, open
 * tails (one pool block each), a query ring for the tail's tokens,
 * dimension-major representatives, selection outputs, scratch and a stream.
 * One decode step per (sequence, layer) appends the current token, scores
 * and selects sealed blocks, attends over the selected blocks plus the open
 * tail, and seals the tail when it reaches 32 tokens (rebuilding the new
 * block's representative from the tail's 32 queries, as
 * cpp/src/online_seal_main.cpp:41 does). Every step call is asynchronous on
 * the context stream, allocates nothing and can be captured in a CUDA graph. */
typedef struct sa_ctx sa_ctx;

typedef struct {
  int32_t device;
  int32_t query_heads;      /* QH */
  int32_t kv_heads;         /* KH; QH/KH in {1,2,4,8} */
  int32_t head_dim;         /* must be 128 */
  int32_t layers;
  int32_t seqs;             /* sequences (batch) */
  int32_t pool_blocks;      /* physical 32-token blocks in the pool */
  int32_t table_blocks;     /* sealed-block capacity per (seq, layer) */
  int32_t budget_blocks;    /* selected sealed blocks per step */
  int32_t init_blocks;      /* forced leading blocks */
  int32_t local_blocks;     /* forced trailing sealed blocks */
  int32_t select_group;     /* query heads per selection group; multiple of QH/KH */
  int32_t rep_window;       /* local-causal window of the seal rebuild (32) */
  int32_t rep_topk;         /* keys averaged per representative (4) */
  int32_t out_fp16;         /* attention output FP16 (1) or FP32 (0) */
  float scale;              /* softmax scale, e.g. 1/sqrt(head_dim) */
} sa_ctx_config;

/* Device pointers owned by a context, for callers that fill or inspect it. */
typedef struct {
  uint16_t* pool;         /* [pool_blocks][KH][2 (K,V)][32][D]: head-major
                             blocks, one 16 KB K+V run per (block, head) */
  float* reps;            /* [seqs*layers][QH][D][table_blocks] */
  int32_t* table;         /* [seqs*layers][table_blocks] logical -> physical */
  int32_t* num_sealed;    /* [seqs*layers] */
  int32_t* tail_block;    /* [seqs*layers] physical block of the open tail */
  int32_t* tail_len;      /* [seqs*layers] tokens in the open tail, 0..31 */
  int32_t* generation;    /* [seqs*layers] seals so far */
  float* query_ring;      /* [seqs*layers][QH][32][D] queries of tail tokens */
  int32_t* selected;      /* [seqs*layers][QH/select_group][budget] logical ids */
  int32_t* selected_count;/* [seqs*layers][QH/select_group] */
  float* scores;          /* [seqs*layers][QH/select_group][table_blocks] */
  int32_t* free_list;     /* [pool_blocks] */
  int32_t* free_top;      /* [1] */
  uint32_t* status;       /* [1] device status bits */
} sa_ctx_ptrs;

SA_API sa_status sa_ctx_create(const sa_ctx_config* config, sa_ctx** out);
SA_API sa_status sa_ctx_destroy(sa_ctx* ctx);
SA_API sa_status sa_ctx_get_ptrs(sa_ctx* ctx, sa_ctx_ptrs* out);
SA_API sa_status sa_ctx_set_stream(sa_ctx* ctx, void* stream);
SA_API void* sa_ctx_stream(sa_ctx* ctx);
/* Empty every sequence, refill the free list, clear the status word. */
SA_API sa_status sa_ctx_reset(sa_ctx* ctx);
/* Give (seq, layer) `blocks` sealed blocks plus an empty open tail, taking
 * blocks from the free list (synchronous). phys_out_host (nullable,
 * capacity blocks + 1) receives the physical ids: sealed blocks in logical
 * order, then the tail block. The caller fills the pool rows itself. */
SA_API sa_status sa_ctx_prefill(sa_ctx* ctx, int32_t seq, int32_t layer,
                                int32_t blocks, int32_t* phys_out_host);
/* Build representatives of sealed blocks [first, first+count) of
 * (seq, layer) from prompt queries [QH][count*32][D] FP32 (device).
 * per_block = 1: each block alone (the online-seal call, T = 32);
 * per_block = 0: one call over the whole range (windows cross blocks). */
SA_API sa_status sa_ctx_build_reps(sa_ctx* ctx, int32_t seq, int32_t layer,
                                   int32_t first, int32_t count,
                                   const float* prompt_queries, int32_t window,
                                   int32_t topk, int32_t per_block);
/* One decode step for every (seq, layer):
 *   query [seqs][layers][QH][D] FP32;
 *   kv_new [seqs][layers][2][KH][D], FP16 (kv_fp32 = 0) or FP32 packed RNE;
 *   out [seqs][layers][QH][D] (FP16 or FP32 per config). */
SA_API sa_status sa_ctx_step(sa_ctx* ctx, const float* query,
                             const void* kv_new, int32_t kv_fp32, void* out);
/* The decode step from raw projections, with the append fused with its
 * producers (head_rms + rope + append_fp16_kv, cpp/src/qwen_layer_main.cpp:
 * 146-183, 270-281, in the order of cpp/src/qwen_chain_main.cpp:370-392):
 * queries and keys are RMS-normalised per head with the layer's q_norm /
 * k_norm weights and rotated (rotate-half RoPE at the sequence's position),
 * then the keys and values are packed to FP16 into the tail.
 *   q_raw [seqs][layers][QH][D], k_raw and v [seqs][layers][KH][D] FP32;
 *   q_norm_w, k_norm_w [layers][D] FP32; positions [seqs] int32 (decode
 *   position of this token); all device pointers; out as in sa_ctx_step.
 * head_dim 128 only. */
SA_API sa_status sa_ctx_step_raw(sa_ctx* ctx, const float* q_raw, const float* k_raw,
                                 const float* v, const float* q_norm_w, const float* k_norm_w,
                                 const int32_t* positions, float rope_theta, float norm_eps,
                                 void* out);
/* The same step from host buffers: H2D inputs, step, D2H output, synchronize
 * (the end-to-end call of a host-side decode loop). Pinned (mapped) buffers
 * are used in place except the queries, which are copied; with all three
 * pinned, no peer gather attached and a non-legacy stream, the first call
 * records the copy and the step's launches into a CUDA graph and later calls
 * with the same buffers replay it. Pageable buffers go through staging
 * copies on every call. */
SA_API sa_status sa_ctx_step_host(sa_ctx* ctx, const float* query_host,
                                  const void* kv_new_host, int32_t kv_fp32,
                                  void* out_host);
/* The step's stages, for callers that interleave their own work. */
SA_API sa_status sa_ctx_append(sa_ctx* ctx, const float* query,
                               const void* kv_new, int32_t kv_fp32);
SA_API sa_status sa_ctx_select(sa_ctx* ctx, const float* query);
SA_API sa_status sa_ctx_attend(sa_ctx* ctx, const float* query, void* out);
SA_API sa_status sa_ctx_seal(sa_ctx* ctx);
/* Synchronize the context stream and fold the device status word into the
 * return code (SA_ERR_DEVICE / SA_ERR_TIMEOUT); *bits_out (nullable) gets it. */
SA_API sa_status sa_ctx_sync(sa_ctx* ctx, uint32_t* bits_out);
/* Kernel launches issued by the context since creation (for accounting). */
SA_API uint64_t sa_ctx_launch_count(const sa_ctx* ctx);
/* Decode-step graphs. No reference counterpart: the reference synchronises
 * after every call (cpp/src/cuda_backend.cpp:397). Between
 * sa_ctx_graph_begin and sa_ctx_graph_end the context's stream-ordered calls
 * (sa_ctx_step, sa_ctx_step_raw, the stage calls, ...) are recorded into a
 * CUDA graph instead of running; sa_ctx_graph_end instantiates and uploads
 * the recording (replacing an earlier one) and sa_ctx_graph_launch replays it
 * on the context's stream, reading and writing the device addresses the
 * recorded calls named. Calls that synchronise or read host memory
 * (sa_ctx_sync, sa_ctx_step_host, setup calls) are refused while a recording
 * is open, and the context's stream must not be the legacy default stream.
 * Replays run back to back without host launch gaps between the kernels. */
SA_API sa_status sa_ctx_graph_begin(sa_ctx* ctx);
SA_API sa_status sa_ctx_graph_end(sa_ctx* ctx);
SA_API sa_status sa_ctx_graph_launch(sa_ctx* ctx);
/* Quality audit of the selection (replaces audit_dense_selection,
 * cpp/src/pipeline_main.cpp:502-574, and the selected-vs-dense comparison of
 * cpp/src/selection_main.cpp:246-252): for every (seq, layer, KV head), the
 * dense softmax of the KV head's query heads over all sealed blocks plus the
 * open tail, summed per block and averaged over those heads.
 *   query    [seqs][layers][QH][D] FP32 (device);
 *   mass_out [seqs*layers][KH][table_blocks + 1] FP32 (device): entry b <
 *            num_sealed = sealed block b, entry table_blocks = the tail,
 *            others 0; each row sums to 1 (when the row has tokens).
 * Asynchronous on the context stream; not part of the decode step. */
SA_API sa_status sa_ctx_audit(sa_ctx* ctx, const float* query, float* mass_out);
/* History-prediction slot table (replaces compare_prediction,
 * cpp/src/pipeline_main.cpp:686-717, and the slot maps of
 * src/solidattention_lab/qwen_decode.py:463-545): a resident window of
 * `budget` slots per (seq, layer, selection group) that holds the blocks
 * predicted for this step (last step's selection). Against the context's
 * current selection (after sa_ctx_select / sa_ctx_step): hits stay; the
 * misses (selected blocks not resident, ascending) overwrite, in order, the
 * slots whose block was not selected (in slot order); slots left over when
 * the selection is shorter than the window are emptied. Empty slots are -1.
 *   slots   [seqs*layers][groups][budget] int32, device, corrected in place;
 *   misses  [seqs*layers][groups][budget] int32, device: blocks to load, -1 padded;
 *   replace [seqs*layers][groups][budget] int32, device: the slot each miss
 *           overwrites, -1 padded;
 *   stats   [seqs*layers][groups][2] int32, device: hits, misses.
 * Asynchronous on the context stream. */
SA_API sa_status sa_ctx_slot_correct(sa_ctx* ctx, int32_t* slots, int32_t* misses,
                                     int32_t* replace, int32_t* stats);
/* Blocks in the reference's main-store format (the rows the reference
 * pwrites per sealed block, cpp/src/kv_lifecycle_main.cpp:104-108, and the
 * layer segments of src/solidattention_lab/qwen_kv_lab.py:77-107): a block is
 * [32 tokens][2 (K,V)][KH][D] FP16, 128 KiB at KH = 8. These copy logical
 * blocks [first, first+count) of (seq, layer) -- through the block table --
 * between the head-major pool and `store` [count][32][2][KH][D], which may be
 * device memory or pinned, mapped host memory (a host tier's staging
 * buffer); 16-byte aligned. Import fills blocks already in the table (after
 * sa_ctx_prefill, or sealed ones being reloaded). Asynchronous on the
 * context stream. */
SA_API sa_status sa_ctx_import_blocks(sa_ctx* ctx, int32_t seq, int32_t layer, int32_t first,
                                      int32_t count, const void* store);
SA_API sa_status sa_ctx_export_blocks(sa_ctx* ctx, int32_t seq, int32_t layer, int32_t first,
                                      int32_t count, void* store);

/* ---- KV-head-sharded contexts: outputs gathered over peer memory ---------
 * No reference counterpart as a function: replaces the all-gather of
 * per-head attention outputs that follows the attention when one long
 * sequence's KV heads are split across `world` GPUs (rank r's context holds
 * KV heads [r*KH, (r+1)*KH), KH = its kv_heads). Once attached, every
 * attention launch of the context also stores each (seq-layer, KV head)
 * output into the current parity slot of every rank's gathered buffer
 * (NVLink P2P stores), laid out [seqs][layers][world*QH][D] (the full head
 * set). After the attention completes, one thread fences at system scope
 * and counts one arrival on every rank's buffer, then waits, bounded, for
 * every rank's arrival (in a decode step's own seal kernel, or in the
 * kernel sa_ctx_gather_wait enqueues). Slots alternate per attention, so a
 * slot stays valid until the attention after next.
 *
 * Setup, per rank: sa_ctx_gather_buffer -> sa_ipc_export the buffer ->
 * exchange the handles (any host channel) -> sa_ipc_open every other rank's
 * handle -> sa_ctx_gather_attach with the [world] pointers (own buffer at
 * index rank). Every rank's context must have the same shape. */
#define SA_IPC_HANDLE_BYTES 64
/* Allocate (once) this rank's gathered buffer for `world` ranks. */
SA_API sa_status sa_ctx_gather_buffer(sa_ctx* ctx, int32_t world, void** buf_out,
                                      size_t* bytes_out);
/* peer_bufs: host array [world] of device pointers, peer_bufs[rank] = own.
 * Attaching (again) synchronizes the context stream and zeroes this rank's
 * arrival counter and epoch. After a wait timed out (SA_ERR_TIMEOUT), late
 * arrivals of that step could satisfy a later wait early, so every rank
 * re-attaches, with no gathered step in flight anywhere, before the next
 * gathered step. */
SA_API sa_status sa_ctx_gather_attach(sa_ctx* ctx, int32_t rank, void* const* peer_bufs);
/* Enqueue the wait for the latest attention's outputs from every rank;
 * *gathered_out (nullable) = the slot holding them [seqs][layers][world*QH][D].
 * A decode step (sa_ctx_step) of an attached context already waits for them
 * in its own seal kernel, so after a step this call only returns the slot
 * and launches nothing; after an attention of its own (sa_ctx_attend,
 * sa_ctx_step_raw) it enqueues the wait kernel.
 * A wait that gives up sets SA_DEV_TIMEOUT in the status word. The slot
 * parity and the expected arrival count are kept on the device, so
 * attention + wait pairs recorded with sa_ctx_graph_begin replay correctly
 * (every attention must be followed by its wait before the next one). A
 * slot address handed out while recording stays fixed in the graph while
 * every replay advances the parity once per gathered attention, so
 * sa_ctx_graph_end refuses (SA_ERR_UNSUPPORTED) a recording that handed one
 * out and holds an odd number of gathered attentions. */
SA_API sa_status sa_ctx_gather_wait(sa_ctx* ctx, void** gathered_out);
/* CUDA IPC handle of a device allocation (SA_IPC_HANDLE_BYTES bytes), and
 * mapping / unmapping another process's allocation on `device`. */
SA_API sa_status sa_ipc_export(int32_t device, const void* dev_ptr, void* handle_out);
SA_API sa_status sa_ipc_open(int32_t device, const void* handle, void** dev_ptr_out);
SA_API sa_status sa_ipc_close(int32_t device, void* dev_ptr);

/* ---- streaming probe (no reference counterpart: a measurement aid) ----
 * Reads entries of 16 KB (one (block, KV head) of the head-major pool) into
 * shared memory the two ways the attention could stage them, two CTAs of
 * 256 threads per SM each streaming a contiguous share of `entry_ids` through
 * three 32 KB stages: mode 0 per-lane 16-byte cp.async copies (the
 * attention's loads), mode 1 one 16 KB cp.async.bulk per entry issued by one
 * thread and completed on an mbarrier (plain loads of this GPU's memory, no
 * cluster multicast). pool: device, 16-byte aligned, pool_entries * 16384
 * bytes; entry_ids: device [n] (ids outside the pool read entry 0);
 * sink: device, at least SA_PROBE_SINK_WORDS uint64 (one word per CTA keeps
 * the reads); status: device word or null (SA_DEV_TIMEOUT when a bounded
 * mbarrier wait gave up). Asynchronous on `stream`; time it with events. */
#define SA_PROBE_SINK_WORDS 1024
SA_API sa_status sa_probe_stream(const void* pool, int64_t pool_entries, const int32_t* entry_ids,
                                 int64_t n, int32_t mode, uint64_t* sink, uint32_t* status,
                                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SA_B200_H */
