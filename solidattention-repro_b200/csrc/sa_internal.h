// sa_internal.h -- parameter blocks and launchers shared between the kernel
// files and the C-ABI implementation (sa_api.cu). Not installed.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "sa_b200.h"

namespace sa {

constexpr int kHeadDim = 128;     // head dimension of every attention kernel
constexpr int kBlockTokens = 32;  // tokens per KV block

// ---- errors ------------------------------------------------------------------

// Records `message` as this thread's last error and returns `status`.
sa_status fail(sa_status status, const std::string& message);
// Maps a CUDA error to SA_ERR_CUDA with the call's name; SA_OK on success.
sa_status cuda_status(cudaError_t err, const char* what);
#define SA_CUDA_TRY(call)                                     \
  do {                                                        \
    const sa_status _s = ::sa::cuda_status((call), #call);    \
    if (_s != SA_OK) return _s;                               \
  } while (0)

// Raises a kernel's dynamic shared memory limit to `bytes` once per device.
// Launches kernel<<<grid, block, smem, stream>>>(args...), with programmatic
// stream serialization when pdl is set (the kernel must pdl_wait before
// reading what the preceding kernel wrote).
template <class... KArgs, class... Args>
cudaError_t launch_kernel(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

sa_status ensure_smem_limit(const void* kernel, int bytes, int* configured_per_device);
constexpr int kMaxDevices = 64;

// Streaming multiprocessors of the current device (cached per device; 148,
// a whole B200, when no device can be queried, e.g. a size query on a host
// without a GPU). Grid plans scale with it, so a context on a partitioned
// device (an MPS or green-context share) gets a plan for the SMs it has.
int device_sm_count();

// ---- decode-context device state (owned by sa_api.cu) -------------------------

struct CtxDev {
  uint16_t* pool;      // head-major: [pool_blocks][kv_heads][K,V][32][128]
  int64_t row_elems;   // 2 * kv_heads * 128 (one token of every head)
  int pool_blocks;
  float* reps;         // [num_sl][qh][128][reps_cap]
  int reps_cap;        // table_blocks rounded up to a multiple of 4
  int32_t* table;      // [num_sl][table_blocks]
  int table_blocks;
  int32_t* num_sealed;
  int32_t* tail_block;
  int32_t* tail_len;
  int32_t* generation;
  float* query_ring;   // [num_sl][qh][32][128]
  int32_t* free_list;
  int32_t* free_top;
  int* seal_counters;  // [0] arrivals of the seal kernel's CTAs; [1] 1 when an append filled a tail (or found it full)
  uint32_t* status;
  uint32_t* status_mirror;  // device-mapped host word the seal commit copies status to (nullable)
  // KV-head-sharded gather (gather_counter null = off): the seal kernel of a
  // decode step also signals this rank's arrival to every rank and waits,
  // bounded, for every rank's (gather_signal_wait with signal; the wait of
  // sa_ctx_gather_wait, without a launch of its own).
  const unsigned long long* gather_counter;
  unsigned long long* gather_epoch;
  void* const* gather_peers;  // device array [gather_world]
  int gather_world;
  size_t gather_counter_bytes;
  int num_sl, qh, kv_heads;
  int rep_window, rep_topk;
  float rep_scale;
};

// ---- attention (sa_attention.cu) -----------------------------------------------

struct AttnParams {
  const void* pool;      // head-major pool base (used when head_major)
  int head_major;        // 1: [block][KV head][K,V][32][128]; 0: token rows at `rows`
  const void* rows;      // token-major rows [token][K,V][KV head][128] FP16 (head_major 0)
  int64_t row_bytes;     // bytes per token row (16-byte multiple)
  int kv_heads;          // KV heads in a pool row
  int group;             // query heads per KV head (1, 2, 4, 8)
  int num_sl;            // (sequence, layer) pairs
  int pool_blocks;       // physical 32-token blocks addressable by the map
  // selected blocks per (sl, selection group): logical ids, ascending
  const int32_t* sel_ids;    // null -> identity 0..n-1
  const int32_t* sel_count;  // null -> fixed_nsel
  int sel_stride;            // ids per selection group
  int n_sel_groups;          // selection groups per sl
  int kv_per_sel_group;      // KV heads sharing one selection group
  int fixed_nsel;
  // logical -> physical block table per sl
  const int32_t* table;  // null -> identity
  int table_stride;
  // open tail per sl (tail_len tokens of physical block tail_block)
  const int32_t* tail_block;  // null -> fixed_tail_block
  const int32_t* tail_len;    // null -> fixed_tail_len
  int fixed_tail_block;
  int fixed_tail_len;
  int tail_pending;    // tokens appended this step but not yet counted in tail_len
  int pdl;             // launched as a programmatic dependent of the previous kernel
  const float* query;  // [num_sl][kv_heads*group][128]
  void* out;           // [num_sl][kv_heads*group][128]
  int out_fp16;
  float scale_log2;     // softmax scale * log2(e)
  int slots_per_unit;   // entry slots of every unit (selected blocks + tail)
  int max_segments;     // CTAs that may cover one unit (partials per unit)
  int ctas;             // grid size
  float* partial;       // [units][max_segments][group][2 + 128]
  int* counters;        // [units], zero between launches
  uint32_t* status;
  // KV-head-sharded gather over peer memory (gather_peers null = off): every
  // unit's output also goes into slot (epoch & 1) of every rank's buffer
  // (slots gather_slot_bytes apart), laid out [sl][world * kv_heads][group]
  // [128] (the full head set, rank r's KV heads at [r * kv_heads,
  // (r + 1) * kv_heads)), followed by one system-scope arrival on each rank's
  // counter. The epoch is this rank's count of completed gathers, kept on the
  // device so that a recorded graph replays correctly.
  void* const* gather_peers;      // device array [gather_world]
  int gather_world;
  int gather_rank;
  size_t gather_slot_bytes;
  size_t gather_counter_bytes;
  const unsigned long long* gather_epoch;
  // 1: every unit's push also counts an arrival on every rank (a standalone
  // attention, waited for by sa_ctx_gather_wait); 0: the decode step's seal
  // kernel signals once per rank for the whole grid
  int gather_unit_arrivals;
};

// The persistent attention schedule: `ctas` CTAs, each owning a contiguous
// range of the flattened (unit, slot) list; a unit is covered by at most
// `max_segments` of them.
struct AttnPlan {
  int slots_per_unit;
  int max_segments;
  int ctas;
};
AttnPlan attention_plan(int units, int slots_per_unit, int group, int sms);
size_t attention_scratch_bytes(const AttnPlan& plan, int units, int group);
sa_status launch_attention(const AttnParams& p, cudaStream_t stream);
// One thread: gather_signal_wait (sa_device.cuh) after a standalone
// gathered attention; SA_DEV_TIMEOUT in *status when the wait gives up.
sa_status launch_gather_wait(void* const* peers, int world, size_t counter_bytes,
                             const unsigned long long* counter, unsigned long long* epoch,
                             unsigned long long per_epoch, uint32_t* status, cudaStream_t stream);

// ---- selection (sa_select.cu) ----------------------------------------------------

struct SelectParams {
  const float* query;  // [num_sl][qh][d]
  const float* reps;
  int64_t s_sl, s_head, s_block, s_dim;  // element strides of reps
  int qh, group, n_groups, d;
  int num_sl;
  const int32_t* nb;  // [num_sl] sealed blocks, null -> fixed_nb
  int fixed_nb;
  int nb_cap;         // capacity of scores rows and of reps along blocks
  int budget, init, local;
  int32_t* ids;       // [num_sl][n_groups][budget]
  int32_t* counts;    // [num_sl][n_groups] (nullable)
  float* scores;      // [num_sl][n_groups][nb_cap]
  int* counters;      // [num_sl][n_groups], zero between launches
  // Groups of more than four heads are split over CTAs, four heads each
  // (select_head_splits): each writes its heads' dot products to
  // head_dots [num_sl * n_groups][group][nb_cap] and the last of a chunk's
  // CTAs (chunk_counters [num_sl * n_groups][select_max_chunks], zero between
  // launches) adds them in head order.
  float* head_dots;
  int* chunk_counters;
  uint32_t* status;
  // Fused append (append_kv null = off): the first CTA of each unit writes
  // the step's K/V of the group's KV heads into row tail_len of the
  // sequence-layer's tail block and the group's queries into the query ring.
  // tail_len itself is left unchanged: the step's attention and seal count
  // the pending token (several units share one sequence-layer's tail).
  CtxDev append_ctx;
  const void* append_kv;  // [num_sl][2][kv_heads][128] FP16, or FP32 when append_kv_fp32
  int append_kv_fp32;
  // Raw projections (raw_k null = off): `query` holds pre-norm queries; every
  // CTA normalises and rotates its group's rows as it loads them, and the
  // first CTA of a unit writes them to raw_qt (for the attention) and the
  // query ring, and appends the normalised, rotated K (raw_k) and V (raw_v)
  // [num_sl][kv_heads][128] FP32 of its KV heads packed to FP16.
  const float* raw_k;
  const float* raw_v;
  const float* q_norm_w;   // [layers][128]
  const float* k_norm_w;   // [layers][128]
  const int32_t* positions;  // [num_sl / layers]
  float* raw_qt;           // [num_sl][qh][128]
  int layers;
  float rope_theta, norm_eps;
  int pdl;  // launched as a programmatic dependent of the previous kernel
};

// Streaming probes (sa_probe.cu): mode 0 per-lane cp.async, 1 bulk copies.
int probe_sink_words();
sa_status launch_probe_stream(const void* pool, long long pool_entries, const int32_t* ids,
                              long long n, int mode, unsigned long long* sink, uint32_t* status,
                              cudaStream_t stream);

int select_max_blocks();
// CTAs a unit's heads are split over (1 for groups of at most four heads),
// chunks of a unit of nb_cap blocks, and the scratch bytes of the split
// (head_dots, then chunk_counters; 0 when there is no split).
int select_head_splits(int group);
int select_max_chunks(int group, int nb_cap);
size_t select_split_scratch_bytes(int units, int group, int nb_cap);
void select_bind_split_scratch(SelectParams& p, void* scratch, int units);
sa_status launch_select(const SelectParams& p, cudaStream_t stream);

// ---- representatives, append, seal (sa_lifecycle.cu) ------------------------------

struct RepParams {
  // keys of token p: token-major kv + row_of(p) * row_stride + kv_head * d, or
  // (head_major) the K plane of block row_of(p) / 32, head kv_head, row p % 32
  const uint16_t* kv;
  int head_major;
  int64_t row_stride;       // elements between token rows
  const int32_t* table;     // null -> row_of(p) = p; else table[table_offset + p/32]*32 + p%32
  int table_offset;
  int kv_heads;
  // queries of head h, position p: q + (h * tokens + p) * d
  const float* q;
  int qh, d;
  int tokens;               // tokens of one call
  int blocks;               // tokens / 32
  int window, topk;
  float scale;              // 1/sqrt(d)
  // value of (head h, block b, dim j) at values + h*o_head + b*o_block + j*o_dim
  float* values;
  int64_t o_head, o_block, o_dim;
  int32_t* offsets;         // [qh][blocks][topk] (nullable)
  uint32_t* status;
};

sa_status launch_build_reps(const RepParams& p, cudaStream_t stream);
// Per-block variant: every block b of a range is its own 32-token call
// (queries q + (h * blocks * 32 + b * 32 + p) * d, i.e. [qh][blocks*32][d]).
sa_status launch_build_reps_per_block(const RepParams& p, cudaStream_t stream);


sa_status launch_append(const CtxDev& c, const float* query, const void* kv_new, int kv_fp32,
                        cudaStream_t stream);
// Rebuild the representative of every full tail and commit the seals.
// pending = tokens appended by a fused append and not yet in tail_len (the
// commit then stores every tail's new length).
sa_status launch_seal(const CtxDev& c, int pending, cudaStream_t stream, bool pdl = false);
// Dense attention mass per block of every (seq-layer, KV head), averaged
// over the KV head's query heads: mass [num_sl][kv_heads][table_blocks + 1],
// entry table_blocks = the open tail (sa_audit.cu).
sa_status launch_audit(const CtxDev& c, const float* query, float* mass, float scale,
                       cudaStream_t stream);
// History-prediction slot correction (sa_slots.cu); see sa_ctx_slot_correct.
sa_status launch_slot_correct(const int32_t* selected, const int32_t* counts, int32_t* slots,
                              int32_t* misses, int32_t* replace, int32_t* stats, int units,
                              int budget, int id_limit, uint32_t* status, cudaStream_t stream);
// Copy sealed blocks [first, first+count) of sequence-layer sl between the
// head-major pool and store rows [count][32][2][KH][128] (sa_lifecycle.cu).
sa_status launch_store_blocks(const CtxDev& c, int sl, int first, int count, void* store,
                              bool import, cudaStream_t stream);
sa_status launch_pack_kv(uint16_t* packed, const float* key, const float* value,
                         size_t token, size_t elements, cudaStream_t stream);
sa_status launch_xor(const uint8_t* in, uint8_t* out, size_t bytes, uint8_t mask,
                     cudaStream_t stream);
sa_status launch_consume(const float* out, int n, float* checksum, cudaStream_t stream);

}  // namespace sa
