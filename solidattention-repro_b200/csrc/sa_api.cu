// sa_api.cu -- implementation of the C ABI declared in include/sa_b200.h.
//
// Host-side runtime of the sparse-KV path: argument validation with the
// reference's error conditions, workspace plans,
// the AcceleratorBackend-style handle (host buffers, event timings) and the
// paged decode context (pool, free list, block tables, tails, seal).
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "sa_internal.h"

namespace sa {

namespace {
thread_local std::string g_last_error;
}

sa_status fail(sa_status status, const std::string& message) {
  g_last_error = message;
  return status;
}

sa_status cuda_status(cudaError_t err, const char* what) {
  if (err == cudaSuccess) return SA_OK;
  return fail(SA_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

namespace {

// Runs the caller's device choice on entry and restores it on exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&previous_) != cudaSuccess) previous_ = -1;
    if (device >= 0 && device != previous_) ok_ = cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (previous_ >= 0) cudaSetDevice(previous_);
  }
  bool ok() const { return ok_; }

 private:
  int previous_ = -1;
  bool ok_ = true;
};

}  // namespace

int device_sm_count() {
  static int cached[kMaxDevices];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    return 148;
  }
  if (cached[dev] <= 0) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        sms <= 0) {
      cudaGetLastError();
      return 148;
    }
    cached[dev] = sms;
  }
  return cached[dev];
}

sa_status ensure_smem_limit(const void* kernel, int bytes, int* configured_per_device) {
  int dev = 0;
  SA_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return fail(SA_ERR_UNSUPPORTED, "device index above 63");
  if (configured_per_device[dev] >= bytes) return SA_OK;
  SA_CUDA_TRY(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  configured_per_device[dev] = bytes;
  return SA_OK;
}

}  // namespace sa

using namespace sa;

// =============================================================== status

struct sa_backend {
  int device = 0;
  cudaStream_t stream = nullptr;
  cudaEvent_t ev[5] = {};
  void* d_kv = nullptr;
  size_t kv_cap = 0;
  float* d_q = nullptr;
  size_t q_cap = 0;
  float* d_out = nullptr;
  size_t out_cap = 0;
  float* d_checksum = nullptr;
  void* d_ws = nullptr;
  size_t ws_cap = 0;
  uint8_t* d_io = nullptr;
  size_t io_cap = 0;
  void* d_buf[6] = {};     // selection / representative staging
  size_t buf_cap[6] = {};
};

struct sa_ctx {
  sa_ctx_config cfg{};
  int num_sl = 0, group = 0, n_sel_groups = 0, table_pad = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  CtxDev dev{};
  int32_t* selected = nullptr;
  int32_t* selected_count = nullptr;
  float* scores = nullptr;
  int* select_counters = nullptr;
  char* select_split = nullptr;  // head-split scratch of groups above four heads
  size_t select_split_bytes = 0;
  float* attn_partial = nullptr;
  int* attn_counters = nullptr;
  AttnPlan attn_plan{};
  // staging for sa_ctx_step_host
  float* d_query = nullptr;
  float* d_qt = nullptr;  // normalised, rotated queries of sa_ctx_step_raw
  void* d_kv_new = nullptr;
  void* d_out = nullptr;
  uint32_t* h_status = nullptr;  // pinned
  uint32_t* h_status_dev = nullptr;  // its device-side address
  std::vector<uint8_t> prefilled;
  uint64_t launches = 0;
  // KV-head-sharded gather over peer memory: two parity slots of
  // [seqs*layers][world * QH][D] outputs, then a 64-bit arrival counter
  uint8_t* gather_buf = nullptr;
  size_t gather_slot_bytes = 0, gather_counter_bytes = 0, gather_bytes = 0;
  int gather_world = 0, gather_rank = -1;
  void** gather_peers = nullptr;  // device array [gather_world]
  uint64_t gather_attends = 0;
  uint64_t gather_waited = 0;  // gathered attends whose wait has been enqueued
  // decode-step graph: recorded between sa_ctx_graph_begin and _end
  bool recording = false;
  uint64_t launches_before_recording = 0;
  uint64_t gather_attends_before_recording = 0;
  uint64_t gather_waited_before_recording = 0;
  bool gather_view_recorded = false;  // a gathered-slot view was handed out while recording
  uint64_t graph_launches = 0;        // kernel launches one replay issues
  uint64_t graph_gather_attends = 0;  // gathered attends one replay issues
  uint64_t graph_gather_waited = 0;   // and the waits it enqueues
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  // sa_ctx_step_host with pinned buffers: the query copy and the step's three
  // launches recorded once and replayed while the call's buffers stay the same
  const void* host_step_key[4] = {nullptr, nullptr, nullptr, nullptr};
  int host_step_kv_fp32 = -1;
  uint64_t host_step_launches = 0;
  cudaGraph_t host_step_graph = nullptr;
  cudaGraphExec_t host_step_exec = nullptr;
};

namespace {
// Calls that synchronise or copy through host memory cannot be recorded into
// a graph; they are refused while a recording is open.
sa_status refuse_while_recording(const char* what) {
  return fail(SA_ERR_INVALID_ARG, std::string(what) + ": not allowed while a graph is being recorded");
}
}  // namespace

extern "C" {

SA_API const char* sa_status_string(sa_status status) {
  switch (status) {
    case SA_OK: return "ok";
    case SA_ERR_INVALID_ARG: return "invalid argument";
    case SA_ERR_UNSUPPORTED: return "unsupported";
    case SA_ERR_CAPACITY: return "capacity exceeded";
    case SA_ERR_CUDA: return "CUDA error";
    case SA_ERR_DEVICE: return "device status error";
    case SA_ERR_TIMEOUT: return "device wait timed out";
    case SA_ERR_NO_MEMORY: return "out of memory";
    default: return "unknown status";
  }
}

SA_API const char* sa_last_error(void) { return g_last_error.c_str(); }

SA_API const char* sa_version(void) { return "sa_b200 0.1 sm_100a"; }

// ===================================================== stateless kernels

SA_API size_t sa_attention_workspace_size(size_t tokens, size_t query_heads, size_t kv_heads) {
  if (kv_heads == 0 || query_heads % kv_heads != 0) return 0;
  if (tokens > 0xffffffffull) return 0;  // beyond what sa_attention_packed accepts
  const int entries = (int)((tokens + kBlockTokens - 1) / kBlockTokens);
  const int units = (int)kv_heads;
  const int group = (int)(query_heads / kv_heads);
  const AttnPlan plan = attention_plan(units, std::max(entries, 1), group, device_sm_count());
  return attention_scratch_bytes(plan, units, group) + (size_t)units * sizeof(int) + 256;
}

SA_API sa_status sa_attention_packed(const uint16_t* kv, const float* query, size_t tokens,
                                     size_t query_heads, size_t kv_heads, size_t head_dim,
                                     float scale, void* out, int out_fp16, void* workspace,
                                     size_t workspace_bytes, void* stream) {
  if (!kv || !query || !out) return fail(SA_ERR_INVALID_ARG, "attention: null pointer");
  if (kv_heads == 0 || query_heads % kv_heads != 0 || tokens == 0)
    return fail(SA_ERR_INVALID_ARG, "invalid GQA attention dimensions");
  if (head_dim != (size_t)kHeadDim) return fail(SA_ERR_UNSUPPORTED, "attention: head_dim must be 128");
  const size_t need = sa_attention_workspace_size(tokens, query_heads, kv_heads);
  if (!workspace || workspace_bytes < need)
    return fail(SA_ERR_CAPACITY, "attention: workspace smaller than sa_attention_workspace_size()");
  if (tokens > 0xffffffffull) return fail(SA_ERR_UNSUPPORTED, "attention: too many tokens");
  if ((reinterpret_cast<uintptr_t>(kv) & 15u) != 0)
    return fail(SA_ERR_INVALID_ARG, "KV buffer must be 16-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int entries = (int)((tokens + kBlockTokens - 1) / kBlockTokens);
  const int units = (int)kv_heads;
  AttnParams p{};
  p.pool = nullptr;
  p.head_major = 0;
  p.rows = kv;
  p.row_bytes = (int64_t)(2 * kv_heads * kHeadDim * sizeof(uint16_t));
  p.kv_heads = (int)kv_heads;
  p.group = (int)(query_heads / kv_heads);
  p.num_sl = 1;
  p.pool_blocks = entries;
  p.sel_ids = nullptr;
  p.sel_count = nullptr;
  p.sel_stride = entries;
  p.n_sel_groups = 1;
  p.kv_per_sel_group = (int)kv_heads;
  p.fixed_nsel = (int)(tokens / kBlockTokens);
  p.table = nullptr;
  p.table_stride = entries;
  p.tail_block = nullptr;
  p.tail_len = nullptr;
  p.fixed_tail_block = (int)(tokens / kBlockTokens);
  p.fixed_tail_len = (int)(tokens % kBlockTokens);
  p.query = query;
  p.out = out;
  p.out_fp16 = out_fp16;
  p.scale_log2 = scale * 1.4426950408889634f;
  const AttnPlan plan = attention_plan(units, entries, p.group, device_sm_count());
  p.slots_per_unit = plan.slots_per_unit;
  p.max_segments = plan.max_segments;
  p.ctas = plan.ctas;
  char* ws = static_cast<char*>(workspace);
  const size_t partial_bytes = attention_scratch_bytes(plan, units, p.group);
  p.partial = reinterpret_cast<float*>(ws);
  p.counters = reinterpret_cast<int*>(ws + ((partial_bytes + 255) & ~size_t(255)));
  p.status = nullptr;
  SA_CUDA_TRY(cudaMemsetAsync(p.counters, 0, (size_t)units * sizeof(int), s));
  return launch_attention(p, s);
}

SA_API size_t sa_select_workspace_size(size_t query_heads, size_t group, size_t blocks) {
  if (group == 0 || query_heads % group != 0) return 0;
  const size_t n_groups = query_heads / group;
  const size_t cap = (blocks + 3) & ~size_t(3);
  const size_t base = (n_groups * cap * sizeof(float) + n_groups * sizeof(int) + 255) & ~size_t(255);
  return base + select_split_scratch_bytes((int)n_groups, (int)group, (int)cap) + 256;
}

SA_API sa_status sa_select_blocks(const float* query, const float* reps, int64_t stride_head,
                                  int64_t stride_block, int64_t stride_dim, size_t query_heads,
                                  size_t group, size_t blocks, size_t head_dim,
                                  size_t budget_blocks, size_t init_blocks, size_t local_blocks,
                                  int32_t* block_ids_out, float* scores_out, void* workspace,
                                  size_t workspace_bytes, void* stream) {
  // The reference's own validation (cpp/src/selection.cpp:99-105).
  if (!query || !reps || query_heads == 0 || blocks == 0 || head_dim == 0 || budget_blocks == 0 ||
      budget_blocks > blocks || init_blocks + local_blocks > budget_blocks)
    return fail(SA_ERR_INVALID_ARG, "invalid representative selection dimensions");
  if (group == 0 || query_heads % group != 0)
    return fail(SA_ERR_INVALID_ARG, "select: group must divide query_heads");
  if (!block_ids_out) return fail(SA_ERR_INVALID_ARG, "select: null block_ids_out");
  if (blocks > (size_t)select_max_blocks())
    return fail(SA_ERR_UNSUPPORTED, "select: more than 16384 blocks");
  const size_t need = sa_select_workspace_size(query_heads, group, blocks);
  if (!workspace || workspace_bytes < need)
    return fail(SA_ERR_CAPACITY, "select: workspace smaller than sa_select_workspace_size()");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t n_groups = query_heads / group;
  const int cap = (int)((blocks + 3) & ~size_t(3));
  SelectParams p{};
  p.query = query;
  p.reps = reps;
  p.s_sl = 0;
  p.s_head = stride_head;
  p.s_block = stride_block;
  p.s_dim = stride_dim;
  p.qh = (int)query_heads;
  p.group = (int)group;
  p.n_groups = (int)n_groups;
  p.d = (int)head_dim;
  p.num_sl = 1;
  p.nb = nullptr;
  p.fixed_nb = (int)blocks;
  p.budget = (int)budget_blocks;
  p.init = (int)init_blocks;
  p.local = (int)local_blocks;
  p.ids = block_ids_out;
  p.counts = nullptr;
  char* ws = static_cast<char*>(workspace);
  p.scores = reinterpret_cast<float*>(ws);
  p.counters = reinterpret_cast<int*>(ws + n_groups * cap * sizeof(float));
  p.status = nullptr;
  // A caller's reps extent along blocks is `blocks`: keep vector loads inside it.
  p.nb_cap = (stride_block == 1 && blocks % 4 != 0) ? (int)blocks : cap;
  SA_CUDA_TRY(cudaMemsetAsync(p.counters, 0, n_groups * sizeof(int), s));
  // groups of more than four heads: the head split's dots and chunk counters
  const size_t base = (n_groups * cap * sizeof(float) + n_groups * sizeof(int) + 255) & ~size_t(255);
  select_bind_split_scratch(p, ws + base, (int)n_groups);
  if (p.chunk_counters)
    SA_CUDA_TRY(cudaMemsetAsync(p.chunk_counters, 0,
                                n_groups * select_max_chunks(p.group, p.nb_cap) * sizeof(int), s));
  const int row = p.nb_cap;
  sa_status st = launch_select(p, s);
  if (st != SA_OK) return st;
  if (scores_out)
    SA_CUDA_TRY(cudaMemcpy2DAsync(scores_out, blocks * sizeof(float), p.scores,
                                  (size_t)row * sizeof(float), blocks * sizeof(float), n_groups,
                                  cudaMemcpyDeviceToDevice, s));
  return SA_OK;
}

SA_API sa_status sa_build_representatives(const float* prompt_queries, const uint16_t* kv,
                                          size_t tokens, size_t query_heads, size_t kv_heads,
                                          size_t head_dim, size_t block_tokens,
                                          size_t local_window, size_t topk, float* values_out,
                                          int32_t* offsets_out, void* stream) {
  // The reference's own validation (cpp/src/selection.cpp:17-22).
  if (!prompt_queries || !kv || tokens == 0 || kv_heads == 0 || query_heads % kv_heads != 0 ||
      block_tokens == 0 || tokens % block_tokens != 0 || local_window == 0 || topk == 0 ||
      topk > block_tokens)
    return fail(SA_ERR_INVALID_ARG, "invalid local-causal representative dimensions");
  if (block_tokens != (size_t)kBlockTokens)
    return fail(SA_ERR_UNSUPPORTED, "representatives: block_tokens must be 32");
  if (!values_out) return fail(SA_ERR_INVALID_ARG, "representatives: null values_out");
  RepParams p{};
  p.kv = kv;
  p.head_major = 0;
  p.row_stride = (int64_t)(2 * kv_heads * head_dim);
  p.table = nullptr;
  p.table_offset = 0;
  p.kv_heads = (int)kv_heads;
  p.q = prompt_queries;
  p.qh = (int)query_heads;
  p.d = (int)head_dim;
  p.tokens = (int)tokens;
  p.blocks = (int)(tokens / block_tokens);
  p.window = (int)local_window;
  p.topk = (int)topk;
  p.scale = 1.0f / std::sqrt((float)head_dim);
  p.values = values_out;
  p.o_head = (int64_t)p.blocks * head_dim;
  p.o_block = (int64_t)head_dim;
  p.o_dim = 1;
  p.offsets = offsets_out;
  p.status = nullptr;
  return launch_build_reps(p, static_cast<cudaStream_t>(stream));
}

SA_API sa_status sa_pack_kv_fp16(uint16_t* packed, const float* key, const float* value,
                                 size_t token, size_t elements, void* stream) {
  if (!packed || !key || !value) return fail(SA_ERR_INVALID_ARG, "pack: null pointer");
  return launch_pack_kv(packed, key, value, token, elements, static_cast<cudaStream_t>(stream));
}

// ========================================================= backend handle

SA_API sa_status sa_backend_create(int device, sa_backend** out) {
  if (!out) return fail(SA_ERR_INVALID_ARG, "backend: null out");
  *out = nullptr;
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(SA_ERR_CUDA, "backend: cudaSetDevice failed");
  auto* b = new (std::nothrow) sa_backend();
  if (!b) return fail(SA_ERR_NO_MEMORY, "backend: allocation failed");
  b->device = device;
  sa_status st = cuda_status(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking),
                             "cudaStreamCreateWithFlags");
  for (int i = 0; st == SA_OK && i < 5; ++i) st = cuda_status(cudaEventCreate(&b->ev[i]), "cudaEventCreate");
  if (st == SA_OK) st = cuda_status(cudaMalloc(&b->d_checksum, sizeof(float)), "cudaMalloc checksum");
  if (st != SA_OK) {
    sa_backend_destroy(b);
    return st;
  }
  *out = b;
  return SA_OK;
}

SA_API sa_status sa_backend_destroy(sa_backend* b) {
  if (!b) return SA_OK;
  DeviceGuard guard(b->device);
  if (b->stream) cudaStreamSynchronize(b->stream);
  cudaFree(b->d_kv);
  cudaFree(b->d_q);
  cudaFree(b->d_out);
  cudaFree(b->d_checksum);
  cudaFree(b->d_ws);
  cudaFree(b->d_io);
  for (void* p : b->d_buf) cudaFree(p);
  for (auto& e : b->ev)
    if (e) cudaEventDestroy(e);
  if (b->stream) cudaStreamDestroy(b->stream);
  delete b;
  return SA_OK;
}

SA_API const char* sa_backend_name(const sa_backend*) { return "b200-sm100a"; }

SA_API sa_status sa_backend_host_alloc(sa_backend* b, size_t bytes, void** out) {
  if (!b || !out) return fail(SA_ERR_INVALID_ARG, "host_alloc: null argument");
  DeviceGuard guard(b->device);
  return cuda_status(cudaHostAlloc(out, bytes, cudaHostAllocDefault), "cudaHostAlloc");
}

SA_API sa_status sa_backend_host_free(sa_backend* b, void* pointer) {
  if (!b) return fail(SA_ERR_INVALID_ARG, "host_free: null backend");
  return cuda_status(cudaFreeHost(pointer), "cudaFreeHost");
}

}  // extern "C"

namespace {
sa_status grow(void** ptr, size_t* cap, size_t bytes) {
  if (bytes <= *cap) return SA_OK;
  cudaFree(*ptr);
  *ptr = nullptr;
  *cap = 0;
  SA_CUDA_TRY(cudaMalloc(ptr, bytes));
  *cap = bytes;
  return SA_OK;
}
}  // namespace

extern "C" {

SA_API sa_status sa_backend_attention(sa_backend* b, const uint16_t* kv_host,
                                      const float* query_host, size_t tokens, size_t query_heads,
                                      size_t kv_heads, size_t head_dim, float scale, int flags,
                                      float* out_host, sa_timings* timings) {
  if (!b || !kv_host || !query_host) return fail(SA_ERR_INVALID_ARG, "backend attention: null pointer");
  if (kv_heads == 0 || query_heads % kv_heads != 0 || tokens == 0)
    return fail(SA_ERR_INVALID_ARG, "invalid GQA attention dimensions");
  if (head_dim != (size_t)kHeadDim) return fail(SA_ERR_UNSUPPORTED, "attention: head_dim must be 128");
  if ((flags & SA_ATTN_COPY_OUTPUT) && !out_host)
    return fail(SA_ERR_INVALID_ARG, "backend attention: null out_host");
  DeviceGuard guard(b->device);
  const size_t kv_bytes = tokens * 2 * kv_heads * head_dim * sizeof(uint16_t);
  const size_t q_bytes = query_heads * head_dim * sizeof(float);
  const size_t ws_bytes = sa_attention_workspace_size(tokens, query_heads, kv_heads);
  sa_status st;
  if ((st = grow(&b->d_kv, &b->kv_cap, kv_bytes)) != SA_OK) return st;
  if ((st = grow(reinterpret_cast<void**>(&b->d_q), &b->q_cap, q_bytes)) != SA_OK) return st;
  if ((st = grow(reinterpret_cast<void**>(&b->d_out), &b->out_cap, q_bytes)) != SA_OK) return st;
  if ((st = grow(&b->d_ws, &b->ws_cap, ws_bytes)) != SA_OK) return st;
  SA_CUDA_TRY(cudaEventRecord(b->ev[0], b->stream));
  SA_CUDA_TRY(cudaMemcpyAsync(b->d_kv, kv_host, kv_bytes, cudaMemcpyHostToDevice, b->stream));
  SA_CUDA_TRY(cudaMemcpyAsync(b->d_q, query_host, q_bytes, cudaMemcpyHostToDevice, b->stream));
  SA_CUDA_TRY(cudaEventRecord(b->ev[1], b->stream));
  st = sa_attention_packed(static_cast<const uint16_t*>(b->d_kv), b->d_q, tokens, query_heads,
                           kv_heads, head_dim, scale, b->d_out, 0, b->d_ws, b->ws_cap, b->stream);
  if (st != SA_OK) return st;
  SA_CUDA_TRY(cudaEventRecord(b->ev[2], b->stream));
  const bool consume = (flags & SA_ATTN_CONSUME) != 0;
  if (consume) {
    if ((st = launch_consume(b->d_out, (int)(query_heads * head_dim), b->d_checksum, b->stream)) != SA_OK)
      return st;
  }
  SA_CUDA_TRY(cudaEventRecord(b->ev[3], b->stream));
  if (flags & SA_ATTN_COPY_OUTPUT) {
    SA_CUDA_TRY(cudaMemcpyAsync(out_host, consume ? b->d_checksum : b->d_out,
                                consume ? sizeof(float) : q_bytes, cudaMemcpyDeviceToHost,
                                b->stream));
  }
  SA_CUDA_TRY(cudaEventRecord(b->ev[4], b->stream));
  SA_CUDA_TRY(cudaEventSynchronize(b->ev[4]));
  if (timings) {
    float ms[4] = {0, 0, 0, 0};
    for (int i = 0; i < 4; ++i) cudaEventElapsedTime(&ms[i], b->ev[i], b->ev[i + 1]);
    timings->h2d_ms = ms[0];
    timings->kernel_ms = ms[1];
    timings->consumer_ms = ms[2];
    timings->d2h_ms = ms[3];
  }
  return SA_OK;
}

SA_API sa_status sa_backend_select(sa_backend* b, const float* query_host, const float* reps_host,
                                   size_t query_heads, size_t blocks, size_t head_dim,
                                   size_t budget_blocks, size_t init_blocks, size_t local_blocks,
                                   int64_t* ids_out_host, float* scores_out_host) {
  if (!b) return fail(SA_ERR_INVALID_ARG, "backend select: null backend");
  // The reference's own validation (cpp/src/selection.cpp:99-105).
  if (!query_host || !reps_host || query_heads == 0 || blocks == 0 || head_dim == 0 ||
      budget_blocks == 0 || budget_blocks > blocks || init_blocks + local_blocks > budget_blocks)
    return fail(SA_ERR_INVALID_ARG, "invalid representative selection dimensions");
  if (!ids_out_host) return fail(SA_ERR_INVALID_ARG, "backend select: null ids_out_host");
  DeviceGuard guard(b->device);
  const size_t q_bytes = query_heads * head_dim * sizeof(float);
  const size_t r_bytes = query_heads * blocks * head_dim * sizeof(float);
  const size_t ws_bytes = sa_select_workspace_size(query_heads, query_heads, blocks);
  const size_t sizes[5] = {q_bytes, r_bytes, budget_blocks * 4, blocks * 4, ws_bytes};
  for (int i = 0; i < 5; ++i) {
    const sa_status st = grow(&b->d_buf[i], &b->buf_cap[i], sizes[i]);
    if (st != SA_OK) return st;
  }
  SA_CUDA_TRY(cudaMemcpyAsync(b->d_buf[0], query_host, q_bytes, cudaMemcpyHostToDevice, b->stream));
  SA_CUDA_TRY(cudaMemcpyAsync(b->d_buf[1], reps_host, r_bytes, cudaMemcpyHostToDevice, b->stream));
  const sa_status st = sa_select_blocks(
      static_cast<const float*>(b->d_buf[0]), static_cast<const float*>(b->d_buf[1]),
      (int64_t)(blocks * head_dim), (int64_t)head_dim, 1, query_heads, query_heads, blocks, head_dim,
      budget_blocks, init_blocks, local_blocks, static_cast<int32_t*>(b->d_buf[2]),
      static_cast<float*>(b->d_buf[3]), b->d_buf[4], b->buf_cap[4], b->stream);
  if (st != SA_OK) return st;
  std::vector<int32_t> ids(budget_blocks);
  SA_CUDA_TRY(cudaMemcpyAsync(ids.data(), b->d_buf[2], budget_blocks * 4, cudaMemcpyDeviceToHost,
                              b->stream));
  if (scores_out_host)
    SA_CUDA_TRY(cudaMemcpyAsync(scores_out_host, b->d_buf[3], blocks * 4, cudaMemcpyDeviceToHost,
                                b->stream));
  SA_CUDA_TRY(cudaStreamSynchronize(b->stream));
  for (size_t i = 0; i < budget_blocks; ++i) ids_out_host[i] = ids[i];
  return SA_OK;
}

SA_API sa_status sa_backend_build_representatives(sa_backend* b, const float* prompt_queries_host,
                                                  const uint16_t* kv_host, size_t tokens,
                                                  size_t query_heads, size_t kv_heads,
                                                  size_t head_dim, size_t block_tokens,
                                                  size_t local_window, size_t topk,
                                                  float* values_out_host,
                                                  int64_t* offsets_out_host) {
  if (!b) return fail(SA_ERR_INVALID_ARG, "backend representatives: null backend");
  // The reference's own validation (cpp/src/selection.cpp:17-22).
  if (!prompt_queries_host || !kv_host || tokens == 0 || kv_heads == 0 ||
      query_heads % kv_heads != 0 || block_tokens == 0 || tokens % block_tokens != 0 ||
      local_window == 0 || topk == 0 || topk > block_tokens)
    return fail(SA_ERR_INVALID_ARG, "invalid local-causal representative dimensions");
  if (!values_out_host) return fail(SA_ERR_INVALID_ARG, "backend representatives: null values_out");
  DeviceGuard guard(b->device);
  const size_t blocks = tokens / block_tokens;
  const size_t q_bytes = query_heads * tokens * head_dim * sizeof(float);
  const size_t kv_bytes = tokens * 2 * kv_heads * head_dim * sizeof(uint16_t);
  const size_t v_bytes = query_heads * blocks * head_dim * sizeof(float);
  const size_t o_bytes = query_heads * blocks * topk * sizeof(int32_t);
  const size_t sizes[4] = {q_bytes, kv_bytes, v_bytes, o_bytes};
  for (int i = 0; i < 4; ++i) {
    const sa_status st = grow(&b->d_buf[i], &b->buf_cap[i], sizes[i]);
    if (st != SA_OK) return st;
  }
  SA_CUDA_TRY(cudaMemcpyAsync(b->d_buf[0], prompt_queries_host, q_bytes, cudaMemcpyHostToDevice,
                              b->stream));
  SA_CUDA_TRY(cudaMemcpyAsync(b->d_buf[1], kv_host, kv_bytes, cudaMemcpyHostToDevice, b->stream));
  const sa_status st = sa_build_representatives(
      static_cast<const float*>(b->d_buf[0]), static_cast<const uint16_t*>(b->d_buf[1]), tokens,
      query_heads, kv_heads, head_dim, block_tokens, local_window, topk,
      static_cast<float*>(b->d_buf[2]), static_cast<int32_t*>(b->d_buf[3]), b->stream);
  if (st != SA_OK) return st;
  std::vector<int32_t> offsets(query_heads * blocks * topk);
  SA_CUDA_TRY(cudaMemcpyAsync(values_out_host, b->d_buf[2], v_bytes, cudaMemcpyDeviceToHost,
                              b->stream));
  SA_CUDA_TRY(cudaMemcpyAsync(offsets.data(), b->d_buf[3], o_bytes, cudaMemcpyDeviceToHost,
                              b->stream));
  SA_CUDA_TRY(cudaStreamSynchronize(b->stream));
  if (offsets_out_host)
    for (size_t i = 0; i < offsets.size(); ++i) offsets_out_host[i] = offsets[i];
  return SA_OK;
}

SA_API sa_status sa_backend_execute(sa_backend* b, void* pinned_input, size_t bytes, uint8_t mask,
                                    sa_timings* timings, uint64_t* checksum_out) {
  if (!b || (!pinned_input && bytes)) return fail(SA_ERR_INVALID_ARG, "execute: null argument");
  DeviceGuard guard(b->device);
  sa_status st;
  if ((st = grow(reinterpret_cast<void**>(&b->d_io), &b->io_cap, 2 * std::max<size_t>(bytes, 1))) != SA_OK)
    return st;
  std::vector<uint8_t> output(bytes);
  uint8_t* d_in = b->d_io;
  uint8_t* d_out = b->d_io + bytes;
  SA_CUDA_TRY(cudaEventRecord(b->ev[0], b->stream));
  SA_CUDA_TRY(cudaMemcpyAsync(d_in, pinned_input, bytes, cudaMemcpyHostToDevice, b->stream));
  SA_CUDA_TRY(cudaEventRecord(b->ev[1], b->stream));
  if ((st = launch_xor(d_in, d_out, bytes, mask, b->stream)) != SA_OK) return st;
  SA_CUDA_TRY(cudaEventRecord(b->ev[2], b->stream));
  SA_CUDA_TRY(cudaMemcpyAsync(output.data(), d_out, bytes, cudaMemcpyDeviceToHost, b->stream));
  SA_CUDA_TRY(cudaEventRecord(b->ev[3], b->stream));
  SA_CUDA_TRY(cudaEventSynchronize(b->ev[3]));
  float ms[3] = {0, 0, 0};
  for (int i = 0; i < 3; ++i) cudaEventElapsedTime(&ms[i], b->ev[i], b->ev[i + 1]);
  if (timings) {
    timings->h2d_ms = ms[0];
    timings->kernel_ms = ms[1];
    timings->consumer_ms = 0;
    timings->d2h_ms = ms[2];
  }
  uint64_t sum = 0;
  for (const uint8_t v : output) sum += v;
  if (checksum_out) *checksum_out = sum;
  return SA_OK;
}

}  // extern "C"

// ================================================== paged decode context

namespace {

sa_status validate_config(const sa_ctx_config& c) {
  if (c.head_dim != kHeadDim) return fail(SA_ERR_UNSUPPORTED, "ctx: head_dim must be 128");
  if (c.query_heads <= 0 || c.kv_heads <= 0 || c.query_heads % c.kv_heads != 0)
    return fail(SA_ERR_INVALID_ARG, "ctx: query_heads must be a positive multiple of kv_heads");
  const int g = c.query_heads / c.kv_heads;
  if (g != 1 && g != 2 && g != 4 && g != 8)
    return fail(SA_ERR_UNSUPPORTED, "ctx: query heads per KV head must be 1, 2, 4 or 8");
  if (c.layers <= 0 || c.seqs <= 0) return fail(SA_ERR_INVALID_ARG, "ctx: layers and seqs must be positive");
  if (c.pool_blocks <= 0 || c.table_blocks <= 0)
    return fail(SA_ERR_INVALID_ARG, "ctx: pool_blocks and table_blocks must be positive");
  if ((int64_t)c.pool_blocks * kBlockTokens > 0x7fffffffLL)
    return fail(SA_ERR_UNSUPPORTED, "ctx: pool too large for 32-bit rows");
  if (c.budget_blocks <= 0 || c.init_blocks < 0 || c.local_blocks < 0 ||
      c.init_blocks + c.local_blocks > c.budget_blocks)
    return fail(SA_ERR_INVALID_ARG, "ctx: need budget >= init + local >= 0");
  if (c.select_group <= 0 || c.query_heads % c.select_group != 0 || c.select_group % g != 0)
    return fail(SA_ERR_INVALID_ARG,
                "ctx: select_group must divide query_heads and be a multiple of query_heads/kv_heads");
  if (c.table_blocks > select_max_blocks())
    return fail(SA_ERR_UNSUPPORTED, "ctx: table_blocks above 16384");
  if (c.rep_window <= 0 || c.rep_window > 64 || c.rep_topk <= 0 || c.rep_topk > kBlockTokens)
    return fail(SA_ERR_UNSUPPORTED, "ctx: rep_window must be 1..64 and rep_topk 1..32");
  if (!(c.scale > 0.f) || !std::isfinite(c.scale)) return fail(SA_ERR_INVALID_ARG, "ctx: bad scale");
  return SA_OK;
}

template <class T>
sa_status dalloc(T** p, size_t count) {
  *p = nullptr;
  if (count == 0) count = 1;
  const cudaError_t e = cudaMalloc(reinterpret_cast<void**>(p), count * sizeof(T));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(SA_ERR_NO_MEMORY, std::string("ctx: cudaMalloc failed: ") + cudaGetErrorString(e));
  }
  return SA_OK;
}

// kv_new non-null: the select kernel also appends the step's token (fused).
SelectParams select_params(sa_ctx* c, const float* query) {
  SelectParams p{};
  p.query = query;
  p.reps = c->dev.reps;
  p.s_dim = c->table_pad;
  p.s_block = 1;
  p.s_head = (int64_t)kHeadDim * c->table_pad;
  p.s_sl = (int64_t)c->cfg.query_heads * p.s_head;
  p.qh = c->cfg.query_heads;
  p.group = c->cfg.select_group;
  p.n_groups = c->n_sel_groups;
  p.d = kHeadDim;
  p.num_sl = c->num_sl;
  p.nb = c->dev.num_sealed;
  p.fixed_nb = 0;
  p.nb_cap = c->table_pad;
  p.budget = c->cfg.budget_blocks;
  p.init = c->cfg.init_blocks;
  p.local = c->cfg.local_blocks;
  p.ids = c->selected;
  p.counts = c->selected_count;
  p.scores = c->scores;
  p.counters = c->select_counters;
  p.status = c->dev.status;
  select_bind_split_scratch(p, c->select_split, c->num_sl * c->n_sel_groups);
  return p;
}

sa_status ctx_select(sa_ctx* c, const float* query, const void* kv_new = nullptr,
                     int kv_fp32 = 0, bool pdl = false) {
  SelectParams p = select_params(c, query);
  p.pdl = pdl;
  if (kv_new) {
    p.append_ctx = c->dev;
    p.append_kv = kv_new;
    p.append_kv_fp32 = kv_fp32;
  }
  ++c->launches;
  return launch_select(p, c->stream);
}

// pending: tokens appended by a fused append this step, not yet in tail_len.
// step_gather: the decode step's seal kernel signals the gather for the
// whole grid (else every unit counts its own arrivals).
sa_status ctx_attend(sa_ctx* c, const float* query, void* out, int pending = 0,
                     bool pdl = false, bool step_gather = false) {
  AttnParams p{};
  p.tail_pending = pending;
  p.pdl = pdl;
  p.pool = c->dev.pool;
  p.head_major = 1;
  p.kv_heads = c->cfg.kv_heads;
  p.group = c->group;
  p.num_sl = c->num_sl;
  p.pool_blocks = c->cfg.pool_blocks;
  p.sel_ids = c->selected;
  p.sel_count = c->selected_count;
  p.sel_stride = c->cfg.budget_blocks;
  p.n_sel_groups = c->n_sel_groups;
  p.kv_per_sel_group = c->cfg.select_group / c->group;
  p.fixed_nsel = 0;
  p.table = c->dev.table;
  p.table_stride = c->cfg.table_blocks;
  p.tail_block = c->dev.tail_block;
  p.tail_len = c->dev.tail_len;
  p.query = query;
  p.out = out;
  p.out_fp16 = c->cfg.out_fp16;
  p.scale_log2 = c->cfg.scale * 1.4426950408889634f;
  p.slots_per_unit = c->attn_plan.slots_per_unit;
  p.max_segments = c->attn_plan.max_segments;
  p.ctas = c->attn_plan.ctas;
  p.partial = c->attn_partial;
  p.counters = c->attn_counters;
  p.status = c->dev.status;
  if (c->gather_peers) {
    p.gather_peers = c->gather_peers;
    p.gather_world = c->gather_world;
    p.gather_rank = c->gather_rank;
    p.gather_slot_bytes = c->gather_slot_bytes;
    p.gather_counter_bytes = c->gather_counter_bytes;
    p.gather_epoch = reinterpret_cast<const unsigned long long*>(c->gather_buf +
                                                                 c->gather_counter_bytes + 8);
    p.gather_unit_arrivals = step_gather ? 0 : 1;
  }
  ++c->launches;
  const sa_status st = launch_attention(p, c->stream);
  if (st == SA_OK && c->gather_peers) ++c->gather_attends;
  return st;
}

}  // namespace

extern "C" {

SA_API sa_status sa_ctx_create(const sa_ctx_config* config, sa_ctx** out) {
  if (!config || !out) return fail(SA_ERR_INVALID_ARG, "ctx: null argument");
  *out = nullptr;
  sa_status st = validate_config(*config);
  if (st != SA_OK) return st;
  DeviceGuard guard(config->device);
  if (!guard.ok()) return fail(SA_ERR_CUDA, "ctx: cudaSetDevice failed");
  auto* c = new (std::nothrow) sa_ctx();
  if (!c) return fail(SA_ERR_NO_MEMORY, "ctx: allocation failed");
  c->cfg = *config;
  const auto& g = c->cfg;
  c->num_sl = g.seqs * g.layers;
  c->group = g.query_heads / g.kv_heads;
  c->n_sel_groups = g.query_heads / g.select_group;
  c->table_pad = (g.table_blocks + 3) & ~3;
  c->prefilled.assign(c->num_sl, 0);
  const size_t nsl = c->num_sl;
  const int64_t row_elems = 2LL * g.kv_heads * kHeadDim;
  CtxDev& d = c->dev;
  d.row_elems = row_elems;
  d.pool_blocks = g.pool_blocks;
  d.table_blocks = g.table_blocks;
  d.reps_cap = c->table_pad;
  d.num_sl = c->num_sl;
  d.qh = g.query_heads;
  d.kv_heads = g.kv_heads;
  d.rep_window = g.rep_window;
  d.rep_topk = g.rep_topk;
  d.rep_scale = 1.0f / std::sqrt((float)kHeadDim);
  const int units = c->num_sl * g.kv_heads;
  c->attn_plan = attention_plan(units, g.budget_blocks + 1, c->group, device_sm_count());

  st = cuda_status(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate");
  c->own_stream = st == SA_OK;
  // d.table_blocks is the table row stride; reps use the padded capacity.
  if (st == SA_OK) st = dalloc(&d.pool, (size_t)g.pool_blocks * kBlockTokens * row_elems);
  if (st == SA_OK) st = dalloc(&d.reps, nsl * g.query_heads * kHeadDim * (size_t)c->table_pad);
  if (st == SA_OK) st = dalloc(&d.table, nsl * g.table_blocks);
  if (st == SA_OK) st = dalloc(&d.num_sealed, nsl);
  if (st == SA_OK) st = dalloc(&d.tail_block, nsl);
  if (st == SA_OK) st = dalloc(&d.tail_len, nsl);
  if (st == SA_OK) st = dalloc(&d.generation, nsl);
  if (st == SA_OK) st = dalloc(&d.query_ring, nsl * g.query_heads * kBlockTokens * kHeadDim);
  if (st == SA_OK) st = dalloc(&d.free_list, (size_t)g.pool_blocks);
  if (st == SA_OK) st = dalloc(&d.free_top, 1);
  if (st == SA_OK) st = dalloc(&d.seal_counters, 2);
  if (st == SA_OK) st = dalloc(&d.status, 1);
  if (st == SA_OK) st = dalloc(&c->selected, nsl * c->n_sel_groups * g.budget_blocks);
  if (st == SA_OK) st = dalloc(&c->selected_count, nsl * c->n_sel_groups);
  if (st == SA_OK) st = dalloc(&c->scores, nsl * c->n_sel_groups * (size_t)c->table_pad);
  if (st == SA_OK) st = dalloc(&c->select_counters, nsl * c->n_sel_groups);
  c->select_split_bytes =
      select_split_scratch_bytes((int)(nsl * c->n_sel_groups), g.select_group, c->table_pad);
  if (st == SA_OK && c->select_split_bytes) st = dalloc(&c->select_split, c->select_split_bytes);
  if (st == SA_OK)
    st = dalloc(reinterpret_cast<char**>(&c->attn_partial),
                attention_scratch_bytes(c->attn_plan, units, c->group));
  if (st == SA_OK) st = dalloc(&c->attn_counters, (size_t)units);
  if (st == SA_OK) st = dalloc(&c->d_query, nsl * g.query_heads * kHeadDim);
  if (st == SA_OK) st = dalloc(&c->d_qt, nsl * g.query_heads * kHeadDim);
  if (st == SA_OK) st = dalloc(reinterpret_cast<float**>(&c->d_kv_new), nsl * row_elems);
  if (st == SA_OK) st = dalloc(reinterpret_cast<float**>(&c->d_out), nsl * g.query_heads * kHeadDim);
  if (st == SA_OK)
    st = cuda_status(cudaHostAlloc(reinterpret_cast<void**>(&c->h_status), sizeof(uint32_t),
                                   cudaHostAllocDefault),
                     "cudaHostAlloc status");
  if (st == SA_OK)
    st = cuda_status(cudaHostGetDevicePointer(reinterpret_cast<void**>(&c->h_status_dev),
                                              c->h_status, 0),
                     "cudaHostGetDevicePointer status");
  if (st == SA_OK) {
    SA_CUDA_TRY(cudaMemset(d.pool, 0, (size_t)g.pool_blocks * kBlockTokens * row_elems * 2));
    SA_CUDA_TRY(cudaMemset(d.reps, 0, nsl * g.query_heads * kHeadDim * (size_t)c->table_pad * 4));
    SA_CUDA_TRY(cudaMemset(d.seal_counters, 0, 2 * sizeof(int)));
    SA_CUDA_TRY(cudaMemset(c->select_counters, 0, nsl * c->n_sel_groups * sizeof(int)));
    if (c->select_split) SA_CUDA_TRY(cudaMemset(c->select_split, 0, c->select_split_bytes));
    SA_CUDA_TRY(cudaMemset(c->attn_counters, 0, (size_t)units * sizeof(int)));
    SA_CUDA_TRY(cudaMemset(c->selected_count, 0, nsl * c->n_sel_groups * sizeof(int)));
    st = sa_ctx_reset(c);
  }
  if (st != SA_OK) {
    const std::string msg = g_last_error;
    sa_ctx_destroy(c);
    g_last_error = msg;
    return st;
  }
  *out = c;
  return SA_OK;
}

SA_API sa_status sa_ctx_destroy(sa_ctx* c) {
  if (!c) return SA_OK;
  DeviceGuard guard(c->cfg.device);
  if (c->recording) {
    cudaGraph_t partial = nullptr;
    cudaStreamEndCapture(c->stream, &partial);
    if (partial) cudaGraphDestroy(partial);
  }
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->graph_exec) cudaGraphExecDestroy(c->graph_exec);
  if (c->graph) cudaGraphDestroy(c->graph);
  if (c->host_step_exec) cudaGraphExecDestroy(c->host_step_exec);
  if (c->host_step_graph) cudaGraphDestroy(c->host_step_graph);
  CtxDev& d = c->dev;
  void* ptrs[] = {d.pool, d.reps, d.table, d.num_sealed, d.tail_block, d.tail_len, d.generation,
                  d.query_ring, d.free_list, d.free_top, d.seal_counters, d.status, c->selected,
                  c->selected_count, c->scores, c->select_counters, c->select_split, c->attn_partial,
                  c->attn_counters, c->d_query, c->d_qt, c->d_kv_new, c->d_out, c->gather_buf,
                  c->gather_peers};
  for (void* p : ptrs) cudaFree(p);
  if (c->h_status) cudaFreeHost(c->h_status);
  if (c->own_stream && c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return SA_OK;
}

SA_API sa_status sa_ctx_get_ptrs(sa_ctx* c, sa_ctx_ptrs* o) {
  if (!c || !o) return fail(SA_ERR_INVALID_ARG, "ctx: null argument");
  o->pool = c->dev.pool;
  o->reps = c->dev.reps;
  o->table = c->dev.table;
  o->num_sealed = c->dev.num_sealed;
  o->tail_block = c->dev.tail_block;
  o->tail_len = c->dev.tail_len;
  o->generation = c->dev.generation;
  o->query_ring = c->dev.query_ring;
  o->selected = c->selected;
  o->selected_count = c->selected_count;
  o->scores = c->scores;
  o->free_list = c->dev.free_list;
  o->free_top = c->dev.free_top;
  o->status = c->dev.status;
  return SA_OK;
}

SA_API sa_status sa_ctx_set_stream(sa_ctx* c, void* stream) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "ctx: null");
  if (c->recording) return refuse_while_recording("set_stream");
  DeviceGuard guard(c->cfg.device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  if (c->own_stream && c->stream) cudaStreamDestroy(c->stream);
  c->own_stream = false;
  c->stream = static_cast<cudaStream_t>(stream);
  return SA_OK;
}

SA_API void* sa_ctx_stream(sa_ctx* c) { return c ? static_cast<void*>(c->stream) : nullptr; }

SA_API sa_status sa_ctx_reset(sa_ctx* c) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "ctx: null");
  if (c->recording) return refuse_while_recording("reset");
  DeviceGuard guard(c->cfg.device);
  const auto& g = c->cfg;
  const size_t nsl = c->num_sl;
  SA_CUDA_TRY(cudaStreamSynchronize(c->stream));
  std::vector<int32_t> free_list(g.pool_blocks);
  for (int i = 0; i < g.pool_blocks; ++i) free_list[i] = g.pool_blocks - 1 - i;  // pops ascend
  const int32_t top = g.pool_blocks;
  SA_CUDA_TRY(cudaMemcpy(c->dev.free_list, free_list.data(), free_list.size() * 4, cudaMemcpyHostToDevice));
  SA_CUDA_TRY(cudaMemcpy(c->dev.free_top, &top, 4, cudaMemcpyHostToDevice));
  SA_CUDA_TRY(cudaMemset(c->dev.table, 0xff, nsl * g.table_blocks * 4));
  SA_CUDA_TRY(cudaMemset(c->dev.num_sealed, 0, nsl * 4));
  SA_CUDA_TRY(cudaMemset(c->dev.tail_block, 0xff, nsl * 4));
  SA_CUDA_TRY(cudaMemset(c->dev.tail_len, 0, nsl * 4));
  SA_CUDA_TRY(cudaMemset(c->dev.generation, 0, nsl * 4));
  SA_CUDA_TRY(cudaMemset(c->dev.status, 0, 4));
  std::fill(c->prefilled.begin(), c->prefilled.end(), 0);
  return SA_OK;
}

SA_API sa_status sa_ctx_prefill(sa_ctx* c, int32_t seq, int32_t layer, int32_t blocks,
                                int32_t* phys_out_host) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "ctx: null");
  if (c->recording) return refuse_while_recording("prefill");
  const auto& g = c->cfg;
  if (seq < 0 || seq >= g.seqs || layer < 0 || layer >= g.layers || blocks < 0)
    return fail(SA_ERR_INVALID_ARG, "prefill: seq/layer/blocks out of range");
  if (blocks > g.table_blocks) return fail(SA_ERR_CAPACITY, "prefill: more blocks than table_blocks");
  const int sl = seq * g.layers + layer;
  if (c->prefilled[sl]) return fail(SA_ERR_INVALID_ARG, "prefill: (seq, layer) already prefilled; reset first");
  DeviceGuard guard(g.device);
  SA_CUDA_TRY(cudaStreamSynchronize(c->stream));
  int32_t top = 0;
  SA_CUDA_TRY(cudaMemcpy(&top, c->dev.free_top, 4, cudaMemcpyDeviceToHost));
  if (top < blocks + 1) return fail(SA_ERR_CAPACITY, "prefill: pool has too few free blocks");
  std::vector<int32_t> slice(blocks + 1);
  SA_CUDA_TRY(cudaMemcpy(slice.data(), c->dev.free_list + (top - blocks - 1), (blocks + 1) * 4,
                         cudaMemcpyDeviceToHost));
  std::vector<int32_t> phys(blocks + 1);
  for (int i = 0; i <= blocks; ++i) phys[i] = slice[blocks - i];  // pop order
  const int32_t new_top = top - blocks - 1;
  const int32_t zero = 0;
  SA_CUDA_TRY(cudaMemcpy(c->dev.free_top, &new_top, 4, cudaMemcpyHostToDevice));
  if (blocks)
    SA_CUDA_TRY(cudaMemcpy(c->dev.table + (size_t)sl * g.table_blocks, phys.data(), blocks * 4,
                           cudaMemcpyHostToDevice));
  SA_CUDA_TRY(cudaMemcpy(c->dev.num_sealed + sl, &blocks, 4, cudaMemcpyHostToDevice));
  SA_CUDA_TRY(cudaMemcpy(c->dev.tail_block + sl, &phys[blocks], 4, cudaMemcpyHostToDevice));
  SA_CUDA_TRY(cudaMemcpy(c->dev.tail_len + sl, &zero, 4, cudaMemcpyHostToDevice));
  SA_CUDA_TRY(cudaMemcpy(c->dev.generation + sl, &zero, 4, cudaMemcpyHostToDevice));
  c->prefilled[sl] = 1;
  if (phys_out_host) std::memcpy(phys_out_host, phys.data(), (blocks + 1) * 4);
  return SA_OK;
}

SA_API sa_status sa_ctx_build_reps(sa_ctx* c, int32_t seq, int32_t layer, int32_t first,
                                   int32_t count, const float* prompt_queries, int32_t window,
                                   int32_t topk, int32_t per_block) {
  if (!c || !prompt_queries) return fail(SA_ERR_INVALID_ARG, "build_reps: null argument");
  const auto& g = c->cfg;
  if (seq < 0 || seq >= g.seqs || layer < 0 || layer >= g.layers || first < 0 || count < 0 ||
      first + count > g.table_blocks)
    return fail(SA_ERR_INVALID_ARG, "build_reps: range out of bounds");
  if (count == 0) return SA_OK;
  DeviceGuard guard(g.device);
  const int sl = seq * g.layers + layer;
  RepParams p{};
  p.kv = c->dev.pool;
  p.head_major = 1;
  p.row_stride = c->dev.row_elems;
  p.table = c->dev.table;
  p.table_offset = sl * g.table_blocks + first;
  p.kv_heads = g.kv_heads;
  p.q = prompt_queries;
  p.qh = g.query_heads;
  p.d = kHeadDim;
  p.tokens = count * kBlockTokens;
  p.blocks = count;
  p.window = window;
  p.topk = topk;
  p.scale = 1.0f / std::sqrt((float)kHeadDim);
  p.values = c->dev.reps + (size_t)sl * g.query_heads * kHeadDim * c->table_pad + first;
  p.o_head = (int64_t)kHeadDim * c->table_pad;
  p.o_block = 1;
  p.o_dim = c->table_pad;
  p.offsets = nullptr;
  p.status = c->dev.status;
  ++c->launches;
  return per_block ? launch_build_reps_per_block(p, c->stream) : launch_build_reps(p, c->stream);
}

SA_API sa_status sa_ctx_append(sa_ctx* c, const float* query, const void* kv_new, int32_t kv_fp32) {
  if (!c || !query || !kv_new) return fail(SA_ERR_INVALID_ARG, "append: null argument");
  DeviceGuard guard(c->cfg.device);
  ++c->launches;
  return launch_append(c->dev, query, kv_new, kv_fp32, c->stream);
}

SA_API sa_status sa_ctx_select(sa_ctx* c, const float* query) {
  if (!c || !query) return fail(SA_ERR_INVALID_ARG, "select: null argument");
  DeviceGuard guard(c->cfg.device);
  return ctx_select(c, query);
}

SA_API sa_status sa_ctx_attend(sa_ctx* c, const float* query, void* out) {
  if (!c || !query || !out) return fail(SA_ERR_INVALID_ARG, "attend: null argument");
  DeviceGuard guard(c->cfg.device);
  // A programmatic dependent of whatever kernel precedes it on the stream, as
  // in a decode step: before griddepcontrol.wait the kernel reads no global
  // memory, so only its launch overlaps the predecessor's last CTAs.
  return ctx_attend(c, query, out, 0, true);
}

SA_API sa_status sa_ctx_seal(sa_ctx* c) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "seal: null ctx");
  DeviceGuard guard(c->cfg.device);
  ++c->launches;
  return launch_seal(c->dev, 0, c->stream);
}

}  // extern "C"

namespace {
sa_status ctx_step(sa_ctx* c, const float* query, const void* kv_new, int32_t kv_fp32, void* out,
                   uint32_t* status_mirror);
}

extern "C" {

SA_API sa_status sa_ctx_step(sa_ctx* c, const float* query, const void* kv_new, int32_t kv_fp32,
                             void* out) {
  if (!c || !query || !kv_new || !out) return fail(SA_ERR_INVALID_ARG, "step: null argument");
  DeviceGuard guard(c->cfg.device);
  return ctx_step(c, query, kv_new, kv_fp32, out, nullptr);
}

}  // extern "C"

namespace {
sa_status ctx_step(sa_ctx* c, const float* query, const void* kv_new, int32_t kv_fp32, void* out,
                   uint32_t* status_mirror) {
  // Three launches: select with the fused append (the new token is written
  // but not yet counted in tail_len), attention counting that pending token,
  // then the seal kernel, which rebuilds full tails and stores every tail's
  // new length. Attention and seal are programmatic dependents of the kernel
  // before them: they launch early and wait on the device before reading
  // its results. The select launches normally: making it a dependent of the
  // previous step's seal as well let three grids queue ahead of each other
  // and cost 29 us per step on a B200, while the two links save 3.6 us.
  sa_status st;
  if ((st = ctx_select(c, query, kv_new, kv_fp32, false)) != SA_OK) return st;
  if ((st = ctx_attend(c, query, out, 1, true, true)) != SA_OK) return st;
  ++c->launches;
  CtxDev d = c->dev;
  d.status_mirror = status_mirror;
  if (c->gather_peers) {
    // the seal kernel also waits for every rank's outputs of this attention
    d.gather_counter =
        reinterpret_cast<const unsigned long long*>(c->gather_buf + c->gather_counter_bytes);
    d.gather_epoch = reinterpret_cast<unsigned long long*>(c->gather_buf + c->gather_counter_bytes + 8);
    d.gather_peers = c->gather_peers;
    d.gather_world = c->gather_world;
    d.gather_counter_bytes = c->gather_counter_bytes;
  }
  st = launch_seal(d, 1, c->stream, true);
  if (st == SA_OK && c->gather_peers) c->gather_waited = c->gather_attends;
  return st;
}

// Device-side address of a pinned, mapped host buffer aligned to `align`
// bytes, or null (pageable memory, or an unaligned pointer).
void* mapped_host(const void* p, uintptr_t align) {
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (a.type != cudaMemoryTypeHost || !a.devicePointer) return nullptr;
  if (reinterpret_cast<uintptr_t>(a.devicePointer) % align) return nullptr;
  return a.devicePointer;
}
}  // namespace
extern "C" {

SA_API sa_status sa_ctx_step_host(sa_ctx* c, const float* query_host, const void* kv_new_host,
                                  int32_t kv_fp32, void* out_host) {
  if (!c || !query_host || !kv_new_host || !out_host)
    return fail(SA_ERR_INVALID_ARG, "step_host: null argument");
  if (c->recording) return refuse_while_recording("step_host");
  DeviceGuard guard(c->cfg.device);
  const auto& g = c->cfg;
  const size_t q_bytes = (size_t)c->num_sl * g.query_heads * kHeadDim * sizeof(float);
  const size_t kv_bytes = (size_t)c->num_sl * c->dev.row_elems * (kv_fp32 ? 4 : 2);
  const size_t out_bytes = (size_t)c->num_sl * g.query_heads * kHeadDim * (g.out_fp16 ? 2 : 4);
  // Pinned, mapped caller buffers are used in place: the fused append reads
  // the new K/V from host memory, the attention writes the output there and
  // the seal copies the status word to a mapped host word, so only the
  // queries (read by every scoring CTA) are copied. Pageable buffers go
  // through device staging copies.
  void* kv_dev = mapped_host(kv_new_host, 16);
  void* out_dev = mapped_host(out_host, 16);
  *reinterpret_cast<volatile uint32_t*>(c->h_status) = 0xffffffffu;  // "not written"
  // All three buffers pinned and no peer gather (whose host-side epoch
  // bookkeeping a replay would skip): replay the call's recorded step, one
  // graph launch instead of a copy and three kernel launches.
  const bool replayable = kv_dev && out_dev && mapped_host(query_host, 16) && !c->gather_peers &&
                          c->stream != nullptr && c->stream != cudaStreamLegacy;
  const bool same = replayable && c->host_step_exec && c->host_step_key[0] == query_host &&
                    c->host_step_key[1] == kv_new_host && c->host_step_key[2] == out_host &&
                    c->host_step_key[3] == kv_dev && c->host_step_kv_fp32 == kv_fp32;
  if (same) {
    SA_CUDA_TRY(cudaGraphLaunch(c->host_step_exec, c->stream));
    c->launches += c->host_step_launches;
  } else {
    if (replayable) {
      if (c->host_step_exec) cudaGraphExecDestroy(c->host_step_exec);
      if (c->host_step_graph) cudaGraphDestroy(c->host_step_graph);
      c->host_step_exec = nullptr;
      c->host_step_graph = nullptr;
      SA_CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    }
    const uint64_t launches0 = c->launches;
    sa_status st = SA_OK;
    cudaError_t e =
        cudaMemcpyAsync(c->d_query, query_host, q_bytes, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess && !kv_dev) {
      e = cudaMemcpyAsync(c->d_kv_new, kv_new_host, kv_bytes, cudaMemcpyHostToDevice, c->stream);
      kv_dev = c->d_kv_new;
    }
    if (e != cudaSuccess) st = cuda_status(e, "step_host: query / K,V copy");
    if (st == SA_OK)
      st = ctx_step(c, c->d_query, kv_dev, kv_fp32, out_dev ? out_dev : c->d_out, c->h_status_dev);
    if (st == SA_OK && !out_dev) {
      e = cudaMemcpyAsync(out_host, c->d_out, out_bytes, cudaMemcpyDeviceToHost, c->stream);
      if (e != cudaSuccess) st = cuda_status(e, "step_host: output copy");
    }
    if (replayable) {
      cudaGraph_t g = nullptr;
      const cudaError_t ec = cudaStreamEndCapture(c->stream, &g);
      if (st == SA_OK && ec != cudaSuccess) st = cuda_status(ec, "step_host: end capture");
      if (st == SA_OK) {
        const cudaError_t ei = cudaGraphInstantiate(&c->host_step_exec, g, 0);
        if (ei != cudaSuccess) st = cuda_status(ei, "step_host: instantiate");
      }
      if (st != SA_OK) {
        if (g) cudaGraphDestroy(g);
        c->host_step_exec = nullptr;
        c->launches = launches0;
        return st;
      }
      c->host_step_graph = g;
      c->host_step_launches = c->launches - launches0;
      c->launches = launches0 + c->host_step_launches;
      c->host_step_key[0] = query_host;
      c->host_step_key[1] = kv_new_host;
      c->host_step_key[2] = out_host;
      c->host_step_key[3] = kv_dev;
      c->host_step_kv_fp32 = kv_fp32;
      SA_CUDA_TRY(cudaGraphLaunch(c->host_step_exec, c->stream));
    } else if (st != SA_OK) {
      return st;
    }
  }
  SA_CUDA_TRY(cudaStreamSynchronize(c->stream));
  if (*reinterpret_cast<volatile uint32_t*>(c->h_status) == 0xffffffffu)
    SA_CUDA_TRY(cudaMemcpy(c->h_status, c->dev.status, sizeof(uint32_t), cudaMemcpyDeviceToHost));
  if (*c->h_status)
    return fail(*c->h_status & SA_DEV_TIMEOUT ? SA_ERR_TIMEOUT : SA_ERR_DEVICE,
                "step_host: device status bits 0x" + std::to_string(*c->h_status));
  return SA_OK;
}

SA_API sa_status sa_probe_stream(const void* pool, int64_t pool_entries, const int32_t* entry_ids,
                                 int64_t n, int32_t mode, uint64_t* sink, uint32_t* status,
                                 void* stream) {
  static_assert(SA_PROBE_SINK_WORDS >= 1024, "sink words");
  return launch_probe_stream(pool, pool_entries, entry_ids, n, mode,
                             reinterpret_cast<unsigned long long*>(sink), status,
                             static_cast<cudaStream_t>(stream));
}

SA_API sa_status sa_ctx_sync(sa_ctx* c, uint32_t* bits_out) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "sync: null ctx");
  if (c->recording) return refuse_while_recording("sync");
  DeviceGuard guard(c->cfg.device);
  SA_CUDA_TRY(cudaStreamSynchronize(c->stream));
  uint32_t bits = 0;
  SA_CUDA_TRY(cudaMemcpy(&bits, c->dev.status, sizeof(bits), cudaMemcpyDeviceToHost));
  if (bits_out) *bits_out = bits;
  if (bits & SA_DEV_TIMEOUT) return fail(SA_ERR_TIMEOUT, "device wait timed out");
  if (bits) return fail(SA_ERR_DEVICE, "device status bits 0x" + std::to_string(bits));
  return SA_OK;
}

SA_API uint64_t sa_ctx_launch_count(const sa_ctx* c) { return c ? c->launches : 0; }

SA_API sa_status sa_ctx_graph_begin(sa_ctx* c) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "graph_begin: null ctx");
  if (c->recording) return fail(SA_ERR_INVALID_ARG, "graph_begin: a recording is already open");
  if (c->stream == nullptr || c->stream == cudaStreamLegacy)
    return fail(SA_ERR_UNSUPPORTED, "graph_begin: the legacy default stream cannot be recorded");
  DeviceGuard guard(c->cfg.device);
  SA_CUDA_TRY(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
  c->recording = true;
  c->launches_before_recording = c->launches;
  c->gather_attends_before_recording = c->gather_attends;
  c->gather_waited_before_recording = c->gather_waited;
  c->gather_view_recorded = false;
  return SA_OK;
}

SA_API sa_status sa_ctx_graph_end(sa_ctx* c) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "graph_end: null ctx");
  if (!c->recording) return fail(SA_ERR_INVALID_ARG, "graph_end: no recording is open");
  DeviceGuard guard(c->cfg.device);
  c->recording = false;
  // recorded calls launched nothing yet
  const uint64_t recorded = c->launches - c->launches_before_recording;
  c->launches = c->launches_before_recording;
  const uint64_t recorded_attends = c->gather_attends - c->gather_attends_before_recording;
  c->gather_attends = c->gather_attends_before_recording;
  const uint64_t recorded_waits = c->gather_waited - c->gather_waited_before_recording;
  c->gather_waited = c->gather_waited_before_recording;
  cudaGraph_t graph = nullptr;
  SA_CUDA_TRY(cudaStreamEndCapture(c->stream, &graph));
  if (c->gather_view_recorded && recorded_attends % 2 == 1) {
    // Every replay flips the device-side slot parity once per gathered
    // attention, while a recorded consumer keeps the slot address it was
    // given at record time: with an odd count it would read the previous
    // step's slot on every second replay.
    cudaGraphDestroy(graph);
    return fail(SA_ERR_UNSUPPORTED,
                "graph_end: a recording that hands out a gathered slot must hold an even "
                "number of gathered attentions");
  }
  cudaGraphExec_t exec = nullptr;
  cudaError_t e = cudaGraphInstantiate(&exec, graph, 0);
  if (e == cudaSuccess) e = cudaGraphUpload(exec, c->stream);
  if (e != cudaSuccess) {
    if (exec) cudaGraphExecDestroy(exec);
    cudaGraphDestroy(graph);
    return cuda_status(e, "graph_end: instantiate");
  }
  if (c->graph_exec) cudaGraphExecDestroy(c->graph_exec);
  if (c->graph) cudaGraphDestroy(c->graph);
  c->graph = graph;
  c->graph_exec = exec;
  c->graph_launches = recorded;
  c->graph_gather_attends = recorded_attends;
  c->graph_gather_waited = recorded_waits;
  return SA_OK;
}

SA_API sa_status sa_ctx_graph_launch(sa_ctx* c) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "graph_launch: null ctx");
  if (c->recording) return refuse_while_recording("graph_launch");
  if (!c->graph_exec) return fail(SA_ERR_INVALID_ARG, "graph_launch: nothing recorded");
  DeviceGuard guard(c->cfg.device);
  SA_CUDA_TRY(cudaGraphLaunch(c->graph_exec, c->stream));
  c->launches += c->graph_launches;
  c->gather_attends += c->graph_gather_attends;
  c->gather_waited += c->graph_gather_waited;
  return SA_OK;
}

SA_API sa_status sa_ctx_audit(sa_ctx* c, const float* query, float* mass_out) {
  if (!c || !query || !mass_out) return fail(SA_ERR_INVALID_ARG, "audit: null argument");
  DeviceGuard guard(c->cfg.device);
  ++c->launches;
  return launch_audit(c->dev, query, mass_out, c->cfg.scale, c->stream);
}

SA_API sa_status sa_ctx_slot_correct(sa_ctx* c, int32_t* slots, int32_t* misses, int32_t* replace,
                                     int32_t* stats) {
  if (!c || !slots || !misses || !replace || !stats)
    return fail(SA_ERR_INVALID_ARG, "slot_correct: null argument");
  DeviceGuard guard(c->cfg.device);
  ++c->launches;
  return launch_slot_correct(c->selected, c->selected_count, slots, misses, replace, stats,
                             c->num_sl * c->n_sel_groups, c->cfg.budget_blocks,
                             c->cfg.table_blocks, c->dev.status, c->stream);
}

SA_API sa_status sa_ctx_step_raw(sa_ctx* c, const float* q_raw, const float* k_raw,
                                 const float* v, const float* q_norm_w, const float* k_norm_w,
                                 const int32_t* positions, float rope_theta, float norm_eps,
                                 void* out) {
  if (!c || !q_raw || !k_raw || !v || !q_norm_w || !k_norm_w || !positions || !out)
    return fail(SA_ERR_INVALID_ARG, "step_raw: null argument");
  if (!(rope_theta > 0.f) || !(norm_eps >= 0.f))
    return fail(SA_ERR_INVALID_ARG, "step_raw: bad rope theta or norm epsilon");
  DeviceGuard guard(c->cfg.device);
  SelectParams p = select_params(c, q_raw);
  p.append_ctx = c->dev;
  p.raw_k = k_raw;
  p.raw_v = v;
  p.q_norm_w = q_norm_w;
  p.k_norm_w = k_norm_w;
  p.positions = positions;
  p.raw_qt = c->d_qt;
  p.layers = c->cfg.layers;
  p.rope_theta = rope_theta;
  p.norm_eps = norm_eps;
  ++c->launches;
  sa_status st = launch_select(p, c->stream);
  if (st != SA_OK) return st;
  if ((st = ctx_attend(c, c->d_qt, out, 1, true)) != SA_OK) return st;
  ++c->launches;
  return launch_seal(c->dev, 1, c->stream, true);
}

namespace {
sa_status ctx_store_blocks(sa_ctx* c, int32_t seq, int32_t layer, int32_t first, int32_t count,
                           void* store, bool import) {
  if (!c || !store) return fail(SA_ERR_INVALID_ARG, "blocks: null argument");
  if (seq < 0 || seq >= c->cfg.seqs || layer < 0 || layer >= c->cfg.layers)
    return fail(SA_ERR_INVALID_ARG, "blocks: sequence or layer out of range");
  if (first < 0 || count < 0 || first + count > c->cfg.table_blocks)
    return fail(SA_ERR_INVALID_ARG, "blocks: logical range beyond the block table");
  DeviceGuard guard(c->cfg.device);
  // the kernel touches `store` directly: it must be this device's memory or
  // pinned host memory mapped for the device (never pageable memory)
  cudaPointerAttributes a{};
  if (cudaPointerGetAttributes(&a, store) != cudaSuccess) {
    cudaGetLastError();
    return fail(SA_ERR_INVALID_ARG, "blocks: store is not device or pinned host memory");
  }
  void* dev = nullptr;
  if ((a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) &&
      a.device == c->cfg.device)
    dev = store;
  else if (a.type == cudaMemoryTypeHost && a.devicePointer)
    dev = a.devicePointer;
  if (!dev)
    return fail(SA_ERR_INVALID_ARG,
                "blocks: store must be memory of the context's device or pinned, mapped host memory");
  if (reinterpret_cast<uintptr_t>(dev) & 15u)
    return fail(SA_ERR_INVALID_ARG, "blocks: store buffer must be 16-byte aligned");
  ++c->launches;
  return launch_store_blocks(c->dev, seq * c->cfg.layers + layer, first, count, dev, import,
                             c->stream);
}
}  // namespace

SA_API sa_status sa_ctx_import_blocks(sa_ctx* c, int32_t seq, int32_t layer, int32_t first,
                                      int32_t count, const void* store) {
  return ctx_store_blocks(c, seq, layer, first, count, const_cast<void*>(store), true);
}

SA_API sa_status sa_ctx_export_blocks(sa_ctx* c, int32_t seq, int32_t layer, int32_t first,
                                      int32_t count, void* store) {
  return ctx_store_blocks(c, seq, layer, first, count, store, false);
}

// ------------------------------------------- KV-head-sharded gather over peer memory

SA_API sa_status sa_ctx_gather_buffer(sa_ctx* c, int32_t world, void** buf_out,
                                      size_t* bytes_out) {
  if (!c || !buf_out || world < 1 || world > 64)
    return fail(SA_ERR_INVALID_ARG, "gather_buffer: bad argument");
  if (c->recording) return refuse_while_recording("gather_buffer");
  if (c->gather_buf && c->gather_world != world)
    return fail(SA_ERR_INVALID_ARG, "gather_buffer: already allocated for another world size");
  DeviceGuard guard(c->cfg.device);
  if (!c->gather_buf) {
    const size_t esz = c->cfg.out_fp16 ? 2 : 4;
    const size_t slot = (size_t)c->num_sl * world * c->cfg.query_heads * kHeadDim * esz;
    c->gather_slot_bytes = (slot + 255) & ~size_t(255);
    c->gather_counter_bytes = 2 * c->gather_slot_bytes;
    c->gather_bytes = c->gather_counter_bytes + 256;
    sa_status st = dalloc(&c->gather_buf, c->gather_bytes);
    if (st != SA_OK) return st;
    SA_CUDA_TRY(cudaMemset(c->gather_buf, 0, c->gather_bytes));
    c->gather_world = world;
  }
  *buf_out = c->gather_buf;
  if (bytes_out) *bytes_out = c->gather_bytes;
  return SA_OK;
}

SA_API sa_status sa_ctx_gather_attach(sa_ctx* c, int32_t rank, void* const* peer_bufs) {
  if (!c || !peer_bufs) return fail(SA_ERR_INVALID_ARG, "gather_attach: null argument");
  if (c->recording) return refuse_while_recording("gather_attach");
  if (!c->gather_buf) return fail(SA_ERR_INVALID_ARG, "gather_attach: call sa_ctx_gather_buffer first");
  if (rank < 0 || rank >= c->gather_world)
    return fail(SA_ERR_INVALID_ARG, "gather_attach: rank outside [0, world)");
  if (peer_bufs[rank] != c->gather_buf)
    return fail(SA_ERR_INVALID_ARG, "gather_attach: peer_bufs[rank] must be this context's buffer");
  for (int r = 0; r < c->gather_world; ++r)
    if (!peer_bufs[r] || (reinterpret_cast<uintptr_t>(peer_bufs[r]) & 255u))
      return fail(SA_ERR_INVALID_ARG, "gather_attach: null or unaligned peer buffer");
  DeviceGuard guard(c->cfg.device);
  if (!c->gather_peers) {
    sa_status st = dalloc(&c->gather_peers, (size_t)c->gather_world);
    if (st != SA_OK) return st;
  }
  SA_CUDA_TRY(cudaMemcpy(c->gather_peers, peer_bufs, sizeof(void*) * c->gather_world,
                         cudaMemcpyHostToDevice));
  // A fresh start: arrival counter and epoch zero (late arrivals of a step
  // whose wait timed out are dropped with them), slot parity even.
  SA_CUDA_TRY(cudaStreamSynchronize(c->stream));
  SA_CUDA_TRY(cudaMemset(c->gather_buf + c->gather_counter_bytes, 0, 24));
  c->gather_attends = 0;
  c->gather_waited = 0;
  c->gather_rank = rank;
  return SA_OK;
}

SA_API sa_status sa_ctx_gather_wait(sa_ctx* c, void** gathered_out) {
  if (!c) return fail(SA_ERR_INVALID_ARG, "gather_wait: null ctx");
  if (!c->gather_peers) return fail(SA_ERR_INVALID_ARG, "gather_wait: gather not attached");
  if (c->gather_attends == 0) return fail(SA_ERR_INVALID_ARG, "gather_wait: no gathered attend yet");
  DeviceGuard guard(c->cfg.device);
  if (c->gather_waited != c->gather_attends) {
    // an attention of its own (sa_ctx_attend): enqueue its wait; a decode
    // step's seal kernel has already enqueued the wait of the step's attention
    ++c->launches;
    const sa_status st = launch_gather_wait(
        c->gather_peers, c->gather_world, c->gather_counter_bytes,
        reinterpret_cast<const unsigned long long*>(c->gather_buf + c->gather_counter_bytes),
        reinterpret_cast<unsigned long long*>(c->gather_buf + c->gather_counter_bytes + 8),
        (unsigned long long)c->gather_world * c->num_sl * c->cfg.kv_heads, c->dev.status,
        c->stream);
    if (st != SA_OK) return st;
    c->gather_waited = c->gather_attends;
  }
  if (gathered_out) {
    *gathered_out = c->gather_buf + ((c->gather_attends - 1) % 2) * c->gather_slot_bytes;
    if (c->recording) c->gather_view_recorded = true;
  }
  return SA_OK;
}

SA_API sa_status sa_ipc_export(int32_t device, const void* dev_ptr, void* handle_out) {
  if (!dev_ptr || !handle_out) return fail(SA_ERR_INVALID_ARG, "ipc_export: null argument");
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(SA_ERR_CUDA, "ipc_export: cudaSetDevice failed");
  cudaIpcMemHandle_t h;
  SA_CUDA_TRY(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
  static_assert(sizeof(h) == SA_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle_out, &h, sizeof(h));
  return SA_OK;
}

SA_API sa_status sa_ipc_open(int32_t device, const void* handle, void** dev_ptr_out) {
  if (!handle || !dev_ptr_out) return fail(SA_ERR_INVALID_ARG, "ipc_open: null argument");
  DeviceGuard guard(device);
  if (!guard.ok()) return fail(SA_ERR_CUDA, "ipc_open: cudaSetDevice failed");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  SA_CUDA_TRY(cudaIpcOpenMemHandle(dev_ptr_out, h, cudaIpcMemLazyEnablePeerAccess));
  return SA_OK;
}

SA_API sa_status sa_ipc_close(int32_t device, void* dev_ptr) {
  if (!dev_ptr) return SA_OK;
  DeviceGuard guard(device);
  SA_CUDA_TRY(cudaIpcCloseMemHandle(dev_ptr));
  return SA_OK;
}

}  // extern "C"
