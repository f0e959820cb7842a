// sa_b200_backend.hpp -- C++ drop-in for the reference's native line, built
// only on the C ABI of sa_b200.h (no CUDA headers needed by the caller).
//
//  * solidattention::make_b200_backend() returns an AcceleratorBackend
//    (cpp/include/solidattention/backend.hpp:41-58) whose attention variants
//    run the sm_100a kernel with the reference's H2D / kernel / consumer / D2H
//    timing split (cpp/src/cuda_backend.cpp:282-415), with no token cap;
//  * solidattention::b200::select_shared_blocks and
//    solidattention::b200::build_local_causal_representatives have the
//    signatures and results of the reference's free functions
//    (cpp/include/solidattention/selection.hpp:19-29) and throw
//    std::runtime_error where those throw.
//
// A driver switches by adding a `--backend b200` branch
// (cpp/src/attention_main.cpp:101-116) and by qualifying the selector calls
// with b200:: (cpp/src/selection_main.cpp:159-181).
#pragma once

#include <cstddef>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "sa_b200.h"
#include "solidattention/backend.hpp"
#include "solidattention/selection.hpp"

namespace solidattention {

namespace b200_detail {
inline void check(sa_status status) {
  if (status != SA_OK) throw std::runtime_error(sa_last_error());
}
}  // namespace b200_detail

class B200Backend final : public AcceleratorBackend {
 public:
  explicit B200Backend(int device = 0) { b200_detail::check(sa_backend_create(device, &handle_)); }
  ~B200Backend() override { sa_backend_destroy(handle_); }
  B200Backend(const B200Backend&) = delete;
  B200Backend& operator=(const B200Backend&) = delete;

  std::string name() const override { return sa_backend_name(handle_); }

  void* allocate_host(std::size_t bytes) override {
    void* pointer = nullptr;
    b200_detail::check(sa_backend_host_alloc(handle_, bytes, &pointer));
    return pointer;
  }

  void free_host(void* pointer) override { b200_detail::check(sa_backend_host_free(handle_, pointer)); }

  TransferResult execute(void* pinned_input, std::size_t bytes, std::uint8_t mask) override {
    sa_timings t{};
    std::uint64_t checksum = 0;
    b200_detail::check(sa_backend_execute(handle_, pinned_input, bytes, mask, &t, &checksum));
    TransferResult r;
    r.h2d_ms = t.h2d_ms;
    r.kernel_ms = t.kernel_ms;
    r.d2h_ms = t.d2h_ms;
    r.checksum = checksum;
    return r;
  }

  // One kernel serves every variant of the reference (C1 serial, C1.1
  // parallel, C1.2 persistent resources): device buffers persist in the handle.
  AttentionResult attention(const AttentionProblem& p) override { return run(p, SA_ATTN_COPY_OUTPUT); }
  AttentionResult attention_optimized(const AttentionProblem& p) override {
    return run(p, SA_ATTN_COPY_OUTPUT);
  }
  AttentionResult attention_persistent(const AttentionProblem& p) override {
    return run(p, SA_ATTN_COPY_OUTPUT);
  }
  // C1.3: the output stays on the device unless this operation is audited.
  AttentionResult attention_resident(const AttentionProblem& p, bool audit_output) override {
    return run(p, audit_output ? SA_ATTN_COPY_OUTPUT : 0);
  }
  // C1.4: a device consumer reduces the output; only its checksum may come back.
  AttentionResult attention_consumed(const AttentionProblem& p, bool audit_checksum) override {
    return run(p, SA_ATTN_CONSUME | (audit_checksum ? SA_ATTN_COPY_OUTPUT : 0));
  }

 private:
  AttentionResult run(const AttentionProblem& p, int flags) {
    AttentionResult r;
    if (flags & SA_ATTN_COPY_OUTPUT) r.output.resize((flags & SA_ATTN_CONSUME) ? 1 : p.query_elements());
    sa_timings t{};
    b200_detail::check(sa_backend_attention(handle_, p.interleaved_kv, p.query, p.tokens,
                                            p.query_heads, p.kv_heads, p.head_dim, p.scale, flags,
                                            r.output.empty() ? nullptr : r.output.data(), &t));
    r.h2d_ms = t.h2d_ms;
    r.kernel_ms = t.kernel_ms;
    r.consumer_ms = t.consumer_ms;
    r.d2h_ms = t.d2h_ms;
    return r;
  }

  sa_backend* handle_ = nullptr;
};

inline std::unique_ptr<AcceleratorBackend> make_b200_backend(int device = 0) {
  return std::make_unique<B200Backend>(device);
}

namespace b200 {

namespace detail {
// The selector functions are free functions in the reference; here each host
// thread lazily owns one backend handle (device 0) for their buffers.
inline sa_backend* thread_backend() {
  struct Holder {
    sa_backend* handle = nullptr;
    ~Holder() {
      if (handle) sa_backend_destroy(handle);
    }
  };
  thread_local Holder holder;
  if (!holder.handle) b200_detail::check(sa_backend_create(0, &holder.handle));
  return holder.handle;
}
}  // namespace detail

inline SelectionResult select_shared_blocks(const float* query, const float* representatives,
                                            std::size_t query_heads, std::size_t blocks,
                                            std::size_t head_dim, std::size_t budget_blocks,
                                            std::size_t init_blocks, std::size_t local_blocks) {
  SelectionResult r;
  std::vector<std::int64_t> ids(budget_blocks ? budget_blocks : 1);
  r.mean_head_scores.resize(blocks);
  b200_detail::check(sa_backend_select(detail::thread_backend(), query, representatives,
                                       query_heads, blocks, head_dim, budget_blocks, init_blocks,
                                       local_blocks, ids.data(), r.mean_head_scores.data()));
  r.block_ids.assign(ids.begin(), ids.begin() + static_cast<std::ptrdiff_t>(budget_blocks));
  return r;
}

inline RepresentativeResult build_local_causal_representatives(
    const float* prompt_queries, const std::uint16_t* interleaved_kv, std::size_t tokens,
    std::size_t query_heads, std::size_t kv_heads, std::size_t head_dim, std::size_t block_tokens,
    std::size_t local_window, std::size_t representative_topk) {
  RepresentativeResult r;
  const std::size_t blocks = block_tokens ? tokens / block_tokens : 0;
  r.values.resize(query_heads * blocks * head_dim);
  std::vector<std::int64_t> offsets(query_heads * blocks * representative_topk);
  b200_detail::check(sa_backend_build_representatives(
      detail::thread_backend(), prompt_queries, interleaved_kv, tokens, query_heads, kv_heads,
      head_dim, block_tokens, local_window, representative_topk, r.values.data(),
      offsets.data()));
  r.chosen_token_offsets.assign(offsets.begin(), offsets.end());
  return r;
}

}  // namespace b200
}  // namespace solidattention
