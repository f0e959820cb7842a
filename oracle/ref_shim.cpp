// ref_shim.cpp -- C entry points over the reference's own C++ functions.
//
// TEST INFRASTRUCTURE ONLY. Built by oracle/Makefile together with the
// reference's unmodified cpp/src/attention_reference.cpp and
// cpp/src/selection.cpp into oracle/_ref/libsa_ref.so, so that Python tests
// can pin the plain-C restatement (sa_oracle.c) against the reference itself
// and bench.py can time the reference's CPU path. Nothing here is part of
// the product library.
//
// Wrapped reference functions (paths relative to the reference project):
//   solidattention::half_to_float / float_to_half  cpp/src/attention_reference.cpp:11-53
//   solidattention::attention_reference            cpp/src/attention_reference.cpp:55-96
//   solidattention::select_shared_blocks           cpp/src/selection.cpp:96-147
//   solidattention::build_local_causal_representatives  cpp/src/selection.cpp:12-94
#include "solidattention/attention_reference.hpp"
#include "solidattention/selection.hpp"

#include <cstdint>
#include <cstring>
#include <exception>
#include <vector>

#ifdef _OPENMP
#include <omp.h>
#endif

namespace sa = solidattention;

extern "C" {

float saref_half_to_float(std::uint16_t v) { return sa::half_to_float(v); }
std::uint16_t saref_float_to_half(float v) { return sa::float_to_half(v); }

int saref_attention(const std::uint16_t* kv, const float* q, std::size_t tokens,
                    std::size_t query_heads, std::size_t kv_heads,
                    std::size_t head_dim, float scale, float* out) {
  try {
    sa::AttentionProblem p{kv, q, tokens, query_heads, kv_heads, head_dim, scale};
    const auto o = sa::attention_reference(p);
    std::memcpy(out, o.data(), o.size() * sizeof(float));
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

int saref_select_shared_blocks(const float* q, const float* reps,
                               std::size_t query_heads, std::size_t blocks,
                               std::size_t head_dim, std::size_t budget,
                               std::size_t init, std::size_t local,
                               std::int64_t* ids_out, std::size_t* n_ids,
                               float* scores_out) {
  try {
    const auto r = sa::select_shared_blocks(q, reps, query_heads, blocks, head_dim,
                                            budget, init, local);
    for (std::size_t i = 0; i < r.block_ids.size(); ++i)
      ids_out[i] = static_cast<std::int64_t>(r.block_ids[i]);
    *n_ids = r.block_ids.size();
    if (scores_out)
      std::memcpy(scores_out, r.mean_head_scores.data(), blocks * sizeof(float));
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

int saref_build_representatives(const float* prompt_queries,
                                const std::uint16_t* kv, std::size_t tokens,
                                std::size_t query_heads, std::size_t kv_heads,
                                std::size_t head_dim, std::size_t block_tokens,
                                std::size_t local_window, std::size_t topk,
                                float* values_out, std::int64_t* offsets_out) {
  try {
    const auto r = sa::build_local_causal_representatives(
        prompt_queries, kv, tokens, query_heads, kv_heads, head_dim,
        block_tokens, local_window, topk);
    std::memcpy(values_out, r.values.data(), r.values.size() * sizeof(float));
    for (std::size_t i = 0; i < r.chosen_token_offsets.size(); ++i)
      offsets_out[i] = static_cast<std::int64_t>(r.chosen_token_offsets[i]);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// One decode step of the sparse path on host cores, for a list of layers:
// per (layer, KV-head group) the reference selector on the group's slice of
// representatives, a packed gather of the chosen 32-token blocks (plus the
// open tail) of that KV head, then the reference attention. Work items run in
// parallel over `threads` OpenMP threads; each item calls the reference's pure
// functions exactly as its drivers do (cpp/src/selection_main.cpp:178-225).
//
// pool:   [pool_blocks][block_tokens][2][kv_heads][head_dim] FP16
// table:  [layers][table_stride] logical block -> pool block
// reps:   [layers][query_heads][blocks][head_dim] FP32
// query:  [layers][query_heads][head_dim] FP32
// tail:   [layers] pool block of the open tail, tail_len tokens valid
// ids:    [layers][kv_heads][budget] out; out: [layers][query_heads][head_dim]
int saref_sparse_step(const std::uint16_t* pool, const std::int32_t* table,
                      std::size_t table_stride, const float* reps,
                      const float* query, const std::int32_t* tail_block,
                      std::size_t tail_len, std::size_t layers,
                      std::size_t query_heads, std::size_t kv_heads,
                      std::size_t head_dim, std::size_t block_tokens,
                      std::size_t blocks, std::size_t budget, std::size_t init,
                      std::size_t local, float scale, int threads,
                      std::int64_t* ids_out, float* out) {
  const std::size_t group = query_heads / kv_heads;
  const std::size_t token_values = 2 * kv_heads * head_dim;
  const long items = static_cast<long>(layers * kv_heads);
  int failed = 0;
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1) reduction(| : failed)
#endif
  for (long item = 0; item < items; ++item) {
    const std::size_t layer = static_cast<std::size_t>(item) / kv_heads;
    const std::size_t h = static_cast<std::size_t>(item) % kv_heads;
    try {
      const float* q = query + (layer * query_heads + h * group) * head_dim;
      const float* r = reps + (layer * query_heads + h * group) * blocks * head_dim;
      const auto sel = sa::select_shared_blocks(q, r, group, blocks, head_dim,
                                                budget, init, local);
      const std::size_t tokens = sel.block_ids.size() * block_tokens + tail_len;
      std::vector<std::uint16_t> packed(tokens * 2 * head_dim);
      std::size_t row = 0;
      auto copy_row = [&](const std::uint16_t* src_row) {
        std::memcpy(&packed[row * 2 * head_dim], src_row + h * head_dim,
                    head_dim * sizeof(std::uint16_t));
        std::memcpy(&packed[row * 2 * head_dim + head_dim],
                    src_row + kv_heads * head_dim + h * head_dim,
                    head_dim * sizeof(std::uint16_t));
        ++row;
      };
      for (std::size_t i = 0; i < sel.block_ids.size(); ++i) {
        ids_out[(layer * kv_heads + h) * budget + i] =
            static_cast<std::int64_t>(sel.block_ids[i]);
        const std::size_t phys =
            static_cast<std::size_t>(table[layer * table_stride + sel.block_ids[i]]);
        for (std::size_t t = 0; t < block_tokens; ++t)
          copy_row(pool + (phys * block_tokens + t) * token_values);
      }
      const std::size_t tail_phys = static_cast<std::size_t>(tail_block[layer]);
      for (std::size_t t = 0; t < tail_len; ++t)
        copy_row(pool + (tail_phys * block_tokens + t) * token_values);
      sa::AttentionProblem p{packed.data(), q, tokens, group, 1, head_dim, scale};
      const auto o = sa::attention_reference(p);
      std::memcpy(out + (layer * query_heads + h * group) * head_dim, o.data(),
                  o.size() * sizeof(float));
    } catch (const std::exception&) {
      failed |= 1;
    }
  }
  return failed ? -1 : 0;
}

// The per-unit body of saref_sparse_step over a caller's list of units, so
// that units of sequence-layers with different block counts share one
// parallel loop. Unit layout as sao_unit (oracle/sa_oracle.h): the unit's
// sealed blocks in logical order followed by its open tail block.
struct saref_unit {
  const std::uint16_t* blocks;
  const float* reps;
  const float* query;
  std::size_t nb;
  std::size_t tail_len;
  std::size_t kv_head;
  std::int64_t* ids_out;
  float* out;
};

int saref_sparse_units(const saref_unit* units, std::size_t n, std::size_t query_heads,
                       std::size_t kv_heads, std::size_t head_dim, std::size_t block_tokens,
                       std::size_t budget, std::size_t init, std::size_t local, float scale,
                       int threads) {
  if (kv_heads == 0 || query_heads % kv_heads != 0) return -1;
  const std::size_t group = query_heads / kv_heads;
  const std::size_t token_values = 2 * kv_heads * head_dim;
  int failed = 0;
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1) reduction(| : failed)
#endif
  for (long i = 0; i < static_cast<long>(n); ++i) {
    const saref_unit& u = units[i];
    const std::size_t h = u.kv_head;
    try {
      const float* q = u.query + h * group * head_dim;
      const float* r = u.reps + h * group * u.nb * head_dim;
      const std::size_t eff = budget < u.nb ? budget : u.nb;
      const std::size_t ini = init < eff ? init : eff;
      const std::size_t loc = local < eff - ini ? local : eff - ini;
      const auto sel = sa::select_shared_blocks(q, r, group, u.nb, head_dim, eff, ini, loc);
      const std::size_t tokens = sel.block_ids.size() * block_tokens + u.tail_len;
      std::vector<std::uint16_t> packed(tokens * 2 * head_dim);
      std::size_t row = 0;
      auto copy_rows = [&](std::size_t block, std::size_t rows) {
        for (std::size_t t = 0; t < rows; ++t, ++row) {
          const std::uint16_t* src = u.blocks + (block * block_tokens + t) * token_values;
          std::memcpy(&packed[row * 2 * head_dim], src + h * head_dim,
                      head_dim * sizeof(std::uint16_t));
          std::memcpy(&packed[row * 2 * head_dim + head_dim],
                      src + kv_heads * head_dim + h * head_dim, head_dim * sizeof(std::uint16_t));
        }
      };
      for (std::size_t k = 0; k < sel.block_ids.size(); ++k) {
        u.ids_out[k] = static_cast<std::int64_t>(sel.block_ids[k]);
        copy_rows(sel.block_ids[k], block_tokens);
      }
      copy_rows(u.nb, u.tail_len);
      sa::AttentionProblem p{packed.data(), q, tokens, group, 1, head_dim, scale};
      const auto o = sa::attention_reference(p);
      std::memcpy(u.out, o.data(), o.size() * sizeof(float));
    } catch (const std::exception&) {
      failed |= 1;
    }
  }
  return failed ? -1 : 0;
}

// Representatives of consecutive blocks, each block its own call of the
// reference's build_local_causal_representatives (T = block_tokens), as the
// online seal builds them (cpp/src/online_seal_main.cpp:41). prompt_queries
// [query_heads][blocks * block_tokens][head_dim]; kv token rows; values_out
// [query_heads][blocks][head_dim]; OpenMP over blocks.
int saref_build_reps_per_block(const float* prompt_queries, const std::uint16_t* kv,
                               std::size_t blocks, std::size_t query_heads,
                               std::size_t kv_heads, std::size_t head_dim,
                               std::size_t block_tokens, std::size_t local_window,
                               std::size_t topk, float* values_out, int threads) {
  const std::size_t tokens = blocks * block_tokens;
  const std::size_t token_values = 2 * kv_heads * head_dim;
  int failed = 0;
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(dynamic, 4) reduction(| : failed)
#endif
  for (long b = 0; b < static_cast<long>(blocks); ++b) {
    try {
      std::vector<float> pq(query_heads * block_tokens * head_dim);
      for (std::size_t h = 0; h < query_heads; ++h)
        std::memcpy(&pq[h * block_tokens * head_dim],
                    prompt_queries + (h * tokens + static_cast<std::size_t>(b) * block_tokens) *
                                         head_dim,
                    block_tokens * head_dim * sizeof(float));
      const auto r = sa::build_local_causal_representatives(
          pq.data(), kv + static_cast<std::size_t>(b) * block_tokens * token_values,
          block_tokens, query_heads, kv_heads, head_dim, block_tokens, local_window, topk);
      for (std::size_t h = 0; h < query_heads; ++h)
        std::memcpy(values_out + (h * blocks + static_cast<std::size_t>(b)) * head_dim,
                    r.values.data() + h * head_dim, head_dim * sizeof(float));
    } catch (const std::exception&) {
      failed |= 1;
    }
  }
  return failed ? -1 : 0;
}

int saref_max_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

}  // extern "C"
