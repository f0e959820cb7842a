/*
 * sa_oracle.h -- CPU restatement of the reference's decode-time sparse-KV path.
 *
 * TEST INFRASTRUCTURE ONLY. This is the parity checker, never the product:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load it. The product library (libsa_b200.so) neither links nor calls it.
 *
 * Every function restates one piece of the reference (ZjuXxxc/solidattention-repro,
 * paths relative to that project) in plain C, keeping the reference's
 * floating-point operation order so that results are bit-identical to the
 * reference compiled with g++ -O2 on x86-64 (no FMA contraction):
 *
 *   sao_half_to_float          cpp/src/attention_reference.cpp:30-53
 *   sao_ref_float_to_half      cpp/src/attention_reference.cpp:11-28 (non-RNE;
 *                              only to regenerate the reference's own fixtures)
 *   sao_attention              cpp/src/attention_reference.cpp:55-96
 *   sao_select_shared_blocks   cpp/src/selection.cpp:96-147
 *   sao_build_representatives  cpp/src/selection.cpp:12-94
 *   sao_c1_fixture             cpp/src/attention_main.cpp:131-156
 *   sao_c21_fixture            cpp/src/selection_main.cpp:113-154
 *   sao_gather_packed          cpp/src/selection_main.cpp:196-218 and
 *                              cpp/src/qwen_chain_main.cpp:360-395 (token order)
 *   sao_lifecycle_run          cpp/src/kv_lifecycle_main.cpp:25-113
 *   sao_slot_correct           cpp/src/pipeline_main.cpp:686-717
 *   sao_head_norm_rope         cpp/src/qwen_layer_main.cpp:146-183
 *
 * Parity of this restatement is pinned against the reference compiled from
 * its own sources (oracle/_ref) and against the reference's published known
 * answers (tests/golden/).
 */
#ifndef SA_ORACLE_H
#define SA_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

float sao_half_to_float(uint16_t value);
uint16_t sao_float_to_half_rne(float value);
uint16_t sao_ref_float_to_half(float value);
void sao_half_to_float_n(const uint16_t* in, float* out, size_t n);
void sao_float_to_half_rne_n(const float* in, uint16_t* out, size_t n);

/* GQA attention over a packed token-major buffer [tokens][2][kv_heads][head_dim]
 * (K plane, then V plane per token). out: [query_heads][head_dim] FP32.
 * Returns 0, or -1 on the reference's invalid-dimension condition. */
int sao_attention(const uint16_t* interleaved_kv, const float* query,
                  size_t tokens, size_t query_heads, size_t kv_heads,
                  size_t head_dim, float scale, float* out);

/* Representative scoring + init/local forcing + stable top-k.
 * query [query_heads][head_dim], representatives [query_heads][blocks][head_dim].
 * block_ids_out receives the chosen ids ascending (capacity budget_blocks),
 * *n_ids_out their count; scores_out (nullable) receives mean_head_scores[blocks].
 * Returns 0 or -1 on invalid dimensions. */
int sao_select_shared_blocks(const float* query, const float* representatives,
                             size_t query_heads, size_t blocks,
                             size_t head_dim, size_t budget_blocks,
                             size_t init_blocks, size_t local_blocks,
                             int64_t* block_ids_out, size_t* n_ids_out,
                             float* scores_out);

/* Per-KV-head selection: the unmodified shared selection applied to each
 * group of `group` consecutive query heads (group == query_heads is the
 * reference's shared mode). ids_out: [query_heads/group][budget_blocks].
 * scores_out (nullable): [query_heads/group][blocks]. */
int sao_select_grouped(const float* query, const float* representatives,
                       size_t query_heads, size_t group, size_t blocks,
                       size_t head_dim, size_t budget_blocks,
                       size_t init_blocks, size_t local_blocks,
                       int64_t* ids_out, float* scores_out);

/* Local-causal received-mass representatives.
 * prompt_queries [query_heads][tokens][head_dim] FP32; interleaved_kv as above.
 * values_out [query_heads][tokens/block_tokens][head_dim];
 * offsets_out [query_heads][tokens/block_tokens][topk] (in-block offsets,
 * rank order); received_out (nullable) [query_heads][tokens]. */
int sao_build_representatives(const float* prompt_queries,
                              const uint16_t* interleaved_kv, size_t tokens,
                              size_t query_heads, size_t kv_heads,
                              size_t head_dim, size_t block_tokens,
                              size_t local_window, size_t topk,
                              float* values_out, int64_t* offsets_out,
                              float* received_out);

/* The reference's deterministic fixtures. */
void sao_c1_fixture(uint16_t* kv /* 128*2*8*128 */, float* query /* 16*128 */);
void sao_c21_fixture(uint16_t* kv /* 512*2*8*128 */,
                     float* prompt_queries /* 16*512*128 */,
                     float* query /* 16*128: last prompt position */);

/* Packed gather: selected blocks (block ids into `store`, ascending as the
 * selector returns them) followed by `tail_tokens` rows of `tail`, copied into
 * `out` as one token-major buffer. token_values = 2*kv_heads*head_dim. */
void sao_gather_packed(const uint16_t* store, const int64_t* block_ids,
                       size_t n_blocks, size_t block_tokens,
                       const uint16_t* tail, size_t tail_tokens,
                       size_t token_values, uint16_t* out);

/* KV lifecycle: append decode tokens to each layer's tail and seal the oldest
 * block while tail >= local_tokens + block_tokens. Token bytes follow the
 * reference's synthetic formula (layer*1009 + token*37 + value*13) & 0xffff.
 * store (nullable) has room for layers*capacity_blocks blocks; every sealed
 * block is written at (layer*capacity_blocks + initial_blocks + sealed)*block.
 * rep_indices_out (nullable) receives [total_seals][q_heads][4].
 * Results: per-layer sealed counts/generation, final tail tokens, audits. */
typedef struct {
  size_t sealed_total;
  size_t representative_audits;
  size_t tail_tokens_layer0;
  size_t generation_layer0;
  size_t capacity_blocks;
} sao_lifecycle_result;

int sao_lifecycle_run(size_t layers, size_t q_heads, size_t kv_heads,
                      size_t head_dim, size_t block_tokens,
                      size_t local_tokens, size_t decode_tokens,
                      size_t initial_blocks, uint16_t* store,
                      int64_t* rep_indices_out, sao_lifecycle_result* result);

/* One CPU decode step over `layers` layers (see sa_oracle.c). pool
 * [pool_blocks][block_tokens][2][kv_heads][head_dim] FP16; table
 * [layers][table_stride]; reps [layers][query_heads][blocks][head_dim];
 * query [layers][query_heads][head_dim]; tail_block [layers];
 * ids_out [layers][kv_heads][budget]; out [layers][query_heads][head_dim]. */
int sao_sparse_step(const uint16_t* pool, const int32_t* table,
                    size_t table_stride, const float* reps, const float* query,
                    const int32_t* tail_block, size_t tail_len, size_t layers,
                    size_t query_heads, size_t kv_heads, size_t head_dim,
                    size_t block_tokens, size_t blocks, size_t budget,
                    size_t init, size_t local, float scale, int threads,
                    int64_t* ids_out, float* out);

/* One decode work unit of the CPU path: a (sequence, layer, KV head).
 * blocks: [nb + 1][block_tokens][2][kv_heads][head_dim] FP16, the nb sealed
 * blocks in logical order followed by the open tail block (tail_len rows
 * valid); reps: [query_heads][nb][head_dim]; query: [query_heads][head_dim]
 * (every head of the sequence-layer; the unit uses its KV head's group);
 * ids_out: [budget]; out: [query_heads / kv_heads][head_dim]. */
typedef struct {
  const uint16_t* blocks;
  const float* reps;
  const float* query;
  size_t nb;
  size_t tail_len;
  size_t kv_head;
  int64_t* ids_out;
  float* out;
} sao_unit;

/* The per-unit body of sao_sparse_step over a list of units, `threads`
 * OpenMP threads over the units. */
int sao_sparse_units(const sao_unit* units, size_t n, size_t query_heads, size_t kv_heads,
                     size_t head_dim, size_t block_tokens, size_t budget, size_t init,
                     size_t local, float scale, int threads);

/* Representatives of `blocks` consecutive blocks, each built alone as the
 * online seal does (cpp/src/online_seal_main.cpp:41: one call of
 * build_local_causal_representatives per block, T = block_tokens):
 * prompt_queries [query_heads][blocks * block_tokens][head_dim], kv token
 * rows [blocks * block_tokens][2][kv_heads][head_dim] FP16, values_out
 * [query_heads][blocks][head_dim]; `threads` OpenMP threads over blocks. */
int sao_build_reps_per_block(const float* prompt_queries, const uint16_t* kv, size_t blocks,
                             size_t query_heads, size_t kv_heads, size_t head_dim,
                             size_t block_tokens, size_t local_window, size_t topk,
                             float* values_out, int threads);

/* The lifecycle's representative audit (kv_lifecycle_main.cpp:93-103): four
 * in-block offsets by descending score, first maximum wins. */
void sao_top4_first_max(const float* scores, size_t block_tokens, int64_t* out);

/* History-prediction slot correction, compare_prediction
 * (cpp/src/pipeline_main.cpp:686-717) per unit, generalised to empty slots
 * (-1, always overwritten) and to selections shorter than the window (the
 * freed slots beyond the misses are emptied). selected [units][budget]
 * ascending with counts [units]; slots [units][budget] corrected in place;
 * misses / replace [units][budget] -1 padded; stats [units][2] = hits, misses. */
void sao_slot_correct(const int32_t* selected, const int32_t* counts, int32_t* slots,
                      int32_t* misses, int32_t* replace, int32_t* stats, size_t units,
                      size_t budget);

/* Dense per-block attention mass of audit_dense_selection
 * (cpp/src/pipeline_main.cpp:517-543) for one dense token set: keys
 * [tokens] rows of head_dim FP16 values, `key_stride` elements apart; query
 * [heads][head_dim] FP32. Per head: FP32 logits (sequential dot, then
 * * scale), the FP32 maximum, expf of the shifted logits, a double
 * denominator; each token adds p / denominator / heads to
 * block_mass[token / block_tokens] (double, zeroed here). */
void sao_dense_block_mass(const uint16_t* keys, size_t key_stride, size_t tokens,
                          const float* query, size_t heads, size_t head_dim,
                          size_t block_tokens, float scale, double* block_mass);

/* The audit's two figures for one selection (pipeline_main.cpp:544-569):
 * selected_mass = the summed mass of the selected blocks plus `extra_mass`
 * (the always-attended open tail); recall = hits / the oracle set's size,
 * where the oracle set is the forced blocks ([0, init) and the last `local`
 * of `blocks`) filled to `budget` from a stable descending sort of the mass.
 * The reference's fixed case is blocks 16, init 1, local 1, budget 4. */
void sao_audit_selection(const double* block_mass, size_t blocks, const int32_t* selected,
                         size_t count, size_t budget, size_t init, size_t local,
                         double extra_mass, double* selected_mass, double* recall);

/* Per-head RMS norm then rotate-half RoPE on rows of 128 floats, in place:
 * head_rms (cpp/src/qwen_layer_main.cpp:146-161, pairwise sum of squares,
 * strides 64..1) and rope (:163-183) at one position. */
void sao_head_norm_rope(float* rows, size_t nrows, const float* weight, int position,
                        float theta, float eps);

/* FNV-1a over 64-bit words, as the C2.1 driver hashes representative offsets
 * (cpp/src/selection_main.cpp:167-171). */
uint64_t sao_fnv_offsets(const int64_t* values, size_t n);

#ifdef __cplusplus
}
#endif

#endif
