/*
 * sa_oracle.c -- CPU restatement of the reference's decode-time sparse-KV path.
 *
 * TEST INFRASTRUCTURE ONLY (see sa_oracle.h). Compiled with
 * -O2 -ffp-contract=off so that every float multiply and add rounds on its
 * own, in the order the reference writes them.
 */
#include "sa_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

static uint32_t f32_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof u);
  return u;
}

static float bits_f32(uint32_t u) {
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

/* attention_reference.cpp:30-53: exact FP16 -> FP32, subnormals normalised. */
float sao_half_to_float(uint16_t value) {
  const uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
  uint32_t exponent = (value >> 10) & 0x1fu;
  uint32_t mantissa = value & 0x3ffu;
  if (exponent == 0) {
    if (mantissa == 0) return bits_f32(sign);
    int shift = 0;
    while ((mantissa & 0x400u) == 0) {
      mantissa <<= 1;
      ++shift;
    }
    mantissa &= 0x3ffu;
    return bits_f32(sign | ((uint32_t)(127 - 14 - shift) << 23) | (mantissa << 13));
  }
  if (exponent == 31) return bits_f32(sign | 0x7f800000u | (mantissa << 13));
  return bits_f32(sign | ((exponent - 15 + 127) << 23) | (mantissa << 13));
}

/* IEEE round-to-nearest-even FP32 -> FP16 (what cvt.rn.f16.f32, _Float16 and
 * numpy's astype(float16) do). Used to generate inputs and to check the
 * device pack; the reference's own device pack is cvt.rn
 * (cpp/src/qwen_layer_main.cpp:270-281). */
uint16_t sao_float_to_half_rne(float value) {
  const uint32_t x = f32_bits(value);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t magnitude = x & 0x7fffffffu;
  if (magnitude >= 0x7f800000u) {
    if (magnitude > 0x7f800000u)
      return (uint16_t)(sign | 0x7e00u | ((magnitude >> 13) & 0x3ffu));
    return (uint16_t)(sign | 0x7c00u);
  }
  const uint32_t biased = magnitude >> 23;
  if (biased >= 113) { /* normal half range (or overflow) */
    uint32_t half = ((biased - 112) << 10) | ((magnitude >> 13) & 0x3ffu);
    const uint32_t rest = magnitude & 0x1fffu;
    if (rest > 0x1000u || (rest == 0x1000u && (half & 1u))) ++half;
    if (half >= 0x7c00u) return (uint16_t)(sign | 0x7c00u);
    return (uint16_t)(sign | half);
  }
  /* subnormal half: value = m * 2^(biased-150), unit 2^-24 */
  const uint32_t shift = 126 - biased;
  if (shift >= 25) return sign;
  const uint32_t m = (magnitude & 0x7fffffu) | 0x800000u;
  uint32_t half = m >> shift;
  const uint32_t rest = m & ((1u << shift) - 1u);
  const uint32_t halfway = 1u << (shift - 1);
  if (rest > halfway || (rest == halfway && (half & 1u))) ++half;
  return (uint16_t)(sign | half);
}

/* attention_reference.cpp:11-28: the reference's truncating conversion. It
 * ORs the rounded mantissa into the exponent field, so a mantissa carry is
 * lost on odd exponents. Only used to regenerate the reference's own sin/cos
 * fixtures, whose known answers are defined over these exact bytes. */
uint16_t sao_ref_float_to_half(float value) {
  const uint32_t bits = f32_bits(value);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const int exponent = (int)((bits >> 23) & 0xffu) - 127 + 15;
  uint32_t mantissa = bits & 0x7fffffu;
  if (exponent <= 0) {
    if (exponent < -10) return (uint16_t)sign;
    mantissa = (mantissa | 0x800000u) >> (1 - exponent);
    return (uint16_t)(sign | ((mantissa + 0x1000u) >> 13));
  }
  if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
  return (uint16_t)(sign | ((uint32_t)exponent << 10) | ((mantissa + 0x1000u) >> 13));
}

void sao_half_to_float_n(const uint16_t* in, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = sao_half_to_float(in[i]);
}

void sao_float_to_half_rne_n(const float* in, uint16_t* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = sao_float_to_half_rne(in[i]);
}

/* attention_reference.cpp:55-96. Two passes per query head: logits with a
 * running maximum, then exp/sum over every logit, then weight = p/den and a
 * token-ordered accumulation of weight*v. */
int sao_attention(const uint16_t* kv, const float* query, size_t tokens,
                  size_t query_heads, size_t kv_heads, size_t head_dim,
                  float scale, float* out) {
  if (kv_heads == 0 || query_heads % kv_heads != 0 || tokens == 0) return -1;
  const size_t groups = query_heads / kv_heads;
  float* logits = (float*)malloc(tokens * sizeof(float));
  if (!logits) return -1;
  for (size_t i = 0; i < query_heads * head_dim; ++i) out[i] = 0.0f;
  for (size_t qh = 0; qh < query_heads; ++qh) {
    const size_t kvh = qh / groups;
    float maximum = -INFINITY;
    for (size_t t = 0; t < tokens; ++t) {
      const size_t base = t * 2 * kv_heads * head_dim + kvh * head_dim;
      float dot = 0.0f;
      for (size_t d = 0; d < head_dim; ++d)
        dot += query[qh * head_dim + d] * sao_half_to_float(kv[base + d]);
      logits[t] = dot * scale;
      if (maximum < logits[t]) maximum = logits[t]; /* std::max(maximum, l) */
    }
    float denominator = 0.0f;
    for (size_t t = 0; t < tokens; ++t) {
      logits[t] = expf(logits[t] - maximum);
      denominator += logits[t];
    }
    for (size_t t = 0; t < tokens; ++t) {
      const size_t vbase = t * 2 * kv_heads * head_dim + kv_heads * head_dim +
                           kvh * head_dim;
      const float weight = logits[t] / denominator;
      for (size_t d = 0; d < head_dim; ++d)
        out[qh * head_dim + d] += weight * sao_half_to_float(kv[vbase + d]);
    }
  }
  free(logits);
  return 0;
}

/* Stable descending order of indices 0..n-1 by key: the result of
 * std::stable_sort(iota, key[l] > key[r]) for non-NaN keys, i.e. descending
 * key with ties kept in ascending index order. Bottom-up merge sort. */
static void stable_order_desc(const float* key, size_t n, size_t* order) {
  size_t* tmp = (size_t*)malloc((n ? n : 1) * sizeof(size_t));
  for (size_t i = 0; i < n; ++i) order[i] = i;
  for (size_t width = 1; width < n; width *= 2) {
    for (size_t lo = 0; lo < n; lo += 2 * width) {
      size_t mid = lo + width < n ? lo + width : n;
      size_t hi = lo + 2 * width < n ? lo + 2 * width : n;
      size_t a = lo, b = mid, o = lo;
      while (a < mid && b < hi) {
        /* take from the right run only when strictly greater: stable */
        if (key[order[b]] > key[order[a]]) tmp[o++] = order[b++];
        else tmp[o++] = order[a++];
      }
      while (a < mid) tmp[o++] = order[a++];
      while (b < hi) tmp[o++] = order[b++];
    }
    memcpy(order, tmp, n * sizeof(size_t));
  }
  free(tmp);
}

/* selection.cpp:96-147. */
int sao_select_shared_blocks(const float* query, const float* reps,
                             size_t query_heads, size_t blocks,
                             size_t head_dim, size_t budget, size_t init,
                             size_t local, int64_t* ids_out, size_t* n_ids,
                             float* scores_out) {
  if (!query || !reps || query_heads == 0 || blocks == 0 || head_dim == 0 ||
      budget == 0 || budget > blocks || init + local > budget)
    return -1;
  float* scores = (float*)calloc(blocks, sizeof(float));
  unsigned char* chosen = (unsigned char*)calloc(blocks, 1);
  size_t* ranked = (size_t*)malloc(blocks * sizeof(size_t));
  for (size_t h = 0; h < query_heads; ++h) {
    for (size_t b = 0; b < blocks; ++b) {
      float dot = 0.0f;
      const float* r = reps + (h * blocks + b) * head_dim;
      for (size_t d = 0; d < head_dim; ++d) dot += query[h * head_dim + d] * r[d];
      scores[b] += dot / (float)query_heads;
    }
  }
  const size_t n_init = init < blocks ? init : blocks;
  const size_t n_local = local < blocks ? local : blocks;
  for (size_t b = 0; b < n_init; ++b) chosen[b] = 1;
  for (size_t b = blocks - n_local; b < blocks; ++b) chosen[b] = 1;
  stable_order_desc(scores, blocks, ranked);
  size_t count = 0;
  for (size_t b = 0; b < blocks; ++b) count += chosen[b];
  for (size_t i = 0; i < blocks; ++i) {
    if (count == budget) break;
    if (!chosen[ranked[i]]) {
      chosen[ranked[i]] = 1;
      ++count;
    }
  }
  size_t n = 0;
  for (size_t b = 0; b < blocks; ++b)
    if (chosen[b]) ids_out[n++] = (int64_t)b;
  *n_ids = n;
  if (scores_out) memcpy(scores_out, scores, blocks * sizeof(float));
  free(scores);
  free(chosen);
  free(ranked);
  return 0;
}

/* Per-KV-head use of the unmodified shared selection: each group of `group`
 * query heads is a contiguous [group][blocks][head_dim] slice of the
 * representatives, so the reference function applies to that slice as is. */
int sao_select_grouped(const float* query, const float* reps,
                       size_t query_heads, size_t group, size_t blocks,
                       size_t head_dim, size_t budget, size_t init,
                       size_t local, int64_t* ids_out, float* scores_out) {
  if (group == 0 || query_heads % group != 0) return -1;
  const size_t groups = query_heads / group;
  for (size_t g = 0; g < groups; ++g) {
    size_t n = 0;
    const int rc = sao_select_shared_blocks(
        query + g * group * head_dim, reps + g * group * blocks * head_dim,
        group, blocks, head_dim, budget, init, local, ids_out + g * budget, &n,
        scores_out ? scores_out + g * blocks : NULL);
    if (rc != 0 || n != budget) return -1;
  }
  return 0;
}

/* selection.cpp:12-94. */
int sao_build_representatives(const float* prompt_queries, const uint16_t* kv,
                              size_t tokens, size_t query_heads,
                              size_t kv_heads, size_t head_dim,
                              size_t block_tokens, size_t local_window,
                              size_t topk, float* values_out,
                              int64_t* offsets_out, float* received_out) {
  if (!prompt_queries || !kv || tokens == 0 || kv_heads == 0 ||
      query_heads % kv_heads != 0 || block_tokens == 0 ||
      tokens % block_tokens != 0 || local_window == 0 || topk == 0 ||
      topk > block_tokens)
    return -1;
  const size_t groups = query_heads / kv_heads;
  const size_t blocks = tokens / block_tokens;
  const float scale = 1.0f / sqrtf((float)head_dim);
  float* received = (float*)calloc(query_heads * tokens, sizeof(float));
  float* logits = (float*)malloc(local_window * sizeof(float));
  for (size_t h = 0; h < query_heads; ++h) {
    const size_t kvh = h / groups;
    for (size_t p = 0; p < tokens; ++p) {
      const size_t start = p + 1 > local_window ? p + 1 - local_window : 0;
      const size_t count = p - start + 1;
      float maximum = -INFINITY;
      for (size_t w = 0; w < count; ++w) {
        const size_t key_base = (start + w) * 2 * kv_heads * head_dim + kvh * head_dim;
        float dot = 0.0f;
        for (size_t d = 0; d < head_dim; ++d)
          dot += prompt_queries[(h * tokens + p) * head_dim + d] *
                 sao_half_to_float(kv[key_base + d]);
        logits[w] = dot * scale;
        if (maximum < logits[w]) maximum = logits[w];
      }
      float denominator = 0.0f;
      for (size_t w = 0; w < count; ++w) {
        logits[w] = expf(logits[w] - maximum);
        denominator += logits[w];
      }
      for (size_t w = 0; w < count; ++w)
        received[h * tokens + start + w] += logits[w] / denominator;
    }
  }
  size_t* order = (size_t*)malloc(block_tokens * sizeof(size_t));
  for (size_t h = 0; h < query_heads; ++h) {
    const size_t kvh = h / groups;
    for (size_t b = 0; b < blocks; ++b) {
      stable_order_desc(received + h * tokens + b * block_tokens, block_tokens, order);
      for (size_t r = 0; r < topk; ++r)
        offsets_out[(h * blocks + b) * topk + r] = (int64_t)order[r];
      for (size_t d = 0; d < head_dim; ++d) {
        float value = 0.0f;
        for (size_t r = 0; r < topk; ++r) {
          const size_t token = b * block_tokens + order[r];
          value += sao_half_to_float(kv[token * 2 * kv_heads * head_dim + kvh * head_dim + d]);
        }
        values_out[(h * blocks + b) * head_dim + d] = value / (float)topk;
      }
    }
  }
  if (received_out) memcpy(received_out, received, query_heads * tokens * sizeof(float));
  free(order);
  free(logits);
  free(received);
  return 0;
}

/* attention_main.cpp:131-156 (C1: 128 tokens, 16/8 heads, head_dim 128). */
void sao_c1_fixture(uint16_t* kv, float* query) {
  const size_t tokens = 128, kv_heads = 8, head_dim = 128, query_heads = 16;
  for (size_t t = 0; t < tokens; ++t)
    for (size_t half = 0; half < 2; ++half)
      for (size_t h = 0; h < kv_heads; ++h)
        for (size_t d = 0; d < head_dim; ++d) {
          const size_t index = t * 2 * kv_heads * head_dim + half * kv_heads * head_dim +
                               h * head_dim + d;
          const float value =
              sinf((float)(t * 17 + h * 13 + d * 3 + half * 19) * 0.013f) * 0.25f;
          kv[index] = sao_ref_float_to_half(value);
        }
  for (size_t i = 0; i < query_heads * head_dim; ++i)
    query[i] = cosf((float)(i * 7) * 0.009f) * 0.2f;
}

/* selection_main.cpp:113-154 (C2.1: 512 tokens, 16/8 heads, head_dim 128). */
void sao_c21_fixture(uint16_t* kv, float* prompt_queries, float* query) {
  const size_t tokens = 512, kv_heads = 8, head_dim = 128, query_heads = 16;
  const size_t groups = query_heads / kv_heads;
  for (size_t t = 0; t < tokens; ++t)
    for (size_t half = 0; half < 2; ++half)
      for (size_t h = 0; h < kv_heads; ++h)
        for (size_t d = 0; d < head_dim; ++d) {
          const size_t index = t * 2 * kv_heads * head_dim + half * kv_heads * head_dim +
                               h * head_dim + d;
          const float value =
              sinf((float)(t * 11 + h * 17 + d * 5 + half * 23) * 0.007f) * 0.2f;
          kv[index] = sao_ref_float_to_half(value);
        }
  for (size_t qh = 0; qh < query_heads; ++qh) {
    const size_t kvh = qh / groups;
    for (size_t t = 0; t < tokens; ++t)
      for (size_t d = 0; d < head_dim; ++d) {
        const size_t key_offset = t * 2 * kv_heads * head_dim + kvh * head_dim + d;
        const float a = sao_half_to_float(kv[key_offset]) * 0.85f;
        const float b = cosf((float)(qh * 19 + t * 7 + d * 3) * 0.011f) * 0.03f;
        prompt_queries[(qh * tokens + t) * head_dim + d] = a + b;
      }
  }
  for (size_t qh = 0; qh < query_heads; ++qh)
    memcpy(query + qh * head_dim, prompt_queries + (qh * tokens + tokens - 1) * head_dim,
           head_dim * sizeof(float));
}

void sao_gather_packed(const uint16_t* store, const int64_t* block_ids,
                       size_t n_blocks, size_t block_tokens,
                       const uint16_t* tail, size_t tail_tokens,
                       size_t token_values, uint16_t* out) {
  const size_t block_values = block_tokens * token_values;
  for (size_t i = 0; i < n_blocks; ++i)
    memcpy(out + i * block_values, store + (size_t)block_ids[i] * block_values,
           block_values * sizeof(uint16_t));
  if (tail_tokens)
    memcpy(out + n_blocks * block_values, tail, tail_tokens * token_values * sizeof(uint16_t));
}

/* kv_lifecycle_main.cpp:25-113 without the O_DIRECT/liburing I/O. */
typedef struct {
  uint16_t* kv;    /* [capacity tokens][token_values] */
  float* score;    /* [q_heads][capacity tokens] */
  size_t tokens;
} lifecycle_tail;

int sao_lifecycle_run(size_t layers, size_t q_heads, size_t kv_heads,
                      size_t head_dim, size_t block_tokens, size_t local_tokens,
                      size_t decode_tokens, size_t initial_blocks,
                      uint16_t* store, int64_t* rep_indices_out,
                      sao_lifecycle_result* result) {
  if (block_tokens < 4 || layers == 0 || q_heads == 0) return -1;
  const size_t token_values = 2 * kv_heads * head_dim;
  const size_t block_values = block_tokens * token_values;
  const size_t capacity_blocks = initial_blocks + (decode_tokens + 31) / 32 + 1;
  const size_t tail_capacity = local_tokens + block_tokens + 1;
  lifecycle_tail* tails = (lifecycle_tail*)calloc(layers, sizeof(lifecycle_tail));
  size_t* sealed = (size_t*)calloc(layers, sizeof(size_t));
  size_t* generation = (size_t*)calloc(layers, sizeof(size_t));
  for (size_t l = 0; l < layers; ++l) {
    tails[l].kv = (uint16_t*)malloc(tail_capacity * token_values * sizeof(uint16_t));
    tails[l].score = (float*)calloc(q_heads * tail_capacity, sizeof(float));
  }
  size_t writes = 0, audits = 0;
  /* append(): push the token's values and a zero score, then every resident
   * token's score grows by ((head+3)*(old+5)+token)%97/97 (:31-45). */
#define SAO_APPEND(L, TOKEN)                                                      \
  do {                                                                            \
    lifecycle_tail* tl = &tails[L];                                               \
    for (size_t v = 0; v < token_values; ++v)                                     \
      tl->kv[tl->tokens * token_values + v] =                                     \
          (uint16_t)(((L) * 1009 + (TOKEN) * 37 + v * 13) & 0xffffu);             \
    ++tl->tokens;                                                                 \
    for (size_t h = 0; h < q_heads; ++h) {                                        \
      tl->score[h * tail_capacity + tl->tokens - 1] = 0.0f;                       \
      for (size_t old = 0; old < tl->tokens; ++old)                               \
        tl->score[h * tail_capacity + old] +=                                     \
            (float)(((h + 3) * (old + 5) + (TOKEN)) % 97) / 97.0f;                \
    }                                                                             \
  } while (0)
  for (size_t l = 0; l < layers; ++l)
    for (size_t t = 0; t < local_tokens; ++t) SAO_APPEND(l, t);
  for (size_t step = 0; step < decode_tokens; ++step) {
    for (size_t l = 0; l < layers; ++l) {
      lifecycle_tail* tl = &tails[l];
      SAO_APPEND(l, local_tokens + step);
      while (tl->tokens >= local_tokens + block_tokens) {
        for (size_t h = 0; h < q_heads; ++h) {
          size_t top[4] = {0, 0, 0, 0};
          const float* s = tl->score + h * tail_capacity;
          for (size_t rank = 0; rank < 4; ++rank) {
            size_t best = block_tokens;
            for (size_t t = 0; t < block_tokens; ++t) {
              int taken = 0;
              for (size_t r = 0; r < rank; ++r) taken |= top[r] == t;
              if (taken) continue;
              if (best == block_tokens || s[t] > s[best]) best = t;
            }
            top[rank] = best;
          }
          audits += top[0] < block_tokens;
          if (rep_indices_out)
            for (size_t r = 0; r < 4; ++r)
              rep_indices_out[(writes * q_heads + h) * 4 + r] = (int64_t)top[r];
        }
        if (store)
          memcpy(store + (l * capacity_blocks + initial_blocks + sealed[l]) * block_values,
                 tl->kv, block_values * sizeof(uint16_t));
        memmove(tl->kv, tl->kv + block_values,
                (tl->tokens - block_tokens) * token_values * sizeof(uint16_t));
        for (size_t h = 0; h < q_heads; ++h)
          memmove(tl->score + h * tail_capacity, tl->score + h * tail_capacity + block_tokens,
                  (tl->tokens - block_tokens) * sizeof(float));
        tl->tokens -= block_tokens;
        ++sealed[l];
        ++generation[l];
        ++writes;
      }
    }
  }
#undef SAO_APPEND
  result->sealed_total = writes;
  result->representative_audits = audits;
  result->tail_tokens_layer0 = tails[0].tokens;
  result->generation_layer0 = generation[0];
  result->capacity_blocks = capacity_blocks;
  for (size_t l = 0; l < layers; ++l) {
    free(tails[l].kv);
    free(tails[l].score);
  }
  free(tails);
  free(sealed);
  free(generation);
  return 0;
}

/* audit_dense_selection, dense part (cpp/src/pipeline_main.cpp:517-543): per
 * head, logits[t] = (sequential FP32 dot) * scale; the FP32 maximum; each
 * logit replaced by expf(logit - maximum) and summed into a double
 * denominator; then block_mass[t / block_tokens] += p / denominator / heads in
 * double, heads in index order. */
void sao_dense_block_mass(const uint16_t* keys, size_t key_stride, size_t tokens,
                          const float* query, size_t heads, size_t head_dim,
                          size_t block_tokens, float scale, double* block_mass) {
  const size_t blocks = (tokens + block_tokens - 1) / block_tokens;
  for (size_t b = 0; b < blocks; ++b) block_mass[b] = 0.0;
  float* logits = (float*)malloc((tokens ? tokens : 1) * sizeof(float));
  for (size_t head = 0; head < heads; ++head) {
    float maximum = -INFINITY;
    for (size_t t = 0; t < tokens; ++t) {
      float dot = 0.0f;
      for (size_t d = 0; d < head_dim; ++d)
        dot += query[head * head_dim + d] * sao_half_to_float(keys[t * key_stride + d]);
      logits[t] = dot * scale;
      if (logits[t] > maximum) maximum = logits[t];
    }
    double denominator = 0.0;
    for (size_t t = 0; t < tokens; ++t) {
      logits[t] = expf(logits[t] - maximum);
      denominator += logits[t];
    }
    for (size_t t = 0; t < tokens; ++t)
      block_mass[t / block_tokens] += logits[t] / denominator / (double)heads;
  }
  free(logits);
}

/* audit_dense_selection, figures (pipeline_main.cpp:544-569). The oracle set
 * starts from the forced blocks (the reference's blocks 0 and 15) and takes
 * blocks in stable descending mass order until it holds `budget`; walking
 * that order and skipping members equals taking, `budget - forced` times, the
 * highest-mass block not yet in the set, the lowest index among equals. */
void sao_audit_selection(const double* block_mass, size_t blocks, const int32_t* selected,
                         size_t count, size_t budget, size_t init, size_t local,
                         double extra_mass, double* selected_mass, double* recall) {
  unsigned char* chosen = (unsigned char*)calloc(blocks ? blocks : 1, 1);
  size_t members = 0;
  for (size_t b = 0; b < blocks; ++b) {
    if (b < init || b + local >= blocks) {
      chosen[b] = 1;
      ++members;
    }
  }
  while (members < budget && members < blocks) {
    size_t best = blocks;
    for (size_t b = 0; b < blocks; ++b)
      if (!chosen[b] && (best == blocks || block_mass[b] > block_mass[best])) best = b;
    chosen[best] = 1;
    ++members;
  }
  double mass = 0.0;
  size_t hits = 0;
  for (size_t i = 0; i < count; ++i) {
    const int32_t b = selected[i];
    if (b < 0 || (size_t)b >= blocks) continue;
    mass += block_mass[b];
    hits += chosen[b];
  }
  *selected_mass = mass + extra_mass;
  *recall = members ? (double)hits / (double)members : 0.0;
  free(chosen);
}

uint64_t sao_fnv_offsets(const int64_t* values, size_t n) {
  uint64_t hash = 1469598103934665603ULL;
  for (size_t i = 0; i < n; ++i) {
    hash ^= (uint64_t)values[i];
    hash *= 1099511628211ULL;
  }
  return hash;
}

/* The CPU decode step of the sparse path over a list of layers, restated on
 * this file's functions: per (layer, KV-head group) the shared selector on
 * the group's slice of representatives, a packed gather of that KV head's
 * chosen blocks and tail rows, then the attention (the same flow as the
 * reference drivers, cpp/src/selection_main.cpp:178-225). Layouts as
 * oracle/ref_shim.cpp's saref_sparse_step. */
int sao_sparse_step(const uint16_t* pool, const int32_t* table,
                    size_t table_stride, const float* reps, const float* query,
                    const int32_t* tail_block, size_t tail_len, size_t layers,
                    size_t query_heads, size_t kv_heads, size_t head_dim,
                    size_t block_tokens, size_t blocks, size_t budget,
                    size_t init, size_t local, float scale, int threads,
                    int64_t* ids_out, float* out) {
  const size_t group = query_heads / kv_heads;
  const size_t token_values = 2 * kv_heads * head_dim;
  const long items = (long)(layers * kv_heads);
  int failed = 0;
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1) reduction(| : failed)
#endif
  for (long item = 0; item < items; ++item) {
    const size_t layer = (size_t)item / kv_heads;
    const size_t h = (size_t)item % kv_heads;
    const float* q = query + (layer * query_heads + h * group) * head_dim;
    const float* r = reps + (layer * query_heads + h * group) * blocks * head_dim;
    int64_t* ids = ids_out + (layer * kv_heads + h) * budget;
    size_t n = 0;
    if (sao_select_shared_blocks(q, r, group, blocks, head_dim, budget, init,
                                 local, ids, &n, NULL) != 0) {
      failed |= 1;
      continue;
    }
    const size_t tokens = n * block_tokens + tail_len;
    uint16_t* packed = (uint16_t*)malloc(tokens * 2 * head_dim * sizeof(uint16_t));
    size_t row = 0;
    for (size_t i = 0; i <= n; ++i) {
      const size_t phys = i < n ? (size_t)table[layer * table_stride + (size_t)ids[i]]
                                : (size_t)tail_block[layer];
      const size_t count = i < n ? block_tokens : tail_len;
      for (size_t t = 0; t < count; ++t, ++row) {
        const uint16_t* src = pool + (phys * block_tokens + t) * token_values;
        memcpy(packed + row * 2 * head_dim, src + h * head_dim, head_dim * sizeof(uint16_t));
        memcpy(packed + row * 2 * head_dim + head_dim, src + kv_heads * head_dim + h * head_dim,
               head_dim * sizeof(uint16_t));
      }
    }
    if (sao_attention(packed, q, tokens, group, 1, head_dim, scale,
                      out + (layer * query_heads + h * group) * head_dim) != 0)
      failed |= 1;
    free(packed);
  }
  return failed ? -1 : 0;
}

/* The unit body of sao_sparse_step (select per KV-head group, packed gather
 * of the chosen blocks and the tail in ascending order as
 * selection_main.cpp:196-218 packs them, attention) over a caller's list. */
int sao_sparse_units(const sao_unit* units, size_t n, size_t query_heads, size_t kv_heads,
                     size_t head_dim, size_t block_tokens, size_t budget, size_t init,
                     size_t local, float scale, int threads) {
  if (kv_heads == 0 || query_heads % kv_heads != 0) return -1;
  const size_t group = query_heads / kv_heads;
  const size_t token_values = 2 * kv_heads * head_dim;
  int failed = 0;
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(dynamic, 1) reduction(| : failed)
#endif
  for (long i = 0; i < (long)n; ++i) {
    const sao_unit* u = &units[i];
    const size_t h = u->kv_head;
    const float* q = u->query + h * group * head_dim;
    const float* r = u->reps + h * group * u->nb * head_dim;
    const size_t eff = budget < u->nb ? budget : u->nb;
    const size_t ini = init < eff ? init : eff;
    const size_t loc = local < eff - ini ? local : eff - ini;
    size_t count = 0;
    if (sao_select_shared_blocks(q, r, group, u->nb, head_dim, eff, ini, loc, u->ids_out,
                                 &count, NULL) != 0) {
      failed |= 1;
      continue;
    }
    const size_t tokens = count * block_tokens + u->tail_len;
    uint16_t* packed = (uint16_t*)malloc((tokens ? tokens : 1) * 2 * head_dim * sizeof(uint16_t));
    size_t row = 0;
    for (size_t k = 0; k <= count; ++k) {
      const size_t block = k < count ? (size_t)u->ids_out[k] : u->nb;
      const size_t rows = k < count ? block_tokens : u->tail_len;
      for (size_t t = 0; t < rows; ++t, ++row) {
        const uint16_t* src = u->blocks + (block * block_tokens + t) * token_values;
        memcpy(packed + row * 2 * head_dim, src + h * head_dim, head_dim * sizeof(uint16_t));
        memcpy(packed + row * 2 * head_dim + head_dim, src + kv_heads * head_dim + h * head_dim,
               head_dim * sizeof(uint16_t));
      }
    }
    if (tokens == 0 || sao_attention(packed, q, tokens, group, 1, head_dim, scale, u->out) != 0)
      failed |= 1;
    free(packed);
  }
  return failed ? -1 : 0;
}

int sao_build_reps_per_block(const float* prompt_queries, const uint16_t* kv, size_t blocks,
                             size_t query_heads, size_t kv_heads, size_t head_dim,
                             size_t block_tokens, size_t local_window, size_t topk,
                             float* values_out, int threads) {
  if (blocks == 0 || block_tokens == 0 || topk == 0) return -1;
  const size_t tokens = blocks * block_tokens;
  const size_t token_values = 2 * kv_heads * head_dim;
  int failed = 0;
#ifdef _OPENMP
#pragma omp parallel for num_threads(threads) schedule(dynamic, 4) reduction(| : failed)
#endif
  for (long b = 0; b < (long)blocks; ++b) {
    float* pq = (float*)malloc(query_heads * block_tokens * head_dim * sizeof(float));
    float* values = (float*)malloc(query_heads * head_dim * sizeof(float));
    int64_t* offsets = (int64_t*)malloc(query_heads * topk * sizeof(int64_t));
    for (size_t h = 0; h < query_heads; ++h)
      memcpy(pq + h * block_tokens * head_dim,
             prompt_queries + (h * tokens + (size_t)b * block_tokens) * head_dim,
             block_tokens * head_dim * sizeof(float));
    if (sao_build_representatives(pq, kv + (size_t)b * block_tokens * token_values, block_tokens,
                                  query_heads, kv_heads, head_dim, block_tokens, local_window,
                                  topk, values, offsets, NULL) != 0)
      failed |= 1;
    else
      for (size_t h = 0; h < query_heads; ++h)
        memcpy(values_out + (h * blocks + (size_t)b) * head_dim, values + h * head_dim,
               head_dim * sizeof(float));
    free(offsets);
    free(values);
    free(pq);
  }
  return failed ? -1 : 0;
}

/* kv_lifecycle_main.cpp:93-103: the four highest-scoring in-block offsets,
 * each pass taking the first strict maximum among offsets not yet taken. */
void sao_top4_first_max(const float* scores, size_t block_tokens, int64_t* out) {
  size_t top[4] = {0, 0, 0, 0};
  for (size_t rank = 0; rank < 4; ++rank) {
    size_t best = block_tokens;
    for (size_t t = 0; t < block_tokens; ++t) {
      int taken = 0;
      for (size_t r = 0; r < rank; ++r) taken |= top[r] == t;
      if (taken) continue;
      if (best == block_tokens || scores[t] > scores[best]) best = t;
    }
    top[rank] = best;
    out[rank] = (int64_t)best;
  }
}

/* compare_prediction (cpp/src/pipeline_main.cpp:686-717): slots whose block
 * is in the new selection are hits (:690-693); the other slots, in slot
 * order, are freed (:694-696); selected blocks not resident, in selection
 * order, are misses (:698-703); the i-th miss goes to the i-th freed slot
 * (:708-710). Empty slots (-1) are never hits; freed slots beyond the misses
 * are emptied (the reference has equal counts and throws otherwise,
 * :704-706). */
void sao_slot_correct(const int32_t* selected, const int32_t* counts, int32_t* slots,
                      int32_t* misses, int32_t* replace, int32_t* stats, size_t units,
                      size_t budget) {
  for (size_t u = 0; u < units; ++u) {
    const int32_t* sel = selected + u * budget;
    int32_t* sl = slots + u * budget;
    int32_t* mi = misses + u * budget;
    int32_t* re = replace + u * budget;
    size_t count = counts[u] < 0 ? 0 : (size_t)counts[u];
    if (count > budget) count = budget;
    size_t nfree = 0, nmiss = 0;
    for (size_t s = 0; s < budget; ++s) mi[s] = re[s] = -1;
    int32_t* freed = (int32_t*)malloc(budget * sizeof(int32_t));
    for (size_t s = 0; s < budget; ++s) {
      int hit = 0;
      for (size_t i = 0; i < count && sl[s] >= 0; ++i) hit |= sel[i] == sl[s];
      if (!hit) freed[nfree++] = (int32_t)s;
    }
    for (size_t i = 0; i < count; ++i) {
      int resident = 0;
      for (size_t s = 0; s < budget; ++s) resident |= sl[s] >= 0 && sl[s] == sel[i];
      if (!resident) mi[nmiss++] = sel[i];
    }
    for (size_t k = 0; k < nfree; ++k) {
      sl[freed[k]] = k < nmiss ? mi[k] : -1;
      if (k < nmiss) re[k] = freed[k];
    }
    stats[2 * u] = (int32_t)(count - nmiss);
    stats[2 * u + 1] = (int32_t)nmiss;
    free(freed);
  }
}

/* head_rms (cpp/src/qwen_layer_main.cpp:146-161): squares reduced pairwise
 * with strides 64, 32, ..., 1 as its 128 threads do, then value *
 * rsqrt(mean + eps) * weight (the reference's device rsqrtf; 1 / sqrtf here).
 * rope (:163-183): dim d pairs with d +- 64, frequency theta^(-2 i / 128),
 * angle = position * frequency, rotate-half. */
void sao_head_norm_rope(float* rows, size_t nrows, const float* weight, int position,
                        float theta, float eps) {
  float red[128], x[128];
  for (size_t r = 0; r < nrows; ++r) {
    float* v = rows + r * 128;
    for (int t = 0; t < 128; ++t) red[t] = v[t] * v[t];
    for (int stride = 64; stride > 0; stride >>= 1)
      for (int t = 0; t < stride; ++t) red[t] += red[t + stride];
    const float inv = 1.0f / sqrtf(red[0] / 128.0f + eps);
    for (int t = 0; t < 128; ++t) x[t] = v[t] * inv * weight[t];
    for (int t = 0; t < 128; ++t) {
      const int paired = t < 64 ? t + 64 : t - 64;
      const int fi = t < 64 ? t : t - 64;
      const float freq = powf(theta, -2.0f * (float)fi / 128.0f);
      const float angle = (float)position * freq;
      const float rotated = t < 64 ? -x[paired] : x[paired];
      v[t] = x[t] * cosf(angle) + rotated * sinf(angle);
    }
  }
}
