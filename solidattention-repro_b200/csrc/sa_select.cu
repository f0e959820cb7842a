// sa_select.cu -- InfLLM representative scoring + deterministic top-k block
// selection for sm_100a.
//
// Replaces select_shared_blocks (cpp/src/selection.cpp:96-147), applied per
// group of `group` query heads (a KV head's G heads, or all QH heads for the
// reference's shared mode).
//
// Scoring keeps the reference's floating-point order exactly: per head a
// sequential head_dim dot product with separately rounded multiply and add
// (no FMA), divided by the group size and added to the block's score head by
// head. A CTA covers 128 (or, for groups under four heads, 256 or 512)
// consecutive blocks; its four warps compute different heads' dot products
// in parallel, each lane owning 4 consecutive blocks, so with
// dimension-major representatives ([head][dim][block]) a warp's loads of one
// dim are 512 contiguous bytes. The per-head dots meet in shared memory and
// each block's score adds them in head order. Scores are therefore
// bit-identical to the reference's.
//
// Top-k: the reference forces [0, init) and the last `local` blocks, then
// stable-sorts by descending score and fills up to the budget, returning ids
// ascending. Equivalent here: pick the K = budget - |forced| largest
// (score, -index) pairs among unforced blocks by an MSB-first radix select
// on order-preserving 32-bit score keys, resolve ties at the threshold key by
// ascending index, and compact the chosen flags in index order. The
// last-arriving CTA of a (sequence-layer, group) does this (atomic counter,
// no spinning), so the result never depends on CTA scheduling.
#include <algorithm>

#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kThreads = 128;
constexpr int kWarps = kThreads / 32;
constexpr int kLaneBlocks = 4;                      // consecutive blocks per lane
constexpr int kWarpBlocks = 32 * kLaneBlocks;       // 128 blocks per warp pass
constexpr int kMaxBlocks = 16384;
constexpr int kDimUnroll = 8;        // dims in flight per warp: occupancy-bound grids
constexpr int kDimUnrollDeep = 16;   // grids of at most kDeepGridCtas CTAs (latency-bound)
constexpr int kDeepCtasPerSm = 5;   // the deep variant's resident CTAs per SM
constexpr unsigned kFull = 0xffffffffu;

constexpr int kTieMax = kThreads;  // threshold buckets this small are ranked directly

// Units of at most this many blocks keep their order keys in shared memory;
// larger ones recompute them from the scores (L2) on every pass, so that the
// dynamic shared memory every CTA reserves stays small (at 4096 blocks a
// 16 KB key array cut the resident CTAs of the scoring from 10 to 9 per SM).
constexpr int kSmemKeyBlocks = 2048;

struct TopkShared {
  int hist[2][256];                      // digit histograms, double-buffered by pass
  unsigned long long cand[kTieMax];      // threshold-bucket members, (key, ~index) packed
  int digit;
  int above;
  int bucket;
  int ncand;
  int warp_count[kWarps];
  int last;
};

// A bucket member's ranking word: larger = earlier in the reference's order
// (score descending, then index ascending).
__device__ __forceinline__ unsigned long long rank_word(uint32_t key, int i) {
  return ((unsigned long long)key << 32) | (uint32_t)~(uint32_t)i;
}
__device__ __forceinline__ int rank_word_index(unsigned long long w) {
  return (int)~(uint32_t)w;
}

// Representatives are read once per step: a read-only load that does not
// allocate in L1 (on a B200 the select ran ~2 us faster with it).
__device__ __forceinline__ float4 ldg_no_l1(const float* src) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(src));
  return v;
}

__device__ __forceinline__ float dot_step(float acc, float q, float r) {
  return __fadd_rn(acc, __fmul_rn(q, r));
}

// CTAs a unit's heads are split over: groups of more than four heads (the
// reference's shared mode puts all query heads in one group) give each CTA
// four heads, one per warp, instead of walking them in sequence.
__host__ __device__ __forceinline__ int head_splits(int group) {
  return group > kWarps ? (group + kWarps - 1) / kWarps : 1;
}

// Warps per head and block sub-chunks of a CTA: with fewer than four heads
// per group the spare warps take further 128-block sub-chunks.
__host__ __device__ __forceinline__ int heads_per_pass(int group) { return group < kWarps ? group : kWarps; }
__host__ __device__ __forceinline__ int sub_chunks(int group) { return kWarps / heads_per_pass(group); }

// One head's dot products for the lane's 4 consecutive blocks b0..b0+3, in
// the reference's order (sequential over dims, multiply and add rounded
// separately).
template <int DU>
__device__ __forceinline__ void head_dots(const SelectParams& p, const float* rh, const float* qj,
                                          int b0, int nb, int vec, float (&dot)[kLaneBlocks]) {
#pragma unroll
  for (int k = 0; k < kLaneBlocks; ++k) dot[k] = 0.f;
  if (vec) {
    const float* col = rh + b0;
    int dd = 0;
    for (; dd + DU <= p.d; dd += DU) {
      float4 r[DU];
#pragma unroll
      for (int u = 0; u < DU; ++u)
        r[u] = ldg_no_l1(col + (size_t)(dd + u) * p.s_dim);
#pragma unroll
      for (int u = 0; u < DU; ++u) {
        const float q = qj[dd + u];
        dot[0] = dot_step(dot[0], q, r[u].x);
        dot[1] = dot_step(dot[1], q, r[u].y);
        dot[2] = dot_step(dot[2], q, r[u].z);
        dot[3] = dot_step(dot[3], q, r[u].w);
      }
    }
    for (; dd < p.d; ++dd) {
      const float4 r = __ldg(reinterpret_cast<const float4*>(col + (size_t)dd * p.s_dim));
      const float q = qj[dd];
      dot[0] = dot_step(dot[0], q, r.x);
      dot[1] = dot_step(dot[1], q, r.y);
      dot[2] = dot_step(dot[2], q, r.z);
      dot[3] = dot_step(dot[3], q, r.w);
    }
  } else {
#pragma unroll
    for (int k = 0; k < kLaneBlocks; ++k) {
      if (b0 + k >= nb) break;
      const float* rb = rh + (size_t)(b0 + k) * p.s_block;
      float acc = 0.f;
      for (int dd = 0; dd < p.d; ++dd) acc = dot_step(acc, qj[dd], __ldg(rb + (size_t)dd * p.s_dim));
      dot[k] = acc;
    }
  }
}

// Raw projections (Qwen3 decode: q_norm / k_norm, then RoPE, then the FP16
// pack -- head_rms, rope and append_fp16_kv of cpp/src/qwen_layer_main.cpp,
// in the order of cpp/src/qwen_chain_main.cpp:370-392): normalise and rotate
// the group's query rows in qs; the unit's first CTA also publishes them
// (raw_qt for the attention, the query ring for the seal) and appends the
// normalised, rotated K and the V of the group's KV heads to the tail row.
// All 128 threads call it; `scratch` holds >= 256 floats.
__device__ void raw_projections(const SelectParams& p, int sl, int g, float* qs, float* scratch) {
  const int t = threadIdx.x;
  const int layer = sl % p.layers;
  const int pos = p.positions[sl / p.layers];
  for (int j = 0; j < p.group; ++j)
    head_norm_rope(qs + j * kHeadDim, scratch, p.q_norm_w + (size_t)layer * kHeadDim, pos,
                   p.rope_theta, p.norm_eps, t);
  if (blockIdx.x != 0) return;
  const CtxDev& c = p.append_ctx;
  const int q0 = g * p.group;
  const int tl = c.tail_len[sl];
  const int phys = c.tail_block[sl];
  const bool ok_tail = tl >= 0 && tl < kBlockTokens;
  const bool ok_block = phys >= 0 && phys < c.pool_blocks;
  if (t == 0 && tl >= kBlockTokens - 1) c.seal_counters[1] = 1;  // the seal's full pass
  if (t == 0 && !ok_tail) raise_status(c.status, SA_DEV_TAIL_FULL);
  if (t == 0 && ok_tail && !ok_block) raise_status(c.status, SA_DEV_BAD_BLOCK);
  for (int j = 0; j < p.group; ++j) {
    const float v = qs[j * kHeadDim + t];
    p.raw_qt[((size_t)sl * p.qh + q0 + j) * kHeadDim + t] = v;
    if (ok_tail && ok_block)
      c.query_ring[(((size_t)sl * c.qh + q0 + j) * kBlockTokens + tl) * kHeadDim + t] = v;
  }
  if (!ok_tail || !ok_block) return;
  const int per_kv = p.qh / c.kv_heads;
  float* row = scratch;
  float* red = scratch + kHeadDim;
  for (int h = q0 / per_kv; h < (q0 + p.group) / per_kv; ++h) {
    const size_t src = ((size_t)sl * c.kv_heads + h) * kHeadDim + t;
    row[t] = p.raw_k[src];
    __syncthreads();
    head_norm_rope(row, red, p.k_norm_w + (size_t)layer * kHeadDim, pos, p.rope_theta,
                   p.norm_eps, t);
    uint16_t* block = c.pool + (((size_t)phys * c.kv_heads + h) * 2) * kBlockTokens * kHeadDim;
    block[(size_t)tl * kHeadDim + t] = f2h_rn(row[t]);
    block[((size_t)kBlockTokens + tl) * kHeadDim + t] = f2h_rn(p.raw_v[src]);
    __syncthreads();
  }
}

// Top-k of one unit over scores[0, nb), run by the unit's last CTA: the
// forced blocks ([0, init) and the last `local`), then the K = budget -
// |forced| unforced blocks that come first in (score descending, index
// ascending) order -- the order of the reference's stable sort -- written
// to ids in ascending index order.
//
// An MSB-first radix select over order-preserving 32-bit keys narrows the
// threshold bucket (the blocks sharing the top bits of the K-th key) 8 bits
// a pass. It stops as soon as the bucket is taken whole, or is small enough
// (<= kTieMax blocks) to rank its members directly by (key, index); only a
// bucket of more than kTieMax exactly equal keys is resolved by index order
// over warp segments. Compaction runs over warp segments too: warp w covers
// blocks [w * seg, (w + 1) * seg), seg a multiple of 32, one block per lane
// per step, so a ballot keeps index order inside a warp and one exchange of
// warp totals keeps it across warps.
// Dynamic shared memory of the top-k: [keys (nb_cap, kSmemKeys only)]
// [tie_bits][pick_bits] (nb_cap / 32 words each): the chosen members of the
// threshold bucket, and the chosen blocks for the ordered compaction.
__host__ __device__ __forceinline__ int bitmap_words(int nb_cap) { return (nb_cap + 31) / 32; }
__host__ __device__ __forceinline__ size_t topk_smem_bytes(int nb_cap) {
  return ((nb_cap <= kSmemKeyBlocks ? (size_t)nb_cap : 0) + 2 * (size_t)bitmap_words(nb_cap)) *
         sizeof(uint32_t);
}

template <bool kSmemKeys>
__device__ void select_top_k(const SelectParams& p, int unit, int nb, const float* scores,
                             uint32_t* dyn, TopkShared& ts) {
  uint32_t* keys = dyn;
  uint32_t* tie_bits = dyn + (kSmemKeys ? p.nb_cap : 0);
  uint32_t* pick_bits = tie_bits + bitmap_words(p.nb_cap);
  auto key_at = [&](int i) -> uint32_t {
    if constexpr (kSmemKeys) return keys[i];
    else return float_order_key(__ldcg(scores + i));
  };
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int budget = min(p.budget, nb);
  const int n_init = min(p.init, nb);
  const int n_local = min(p.local, nb);
  const int local_begin = nb - n_local;
  const int n_forced = n_init + n_local - max(0, n_init - local_begin);
  const int K = max(0, budget - n_forced);
  auto forced = [&](int i) { return i < n_init || i >= local_begin; };
  const int seg = (nb + kThreads - 1) / kThreads * 32;
  const int lo = warp * seg, hi = min(nb, lo + seg);
  const uint32_t lanes_below = (1u << lane) - 1u;
  // f(i, key) for this thread's blocks i = tid, tid + kThreads, ... < nb;
  // keys recomputed from L2 arrive kKeyBatch loads at a time
  constexpr int kKeyBatch = 16;
  auto for_keys = [&](auto&& f) {
    if constexpr (kSmemKeys) {
#pragma unroll 4
      for (int i = tid; i < nb; i += kThreads) f(i, keys[i]);
    } else {
      for (int base = 0; base < nb; base += kThreads * kKeyBatch) {
        uint32_t k[kKeyBatch];
#pragma unroll
        for (int u = 0; u < kKeyBatch; ++u) {
          const int i = base + u * kThreads + tid;
          k[u] = i < nb ? float_order_key(__ldcg(scores + i)) : 0u;
        }
#pragma unroll
        for (int u = 0; u < kKeyBatch; ++u) {
          const int i = base + u * kThreads + tid;
          if (i < nb) f(i, k[u]);
        }
      }
    }
  };

  // keys, with every load of a batch in flight at once
  constexpr int kLoadBatch = 16;
  bool nan_seen = false;
  for (int base = 0; base < nb; base += kThreads * kLoadBatch) {
    float v[kLoadBatch];
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * kThreads + tid;
      v[u] = i < nb ? __ldcg(scores + i) : 0.f;
    }
#pragma unroll
    for (int u = 0; u < kLoadBatch; ++u) {
      const int i = base + u * kThreads + tid;
      if (i < nb) {
        nan_seen |= isnan(v[u]);
        if constexpr (kSmemKeys) keys[i] = float_order_key(v[u]);
      }
    }
  }
  if (nan_seen) raise_status(p.status, SA_DEV_NONFINITE);
  for (int w = tid; w < (nb + 31) / 32; w += kThreads) tie_bits[w] = 0;
  for (int i = tid; i < 256; i += kThreads) ts.hist[0][i] = 0;
  if (tid == 0) ts.ncand = 0;
  __syncthreads();

  // threshold bucket: `bucket` unforced blocks have (key & mask) == prefix,
  // the first `remaining` of them (in the sort order) are chosen
  uint32_t prefix = 0, mask = 0;
  int remaining = K, bucket = nb - n_forced;
  bool whole = true;  // every bucket member chosen; else tie_bits marks them
  if (K > 0) {
    for (int pass = 0;; ++pass) {
      if (bucket == remaining) break;
      if (bucket <= kTieMax) {
        // gather the members (in any order) and rank each among them
        // (one shared-memory atomic per warp and 32 blocks: with many equal
        // keys the members crowd into few warps)
        constexpr int kGatherBatch = kSmemKeys ? 4 : 16;  // key loads in flight together
        for (int base = 0; base < nb; base += kThreads * kGatherBatch) {
          uint32_t k[kGatherBatch];
#pragma unroll
          for (int u = 0; u < kGatherBatch; ++u) {
            const int i = base + u * kThreads + tid;
            k[u] = i < nb ? key_at(i) : 0u;
          }
#pragma unroll
          for (int u = 0; u < kGatherBatch; ++u) {
            const int i = base + u * kThreads + tid;
            const bool m = i < nb && !forced(i) && (k[u] & mask) == prefix;
            const uint32_t b = __ballot_sync(kFull, m);
            int slot = 0;
            if (lane == 0 && b) slot = atomicAdd(&ts.ncand, __popc(b));
            slot = __shfl_sync(kFull, slot, 0);
            if (m) ts.cand[slot + __popc(b & lanes_below)] = rank_word(k[u], i);
          }
        }
        __syncthreads();
        if (tid < bucket) {
          // a packed word per member: one compare of the (key, index) order
          const unsigned long long mine = ts.cand[tid];
          int rank = 0;
#pragma unroll 4
          for (int j = 0; j < bucket; ++j) rank += ts.cand[j] > mine;
          const int i = rank_word_index(mine);
          if (rank < remaining) atomicOr(&tie_bits[i >> 5], 1u << (i & 31));
        }
        __syncthreads();
        whole = false;
        break;
      }
      if (pass == 4) {
        // more than kTieMax equal keys: the first `remaining` by index
        auto member = [&](int i) { return i < hi && !forced(i) && key_at(i) == prefix; };
        int n = 0;
        for (int base = lo; base < hi; base += 32) n += __popc(__ballot_sync(kFull, member(base + lane)));
        if (lane == 0) ts.warp_count[warp] = n;
        __syncthreads();
        int before = 0;
        for (int w = 0; w < warp; ++w) before += ts.warp_count[w];
        for (int base = lo; base < hi; base += 32) {
          const bool m = member(base + lane);
          const uint32_t b = __ballot_sync(kFull, m);
          const uint32_t take =
              __ballot_sync(kFull, m && before + __popc(b & lanes_below) < remaining);
          if (lane == 0) tie_bits[base >> 5] = take;
          before += __popc(b);
        }
        __syncthreads();
        whole = false;
        break;
      }
      // histogram of the next 8 bits over the bucket; the other buffer is
      // cleared for the pass after this one
      const int shift = 24 - 8 * pass;
      int* hist = ts.hist[pass & 1];
      for (int i = tid; i < 256; i += kThreads) ts.hist[(pass + 1) & 1][i] = 0;
      for_keys([&](int i, uint32_t k) {
        if (!forced(i) && (k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1);
      });
      __syncthreads();
      if (warp == 0) {
        // digits in descending order: lane l holds digits 255 - 8l - j
        int c[8];
        int local = 0;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          c[j] = hist[255 - 8 * lane - j];
          local += c[j];
        }
        int incl = local;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int v = __shfl_up_sync(kFull, incl, o);
          if (lane >= o) incl += v;
        }
        int acc = incl - local;
        if (acc < remaining && remaining <= incl) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            if (acc < remaining && acc + c[j] >= remaining) {
              ts.digit = 255 - 8 * lane - j;
              ts.above = acc;
              ts.bucket = c[j];
            }
            acc += c[j];
          }
        }
      }
      __syncthreads();
      prefix |= (uint32_t)ts.digit << shift;
      mask |= 0xffu << shift;
      remaining -= ts.above;
      bucket = ts.bucket;
    }
  }

  // chosen blocks in index order
  auto chosen = [&](int i, uint32_t key) {
    if (i >= hi) return false;
    if (forced(i)) return true;
    if (K == 0) return false;
    const uint32_t km = key & mask;
    if (km != prefix) return km > prefix;
    return whole || (tie_bits[i >> 5] >> (i & 31) & 1u) != 0u;
  };
  int n = 0;
  constexpr int kWordBatch = kSmemKeys ? 1 : 8;  // 32-block words whose keys load together
  for (int base0 = lo; base0 < hi; base0 += 32 * kWordBatch) {
    uint32_t k[kWordBatch];
#pragma unroll
    for (int u = 0; u < kWordBatch; ++u) {
      const int i = base0 + 32 * u + lane;
      k[u] = i < hi ? key_at(i) : 0u;
    }
#pragma unroll
    for (int u = 0; u < kWordBatch; ++u) {
      const int base = base0 + 32 * u;
      if (base >= hi) break;
      const uint32_t b = __ballot_sync(kFull, chosen(base + lane, k[u]));
      if (lane == 0) pick_bits[base >> 5] = b;
      n += __popc(b);
    }
  }
  if (lane == 0) ts.warp_count[warp] = n;
  __syncthreads();
  int pos = 0, total = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const int c = ts.warp_count[w];
    pos += w < warp ? c : 0;
    total += c;
  }
  int32_t* ids = p.ids + (size_t)unit * p.budget;
  for (int base = lo; base < hi; base += 32) {
    const uint32_t b = pick_bits[base >> 5];
    if (b >> lane & 1u) {
      const int at = pos + __popc(b & lanes_below);
      if (at < p.budget) ids[at] = base + lane;
    }
    pos += __popc(b);
  }
  if (tid == 0 && p.counts) p.counts[unit] = min(total, p.budget);
}

// 10 resident CTAs per SM (48 registers): with the no-allocate loads the
// select ran 100.3 us at cfg3 against 103.0 us at the compiler's 56 registers
// (9 CTAs) and 104.4 / 118.5 us at 12 / 16 CTAs.
// The deep variant keeps 16 dims (8 KB a warp) in flight for grids too small
// to fill the SMs (cfg2: 448 CTAs), where only more bytes in flight per warp
// hide the load latency.
template <int DU, int kMinBlocks>
__global__ void __launch_bounds__(kThreads, kMinBlocks)
    select_kernel(const SelectParams p, const int vec) {
  // dynamic shared memory: q [group][d], head dots [group][chunk], then (last
  // CTA) order keys [nb_cap]
  extern __shared__ float smem[];
  __shared__ TopkShared ts;
  pdl_launch_dependents();
  pdl_wait();  // sealed counts, tails and representatives of the previous step
  const int unit = blockIdx.y;
  const int sl = unit / p.n_groups;
  const int g = unit - sl * p.n_groups;
  const int nb = max(0, min(p.nb ? p.nb[sl] : p.fixed_nb, p.nb_cap));
  const int hp = heads_per_pass(p.group);
  const int sub = sub_chunks(p.group);
  const int chunk = sub * kWarpBlocks;
  const int nchunks = max(1, (nb + chunk - 1) / chunk);
  if ((int)blockIdx.x >= nchunks) return;
  // heads [hb, hb + nh) of the group are this CTA's
  const int hsplit = head_splits(p.group);
  const int hb = (int)blockIdx.z * kWarps;
  const int nh = hsplit > 1 ? min(kWarps, p.group - hb) : p.group;
  float* qs = smem;
  float* dots = smem + ((nh * p.d + 3) & ~3);  // 16-byte aligned

  if (p.append_kv && blockIdx.x == 0 && blockIdx.z == 0) {
    // fused decode-tail append of this group's heads (tail_len unchanged)
    const int q0 = g * p.group;
    const int per_kv = p.qh / p.append_ctx.kv_heads;
    append_token(p.append_ctx, sl, p.query, p.append_kv, p.append_kv_fp32, q0 / per_kv,
                 (q0 + p.group) / per_kv, q0, q0 + p.group, threadIdx.x, kThreads);
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sc = warp / hp;
  const int cbase = blockIdx.x * chunk;
  // The lines of the first DU dims of the warp's first head are requested
  // into L2 before the query is staged (one prefetch per 128-byte line, no
  // registers held), so that the query's round trip overlaps theirs. Units
  // of one chunk skip it: their select is the top-k's latency, and on a B200
  // the prefetches made a 64-block unit's select 0.7 us slower (cfg3 2.4 us
  // faster, cfg2 0.9 us).
  if (vec && nchunks > 1 && sc < sub && warp % hp < nh && (lane & 7) == 0 &&
      cbase + sc * kWarpBlocks + lane * kLaneBlocks < nb) {
    const float* col = p.reps + (size_t)sl * p.s_sl +
                       (size_t)(g * p.group + hb + warp % hp) * p.s_head + cbase +
                       sc * kWarpBlocks + lane * kLaneBlocks;
#pragma unroll
    for (int u = 0; u < DU; ++u)
      if (u < p.d) asm volatile("prefetch.global.L2 [%0];" ::"l"(col + (size_t)u * p.s_dim));
  }
  const float* qsrc = p.query + ((size_t)sl * p.qh + (size_t)g * p.group + hb) * p.d;
  for (int i = threadIdx.x; i < nh * p.d; i += kThreads) qs[i] = qsrc[i];
  __syncthreads();
  if (p.raw_k) raw_projections(p, sl, g, qs, dots);

  // ---- per-head dot products: warp w takes head w % hp (+ hp, ...) of
  // sub-chunk w / hp ----
  if (sc < sub) {
    const int lb = sc * kWarpBlocks + lane * kLaneBlocks;  // chunk-local first block
    const int b0 = cbase + lb;
    for (int j = warp % hp; j < nh; j += hp) {
      float dot[kLaneBlocks] = {0.f, 0.f, 0.f, 0.f};
      if (b0 < nb) {
        const int h = g * p.group + hb + j;
        head_dots<DU>(p, p.reps + (size_t)sl * p.s_sl + (size_t)h * p.s_head, qs + j * p.d, b0, nb,
                  vec, dot);
      }
      *reinterpret_cast<float4*>(dots + (size_t)j * chunk + lb) =
          make_float4(dot[0], dot[1], dot[2], dot[3]);
    }
  }
  __syncthreads();
  // ---- block scores: sum over the group's heads in head order ----
  float* scores = p.scores + (size_t)unit * p.nb_cap;
  const float divisor = (float)p.group;
  if (hsplit == 1) {
    for (int lb = threadIdx.x; lb < chunk; lb += kThreads) {
      const int b = cbase + lb;
      if (b >= nb) break;
      float score = 0.f;
      for (int j = 0; j < p.group; ++j)
        score = __fadd_rn(score, __fdiv_rn(dots[(size_t)j * chunk + lb], divisor));
      scores[b] = score;
    }
  } else {
    // publish this CTA's heads; the chunk's last CTA adds all heads in order
    float* hd = p.head_dots + (size_t)unit * p.group * p.nb_cap;
    for (int i = threadIdx.x; i < nh * chunk; i += kThreads) {
      const int j = i / chunk, lb = i - j * chunk, b = cbase + lb;
      if (b < nb) hd[(size_t)(hb + j) * p.nb_cap + b] = dots[(size_t)j * chunk + lb];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      // the barrier orders the CTA's dot stores before this fence
      __threadfence();
      int* cc = p.chunk_counters + (size_t)unit * ((p.nb_cap + chunk - 1) / chunk) + blockIdx.x;
      ts.last = atomicAdd(cc, 1) == hsplit - 1;
      if (ts.last) {
        __threadfence();
        *cc = 0;
      }
    }
    __syncthreads();
    if (!ts.last) return;
    for (int lb = threadIdx.x; lb < chunk; lb += kThreads) {
      const int b = cbase + lb;
      if (b >= nb) break;
      float score = 0.f;
      for (int j = 0; j < p.group; ++j)
        score = __fadd_rn(score, __fdiv_rn(__ldcg(hd + (size_t)j * p.nb_cap + b), divisor));
      scores[b] = score;
    }
  }

  // ---- the last CTA of this (sl, group) selects ----
  __syncthreads();
  if (nchunks > 1) {
    if (threadIdx.x == 0) {
      // the barrier orders the CTA's score stores before the arrival
      ts.last = arrive_acq_rel(&p.counters[unit]) == nchunks - 1;
      if (ts.last) p.counters[unit] = 0;
    }
    __syncthreads();
    if (!ts.last) return;
  }

  // q and dots are no longer needed: the top-k reuses the dynamic shared memory
  if (p.nb_cap <= kSmemKeyBlocks)
    select_top_k<true>(p, unit, nb, scores, reinterpret_cast<uint32_t*>(smem), ts);
  else
    select_top_k<false>(p, unit, nb, scores, reinterpret_cast<uint32_t*>(smem), ts);
}

}  // namespace

int select_max_blocks() { return kMaxBlocks; }

int select_head_splits(int group) { return head_splits(group); }

int select_max_chunks(int group, int nb_cap) {
  const int chunk = sub_chunks(group) * kWarpBlocks;
  return std::max(1, (nb_cap + chunk - 1) / chunk);
}

size_t select_split_scratch_bytes(int units, int group, int nb_cap) {
  if (head_splits(group) == 1) return 0;
  const size_t dots = ((size_t)units * group * nb_cap * sizeof(float) + 255) & ~size_t(255);
  return dots + (size_t)units * select_max_chunks(group, nb_cap) * sizeof(int);
}

void select_bind_split_scratch(SelectParams& p, void* scratch, int units) {
  if (head_splits(p.group) == 1 || !scratch) return;
  const size_t dots = ((size_t)units * p.group * p.nb_cap * sizeof(float) + 255) & ~size_t(255);
  p.head_dots = static_cast<float*>(scratch);
  p.chunk_counters = reinterpret_cast<int*>(static_cast<char*>(scratch) + dots);
}

sa_status launch_select(const SelectParams& p, cudaStream_t stream) {
  if (p.num_sl <= 0 || p.n_groups <= 0) return SA_OK;
  if (p.nb_cap > kMaxBlocks)
    return fail(SA_ERR_UNSUPPORTED, "select: more than 16384 candidate blocks");
  if ((size_t)p.num_sl * p.n_groups > 65535u)
    return fail(SA_ERR_UNSUPPORTED, "select: more than 65535 (sequence-layer, group) units");
  const int vec = p.s_block == 1 && p.s_dim % 4 == 0 && p.s_head % 4 == 0 && p.s_sl % 4 == 0 &&
                  p.nb_cap % 4 == 0 && (reinterpret_cast<uintptr_t>(p.reps) & 15u) == 0;
  const int chunk = sub_chunks(p.group) * kWarpBlocks;
  const int hsplit = head_splits(p.group);
  if (hsplit > 1 && (!p.head_dots || !p.chunk_counters))
    return fail(SA_ERR_INVALID_ARG, "select: groups of more than 4 heads need the split scratch");
  if (hsplit > 1 && p.raw_k)
    return fail(SA_ERR_UNSUPPORTED, "select: raw projections need groups of at most 4 heads");
  const size_t nh = hsplit > 1 ? (size_t)kWarps : (size_t)p.group;
  const size_t smem =
      std::max((((nh * p.d + 3) & ~size_t(3)) + nh * chunk) * sizeof(float),
               topk_smem_bytes(p.nb_cap));
  const int nchunks = std::max(1, (p.nb_cap + chunk - 1) / chunk);
  const dim3 grid(nchunks, p.num_sl * p.n_groups, hsplit);
  const bool deep =
      (long long)nchunks * p.num_sl * p.n_groups * hsplit <= (long long)kDeepCtasPerSm * device_sm_count();
  auto kernel = deep ? select_kernel<kDimUnrollDeep, 5> : select_kernel<kDimUnroll, 10>;
  static int configured[2][kMaxDevices];
  const sa_status st = ensure_smem_limit((const void*)kernel, (int)std::max<size_t>(smem, 48 * 1024),
                                         configured[deep ? 1 : 0]);
  if (st != SA_OK) return st;
  const cudaError_t e = launch_kernel(kernel, grid, dim3(kThreads), smem, stream, p.pdl != 0, p, vec);
  if (e != cudaSuccess) return cuda_status(e, "select_kernel launch");
  return cuda_status(cudaGetLastError(), "select_kernel launch");
}

}  // namespace sa
