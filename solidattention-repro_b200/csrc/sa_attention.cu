// sa_attention.cu -- block-sparse GQA decode attention for sm_100a.
//
// Replaces the reference's attention (cpp/src/attention_reference.cpp:55-96)
// and its device kernels sparse_attention_parallel
// (cpp/src/cuda_backend.cpp:109-158) and sparse_fp16_attention
// (cpp/src/qwen_layer_main.cpp:224-268).
//
// Work unit: one (sequence-layer, KV head). Its token set is a list of
// entries: the selected sealed blocks (logical ids -> physical pool blocks
// through the block table) followed by the open tail (tail_len tokens). Every
// unit owns `slots_per_unit` entry slots; slots past its entries are empty.
//
// Persistent schedule: the flattened slot list of all units is cut into one
// contiguous range per (virtual) CTA, about one wave: two 256-thread virtual
// CTAs per 512-thread CTA and SM (see virt_ctas). A CTA streams its range across
// unit boundaries without draining its load pipeline; the part of its range
// inside one unit is a segment. The (physical block, token count) pair of
// every slot in the range is resolved once, in parallel, into shared memory.
//
// Pipeline: a stage holds two entries of one segment (2 x 16 KB: the K rows
// then the V rows of the unit's KV head, 32 x 256 B each) in a ring of three
// stages. Every lane reads only its own sixteen-byte column of its own rows
// (below), so every lane also loads exactly those bytes itself, with 16-byte
// cp.async copies through the load/store unit, one commit group per stage: a
// lane waits only for its own copies and refills its part of a stage as soon
// as it has computed on it, with no producer thread and no cross-warp release.
// (On a B200, streaming random 16 KB blocks: one thread per SM issuing 16 KB
// bulk copies read at most 4.3 TB/s and two such threads per SM 6.6 TB/s,
// whatever the number of copies in flight, while 16-byte cp.async copies
// reached 7.2 TB/s with 128 KB in flight per SM.) Rows come from the decode
// context's head-major pool or from a caller's token-major rows; the
// shared-memory layout is the same.
//
// Warp w, per stage: half-warp h takes entry h of the stage and its tokens
// [4w, 4w+4); lane l covers head dims [8(l%16), 8(l%16)+8). A quarter-warp
// reads 128 contiguous bytes of one row: conflict-free. QK uses packed FP32
// FMA (__ffma2_rn) with the softmax scale folded into q, then a 16-lane
// transpose-reduce leaves one (token, head) logit per lane. The warp keeps an
// FP32 online softmax per head (exp2 domain, running max shared by both
// half-warps) and skips the accumulator rescale when no running max moved.
//
// At the end of a segment the eight warps merge by log-sum-exp through the
// segment's last stage buffer, which is released only afterwards. A unit
// covered by several CTAs gets one partial (m, l, o[128]) per CTA; the last
// CTA to arrive (atomic counter, no spinning) merges them in range order, so
// the result does not depend on CTA timing.
#include <algorithm>

#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = kConsumerWarps * 32;
constexpr int kStages = 3;
constexpr int kRowBytes = kHeadDim * 2;                 // one token of one head, FP16
constexpr int kPlaneBytes = kBlockTokens * kRowBytes;   // 32 rows: 8 KB
constexpr int kEntryBytes = 2 * kPlaneBytes;            // K plane then V plane
constexpr int kStageBytes = 2 * kEntryBytes;            // two entries per stage
constexpr int kPartialStride = 2 + kHeadDim;            // m, l, o[128]
constexpr int kMaxCtaSlots = 512;                       // slots one CTA may own
constexpr int kMaxSegments = 32;                        // units one CTA may touch
constexpr unsigned kFull = 0xffffffffu;
constexpr float kLazyRescale = 8.f;                     // log2 units

constexpr int kMaxStages = kMaxCtaSlots / 2 + kMaxSegments;

// Stage table word: tokens of the stage's two entries (6 bits each), its
// first CTA-local slot (9 bits), its segment (5 bits), and whether it opens /
// closes the segment.
constexpr uint32_t kInfoStart = 1u << 26;
constexpr uint32_t kInfoEnd = 1u << 27;
__host__ __device__ constexpr uint32_t stage_word(int ntok0, int ntok1, int e0, int seg,
                                                   bool start, bool end) {
  return (uint32_t)ntok0 | ((uint32_t)ntok1 << 6) | ((uint32_t)e0 << 12) |
         ((uint32_t)seg << 21) | (start ? kInfoStart : 0u) | (end ? kInfoEnd : 0u);
}
__device__ __forceinline__ int info_ntok(uint32_t w, int i) { return (w >> (6 * i)) & 0x3f; }
__device__ __forceinline__ int info_e0(uint32_t w) { return (w >> 12) & 0x1ff; }
__device__ __forceinline__ int info_seg(uint32_t w) { return (w >> 21) & 0x1f; }

// Virtual CTAs: with up to four query heads per KV head, one 512-thread CTA
// runs two independent 256-thread halves ("virtual CTAs", each with its own
// shared-memory state and named barrier), one per SM. Two separate CTAs per
// SM would also fit, but the warp scheduler favours the older CTA: on a
// B200 the second CTA of every SM finished ~20% later and then streamed
// alone. The halves of one CTA are scheduled evenly, which balances the
// SM's two shares of the work without changing the work split or any
// result bit.
template <int G>
constexpr int virt_ctas() { return G <= 4 ? 2 : 1; }
template <int V>
__device__ __forceinline__ int vtid() { return V == 1 ? (int)threadIdx.x : (int)(threadIdx.x & 255); }
template <int V>
__device__ __forceinline__ int vhalf() { return V == 1 ? 0 : (int)(threadIdx.x >> 8); }
template <int V>
__device__ __forceinline__ int vbid() { return (int)blockIdx.x * V + vhalf<V>(); }
template <int V>
__device__ __forceinline__ void vsync() {
  asm volatile("bar.sync %0, 256;" ::"r"(1 + vhalf<V>()) : "memory");
}

template <int G>
struct alignas(128) AttnSmem {
  uint8_t tiles[kStages][kStageBytes];
  float2 pbuf[kConsumerWarps][2][4][G];  // probabilities (p, p) [half][token][head]
  float2 abuf[kConsumerWarps][G];        // rescale factor (a, a) per head
  float wscale[kConsumerWarps][G];
  float mw[kConsumerWarps][G];           // warp softmax states at a segment end
  float lw[kConsumerWarps][G];
  float cta_m[G];
  float cta_l[G];
  int ent_phys[kMaxCtaSlots];
  uint8_t ent_ntok[kMaxCtaSlots];
  uint32_t stage_info[kMaxStages];
  int seg_slot0[kMaxSegments + 1];   // first CTA-local slot of each segment
  int seg_stage0[kMaxSegments + 1];  // first stage of each segment
  int seg_unit[kMaxSegments];
  int seg_index[kMaxSegments];       // the CTA's place among its unit's CTAs
  int seg_count[kMaxSegments];       // CTAs covering the unit
  alignas(16) uint8_t ostage[G * kHeadDim * 4];  // a unit's output, for peer stores
  int nseg;
  int nstages;
  int last_flag;
};

// spec_id: the selected id at slot e (loaded by the caller together with the
// count, before knowing whether e holds a selected block).
__device__ __forceinline__ void unit_entry(const AttnParams& p, int sl, int sgroup, int nsel,
                                           int tail_len, int e, int spec_id, int* phys,
                                           int* ntok) {
  *phys = 0;
  *ntok = 0;
  int r;
  if (e < nsel) {
    const int logical = p.sel_ids ? spec_id : e;
    if (p.table) {
      if (logical < 0 || logical >= p.table_stride) {
        raise_status(p.status, SA_DEV_BAD_BLOCK);
        return;
      }
      r = p.table[(size_t)sl * p.table_stride + logical];
    } else {
      r = logical;
    }
    *ntok = kBlockTokens;
  } else if (e == nsel && tail_len > 0) {
    r = p.tail_block ? p.tail_block[sl] : p.fixed_tail_block;
    *ntok = tail_len;
  } else {
    return;  // an empty slot
  }
  if (r < 0 || r >= p.pool_blocks) {
    raise_status(p.status, SA_DEV_BAD_BLOCK);
    *ntok = 0;
    return;
  }
  *phys = r;
}

// The CTA owning flattened slot x when `total` slots are cut into `ctas`
// ranges [c * total / ctas, (c + 1) * total / ctas).
__device__ __forceinline__ int cta_of_slot(long long x, long long total, int ctas) {
  return (int)(((x + 1) * ctas - 1) / total);
}

// The hardware base-2 exponential (ex2.approx, ~2 ulp).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// In-warp transpose-reduce over lane bits OFF, OFF/2, ...: at each level a
// lane keeps positions [0, M/2) of its M values and adds its partner's
// positions [M/2, M). Each lane computes its values in an order XOR-permuted
// by its own lane bits, so both partners' kept and received positions name
// the same (token, head) pair and no selects are needed.
template <int M, int OFF>
struct Halve {
  __device__ __forceinline__ static void run(float* a) {
    if constexpr (M > 1 && OFF >= 1) {
#pragma unroll
      for (int j = 0; j < M / 2; ++j) a[j] += __shfl_xor_sync(kFull, a[j + M / 2], OFF);
      Halve<M / 2, OFF / 2>::run(a);
    }
  }
};

__device__ __forceinline__ void unpack8(const uint4& u, float2 (&f)[4]) {
  f[0] = h2x2f(u.x);
  f[1] = h2x2f(u.y);
  f[2] = h2x2f(u.z);
  f[3] = h2x2f(u.w);
}

// G duplicated pairs from shared memory with the widest loads.
template <int G>
__device__ __forceinline__ void load_pairs(const float2* src, float2 (&v)[G]) {
  if constexpr (G == 1) {
    v[0] = src[0];
  } else {
#pragma unroll
    for (int g = 0; g < G; g += 2) {
      const float4 t = *reinterpret_cast<const float4*>(src + g);
      v[g] = make_float2(t.x, t.y);
      v[g + 1] = make_float2(t.z, t.w);
    }
  }
}

// This lane's copies for stage j into shared-memory stage `slot`: rows
// [t0, t0 + 4) of entry `half`, K then V plane, 16 bytes at column l16 --
// exactly the bytes the lane reads; rows at or past the entry's token count
// are not copied (the compute masks them).
template <int G, bool kHeadMajor>
__device__ __forceinline__ void load_stage(AttnSmem<G>& s, const AttnParams& p, int j, int slot,
                                           int half, int t0, int l16) {
  const uint32_t w = s.stage_info[j];
  const int ntok = info_ntok(w, half);
  if (ntok <= t0) return;
  const int phys = s.ent_phys[info_e0(w) + half];
  const int kvh = s.seg_unit[info_seg(w)] % p.kv_heads;
  const uint8_t* src;
  size_t row_stride, plane;
  if constexpr (kHeadMajor) {
    src = reinterpret_cast<const uint8_t*>(p.pool) +
          ((size_t)phys * p.kv_heads + kvh) * kEntryBytes + (size_t)t0 * kRowBytes;
    row_stride = kRowBytes;
    plane = kPlaneBytes;
  } else {
    src = reinterpret_cast<const uint8_t*>(p.rows) +
          ((size_t)phys * kBlockTokens + t0) * (size_t)p.row_bytes + (size_t)kvh * kRowBytes;
    row_stride = (size_t)p.row_bytes;
    plane = (size_t)p.kv_heads * kRowBytes;
  }
  src += l16 * 16;
  uint8_t* dst = s.tiles[slot] + half * kEntryBytes + t0 * kRowBytes + l16 * 16;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    if (t0 + r < ntok) {
      cp_async16(dst + r * kRowBytes, src + r * row_stride);
      cp_async16(dst + kPlaneBytes + r * kRowBytes, src + plane + r * row_stride);
    }
  }
}

// Stores output element idx of unit u (local layout) and, when gathering,
// stages it for the peer stores.
template <int G>
__device__ __forceinline__ void store_out(const AttnParams& p, AttnSmem<G>& s, size_t base,
                                          int idx, float v) {
  if (p.out_fp16) {
    const uint16_t h = f2h_rn(v);
    reinterpret_cast<uint16_t*>(p.out)[base + idx] = h;
    if (p.gather_peers) reinterpret_cast<uint16_t*>(s.ostage)[idx] = h;
  } else {
    reinterpret_cast<float*>(p.out)[base + idx] = v;
    if (p.gather_peers) reinterpret_cast<float*>(s.ostage)[idx] = v;
  }
}

// Copies unit u's staged output into every rank's gathered buffer (16-byte
// P2P stores over NVLink; the own rank's buffer is local). In a decode step
// nothing else happens here: once the whole attention grid has completed,
// one thread of the step's seal kernel fences once at system scope and
// signals every rank (gather_signal_wait). A standalone attention also
// counts the unit's arrival on every rank (one fence and one remote atomic
// per rank for every unit: at eight GPUs that per-unit work was a large
// part of the step).
template <int G>
__device__ __forceinline__ void gather_push(const AttnParams& p, AttnSmem<G>& s, int u) {
  vsync<virt_ctas<G>()>();
  const int esz = p.out_fp16 ? 2 : 4;
  const int chunks = G * kHeadDim * esz / 16;
  const int sl = u / p.kv_heads;
  const int kvh = u - sl * p.kv_heads;
  const size_t off = (size_t)(*p.gather_epoch & 1ull) * p.gather_slot_bytes +
                     (((size_t)sl * p.gather_world + p.gather_rank) * p.kv_heads + kvh) *
                         (size_t)(G * kHeadDim * esz);
  for (int i = vtid<virt_ctas<G>()>(); i < chunks * p.gather_world; i += kThreads) {
    const int r = i / chunks;
    const int c = i - r * chunks;
    uint8_t* dst = reinterpret_cast<uint8_t*>(p.gather_peers[r]) + off + (size_t)c * 16;
    *reinterpret_cast<uint4*>(dst) = reinterpret_cast<const uint4*>(s.ostage)[c];
  }
  if (!p.gather_unit_arrivals) return;
  vsync<virt_ctas<G>()>();
  if (vtid<virt_ctas<G>()>() == 0) {
    // release pattern at system scope: the fence orders the CTA's stores
    // (ordered before it by the barrier) before the relaxed arrivals
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    for (int r = 0; r < p.gather_world; ++r) {
      const unsigned long long* ctr = reinterpret_cast<const unsigned long long*>(
          reinterpret_cast<uint8_t*>(p.gather_peers[r]) + p.gather_counter_bytes);
      asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
    }
  }
}

// acc[g] += p(token, g) * v(token) over the half-warp's 4 tokens; tokens at
// or past ntok are skipped when kMasked (their rows may hold stale data).
template <int G, bool kMasked>
__device__ __forceinline__ void pv_tokens(const uint8_t* vrow, const float2 (*pb)[G], int t0,
                                          int ntok, float2 (&acc)[G][4]) {
#pragma unroll
  for (int tt = 0; tt < 4; ++tt) {
    if (!kMasked || t0 + tt < ntok) {
      float2 v[4];
      unpack8(*reinterpret_cast<const uint4*>(vrow + tt * kRowBytes), v);
      float2 pp[G];
      load_pairs<G>(pb[tt], pp);
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[g][c] = __ffma2_rn(pp[g], v[c], acc[g][c]);
    }
  }
}

template <int G, bool kHeadMajor>
__global__ void __launch_bounds__(kThreads * virt_ctas<G>(), 1)
    attention_kernel(const AttnParams p) {
  // Pairs (token, head) per half-warp: 4G over 16 lanes -> VPL per lane.
  constexpr int NPH = 4 * G;
  constexpr int VPL = NPH > 16 ? NPH / 16 : 1;
  constexpr int kPairShift = NPH >= 16 ? 0 : (NPH == 8 ? 1 : 2);  // lanes per pair = 1 << shift
  extern __shared__ __align__(128) uint8_t smem_raw[];
  if (vbid<virt_ctas<G>()>() >= p.ctas) return;  // the idle half of an odd plan
  AttnSmem<G>& s = *reinterpret_cast<AttnSmem<G>*>(
      smem_raw + (size_t)vhalf<virt_ctas<G>()>() * sizeof(AttnSmem<G>));
  const int warp = vtid<virt_ctas<G>()>() >> 5;
  const int lane = vtid<virt_ctas<G>()>() & 31;
  pdl_launch_dependents();

  // ---- this CTA's slot range, its segments and its stage table ----
  const long long E = p.slots_per_unit;
  const long long total = (long long)p.num_sl * p.kv_heads * E;
  const long long lo = (long long)vbid<virt_ctas<G>()>() * total / p.ctas;
  const long long hi = (long long)(vbid<virt_ctas<G>()>() + 1) * total / p.ctas;
  const int n = (int)min(hi - lo, (long long)kMaxCtaSlots);
  if (vtid<virt_ctas<G>()>() == 0) {
    if (hi - lo > kMaxCtaSlots) raise_status(p.status, SA_DEV_BAD_BLOCK);
    int nseg = 0, stages = 0;
    if (n > 0) {
      const long long u0 = lo / E;
      const long long u1 = (lo + n - 1) / E;
      nseg = (int)min(u1 - u0 + 1, (long long)kMaxSegments);
      for (int k = 0; k < nseg; ++k) {
        const long long u = u0 + k;
        const int a = (int)(max(lo, u * E) - lo);
        const int b = (int)(min(lo + n, (u + 1) * E) - lo);
        const int cf = cta_of_slot(u * E, total, p.ctas);
        const int cl = cta_of_slot((u + 1) * E - 1, total, p.ctas);
        s.seg_unit[k] = (int)u;
        s.seg_index[k] = (int)vbid<virt_ctas<G>()>() - cf;
        s.seg_count[k] = cl - cf + 1;
        s.seg_slot0[k] = a;
        s.seg_stage0[k] = stages;
        stages += (b - a + 1) / 2;
      }
      s.seg_slot0[nseg] = (int)(min(lo + n, (u0 + nseg) * E) - lo);
    } else {
      s.seg_slot0[0] = 0;
    }
    s.seg_stage0[nseg] = stages;
    s.nseg = nseg;
    s.nstages = stages;
  }
  pdl_wait();  // the selection (and the append) of this step
  for (int i = vtid<virt_ctas<G>()>(); i < n; i += kThreads) {
    const long long x = lo + i;
    const int u = (int)(x / E);
    const int e = (int)(x - (long long)u * E);
    const int sl = u / p.kv_heads;
    const int kvh = u - sl * p.kv_heads;
    const int sgroup = kvh / p.kv_per_sel_group;
    // the count, the tail length and the id at this slot in one round of loads
    const int spec_id = p.sel_ids && e < p.sel_stride
                            ? __ldcg(p.sel_ids + (sl * p.n_sel_groups + sgroup) * p.sel_stride + e)
                            : 0;
    int nsel = p.sel_count ? __ldcg(p.sel_count + sl * p.n_sel_groups + sgroup) : p.fixed_nsel;
    nsel = max(0, min(nsel, p.sel_ids ? p.sel_stride : nsel));
    int tail_len = p.tail_len ? __ldcg(p.tail_len + sl) : p.fixed_tail_len;
    if (tail_len < kBlockTokens) tail_len += p.tail_pending;
    tail_len = max(0, min(tail_len, kBlockTokens));
    int phys, ntok;
    unit_entry(p, sl, sgroup, nsel, tail_len, e, spec_id, &phys, &ntok);
    s.ent_phys[i] = phys;
    s.ent_ntok[i] = (uint8_t)ntok;
  }
  vsync<virt_ctas<G>()>();
  // stage table, one stage per thread
  for (int j = vtid<virt_ctas<G>()>(); j < s.nstages; j += kThreads) {
    int k = 0;
    while (k + 1 < s.nseg && s.seg_stage0[k + 1] <= j) ++k;
    const int j0 = s.seg_stage0[k], j1 = s.seg_stage0[k + 1];
    const int send = s.seg_slot0[k + 1];
    const int e0 = s.seg_slot0[k] + 2 * (j - j0);
    s.stage_info[j] = stage_word(s.ent_ntok[e0], e0 + 1 < send ? s.ent_ntok[e0 + 1] : 0, e0, k,
                                 j == j0, j + 1 == j1);
  }
  vsync<virt_ctas<G>()>();
  const int nstages = s.nstages;

  const int half = lane >> 4;      // which entry of the stage
  const int l16 = lane & 15;       // 16 B (8 dims) column of a 256 B row
  const int t0 = 4 * warp;
  // This lane's reduced (token, head) pairs after QK: v = pair0 + i, with
  // v = token * G + head. QK runs in the order v ^ pair0 (see Halve): token
  // tt reads row tt ^ tsw, head g uses q of head g ^ gsw.
  const int pair0 = (l16 >> kPairShift) * VPL;
  const int tsw = pair0 / G;
  const int gsw = pair0 % G;
  const bool pair_writer = (l16 & ((1 << kPairShift) - 1)) == 0;
  // Byte offsets of this lane's 16 B column in its entry's K plane, per token.
  const int col_off = half * kEntryBytes + t0 * kRowBytes + l16 * 16;
  // one commit group per stage, the first kStages in flight before the loop
#pragma unroll
  for (int j = 0; j < kStages; ++j) {
    if (j < nstages) load_stage<G, kHeadMajor>(s, p, j, j, half, t0, l16);
    cp_async_commit();
  }

  float m_run[VPL], m_thr[VPL], l_run[VPL];
  float2 acc[G][4];
  float2 q[G][4];  // q[g] holds head g ^ gsw
  int stage = 0;

  for (int j = 0; j < nstages; ++j) {
    const uint32_t info = s.stage_info[j];
    if (info & kInfoStart) {
      // ---- a new segment: its unit's q (scaled into the exp2 domain), fresh state ----
      const float* qbase = p.query + (size_t)s.seg_unit[info_seg(info)] * G * kHeadDim + 8 * l16;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float* qh = qbase + (g ^ gsw) * kHeadDim;
        const float4 a = __ldg(reinterpret_cast<const float4*>(qh));
        const float4 b = __ldg(reinterpret_cast<const float4*>(qh + 4));
        q[g][0] = make_float2(a.x * p.scale_log2, a.y * p.scale_log2);
        q[g][1] = make_float2(a.z * p.scale_log2, a.w * p.scale_log2);
        q[g][2] = make_float2(b.x * p.scale_log2, b.y * p.scale_log2);
        q[g][3] = make_float2(b.z * p.scale_log2, b.w * p.scale_log2);
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[g][c] = make_float2(0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        m_run[i] = -INFINITY;
        m_thr[i] = -INFINITY;
        l_run[i] = 0.f;
      }
    }
    cp_async_wait<kStages - 1>();  // this lane's copies of stage j have landed
    const int ntok = info_ntok(info, half);
    const int ntok_other = info_ntok(info, half ^ 1);
    const uint8_t* tile = s.tiles[stage];
    if (t0 < ntok || t0 < ntok_other) {
      const uint8_t* kcol = tile + col_off;
      // ---- QK over this lane's 8 dims, 4 tokens x G heads (permuted order) ----
      float part[NPH];
#pragma unroll
      for (int tt = 0; tt < 4; ++tt) {
        float2 k[4];
        unpack8(*reinterpret_cast<const uint4*>(kcol + (tt ^ tsw) * kRowBytes), k);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float2 a = __fmul2_rn(q[g][0], k[0]);
          a = __ffma2_rn(q[g][1], k[1], a);
          a = __ffma2_rn(q[g][2], k[2], a);
          a = __ffma2_rn(q[g][3], k[3], a);
          part[tt * G + g] = a.x + a.y;
        }
      }
      Halve<NPH, 8>::run(part);
      if constexpr (NPH < 16) {
#pragma unroll
        for (int off = 1 << (kPairShift - 1); off >= 1; off >>= 1)
          part[0] += __shfl_xor_sync(kFull, part[0], off);
      }
      // ---- online softmax over 8 tokens (4 per half-warp) per head, lazily
      // rescaled: the running max moves only when a logit exceeds it by more
      // than kLazyRescale (log2 units), so probabilities stay below
      // 2^kLazyRescale and most stages skip the max reduction and rescale ----
      float x[VPL];
      bool over = false;
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const int tt = (pair0 + i) / G;
        x[i] = (t0 + tt < ntok) ? part[i] : -INFINITY;
        over |= x[i] > m_thr[i];
      }
      const bool rescale = __any_sync(kFull, over);
      if (rescale) {
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          float bm = fmaxf(x[i], __shfl_xor_sync(kFull, x[i], 4));
          bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 8));
          bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 16));
          const float m_new = fmaxf(m_run[i], bm);
          const float alpha = m_new == -INFINITY ? 1.f : fast_exp2(m_run[i] - m_new);
          m_run[i] = m_new;
          m_thr[i] = m_new + kLazyRescale;
          l_run[i] *= alpha;
          const int v = pair0 + i;
          if (pair_writer && half == 0 && v / G == 0) s.abuf[warp][v % G] = make_float2(alpha, alpha);
        }
      }
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        const float pr = x[i] == -INFINITY ? 0.f : fast_exp2(x[i] - m_run[i]);
        l_run[i] += pr;
        const int v = pair0 + i;
        if (pair_writer) s.pbuf[warp][half][v / G][v % G] = make_float2(pr, pr);
      }
      __syncwarp();
      // ---- PV over the half-warp's 4 tokens ----
      if (rescale) {
        float2 aa[G];
        load_pairs<G>(s.abuf[warp], aa);
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
          for (int c = 0; c < 4; ++c) acc[g][c] = __fmul2_rn(acc[g][c], aa[g]);
      }
      const uint8_t* vrow = tile + col_off + kPlaneBytes;
      if (ntok >= kBlockTokens) pv_tokens<G, false>(vrow, s.pbuf[warp][half], t0, ntok, acc);
      else pv_tokens<G, true>(vrow, s.pbuf[warp][half], t0, ntok, acc);
      __syncwarp();
    }

    if (info & kInfoEnd) {
      // ---- segment end: merge the 8 warps through this stage's buffer ----
      vsync<virt_ctas<G>()>();  // every warp is done reading the stage
      float* accw = reinterpret_cast<float*>(s.tiles[stage]);  // [8][G][128]
      // the two half-warps hold different tokens of the same dims
#pragma unroll
      for (int g = 0; g < G; ++g)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          acc[g][c].x += __shfl_xor_sync(kFull, acc[g][c].x, 16);
          acc[g][c].y += __shfl_xor_sync(kFull, acc[g][c].y, 16);
        }
      // l of each head summed over the warp's 8 token slots
#pragma unroll
      for (int i = 0; i < VPL; ++i) {
        float ls = l_run[i] + __shfl_xor_sync(kFull, l_run[i], 4);
        ls += __shfl_xor_sync(kFull, ls, 8);
        ls += __shfl_xor_sync(kFull, ls, 16);
        const int v = pair0 + i;
        if (pair_writer && half == 0 && v / G == 0) {
          s.mw[warp][v % G] = m_run[i];
          s.lw[warp][v % G] = ls;
        }
      }
      if (half == 0) {
#pragma unroll
        for (int g = 0; g < G; ++g) {
          float* dst = &accw[(warp * G + g) * kHeadDim + 8 * l16];
          *reinterpret_cast<float4*>(dst) =
              make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
          *reinterpret_cast<float4*>(dst + 4) =
              make_float4(acc[g][2].x, acc[g][2].y, acc[g][3].x, acc[g][3].y);
        }
      }
      vsync<virt_ctas<G>()>();
      if (vtid<virt_ctas<G>()>() < G) {
        const int g = vtid<virt_ctas<G>()>();
        float M = -INFINITY;
        for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, s.mw[w][g]);
        float L = 0.f;
        for (int w = 0; w < kConsumerWarps; ++w) {
          const float f = (M == -INFINITY) ? 0.f : exp2f(s.mw[w][g] - M);
          s.wscale[w][g] = f;
          L += s.lw[w][g] * f;
        }
        s.cta_m[g] = M;
        s.cta_l[g] = L;
      }
      vsync<virt_ctas<G>()>();
      const int seg = info_seg(info);
      const int u = s.seg_unit[seg];
      const size_t out_base = (size_t)u * G * kHeadDim;
      const int nparts = s.seg_count[seg];
      if (nparts == 1) {
        for (int idx = vtid<virt_ctas<G>()>(); idx < G * kHeadDim; idx += kThreads) {
          const int g = idx / kHeadDim, d = idx % kHeadDim;
          float o = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w)
            o += accw[(w * G + g) * kHeadDim + d] * s.wscale[w][g];
          const float L = s.cta_l[g];
          store_out<G>(p, s, out_base, idx, L > 0.f ? o / L : 0.f);
        }
        if (p.gather_peers) gather_push<G>(p, s, u);
      } else {
        float* part =
            p.partial + ((size_t)u * p.max_segments + s.seg_index[seg]) * G * kPartialStride;
        for (int idx = vtid<virt_ctas<G>()>(); idx < G * kHeadDim; idx += kThreads) {
          const int g = idx / kHeadDim, d = idx % kHeadDim;
          float o = 0.f;
#pragma unroll
          for (int w = 0; w < kConsumerWarps; ++w)
            o += accw[(w * G + g) * kHeadDim + d] * s.wscale[w][g];
          part[g * kPartialStride + 2 + d] = o;
          if (d == 0) {
            part[g * kPartialStride] = s.cta_m[g];
            part[g * kPartialStride + 1] = s.cta_l[g];
          }
        }
        vsync<virt_ctas<G>()>();
        if (vtid<virt_ctas<G>()>() == 0)  // the barrier orders the partial stores before it
          s.last_flag = arrive_acq_rel(&p.counters[u]) == nparts - 1;
        vsync<virt_ctas<G>()>();
        if (s.last_flag) {
          const float* parts = p.partial + (size_t)u * p.max_segments * G * kPartialStride;
          // The partials' loads go out kMergeBatch at a time (a loop of
          // dependent L2 round trips took ~7 us when a unit had 9 parts);
          // they are still combined in range order.
          constexpr int kMergeBatch = 8;
          for (int idx = vtid<virt_ctas<G>()>(); idx < G * kHeadDim; idx += kThreads) {
            const int g = idx / kHeadDim, d = idx % kHeadDim;
            float M = -INFINITY;
            for (int k0 = 0; k0 < nparts; k0 += kMergeBatch) {
              float mk[kMergeBatch];
#pragma unroll
              for (int b = 0; b < kMergeBatch; ++b)
                mk[b] = k0 + b < nparts ? __ldcg(parts + ((k0 + b) * G + g) * kPartialStride)
                                        : -INFINITY;
#pragma unroll
              for (int b = 0; b < kMergeBatch; ++b) M = fmaxf(M, mk[b]);
            }
            float L = 0.f, o = 0.f;
            if (M != -INFINITY) {
              for (int k0 = 0; k0 < nparts; k0 += kMergeBatch) {
                float mk[kMergeBatch], lk[kMergeBatch], ok[kMergeBatch];
#pragma unroll
                for (int b = 0; b < kMergeBatch; ++b) {
                  const float* pk = parts + ((k0 + b) * G + g) * kPartialStride;
                  const bool in = k0 + b < nparts;
                  mk[b] = in ? __ldcg(pk) : 0.f;
                  lk[b] = in ? __ldcg(pk + 1) : 0.f;
                  ok[b] = in ? __ldcg(pk + 2 + d) : 0.f;
                }
#pragma unroll
                for (int b = 0; b < kMergeBatch; ++b) {
                  if (k0 + b < nparts) {
                    const float f = exp2f(mk[b] - M);
                    L += lk[b] * f;
                    o += ok[b] * f;
                  }
                }
              }
            }
            store_out<G>(p, s, out_base, idx, L > 0.f ? o / L : 0.f);
          }
          if (vtid<virt_ctas<G>()>() == 0) p.counters[u] = 0;
          if (p.gather_peers) gather_push<G>(p, s, u);
        }
      }
      vsync<virt_ctas<G>()>();  // the stage buffer is free again
    }

    // Refill this lane's part of the stage with stage j + kStages (after a
    // segment end only now: the merge used the stage as scratch).
    if (j + kStages < nstages) load_stage<G, kHeadMajor>(s, p, j + kStages, stage, half, t0, l16);
    cp_async_commit();
    if (++stage == kStages) stage = 0;
  }
  cp_async_wait<0>();  // only empty groups remain; nothing lands after exit
}

template <int G, bool kHeadMajor>
sa_status launch_layout(const AttnParams& p, cudaStream_t stream) {
  constexpr int kV = virt_ctas<G>();
  const size_t smem = kV * sizeof(AttnSmem<G>);
  static int configured[kMaxDevices];
  const sa_status st =
      ensure_smem_limit((const void*)attention_kernel<G, kHeadMajor>, (int)smem, configured);
  if (st != SA_OK) return st;
  const cudaError_t e = launch_kernel(attention_kernel<G, kHeadMajor>, dim3((p.ctas + kV - 1) / kV),
                                      dim3(kThreads * kV),
                                      smem, stream, p.pdl != 0, p);
  if (e != cudaSuccess) return cuda_status(e, "attention_kernel launch");
  return cuda_status(cudaGetLastError(), "attention_kernel launch");
}

template <int G>
sa_status launch_g(const AttnParams& p, cudaStream_t stream) {
  return p.head_major ? launch_layout<G, true>(p, stream) : launch_layout<G, false>(p, stream);
}

// Waits (bounded) until this rank's counter holds the arrivals of gather
// epoch + 1, then advances the epoch: the next attention writes the other
// slot. Epoch and expected count live on the device, so a recorded graph
// replays them correctly.
__global__ void gather_wait_kernel(void* const* peers, int world, size_t counter_bytes,
                                   const unsigned long long* counter, unsigned long long* epoch,
                                   unsigned long long per_epoch, uint32_t* status) {
  if (threadIdx.x != 0) return;
  gather_signal_wait(peers, world, counter_bytes, counter, epoch, per_epoch, false, status);
}

}  // namespace

sa_status launch_gather_wait(void* const* peers, int world, size_t counter_bytes,
                             const unsigned long long* counter, unsigned long long* epoch,
                             unsigned long long per_epoch, uint32_t* status, cudaStream_t stream) {
  gather_wait_kernel<<<1, 32, 0, stream>>>(peers, world, counter_bytes, counter, epoch, per_epoch,
                                           status);
  return cuda_status(cudaGetLastError(), "gather_wait_kernel launch");
}

AttnPlan attention_plan(int units, int slots_per_unit, int group, int sms) {
  const long long E = std::max(1, slots_per_unit);
  const long long U = std::max(1, units);
  const long long total = U * E;
  const long long wave = (long long)std::max(1, sms) * (group <= 4 ? 2 : 1);  // resident CTAs
  // Estimated time of a CTA count, in stage times (two slots per stage): the
  // CTAs run in ceil(C / wave) waves; a segment end (the 8-warp merge and the
  // next unit's start) costs about five stages, and a unit split over n CTAs
  // 2 + n/8 more (its partials and their merge by the last CTA). Five, not
  // three: at cfg2 (224 units of 65 slots) one whole unit per CTA ran the
  // attention in 44.2 us, against 47.9 us for 296 CTAs splitting units.
  auto cost = [&](long long C) -> double {
    if (C < 1 || C > total) return 1e30;
    const long long per = (total + C - 1) / C;
    if (per > kMaxCtaSlots) return 1e30;
    long long segs, stages;
    bool split;
    if (C % U == 0) {  // k CTAs per unit, ranges aligned to units
      segs = 1;
      stages = (per + 1) / 2;
      split = C > U;
    } else if (U % C == 0) {  // k whole units per CTA
      segs = U / C;
      stages = segs * ((E + 1) / 2);
      split = false;
    } else {
      segs = (per + E - 2) / E + 1;
      stages = (per + 1) / 2 + segs - 1;
      split = true;
    }
    if (segs > kMaxSegments) return 1e30;
    const long long waves = (C + wave - 1) / wave;
    const double parts = split ? (double)((E + per - 1) / per + 1) : 0.0;
    return (double)waves * (double)(stages + 5 * segs) + (split ? 2.0 + parts / 8.0 : 0.0);
  };
  long long best = 0;
  double best_cost = 1e30;
  auto consider = [&](long long C) {
    const double c = cost(C);
    if (c < best_cost || (c == best_cost && C < best)) {
      best_cost = c;
      best = C;
    }
  };
  for (long long k = 1; k <= 64; ++k) consider(U * k);
  for (long long k = 2; k <= kMaxSegments; ++k)
    if (U % k == 0) consider(U / k);
  for (long long w = 1; w <= 8; ++w) {
    const long long per = (total + wave * w - 1) / (wave * w);
    consider((total + per - 1) / per);
  }
  if (best == 0) best = (total + kMaxCtaSlots - 1) / kMaxCtaSlots;  // always feasible
  AttnPlan plan{};
  plan.slots_per_unit = (int)E;
  plan.ctas = (int)best;
  // every CTA owns at least floor(total / ctas) slots
  const long long min_slots = std::max<long long>(1, total / best);
  plan.max_segments = (int)((E + min_slots - 1) / min_slots + 1);
  return plan;
}

size_t attention_scratch_bytes(const AttnPlan& plan, int units, int group) {
  return (size_t)units * plan.max_segments * group * kPartialStride * sizeof(float);
}

sa_status launch_attention(const AttnParams& p, cudaStream_t stream) {
  if (p.num_sl <= 0 || p.kv_heads <= 0 || p.ctas <= 0) return SA_OK;
  switch (p.group) {
    case 1: return launch_g<1>(p, stream);
    case 2: return launch_g<2>(p, stream);
    case 4: return launch_g<4>(p, stream);
    case 8: return launch_g<8>(p, stream);
    default: return fail(SA_ERR_UNSUPPORTED, "attention: query heads per KV head must be 1, 2, 4 or 8");
  }
}

}  // namespace sa
