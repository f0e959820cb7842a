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
// stages. Every warp reads only its own rows (below), so its lanes load
// exactly those rows themselves, with 16-byte cp.async copies through the
// load/store unit, one commit group per stage: a warp waits only for its own
// copies and refills its part of a stage as soon as it has computed on it,
// with no producer thread and no cross-warp release.
// (On a B200, streaming random 16 KB blocks: one thread per SM issuing 16 KB
// bulk copies read at most 4.3 TB/s and two such threads per SM 6.6 TB/s,
// whatever the number of copies in flight, while 16-byte cp.async copies
// reached 7.2 TB/s with 128 KB in flight per SM.) Rows come from the decode
// context's head-major pool or from a caller's token-major rows; the
// shared-memory layout is the same.
//
// Warp w, per stage: rows [4w, 4w + 4) of both entries, 8 token rows, which
// are also exactly the rows its lanes copy (so a warp waits only for its own
// copies). The products run on the tensor cores (mma.sync, FP16 operands,
// FP32 accumulation) with FP32-level accuracy: the FP32 query and the FP32
// probabilities enter as FP16 hi + lo pairs (each pre-scaled by a power of
// two), K and V are FP16 already, so every product is exact and the two
// parts carry about 22 bits. S^T (8 rows x 8 head columns) = K . q^T takes
// 16 m16n8k16 MMAs (A from ldmatrix, q^T held in registers for the
// segment); the FP32 online softmax (exp2 domain, running max per head over
// the warp's rows, rescaled lazily: only when a logit exceeds it by 2^8)
// works on the accumulator fragments; movmatrix turns the probabilities into
// the P^T operand, and O^T (128 dims x 8 head columns) += V^T . P^T takes 16
// m16n8k8 MMAs (A from ldmatrix.trans). Per lane and stage that is ~110
// instructions where FP32 FMAs on converted FP16 pairs took ~300. Shared
// memory holds chunk c of warp-local row r at chunk c ^ r (conflict-free
// ldmatrix); rows past an entry's token count are zeroed.
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

// ---- tensor-core fragments (mma.sync, FP16 operands, FP32 accumulation) ----
//
// A warp owns 8 rows of a stage: tokens [t0, t0 + 4) of entry 0 (rows 0-3)
// and of entry 1 (rows 4-7). In shared memory the 16-byte chunk c of row r
// lives at chunk c ^ r, so the 8 row addresses of one ldmatrix fall into 8
// different bank groups.
__device__ __forceinline__ uint32_t smem_u32(const void* ptr) {
  return (uint32_t)__cvta_generic_to_shared(ptr);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// d += A (16 x 16, rows 8-15 zero: a1 = a3 = 0) * B (16 x 8)
__device__ __forceinline__ void mma_k16_top(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0,
                                            uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

// d += A (16 x 8) * B (8 x 8)
__device__ __forceinline__ void mma_k8(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5}, {%6}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(b0));
}

// The transpose of an 8 x 8 matrix of 16-bit values held one pair per lane.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t a) {
  uint32_t d;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(d) : "r"(a));
  return d;
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// (x, y) as FP16 hi + lo pairs: x = hi.x + lo.x to about 2^-22 relative.
__device__ __forceinline__ void split_f16x2(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 hf = __half22float2(h);
  hi = h2_bits(h);
  lo = h2_bits(__floats2half2_rn(x - hf.x, y - hf.y));
}

// 2^e as a float, e in [-126, 127].
__device__ __forceinline__ float exp2_int(int e) { return __int_as_float((e + 127) << 23); }

// This lane's copies for stage j into shared-memory stage `slot`: rows
// [t0, t0 + 4) of entry `half`, K then V plane, the 16 bytes of chunk l16
// (placed at chunk l16 ^ r for the warp-local row r = 4 half + row). Rows at
// or past the entry's token count are zeroed instead: the MMAs multiply
// them by zero probabilities, and stale bytes there could be NaN patterns.
template <int G, bool kHeadMajor>
__device__ __forceinline__ void load_stage(AttnSmem<G>& s, const AttnParams& p, int j, int slot,
                                           int half, int t0, int l16) {
  const uint32_t w = s.stage_info[j];
  const int ntok = info_ntok(w, half);
  uint8_t* dst = s.tiles[slot] + half * kEntryBytes + t0 * kRowBytes;
  if (ntok <= t0) {
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int c = (l16 ^ (4 * half + r)) * 16;
      *reinterpret_cast<uint4*>(dst + r * kRowBytes + c) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(dst + kPlaneBytes + r * kRowBytes + c) = make_uint4(0u, 0u, 0u, 0u);
    }
    return;
  }
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
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    uint8_t* d = dst + r * kRowBytes + (l16 ^ (4 * half + r)) * 16;
    if (t0 + r < ntok) {
      cp_async16(d, src + r * row_stride);
      cp_async16(d + kPlaneBytes, src + plane + r * row_stride);
    } else {
      *reinterpret_cast<uint4*>(d) = make_uint4(0u, 0u, 0u, 0u);
      *reinterpret_cast<uint4*>(d + kPlaneBytes) = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

// One plane (0: K rows, 1: V rows) of load_stage's copies. Loading a stage
// plane by plane (all K rows, then all V rows) instead of row by row runs
// the attention faster on some plans and slower on others (see launch_g).
template <int G, bool kHeadMajor>
__device__ __forceinline__ void load_plane(AttnSmem<G>& s, const AttnParams& p, int j, int slot,
                                           int pl, int half, int t0, int l16) {
  const uint32_t w = s.stage_info[j];
  const int ntok = info_ntok(w, half);
  uint8_t* dst = s.tiles[slot] + half * kEntryBytes + pl * kPlaneBytes + t0 * kRowBytes;
  if (ntok <= t0) {
#pragma unroll
    for (int r = 0; r < 4; ++r)
      *reinterpret_cast<uint4*>(dst + r * kRowBytes + (l16 ^ (4 * half + r)) * 16) =
          make_uint4(0u, 0u, 0u, 0u);
    return;
  }
  const int phys = s.ent_phys[info_e0(w) + half];
  const int kvh = s.seg_unit[info_seg(w)] % p.kv_heads;
  const uint8_t* src;
  size_t row_stride;
  if constexpr (kHeadMajor) {
    src = reinterpret_cast<const uint8_t*>(p.pool) +
          ((size_t)phys * p.kv_heads + kvh) * kEntryBytes + (size_t)pl * kPlaneBytes +
          (size_t)t0 * kRowBytes;
    row_stride = kRowBytes;
  } else {
    src = reinterpret_cast<const uint8_t*>(p.rows) +
          ((size_t)phys * kBlockTokens + t0) * (size_t)p.row_bytes +
          (size_t)(pl * p.kv_heads + kvh) * kRowBytes;
    row_stride = (size_t)p.row_bytes;
  }
  src += l16 * 16;
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    uint8_t* d = dst + r * kRowBytes + (l16 ^ (4 * half + r)) * 16;
    if (t0 + r < ntok) cp_async16(d, src + r * row_stride);
    else *reinterpret_cast<uint4*>(d) = make_uint4(0u, 0u, 0u, 0u);
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

template <int G, bool kHeadMajor, bool kPlaneOrder>
__global__ void __launch_bounds__(kThreads * virt_ctas<G>(), 1)
    attention_kernel(const AttnParams p) {
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

  const int half = lane >> 4;      // the entry this lane copies
  const int l16 = lane & 15;       // the 16-byte chunk of a 256-byte row it copies
  const int t0 = 4 * warp;
  // MMA fragment coordinates: row group g (a token row of the warp, or a
  // head for the q and P^T operands), pair t (heads 2t, 2t + 1 of the
  // logits and the accumulators).
  const int g = lane >> 2, t = lane & 3;
  // ldmatrix: lane L gives the address of row L & 7 of matrix L >> 3.
  const int lr = lane & 7;
  const uint32_t row_off = (uint32_t)((lr >> 2) * kEntryBytes + (t0 + (lr & 3)) * kRowBytes);
  // chunk 4 kk + (lane >> 3) of row lr sits at chunk_off(kk)
  auto chunk_off = [&](int kk) { return (uint32_t)(((4 * kk + (lane >> 3)) ^ lr) * 16); };
  // logit row g is token t0 + (g & 3) of entry g >> 2
  const int my_tok = t0 + (g & 3);
  const int my_ent = g >> 2;
  // one commit group per stage, the first kStages in flight before the loop
#pragma unroll
  for (int j = 0; j < kStages; ++j) {
    if (j < nstages) {
      if constexpr (kPlaneOrder) {
        load_plane<G, kHeadMajor>(s, p, j, j, 0, half, t0, l16);
        load_plane<G, kHeadMajor>(s, p, j, j, 1, half, t0, l16);
      } else {
        load_stage<G, kHeadMajor>(s, p, j, j, half, t0, l16);
      }
    }
    cp_async_commit();
  }

  // per head 2t + i: running max (log2 units), lazy-rescale threshold, sum of
  // this lane's row's probabilities
  float m_run[2], m_thr[2], l_run[2];
  float acc[8][4];       // O^T: dims 16 m + g (+ 8) x heads 2t, 2t + 1, probabilities x 2^7
  uint32_t qh[8][2], ql[8][2];  // q^T fragments of head g, hi and lo FP16 parts
  float q_unscale = 1.f;        // logits = MMA result * q_unscale
  int stage = 0;

  for (int j = 0; j < nstages; ++j) {
    const uint32_t info = s.stage_info[j];
    if (info & kInfoStart) {
      // ---- a new segment: its unit's q in the exp2 domain, scaled by a power
      // of two so that its largest element is in [2^14, 2^15), split into
      // FP16 hi + lo parts; fresh softmax state ----
      const float* qrow = p.query + ((size_t)s.seg_unit[info_seg(info)] * G + g) * kHeadDim + 2 * t;
      float2 qv[8][2];
      uint32_t amax = 0u;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float2 v = make_float2(0.f, 0.f);
          if (g < G) v = __ldg(reinterpret_cast<const float2*>(qrow + 16 * k + 8 * h));
          v.x *= p.scale_log2;
          v.y *= p.scale_log2;
          qv[k][h] = v;
          amax = max(amax, max(__float_as_uint(fabsf(v.x)), __float_as_uint(fabsf(v.y))));
        }
      }
      amax = __reduce_max_sync(kFull, amax);
      const int e = amax == 0u ? 0 : (int)((amax >> 23) & 0xff) - 127;
      const int qe = max(-100, min(100, 14 - e));
      const float up = exp2_int(qe);
      q_unscale = exp2_int(-qe);
#pragma unroll
      for (int k = 0; k < 8; ++k)
#pragma unroll
        for (int h = 0; h < 2; ++h)
          split_f16x2(qv[k][h].x * up, qv[k][h].y * up, qh[k][h], ql[k][h]);
#pragma unroll
      for (int m = 0; m < 8; ++m)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[m][c] = 0.f;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        m_run[i] = -INFINITY;
        m_thr[i] = -INFINITY;
        l_run[i] = 0.f;
      }
    }
    cp_async_wait<kStages - 1>();  // this lane's copies of stage j have landed
    __syncwarp();                  // ... and the other lanes' (ldmatrix reads them)
    const int ntok0 = info_ntok(info, 0);
    const int ntok1 = info_ntok(info, 1);
    const bool active = t0 < ntok0 || t0 < ntok1;
    const uint32_t kbase = smem_u32(s.tiles[stage]) + row_off;
    float x[2] = {-INFINITY, -INFINITY};
    if (active) {
      // ---- S^T (8 token rows x 8 heads) = K rows . q^T, hi and lo parts ----
      // four independent accumulation chains (hi / lo x even / odd k-steps)
      float sh0[4] = {0.f, 0.f, 0.f, 0.f}, sh1[4] = {0.f, 0.f, 0.f, 0.f};
      float sl0[4] = {0.f, 0.f, 0.f, 0.f}, sl1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t a[4];
        ldsm_x4(kbase + chunk_off(kk), a);
        mma_k16_top(sh0, a[0], a[1], qh[2 * kk][0], qh[2 * kk][1]);
        mma_k16_top(sh1, a[2], a[3], qh[2 * kk + 1][0], qh[2 * kk + 1][1]);
        mma_k16_top(sl0, a[0], a[1], ql[2 * kk][0], ql[2 * kk][1]);
        mma_k16_top(sl1, a[2], a[3], ql[2 * kk + 1][0], ql[2 * kk + 1][1]);
      }
      const bool valid = my_tok < (my_ent ? ntok1 : ntok0);
      x[0] = valid ? ((sh0[0] + sh1[0]) + (sl0[0] + sl1[0])) * q_unscale : -INFINITY;
      x[1] = valid ? ((sh0[1] + sh1[1]) + (sl0[1] + sl1[1])) * q_unscale : -INFINITY;
    }
    // (QK and the softmax + PV in two blocks around a warp barrier: on a
    // B200 the per-rank share of eight GPUs ran 20.4 -> 19.6 us)
    __syncwarp();
    if (active) {
      // ---- online softmax over the warp's 8 rows per head, lazily rescaled:
      // the running max moves only when a logit exceeds it by more than
      // kLazyRescale (log2 units), so probabilities stay below 2^kLazyRescale ----
      const bool rescale = __any_sync(kFull, x[0] > m_thr[0] || x[1] > m_thr[1]);
      if (rescale) {
        float alpha[2];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          float bm = fmaxf(x[i], __shfl_xor_sync(kFull, x[i], 4));
          bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 8));
          bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 16));
          const float m_new = fmaxf(m_run[i], bm);
          alpha[i] = m_new == -INFINITY ? 1.f : fast_exp2(m_run[i] - m_new);
          m_run[i] = m_new;
          m_thr[i] = m_new + kLazyRescale;
          l_run[i] *= alpha[i];
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
          acc[m][0] *= alpha[0];
          acc[m][1] *= alpha[1];
          acc[m][2] *= alpha[0];
          acc[m][3] *= alpha[1];
        }
      }
      float pr[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        pr[i] = x[i] == -INFINITY ? 0.f : fast_exp2(x[i] - m_run[i]);
        l_run[i] += pr[i];
      }
      // ---- P^T operand: (row g, heads 2t, 2t+1) pairs, scaled by 2^7 and split
      // into FP16 hi + lo, transposed to (rows 2t, 2t+1, head g) ----
      uint32_t ph, pl;
      split_f16x2(pr[0] * 128.f, pr[1] * 128.f, ph, pl);
      ph = movmatrix_trans(ph);
      pl = movmatrix_trans(pl);
      // ---- O^T (128 dims x 8 heads) += V^T . P^T ----
      const uint32_t vbase = kbase + kPlaneBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t v[4];
        ldsm_x4_trans(vbase + chunk_off(kk), v);
        mma_k8(acc[2 * kk], v[0], v[1], ph);
        mma_k8(acc[2 * kk], v[0], v[1], pl);
        mma_k8(acc[2 * kk + 1], v[2], v[3], ph);
        mma_k8(acc[2 * kk + 1], v[2], v[3], pl);
      }
    }
    __syncwarp();  // the warp's ldmatrix reads of this stage are done before its refill

    if (info & kInfoEnd) {
      // ---- segment end: merge the 8 warps through this stage's buffer ----
      vsync<virt_ctas<G>()>();  // every warp is done reading the stage
      float* accw = reinterpret_cast<float*>(s.tiles[stage]);  // [8][G][128]
      // l of each head summed over the warp's 8 rows (the lanes sharing t)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        float ls = l_run[i] + __shfl_xor_sync(kFull, l_run[i], 4);
        ls += __shfl_xor_sync(kFull, ls, 8);
        ls += __shfl_xor_sync(kFull, ls, 16);
        const int h = 2 * t + i;
        if (g == 0 && h < G) {
          s.mw[warp][h] = m_run[i];
          s.lw[warp][h] = ls;
        }
      }
      // the warp's O^T fragments, back to unscaled probabilities
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int h = 2 * t + i;
        if (h < G) {
          float* dst = &accw[(warp * G + h) * kHeadDim + g];
#pragma unroll
          for (int m = 0; m < 8; ++m) {
            dst[16 * m] = acc[m][i] * (1.f / 128.f);
            dst[16 * m + 8] = acc[m][2 + i] * (1.f / 128.f);
          }
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
    if (j + kStages < nstages) {
      if constexpr (kPlaneOrder) {
        load_plane<G, kHeadMajor>(s, p, j + kStages, stage, 0, half, t0, l16);
        load_plane<G, kHeadMajor>(s, p, j + kStages, stage, 1, half, t0, l16);
      } else {
        load_stage<G, kHeadMajor>(s, p, j + kStages, stage, half, t0, l16);
      }
    }
    cp_async_commit();
    if (++stage == kStages) stage = 0;
  }
  cp_async_wait<0>();  // only empty groups remain; nothing lands after exit
}

template <int G, bool kHeadMajor, bool kPlaneOrder>
sa_status launch_layout(const AttnParams& p, cudaStream_t stream) {
  constexpr int kV = virt_ctas<G>();
  const size_t smem = kV * sizeof(AttnSmem<G>);
  static int configured[kMaxDevices];
  const sa_status st = ensure_smem_limit((const void*)attention_kernel<G, kHeadMajor, kPlaneOrder>,
                                         (int)smem, configured);
  if (st != SA_OK) return st;
  const cudaError_t e = launch_kernel(attention_kernel<G, kHeadMajor, kPlaneOrder>,
                                      dim3((p.ctas + kV - 1) / kV),
                                      dim3(kThreads * kV),
                                      smem, stream, p.pdl != 0, p);
  if (e != cudaSuccess) return cuda_status(e, "attention_kernel launch");
  return cuda_status(cudaGetLastError(), "attention_kernel launch");
}

template <int G>
sa_status launch_g(const AttnParams& p, cudaStream_t stream) {
  // Stages load plane by plane (load_plane) when the virtual CTAs fill about
  // a wave, every one streams a range inside one unit (k per unit) and the
  // ranges are long: on a B200, 288 units of 129 slots on 288 virtual CTAs
  // 104.5 -> 94.7 us, 144 units on 288 (two per unit) 57.3 -> 54.6 us;
  // shorter ranges (72 units on 288: 33.7 -> 34.0 us; 36 on 288: 19.6 ->
  // 21.7 us), several units per CTA (2,304 units on 296: 368 -> 439 us) or
  // a part of the SMs idle (224 units on 224: 43.4 -> 49.9 us) run slower.
  const long long units = (long long)p.num_sl * p.kv_heads;
  const long long slots = units * p.slots_per_unit;
  const long long wave = (long long)device_sm_count() * virt_ctas<G>();
  const bool plane_order = (long long)p.ctas * 10 >= wave * 9 && p.ctas % units == 0 &&
                           slots >= 64LL * p.ctas;
  if (p.head_major)
    return plane_order ? launch_layout<G, true, true>(p, stream)
                       : launch_layout<G, true, false>(p, stream);
  return plane_order ? launch_layout<G, false, true>(p, stream)
                     : launch_layout<G, false, false>(p, stream);
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
