// sa_attention.cu -- block-sparse GQA decode attention for sm_100a.
//
// Replaces the reference's attention (cpp/src/attention_reference.cpp:55-96)
// and its device kernels sparse_attention_parallel
// (cpp/src/cuda_backend.cpp:109-158) and sparse_fp16_attention
// (cpp/src/qwen_layer_main.cpp:224-268).
//
// Work unit: one (sequence-layer, KV head). Its token set is a list of
// entries: the selected sealed blocks (logical ids -> physical pool blocks
// through the block table) followed by the open tail (tail_len tokens).
// A CTA takes `split_entries` consecutive entries of one unit; their
// (physical block, token count) pairs are resolved once, in parallel, into
// shared memory.
//
// Pipeline: a stage holds two entries (2 x 16 KB: the K rows then the V rows
// of the unit's KV head, 32 x 256 B each) in a ring of three stages. Entries
// of the decode context's head-major pool arrive as one contiguous 16 KB
// bulk copy; entries of a caller's token-major buffer as two 8 KB TMA tiles
// (32 rows x 256 B) -- the shared-memory layout is the same. A stage's TMA loads complete a "full" mbarrier (bounded
// waits); the last of the eight warps to release a stage (a shared-memory
// arrival counter) issues the loads that refill it, so no warp ever blocks
// on a producer.
//
// Consumer warp w, per stage: half-warp h takes entry h of the stage and its
// tokens [4w, 4w+4); lane l covers head dims [8(l%16), 8(l%16)+8). A
// quarter-warp reads 128 contiguous bytes of one row: conflict-free. QK uses packed FP32
// FMA (__ffma2_rn) with the softmax scale folded into q, then a 16-lane
// transpose-reduce leaves one (token, head) logit per lane. The warp keeps an
// FP32 online softmax per head (exp2 domain, running max shared by both
// half-warps) and skips the accumulator rescale when no running max moved.
// At the end the warps merge by log-sum-exp; with several splits per unit
// each CTA writes a partial (m, l, o[128]) and the last CTA to arrive (atomic
// counter, no spinning) merges them in split order, so the result does not
// depend on CTA timing.
#include <algorithm>

#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = kConsumerWarps * 32;
constexpr int kStages = 3;
constexpr int kRowBytes = kHeadDim * 2;          // one token of one head, FP16
constexpr int kPlaneBytes = kBlockTokens * kRowBytes;  // 32 rows: 8 KB
constexpr int kEntryBytes = 2 * kPlaneBytes;     // K plane then V plane
constexpr int kStageBytes = 2 * kEntryBytes;     // two entries per stage
constexpr int kPartialStride = 2 + kHeadDim;     // m, l, o[128]
constexpr int kMaxSplitEntries = 64;
constexpr unsigned kFull = 0xffffffffu;

template <int G>
struct alignas(128) AttnSmem {
  uint8_t tiles[kStages][kStageBytes];
  float pbuf[kConsumerWarps][2][4][G];  // probabilities [half][token][head]
  float abuf[kConsumerWarps][G];        // rescale factor per head
  float wscale[kConsumerWarps][G];
  float cta_m[G];
  float cta_l[G];
  int ent_phys[kMaxSplitEntries];
  int ent_ntok[kMaxSplitEntries];
  uint64_t full[kStages];
  int released[kStages];      // warps done with the stage's current contents
  int stage_issues[kStages];  // loads issued into the stage so far
  int abort_flag;
  int last_flag;
};

struct Entry {
  int phys;
  int ntok;
};

__device__ __forceinline__ Entry unit_entry(const AttnParams& p, int sl, int sgroup, int nsel,
                                            int tail_len, int e) {
  Entry r;
  if (e < nsel) {
    const int logical =
        p.sel_ids ? p.sel_ids[(sl * p.n_sel_groups + sgroup) * p.sel_stride + e] : e;
    if (p.table) {
      if (logical < 0 || logical >= p.table_stride) {
        raise_status(p.status, SA_DEV_BAD_BLOCK);
        return {0, 0};
      }
      r.phys = p.table[(size_t)sl * p.table_stride + logical];
    } else {
      r.phys = logical;
    }
    r.ntok = kBlockTokens;
  } else {
    r.phys = p.tail_block ? p.tail_block[sl] : p.fixed_tail_block;
    r.ntok = tail_len;
  }
  if (r.phys < 0 || r.phys >= p.pool_blocks) {
    raise_status(p.status, SA_DEV_BAD_BLOCK);
    return {0, 0};
  }
  return r;
}

// The hardware base-2 exponential (ex2.approx, ~2 ulp).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// In-warp transpose-reduce step chain: M values per lane, halving at lane
// offset OFF, then OFF/2, ...; a lane keeps the lower half of its values when
// its OFF bit is clear (the upper half otherwise) and adds the partner's copy.
template <int M, int OFF>
struct Halve {
  __device__ __forceinline__ static void run(float* a, int lane) {
    if constexpr (M > 1 && OFF >= 1) {
      const bool upper = (lane & OFF) != 0;
#pragma unroll
      for (int j = 0; j < M / 2; ++j) {
        const float keep = upper ? a[j + M / 2] : a[j];
        const float send = upper ? a[j] : a[j + M / 2];
        a[j] = keep + __shfl_xor_sync(kFull, send, OFF);
      }
      Halve<M / 2, OFF / 2>::run(a, lane);
    }
  }
};

__device__ __forceinline__ void unpack8(const uint4& u, float2 (&f)[4]) {
  f[0] = h2x2f(u.x);
  f[1] = h2x2f(u.y);
  f[2] = h2x2f(u.z);
  f[3] = h2x2f(u.w);
}

// Issues the loads of stage j (entries 2j, 2j+1 of the CTA's range): one 16 KB
// bulk copy per entry from a head-major pool, or two 8 KB TMA tiles per entry
// from a token-major buffer.
template <int G, bool kHeadMajor>
__device__ __forceinline__ void issue_stage(AttnSmem<G>& s, const CUtensorMap* map,
                                            const uint8_t* pool, int kv_heads, int kvh, int n,
                                            int j) {
  const int stage = j % kStages;
  uint32_t tx = 0;
  for (int e = 2 * j; e < min(n, 2 * j + 2); ++e) tx += s.ent_ntok[e] > 0 ? kEntryBytes : 0;
  if (tx) {
    mbar_arrive_expect_tx(&s.full[stage], tx);
    for (int e = 2 * j; e < min(n, 2 * j + 2); ++e) {
      if (s.ent_ntok[e] <= 0) continue;
      uint8_t* dst = s.tiles[stage] + (e & 1) * kEntryBytes;
      if constexpr (kHeadMajor) {
        bulk_load(dst, pool + ((size_t)s.ent_phys[e] * kv_heads + kvh) * kEntryBytes, kEntryBytes,
                  &s.full[stage]);
      } else {
        const int y = s.ent_phys[e] * kBlockTokens;
        tma_load_2d(dst, map, &s.full[stage], kvh * kHeadDim, y);
        tma_load_2d(dst + kPlaneBytes, map, &s.full[stage], (kv_heads + kvh) * kHeadDim, y);
      }
    }
  } else {
    mbar_arrive(&s.full[stage]);
  }
  s.stage_issues[stage] += 1;
}

template <int G, bool kHeadMajor>
__global__ void __launch_bounds__(kThreads, (G <= 4 ? 2 : 1))
    attention_kernel(const __grid_constant__ CUtensorMap map, const AttnParams p) {
  // Pairs (token, head) per half-warp: 4G over 16 lanes -> VPL per lane.
  constexpr int NPH = 4 * G;
  constexpr int VPL = NPH > 16 ? NPH / 16 : 1;
  constexpr int kPairShift = NPH >= 16 ? 0 : (NPH == 8 ? 1 : 2);  // lanes per pair = 1 << shift
  extern __shared__ __align__(128) uint8_t smem_raw[];
  AttnSmem<G>& s = *reinterpret_cast<AttnSmem<G>*>(smem_raw);
  const uint8_t* pool = reinterpret_cast<const uint8_t*>(p.pool);

  const int unit = blockIdx.y;
  const int split = blockIdx.x;
  const int sl = unit / p.kv_heads;
  const int kvh = unit - sl * p.kv_heads;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int sgroup = kvh / p.kv_per_sel_group;
  int nsel = p.sel_count ? p.sel_count[sl * p.n_sel_groups + sgroup] : p.fixed_nsel;
  nsel = max(0, min(nsel, p.sel_ids ? p.sel_stride : nsel));
  int tail_len = p.tail_len ? p.tail_len[sl] : p.fixed_tail_len;
  tail_len = max(0, min(tail_len, kBlockTokens));
  const int entries = nsel + (tail_len > 0 ? 1 : 0);
  const int nsplit = max(1, (entries + p.split_entries - 1) / p.split_entries);
  if (split >= nsplit) return;
  const int e_begin = split * p.split_entries;
  const int n = max(0, min(min(entries, e_begin + p.split_entries) - e_begin, kMaxSplitEntries));
  const int nstages = (n + 1) / 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&s.full[i], 1);
      s.released[i] = 0;
      s.stage_issues[i] = 0;
    }
    s.abort_flag = 0;
    mbar_fence_init();
    if constexpr (!kHeadMajor) tma_prefetch_desc(&map);
  }
  for (int i = threadIdx.x; i < n; i += kThreads) {
    const Entry en = unit_entry(p, sl, sgroup, nsel, tail_len, e_begin + i);
    s.ent_phys[i] = en.phys;
    s.ent_ntok[i] = en.ntok;
  }
  __syncthreads();

  const int half = lane >> 4;      // which entry of the stage
  const int l16 = lane & 15;       // 16 B (8 dims) column of a 256 B row
  const int t0 = 4 * warp;
  // Byte offset of this lane's first K row inside its entry's tile.
  const int lane_off = half * kEntryBytes + t0 * kRowBytes + l16 * 16;

  float m_run[VPL], l_run[VPL];
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    m_run[j] = -INFINITY;
    l_run[j] = 0.f;
  }
  float2 acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[g][c] = make_float2(0.f, 0.f);

  if (threadIdx.x == 0)
    for (int j = 0; j < min(kStages, nstages); ++j)
      issue_stage<G, kHeadMajor>(s, &map, pool, p.kv_heads, kvh, n, j);
  {
    // ---------------- every warp consumes ----------------
    // q of this lane's 8 dims for the unit's G heads, pre-scaled into the
    // exp2 domain.
    float2 q[G][4];
    {
      const float* qbase = p.query + ((size_t)sl * p.kv_heads * G + (size_t)kvh * G) * kHeadDim +
                           8 * l16;
#pragma unroll
      for (int g = 0; g < G; ++g) {
        const float4 a = __ldg(reinterpret_cast<const float4*>(qbase + g * kHeadDim));
        const float4 b = __ldg(reinterpret_cast<const float4*>(qbase + g * kHeadDim + 4));
        q[g][0] = make_float2(a.x * p.scale_log2, a.y * p.scale_log2);
        q[g][1] = make_float2(a.z * p.scale_log2, a.w * p.scale_log2);
        q[g][2] = make_float2(b.x * p.scale_log2, b.y * p.scale_log2);
        q[g][3] = make_float2(b.z * p.scale_log2, b.w * p.scale_log2);
      }
    }

    for (int j = 0; j < nstages; ++j) {
      const int stage = j % kStages;
      if (*reinterpret_cast<volatile int*>(&s.abort_flag)) break;
      if (!mbar_wait_bounded(&s.full[stage], (j / kStages) & 1, p.status)) {
        atomicExch(&s.abort_flag, 1);
        break;
      }
      const int e = 2 * j + half;
      const int ntok = e < n ? s.ent_ntok[e] : 0;
      const int e_other = 2 * j + (half ^ 1);
      const int ntok_other = e_other < n ? s.ent_ntok[e_other] : 0;
      if (t0 < ntok || t0 < ntok_other) {
        const uint8_t* krow = s.tiles[stage] + lane_off;
        const uint8_t* vrow = krow + kPlaneBytes;
        // ---- QK over this lane's 8 dims, 4 tokens x G heads ----
        float part[NPH];
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
          float2 k[4];
          unpack8(*reinterpret_cast<const uint4*>(krow + tt * kRowBytes), k);
#pragma unroll
          for (int g = 0; g < G; ++g) {
            float2 a = __fmul2_rn(q[g][0], k[0]);
            a = __ffma2_rn(q[g][1], k[1], a);
            a = __ffma2_rn(q[g][2], k[2], a);
            a = __ffma2_rn(q[g][3], k[3], a);
            part[tt * G + g] = a.x + a.y;
          }
        }
        // 16-lane transpose-reduce: lane keeps VPL logits of pairs
        // v = ((l16 >> kPairShift) * VPL + i) = (token tt, head g) as tt * G + g.
        Halve<NPH, 8>::run(part, lane);
        if constexpr (NPH < 16) {
#pragma unroll
          for (int off = 1 << (kPairShift - 1); off >= 1; off >>= 1)
            part[0] += __shfl_xor_sync(kFull, part[0], off);
        }
        // ---- online softmax: 8 tokens (4 per half-warp) per head ----
        float pr[VPL], alpha[VPL];
        bool moved = false;
#pragma unroll
        for (int i = 0; i < VPL; ++i) {
          const int v = (l16 >> kPairShift) * VPL + i;
          const int tt = v / G;
          const float x = (t0 + tt < ntok) ? part[i] : -INFINITY;
          float bm = fmaxf(x, __shfl_xor_sync(kFull, x, 4));
          bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 8));
          bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 16));
          const float m_new = fmaxf(m_run[i], bm);
          alpha[i] = 1.f;
          pr[i] = 0.f;
          if (m_new != -INFINITY) {
            alpha[i] = fast_exp2(m_run[i] - m_new);
            pr[i] = fast_exp2(x - m_new);
          }
          moved |= m_new != m_run[i];
          m_run[i] = m_new;
          l_run[i] = l_run[i] * alpha[i] + pr[i];
        }
        if ((l16 & ((1 << kPairShift) - 1)) == 0) {
#pragma unroll
          for (int i = 0; i < VPL; ++i) {
            const int v = (l16 >> kPairShift) * VPL + i;
            s.pbuf[warp][half][v / G][v % G] = pr[i];
            if (half == 0 && v / G == 0) s.abuf[warp][v % G] = alpha[i];
          }
        }
        const bool rescale = __any_sync(kFull, moved);
        __syncwarp();
        // ---- PV over the half-warp's 4 tokens ----
        if (rescale) {
#pragma unroll
          for (int g = 0; g < G; ++g) {
            const float a = s.abuf[warp][g];
            const float2 aa = make_float2(a, a);
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[g][c] = __fmul2_rn(acc[g][c], aa);
          }
        }
#pragma unroll
        for (int tt = 0; tt < 4; ++tt) {
          if (t0 + tt < ntok) {
            float2 v[4];
            unpack8(*reinterpret_cast<const uint4*>(vrow + tt * kRowBytes), v);
            const float* pt = &s.pbuf[warp][half][tt][0];
#pragma unroll
            for (int g = 0; g < G; ++g) {
              const float pg = pt[g];
              const float2 pp = make_float2(pg, pg);
#pragma unroll
              for (int c = 0; c < 4; ++c) acc[g][c] = __ffma2_rn(pp, v[c], acc[g][c]);
            }
          }
        }
        __syncwarp();
      }
      // Release the stage; its last user refills it with stage j + kStages.
      if (lane == 0) {
        __threadfence_block();
        if (atomicAdd(&s.released[stage], 1) == kConsumerWarps - 1) {
          s.released[stage] = 0;
          __threadfence_block();
          fence_proxy_async_shared();
          if (j + kStages < nstages && !*reinterpret_cast<volatile int*>(&s.abort_flag))
            issue_stage<G, kHeadMajor>(s, &map, pool, p.kv_heads, kvh, n, j + kStages);
        }
      }
    }
  }

  __syncthreads();
  if (s.abort_flag) {
    // Let the loads still in flight land (bounded) before the CTA exits.
    if (threadIdx.x == 0)
      for (int st = 0; st < kStages; ++st)
        if (s.stage_issues[st] > 0)
          mbar_wait_bounded(&s.full[st], (s.stage_issues[st] - 1) & 1, p.status);
    __syncthreads();
    return;
  }

  // ---- merge the 8 warps (log-sum-exp) ----
  float* accw = reinterpret_cast<float*>(s.tiles);    // [8][G][128]
  float* mw = accw + kConsumerWarps * G * kHeadDim;   // [8][G]
  float* lw = mw + kConsumerWarps * G;                // [8][G]
  {
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
      const int v = (l16 >> kPairShift) * VPL + i;
      if (lane == ((v % G) / VPL) << kPairShift && v / G == 0) {
        mw[warp * G + v % G] = m_run[i];
        lw[warp * G + v % G] = ls;
      }
    }
    if (half == 0) {
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float* dst = &accw[(warp * G + g) * kHeadDim + 8 * l16];
        *reinterpret_cast<float4*>(dst) = make_float4(acc[g][0].x, acc[g][0].y, acc[g][1].x, acc[g][1].y);
        *reinterpret_cast<float4*>(dst + 4) =
            make_float4(acc[g][2].x, acc[g][2].y, acc[g][3].x, acc[g][3].y);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float M = -INFINITY;
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, mw[w * G + g]);
    float L = 0.f;
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float f = (M == -INFINITY) ? 0.f : exp2f(mw[w * G + g] - M);
      s.wscale[w][g] = f;
      L += lw[w * G + g] * f;
    }
    s.cta_m[g] = M;
    s.cta_l[g] = L;
  }
  __syncthreads();

  const size_t out_base = ((size_t)sl * p.kv_heads * G + (size_t)kvh * G) * kHeadDim;
  if (nsplit == 1) {
    for (int idx = threadIdx.x; idx < G * kHeadDim; idx += kThreads) {
      const int g = idx / kHeadDim, d = idx % kHeadDim;
      float o = 0.f;
#pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) o += accw[(w * G + g) * kHeadDim + d] * s.wscale[w][g];
      const float L = s.cta_l[g];
      const float v = L > 0.f ? o / L : 0.f;
      if (p.out_fp16) reinterpret_cast<uint16_t*>(p.out)[out_base + idx] = f2h_rn(v);
      else reinterpret_cast<float*>(p.out)[out_base + idx] = v;
    }
    return;
  }

  float* part = p.partial + ((size_t)unit * p.max_splits + split) * G * kPartialStride;
  for (int idx = threadIdx.x; idx < G * kHeadDim; idx += kThreads) {
    const int g = idx / kHeadDim, d = idx % kHeadDim;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) o += accw[(w * G + g) * kHeadDim + d] * s.wscale[w][g];
    part[g * kPartialStride + 2 + d] = o;
    if (d == 0) {
      part[g * kPartialStride] = s.cta_m[g];
      part[g * kPartialStride + 1] = s.cta_l[g];
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s.last_flag = atomicAdd(&p.counters[unit], 1) == nsplit - 1;
  __syncthreads();
  if (!s.last_flag) return;
  __threadfence();
  const float* parts = p.partial + (size_t)unit * p.max_splits * G * kPartialStride;
  for (int idx = threadIdx.x; idx < G * kHeadDim; idx += kThreads) {
    const int g = idx / kHeadDim, d = idx % kHeadDim;
    float M = -INFINITY;
    for (int k = 0; k < nsplit; ++k) M = fmaxf(M, __ldcg(parts + (k * G + g) * kPartialStride));
    float L = 0.f, o = 0.f;
    if (M != -INFINITY) {
      for (int k = 0; k < nsplit; ++k) {
        const float* pk = parts + (k * G + g) * kPartialStride;
        const float f = exp2f(__ldcg(pk) - M);
        L += __ldcg(pk + 1) * f;
        o += __ldcg(pk + 2 + d) * f;
      }
    }
    const float v = L > 0.f ? o / L : 0.f;
    if (p.out_fp16) reinterpret_cast<uint16_t*>(p.out)[out_base + idx] = f2h_rn(v);
    else reinterpret_cast<float*>(p.out)[out_base + idx] = v;
  }
  if (threadIdx.x == 0) p.counters[unit] = 0;
}

template <int G, bool kHeadMajor>
sa_status launch_layout(const AttnParams& p, const CUtensorMap& map, cudaStream_t stream) {
  const size_t smem = sizeof(AttnSmem<G>);
  static int configured[kMaxDevices];
  const sa_status st =
      ensure_smem_limit((const void*)attention_kernel<G, kHeadMajor>, (int)smem, configured);
  if (st != SA_OK) return st;
  const dim3 grid(p.max_splits, p.num_sl * p.kv_heads);
  attention_kernel<G, kHeadMajor><<<grid, kThreads, smem, stream>>>(map, p);
  return cuda_status(cudaGetLastError(), "attention_kernel launch");
}

template <int G>
sa_status launch_g(const AttnParams& p, const CUtensorMap& map, cudaStream_t stream) {
  return p.head_major ? launch_layout<G, true>(p, map, stream)
                      : launch_layout<G, false>(p, map, stream);
}

}  // namespace

int attention_plan_splits(int units, int max_entries, int* split_entries) {
  // About four waves of two CTAs per SM on 148 SMs; even entry counts (a
  // stage holds two), 4..64 entries per CTA.
  const int target_ctas = 148 * 2 * 4;
  const int per_unit = std::max(1, (target_ctas + units - 1) / std::max(units, 1));
  int split = std::max(4, (max_entries + per_unit - 1) / per_unit);
  split = std::min(split, kMaxSplitEntries);
  const int nsplit = std::max(1, (max_entries + split - 1) / split);
  split = std::max(1, (max_entries + nsplit - 1) / nsplit);
  split = std::min(kMaxSplitEntries, (split + 1) & ~1);
  *split_entries = split;
  return std::max(1, (max_entries + split - 1) / split);
}

size_t attention_scratch_bytes(int units, int max_splits, int group) {
  return (size_t)units * max_splits * group * kPartialStride * sizeof(float);
}

sa_status launch_attention(const AttnParams& p, const CUtensorMap& map, cudaStream_t stream) {
  if (p.num_sl <= 0 || p.kv_heads <= 0) return SA_OK;
  if ((size_t)p.num_sl * p.kv_heads > 65535u)
    return fail(SA_ERR_UNSUPPORTED, "attention: more than 65535 (sequence-layer, KV head) units");
  if (p.split_entries > kMaxSplitEntries)
    return fail(SA_ERR_UNSUPPORTED, "attention: split larger than 64 entries");
  switch (p.group) {
    case 1: return launch_g<1>(p, map, stream);
    case 2: return launch_g<2>(p, map, stream);
    case 4: return launch_g<4>(p, map, stream);
    case 8: return launch_g<8>(p, map, stream);
    default: return fail(SA_ERR_UNSUPPORTED, "attention: query heads per KV head must be 1, 2, 4 or 8");
  }
}

}  // namespace sa
