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
// A CTA takes `split_entries` consecutive entries of one unit.
//
// Data path per entry (one KV head of one 32-token block = 16 KB):
//   thread 0 issues four TMA tile loads (K lo/hi, V lo/hi: 32 rows x 128 B,
//   128 B swizzle) into a 4-stage ring guarded by mbarriers;
//   QK:  warp w owns head dims [16w, 16w+16), lane = token; q lives in
//        registers, K is read from swizzled smem conflict-free; packed
//        __ffma2_rn accumulates, partial logits go to smem;
//   softmax: warp w owns tokens [4w, 4w+4); it sums the 8 partials, keeps a
//        running max / sum per head (FP32, exp2 domain) -- an online softmax
//        per warp over its token subset;
//   PV:  lane owns dims [4 lane, 4 lane + 4) of the warp's tokens.
// At the end the 8 warp states are merged by log-sum-exp; with several
// splits per unit every CTA writes a partial (m, l, o[128]) and the last CTA
// to arrive (atomic counter, no spinning) merges them in split order, so
// results do not depend on CTA timing.
#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kStages = 4;
constexpr int kSubTile = kBlockTokens * 128;  // 32 rows x 128 B
constexpr int kTileBytes = 4 * kSubTile;     // K lo, K hi, V lo, V hi
constexpr int kPartialStride = 2 + kHeadDim; // m, l, o[128]
constexpr unsigned kFull = 0xffffffffu;

template <int G>
struct alignas(1024) AttnSmem {
  uint8_t tiles[kStages][kTileBytes];
  float plog[2][kWarps][kBlockTokens][G];
  float pw[kWarps][4][G];
  float aw[kWarps][G];
  float wscale[kWarps][G];
  uint64_t full[kStages];
  int ntok[kStages];
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
    int logical = p.sel_ids ? p.sel_ids[(sl * p.n_sel_groups + sgroup) * p.sel_stride + e] : e;
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

// One lane's G partial logits as the widest conflict-free stores.
template <int G>
__device__ __forceinline__ void store_partials(float* dst, const float (&v)[G]) {
  if constexpr (G == 1) {
    dst[0] = v[0];
  } else if constexpr (G == 2) {
    *reinterpret_cast<float2*>(dst) = make_float2(v[0], v[1]);
  } else {
#pragma unroll
    for (int g = 0; g < G; g += 4)
      *reinterpret_cast<float4*>(dst + g) = make_float4(v[g], v[g + 1], v[g + 2], v[g + 3]);
  }
}

template <int G>
__global__ void __launch_bounds__(kThreads, (G <= 4 ? 2 : 1))
    attention_kernel(const __grid_constant__ CUtensorMap map, const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  AttnSmem<G>& s = *reinterpret_cast<AttnSmem<G>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

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
  const int n = max(0, min(entries, e_begin + p.split_entries) - e_begin);

  int issued = 0;  // meaningful in thread 0 only
  auto issue = [&](int i) {
    const int stage = i % kStages;
    const Entry en = unit_entry(p, sl, sgroup, nsel, tail_len, e_begin + i);
    s.ntok[stage] = en.ntok;
    if (en.ntok > 0) {
      mbar_arrive_expect_tx(&s.full[stage], kTileBytes);
      const int x = kvh * kHeadDim;
      const int xv = p.kv_heads * kHeadDim + x;
      const int y = en.phys * kBlockTokens;
      uint8_t* dst = s.tiles[stage];
      tma_load_2d(dst, &map, &s.full[stage], x, y);
      tma_load_2d(dst + kSubTile, &map, &s.full[stage], x + 64, y);
      tma_load_2d(dst + 2 * kSubTile, &map, &s.full[stage], xv, y);
      tma_load_2d(dst + 3 * kSubTile, &map, &s.full[stage], xv + 64, y);
    } else {
      mbar_arrive(&s.full[stage]);
    }
    issued = i + 1;
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < kStages; ++i) mbar_init(&s.full[i], 1);
    s.abort_flag = 0;
    mbar_fence_init();
    tma_prefetch_desc(&map);
  }
  __syncthreads();
  if (threadIdx.x == 0)
    for (int i = 0; i < min(kStages, n); ++i) issue(i);

  // q slice for QK: dims [16 warp, 16 warp + 16) of the unit's G heads.
  const float* qbase = p.query + ((size_t)sl * p.kv_heads * G + (size_t)kvh * G) * kHeadDim;
  float2 q2[G][8];
#pragma unroll
  for (int g = 0; g < G; ++g) {
    const float4* src = reinterpret_cast<const float4*>(qbase + g * kHeadDim + 16 * warp);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 v = __ldg(src + i);
      q2[g][2 * i] = make_float2(v.x, v.y);
      q2[g][2 * i + 1] = make_float2(v.z, v.w);
    }
  }

  const int kd_half = warp >> 2;
  const int kd_chunk = (warp & 3) * 2;
  const int pv_half = lane >> 4;
  const int pv_chunk = (lane & 15) >> 1;
  const int pv_sub = (lane & 1) * 8;
  const int sm_t = lane / G;  // softmax pair (token index in warp, head)
  const int sm_g = lane % G;
  const bool sm_active = lane < 4 * G;

  float acc[G][4];
#pragma unroll
  for (int g = 0; g < G; ++g)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[g][c] = 0.f;
  float m_run = -INFINITY;
  float l_run = 0.f;
  int consumed = 0;

  for (int i = 0; i < n; ++i) {
    const int stage = i % kStages;
    if (!mbar_wait_bounded(&s.full[stage], (i / kStages) & 1, p.status)) s.abort_flag = 1;
    const uint8_t* tile = s.tiles[stage];
    const int ntok = s.ntok[stage];

    // ---- QK partial dot products (lane = token) ----
    {
      const uint8_t* row = tile + kd_half * kSubTile + lane * 128;
      const int sw = lane & 7;
      const uint4 c0 = *reinterpret_cast<const uint4*>(row + ((kd_chunk ^ sw) << 4));
      const uint4 c1 = *reinterpret_cast<const uint4*>(row + (((kd_chunk + 1) ^ sw) << 4));
      float2 k[8];
      k[0] = h2x2f(c0.x); k[1] = h2x2f(c0.y); k[2] = h2x2f(c0.z); k[3] = h2x2f(c0.w);
      k[4] = h2x2f(c1.x); k[5] = h2x2f(c1.y); k[6] = h2x2f(c1.z); k[7] = h2x2f(c1.w);
      float part[G];
#pragma unroll
      for (int g = 0; g < G; ++g) {
        float2 a = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 8; ++j) a = __ffma2_rn(q2[g][j], k[j], a);
        part[g] = a.x + a.y;
      }
      store_partials<G>(&s.plog[i & 1][warp][lane][0], part);
    }
    __syncthreads();
    if (s.abort_flag) break;
    consumed = i + 1;
    // Every warp is past its PV of entry i-1: its stage can be refilled.
    if (threadIdx.x == 0 && i >= 1 && i - 1 + kStages < n) issue(i - 1 + kStages);

    // ---- online softmax over this warp's 4 tokens ----
    float x = -INFINITY;
    if (sm_active) {
      const int t = 4 * warp + sm_t;
      if (t < ntok) {
        float sum = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) sum += s.plog[i & 1][w2][t][sm_g];
        x = sum * p.scale_log2;
      }
    }
    float bm = fmaxf(x, __shfl_xor_sync(kFull, x, G));
    bm = fmaxf(bm, __shfl_xor_sync(kFull, bm, 2 * G));
    const float m_new = fmaxf(m_run, bm);
    float alpha = 1.f, pr = 0.f;
    if (m_new != -INFINITY) {
      alpha = exp2f(m_run - m_new);
      pr = exp2f(x - m_new);
    }
    m_run = m_new;
    l_run = l_run * alpha + pr;
    if (sm_active) s.pw[warp][sm_t][sm_g] = pr;
    if (lane < G) s.aw[warp][lane] = alpha;
    __syncwarp();

    // ---- PV over the warp's tokens (lane = 4 dims) ----
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const float a = s.aw[warp][g];
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[g][c] *= a;
    }
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
      const int t = 4 * warp + tt;
      if (t < ntok) {
        const uint8_t* vrow = tile + (2 + pv_half) * kSubTile + t * 128;
        const uint2 v = *reinterpret_cast<const uint2*>(vrow + ((pv_chunk ^ (t & 7)) << 4) + pv_sub);
        const float2 v01 = h2x2f(v.x);
        const float2 v23 = h2x2f(v.y);
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const float pg = s.pw[warp][tt][g];
          const float2 pp = make_float2(pg, pg);
          const float2 a01 = __ffma2_rn(pp, v01, make_float2(acc[g][0], acc[g][1]));
          const float2 a23 = __ffma2_rn(pp, v23, make_float2(acc[g][2], acc[g][3]));
          acc[g][0] = a01.x; acc[g][1] = a01.y; acc[g][2] = a23.x; acc[g][3] = a23.y;
        }
      }
    }
    __syncwarp();
  }

  if (s.abort_flag) {
    // Drain the loads still in flight (bounded) before the CTA exits.
    if (threadIdx.x == 0)
      for (int k = consumed; k < issued; ++k)
        mbar_wait_bounded(&s.full[k % kStages], (k / kStages) & 1, p.status);
    __syncthreads();
    return;
  }

  // ---- merge the 8 warp states (log-sum-exp) ----
  __syncthreads();  // all tiles consumed: reuse them as the merge area
  float* accw = reinterpret_cast<float*>(s.tiles);   // [8][G][128]
  float* mw = accw + kWarps * G * kHeadDim;           // [8][G]
  float* lw = mw + kWarps * G;                        // [8][G]
  float lsum = l_run + __shfl_xor_sync(kFull, l_run, G);
  lsum += __shfl_xor_sync(kFull, lsum, 2 * G);
  if (lane < G) {
    mw[warp * G + lane] = m_run;
    lw[warp * G + lane] = lsum;
  }
#pragma unroll
  for (int g = 0; g < G; ++g)
    *reinterpret_cast<float4*>(&accw[(warp * G + g) * kHeadDim + 4 * lane]) =
        make_float4(acc[g][0], acc[g][1], acc[g][2], acc[g][3]);
  __syncthreads();
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float M = -INFINITY;
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, mw[w * G + g]);
    float L = 0.f;
    for (int w = 0; w < kWarps; ++w) {
      const float f = (M == -INFINITY) ? 0.f : exp2f(mw[w * G + g] - M);
      s.wscale[w][g] = f;
      L += lw[w * G + g] * f;
    }
    mw[g] = M;  // warp 0's slots are read below only through wscale/mw[g], lw[g]
    lw[g] = L;
  }
  __syncthreads();

  const size_t out_base = ((size_t)sl * p.kv_heads * G + (size_t)kvh * G) * kHeadDim;
  if (nsplit == 1) {
    for (int idx = threadIdx.x; idx < G * kHeadDim; idx += kThreads) {
      const int g = idx / kHeadDim, d = idx % kHeadDim;
      float o = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) o += accw[(w * G + g) * kHeadDim + d] * s.wscale[w][g];
      const float L = lw[g];
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
    for (int w = 0; w < kWarps; ++w) o += accw[(w * G + g) * kHeadDim + d] * s.wscale[w][g];
    part[g * kPartialStride + 2 + d] = o;
    if (d == 0) {
      part[g * kPartialStride] = mw[g];
      part[g * kPartialStride + 1] = lw[g];
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

template <int G>
sa_status launch_g(const AttnParams& p, const CUtensorMap& map, cudaStream_t stream) {
  const size_t smem = sizeof(AttnSmem<G>) + 1024;
  static int configured[kMaxDevices];
  const sa_status st = ensure_smem_limit((const void*)attention_kernel<G>, (int)smem, configured);
  if (st != SA_OK) return st;
  const dim3 grid(p.max_splits, p.num_sl * p.kv_heads);
  attention_kernel<G><<<grid, kThreads, smem, stream>>>(map, p);
  return cuda_status(cudaGetLastError(), "attention_kernel launch");
}

}  // namespace

int attention_plan_splits(int units, int max_entries, int* split_entries) {
  // About four waves of two CTAs per SM on 148 SMs, at least 4 entries each.
  const int target_ctas = 148 * 2 * 4;
  const int per_unit = std::max(1, (target_ctas + units - 1) / std::max(units, 1));
  int split = std::max(4, (max_entries + per_unit - 1) / per_unit);
  int nsplit = std::max(1, (max_entries + split - 1) / split);
  split = std::max(1, (max_entries + nsplit - 1) / nsplit);
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
  switch (p.group) {
    case 1: return launch_g<1>(p, map, stream);
    case 2: return launch_g<2>(p, map, stream);
    case 4: return launch_g<4>(p, map, stream);
    case 8: return launch_g<8>(p, map, stream);
    default: return fail(SA_ERR_UNSUPPORTED, "attention: query heads per KV head must be 1, 2, 4 or 8");
  }
}

}  // namespace sa
