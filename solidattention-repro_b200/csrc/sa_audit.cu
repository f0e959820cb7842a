// sa_audit.cu -- dense attention mass per block: the quality audit of the
// selection.
//
// Replaces the reference's dense audits, audit_dense_selection
// (cpp/src/pipeline_main.cpp:502-574: per-block mass of the dense softmax,
// averaged over query heads, then the selected mass and the recall of the
// mass-ranked oracle set) and the selected-vs-dense comparison of
// cpp/src/selection_main.cpp:246-252. Selection here is per KV head, so the
// audit is per (sequence-layer, KV head) and averages over that KV head's G
// query heads; the open tail is part of the dense token set (it is always
// attended) and its mass is reported as one extra entry.
//
// Not on the timed path: one CTA per unit makes three passes over the unit's
// K rows (per-head maximum, denominator, per-block mass), recomputing the
// logits each time instead of storing them. A warp takes one 32-token block
// at a time, one token per lane.
#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kAuditThreads = 256;
constexpr int kAuditWarps = kAuditThreads / 32;
constexpr int kMaxAuditGroup = 32;
constexpr unsigned kFull = 0xffffffffu;

struct AuditParams {
  CtxDev c;
  const float* query;  // [num_sl][qh][128]
  float* mass;         // [num_sl][kv_heads][table_blocks + 1]
  float scale_log2;
};

// Logits (log2 domain) of the lane's token for the G heads of KV head kvh.
__device__ __forceinline__ void token_logits(const uint16_t* krow, const float* qs, int group,
                                             float scale_log2, float* out) {
  for (int g = 0; g < group; ++g) out[g] = 0.f;
  for (int d = 0; d < kHeadDim; d += 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(krow + d);
    const float2 k0 = h2x2f(u.x), k1 = h2x2f(u.y), k2 = h2x2f(u.z), k3 = h2x2f(u.w);
    for (int g = 0; g < group; ++g) {
      const float* q = qs + g * kHeadDim + d;
      float a = out[g];
      a = fmaf(q[0], k0.x, a);
      a = fmaf(q[1], k0.y, a);
      a = fmaf(q[2], k1.x, a);
      a = fmaf(q[3], k1.y, a);
      a = fmaf(q[4], k2.x, a);
      a = fmaf(q[5], k2.y, a);
      a = fmaf(q[6], k3.x, a);
      a = fmaf(q[7], k3.y, a);
      out[g] = a;
    }
  }
  for (int g = 0; g < group; ++g) out[g] *= scale_log2;
}

__global__ void __launch_bounds__(kAuditThreads) audit_kernel(const AuditParams p) {
  __shared__ float qs[kMaxAuditGroup * kHeadDim];
  __shared__ float red[kAuditWarps][kMaxAuditGroup];
  __shared__ float stat[kMaxAuditGroup];  // per head: maximum, then 1 / denominator
  const CtxDev& c = p.c;
  const int group = c.qh / c.kv_heads;
  const int unit = blockIdx.x;
  const int sl = unit / c.kv_heads;
  const int kvh = unit - sl * c.kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = max(0, min(c.num_sealed[sl], c.table_blocks));
  const int tl = max(0, min(c.tail_len[sl], kBlockTokens));
  const int nblk = nb + (tl > 0 ? 1 : 0);
  float* mass = p.mass + (size_t)unit * (c.table_blocks + 1);
  for (int i = threadIdx.x; i < group * kHeadDim; i += kAuditThreads)
    qs[i] = p.query[((size_t)sl * c.qh + (size_t)kvh * group) * kHeadDim + i];
  for (int i = threadIdx.x; i <= c.table_blocks; i += kAuditThreads) mass[i] = 0.f;
  __syncthreads();

  // K row of token `lane` of dense block b (the tail is block nb)
  auto krow = [&](int b) -> const uint16_t* {
    const int phys = b < nb ? c.table[(size_t)sl * c.table_blocks + b] : c.tail_block[sl];
    if (phys < 0 || phys >= c.pool_blocks) return nullptr;
    return c.pool + ((((size_t)phys * c.kv_heads + kvh) * 2) * kBlockTokens + lane) * kHeadDim;
  };
  float l[kMaxAuditGroup];
  for (int pass = 0; pass < 3; ++pass) {
    float acc[kMaxAuditGroup];
    for (int g = 0; g < group; ++g) acc[g] = pass == 0 ? -INFINITY : 0.f;
    for (int b = warp; b < nblk; b += kAuditWarps) {
      const uint16_t* row = krow(b);
      const bool valid = row != nullptr && (b < nb || lane < tl);
      if (row == nullptr && lane == 0) raise_status(c.status, SA_DEV_BAD_BLOCK);
      if (valid) token_logits(row, qs, group, p.scale_log2, l);
      if (pass == 0) {
        for (int g = 0; g < group; ++g) acc[g] = fmaxf(acc[g], valid ? l[g] : -INFINITY);
      } else {
        float bm = 0.f;  // pass 2: this block's share of the heads' normalised mass
        for (int g = 0; g < group; ++g) {
          const float e = valid ? exp2f(l[g] - stat[g]) : 0.f;
          if (pass == 1) acc[g] += e;
          else bm += e * stat[kMaxAuditGroup / 2 + g];
        }
        if (pass == 2) {
          for (int off = 16; off >= 1; off >>= 1) bm += __shfl_xor_sync(kFull, bm, off);
          if (lane == 0) mass[b < nb ? b : c.table_blocks] = bm / group;
        }
      }
    }
    if (pass == 2) break;
    for (int g = 0; g < group; ++g) {
      float v = acc[g];
      for (int off = 16; off >= 1; off >>= 1) {
        const float o = __shfl_xor_sync(kFull, v, off);
        v = pass == 0 ? fmaxf(v, o) : v + o;
      }
      if (lane == 0) red[warp][g] = v;
    }
    __syncthreads();
    if (threadIdx.x < group) {
      const int g = threadIdx.x;
      float v = pass == 0 ? -INFINITY : 0.f;
      for (int w = 0; w < kAuditWarps; ++w) v = pass == 0 ? fmaxf(v, red[w][g]) : v + red[w][g];
      if (pass == 0) stat[g] = v;
      else stat[kMaxAuditGroup / 2 + g] = v > 0.f ? 1.f / v : 0.f;
    }
    __syncthreads();
  }
}

}  // namespace

sa_status launch_audit(const CtxDev& c, const float* query, float* mass, float scale,
                       cudaStream_t stream) {
  const int group = c.qh / c.kv_heads;
  if (group > kMaxAuditGroup / 2)
    return fail(SA_ERR_UNSUPPORTED, "audit: more than 16 query heads per KV head");
  AuditParams p{};
  p.c = c;
  p.query = query;
  p.mass = mass;
  p.scale_log2 = scale * 1.4426950408889634f;
  const int units = c.num_sl * c.kv_heads;
  if (units <= 0) return SA_OK;
  audit_kernel<<<units, kAuditThreads, 0, stream>>>(p);
  return cuda_status(cudaGetLastError(), "audit_kernel launch");
}

}  // namespace sa
