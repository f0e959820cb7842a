// sa_lifecycle.cu -- KV block lifecycle kernels for sm_100a: representative
// rebuild, decode-tail append, seal into the paged pool, FP16 pack, and the
// two small helper kernels of the backend handle.
//
// Representative rebuild restates build_local_causal_representatives
// (cpp/src/selection.cpp:12-94): for query head h and query position p the
// softmax over the causal window [p-W+1, p] gives every window key a received
// probability; a key's mass is the sum of what it receives, in query order;
// the block's representative is the mean (in rank order, FP32) of its top-k
// keys by mass (stable: ties go to the lower offset). Every dot product,
// maximum, sum and division keeps the reference's order and rounding, so the
// only difference from the CPU is the last bit of expf.
//
// The seal follows the lifecycle of cpp/src/kv_lifecycle_main.cpp:92-113 and
// cpp/src/online_seal_main.cpp:41-46: when a tail holds 32 tokens it becomes
// the next sealed block. Here the tail already lives in a pool block, so the
// seal moves no KV bytes: it rebuilds the representative from the tail's 32
// queries, appends the block to the table, takes a fresh tail block from the
// free list and bumps the generation.
#include <algorithm>

#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kRepThreads = 256;
constexpr int kRepWarps = kRepThreads / 32;
constexpr int kRepMaxWindow = 64;
constexpr int kRepMaxDim = 128;
constexpr int kRepKeyLd = 162;  // >= 32 + 2*(64-1) keys; 81 words per row, odd -> conflict-free
constexpr int kRepMaxQueries = kBlockTokens + kRepMaxWindow - 1;      // 95
constexpr unsigned kFull = 0xffffffffu;

struct RepSmem {
  uint16_t kT[kRepMaxDim][kRepKeyLd];           // keys, transposed [dim][key]
  float qbuf[kRepWarps][kRepMaxDim];            // one query row per warp
  float contrib[kRepMaxQueries][kBlockTokens];  // probability query -> block key
  float qall[kBlockTokens][kRepMaxDim];         // every query row (one-warp calls)
  int order[kBlockTokens];
};

struct RepCall {
  const float* q;        // query of position pos at q + pos * d
  int tokens;            // T of the call
  int block;             // block within the call
  const uint16_t* kv;
  int head_major;        // kv is a head-major pool [block][kv_heads][K,V][32][d]
  int kv_heads;
  int64_t row_stride;
  int kv_head;
  int d;
  const int32_t* table;  // null -> row = row_base + token
  int table_base;
  int64_t row_base;
  int64_t pool_rows;     // rows addressable (bounds check), <= 0: unchecked
  int window, topk;
  float scale;
  float* out_values;     // dim j at out_values[j * o_dim]
  int64_t o_dim;
  int32_t* out_offsets;  // topk ids, nullable
  uint32_t* status;
};

__device__ __forceinline__ const uint16_t* key_row(const RepCall& c, int token) {
  int64_t row;
  if (c.table) {
    const int blk = c.table[c.table_base + token / kBlockTokens];
    row = (int64_t)blk * kBlockTokens + token % kBlockTokens;
  } else {
    row = c.row_base + token;
  }
  if (row < 0 || (c.pool_rows > 0 && row >= c.pool_rows)) return nullptr;
  if (c.head_major) {
    const int64_t blk = row / kBlockTokens;
    return c.kv + ((blk * c.kv_heads + c.kv_head) * 2 * kBlockTokens + row % kBlockTokens) * c.d;
  }
  return c.kv + row * c.row_stride + (int64_t)c.kv_head * c.d;
}

// One (head, block) of the representative build; whole CTA participates.
__device__ void rep_block(const RepCall& c, RepSmem& s) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int W = c.window, T = c.tokens, D = c.d;
  const int blk0 = c.block * kBlockTokens;
  const int p_lo = blk0;
  const int p_hi = min(T, blk0 + kBlockTokens + W - 1);
  const int nq = p_hi - p_lo;
  const int k_lo = max(0, p_lo - W + 1);
  const int nk = p_hi - k_lo;

  // One-warp calls: every key of the call fits the 32 lanes of a warp (the
  // seal of a block and per-block builds, window <= 32), and rows can be
  // read 16 bytes at a time. A warp then scores four queries at once, lane =
  // key, instead of one query per pass.
  const bool one_warp = nk <= 32 && D == kRepMaxDim &&
                        (reinterpret_cast<uintptr_t>(c.kv) & 15u) == 0 &&
                        (c.head_major || c.row_stride % 8 == 0) &&
                        (reinterpret_cast<uintptr_t>(c.q) & 15u) == 0;
  bool bad = false;
  if (one_warp) {
    constexpr int kChunks8 = kRepMaxDim / 8;
#pragma unroll 2
    for (int idx = tid; idx < nk * kChunks8; idx += kRepThreads) {
      const int r = idx / kChunks8, c8 = idx - r * kChunks8;
      const uint16_t* row = key_row(c, k_lo + r);
      bad |= row == nullptr;
      uint4 u = make_uint4(0u, 0u, 0u, 0u);
      if (row) u = *reinterpret_cast<const uint4*>(row + c8 * 8);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s.kT[c8 * 8 + 2 * j][r] = (uint16_t)(w[j] & 0xffffu);
        s.kT[c8 * 8 + 2 * j + 1][r] = (uint16_t)(w[j] >> 16);
      }
    }
    constexpr int kChunks4 = kRepMaxDim / 4;
#pragma unroll 4
    for (int idx = tid; idx < nq * kChunks4; idx += kRepThreads) {
      const int qi = idx / kChunks4, c4 = idx - qi * kChunks4;
      *reinterpret_cast<float4*>(&s.qall[qi][c4 * 4]) =
          *reinterpret_cast<const float4*>(c.q + (int64_t)(p_lo + qi) * D + c4 * 4);
    }
  } else {
    for (int idx = tid; idx < nk * D; idx += kRepThreads) {
      const int r = idx / D, dim = idx - r * D;
      const uint16_t* row = key_row(c, k_lo + r);
      bad |= row == nullptr;
      s.kT[dim][r] = row ? row[dim] : (uint16_t)0;
    }
  }
  if (bad) raise_status(c.status, SA_DEV_BAD_BLOCK);
  for (int idx = tid; idx < nq * kBlockTokens; idx += kRepThreads)
    s.contrib[idx / kBlockTokens][idx % kBlockTokens] = 0.f;
  __syncthreads();

  if (one_warp) {
    // lane = key k_lo + lane; a warp takes queries q0 + j * kRepWarps, j < 4.
    // Each dot keeps the reference's order (sequential over dims, multiply
    // and add rounded separately); lanes outside a query's window compute a
    // dot that is discarded, and their zero terms leave the ordered
    // denominator unchanged.
    const int key = k_lo + lane;
    for (int q0 = warp; q0 < nq; q0 += 4 * kRepWarps) {
      const float* qr[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) qr[j] = s.qall[min(q0 + j * kRepWarps, nq - 1)];
      float dot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int dim = 0; dim < kRepMaxDim; dim += 4) {
        float kf[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) kf[u] = h2f(s.kT[dim + u][lane]);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 qv = *reinterpret_cast<const float4*>(qr[j] + dim);
          dot[j] = __fadd_rn(dot[j], __fmul_rn(qv.x, kf[0]));
          dot[j] = __fadd_rn(dot[j], __fmul_rn(qv.y, kf[1]));
          dot[j] = __fadd_rn(dot[j], __fmul_rn(qv.z, kf[2]));
          dot[j] = __fadd_rn(dot[j], __fmul_rn(qv.w, kf[3]));
        }
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int qi = q0 + j * kRepWarps;
        if (qi >= nq) break;
        const int pos = p_lo + qi;
        const bool valid = lane < nk && key >= max(0, pos - W + 1) && key <= pos;
        const float lg = valid ? __fmul_rn(dot[j], c.scale) : -INFINITY;
        float maxv = lg;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) maxv = fmaxf(maxv, __shfl_xor_sync(kFull, maxv, o));
        const float e = valid ? expf(__fsub_rn(lg, maxv)) : 0.f;
        float den = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) den = __fadd_rn(den, __shfl_sync(kFull, e, i));
        if (valid && key >= blk0 && key < blk0 + kBlockTokens)
          s.contrib[qi][key - blk0] = __fdiv_rn(e, den);
      }
    }
  }
  for (int qi = one_warp ? nq : warp; qi < nq; qi += kRepWarps) {
    const int pos = p_lo + qi;
    const float* qrow = c.q + (int64_t)pos * D;
    for (int dim = lane; dim < D; dim += 32) s.qbuf[warp][dim] = qrow[dim];
    __syncwarp();
    const int start = max(0, pos - W + 1);
    const int count = pos - start + 1;
    float lg[2] = {-INFINITY, -INFINITY};
    float maxv = -INFINITY;
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const int w = ch * 32 + lane;
      if (w < count) {
        const int key = start + w - k_lo;
        float dot = 0.f;
        for (int dim = 0; dim < D; ++dim)
          dot = __fadd_rn(dot, __fmul_rn(s.qbuf[warp][dim], h2f(s.kT[dim][key])));
        lg[ch] = __fmul_rn(dot, c.scale);
      }
      maxv = fmaxf(maxv, lg[ch]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) maxv = fmaxf(maxv, __shfl_xor_sync(kFull, maxv, o));
    float e[2];
#pragma unroll
    for (int ch = 0; ch < 2; ++ch)
      e[ch] = (ch * 32 + lane < count) ? expf(__fsub_rn(lg[ch], maxv)) : 0.f;
    // Denominator in window order, as the reference sums it.
    float den = 0.f;
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      if (ch * 32 >= count) break;
      const int lim = min(32, count - ch * 32);
      for (int i = 0; i < lim; ++i) den = __fadd_rn(den, __shfl_sync(kFull, e[ch], i));
    }
#pragma unroll
    for (int ch = 0; ch < 2; ++ch) {
      const int w = ch * 32 + lane;
      if (w < count) {
        const int key = start + w;
        if (key >= blk0 && key < blk0 + kBlockTokens)
          s.contrib[qi][key - blk0] = __fdiv_rn(e[ch], den);
      }
    }
    __syncwarp();
  }
  __syncthreads();

  if (warp == 0) {
    float r = 0.f;
    for (int qi = 0; qi < nq; ++qi) r = __fadd_rn(r, s.contrib[qi][lane]);
    int rank = 0;
    for (int j = 0; j < 32; ++j) {
      const float rj = __shfl_sync(kFull, r, j);
      rank += (rj > r) || (rj == r && j < lane);
    }
    if (rank < c.topk) s.order[rank] = lane;
  }
  __syncthreads();
  const float divisor = (float)c.topk;
  for (int dim = tid; dim < D; dim += kRepThreads) {
    float v = 0.f;
    for (int rk = 0; rk < c.topk; ++rk) v = __fadd_rn(v, h2f(s.kT[dim][blk0 + s.order[rk] - k_lo]));
    c.out_values[(int64_t)dim * c.o_dim] = __fdiv_rn(v, divisor);
  }
  if (c.out_offsets && tid < c.topk) c.out_offsets[tid] = s.order[tid];
  __syncthreads();
}

__device__ __forceinline__ RepSmem& rep_smem() {
  extern __shared__ __align__(16) uint8_t rep_raw[];
  return *reinterpret_cast<RepSmem*>(rep_raw);
}

// grid (qh, blocks): a call over `tokens` tokens; block b of it.
__global__ void __launch_bounds__(kRepThreads) reps_kernel(const RepParams p, int per_block) {
  const int h = blockIdx.x, b = blockIdx.y;
  const int group = p.qh / p.kv_heads;
  RepCall c;
  const int call_tokens = per_block ? kBlockTokens : p.tokens;
  const int64_t q_head_stride = (int64_t)p.tokens * p.d;  // [qh][tokens][d]
  c.q = p.q + h * q_head_stride + (per_block ? (int64_t)b * kBlockTokens * p.d : 0);
  c.tokens = call_tokens;
  c.block = per_block ? 0 : b;
  c.kv = p.kv;
  c.head_major = p.head_major;
  c.kv_heads = p.kv_heads;
  c.row_stride = p.row_stride;
  c.kv_head = h / group;
  c.d = p.d;
  c.table = p.table;
  c.table_base = p.table_offset + (per_block ? b : 0);
  c.row_base = per_block ? (int64_t)b * kBlockTokens : 0;
  c.pool_rows = 0;
  c.window = p.window;
  c.topk = p.topk;
  c.scale = p.scale;
  c.out_values = p.values + h * p.o_head + b * p.o_block;
  c.o_dim = p.o_dim;
  c.out_offsets = p.offsets ? p.offsets + ((int64_t)h * p.blocks + b) * p.topk : nullptr;
  c.status = p.status;
  rep_block(c, rep_smem());
}

// Tail length of sequence-layer sl once the step's pending tokens count (a
// tail that was already full received no append).
__device__ __forceinline__ int effective_tail(const CtxDev& c, int sl, int pending) {
  const int tl = c.tail_len[sl];
  return tl < kBlockTokens ? tl + pending : tl;
}

// Rebuild the representative of query head h of sequence-layer sl if its
// tail is full.
__device__ void seal_rebuild(const CtxDev& c, int h, int sl, int pending) {
  if (effective_tail(c, sl, pending) < kBlockTokens || c.num_sealed[sl] >= c.table_blocks) return;
  const int nb = c.num_sealed[sl];
  const int phys = c.tail_block[sl];
  if (phys < 0 || phys >= c.pool_blocks) return;
  RepCall r;
  r.q = c.query_ring + ((int64_t)sl * c.qh + h) * kBlockTokens * kHeadDim;
  r.tokens = kBlockTokens;
  r.block = 0;
  r.kv = c.pool;
  r.head_major = 1;
  r.kv_heads = c.kv_heads;
  r.row_stride = c.row_elems;
  r.kv_head = h / (c.qh / c.kv_heads);
  r.d = kHeadDim;
  r.table = nullptr;
  r.table_base = 0;
  r.row_base = (int64_t)phys * kBlockTokens;
  r.pool_rows = (int64_t)c.pool_blocks * kBlockTokens;
  r.window = c.rep_window;
  r.topk = c.rep_topk;
  r.scale = c.rep_scale;
  r.out_values = c.reps + ((int64_t)sl * c.qh + h) * kHeadDim * c.reps_cap + nb;
  r.o_dim = c.reps_cap;
  r.out_offsets = nullptr;
  r.status = c.status;
  rep_block(r, rep_smem());
}

// One CTA: commit every full tail in (sequence-layer) order, so the physical
// block each new tail receives is deterministic; with pending tokens, store
// every other tail's new length.
__device__ void seal_commit(const CtxDev& c, int pending) {
  __shared__ int scan[33];
  __shared__ int base_top;
  if (threadIdx.x == 0) base_top = *c.free_top;
  __syncthreads();
  int taken_before = 0;
  for (int sl0 = 0; sl0 < c.num_sl; sl0 += blockDim.x) {
    const int sl = sl0 + threadIdx.x;
    int want = 0;
    int len = 0;
    if (sl < c.num_sl) {
      len = effective_tail(c, sl, pending);
      if (len >= kBlockTokens) {
        if (c.num_sealed[sl] >= c.table_blocks) raise_status(c.status, SA_DEV_TABLE_FULL);
        else if (c.tail_block[sl] < 0 || c.tail_block[sl] >= c.pool_blocks)
          raise_status(c.status, SA_DEV_BAD_BLOCK);
        else want = 1;
      }
    }
    int total = 0;
    const int rank = taken_before + block_exclusive_scan(want, scan, &total);
    if (want) {
      const int top = base_top - 1 - rank;
      if (top < 0) {
        raise_status(c.status, SA_DEV_POOL_EMPTY);
        want = 0;
      } else {
        const int nb = c.num_sealed[sl];
        c.table[(int64_t)sl * c.table_blocks + nb] = c.tail_block[sl];
        c.num_sealed[sl] = nb + 1;
        c.tail_block[sl] = c.free_list[top];
        c.tail_len[sl] = 0;
        c.generation[sl] += 1;
      }
    }
    if (!want && pending && sl < c.num_sl) c.tail_len[sl] = len;
    taken_before += total;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    *c.free_top = max(0, base_top - taken_before);
    if (c.status_mirror) {
      // every kernel of the step has finished writing status bits by now
      __threadfence();
      *reinterpret_cast<volatile uint32_t*>(c.status_mirror) =
          *reinterpret_cast<volatile uint32_t*>(c.status);
      __threadfence_system();
    }
  }
}

// Grid-stride over (query head, sequence-layer) items: rebuild the
// representative of every full tail; the last CTA to finish commits the
// seals (an atomic arrival count, reset by that CTA; no spinning).
// Three CTAs per SM (74 KB of shared memory each, <= 85 registers): a full
// seal of every head of every layer spreads over 444 CTAs.
__global__ void __launch_bounds__(kRepThreads, 3) seal_kernel(const CtxDev c, int pending) {
  __shared__ int last;
  pdl_launch_dependents();
  pdl_wait();  // the attention of this step still reads the tails
  // A gathered step also signals and waits here for every rank's outputs
  // (CTA 0, before the commit and the status mirror, which its barriers
  // order after it).
  if (c.gather_counter && blockIdx.x == 0 && threadIdx.x == 0)
    gather_signal_wait(c.gather_peers, c.gather_world, c.gather_counter_bytes, c.gather_counter,
                       c.gather_epoch, (unsigned long long)c.gather_world, true, c.status);
  if (pending && __ldcg(c.seal_counters + 1) == 0) {
    // The step's appends filled no tail (the fused append flags one that it
    // fills or finds full): only the tail lengths move, by one CTA.
    if (blockIdx.x == 0) seal_commit(c, pending);
    return;
  }
  const int items = c.qh * c.num_sl;
  // Most steps fill no tail: test all of this CTA's items in one round of
  // loads (one item per thread) before walking them one at a time.
  int full = 0;
  for (int i = blockIdx.x + (int)threadIdx.x * (int)gridDim.x; i < items;
       i += (int)(blockDim.x * gridDim.x))
    full |= effective_tail(c, i / c.qh, pending) >= kBlockTokens;
  if (__syncthreads_or(full)) {
    for (int i = blockIdx.x; i < items; i += gridDim.x) {
      seal_rebuild(c, i % c.qh, i / c.qh, pending);
      __syncthreads();  // the next item reuses the shared buffers
    }
  }
  if (threadIdx.x == 0) {
    // the barrier orders the CTA's representative stores before this fence
    __threadfence();
    last = atomicAdd(c.seal_counters, 1) == (int)gridDim.x - 1;
    if (last) {
      __threadfence();
      c.seal_counters[0] = 0;
      c.seal_counters[1] = 0;  // every CTA has read the flag
    }
  }
  __syncthreads();
  if (last) seal_commit(c, pending);
}

// grid num_sl: write the current token's K/V into its tail row (one row of
// each KV head's K and V planes of the head-major tail block) and its query
// into the tail's query ring.
__global__ void __launch_bounds__(256)
    append_kernel(const CtxDev c, const float* query, const void* kv_new, int kv_fp32) {
  const int sl = blockIdx.x;
  const int tl = c.tail_len[sl];
  if (!append_token(c, sl, query, kv_new, kv_fp32, 0, c.kv_heads, 0, c.qh, threadIdx.x,
                    blockDim.x))
    return;
  __syncthreads();
  if (threadIdx.x == 0) c.tail_len[sl] = tl + 1;
}

__global__ void pack_kv_kernel(uint16_t* packed, const float* key, const float* value,
                               size_t token, size_t elements) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= elements) return;
  uint16_t* row = packed + token * 2 * elements;
  row[i] = f2h_rn(key[i]);
  row[elements + i] = f2h_rn(value[i]);
}

__global__ void xor_kernel(const uint8_t* in, uint8_t* out, size_t bytes, uint8_t mask) {
  const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < bytes) out[i] = in[i] ^ mask;
}

// checksum = sum(out[i] * (1 + (i % 17) * 1e-3)), the C1.4 consumer
// (cpp/src/cuda_backend.cpp:160-168), as one block-wide reduction.
__global__ void consume_kernel(const float* out, int n, float* checksum) {
  __shared__ float part[32];
  float acc = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x)
    acc += out[i] * (1.0f + (float)(i % 17) * 0.001f);
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(kFull, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(kFull, v, o);
    if (threadIdx.x == 0) *checksum = v;
  }
}

int g_reps_smem[kMaxDevices];
int g_seal_smem[kMaxDevices];

sa_status check_rep_params(int d, int window, int topk) {
  if (d <= 0 || d > kRepMaxDim) return fail(SA_ERR_UNSUPPORTED, "representatives: head_dim must be 1..128");
  if (window <= 0 || window > kRepMaxWindow)
    return fail(SA_ERR_UNSUPPORTED, "representatives: local_window must be 1..64");
  if (topk <= 0 || topk > kBlockTokens) return fail(SA_ERR_INVALID_ARG, "representatives: topk must be 1..32");
  return SA_OK;
}

}  // namespace

sa_status launch_build_reps(const RepParams& p, cudaStream_t stream) {
  sa_status st = check_rep_params(p.d, p.window, p.topk);
  if (st != SA_OK) return st;
  if ((st = ensure_smem_limit((const void*)reps_kernel, (int)sizeof(RepSmem), g_reps_smem)) != SA_OK)
    return st;
  if (p.blocks <= 0) return SA_OK;
  if (p.blocks > 65535) return fail(SA_ERR_UNSUPPORTED, "representatives: more than 65535 blocks");
  reps_kernel<<<dim3(p.qh, p.blocks), kRepThreads, sizeof(RepSmem), stream>>>(p, 0);
  return cuda_status(cudaGetLastError(), "reps_kernel launch");
}

sa_status launch_build_reps_per_block(const RepParams& p, cudaStream_t stream) {
  sa_status st = check_rep_params(p.d, p.window, p.topk);
  if (st != SA_OK) return st;
  if ((st = ensure_smem_limit((const void*)reps_kernel, (int)sizeof(RepSmem), g_reps_smem)) != SA_OK)
    return st;
  if (p.blocks <= 0) return SA_OK;
  if (p.blocks > 65535) return fail(SA_ERR_UNSUPPORTED, "representatives: more than 65535 blocks");
  reps_kernel<<<dim3(p.qh, p.blocks), kRepThreads, sizeof(RepSmem), stream>>>(p, 1);
  return cuda_status(cudaGetLastError(), "reps_kernel launch");
}

sa_status launch_append(const CtxDev& c, const float* query, const void* kv_new, int kv_fp32,
                        cudaStream_t stream) {
  append_kernel<<<c.num_sl, 256, 0, stream>>>(c, query, kv_new, kv_fp32);
  return cuda_status(cudaGetLastError(), "append_kernel launch");
}

sa_status launch_seal(const CtxDev& c, int pending, cudaStream_t stream, bool pdl) {
  sa_status st = check_rep_params(kHeadDim, c.rep_window, c.rep_topk);
  if (st != SA_OK) return st;
  if ((st = ensure_smem_limit((const void*)seal_kernel, (int)sizeof(RepSmem), g_seal_smem)) != SA_OK)
    return st;
  // three CTAs per SM at most; a step that fills no tail runs CTA 0 alone
  const int items = c.qh * c.num_sl;
  const int grid = std::max(1, std::min(items, 3 * device_sm_count()));
  return cuda_status(launch_kernel(seal_kernel, dim3(grid), dim3(kRepThreads), sizeof(RepSmem),
                                   stream, pdl, c, pending),
                     "seal_kernel launch");
}

sa_status launch_pack_kv(uint16_t* packed, const float* key, const float* value, size_t token,
                         size_t elements, cudaStream_t stream) {
  if (elements == 0) return SA_OK;
  pack_kv_kernel<<<(unsigned)((elements + 255) / 256), 256, 0, stream>>>(packed, key, value, token,
                                                                        elements);
  return cuda_status(cudaGetLastError(), "pack_kv_kernel launch");
}

sa_status launch_xor(const uint8_t* in, uint8_t* out, size_t bytes, uint8_t mask,
                     cudaStream_t stream) {
  if (bytes == 0) return SA_OK;
  xor_kernel<<<(unsigned)((bytes + 255) / 256), 256, 0, stream>>>(in, out, bytes, mask);
  return cuda_status(cudaGetLastError(), "xor_kernel launch");
}

sa_status launch_consume(const float* out, int n, float* checksum, cudaStream_t stream) {
  consume_kernel<<<1, 1024, 0, stream>>>(out, n, checksum);
  return cuda_status(cudaGetLastError(), "consume_kernel launch");
}

}  // namespace sa

namespace sa {

namespace {

// grid (count, kv_heads): one (block, KV head) = 16 KB per CTA. Token-major
// store rows [32][2][KH][128] <-> the head-major pool's [KH][2][32][128].
template <bool kImport>
__global__ void __launch_bounds__(256)
    store_blocks_kernel(const CtxDev c, int sl, int first, uint16_t* store) {
  const int b = blockIdx.x, h = blockIdx.y;
  const int logical = first + b;
  if (logical < 0 || logical >= c.table_blocks) {
    if (threadIdx.x == 0) raise_status(c.status, SA_DEV_BAD_BLOCK);
    return;
  }
  const int phys = c.table[(int64_t)sl * c.table_blocks + logical];
  if (phys < 0 || phys >= c.pool_blocks) {
    if (threadIdx.x == 0) raise_status(c.status, SA_DEV_BAD_BLOCK);
    return;
  }
  uint16_t* pool = c.pool + ((int64_t)phys * c.kv_heads + h) * 2 * kBlockTokens * kHeadDim;
  uint16_t* rows = store + (int64_t)b * kBlockTokens * c.row_elems;
  constexpr int kChunks = 2 * kBlockTokens * kHeadDim / 8;  // 16-byte chunks of the (block, head)
  for (int i = threadIdx.x; i < kChunks; i += blockDim.x) {
    const int kv = i / (kBlockTokens * kHeadDim / 8);
    const int t = (i / (kHeadDim / 8)) % kBlockTokens;
    const int d = (i % (kHeadDim / 8)) * 8;
    uint4* p = reinterpret_cast<uint4*>(pool + ((int64_t)kv * kBlockTokens + t) * kHeadDim + d);
    uint4* r = reinterpret_cast<uint4*>(rows + ((int64_t)t * 2 + kv) * c.kv_heads * kHeadDim +
                                        (int64_t)h * kHeadDim + d);
    if (kImport) *p = *r;
    else *r = *p;
  }
}

}  // namespace

sa_status launch_store_blocks(const CtxDev& c, int sl, int first, int count, void* store,
                              bool import, cudaStream_t stream) {
  if (count <= 0) return SA_OK;
  if (count > 65535) return fail(SA_ERR_UNSUPPORTED, "blocks: more than 65535 blocks per call");
  const dim3 grid(count, c.kv_heads);
  if (import)
    store_blocks_kernel<true><<<grid, 256, 0, stream>>>(c, sl, first, static_cast<uint16_t*>(store));
  else
    store_blocks_kernel<false><<<grid, 256, 0, stream>>>(c, sl, first, static_cast<uint16_t*>(store));
  return cuda_status(cudaGetLastError(), "store_blocks_kernel launch");
}

}  // namespace sa
