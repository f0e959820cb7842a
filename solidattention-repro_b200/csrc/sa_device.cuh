// sa_device.cuh -- device-side helpers shared by the sm_100a kernels:
// status bits, 16-byte cp.async copies, FP16 conversion, small block-wide
// scans, programmatic-launch hooks and the decode-tail append.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "sa_b200.h"
#include "sa_internal.h"

namespace sa {

// A bounded wait gives up after this many SM clock cycles (~1 s at 1.9 GHz),
// sets SA_DEV_TIMEOUT and lets the kernel return instead of hanging.
constexpr long long kWaitLimitCycles = 2000000000LL;

__device__ __forceinline__ void raise_status(uint32_t* status, uint32_t bit) {
  if (status) atomicOr(status, bit);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- cp.async (16-byte copies through the load/store unit) ------------------

// Asynchronous 16-byte copy global -> shared (both 16-byte aligned); it lands
// when a later cp_async_wait covers its commit group.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)),
               "l"(reinterpret_cast<uint64_t>(src))
               : "memory");
}

__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Waits until at most N of this thread's commit groups are still in flight.
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- arrival counters ----------------------------------------------------------

// One arrival on a GPU-scope counter with acquire-release semantics; returns
// the count before it. Called by one thread after a barrier: the CTA's
// earlier stores are visible before the arrival, and an arriver that sees
// the last count sees every earlier arriver's stores (one atomic round trip,
// where a fence, the atomic and a second fence took three).
__device__ __forceinline__ int arrive_acq_rel(int* counter) {
  int prev;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
               : "=r"(prev)
               : "l"(counter)
               : "memory");
  return prev;
}

// ---- conversions -----------------------------------------------------------

__device__ __forceinline__ float h2f(uint16_t h) {
  return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t f2h_rn(float f) {
  return __half_as_ushort(__float2half_rn(f));
}

__device__ __forceinline__ float2 h2x2f(uint32_t packed) {
  __half2 h;
  *reinterpret_cast<uint32_t*>(&h) = packed;
  return __half22float2(h);
}

// Order-preserving map of a float to uint32 (larger float -> larger key).
// -0.0 is folded onto +0.0 so that the two compare equal, as `>` does.
__device__ __forceinline__ uint32_t float_order_key(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) == 0) u = 0;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// ---- block scans -------------------------------------------------------------

// Exclusive prefix sum over the threads of a block (blockDim.x <= 1024,
// multiple of 32). `scratch` holds >= 33 ints of shared memory. Returns the
// exclusive prefix; *total gets the block sum. Contains __syncthreads.
__device__ __forceinline__ int block_exclusive_scan(int value, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = blockDim.x >> 5;
  int inclusive = value;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, inclusive, o);
    if (lane >= o) inclusive += n;
  }
  if (lane == 31) scratch[warp] = inclusive;
  __syncthreads();
  if (warp == 0) {
    int w = lane < warps ? scratch[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    if (lane < warps) scratch[lane] = w;  // inclusive warp sums
    if (lane == warps - 1) scratch[32] = w;
  }
  __syncthreads();
  const int before = (warp > 0 ? scratch[warp - 1] : 0) + inclusive - value;
  *total = scratch[32];
  __syncthreads();
  return before;
}

// ---- programmatic dependent launch ------------------------------------------

// Lets the next kernel of the stream launch (its CTAs become resident and run
// up to their own pdl_wait) before this grid completes.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
// Blocks until the preceding grid of the stream has completed and its memory
// is visible; returns at once when the kernel was launched without the
// programmatic-serialization attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// ---- KV-head-sharded gather ----------------------------------------------------

// One thread, after a gathered attention grid has completed (every unit's
// output stored into every rank's gathered slot). The gather buffer's
// control words are [counter][epoch][target]: arrivals so far, gathers
// completed, and the arrivals that complete the latest one.
// signal: a decode step's seal kernel signals this rank's arrival to every
// rank itself -- one system-scope fence, cumulative over the attention
// grid's peer stores (which happen before its grid dependency wait), then
// one relaxed arrival per rank -- and this gather expects `per_epoch` =
// world arrivals; after a standalone attention, whose units each arrived on
// every rank, it expects world * units and signals nothing.
// Then it waits, bounded, with system-scope acquire loads, until the
// counter reaches the target, and advances the epoch (the next attention
// writes the other slot). A wait that gives up raises SA_DEV_TIMEOUT and
// still advances the epoch.
__device__ __forceinline__ void gather_signal_wait(void* const* peers, int world,
                                                   size_t counter_bytes,
                                                   const unsigned long long* counter,
                                                   unsigned long long* epoch,
                                                   unsigned long long per_epoch, bool signal,
                                                   uint32_t* status) {
  if (signal) {
    asm volatile("fence.sc.sys;" ::: "memory");
    for (int r = 0; r < world; ++r) {
      const unsigned long long* ctr = reinterpret_cast<const unsigned long long*>(
          reinterpret_cast<const uint8_t*>(peers[r]) + counter_bytes);
      asm volatile("red.relaxed.sys.global.add.u64 [%0], 1;" ::"l"(ctr) : "memory");
    }
  }
  unsigned long long* target = epoch + 1;
  const unsigned long long expected = *reinterpret_cast<volatile unsigned long long*>(target) +
                                      per_epoch;
  *target = expected;
  const long long start = clock64();
  for (;;) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(counter) : "memory");
    if (v >= expected) break;
    if (clock64() - start > kWaitLimitCycles) {
      raise_status(status, SA_DEV_TIMEOUT);
      break;
    }
    __nanosleep(128);
  }
  *epoch = *reinterpret_cast<volatile unsigned long long*>(epoch) + 1;
}

// ---- per-head RMS norm + rotary embedding (Qwen3 q/k norm) --------------------

// One 128-wide head row held in shared memory `row`, transformed in place by
// the 128 threads of a CTA (thread t owns element t): RMS norm with the
// reference's pairwise reduction order (head_rms, cpp/src/qwen_layer_main.cpp:
// 146-161: square, then strides 64, 32, ..., 1), then rotate-half RoPE at
// `position` (rope, :163-183). `red` is 128 floats of scratch. Both must be
// called by all 128 threads.
__device__ __forceinline__ void head_norm_rope(float* row, float* red, const float* weight,
                                               int position, float theta, float eps, int t) {
  const float v = row[t];
  red[t] = v * v;
  __syncthreads();
  for (int stride = 64; stride > 0; stride >>= 1) {
    if (t < stride) red[t] += red[t + stride];
    __syncthreads();
  }
  row[t] = v * rsqrtf(red[0] / 128.0f + eps) * weight[t];
  __syncthreads();
  const int half = 64;
  const int paired = t < half ? t + half : t - half;
  const int fi = t < half ? t : t - half;
  const float freq = powf(theta, -2.0f * fi / 128.0f);
  const float angle = position * freq;
  const float x = row[t];
  const float rotated = t < half ? -row[paired] : row[paired];
  __syncthreads();
  row[t] = x * cosf(angle) + rotated * sinf(angle);
  __syncthreads();
}

// ---- decode-tail append ------------------------------------------------------

// Writes the step's K/V of KV heads [kvh0, kvh1) of sequence-layer sl into
// row tail_len[sl] of its head-major tail block (plane (h, kv) row tl) and
// the queries of query heads [qh0, qh1) into the tail's query ring. tail_len
// is not changed. kv_new rows are [num_sl][2][kv_heads][128], FP16 or FP32
// (packed to FP16 with round-to-nearest-even). Every thread of the CTA calls
// it (index tid of nthreads); false, with a status bit, when the tail is
// full or its block id is invalid (the decision is uniform over the CTA).
__device__ __forceinline__ bool append_token(const CtxDev& c, int sl, const float* query,
                                             const void* kv_new, int kv_fp32, int kvh0, int kvh1,
                                             int qh0, int qh1, int tid, int nthreads) {
  const int tl = c.tail_len[sl];
  const int phys = c.tail_block[sl];
  // a tail this token fills (or one already full) needs the seal's full pass
  if (tid == 0 && tl >= kBlockTokens - 1) c.seal_counters[1] = 1;
  if (tl < 0 || tl >= kBlockTokens) {
    if (tid == 0) raise_status(c.status, SA_DEV_TAIL_FULL);
    return false;
  }
  if (phys < 0 || phys >= c.pool_blocks) {
    if (tid == 0) raise_status(c.status, SA_DEV_BAD_BLOCK);
    return false;
  }
  uint16_t* block = c.pool + (int64_t)phys * c.kv_heads * 2 * kBlockTokens * kHeadDim;
  constexpr int kChunksPerPlane = kHeadDim / 8;  // 16-byte FP16 chunks of one head row
  const int heads = kvh1 - kvh0;
  const int chunks = 2 * heads * kChunksPerPlane;
  for (int i = tid; i < chunks; i += nthreads) {
    const int kv = i / (heads * kChunksPerPlane);
    const int rem = i - kv * heads * kChunksPerPlane;
    const int h = kvh0 + rem / kChunksPerPlane;
    const int d = (rem % kChunksPerPlane) * 8;
    const int64_t src = (((int64_t)sl * 2 + kv) * c.kv_heads + h) * kHeadDim + d;
    uint4* dst = reinterpret_cast<uint4*>(block + (((int64_t)h * 2 + kv) * kBlockTokens + tl) *
                                                      kHeadDim + d);
    if (kv_fp32) {
      const float4* f = reinterpret_cast<const float4*>(static_cast<const float*>(kv_new) + src);
      const float4 a = f[0], b = f[1];
      *dst = make_uint4((uint32_t)f2h_rn(a.x) | ((uint32_t)f2h_rn(a.y) << 16),
                        (uint32_t)f2h_rn(a.z) | ((uint32_t)f2h_rn(a.w) << 16),
                        (uint32_t)f2h_rn(b.x) | ((uint32_t)f2h_rn(b.y) << 16),
                        (uint32_t)f2h_rn(b.z) | ((uint32_t)f2h_rn(b.w) << 16));
    } else {
      *dst = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(kv_new) + src);
    }
  }
  float* ring = c.query_ring + (int64_t)sl * c.qh * kBlockTokens * kHeadDim;
  const float* q = query + (int64_t)sl * c.qh * kHeadDim;
  const int qchunks = (qh1 - qh0) * kHeadDim / 4;
  for (int i = tid; i < qchunks; i += nthreads) {
    const int h = qh0 + (4 * i) / kHeadDim;
    const int d = (4 * i) % kHeadDim;
    *reinterpret_cast<float4*>(ring + ((int64_t)h * kBlockTokens + tl) * kHeadDim + d) =
        *reinterpret_cast<const float4*>(q + (int64_t)h * kHeadDim + d);
  }
  return true;
}

}  // namespace sa
