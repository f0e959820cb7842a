// sa_probe.cu -- streaming probes: how fast the two ways of staging 16 KB
// pool blocks into shared memory read from HBM on this GPU.
//
// Not on the decode path. The attention kernel stages every selected
// (block, KV head) entry (16 KB: its K and V planes) into a ring of three
// 32 KB stages. Two ways to fill a stage were measured on a B200, and these
// kernels let anyone measure them again (bench.py --probe-streaming):
//
//  * per-lane cp.async: every thread copies 16-byte pieces itself and waits
//    only for its own commit groups (the attention's choice);
//  * bulk copies: one thread per CTA issues one 16 KB cp.async.bulk per
//    entry, completing on the stage's mbarrier, and all threads wait on it.
//    Plain bulk loads from this GPU's own pool (no cluster multicast).
//
// Both run two CTAs of 256 threads per SM with the attention's ring (three
// stages of two entries) and read one word of every entry after it lands,
// so nothing else limits the stream. Every mbarrier wait is bounded (about
// a second of %globaltimer): a wait that gives up sets SA_DEV_TIMEOUT and
// the CTA stops issuing copies, then waits (bounded again) for the copies
// it has in flight before it exits.
#include <algorithm>

#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kProbeThreads = 256;
constexpr int kProbeStages = 3;
constexpr int kEntry = 16384;             // one (block, KV head): K and V planes
constexpr int kProbeStage = 2 * kEntry;   // two entries a stage, as the attention
constexpr unsigned long long kWaitNs = 1000000000ull;  // one second

struct ProbeParams {
  const uint8_t* pool;   // entries of kEntry bytes
  const int32_t* ids;    // entry ids to read, in order
  int n;                 // ids
  int pool_entries;
  unsigned long long* sink;  // [grid]: one word per CTA (keeps the reads)
  uint32_t* status;
};

// The CTA's contiguous share of the ids.
__device__ __forceinline__ void cta_range(int n, int* lo, int* hi) {
  *lo = (int)((long long)blockIdx.x * n / gridDim.x);
  *hi = (int)((long long)(blockIdx.x + 1) * n / gridDim.x);
}

__device__ __forceinline__ const uint8_t* entry_src(const ProbeParams& p, int k) {
  const int id = p.ids[k];
  return p.pool + (size_t)(id >= 0 && id < p.pool_entries ? id : 0) * kEntry;
}

// Per-lane copies: thread t copies 16-byte pieces t, t + 256, ... of the
// stage's 32 KB (eight pieces) and reads back its first one.
__global__ void __launch_bounds__(kProbeThreads) probe_cp_async_kernel(const ProbeParams p) {
  extern __shared__ __align__(128) uint8_t ring[];
  int lo, hi;
  cta_range(p.n, &lo, &hi);
  const int stages = (hi - lo + 1) / 2;
  auto load = [&](int j, int slot) {
#pragma unroll
    for (int r = 0; r < kProbeStage / 16 / kProbeThreads; ++r) {
      const int piece = threadIdx.x + r * kProbeThreads;
      const int e = piece / (kEntry / 16);
      const int k = lo + 2 * j + e;
      if (k < hi)
        cp_async16(ring + slot * kProbeStage + piece * 16,
                   entry_src(p, k) + (piece - e * (kEntry / 16)) * 16);
    }
  };
#pragma unroll
  for (int j = 0; j < kProbeStages; ++j) {
    if (j < stages) load(j, j);
    cp_async_commit();
  }
  unsigned long long acc = 0;
  int slot = 0;
  for (int j = 0; j < stages; ++j) {
    cp_async_wait<kProbeStages - 1>();
    if (lo + 2 * j < hi)
      acc ^= *reinterpret_cast<const unsigned long long*>(ring + slot * kProbeStage +
                                                          threadIdx.x * 16);
    if (j + kProbeStages < stages) load(j + kProbeStages, slot);
    cp_async_commit();
    if (++slot == kProbeStages) slot = 0;
  }
  cp_async_wait<0>();
  acc = __reduce_xor_sync(0xffffffffu, (unsigned)acc) ^ (acc >> 32);
  if (threadIdx.x == 0) p.sink[blockIdx.x] = acc;
}

__device__ __forceinline__ unsigned long long probe_time() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(bytes)
               : "memory");
}

// One bulk copy of `bytes` (a multiple of 16, both addresses 16-byte
// aligned) from this GPU's global memory into this CTA's shared memory,
// completing on `bar`.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase of `bar` with this parity; false after about a second.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  const unsigned long long t0 = probe_time();
  while (!mbar_try_wait(bar, parity))
    if (probe_time() - t0 > kWaitNs) return false;
  return true;
}

// One thread issues a stage's two 16 KB bulk copies on the stage's
// mbarrier; every thread waits for the phase, reads, and after a barrier the
// thread refills the stage.
__global__ void __launch_bounds__(kProbeThreads) probe_bulk_kernel(const ProbeParams p) {
  extern __shared__ __align__(128) uint8_t ring[];
  __shared__ __align__(8) uint64_t bar[kProbeStages];
  __shared__ int failed;
  int lo, hi;
  cta_range(p.n, &lo, &hi);
  const int stages = (hi - lo + 1) / 2;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kProbeStages; ++s) mbar_init(&bar[s]);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    failed = 0;
  }
  __syncthreads();
  auto issue = [&](int j, int slot) {
    const int k0 = lo + 2 * j;
    const int cnt = min(2, hi - k0);
    mbar_expect_tx(&bar[slot], (uint32_t)(cnt * kEntry));
    for (int e = 0; e < cnt; ++e)
      bulk_load(ring + slot * kProbeStage + e * kEntry, entry_src(p, k0 + e), kEntry, &bar[slot]);
  };
  if (threadIdx.x == 0)
    for (int j = 0; j < kProbeStages && j < stages; ++j) issue(j, j);
  unsigned long long acc = 0;
  int slot = 0, j = 0;
  for (; j < stages; ++j) {
    if (!mbar_wait_bounded(&bar[slot], (uint32_t)((j / kProbeStages) & 1))) failed = 1;
    __syncthreads();
    if (failed) break;
    acc ^= *reinterpret_cast<const unsigned long long*>(ring + slot * kProbeStage + threadIdx.x * 16);
    __syncthreads();  // every read of the stage is done before its refill
    if (threadIdx.x == 0 && j + kProbeStages < stages) issue(j + kProbeStages, slot);
    if (++slot == kProbeStages) slot = 0;
  }
  if (failed) {
    // stop issuing; wait (bounded) for the stages still in flight
    if (threadIdx.x == 0) {
      raise_status(p.status, SA_DEV_TIMEOUT);
      for (int q = j; q < stages && q < j + kProbeStages; ++q)
        mbar_wait_bounded(&bar[q % kProbeStages], (uint32_t)((q / kProbeStages) & 1));
    }
    __syncthreads();
    return;
  }
  acc = __reduce_xor_sync(0xffffffffu, (unsigned)acc) ^ (acc >> 32);
  if (threadIdx.x == 0) p.sink[blockIdx.x] = acc;
}

}  // namespace

int probe_sink_words() { return 1024; }

sa_status launch_probe_stream(const void* pool, long long pool_entries, const int32_t* ids,
                              long long n, int mode, unsigned long long* sink, uint32_t* status,
                              cudaStream_t stream) {
  if (!pool || !ids || !sink || pool_entries <= 0 || n <= 0 || n > 0x7fffffffLL ||
      pool_entries > 0x7fffffffLL || (mode != 0 && mode != 1))
    return fail(SA_ERR_INVALID_ARG, "probe_stream: bad argument");
  if ((reinterpret_cast<uintptr_t>(pool) & 15u) != 0)
    return fail(SA_ERR_INVALID_ARG, "probe_stream: the pool must be 16-byte aligned");
  ProbeParams p{};
  p.pool = static_cast<const uint8_t*>(pool);
  p.ids = ids;
  p.n = (int)n;
  p.pool_entries = (int)pool_entries;
  p.sink = sink;
  p.status = status;
  const int grid = std::min(2 * device_sm_count(), probe_sink_words());
  const int smem = kProbeStages * kProbeStage;
  static int configured[2][kMaxDevices];
  const void* k = mode == 0 ? (const void*)probe_cp_async_kernel : (const void*)probe_bulk_kernel;
  const sa_status st = ensure_smem_limit(k, smem, configured[mode]);
  if (st != SA_OK) return st;
  if (mode == 0)
    probe_cp_async_kernel<<<grid, kProbeThreads, smem, stream>>>(p);
  else
    probe_bulk_kernel<<<grid, kProbeThreads, smem, stream>>>(p);
  return cuda_status(cudaGetLastError(), "probe kernel launch");
}

}  // namespace sa
