// sa_slots.cu -- history-prediction slot table: correct a resident window
// of selected blocks against the current selection.
//
// Replaces compare_prediction (cpp/src/pipeline_main.cpp:686-717) and the
// slot maps of the Python decode loop (src/solidattention_lab/qwen_decode.py:
// 463-545), the consumer of the selector output in the reference's tiered
// pipeline: `budget` slots per (sequence-layer, selection group) hold the
// blocks predicted for this step (last step's selection); a block of the
// current selection that is resident is a hit, one that is not is a miss
// (in the selection's ascending order), and the misses overwrite, in order,
// the slots whose block was not selected (in slot order). The reference
// requires both sets to have `budget` blocks; here empty slots (-1) count as
// slots to overwrite, and slots left over when the selection is shorter than
// the window are emptied, so the first step and short contexts work too.
//
// One CTA per unit: residency of selected blocks through a shared-memory
// bitmap over block ids, both orders kept by block-wide exclusive scans.
#include "sa_device.cuh"
#include "sa_internal.h"

namespace sa {

namespace {

constexpr int kSlotThreads = 256;

struct SlotParams {
  const int32_t* selected;  // [units][budget] ascending
  const int32_t* counts;    // [units]
  int32_t* slots;           // [units][budget], -1 = empty
  int32_t* misses;          // [units][budget], -1 padded
  int32_t* replace;         // [units][budget], -1 padded
  int32_t* stats;           // [units][2]: hits, misses
  int budget;
  int id_limit;             // block ids are < id_limit (bitmap size in bits)
  uint32_t* status;
};

__global__ void __launch_bounds__(kSlotThreads) slot_correct_kernel(const SlotParams p) {
  extern __shared__ uint32_t resident[];  // bitmap over block ids
  __shared__ int scan[33];
  const int unit = blockIdx.x;
  const int32_t* sel = p.selected + (size_t)unit * p.budget;
  int32_t* slots = p.slots + (size_t)unit * p.budget;
  int32_t* misses = p.misses + (size_t)unit * p.budget;
  int32_t* replace = p.replace + (size_t)unit * p.budget;
  const int words = (p.id_limit + 31) / 32;
  const int count = max(0, min(p.counts[unit], p.budget));
  for (int w = threadIdx.x; w < words; w += kSlotThreads) resident[w] = 0;
  __syncthreads();
  // Each thread owns a contiguous run of slots (and of selected ids), so the
  // scans below keep slot order and selection order.
  const int per = (p.budget + kSlotThreads - 1) / kSlotThreads;
  const int lo = min(p.budget, (int)threadIdx.x * per);
  const int hi = min(p.budget, lo + per);
  for (int s = lo; s < hi; ++s) {
    const int b = slots[s];
    if (b >= 0 && b < p.id_limit) atomicOr(&resident[b >> 5], 1u << (b & 31));
    else if (b >= p.id_limit) raise_status(p.status, SA_DEV_BAD_BLOCK);
  }
  __syncthreads();
  // a slot is kept when its block is selected (binary search of the sorted selection)
  auto selected = [&](int b) {
    int l = 0, r = count;
    while (l < r) {
      const int m = (l + r) >> 1;
      if (sel[m] < b) l = m + 1;
      else r = m;
    }
    return l < count && sel[l] == b;
  };
  int evict_local = 0, miss_local = 0;
  for (int s = lo; s < hi; ++s) evict_local += !(slots[s] >= 0 && selected(slots[s]));
  for (int i = lo; i < min(hi, count); ++i) {
    const int b = sel[i];
    miss_local += !(b >= 0 && b < p.id_limit && (resident[b >> 5] >> (b & 31) & 1u));
  }
  int evict_total = 0, miss_total = 0;
  int evict_pos = block_exclusive_scan(evict_local, scan, &evict_total);
  __syncthreads();
  int miss_pos = block_exclusive_scan(miss_local, scan, &miss_total);
  // lists, -1 padded
  for (int s = lo; s < hi; ++s) {
    misses[s] = -1;
    replace[s] = -1;
  }
  __syncthreads();
  for (int s = lo; s < hi; ++s)
    if (!(slots[s] >= 0 && selected(slots[s]))) replace[evict_pos++] = s;
  for (int i = lo; i < min(hi, count); ++i) {
    const int b = sel[i];
    if (!(b >= 0 && b < p.id_limit && (resident[b >> 5] >> (b & 31) & 1u))) misses[miss_pos++] = b;
  }
  __syncthreads();
  // apply: the i-th miss overwrites the i-th freed slot; freed slots beyond
  // the misses are emptied
  for (int i = threadIdx.x; i < evict_total; i += kSlotThreads)
    slots[replace[i]] = i < miss_total ? misses[i] : -1;
  __syncthreads();  // replace[] is read above before its tail is cleared
  for (int i = miss_total + threadIdx.x; i < evict_total; i += kSlotThreads) replace[i] = -1;
  if (threadIdx.x == 0) {
    p.stats[2 * unit] = count - miss_total;
    p.stats[2 * unit + 1] = miss_total;
  }
}

}  // namespace

sa_status launch_slot_correct(const int32_t* selected, const int32_t* counts, int32_t* slots,
                              int32_t* misses, int32_t* replace, int32_t* stats, int units,
                              int budget, int id_limit, uint32_t* status, cudaStream_t stream) {
  if (units <= 0 || budget <= 0) return SA_OK;
  SlotParams p{selected, counts, slots, misses, replace, stats, budget, id_limit, status};
  const size_t smem = (size_t)((id_limit + 31) / 32) * sizeof(uint32_t);
  if (smem > 48 * 1024) return fail(SA_ERR_UNSUPPORTED, "slots: block ids above 393216");
  slot_correct_kernel<<<units, kSlotThreads, smem, stream>>>(p);
  return cuda_status(cudaGetLastError(), "slot_correct_kernel launch");
}

}  // namespace sa
