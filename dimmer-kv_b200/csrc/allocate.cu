// allocate.cu — the per-token rung allocator of DimmerKV on the GPU.
//
// Replaces kvtc.allocate_rungs (scripts/kvtc.py:277-298): every slot (token of the key or the value
// stream) starts at its coarsest rung; each upgrade l -> l+1 is worth
//   value = max(err[l] - err[l+1], 0) / (size[l+1] - size[l])      (float32 difference, double quotient)
// made non-increasing along a slot's upgrades with a running minimum; all upgrades are sorted by value,
// descending and stable (ties by flat index slot * (levels - 1) + l), and the longest prefix whose summed
// cost fits the budget is taken; a slot's count is the number of its upgrades taken.
//
// Instead of sorting, the cut is found by a radix select on the order of the values: each value becomes a
// 64-bit key whose ascending order is the values' descending order; eight passes over 8 bits each build
// a histogram of upgrade costs per digit among the keys that match the digits chosen so far, and a
// one-CTA pass picks the digit where the running cost crosses the remaining budget. That leaves one key
// K (the value group the cut falls in) and the budget left for it: every upgrade with a smaller key is
// taken, none with a larger one, and those with key K are taken in flat-index order while their running
// cost fits (a scan over slots). Sizes and costs are integers, so every sum is exact and the result equals
// the sort-based one bit for bit.
#include <cstdint>

#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kAllocThreads = 256;
constexpr int kMaxLevels = 64;

// Ascending key order = descending value order; -0.0 ties with +0.0; NaN (a NaN error) sorts first.
__device__ __forceinline__ uint64_t desc_key(double v) {
  if (v != v) return 0ull;
  if (v == 0.0) v = 0.0;
  uint64_t b = static_cast<uint64_t>(__double_as_longlong(v));
  b = (b & 0x8000000000000000ull) ? ~b : (b | 0x8000000000000000ull);  // ascending order of v
  return ~b;                                                             // descending
}

// State of the select, in the workspace: [0] key prefix, [1] remaining budget, [2] 1 when every upgrade
// fits (no cut).
struct SelectState {
  unsigned long long prefix, remaining, all_fit, pad;
};
}  // namespace

// One thread per slot: the slot's upgrade keys and costs.
__global__ void alloc_prepare_kernel(const AllocParams p, uint64_t* keys, uint64_t* costs, int* status) {
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (slot >= p.slots) return;
  const int L = p.levels;
  const int64_t* size = p.level_bytes + (slot < p.middle ? 0 : L);
  const float* err = p.errors + slot * L;
  double run = 0.0;
  for (int l = 0; l + 1 < L; ++l) {
    const int64_t c = size[l + 1] - size[l];
    if (c <= 0) {
      record_error(status, kErrBadDescriptor);  // level sizes must grow
      return;
    }
    float g = __fsub_rn(err[l], err[l + 1]);
    g = (g != g) ? g : fmaxf(g, 0.f);  // clamp_min(0) keeps NaN
    const double v = __ddiv_rn(static_cast<double>(g), static_cast<double>(c));
    run = (l == 0) ? v : ((v != v || run != run) ? (run != run ? run : v) : fmin(run, v));
    keys[slot * (L - 1) + l] = desc_key(run);
    costs[slot * (L - 1) + l] = static_cast<uint64_t>(c);
  }
}

// Pass `pass` (0..7): cost histogram of digit `pass` over the keys matching the chosen prefix.
__global__ void alloc_hist_kernel(int64_t n, const uint64_t* keys, const uint64_t* costs, const SelectState* st,
                                  unsigned long long* hist, int pass) {
  __shared__ unsigned long long h[256];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) h[i] = 0ull;
  __syncthreads();
  const int shift = 56 - 8 * pass;
  const uint64_t mask = pass == 0 ? 0ull : (~0ull << (64 - 8 * pass));
  const uint64_t prefix = st->prefix;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint64_t k = keys[i];
    if ((k & mask) == (prefix & mask)) atomicAdd(&h[(k >> shift) & 255u], static_cast<unsigned long long>(costs[i]));
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 256; i += blockDim.x)
    if (h[i]) atomicAdd(&hist[i], h[i]);
}

// The select's state and histogram from zero; the remaining budget as given.
__global__ void alloc_init_kernel(SelectState* st, unsigned long long* hist, unsigned long long remaining) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0ull;
  if (threadIdx.x == 0) {
    st->prefix = 0ull;
    st->remaining = remaining;
    st->all_fit = 0ull;
    st->pad = 0ull;
  }
}

// One thread: the digit where the running cost (ascending keys) crosses the remaining budget.
__global__ void alloc_decide_kernel(SelectState* st, unsigned long long* hist, int pass) {
  if (threadIdx.x != 0) return;
  if (st->all_fit) {
    for (int i = 0; i < 256; ++i) hist[i] = 0ull;
    return;
  }
  unsigned long long acc = 0ull;
  const unsigned long long r = st->remaining;
  int d = 0;
  for (; d < 256; ++d) {
    if (acc + hist[d] > r) break;
    acc += hist[d];
  }
  if (d == 256) {
    st->all_fit = 1ull;  // every upgrade under this prefix fits (only possible on the first pass)
  } else {
    st->remaining = r - acc;
    st->prefix |= static_cast<unsigned long long>(d) << (56 - 8 * pass);
  }
  for (int i = 0; i < 256; ++i) hist[i] = 0ull;
}

// Cost of each slot's upgrades whose key is the cut key (the tie group), summed per block of slots.
__global__ void alloc_tie_sums_kernel(const AllocParams p, const uint64_t* keys, const uint64_t* costs,
                                      const SelectState* st, unsigned long long* slot_tie,
                                      unsigned long long* block_sums) {
  __shared__ unsigned long long red[kAllocThreads / 32];
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  unsigned long long t = 0ull;
  if (slot < p.slots && !st->all_fit) {
    const int L1 = p.levels - 1;
    for (int l = 0; l < L1; ++l)
      if (keys[slot * L1 + l] == st->prefix) t += costs[slot * L1 + l];
  }
  if (slot < p.slots) slot_tie[slot] = t;
  unsigned long long w = t;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) w += __shfl_xor_sync(0xffffffffu, w, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = w;
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
    for (int i = 0; i < kAllocThreads / 32; ++i) b += red[i];
    block_sums[blockIdx.x] = b;
  }
}

// Exclusive scan of the block sums (one CTA, in order).
__global__ void alloc_scan_blocks_kernel(unsigned long long* block_sums, int n_blocks) {
  if (threadIdx.x != 0) return;
  unsigned long long acc = 0ull;
  for (int b = 0; b < n_blocks; ++b) {
    const unsigned long long v = block_sums[b];
    block_sums[b] = acc;
    acc += v;
  }
}

// Per slot: upgrades below the cut key are taken; those at the cut key while the running tie cost (flat
// index order) fits the remaining budget.
__global__ void alloc_count_kernel(const AllocParams p, const uint64_t* keys, const uint64_t* costs,
                                   const SelectState* st, const unsigned long long* slot_tie,
                                   const unsigned long long* block_offsets) {
  __shared__ unsigned long long scan[kAllocThreads];
  const int64_t slot = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const unsigned long long mine = slot < p.slots ? slot_tie[slot] : 0ull;
  // Exclusive prefix of the tie costs of the block's slots (Hillis-Steele in shared memory).
  scan[threadIdx.x] = mine;
  __syncthreads();
  for (int o = 1; o < kAllocThreads; o <<= 1) {
    const unsigned long long add = threadIdx.x >= o ? scan[threadIdx.x - o] : 0ull;
    __syncthreads();
    scan[threadIdx.x] += add;
    __syncthreads();
  }
  if (slot >= p.slots) return;
  unsigned long long running = block_offsets[blockIdx.x] + scan[threadIdx.x] - mine;
  const int L1 = p.levels - 1;
  const bool all = st->all_fit != 0ull;
  const uint64_t cut = st->prefix;
  const unsigned long long budget = st->remaining;
  int taken = 0;
  for (int l = 0; l < L1; ++l) {
    const uint64_t k = keys[slot * L1 + l];
    if (all || k < cut) {
      ++taken;
    } else if (k == cut) {
      running += costs[slot * L1 + l];
      if (running <= budget) ++taken;
    }
  }
  p.counts[slot] = taken;
}

int64_t alloc_workspace_bytes(int64_t slots, int levels) {
  if (slots < 0 || levels < 2 || levels > kMaxLevels) return -1;
  const int64_t n = slots * (levels - 1);
  const int64_t blocks = (slots + kAllocThreads - 1) / kAllocThreads;
  return 256 + 256 * 8 + n * 16 + slots * 8 + (blocks + 1) * 8;
}

int run_allocate(const AllocParams& p, cudaStream_t stream) {
  if (p.slots < 0 || p.levels < 2 || p.levels > kMaxLevels || p.middle < 0 || p.middle > p.slots ||
      p.remaining < 0)
    return kDkvErrArgs;
  const int64_t need = alloc_workspace_bytes(p.slots, p.levels);
  if (p.workspace == nullptr || p.workspace_bytes < need || (reinterpret_cast<uintptr_t>(p.workspace) & 255u))
    return kDkvErrArgs;
  if (p.slots == 0) return kDkvOk;
  uint8_t* w = static_cast<uint8_t*>(p.workspace);
  SelectState* st = reinterpret_cast<SelectState*>(w);
  unsigned long long* hist = reinterpret_cast<unsigned long long*>(w + 256);
  const int64_t n = p.slots * (p.levels - 1);
  uint64_t* keys = reinterpret_cast<uint64_t*>(w + 256 + 256 * 8);
  uint64_t* costs = keys + n;
  unsigned long long* slot_tie = reinterpret_cast<unsigned long long*>(costs + n);
  unsigned long long* block_sums = slot_tie + p.slots;
  const int blocks = static_cast<int>((p.slots + kAllocThreads - 1) / kAllocThreads);
  alloc_init_kernel<<<1, 256, 0, stream>>>(st, hist, static_cast<unsigned long long>(p.remaining));
  alloc_prepare_kernel<<<blocks, kAllocThreads, 0, stream>>>(p, keys, costs, p.status);
  const int64_t want_blocks = (n + kAllocThreads - 1) / kAllocThreads;
  const int hist_blocks = static_cast<int>(want_blocks < 4 * 148 ? want_blocks : 4 * 148);
  for (int pass = 0; pass < 8; ++pass) {
    alloc_hist_kernel<<<hist_blocks, kAllocThreads, 0, stream>>>(n, keys, costs, st, hist, pass);
    alloc_decide_kernel<<<1, 32, 0, stream>>>(st, hist, pass);
  }
  alloc_tie_sums_kernel<<<blocks, kAllocThreads, 0, stream>>>(p, keys, costs, st, slot_tie, block_sums);
  alloc_scan_blocks_kernel<<<1, 32, 0, stream>>>(block_sums, blocks);
  alloc_count_kernel<<<blocks, kAllocThreads, 0, stream>>>(p, keys, costs, st, slot_tie, block_sums);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
