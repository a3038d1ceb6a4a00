// demote.cu — tier management: demote hot tokens by dropping their least significant planes.
//
// The progressive codec's planes are ordered most significant first, and a token holding its first m
// planes decodes at that precision (scripts/progressive.py:47-55). Dropping d planes from every token of
// a tile keeps the tile's tokens sorted by plane count, so each (tile, group) block stays a block of the
// same layout: the holders of plane j become the old holders of plane j + d, a suffix of the old
// holders of plane j. The new block is therefore the concatenation of contiguous pieces of the old one:
// the headers of the tokens that keep a plane, then for every plane j the words of its new holders. The
// dropped planes stay in the cold tier, which holds every plane of every token.
//
// Persistent CTAs (8 per SM) walk the new blocks with a stride of the grid; the host lays the new blocks
// out (offsets, sizes, first tables) from the old descriptors and the planes dropped. Each CTA runs a
// software pipeline, one step per block and one commit group of asynchronous copies (cp.async) per step.
// Block j: its old index and token count are copied at step j - 2A - 1, its old and new descriptors at
// step j - A - 1; at step j - 1 warp 0 checks them and turns them into a copy plan (per segment: first
// old word, first new word, words); step j copies the surviving pieces into shared memory and step
// j + A - 1 writes them to their new place. A = 3 blocks of data per CTA are in flight, the checks run
// once per block, and every wait is cp.async.wait_group on the thread's own copies.
#include "dkv_format.cuh"
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kDemoteThreads = 128;
constexpr int kDemoteCtasPerSm = 8;
constexpr int kMaxCodePlanes = 8;          // planes of a progressive code (quantize8)
constexpr int kAhead = 3;                  // A: blocks whose data is in flight per CTA
constexpr int kLag = kAhead - 1;           // a block is written kLag steps after its data copy is issued
constexpr int kDataSlots = kAhead;
constexpr int kDescSlots = 2 * kAhead + 1;
constexpr int kIndexSlots = kAhead + 1;
static_assert(kDemoteThreads >= kTileTokens, "one thread per token slot of a tile");

// Shared-memory image of one block's surviving pieces: thread t's header and plane words at [t].
struct DataSlot {
  uint32_t hdr[kTileTokens];
  uint64_t plane[kMaxCodePlanes][kTileTokens];
};
// A block's descriptors (old and new GroupDesc, copied 16 bytes at a time), its tile's token count,
// whether its old index was in range, and the copy plan built from them.
struct alignas(16) DescSlot {
  GroupDesc od;
  GroupDesc nd;
  int n;
  int oi_ok;
  int ok;                          // the block passed every check: the plan may be used
  uint32_t hdr_src, hdr_dst, hdr_cnt;  // header words (32-bit units of the code buffers)
  uint32_t src[kMaxCodePlanes];    // first old word of plane j's survivors (64-bit units of old_code)
  uint32_t dst[kMaxCodePlanes];    // first new word of plane j (64-bit units of new_code)
  uint32_t cnt[kMaxCodePlanes];    // holders of plane j in the new block
};
struct IndexSlot {
  int oi;
  int n;
};
struct DemoteShared {
  DataSlot data[kDataSlots];
  DescSlot desc[kDescSlots];
  IndexSlot index[kIndexSlots];
};
static_assert(sizeof(DemoteShared) <= 48 * 1024, "static shared memory");

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_lag() { asm volatile("cp.async.wait_group %0;" ::"n"(kLag) : "memory"); }

// Warp 0 checks one block's descriptors and writes its copy plan; lane j < 8 handles plane j (and the
// first-table entry j + 8). Checks: both blocks progressive codes inside their buffers, first tables
// inside the tile, each new holder range a suffix of the old one, no plane beyond the 8 of a progressive
// code, every segment inside its block.
__device__ __forceinline__ void build_plan(DescSlot& d, const DemoteParams& p, uint32_t lane) {
  const int n = d.n;
  const uint32_t un = static_cast<uint32_t>(n);
  const GroupDesc& od = d.od;
  const GroupDesc& nd = d.nd;
  const uint32_t j = lane & 7u;
  const uint32_t ofj = od.first[j], nfj = nd.first[j];
  const uint32_t of0 = od.first[0], nf0 = nd.first[0];
  bool ok = d.oi_ok != 0 && n >= 1 && n <= kTileTokens && od.kind == kKindProgressive &&
            od.max_planes <= kMaxCodePlanes && static_cast<uint64_t>(od.code_offset) + od.code_bytes <= p.old_code_size &&
            static_cast<uint64_t>(nd.code_offset) + nd.code_bytes <= p.new_code_size;
  ok = ok && ofj <= un && nfj <= un && nfj >= ofj && of0 <= un && nf0 <= un;
  ok = ok && od.first[j + 8] == un && nd.first[j + 8] == un;
  // Segment sizes in 64-bit words (ok guarantees no wrap) and their exclusive prefix over planes.
  const uint32_t old_words = ok ? un - ofj : 0u, new_words = ok ? un - nfj : 0u;
  uint32_t old_pre = old_words, new_pre = new_words;
#pragma unroll
  for (int k = 1; k < 8; k <<= 1) {
    const uint32_t o = __shfl_up_sync(0xFFFFFFFFu, old_pre, k, 8);
    const uint32_t w = __shfl_up_sync(0xFFFFFFFFu, new_pre, k, 8);
    if (j >= static_cast<uint32_t>(k)) {
      old_pre += o;
      new_pre += w;
    }
  }
  const uint32_t old_all = __shfl_sync(0xFFFFFFFFu, old_pre, 7, 8), new_all = __shfl_sync(0xFFFFFFFFu, new_pre, 7, 8);
  old_pre -= old_words;
  new_pre -= new_words;
  const uint32_t old_hdr = ok ? ((un - of0) * 4u + 7u) / 8u : 0u, new_hdr = ok ? ((un - nf0) * 4u + 7u) / 8u : 0u;
  ok = ok && (old_hdr + old_all) * 8ull <= od.code_bytes && (new_hdr + new_all) * 8ull <= nd.code_bytes;
  ok = __all_sync(0xFFFFFFFFu, ok);
  if (lane < 8) {
    d.src[j] = od.code_offset / 8u + old_hdr + old_pre + (nfj - ofj);
    d.dst[j] = nd.code_offset / 8u + new_hdr + new_pre;
    d.cnt[j] = ok ? un - nfj : 0u;
  }
  if (lane == 0) {
    d.hdr_src = od.code_offset / 4u + (nf0 - of0);
    d.hdr_dst = nd.code_offset / 4u;
    d.hdr_cnt = ok ? un - nf0 : 0u;
    d.ok = ok ? 1 : 0;
  }
}
}  // namespace

__global__ void __launch_bounds__(kDemoteThreads, kDemoteCtasPerSm) demote_kernel(const DemoteParams p) {
  __shared__ DemoteShared sm;
  const uint32_t t = threadIdx.x;
  const int64_t stride = gridDim.x;
  const int64_t base = blockIdx.x;
  const int n_mine = static_cast<int>((p.n_new - base + stride - 1) / stride);  // blocks of this CTA (>= 1)
  const uint32_t* __restrict__ old32 = reinterpret_cast<const uint32_t*>(p.old_code);
  const uint64_t* __restrict__ old64 = reinterpret_cast<const uint64_t*>(p.old_code);
  uint32_t* __restrict__ new32 = reinterpret_cast<uint32_t*>(p.new_code);
  uint64_t* __restrict__ new64 = reinterpret_cast<uint64_t*>(p.new_code);
  for (int i = -2 * kAhead - 1; i < n_mine + kLag; ++i) {
    // Index and token count of block i + 2A + 1.
    const int jx = i + 2 * kAhead + 1;
    if (jx < n_mine && (t == 4 || t == 5)) {
      IndexSlot& x = sm.index[jx % kIndexSlots];
      const int64_t b = base + jx * stride;
      if (t == 4) cp_async4(&x.oi, p.old_index + b);
      else cp_async4(&x.n, p.n_tokens + b);
    }
    // Descriptors of block i + A + 1 (its index arrived A steps ago).
    const int jd = i + kAhead + 1;
    if (jd >= 0 && jd < n_mine && t < 5) {
      const IndexSlot& x = sm.index[jd % kIndexSlots];
      DescSlot& d = sm.desc[jd % kDescSlots];
      const int oi = x.oi;
      const bool oi_ok = oi >= 0 && oi < p.n_old_groups;
      const int64_t b = base + jd * stride;
      if (t < 2) {
        if (oi_ok) cp_async16(reinterpret_cast<uint8_t*>(&d.od) + 16 * t, reinterpret_cast<const uint8_t*>(p.old_groups + oi) + 16 * t);
      } else if (t < 4) {
        cp_async16(reinterpret_cast<uint8_t*>(&d.nd) + 16 * (t - 2), reinterpret_cast<const uint8_t*>(p.new_groups + b) + 16 * (t - 2));
      } else {
        d.n = x.n;
        d.oi_ok = oi_ok ? 1 : 0;
      }
    }
    // Copy plan of block i + 1 (its descriptors arrived A steps ago).
    const int jp = i + 1;
    if (jp >= 0 && jp < n_mine && t < 32) build_plan(sm.desc[jp % kDescSlots], p, t);
    // Surviving pieces of block i into shared memory.
    if (i >= 0 && i < n_mine) {
      const DescSlot& d = sm.desc[i % kDescSlots];
      DataSlot& ds = sm.data[i % kDataSlots];
      if (t < d.hdr_cnt) cp_async4(&ds.hdr[t], old32 + d.hdr_src + t);
#pragma unroll
      for (int j = 0; j < kMaxCodePlanes; ++j)
        if (t < d.cnt[j]) cp_async8(&ds.plane[j][t], old64 + d.src[j] + t);
    }
    cp_async_commit();
    cp_async_wait_lag();  // this thread's copies of step i - lag have landed
    // Block i - lag to its new place.
    const int jw = i - kLag;
    if (jw >= 0 && jw < n_mine) {
      const DescSlot& d = sm.desc[jw % kDescSlots];
      const DataSlot& ds = sm.data[jw % kDataSlots];
      if (t < d.hdr_cnt) new32[d.hdr_dst + t] = ds.hdr[t];
#pragma unroll
      for (int j = 0; j < kMaxCodePlanes; ++j)
        if (t < d.cnt[j]) new64[d.dst[j] + t] = ds.plane[j][t];
      if (t == 0 && !d.ok) record_error(p.status, kErrBadDescriptor);
    }
    __syncthreads();  // what some threads copied or planned is read by all in later steps
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

int run_demote(const DemoteParams& p, cudaStream_t stream) {
  if (p.n_new < 0 || p.n_old_groups < 0) return kDkvErrArgs;
  if ((reinterpret_cast<uintptr_t>(p.old_code) & 15u) || (reinterpret_cast<uintptr_t>(p.new_code) & 15u) ||
      (reinterpret_cast<uintptr_t>(p.old_groups) & 15u) || (reinterpret_cast<uintptr_t>(p.new_groups) & 15u) ||
      (reinterpret_cast<uintptr_t>(p.old_index) & 3u) || (reinterpret_cast<uintptr_t>(p.n_tokens) & 3u))
    return kDkvErrArgs;
  if (p.n_new == 0) return kDkvOk;
  if (p.n_new > 0x7FFFFFFF) return kDkvErrConfig;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return kDkvErrCuda;
  // Eight CTAs of this kernel's static shared memory need the largest shared-memory carveout.
  if (cudaFuncSetAttribute(demote_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100) != cudaSuccess)
    return kDkvErrCuda;
  const int64_t grid = p.n_new < static_cast<int64_t>(sms) * kDemoteCtasPerSm ? p.n_new
                                                                                 : static_cast<int64_t>(sms) * kDemoteCtasPerSm;
  demote_kernel<<<static_cast<unsigned>(grid), kDemoteThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
