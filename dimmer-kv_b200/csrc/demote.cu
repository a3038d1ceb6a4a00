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
// out (offsets, sizes, first tables) from the old descriptors and the planes dropped. A block's
// descriptors (its old index, token count, old and new GroupDesc) are fetched into shared memory one
// block ahead, while the block before it is copied, so each block costs one round trip to HBM.
#include "dkv_format.cuh"
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kDemoteThreads = 128;
constexpr int kDemoteCtasPerSm = 8;
constexpr int kStageThreads = 18;  // threads that fetch a block's descriptors
constexpr int kMaxCodePlanes = 8;  // planes of a progressive code (quantize8)
static_assert(kDemoteThreads >= kTileTokens, "one thread per token slot of a tile");

// One block's descriptors in shared memory: the old and new GroupDesc as words, the old index (-1 when
// out of range) and the token count of the block's tile.
struct DemoteStage {
  uint32_t od[8];
  uint32_t nd[8];
  int oi;
  int n;
};

// Threads 0..17 fetch block b's descriptors: 0-7 the old descriptor's words, 8-15 the new one's, 16 the
// token count, 17 the old index. Every one of them holds oi, the block's old index.
__device__ __forceinline__ void fetch_stage(const DemoteParams& p, int64_t b, int oi, DemoteStage& s) {
  const int t = threadIdx.x;
  const bool oi_ok = oi >= 0 && oi < p.n_old_groups;
  if (t < 8) {
    s.od[t] = oi_ok ? __ldg(reinterpret_cast<const uint32_t*>(p.old_groups + oi) + t) : 0u;
  } else if (t < 16) {
    s.nd[t - 8] = __ldg(reinterpret_cast<const uint32_t*>(p.new_groups + b) + (t - 8));
  } else if (t == 16) {
    s.n = __ldg(p.n_tokens + b);
  } else if (t == 17) {
    s.oi = oi_ok ? oi : -1;
  }
}

__device__ __forceinline__ uint32_t first_byte(const uint32_t* first4, int j) {
  return (first4[j >> 2] >> ((j & 3) * 8)) & 0xFFu;
}
}  // namespace

__global__ void __launch_bounds__(kDemoteThreads, kDemoteCtasPerSm) demote_kernel(const DemoteParams p) {
  __shared__ DemoteStage stage[2];
  const uint32_t t = threadIdx.x;
  const int64_t stride = gridDim.x;
  int64_t b = blockIdx.x;
  int oi_next = -1;  // threads 0..17: the old index of the block after the one staged last
  if (t < kStageThreads) {
    fetch_stage(p, b, __ldg(p.old_index + b), stage[0]);
    if (b + stride < p.n_new) oi_next = __ldg(p.old_index + b + stride);
  }
  __syncthreads();
  for (int k = 0; b < p.n_new; ++k, b += stride) {
    const DemoteStage& s = stage[k & 1];
    const int n = s.n;
    const uint32_t od_off = s.od[1], od_bytes = s.od[2], od_kind = s.od[3] & 0xFFu, od_max = (s.od[3] >> 8) & 0xFFu;
    const uint32_t nd_off = s.nd[1], nd_bytes = s.nd[2];
    uint32_t of4[4], nf4[4];
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      of4[w] = s.od[4 + w];
      nf4[w] = s.nd[4 + w];
    }
    // Both blocks: progressive codes (raw and ladder blocks have no planes to drop), first tables inside the
    // tile, each new holder range inside the old one.
    bool ok = s.oi >= 0 && n >= 1 && n <= kTileTokens && od_kind == static_cast<uint32_t>(kKindProgressive) &&
              od_max <= 8u && static_cast<uint64_t>(od_off) + od_bytes <= p.old_code_size &&
              static_cast<uint64_t>(nd_off) + nd_bytes <= p.new_code_size;
    const uint32_t of0 = first_byte(of4, 0), nf0 = first_byte(nf4, 0);
    uint32_t old_seg = ((n - of0) * 4u + 7u) & ~7u;
    const uint32_t new_seg = ((n - nf0) * 4u + 7u) & ~7u;
    uint32_t old_total = old_seg, new_total = new_seg;
#pragma unroll
    for (int j = 0; j < kMaxCodePlanes; ++j) {
      const uint32_t ofj = first_byte(of4, j), nfj = first_byte(nf4, j);
      ok = ok && ofj <= static_cast<uint32_t>(n) && nfj <= static_cast<uint32_t>(n) && nfj >= ofj;
      old_total += (n - ofj) * 8u;
      new_total += (n - nfj) * 8u;
    }
    // A progressive block stores at most 8 planes: no token of either block holds a plane beyond them.
#pragma unroll
    for (int j = kMaxCodePlanes; j < 16; ++j)
      ok = ok && first_byte(of4, j) == static_cast<uint32_t>(n) && first_byte(nf4, j) == static_cast<uint32_t>(n);
    ok = ok && old_total <= od_bytes && new_total <= nd_bytes;
    // Thread t owns token slot t of the new block's header segment and of every plane segment: all its
    // loads are issued before any store, so each thread keeps up to 9 independent loads in flight.
    const uint32_t* __restrict__ src = reinterpret_cast<const uint32_t*>(p.old_code + od_off);
    uint32_t* __restrict__ dst = reinterpret_cast<uint32_t*>(p.new_code + nd_off);
    const uint64_t* __restrict__ src64 = reinterpret_cast<const uint64_t*>(src);
    uint64_t* __restrict__ dst64 = reinterpret_cast<uint64_t*>(dst);
    const bool has_hdr = ok && t + nf0 < static_cast<uint32_t>(n);
    uint32_t hdr = 0u;
    if (has_hdr) hdr = __ldg(src + (nf0 - of0) + t);  // headers of the tokens keeping a plane
    uint64_t word[kMaxCodePlanes];
#pragma unroll
    for (int j = 0; j < kMaxCodePlanes; ++j) {
      const uint32_t ofj = first_byte(of4, j), nfj = first_byte(nf4, j);
      if (ok && t + nfj < static_cast<uint32_t>(n)) word[j] = __ldg(src64 + old_seg / 8 + (nfj - ofj) + t);
      old_seg += (n - ofj) * 8u;
    }
    // The other stage was last read before the barrier that ended the previous iteration: fetch the next
    // block's descriptors into it while this block's loads are in flight.
    const int64_t b1 = b + stride;
    if (t < kStageThreads && b1 < p.n_new) {
      fetch_stage(p, b1, oi_next, stage[(k + 1) & 1]);
      oi_next = b1 + stride < p.n_new ? __ldg(p.old_index + b1 + stride) : -1;
    }
    if (ok) {
      if (has_hdr) dst[t] = hdr;
      uint32_t at = new_seg / 8 + t;  // slot t's word in plane j of the new block
#pragma unroll
      for (int j = 0; j < kMaxCodePlanes; ++j) {
        const uint32_t nfj = first_byte(nf4, j);
        if (t + nfj < static_cast<uint32_t>(n)) dst64[at] = word[j];
        at += n - nfj;
      }
    } else if (t == 0) {
      record_error(p.status, kErrBadDescriptor);
    }
    __syncthreads();
  }
}

int run_demote(const DemoteParams& p, cudaStream_t stream) {
  if (p.n_new < 0 || p.n_old_groups < 0) return kDkvErrArgs;
  if ((reinterpret_cast<uintptr_t>(p.old_code) & 15u) || (reinterpret_cast<uintptr_t>(p.new_code) & 15u))
    return kDkvErrArgs;
  if (p.n_new == 0) return kDkvOk;
  if (p.n_new > 0x7FFFFFFF) return kDkvErrConfig;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
    return kDkvErrCuda;
  const int64_t grid = p.n_new < static_cast<int64_t>(sms) * kDemoteCtasPerSm ? p.n_new
                                                                                 : static_cast<int64_t>(sms) * kDemoteCtasPerSm;
  demote_kernel<<<static_cast<unsigned>(grid), kDemoteThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
