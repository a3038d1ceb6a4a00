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
// One CTA per new block, given the old block it comes from and its tile's token count; the host lays
// the new blocks out (offsets, sizes, first tables) from the old descriptors and the planes dropped.
#include "dkv_format.cuh"
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kDemoteThreads = 128;

__device__ __forceinline__ uint32_t first_of(const GroupDesc& g, int j) { return g.first[j]; }
}  // namespace

__global__ void __launch_bounds__(kDemoteThreads) demote_kernel(const DemoteParams p) {
  const int64_t i = blockIdx.x;
  const int oi = p.old_index[i];
  const int n = p.n_tokens[i];
  if (oi < 0 || oi >= p.n_old_groups || n < 1 || n > kTileTokens) {
    if (threadIdx.x == 0) record_error(p.status, kErrBadDescriptor);
    return;
  }
  const GroupDesc od = p.old_groups[oi];
  const GroupDesc nd = p.new_groups[i];
  // Both blocks: progressive codes (raw and ladder blocks have no planes to drop), first tables inside the
  // tile, each new holder range inside the old one.
  bool ok = od.kind == kKindProgressive && od.max_planes <= 8 &&
            static_cast<uint64_t>(od.code_offset) + od.code_bytes <= p.old_code_size &&
            static_cast<uint64_t>(nd.code_offset) + nd.code_bytes <= p.new_code_size;
  uint32_t old_seg = ((n - first_of(od, 0)) * 4u + 7u) & ~7u;
  uint32_t new_seg = ((n - first_of(nd, 0)) * 4u + 7u) & ~7u;
  uint32_t old_total = old_seg, new_total = new_seg;
  for (int j = 0; j < 16; ++j) {
    ok = ok && first_of(od, j) <= static_cast<uint32_t>(n) && first_of(nd, j) <= static_cast<uint32_t>(n) &&
         first_of(nd, j) >= first_of(od, j);
    old_total += (n - first_of(od, j)) * 8u;
    new_total += (n - first_of(nd, j)) * 8u;
  }
  ok = ok && old_total <= od.code_bytes && new_total <= nd.code_bytes;
  if (!ok) {
    if (threadIdx.x == 0) record_error(p.status, kErrBadDescriptor);
    return;
  }
  const uint32_t* src = reinterpret_cast<const uint32_t*>(p.old_code + od.code_offset);
  uint32_t* dst = reinterpret_cast<uint32_t*>(p.new_code + nd.code_offset);
  // Headers of the tokens that keep at least one plane.
  {
    const uint32_t skip = first_of(nd, 0) - first_of(od, 0);
    const uint32_t words = n - first_of(nd, 0);
    for (uint32_t w = threadIdx.x; w < words; w += blockDim.x) dst[w] = src[skip + w];
  }
  // Plane j: the 64-bit words of its new holders (plane segments start on 8-byte boundaries).
  const uint64_t* src64 = reinterpret_cast<const uint64_t*>(src);
  uint64_t* dst64 = reinterpret_cast<uint64_t*>(dst);
  for (int j = 0; j < 16; ++j) {
    const uint32_t old_holders = n - first_of(od, j), new_holders = n - first_of(nd, j);
    if (new_holders > 0) {
      const uint64_t* s = src64 + old_seg / 8 + (first_of(nd, j) - first_of(od, j));
      uint64_t* d = dst64 + new_seg / 8;
      for (uint32_t w = threadIdx.x; w < new_holders; w += blockDim.x) d[w] = s[w];
    }
    old_seg += old_holders * 8u;
    new_seg += new_holders * 8u;
  }
}

int run_demote(const DemoteParams& p, cudaStream_t stream) {
  if (p.n_new < 0 || p.n_old_groups < 0) return kDkvErrArgs;
  if ((reinterpret_cast<uintptr_t>(p.old_code) & 15u) || (reinterpret_cast<uintptr_t>(p.new_code) & 15u))
    return kDkvErrArgs;
  if (p.n_new == 0) return kDkvOk;
  if (p.n_new > 0x7FFFFFFF) return kDkvErrConfig;
  demote_kernel<<<static_cast<unsigned>(p.n_new), kDemoteThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
