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
static_assert(kDemoteThreads >= kTileTokens, "one thread per token slot of a tile");

__device__ __forceinline__ uint32_t first_of(const GroupDesc& g, int j) { return g.first[j]; }
}  // namespace

__global__ void __launch_bounds__(kDemoteThreads, 8) demote_kernel(const DemoteParams p) {
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
  // Thread t owns token slot t of the new block's header segment and of every plane segment: all its
  // loads are issued before any store, so each thread keeps up to 17 independent loads in flight.
  const uint32_t t = threadIdx.x;
  const uint32_t* __restrict__ src = reinterpret_cast<const uint32_t*>(p.old_code + od.code_offset);
  uint32_t* __restrict__ dst = reinterpret_cast<uint32_t*>(p.new_code + nd.code_offset);
  const uint64_t* __restrict__ src64 = reinterpret_cast<const uint64_t*>(src);
  uint64_t* __restrict__ dst64 = reinterpret_cast<uint64_t*>(dst);
  const uint32_t nf0 = first_of(nd, 0);
  const bool has_hdr = t + nf0 < static_cast<uint32_t>(n);
  uint32_t hdr = 0u;
  if (has_hdr) hdr = __ldg(src + (nf0 - first_of(od, 0)) + t);  // headers of the tokens keeping a plane
  uint64_t word[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t ofj = first_of(od, j), nfj = first_of(nd, j);
    if (t + nfj < static_cast<uint32_t>(n)) word[j] = __ldg(src64 + old_seg / 8 + (nfj - ofj) + t);
    old_seg += (n - ofj) * 8u;
  }
  if (has_hdr) dst[t] = hdr;
  uint32_t at = new_seg / 8 + t;  // slot t's word in plane j of the new block
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint32_t nfj = first_of(nd, j);
    if (t + nfj < static_cast<uint32_t>(n)) dst64[at] = word[j];
    at += n - nfj;
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
