// value_dense.cu — attention probabilities applied to value coefficients that were decoded once per
// decode step, streamed from HBM by TMA (the value stage at HBM speed instead of decode speed).
//
// Replaces, like value_weights.cu, the per-block value products of CompressedContext.attend
// (scripts/compressed_attention.py:127, 132-133):
//   p_c = softmax(...)[..., :middle].to(dtype)
//   weighted += einsum("bhgqn,nr->bhgqr", p_c[..., block.index], block.coefficients)
// The value coefficients are the same for every layer (the cross-layer basis spans all of them,
// compressed_attention.py:128-134 use block["coefficients"] for every layer), so the plane streams are
// decoded once per decode step by dkv_unpack into a tile-padded bf16 buffer (tile t's tokens at rows
// t * 128 .., the rows past a tile's tokens zero) and every layer reads that buffer instead of decoding
// the planes again: one decode per step instead of one per layer.
//
// One CTA per SM walks its list of work items (conversation, run of value tiles, range of union groups;
// the same items and schedule as the decoding kernel). Roles (256 threads):
//   warp 0     P / descriptor producer: per (item, tile) the tile's P^T image (bf16 probabilities built by
//              vprobs_kernel in the MMA's B-operand layout) and the tile's block descriptors inside the
//              item's groups, each with one bulk copy into a double buffer
//   warp 1     MMA issuer: per group pair of a tile, 8 tcgen05.mma (M = 128 components, N = rows,
//              K = 16 tokens each) into the item's TMEM accumulator (two of 256 columns, items alternate)
//   warp 2     A producer: per group pair, two TMA boxes of 64 components x 128 tokens (128B swizzle) of
//              the decoded buffer into a ring of A stages (a pair's absent group reads zeros there)
//   warps 4-7  epilogue, one per TMEM lane quarter: the finished accumulator -> fp32 partial sums,
//              reduced by finalize.cu, while the next item accumulates into the other half of TMEM
// Every wait is bounded and abort-aware (dkv_ptx.cuh); the kernel does no work when the call's status
// word is already set.
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {

constexpr int kDThreads = 256;
constexpr int kDPairTile = 32768;       // two groups x 128 tokens x 128 B
constexpr int kDHalf = 16384;
constexpr int kDMaxRangeGroups = 64;
constexpr int kDAccumCols = 256;
constexpr int kDMaxStages = 6;

// Next group pair of a tile's descriptor list (in shared memory, sorted by union group).
__device__ __forceinline__ int dense_next_pair(const GroupDesc* d, int n, int g0, int& i) {
  if (i >= n) return -1;
  const int g = static_cast<int>(d[i].group);
  const int pair = (g - g0) >> 1;
  ++i;
  if (((g - g0) & 1) == 0 && i < n && static_cast<int>(d[i].group) == g + 1) ++i;
  return pair;
}

}  // namespace

template <bool F16>
__global__ void __launch_bounds__(kDThreads, 1)
    value_dense_kernel(const __grid_constant__ CUtensorMap vmap, const ValueWeightParams p, int a_stages) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NR = p.n_rows_pad;                        // MMA N (multiple of 16, <= 128)
  const int p_tile = NR * 256;                        // P^T image: two K atoms of 64 tokens
  uint8_t* a_tiles = smem;                            // [a_stages][kDPairTile]
  uint8_t* p_tiles = a_tiles + a_stages * kDPairTile;  // [2][p_tile]
  GroupDesc* descs = reinterpret_cast<GroupDesc*>(p_tiles + 2 * p_tile);  // [2][kDMaxRangeGroups]
  uint64_t* bars = reinterpret_cast<uint64_t*>(descs + 2 * kDMaxRangeGroups);
  uint64_t* a_full = bars;                   // [a_stages] the A producer's two TMA boxes
  uint64_t* a_empty = a_full + kDMaxStages;  // [a_stages] MMA commit
  uint64_t* p_full = a_empty + kDMaxStages;  // [2] bulk copy of a P image
  uint64_t* p_empty = p_full + 2;            // [2] MMA commit
  uint64_t* d_full = p_empty + 2;            // [2] bulk copy of a tile's descriptors
  uint64_t* d_empty = d_full + 2;            // [2] A producer + MMA issuer
  uint64_t* accum_full = d_empty + 2;        // [2] MMA commit at the end of an item
  uint64_t* accum_empty = accum_full + 2;    // [2] the 4 epilogue warps
  uint64_t* mma_done = accum_empty + 2;      // every issued MMA has completed (exit path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t idesc = idesc_f16(128, NR, /*is_bf16=*/!F16, /*a_mn=*/true, /*b_mn=*/false);
  const int item_cols = p.item_groups * 64;
  const int n_pairs = p.item_groups / 2;
  const ItemRange items(p.cta_begin, p.item_order, p.n_items);

  if (tid == 0) {
    for (int i = 0; i < a_stages; ++i) {
      mbar_init(&a_full[i], 1);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], 1);
      mbar_init(&p_empty[i], 1);
      mbar_init(&d_full[i], 1);
      mbar_init(&d_empty[i], 2);
      mbar_init(&accum_full[i], 1);
      mbar_init(&accum_empty[i], 128);
    }
    mbar_init(mma_done, 1);
    // A kernel whose call has already failed does no work (every role sees the flag and skips).
    *abort_flag = status_at_entry(p.status) != 0 ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  auto tile_range = [&](int it, int t, int tb, int& d0, int& d1) {
    const int64_t at = (static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2;
    d0 = p.item_ranges[at];
    d1 = p.item_ranges[at + 1];
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer: P images and descriptors
    if (lane == 0) {
      uint32_t d_iter = 0, p_iter = 0;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        const int it = items.at(k);
        if (it < 0) {
          record_error(p.status, kSiteValueDense + kErrBadDescriptor);
          *abort_flag = 1;
          break;
        }
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2];
        for (int t = tb; t < te && !*abort_flag; ++t) {
          int d0, d1;
          tile_range(it, t, tb, d0, d1);
          const int n = d1 - d0;
          if (n < 0 || n > kDMaxRangeGroups || t < 0 || t >= p.n_tiles) {
            record_error(p.status, kSiteValueDense + kErrBadDescriptor);
            *abort_flag = 1;
            break;
          }
          const int pb = p_iter & 1, db = d_iter & 1;
          if (p_iter >= 2 && !mbar_wait(&p_empty[pb], ((p_iter >> 1) - 1) & 1, p.status, kSiteValueDense + kErrWaitEmpty, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&p_full[pb], p_tile);
          bulk_load(p_tiles + pb * p_tile, p.p_img + static_cast<int64_t>(t) * p_tile, p_tile, &p_full[pb]);
          ++p_iter;
          if (d_iter >= 2 && !mbar_wait(&d_empty[db], ((d_iter >> 1) - 1) & 1, p.status, kSiteValueDense + kErrWaitEmpty, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          if (n > 0) {
            mbar_arrive_expect_tx(&d_full[db], n * 32);
            bulk_load(descs + db * kDMaxRangeGroups, p.groups + d0, n * 32, &d_full[db]);
          } else {
            mbar_arrive(&d_full[db]);
          }
          ++d_iter;
        }
      }
      // Drain: every copy this producer issued has landed before the CTA can leave.
      for (int s = 0; s < 2 && s < static_cast<int>(d_iter); ++s) {
        const uint32_t last = d_iter - 1 - ((d_iter - 1 - s) % 2);
        mbar_wait(&d_full[s], (last / 2) & 1, p.status, kSiteValueDense + kErrWaitDrain);
      }
      for (int s = 0; s < 2 && s < static_cast<int>(p_iter); ++s) {
        const uint32_t last = p_iter - 1 - ((p_iter - 1 - s) % 2);
        mbar_wait(&p_full[s], (last / 2) & 1, p.status, kSiteValueDense + kErrWaitDrain);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ A producer: decoded coefficients by TMA
    if (lane == 0) {
      prefetch_tensormap(&vmap);
      uint32_t a_iter = 0, d_iter = 0;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        const int it = items.at(k);
        if (it < 0) break;  // reported by the descriptor producer
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
        for (int t = tb; t < te && !*abort_flag; ++t) {
          int d0, d1;
          tile_range(it, t, tb, d0, d1);
          const int n = d1 - d0;
          const int db = d_iter & 1;
          if (!mbar_wait(&d_full[db], (d_iter >> 1) & 1, p.status, kSiteValueDense + kErrWaitCodes, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          const GroupDesc* d = descs + db * kDMaxRangeGroups;
          int i = 0, pair;
          bool ok = n >= 0 && n <= kDMaxRangeGroups;
          while (ok && (pair = dense_next_pair(d, n, g0, i)) >= 0) {
            if (pair >= n_pairs || d[i - 1].group < static_cast<uint32_t>(g0)) {  // outside the item's groups
              record_error(p.status, kSiteValueDense + kErrBadDescriptor);
              ok = false;
              break;
            }
            const int st = a_iter % a_stages;
            if (a_iter >= static_cast<uint32_t>(a_stages) &&
                !mbar_wait(&a_empty[st], ((a_iter / a_stages) - 1) & 1, p.status, kSiteValueDense + kErrWaitEmpty, abort_flag)) {
              ok = false;
              break;
            }
            // x: the pair's first component (a multiple of 64 elements, 128 bytes); y: the tile's first row.
            const int x = (g0 + 2 * pair) * kGroup;
            const int y = t * kTileTokens;
            mbar_arrive_expect_tx(&a_full[st], kDPairTile);
            tma_load_2d(a_tiles + st * kDPairTile, &vmap, &a_full[st], x, y);
            tma_load_2d(a_tiles + st * kDPairTile + kDHalf, &vmap, &a_full[st], x + kGroup, y);
            ++a_iter;
          }
          mbar_arrive(&d_empty[db]);  // done reading this tile's descriptors
          ++d_iter;
          if (!ok) {
            *abort_flag = 1;
            break;
          }
        }
      }
      // Drain: every TMA box this producer issued has landed before the CTA can leave.
      for (int s = 0; s < a_stages && s < static_cast<int>(a_iter); ++s) {
        const uint32_t last = a_iter - 1 - ((a_iter - 1 - s) % a_stages);
        mbar_wait(&a_full[s], (last / a_stages) & 1, p.status, kSiteValueDense + kErrWaitDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t a_iter = 0, p_iter = 0, d_iter = 0, item_iter = 0;
      bool issued = false;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        const int it = items.at(k);
        if (it < 0) break;  // reported by the descriptor producer
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
        const uint32_t acc_base = tmem + (item_iter & 1) * kDAccumCols;
        if (item_iter >= 2 &&
            !mbar_wait(&accum_empty[item_iter & 1], ((item_iter >> 1) - 1) & 1, p.status, kSiteValueDense + kErrWaitAccumFree,
                       abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint32_t started = 0;  // pairs whose accumulator has been initialised in this item
        bool ok = true;
        for (int t = tb; t < te && ok; ++t) {
          int d0, d1;
          tile_range(it, t, tb, d0, d1);
          const int n = d1 - d0;
          const int pb = p_iter & 1, db = d_iter & 1;
          if (!mbar_wait(&p_full[pb], (p_iter >> 1) & 1, p.status, kSiteValueDense + kErrWaitA, abort_flag) ||
              !mbar_wait(&d_full[db], (d_iter >> 1) & 1, p.status, kSiteValueDense + kErrWaitCodes, abort_flag)) {
            ok = false;
            break;
          }
          const GroupDesc* d = descs + db * kDMaxRangeGroups;
          const uint32_t p_base = smem_u32(p_tiles + pb * p_tile);
          int i = 0, pair;
          while ((pair = dense_next_pair(d, n, g0, i)) >= 0) {
            if (pair >= n_pairs || d[i - 1].group < static_cast<uint32_t>(g0)) {  // the A producer reports it
              ok = false;
              break;
            }
            const int st = a_iter % a_stages;
            if (!mbar_wait(&a_full[st], (a_iter / a_stages) & 1, p.status, kSiteValueDense + kErrWaitA, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(a_tiles + st * kDPairTile);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              // A: 128 components (two groups, 64 each: LBO = 16 KB between them) x 16 tokens (rows of
              // 128 B, SBO = 1 KB per 8 rows), MN-major. B: P^T, K-major, two atoms of 64 tokens.
              const uint64_t adesc = smem_desc_sw128(a_base + kk * 2048, kDHalf, 1024);
              const uint64_t bdesc = smem_desc_sw128(p_base + (kk >> 2) * (NR * 128) + (kk & 3) * 32, 16, 1024);
              const uint32_t acc = ((started >> pair) & 1u) || kk > 0 ? 1u : 0u;
              mma_f16(acc_base + pair * NR, adesc, bdesc, idesc, acc);
            }
            issued = true;
            started |= 1u << pair;
            mma_commit(&a_empty[st]);
            ++a_iter;
          }
          if (!ok) break;
          mma_commit(&p_empty[pb]);
          mbar_arrive(&d_empty[db]);
          ++p_iter;
          ++d_iter;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mma_commit(&accum_full[item_iter & 1]);
        ++item_iter;
      }
      if (issued) {
        // Every exit: no MMA may still read shared memory or TMEM past this point.
        mma_commit(mma_done);
        mbar_wait(mma_done, 0, p.status, kSiteValueDense + kErrWaitDrain);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue: TMEM -> partial sums
    const int c = (warp & 3) * 32 + lane;  // component within the pair == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t item_iter = 0;
    for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
      const int it = items.at(k);
      if (it < 0) break;  // reported by the descriptor producer
      const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
      // Pairs with a block in some tile of the item (the MMA started exactly those).
      uint32_t live_mask = 0;
      for (int t = tb; t < te; ++t) {
        int d0, d1;
        tile_range(it, t, tb, d0, d1);
        for (int i2 = d0; i2 < d1; ++i2) live_mask |= 1u << ((static_cast<int>(__ldg(&p.groups[i2].group)) - g0) >> 1);
      }
      if (!warp_wait(&accum_full[item_iter & 1], (item_iter >> 1) & 1, p.status, kSiteValueDense + kErrWaitAccum, abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      float* dst = p.partial + static_cast<int64_t>(it) * NR * item_cols;
      for (int pair2 = 0; pair2 < n_pairs; ++pair2) {
        const bool live = (live_mask >> pair2) & 1u;
        for (int n0 = 0; n0 < NR; n0 += 16) {
          uint32_t v[16];
          if (live) {
            tmem_ld16(tmem + (item_iter & 1) * kDAccumCols + lane_base + pair2 * NR + n0, v);
            tmem_ld_wait();
          } else {
#pragma unroll
            for (int i2 = 0; i2 < 16; ++i2) v[i2] = 0u;
          }
#pragma unroll
          for (int i2 = 0; i2 < 16; ++i2)
            dst[static_cast<int64_t>(n0 + i2) * item_cols + pair2 * 128 + c] = __uint_as_float(v[i2]);
        }
      }
      tc_fence_before();
      mbar_arrive(&accum_empty[item_iter & 1]);
      ++item_iter;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

int dense_value_stages(int n_rows_pad) {
  const int fixed = 1024 + 2 * n_rows_pad * 256 + 2 * kDMaxRangeGroups * 32 + 32 * 8 + 16;
  const int stages = (232448 - fixed) / kDPairTile;
  return stages < kDMaxStages ? stages : kDMaxStages;
}

int run_value_dense(const CUtensorMap& vmap, const ValueWeightParams& p, int grid, cudaStream_t stream) {
  if (p.n_rows_pad % 16 != 0 || p.n_rows_pad < 16 || p.n_rows_pad > 128 || p.n_rows > p.n_rows_pad)
    return kDkvErrConfig;
  if ((p.item_groups / 2) * p.n_rows_pad > kDAccumCols || p.item_groups % 2 != 0 || p.item_groups > kDMaxRangeGroups)
    return kDkvErrConfig;
  if (p.p_img == nullptr || p.n_tiles <= 0 || (reinterpret_cast<uintptr_t>(p.p_img) & 15u)) return kDkvErrArgs;
  if (p.n_items == 0) return kDkvOk;
  const int stages = dense_value_stages(p.n_rows_pad);
  if (stages < 2) return kDkvErrConfig;
  const int smem = 1024 + stages * kDPairTile + 2 * p.n_rows_pad * 256 + 2 * kDMaxRangeGroups * 32 + 32 * 8 + 16;
  const int rc = run_vprobs(p, stream);  // P^T images of every value tile for this call's rows
  if (rc != kDkvOk) return rc;
  if (p.f16) {
    if (cudaFuncSetAttribute(value_dense_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return kDkvErrCuda;
    value_dense_kernel<true><<<grid, kDThreads, smem, stream>>>(vmap, p, stages);
  } else {
    if (cudaFuncSetAttribute(value_dense_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return kDkvErrCuda;
    value_dense_kernel<false><<<grid, kDThreads, smem, stream>>>(vmap, p, stages);
  }
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
