// value_weights.cu — attention probabilities applied to value coefficients (values never decoded).
//
// Replaces the per-block value products of CompressedContext.attend
// (scripts/compressed_attention.py:127, 132-133):
//   p_c = softmax(...)[..., :middle].to(dtype)
//   weighted += einsum("bhgqn,nr->bhgqr", p_c[..., block.index], block.coefficients)
// for a batch of conversations. One work item = (conversation, run of value tiles, range of
// union groups). Two sets of 8 worker warps share every tile: they decode alternate pairs of
// coefficient groups (pair ordinal k of a tile goes to set k % 2, into that set's own ring of A
// tiles) into 128-component x 128-token bf16 tiles (MN-major operand: token rows of 64 components,
// 128B swizzle), so two decodes are in flight. The B operand is P^T (rows = query head x query row,
// K = the tile's 128 tokens) in bf16, exactly the reference's rounding of p to the cache dtype,
// 128B-swizzled K-major: with p_img (PIMG) vprobs_kernel builds it once per value tile and call (it is
// the same for every group range of a tile) and a producer fetches it with one bulk copy; without, both
// worker sets build it in shared memory from the fp32 scores and the softmax statistics.
// The MMA warp accumulates D[128 components, rows] += C^T P^T with tcgen05 (M=128, N=rows,
// K=16 tokens per instruction) into one TMEM column range per group pair, inside one of two
// 256-column accumulators that consecutive items alternate between. At the end of an item warps 4, 5,
// 14 and 15 (one per TMEM lane quarter, two from each set) write its accumulator to `partial` (fp32,
// reduced by finalize.cu) while the next item accumulates into the other.
// Producers: warp 19 copies each tile's P image and its descriptors (the host lists, per item and
// tile, the range of descriptors inside the item's groups) into shared memory with bulk copies; every
// role walks the group pairs there; warps 0 and 18 stream the code blocks of set 0's and set 1's pairs
// into one ring of slots each, so a set never waits on a slot the other set still holds.
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {

// Warps: 0 and 18 code producers (one ring per worker set), 1 MMA, 2-9 worker set 0, 10-17 worker set
// 1 (4, 5, 14, 15 also drain the accumulators), 19 P-image / descriptor producer.
constexpr int kVThreads = 640;
constexpr int kPairTile = 32768;  // two groups x 128 tokens x 128 B
constexpr int kMaxRangeGroups = 64;
constexpr int kAccumCols = 256;   // TMEM columns of one item's accumulator (two alternate in the 512)

template <bool RAW>
struct ValueSmem {
  static constexpr int kCodeSlots = RAW ? 2 : 3;  // per worker set
  static constexpr int kCodeSlot = RAW ? 17408 : 8960;
};

// Next group pair of a tile's descriptor list (in shared memory, sorted by union group).
__device__ __forceinline__ int next_pair(const GroupDesc* d, int n, int g0, int& i, int& lo, int& hi) {
  lo = hi = -1;
  if (i >= n) return -1;
  const int g = static_cast<int>(d[i].group);
  const int pair = (g - g0) >> 1;
  if (((g - g0) & 1) == 0) {
    lo = i++;
    if (i < n && static_cast<int>(d[i].group) == g + 1) hi = i++;
  } else {
    hi = i++;
  }
  return pair;
}

}  // namespace

// One CTA per value tile: the tile's P^T image for the call's rows (bf16 probabilities, rounded as the
// reference rounds p to the cache dtype, compressed_attention.py:127), laid out exactly as the MMA's
// B operand sits in shared memory (two atoms of 64 tokens, n_rows_pad rows x 128 B, 128B swizzle),
// built in shared memory and written out whole.
__global__ void __launch_bounds__(256) vprobs_kernel(const ValueWeightParams p) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  extern __shared__ __align__(16) uint8_t img[];  // [2][NR][128]
  const int NR = p.n_rows_pad;
  const int t = blockIdx.x;
  const TileDesc tile = p.tiles[t];
  const bool tile_ok = tile.n_tokens >= 1 && tile.n_tokens <= kTileTokens;
  if (!tile_ok && threadIdx.x == 0) record_error(p.status, kSiteValue + kErrBadDescriptor);
  const int s = tile.seq;
  const int r = threadIdx.x & 127;
  const bool tok_ok = tile_ok && r < tile.n_tokens;
  const int64_t m_s = tile_ok ? p.seq_m[s] : 0;
  const float* sc = p.scores + (tile_ok ? p.seq_score_off[s] : 0);
  const int sidx = tok_ok ? p.tok_sidx[tile.token_base + r] : 0;
  const int atom = r >> 6, chunk = (r & 63) >> 3, within = (r & 7) * 2;
  for (int n = threadIdx.x >> 7; n < NR; n += 2) {
    float prob = 0.f;
    if (tok_ok && n < p.n_rows) {
      const float x = sc[static_cast<int64_t>(p.row_begin + n) * m_s + sidx];
      const float* st = p.row_stats + (static_cast<int64_t>(s) * p.n_q_heads * p.q_len + p.row_begin + n) * 4;
      prob = (x == -INFINITY) ? 0.f : expf(x - st[0]) * st[1];
    }
    *reinterpret_cast<uint16_t*>(img + atom * (NR * 128) + sw128_offset(n, chunk) + within) =
        p.f16 ? float_to_half<true>(prob) : float_to_half<false>(prob);
  }
  __syncthreads();
  uint4* dst = reinterpret_cast<uint4*>(p.p_img + static_cast<int64_t>(t) * NR * 256);
  for (int i = threadIdx.x; i < NR * 16; i += blockDim.x) dst[i] = reinterpret_cast<const uint4*>(img)[i];
}

template <bool RAW, bool PIMG, bool F16>
__global__ void __launch_bounds__(kVThreads, 1) value_weights_kernel(const ValueWeightParams p, int a_slots) {
  using L = ValueSmem<RAW>;
  constexpr int kCodeSlots = L::kCodeSlots;
  constexpr int kCodeSlot = L::kCodeSlot;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NR = p.n_rows_pad;  // MMA N (multiple of 16, <= 128)
  const int p_tile = NR * 256;  // two K atoms of 64 tokens
  uint8_t* a_tiles = smem;                                              // [2 sets][a_slots][kPairTile]
  uint8_t* p_tiles = a_tiles + 2 * a_slots * kPairTile;                 // [2][p_tile]
  GroupDesc* descs = reinterpret_cast<GroupDesc*>(p_tiles + 2 * p_tile);  // [2][kMaxRangeGroups]
  float* stats_s = reinterpret_cast<float*>(descs + 2 * kMaxRangeGroups);  // [3][128][2] max, 1/sum
  uint8_t* c_slots = reinterpret_cast<uint8_t*>(stats_s + 3 * 256);        // [2 sets][kCodeSlots][kCodeSlot]
  uint64_t* bars = reinterpret_cast<uint64_t*>(c_slots + 2 * kCodeSlots * kCodeSlot);
  uint64_t* code_full = bars;                       // [2 sets][kCodeSlots]
  uint64_t* code_empty = code_full + 2 * kCodeSlots;  // [2 sets][kCodeSlots]
  uint64_t* a_full = code_empty + 2 * kCodeSlots;  // [2 sets][2]
  uint64_t* a_empty = a_full + 4;              // [2 sets][2]
  uint64_t* p_full = a_empty + 4;              // [2]
  uint64_t* p_empty = p_full + 2;              // [2]
  uint64_t* d_full = p_empty + 2;              // [2]
  uint64_t* d_empty = d_full + 2;              // [2]
  uint64_t* stats_ready = d_empty + 2;         // [3]
  uint64_t* accum_full = stats_ready + 3;      // [2] TMEM accumulator halves (items alternate)
  uint64_t* accum_empty = accum_full + 2;      // [2]
  uint64_t* mma_done = accum_empty + 2;        // MMA issuer: its MMAs completed (early exit)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t idesc = idesc_f16(128, NR, /*is_bf16=*/!F16, /*a_mn=*/true, /*b_mn=*/false);
  const int item_cols = p.item_groups * 64;
  const int n_pairs = p.item_groups / 2;
  const ItemRange items(p.cta_begin, p.item_order, p.n_items);

  if (tid == 0) {
    for (int i = 0; i < 2 * kCodeSlots; ++i) {
      mbar_init(&code_full[i], 1);
      mbar_init(&code_empty[i], 256);  // the 256 threads of the set that decodes the block
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&a_full[i], 256);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&p_full[i], PIMG ? 1 : 512);  // the producer's bulk copy, or the 512 workers
      mbar_init(&p_empty[i], 1);
      mbar_init(&d_full[i], 1);
      mbar_init(&d_empty[i], 515);  // the 512 workers, the MMA issuer and the two code producers
    }
    for (int i = 0; i < 3; ++i) mbar_init(&stats_ready[i], 512);
    for (int i = 0; i < 2; ++i) {
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

  if (warp == 19) {
    // ------------------------------------------------------------ producer: P images and descriptors
    if (lane == 0) {
      uint32_t d_iter = 0, p_iter = 0;
      const int p_tile = p.n_rows_pad * 256;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        const int it = items.at(k);
        if (it < 0) {
          record_error(p.status, kSiteValue + kErrBadDescriptor);
          *abort_flag = 1;
          break;
        }
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2];
        for (int t = tb; t < te && !*abort_flag; ++t) {
          const int d0 = p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2];
          const int d1 = p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2 + 1];
          const int n = d1 - d0;
          const int db = d_iter & 1;
          if (n < 0 || n > kMaxRangeGroups) {
            record_error(p.status, kSiteValue + kErrBadDescriptor);
            *abort_flag = 1;
            break;
          }
          if (PIMG) {
            if (t < 0 || t >= p.n_tiles) {
              record_error(p.status, kSiteValue + kErrBadDescriptor);
              *abort_flag = 1;
              break;
            }
            const int pb = p_iter & 1;
            if (p_iter >= 2 && !mbar_wait(&p_empty[pb], ((p_iter >> 1) - 1) & 1, p.status, kSiteValue + kErrWaitEmpty, abort_flag)) {
              *abort_flag = 1;
              break;
            }
            mbar_arrive_expect_tx(&p_full[pb], p_tile);
            bulk_load(p_tiles + pb * p_tile, p.p_img + static_cast<int64_t>(t) * p_tile, p_tile, &p_full[pb]);
            ++p_iter;
          }
          if (d_iter >= 2 && !mbar_wait(&d_empty[db], ((d_iter >> 1) - 1) & 1, p.status, kSiteValue + kErrWaitEmpty, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          if (n > 0) {
            mbar_arrive_expect_tx(&d_full[db], n * 32);
            bulk_load(descs + db * kMaxRangeGroups, p.groups + d0, n * 32, &d_full[db]);
          } else {
            mbar_arrive(&d_full[db]);
          }
          ++d_iter;
        }
      }
      // Drain: every copy this producer issued has landed before the CTA can leave.
      for (int s = 0; s < 2 && s < static_cast<int>(d_iter); ++s) {
        const uint32_t last = d_iter - 1 - ((d_iter - 1 - s) % 2);
        mbar_wait(&d_full[s], (last / 2) & 1, p.status, kSiteValue + kErrWaitDrain);
      }
      for (int s = 0; PIMG && s < 2 && s < static_cast<int>(p_iter); ++s) {
        const uint32_t last = p_iter - 1 - ((p_iter - 1 - s) % 2);
        mbar_wait(&p_full[s], (last / 2) & 1, p.status, kSiteValue + kErrWaitDrain);
      }
    }
  } else if (warp == 0 || warp == 18) {
    // ------------------------------------------------------------ producers: code blocks of one worker set
    // Warp 0 streams the blocks of the pairs set 0 decodes (even ordinals of a tile) into ring 0, warp 18
    // those of set 1 into ring 1, so neither set waits on a slot the other still holds.
    if (lane == 0) {
      const int ring = warp == 18 ? 1 : 0;
      uint8_t* slots = c_slots + ring * kCodeSlots * kCodeSlot;
      uint64_t* r_full = code_full + ring * kCodeSlots;
      uint64_t* r_empty = code_empty + ring * kCodeSlots;
      uint32_t c_iter = 0, d_iter = 0;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        const int it = items.at(k);
        if (it < 0) {
          record_error(p.status, kSiteValue + kErrBadDescriptor);
          *abort_flag = 1;
          break;
        }
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
        for (int t = tb; t < te && !*abort_flag; ++t) {
          const int n = p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2 + 1] -
                        p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2];
          const int db = d_iter & 1;
          if (!mbar_wait(&d_full[db], (d_iter >> 1) & 1, p.status, kSiteValue + kErrWaitCodes, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          const GroupDesc* d = descs + db * kMaxRangeGroups;
          int i = 0, lo, hi, pair, ord = 0;
          bool ok = n >= 0 && n <= kMaxRangeGroups;
          while (ok && (pair = next_pair(d, n, g0, i, lo, hi)) >= 0) {
            if ((ord++ & 1) != ring) continue;
            for (int half = 0; half < 2 && ok; ++half) {
              const int gi = half ? hi : lo;
              if (gi < 0) continue;
              const uint32_t off = d[gi].code_offset, bytes = d[gi].code_bytes;
              if (bytes > static_cast<uint32_t>(kCodeSlot) || static_cast<uint64_t>(off) + bytes > p.code_size) {
                record_error(p.status, kSiteValue + kErrBadDescriptor);
                ok = false;
                break;
              }
              const int cs = c_iter % kCodeSlots;
              if (c_iter >= kCodeSlots &&
                  !mbar_wait(&r_empty[cs], ((c_iter / kCodeSlots) - 1) & 1, p.status, kSiteValue + kErrWaitEmpty, abort_flag)) {
                ok = false;
                break;
              }
              mbar_arrive_expect_tx(&r_full[cs], bytes);
              bulk_load(slots + cs * kCodeSlot, p.code + off, bytes, &r_full[cs]);
              ++c_iter;
            }
          }
          mbar_arrive(&d_empty[db]);  // done reading this tile's descriptors
          ++d_iter;
          if (!ok) {
            *abort_flag = 1;
            break;
          }
        }
      }
      // Drain: every copy this producer issued has landed before the CTA can leave.
      for (int s = 0; s < kCodeSlots && s < static_cast<int>(c_iter); ++s) {
        const uint32_t last = c_iter - 1 - ((c_iter - 1 - s) % kCodeSlots);
        mbar_wait(&r_full[s], (last / kCodeSlots) & 1, p.status, kSiteValue + kErrWaitDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t a_iter[2] = {0, 0};
      uint32_t p_iter = 0, d_iter = 0, item_iter = 0;
      bool issued = false;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        const int it = items.at(k);
        if (it < 0) {
          record_error(p.status, kSiteValue + kErrBadDescriptor);
          *abort_flag = 1;
          break;
        }
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
        // Two accumulators of kAccumCols columns: item i uses half i % 2, so the epilogue of an item
        // drains one half while the next item accumulates into the other.
        const uint32_t acc_base = tmem + (item_iter & 1) * kAccumCols;
        if (item_iter >= 2 &&
            !mbar_wait(&accum_empty[item_iter & 1], ((item_iter >> 1) - 1) & 1, p.status, kSiteValue + kErrWaitAccumFree, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint32_t started = 0;  // pairs whose accumulator has been initialised in this item
        bool ok = true;
        for (int t = tb; t < te && ok; ++t) {
          const int pb = p_iter & 1, db = d_iter & 1;
          const int n = p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2 + 1] -
                        p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2];
          if (!mbar_wait(&p_full[pb], (p_iter >> 1) & 1, p.status, kSiteValue + kErrWaitA, abort_flag) ||
              !mbar_wait(&d_full[db], (d_iter >> 1) & 1, p.status, kSiteValue + kErrWaitCodes, abort_flag)) {
            ok = false;
            break;
          }
          const GroupDesc* d = descs + db * kMaxRangeGroups;
          int i = 0, lo, hi, pair, ord = 0;
          while ((pair = next_pair(d, n, g0, i, lo, hi)) >= 0) {
            const int set = ord & 1;
            const int slot = a_iter[set] % a_slots;
            if (!mbar_wait(&a_full[set * 2 + slot], (a_iter[set] / a_slots) & 1, p.status, kSiteValue + kErrWaitA, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(a_tiles + (set * a_slots + slot) * kPairTile);
            const uint32_t p_base = smem_u32(p_tiles + pb * p_tile);
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {
              const uint64_t adesc = smem_desc_sw128(a_base + kk * 2048, 16384, 1024);
              const uint64_t bdesc = smem_desc_sw128(p_base + (kk >> 2) * (NR * 128) + (kk & 3) * 32, 16, 1024);
              const uint32_t acc = ((started >> pair) & 1u) || kk > 0 ? 1u : 0u;
              mma_f16(acc_base + pair * NR, adesc, bdesc, idesc, acc);
            }
            issued = true;
            started |= 1u << pair;
            mma_commit(&a_empty[set * 2 + slot]);
            ++a_iter[set];
            ++ord;
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
        // Every exit (also one where the epilogue gave up): no MMA may still read shared memory or TMEM
        // past this point.
        mma_commit(mma_done);
        mbar_wait(mma_done, 0, p.status, kSiteValue + kErrWaitDrain);
      }
    }
  } else {
    // ------------------------------------------------------------ worker sets (P, decode; warps 4-7 epilogue)
    const int set = warp >= 10 ? 1 : 0;
    const int u = tid - (set ? 320 : 64);  // 0..255 within the set
    const int w = tid - 64;                // 0..511 over both sets
    const int r = u & 127;                 // token row (decode) / token column (P)
    const int h = u >> 7;                  // component half (decode) / row quarter within the set's half (P)
    uint32_t c_iter = 0, a_iter = 0, p_iter = 0, d_iter = 0, item_iter = 0;
    for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
      const int it = items.at(k);
      if (it < 0) {
        record_error(p.status, kSiteValue + kErrBadDescriptor);
        *abort_flag = 1;
        break;
      }
      const int s = p.items[4 * it], tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
      const int64_t m_s = p.seq_m[s];
      const float* sc = p.scores + p.seq_score_off[s];
      // Softmax statistics of the item's rows, staged once per item in one of three buffers: a worker
      // can be at most two items ahead of the slowest one (each P tile waits for the MMA of the tile
      // two before it, which waits for every worker), so three buffers never collide.
      float* st_s = stats_s + (item_iter % 3) * 256;
      if (!PIMG) {
      if (w < NR) {
        float mx = 0.f, inv = 0.f;
        if (w < p.n_rows) {
          const float* st = p.row_stats + (static_cast<int64_t>(s) * p.n_q_heads * p.q_len + p.row_begin + w) * 4;
          mx = st[0];
          inv = st[1];
        }
        st_s[2 * w] = mx;
        st_s[2 * w + 1] = inv;
      }
      mbar_arrive(&stats_ready[item_iter % 3]);
      if (!warp_wait(&stats_ready[item_iter % 3], (item_iter / 3) & 1, p.status, kSiteValue + kErrWaitA, abort_flag)) {
        *abort_flag = 1;
        break;
      }
      }
      for (int t = tb; t < te && !*abort_flag; ++t) {
        const TileDesc tile = p.tiles[t];
        // ---- P^T tile: rows x 128 tokens, bf16 (the reference rounds p to the cache dtype); set s builds
        //      rows [s*NR/2, (s+1)*NR/2), thread half h a quarter of them.
        const int pb = p_iter & 1;
        if (!PIMG && p_iter >= 2 && !warp_wait(&p_empty[pb], ((p_iter >> 1) - 1) & 1, p.status, kSiteValue + kErrWaitEmpty, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        if (!PIMG) {
          uint8_t* pt = p_tiles + pb * p_tile;
          const bool tok_ok = r < tile.n_tokens;
          const int sidx = tok_ok ? p.tok_sidx[tile.token_base + r] : 0;
          const int atom = r >> 6, chunk = (r & 63) >> 3, within = (r & 7) * 2;
          const int quarter = NR / 4;
          const int rb = set * (NR / 2) + h * quarter;
          for (int n0 = rb; n0 < rb + quarter; n0 += 4) {
            float x[4];
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int n = n0 + kk;
              x[kk] = (tok_ok && n < p.n_rows) ? sc[static_cast<int64_t>(p.row_begin + n) * m_s + sidx] : -INFINITY;
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const int n = n0 + kk;
              const float prob = (x[kk] == -INFINITY) ? 0.f : expf(x[kk] - st_s[2 * n]) * st_s[2 * n + 1];
              *reinterpret_cast<uint16_t*>(pt + atom * (NR * 128) + sw128_offset(n, chunk) + within) =
                  float_to_half<F16>(prob);
            }
          }
          fence_async_shared();
          mbar_arrive(&p_full[pb]);
          ++p_iter;
        }
        // ---- coefficient pairs: this set takes the pairs of its ordinal parity
        const int db = d_iter & 1;
        const int n = p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2 + 1] -
                      p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2];
        if (!warp_wait(&d_full[db], (d_iter >> 1) & 1, p.status, kSiteValue + kErrWaitCodes, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        const GroupDesc* d = descs + db * kMaxRangeGroups;
        int i = 0, lo, hi, pair, ord = 0;
        while ((pair = next_pair(d, n, g0, i, lo, hi)) >= 0) {
          if ((ord & 1) != set) {  // the other set's pair (its blocks are in the other ring)
            ++ord;
            continue;
          }
          const int slot = a_iter % a_slots;
          if (a_iter >= static_cast<uint32_t>(a_slots) &&
              !warp_wait(&a_empty[set * 2 + slot], ((a_iter / a_slots) - 1) & 1, p.status, kSiteValue + kErrWaitEmpty, abort_flag)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* a = a_tiles + (set * a_slots + slot) * kPairTile;
          for (int half = 0; half < 2; ++half) {
            const int gi = half ? hi : lo;
            uint8_t* dst = a + half * 16384;
            uint32_t out[16];
            if (gi >= 0) {
              const int cs = set * kCodeSlots + c_iter % kCodeSlots;  // this set's ring
              if (!warp_wait(&code_full[cs], (c_iter / kCodeSlots) & 1, p.status, kSiteValue + kErrWaitCodes, abort_flag)) {
                *abort_flag = 1;
                break;
              }
              const uint4* dw = reinterpret_cast<const uint4*>(d + gi);
              const GroupRegs gr = group_from_words(dw[0], dw[1]);
              decode_half<F16>(c_slots + cs * kCodeSlot, gr, tile.n_tokens, r, h, out);
              mbar_arrive(&code_empty[cs]);
              ++c_iter;
            } else {
#pragma unroll
              for (int kk = 0; kk < 16; ++kk) out[kk] = 0u;
            }
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              *reinterpret_cast<uint4*>(dst + sw128_offset(r, 4 * h + kk)) =
                  make_uint4(out[4 * kk], out[4 * kk + 1], out[4 * kk + 2], out[4 * kk + 3]);
          }
          if (*abort_flag) break;
          fence_async_shared();
          mbar_arrive(&a_full[set * 2 + slot]);
          ++a_iter;
          ++ord;
        }
        mbar_arrive(&d_empty[db]);
        ++d_iter;
      }
      if (*abort_flag) break;
      // ---- epilogue (warps 4..7, one per TMEM lane quarter): TMEM -> partial sums
      if (warp == 4 || warp == 5 || warp == 14 || warp == 15) {
        if (!warp_wait(&accum_full[item_iter & 1], (item_iter >> 1) & 1, p.status, kSiteValue + kErrWaitAccum, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const int c = (warp & 3) * 32 + lane;  // component within the pair == TMEM lane (quarter warp % 4)
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        float* dst = p.partial + static_cast<int64_t>(it) * NR * item_cols;
        // Pairs started by either set: the MMA started every pair that has a block in the item.
        uint32_t live_mask = 0;
        for (int t = tb; t < te; ++t) {
          const int d0 = p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2];
          const int d1 = p.item_ranges[(static_cast<int64_t>(it) * p.tile_chunk + (t - tb)) * 2 + 1];
          for (int i2 = d0; i2 < d1; ++i2) live_mask |= 1u << ((static_cast<int>(__ldg(&p.groups[i2].group)) - g0) >> 1);
        }
        for (int pair2 = 0; pair2 < n_pairs; ++pair2) {
          const bool live = (live_mask >> pair2) & 1u;
          for (int n0 = 0; n0 < NR; n0 += 16) {
            uint32_t v[16];
            if (live) {
              tmem_ld16(tmem + (item_iter & 1) * kAccumCols + lane_base + pair2 * NR + n0, v);
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
      }
      ++item_iter;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

template <bool RAW, bool PIMG, bool F16>
static int launch_vw3(const ValueWeightParams& p, int grid, int smem, int a_slots, cudaStream_t stream) {
  if (cudaFuncSetAttribute(value_weights_kernel<RAW, PIMG, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return kDkvErrCuda;
  value_weights_kernel<RAW, PIMG, F16><<<grid, kVThreads, smem, stream>>>(p, a_slots);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

template <bool RAW, bool PIMG>
static int launch_vw(const ValueWeightParams& p, int grid, int smem, int a_slots, cudaStream_t stream) {
  return p.f16 ? launch_vw3<RAW, PIMG, true>(p, grid, smem, a_slots, stream)
               : launch_vw3<RAW, PIMG, false>(p, grid, smem, a_slots, stream);
}

int run_vprobs(const ValueWeightParams& p, cudaStream_t stream) {
  if (p.n_tiles <= 0 || p.p_img == nullptr || (reinterpret_cast<uintptr_t>(p.p_img) & 15u)) return kDkvErrArgs;
  vprobs_kernel<<<p.n_tiles, 256, p.n_rows_pad * 256, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

int run_value_weights(const ValueWeightParams& p, int grid, cudaStream_t stream) {
  if (p.n_rows_pad % 16 != 0 || p.n_rows_pad < 16 || p.n_rows_pad > 128 || p.n_rows > p.n_rows_pad)
    return kDkvErrConfig;
  if ((p.item_groups / 2) * p.n_rows_pad > kAccumCols || p.item_groups % 2 != 0 || p.item_groups > kMaxRangeGroups)
    return kDkvErrConfig;
  if (p.n_items == 0) return kDkvOk;
  const bool raw = p.max_planes > 8;
  const int slots = 2 * (raw ? ValueSmem<true>::kCodeSlots * ValueSmem<true>::kCodeSlot
                             : ValueSmem<false>::kCodeSlots * ValueSmem<false>::kCodeSlot);
  const int a_slots = p.n_rows_pad > 64 ? 1 : 2;  // two A tiles per set where the P tiles leave room
  const int smem = 1024 + 2 * a_slots * kPairTile + 2 * p.n_rows_pad * 256 + 2 * kMaxRangeGroups * 32 + 3 * 256 * 4 +
                   slots + 48 * 8;
  if (smem > 232448) return kDkvErrConfig;
  if (p.p_img != nullptr) {
    // P^T images of every value tile for this call's rows, then the weighting that fetches them.
    const int rc = run_vprobs(p, stream);
    if (rc != kDkvOk) return rc;
    return raw ? launch_vw<true, true>(p, grid, smem, a_slots, stream) : launch_vw<false, true>(p, grid, smem, a_slots, stream);
  }
  return raw ? launch_vw<true, false>(p, grid, smem, a_slots, stream) : launch_vw<false, false>(p, grid, smem, a_slots, stream);
}

}  // namespace dkv
