// key_scores_dense.cu — key rebuild + RoPE + q.k over key coefficients that were decoded once per decode
// step, both tcgen05 operands streamed by TMA (CTA pairs, cta_group::2).
//
// Replaces, like key_scores_pair.cu, CompressedContext._keys + the score product of attend
// (scripts/compressed_attention.py:105-111, 118-122):
//   keys = rerotate(block["coefficients"] @ basis[layer] + mean[layer], cos, sin)
//   scores = query @ keys^T * scaling
// The key coefficients are the same for every layer (one cross-layer basis, compressed_attention.py:
// 105-111 use block["coefficients"] for every layer), so dkv_unpack decodes the key planes once per step
// into a tile-padded 16-bit buffer (key tile t's tokens at rows t * 128 .., column = union group * 64 +
// component, zeros for groups the tile does not hold) and every layer's rebuild reads that buffer with
// TMA instead of decoding the planes again in the kernel.
//
// Work items and schedule are the CTA-pair kernel's: a pair of key tiles (one per CTA of a cluster of
// two) x 512 key columns, its groups the sorted union of the two tiles' groups. Per merged group each CTA
// loads one stage: its tile's 128 x 64 coefficient box (A, 16 KB) and 128 of each pair MMA's 256 basis
// rows (B, 2 x 16 KB). The even CTA issues M = 256 (128 rows of each CTA) x N = 256 pair MMAs, two per
// K step, into a 512-column fp32 accumulator per CTA. Roles (384 threads, 168 registers each, no register
// reallocation):
//   warp 0      producer: A and B boxes of every merged group into a ring of stages (TMA, no multicast)
//   warp 1      even CTA: pair MMA issuer; odd CTA: forwards its stage completions to the even CTA
//   warps 4-11  epilogue, two warps per TMEM lane quarter (warp % 4), each half of every head's RoPE pairs:
//               TMEM -> + mean -> RoPE -> q.k for each head's query group (packed fp32x2 arithmetic), the
//               two halves' products added through shared memory -> fp32 scores
// Every wait is bounded and abort-aware (dkv_ptx.cuh); the abort flag is cluster-wide; the kernel does
// no work when the call's status word is already set.
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {

// Epilogue: 8 warps, two per TMEM lane quarter. The two warps of a quarter split every head's RoPE pairs (so
// each token's cos / sin words are loaded by one warp, not two), take all of the item's heads, load two heads'
// TMEM columns before one wait, and add their partial q.k products through shared memory.
constexpr int kKdEpilogueWarps = 8;
constexpr int kKdEpilogueThreads = kKdEpilogueWarps * 32;
constexpr int kKdThreads = 128 + kKdEpilogueThreads;
constexpr int kKdCols = 512;                 // key columns per item (one 512-column TMEM accumulator)
constexpr int kKdMmaN = 256;                 // N of one pair MMA (two per K step)
constexpr int kKdHalfCols = 128;             // basis rows of one pair MMA loaded by each CTA
constexpr int kKdA = 16384;                  // 128 token rows x 64 components x 16 bit (128B swizzle)
constexpr int kKdBHalf = kKdHalfCols * 128;  // 128 basis rows x 64 components x 16 bit
constexpr int kKdStage = kKdA + 2 * kKdBHalf;
constexpr int kKdStages = 4;

}  // namespace

template <int D, int G, bool F16>
__global__ void __launch_bounds__(kKdThreads, 1)
    key_scores_dense_kernel(const __grid_constant__ CUtensorMap bmap, const __grid_constant__ CUtensorMap amap,
                            const KeyScoreParams p) {
  constexpr int kHeads = kKdCols / D;        // KV heads per item
  constexpr int kPairSpan = D / 4;           // RoPE pair dims of one warp's part: half of each head's D / 2
  constexpr int kLoadHeads = 2;              // heads whose TMEM columns one wait covers
  constexpr uint32_t kIdesc = idesc_f16(256, kKdMmaN, /*is_bf16=*/!F16, false, false);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* stages = smem;                                                // [kKdStages][A | B half 0 | B half 1]
  float* q_s = reinterpret_cast<float*>(smem + kKdStages * kKdStage);   // [kHeads * G][D]
  float* mean_s = q_s + kHeads * G * D;                                  // [kKdCols]
  float* red_s = mean_s + kKdCols;                                       // [kHeads][G][128] second parts' q.k
  uint64_t* bars = reinterpret_cast<uint64_t*>(red_s + kHeads * G * 128);
  uint64_t* full = bars;                       // [kKdStages] this CTA's A and B boxes (TMA)
  uint64_t* peer_full = full + kKdStages;      // [kKdStages] even CTA: the odd CTA's forward
  uint64_t* empty = peer_full + kKdStages;     // [kKdStages] pair-MMA commit (both CTAs)
  uint64_t* accum_full = empty + kKdStages;    // pair-MMA commit at the end of an item
  uint64_t* accum_empty = accum_full + 1;      // even CTA: 2 x 16 epilogue warp arrivals
  uint64_t* mma_done = accum_empty + 1;        // even CTA: every issued pair MMA has completed
  uint64_t* ep_sync = mma_done + 1;            // [2] epilogue rendezvous (512 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ep_sync + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int nblocks = p.n_cols / kKdCols;
  // Cluster c processes list c of the schedule.
  const ItemRange items(p.cta_begin, p.item_order, p.n_items, blockIdx.x >> 1, gridDim.x >> 1);

  if (tid == 0) {
    for (int i = 0; i < kKdStages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&peer_full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(accum_empty, 2 * kKdEpilogueWarps);
    mbar_init(mma_done, 1);
    mbar_init(&ep_sync[0], kKdEpilogueThreads);
    mbar_init(&ep_sync[1], kKdEpilogueThreads);
    // A kernel whose call has already failed does no work (every role sees the flag and skips).
    *abort_flag = status_at_entry(p.status) != 0 ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kKdCols);
  __syncthreads();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t peer_full_lead = mapa_shared(smem_u32(peer_full), 0);
  const uint32_t accum_empty_lead = mapa_shared(smem_u32(accum_empty), 0);
  // Cluster-wide abort: a role that gives up sets the flag in both CTAs (its own and, through
  // st.shared::cluster, the peer's); both CTAs stay resident until the final cluster barrier.
  auto give_up = [abort_flag]() {
    *abort_flag = 1;
    st_cluster_u32(mapa_shared(smem_u32(const_cast<int*>(abort_flag)), cluster_ctarank() ^ 1u), 1u);
  };
  if (tid == 0 && *abort_flag) give_up();  // the entry check of either CTA stops both

  // The item of schedule position k: (pair, column block, merged groups, first entry), or false.
  auto item_at = [&](int k, int& pair, int& nblk, int& n_merged, int& first) -> bool {
    const int it = items.at(k);
    if (it < 0) return false;
    const int code = p.items[it];
    pair = code / nblocks;
    nblk = code % nblocks;
    const int4 pr = __ldg(reinterpret_cast<const int4*>(p.pairs) + pair);
    n_merged = pr.z;
    first = pr.w;
    return true;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer: A and B boxes per merged group
    if (lane == 0) {
      prefetch_tensormap(&bmap);
      prefetch_tensormap(&amap);
      uint32_t s_iter = 0;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        int pair, nblk, n_merged, first;
        if (!item_at(k, pair, nblk, n_merged, first)) {
          record_error(p.status, kSiteKeyDense + kErrBadDescriptor);
          give_up();
          break;
        }
        if (n_merged <= 0) continue;  // nothing to accumulate: the epilogue writes the mean-only keys
        const int ti = p.pairs[4 * pair + rank];
        if (ti >= p.n_tiles) {
          record_error(p.status, kSiteKeyDense + kErrBadDescriptor);
          give_up();
          break;
        }
        bool ok = true;
        for (int gi = 0; gi < n_merged; ++gi) {
          const uint32_t g = static_cast<uint32_t>(__ldg(p.pair_groups + 4 * (first + gi)));
          if (g >= p.n_union_groups) {
            record_error(p.status, kSiteKeyDense + kErrBadDescriptor);
            ok = false;
            break;
          }
          const int s = s_iter % kKdStages;
          if (s_iter >= kKdStages &&
              !mbar_wait(&empty[s], ((s_iter / kKdStages) - 1) & 1, p.status, kSiteKeyDense + kErrWaitEmpty, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = stages + s * kKdStage;
          // A: this CTA's tile, 128 rows of the group's 64 components (zeros where the tile lacks the group).
          // A CTA without a tile (the odd one of a single-tile pair) loads no A: its accumulator rows are
          // never read.
          mbar_arrive_expect_tx(&full[s], (ti >= 0 ? kKdA : 0) + 2 * kKdBHalf);
          if (ti >= 0) tma_load_2d(st, &amap, &full[s], static_cast<int>(g) * kGroup, ti * kTileTokens);
#pragma unroll
          for (int hf = 0; hf < 2; ++hf)
            tma_load_2d(st + kKdA + hf * kKdBHalf, &bmap, &full[s], static_cast<int>(g) * kGroup,
                        p.layer * p.n_cols + nblk * kKdCols + hf * kKdMmaN + rank * kKdHalfCols);
          ++s_iter;
        }
        if (!ok) {
          give_up();
          break;
        }
      }
      // Drain: every box this CTA issued has landed before the CTA can leave.
      for (int s = 0; s < kKdStages && s < static_cast<int>(s_iter); ++s) {
        const uint32_t last = s_iter - 1 - ((s_iter - 1 - s) % kKdStages);
        mbar_wait(&full[s], (last / kKdStages) & 1, p.status, kSiteKeyDense + kErrWaitDrain);
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------------------------------------------------- pair MMA issuer (even CTA)
      if (lane == 0) {
        uint32_t s_iter = 0, item_iter = 0;
        for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
          int pair, nblk, n_merged, first;
          if (!item_at(k, pair, nblk, n_merged, first)) break;  // reported by the producer
          if (n_merged <= 0) continue;
          if (item_iter >= 1 &&
              !mbar_wait(accum_empty, (item_iter - 1) & 1, p.status, kSiteKeyDense + kErrWaitAccumFree, abort_flag)) {
            give_up();
            break;
          }
          tc_fence_after();
          bool ok = true;
          for (int gi = 0; gi < n_merged; ++gi) {
            const int s = s_iter % kKdStages;
            const uint32_t par = (s_iter / kKdStages) & 1;
            if (!mbar_wait(&full[s], par, p.status, kSiteKeyDense + kErrWaitA, abort_flag) ||
                !mbar_wait(&peer_full[s], par, p.status, kSiteKeyDense + kErrWaitBasis, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(stages + s * kKdStage);
            const uint32_t b_base = a_base + kKdA;
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t adesc = smem_desc_sw128(a_base + 32 * kk, 16, 1024);
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const uint64_t bdesc = smem_desc_sw128(b_base + hf * kKdBHalf + 32 * kk, 16, 1024);
                mma_f16_pair(tmem + hf * kKdMmaN, adesc, bdesc, kIdesc, (gi > 0 || kk > 0) ? 1u : 0u);
              }
            }
            mma_commit_pair(&empty[s], 0x3);
            ++s_iter;
          }
          if (!ok) {
            give_up();
            break;
          }
          mma_commit_pair(accum_full, 0x3);
          ++item_iter;
        }
        // Also on an early exit: no pair MMA may still read shared memory or TMEM past this point.
        if (s_iter > 0) {
          mma_commit_pair(mma_done, 0x1);
          mbar_wait(mma_done, 0, p.status, kSiteKeyDense + kErrWaitDrain);
        }
      }
    } else {
      // ---------------------------------------------------------- stage forwarder (odd CTA)
      if (lane == 0) {
        uint32_t s_iter = 0;
        for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
          int pair, nblk, n_merged, first;
          if (!item_at(k, pair, nblk, n_merged, first)) break;  // reported by the producer
          bool ok = true;
          for (int gi = 0; gi < n_merged; ++gi) {
            const int s = s_iter % kKdStages;
            if (!mbar_wait(&full[s], (s_iter / kKdStages) & 1, p.status, kSiteKeyDense + kErrWaitBasis, abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_cluster(peer_full_lead + s * 8);
            ++s_iter;
          }
          if (!ok) {
            give_up();
            break;
          }
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue warps
    // Warp w reads TMEM lane quarter w % 4 (the tile rows 32 (w % 4) ..); warps 4..7 take the first half of
    // every head's RoPE pairs (dims [0, D / 4) and [D / 2, 3 D / 4)), warps 8..11 the second half.
    const int r = (warp & 3) * 32 + lane;  // TMEM lane == tile token row
    const int et = tid - 128;              // 0..511 within the epilogue group
    const int part = (warp - 4) >> 2;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t item_iter = 0, n_sync = 0;
    bool failed = false;
    for (int k = items.k; k < items.end && !*abort_flag && !failed; k += items.step) {
      int pair, nblk, n_merged, first;
      if (!item_at(k, pair, nblk, n_merged, first)) break;  // reported by the producer
      const int ti = p.pairs[4 * pair + rank];
      const bool accumulated = n_merged > 0;
      // The token's RoPE row is located before waiting for the accumulator.
      const bool has_tile = ti >= 0 && ti < p.n_tiles;
      const TileDesc tile = has_tile ? p.tiles[ti] : TileDesc{};
      const bool valid = has_tile && r < tile.n_tokens;
      int pos = valid ? p.tok_pos[tile.token_base + r] : 0;
      const bool hidden = pos < 0;  // refined or evicted token: excluded from the softmax
      pos = hidden ? 0 : (pos >= p.max_pos ? p.max_pos - 1 : pos);
      const uint16_t* cosrow = reinterpret_cast<const uint16_t*>(p.cos_t) + static_cast<int64_t>(pos) * (D / 2);
      const uint16_t* sinrow = reinterpret_cast<const uint16_t*>(p.sin_t) + static_cast<int64_t>(pos) * (D / 2);
      // The accumulator is waited for as late as possible: the first query row's q and mean loads (and the
      // RoPE rows' way into L1) happen while the item's MMAs still run.
      auto wait_accum = [&]() -> bool {
        if (!warp_wait(accum_full, item_iter & 1, p.status, kSiteKeyDense + kErrWaitAccum, abort_flag)) return false;
        tc_fence_after();
        return true;
      };
      if (accumulated && !has_tile && !wait_accum()) {
        give_up();
        break;
      }
      if (has_tile) {
        prefetch_l1(cosrow);
        prefetch_l1(sinrow);
        const int s = tile.seq;
        const int64_t m_s = p.seq_m[s];
        float* out_base = p.scores + p.seq_score_off[s];
        const int kv0 = nblk * kHeads;
        for (int qi = 0; qi < p.q_len; ++qi) {
          if (!group_sync(ep_sync, n_sync, p.status, kSiteKeyDense + kErrWaitAccum, abort_flag)) {
            give_up();
            failed = true;
            break;
          }
          for (int i = et; i < kHeads * G * D; i += kKdEpilogueThreads) {
            const int hq = kv0 * G + i / D;
            const int d = i % D;
            q_s[i] = half_to_float<F16>(reinterpret_cast<const uint16_t*>(
                p.query)[((static_cast<int64_t>(s) * p.n_q_heads + hq) * p.q_len + qi) * D + d]);
          }
          if (qi == 0) {
            const uint16_t* mrow = reinterpret_cast<const uint16_t*>(p.mean) + static_cast<int64_t>(s) * p.mean_seq_stride +
                                   static_cast<int64_t>(p.layer) * p.n_cols + nblk * kKdCols;
            for (int i = et; i < kKdCols; i += kKdEpilogueThreads) mean_s[i] = half_to_float<F16>(mrow[i]);
          }
          if (!group_sync(ep_sync, n_sync, p.status, kSiteKeyDense + kErrWaitAccum, abort_flag) ||
              (qi == 0 && accumulated && !wait_accum())) {
            give_up();
            failed = true;
            break;
          }
          float acc[kHeads][G];
#pragma unroll
          for (int e = 0; e < kHeads; ++e)
#pragma unroll
            for (int j = 0; j < G; ++j) acc[e][j] = 0.f;
#pragma unroll 1
          for (int c = part * kPairSpan; c < (part + 1) * kPairSpan; c += 16) {
            // The token's cos / sin for these 16 dims (8 pairs of 16-bit values), shared by the warp's heads.
            const uint4* cp = reinterpret_cast<const uint4*>(cosrow + c);
            const uint4* sp = reinterpret_cast<const uint4*>(sinrow + c);
            const uint4 c0 = __ldg(cp), c1 = __ldg(cp + 1), s0 = __ldg(sp), s1 = __ldg(sp + 1);
            const uint32_t cbv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
            const uint32_t sbv[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
#pragma unroll
            for (int hp = 0; hp < kHeads; hp += kLoadHeads) {
              uint32_t xs1[kLoadHeads][16], xs2[kLoadHeads][16];
              if (accumulated) {
#pragma unroll
                for (int e = 0; e < kLoadHeads; ++e) {
                  tmem_ld16(tmem + lane_base + (hp + e) * D + c, xs1[e]);
                  tmem_ld16(tmem + lane_base + (hp + e) * D + D / 2 + c, xs2[e]);
                }
                tmem_ld_wait();
#pragma unroll
                for (int e = 0; e < kLoadHeads; ++e) {
                  tmem_reg_fence(xs1[e]);
                  tmem_reg_fence(xs2[e]);
                }
              } else {
#pragma unroll
                for (int e = 0; e < kLoadHeads; ++e)
#pragma unroll
                  for (int i = 0; i < 16; ++i) xs1[e][i] = xs2[e][i] = 0u;
              }
#pragma unroll
            for (int e = hp; e < hp + kLoadHeads; ++e) {
              const int hh = e;
              uint32_t* x1 = xs1[e - hp];
              uint32_t* x2 = xs2[e - hp];
              // Pairs of dims (c + 2k, c + 2k + 1) in packed fp32x2 arithmetic: + mean, RoPE, q.k.
              const ulonglong2* m1 = reinterpret_cast<const ulonglong2*>(mean_s + hh * D + c);
              const ulonglong2* m2 = reinterpret_cast<const ulonglong2*>(mean_s + hh * D + D / 2 + c);
              uint64_t r1[8], r2[8];
#pragma unroll
              for (int k2 = 0; k2 < 8; k2 += 2) {
                const ulonglong2 ma = m1[k2 / 2], mb = m2[k2 / 2];
#pragma unroll
                for (int u = 0; u < 2; ++u) {
                  const int k = k2 + u;
                  const float2 cf = half2_to_float2<F16>(cbv[k]);
                  const float2 sf = half2_to_float2<F16>(sbv[k]);
                  const uint64_t cc = f32x2_pack(__float_as_uint(cf.x), __float_as_uint(cf.y));
                  const uint64_t ss = f32x2_pack(__float_as_uint(sf.x), __float_as_uint(sf.y));
                  const uint64_t ns = ss ^ 0x8000000080000000ull;  // -sin, both lanes
                  const uint64_t k1 = add_f32x2(f32x2_pack(x1[2 * k], x1[2 * k + 1]), u ? ma.y : ma.x);
                  const uint64_t kb = add_f32x2(f32x2_pack(x2[2 * k], x2[2 * k + 1]), u ? mb.y : mb.x);
                  r1[k] = fma_f32x2(k1, cc, mul_f32x2(kb, ns));  // k1 cos - k2 sin
                  r2[k] = fma_f32x2(kb, cc, mul_f32x2(k1, ss));  // k2 cos + k1 sin
                }
              }
#pragma unroll
              for (int j = 0; j < G; ++j) {
                const ulonglong2* q1 = reinterpret_cast<const ulonglong2*>(q_s + (hh * G + j) * D + c);
                const ulonglong2* q2 = reinterpret_cast<const ulonglong2*>(q_s + (hh * G + j) * D + D / 2 + c);
                uint64_t a2 = 0ull;  // (+0.0, +0.0)
#pragma unroll
                for (int k2 = 0; k2 < 8; k2 += 2) {
                  const ulonglong2 qa = q1[k2 / 2], qb = q2[k2 / 2];
                  a2 = fma_f32x2(qa.x, r1[k2], a2);
                  a2 = fma_f32x2(qa.y, r1[k2 + 1], a2);
                  a2 = fma_f32x2(qb.x, r2[k2], a2);
                  a2 = fma_f32x2(qb.y, r2[k2 + 1], a2);
                }
                const float a = f32x2_sum(a2);
                acc[e][j] += a;
              }
            }
            }
          }
          // The second part's partial products go through shared memory to the first part's warp.
          if (part == 1) {
#pragma unroll
            for (int e = 0; e < kHeads; ++e)
#pragma unroll
              for (int j = 0; j < G; ++j) red_s[(e * G + j) * 128 + r] = acc[e][j];
          }
          if (!group_sync(ep_sync, n_sync, p.status, kSiteKeyDense + kErrWaitAccum, abort_flag)) {
            give_up();
            failed = true;
            break;
          }
          if (part == 0) {
#pragma unroll
            for (int e = 0; e < kHeads; ++e)
#pragma unroll
              for (int j = 0; j < G; ++j) acc[e][j] += red_s[(e * G + j) * 128 + r];
          }
          if (valid && part == 0) {
#pragma unroll
            for (int e = 0; e < kHeads; ++e)
#pragma unroll
              for (int j = 0; j < G; ++j) {
                const int hq = (kv0 + e) * G + j;
                out_base[(static_cast<int64_t>(hq) * p.q_len + qi) * m_s + tile.score_base + r] =
                    hidden ? -INFINITY : acc[e][j] * p.scaling;
              }
          }
        }
      }
      if (accumulated) {
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(accum_empty_lead);
        ++item_iter;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no cross-CTA arrive, commit or MMA operand read is outstanding past here
  if (warp == 1) tmem_dealloc_pair(tmem, kKdCols);
  cluster_sync_all();
}

template <int D, int G, bool F16>
static int launch_dense(const CUtensorMap& bmap, const CUtensorMap& amap, const KeyScoreParams& p, int grid,
                        cudaStream_t stream) {
  const int smem = 1024 + kKdStages * kKdStage + (kKdCols / D) * G * D * 4 + kKdCols * 4 +
                   (kKdCols / D) * G * 128 * 4 + 32 * 8 + 32;
  if (smem > 232448) return kDkvErrConfig;
  cudaError_t e =
      cudaFuncSetAttribute(key_scores_dense_kernel<D, G, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return kDkvErrCuda;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kKdThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, key_scores_dense_kernel<D, G, F16>, bmap, amap, p);
  return e == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

template <int D, bool F16>
static int dense_dispatch_g(const CUtensorMap& bmap, const CUtensorMap& amap, const KeyScoreParams& p, int grid,
                            cudaStream_t stream) {
  switch (p.q_per_kv) {
    case 1: return launch_dense<D, 1, F16>(bmap, amap, p, grid, stream);
    case 2: return launch_dense<D, 2, F16>(bmap, amap, p, grid, stream);
    case 3: return launch_dense<D, 3, F16>(bmap, amap, p, grid, stream);
    case 4: return launch_dense<D, 4, F16>(bmap, amap, p, grid, stream);
    default: return kDkvErrConfig;
  }
}

// grid: CTAs (an even number; two per cluster). amap: the decoded key buffer, [n_tiles * 128 rows][union
// components], 64 x 128 boxes with 128B swizzle; bmap: the key basis as for run_key_scores_pair.
int run_key_scores_dense(const CUtensorMap& bmap, const CUtensorMap& amap, const KeyScoreParams& p, int grid,
                         cudaStream_t stream) {
  if (grid < 2 || grid % 2 != 0 || p.n_cols % kKdCols != 0 || p.pairs == nullptr || p.pair_groups == nullptr ||
      kKdCols % p.head_dim != 0 || p.n_tiles < 0)
    return kDkvErrConfig;
  if (p.head_dim == 128) return p.f16 ? dense_dispatch_g<128, true>(bmap, amap, p, grid, stream)
                                      : dense_dispatch_g<128, false>(bmap, amap, p, grid, stream);
  if (p.head_dim == 64) return p.f16 ? dense_dispatch_g<64, true>(bmap, amap, p, grid, stream)
                                     : dense_dispatch_g<64, false>(bmap, amap, p, grid, stream);
  return kDkvErrConfig;
}

}  // namespace dkv
