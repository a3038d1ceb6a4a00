// key_scores.cu — per-layer key rebuild fused with RoPE and the query-key products.
//
// Replaces, for one layer and a whole batch of compressed conversations:
//   CompressedContext._keys   (scripts/compressed_attention.py:105-111)  C_b @ B_l + mean, RoPE
//   the compressed half of    CompressedContext.attend (:118-120)        einsum(q, K) * scaling
// without materialising the rebuilt keys anywhere but TMEM.
//
// One work item = (tile of <=128 key tokens of one conversation, block of NB key columns).
// Per coefficient group (64 PCA components) of the tile (576 threads: warp 0 producer, warp 1 MMA,
// warps 2-9 decode, warps 10-17 epilogue):
//   producer thread  : two independent streams: cp.async.bulk of the tile's plane block into a ring
//                      of code slots, and TMA of the basis rows (NB columns x 64 components, 128B
//                      swizzle) into a ring of B stages; it polls both rings' free barriers so that
//                      neither stream waits for the other
//   8 decode warps   : bit-plane decode -> bf16 A tile (128 tokens x 64 components, 128B swizzle),
//                      ring of A stages
//   MMA warp         : tcgen05.mma M=128, N=min(NB,256), K=16 x 4, fp32 accumulator in TMEM;
//                      one commit frees the A stage, another the B stage
// After the tile's last group the 8 epilogue warps read the accumulator (one token per thread, two
// warps per TMEM lane quarter, each taking half of the block's KV heads), add the mean, apply RoPE
// with the token's position, dot with the GQA query heads and write fp32 scores.
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {

constexpr int kThreads = 576;  // producer, MMA, 8 decode warps, 8 epilogue warps
constexpr int kStagesB = 2;
constexpr int kATile = 16384;  // 128 rows x 128 B

// RAW: the stream holds raw (16-plane) blocks, which need 17 KB code slots; otherwise blocks hold at
// most 8 planes (<= 8.75 KB) and the saved shared memory buys a third A stage and a fourth code slot.
template <int NB, bool RAW>
struct KeySmem {
  static constexpr int kStagesA = RAW ? 2 : 3;
  static constexpr int kStagesC = RAW ? 3 : 4;
  static constexpr int kCodeSlot = RAW ? 17408 : 8960;  // block + the stashed 32-byte descriptor
  static constexpr int kBStage = NB * 128;
  static constexpr int kA = 0;
  static constexpr int kB = kA + kStagesA * kATile;
  static constexpr int kC = kB + kStagesB * kBStage;
  static constexpr int kQ = kC + kStagesC * kCodeSlot;
};

// Walks the (item, group) sequence of this CTA; the producer keeps two of these (code blocks, basis
// tiles) and the decode and MMA roles one each, so every role sees the same order.
struct GroupCursor {
  ItemRange ir;     // this CTA's items
  int k;            // position in ir
  int gi;           // group within the item's tile
  int n_groups, group_base, nblk;

  __device__ __forceinline__ GroupCursor(const ItemRange& r) : ir(r), k(r.k), gi(0), n_groups(0), group_base(0), nblk(0) {}

  __device__ __forceinline__ void load(const KeyScoreParams& p, int nblocks) {
    while (k < ir.end) {
      const int it = ir.at(k);
      if (it < 0) {
        record_error(p.status, kSiteKey + kErrBadDescriptor);
        k = ir.end;
        return;
      }
      const int item = p.items[it];
      const TileDesc& t = p.tiles[item / nblocks];
      n_groups = t.n_groups;
      group_base = t.group_base;
      nblk = item % nblocks;
      if (n_groups > 0) return;
      k += ir.step;
    }
  }
  __device__ __forceinline__ bool done() const { return k >= ir.end; }
  __device__ __forceinline__ void advance(const KeyScoreParams& p, int nblocks) {
    if (++gi >= n_groups) {
      gi = 0;
      k += ir.step;
      load(p, nblocks);
    }
  }
};

}  // namespace

template <int D, int NB, int G, bool RAW>
__global__ void __launch_bounds__(kThreads, 1)
    key_scores_kernel(const __grid_constant__ CUtensorMap bmap, const KeyScoreParams p) {
  constexpr int kHeads = NB / D;                // KV heads per work item
  constexpr int kHalfHeads = (kHeads + 1) / 2;  // heads of the first epilogue half
  constexpr int kNMma = NB > 256 ? 256 : NB;
  constexpr int kNHalf = NB / kNMma;
  constexpr uint32_t kIdesc = idesc_f16(128, kNMma, true, false, false);
  using L = KeySmem<NB, RAW>;
  constexpr int kStagesA = L::kStagesA;
  constexpr int kStagesC = L::kStagesC;
  constexpr int kCodeSlot = L::kCodeSlot;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem + L::kA;
  uint8_t* b_tiles = smem + L::kB;
  uint8_t* c_slots = smem + L::kC;
  float* q_s = reinterpret_cast<float*>(smem + L::kQ);  // [kHeads * G][D]
  float* mean_s = q_s + kHeads * G * D;                  // [NB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(mean_s + NB);
  uint64_t* code_full = bars;                     // [kStagesC]
  uint64_t* code_empty = code_full + kStagesC;    // [kStagesC]
  uint64_t* a_full = code_empty + kStagesC;       // [kStagesA]
  uint64_t* a_empty = a_full + kStagesA;          // [kStagesA]
  uint64_t* b_full = a_empty + kStagesA;          // [kStagesB]
  uint64_t* b_empty = b_full + kStagesB;          // [kStagesB]
  uint64_t* accum_full = b_empty + kStagesB;
  uint64_t* accum_empty = accum_full + 1;
  uint64_t* ep_sync = accum_empty + 1;  // [2] epilogue rendezvous (256 arrivals)
  uint64_t* mma_done = ep_sync + 2;      // every issued MMA has completed (exit path)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nblocks = p.n_cols / NB;
  const ItemRange items(p.cta_begin, p.item_order, p.n_items);

  if (tid == 0) {
    for (int i = 0; i < kStagesC; ++i) {
      mbar_init(&code_full[i], 1);
      mbar_init(&code_empty[i], 256);
    }
    for (int i = 0; i < kStagesA; ++i) {
      mbar_init(&a_full[i], 256);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kStagesB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(accum_empty, 256);
    mbar_init(&ep_sync[0], 256);
    mbar_init(&ep_sync[1], 256);
    mbar_init(mma_done, 1);
    // A kernel whose call has already failed does no work (every role sees the flag and skips).
    *abort_flag = status_at_entry(p.status) != 0 ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, NB);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&bmap);
      GroupCursor cc(items), cb(items);
      cc.load(p, nblocks);
      cb.load(p, nblocks);
      uint32_t c_iter = 0, b_iter = 0;
      WaitClock idle;
      bool idling = false;
      while ((!cc.done() || !cb.done()) && !*abort_flag) {
        bool progress = false;
        if (!cc.done()) {
          const int cs = c_iter % kStagesC;
          if (c_iter < kStagesC || mbar_test_wait(&code_empty[cs], ((c_iter / kStagesC) - 1) & 1)) {
            const GroupDesc* gd = &p.groups[cc.group_base + cc.gi];
            const GroupRegs gr = load_group(gd);
            if (gr.code_bytes > static_cast<uint32_t>(kCodeSlot - 32) ||
                static_cast<uint64_t>(gr.code_offset) + gr.code_bytes > p.code_size || gr.group >= p.n_union_groups) {
              record_error(p.status, kSiteKey + kErrBadDescriptor);
              *abort_flag = 1;
              break;
            }
            stash_group(c_slots + (cs + 1) * kCodeSlot, gd);
            mbar_arrive_expect_tx(&code_full[cs], gr.code_bytes);
            bulk_load(c_slots + cs * kCodeSlot, p.code + gr.code_offset, gr.code_bytes, &code_full[cs]);
            ++c_iter;
            cc.advance(p, nblocks);
            progress = true;
          }
        }
        if (!cb.done()) {
          const int sb = b_iter % kStagesB;
          if (b_iter < kStagesB || mbar_test_wait(&b_empty[sb], ((b_iter / kStagesB) - 1) & 1)) {
            const uint32_t group = __ldg(&p.groups[cb.group_base + cb.gi].group);
            mbar_arrive_expect_tx(&b_full[sb], L::kBStage);
            for (int hf = 0; hf < kNHalf; ++hf)
              tma_load_2d(b_tiles + sb * L::kBStage + hf * kNMma * 128, &bmap, &b_full[sb],
                          static_cast<int>(group) * kGroup, p.layer * p.n_cols + cb.nblk * NB + hf * kNMma);
            ++b_iter;
            cb.advance(p, nblocks);
            progress = true;
          }
        }
        if (progress) {
          idling = false;
        } else if (!idling) {
          idle = WaitClock();
          idling = true;
        } else if (idle.expired()) {
          record_error(p.status, kSiteKey + kErrWaitEmpty);
          *abort_flag = 1;
        }
      }
      // Drain: every copy this producer issued has landed before the CTA can leave.
      for (int s = 0; s < kStagesC && s < static_cast<int>(c_iter); ++s) {
        const uint32_t last = c_iter - 1 - ((c_iter - 1 - s) % kStagesC);
        mbar_wait(&code_full[s], (last / kStagesC) & 1, p.status, kSiteKey + kErrWaitDrain);
      }
      for (int s = 0; s < kStagesB && s < static_cast<int>(b_iter); ++s) {
        const uint32_t last = b_iter - 1 - ((b_iter - 1 - s) % kStagesB);
        mbar_wait(&b_full[s], (last / kStagesB) & 1, p.status, kSiteKey + kErrWaitDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t a_iter = 0, b_iter = 0, item_iter = 0;
      for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
        const int it = items.at(k);
        if (it < 0) {
          record_error(p.status, kSiteKey + kErrBadDescriptor);
          *abort_flag = 1;
          break;
        }
        const int item = p.items[it];
        const TileDesc tile = p.tiles[item / nblocks];
        if (item_iter > 0 && !mbar_wait(accum_empty, (item_iter - 1) & 1, p.status, kSiteKey + kErrWaitAccumFree, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int gi = 0; gi < tile.n_groups; ++gi) {
          const int sa = a_iter % kStagesA, sb = b_iter % kStagesB;
          if (!mbar_wait(&a_full[sa], (a_iter / kStagesA) & 1, p.status, kSiteKey + kErrWaitA, abort_flag) ||
              !mbar_wait(&b_full[sb], (b_iter / kStagesB) & 1, p.status, kSiteKey + kErrWaitBasis, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(a_tiles + sa * kATile);
          const uint32_t b_base = smem_u32(b_tiles + sb * L::kBStage);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t adesc = smem_desc_sw128(a_base + 32 * k, 16, 1024);
#pragma unroll
            for (int hf = 0; hf < kNHalf; ++hf) {
              const uint64_t bdesc = smem_desc_sw128(b_base + hf * kNMma * 128 + 32 * k, 16, 1024);
              mma_f16(tmem + hf * kNMma, adesc, bdesc, kIdesc, (gi > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit(&a_empty[sa]);
          mma_commit(&b_empty[sb]);
          ++a_iter;
          ++b_iter;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mma_commit(accum_full);
        ++item_iter;
      }
      // Also on an early exit: no MMA may still read shared memory or TMEM past this point.
      if (a_iter > 0) {
        mma_commit(mma_done);
        mbar_wait(mma_done, 0, p.status, kSiteKey + kErrWaitDrain);
      }
    }
  } else if (warp >= 2 && warp < 10) {
    // ------------------------------------------------------------ decode warps
    const int u = tid - 64;
    const int r = u & 127;
    const int h = u >> 7;
    uint32_t c_iter = 0, a_iter = 0;
    for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
      const int it = items.at(k);
      if (it < 0) {
        record_error(p.status, kSiteKey + kErrBadDescriptor);
        *abort_flag = 1;
        break;
      }
      const int item = p.items[it];
      const TileDesc tile = p.tiles[item / nblocks];
      for (int gi = 0; gi < tile.n_groups; ++gi) {
        const int cs = c_iter % kStagesC;
        const int sa = a_iter % kStagesA;
        if (!warp_wait(&code_full[cs], (c_iter / kStagesC) & 1, p.status, kSiteKey + kErrWaitCodes, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        if (a_iter >= kStagesA &&
            !warp_wait(&a_empty[sa], ((a_iter / kStagesA) - 1) & 1, p.status, kSiteKey + kErrWaitEmpty, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        const GroupRegs gr = stashed_group(c_slots + (cs + 1) * kCodeSlot);
        uint32_t out[16];
        decode_half(c_slots + cs * kCodeSlot, gr, tile.n_tokens, r, h, out);
        uint8_t* a = a_tiles + sa * kATile;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(a + sw128_offset(r, 4 * h + k)) =
              make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
        fence_async_shared();
        mbar_arrive(&a_full[sa]);
        mbar_arrive(&code_empty[cs]);
        ++c_iter;
        ++a_iter;
      }
      if (*abort_flag) break;
    }
  } else if (warp >= 10) {
    // ------------------------------------------------------------ epilogue warps
    // A warp reads the TMEM lane quarter (warp % 4); warps 10..13 and 14..17 each cover quarters
    // 2, 3, 0, 1, the first four taking the first half of the KV heads, the others the second.
    const int r = (warp & 3) * 32 + lane;          // TMEM lane == tile token row
    const int et = tid - 320;                      // 0..255 within the epilogue group
    const int head_half = (warp - 10) >> 2;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t item_iter = 0, n_sync = 0;
    bool failed = false;
    for (int k = items.k; k < items.end && !failed && !*abort_flag; k += items.step) {
      const int it = items.at(k);
      if (it < 0) {
        record_error(p.status, kSiteKey + kErrBadDescriptor);
        *abort_flag = 1;
        break;
      }
      const int item = p.items[it];
      const int ti = item / nblocks, nblk = item % nblocks;
      const TileDesc tile = p.tiles[ti];
      // The token's RoPE row (cos, sin for the first head_dim/2 dims; bf16 pairs) is fetched before
      // waiting for the accumulator so that its latency hides behind the MMAs.
      const int s = tile.seq;
      const bool valid = r < tile.n_tokens;
      const int token = tile.token_base + (valid ? r : 0);
      int pos = p.tok_pos[token];
      const bool hidden = pos < 0;  // refined or evicted token: excluded from the softmax
      pos = hidden ? 0 : (pos >= p.max_pos ? p.max_pos - 1 : pos);
      const __nv_bfloat16* cosrow = p.cos_t + static_cast<int64_t>(pos) * (D / 2);
      const __nv_bfloat16* sinrow = p.sin_t + static_cast<int64_t>(pos) * (D / 2);
      if (!warp_wait(accum_full, item_iter & 1, p.status, kSiteKey + kErrWaitAccum, abort_flag)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int64_t m_s = p.seq_m[s];
      float* out_base = p.scores + p.seq_score_off[s];
      const int kv0 = nblk * kHeads;
      for (int qi = 0; qi < p.q_len; ++qi) {
        if (!group_sync(ep_sync, n_sync, p.status, kSiteKey + kErrWaitAccum, abort_flag)) {
          *abort_flag = 1;
          failed = true;
          break;
        }
        // Stage this query row for the block's heads, and the block's mean slice.
        for (int i = et; i < kHeads * G * D; i += 256) {
          const int hq = kv0 * G + i / D;  // query head
          const int d = i % D;
          q_s[i] = __bfloat162float(p.query[((static_cast<int64_t>(s) * p.n_q_heads + hq) * p.q_len + qi) * D + d]);
        }
        if (qi == 0) {
          const __nv_bfloat16* mrow = p.mean + static_cast<int64_t>(s) * p.mean_seq_stride +
                                      static_cast<int64_t>(p.layer) * p.n_cols + nblk * NB;
          for (int i = et; i < NB; i += 256) mean_s[i] = __bfloat162float(mrow[i]);
        }
        if (!group_sync(ep_sync, n_sync, p.status, kSiteKey + kErrWaitAccum, abort_flag)) {
          *abort_flag = 1;
          failed = true;
          break;
        }
#pragma unroll 1
        for (int hh = head_half * kHalfHeads; hh < (head_half ? kHeads : kHalfHeads); ++hh) {
          float acc[G];
#pragma unroll
          for (int j = 0; j < G; ++j) acc[j] = 0.f;
#pragma unroll 1
          for (int c = 0; c < D / 2; c += 16) {
            uint32_t x1[16], x2[16];
            if (tile.n_groups > 0) {
              tmem_ld16(tmem + lane_base + hh * D + c, x1);
              tmem_ld16(tmem + lane_base + hh * D + D / 2 + c, x2);
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) x1[i] = x2[i] = 0u;
            }
            const uint4* cp = reinterpret_cast<const uint4*>(cosrow + c);
            const uint4* sp = reinterpret_cast<const uint4*>(sinrow + c);
            const uint4 cv[2] = {__ldg(cp), __ldg(cp + 1)};
            const uint4 sv[2] = {__ldg(sp), __ldg(sp + 1)};
            const __nv_bfloat162* cb = reinterpret_cast<const __nv_bfloat162*>(cv);
            const __nv_bfloat162* sb = reinterpret_cast<const __nv_bfloat162*>(sv);
            tmem_ld_wait();
            const float4* m1 = reinterpret_cast<const float4*>(mean_s + hh * D + c);
            const float4* m2 = reinterpret_cast<const float4*>(mean_s + hh * D + D / 2 + c);
#pragma unroll
            for (int i = 0; i < 16; i += 2) {
              const float2 cf = __bfloat1622float2(cb[i / 2]);
              const float2 sf = __bfloat1622float2(sb[i / 2]);
              const float4 ma = m1[i / 4], mb = m2[i / 4];
              const float k1a = __uint_as_float(x1[i]) + ((i & 2) ? ma.z : ma.x);
              const float k1b = __uint_as_float(x1[i + 1]) + ((i & 2) ? ma.w : ma.y);
              const float k2a = __uint_as_float(x2[i]) + ((i & 2) ? mb.z : mb.x);
              const float k2b = __uint_as_float(x2[i + 1]) + ((i & 2) ? mb.w : mb.y);
              x1[i] = __float_as_uint(k1a * cf.x - k2a * sf.x);
              x1[i + 1] = __float_as_uint(k1b * cf.y - k2b * sf.y);
              x2[i] = __float_as_uint(k2a * cf.x + k1a * sf.x);
              x2[i + 1] = __float_as_uint(k2b * cf.y + k1b * sf.y);
            }
#pragma unroll
            for (int j = 0; j < G; ++j) {
              const float4* q1 = reinterpret_cast<const float4*>(q_s + (hh * G + j) * D + c);
              const float4* q2 = reinterpret_cast<const float4*>(q_s + (hh * G + j) * D + D / 2 + c);
              float a = 0.f;
#pragma unroll
              for (int i = 0; i < 16; i += 4) {
                const float4 qa = q1[i / 4], qb = q2[i / 4];
                a += qa.x * __uint_as_float(x1[i]) + qa.y * __uint_as_float(x1[i + 1]) +
                     qa.z * __uint_as_float(x1[i + 2]) + qa.w * __uint_as_float(x1[i + 3]);
                a += qb.x * __uint_as_float(x2[i]) + qb.y * __uint_as_float(x2[i + 1]) +
                     qb.z * __uint_as_float(x2[i + 2]) + qb.w * __uint_as_float(x2[i + 3]);
              }
              acc[j] += a;
            }
          }
          if (valid) {
#pragma unroll
            for (int j = 0; j < G; ++j) {
              const int hq = (kv0 + hh) * G + j;
              out_base[(static_cast<int64_t>(hq) * p.q_len + qi) * m_s + tile.score_base + r] =
                  hidden ? -INFINITY : acc[j] * p.scaling;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(accum_empty);
      ++item_iter;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, NB);
}

template <int D, int NB, int G, bool RAW>
static int launch_key_scores(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  using L = KeySmem<NB, RAW>;
  const int smem = 1024 + L::kQ + (NB / D) * G * D * 4 + NB * 4 + 24 * 8 + 32;
  static_assert(2 * (L::kStagesC + L::kStagesA + kStagesB) + 5 <= 24, "barrier space");
  if (smem > 232448) return kDkvErrConfig;
  cudaError_t e =
      cudaFuncSetAttribute(key_scores_kernel<D, NB, G, RAW>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return kDkvErrCuda;
  key_scores_kernel<D, NB, G, RAW><<<grid, kThreads, smem, stream>>>(bmap, p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

template <int D, int NB, int G>
static int launch_raw(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  return p.max_planes > 8 ? launch_key_scores<D, NB, G, true>(bmap, p, grid, stream)
                          : launch_key_scores<D, NB, G, false>(bmap, p, grid, stream);
}

template <int D, int NB>
static int dispatch_g(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  switch (p.q_per_kv) {
    case 1: return launch_raw<D, NB, 1>(bmap, p, grid, stream);
    case 2: return launch_raw<D, NB, 2>(bmap, p, grid, stream);
    case 3: return launch_raw<D, NB, 3>(bmap, p, grid, stream);
    case 4: return launch_raw<D, NB, 4>(bmap, p, grid, stream);
    default: return kDkvErrConfig;
  }
}

int run_key_scores(const CUtensorMap& bmap, const KeyScoreParams& p, int nb, int grid, cudaStream_t stream) {
  if (p.head_dim == 128) {
    if (nb == 512) return dispatch_g<128, 512>(bmap, p, grid, stream);
    if (nb == 256) return dispatch_g<128, 256>(bmap, p, grid, stream);
    if (nb == 128) return dispatch_g<128, 128>(bmap, p, grid, stream);
  } else if (p.head_dim == 64) {
    if (nb == 512) return dispatch_g<64, 512>(bmap, p, grid, stream);
    if (nb == 256) return dispatch_g<64, 256>(bmap, p, grid, stream);
    if (nb == 128) return dispatch_g<64, 128>(bmap, p, grid, stream);
  }
  return kDkvErrConfig;
}

}  // namespace dkv
