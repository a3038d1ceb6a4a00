// key_scores_pair.cu — per-layer key rebuild fused with RoPE and the query-key products, on CTA pairs.
//
// Replaces, for one layer and a whole batch of compressed conversations:
//   CompressedContext._keys   (scripts/compressed_attention.py:105-111)  C_b @ B_l + mean, RoPE
//   the compressed half of    CompressedContext.attend (:118-120)        einsum(q, K) * scaling
// without materialising the rebuilt keys anywhere but TMEM.
//
// A cluster of two CTAs (two SMs of one TPC) works on one item at a time: a pair of key tiles (up to
// 128 tokens each, usually two neighbouring tiles of one conversation) x a block of 512 key columns.
// The pair MMA (tcgen05.mma.cta_group::2, M = 256, N = 256, K = 16; two per K step for the two
// column halves) takes the A rows of each CTA's tile from that CTA's shared memory and each half of
// the 256 basis columns of an MMA from one CTA, so every SM loads 256 of the item's 512 basis columns
// per coefficient group: half the L2 traffic of a single-CTA tile, and twice the pipeline depth in the
// same shared memory. Each token's codes are decoded twice per layer (two column blocks).
//
// The two tiles' groups are merged (both CTAs walk the same sorted union); a CTA whose tile lacks a
// group decodes zeros for it. Roles per CTA (896 threads, seven warpgroups):
//   warp 0     code producer: plane blocks of its own tile (cp.async.bulk, ring of code slots)
//   warp 1     even CTA: the pair MMA issuer; odd CTA: forwards its B-stage completions to the even
//              CTA (a TMA completes on the issuing CTA's own barrier, so every CTA can drain its copies)
//   warp 2     basis producer: its half of the basis rows of every MMA (TMA, ring of B stages)
//   warps 4-19 decode, two sets of 8 warps taking alternate groups: bit planes -> bf16 A tile (128
//              tokens x 64 components, 128B swizzle); they follow the producer's slots (each slot carries
//              its descriptor, the tile's token count and an end mark), so they hold no item state
//   warps 20-27 epilogue: TMEM -> + mean -> RoPE -> q.k -> fp32 scores, two heads' accumulators
//              loaded per TMEM wait
// Cross-CTA signals: decode and epilogue warps arrive on the even CTA's a_full / accum_empty barriers
// (one arrival per warp, after the operand writes are fenced to the async proxy); the MMA commits multicast to both CTAs' a_empty / b_empty /
// accum_full barriers. Every wait is bounded; on any error both CTAs stop issuing, drain their own
// copies and meet at the final cluster barrier.
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {

constexpr int kPairThreads = 896;
// Register split per warpgroup (setmaxnreg): the launch gives every thread kLaunchRegs; the control
// warpgroup drops to 24, the four decode warpgroups to 40, the two epilogue warpgroups take 160:
// 128*24 + 512*40 + 256*160 = 64512 <= 896*72 = 64512. The launch checks the compiled count first.
// Registers move between warps of the same SM sub-partition only (warp w runs on sub-partition w % 4), and
// each sub-partition holds one control warp, four decode warps and two epilogue warps: 32*(72-24) +
// 4*32*(72-40) = 5632 registers released there, exactly the 2*32*(160-72) its two epilogue warps take.
// (Measured against 40/48/136, 40/40/152 and 24/48/144 on the bench's 64 conversations: 0.9 % faster
// than the next best; ptxas reports the fewest spills for it.)
// The balance is exact, so no warp may take registers back (its setmaxnreg.inc at the bottom of its
// branch) before both epilogue warps of its sub-partition hold their 160: the idle control warp 3 would
// otherwise reach its inc at once and could starve an epilogue warp of sub-partition 3 for good. Every
// warp therefore meets the others on named barrier kRegBarrier right after its first setmaxnreg.
constexpr int kLaunchRegs = 72;
#ifndef DKV_REGS_CONTROL
#define DKV_REGS_CONTROL 24
#define DKV_REGS_DECODE 40
#define DKV_REGS_EPILOGUE 160
#endif
constexpr int kRegsControl = DKV_REGS_CONTROL, kRegsDecode = DKV_REGS_DECODE, kRegsEpilogue = DKV_REGS_EPILOGUE;
static_assert(128 * kRegsControl + 512 * kRegsDecode + 256 * kRegsEpilogue <= kPairThreads * kLaunchRegs,
              "register split exceeds the launch allocation");
constexpr int kRegBarrier = 1;              // named barrier of the register hand-over (0 is __syncthreads)
constexpr int kPairCols = 512;              // key columns per item
constexpr int kMmaN = 256;                  // N of one pair MMA (two per K step)
constexpr int kHalfCols = 128;              // basis columns of one pair MMA loaded by each CTA
constexpr int kATilePair = 16384;           // 128 rows x 128 B
constexpr int kBHalf = kHalfCols * 128;     // 128 basis rows x 64 components x bf16
constexpr int kBStagePair = 2 * kBHalf;     // both MMA halves

template <bool RAW>
struct PairSmem {
  static constexpr int kStagesA = RAW ? 2 : 3;
  static constexpr int kStagesB = 4;
  static constexpr int kStagesC = RAW ? 3 : 4;
  static constexpr int kCodeSlot = RAW ? 17408 : 8960;  // block + the stashed 32-byte descriptor
  static constexpr int kA = 0;
  static constexpr int kB = kA + kStagesA * kATilePair;
  static constexpr int kC = kB + kStagesB * kBStagePair;
  static constexpr int kQ = kC + kStagesC * kCodeSlot;
};

// Walks the merged group sequence of one CTA pair's items. The host lists, per pair, the sorted union
// of the two tiles' groups as (group, descriptor of tile 0 or -1, descriptor of tile 1 or -1, 0)
// entries (pair_groups); both CTAs read the same entries, one 16-byte load per group.
struct PairCursor {
  ItemRange ir;
  int k;
  int nblk;
  int off, n, i;  // current item: its entries [off, off + n), position i
  int tok[2];      // token counts of the item's two tiles (0: no tile)

  __device__ __forceinline__ explicit PairCursor(const ItemRange& r) : ir(r), k(r.k), nblk(0), off(0), n(0), i(0) {
    tok[0] = tok[1] = 0;
  }

  // Load items from position k on until one has a group. Returns false when done (or on a bad entry).
  __device__ __forceinline__ bool load(const KeyScoreParams& p, int nblocks) {
    while (k < ir.end) {
      const int it = ir.at(k);
      if (it < 0) {
        record_error(p.status, kSiteKeyPair + kErrBadDescriptor);
        k = ir.end;
        break;
      }
      const int code = p.items[it];
      const int4 pr = __ldg(reinterpret_cast<const int4*>(p.pairs) + code / nblocks);
      nblk = code % nblocks;
      n = pr.z;
      off = pr.w;
      i = 0;
      if (n > 0) {
        tok[0] = pr.x >= 0 ? p.tiles[pr.x].n_tokens : 0;
        tok[1] = pr.y >= 0 ? p.tiles[pr.y].n_tokens : 0;
        return true;
      }
      k += ir.step;
    }
    return false;
  }
  __device__ __forceinline__ bool done() const { return k >= ir.end; }
  // Current merged group and, for CTA `rank`, the descriptor index of its tile's block (-1: none).
  __device__ __forceinline__ uint32_t group(const KeyScoreParams& p, int rank, int& desc) const {
    const int4 e = __ldg(reinterpret_cast<const int4*>(p.pair_groups) + off + i);
    desc = rank ? e.z : e.y;
    return static_cast<uint32_t>(e.x);
  }
  __device__ __forceinline__ void advance(const KeyScoreParams& p, int nblocks) {
    if (++i >= n) {
      k += ir.step;
      load(p, nblocks);
    }
  }
};

// Stash flags (GroupDesc pad bytes of a code slot's stashed descriptor).
constexpr uint32_t kStashEnd = 1u;  // no more groups for this CTA

}  // namespace

template <int D, int G, bool RAW, bool F16>
__global__ void __launch_bounds__(kPairThreads, 1)
    key_scores_pair_kernel(const __grid_constant__ CUtensorMap bmap, const KeyScoreParams p) {
  constexpr int kHeads = kPairCols / D;     // KV heads per item
  constexpr int kHalfHeads = kHeads / 2;    // heads per epilogue half
  constexpr uint32_t kIdesc = idesc_f16(256, kMmaN, /*is_bf16=*/!F16, false, false);
  using L = PairSmem<RAW>;
  constexpr int kStagesA = L::kStagesA;
  constexpr int kStagesB = L::kStagesB;
  constexpr int kStagesC = L::kStagesC;
  constexpr int kCodeSlot = L::kCodeSlot;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem + L::kA;
  uint8_t* b_tiles = smem + L::kB;
  uint8_t* c_slots = smem + L::kC;
  float* q_s = reinterpret_cast<float*>(smem + L::kQ);  // [kHeads * G][D]
  float* mean_s = q_s + kHeads * G * D;                  // [kPairCols]
  uint64_t* bars = reinterpret_cast<uint64_t*>(mean_s + kPairCols);
  uint64_t* code_full = bars;                    // [kStagesC]
  uint64_t* code_empty = code_full + kStagesC;   // [kStagesC]
  uint64_t* a_full = code_empty + kStagesC;      // [kStagesA] (even CTA: 16 warp arrivals)
  uint64_t* a_empty = a_full + kStagesA;         // [kStagesA] (pair-MMA commit)
  uint64_t* b_full = a_empty + kStagesA;         // [kStagesB] (this CTA's TMA)
  uint64_t* b_peer = b_full + kStagesB;          // [kStagesB] (even CTA: the odd CTA's forward)
  uint64_t* b_empty = b_peer + kStagesB;         // [kStagesB] (pair-MMA commit)
  uint64_t* accum_full = b_empty + kStagesB;     // pair-MMA commit
  uint64_t* accum_empty = accum_full + 1;        // even CTA: 16 warp arrivals
  uint64_t* mma_done = accum_empty + 1;          // even CTA: every issued pair MMA has completed
  uint64_t* ep_sync = mma_done + 1;              // [2] epilogue rendezvous (256 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ep_sync + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int nblocks = p.n_cols / kPairCols;
  // Cluster c processes list c of the schedule.
  const ItemRange items(p.cta_begin, p.item_order, p.n_items, blockIdx.x >> 1, gridDim.x >> 1);

  if (tid == 0) {
    for (int i = 0; i < kStagesC; ++i) {
      mbar_init(&code_full[i], 1);
      mbar_init(&code_empty[i], 256);
    }
    for (int i = 0; i < kStagesA; ++i) {
      mbar_init(&a_full[i], 16);
      mbar_init(&a_empty[i], 1);
    }
    for (int i = 0; i < kStagesB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&b_peer[i], 1);
      mbar_init(&b_empty[i], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(accum_empty, 16);
    mbar_init(mma_done, 1);
    mbar_init(&ep_sync[0], 256);
    mbar_init(&ep_sync[1], 256);
    // A kernel whose call has already failed does no work (every role sees the flag and skips).
    *abort_flag = status_at_entry(p.status) != 0 ? 1 : 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kPairCols);
  __syncthreads();
  cluster_sync_all();  // barriers of both CTAs initialised before any cross-CTA arrive
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Even-CTA addresses of the barriers that take arrivals from both CTAs.
  const uint32_t a_full_lead = mapa_shared(smem_u32(a_full), 0);
  const uint32_t b_peer_lead = mapa_shared(smem_u32(b_peer), 0);
  const uint32_t accum_empty_lead = mapa_shared(smem_u32(accum_empty), 0);
  // The abort flag is cluster-wide: a role that gives up sets it in both CTAs (its own and, through
  // st.shared::cluster, the peer's), so that no role of either CTA keeps waiting on a partner that has
  // stopped. Both CTAs stay resident until the final cluster barrier, so the peer's flag is valid.
  auto give_up = [abort_flag]() {
    *abort_flag = 1;
    st_cluster_u32(mapa_shared(smem_u32(const_cast<int*>(abort_flag)), cluster_ctarank() ^ 1u), 1u);
  };
  if (tid == 0 && *abort_flag) give_up();  // the entry check of either CTA stops both

  // Each role's register budget is set at the top of its warpgroup's branch (so that it governs the
  // role's code) and the launch budget restored at the bottom, before the common exit path; the
  // epilogue warpgroups release their extra registers there, which the others then take back. Between
  // the two, every warp passes the register hand-over barrier once all epilogue warps hold their budget.
  if (warp < 4) {
  setmaxnreg_dec<kRegsControl>();
  named_barrier_sync(kRegBarrier, kPairThreads);
  if (warp == 0) {
    // ------------------------------------------------------------ code producer
    if (lane == 0) {
      PairCursor cc(items);
      cc.load(p, nblocks);
      uint32_t c_iter = 0;
      bool c_ended = false;  // the end mark has been written
      while (!c_ended && !*abort_flag) {
        const int cs = c_iter % kStagesC;
        if (c_iter >= kStagesC &&
            !mbar_wait(&code_empty[cs], ((c_iter / kStagesC) - 1) & 1, p.status, kSiteKeyPair + kErrWaitEmpty, abort_flag)) {
          give_up();
          break;
        }
        if (cc.done()) {
          c_ended = true;  // the end marks follow below
          break;
        }
        uint8_t* slot_end = c_slots + (cs + 1) * kCodeSlot;
        uint4* stash = reinterpret_cast<uint4*>(slot_end - 32);
        int desc;
        const uint32_t g = cc.group(p, rank, desc);
        const uint32_t n_tok = static_cast<uint32_t>(cc.tok[rank]);
        if (desc >= 0) {
          const GroupDesc* gd = &p.groups[desc];
          const uint4* src = reinterpret_cast<const uint4*>(gd);
          uint4 w0 = __ldg(src);
          const uint4 w1 = __ldg(src + 1);
          const GroupRegs gr = group_from_words(w0, w1);
          if (gr.code_bytes > static_cast<uint32_t>(kCodeSlot - 32) ||
              static_cast<uint64_t>(gr.code_offset) + gr.code_bytes > p.code_size ||
              gr.group >= p.n_union_groups) {
            record_error(p.status, kSiteKeyPair + kErrBadDescriptor);
            give_up();
            break;
          }
          w0.w = (w0.w & 0xFFFFu) | (n_tok << 16);  // pad0: the tile's token count
          stash[0] = w0;
          stash[1] = w1;
          mbar_arrive_expect_tx(&code_full[cs], gr.code_bytes);
          bulk_load(c_slots + cs * kCodeSlot, p.code + gr.code_offset, gr.code_bytes, &code_full[cs]);
        } else {
          // This CTA's tile has no block for the group: no token holds a plane (first[j] = 128).
          stash[0] = make_uint4(g, 0u, 0u, n_tok << 16);
          stash[1] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
          mbar_arrive(&code_full[cs]);
        }
        cc.advance(p, nblocks);
        ++c_iter;
      }
      // End marks in the next two slots, one for each decode set (also after an error, to release them).
      for (int e = 0; e < 2; ++e) {
        const int cs = c_iter % kStagesC;
        if (c_iter >= kStagesC &&
            !mbar_wait(&code_empty[cs], ((c_iter / kStagesC) - 1) & 1, p.status, kSiteKeyPair + kErrWaitDrain, abort_flag))
          break;
        uint4* stash = reinterpret_cast<uint4*>(c_slots + (cs + 1) * kCodeSlot - 32);
        stash[0] = make_uint4(0u, 0u, 0u, kStashEnd << 24);
        stash[1] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
        mbar_arrive(&code_full[cs]);
        ++c_iter;
      }
      // Drain: every plane-block copy this CTA issued has landed before the CTA can leave.
      for (int s = 0; s < kStagesC && s < static_cast<int>(c_iter); ++s) {
        const uint32_t last = c_iter - 1 - ((c_iter - 1 - s) % kStagesC);
        mbar_wait(&code_full[s], (last / kStagesC) & 1, p.status, kSiteKeyPair + kErrWaitDrain);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ basis producer
    if (lane == 0) {
      prefetch_tensormap(&bmap);
      PairCursor cb(items);
      cb.load(p, nblocks);
      uint32_t b_iter = 0;
      while (!cb.done() && !*abort_flag) {
        const int sb = b_iter % kStagesB;
        if (b_iter >= kStagesB &&
            !mbar_wait(&b_empty[sb], ((b_iter / kStagesB) - 1) & 1, p.status, kSiteKeyPair + kErrWaitEmpty, abort_flag)) {
          give_up();
          break;
        }
        int desc;
        const uint32_t g = cb.group(p, rank, desc);
        mbar_arrive_expect_tx(&b_full[sb], kBStagePair);
#pragma unroll
        for (int hf = 0; hf < 2; ++hf)
          tma_load_2d(b_tiles + sb * kBStagePair + hf * kBHalf, &bmap, &b_full[sb], static_cast<int>(g) * kGroup,
                      p.layer * p.n_cols + cb.nblk * kPairCols + hf * kMmaN + rank * kHalfCols);
        ++b_iter;
        cb.advance(p, nblocks);
      }
      // Drain: every basis copy this CTA issued has landed before the CTA can leave.
      for (int s = 0; s < kStagesB && s < static_cast<int>(b_iter); ++s) {
        const uint32_t last = b_iter - 1 - ((b_iter - 1 - s) % kStagesB);
        mbar_wait(&b_full[s], (last / kStagesB) & 1, p.status, kSiteKeyPair + kErrWaitDrain);
      }
    }
  } else if (warp == 1) {
    if (rank == 0) {
      // ---------------------------------------------------------- pair MMA issuer (even CTA)
      if (lane == 0) {
        uint32_t a_iter = 0, b_iter = 0, item_iter = 0;
        for (int k = items.k; k < items.end && !*abort_flag; k += items.step) {
          const int it = items.at(k);
          if (it < 0) {
            record_error(p.status, kSiteKeyPair + kErrBadDescriptor);
            give_up();
            break;
          }
          const int n_merged = p.pairs[4 * (p.items[it] / nblocks) + 2];
          if (n_merged <= 0) continue;  // nothing accumulated; the epilogue writes the mean-only keys
          if (item_iter >= 1 &&
              !mbar_wait(accum_empty, (item_iter - 1) & 1, p.status, kSiteKeyPair + kErrWaitAccumFree, abort_flag)) {
            give_up();
            break;
          }
          tc_fence_after();
          bool ok = true;
          for (int gi = 0; gi < n_merged; ++gi) {
            const int sa = a_iter % kStagesA, sb = b_iter % kStagesB;
            if (!mbar_wait(&a_full[sa], (a_iter / kStagesA) & 1, p.status, kSiteKeyPair + kErrWaitA, abort_flag) ||
                !mbar_wait(&b_full[sb], (b_iter / kStagesB) & 1, p.status, kSiteKeyPair + kErrWaitBasis, abort_flag) ||
                !mbar_wait(&b_peer[sb], (b_iter / kStagesB) & 1, p.status, kSiteKeyPair + kErrWaitBasis, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(a_tiles + sa * kATilePair);
            const uint32_t b_base = smem_u32(b_tiles + sb * kBStagePair);
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint64_t adesc = smem_desc_sw128(a_base + 32 * kk, 16, 1024);
#pragma unroll
              for (int hf = 0; hf < 2; ++hf) {
                const uint64_t bdesc = smem_desc_sw128(b_base + hf * kBHalf + 32 * kk, 16, 1024);
                mma_f16_pair(tmem + hf * kMmaN, adesc, bdesc, kIdesc, (gi > 0 || kk > 0) ? 1u : 0u);
              }
            }
            mma_commit_pair(&a_empty[sa], 0x3);
            mma_commit_pair(&b_empty[sb], 0x3);
            ++a_iter;
            ++b_iter;
          }
          if (!ok) {
            give_up();
            break;
          }
          mma_commit_pair(accum_full, 0x3);
          ++item_iter;
        }
        // Also on an early exit: no pair MMA may still read shared memory or TMEM past this point.
        if (a_iter > 0) {
          mma_commit_pair(mma_done, 0x1);
          mbar_wait(mma_done, 0, p.status, kSiteKeyPair + kErrWaitDrain);
        }
      }
    } else {
      // ---------------------------------------------------------- B-stage forwarder (odd CTA)
      if (lane == 0) {
        PairCursor cf(items);
        cf.load(p, nblocks);
        uint32_t b_iter = 0;
        while (!cf.done() && !*abort_flag) {
          const int sb = b_iter % kStagesB;
          if (!mbar_wait(&b_full[sb], (b_iter / kStagesB) & 1, p.status, kSiteKeyPair + kErrWaitBasis, abort_flag)) {
            give_up();
            break;
          }
          mbar_arrive_cluster(b_peer_lead + sb * 8);
          ++b_iter;
          cf.advance(p, nblocks);
        }
      }
    }
  }
  setmaxnreg_inc<kLaunchRegs>();
  } else if (warp < 20) {
    setmaxnreg_dec<kRegsDecode>();
    named_barrier_sync(kRegBarrier, kPairThreads);
    // ------------------------------------------------------------ decode warps (follow the slots)
    // Set 0 (warps 4-11) takes the even positions of the group sequence, set 1 (warps 12-19) the odd.
    const int set = (warp - 4) >> 3;
    const int u = tid - 128 - set * 256;
    const int r = u & 127;
    const int h = u >> 7;
    for (uint32_t i = set;; i += 2) {  // position in the sequence: code slot i % kStagesC, A stage i % kStagesA
      const int cs = i % kStagesC;
      if (!warp_wait(&code_full[cs], (i / kStagesC) & 1, p.status, kSiteKeyPair + kErrWaitCodes, abort_flag)) {
        give_up();
        break;
      }
      const uint8_t* slot = c_slots + cs * kCodeSlot;
      const uint4 w0 = *reinterpret_cast<const uint4*>(slot + kCodeSlot - 32);
      if ((w0.w >> 24) & kStashEnd) break;
      const int sa = i % kStagesA;
      if (i >= static_cast<uint32_t>(kStagesA) &&
          !warp_wait(&a_empty[sa], ((i / kStagesA) - 1) & 1, p.status, kSiteKeyPair + kErrWaitEmpty, abort_flag)) {
        give_up();
        break;
      }
      const GroupRegs gr = group_from_words(w0, *reinterpret_cast<const uint4*>(slot + kCodeSlot - 16));
      const int n_tok = static_cast<int>((w0.w >> 16) & 0xFFu);
      uint32_t out[16];
      decode_half<F16>(slot, gr, n_tok, r, h, out);
      uint8_t* a = a_tiles + sa * kATilePair;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        *reinterpret_cast<uint4*>(a + sw128_offset(r, 4 * h + kk)) =
            make_uint4(out[4 * kk], out[4 * kk + 1], out[4 * kk + 2], out[4 * kk + 3]);
      fence_async_shared();
      mbar_arrive(&code_empty[cs]);
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(a_full_lead + sa * 8);
    }
    setmaxnreg_inc<kLaunchRegs>();
  } else {
    setmaxnreg_inc<kRegsEpilogue>();
    named_barrier_sync(kRegBarrier, kPairThreads);
    // ------------------------------------------------------------ epilogue warps
    // A warp reads the TMEM lane quarter (warp % 4); warps 20..23 and 24..27 each cover quarters
    // 0..3, the first four taking the first half of the item's KV heads, the others the second.
    const int r = (warp & 3) * 32 + lane;  // TMEM lane == tile token row
    const int et = tid - 640;              // 0..255 within the epilogue group
    const int head_half = (warp - 20) >> 2;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t item_iter = 0, n_sync = 0;
    bool failed = false;
    for (int k = items.k; k < items.end && !*abort_flag && !failed; k += items.step) {
      const int it = items.at(k);
      if (it < 0) {
        record_error(p.status, kSiteKeyPair + kErrBadDescriptor);
        give_up();
        break;
      }
      const int code = p.items[it];
      const int pair = code / nblocks, nblk = code % nblocks;
      const int ti = p.pairs[4 * pair + rank];
      const bool accumulated = p.pairs[4 * pair + 2] > 0;
      // The token's RoPE row is located before waiting for the accumulator.
      const bool has_tile = ti >= 0;
      const TileDesc tile = has_tile ? p.tiles[ti] : TileDesc{};
      const bool valid = has_tile && r < tile.n_tokens;
      int pos = valid ? p.tok_pos[tile.token_base + r] : 0;
      const bool hidden = pos < 0;  // refined or evicted token: excluded from the softmax
      pos = hidden ? 0 : (pos >= p.max_pos ? p.max_pos - 1 : pos);
      const uint16_t* cosrow = reinterpret_cast<const uint16_t*>(p.cos_t) + static_cast<int64_t>(pos) * (D / 2);
      const uint16_t* sinrow = reinterpret_cast<const uint16_t*>(p.sin_t) + static_cast<int64_t>(pos) * (D / 2);
      if (accumulated) {
        if (!warp_wait(accum_full, item_iter & 1, p.status, kSiteKeyPair + kErrWaitAccum, abort_flag)) {
          give_up();
          break;
        }
        tc_fence_after();
      }
      if (has_tile) {
        const int s = tile.seq;
        const int64_t m_s = p.seq_m[s];
        float* out_base = p.scores + p.seq_score_off[s];
        const int kv0 = nblk * kHeads;
        const int h0 = head_half * kHalfHeads;  // first head of this half
        for (int qi = 0; qi < p.q_len; ++qi) {
          if (!group_sync(ep_sync, n_sync, p.status, kSiteKeyPair + kErrWaitAccum, abort_flag)) {
            give_up();
            failed = true;
            break;
          }
          for (int i = et; i < kHeads * G * D; i += 256) {
            const int hq = kv0 * G + i / D;
            const int d = i % D;
            q_s[i] = half_to_float<F16>(reinterpret_cast<const uint16_t*>(
                p.query)[((static_cast<int64_t>(s) * p.n_q_heads + hq) * p.q_len + qi) * D + d]);
          }
          if (qi == 0) {
            const uint16_t* mrow = reinterpret_cast<const uint16_t*>(p.mean) + static_cast<int64_t>(s) * p.mean_seq_stride +
                                   static_cast<int64_t>(p.layer) * p.n_cols + nblk * kPairCols;
            for (int i = et; i < kPairCols; i += 256) mean_s[i] = half_to_float<F16>(mrow[i]);
          }
          if (!group_sync(ep_sync, n_sync, p.status, kSiteKeyPair + kErrWaitAccum, abort_flag)) {
            give_up();
            failed = true;
            break;
          }
          float acc[kHalfHeads][G];
#pragma unroll
          for (int e = 0; e < kHalfHeads; ++e)
#pragma unroll
            for (int j = 0; j < G; ++j) acc[e][j] = 0.f;
#pragma unroll 1
          for (int c = 0; c < D / 2; c += 16) {
            // The token's cos / sin for these 16 dims, shared by every head of the half.
            const uint4* cp = reinterpret_cast<const uint4*>(cosrow + c);
            const uint4* sp = reinterpret_cast<const uint4*>(sinrow + c);
            const uint4 cv[2] = {__ldg(cp), __ldg(cp + 1)};
            const uint4 sv[2] = {__ldg(sp), __ldg(sp + 1)};
            const uint32_t* cbv = reinterpret_cast<const uint32_t*>(cv);  // 8 pairs of 16-bit values
            const uint32_t* sbv = reinterpret_cast<const uint32_t*>(sv);
#pragma unroll
            for (int hp = 0; hp < kHalfHeads; hp += 2) {
              uint32_t x1[2][16], x2[2][16];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int hh = h0 + hp + e;
                if (accumulated) {
                  tmem_ld16(tmem + lane_base + hh * D + c, x1[e]);
                  tmem_ld16(tmem + lane_base + hh * D + D / 2 + c, x2[e]);
                } else {
#pragma unroll
                  for (int i = 0; i < 16; ++i) x1[e][i] = x2[e][i] = 0u;
                }
              }
              if (accumulated) tmem_ld_wait();
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const int hh = h0 + hp + e;
                const float4* m1 = reinterpret_cast<const float4*>(mean_s + hh * D + c);
                const float4* m2 = reinterpret_cast<const float4*>(mean_s + hh * D + D / 2 + c);
#pragma unroll
                for (int i = 0; i < 16; i += 2) {
                  const float2 cf = half2_to_float2<F16>(cbv[i / 2]);
                  const float2 sf = half2_to_float2<F16>(sbv[i / 2]);
                  const float4 ma = m1[i / 4], mb = m2[i / 4];
                  const float k1a = __uint_as_float(x1[e][i]) + ((i & 2) ? ma.z : ma.x);
                  const float k1b = __uint_as_float(x1[e][i + 1]) + ((i & 2) ? ma.w : ma.y);
                  const float k2a = __uint_as_float(x2[e][i]) + ((i & 2) ? mb.z : mb.x);
                  const float k2b = __uint_as_float(x2[e][i + 1]) + ((i & 2) ? mb.w : mb.y);
                  x1[e][i] = __float_as_uint(k1a * cf.x - k2a * sf.x);
                  x1[e][i + 1] = __float_as_uint(k1b * cf.y - k2b * sf.y);
                  x2[e][i] = __float_as_uint(k2a * cf.x + k1a * sf.x);
                  x2[e][i + 1] = __float_as_uint(k2b * cf.y + k1b * sf.y);
                }
#pragma unroll
                for (int j = 0; j < G; ++j) {
                  const float4* q1 = reinterpret_cast<const float4*>(q_s + (hh * G + j) * D + c);
                  const float4* q2 = reinterpret_cast<const float4*>(q_s + (hh * G + j) * D + D / 2 + c);
                  float a = 0.f;
#pragma unroll
                  for (int i = 0; i < 16; i += 4) {
                    const float4 qa = q1[i / 4], qb = q2[i / 4];
                    a += qa.x * __uint_as_float(x1[e][i]) + qa.y * __uint_as_float(x1[e][i + 1]) +
                         qa.z * __uint_as_float(x1[e][i + 2]) + qa.w * __uint_as_float(x1[e][i + 3]);
                    a += qb.x * __uint_as_float(x2[e][i]) + qb.y * __uint_as_float(x2[e][i + 1]) +
                         qb.z * __uint_as_float(x2[e][i + 2]) + qb.w * __uint_as_float(x2[e][i + 3]);
                  }
                  acc[hp + e][j] += a;
                }
              }
            }
          }
          if (valid) {
#pragma unroll
            for (int e = 0; e < kHalfHeads; ++e)
#pragma unroll
              for (int j = 0; j < G; ++j) {
                const int hq = (kv0 + h0 + e) * G + j;
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
    setmaxnreg_dec<kLaunchRegs>();
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no cross-CTA arrive, commit or MMA operand read is outstanding past here
  if (warp == 1) tmem_dealloc_pair(tmem, kPairCols);
  cluster_sync_all();
}

template <int D, int G, bool RAW, bool F16>
static int launch_pair(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  using L = PairSmem<RAW>;
  const int smem = 1024 + L::kQ + (kPairCols / D) * G * D * 4 + kPairCols * 4 + 48 * 8 + 32;
  if (smem > 232448) return kDkvErrConfig;
  // The warpgroup register split assumes exactly kLaunchRegs per thread at launch; with any other
  // count setmaxnreg.inc could wait for registers that never come, so refuse to launch.
  cudaFuncAttributes fattr{};
  if (cudaFuncGetAttributes(&fattr, key_scores_pair_kernel<D, G, RAW, F16>) != cudaSuccess) return kDkvErrCuda;
  if (fattr.numRegs != kLaunchRegs) return kDkvErrConfig;
  cudaError_t e =
      cudaFuncSetAttribute(key_scores_pair_kernel<D, G, RAW, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return kDkvErrCuda;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, key_scores_pair_kernel<D, G, RAW, F16>, bmap, p);
  return e == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

template <int D, bool F16>
static int pair_dispatch_g(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  const bool raw = p.max_planes > 8;
  switch (p.q_per_kv) {
    case 1: return raw ? launch_pair<D, 1, true, F16>(bmap, p, grid, stream) : launch_pair<D, 1, false, F16>(bmap, p, grid, stream);
    case 2: return raw ? launch_pair<D, 2, true, F16>(bmap, p, grid, stream) : launch_pair<D, 2, false, F16>(bmap, p, grid, stream);
    case 3: return raw ? launch_pair<D, 3, true, F16>(bmap, p, grid, stream) : launch_pair<D, 3, false, F16>(bmap, p, grid, stream);
    case 4: return raw ? launch_pair<D, 4, true, F16>(bmap, p, grid, stream) : launch_pair<D, 4, false, F16>(bmap, p, grid, stream);
    default: return kDkvErrConfig;
  }
}

// grid: CTAs (an even number; two per cluster).
int run_key_scores_pair(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  if (grid < 2 || grid % 2 != 0 || p.n_cols % kPairCols != 0 || p.pairs == nullptr || kPairCols % p.head_dim != 0)
    return kDkvErrConfig;
  if (p.head_dim == 128) return p.f16 ? pair_dispatch_g<128, true>(bmap, p, grid, stream) : pair_dispatch_g<128, false>(bmap, p, grid, stream);
  if (p.head_dim == 64) return p.f16 ? pair_dispatch_g<64, true>(bmap, p, grid, stream) : pair_dispatch_g<64, false>(bmap, p, grid, stream);
  return kDkvErrConfig;
}

}  // namespace dkv
