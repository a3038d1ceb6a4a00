// value_weights.cu — attention probabilities applied to value coefficients (values never decoded).
//
// Replaces the per-block value products of CompressedContext.attend
// (scripts/compressed_attention.py:127, 132-133):
//   p_c = softmax(...)[..., :middle].to(dtype)
//   weighted += einsum("bhgqn,nr->bhgqr", p_c[..., block.index], block.coefficients)
// for a batch of conversations. One work item = (conversation, run of value tiles, range of
// union groups). For every tile the 8 worker warps
//   - build P^T (rows = query head x query row, K = the tile's 128 tokens) in bf16 from the
//     fp32 scores and the softmax statistics (exactly the reference's rounding of p to the
//     cache dtype), 128B-swizzled K-major;
//   - decode each pair of coefficient groups into a 128-component x 128-token bf16 tile
//     (MN-major operand: token rows of 64 components, 128B swizzle).
// The MMA warp accumulates D[128 components, rows] += C^T P^T with tcgen05 (M=128, N=rows,
// K=16 tokens per instruction) into one TMEM column range per group pair. At the end of the
// item the accumulators are written to `partial` (fp32), which finalize.cu reduces.
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {

constexpr int kVThreads = 384;
constexpr int kVCodeSlots = 4;
constexpr int kVCodeSlot = 17408;
constexpr int kPairTile = 32768;  // two groups x 128 tokens x 128 B

// Walks the groups of one tile that fall in [g0, g0 + ng): every role of the kernel uses the
// same walk, so all agree on the sequence of code blocks and group pairs.
struct PairWalk {
  const GroupDesc* groups;
  int base, count, g0, ng;
  int gi;  // next group index (absolute)

  __device__ __forceinline__ void begin(const TileDesc& t, const GroupDesc* all, int first_group, int n_groups) {
    groups = all;
    base = t.group_base;
    count = t.n_groups;
    g0 = first_group;
    ng = n_groups;
    gi = base;
    while (gi < base + count && static_cast<int>(__ldg(&groups[gi].group)) < g0) ++gi;
  }
  // Next pair present in the tile: returns pair index or -1; sets descriptors of its halves.
  __device__ __forceinline__ int next(int& lo_gi, int& hi_gi) {
    lo_gi = hi_gi = -1;
    if (gi >= base + count) return -1;
    const int g = static_cast<int>(__ldg(&groups[gi].group));
    if (g >= g0 + ng) return -1;
    const int pair = (g - g0) >> 1;
    if (((g - g0) & 1) == 0) {
      lo_gi = gi++;
      if (gi < base + count && static_cast<int>(__ldg(&groups[gi].group)) == g + 1) hi_gi = gi++;
    } else {
      hi_gi = gi++;
    }
    return pair;
  }
};

}  // namespace

__global__ void __launch_bounds__(kVThreads, 1) value_weights_kernel(const ValueWeightParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int NR = p.n_rows_pad;            // MMA N (multiple of 16, <= 128)
  const int p_tile = NR * 256;            // two K atoms of 64 tokens
  uint8_t* a_tiles = smem;                                  // [2][kPairTile]
  uint8_t* p_tiles = a_tiles + 2 * kPairTile;               // [2][p_tile]
  uint8_t* c_slots = p_tiles + 2 * p_tile;                  // [kVCodeSlots][kVCodeSlot]
  uint64_t* bars = reinterpret_cast<uint64_t*>(c_slots + kVCodeSlots * kVCodeSlot);
  uint64_t* code_full = bars;
  uint64_t* code_empty = code_full + kVCodeSlots;
  uint64_t* a_full = code_empty + kVCodeSlots;    // [2]
  uint64_t* a_empty = a_full + 2;                 // [2]
  uint64_t* p_full = a_empty + 2;                 // [2]
  uint64_t* p_empty = p_full + 2;                 // [2]
  uint64_t* accum_full = p_empty + 2;
  uint64_t* accum_empty = accum_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t idesc = idesc_f16(128, NR, true, /*a_mn=*/true, /*b_mn=*/false);
  const int item_cols = p.item_groups * 64;
  const int n_pairs = p.item_groups / 2;

  if (tid == 0) {
    for (int i = 0; i < kVCodeSlots; ++i) {
      mbar_init(&code_full[i], 1);
      mbar_init(&code_empty[i], 256);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&a_full[i], 256);
      mbar_init(&a_empty[i], 1);
      mbar_init(&p_full[i], 256);
      mbar_init(&p_empty[i], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(accum_empty, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer: code blocks
    if (lane == 0) {
      uint32_t c_iter = 0;
      for (int it = blockIdx.x; it < p.n_items && !*abort_flag; it += gridDim.x) {
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
        for (int t = tb; t < te && !*abort_flag; ++t) {
          const TileDesc tile = p.tiles[t];
          PairWalk walk;
          walk.begin(tile, p.groups, g0, p.item_groups);
          int lo, hi;
          while (walk.next(lo, hi) >= 0) {
            for (int half = 0; half < 2; ++half) {
              const int gi = half ? hi : lo;
              if (gi < 0) continue;
              const GroupRegs gr = load_group(&p.groups[gi]);
              if (gr.code_bytes > static_cast<uint32_t>(kVCodeSlot - 32) ||
                  static_cast<uint64_t>(gr.code_offset) + gr.code_bytes > p.code_size) {
                record_error(p.status, kErrBadDescriptor);
                *abort_flag = 1;
                break;
              }
              const int cs = c_iter % kVCodeSlots;
              if (c_iter >= kVCodeSlots &&
                  !mbar_wait(&code_empty[cs], ((c_iter / kVCodeSlots) - 1) & 1, p.status, kErrWaitEmpty)) {
                *abort_flag = 1;
                break;
              }
              stash_group(c_slots + (cs + 1) * kVCodeSlot, &p.groups[gi]);
              mbar_arrive_expect_tx(&code_full[cs], gr.code_bytes);
              bulk_load(c_slots + cs * kVCodeSlot, p.code + gr.code_offset, gr.code_bytes, &code_full[cs]);
              ++c_iter;
            }
            if (*abort_flag) break;
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t a_iter = 0, p_iter = 0, item_iter = 0;
      for (int it = blockIdx.x; it < p.n_items && !*abort_flag; it += gridDim.x) {
        const int tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
        if (item_iter > 0 && !mbar_wait(accum_empty, (item_iter - 1) & 1, p.status, kErrWaitAccumFree)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        uint32_t started = 0;  // pairs whose accumulator has been initialised in this item
        bool ok = true;
        for (int t = tb; t < te && ok; ++t) {
          const TileDesc tile = p.tiles[t];
          const int pb = p_iter & 1;
          if (!mbar_wait(&p_full[pb], (p_iter >> 1) & 1, p.status, kErrWaitA)) {
            ok = false;
            break;
          }
          PairWalk walk;
          walk.begin(tile, p.groups, g0, p.item_groups);
          int lo, hi, pair;
          while ((pair = walk.next(lo, hi)) >= 0) {
            const int slot = a_iter & 1;
            if (!mbar_wait(&a_full[slot], (a_iter >> 1) & 1, p.status, kErrWaitA)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = smem_u32(a_tiles + slot * kPairTile);
            const uint32_t p_base = smem_u32(p_tiles + pb * p_tile);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const uint64_t adesc = smem_desc_sw128(a_base + i * 2048, 16384, 1024);
              const uint64_t bdesc = smem_desc_sw128(p_base + (i >> 2) * (NR * 128) + (i & 3) * 32, 16, 1024);
              const uint32_t acc = ((started >> pair) & 1u) || i > 0 ? 1u : 0u;
              mma_f16(tmem + pair * NR, adesc, bdesc, idesc, acc);
            }
            started |= 1u << pair;
            mma_commit(&a_empty[slot]);
            ++a_iter;
          }
          if (!ok) break;
          mma_commit(&p_empty[pb]);
          ++p_iter;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mma_commit(accum_full);
        ++item_iter;
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ worker warps (P, decode, epilogue)
    const int u = tid - 128;
    const int r = u & 127;  // token row (decode) / token column (P)
    const int h = u >> 7;   // component half (decode) / row half (P)
    uint32_t c_iter = 0, a_iter = 0, p_iter = 0, item_iter = 0;
    for (int it = blockIdx.x; it < p.n_items && !*abort_flag; it += gridDim.x) {
      const int s = p.items[4 * it], tb = p.items[4 * it + 1], te = p.items[4 * it + 2], g0 = p.items[4 * it + 3];
      const int64_t m_s = p.seq_m[s];
      const float* sc = p.scores + p.seq_score_off[s];
      const float* stats = p.row_stats + static_cast<int64_t>(s) * p.n_q_heads * p.q_len * 4;
      uint32_t started = 0;
      for (int t = tb; t < te && !*abort_flag; ++t) {
        const TileDesc tile = p.tiles[t];
        // ---- P^T tile: rows x 128 tokens, bf16
        const int pb = p_iter & 1;
        if (p_iter >= 2 && !mbar_wait(&p_empty[pb], ((p_iter >> 1) - 1) & 1, p.status, kErrWaitEmpty)) {
          *abort_flag = 1;
          break;
        }
        {
          uint8_t* pt = p_tiles + pb * p_tile;
          const bool tok_ok = r < tile.n_tokens;
          const int sidx = tok_ok ? p.tok_sidx[tile.token_base + r] : 0;
          const int atom = r >> 6, chunk = (r & 63) >> 3, within = (r & 7) * 2;
          const int rows_half = NR / 2;
          for (int n = h * rows_half; n < (h + 1) * rows_half; ++n) {
            float prob = 0.f;
            if (tok_ok && n < p.n_rows) {
              const int row = p.row_begin + n;
              const float x = sc[static_cast<int64_t>(row) * m_s + sidx];
              prob = (x == -INFINITY) ? 0.f : expf(x - stats[row * 4]) * stats[row * 4 + 1];
            }
            *reinterpret_cast<__nv_bfloat16*>(pt + atom * (NR * 128) + sw128_offset(n, chunk) + within) =
                __float2bfloat16_rn(prob);
          }
          fence_async_shared();
          mbar_arrive(&p_full[pb]);
          ++p_iter;
        }
        // ---- coefficient pairs
        PairWalk walk;
        walk.begin(tile, p.groups, g0, p.item_groups);
        int lo, hi, pair;
        while ((pair = walk.next(lo, hi)) >= 0) {
          const int slot = a_iter & 1;
          if (a_iter >= 2 && !mbar_wait(&a_empty[slot], ((a_iter >> 1) - 1) & 1, p.status, kErrWaitEmpty)) {
            *abort_flag = 1;
            break;
          }
          uint8_t* a = a_tiles + slot * kPairTile;
          for (int half = 0; half < 2; ++half) {
            const int gi = half ? hi : lo;
            uint8_t* dst = a + half * 16384;
            uint32_t out[16];
            if (gi >= 0) {
              const int cs = c_iter % kVCodeSlots;
              if (!mbar_wait(&code_full[cs], (c_iter / kVCodeSlots) & 1, p.status, kErrWaitCodes)) {
                *abort_flag = 1;
                break;
              }
              const GroupRegs gr = stashed_group(c_slots + (cs + 1) * kVCodeSlot);
              decode_half(c_slots + cs * kVCodeSlot, gr, tile.n_tokens, r, h, out);
              mbar_arrive(&code_empty[cs]);
              ++c_iter;
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) out[i] = 0u;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k)
              *reinterpret_cast<uint4*>(dst + sw128_offset(r, 4 * h + k)) =
                  make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
          }
          if (*abort_flag) break;
          fence_async_shared();
          mbar_arrive(&a_full[slot]);
          ++a_iter;
          started |= 1u << pair;
        }
      }
      if (*abort_flag) break;
      // ---- epilogue (warps 4..7): TMEM -> partial sums
      if (warp < 8) {
        if (!mbar_wait(accum_full, item_iter & 1, p.status, kErrWaitAccum)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        const int c = (warp - 4) * 32 + lane;  // component within the pair == TMEM lane
        const uint32_t lane_base = static_cast<uint32_t>((warp - 4) * 32) << 16;
        float* dst = p.partial + static_cast<int64_t>(it) * NR * item_cols;
        for (int pair2 = 0; pair2 < n_pairs; ++pair2) {
          const bool live = (started >> pair2) & 1u;
          for (int n0 = 0; n0 < NR; n0 += 16) {
            uint32_t v[16];
            if (live) {
              tmem_ld16(tmem + lane_base + pair2 * NR + n0, v);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) v[i] = 0u;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i)
              dst[static_cast<int64_t>(n0 + i) * item_cols + pair2 * 128 + c] = __uint_as_float(v[i]);
          }
        }
        tc_fence_before();
        mbar_arrive(accum_empty);
      }
      ++item_iter;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, 512);
}

int run_value_weights(const ValueWeightParams& p, int grid, cudaStream_t stream) {
  if (p.n_rows_pad % 16 != 0 || p.n_rows_pad < 16 || p.n_rows_pad > 128 || p.n_rows > p.n_rows_pad)
    return kDkvErrConfig;
  if ((p.item_groups / 2) * p.n_rows_pad > 512 || p.item_groups % 2 != 0 || p.item_groups > 64) return kDkvErrConfig;
  if (p.n_items == 0) return kDkvOk;
  const int smem = 1024 + 2 * kPairTile + 2 * p.n_rows_pad * 256 + kVCodeSlots * kVCodeSlot + 32 * 8;
  if (cudaFuncSetAttribute(value_weights_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kDkvErrCuda;
  value_weights_kernel<<<grid, kVThreads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
