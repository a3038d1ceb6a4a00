// key_scores.cu — per-layer key rebuild fused with RoPE and the query-key products.
//
// Replaces, for one layer and a whole batch of compressed conversations:
//   CompressedContext._keys   (scripts/compressed_attention.py:105-111)  C_b @ B_l + mean, RoPE
//   the compressed half of    CompressedContext.attend (:118-120)        einsum(q, K) * scaling
// without materialising the rebuilt keys anywhere but TMEM.
//
// One work item = (tile of <=128 key tokens of one conversation, block of NB key columns).
// Per coefficient group (64 PCA components) of the tile:
//   producer warp    : cp.async.bulk of the tile's plane block -> shared; TMA of the basis rows
//                      (NB columns x 64 components, 128B swizzle) -> shared
//   8 unpack warps   : bit-plane decode -> bf16 A tile (128 tokens x 64 components, 128B swizzle)
//   MMA warp         : tcgen05.mma M=128, N=min(NB,256), K=16 x 4, fp32 accumulator in TMEM
// After the tile's last group the 4 epilogue warps read the accumulator (one token per thread),
// add the mean, apply RoPE with the token's position, dot with the query heads of every KV head
// in the block and write fp32 scores.
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {

constexpr int kThreads = 512;
constexpr int kStagesAB = 2;
constexpr int kStagesC = 3;
constexpr int kCodeSlot = 17408;  // >= headers (512 B) + 16 planes x 1 KB
constexpr int kATile = 16384;     // 128 rows x 128 B

__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

template <int NB>
struct KeySmem {
  static constexpr int kBStage = NB * 128;
  static constexpr int kA = 0;
  static constexpr int kB = kA + kStagesAB * kATile;
  static constexpr int kC = kB + kStagesAB * kBStage;
  static constexpr int kQ = kC + kStagesC * kCodeSlot;
};

}  // namespace

template <int D, int NB, int G>
__global__ void __launch_bounds__(kThreads, 1)
    key_scores_kernel(const __grid_constant__ CUtensorMap bmap, const KeyScoreParams p) {
  constexpr int kHeads = NB / D;           // KV heads per work item
  constexpr int kNMma = NB > 256 ? 256 : NB;
  constexpr int kNHalf = NB / kNMma;
  constexpr uint32_t kIdesc = idesc_f16(128, kNMma, true, false, false);
  using L = KeySmem<NB>;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* a_tiles = smem + L::kA;
  uint8_t* b_tiles = smem + L::kB;
  uint8_t* c_slots = smem + L::kC;
  float* q_s = reinterpret_cast<float*>(smem + L::kQ);         // [kHeads * G][D]
  float* mean_s = q_s + kHeads * G * D;                         // [NB]
  uint64_t* bars = reinterpret_cast<uint64_t*>(mean_s + NB);
  uint64_t* code_full = bars;                                   // [kStagesC]
  uint64_t* code_empty = code_full + kStagesC;                  // [kStagesC]
  uint64_t* b_full = code_empty + kStagesC;                     // [kStagesAB]
  uint64_t* a_full = b_full + kStagesAB;                        // [kStagesAB]
  uint64_t* stage_empty = a_full + kStagesAB;                   // [kStagesAB]
  uint64_t* accum_full = stage_empty + kStagesAB;
  uint64_t* accum_empty = accum_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accum_empty + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nblocks = p.n_cols / NB;

  if (tid == 0) {
    for (int i = 0; i < kStagesC; ++i) {
      mbar_init(&code_full[i], 1);
      mbar_init(&code_empty[i], 256);
    }
    for (int i = 0; i < kStagesAB; ++i) {
      mbar_init(&b_full[i], 1);
      mbar_init(&a_full[i], 256);
      mbar_init(&stage_empty[i], 1);
    }
    mbar_init(accum_full, 1);
    mbar_init(accum_empty, 128);
    *abort_flag = 0;
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
      uint32_t c_iter = 0, s_iter = 0;
      for (int it = blockIdx.x; it < p.n_items && !*abort_flag; it += gridDim.x) {
        const int item = p.items[it];
        const int ti = item / nblocks, nblk = item % nblocks;
        const TileDesc tile = p.tiles[ti];
        for (int gi = 0; gi < tile.n_groups && !*abort_flag; ++gi) {
          const GroupRegs gr = load_group(&p.groups[tile.group_base + gi]);
          if (gr.code_bytes > static_cast<uint32_t>(kCodeSlot) ||
              static_cast<uint64_t>(gr.code_offset) + gr.code_bytes > p.code_size || gr.group >= p.n_union_groups) {
            record_error(p.status, kErrBadDescriptor);
            *abort_flag = 1;
            break;
          }
          const int cs = c_iter % kStagesC;
          if (c_iter >= kStagesC &&
              !mbar_wait(&code_empty[cs], ((c_iter / kStagesC) - 1) & 1, p.status, kErrWaitEmpty)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&code_full[cs], gr.code_bytes);
          bulk_load(c_slots + cs * kCodeSlot, p.code + gr.code_offset, gr.code_bytes, &code_full[cs]);
          ++c_iter;
          const int ss = s_iter % kStagesAB;
          if (s_iter >= kStagesAB &&
              !mbar_wait(&stage_empty[ss], ((s_iter / kStagesAB) - 1) & 1, p.status, kErrWaitEmpty)) {
            *abort_flag = 1;
            break;
          }
          mbar_arrive_expect_tx(&b_full[ss], L::kBStage);
          for (int hf = 0; hf < kNHalf; ++hf)
            tma_load_2d(b_tiles + ss * L::kBStage + hf * kNMma * 128, &bmap, &b_full[ss],
                        static_cast<int>(gr.group) * kGroup, p.layer * p.n_cols + nblk * NB + hf * kNMma);
          ++s_iter;
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t s_iter = 0, item_iter = 0;
      for (int it = blockIdx.x; it < p.n_items && !*abort_flag; it += gridDim.x) {
        const int item = p.items[it];
        const TileDesc tile = p.tiles[item / nblocks];
        if (item_iter > 0 && !mbar_wait(accum_empty, (item_iter - 1) & 1, p.status, kErrWaitAccumFree)) {
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        bool ok = true;
        for (int gi = 0; gi < tile.n_groups; ++gi) {
          const int ss = s_iter % kStagesAB;
          const uint32_t par = (s_iter / kStagesAB) & 1;
          if (!mbar_wait(&a_full[ss], par, p.status, kErrWaitA) ||
              !mbar_wait(&b_full[ss], par, p.status, kErrWaitBasis)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_base = smem_u32(a_tiles + ss * kATile);
          const uint32_t b_base = smem_u32(b_tiles + ss * L::kBStage);
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint64_t adesc = smem_desc_sw128(a_base + 32 * k, 16, 1024);
#pragma unroll
            for (int hf = 0; hf < kNHalf; ++hf) {
              const uint64_t bdesc = smem_desc_sw128(b_base + hf * kNMma * 128 + 32 * k, 16, 1024);
              mma_f16(tmem + hf * kNMma, adesc, bdesc, kIdesc, (gi > 0 || k > 0) ? 1u : 0u);
            }
          }
          mma_commit(&stage_empty[ss]);
          ++s_iter;
        }
        if (!ok) {
          *abort_flag = 1;
          break;
        }
        mma_commit(accum_full);
        ++item_iter;
      }
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ unpack warps
    const int u = tid - 128;
    const int r = u & 127;
    const int h = u >> 7;
    uint32_t c_iter = 0, s_iter = 0;
    for (int it = blockIdx.x; it < p.n_items && !*abort_flag; it += gridDim.x) {
      const int item = p.items[it];
      const TileDesc tile = p.tiles[item / nblocks];
      for (int gi = 0; gi < tile.n_groups; ++gi) {
        const GroupRegs gr = load_group(&p.groups[tile.group_base + gi]);
        const int cs = c_iter % kStagesC;
        const int ss = s_iter % kStagesAB;
        if (!mbar_wait(&code_full[cs], (c_iter / kStagesC) & 1, p.status, kErrWaitCodes)) {
          *abort_flag = 1;
          break;
        }
        if (s_iter >= kStagesAB &&
            !mbar_wait(&stage_empty[ss], ((s_iter / kStagesAB) - 1) & 1, p.status, kErrWaitEmpty)) {
          *abort_flag = 1;
          break;
        }
        uint32_t out[16];
        decode_half(c_slots + cs * kCodeSlot, gr, tile.n_tokens, r, h, out);
        uint8_t* a = a_tiles + ss * kATile;
#pragma unroll
        for (int k = 0; k < 4; ++k)
          *reinterpret_cast<uint4*>(a + sw128_offset(r, 4 * h + k)) =
              make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
        fence_async_shared();
        mbar_arrive(&a_full[ss]);
        mbar_arrive(&code_empty[cs]);
        ++c_iter;
        ++s_iter;
      }
      if (*abort_flag) break;
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ epilogue warps
    const int r = tid - 384;                       // TMEM lane == tile token row
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t item_iter = 0;
    for (int it = blockIdx.x; it < p.n_items && !*abort_flag; it += gridDim.x) {
      const int item = p.items[it];
      const int ti = item / nblocks, nblk = item % nblocks;
      const TileDesc tile = p.tiles[ti];
      if (!mbar_wait(accum_full, item_iter & 1, p.status, kErrWaitAccum)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int s = tile.seq;
      const bool valid = r < tile.n_tokens;
      const int token = tile.token_base + (valid ? r : 0);
      int pos = p.tok_pos[token];
      const bool hidden = pos < 0;  // refined or evicted token: excluded from the softmax
      pos = hidden ? 0 : (pos >= p.max_pos ? p.max_pos - 1 : pos);
      const __nv_bfloat16* cosrow = p.cos_t + static_cast<int64_t>(pos) * (D / 2);
      const __nv_bfloat16* sinrow = p.sin_t + static_cast<int64_t>(pos) * (D / 2);
      const int64_t m_s = p.seq_m[s];
      float* out_base = p.scores + p.seq_score_off[s];
      const int kv0 = nblk * kHeads;
      for (int qi = 0; qi < p.q_len; ++qi) {
        named_sync(1, 128);
        // Stage this query row for the block's heads, and the block's mean slice.
        for (int i = r; i < kHeads * G * D; i += 128) {
          const int hq = kv0 * G + i / D;  // query head
          const int d = i % D;
          q_s[i] = __bfloat162float(p.query[((static_cast<int64_t>(s) * p.n_q_heads + hq) * p.q_len + qi) * D + d]);
        }
        if (qi == 0) {
          const __nv_bfloat16* mrow = p.mean + static_cast<int64_t>(s) * p.mean_seq_stride +
                                      static_cast<int64_t>(p.layer) * p.n_cols + nblk * NB;
          for (int i = r; i < NB; i += 128) mean_s[i] = __bfloat162float(mrow[i]);
        }
        named_sync(1, 128);
#pragma unroll 1
        for (int hh = 0; hh < kHeads; ++hh) {
          float acc[G];
#pragma unroll
          for (int j = 0; j < G; ++j) acc[j] = 0.f;
#pragma unroll 1
          for (int c = 0; c < D / 2; c += 16) {
            float cs[16], sn[16];
            {
              const uint4* cp = reinterpret_cast<const uint4*>(cosrow + c);
              const uint4* sp = reinterpret_cast<const uint4*>(sinrow + c);
              uint4 cv[2] = {__ldg(cp), __ldg(cp + 1)};
              uint4 sv[2] = {__ldg(sp), __ldg(sp + 1)};
              const __nv_bfloat16* cb = reinterpret_cast<const __nv_bfloat16*>(cv);
              const __nv_bfloat16* sb = reinterpret_cast<const __nv_bfloat16*>(sv);
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                cs[i] = __bfloat162float(cb[i]);
                sn[i] = __bfloat162float(sb[i]);
              }
            }
            uint32_t x1[16], x2[16];
            if (tile.n_groups > 0) {
              tmem_ld16(tmem + lane_base + hh * D + c, x1);
              tmem_ld16(tmem + lane_base + hh * D + D / 2 + c, x2);
              tmem_ld_wait();
            } else {
#pragma unroll
              for (int i = 0; i < 16; ++i) x1[i] = x2[i] = 0u;
            }
            float r1[16], r2[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float k1 = __uint_as_float(x1[i]) + mean_s[hh * D + c + i];
              const float k2 = __uint_as_float(x2[i]) + mean_s[hh * D + D / 2 + c + i];
              r1[i] = k1 * cs[i] - k2 * sn[i];
              r2[i] = k2 * cs[i] + k1 * sn[i];
            }
#pragma unroll
            for (int j = 0; j < G; ++j) {
              const float* qrow = q_s + (hh * G + j) * D;
              float a = 0.f;
#pragma unroll
              for (int i = 0; i < 16; ++i) a += qrow[c + i] * r1[i] + qrow[D / 2 + c + i] * r2[i];
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

template <int D, int NB, int G>
static int launch_key_scores(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  using L = KeySmem<NB>;
  const int smem = 1024 + L::kQ + (NB / D) * G * D * 4 + NB * 4 + 16 * 8 + 16;
  if (smem > 232448) return kDkvErrConfig;
  cudaError_t e = cudaFuncSetAttribute(key_scores_kernel<D, NB, G>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return kDkvErrCuda;
  key_scores_kernel<D, NB, G><<<grid, kThreads, smem, stream>>>(bmap, p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

template <int D, int NB>
static int dispatch_g(const CUtensorMap& bmap, const KeyScoreParams& p, int grid, cudaStream_t stream) {
  switch (p.q_per_kv) {
    case 1: return launch_key_scores<D, NB, 1>(bmap, p, grid, stream);
    case 2: return launch_key_scores<D, NB, 2>(bmap, p, grid, stream);
    case 3: return launch_key_scores<D, NB, 3>(bmap, p, grid, stream);
    case 4: return launch_key_scores<D, NB, 4>(bmap, p, grid, stream);
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
