// unpack.cu — ragged bit-plane unpack to dense PCA coefficients.
//
// Replaces progressive.dequantize (scripts/progressive.py:47-55) for a packed stream, and the
// ladder decode of kvtc.quantize_groups (scripts/kvtc.py:78): every token of every tile is
// decoded at its own plane count and written as a dense row of out_cols coefficients (stream
// order; column = union group * 64 + component; zeros for groups the tile does not hold).
//
// One CTA per tile. A producer warp stages the tile's plane blocks into a ring of shared-memory
// slots with cp.async.bulk (completion on mbarriers); eight decode warps take two threads per
// token (32 components each), decode from shared memory, and write through a per-warp staging
// buffer so that every store instruction covers whole 32-byte sectors: the kernel is bound by
// the HBM write of the dense output (2 or 4 bytes per component) plus the code read.
#include "dkv_format.cuh"
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {

constexpr int kUnpackSlots = 4;
constexpr int kUnpackDecodeThreads = 256;
constexpr int kUnpackThreads = kUnpackDecodeThreads + 32;

// RAW: the stream holds raw (16-plane) blocks of up to 16896 bytes (128 headers + 16 planes x 128
// words); otherwise blocks hold at most 8 planes (<= 8704 bytes) and the smaller slots let more CTAs
// share an SM.
template <bool BF16, bool RAW>
struct UnpackSmem {
  static constexpr int kSlotBytes = RAW ? 16896 : 8704;
  static constexpr int kSlotStride = kSlotBytes + 32;          // the block, then its descriptor
  static constexpr int kHalfBytes = BF16 ? 64 : 128;           // 32 components of one row
  static constexpr int kStageWarp = 32 * kHalfBytes;           // one warp's 32 rows
  static constexpr int kStage = kUnpackSlots * kSlotStride;
  static constexpr int kBars = kStage + 8 * kStageWarp;
  static constexpr int kBytes = kBars + 2 * kUnpackSlots * 8 + 16;
};

// Store 32 rows x (32 components) held one row per lane (in regs, 16 B chunks) to global memory:
// through the warp's staging buffer (chunk index XOR-swizzled against bank conflicts) so that each
// store instruction writes whole sectors (4 lanes per 64-byte row half for bf16, 8 per 128 bytes
// for fp32). Rows at or past n_valid are not written.
template <bool BF16>
__device__ __forceinline__ void store_rows(uint8_t* stage, const uint4 (&chunks)[BF16 ? 4 : 8],
                                           uint8_t* out_row0, int64_t row_stride_bytes, int lane, int n_valid) {
  constexpr int kC = BF16 ? 4 : 8;  // 16-byte chunks per row half
  const int sw = BF16 ? ((lane >> 1) & 3) : (lane & 7);
#pragma unroll
  for (int c = 0; c < kC; ++c)
    *reinterpret_cast<uint4*>(stage + lane * (kC * 16) + ((c ^ sw) * 16)) = chunks[c];
  __syncwarp();
#pragma unroll
  for (int j = 0; j < kC; ++j) {
    const int k = lane + 32 * j;
    const int row = k / kC;
    const int c = k % kC;
    const int swr = BF16 ? ((row >> 1) & 3) : (row & 7);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + row * (kC * 16) + ((c ^ swr) * 16));
    if (row < n_valid) *reinterpret_cast<uint4*>(out_row0 + row * row_stride_bytes + c * 16) = v;
  }
  __syncwarp();
}

template <bool BF16>
__device__ __forceinline__ void store_zero_rows(uint8_t* out_row0, int64_t row_stride_bytes, int lane, int n_valid) {
  constexpr int kC = BF16 ? 4 : 8;
#pragma unroll
  for (int j = 0; j < kC; ++j) {
    const int k = lane + 32 * j;
    const int row = k / kC;
    if (row < n_valid)
      *reinterpret_cast<uint4*>(out_row0 + row * row_stride_bytes + (k % kC) * 16) = make_uint4(0u, 0u, 0u, 0u);
  }
}

}  // namespace

template <bool BF16, bool RAW, bool F16>
__global__ void __launch_bounds__(kUnpackThreads, BF16 ? 4 : 1) unpack_kernel(const UnpackParams p) {
  using S = UnpackSmem<BF16, RAW>;
  constexpr int kUnpackSlotBytes = S::kSlotBytes;
  constexpr int kC = S::kHalfBytes / 16;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBars);
  uint64_t* empty = full + kUnpackSlots;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + kUnpackSlots);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed: no work
  const TileDesc tile = p.tiles[blockIdx.x];
  const int n_union = static_cast<int>(p.out_cols / kGroup);
  if (tile.n_tokens < 1 || tile.n_tokens > kTileTokens || tile.n_groups < 0 || tile.n_groups > n_union) {
    if (tid == 0) record_error(p.status, kSiteUnpack + kErrBadDescriptor);
    return;  // uniform over the CTA: nothing initialised yet
  }
  if (tid == 0) {
    for (int i = 0; i < kUnpackSlots; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kUnpackDecodeThreads);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == 8) {
    // ------------------------------------------------------------ producer: blocks in tile order
    if (lane == 0) {
      int issued = 0;
      for (int gi = 0; gi < tile.n_groups && !*abort_flag; ++gi) {
        const GroupRegs gr = load_group(&p.groups[tile.group_base + gi]);
        if (gr.code_bytes == 0 || gr.code_bytes > static_cast<uint32_t>(kUnpackSlotBytes) || (gr.code_bytes & 15u) ||
            (gr.code_offset & 15u) || static_cast<uint64_t>(gr.code_offset) + gr.code_bytes > p.code_size) {
          record_error(p.status, kSiteUnpack + kErrBadDescriptor);
          *abort_flag = 1;
          break;
        }
        const int s = issued % kUnpackSlots;
        if (issued >= kUnpackSlots &&
            !mbar_wait(&empty[s], ((issued / kUnpackSlots) - 1) & 1, p.status, kSiteUnpack + kErrWaitEmpty, abort_flag)) {
          *abort_flag = 1;
          break;
        }
        // The block's descriptor goes into the slot's tail before the copy is issued; the decoders read
        // it after the slot's barrier completes (arrive releases, the wait acquires).
        uint4* stash = reinterpret_cast<uint4*>(smem + s * S::kSlotStride + kUnpackSlotBytes);
        const uint4* src = reinterpret_cast<const uint4*>(&p.groups[tile.group_base + gi]);
        stash[0] = __ldg(src);
        stash[1] = __ldg(src + 1);
        mbar_arrive_expect_tx(&full[s], gr.code_bytes);
        bulk_load(smem + s * S::kSlotStride, p.code + gr.code_offset, gr.code_bytes, &full[s]);
        ++issued;
      }
      // Drain: the CTA must not exit with a copy into its shared memory in flight.
      const int first = issued > kUnpackSlots ? issued - kUnpackSlots : 0;
      for (int i = first; i < issued; ++i)
        mbar_wait(&full[i % kUnpackSlots], (i / kUnpackSlots) & 1, p.status, kSiteUnpack + kErrWaitCodes);
    }
    return;
  }

  // -------------------------------------------------------------- decode warps
  // Thread (r, h): token row r of the tile, components 32h..32h+31 of each group. Warp w holds rows
  // 32 (w % 4) .. +31 of half h = w / 4 and stores them itself.
  const int r = tid & 127;
  const int h = tid >> 7;
  const int row0 = (warp & 3) * 32;
  const int n_valid = tile.n_tokens - row0;  // rows of this warp inside the tile (may be <= 0)
  uint8_t* stage = smem + S::kStage + warp * S::kStageWarp;
  const int64_t stride = p.out_cols * (BF16 ? 2 : 4);
  const int64_t first_row = p.out_tile_rows > 0 ? static_cast<int64_t>(blockIdx.x) * p.out_tile_rows : tile.token_base;
  uint8_t* out_base = reinterpret_cast<uint8_t*>(p.out) + (first_row + row0) * stride +
                      static_cast<int64_t>(h) * S::kHalfBytes;
  // Blocks arrive in the tile's order (ascending union group); the groups before each block and after
  // the last one are written as zeros.
  int g_done = 0;  // groups [0, g_done) of the rows are written
  for (int i = 0; i < tile.n_groups; ++i) {
    const int s = i % kUnpackSlots;
    // The warp leaves together (its stores end in __syncwarp): one lane giving up ends the warp.
    const bool landed = mbar_wait(&full[s], (i / kUnpackSlots) & 1, p.status, kSiteUnpack + kErrWaitCodes, abort_flag);
    if (!__all_sync(0xffffffffu, landed)) {
      *abort_flag = 1;
      return;
    }
    const uint8_t* blk = smem + s * S::kSlotStride;
    const uint4* stash = reinterpret_cast<const uint4*>(blk + kUnpackSlotBytes);
    const GroupRegs gr = group_from_words(stash[0], stash[1]);
    const int g = static_cast<int>(gr.group);
    if (g < g_done || g >= n_union) {  // descriptors out of union order, or a group past out_cols / 64
      record_error(p.status, kSiteUnpack + kErrBadDescriptor);
      *abort_flag = 1;
      return;
    }
    for (; g_done < g; ++g_done)
      if (n_valid > 0) store_zero_rows<BF16>(out_base + static_cast<int64_t>(g_done) * kGroup * (BF16 ? 2 : 4), stride,
                                             lane, n_valid);
    uint4 chunks[kC];
    if (BF16) {
      uint32_t out[16];
      decode_half<F16>(blk, gr, tile.n_tokens, r, h, out);
#pragma unroll
      for (int k = 0; k < 4; ++k) chunks[k] = make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
    } else {
      float out[32];
      decode_half_f32<F16>(blk, gr, tile.n_tokens, r, h, out);
#pragma unroll
      for (int k = 0; k < kC; ++k)
        chunks[k] = make_uint4(__float_as_uint(out[4 * k]), __float_as_uint(out[4 * k + 1]),
                               __float_as_uint(out[4 * k + 2]), __float_as_uint(out[4 * k + 3]));
    }
    mbar_arrive(&empty[s]);
    if (n_valid > 0)
      store_rows<BF16>(stage, chunks, out_base + static_cast<int64_t>(g) * kGroup * (BF16 ? 2 : 4), stride, lane,
                       n_valid);
    g_done = g + 1;
  }
  for (; g_done < n_union; ++g_done)
    if (n_valid > 0)
      store_zero_rows<BF16>(out_base + static_cast<int64_t>(g_done) * kGroup * (BF16 ? 2 : 4), stride, lane, n_valid);
}

template <bool BF16, bool RAW, bool F16>
static int launch_unpack3(const UnpackParams& p, cudaStream_t stream) {
  const int smem = UnpackSmem<BF16, RAW>::kBytes + 128;
  if (cudaFuncSetAttribute(unpack_kernel<BF16, RAW, F16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
      cudaSuccess)
    return kDkvErrCuda;
  unpack_kernel<BF16, RAW, F16><<<p.n_tiles, kUnpackThreads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

// BF16: 16-bit output (in fp16 with p.f16, else bf16); otherwise float32. p.f16 also says that raw blocks hold
// fp16 patterns.
template <bool BF16, bool RAW>
static int launch_unpack(const UnpackParams& p, cudaStream_t stream) {
  return p.f16 ? launch_unpack3<BF16, RAW, true>(p, stream) : launch_unpack3<BF16, RAW, false>(p, stream);
}

int run_unpack(const UnpackParams& p, cudaStream_t stream) {
  if (p.n_tiles == 0) return kDkvOk;
  if (p.out_cols % 64 != 0 || p.out_cols <= 0) return kDkvErrArgs;
  if (reinterpret_cast<uintptr_t>(p.out) & 15u) return kDkvErrArgs;
  if (p.out_tile_rows != 0 && p.out_tile_rows != kTileTokens) return kDkvErrArgs;
  const bool raw = p.max_planes <= 0 || p.max_planes > 8;
  if (p.out_bf16)
    return raw ? launch_unpack<true, true>(p, stream) : launch_unpack<true, false>(p, stream);
  return raw ? launch_unpack<false, true>(p, stream) : launch_unpack<false, false>(p, stream);
}

}  // namespace dkv
