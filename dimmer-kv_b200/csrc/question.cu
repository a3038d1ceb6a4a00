// question.cu — question-time scoring, top-k selection and the cold-plane merge of refined tokens.
//
// importance : replaces the scoring branch of dimmer_attention (scripts/dimmer.py:62-75) as summed by
//              question_importance (scripts/progressive.py:239-254): for every context token, the
//              attention probability it receives, summed over query heads and question rows (and, by
//              repeated calls, over layers). Compressed tokens are read from the fp32 score buffer and
//              the softmax statistics of the layer; exact tokens from their probabilities.
// topk       : replaces importance[start:end].topk(count) (scripts/methods.py:246-247) with a radix
//              select on order-preserving keys; equal values are taken by lowest position (torch.topk
//              leaves ties unspecified). Output: selected positions in ascending order.
// refine     : replaces ProgressiveCache.refine's decode of the selected rows at all planes
//              (scripts/progressive.py:224-236): the hot planes of each selected token (from the packed
//              hot stream) and its cold planes (staged from pinned host memory) are merged into new
//              full-precision blocks, one 8-plane block per (refined tile, group).
#include <cfloat>
#include <cmath>

#include "dkv_format.cuh"
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

// ------------------------------------------------------------------ importance
__global__ void __launch_bounds__(256) importance_kernel(const ImportanceParams p) {
  extern __shared__ float st[];  // [rows][2]: max, 1/sum
  const int s = blockIdx.y;
  const int rows = p.n_q_heads * p.q_len;
  const float* stats = p.row_stats + static_cast<int64_t>(s) * rows * 4;
  for (int r = threadIdx.x; r < rows; r += blockDim.x) {
    st[2 * r] = stats[4 * r];
    st[2 * r + 1] = stats[4 * r + 1];
  }
  __syncthreads();
  const int64_t m_s = p.seq_m[s];
  const int64_t n = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (n < m_s) {
    const float* sc = p.scores + p.seq_score_off[s] + n;
    float acc = 0.f;
    for (int r = 0; r < rows; ++r) {
      const float x = sc[static_cast<int64_t>(r) * m_s];
      if (x != -INFINITY) acc += expf(x - st[2 * r]) * st[2 * r + 1];
    }
    p.imp_compressed[p.seq_k_base[s] + n] += acc;
  }
  if (blockIdx.x == 0) {
    for (int e = threadIdx.x; e < p.n_exact; e += blockDim.x) {
      float acc = 0.f;
      for (int r = 0; r < rows; ++r) acc += p.p_exact[(static_cast<int64_t>(s) * rows + r) * p.n_exact + e];
      p.imp_exact[static_cast<int64_t>(s) * p.n_exact + e] += acc;
    }
  }
}

int run_importance(const ImportanceParams& p, int max_m, cudaStream_t stream) {
  if (p.n_seq == 0 || max_m == 0) return kDkvOk;
  const int rows = p.n_q_heads * p.q_len;
  const int smem = rows * 2 * 4;
  if (smem > 200 * 1024) return kDkvErrConfig;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(importance_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kDkvErrCuda;
  dim3 grid((max_m + 255) / 256, p.n_seq);
  importance_kernel<<<grid, 256, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

// ------------------------------------------------------------------ top-k
namespace {
constexpr int kTopkThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float x) {
  const uint32_t u = __float_as_uint(x) == 0x80000000u ? 0u : __float_as_uint(x);  // -0 ties with +0
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);  // larger float -> larger key
}

// Radix-select the value of rank `want` (1-based) among the selected elements, in descending order of
// `key(i)` when descending, else ascending. hist is 256 shared counters. Returns (threshold, rank left).
template <typename KeyFn, typename SelFn>
__device__ void radix_select(int n, KeyFn key, SelFn sel, bool descending, uint32_t want, unsigned* hist,
                             uint32_t* result) {
  uint32_t prefix = 0, mask = 0;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int b = threadIdx.x; b < 256; b += blockDim.x) hist[b] = 0;
    __syncthreads();
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      if (!sel(i)) continue;
      const uint32_t k = key(i);
      if ((k & mask) == prefix) atomicAdd(&hist[(k >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      uint32_t cum = 0;
      int chosen = descending ? 0 : 255;
      for (int step = 0; step < 256; ++step) {
        const int b = descending ? 255 - step : step;
        if (cum + hist[b] >= want) {
          chosen = b;
          break;
        }
        cum += hist[b];
      }
      want -= cum;
      result[0] = prefix | (static_cast<uint32_t>(chosen) << shift);
      result[1] = want;
    }
    __syncthreads();
    prefix = result[0];
    want = result[1];
    mask |= 255u << shift;
    __syncthreads();
  }
}
}  // namespace

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(const TopkParams p) {
  __shared__ unsigned hist[256];
  __shared__ uint32_t res[2];
  __shared__ unsigned count;
  extern __shared__ int32_t picked[];  // [k]
  const int s = blockIdx.x;
  const int base = p.seq_k_base[s];
  const int n = p.seq_m[s];
  const int k = p.counts[s];
  int32_t* out = p.out + p.out_offset[s];
  const float* imp = p.importance + base;
  const int32_t* pos = p.positions + base;
  auto valid = [&](int i) { return pos[i] >= 0; };
  auto vkey = [&](int i) { return order_key(imp[i]); };
  if (k <= 0 || n <= 0) return;
  // Threshold key T of the k-th largest value, and how many elements equal to T are taken.
  radix_select(n, vkey, valid, true, static_cast<uint32_t>(k), hist, res);
  const uint32_t T = res[0];
  const uint32_t take_eq = res[1];
  // Among the elements equal to T, the take_eq lowest positions: radix-select the position bound.
  auto tie = [&](int i) { return valid(i) && vkey(i) == T; };
  auto pkey = [&](int i) { return static_cast<uint32_t>(pos[i]); };
  radix_select(n, pkey, tie, false, take_eq, hist, res);
  const uint32_t P = res[0];
  if (threadIdx.x == 0) count = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    if (!valid(i)) continue;
    const uint32_t key = vkey(i);
    if (key > T || (key == T && static_cast<uint32_t>(pos[i]) <= P)) {
      const unsigned slot = atomicAdd(&count, 1u);
      if (slot < static_cast<unsigned>(k)) picked[slot] = pos[i];
    }
  }
  __syncthreads();
  const int got = min(static_cast<int>(count), k);
  // Ascending positions: every element's rank is the number of smaller picked positions.
  for (int i = threadIdx.x; i < got; i += blockDim.x) {
    int rank = 0;
    const int v = picked[i];
    for (int j = 0; j < got; ++j) rank += picked[j] < v;
    out[rank] = v;
  }
  if (threadIdx.x == 0 && got != k && p.status != nullptr) atomicCAS(p.status, 0, kErrBadDescriptor);
}

int run_topk(const TopkParams& p, int max_k, cudaStream_t stream) {
  if (p.n_seq == 0) return kDkvOk;
  if (max_k > 16384) return kDkvErrConfig;
  const int smem = max_k * 4;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(topk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kDkvErrCuda;
  topk_kernel<<<p.n_seq, kTopkThreads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

// ------------------------------------------------------------------ refine merge
// One thread per (selected token, refined group). The refined segment's blocks are uniform: every
// token holds 8 planes on every group, so block (tile j, group g) = headers (n x 4 B, padded to 8)
// then 8 planes of n words; the host laid out the descriptors and offsets.
__global__ void __launch_bounds__(256) refine_kernel(const RefineParams p) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(p.n_selected) * p.n_groups) return;
  const int i = static_cast<int>(idx / p.n_groups);  // selected token
  const int gl = static_cast<int>(idx % p.n_groups);  // refined group (local)
  const int tile_j = i / kTileTokens, r = i % kTileTokens;
  const int n_tile = min(kTileTokens, p.n_selected - tile_j * kTileTokens);
  const GroupDesc& od = p.out_groups[tile_j * p.n_groups + gl];
  uint8_t* blk = p.out_code + od.code_offset;
  const uint32_t group = od.group;
  // Hot block of this token and group (if the hot tier holds a plane of it).
  const TileDesc ht = p.hot_tiles[p.hot_tile[i]];
  const int hr = p.hot_row[i];
  int m_hot = 0;
  const uint8_t* hblk = nullptr;
  GroupRegs hg{};
  for (int d = 0; d < ht.n_groups; ++d) {
    const GroupRegs g = load_group(&p.hot_groups[ht.group_base + d]);
    if (g.group == group) {
      hg = g;
      hblk = p.hot_code + g.code_offset;
      m_hot = planes_of(g, hr, ht.n_tokens);
      break;
    }
  }
  if (m_hot == kMaxPlanes || m_hot > 8) {  // raw hot blocks are never refined
    record_error(p.status, kErrBadDescriptor);
    return;
  }
  // Cold record of this token and group: header + the 8 plane words of the full code.
  const uint64_t* cold = p.cold_words + (static_cast<int64_t>(i) * p.n_groups + gl) * 8;
  uint32_t header = p.cold_headers[static_cast<int64_t>(i) * p.n_groups + gl];
  uint64_t words[8];
  for (int j = 0; j < 8; ++j) words[j] = cold[j];
  if (m_hot > 0) {
    header = *reinterpret_cast<const uint32_t*>(hblk + static_cast<uint32_t>(hr - first_at(hg, 0)) * 4u);
    uint32_t seg = ((static_cast<uint32_t>(ht.n_tokens) - first_at(hg, 0)) * 4u + 7u) & ~7u;
    for (int j = 0; j < m_hot; ++j) {
      const uint32_t fj = first_at(hg, j);
      words[j] = *reinterpret_cast<const uint64_t*>(hblk + seg + (static_cast<uint32_t>(hr) - fj) * 8u);
      seg += (static_cast<uint32_t>(ht.n_tokens) - fj) * 8u;
    }
  }
  *reinterpret_cast<uint32_t*>(blk + r * 4) = header;
  const uint32_t seg0 = (static_cast<uint32_t>(n_tile) * 4u + 7u) & ~7u;
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint64_t*>(blk + seg0 + static_cast<uint32_t>(j * n_tile + r) * 8u) = words[j];
}

int run_refine(const RefineParams& p, cudaStream_t stream) {
  const int64_t total = static_cast<int64_t>(p.n_selected) * p.n_groups;
  if (total == 0) return kDkvOk;
  refine_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
