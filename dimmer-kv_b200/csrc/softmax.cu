// softmax.cu — one softmax over compressed and exact tokens, as statistics.
//
// Replaces the normalisation of CompressedContext.attend (scripts/compressed_attention.py:122-128):
// scores_e = q . k_exact * scaling (+ mask), then softmax over cat(scores_c, scores_e) in float32.
// Instead of materialising probabilities for the compressed tokens, each (conversation, query
// head, query row) gets its row maximum, 1 / sum of exponentials and the probability mass of the
// compressed part; the exact tokens' probabilities are written out (there are few of them).
// Split-K over GPUs (one conversation's tokens sharded): mode kSoftmaxLocal writes each row's local
// (max, sum of exponentials); after the shards are merged into the global (max, 1 / sum), mode
// kSoftmaxGlobal computes the compressed mass and the exact-token probabilities with them, so every
// shard rounds its probabilities exactly as one softmax over all tokens would.
#include <cfloat>
#include <cmath>
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"
#include "dkv_kernels.h"

namespace dkv {

namespace {
constexpr int kSoftmaxThreads = 256;

// x rounded to the cache dtype (the reference's p.to(dtype)), bf16 or fp16 by the call's flag.
__device__ __forceinline__ float dtype_round(float x, int f16) { return f16 ? round_half<true>(x) : round_half<false>(x); }
__device__ __forceinline__ float load_half(const __nv_bfloat16* ptr, int64_t i, int f16) {
  const uint16_t bits = reinterpret_cast<const uint16_t*>(ptr)[i];
  return f16 ? half_to_float<true>(bits) : half_to_float<false>(bits);
}

__device__ __forceinline__ void merge_ml(float& m, float& l, float m2, float l2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) {
    m = m2;
    l = l2;
    return;
  }
  if (m2 > m) {
    l = l * expf(m - m2) + l2;
    m = m2;
  } else {
    l = l + l2 * expf(m2 - m);
  }
}
// Row `row`'s compressed scores and its slice [lo, hi) of `splits` slices.
struct RowSlice {
  const float* sc;
  int64_t lo, hi;
};
__device__ __forceinline__ RowSlice row_slice(const SoftmaxParams& p, int row, int slice, int splits) {
  const int qi = row % p.q_len;
  const int hq = (row / p.q_len) % p.n_q_heads;
  const int s = row / (p.q_len * p.n_q_heads);
  const int64_t m_s = p.seq_m[s];
  const int64_t chunk = (m_s + splits - 1) / splits;
  RowSlice r;
  r.sc = p.scores + p.seq_score_off[s] + (static_cast<int64_t>(hq) * p.q_len + qi) * m_s;
  r.lo = min(m_s, chunk * slice);
  r.hi = min(m_s, r.lo + chunk);
  return r;
}

// Running (max, sum of exp) over sc[lo, hi), reduced over the block into (m, l) of thread 0.
__device__ __forceinline__ void block_max_sum(const float* sc, int64_t lo, int64_t hi, float* red_m, float* red_l,
                                              float& m_out, float& l_out) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float m = -INFINITY, l = 0.f;
  for (int64_t n = lo + tid; n < hi; n += blockDim.x) {
    const float x = sc[n];
    if (x == -INFINITY) continue;
    if (x > m) {
      l = (m == -INFINITY ? 0.f : l * expf(m - x)) + 1.f;
      m = x;
    } else {
      l += expf(x - m);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
    const float l2 = __shfl_xor_sync(0xffffffffu, l, o);
    merge_ml(m, l, m2, l2);
  }
  if (lane == 0) {
    red_m[warp] = m;
    red_l[warp] = l;
  }
  __syncthreads();
  m_out = -INFINITY;
  l_out = 0.f;
  if (tid == 0)
    for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) merge_ml(m_out, l_out, red_m[w], red_l[w]);
}
}  // namespace

// Few long rows (one long conversation): each row's compressed scores are cut into `splits` slices, one
// CTA per (row, slice) writes the slice's (max, sum of exponentials) to scratch[row][slice].
__global__ void __launch_bounds__(kSoftmaxThreads) softmax_partial_kernel(const SoftmaxParams p, int splits) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  __shared__ float red_m[16], red_l[16];
  const int row = blockIdx.x, slice = blockIdx.y;
  const RowSlice r = row_slice(p, row, slice, splits);
  float m, l;
  block_max_sum(r.sc, r.lo, r.hi, red_m, red_l, m, l);
  if (threadIdx.x == 0) {
    float* out = p.scratch + (static_cast<int64_t>(row) * splits + slice) * 2;
    out[0] = m;
    out[1] = l;
  }
}

// The compressed probability mass of each slice with the row's final (max, 1 / sum): the sum of the
// bf16-rounded probabilities (the reference's p_c.to(dtype), compressed_attention.py:127-130).
__global__ void __launch_bounds__(kSoftmaxThreads) softmax_mass_kernel(const SoftmaxParams p, int splits) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  __shared__ float red[8];
  const int row = blockIdx.x, slice = blockIdx.y;
  const RowSlice r = row_slice(p, row, slice, splits);
  const float* st = p.row_stats + static_cast<int64_t>(row) * 4;
  const float mx = st[0], inv = st[1];
  float mass = 0.f;
  for (int64_t n = r.lo + threadIdx.x; n < r.hi; n += blockDim.x) {
    const float x = r.sc[n];
    if (x != -INFINITY) mass += dtype_round(expf(x - mx) * inv, p.f16);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mass += __shfl_xor_sync(0xffffffffu, mass, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mass;
  __syncthreads();
  if (threadIdx.x == 0) {
    float total = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) total += red[w];
    p.scratch[static_cast<int64_t>(p.n_seq) * p.n_q_heads * p.q_len * splits * 2 +
              static_cast<int64_t>(row) * splits + slice] = total;
  }
}

// Sums each row's slice masses in slice order into row_stats[2].
__global__ void softmax_mass_sum_kernel(const SoftmaxParams p, int splits, int rows) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  const float* part = p.scratch + static_cast<int64_t>(rows) * splits * 2 + static_cast<int64_t>(row) * splits;
  float total = 0.f;
  for (int s = 0; s < splits; ++s) total += part[s];
  p.row_stats[static_cast<int64_t>(row) * 4 + 2] = total;
}

__global__ void __launch_bounds__(kSoftmaxThreads) softmax_stats_kernel(const SoftmaxParams p, int splits) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  extern __shared__ float sh[];
  const int D = p.head_dim;
  float* qv = sh;                     // [D]
  float* se = qv + D;                 // [n_exact]
  float* red_m = se + p.n_exact;      // [16]
  float* red_l = red_m + 16;          // [8]

  const int row = blockIdx.x;
  const int qi = row % p.q_len;
  const int hq = (row / p.q_len) % p.n_q_heads;
  const int s = row / (p.q_len * p.n_q_heads);
  const int kvh = hq / p.q_per_kv;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  const int64_t q0 = ((static_cast<int64_t>(s) * p.n_q_heads + hq) * p.q_len + qi) * D;
  for (int d = tid; d < D; d += blockDim.x) qv[d] = load_half(p.query, q0 + d, p.f16);
  __syncthreads();

  // Exact-token scores, one warp per token.
  const int64_t kbase = (static_cast<int64_t>(s) * (p.n_q_heads / p.q_per_kv) + kvh) * static_cast<int64_t>(p.n_exact) * D;
  for (int e = warp; e < p.n_exact; e += blockDim.x / 32) {
    const int64_t k = kbase + static_cast<int64_t>(e) * D;
    float dot = 0.f;
    for (int d = lane; d < D; d += 32) dot += qv[d] * load_half(p.exact_k, k + d, p.f16);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if (lane == 0) {
      float v = dot * p.scaling;
      if (p.mask != nullptr) v += p.mask[(static_cast<int64_t>(s) * p.q_len + qi) * p.n_exact + e];
      se[e] = v;
    }
  }

  // Compressed part: running (max, sum of exp) per thread, then a block reduction; or, for rows split into
  // slices, the slices' partials merged in slice order.
  const int64_t m_s = p.seq_m[s];
  const float* sc = p.scores + p.seq_score_off[s] + (static_cast<int64_t>(hq) * p.q_len + qi) * m_s;
  float mc = -INFINITY, lc = 0.f;
  if (splits > 1) {
    __syncthreads();  // the exact scores (se) are complete
    if (tid == 0)
      for (int sl = 0; sl < splits; ++sl) {
        const float* part = p.scratch + (static_cast<int64_t>(row) * splits + sl) * 2;
        merge_ml(mc, lc, part[0], part[1]);
      }
  } else {
    block_max_sum(sc, 0, m_s, red_m, red_l, mc, lc);
  }
  if (tid == 0) {
    float mx = mc;
    for (int e = 0; e < p.n_exact; ++e) mx = fmaxf(mx, se[e]);
    float sum = (mc == -INFINITY) ? 0.f : lc * expf(mc - mx);
    for (int e = 0; e < p.n_exact; ++e) sum += (mx == -INFINITY) ? 0.f : expf(se[e] - mx);
    float* st = p.row_stats + static_cast<int64_t>(row) * 4;
    if (p.mode == kSoftmaxLocal) {
      // Split-K, first pass: this shard's (max, sum of exponentials); the caller merges the shards.
      st[0] = mx;
      st[1] = sum;
      st[2] = 0.f;
      st[3] = 0.f;
    } else if (p.mode == kSoftmaxGlobal) {
      // Split-K, second pass: the merged (max, 1 / sum) over every shard.
      mx = st[0];
      sum = 1.f / st[1];
    }
    red_m[0] = mx;
    red_l[0] = 1.f / sum;
  }
  __syncthreads();
  if (p.mode == kSoftmaxLocal) return;
  const float mx = red_m[0], inv = red_l[0];
  if (splits > 1) {  // the slices' masses follow (softmax_mass_kernel); the exact probabilities here
    for (int e = tid; e < p.n_exact; e += blockDim.x)
      p.p_exact[static_cast<int64_t>(row) * p.n_exact + e] = expf(se[e] - mx) * inv;
    if (tid == 0) {
      float* st = p.row_stats + static_cast<int64_t>(row) * 4;
      st[0] = mx;
      st[1] = inv;
      st[2] = 0.f;
      st[3] = 0.f;
    }
    return;
  }
  // The reference casts the probabilities to the cache dtype before the value products
  // (compressed_attention.py:127-128, 130): the compressed mass used by the mean term is a sum of
  // bf16-rounded probabilities. Exact probabilities are stored in fp32 (the finalize kernel rounds
  // them at use; question-time scoring sums them unrounded, as dimmer.py:64-66 does).
  for (int e = tid; e < p.n_exact; e += blockDim.x)
    p.p_exact[static_cast<int64_t>(row) * p.n_exact + e] = expf(se[e] - mx) * inv;
  float mass = 0.f;
  for (int64_t n = tid; n < m_s; n += blockDim.x) {
    const float x = sc[n];
    if (x != -INFINITY) mass += dtype_round(expf(x - mx) * inv, p.f16);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mass += __shfl_xor_sync(0xffffffffu, mass, o);
  __syncthreads();
  if (lane == 0) red_m[8 + warp] = mass;
  __syncthreads();
  if (tid == 0) {
    float total = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x / 32); ++w) total += red_m[8 + w];
    float* st = p.row_stats + static_cast<int64_t>(row) * 4;
    st[0] = mx;
    st[1] = inv;
    st[2] = total;
    st[3] = 0.f;
  }
}

int run_softmax_stats(const SoftmaxParams& p, cudaStream_t stream) {
  if (p.n_exact < 0 || p.n_exact > 16384 || p.head_dim > 256) return kDkvErrConfig;
  const int rows = p.n_seq * p.n_q_heads * p.q_len;
  if (rows == 0) return kDkvOk;
  const int smem = (p.head_dim + p.n_exact + 24) * 4;
  if (smem > 48 * 1024) {
    if (cudaFuncSetAttribute(softmax_stats_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
      return kDkvErrCuda;
  }
  // Few rows (one or a few long conversations at bs1): cut each row's scores into slices so that about
  // two CTAs per SM scan them; the partials live in the caller's scratch.
  int splits = 1;
  if (p.scratch != nullptr && p.n_sms > 0 && rows < 2 * p.n_sms) {
    splits = min(64, (2 * p.n_sms + rows - 1) / rows);
    if (static_cast<int64_t>(rows) * splits * 3 > p.scratch_floats) splits = 1;
  }
  if (splits > 1) {
    softmax_partial_kernel<<<dim3(rows, splits), kSoftmaxThreads, 0, stream>>>(p, splits);
    if (cudaGetLastError() != cudaSuccess) return kDkvErrCuda;
  }
  softmax_stats_kernel<<<rows, kSoftmaxThreads, smem, stream>>>(p, splits);
  if (cudaGetLastError() != cudaSuccess) return kDkvErrCuda;
  if (splits > 1 && p.mode != kSoftmaxLocal) {
    softmax_mass_kernel<<<dim3(rows, splits), kSoftmaxThreads, 0, stream>>>(p, splits);
    if (cudaGetLastError() != cudaSuccess) return kDkvErrCuda;
    softmax_mass_sum_kernel<<<(rows + 255) / 256, 256, 0, stream>>>(p, splits, rows);
  }
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
