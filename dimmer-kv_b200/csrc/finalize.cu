// finalize.cu — value basis applied once per head, plus the mean and exact-token terms.
//
// Replaces the tail of CompressedContext.attend (scripts/compressed_attention.py:130-137):
//   out_c = sum(p_c) * mean_v + (p_c @ C_v) @ B_v[layer, head]     (values never decoded)
//   out   = out_c + p_e @ V_exact
// The probability-weighted coefficients p_c @ C_v arrive as per-item partial sums from
// value_weights.cu; this kernel reduces them, applies the value basis of the layer for one KV
// head and writes the output in the HF layout [batch, q_len, q_heads, head_dim] (bf16).
#include "dkv_kernels.h"

namespace dkv {

namespace {
constexpr int kFinalizeThreads = 256;
}

__global__ void __launch_bounds__(kFinalizeThreads) finalize_kernel(const FinalizeParams p) {
  extern __shared__ float w[];  // [G][r_v] weighted coefficients of one query row, then reduction scratch
  const int n_kv = p.n_q_heads / p.q_per_kv;
  const int s = blockIdx.x / n_kv;
  const int kvh = blockIdx.x % n_kv;
  const int D = p.head_dim;
  const int G = p.q_per_kv;
  const int R = p.r_v;
  const int parts = blockDim.x / (D / 2);   // component slices
  const int d2 = threadIdx.x % (D / 2);     // output dims 2*d2, 2*d2+1
  const int part = threadIdx.x / (D / 2);
  const int d = threadIdx.x;                // output dim of the final combine (threads 0 .. D-1)
  float* red = w + G * R;  // [parts][G][D]
  const int item_cols = p.item_groups * 64;

  for (int qi = 0; qi < p.q_len; ++qi) {
    // Only rows computed by the matching value_weights call.
    bool any = false;
    for (int j = 0; j < G; ++j) {
      const int row = (kvh * G + j) * p.q_len + qi - p.row_begin;
      any |= (row >= 0 && row < p.n_rows);
    }
    if (!any) continue;
    for (int i = threadIdx.x; i < G * R; i += blockDim.x) w[i] = 0.f;
    __syncthreads();
    const int it0 = p.seq_items[2 * s], it1 = p.seq_items[2 * s + 1];
    for (int it = it0; it < it1; ++it) {
      const int g0 = p.items[4 * it + 3];
      for (int j = 0; j < G; ++j) {
        const int row = (kvh * G + j) * p.q_len + qi - p.row_begin;
        if (row < 0 || row >= p.n_rows) continue;
        const float* src = p.partial + (static_cast<int64_t>(it) * p.n_rows_pad + row) * item_cols;
        for (int c = threadIdx.x; c < item_cols; c += blockDim.x) {
          const int col = g0 * 64 + c;
          if (col < R) w[j * R + col] += src[c];
        }
      }
    }
    __syncthreads();
    // Value basis of this KV head: each thread owns two adjacent output dims (one bf16x2 load per
    // component) and a slice of the components; slices are summed through shared memory.
    float acc[4][2] = {{0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}, {0.f, 0.f}};
    const __nv_bfloat162* bv = reinterpret_cast<const __nv_bfloat162*>(
        p.basis_v + static_cast<int64_t>(p.layer) * R * p.n_cols + kvh * D + 2 * d2);
    const int64_t bstride = p.n_cols / 2;
#pragma unroll 4
    for (int r = part; r < R; r += parts) {
      const float2 b = __bfloat1622float2(bv[static_cast<int64_t>(r) * bstride]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j < G) {
          const float wv = w[j * R + r];
          acc[j][0] += wv * b.x;
          acc[j][1] += wv * b.y;
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j < G) {
        red[(part * G + j) * D + 2 * d2] = acc[j][0];
        red[(part * G + j) * D + 2 * d2 + 1] = acc[j][1];
      }
    }
    __syncthreads();
    if (threadIdx.x < D) {
      const float mean = __bfloat162float(p.mean_v[static_cast<int64_t>(s) * p.mean_seq_stride +
                                                   static_cast<int64_t>(p.layer) * p.n_cols + kvh * D + d]);
      const __nv_bfloat16* vex = p.exact_v + (static_cast<int64_t>(s) * n_kv + kvh) * p.n_exact * D + d;
      for (int j = 0; j < G; ++j) {
        const int hq = kvh * G + j;
        const int row = hq * p.q_len + qi - p.row_begin;
        if (row < 0 || row >= p.n_rows) continue;
        float o = 0.f;
        for (int q2 = 0; q2 < parts; ++q2) o += red[(q2 * G + j) * D + d];
        const int64_t srow = (static_cast<int64_t>(s) * p.n_q_heads + hq) * p.q_len + qi;
        o += mean * p.row_stats[srow * 4 + 2];
        const float* pe = p.p_exact + srow * p.n_exact;
        // Exact probabilities are kept unrounded (question-time scoring sums them); the value product uses
        // them rounded to the cache dtype, as the reference does (compressed_attention.py:128, 135).
        for (int e = 0; e < p.n_exact; ++e)
          o += __bfloat162float(__float2bfloat16_rn(pe[e])) * __bfloat162float(vex[static_cast<int64_t>(e) * D]);
        const int64_t oi = ((static_cast<int64_t>(s) * p.q_len + qi) * p.n_q_heads + hq) * D + d;
        if (p.out_f32)
          static_cast<float*>(p.out)[oi] = o;
        else
          static_cast<__nv_bfloat16*>(p.out)[oi] = __float2bfloat16_rn(o);
      }
    }
    __syncthreads();
  }
}

int run_finalize(const FinalizeParams& p, cudaStream_t stream) {
  if (p.q_per_kv > 4 || p.head_dim > 256 || kFinalizeThreads % p.head_dim != 0) return kDkvErrConfig;
  const int parts = kFinalizeThreads / (p.head_dim / 2);
  const int smem = (p.q_per_kv * p.r_v + parts * p.q_per_kv * p.head_dim) * 4;
  if (smem > 227 * 1024) return kDkvErrConfig;
  if (cudaFuncSetAttribute(finalize_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kDkvErrCuda;
  const int grid = p.n_seq * (p.n_q_heads / p.q_per_kv);
  if (grid == 0) return kDkvOk;
  finalize_kernel<<<grid, kFinalizeThreads, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
