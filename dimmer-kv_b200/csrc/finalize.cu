// finalize.cu — value basis applied once per head, plus the mean and exact-token terms.
//
// Replaces the tail of CompressedContext.attend (scripts/compressed_attention.py:130-137):
//   out_c = sum(p_c) * mean_v + (p_c @ C_v) @ B_v[layer, head]     (values never decoded)
//   out   = out_c + p_e @ V_exact
// The probability-weighted coefficients p_c @ C_v arrive as per-item partial sums from the value stage
// (value_dense.cu / value_weights.cu). Three kernels:
//   wsum    : one CTA per (conversation, 64 components, block of rows): sums the conversation's items that cover the
//             components, in item order (deterministic), into W [conversation][row][component] (fp32).
//   vbasis  : per KV head a fp32 product W[rows of the head, all conversations] x B_v[layer][:, head] on the
//             CUDA cores (the reference's product is fp32-accurate; tensor-core inputs would round W),
//             tiled 32 rows x head_dim columns x 32 components through shared memory, the components split
//             into up to kMaxKSplit slices so that the grid covers the SMs. Output: per-slice partial outputs
//             [slices][conversations][rows][head_dim].
//   combine : sums the slices in a fixed order (deterministic), adds the mean term and the exact
//             tokens, and writes the HF layout [batch, q_len, q_heads, head_dim].
// Scratch (vpart): W [n_seq][rows_pad][r_v], then the slices' partial outputs.
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"

namespace dkv {

namespace {
constexpr int kWsumComps = 64;       // components per wsum CTA (one group; item ranges hold whole groups)
constexpr int kWsumThreads = 256;    // 64 components x 4 row phases
constexpr int kWsumRows = 8;         // rows per wsum CTA when few conversations leave the grid small
constexpr int kGemmThreads = 256;
constexpr int kGemmBM = 32;          // rows per vbasis CTA
constexpr int kGemmBK = 32;          // components per shared-memory step
constexpr int kMaxKSplit = 16;       // component slices of vbasis (partial outputs summed by combine)
constexpr int kCombineThreads = 128;
constexpr int kCombineRows = 8;      // rows of one KV head per combine CTA (one when a head has many rows)
}  // namespace

// W[s][lr][c] = sum over the conversation's items covering component c (item order) of
// partial[item][lr][c - first component of the item]. Rows lr in [0, n_rows). A conversation's items are
// ordered by first group (then tile), so the items covering one block are consecutive: found by a binary
// search, then summed with independent loads.
__global__ void __launch_bounds__(kWsumThreads) wsum_kernel(const FinalizeParams p, float* w, int row_block) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  const int s = blockIdx.x;
  const int c0 = blockIdx.y * kWsumComps;
  const int c = c0 + (threadIdx.x % kWsumComps);
  const int phase = threadIdx.x / kWsumComps;
  const int item_cols = p.item_groups * 64;
  const int g_first = (c0 / item_cols) * p.item_groups;  // first group of the items covering this block
  const int it0 = __ldg(p.seq_items + 2 * s), it1 = __ldg(p.seq_items + 2 * s + 1);
  int lo = it0, hi = it1;  // first item whose first group is >= g_first
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(p.items + 4 * mid + 3) < g_first) lo = mid + 1;
    else hi = mid;
  }
  int end = lo;
  while (end < it1 && __ldg(p.items + 4 * end + 3) == g_first) ++end;
  const int cb = g_first * 64;
  const int lr_end = min(p.n_rows, static_cast<int>(blockIdx.z + 1) * row_block);
  for (int lr = blockIdx.z * row_block + phase; lr < lr_end; lr += kWsumThreads / kWsumComps) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int it = lo;
    for (; it + 4 <= end; it += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        acc[u] += p.partial[(static_cast<int64_t>(it + u) * p.n_rows_pad + lr) * item_cols + (c - cb)];
    }
#pragma unroll
    for (int u = 0; u < 3; ++u)
      if (it + u < end) acc[u] += p.partial[(static_cast<int64_t>(it + u) * p.n_rows_pad + lr) * item_cols + (c - cb)];
    w[(static_cast<int64_t>(s) * p.n_rows_pad + lr) * p.r_v + c] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  }
}

// Rows of KV head kvh inside the call: [head_lo, head_hi) (absolute row indices), nrh of them.
__device__ __forceinline__ void head_rows(const FinalizeParams& p, int kvh, int& head_lo, int& nrh) {
  const int G = p.q_per_kv;
  head_lo = max(p.row_begin, kvh * G * p.q_len);
  const int head_hi = min(p.row_begin + p.n_rows, (kvh + 1) * G * p.q_len);
  nrh = max(0, head_hi - head_lo);
}

// vpart[slice][s][lr][d] = sum over components k of the slice of W[s][lr][k] * B_v[layer][k][kvh * D + d], for
// the rows lr of KV head kvh = blockIdx.y of every conversation (GEMM rows m = s * nrh + row within the head).
template <int D>
__global__ void __launch_bounds__(kGemmThreads) vbasis_kernel(const FinalizeParams p, const float* w, float* vpart,
                                                             int k_slice) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  constexpr int kTN = 4;                      // columns per thread
  constexpr int kThreadsN = D / kTN;          // 32 (D = 128) or 16 (D = 64)
  constexpr int kThreadsM = kGemmThreads / kThreadsN;
  constexpr int kTM = kGemmBM / kThreadsM;    // rows per thread: 4 or 2
  __shared__ float as[kGemmBK][kGemmBM + 4];  // W tile, component-major (rows contiguous)
  __shared__ float bs[kGemmBK][D];            // B_v tile in fp32
  const int kvh = blockIdx.y;
  int head_lo, nrh;
  head_rows(p, kvh, head_lo, nrh);
  const int M = p.n_seq * nrh;
  const int m0 = blockIdx.x * kGemmBM;
  if (nrh == 0 || m0 >= M) return;
  const int k0 = blockIdx.z * k_slice;
  const int k1 = min(p.r_v, k0 + k_slice);
  const int tid = threadIdx.x;
  const int tn = tid % kThreadsN, tm = tid / kThreadsN;
  float acc[kTM][kTN];
#pragma unroll
  for (int i = 0; i < kTM; ++i)
#pragma unroll
    for (int j = 0; j < kTN; ++j) acc[i][j] = 0.f;
  const uint16_t* bsrc = reinterpret_cast<const uint16_t*>(p.basis_v) + static_cast<int64_t>(p.layer) * p.r_v * p.n_cols +
                         kvh * D;
  for (int kb = k0; kb < k1; kb += kGemmBK) {
    // W tile: kGemmBM rows x kGemmBK components (rows past M or components past the slice read as 0).
    for (int i = tid; i < kGemmBM * kGemmBK; i += kGemmThreads) {
      const int mm = i / kGemmBK, kk = i % kGemmBK;
      const int m = m0 + mm, k = kb + kk;
      float v = 0.f;
      if (m < M && k < k1) {
        const int sq = m / nrh, lr = head_lo - p.row_begin + m % nrh;
        v = w[(static_cast<int64_t>(sq) * p.n_rows_pad + lr) * p.r_v + k];
      }
      as[kk][mm] = v;
    }
    // B_v tile: kGemmBK components x D columns of this head, 16-bit -> fp32.
    for (int i = tid; i < kGemmBK * (D / 2); i += kGemmThreads) {
      const int kk = i / (D / 2), dp = i % (D / 2);
      const int k = kb + kk;
      float2 b = make_float2(0.f, 0.f);
      if (k < k1) {
        const uint32_t bits = *reinterpret_cast<const uint32_t*>(bsrc + static_cast<int64_t>(k) * p.n_cols + 2 * dp);
        b = p.f16 ? half2_to_float2<true>(bits) : half2_to_float2<false>(bits);
      }
      bs[kk][2 * dp] = b.x;
      bs[kk][2 * dp + 1] = b.y;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < kGemmBK; ++kk) {
      float a[kTM];
#pragma unroll
      for (int i = 0; i < kTM; ++i) a[i] = as[kk][tm * kTM + i];
      const float4 b = *reinterpret_cast<const float4*>(&bs[kk][tn * kTN]);
#pragma unroll
      for (int i = 0; i < kTM; ++i) {
        acc[i][0] = fmaf(a[i], b.x, acc[i][0]);
        acc[i][1] = fmaf(a[i], b.y, acc[i][1]);
        acc[i][2] = fmaf(a[i], b.z, acc[i][2]);
        acc[i][3] = fmaf(a[i], b.w, acc[i][3]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < kTM; ++i) {
    const int m = m0 + tm * kTM + i;
    if (m >= M) continue;
    const int sq = m / nrh, lr = head_lo - p.row_begin + m % nrh;
    float4* dst = reinterpret_cast<float4*>(
        vpart + ((static_cast<int64_t>(blockIdx.z) * p.n_seq + sq) * p.n_rows_pad + lr) * D + tn * kTN);
    *dst = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
  }
}

// One CTA per (conversation, KV head, block of 8 rows of the head); a thread per output dim.
__global__ void __launch_bounds__(kCombineThreads) combine_kernel(const FinalizeParams p, int n_chunks,
                                                                   int rows_per_cta) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  const int G = p.q_per_kv;
  const int n_kv = p.n_q_heads / G;
  const int s = blockIdx.x / n_kv, kvh = blockIdx.x % n_kv;
  const int D = p.head_dim;
  const int head_lo = max(p.row_begin, kvh * G * p.q_len);
  const int head_hi = min(p.row_begin + p.n_rows, (kvh + 1) * G * p.q_len);
  const int rlo = head_lo + blockIdx.y * rows_per_cta;
  const int rhi = min(head_hi, rlo + rows_per_cta);
  for (int i = threadIdx.x; i < (rhi - rlo) * D; i += blockDim.x) {
    const int row = rlo + i / D, d = i % D;
    const int lr = row - p.row_begin;
    const int hq = row / p.q_len, qi = row % p.q_len;
    // Chunks summed in a fixed order with independent loads in flight.
    const float* vp = p.vpart + (static_cast<int64_t>(s) * p.n_rows_pad + lr) * D + d;
    const int64_t cstride = static_cast<int64_t>(p.n_seq) * p.n_rows_pad * D;
    float part[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int ch = 0;
    for (; ch + 8 <= n_chunks; ch += 8) {
#pragma unroll
      for (int u = 0; u < 8; ++u) part[u] += vp[(ch + u) * cstride];
    }
    float tail = 0.f;
    for (; ch < n_chunks; ++ch) tail += vp[ch * cstride];
    float o = ((part[0] + part[1]) + (part[2] + part[3])) + ((part[4] + part[5]) + (part[6] + part[7])) + tail;
    const int64_t srow = (static_cast<int64_t>(s) * p.n_q_heads + hq) * p.q_len + qi;
    const uint16_t mbits = reinterpret_cast<const uint16_t*>(
        p.mean_v)[static_cast<int64_t>(s) * p.mean_seq_stride + static_cast<int64_t>(p.layer) * p.n_cols + kvh * D + d];
    const float mean = p.f16 ? half_to_float<true>(mbits) : half_to_float<false>(mbits);
    o += mean * p.row_stats[srow * 4 + 2];
    // Exact probabilities are kept unrounded (question-time scoring sums them); the value product uses
    // them rounded to the cache dtype, as the reference does (compressed_attention.py:128, 135).
    const float* pe = p.p_exact + srow * p.n_exact;
    const uint16_t* vex = reinterpret_cast<const uint16_t*>(p.exact_v) + (static_cast<int64_t>(s) * n_kv + kvh) * p.n_exact * D + d;
    float ex[4] = {0.f, 0.f, 0.f, 0.f};
    float ex_tail = 0.f;
    int e = 0;
    if (p.f16) {
      for (; e + 4 <= p.n_exact; e += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          ex[u] += round_half<true>(pe[e + u]) * half_to_float<true>(vex[static_cast<int64_t>(e + u) * D]);
      }
      for (; e < p.n_exact; ++e) ex_tail += round_half<true>(pe[e]) * half_to_float<true>(vex[static_cast<int64_t>(e) * D]);
    } else {
      for (; e + 4 <= p.n_exact; e += 4) {
#pragma unroll
        for (int u = 0; u < 4; ++u)
          ex[u] += round_half<false>(pe[e + u]) * half_to_float<false>(vex[static_cast<int64_t>(e + u) * D]);
      }
      for (; e < p.n_exact; ++e)
        ex_tail += round_half<false>(pe[e]) * half_to_float<false>(vex[static_cast<int64_t>(e) * D]);
    }
    o += ((ex[0] + ex[1]) + (ex[2] + ex[3])) + ex_tail;
    const int64_t oi = ((static_cast<int64_t>(s) * p.q_len + qi) * p.n_q_heads + hq) * D + d;
    if (p.out_f32)
      static_cast<float*>(p.out)[oi] = o;
    else
      static_cast<uint16_t*>(p.out)[oi] = p.f16 ? float_to_half<true>(o) : float_to_half<false>(o);
  }
}

int64_t finalize_vpart_floats(int r_v, int n_seq, int rows_pad, int head_dim) {
  return static_cast<int64_t>(n_seq) * rows_pad * (static_cast<int64_t>(r_v) + kMaxKSplit * head_dim);
}

template <int D>
static int launch_vbasis(const FinalizeParams& p, const float* w, float* vpart, int m_tiles, int n_kv, int splits,
                         int k_slice, cudaStream_t stream) {
  vbasis_kernel<D><<<dim3(m_tiles, n_kv, splits), kGemmThreads, 0, stream>>>(p, w, vpart, k_slice);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

int run_finalize(const FinalizeParams& p, cudaStream_t stream) {
  if ((p.head_dim != 64 && p.head_dim != 128) || p.q_per_kv < 1 || p.n_q_heads % p.q_per_kv != 0 ||
      p.vpart == nullptr || p.item_groups % 2 != 0 || p.n_rows > p.n_rows_pad || p.r_v % kWsumComps != 0)
    return kDkvErrConfig;
  if (p.n_seq == 0 || p.n_rows == 0) return kDkvOk;
  float* w = p.vpart;                                                              // [n_seq][rows_pad][r_v]
  float* vpart = p.vpart + static_cast<int64_t>(p.n_seq) * p.n_rows_pad * p.r_v;  // [splits][n_seq][rows_pad][D]
  // Rows per CTA: all of the call's rows when (conversation, component block) CTAs already fill the GPU a few
  // times over, else blocks of kWsumRows (question-length calls of one conversation).
  const int row_block = static_cast<int64_t>(p.n_seq) * (p.r_v / kWsumComps) >= 1024 ? p.n_rows : kWsumRows;
  wsum_kernel<<<dim3(p.n_seq, p.r_v / kWsumComps, (p.n_rows + row_block - 1) / row_block), kWsumThreads, 0, stream>>>(
      p, w, row_block);
  if (cudaGetLastError() != cudaSuccess) return kDkvErrCuda;
  // GEMM rows per KV head: every conversation's rows of the head inside this call.
  const int n_kv = p.n_q_heads / p.q_per_kv;
  int max_rows = 0;
  for (int kvh = 0; kvh < n_kv; ++kvh) {
    const int lo = max(p.row_begin, kvh * p.q_per_kv * p.q_len);
    const int hi = min(p.row_begin + p.n_rows, (kvh + 1) * p.q_per_kv * p.q_len);
    max_rows = max(max_rows, hi - lo);
  }
  const int m_tiles = (p.n_seq * max_rows + kGemmBM - 1) / kGemmBM;
  // Component slices: enough CTAs for about two per SM, each slice a multiple of kGemmBK components.
  int splits = (2 * 148 + m_tiles * n_kv - 1) / (m_tiles * n_kv);
  splits = max(1, min(kMaxKSplit, min(splits, p.r_v / kGemmBK)));
  const int k_slice = ((p.r_v + splits - 1) / splits + kGemmBK - 1) / kGemmBK * kGemmBK;
  splits = (p.r_v + k_slice - 1) / k_slice;
  const int rc = p.head_dim == 128 ? launch_vbasis<128>(p, w, vpart, m_tiles, n_kv, splits, k_slice, stream)
                                   : launch_vbasis<64>(p, w, vpart, m_tiles, n_kv, splits, k_slice, stream);
  if (rc != kDkvOk) return rc;
  FinalizeParams pc = p;
  pc.vpart = vpart;
  const int rows_per_head = min(p.n_rows, p.q_per_kv * p.q_len);
  // Question-length queries put many rows on a head: one row per CTA then keeps the SMs busy.
  const int rows_per_cta = rows_per_head >= 32 ? 1 : kCombineRows;
  const dim3 cgrid(p.n_seq * n_kv, (rows_per_head + rows_per_cta - 1) / rows_per_cta);
  combine_kernel<<<cgrid, kCombineThreads, 0, stream>>>(pc, splits, rows_per_cta);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
