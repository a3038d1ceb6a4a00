// finalize.cu — value basis applied once per head, plus the mean and exact-token terms.
//
// Replaces the tail of CompressedContext.attend (scripts/compressed_attention.py:130-137):
//   out_c = sum(p_c) * mean_v + (p_c @ C_v) @ B_v[layer, head]     (values never decoded)
//   out   = out_c + p_e @ V_exact
// The probability-weighted coefficients p_c @ C_v arrive as per-item partial sums from
// value_weights.cu. Two kernels:
//   vbasis  : one CTA per (chunk of 128 basis components, KV head, block of 8 conversations). The
//             CTA stages its basis slice [128 components x head_dim] in shared memory, reduces the
//             items' partial sums of those components for its conversations and multiplies them by
//             the slice: the layer's value basis is read once per 8 conversations instead of once per
//             conversation. Output: per-chunk partial outputs [chunks][conversations][rows][head_dim].
//   combine : sums the chunks in a fixed order (deterministic), adds the mean term and the exact
//             tokens, and writes the HF layout [batch, q_len, q_heads, head_dim].
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"
#include "dkv_format.cuh"

namespace dkv {

namespace {
constexpr int kFinalizeThreads = 256;
constexpr int kCombineThreads = 128;
constexpr int kCombineRows = 8;  // rows of one KV head per combine CTA (one when a head has many rows)
constexpr int kRChunk = 128;   // basis components per vbasis CTA
constexpr int kSeqBlock = 8;   // conversations per vbasis CTA (fewer when many rows share a KV head)
constexpr int kCoverPerSeq = 512;  // items of one conversation that cover a component chunk
}  // namespace

__global__ void __launch_bounds__(kFinalizeThreads) vbasis_kernel(const FinalizeParams p, int seq_block,
                                                                  int row_block, int n_row_blocks) {
  if (cta_failed_at_entry(p.status)) return;  // an earlier kernel of the call failed
  extern __shared__ float smem_f[];
  const int D = p.head_dim;
  const int D2 = D / 2;
  const int G = p.q_per_kv;
  const int chunk = blockIdx.x, kvh = blockIdx.y;
  const int s0 = (blockIdx.z / n_row_blocks) * seq_block;
  const int n_s = min(seq_block, p.n_seq - s0);
  const int r0 = chunk * kRChunk;
  // Rows of this KV head inside the call, then this CTA's block of them (many query rows per head,
  // few conversations: the rows are spread over more CTAs).
  const int head_lo = max(p.row_begin, kvh * G * p.q_len);
  const int head_hi = min(p.row_begin + p.n_rows, (kvh + 1) * G * p.q_len);
  const int rlo = head_lo + static_cast<int>(blockIdx.z % n_row_blocks) * row_block;
  const int rhi = min(head_hi, rlo + row_block);
  const int nr = rhi - rlo;
  if (nr <= 0 || n_s <= 0) return;
  uint32_t* bs = reinterpret_cast<uint32_t*>(smem_f);  // [kRChunk][D/2] pairs of 16-bit basis values
  float* ws = smem_f + kRChunk * D2;                                // [n_s][nr][kRChunk]
  const int tid = threadIdx.x;
  const int item_cols = p.item_groups * 64;

  // Basis slice of this KV head: rows r0 .. r0+127 of [layer][r_v][n_cols], columns kvh*D .. +D.
  const uint32_t* bsrc =
      reinterpret_cast<const uint32_t*>(p.basis_v + static_cast<int64_t>(p.layer) * p.r_v * p.n_cols) + kvh * D2;
  for (int i = tid; i < kRChunk * D2; i += kFinalizeThreads) {
    const int r = i / D2, dp = i % D2;
    bs[i] = (r0 + r < p.r_v) ? bsrc[static_cast<int64_t>(r0 + r) * (p.n_cols / 2) + dp] : 0u;  // +0.0 in both
  }
  // Weighted coefficients of the block's conversations. First the items of each conversation that cover
  // this chunk (in item order), then every element sums them with independent loads.
  // One warp per conversation builds its list (at most kCoverPerSeq items).
  __shared__ int cover[kSeqBlock * kCoverPerSeq];
  __shared__ int n_cover[kSeqBlock];
  {
    const int sl = tid >> 5, ln = tid & 31;
    if (sl < n_s) {
      const int it0 = p.seq_items[2 * (s0 + sl)], it1 = p.seq_items[2 * (s0 + sl) + 1];
      int n = 0;
      for (int base = it0; base < it1; base += 32) {
        const int it = base + ln;
        bool hit = false;
        if (it < it1) {
          const int cb = p.items[4 * it + 3] * 64;
          hit = r0 >= cb && r0 < cb + item_cols;
        }
        const unsigned mask = __ballot_sync(0xffffffffu, hit);
        const int slot = n + __popc(mask & ((1u << ln) - 1u));
        if (hit) {
          if (slot < kCoverPerSeq)
            cover[sl * kCoverPerSeq + slot] = it;
          else  // more covering items than the list holds: report, never drop silently
            record_error(p.status, kErrBadDescriptor);
        }
        n += __popc(mask);
      }
      if (ln == 0) n_cover[sl] = n < kCoverPerSeq ? n : kCoverPerSeq;
    }
  }
  __syncthreads();
  for (int i = tid; i < n_s * nr * kRChunk; i += kFinalizeThreads) {
    const int sl = i / (nr * kRChunk);
    const int rr = (i / kRChunk) % nr, c = i % kRChunk;
    const int64_t col = (rlo - p.row_begin + rr) * static_cast<int64_t>(item_cols) + (r0 % item_cols) + c;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int j = sl * kCoverPerSeq;
    const int j1 = j + n_cover[sl];
    for (; j + 4 <= j1; j += 4) {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        acc[u] += p.partial[static_cast<int64_t>(cover[j + u]) * p.n_rows_pad * item_cols + col];
    }
    float tail = 0.f;
    for (; j < j1; ++j) tail += p.partial[static_cast<int64_t>(cover[j]) * p.n_rows_pad * item_cols + col];
    ws[i] = ((acc[0] + acc[1]) + (acc[2] + acc[3])) + tail;
  }
  __syncthreads();
  const int dp = tid % D2;
  const int rg = tid / D2;
  const int n_rg = kFinalizeThreads / D2;
  for (int j = rg; j < n_s * nr; j += n_rg) {
    const float* w = ws + j * kRChunk;
    float ax = 0.f, ay = 0.f;
    if (p.f16) {
#pragma unroll 8
      for (int c = 0; c < kRChunk; ++c) {
        const float2 b = half2_to_float2<true>(bs[c * D2 + dp]);
        ax = fmaf(w[c], b.x, ax);
        ay = fmaf(w[c], b.y, ay);
      }
    } else {
#pragma unroll 8
      for (int c = 0; c < kRChunk; ++c) {
        const float2 b = half2_to_float2<false>(bs[c * D2 + dp]);
        ax = fmaf(w[c], b.x, ax);
        ay = fmaf(w[c], b.y, ay);
      }
    }
    const int s = s0 + j / nr, rr = j % nr;
    float2* dst = reinterpret_cast<float2*>(
        p.vpart + ((static_cast<int64_t>(chunk) * p.n_seq + s) * p.n_rows_pad + (rlo - p.row_begin + rr)) * D);
    dst[dp] = make_float2(ax, ay);
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

int finalize_chunks(int r_v) { return (r_v + kRChunk - 1) / kRChunk; }

int run_finalize(const FinalizeParams& p, cudaStream_t stream) {
  if (p.head_dim % 64 != 0 || p.head_dim > 256 || p.q_per_kv < 1 || p.n_q_heads % p.q_per_kv != 0 ||
      p.vpart == nullptr || p.item_groups % 2 != 0 || p.n_rows > p.n_rows_pad)
    return kDkvErrConfig;
  if (p.n_seq == 0 || p.n_rows == 0) return kDkvOk;
  // Rows of one KV head inside this call: at most q_per_kv * q_len and at most n_rows.
  const int nr_max = min(p.n_rows, p.q_per_kv * p.q_len);
  const int n_chunks = finalize_chunks(p.r_v);
  const int n_kv = p.n_q_heads / p.q_per_kv;
  // Many rows per KV head and few conversations (question-length queries): cut each head's rows into
  // blocks of 16 so that the grid covers the SMs (a call's rows then span one or two KV heads).
  int row_block = nr_max;
  if (p.n_seq < kSeqBlock && nr_max > 16) row_block = 16;
  const int n_row_blocks = (nr_max + row_block - 1) / row_block;
  const int basis_bytes = kRChunk * p.head_dim / 2 * 4;
  const int per_seq = row_block * kRChunk * 4;
  const int seq_block = min(kSeqBlock, (200 * 1024 - basis_bytes) / per_seq);
  if (seq_block < 1) return kDkvErrConfig;
  const int smem = basis_bytes + seq_block * per_seq;
  if (cudaFuncSetAttribute(vbasis_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return kDkvErrCuda;
  const int seq_blocks = (p.n_seq + seq_block - 1) / seq_block;
  vbasis_kernel<<<dim3(n_chunks, n_kv, seq_blocks * n_row_blocks), kFinalizeThreads, smem, stream>>>(
      p, seq_block, row_block, n_row_blocks);
  if (cudaGetLastError() != cudaSuccess) return kDkvErrCuda;
  const int rows_per_head = min(p.n_rows, p.q_per_kv * p.q_len);
  // Question-length queries put many rows on a head: one row per CTA then keeps the SMs busy.
  const int rows_per_cta = rows_per_head >= 32 ? 1 : kCombineRows;
  const dim3 cgrid(p.n_seq * n_kv, (rows_per_head + rows_per_cta - 1) / rows_per_cta);
  combine_kernel<<<cgrid, kCombineThreads, 0, stream>>>(p, n_chunks, rows_per_cta);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
