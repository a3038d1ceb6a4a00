// encode.cu — encode side of the progressive codec: quantize8 and the per-rung error of every token.
//
// Replaces quantize8 (scripts/progressive.py:37-44) and the error table of ProgressiveCodec.encode
// (scripts/progressive.py:152-163). The reference builds a [tokens, groups, 9] float32 table of the
// squared error of each (token, group) decoded at 0..8 planes, gathers it at each rung's plane count
// per group and sums over groups. Here each group is read once: its min / max, f16 low and span, the
// 8-bit codes, the nine errors and the rungs' sums are formed in registers; the table never exists.
//
// Arithmetic, as the reference's float32 torch ops:
//   low  = f16(min), span = f16(max(max - low, 1e-8))
//   code = clamp(floor((x - low) / span * 256), 0, 255)    (IEEE divide; NaN -> 0 like the cast)
//   v_m  = low + (code >> (8 - m) + 0.5) * span / 2^m       (m >= 1; the product is exact, so one
//          fused multiply-add rounds once, like the reference's multiply, divide, add)
//   err_m = sum over the group of (x - v_m)^2, v_0 = 0
// The codes, low and span are bit-exact; the error sums are float32 in a fixed order of their own.
//
// Layout: one CTA of 8 warps per 4 tokens, two warps per token; a warp takes two adjacent groups at a
// time (one per half-warp, four coefficients per lane, one 512-byte load per warp), with the next pair
// loaded before the current one is processed. Each lane r < n_rungs of a warp keeps rung r's sum; the
// two warps of a token add theirs at the end.
#include <cuda_fp16.h>

#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kEncodeWarps = 8;
constexpr int kEncodeTokensPerCta = 4;
constexpr int kEncodeMaxRungs = 32;
constexpr int kEncodeMaxGroups = 1024;  // rung table staged in shared memory: n_rungs x groups bytes
}  // namespace

__global__ void __launch_bounds__(kEncodeWarps * 32) encode_kernel(const EncodeParams p) {
  extern __shared__ uint8_t rung_planes_s[];  // [n_rungs][groups]
  __shared__ float scratch[kEncodeWarps][2][9];
  __shared__ float red[kEncodeTokensPerCta][kEncodeMaxRungs + 1];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int half = lane >> 4;
  const int l16 = lane & 15;
  const int groups = p.features / 64;
  for (int i = tid; i < p.n_rungs * groups; i += blockDim.x) {
    uint8_t m = p.rung_planes[i];
    if (m > 8) {  // a plane count the codes cannot hold: report it, never index past the nine errors
      record_error(p.status, kErrBadDescriptor);
      m = 8;
    }
    rung_planes_s[i] = m;
  }
  __syncthreads();

  const int tl = warp >> 1;                           // token of the CTA
  const int wt = warp & 1;                            // warp of the token
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kEncodeTokensPerCta + tl;
  const bool active = t < p.tokens;
  float acc_rung = 0.f;    // lane r: rung r's sum over this warp's groups
  float acc_energy = 0.f;  // lane 0
  if (active) {
    const float* row = p.coeff + t * p.coeff_stride;
    // Warp wt takes the group pairs (2 (wt + 2k), 2 (wt + 2k) + 1), k = 0, 1, ...
    int g = 2 * wt + half;
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (g < groups) x = __ldg(reinterpret_cast<const float4*>(row + g * 64) + l16);
    for (int pair = 2 * wt; pair < groups; pair += 4) {
      const int gnext = g + 4;
      float4 xn = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gnext < groups) xn = __ldg(reinterpret_cast<const float4*>(row + gnext * 64) + l16);
      const bool valid = g < groups;
      const float xv[4] = {x.x, x.y, x.z, x.w};
      // Min and max over the 64 values of the half-warp's group.
      float mn = fminf(fminf(xv[0], xv[1]), fminf(xv[2], xv[3]));
      float mx = fmaxf(fmaxf(xv[0], xv[1]), fmaxf(xv[2], xv[3]));
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      }
      const __half low_h = __float2half_rn(mn);
      const float low = __half2float(low_h);
      const __half span_h = __float2half_rn(fmaxf(__fsub_rn(mx, low), 1e-8f));
      const float span = __half2float(span_h);
      uint32_t code[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float q = floorf(__fmul_rn(__fdiv_rn(__fsub_rn(xv[k], low), span), 256.f));
        q = fminf(fmaxf(q, 0.f), 255.f);  // NaN (0 / 0 of a constant group) -> 0, like the uint8 cast
        code[k] = static_cast<uint32_t>(q);
      }
      // Squared error at 0..8 planes.
      float e[9];
      e[0] = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) e[0] = fmaf(xv[k], xv[k], e[0]);
#pragma unroll
      for (int m = 1; m <= 8; ++m) {
        const float scale = __fmul_rn(span, __int_as_float((127 - m) << 23));  // span / 2^m, exact
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float idx = __fsub_rn(__uint_as_float(0x4B000000u | (code[k] >> (8 - m))), 8388607.5f);  // + 0.5
          const float d = __fsub_rn(xv[k], __fmaf_rn(idx, scale, low));
          s = fmaf(d, d, s);
        }
        e[m] = s;
      }
#pragma unroll
      for (int o = 8; o >= 1; o >>= 1) {
#pragma unroll
        for (int m = 0; m <= 8; ++m) e[m] += __shfl_xor_sync(0xffffffffu, e[m], o);
      }
      if (valid) {
        const int64_t col = static_cast<int64_t>(g) * 64 + 4 * l16;
        *reinterpret_cast<uint32_t*>(p.codes + t * p.features + col) =
            code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
        if (l16 == 0) {
          p.low[t * groups + g] = __half_as_ushort(low_h);
          p.span[t * groups + g] = __half_as_ushort(span_h);
        }
      }
#pragma unroll
      for (int m = 0; m <= 8; ++m)
        if (l16 == m) scratch[warp][half][m] = valid ? e[m] : 0.f;
      __syncwarp();
      if (lane < p.n_rungs) {
        const int g0 = pair;  // the half-warps hold groups pair and pair + 1
        float a = scratch[warp][0][rung_planes_s[lane * groups + g0]];
        if (g0 + 1 < groups) a += scratch[warp][1][rung_planes_s[lane * groups + g0 + 1]];
        acc_rung += a;
      }
      if (lane == 0) acc_energy += scratch[warp][0][0] + scratch[warp][1][0];
      __syncwarp();
      x = xn;
      g = gnext;
    }
  }
  // The token's two warps: warp 1 hands its sums to warp 0, which writes them.
  if (wt == 1) {
    if (lane < p.n_rungs) red[tl][lane] = acc_rung;
    if (lane == 0) red[tl][kEncodeMaxRungs] = acc_energy;
  }
  __syncthreads();
  if (wt == 0 && active) {
    if (lane < p.n_rungs) p.rung_error[t * p.n_rungs + lane] = acc_rung + red[tl][lane];
    if (lane == 0 && p.energy != nullptr) p.energy[t] = acc_energy + red[tl][kEncodeMaxRungs];
  }
}

int run_encode(const EncodeParams& p, cudaStream_t stream) {
  if (p.tokens < 0 || p.features <= 0 || p.features % 64 != 0 || p.n_rungs < 1 || p.n_rungs > kEncodeMaxRungs ||
      p.coeff_stride < p.features || p.coeff_stride % 4 != 0)
    return kDkvErrArgs;
  if ((reinterpret_cast<uintptr_t>(p.coeff) & 15u) || (reinterpret_cast<uintptr_t>(p.codes) & 3u) ||
      (reinterpret_cast<uintptr_t>(p.low) & 1u) || (reinterpret_cast<uintptr_t>(p.span) & 1u))
    return kDkvErrArgs;
  const int groups = p.features / 64;
  if (groups > kEncodeMaxGroups) return kDkvErrConfig;
  if (p.tokens == 0) return kDkvOk;
  const int smem = p.n_rungs * groups;  // <= 32 KB
  const int grid = (p.tokens + kEncodeTokensPerCta - 1) / kEncodeTokensPerCta;
  encode_kernel<<<grid, kEncodeWarps * 32, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
