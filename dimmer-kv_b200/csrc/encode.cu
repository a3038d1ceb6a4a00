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
//   code = clamp(floor((x - low) / span * 256), 0, 255)    (IEEE quotient; NaN -> 0 like the cast)
//   err_m = sum over the group of (x - v_m)^2,  v_m = low + (code >> (8 - m) + 0.5) * span / 2^m,  v_0 = 0
// The codes, low and span are bit-exact. The quotient is first taken as (x - low) * (256 / span);
// that product is within 3 * 2^-24 relative of 256 * fl((x - low) / span), i.e. within 7e-5 for
// every value up to 384 (the largest a group reaches: span is its f16-rounded range, at worst half a
// subnormal step short), so when its fraction is farther than 1e-4 from an integer both floor alike,
// and only the rest (values on a bin edge, NaN, infinities) takes the correctly rounded division.
// The error sums are float32 in a fixed order of their own (d = (x - low) - (idx + 0.5) * span / 2^m,
// fused into the square-add).
//
// Layout: one CTA of 8 warps per 4 tokens, two warps per token; a warp takes two adjacent groups at a
// time (one per half-warp, four coefficients per lane, one 512-byte load per warp), with the next pair
// loaded before the current one is processed. Each lane keeps its own running sum for every rung (the
// rung's plane count of the lane's group picks one of the lane's nine errors), and the lanes' sums are
// added once per token at the end.
#include <cuda_fp16.h>

#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kEncodeWarps = 8;
constexpr int kEncodeTokensPerCta = 4;
constexpr int kEncodeMaxRungs = 32;
constexpr int kEncodeMaxGroups = 1024;  // rung table staged in shared memory: groups x n_rungs bytes

// floor((x - low) / span * 256) clamped to [0, 255], bit-exact with the IEEE quotient.
__device__ __forceinline__ uint32_t code_of(float y, float scale256, float span) {
  const float q = __fmul_rn(y, scale256);
  float k = floorf(q);
  const float frac = q - k;
  if (!(frac > 1e-4f && frac < 0.9999f)) k = floorf(__fmul_rn(__fdiv_rn(y, span), 256.f));
  k = fminf(fmaxf(k, 0.f), 255.f);  // NaN (0 / 0 of a constant group) -> 0, like the uint8 cast
  return static_cast<uint32_t>(k);
}
}  // namespace

template <int R>
__global__ void __launch_bounds__(kEncodeWarps * 32) encode_kernel(const EncodeParams p) {
  extern __shared__ uint8_t rung_planes_s[];  // [groups][n_rungs] (transposed: a group's rungs are adjacent)
  __shared__ float err_s[kEncodeWarps][32][9];  // a lane's nine errors (odd row stride: no bank conflicts)
  __shared__ float red[kEncodeTokensPerCta][R + 1];

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int half = lane >> 4;
  const int l16 = lane & 15;
  const int groups = p.features / 64;
  const int nr = p.n_rungs;
  for (int i = tid; i < nr * groups; i += blockDim.x) {
    const int r = i / groups, g = i % groups;  // read coalesced, store transposed
    uint8_t m = p.rung_planes[i];
    if (m > 8) {  // a plane count the codes cannot hold: report it, never index past the nine errors
      record_error(p.status, kErrBadDescriptor);
      m = 8;
    }
    rung_planes_s[g * nr + r] = m;
  }
  __syncthreads();

  const int tl = warp >> 1;                           // token of the CTA
  const int wt = warp & 1;                            // warp of the token
  const int64_t t = static_cast<int64_t>(blockIdx.x) * kEncodeTokensPerCta + tl;
  const bool active = t < p.tokens;
  float acc[R];     // this lane's sum for every rung
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  float energy = 0.f;
  float* my_err = err_s[warp][lane];
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
      const float scale256 = __fdiv_rn(256.f, span);
      float y[4];
      uint32_t code[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        y[k] = __fsub_rn(xv[k], low);
        code[k] = code_of(y[k], scale256, span);
      }
      // This lane's squared error at 0..8 planes (its four values).
      float e[9];
      e[0] = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) e[0] = fmaf(xv[k], xv[k], e[0]);
#pragma unroll
      for (int m = 1; m <= 8; ++m) {
        const float s = __fmul_rn(span, __int_as_float((127 - m) << 23));  // span / 2^m, exact
        float a = 0.f;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float idx = __fsub_rn(__uint_as_float(0x4B000000u | (code[k] >> (8 - m))), 8388607.5f);  // + 0.5
          const float d = fmaf(-idx, s, y[k]);
          a = fmaf(d, d, a);
        }
        e[m] = a;
      }
      if (valid) {
        const int64_t col = static_cast<int64_t>(g) * 64 + 4 * l16;
        *reinterpret_cast<uint32_t*>(p.codes + t * p.features + col) =
            code[0] | (code[1] << 8) | (code[2] << 16) | (code[3] << 24);
        if (l16 == 0) {
          p.low[t * groups + g] = __half_as_ushort(low_h);
          p.span[t * groups + g] = __half_as_ushort(span_h);
        }
        energy += e[0];
        // Each rung's plane count for this group picks one of the nine errors.
#pragma unroll
        for (int m = 0; m <= 8; ++m) my_err[m] = e[m];
        const uint8_t* planes = rung_planes_s + g * nr;
#pragma unroll
        for (int r = 0; r < R; ++r)
          if (r < nr) acc[r] += my_err[planes[r]];
      }
      x = xn;
      g = gnext;
    }
  }
  // Sum the lanes, then the token's two warps: warp 1 hands its sums to warp 0, which writes them.
#pragma unroll
  for (int r = 0; r < R; ++r) {
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], o);
  }
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) energy += __shfl_xor_sync(0xffffffffu, energy, o);
  if (wt == 1 && lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r) red[tl][r] = acc[r];
    red[tl][R] = energy;
  }
  __syncthreads();
  if (wt == 0 && active && lane == 0) {
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (r < nr) p.rung_error[t * nr + r] = acc[r] + red[tl][r];
    if (p.energy != nullptr) p.energy[t] = energy + red[tl][R];
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
  if (p.n_rungs <= 16)
    encode_kernel<16><<<grid, kEncodeWarps * 32, smem, stream>>>(p);
  else
    encode_kernel<32><<<grid, kEncodeWarps * 32, smem, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
