// unpack.cu — ragged bit-plane unpack to dense PCA coefficients.
//
// Replaces progressive.dequantize (scripts/progressive.py:47-55) for a packed stream, and the
// ladder decode of kvtc.quantize_groups (scripts/kvtc.py:78): every token of every tile is
// decoded at its own plane count, one CTA per tile, two threads per token (32 components each).
// Plane words are read straight from global memory with 128-bit loads per 4 words where
// aligned; output rows are written in stream order, columns = union group * 64 + component.
#include "dkv_format.cuh"
#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

__global__ void __launch_bounds__(256) unpack_kernel(const UnpackParams p) {
  const int ti = blockIdx.x;
  const TileDesc tile = p.tiles[ti];
  const int r = threadIdx.x & 127;
  const int h = threadIdx.x >> 7;
  if (tile.n_tokens < 1 || tile.n_tokens > kTileTokens) {
    record_error(p.status, kErrBadDescriptor);
    return;
  }
  if (r >= tile.n_tokens) return;
  const int64_t row = static_cast<int64_t>(tile.token_base + r);
  for (int gi = 0; gi < tile.n_groups; ++gi) {
    const GroupRegs gr = load_group(&p.groups[tile.group_base + gi]);
    if (static_cast<uint64_t>(gr.code_offset) + gr.code_bytes > p.code_size ||
        static_cast<int64_t>(gr.group + 1) * kGroup > p.out_cols) {
      record_error(p.status, kErrBadDescriptor);
      return;
    }
    const uint8_t* blk = p.code + gr.code_offset;
    const int64_t col = static_cast<int64_t>(gr.group) * kGroup + 32 * h;
    if (p.out_bf16) {
      uint32_t out[16];
      decode_half(blk, gr, tile.n_tokens, r, h, out);
      uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(p.out) + row * p.out_cols + col);
#pragma unroll
      for (int k = 0; k < 4; ++k) dst[k] = make_uint4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
    } else {
      float out[32];
      decode_half_f32(blk, gr, tile.n_tokens, r, h, out);
      float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + row * p.out_cols + col);
#pragma unroll
      for (int k = 0; k < 8; ++k) dst[k] = make_float4(out[4 * k], out[4 * k + 1], out[4 * k + 2], out[4 * k + 3]);
    }
  }
}

int run_unpack(const UnpackParams& p, cudaStream_t stream) {
  if (p.n_tiles == 0) return kDkvOk;
  if (p.out_cols % 64 != 0) return kDkvErrArgs;
  unpack_kernel<<<p.n_tiles, 256, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
