// storage.cu — restore of the kvtc byte format: bit-packed ladder codes -> dense coefficients.
//
// Replaces the per-rung, per-width loop of kvtc_storage.decode_bytes (scripts/kvtc_storage.py:103-114):
// for every (rung, bit width) segment of a stream, the packed w-bit codes of count tokens x n_groups
// groups x 64 components (8 / w codes per byte, the first in the low bits) and their f16 low and scale
// become codes * scale + low (float32 multiply, then add, as the reference's torch ops) in the rows of
// the segment's tokens and the columns of its groups. The host walks the format (the rung of every
// token is in the clear, so every segment's offsets follow) and lists the segments; one launch
// restores a whole stream.
//
// One thread per 16 consecutive components of a (token, group): their codes are 4 (w = 2), 8 (w = 4) or
// 16 (w = 8) bytes, read byte by byte because the format packs its arrays without alignment; the values
// go out as four 16-byte stores. The segment record is read once per CTA.
#include <cuda_fp16.h>

#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kStorageThreads = 256;

__device__ __forceinline__ float f16_at(const uint8_t* data, uint64_t at) {
  const unsigned short bits = static_cast<unsigned short>(data[at] | (data[at + 1] << 8));
  return __half2float(__ushort_as_half(bits));
}
}  // namespace

__global__ void __launch_bounds__(kStorageThreads) storage_unpack_kernel(const StorageParams p) {
  __shared__ StorageSegment sg_s;
  if (threadIdx.x == 0) sg_s = p.segments[blockIdx.y];
  __syncthreads();
  const StorageSegment sg = sg_s;
  if (sg.count < 0 || sg.n_groups <= 0 || static_cast<int64_t>(sg.count) * sg.n_groups * 4 > p.max_units) {
    if (threadIdx.x == 0 && blockIdx.x == 0) record_error(p.status, kErrBadDescriptor);
    return;
  }
  // Units of a segment: at most max_units < 2^31 (checked here and on the host), so 32-bit index math.
  const uint32_t units = static_cast<uint32_t>(sg.count) * static_cast<uint32_t>(sg.n_groups) * 4u;
  const uint32_t q = blockIdx.x * kStorageThreads + threadIdx.x;
  if (q >= units) return;
  const int w = sg.width;
  if (w != 2 && w != 4 && w != 8) {
    record_error(p.status, kErrBadDescriptor);
    return;
  }
  const uint32_t tg = q >> 2;                   // (token, group) index
  const int i = static_cast<int>(tg / static_cast<uint32_t>(sg.n_groups));
  const int j = static_cast<int>(tg - static_cast<uint32_t>(i) * static_cast<uint32_t>(sg.n_groups));
  const int c = static_cast<int>(q & 3u) * 16;  // first of the thread's 16 components
  const uint64_t byte0 = sg.codes_offset + (static_cast<uint64_t>(q) * 16u * static_cast<uint32_t>(w)) / 8u;
  const int nbytes = 2 * w;                      // 16 codes x w bits
  const uint64_t hdr = static_cast<uint64_t>(tg) * 2;
  if (byte0 + nbytes > p.data_size || sg.low_offset + hdr + 2 > p.data_size ||
      sg.scale_offset + hdr + 2 > p.data_size) {
    record_error(p.status, kErrBadDescriptor);
    return;
  }
  if (sg.rows_offset < 0 || sg.groups_offset < 0 || static_cast<int64_t>(sg.rows_offset) + i >= p.n_rows_idx ||
      static_cast<int64_t>(sg.groups_offset) + j >= p.n_groups_idx) {
    record_error(p.status, kErrBadDescriptor);
    return;
  }
  const int row = p.rows[sg.rows_offset + i];
  const int group = p.groups[sg.groups_offset + j];
  if (row < 0 || row >= p.out_rows || group < 0 || (static_cast<int64_t>(group) + 1) * 64 > p.out_cols) {
    record_error(p.status, kErrBadDescriptor);
    return;
  }
  // The thread's 2w bytes of codes, read byte by byte (the format aligns nothing), as little-endian words.
  uint32_t words[4] = {0u, 0u, 0u, 0u};
#pragma unroll
  for (int b = 0; b < 16; ++b)
    if (b < nbytes) words[b >> 2] |= static_cast<uint32_t>(p.data[byte0 + b]) << (8 * (b & 3));
  const uint32_t mask = (1u << w) - 1u;
  const float low = f16_at(p.data, sg.low_offset + hdr);
  const float scale = f16_at(p.data, sg.scale_offset + hdr);
  float4* dst = reinterpret_cast<float4*>(p.out + static_cast<int64_t>(row) * p.out_cols + group * 64 + c);
#pragma unroll
  for (int k4 = 0; k4 < 4; ++k4) {
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int bit = (4 * k4 + k) * w;  // bit of code 4 k4 + k in the thread's little-endian run
      const float code = static_cast<float>((words[bit >> 5] >> (bit & 31)) & mask);
      v[k] = __fadd_rn(__fmul_rn(code, scale), low);
    }
    dst[k4] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

int run_storage_unpack(const StorageParams& p, cudaStream_t stream) {
  if (p.n_segments < 0 || p.out_cols % 64 != 0 || p.max_units < 0) return kDkvErrArgs;
  if (reinterpret_cast<uintptr_t>(p.out) & 15u) return kDkvErrArgs;
  if (p.n_segments == 0 || p.max_units == 0) return kDkvOk;
  if (p.n_segments > 65535 || p.max_units >= (int64_t{1} << 31)) return kDkvErrConfig;
  const int64_t blocks = (p.max_units + kStorageThreads - 1) / kStorageThreads;
  storage_unpack_kernel<<<dim3(static_cast<unsigned>(blocks), p.n_segments), kStorageThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
