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
// A unit is 16 consecutive components of a (token, group): their codes are 4 (w = 2), 8 (w = 4) or 16
// (w = 8) bytes, read byte by byte because the format packs its arrays without alignment; the values go
// out as four 16-byte stores. Each thread restores two units (units t and t + 256 of its CTA's 512) and
// loads both units' codes before it reads their row and group indices. The segment record is read once
// per CTA.
#include <cuda_fp16.h>

#include "dkv_kernels.h"
#include "dkv_ptx.cuh"

namespace dkv {

namespace {
constexpr int kStorageThreads = 256;
constexpr int kUnitsPerThread = 2;  // units of 16 components restored by each thread

__device__ __forceinline__ float f16_at(const uint8_t* data, uint64_t at) {
  const unsigned short bits = static_cast<unsigned short>(__ldg(data + at) | (__ldg(data + at + 1) << 8));
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
  const uint32_t q0 = blockIdx.x * (kStorageThreads * kUnitsPerThread) + threadIdx.x;
  if (q0 >= units) return;
  const int w = sg.width;
  if (w != 2 && w != 4 && w != 8) {
    record_error(p.status, kErrBadDescriptor);
    return;
  }
  const int nbytes = 2 * w;  // 16 codes x w bits
  // Phase 1, for each of the thread's units: the 2w bytes of codes, read byte by byte (the format aligns
  // nothing) as little-endian words, and the group's f16 low / scale. They depend only on the segment
  // record, so every unit's loads are issued before the row and group indices are read.
  uint32_t words[kUnitsPerThread][4];
  float low[kUnitsPerThread], scale[kUnitsPerThread];
  bool live[kUnitsPerThread];
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    const uint32_t q = q0 + u * kStorageThreads;
    const uint32_t tg = q >> 2;  // (token, group) index
    const uint64_t byte0 = sg.codes_offset + (static_cast<uint64_t>(q) * 16u * static_cast<uint32_t>(w)) / 8u;
    const uint64_t hdr = static_cast<uint64_t>(tg) * 2;
    live[u] = q < units;
    words[u][0] = words[u][1] = words[u][2] = words[u][3] = 0u;
    low[u] = scale[u] = 0.0f;
    if (!live[u]) continue;
    if (byte0 + nbytes > p.data_size || sg.low_offset + hdr + 2 > p.data_size ||
        sg.scale_offset + hdr + 2 > p.data_size) {
      record_error(p.status, kErrBadDescriptor);
      live[u] = false;
      continue;
    }
#pragma unroll
    for (int b = 0; b < 16; ++b)
      if (b < nbytes) words[u][b >> 2] |= static_cast<uint32_t>(__ldg(p.data + byte0 + b)) << (8 * (b & 3));
    low[u] = f16_at(p.data, sg.low_offset + hdr);
    scale[u] = f16_at(p.data, sg.scale_offset + hdr);
  }
  // Phase 2: row and group of each unit, then its 16 values (code * scale + low, a float32 multiply then
  // add as the reference's torch ops) as four 16-byte stores.
  const uint32_t mask = (1u << w) - 1u;
#pragma unroll
  for (int u = 0; u < kUnitsPerThread; ++u) {
    if (!live[u]) continue;
    const uint32_t q = q0 + u * kStorageThreads;
    const uint32_t tg = q >> 2;
    const int i = static_cast<int>(tg / static_cast<uint32_t>(sg.n_groups));
    const int j = static_cast<int>(tg - static_cast<uint32_t>(i) * static_cast<uint32_t>(sg.n_groups));
    const int c = static_cast<int>(q & 3u) * 16;  // first of the unit's 16 components
    if (sg.rows_offset < 0 || sg.groups_offset < 0 || static_cast<int64_t>(sg.rows_offset) + i >= p.n_rows_idx ||
        static_cast<int64_t>(sg.groups_offset) + j >= p.n_groups_idx) {
      record_error(p.status, kErrBadDescriptor);
      continue;
    }
    const int row = __ldg(p.rows + sg.rows_offset + i);
    const int group = __ldg(p.groups + sg.groups_offset + j);
    if (row < 0 || row >= p.out_rows || group < 0 || (static_cast<int64_t>(group) + 1) * 64 > p.out_cols) {
      record_error(p.status, kErrBadDescriptor);
      continue;
    }
    float4* dst = reinterpret_cast<float4*>(p.out + static_cast<int64_t>(row) * p.out_cols + group * 64 + c);
#pragma unroll
    for (int k4 = 0; k4 < 4; ++k4) {
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int bit = (4 * k4 + k) * w;  // bit of code 4 k4 + k in the unit's little-endian run
        const float code = static_cast<float>((words[u][bit >> 5] >> (bit & 31)) & mask);
        v[k] = __fadd_rn(__fmul_rn(code, scale[u]), low[u]);
      }
      dst[k4] = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}

int run_storage_unpack(const StorageParams& p, cudaStream_t stream) {
  if (p.n_segments < 0 || p.out_cols % 64 != 0 || p.max_units < 0) return kDkvErrArgs;
  if (reinterpret_cast<uintptr_t>(p.out) & 15u) return kDkvErrArgs;
  if (p.n_segments == 0 || p.max_units == 0) return kDkvOk;
  if (p.n_segments > 65535 || p.max_units >= (int64_t{1} << 31)) return kDkvErrConfig;
  const int64_t per_cta = static_cast<int64_t>(kStorageThreads) * kUnitsPerThread;
  const int64_t blocks = (p.max_units + per_cta - 1) / per_cta;
  storage_unpack_kernel<<<dim3(static_cast<unsigned>(blocks), p.n_segments), kStorageThreads, 0, stream>>>(p);
  return cudaGetLastError() == cudaSuccess ? kDkvOk : kDkvErrCuda;
}

}  // namespace dkv
