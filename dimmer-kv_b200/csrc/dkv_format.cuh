// dkv_format.cuh — the packed plane-stream layout and its decoder.
//
// A compressed stream (keys or values of a batch of conversations) is a list of
// tiles of up to 128 tokens. Tokens inside a tile are sorted by precision step,
// so for every coefficient group the tokens that hold plane j form a suffix of
// the tile. Each (tile, group) block stores, contiguously:
//   headers  : one (f16 low, f16 mult) pair per token holding >= 1 plane, padded to 8 B
//   plane j  : one 64-bit word per token holding plane j (bit c = component c), j = 0, 1, ...
// padded to 16 B so that blocks can be fetched with cp.async.bulk.
// A token with m planes stores the m-bit index most-significant plane first.
// Decoding (the reference arithmetic, float32, no contraction):
//   progressive (scripts/progressive.py:47-55):  v = low + (idx + 0.5) * mult / 2^m
//   ladder      (scripts/kvtc.py:78):             v = idx * mult + low
//   m == 16 ("raw", the ladder's exact rung):     the 16 index bits are the bf16 value
#pragma once
#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace dkv {

constexpr int kTileTokens = 128;
constexpr int kGroup = 64;
constexpr int kMaxPlanes = 16;
constexpr int kKindProgressive = 0;
constexpr int kKindLadder = 1;

struct TileDesc {
  int32_t seq;         // conversation index in the batch
  int32_t token_base;  // first token of the tile in the stream's per-token arrays
  int32_t n_tokens;    // 1..128
  int32_t n_groups;    // blocks stored for this tile
  int32_t group_base;  // first GroupDesc of the tile
  int32_t score_base;  // position of the tile's first token inside its conversation's score order
  int32_t reserved0;
  int32_t reserved1;
};
static_assert(sizeof(TileDesc) == 32, "TileDesc is 32 bytes");

struct GroupDesc {
  uint32_t group;        // union group index (coefficient columns group*64 .. group*64+63)
  uint32_t code_offset;  // byte offset of the block in the code buffer (16-byte aligned)
  uint32_t code_bytes;   // block size (multiple of 16)
  uint8_t kind;          // kKindProgressive or kKindLadder
  uint8_t max_planes;    // planes stored for the finest token of the tile
  uint8_t pad0, pad1;
  uint8_t first[16];     // first[j]: first token (in the tile) holding plane j; n_tokens if none
};
static_assert(sizeof(GroupDesc) == 32, "GroupDesc is 32 bytes");

// A GroupDesc held in registers (the 16 'first' bytes as four words).
struct GroupRegs {
  uint32_t group, code_offset, code_bytes;
  int kind, max_planes;
  uint32_t first4[4];
  __device__ __forceinline__ int first(int j) const { return (first4[j >> 2] >> ((j & 3) * 8)) & 0xFF; }
};

__device__ __forceinline__ GroupRegs group_from_words(uint4 a, uint4 b) {
  GroupRegs r;
  r.group = a.x;
  r.code_offset = a.y;
  r.code_bytes = a.z;
  r.kind = static_cast<int>(a.w & 0xFF);
  r.max_planes = static_cast<int>((a.w >> 8) & 0xFF);
  r.first4[0] = b.x;
  r.first4[1] = b.y;
  r.first4[2] = b.z;
  r.first4[3] = b.w;
  return r;
}

__device__ __forceinline__ GroupRegs load_group(const GroupDesc* g) {
  const uint4* p = reinterpret_cast<const uint4*>(g);
  return group_from_words(__ldg(p), __ldg(p + 1));
}

// A code slot keeps the 32-byte descriptor of the block it holds in its last 32 bytes: the
// producer writes it before issuing the block's bulk copy, the consumers read it after the copy's
// mbarrier completes (arrive has release, try_wait acquire semantics).
__device__ __forceinline__ void stash_group(uint8_t* slot_end, const GroupDesc* g) {
  const uint4* src = reinterpret_cast<const uint4*>(g);
  uint4* dst = reinterpret_cast<uint4*>(slot_end - 32);
  dst[0] = __ldg(src);
  dst[1] = __ldg(src + 1);
}

__device__ __forceinline__ GroupRegs stashed_group(const uint8_t* slot_end) {
  const uint4* src = reinterpret_cast<const uint4*>(slot_end - 32);
  return group_from_words(src[0], src[1]);
}

// Byte j (0..15, runtime) of the 'first' table.
__device__ __forceinline__ uint32_t first_at(const GroupRegs& g, int j) {
  const uint32_t lo = (j & 4) ? g.first4[1] : g.first4[0];
  const uint32_t hi = (j & 4) ? g.first4[3] : g.first4[2];
  return (((j & 8) ? hi : lo) >> ((j & 3) * 8)) & 0xFFu;
}

// Plane count of tile token r for this group: the number of planes j with first[j] <= r (the
// table is non-decreasing and holds n_tokens past max_planes), four bytes per SIMD compare.
__device__ __forceinline__ int planes_of(const GroupRegs& g, int r, int n_tokens) {
  if (r >= n_tokens) return 0;
  const uint32_t rr = static_cast<uint32_t>(r) * 0x01010101u;
  return (__popc(__vcmpgeu4(rr, g.first4[0])) + __popc(__vcmpgeu4(rr, g.first4[1])) +
          __popc(__vcmpgeu4(rr, g.first4[2])) + __popc(__vcmpgeu4(rr, g.first4[3]))) >> 3;
}

// Spread the four bits (4b .. 4b+3) of a plane word into bit s of four bytes.
__device__ __forceinline__ uint32_t spread4(uint32_t w, int b, uint32_t s) {
  return ((((w >> (4 * b)) & 0xFu) * (0x204081u << s)) & (0x01010101u << s));
}

// Decode 32 components (half h of the 64-component group) of token r from a block that starts
// at `blk` (shared or global memory). `out` receives 16 packed bf16x2 words (components 32h..32h+31).
// Only the token's own planes are visited; the float arithmetic is the reference's, in float32
// with no contraction, then rounded to bf16 (the reference's .to(dtype), compressed_attention.py:76).
__device__ __forceinline__ void decode_half(const uint8_t* blk, const GroupRegs& g, int n_tokens, int r, int h,
                                            uint32_t (&out)[16]) {
  const int m = planes_of(g, r, n_tokens);
  if (m == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = 0u;
    return;
  }
  const uint32_t n = static_cast<uint32_t>(n_tokens);
  const uint32_t f0 = first_at(g, 0);
  uint32_t seg = ((n - f0) * 4u + 7u) & ~7u;
  if (m == kMaxPlanes) {
    // Raw bf16: planes 0..7 carry the high byte, 8..15 the low byte.
    uint32_t hi[8] = {0, 0, 0, 0, 0, 0, 0, 0}, lo[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    for (int j = 0; j < kMaxPlanes; ++j) {
      const uint32_t fj = first_at(g, j);
      const uint32_t w = *reinterpret_cast<const uint32_t*>(blk + seg + (static_cast<uint32_t>(r) - fj) * 8u + 4u * h);
      seg += (n - fj) * 8u;
      const uint32_t s = 7u - static_cast<uint32_t>(j & 7);
      if (j < 8) {
#pragma unroll
        for (int b = 0; b < 8; ++b) hi[b] |= spread4(w, b, s);
      } else {
#pragma unroll
        for (int b = 0; b < 8; ++b) lo[b] |= spread4(w, b, s);
      }
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      out[2 * b] = __byte_perm(lo[b], hi[b], 0x5140);
      out[2 * b + 1] = __byte_perm(lo[b], hi[b], 0x7362);
    }
    return;
  }
  // Gather the m index bits of every component into the bytes of acc[b] (components 4b..4b+3).
  uint32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int j = 0; j < m; ++j) {
    const uint32_t fj = first_at(g, j);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(blk + seg + (static_cast<uint32_t>(r) - fj) * 8u + 4u * h);
    seg += (n - fj) * 8u;
    const uint32_t s = static_cast<uint32_t>(m - 1 - j);
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[b] |= spread4(w, b, s);
  }
  // Header: f16 low, f16 mult.
  const uint32_t hdr = *reinterpret_cast<const uint32_t*>(blk + (static_cast<uint32_t>(r) - f0) * 4u);
  const float low = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr & 0xFFFFu)));
  const float mult = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr >> 16)));
  // progressive: (idx + 0.5) * (span * 2^-m)  == ((idx + 0.5) * span) / 2^m exactly (power-of-two scaling)
  // ladder:      idx * scale
  const bool prog = (g.kind == kKindProgressive);
  const float scale = prog ? __fmul_rn(mult, __int_as_float((127 - m) << 23)) : mult;
  const float bias = prog ? 8388607.5f : 8388608.0f;  // float(0x4B000000 | idx) - bias = idx (+ 0.5)
  if (m <= 2) {
    // At most four distinct values: decode them once (same arithmetic), then every output pair is
    // one byte permute selecting bf16 halves: pair (idx0, idx1) <- selector 0x1010 + 34*(idx0 | idx1 << 8).
    float t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) t[i] = __fadd_rn(__fmul_rn(__fsub_rn(8388608.0f + i, bias), scale), low);
    __nv_bfloat162 v01 = __floats2bfloat162_rn(t[0], t[1]);
    __nv_bfloat162 v23 = __floats2bfloat162_rn(t[2], t[3]);
    const uint32_t lo = *reinterpret_cast<uint32_t*>(&v01), hi = *reinterpret_cast<uint32_t*>(&v23);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      out[2 * b] = __byte_perm(lo, hi, 0x1010u + 34u * (acc[b] & 0xFFFFu));
      out[2 * b + 1] = __byte_perm(lo, hi, 0x1010u + 34u * (acc[b] >> 16));
    }
    return;
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = __uint_as_float(__byte_perm(acc[b], 0x4B000000u, 0x7440u | k));
      v[k] = __fadd_rn(__fmul_rn(__fsub_rn(x, bias), scale), low);
    }
    __nv_bfloat162 p0 = __floats2bfloat162_rn(v[0], v[1]);
    __nv_bfloat162 p1 = __floats2bfloat162_rn(v[2], v[3]);
    out[2 * b] = *reinterpret_cast<uint32_t*>(&p0);
    out[2 * b + 1] = *reinterpret_cast<uint32_t*>(&p1);
  }
}

// float32 variant of the decoder (used by the standalone unpack kernel).
__device__ __forceinline__ void decode_half_f32(const uint8_t* blk, const GroupRegs& g, int n_tokens, int r, int h,
                                                float (&out)[32]) {
  const int m = planes_of(g, r, n_tokens);
  if (m == 0 || m == kMaxPlanes) {
    uint32_t packed[16];
    decode_half(blk, g, n_tokens, r, h, packed);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      out[2 * i] = __uint_as_float(packed[i] << 16);
      out[2 * i + 1] = __uint_as_float(packed[i] & 0xFFFF0000u);
    }
    return;
  }
  const uint32_t n = static_cast<uint32_t>(n_tokens);
  const uint32_t f0 = first_at(g, 0);
  uint32_t seg = ((n - f0) * 4u + 7u) & ~7u;
  uint32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  for (int j = 0; j < m; ++j) {
    const uint32_t fj = first_at(g, j);
    const uint32_t w = *reinterpret_cast<const uint32_t*>(blk + seg + (static_cast<uint32_t>(r) - fj) * 8u + 4u * h);
    seg += (n - fj) * 8u;
    const uint32_t s = static_cast<uint32_t>(m - 1 - j);
#pragma unroll
    for (int b = 0; b < 8; ++b) acc[b] |= spread4(w, b, s);
  }
  const uint32_t hdr = *reinterpret_cast<const uint32_t*>(blk + (static_cast<uint32_t>(r) - f0) * 4u);
  const float low = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr & 0xFFFFu)));
  const float mult = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr >> 16)));
  const bool prog = (g.kind == kKindProgressive);
  const float scale = prog ? __fmul_rn(mult, __int_as_float((127 - m) << 23)) : mult;
  const float bias = prog ? 8388607.5f : 8388608.0f;
#pragma unroll
  for (int b = 0; b < 8; ++b) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = __uint_as_float(__byte_perm(acc[b], 0x4B000000u, 0x7440u | k));
      out[4 * b + k] = __fadd_rn(__fmul_rn(__fsub_rn(x, bias), scale), low);
    }
  }
}

}  // namespace dkv
