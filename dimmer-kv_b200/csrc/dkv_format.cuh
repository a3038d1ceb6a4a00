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

// The work items one CTA processes: with a static schedule, the list order[cta_begin[b] ..
// cta_begin[b+1]) (order NULL: the list positions themselves); without one, every gridDim.x-th item
// from blockIdx.x. at() returns -1 for an entry outside [0, n_items), which the caller reports.
struct ItemRange {
  int k, end, step, n_items;
  const int32_t* order;

  __device__ __forceinline__ ItemRange(const int32_t* cta_begin, const int32_t* item_order, int n)
      : ItemRange(cta_begin, item_order, n, static_cast<int>(blockIdx.x), static_cast<int>(gridDim.x)) {}
  // List `b` of `nb` (a cluster of CTAs shares one list).
  __device__ __forceinline__ ItemRange(const int32_t* cta_begin, const int32_t* item_order, int n, int b, int nb) {
    n_items = n;
    if (cta_begin != nullptr) {
      k = max(0, __ldg(cta_begin + b));
      end = __ldg(cta_begin + b + 1);
      step = 1;
      order = item_order;
      if (order == nullptr) end = min(end, n);
    } else {
      k = b;
      end = n;
      step = nb;
      order = nullptr;
    }
  }
  __device__ __forceinline__ int at(int kk) const {
    const int it = order != nullptr ? __ldg(order + kk) : kk;
    return (it >= 0 && it < n_items) ? it : -1;
  }
};

// ---------------------------------------------------------------- the cache dtype (bf16 or fp16)
// The kernels read and write 16-bit operands in the cache dtype of the call: bf16 (F16 = false) or fp16
// (F16 = true, the reference's default CompressedContext dtype). Values are kept as raw 16-bit patterns.
template <bool F16>
__device__ __forceinline__ float half_to_float(uint16_t bits) {
  if constexpr (F16) return __half2float(__ushort_as_half(bits));
  else return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}
// Two packed 16-bit values (low half first) -> float2.
template <bool F16>
__device__ __forceinline__ float2 half2_to_float2(uint32_t bits) {
  if constexpr (F16) {
    const __half2 h = *reinterpret_cast<const __half2*>(&bits);
    return __half22float2(h);
  } else {
    return make_float2(__uint_as_float(bits << 16), __uint_as_float(bits & 0xFFFF0000u));
  }
}
// Round to nearest even in the cache dtype; returns the 16-bit pattern.
template <bool F16>
__device__ __forceinline__ uint16_t float_to_half(float x) {
  if constexpr (F16) return __half_as_ushort(__float2half_rn(x));
  else return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
// Two floats rounded to the cache dtype, packed (a in the low half).
template <bool F16>
__device__ __forceinline__ uint32_t float2_to_half2(float a, float b) {
  if constexpr (F16) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}
// x rounded to the cache dtype, as a float (the reference's .to(dtype)).
template <bool F16>
__device__ __forceinline__ float round_half(float x) {
  return half_to_float<F16>(float_to_half<F16>(x));
}

// Byte j (0..15, runtime) of the 'first' table.
__device__ __forceinline__ uint32_t first_at(const GroupRegs& g, int j) {
  const uint32_t lo = (j & 4) ? g.first4[1] : g.first4[0];
  const uint32_t hi = (j & 4) ? g.first4[3] : g.first4[2];
  return (((j & 8) ? hi : lo) >> ((j & 3) * 8)) & 0xFFu;
}

// Plane count of tile token r for this group: the number of planes j with first[j] <= r (the
// table is non-decreasing and holds n_tokens past max_planes). Four bytes per subtraction: with
// r, first[j] <= 128, byte (0x80 | r) - first[j] never borrows and keeps its top bit iff r >= first[j].
__device__ __forceinline__ int planes_of(const GroupRegs& g, int r, int n_tokens) {
  if (r >= n_tokens) return 0;
  const uint32_t rr = (static_cast<uint32_t>(r) * 0x01010101u) | 0x80808080u;
  return __popc((rr - g.first4[0]) & 0x80808080u) + __popc((rr - g.first4[1]) & 0x80808080u) +
         __popc((rr - g.first4[2]) & 0x80808080u) + __popc((rr - g.first4[3]) & 0x80808080u);
}

// Bit order of a plane word: in each 32-bit half, bit 8k + b holds component 4b + k (byte k holds
// components k, k+4, ..., k+28). gather_plane drops the 32 bits of one half-word into bit s of the
// per-component bytes: byte k of acc[b] collects component 4b + k. Rotating left by s and then right
// by b moves bit 8k + b to 8k + s (and no other bit there), so each group of four components costs
// one rotate and one masked OR.
__device__ __forceinline__ void gather_plane(uint32_t (&acc)[8], uint32_t w, uint32_t s) {
  const uint32_t ws = __funnelshift_l(w, w, s);
  const uint32_t mask = 0x01010101u << s;
#pragma unroll
  for (int b = 0; b < 8; ++b) acc[b] |= __funnelshift_r(ws, ws, b) & mask;
}

// Plane words of a token with exactly M planes: all M loads are issued before any is used (one
// memory latency instead of M), then each is gathered into the per-component bytes.
template <int M>
__device__ __forceinline__ void gather_fixed(const uint8_t* blk, const GroupRegs& g, uint32_t n, uint32_t ru, int h,
                                             uint32_t seg, uint32_t (&acc)[8]) {
  uint32_t w[M];
#pragma unroll
  for (int j = 0; j < M; ++j) {
    const uint32_t fj = (g.first4[j >> 2] >> ((j & 3) * 8)) & 0xFFu;
    w[j] = *reinterpret_cast<const uint32_t*>(blk + seg + (ru - fj) * 8u + 4u * h);
    seg += (n - fj) * 8u;
  }
#pragma unroll
  for (int j = 0; j < M; ++j) gather_plane(acc, w[j], static_cast<uint32_t>(M - 1 - j));
}

// Index bits of the 32 components of half h of token r: byte k of acc[b] = index of component 4b + k
// (raw bf16: acc the high byte, acc_lo the low byte). Returns the token's plane count m (0: no planes;
// acc untouched). Tokens of a tile are sorted by plane count, so the switch is warp-uniform almost
// everywhere.
__device__ __forceinline__ int gather_index(const uint8_t* blk, const GroupRegs& g, int n_tokens, int r, int h,
                                            uint32_t (&acc)[8], uint32_t (&acc_lo)[8]) {
  const int m = planes_of(g, r, n_tokens);
  if (m == 0) return 0;
  const uint32_t n = static_cast<uint32_t>(n_tokens);
  const uint32_t ru = static_cast<uint32_t>(r);
  const uint32_t f0 = g.first4[0] & 0xFFu;
  const uint32_t seg = ((n - f0) * 4u + 7u) & ~7u;
  switch (m) {
    case 1: gather_fixed<1>(blk, g, n, ru, h, seg, acc); break;
    case 2: gather_fixed<2>(blk, g, n, ru, h, seg, acc); break;
    case 3: gather_fixed<3>(blk, g, n, ru, h, seg, acc); break;
    case 4: gather_fixed<4>(blk, g, n, ru, h, seg, acc); break;
    case 5: gather_fixed<5>(blk, g, n, ru, h, seg, acc); break;
    case 6: gather_fixed<6>(blk, g, n, ru, h, seg, acc); break;
    case 7: gather_fixed<7>(blk, g, n, ru, h, seg, acc); break;
    case 8: gather_fixed<8>(blk, g, n, ru, h, seg, acc); break;
    default: {
      // Raw bf16 (m == 16): planes 0..7 carry the high byte, 8..15 the low byte.
      uint32_t sg = seg;
      for (int j = 0; j < kMaxPlanes; ++j) {
        const uint32_t fj = first_at(g, j);
        const uint32_t w = *reinterpret_cast<const uint32_t*>(blk + sg + (ru - fj) * 8u + 4u * h);
        sg += (n - fj) * 8u;
        if (j < 8)
          gather_plane(acc, w, static_cast<uint32_t>(7 - j));
        else
          gather_plane(acc_lo, w, static_cast<uint32_t>(15 - j));
      }
    }
  }
  return m;
}

// Decode 32 components (half h of the 64-component group) of token r from a block that starts
// at `blk` (shared or global memory). `out` receives 16 packed words of two values in the cache dtype
// (bf16, or fp16 with F16; components 32h..32h+31). Raw blocks (m == 16) hold the 16-bit pattern of the
// cache dtype itself and are passed through.
// Only the token's own planes are visited. The value is the reference's float32 arithmetic then
// rounded to bf16 (the reference's .to(dtype), compressed_attention.py:76):
//   progressive (idx + 0.5) * mult / 2^m + low, ladder idx * mult + low.
// For m <= 8 the product is exact in float32 ((idx + 0.5) has at most 9 significant bits and
// mult / 2^m at most 11, an f16 value scaled by a power of two), so one fused multiply-add rounds
// exactly once, like the reference's separate multiply (exact) and add.
template <bool F16 = false>
__device__ __forceinline__ void decode_half(const uint8_t* blk, const GroupRegs& g, int n_tokens, int r, int h,
                                            uint32_t (&out)[16]) {
  uint32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  uint32_t lo[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int m = gather_index(blk, g, n_tokens, r, h, acc, lo);
  if (m == 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = 0u;
    return;
  }
  if (m == kMaxPlanes) {
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      out[2 * b] = __byte_perm(lo[b], acc[b], 0x5140);
      out[2 * b + 1] = __byte_perm(lo[b], acc[b], 0x7362);
    }
    return;
  }
  // Header: f16 low, f16 mult.
  const uint32_t f0 = first_at(g, 0);
  const uint32_t hdr = *reinterpret_cast<const uint32_t*>(blk + (static_cast<uint32_t>(r) - f0) * 4u);
  const float low = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr & 0xFFFFu)));
  const float mult = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr >> 16)));
  const bool prog = (g.kind == kKindProgressive);
  const float scale = prog ? __fmul_rn(mult, __int_as_float((127 - m) << 23)) : mult;  // exact (power of two)
  const float bias = prog ? 8388607.5f : 8388608.0f;  // float(0x4B000000 | idx) - bias = idx (+ 0.5)
  if (m <= 2) {
    // At most four distinct values: decode them once, then every output pair is one byte permute
    // selecting bf16 halves of (t0, t1 | t2, t3): the selector of pair (i0, i1) is
    // 0x1010 + 34 * (i0 | i1 << 8), computed for two pairs at once (each byte stays below 256).
    float t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) t[i] = __fmaf_rn(__fsub_rn(8388608.0f + i, bias), scale, low);
    const uint32_t tlo = float2_to_half2<F16>(t[0], t[1]), thi = float2_to_half2<F16>(t[2], t[3]);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t sel = acc[b] * 34u + 0x10101010u;
      out[2 * b] = __byte_perm(tlo, thi, sel);
      out[2 * b + 1] = __byte_perm(tlo, thi, sel >> 16);
    }
    return;
  }
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float x = __uint_as_float(__byte_perm(acc[b], 0x4B000000u, 0x7440u | k));
      v[k] = __fmaf_rn(__fsub_rn(x, bias), scale, low);
    }
    out[2 * b] = float2_to_half2<F16>(v[0], v[1]);
    out[2 * b + 1] = float2_to_half2<F16>(v[2], v[3]);
  }
}

// float32 variant of the decoder (used by the standalone unpack kernel). F16: raw blocks hold fp16
// patterns (a stream packed for an fp16 cache) instead of bf16.
template <bool F16 = false>
__device__ __forceinline__ void decode_half_f32(const uint8_t* blk, const GroupRegs& g, int n_tokens, int r, int h,
                                                float (&out)[32]) {
  uint32_t acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  uint32_t lo[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  const int m = gather_index(blk, g, n_tokens, r, h, acc, lo);
  if (m == 0 || m == kMaxPlanes) {
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      // Raw 16-bit values widened to float32 (zero when there are no planes: acc and lo are zero).
      const uint32_t p0 = __byte_perm(lo[b], acc[b], 0x5140), p1 = __byte_perm(lo[b], acc[b], 0x7362);
      const float2 a = half2_to_float2<F16>(p0), c = half2_to_float2<F16>(p1);
      out[4 * b] = a.x;
      out[4 * b + 1] = a.y;
      out[4 * b + 2] = c.x;
      out[4 * b + 3] = c.y;
    }
    return;
  }
  const uint32_t f0 = first_at(g, 0);
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
      out[4 * b + k] = __fmaf_rn(__fsub_rn(x, bias), scale, low);
    }
  }
}

}  // namespace dkv
