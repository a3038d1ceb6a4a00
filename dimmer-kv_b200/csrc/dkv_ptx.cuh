// dkv_ptx.cuh — sm_100a building blocks used by every DimmerKV kernel:
// mbarriers with bounded waits, bulk / tensor (TMA) copies, tcgen05 MMA,
// TMEM allocation and loads, shared-memory matrix descriptors.
//
// Every wait in this file is bounded (about two seconds, on two independent
// clocks). A wait that runs out records an error code in the caller's status
// word and returns false; callers then stop issuing work and leave through the
// normal exit path (TMEM freed, no copy left in flight that the CTA still waits
// on). Kernels also read the status word as they start and do no work when an
// earlier kernel has recorded an error.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda.h>

namespace dkv {

// ---------------------------------------------------------------- errors
// Status words written by kernels (first error wins).
enum DeviceError : int {
  kErrNone = 0,
  kErrWaitCodes = 101,     // waiting for a plane block copy
  kErrWaitBasis = 102,     // waiting for a basis tile (TMA)
  kErrWaitA = 103,         // MMA waiting for an unpacked operand tile
  kErrWaitEmpty = 104,     // producer waiting for a free stage
  kErrWaitAccum = 105,     // epilogue waiting for the accumulator
  kErrWaitAccumFree = 106, // MMA waiting for the epilogue to drain TMEM
  kErrWaitDrain = 107,     // exit path waiting for outstanding async work
  kErrBadDescriptor = 110, // a tile / group descriptor failed its bounds check
};
// The kernel that recorded an error, added to the code (the host names it): status = site + error.
constexpr int kSiteKeyPair = 1000;     // key_scores_pair_kernel (CTA pairs)
constexpr int kSiteKey = 2000;         // key_scores_kernel (one CTA per item)
constexpr int kSiteValue = 3000;       // value_weights_kernel / vprobs_kernel (planes decoded per layer)
constexpr int kSiteValueDense = 4000;  // value_dense_kernel (coefficients decoded once per step)
constexpr int kSiteUnpack = 5000;      // unpack_kernel
constexpr int kSiteKeyDense = 6000;    // key_scores_dense_kernel (coefficients decoded once per step)

// Bound on one wait. Healthy waits in these kernels last microseconds; a wait gives up after 2 s of
// %globaltimer time. The time is summed over polls in steps clamped to 100 ms (a step backwards counts as
// nothing), so that a jump of the timer (it follows the host's clock) cannot end a healthy wait early.
// Polls are mbarrier.try_wait, which suspends the thread until the phase completes (the efficient wait of
// a pipeline) or for at most the suspend-time hint, kPollSuspendNs; the deadline is checked between polls.
// Times are kept in units of 1.024 us (ns >> 10).
constexpr uint32_t kWaitDeadline1024 = 2000000000u / 1024u;
constexpr uint32_t kWaitStepCap1024 = 100000000u / 1024u;
constexpr uint32_t kPollSuspendNs = 1000000u;

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Elapsed-time bookkeeping of one bounded wait (started after its first unsuccessful poll).
struct WaitClock {
  uint32_t last, elapsed;
  __device__ __forceinline__ WaitClock() : last(static_cast<uint32_t>(global_ns() >> 10)), elapsed(0) {}
  // True once the wait has run out.
  __device__ __forceinline__ bool expired() {
    const uint32_t t = static_cast<uint32_t>(global_ns() >> 10);
    const int32_t step = static_cast<int32_t>(t - last);
    last = t;
    if (step > 0) elapsed += static_cast<uint32_t>(step) < kWaitStepCap1024 ? static_cast<uint32_t>(step) : kWaitStepCap1024;
    return elapsed > kWaitDeadline1024;
  }
};

__device__ __forceinline__ void record_error(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

// A wait that ran out: its code (kernel site + error, below 10^4) and, in the decimal digits above, the
// barrier that did not complete (its shared-memory address / 8, modulo 10^5): status = barrier * 10^4 +
// code. The host prints both.
__device__ __forceinline__ void record_wait_error(int* status, int code, uint32_t bar_saddr) {
  record_error(status, static_cast<int>((bar_saddr >> 3) % 100000u) * 10000 + code);
}

// The call's status word as the kernel starts: non-zero when an earlier kernel of the call (or of an
// earlier call sharing the word) failed. Kernels that find it set do no work and leave at once.
__device__ __forceinline__ int status_at_entry(const int* status) {
  return status != nullptr ? *reinterpret_cast<const volatile int*>(status) : 0;
}

// CTA-uniform entry check for kernels that use __syncthreads: every thread gets the same answer.
__device__ __forceinline__ bool cta_failed_at_entry(const int* status) {
  return __syncthreads_or(threadIdx.x == 0 && status_at_entry(status) != 0) != 0;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Non-blocking test of the phase with the given parity (for a thread that polls several barriers).
// Test of the phase with the given parity that may suspend the thread until the phase completes, for at
// most kPollSuspendNs.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kPollSuspendNs)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. With `abort` (the CTA's abort flag in
// shared memory), the wait also ends, without an error of its own, as soon as another role of the CTA
// (or of its cluster) has given up, so that one failure ends every wait within microseconds. Waits
// that drain the thread's own copies or MMAs in flight pass no abort flag: those always complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          const volatile int* abort = nullptr) {
  if (mbar_try_wait(bar, parity)) return true;
  WaitClock clock;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort != nullptr && *abort != 0) return false;
    if (clock.expired()) {
      record_wait_error(status, code, smem_u32(bar));
      return false;
    }
  }
}

// The same wait taken by every lane of a warp, with one answer for the whole warp (a warp vote), so
// that the lanes never split between a loop's exit and the warp-wide (.sync.aligned) instructions that
// follow a wait (tcgen05.ld, setmaxnreg, __syncwarp). All 32 lanes must call it.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, int* status, int code,
                                          const volatile int* abort) {
  return __all_sync(0xffffffffu, mbar_wait(bar, parity, status, code, abort)) != 0;
}

// Rendezvous of a fixed group of threads on one of two mbarriers used alternately (each initialised
// with the group's size), bounded like every other wait, so a thread that gave up on an earlier wait
// never leaves the rest of the group blocked. n counts this thread's rendezvous so far. Called by whole
// warps; the answer is the same for every lane of a warp.
__device__ __forceinline__ bool group_sync(uint64_t* bars2, uint32_t& n, int* status, int code,
                                           const volatile int* abort) {
  uint64_t* bar = bars2 + (n & 1);
  const uint32_t parity = (n >> 1) & 1;
  ++n;
  mbar_arrive(bar);
  return warp_wait(bar, parity, status, code, abort);
}

// ---------------------------------------------------------------- copies
// 1-D bulk copy global -> shared, completion counted on an mbarrier in bytes.
// Both addresses 16-byte aligned, size a multiple of 16.
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 2-D tiled tensor copy (TMA) global -> shared. x is the innermost coordinate.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------- packed fp32 pairs (sm_100)
// Two fp32 values in one 64-bit register, low word first; each lane of add / mul / fma.rn.f32x2 rounds like
// the scalar fp32 instruction.
__device__ __forceinline__ uint64_t f32x2_pack(uint32_t lo, uint32_t hi) {
  uint64_t d;
  asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "r"(lo), "r"(hi));
  return d;
}
__device__ __forceinline__ float f32x2_sum(uint64_t v) {
  uint32_t lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(lo), "=r"(hi) : "l"(v));
  return __uint_as_float(lo) + __uint_as_float(hi);
}
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t mul_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t fma_f32x2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}

// Bring the line holding addr into L1 (no data returned, nothing to wait for).
__device__ __forceinline__ void prefetch_l1(const void* addr) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<uint64_t>(addr)));
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async
// proxy (tcgen05.mma operand reads, bulk copies).
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 or fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; the warp's lane quarter is encoded in taddr[31:16].
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// After tmem_ld_wait: ties the registers a tcgen05.ld wrote to the wait, so that no use of them can be
// scheduled before it (the load writes them asynchronously).
__device__ __forceinline__ void tmem_reg_fence(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]));
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 "version 1" layout).
//   K-major operand:  SBO = byte stride between 8-row groups (1024 for dense rows of 128 B), LBO unused (16).
//   MN-major operand: LBO = byte stride between 64-element MN atoms, SBO = byte stride between 8-row K groups.
// The tile base must be 1024-byte aligned; K steps inside a K-major atom advance the start by 32 B.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
// is_bf16: A and B are bf16 (else fp16; both operands always share one type).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool is_bf16, bool a_mn_major, bool b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | ((is_bf16 ? 1u : 0u) << 7)                // A format
         | ((is_bf16 ? 1u : 0u) << 10)               // B format
         | ((a_mn_major ? 1u : 0u) << 15)            // A major-ness
         | ((b_mn_major ? 1u : 0u) << 16)            // B major-ness
         | (static_cast<uint32_t>(N >> 3) << 17)     // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);    // M / 16
}

// Byte offset of the 16-byte chunk `chunk` (0..7) of row `row` inside a
// 128B-swizzled tile whose rows are 128 bytes long.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

// ---------------------------------------------------------------- clusters (CTA pairs)
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's). Default
// semantics (release, CTA scope), as the CUTLASS two-SM pipelines use for operand hand-off: a writer of
// an MMA operand issues fence.proxy.async first; a cluster-scope release here would be a full fence
// per arrival.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// Store a 32-bit word at a shared::cluster address (this CTA's or the peer's shared memory).
__device__ __forceinline__ void st_cluster_u32(uint32_t cluster_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cluster_addr), "r"(v) : "memory");
}

__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMEM shared by a CTA pair: issued by the same warp in both CTAs, with the same destination slot.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A x B over the CTA pair (M = 256: rows 0-127 from this CTA's A tile, 128-255 from the
// peer's at the same shared-memory address; B's N columns likewise split between the two CTAs).
// Issued by one thread of the even CTA.
__device__ __forceinline__ void mma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the mbarrier at this shared-memory offset in every CTA of `cta_mask` once the pair MMAs
// issued so far complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// Per-warpgroup register budgets (all four warps of a warpgroup execute the same instruction).
// The budgets of a CTA's warpgroups must fit the registers it was launched with.
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

// Named barrier `id` over `threads` threads (a multiple of 32): every warp of the participating set
// executes it once, from whatever code location its role is at.
__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ uint32_t elect_lane0() { return (threadIdx.x & 31u) == 0u; }

__device__ __forceinline__ int warp_id() { return static_cast<int>(threadIdx.x >> 5); }

}  // namespace dkv
