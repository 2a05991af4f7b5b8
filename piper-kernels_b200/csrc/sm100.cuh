// sm_100a primitives used by the Piper Attention kernels: mbarriers with
// bounded waits, TMA tile loads (no multicast), 1-D bulk copies, TMEM
// allocation, tcgen05.mma kind::i8 issue/commit, tcgen05.ld/st.
//
// Every wait here is bounded: it gives up after a wall-clock budget (the
// %globaltimer nanosecond clock), records a status word in device memory and
// returns false, so no kernel built on these helpers can spin forever.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace piper {

// Device-side status word: 0 = ok.  Bits record which class of wait gave up.
enum : uint32_t {
  kStatusTimeoutFull = 1u << 0,   // consumer waited for data that never arrived
  kStatusTimeoutEmpty = 1u << 1,  // producer waited for a slot that never freed
  kStatusTimeoutMma = 1u << 2,    // tensor-core completion never signalled
  kStatusTimeoutDrain = 1u << 3,  // in-flight copies not drained at exit
  kStatusBadLaunch = 1u << 4,     // launch shape inconsistent with the plan
  kStatusTimeoutProbe = 1u << 5,  // the self-test wait (nothing ever arrives)
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Largest of three floats (a NaN input is ignored, as by fmaxf).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// ---------------------------------------------------------------- mbarrier
// Barriers and flags are addressed by 32-bit shared-window addresses
// (smem_u32), which keeps them out of 64-bit generic registers.
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

// Non-blocking probe of a phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// CTA-wide abort flag in shared memory (0 = keep going); address 0 = none.
__device__ __forceinline__ uint32_t flag_get(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.volatile.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ void flag_set(uint32_t addr, uint32_t v) {
  asm volatile("st.volatile.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

// Waits until the phase with the given parity has completed.  Returns false
// (after recording `status_bit` in *status and raising the abort flag) when
// `budget_ns` of wall-clock time passes first, or as soon as another warp
// has raised the abort flag.
//
// The probe is the non-suspending test_wait: a suspended warp is woken
// noticeably later than a spinning one sees the phase flip, and every waiter
// here sits on the critical path of the pipeline.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, uint64_t budget_ns, uint32_t* status,
                                          uint32_t status_bit, uint32_t abort_addr) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_test(bar, parity)) return true;
    if ((++spins & 3u) == 0) {
      if (abort_addr != 0 && flag_get(abort_addr) != 0) return false;
      if (global_timer_ns() - start > budget_ns) {
        if (status != nullptr) atomicOr(status, status_bit);
        if (abort_addr != 0) flag_set(abort_addr, 1u);
        return false;
      }
    }
  }
}

// Suspending probe: the thread may sleep in hardware until the phase
// completes or about `hint_ns` pass, instead of spinning.
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// mbar_wait for waits that are long by design (a tile waiting for the tensor
// pipe while the other tile computes): the waiting warp sleeps in try_wait
// instead of spinning, so it does not take issue slots from the warps that
// share its SMSP.  Bounded in the same way.
__device__ __forceinline__ bool mbar_wait_sleep(uint32_t bar, uint32_t parity, uint64_t budget_ns, uint32_t* status,
                                                uint32_t status_bit, uint32_t abort_addr) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    if (mbar_try(bar, parity, 1000u)) return true;
    if (abort_addr != 0 && flag_get(abort_addr) != 0) return false;
    if (global_timer_ns() - start > budget_ns) {
      if (status != nullptr) atomicOr(status, status_bit);
      if (abort_addr != 0) flag_set(abort_addr, 1u);
      return false;
    }
  }
}

__device__ __forceinline__ bool mbar_wait_sleep_warp(uint32_t bar, uint32_t parity, uint64_t budget_ns,
                                                     uint32_t* status, uint32_t status_bit, uint32_t abort_addr) {
  const bool ok = mbar_wait_sleep(bar, parity, budget_ns, status, status_bit, abort_addr);
  return __all_sync(0xffffffffu, ok) != 0;
}

// Warp-uniform variant for code that synchronises the warp afterwards: every
// lane waits (each bounded), then the warp agrees on success, so no lane can
// leave a loop that its siblings stay in.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, uint64_t budget_ns, uint32_t* status,
                                               uint32_t status_bit, uint32_t abort_addr) {
  const bool ok = mbar_wait(bar, parity, budget_ns, status, status_bit, abort_addr);
  return __all_sync(0xffffffffu, ok) != 0;
}

// ---------------------------------------------------------------- proxies
__device__ __forceinline__ void fence_proxy_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 3-D tiled load into this CTA's shared memory; completion is signalled on
// `bar` as transaction bytes.  The innermost coordinate c0 must be a multiple
// of 16 bytes (all callers pass 0 or multiples of 64 bytes).
__device__ __forceinline__ void tma_load_3d(uint32_t smem_dst, const CUtensorMap* map, uint32_t bar, int c0, int c1,
                                            int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

// 1-D bulk copy global -> shared (16-byte aligned addresses, size % 16 == 0).
__device__ __forceinline__ void bulk_load(uint32_t smem_dst, const void* gmem_src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_dst),
      "l"(reinterpret_cast<uint64_t>(gmem_src)), "r"(bytes), "r"(bar)
      : "memory");
}

// ---------------------------------------------------------------- TMEM
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(smem_result)),
               "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// ---------------------------------------------------------------- UMMA descriptors
// Shared-memory matrix descriptor for a K-major operand stored in the
// canonical swizzled layout that TMA writes (rows of `row_bytes` = 64 or 128
// bytes, 8-row groups `8*row_bytes` apart).  Fields: start address >> 4
// (bits 0-13), leading byte offset >> 4 (16-29; 1 for swizzled K-major),
// stride byte offset >> 4 (32-45), version 1 (46-47), swizzle mode (61-63:
// 2 = 128B, 4 = 64B).
__device__ __forceinline__ uint64_t umma_desc_kmajor(uint32_t smem_addr, uint32_t row_bytes) {
  const uint64_t sbo = (8u * row_bytes) >> 4;
  const uint64_t layout = row_bytes == 128 ? 2ull : 4ull;
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= 1ull << 16;
  d |= (sbo & 0x3FFFull) << 32;
  d |= 1ull << 46;
  d |= layout << 61;
  return d;
}

// Instruction descriptor for tcgen05.mma kind::i8: S32 accumulator (bits 4-5
// = 2), A/B signedness (bits 7-9 / 10-12: 0 = u8, 1 = s8), both K-major,
// N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_i8(bool a_signed, bool b_signed, int m, int n) {
  return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
         (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for tcgen05.mma kind::f8f6f4 with e4m3 A and B
// (format 0 in bits 7-9 / 10-12), an F32 accumulator (bits 4-5 = 1), both
// K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
__host__ __device__ constexpr uint32_t umma_idesc_e4m3(int m, int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor for tcgen05.mma kind::f16 with F16 A and B (format
// 0 in bits 7-9 / 10-12), an F32 accumulator (bits 4-5 = 1), both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
  return (1u << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// kind::f16 MMA whose A operand (M x 16 fp16, two per 32-bit column, row m
// in lane m) is read from TMEM at `a_tmem` instead of shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// ---------------------------------------------------------------- TMEM <-> registers
// 32x32b shape: warp w of a warpgroup reads TMEM lanes 32w..32w+31, thread
// lane i gets lane 32w+i; .xN reads N consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// Same as tmem_ld32, issued as four .x8 loads: the destination of one load
// must be a contiguous register block, and eight is far easier to place than
// thirty-two when most registers already hold live state.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld32_split(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld8(taddr, r);
  tmem_ld8(taddr + 8, r + 8);
  tmem_ld8(taddr + 16, r + 16);
  tmem_ld8(taddr + 24, r + 24);
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Writes 8 values into 8 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t* v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(v[0]),
               "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
               : "memory");
}

// Writes the same 32-bit value into 4 consecutive columns of this thread's lane.
__device__ __forceinline__ void tmem_st4_same(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%1,%1,%1};" ::"r"(taddr), "r"(v) : "memory");
}

// 16-byte shared load the compiler keeps in program order relative to the
// other volatile asm (it will not hoist a whole block of them ahead of the
// TMEM waits, which would pin 64 extra registers).
__device__ __forceinline__ float4 lds128(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// ---------------------------------------------------------------- math
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace piper
