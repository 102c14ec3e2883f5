// Device helpers shared by the attention kernels (sm_100a).
//
// Everything that waits on the device waits with a time limit: a wait that
// gives up sets a bit in the device error word and the kernel returns, so a
// lost wake-up never hangs the GPU.  The host reads and clears the word with
// llmi_cuda_poll_error().
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace llmi {

// Bits of the device error word.
enum : unsigned {
  kErrWaitTimeout = 1u,      // an mbarrier wait ran out of time
  kErrTmemAlloc = 2u,        // tensor-memory allocation did not complete
  kErrBadLaunch = 4u,        // a kernel saw a launch shape it cannot serve
};

// The device error word (one per device and loaded module).
__device__ unsigned g_error_word;

// 2 s: far above any legitimate wait in these kernels (whole launches take
// microseconds to milliseconds), far below a watchdog.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void raise_error(unsigned bits) { atomicOr(&g_error_word, bits); }

// Programmatic dependent launch (griddepcontrol).  A kernel launched with
// programmatic stream serialization may become resident once every CTA of the
// kernel before it has called launch_dependents() (or exited); wait_primary()
// then blocks until that kernel has completed and its memory is visible.
// Decode-path kernels call both at entry, before any global access (L2
// prefetches aside) or early return: the next launch's set-up and CTA ramp
// overlap this one's tail, and
// since every kernel waits for its predecessor before finishing, the chain
// stays ordered.  Without the launch attribute both are no-ops.
// The one exception is a call flagged `settled` by its caller (the session
// between synchronised or separately launched steps): the operands it only
// carries over from earlier steps (cache rows before the newest, the
// recurrent state) are then known complete, and the kernel reads them before
// its wait, while the kernel ahead still runs.
__device__ __forceinline__ void launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void wait_primary() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_enter() {
  launch_dependents();
  wait_primary();
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// Makes initialised barriers visible to the async proxy (TMA) and the CTA.
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Non-suspending test of a phase: cheaper than try_wait when the phase has
// already completed, which matters in a thread that issues tensor-core MMAs
// (a suspending wait there leaves the MMA queue to run dry).
__device__ __forceinline__ bool mbar_test_wait(uint64_t *bar, unsigned parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// The waits below test the phase inline (one instruction when it has
// completed) and keep the spin-and-timeout loop out of line: the kernels
// wait at dozens of places, and inlining every loop bloats their code past
// what the instruction cache holds.

// Waits for the phase with the given parity to complete.  Returns false (and
// raises kErrWaitTimeout) if it has not completed within kWaitLimitNs.
__device__ __noinline__ bool mbar_wait_slow(uint64_t *bar, unsigned parity) {
  const uint64_t start = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity))
        return true;
    if (global_timer_ns() - start > kWaitLimitNs) {
      raise_error(kErrWaitTimeout);
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, unsigned parity) {
  return mbar_test_wait(bar, parity) || mbar_wait_slow(bar, parity);
}

// Bounded wait for kernels whose roles depend on one another: it also gives
// up as soon as another role has set the CTA's abort flag, and a wait that
// times out sets that flag, so every role leaves its loop.
__device__ __noinline__ bool wait_or_abort_slow(uint64_t *bar, unsigned parity,
                                                volatile uint32_t *abort) {
  const uint64_t start = global_timer_ns();
  while (true) {
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(bar, parity))
        return true;
    if (*abort)
      return false;
    if (global_timer_ns() - start > kWaitLimitNs) {
      raise_error(kErrWaitTimeout);
      *abort = 1u;
      return false;
    }
  }
}
__device__ __forceinline__ bool wait_or_abort(uint64_t *bar, unsigned parity,
                                              volatile uint32_t *abort) {
  return mbar_test_wait(bar, parity) || wait_or_abort_slow(bar, parity, abort);
}

// ---- cp.async -----------------------------------------------------------------

// cp.async of 16 (or 4) bytes global -> shared; `bytes_valid` 0 writes zeros
// without reading.
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t bytes_valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(bytes_valid)
               : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src, uint32_t bytes_valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(bytes_valid)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// ---- bulk copies (TMA engine, no multicast) ----------------------------------

// 1-D bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1], %2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Bulk prefetch of [src, src + bytes) into L2: no destination, no barrier.
// src 16-byte aligned, bytes a multiple of 16.  A prefetch only warms L2 and
// never changes what a later load returns, so a kernel may issue it before
// wait_primary(), while the kernel ahead of it still runs.
__device__ __forceinline__ void prefetch_l2(const void *src, unsigned bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- streaming global access ---------------------------------------------------

__device__ __forceinline__ float4 ld_stream_f4(const float *p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void st_stream_f4(float *p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z),
               "f"(v.w)
               : "memory");
}

// ---- warp-level tensor-core fragments (m16n8k16, f16 in, f32 accumulate) ------

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// Transposes an 8x8 b16 matrix held in the standard fragment layout (thread t
// holds row t/4, columns 2*(t%4) and 2*(t%4)+1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 arithmetic of sm_100 (two lanes per instruction, each lane
// rounded as the scalar operation would be) and the three-input maximum.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// log2(x) for x > 0, subnormal inputs included (MUFU approximation).
__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace llmi
