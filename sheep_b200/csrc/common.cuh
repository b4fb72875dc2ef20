// Shared device helpers for the sm_100a decode engine.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#define SB_DEV __device__ __forceinline__

namespace sb {

constexpr int kGroup = 32;      // weights per group (one step/min field)
constexpr int kGps = 8;         // groups per 256-weight superblock
constexpr int kUnit = 64;       // weights one lane handles per step: 4 groups x 16 columns

SB_DEV float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
SB_DEV double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
SB_DEV int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
SB_DEV float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Weights are read once per token: stream them past L1 and mark them first to
// leave L2, so the KV cache and activations stay resident.
SB_DEV uint4 ld_stream(const void * p) {
    uint4 v;
    asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}
SB_DEV uint32_t ld_u32(const void * p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }
SB_DEV uint16_t ld_u16(const void * p) { return __ldg(reinterpret_cast<const unsigned short *>(p)); }
SB_DEV uint8_t ld_u8(const void * p) { return __ldg(reinterpret_cast<const unsigned char *>(p)); }

SB_DEV float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
SB_DEV uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Programmatic dependent launch (PTX griddepcontrol, sm_90+). The next kernel
// in the stream may start once every CTA here has signalled; it must call
// pdl_wait() before reading anything this kernel writes.
SB_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
SB_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Bulk prefetch of a byte range into L2 (cp.async.bulk.prefetch, sm_90+). The
// range is widened to 16-byte boundaries; callers allocate with slack so the
// widening stays inside the buffer.
SB_DEV void prefetch_l2(const void * p, size_t n) {
    if (!n) return;
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    uintptr_t lo = a & ~uintptr_t(15), hi = (a + n + 15) & ~uintptr_t(15);
    while (lo < hi) {
        const uint32_t chunk = (hi - lo) > (1u << 20) ? (1u << 20) : uint32_t(hi - lo);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" :: "l"(lo), "r"(chunk) : "memory");
        lo += chunk;
    }
}

// ---------------------------------------------------------------- async copies
// mbarrier + cp.async.bulk (sm_90+), one-dimensional bulk copies global ->
// shared with transaction-count completion. Every wait is bounded in time:
// after kWaitNs of the global timer it records an error and returns false, so
// a kernel can never spin forever on a copy that does not arrive.
//
// try_wait.parity(P) reports the phase with parity P complete whenever the
// barrier's current phase parity differs from P, so a waiter must never be
// more than one phase ahead of a barrier: each stage of a ring is consumed by
// one fixed warp, in order.

constexpr unsigned long long kWaitNs = 2000000000ull;   // 2 s

SB_DEV unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

SB_DEV uint32_t smem_u32(const void * p) { return (uint32_t) __cvta_generic_to_shared(p); }

SB_DEV void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
SB_DEV void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }

SB_DEV void mbar_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
SB_DEV void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
SB_DEV bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}
SB_DEV bool mbar_wait(uint64_t * bar, uint32_t parity, int * err, int code) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = global_ns();
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (global_ns() - t0 > kWaitNs) break;
    }
    if (err) atomicExch(err, code);
    return false;
}

// Bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned) into
// this CTA's shared memory, completing on `bar`.
SB_DEV void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Named barrier over the first `n` threads (a subset of the block).
SB_DEV void bar_sync(int id, int n) { asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory"); }

// Timestamps of the trace build (-DSB_TRACE): thread 0 of each CTA writes
// trace[(launch * kTraceCtas + blockIdx) * 8 + slot]: slot 0 the global timer
// at entry, later slots that time plus the SM cycles since, at the nominal
// 1965 MHz (finer than the global timer's steps).
constexpr int kTraceCtas = 160;
#ifdef SB_TRACE
SB_DEV unsigned long long & trace_ns0() { __shared__ unsigned long long v; return v; }
SB_DEV long long & trace_clk0() { __shared__ long long v; return v; }
SB_DEV unsigned long long trace_now(int slot) {
    if (slot == 0) {
        trace_clk0() = clock64();
        trace_ns0() = global_ns();
        return trace_ns0();
    }
    return trace_ns0() + (unsigned long long) ((clock64() - trace_clk0()) * 1000 / 1965);
}
#define SB_MARK(tr, launch, slot)                                                              \
    do {                                                                                       \
        if ((tr) && threadIdx.x == 0 && blockIdx.y == 0 && blockIdx.x < kTraceCtas)            \
            (tr)[((size_t) (launch) * kTraceCtas + blockIdx.x) * 8 + (slot)] = trace_now(slot); \
    } while (0)
#else
#define SB_MARK(tr, launch, slot) do { } while (0)
#endif

// Bounds checks of the checked build (-DSB_CHECKED): a failed check records
// its site in *err and the access is skipped. Compiled out otherwise.
#ifdef SB_CHECKED
#define SB_CHECK(err, cond, code) ((cond) ? true : (((err) ? atomicCAS((err), 0, (code)) : 0), false))
#else
#define SB_CHECK(err, cond, code) true
#endif

// Spread the low 4 bits of n into the low bit of each byte (bit i -> byte i).
SB_DEV uint32_t nib_to_bytes(uint32_t n) { return (n * 0x00204081u) & 0x01010101u; }

}  // namespace sb
