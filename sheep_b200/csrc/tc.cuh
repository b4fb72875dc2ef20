// 5th-generation tensor core (tcgen05) building blocks for sm_100a: shared-
// memory operand descriptors, the instruction descriptor of the int8 MMA, the
// tensor-memory (TMEM) accumulator's allocation and loads.
//
// Operands sit in shared memory in the canonical K-major layout without
// swizzle: "core matrices" of 8 rows x 16 bytes (128 contiguous bytes, row r
// at 16 r). One MMA of kind::i8 consumes K = 32 bytes of every row, i.e. two
// core matrices side by side in K; the descriptor's leading byte offset is the
// distance between those two, its stride byte offset the distance between
// successive groups of 8 rows. Here a tile of R rows x KB bytes keeps, for each
// 16-byte column chunk c, its R/8 core matrices contiguous:
//
//   byte (row, k) at  ((k / 16) * (R / 8) + row / 8) * 128 + (row % 8) * 16 + k % 16
//
// so LBO = R/8 * 128 and SBO = 128, and the MMA for K bytes [32 j, 32 j + 32)
// starts at chunk 2 j. The accumulator D (M = 128 rows) lives in TMEM: row i in
// lane i, column n in column base + n, one 32-bit word each; warp w of the CTA
// may read lanes 32 (w % 4) .. 32 (w % 4) + 31 (address: lane << 16 | column).
#pragma once

#include "common.cuh"

namespace sb {

// Byte offset of (row, k) in a tile of `rows` rows laid out as above.
__host__ __device__ inline uint32_t tc_off(int rows, int row, int k) {
    return (uint32_t) (((k >> 4) * (rows >> 3) + (row >> 3)) * 128 + (row & 7) * 16 + (k & 15));
}

// Shared-memory matrix descriptor (K-major, no swizzle, sm100 version 1).
SB_DEV uint64_t tc_desc(const void * smem_ptr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    const uint32_t a = smem_u32(smem_ptr);
    return (uint64_t) ((a & 0x3FFFFu) >> 4) | ((uint64_t) ((lbo_bytes >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo_bytes >> 4) & 0x3FFFu) << 32) | (1ull << 46);
}

// Instruction descriptor of tcgen05.mma kind::i8: signed 8-bit A and B, both
// K-major, 32-bit signed accumulate, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_s8(int M, int N) {
    return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t) (N >> 3) << 17) | ((uint32_t) (M >> 4) << 24);
}

// TMEM columns to allocate for n 32-bit accumulator columns (a power of two, >= 32).
__host__ __device__ constexpr uint32_t tc_cols(int n) {
    return n <= 32 ? 32u : n <= 64 ? 64u : n <= 128 ? 128u : n <= 256 ? 256u : 512u;
}

// Warp-collective allocation; the TMEM address lands in *dst (shared memory).
SB_DEV void tmem_alloc(uint32_t * dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst)), "r"(ncols) : "memory");
}
SB_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
SB_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols) : "memory");
}

// Ordering of tcgen05 operations around thread synchronization, and of
// generic-proxy shared-memory writes before the tensor core reads them.
SB_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
SB_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
SB_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// D (TMEM) = A * B^T (+ D when accumulate), one thread issues.
SB_DEV void tc_mma_s8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
    const uint32_t z = 0;
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t) accumulate),
                    "r"(z), "r"(z), "r"(z), "r"(z)
                 : "memory");
}

// D (TMEM, fp32) = A * B^T (+ D), fp16 operands (kind::f16), one thread issues.
SB_DEV void tc_mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool accumulate) {
    const uint32_t z = 0;
    asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}"
                 :: "r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"((uint32_t) accumulate),
                    "r"(z), "r"(z), "r"(z), "r"(z)
                 : "memory");
}

// Arrive once on *bar when every MMA this thread issued before has completed.
SB_DEV void tc_commit(uint64_t * bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
}

// 8 consecutive 32-bit columns of this thread's TMEM lane.
SB_DEV void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}
SB_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Thread-block clusters: a barrier over every thread of the cluster (release /
// acquire: shared-memory stores before it are visible after it), and stores
// into another CTA's shared memory by its rank in the cluster.
SB_DEV void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
SB_DEV uint32_t cluster_map(const void * smem_ptr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(smem_ptr)), "r"(rank));
    return r;
}
SB_DEV void st_cluster(uint32_t addr, float v) {
    asm volatile("st.shared::cluster.f32 [%0], %1;" :: "r"(addr), "f"(v) : "memory");
}
SB_DEV void st_cluster4(uint32_t addr, float a, float b, float c, float d) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" :: "r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
                 : "memory");
}

}  // namespace sb
