// The int8 tensor-core tile product on tcgen05: C[M][N] (int32) =
// A[M][K] * B[N][K]^T, A and B signed 8-bit, row-major (K contiguous).
//
// One CTA per 128 rows of A; K is staged through shared memory 256 bytes at a
// time in the canonical core-matrix layout (tc.cuh), one thread issues the
// eight K = 32 MMAs of a stage into the TMEM accumulator and commits them to an
// mbarrier, and four warps read the accumulator back (warp w: rows 32 w ..
// 32 w + 31). This is the integer core of the batched path (the reference's
// sml_g_tcm9, sml/sml-gpu-fast.cu:3149, on mma.sync); the sum per 256 columns
// is the unit its per-superblock epilogue scales.
#include "tc.cuh"
#include "sheep_b200.h"

#include <cstdio>

using namespace sb;

namespace {

constexpr int kTcM = 128;      // rows per CTA (the MMA's M)
constexpr int kTcKC = 256;     // K bytes staged per pass
char g_err[256];

template <int N>
__global__ void __launch_bounds__(128) k_tc_imma(const int8_t * A, const int8_t * B, int32_t * C, int K, int * err) {
    extern __shared__ __align__(1024) uint8_t sm[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t tslot;
    uint8_t * As = sm;                        // kTcM x kTcKC
    uint8_t * Bs = sm + kTcM * kTcKC;         // N x kTcKC
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m0 = blockIdx.x * kTcM;
    constexpr uint32_t ncols = tc_cols(N);
    if (warp == 0) tmem_alloc(&tslot, ncols);
    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    if (warp == 0) tmem_relinquish();
    bool ok = true;
    constexpr uint32_t idesc = tc_idesc_s8(kTcM, N);
    for (int kc = 0, ph = 0; kc < K; kc += kTcKC, ph++) {
        const int kb = K - kc < kTcKC ? K - kc : kTcKC;   // a multiple of 32
        const int nc = kb / 16;                            // 16-byte chunks per row
        for (int i = tid; i < kTcM * nc; i += 128) {
            const int row = i / nc, c = i - row * nc;
            *reinterpret_cast<uint4 *>(As + tc_off(kTcM, row, 16 * c)) =
                *reinterpret_cast<const uint4 *>(A + (size_t) (m0 + row) * K + kc + 16 * c);
        }
        for (int i = tid; i < N * nc; i += 128) {
            const int row = i / nc, c = i - row * nc;
            *reinterpret_cast<uint4 *>(Bs + tc_off(N, row, 16 * c)) =
                *reinterpret_cast<const uint4 *>(B + (size_t) row * K + kc + 16 * c);
        }
        fence_proxy_async_smem();   // the tensor core reads shared memory through the async proxy
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            for (int j = 0; j < kb / 32; j++) {
                const uint64_t ad = tc_desc(As + tc_off(kTcM, 0, 32 * j), (kTcM / 8) * 128, 128);
                const uint64_t bd = tc_desc(Bs + tc_off(N, 0, 32 * j), (N / 8) * 128, 128);
                tc_mma_s8(tmem, ad, bd, idesc, kc > 0 || j > 0);
            }
            tc_commit(&bar);
        }
        // the stage's MMAs finish before its shared memory is rewritten or D is read
        if (!mbar_wait(&bar, ph & 1, err, 30)) ok = false;
        tc_fence_after();
        __syncthreads();
    }
    const int row = 32 * warp + lane;
    for (int c = 0; c < N; c += 8) {
        uint32_t r[8];
        tmem_ld8(tmem + ((uint32_t) (32 * warp) << 16) + (uint32_t) c, r);
        tmem_wait_ld();
        if (ok) {
            int4 * dst = reinterpret_cast<int4 *>(C + (size_t) (m0 + row) * N + c);
            dst[0] = make_int4((int) r[0], (int) r[1], (int) r[2], (int) r[3]);
            dst[1] = make_int4((int) r[4], (int) r[5], (int) r[6], (int) r[7]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, ncols);
}

// Shared memory: the two tiles need (128 + N) x 256 bytes; 160 KB are
// allocated so that every descriptor read stays inside the allocation even
// for offsets read the other way round (then results, not memory, go wrong).
constexpr int kTcSmem = 160 * 1024;

template <int N>
cudaError_t launch_imma(const int8_t * A, const int8_t * B, int32_t * C, int M, int K, int * err, cudaStream_t st) {
    const int smem = kTcSmem;
    static_assert((kTcM + N) * kTcKC <= kTcSmem, "tiles exceed the shared memory");
    cudaError_t e = cudaFuncSetAttribute(k_tc_imma<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    k_tc_imma<N><<<M / kTcM, 128, smem, st>>>(A, B, C, K, err);
    return cudaGetLastError();
}

}  // namespace

extern "C" const char * sb_tc_last_error(void) { return g_err; }

extern "C" int sb_tc_imma(const int8_t * A, const int8_t * B, int32_t * C, int M, int N, int K, int * err,
                          void * stream) {
    g_err[0] = 0;
    if (!A || !B || !C || !err || M <= 0 || M % kTcM || K <= 0 || K % 32 ||
        (N != 16 && N != 32 && N != 64 && N != 128 && N != 256) ||
        (((uintptr_t) A | (uintptr_t) B | (uintptr_t) C) & 15)) {
        snprintf(g_err, sizeof g_err, "M a multiple of 128, N in 16/32/64/128/256, K of 32; 16-byte aligned buffers");
        return 0;
    }
    const cudaStream_t st = (cudaStream_t) stream;
    cudaError_t e = cudaErrorInvalidValue;
    switch (N) {
    case 16: e = launch_imma<16>(A, B, C, M, K, err, st); break;
    case 32: e = launch_imma<32>(A, B, C, M, K, err, st); break;
    case 64: e = launch_imma<64>(A, B, C, M, K, err, st); break;
    case 128: e = launch_imma<128>(A, B, C, M, K, err, st); break;
    default: e = launch_imma<256>(A, B, C, M, K, err, st); break;
    }
    if (e != cudaSuccess) {
        snprintf(g_err, sizeof g_err, "k_tc_imma: %s", cudaGetErrorString(e));
        return 0;
    }
    return 1;
}
