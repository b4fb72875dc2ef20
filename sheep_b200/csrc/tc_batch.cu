// The batched path on the tensor cores: y[t] = W x[t] for T >= 16 rows of x,
// with the reference's batched arithmetic (sml_g_requant8 and the int8 tiles,
// sml/sml-gpu-fast.cu:1804-1880, 2025-2031): the weights re-quantized to int8
// with one fp32 scale per row per 256 (the group scale and min folded in), x
// quantized per 256, the int32 dot of a superblock from tcgen05.mma, and one
// float epilogue per superblock, acc = fma(s8 * xs, dot, acc), superblocks in
// order -- so results equal the CPU restatement bit for bit.
//
//   k_requant8   one warp per (row, superblock): the bound of its groups, s8,
//                and the 256 int8 weights, written as the GEMM's A operand:
//                a 32 KB block per (128 rows, superblock) in the core-matrix
//                layout of tc.cuh. Done once per tensor, kept on the device
//                (the reference re-makes it per call).
//   k_quant_rows one CTA per token (row of x), one warp per superblock: the
//                row gathered through the tensor's column order (optionally
//                RMS-normalized, or SiLU(gate) * up), the B operand, a block of
//                N x 256 bytes per (N tokens, superblock), and the scale.
//   k_tcgemm<N>  one CTA per (128 rows, N tokens, slice of the superblocks),
//                ten warps: a producer (bulk copies of both blocks of a
//                superblock into a 4-stage ring), an MMA issuer (8 MMAs of
//                K = 32 per superblock into one of four TMEM accumulators, then
//                commits), and eight epilogue warps, two per quarter of the TMEM
//                lanes (rows), each taking half the tokens, that apply the
//                superblock's scales while the next superblock multiplies. The slices of a tile run as one thread-block
//                cluster and meet in the leader CTA's shared memory, where
//                they are added in slice order (split-K). The epilogue may add
//                a bias or accumulate into y (a residual).
#include "tc.cuh"
#include "decode.cuh"
#include "sheep_b200.h"
#include "tc_batch.h"

#include <cstdio>

namespace sb {

constexpr int kTcStages = 4;
constexpr int kTcAcc = 4;        // TMEM accumulators: the MMAs run up to 3 superblocks ahead of the epilogue
constexpr int kTcEpiWarps = 8;   // two per quarter of the TMEM lanes, each half of the tokens
constexpr int kTcThreads = (2 + kTcEpiWarps) * 32;


#ifdef SB_TRACE
// Trace build: global-timer marks of the last tensor-core product, per CTA
// (blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z) < kTcTraceCtas).
constexpr int kTcTraceCtas = 1024;
__device__ unsigned long long g_tc_trace[kTcTraceCtas * 8];
#define TC_MARK(slot)                                                                                   \
    do {                                                                                                \
        const unsigned cta_ = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);          \
        if (cta_ < (unsigned) kTcTraceCtas) g_tc_trace[cta_ * 8 + (slot)] = global_ns();              \
    } while (0)
#else
#define TC_MARK(slot) do { } while (0)
#endif
constexpr uint32_t kTcABytes = 128 * 256;

template <int NB, int SIX>
__global__ void __launch_bounds__(256) k_requant8(const __grid_constant__ QT t, uint8_t * wblk, float * s8,
                                                  int rows_pad, int nsb, int row_off, int rows_here) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const long item = (long) blockIdx.x * 8 + warp;
    if (item >= (long) rows_here * nsb) return;
    const int r = (int) (item / nsb), sb = (int) (item % nsb);   // r: row of t; row_off + r: row of the plan
    const int ng = t.cols / kGroup, g = sb * 8 + (lane >> 2), part = lane & 3;
    const bool live = r < t.rows && g < ng;
    const float cmax = (float) ((1 << NB) - 1);
    float s = 0.0f, m = 0.0f, bound = 0.0f;
    if (live) {
        s = __fmul_rn(h2f(t.sd[(size_t) r * t.nsb + sb]), (float) field_at<SIX>(t.sq, t.frow, r, g));
        if (t.has_min)
            m = __fmul_rn(h2f(t.md[(size_t) r * t.nsb + sb]), __fsub_rn((float) field_at<SIX>(t.mq, t.frow, r, g), t.mbias));
        const float top = __fmaf_rn(s, cmax, m);
        bound = fmaxf(fabsf(m), fabsf(top));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) bound = fmaxf(bound, __shfl_xor_sync(0xffffffffu, bound, o));
    if (lane == 0) s8[(size_t) sb * rows_pad + row_off + r] = __fdiv_rn(bound, 127.0f);
    const float inv = bound > 0.0f ? __fdiv_rn(127.0f, bound) : 0.0f;
    const float ka = __fmul_rn(s, inv), kb = __fmul_rn(m, inv);
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int j = 0; j < 8; j++) {
        const int i = g * kGroup + part * 8 + j;
        const int q = live ? __float2int_rn(__fmaf_rn((float) code_at<NB>(t, r, i), ka, kb)) : 0;
        w[j >> 2] |= ((uint32_t) (q & 0xff)) << (8 * (j & 3));
    }
    const int k = (lane >> 2) * kGroup + part * 8;
    const int pr = row_off + r;
    *reinterpret_cast<uint2 *>(wblk + ((size_t) (pr >> 7) * nsb + sb) * kTcABytes + tc_off(128, pr & 127, k)) =
        make_uint2(w[0], w[1]);
}

// One CTA per (row of x, 8 superblocks), one warp per superblock: the row's
// values in the tensor's column order (plain; RMS-normalized with a gain, the
// norm's sum of squares over the whole row in double as the decode GEMVs take
// it; or SiLU(gate) * up from a row holding gate | up), quantized per 256 into
// the B operand blocks (N tokens per block) and the per-superblock scales.
// Rows past T are zeros.
template <int MODE>
__global__ void __launch_bounds__(256) k_quant_rows(const TcQuantArgs a) {
    __shared__ double red[8];
    const int tok = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool live = tok < a.T;
    const float * row = a.x + (size_t) tok * a.ldx;
    float s = 1.0f;
    if (MODE == TQ_NORM) {
        double q = 0.0;
        if (live)
            for (int i = threadIdx.x; i < a.cols; i += 256) q += (double) row[i] * (double) row[i];
        q = warp_sum_d(q);
        if (lane == 0) red[warp] = q;
        __syncthreads();
        double ss = 0.0;
        for (int k = 0; k < 8; k++) ss += red[k];
        s = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float) (ss / a.cols), a.eps)));
    }
    const int sb = blockIdx.y * 8 + warp;
    if (sb < a.nsb) {
        const int k0 = lane * 8;
        float v[8];
        float amax = 0.0f;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int i = sb * 256 + k0 + j;
            float x = 0.0f;
            if (live && i < a.cols) {
                const int p = a.perm[i];
                if (MODE == TQ_PLAIN) x = row[p];
                else if (MODE == TQ_NORM) x = __fmul_rn(__fmul_rn(row[p], s), a.gain[p]);
                else x = silu_mul(row[p], row[a.up_off + p]);
            }
            v[j] = x;
            amax = fmaxf(amax, fabsf(x));
        }
        amax = warp_max(amax);
        const float sc = __fdiv_rn(amax, 127.0f);
        const float is = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
        uint32_t w[2] = {0u, 0u};
#pragma unroll
        for (int j = 0; j < 8; j++) {
            int q = __float2int_rn(__fmul_rn(v[j], is));
            q = q > 127 ? 127 : q < -127 ? -127 : q;
            w[j >> 2] |= ((uint32_t) (q & 0xff)) << (8 * (j & 3));
        }
        *reinterpret_cast<uint2 *>(a.xblk + ((size_t) (tok / a.N) * a.nsb + sb) * (size_t) (a.N * 256) +
                                   tc_off(a.N, tok % a.N, k0)) = make_uint2(w[0], w[1]);
        if (lane == 0) a.xs[(size_t) sb * a.T_pad + tok] = sc;
    }
}

// A wait that gives up at once when another role of the CTA already has.
SB_DEV bool tc_wait(uint64_t * bar, uint32_t parity, int * err, int code, volatile int * fail) {
    if (*fail) return false;
    if (mbar_wait(bar, parity, err, code)) return true;
    *fail = 1;
    return false;
}

template <int N>
__global__ void __launch_bounds__(kTcThreads, 1) k_tcgemm(const __grid_constant__ TcArgs g) {
    extern __shared__ __align__(1024) uint8_t tsm[];
    __shared__ __align__(8) uint64_t full[kTcStages], empty[kTcStages], accf[kTcAcc], acce[kTcAcc];
    __shared__ uint32_t tslot;
    __shared__ volatile int fail;
    // a stage: A block | B block | the rows' s8 (128 floats) | the tokens' xs (N floats)
    constexpr uint32_t BB = N * 256, SB = kTcABytes + BB + 512 + N * 4;
    static_assert((size_t) kTcStages * SB >= (size_t) (kTcMaxSplit - 1) * 128 * N * 4,
                  "a cluster's partial tiles must fit in the leader's ring");
    constexpr uint32_t ncols = tc_cols(kTcAcc * N);
    constexpr uint32_t idesc = tc_idesc_s8(128, N);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mb = blockIdx.x, tb = blockIdx.y, z = blockIdx.z;
    // this CTA's superblocks: slice z of the deep sum
    const int per = (g.nsb + g.split - 1) / g.split;
    const int s0 = z * per, ns = min(g.nsb, s0 + per) - s0;
    if (warp == 1) tmem_alloc(&tslot, ncols);
    if (tid == 0) {
        // a stage is free once its MMAs are done (commit) and the epilogue warps read its scales
        for (int s = 0; s < kTcStages; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], kTcEpiWarps + 1); }
        for (int b = 0; b < kTcAcc; b++) { mbar_init(&accf[b], 1); mbar_init(&acce[b], kTcEpiWarps); }
        fail = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    if (warp == 1) tmem_relinquish();
    if (tid == 0) TC_MARK(0);
    // epilogue warps: TMEM lane = row (a warp may read lanes 32 (warp % 4) ..),
    // tokens c0 .. c0 + H - 1
    constexpr int H = N / 2;
    const int q = warp & 3, row = 32 * q + lane, r = mb * 128 + row, c0 = warp >= 6 ? H : 0;
    float acc[H];
    bool ok = true;

    if (warp == 0) {
        // ---------------- producer: both operand blocks of every superblock
        if (lane == 0) {
            for (int i = 0; i < ns; i++) {
                const int s = i % kTcStages, lap = i / kTcStages, sb = s0 + i;
                if (lap > 0 && !tc_wait(&empty[s], (lap - 1) & 1, g.err, 40, &fail)) break;
                mbar_expect_tx(&full[s], SB);
                bulk_g2s(tsm + (size_t) s * SB, g.wblk + ((size_t) mb * g.nsb + sb) * kTcABytes, kTcABytes, &full[s]);
                bulk_g2s(tsm + (size_t) s * SB + kTcABytes, g.xblk + ((size_t) tb * g.nsb + sb) * BB, BB, &full[s]);
                bulk_g2s(tsm + (size_t) s * SB + kTcABytes + BB, g.s8 + (size_t) sb * g.rows_pad + mb * 128, 512,
                         &full[s]);
                bulk_g2s(tsm + (size_t) s * SB + kTcABytes + BB + 512, g.xs + (size_t) sb * g.T_pad + tb * N, N * 4,
                         &full[s]);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer: 8 x K=32 per superblock into accumulator sb % 2
        if (lane == 0) {
            for (int i = 0; i < ns; i++) {
                const int s = i % kTcStages, buf = i % kTcAcc;
                if (!tc_wait(&full[s], (i / kTcStages) & 1, g.err, 41, &fail)) break;
                if (i >= kTcAcc && !tc_wait(&acce[buf], (i / kTcAcc - 1) & 1, g.err, 42, &fail)) break;
                tc_fence_after();
                const uint8_t * As = tsm + (size_t) s * SB, * Bs = As + kTcABytes;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    tc_mma_s8(tmem + (uint32_t) (buf * N), tc_desc(As + tc_off(128, 0, 32 * j), 16 * 128, 128),
                              tc_desc(Bs + tc_off(N, 0, 32 * j), (N / 8) * 128, 128), idesc, j > 0);
                tc_commit(&empty[s]);     // the stage may be refilled once these MMAs are done
                tc_commit(&accf[buf]);    // and the accumulator read
            }
        }
    } else {
        // ---------------- epilogue: TMEM lanes (rows) 32 q .. 32 q + 31, tokens c0 ..
        for (int t = 0; t < H; t++) acc[t] = 0.0f;
        for (int i = 0; i < ns; i++) {
            const int buf = i % kTcAcc, s = i % kTcStages;
            // the stage's scales: landed with its operands, and the stage is held
            // (empty needs this warp's arrival) until they are read
            ok = ok && tc_wait(&full[s], (i / kTcStages) & 1, g.err, 44, &fail);
            const float * ssc = reinterpret_cast<const float *>(tsm + (size_t) s * SB + kTcABytes + BB);
            const float s8v = ssc[row];
            float xsv[H];
#pragma unroll
            for (int t = 0; t < H; t += 4) {
                const float4 v4 = *reinterpret_cast<const float4 *>(ssc + 128 + c0 + t);
                xsv[t] = v4.x; xsv[t + 1] = v4.y; xsv[t + 2] = v4.z; xsv[t + 3] = v4.w;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            ok = ok && tc_wait(&accf[buf], (i / kTcAcc) & 1, g.err, 43, &fail);
            if (i == 0 && tid == 64) TC_MARK(1);
            tc_fence_after();
            uint32_t d[H];
#pragma unroll
            for (int c = 0; c < H; c += 8) {
                uint32_t r8[8];
                tmem_ld8(tmem + ((uint32_t) (32 * q) << 16) + (uint32_t) (buf * N + c0 + c), r8);
#pragma unroll
                for (int k = 0; k < 8; k++) d[c + k] = r8[k];
            }
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acce[buf]);
#pragma unroll
            for (int t = 0; t < H; t++) acc[t] = __fmaf_rn(__fmul_rn(s8v, xsv[t]), (float) (int) d[t], acc[t]);
        }
        if (tid == 64) TC_MARK(2);
    }
    if (g.split > 1) {
        // The slices of a tile are one cluster (rank = z). Once every CTA is past
        // its main loop (the leader's ring is idle), slices 1.. store their sums
        // into the leader's ring as [slice - 1][token / 4][row][4] (four tokens
        // per 16-byte store; a warp's 32 rows are 512 contiguous bytes); the
        // leader adds them in slice order, so the sum does not depend on arrival
        // order (sml_g_splitk_sum, sml/sml-gpu-fast.cu:2057-2065).
        cluster_sync();
        float * pbuf = reinterpret_cast<float *>(tsm);
        if (warp >= 2 && z > 0) {
            const uint32_t base = cluster_map(pbuf + (size_t) (z - 1) * N * 128 + row * 4, 0);
#pragma unroll
            for (int t = 0; t < H; t += 4)
                st_cluster4(base + (uint32_t) ((c0 + t) * 128 * 4), acc[t], acc[t + 1], acc[t + 2], acc[t + 3]);
        }
        cluster_sync();
        if (warp >= 2) {
            if (z == 0) {
                for (int k = 1; k < g.split; k++) {
                    const float * pk = pbuf + (size_t) (k - 1) * N * 128 + row * 4;
#pragma unroll
                    for (int t = 0; t < H; t += 4) {
                        const float4 v = *reinterpret_cast<const float4 *>(pk + (c0 + t) * 128);
                        acc[t] = __fadd_rn(acc[t], v.x);
                        acc[t + 1] = __fadd_rn(acc[t + 1], v.y);
                        acc[t + 2] = __fadd_rn(acc[t + 2], v.z);
                        acc[t + 3] = __fadd_rn(acc[t + 3], v.w);
                    }
                }
            } else {
                ok = false;   // only the leader writes the tile
            }
        }
    }
    if (warp >= 2) {
        if (tid == 64) TC_MARK(3);
        if (ok && r < g.rows) {
            const int nt = min(N, g.T - tb * N) - c0;
            float * yr = g.y + ((size_t) tb * N + c0) * g.ldy + r;
            if (g.accumulate) {
                // every token's old value read before any is written (they never alias)
                float old[H];
#pragma unroll
                for (int t = 0; t < H; t++) old[t] = t < nt ? yr[(size_t) t * g.ldy] : 0.0f;
#pragma unroll
                for (int t = 0; t < H; t++)
                    if (t < nt) yr[(size_t) t * g.ldy] = __fadd_rn(old[t], acc[t]);
            } else {
                const float b = g.bias ? g.bias[r] : 0.0f;
#pragma unroll
                for (int t = 0; t < H; t++)
                    if (t < nt) yr[(size_t) t * g.ldy] = g.bias ? __fadd_rn(acc[t], b) : acc[t];
            }
        }
    }
    if (tid == 64) TC_MARK(4);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, ncols);
    }
    if (tid == 0) TC_MARK(5);
}

template <int NB, int SIX>
static void launch_requant(const QT & t, uint8_t * wblk, float * s8, int rows_pad, int nsb, int row_off,
                           cudaStream_t st, cudaError_t * r) {
    const long items = (long) t.rows * nsb;
    k_requant8<NB, SIX><<<(unsigned) ((items + 7) / 8), 256, 0, st>>>(t, wblk, s8, rows_pad, nsb, row_off, t.rows);
    *r = cudaGetLastError();
}

cudaError_t tc_requant(const QT & t, const TcPlan & p, int row_off, cudaStream_t st) {
    cudaError_t r = cudaErrorInvalidValue;
    if (row_off + t.rows > p.rows_pad || (t.cols / kGroup + 7) / 8 != p.nsb) return r;
    SB_DISPATCH_QT(t.nbits, t.six, launch_requant, t, p.wblk, p.s8, p.rows_pad, p.nsb, row_off, st, &r);
    return r;
}

int tc_tile_n(int T) { return T <= 16 ? 16 : T <= 32 ? 32 : 64; }
int tc_tokens_pad(int T) { const int N = tc_tile_n(T); return (T + N - 1) / N * N; }

cudaError_t tc_quant(int mode, const TcQuantArgs & a, cudaStream_t st) {
    const dim3 grid(a.T_pad, (a.nsb + 7) / 8);
    if (mode == TQ_NORM) k_quant_rows<TQ_NORM><<<grid, 256, 0, st>>>(a);
    else if (mode == TQ_SILU) k_quant_rows<TQ_SILU><<<grid, 256, 0, st>>>(a);
    else k_quant_rows<TQ_PLAIN><<<grid, 256, 0, st>>>(a);
    return cudaGetLastError();
}

template <int N>
static cudaError_t launch_gemm(const TcArgs & a, cudaStream_t st) {
    constexpr int smem = kTcStages * (int) (kTcABytes + N * 256 + 512 + N * 4);
    static bool attr = false;
    if (!attr) {
        const cudaError_t e = cudaFuncSetAttribute(k_tcgemm<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.rows_pad / 128, a.T_pad / N, a.split);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = (unsigned) a.split;   // one tile's slices
    cfg.attrs = at;
    cfg.numAttrs = a.split > 1 ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_tcgemm<N>, a);
}

int tc_split(int nsb, int split) {
    if (split < 1) split = 1;
    if (split > nsb) split = nsb;
    const int per = (nsb + split - 1) / split;
    return (nsb + per - 1) / per;
}

cudaError_t tc_mma(const TcArgs & a, cudaStream_t st) {
    if (a.split < 1 || a.split > kTcMaxSplit || a.split != tc_split(a.nsb, a.split)) return cudaErrorInvalidValue;
    const int N = tc_tile_n(a.T);
    return N == 16 ? launch_gemm<16>(a, st) : N == 32 ? launch_gemm<32>(a, st) : launch_gemm<64>(a, st);
}

cudaError_t tc_gemm(const QT & t, const TcPlan & p, const float * x, int T, uint8_t * xblk, float * xs, float * y,
                    int * err, cudaStream_t st) {
    TcQuantArgs q;
    memset(&q, 0, sizeof q);
    q.x = x; q.ldx = t.cols; q.perm = t.perm; q.cols = t.cols; q.T = T; q.T_pad = tc_tokens_pad(T);
    q.N = tc_tile_n(T); q.nsb = p.nsb; q.xblk = xblk; q.xs = xs;
    cudaError_t e = tc_quant(TQ_PLAIN, q, st);
    if (e != cudaSuccess) return e;
    TcArgs a;
    memset(&a, 0, sizeof a);
    a.wblk = p.wblk; a.s8 = p.s8; a.xblk = xblk; a.xs = xs; a.y = y; a.ldy = t.rows;
    a.rows = t.rows; a.rows_pad = p.rows_pad; a.nsb = p.nsb; a.T = T; a.T_pad = q.T_pad; a.err = err;
    a.split = 1;
    return tc_mma(a, st);
}

}  // namespace sb

// The global-timer marks of the last tensor-core product (trace build only):
// per CTA [start, first accumulator read, main loop done, slices added,
// stored, exit, -, -]; returns the CTAs copied (0 without SB_TRACE).
extern "C" int sb_tc_trace(unsigned long long * out, int cap_ctas) {
#ifdef SB_TRACE
    const int n = cap_ctas < sb::kTcTraceCtas ? cap_ctas : sb::kTcTraceCtas;
    if (cudaMemcpyFromSymbol(out, sb::g_tc_trace, (size_t) n * 8 * 8) != cudaSuccess) return 0;
    return n;
#else
    (void) out; (void) cap_ctas;
    return 0;
#endif
}
