// Mixture-of-experts FFN on the tensor cores, for 16 or more rows per call.
//
// With many rows per call most chosen experts serve several rows, and the
// expert products become small dense contractions: rows of one expert (a
// chunk of up to 64, the dispatch the router already builds) times the
// expert's weights. The reference batches them the same way (sml_g_moe_*
// with gatherb / scatterb around its batched kernels, sml/sml-gpu-fast.cu:
// 3582-3612; moe_ffn_batch on the CPU, sml/sml-run.c:3182). Here each product
// is a tcgen05 MMA of kind::f16: the expert's Q4 tiles are decoded to fp16 in
// shared memory (code * (d * sq) + md * (mq - bias), the group's step and
// minimum rounded to fp16 once), the rows are fp16, and the sums are fp32 in
// tensor memory. This is not the decode arithmetic (int8 activations per 32,
// the reference's float order): results agree with it to about 1e-3 relative
// (fp16 operands, fp32 accumulation), and the one-row decode keeps its exact
// kernels.
//
//   k_moe_xg       per (chunk, 128 columns): the chunk's rows gathered through
//                  the expert's column order, fp16, as the MMA's B operand
//                  (Np x 128, Np = rows rounded up to 16, core-matrix layout).
//   k_moe_tc<GU>   per (chunk, 64 gate rows + the same 64 up rows): the MMA
//                  over the expert's columns; the epilogue forms
//                  SiLU(gate) * up and stores it, fp16, at down's column
//                  positions as the B operand of the down product.
//   k_moe_tc<DN>   per (chunk, 128 down rows): the MMA over the hidden width;
//                  fp32 rows per choice ([T*k][E]), summed by k_moe_comb.
//
// A k_moe_tc CTA: warps 0-3 copy (16-byte asynchronous copies) the 128 rows'
// group fields for the whole width once, then per 128 columns the rows' code
// bytes and the B block into a 3-stage ring two chunks ahead, and decode a
// stage's codes into its fp16 A block (one A row per thread); warp 4 issues
// the 8 MMAs of K = 16 per stage and commits; after the last, warps 0-3 read
// the accumulator (TMEM lane = row) for the epilogue. Every wait is bounded
// and reports an error code.
#include "moe_host.h"
#include "tc.cuh"

#include <cuda_fp16.h>

namespace sb {

constexpr int kXN = 64;                 // most rows of a chunk (the MMA's N)
constexpr int kXStages = 3;
constexpr int kXThreads = 160;
constexpr uint32_t kXABytes = 128 * 256;          // 128 rows x 128 fp16
constexpr uint32_t kXBBytes = kXN * 256;          // 64 rows x 128 fp16
constexpr uint32_t kXCodeBytes = 128 * 64;        // 128 rows x 128 four-bit codes

// Bytes of one chunk's B operand over K columns (a block of kXBBytes per 128).
__host__ __device__ inline size_t moe_xb_bytes(int K) { return (size_t) (K / 128) * kXBBytes; }

struct MoeTcArgs {
    TT t;                                // geometry of every expert's tiles (t.tiles unused)
    const uint8_t * const * tiles;       // [expert] tile base
    const int32_t * const * perm;        // [expert] GU: input gather
    const int32_t * const * scatter;     // [expert] GU: where hidden value f goes in down's order
    const float * in;                    // xg: input rows
    int in_stride, in_div;               // floats per input row; input row = slot / in_div
    const uint8_t * bop;                 // B operands: [chunk] blocks of moe_xb_bytes(K)
    uint8_t * hb;                        // GU: the down product's B operands (K = ffn_f)
    float * out;                         // DN: rows per choice
    int out_stride;
    int ffn_f;
    const int * slots, * ch_e, * ch_s0, * ch_n, * meta;
    int * err;
};

SB_DEV int round16(int n) { return (n + 15) & ~15; }

// ---------------------------------------------------------------- gather

// grid (K / 128, chunks), 128 threads: thread i fills 8 columns (i % 16) of
// rows i / 16, i / 16 + 8, ... of its chunk's B block; rows past the chunk's
// count (up to Np) are zeros.
__global__ void __launch_bounds__(128) k_moe_xg(const __grid_constant__ MoeTcArgs g, int K) {
    pdl_launch_dependents();
    pdl_wait();
    const int c = blockIdx.y, kc = blockIdx.x;
    if (c >= g.meta[0]) return;
    const int e = g.ch_e[c], ntok = g.ch_n[c], s0 = g.ch_s0[c], Np = round16(ntok);
    const int kg = threadIdx.x & 15, t0 = threadIdx.x >> 4;
    const int32_t * pm = g.perm[e] + kc * 128 + 8 * kg;
    int idx[8];
#pragma unroll
    for (int m = 0; m < 8; m++) idx[m] = pm[m];
    uint8_t * blk = const_cast<uint8_t *>(g.bop) + (size_t) c * moe_xb_bytes(K) + (size_t) kc * kXBBytes;
    for (int t = t0; t < Np; t += 8) {
        uint32_t h[4] = {0u, 0u, 0u, 0u};
        if (t < ntok) {
            const float * row = g.in + (size_t) (g.slots[s0 + t] / g.in_div) * g.in_stride;
#pragma unroll
            for (int m = 0; m < 8; m += 2) {
                const __half2 v = __floats2half2_rn(row[idx[m]], row[idx[m + 1]]);
                h[m >> 1] = *reinterpret_cast<const uint32_t *>(&v);
            }
        }
        *reinterpret_cast<uint4 *>(blk + tc_off(Np, t, 16 * kg)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// ---------------------------------------------------------------- the product

// Eight fp16 weights from eight code bytes (w0: bytes 0-3, w1: 4-7), their low
// (HI = false) or high nibbles: code * s + m, one rounding (fma), as a uint4 in
// column order.
template <bool HI>
SB_DEV uint4 dq8(uint32_t w0, uint32_t w1, __half2 s, __half2 m) {
    const __half2 k1024 = __float2half2_rn(1024.0f);
    uint32_t o[4];
    const uint32_t src[2] = {w0, w1};
#pragma unroll
    for (int q = 0; q < 4; q++) {
        // bytes (2q, 2q + 1) of the eight into the two 16-bit halves
        const uint32_t t = __byte_perm(src[q >> 1], 0u, (q & 1) ? 0x4342u : 0x4140u);
        const uint32_t n = ((HI ? (t >> 4) : t) & 0x000F000Fu) | 0x64006400u;   // 1024 + code, exactly
        __half2 h = *reinterpret_cast<const __half2 *>(&n);
        h = __hfma2(__hsub2(h, k1024), s, m);
        o[q] = *reinterpret_cast<const uint32_t *>(&h);
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

SB_DEV bool xt_wait(uint64_t * bar, uint32_t parity, int * err, int code, volatile int * fail) {
    if (*fail) return false;
    if (mbar_wait(bar, parity, err, code)) return true;
    *fail = 1;
    return false;
}

// 16-byte asynchronous copies global -> shared (bypassing L1), in commit groups.
SB_DEV void xa_cp16(void * dst, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}
SB_DEV void xa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SB_DEV void xa_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// MODE: MG_GU (gate / up interleaved tiles, TR/2 gate rows then TR/2 up rows)
// or MG_DN. Four-bit codes with 8-bit group fields. Warps 0-3 copy (16-byte
// asynchronous copies, two chunks ahead), decode and run the epilogue; warp 4
// owns the tensor memory and issues the MMAs.
template <int MODE>
__global__ void __launch_bounds__(kXThreads, 1) k_moe_tc(const __grid_constant__ MoeTcArgs g) {
    extern __shared__ __align__(1024) uint8_t xsm[];
    __shared__ __align__(8) uint64_t full_a[kXStages], empty[kXStages], done;
    __shared__ uint32_t tslot;
    __shared__ volatile int fail;
    __shared__ volatile int cfail[2];
    pdl_launch_dependents();
    const TT & t = g.t;
    const int K = t.cols, TR = t.TR, nkc = K / 128;
    const TileGeom tg = tile_geom(K, TR, 4, 0, t.has_min);
    const uint32_t f_sq = pad16((uint32_t) tg.P * TR * 4), f_sd = pad16((uint32_t) tg.S * TR * 2);
    const uint32_t fb = 2 * f_sq + 2 * f_sd;                  // one tile's fields in shared memory
    const int ntl = 128 / TR;                                 // tiles of the 128 rows
    const uint32_t stage_b = kXABytes + kXBBytes + kXCodeBytes;
    uint8_t * fields = xsm + (size_t) kXStages * stage_b;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int mb = blockIdx.x, c = blockIdx.y;
    if (warp == 4) tmem_alloc(&tslot, 64);
    if (tid == 0) {
        for (int s = 0; s < kXStages; s++) { mbar_init(&full_a[s], 4); mbar_init(&empty[s], 1); }
        mbar_init(&done, 1);
        fail = 0;
        cfail[0] = cfail[1] = 0;
        mbar_fence_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tslot;
    if (warp == 4) tmem_relinquish();
    pdl_wait();
    const int nch = g.meta[0];
    const bool live = c < nch;
    const int e = live ? g.ch_e[c] : 0, ntok = live ? g.ch_n[c] : 0, s0 = live ? g.ch_s0[c] : 0;
    const int Np = round16(ntok > 0 ? ntok : 1);
    // the tiles of this CTA's 128 rows: GU 64 gate rows (and their up rows)
    // from row 64 mb, DN 128 rows from 128 mb
    const int tile0 = MODE == MG_GU ? (64 * mb) / (TR / 2) : (128 * mb) / TR;
    const uint8_t * tiles = live ? g.tiles[e] + (size_t) tile0 * t.tb : nullptr;
    const uint8_t * bsrc = g.bop + (size_t) c * moe_xb_bytes(K);

    if (live && warp == 4) {
        // ---------------- MMA issuer
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | ((uint32_t) (Np >> 3) << 17) | ((uint32_t) (128 >> 4) << 24);
            for (int kc = 0; kc < nkc; kc++) {
                const int s = kc % kXStages;
                if (!xt_wait(&full_a[s], (kc / kXStages) & 1, g.err, 123, &fail)) break;
                tc_fence_after();
                const uint8_t * As = xsm + (size_t) s * stage_b, * Bs = As + kXABytes;
#pragma unroll
                for (int j = 0; j < 8; j++)
                    tc_mma_f16(tmem, tc_desc(As + tc_off(128, 0, 32 * j), 16 * 128, 128),
                               tc_desc(Bs + tc_off(Np, 0, 32 * j), (uint32_t) (Np / 8) * 128, 128), idesc,
                               kc > 0 || j > 0);
                tc_commit(&empty[s]);
            }
            tc_commit(&done);
        }
    } else if (live) {
        // ---------------- copies, decode (one A row per thread), epilogue
        const int r = tid;                                    // A row 0..127
        int i, j;
        if (MODE == MG_GU) {
            const int h = TR / 2, f = r & 63;
            i = f / h;
            j = (r < 64 ? 0 : h) + f % h;
        } else {
            i = r / TR;
            j = r % TR;
        }
        const uint32_t run = 32u * TR, ptile = 2 * run;       // one tile's code bytes per chunk: two runs
        // chunk kc into stage kc % 3: the rows' code bytes and the chunk's B block
        auto issue = [&](int kc) {
            uint8_t * st = xsm + (size_t) (kc % kXStages) * stage_b;
            const int pr = (int) (run / 16), pt = 2 * pr;
            for (int p = tid; p < ntl * pt; p += 128) {
                const int ti = p / pt, rem = p % pt, sec = rem / pr, off = rem % pr;
                const uint8_t * src = tiles + (size_t) ti * t.tb + tg.pl_off[0] + (sec ? tg.pl_sec[0] : 0) +
                                      (size_t) (2 * kc) * TR * 16 + (size_t) off * 16;
                xa_cp16(st + kXABytes + kXBBytes + (size_t) ti * ptile + (size_t) sec * run + (size_t) off * 16, src);
            }
            for (int p = tid; p < Np * 16; p += 128)
                xa_cp16(st + kXABytes + (size_t) p * 16, bsrc + (size_t) kc * kXBBytes + (size_t) p * 16);
        };
        // the rows' group fields over the whole width, then the first two chunks
        {
            const int pf = (int) (fb / 16);
            for (int p = tid; p < ntl * pf; p += 128) {
                const int ti = p / pf;
                const uint32_t q = (uint32_t) (p % pf) * 16;
                const uint8_t * tl = tiles + (size_t) ti * t.tb;
                const uint8_t * src = q < f_sq ? tl + tg.sq_off + q
                                    : q < 2 * f_sq ? (t.has_min ? tl + tg.mq_off : tl + tg.sq_off) + (q - f_sq)
                                    : q < 2 * f_sq + f_sd ? tl + tg.sd_off + (q - 2 * f_sq)
                                    : (t.has_min ? tl + tg.md_off : tl + tg.sd_off) + (q - 2 * f_sq - f_sd);
                xa_cp16(fields + (size_t) ti * fb + q, src);
            }
        }
        issue(0);
        xa_commit();
        if (nkc > 1) issue(1);
        xa_commit();
        const uint8_t * fl = fields + (size_t) i * fb;
        bool ok = true;
        for (int kc = 0; kc < nkc; kc++) {
            const int s = kc % kXStages;
            // chunk kc + 2 into its stage once the MMAs of chunk kc - 1, its last user, are done
            bool bad = false;
            if (kc + 2 < nkc) {
                if (kc >= 1 && !xt_wait(&empty[(kc + 2) % kXStages], ((kc - 1) / kXStages) & 1, g.err, 120, &fail))
                    bad = true;
                if (!bad) issue(kc + 2);
            }
            xa_commit();
            xa_wait<2>();                                     // this thread's copies of chunk kc have landed
            if (bad) cfail[kc & 1] = 1;
            bar_sync(1, 128);                                 // and every thread's
            if (cfail[kc & 1]) { ok = false; break; }
            uint8_t * As = xsm + (size_t) s * stage_b;
            const uint8_t * raw = As + kXABytes + kXBBytes + (size_t) i * ptile;
            // fields of the quad kc: four groups' sq and mq, the superblock's d and md
            const uint32_t sq4 = *reinterpret_cast<const uint32_t *>(fl + (size_t) (kc * TR + j) * 4);
            const uint32_t mq4 = *reinterpret_cast<const uint32_t *>(fl + f_sq + (size_t) (kc * TR + j) * 4);
            const float d = h2f(*reinterpret_cast<const uint16_t *>(fl + 2 * f_sq + (size_t) ((kc >> 1) * TR + j) * 2));
            const float md = t.has_min
                ? h2f(*reinterpret_cast<const uint16_t *>(fl + 2 * f_sq + f_sd + (size_t) ((kc >> 1) * TR + j) * 2))
                : 0.0f;
            __half2 sg[4], mg[4];
#pragma unroll
            for (int q = 0; q < 4; q++) {
                const float sv = d * (float) ((sq4 >> (8 * q)) & 0xffu);
                const float mv = t.has_min ? md * ((float) ((mq4 >> (8 * q)) & 0xffu) - t.mbias) : 0.0f;
                sg[q] = __float2half2_rn(sv);
                mg[q] = __float2half2_rn(mv);
            }
            // code words: lo section units 0, 1 (groups 0 | 1), hi section units 0, 1 (groups 2 | 3)
            const uint4 l0 = *reinterpret_cast<const uint4 *>(raw + (size_t) j * 16);
            const uint4 l1 = *reinterpret_cast<const uint4 *>(raw + (size_t) (TR + j) * 16);
            const uint4 h0 = *reinterpret_cast<const uint4 *>(raw + run + (size_t) j * 16);
            const uint4 h1 = *reinterpret_cast<const uint4 *>(raw + run + (size_t) (TR + j) * 16);
            // column k of the 128: group k / 32, position k % 32; a 16-byte
            // store holds columns 8 m .. 8 m + 7
            auto put = [&](int m, uint4 v) { *reinterpret_cast<uint4 *>(As + tc_off(128, r, 16 * m)) = v; };
            put(0, dq8<false>(l0.x, l0.y, sg[0], mg[0]));
            put(1, dq8<false>(l0.z, l0.w, sg[0], mg[0]));
            put(2, dq8<false>(l1.x, l1.y, sg[0], mg[0]));
            put(3, dq8<false>(l1.z, l1.w, sg[0], mg[0]));
            put(4, dq8<true>(l0.x, l0.y, sg[1], mg[1]));
            put(5, dq8<true>(l0.z, l0.w, sg[1], mg[1]));
            put(6, dq8<true>(l1.x, l1.y, sg[1], mg[1]));
            put(7, dq8<true>(l1.z, l1.w, sg[1], mg[1]));
            put(8, dq8<false>(h0.x, h0.y, sg[2], mg[2]));
            put(9, dq8<false>(h0.z, h0.w, sg[2], mg[2]));
            put(10, dq8<false>(h1.x, h1.y, sg[2], mg[2]));
            put(11, dq8<false>(h1.z, h1.w, sg[2], mg[2]));
            put(12, dq8<true>(h0.x, h0.y, sg[3], mg[3]));
            put(13, dq8<true>(h0.z, h0.w, sg[3], mg[3]));
            put(14, dq8<true>(h1.x, h1.y, sg[3], mg[3]));
            put(15, dq8<true>(h1.z, h1.w, sg[3], mg[3]));
            // the B block was written by copies (generic proxy) and A here:
            // both must be visible to the tensor core's reads
            fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) mbar_arrive(&full_a[s]);
        }
        xa_wait<0>();                                         // no copy lands after the CTA leaves
        ok = ok && xt_wait(&done, 0, g.err, 126, &fail);
        // every copy/decode warp knows whether the CTA failed before it reads TMEM
        bar_sync(1, 128);
        ok = ok && !fail;
        const int q = warp;                                   // TMEM lanes 32 q .. 32 q + 31
        float dv[kXN];
        if (ok) {
            tc_fence_after();
#pragma unroll
            for (int cc = 0; cc < kXN; cc += 8) {
                if (cc < Np) {
                    uint32_t r8[8];
                    tmem_ld8(tmem + ((uint32_t) (32 * q) << 16) + (uint32_t) cc, r8);
#pragma unroll
                    for (int k = 0; k < 8; k++) dv[cc + k] = __uint_as_float(r8[k]);
                }
            }
            tmem_wait_ld();
        }
        if (MODE == MG_DN) {
            if (ok) {
                const int row = 128 * mb + r;
                for (int tt = 0; tt < ntok; tt++)
                    g.out[(size_t) g.slots[s0 + tt] * g.out_stride + row] = dv[tt];
            }
        } else {
            // up rows (TMEM lanes 64..127) to the gate rows' threads through
            // shared memory (stage 0's A block: every MMA is done)
            float * xch = reinterpret_cast<float *>(xsm);
            if (ok && r >= 64)
                for (int tt = 0; tt < ntok; tt++) xch[(r - 64) * (kXN + 1) + tt] = dv[tt];
            bar_sync(1, 128);
            if (ok && r < 64) {
                const int f = 64 * mb + r;
                const int k = g.scatter[e][f];
                uint8_t * blk = g.hb + (size_t) c * moe_xb_bytes(g.ffn_f) + (size_t) (k >> 7) * kXBBytes;
                if (SB_CHECK(g.err, k >= 0 && k < g.ffn_f, 127)) {
                    for (int tt = 0; tt < Np; tt++) {
                        const float hv = tt < ntok ? silu_mul(dv[tt], xch[r * (kXN + 1) + tt]) : 0.0f;
                        *reinterpret_cast<__half *>(blk + tc_off(Np, tt, 2 * (k & 127))) = __float2half_rn(hv);
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        tc_fence_after();
        tmem_dealloc(tmem, 64);
    }
}

// ---------------------------------------------------------------- host

bool moe_tc_ok(const MoeLayer & m) {
    const TT & gu = m.gu, & dn = m.dn;
    return gu.nbits == 4 && dn.nbits == 4 && !gu.six && !dn.six && m.F % 128 == 0 && m.E % 128 == 0 &&
           gu.TR >= 2 && gu.TR % 2 == 0 && 64 % (gu.TR / 2) == 0 && 128 % dn.TR == 0 &&
           gu.cols == m.E && dn.cols == m.F;
}

int moe_tc_chunks(const MoeLayer & m, int T) {
    const int ns = T * m.k, held = m.e_hi - m.e_lo;
    const int c = held + (ns + kXN - 1) / kXN;
    return c < ns ? c : ns;
}

size_t moe_tc_smem(int K, int TR, int has_min) {
    const TileGeom tg = tile_geom(K, TR, 4, 0, has_min);
    const size_t fb = 2 * pad16((uint32_t) tg.P * TR * 4) + 2 * pad16((uint32_t) tg.S * TR * 2);
    return (size_t) kXStages * (kXABytes + kXBBytes + kXCodeBytes) + (size_t) (128 / TR) * fb;
}

size_t moe_tc_scratch(const MoeLayer & m, int T) {
    const size_t ch = (size_t) moe_tc_chunks(m, T);
    return ch * (moe_xb_bytes(m.E) + moe_xb_bytes(m.F));
}

cudaError_t moe_tc_enqueue(const MoeLayer & m, const MoeScratch & s, const float * in, int T, int nch_max,
                           cudaStream_t st, bool pdl, int * err) {
    MoeTcArgs a;
    memset(&a, 0, sizeof a);
    a.slots = s.r.slots; a.ch_e = s.r.ch_e; a.ch_s0 = s.r.ch_s0; a.ch_n = s.r.ch_n; a.meta = s.r.meta;
    a.err = err; a.ffn_f = m.F;
    uint8_t * xb = s.xb, * hb = s.xb + (size_t) nch_max * moe_xb_bytes(m.E);
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.stream = st;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    {
        MoeTcArgs x = a;
        x.perm = m.gu_perm; x.in = in; x.in_stride = m.E; x.in_div = m.k; x.bop = xb;
        cfg.gridDim = dim3(m.E / 128, nch_max);
        cfg.blockDim = dim3(128);
        cfg.dynamicSmemBytes = 0;
        const cudaError_t r = cudaLaunchKernelEx(&cfg, k_moe_xg, x, m.E);
        if (r != cudaSuccess) return r;
    }
    {
        MoeTcArgs x = a;
        x.t = m.gu; x.tiles = m.gu_tiles; x.scatter = m.dn_iperm; x.bop = xb; x.hb = hb;
        const size_t smem = moe_tc_smem(m.E, m.gu.TR, m.gu.has_min);
        static bool attr = false;
        if (!attr) {
            // the dynamic limit: the device's opt-in maximum less the kernel's static shared memory
            int dev = 0, optin = 0;
            cudaGetDevice(&dev);
            cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
            cudaFuncAttributes fa;
            if (cudaFuncGetAttributes(&fa, k_moe_tc<MG_GU>) == cudaSuccess)
                cudaFuncSetAttribute(k_moe_tc<MG_GU>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     optin - (int) fa.sharedSizeBytes);
            if (cudaFuncGetAttributes(&fa, k_moe_tc<MG_DN>) == cudaSuccess)
                cudaFuncSetAttribute(k_moe_tc<MG_DN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     optin - (int) fa.sharedSizeBytes);
            attr = true;
        }
        cfg.gridDim = dim3(m.F / 64, nch_max);
        cfg.blockDim = dim3(kXThreads);
        cfg.dynamicSmemBytes = smem;
        const cudaError_t r = cudaLaunchKernelEx(&cfg, k_moe_tc<MG_GU>, x);
        if (r != cudaSuccess) return r;
    }
    {
        MoeTcArgs x = a;
        x.t = m.dn; x.tiles = m.dn_tiles; x.bop = hb; x.out = s.yk; x.out_stride = m.E;
        cfg.gridDim = dim3(m.E / 128, nch_max);
        cfg.blockDim = dim3(kXThreads);
        cfg.dynamicSmemBytes = moe_tc_smem(m.F, m.dn.TR, m.dn.has_min);
        return cudaLaunchKernelEx(&cfg, k_moe_tc<MG_DN>, x);
    }
}

}  // namespace sb
