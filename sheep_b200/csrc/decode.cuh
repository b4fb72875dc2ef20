// Decode-step kernels: one token through the stack, device-resident.
//
// Per layer (the reference's f2_layer order, sml/sml-gpu-fwd.c:604-633, and the
// CPU forward sml/sml-run.c:3340-3520):
//   k_tgemv<QKV>   RMSNorm + gather + int8 quant (prologue), q|k|v rows, + bias
//   k_attn         Q/K norm (if any), RoPE, fp16 KV write, split-position attention
//   k_tgemv<O>     gather + quant of the attention output, o rows, x += y
//   k_tgemv<FFN>   RMSNorm + quant, gate and up rows, silu(g)*u written in the
//                  down projection's permuted order
//   k_tgemv<DOWN>  quant, down rows, x += y
// then k_tgemv<HEAD> (final norm, head rows, logits, greedy argmax). The GEMV
// kernels live in tgemv.cuh; this file holds the rest.
//
// Every kernel signals its dependents at entry (programmatic dependent
// launch) and every CTA calls pdl_wait() before it can exit: a grid may only
// complete after its predecessor has.
#pragma once

#include "expf_libm.h"
#include "qgemv.cuh"

namespace sb {

enum GemvMode { GM_QKV = 0, GM_O = 1, GM_FFN = 2, GM_DOWN = 3, GM_HEAD = 4, GM_PLAIN = 5 };

// Shared memory for the activation of a width-n input.
__host__ __device__ inline size_t act_smem_bytes(int n) {
    return (size_t) n + (size_t) (n / kGroup) * 8 + 64;
}

SB_DEV ActS act_carve(uint8_t * smem, int n) {
    ActS a;
    a.q = reinterpret_cast<int8_t *>(smem);
    a.xs = reinterpret_cast<float *>(smem + n);
    a.xsum = a.xs + n / kGroup;
    a.n = n;
    return a;
}

// The reference's exponential for SiLU (sml_exp_ps, sml/sml-run.c:392-413, the
// AVX2 build's): x clamped to [-88, 88], f = x*log2(e), r = f rounded to
// nearest even, 2^(f - r) by a degree-5 polynomial in Horner form (each step
// one fused multiply-add, as gcc contracts the intrinsics' add(mul(p, g), c)),
// scaled by 2^r through the exponent field. Restated with the same constants so
// the hidden vector equals the reference's bit for bit.
SB_DEV float exp_silu(float x) {
    x = fminf(fmaxf(x, -88.0f), 88.0f);
    const float f = __fmul_rn(x, 1.44269504088896341f);
    const float r = rintf(f);
    const float g = __fsub_rn(f, r);
    float p = 1.3697664e-3f;
    p = __fmaf_rn(p, g, 8.3013611e-3f);
    p = __fmaf_rn(p, g, 5.5826318e-2f);
    p = __fmaf_rn(p, g, 2.4022652e-1f);
    p = __fmaf_rn(p, g, 6.9314718e-1f);
    p = __fmaf_rn(p, g, 1.0f);
    return __fmul_rn(p, __int_as_float(((int) r + 127) << 23));
}

SB_DEV float silu_mul(float g, float u) {
    // silu_mul (sml/sml-run.c:436-446), the vector arm every hidden width that
    // is a multiple of 8 takes: (g / (1 + exp(0 - g))) * u, IEEE division
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, exp_silu(__fsub_rn(0.0f, g)))), u);
}

// ---------------------------------------------------------------- embedding

// One code of row `row`, column i (permuted order), from every plane.
template <int NB>
SB_DEV int code_at(const QT & t, int row, int i) {
    const int n = t.cols, grp = i / kGroup, j = i % kGroup;
    auto nib = [&](const uint8_t * pl) {
        const uint8_t b = pl[(size_t) row * (n / 2) + (grp / 4) * 64 + ((grp & 3) >= 2 ? 32 : 0) + j];
        return (grp & 1) ? (b >> 4) & 15 : b & 15;
    };
    auto two = [&](const uint8_t * pl) {
        return (pl[(size_t) row * (n / 4) + (grp / 4) * 32 + j] >> (2 * (grp & 3))) & 3;
    };
    auto one = [&](const uint8_t * pl) {
        return (pl[(size_t) row * (n / 8) + grp * 4 + j / 8] >> (j & 7)) & 1;
    };
    switch (NB) {
    case 2: return two(t.pl[0]);
    case 3: return two(t.pl[0]) + (one(t.pl[1]) << 2);
    case 4: return nib(t.pl[0]);
    case 5: return nib(t.pl[0]) + (one(t.pl[1]) << 4);
    case 6: return (two(t.pl[0]) << 4) + nib(t.pl[1]);
    case 7: return nib(t.pl[0]) + (two(t.pl[1]) << 4) + (one(t.pl[2]) << 6);
    default: return nib(t.pl[0]) + (nib(t.pl[1]) << 4);
    }
}

template <int SIX>
SB_DEV int field_at(const uint8_t * f, int frow, int row, int grp) {
    if (!SIX) return f[(size_t) row * frow + grp];
    const uint8_t * p = f + (size_t) row * frow + (grp >> 2) * 3;
    const uint32_t b0 = p[0], b1 = p[1], b2 = p[2];
    switch (grp & 3) {
    case 0: return (int) (b0 & 63u);
    case 1: return (int) (((b0 >> 6) | (b1 << 2)) & 63u);
    case 2: return (int) (((b1 >> 4) | (b2 << 4)) & 63u);
    default: return (int) ((b2 >> 2) & 63u);
    }
}

// w = code * (d * sq) + md * (mq - bias), multiply and add rounded separately
// (sml/sml-kernel.c:2146-2157).
template <int NB, int SIX>
SB_DEV float dequant_at(const QT & t, int row, int i) {
    const int grp = i / kGroup;
    const float step = __fmul_rn(h2f(t.sd[(size_t) row * t.nsb + grp / kGps]), (float) field_at<SIX>(t.sq, t.frow, row, grp));
    float mn = 0.0f;
    if (t.has_min)
        mn = __fmul_rn(h2f(t.md[(size_t) row * t.nsb + grp / kGps]),
                       __fsub_rn((float) field_at<SIX>(t.mq, t.frow, row, grp), t.mbias));
    return __fadd_rn(__fmul_rn((float) code_at<NB>(t, row, i), step), mn);
}

// x[perm[i]] = dequant(emb[tok], i): the embedding row scattered back to
// natural order (sml/sml-run.c:3332-3336). tok is read from device memory so a
// captured graph replays the greedy loop without the host.
template <int NB, int SIX>
__global__ void k_embed(const __grid_constant__ QT t, const int * dtok, float * x, int * err, unsigned * seq) {
    pdl_launch_dependents();
    pdl_wait();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (seq && i == 0) *seq += 1u;   // tokens run (a tensor-parallel engine's exchange events count by it)
    if (i >= t.cols) return;
    const int tok = *dtok;
    if (!SB_CHECK(err, tok >= 0 && tok < t.rows, 301)) return;
    x[t.perm[i]] = dequant_at<NB, SIX>(t, tok, i);
}

// Standalone activation quantization (sml_quantize_act after sml_gather):
// q in natural group order. One warp per group.
static __global__ void k_quant_act(const float * x, const int32_t * perm, int n, int8_t * q, float * s, int32_t * sums) {
    const int lane = threadIdx.x & 31;
    const int grp = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (grp >= n / kGroup) return;
    const int i = grp * kGroup + lane;
    const float v = x[perm ? perm[i] : i];
    const float amax = warp_max(fabsf(v));
    const float sc = __fdiv_rn(amax, 127.0f);
    const float is = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    int c = __float2int_rn(__fmul_rn(v, is));
    c = c > 127 ? 127 : c < -127 ? -127 : c;
    const int sum = warp_sum_i(c);
    q[i] = (int8_t) c;
    if (lane == 0) { s[grp] = sc; sums[grp] = sum; }
}

template <int NB, int SIX>
__global__ void k_dequant_rows(const __grid_constant__ QT t, const int * rows, int nrows, float * out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int r = blockIdx.y;
    if (i >= t.cols || r >= nrows) return;
    out[(size_t) r * t.cols + i] = dequant_at<NB, SIX>(t, rows[r], i);
}

// ---------------------------------------------------------------- attention

struct AttnArgs {
    const float * qkv;       // [q | k | v] of this token, before RoPE
    int n_head, n_kv, hd, qd, kvd;
    const float * qn, * kn;  // Q/K norm gains (per head, hd long) or NULL
    float eps;
    const float * rcos, * rsin;   // [n_ctx][hd/2] RoPE tables
    uint16_t * kc, * vc;     // this layer's cache, [n_ctx][kvd] fp16
    int n_ctx;
    const int * pos;         // device position, or NULL: pos_imm
    int pos_imm;
    int chunk;               // positions per CTA
    float scale;             // 1/sqrt(hd)
    float * part;            // [n_head][max_chunks][hd + 2]
    unsigned * cnt;          // [n_head]
    int max_chunks;
    float * out;             // [qd] attention output
    const ExpfEntry * xtab;  // expf_libm.h table (k_attn_seq), or NULL: exp rounded from double
    float xnear;             // ... consulted within this distance of a rounding midpoint
    int qkv_ld, out_ld;      // k_attn_seq over a prompt chunk: token blockIdx.y at qkv + y*qkv_ld,
                             // position pos_imm + y, output out + y*out_ld
    int * err;
    unsigned long long * trace;
    int launch_id;
};

constexpr int kAttnThreads = 256;

// Per-head RMS norm (sml/sml-run.c:295-325, one head at a time) then RoPE by
// halved pairs (sml/sml-run.c:339-375) of a 128-thread block's head vector.
SB_DEV void norm_rope(float * v, const float * w, float eps, int hd, const float * cs, const float * sn, double * red) {
    if (w) {
        const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
        double s = 0.0;
        for (int i = threadIdx.x; i < hd; i += blockDim.x) s += (double) v[i] * (double) v[i];
        s = warp_sum_d(s);
        if (lane == 0) red[wp] = s;
        __syncthreads();
        double ss = 0.0;
        for (int k = 0; k < (int) (blockDim.x >> 5); k++) ss += red[k];
        const float f = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float) (ss / hd), eps)));
        __syncthreads();
        for (int i = threadIdx.x; i < hd; i += blockDim.x) v[i] = __fmul_rn(__fmul_rn(v[i], f), w[i]);
        __syncthreads();
    }
    const int half = hd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float a = v[i], b = v[i + half];
        // as the reference's build computes it (sml/sml-run.c:363-366 under gcc's
        // contraction): v[i] = fma(a, cos, -(b sin)), v[i + half] = fma(a, sin, b cos)
        v[i] = __fmaf_rn(a, cs[i], -__fmul_rn(b, sn[i]));
        v[i + half] = __fmaf_rn(a, sn[i], __fmul_rn(b, cs[i]));
    }
    __syncthreads();
}

// The host libm's expf on the device (expf_libm.h): exp in double rounded
// once; where that double lies within `near` float ulps of a rounding midpoint
// (about 0.2 % of arguments), the table says whether the host's expf rounds the
// other way.
SB_DEV float expf_libm(float x, const ExpfEntry * tab, float near) {
    const double d = exp((double) x);
    float y = __double2float_rn(d);
    if (tab && x < 0.0f) {
        const double r = d - (double) y;   // exact: d and y agree to a float ulp
        const uint32_t yb = __float_as_uint(y);
        const float nb = __uint_as_float(r > 0.0 ? yb + 1u : yb - 1u);   // neighbour on d's side (y > 0)
        const double side = fabs((double) nb - (double) y);
        if (r != 0.0 && 0.5 * side - fabs(r) < (double) near * side) {
            const uint32_t k = __float_as_uint(x), mask = (1u << kExpfBits) - 1u;
            uint32_t h = expf_slot(k);
            for (int i = 0; i < 64; i++) {   // the table is at most half full: a run ends well before
                const ExpfEntry e = tab[h];
                if (e.x == k) { y = __uint_as_float(e.y); break; }
                if (e.x == 0xffffffffu) break;
                h = (h + 1) & mask;
            }
        }
    }
    return y;
}

// RoPE by halved pairs as the reference's build computes it
// (sml/sml-run.c:363-366 under gcc's contraction): v[i] = fma(a, cos, -(b sin)),
// v[i + half] = fma(a, sin, b cos), a = v[i], b = v[i + half].
SB_DEV void rope_ref(float * v, int hd, const float * cs, const float * sn) {
    const int half = hd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const float a = v[i], b = v[i + half];
        v[i] = __fmaf_rn(a, cs[i], -__fmul_rn(b, sn[i]));
        v[i + half] = __fmaf_rn(a, sn[i], __fmul_rn(b, cs[i]));
    }
}

// Per-head RMS norm of Q or K (sml/sml-run.c:329-333): the sum of squares in
// double, s = 1/sqrtf((float)(ss/hd) + eps), v = (v*s)*w.
SB_DEV void head_norm(float * v, const float * w, float eps, int hd, double * red) {
    const int lane = threadIdx.x & 31, wp = threadIdx.x >> 5;
    double s = 0.0;
    for (int i = threadIdx.x; i < hd; i += blockDim.x) s += (double) v[i] * (double) v[i];
    s = warp_sum_d(s);
    if (lane == 0) red[wp] = s;
    __syncthreads();
    double ss = 0.0;
    for (int k = 0; k < (int) (blockDim.x >> 5); k++) ss += red[k];
    const float f = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float) (ss / hd), eps)));
    __syncthreads();
    for (int i = threadIdx.x; i < hd; i += blockDim.x) v[i] = __fmul_rn(__fmul_rn(v[i], f), w[i]);
    __syncthreads();
}

constexpr int kSeqThreads = 256;
constexpr int kSeqCap = 192;      // cached positions whose K and V rows are staged in shared memory
                                  // (96 KB at head size 128: the CTA still fits beside a GEMV's)

SB_DEV void cp_async16(void * dst, const void * src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(dst)), "l"(src) : "memory");
}
SB_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
SB_DEV void cp_async_group() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SB_DEV void cp_async_wait_group() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }

// Shared memory of k_attn_seq: q, k, v, cos, sin, a score per position, and
// the K and V rows of the first kSeqCap positions (K rows padded by 16 bytes so
// a warp's 16-byte reads of 32 rows fall in distinct banks).
__host__ __device__ inline int attn_seq_cap(int n_ctx) { return n_ctx < kSeqCap ? n_ctx : kSeqCap; }
__host__ __device__ inline size_t attn_seq_smem_bytes(int hd, int n_ctx) {
    return (size_t) (4 * hd + ((n_ctx + 3) & ~3)) * 4 + (size_t) attn_seq_cap(n_ctx) * (2 * hd + 8) * 2;
}

// Decode attention of one query head per CTA, in the reference's float order
// (attn_row, sml/sml-run.c:180-266, AVX2 arm):
//   score(t) = (((c0+c4)+(c1+c5)) + ((c2+c6)+(c3+c7))) * scale, chain c_l the
//              fused multiply-adds over dims l, l+8, ... (one thread per position);
//   softmax    max, e_t = expf(s_t - max) (the host libm's, expf_libm), their sum
//              in position order (one thread), p_t = e_t * (1/sum);
//   out[d]     = fma chain over positions 0..pos in order (one thread per dim).
// The cached rows (positions before pos, up to kSeqCap of them) do not depend on
// the previous kernel: they are copied into shared memory (cp.async) before
// the dependency wait; past kSeqCap, keys are read from the cache in place and
// values pass through the keys' staging area (free once the scores are done)
// in double-buffered blocks of kSeqCap / 2 rows.
// After the wait: Q/K norm if any, RoPE (rope_ref), the new key/value rounded
// to fp16, written to the cache by the group's first head and into this CTA's
// staged rows. The serial loops (the softmax sum, each dim's chain) load a
// block of 32 positions before its arithmetic.
template <int HD>
// 32 registers a thread (8 CTAs' worth by the bound): two of its warps fit
// beside a streaming GEMV's on each SM sub-partition (tgemv.cuh k_tgemv).
__global__ void __launch_bounds__(kSeqThreads, 8) k_attn_seq(const __grid_constant__ AttnArgs g) {
    extern __shared__ __align__(16) float sm[];
    __shared__ double red[kSeqThreads / 32];
    __shared__ float wred[kSeqThreads / 32];
    __shared__ float s_inv;
    pdl_launch_dependents();
    SB_MARK(g.trace, g.launch_id, 0);
    constexpr int hd = HD;
    const int h = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wp = tid >> 5;
    const int pos = g.pos ? *g.pos : g.pos_imm + (int) blockIdx.y;
    const float * qkv = g.qkv + (size_t) blockIdx.y * g.qkv_ld;
    float * gout = g.out + (size_t) blockIdx.y * g.out_ld;
    if (!SB_CHECK(g.err, pos >= 0 && pos < g.n_ctx && g.hd == HD, 211)) { pdl_wait(); return; }
    const int rep = g.n_head / g.n_kv, kvh = h / rep, np = pos + 1;
    const int cap = attn_seq_cap(g.n_ctx), nst = pos < cap ? pos : cap;   // staged cached rows
    const int ks = hd + 8;                                                // K row stride (halves)
    float * q = sm, * kn = sm + hd, * vn = sm + 2 * hd, * cs = sm + 3 * hd, * sn = cs + hd / 2;
    float * sc = sm + 4 * hd;
    uint16_t * Ks = reinterpret_cast<uint16_t *>(sc + ((g.n_ctx + 3) & ~3));   // [cap][hd + 8]
    uint16_t * Vs = Ks + (size_t) cap * ks;                                     // [cap][hd]
    const size_t row0 = (size_t) kvh * hd;
    {
        const int per = hd / 8;
        for (int idx = tid; idx < nst * per; idx += kSeqThreads) {
            const int t = idx / per, part = idx % per;
            const size_t at = (size_t) t * g.kvd + row0 + part * 8;
            cp_async16(Ks + (size_t) t * ks + part * 8, g.kc + at);
            cp_async16(Vs + (size_t) t * hd + part * 8, g.vc + at);
        }
    }
    for (int i = tid; i < hd / 2; i += blockDim.x) {
        cs[i] = g.rcos[(size_t) pos * (hd / 2) + i];
        sn[i] = g.rsin[(size_t) pos * (hd / 2) + i];
    }
    pdl_wait();
    SB_MARK(g.trace, g.launch_id, 1);
    for (int i = tid; i < hd; i += blockDim.x) {
        q[i] = qkv[h * hd + i];
        kn[i] = qkv[g.qd + kvh * hd + i];
        vn[i] = qkv[g.qd + g.kvd + kvh * hd + i];
    }
    __syncthreads();
    if (g.qn) head_norm(q, g.qn, g.eps, hd, red);
    if (g.kn) head_norm(kn, g.kn, g.eps, hd, red);
    rope_ref(q, hd, cs, sn);
    rope_ref(kn, hd, cs, sn);
    __syncthreads();
    // the new row (rows past the staged ones are read from the cache, so a
    // position beyond kSeqCap must reach it before the scores: a fence and the
    // barrier below order the stores)
    for (int i = tid; i < hd; i += blockDim.x) {
        const uint16_t kh = f2h(kn[i]), vh = f2h(vn[i]);
        if (pos < cap) { Ks[(size_t) pos * ks + i] = kh; Vs[(size_t) pos * hd + i] = vh; }
        if (h % rep == 0 || pos >= cap) { g.kc[(size_t) pos * g.kvd + row0 + i] = kh; g.vc[(size_t) pos * g.kvd + row0 + i] = vh; }
    }
    if (pos >= cap) __threadfence_block();
    cp_async_wait_all();
    __syncthreads();
    SB_MARK(g.trace, g.launch_id, 2);
    // scores, one position per thread
    float m = -INFINITY;
    for (int t = tid; t < np; t += blockDim.x) {
        float c[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        const uint16_t * kr = t < cap ? Ks + (size_t) t * ks : g.kc + (size_t) t * g.kvd + row0;
#pragma unroll
        for (int i0 = 0; i0 < hd; i0 += 8) {
            const uint4 w = *reinterpret_cast<const uint4 *>(kr + i0);
            const float4 qa = *reinterpret_cast<const float4 *>(q + i0), qb = *reinterpret_cast<const float4 *>(q + i0 + 4);
            c[0] = __fmaf_rn(qa.x, h2f((uint16_t) (w.x & 0xffffu)), c[0]);
            c[1] = __fmaf_rn(qa.y, h2f((uint16_t) (w.x >> 16)), c[1]);
            c[2] = __fmaf_rn(qa.z, h2f((uint16_t) (w.y & 0xffffu)), c[2]);
            c[3] = __fmaf_rn(qa.w, h2f((uint16_t) (w.y >> 16)), c[3]);
            c[4] = __fmaf_rn(qb.x, h2f((uint16_t) (w.z & 0xffffu)), c[4]);
            c[5] = __fmaf_rn(qb.y, h2f((uint16_t) (w.z >> 16)), c[5]);
            c[6] = __fmaf_rn(qb.z, h2f((uint16_t) (w.w & 0xffffu)), c[6]);
            c[7] = __fmaf_rn(qb.w, h2f((uint16_t) (w.w >> 16)), c[7]);
        }
        const float s = __fadd_rn(__fadd_rn(__fadd_rn(c[0], c[4]), __fadd_rn(c[1], c[5])),
                                  __fadd_rn(__fadd_rn(c[2], c[6]), __fadd_rn(c[3], c[7])));
        sc[t] = __fmul_rn(s, g.scale);
        m = fmaxf(m, sc[t]);
    }
    SB_MARK(g.trace, g.launch_id, 5);
    m = warp_max(m);
    if (lane == 0) wred[wp] = m;
    __syncthreads();
    m = wred[0];
    for (int k = 1; k < (int) (blockDim.x >> 5); k++) m = fmaxf(m, wred[k]);
    for (int t = tid; t < np; t += blockDim.x) sc[t] = expf_libm(__fsub_rn(sc[t], m), g.xtab, g.xnear);
    __syncthreads();
    SB_MARK(g.trace, g.launch_id, 6);
    if (tid == 0) {
        // the sum in position order, each block of 32 loaded (as float4) before it is added
        float sum = 0.0f;
        int t = 0;
        for (; t + 32 <= np; t += 32) {
            float4 e[8];
#pragma unroll
            for (int u = 0; u < 8; u++) e[u] = *reinterpret_cast<const float4 *>(sc + t + 4 * u);
#pragma unroll
            for (int u = 0; u < 8; u++) {
                sum = __fadd_rn(sum, e[u].x); sum = __fadd_rn(sum, e[u].y);
                sum = __fadd_rn(sum, e[u].z); sum = __fadd_rn(sum, e[u].w);
            }
        }
        for (; t < np; t++) sum = __fadd_rn(sum, sc[t]);
        s_inv = __fdiv_rn(1.0f, sum);
    }
    __syncthreads();
    SB_MARK(g.trace, g.launch_id, 3);
    const float inv = s_inv;
    for (int t = tid; t < np; t += blockDim.x) sc[t] = __fmul_rn(sc[t], inv);
    __syncthreads();
    SB_MARK(g.trace, g.launch_id, 7);
    // two dims per thread (one 4-byte load of V per position), two chains over
    // the positions in order: rows [t0, t1) of a staged block V0 (row t at
    // V0 + (t - t0) * hd), a block of 32 loaded before its arithmetic
    const int d = 2 * tid;
    float o0 = 0.0f, o1 = 0.0f;
    auto chain = [&](const uint16_t * V0, int t0, int t1) {
        const uint32_t * vcol = reinterpret_cast<const uint32_t *>(V0 + d);
        int t = t0;
        for (; t + 32 <= t1; t += 32) {
            float4 p[8];
            uint32_t v[32];
#pragma unroll
            for (int u = 0; u < 8; u++) p[u] = *reinterpret_cast<const float4 *>(sc + t + 4 * u);
#pragma unroll
            for (int u = 0; u < 32; u++) v[u] = vcol[(size_t) (t - t0 + u) * (hd / 2)];
#pragma unroll
            for (int u = 0; u < 8; u++) {
                const float pp[4] = {p[u].x, p[u].y, p[u].z, p[u].w};
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const uint32_t vv = v[4 * u + w];
                    o0 = __fmaf_rn(pp[w], h2f((uint16_t) (vv & 0xffffu)), o0);
                    o1 = __fmaf_rn(pp[w], h2f((uint16_t) (vv >> 16)), o1);
                }
            }
        }
        for (; t < t1; t++) {
            const uint32_t vv = vcol[(size_t) (t - t0) * (hd / 2)];
            o0 = __fmaf_rn(sc[t], h2f((uint16_t) (vv & 0xffffu)), o0);
            o1 = __fmaf_rn(sc[t], h2f((uint16_t) (vv >> 16)), o1);
        }
    };
    const int ns = np < cap ? np : cap;
    if (tid < hd / 2) chain(Vs, 0, ns);
    if (np > cap) {
        // rows past the staged ones: blocks of VB rows through the keys' area
        // (2 VB rows of hd fit in its cap rows of hd + 8), the next block's
        // copies issued before this block's chains
        const int VB = cap / 2, per = hd / 8;
        auto issue = [&](uint16_t * buf, int t0) {
            const int n = (np - t0 < VB ? np - t0 : VB) * per;
            for (int idx = tid; idx < n; idx += kSeqThreads) {
                const int r = idx / per, part = idx % per;
                cp_async16(buf + (size_t) r * hd + part * 8, g.vc + (size_t) (t0 + r) * g.kvd + row0 + part * 8);
            }
            cp_async_group();
        };
        issue(Ks, cap);
        int b = 0;
        for (int t0 = cap; t0 < np; t0 += VB, b ^= 1) {
            uint16_t * cur = Ks + (size_t) b * VB * hd;
            if (t0 + VB < np) {
                issue(Ks + (size_t) (b ^ 1) * VB * hd, t0 + VB);
                cp_async_wait_group<1>();
            } else {
                cp_async_wait_group<0>();
            }
            __syncthreads();
            if (tid < hd / 2) chain(cur, t0, t0 + VB < np ? t0 + VB : np);
            __syncthreads();   // this buffer is refilled two blocks on
        }
    }
    if (tid < hd / 2) *reinterpret_cast<float2 *>(gout + h * hd + d) = make_float2(o0, o1);
    SB_MARK(g.trace, g.launch_id, 4);
}

// A prompt chunk's embedding rows: token t's row dequantized and scattered to
// natural order into x + t*E (as k_embed, one row per blockIdx.y).
template <int NB, int SIX>
__global__ void k_embed_rows(const __grid_constant__ QT t, const int * tok, float * x, int * err) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x, r = blockIdx.y;
    if (i >= t.cols) return;
    const int tk = tok[r];
    if (tk < 0 || tk >= t.rows) { if (i == 0) atomicExch(err, 303); return; }
    x[(size_t) r * t.cols + t.perm[i]] = dequant_at<NB, SIX>(t, tk, i);
}

// A prompt chunk's keys and values into the cache before its attention: token
// blockIdx.y (position pos0 + y), KV head blockIdx.x; K normed if kn, RoPE'd
// (rope_ref) and V as they are, both rounded to fp16 -- the values k_attn_seq
// computes for its own position, so every later read of these rows sees what
// the token's own attention writes.
template <int HD>
__global__ void __launch_bounds__(128) k_chunk_kv(const float * qkv, int ldq, int qd, int kvd, const float * kn,
                                                   float eps, const float * rcos, const float * rsin, uint16_t * kc,
                                                   uint16_t * vc, int pos0) {
    __shared__ float k[HD], cs[HD / 2], sn[HD / 2];
    __shared__ double red[4];
    const int kvh = blockIdx.x, t = blockIdx.y, pos = pos0 + t;
    const float * row = qkv + (size_t) t * ldq;
    for (int i = threadIdx.x; i < HD / 2; i += blockDim.x) {
        cs[i] = rcos[(size_t) pos * (HD / 2) + i];
        sn[i] = rsin[(size_t) pos * (HD / 2) + i];
    }
    for (int i = threadIdx.x; i < HD; i += blockDim.x) k[i] = row[qd + kvh * HD + i];
    __syncthreads();
    if (kn) head_norm(k, kn, eps, HD, red);
    rope_ref(k, HD, cs, sn);
    __syncthreads();
    for (int i = threadIdx.x; i < HD; i += blockDim.x) {
        kc[(size_t) pos * kvd + kvh * HD + i] = f2h(k[i]);
        vc[(size_t) pos * kvd + kvh * HD + i] = f2h(row[qd + kvd + kvh * HD + i]);
    }
}

// Greedy choice over the whole logit vector of a tensor-parallel engine, once
// every rank's rows have arrived: the first largest logit (ties to the lower
// index, sml/sml-run.c:3539-3544) becomes the next token; the position
// advances and the choice is logged.
constexpr int kArgmaxThreads = 1024;
// Shared memory of k_attn for head width hd and `chunk` positions.
__host__ __device__ inline size_t attn_smem_bytes(int hd, int chunk) {
    return (size_t) (4 * hd + chunk) * 4 + (size_t) chunk * (hd + 4) * 2 + (size_t) chunk * hd * 2;
}

// One CTA per (query head, chunk of positions): RoPE of q and of the new key,
// the fp16 KV write at pos (by one CTA per KV head), then attention over the
// chunk. The chunk's keys and values and the position's RoPE row are loaded
// into shared memory with every load issued at once. Scores take two threads
// per position, alternating 4-byte words of a key row padded to hd+4 halves
// (a warp's 32 reads fall in 32 banks); weighted values one thread per
// dimension. Chunks are combined by the last CTA of the head, in chunk order
// (flash-decoding partials).
static __global__ void __launch_bounds__(kAttnThreads) k_attn(const __grid_constant__ AttnArgs g) {
    extern __shared__ __align__(16) float sm[];
    __shared__ double red[kAttnThreads / 32];
    __shared__ float wred[kAttnThreads / 32];
    __shared__ unsigned last_flag;
    pdl_launch_dependents();
    SB_MARK(g.trace, g.launch_id, 0);
    const int h = blockIdx.x, c = blockIdx.y, hd = g.hd, tid = threadIdx.x;
    // the position comes from the previous token; the cached keys and values
    // before it from earlier tokens: neither waits on the previous kernel
    const int pos = g.pos ? *g.pos : g.pos_imm;
    const int nchunk = pos / g.chunk + 1;
    if (c >= nchunk) return;
    const int t0 = c * g.chunk, t1 = min(pos + 1, t0 + g.chunk), nt = t1 - t0;
    if (!SB_CHECK(g.err, pos >= 0 && pos < g.n_ctx && nchunk <= g.max_chunks && nt <= g.chunk && (hd & 7) == 0, 201))
        return;
    const int rep = g.n_head / g.n_kv, kvh = h / rep;
    float * q = sm, * kn = sm + hd, * vn = sm + 2 * hd, * cs = sm + 3 * hd, * sn = cs + hd / 2;
    float * sc = sm + 4 * hd;
    uint16_t * Ks = reinterpret_cast<uint16_t *>(sm + 4 * hd + g.chunk);   // [chunk][hd + 4]
    uint16_t * Vs = Ks + (size_t) g.chunk * (hd + 4);                        // [chunk][hd]
    const int kst = hd + 4;
    for (int i = tid; i < hd / 2; i += blockDim.x) {
        cs[i] = g.rcos[(size_t) pos * (hd / 2) + i];
        sn[i] = g.rsin[(size_t) pos * (hd / 2) + i];
    }
    const int per = hd / 8;   // 16-byte pieces per row
    // in batches of kB pieces per thread: all of a batch's loads before its stores
    constexpr int kB = 8;
    for (int b0 = 0; b0 < nt * per; b0 += kB * (int) blockDim.x) {
        uint4 kv[kB], vv[kB];
#pragma unroll
        for (int r = 0; r < kB; r++) {
            const int idx = b0 + r * blockDim.x + tid;
            const int t = t0 + idx / per, part = idx % per;
            if (idx < nt * per && t != pos) {
                const size_t at = (size_t) t * g.kvd + (size_t) kvh * hd + part * 8;
                kv[r] = *reinterpret_cast<const uint4 *>(g.kc + at);
                vv[r] = *reinterpret_cast<const uint4 *>(g.vc + at);
            }
        }
#pragma unroll
        for (int r = 0; r < kB; r++) {
            const int idx = b0 + r * blockDim.x + tid;
            const int t = t0 + idx / per, part = idx % per;
            if (idx < nt * per && t != pos) {
                *reinterpret_cast<uint2 *>(Ks + (size_t) (t - t0) * kst + part * 8) = make_uint2(kv[r].x, kv[r].y);
                *reinterpret_cast<uint2 *>(Ks + (size_t) (t - t0) * kst + part * 8 + 4) = make_uint2(kv[r].z, kv[r].w);
                *reinterpret_cast<uint4 *>(Vs + (size_t) (t - t0) * hd + part * 8) = vv[r];
            }
        }
    }
    pdl_wait();
    SB_MARK(g.trace, g.launch_id, 1);
    for (int i = tid; i < hd; i += blockDim.x) {
        q[i] = g.qkv[h * hd + i];
        kn[i] = g.qkv[g.qd + kvh * hd + i];
        vn[i] = g.qkv[g.qd + g.kvd + kvh * hd + i];
    }
    __syncthreads();
    SB_MARK(g.trace, g.launch_id, 2);
    norm_rope(q, g.qn, g.eps, hd, cs, sn, red);
    norm_rope(kn, g.kn, g.eps, hd, cs, sn, red);
    // the new key and value as the cache stores them (fp16, round to nearest even)
    const size_t at = (size_t) pos * g.kvd + (size_t) kvh * hd;
    const bool mine = pos >= t0 && pos < t1;
    for (int i = tid; i < hd; i += blockDim.x) {
        const uint16_t kh = f2h(kn[i]), vh = f2h(vn[i]);
        if (mine) { Ks[(size_t) (pos - t0) * kst + i] = kh; Vs[(size_t) (pos - t0) * hd + i] = vh; }
        if (h % rep == 0 && mine) { g.kc[at + i] = kh; g.vc[at + i] = vh; }
    }
    __syncthreads();
    // scores, two threads per position (sml/sml-run.c:180-235: dot * 1/sqrt(hd))
    const int lane = tid & 31, wp = tid >> 5, nw = blockDim.x >> 5;
    for (int base = 0; base < nt; base += blockDim.x / 2) {
        const int p = base + (tid >> 1), half = tid & 1;
        float s = 0.0f;
        if (p < nt) {
            const uint32_t * kr = reinterpret_cast<const uint32_t *>(Ks + (size_t) p * kst);
            for (int i = half; i < hd / 2; i += 2) {
                const uint32_t w2 = kr[i];
                s += q[2 * i] * h2f((uint16_t) (w2 & 0xffffu));
                s += q[2 * i + 1] * h2f((uint16_t) (w2 >> 16));
            }
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (p < nt && half == 0) sc[p] = s * g.scale;
    }
    __syncthreads();
    SB_MARK(g.trace, g.launch_id, 3);
    float m = -INFINITY;
    for (int t = tid; t < nt; t += blockDim.x) m = fmaxf(m, sc[t]);
    m = warp_max(m);
    if (lane == 0) wred[wp] = m;
    __syncthreads();
    m = wred[0];
    for (int k = 1; k < nw; k++) m = fmaxf(m, wred[k]);
    __syncthreads();
    float l = 0.0f;
    for (int t = tid; t < nt; t += blockDim.x) { const float e = expf(sc[t] - m); sc[t] = e; l += e; }
    l = warp_sum(l);
    if (lane == 0) wred[wp] = l;
    __syncthreads();
    l = 0.0f;
    for (int k = 0; k < nw; k++) l += wred[k];
    SB_MARK(g.trace, g.launch_id, 4);
    // weighted values: one dimension per thread
    for (int i = tid; i < hd; i += blockDim.x) {
        float o = 0.0f;
        for (int t = 0; t < nt; t++) o += sc[t] * h2f(Vs[(size_t) t * hd + i]);
        if (nchunk == 1) g.out[h * hd + i] = o / l;
        else g.part[((size_t) h * g.max_chunks + c) * (hd + 2) + 2 + i] = o;
    }
    SB_MARK(g.trace, g.launch_id, 5);
    if (nchunk == 1) return;
    if (tid == 0) {
        g.part[((size_t) h * g.max_chunks + c) * (hd + 2)] = m;
        g.part[((size_t) h * g.max_chunks + c) * (hd + 2) + 1] = l;
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_flag = atomicAdd(&g.cnt[h], 1u) == (unsigned) nchunk - 1;
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
#ifdef SB_TRACE
    if (g.trace && tid == 0 && h < kTraceCtas) g.trace[((size_t) g.launch_id * kTraceCtas + h) * 8 + 6] = global_ns();
#endif
    // the last chunk of this head combines every chunk, in chunk order. The
    // partials are read through L2 (after the fence above) with plain loads; up
    // to 8 chunks, a thread issues every load it needs (each chunk's max and sum,
    // and its own output element's partials) before using any, so the combine
    // costs one round trip. The arithmetic is the same for any chunk count.
    const float * P = g.part + (size_t) h * g.max_chunks * (hd + 2);
    if (nchunk <= 8) {
        float mk[8], lk[8];
#pragma unroll
        for (int k = 0; k < 8; k++) {
            mk[k] = k < nchunk ? __ldcg(P + k * (hd + 2)) : -INFINITY;
            lk[k] = k < nchunk ? __ldcg(P + k * (hd + 2) + 1) : 0.0f;
        }
        for (int i = tid; i < hd; i += blockDim.x) {
            float pk[8];
#pragma unroll
            for (int k = 0; k < 8; k++) pk[k] = k < nchunk ? __ldcg(P + k * (hd + 2) + 2 + i) : 0.0f;
            float M = -INFINITY;
#pragma unroll
            for (int k = 0; k < 8; k++) if (k < nchunk) M = fmaxf(M, mk[k]);
            float Lsum = 0.0f, o = 0.0f;
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (k < nchunk) Lsum += lk[k] * expf(mk[k] - M);
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (k < nchunk) o += pk[k] * expf(mk[k] - M);
            g.out[h * hd + i] = o / Lsum;
        }
    } else {
        float M = -INFINITY;
        for (int k = 0; k < nchunk; k++) M = fmaxf(M, __ldcg(P + k * (hd + 2)));
        float Lsum = 0.0f;
        for (int k = 0; k < nchunk; k++) Lsum += __ldcg(P + k * (hd + 2) + 1) * expf(__ldcg(P + k * (hd + 2)) - M);
        for (int i = tid; i < hd; i += blockDim.x) {
            float o = 0.0f;
            for (int k = 0; k < nchunk; k++) o += __ldcg(P + k * (hd + 2) + 2 + i) * expf(__ldcg(P + k * (hd + 2)) - M);
            g.out[h * hd + i] = o / Lsum;
        }
    }
    if (tid == 0) g.cnt[h] = 0;
#ifdef SB_TRACE
    __syncthreads();
    if (g.trace && tid == 0 && h < kTraceCtas) g.trace[((size_t) g.launch_id * kTraceCtas + h) * 8 + 7] = global_ns();
#endif
}

}  // namespace sb
