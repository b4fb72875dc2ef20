// The whole decode step of a dense decoder as ONE persistent kernel.
//
// The multi-kernel chain (engine.cu: per layer q|k|v, attention, o, gate/up,
// down) pays, per kernel, a launch, a ramp of its weight stream and the
// staging of its activation; at batch 1 those, not HBM, set the token time.
// Here one CTA per SM stays resident for the token and runs every phase:
//
//   embed | per layer: q|k|v, attention, o, gate/up, down | head + argmax
//
// Weights never depend on activations, so the producer warp streams this
// CTA's tiles of EVERY phase, in phase order, into the shared-memory ring
// without waiting for anything but ring space; it runs ahead as far as the
// ring allows, and a phase finds its tiles already resident. Each matrix is
// cut into tiles as for the chain (tiles.h) and CTA b takes the same share
// [T*b/G, T*(b+1)/G) of every matrix. Tiles differ in size (a row of down
// against a pair of q rows), so the ring is a byte ring: item k takes the
// next tb bytes (wrapping to the start when they do not fit) and mbarrier
// slot k % 32, whose offset the producer publishes before arming it. Item k is
// consumed by warp k % 16 whatever the phase, so each slot has one consumer
// warp, which takes its items in order -- the mbarrier parity rule of tgemv.cuh.
//
// Phases meet at a grid barrier, and every value one phase hands to the next
// (residual stream, q|k|v, attention partials, hidden vector) carries its
// version. The barrier is a counter: consumer thread 0 of every CTA adds 1
// once the CTA's writes of the phase are issued, then waits until the counter
// reaches G times the barriers passed (the last CTA of the token resets it).
// It has no release fence: on this GPU a gpu-scope fence waits for the SM's
// outstanding memory traffic, the weight stream included, and roughly doubled
// the barrier. The versions make that safe: a value and its tag travel in one
// 64-bit word (single-copy atomic), and a reader that finds an older tag -- a
// store of the previous phase not yet visible -- polls that word again. Reads
// of a version finish before their CTA arrives, and the next version is
// written only after a later barrier, so a reader never sees a newer one.
// Work that does not depend on the other CTAs -- the next phase's column
// order and gain, an attention item's cached keys and values -- is issued
// between arriving and waiting.
//
// Per staged phase the consumers wait for the column order and norm gain (bulk
// copies issued one phase earlier), stage the int8 activation from the
// previous phase's output (read through L2), run their tiles, and write the phase's output. Attention runs as
// (head, chunk) items spread over the CTAs; every CTA combines the chunk
// partials itself while staging o. Arithmetic, epilogues and the order of
// every sum are the chain's kernels', so the logits equal the chain's.
//
// Every wait is bounded in time (2 s); once any wait in the grid has given up
// the others return at once, so a fault cannot hang the GPU. All G CTAs must
// be resident together (they wait on one another): the kernel is launched
// cooperatively, which guarantees that or fails.
#pragma once

#include "tgemv.cuh"

namespace sb {

struct MegaLayer {
    TT qkv, o, gu, dn;
    const float * an, * fn;        // RMSNorm gains
    const float * qkv_b;           // q|k|v bias or NULL
    const float * qn, * kn;        // Q/K norm gains or NULL
    const int32_t * dn_iperm;      // gate/up hidden value i goes to hp[dn_iperm[i]]
    uint16_t * kc, * vc;           // this layer's fp16 KV cache [n_ctx][kvd]
};

// A value and its version in one 64-bit word: the float in the low half, the
// tag in the high half.
typedef unsigned long long tagged_t;

struct MegaArgs {
    const MegaLayer * L;
    int n_layer;
    QT emb;
    TT head;
    const float * out_norm;
    tagged_t * x;                  // [E] residual stream
    tagged_t * qkv;                // [qd + 2 kvd] this layer's q | k | v, before RoPE
    tagged_t * part;               // [nh][max_chunks][hd + 2] attention partials: max, sum, unnormalized out
    tagged_t * hp;                 // [F] SiLU(gate) * up in down's column order
    float * logits;
    int E, nh, nkv, hd, qd, kvd, F, V, n_ctx;
    float eps, scale;
    const float * rcos, * rsin;
    int attn_chunk, max_chunks;
    int * tok, * pos, * tlog;
    float * am_val;
    int * am_idx;
    unsigned * am_cnt;
    unsigned * bar;                // grid barrier arrivals this token
    unsigned * seq;                // tokens run: the base of this token's tags
    uint32_t ring_bytes;           // the tile ring (bytes)
    uint32_t stage_bytes;          // the largest tile
    // shared memory: [x kept (E floats) | act + input + combine weights, or attention | statics | ring]
    uint32_t work_off, xin_off, stat_off, ring_off;
    int * err;
    unsigned long long * trace;
};

// ---------------------------------------------------------------- barrier

SB_DEV unsigned ld_relaxed_u32(const unsigned * p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
SB_DEV void red_relaxed_add(unsigned * p, unsigned v) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
SB_DEV void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Arrive: once every consumer's writes of the phase are issued (named
// barrier), thread 0 counts this CTA in.
SB_DEV void bar_arrive(const MegaArgs & g) {
    bar_sync(1, kConsThreads);
    if (threadIdx.x == 0) red_relaxed_add(g.bar, 1u);
}

// Wait until every CTA has arrived n times: thread 0 polls (bounded; it gives
// up at once if any wait of the grid already has), then the named barrier
// releases the other consumers.
SB_DEV void bar_wait(const MegaArgs & g, unsigned n, bool & failed) {
    if (threadIdx.x == 0 && !failed) {
        const unsigned target = n * gridDim.x;
        if (ld_relaxed_u32(g.bar) < target) {
            const unsigned long long t0 = global_ns();
            for (;;) {
                bool ok = false;
                for (int i = 0; i < 32 && !ok; i++) ok = ld_relaxed_u32(g.bar) >= target;
                if (ok) break;
                if (*(volatile int *) g.err || global_ns() - t0 > kWaitNs) {
                    atomicCAS(g.err, 0, 20);
                    failed = true;
                    break;
                }
            }
        }
    }
    bar_sync(1, kConsThreads);
}

// ---------------------------------------------------------------- versions

SB_DEV void st_tag(tagged_t * p, float v, unsigned tag) {
    const tagged_t w = ((tagged_t) tag << 32) | (tagged_t) __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.b64 [%0], %1;" :: "l"(p), "l"(w) : "memory");
}
SB_DEV tagged_t ld_tag(const tagged_t * p) {
    tagged_t w;
    asm volatile("ld.relaxed.gpu.global.b64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
SB_DEV bool tag_is(tagged_t w, unsigned tag) { return (unsigned) (w >> 32) == tag; }

// The value of the word at p (w: a first load of it) once it carries `tag`.
// Bounded: after kWaitNs, or at once if any wait of the grid has given up, it
// records the failure and returns what it has.
SB_DEV float tag_val(const tagged_t * p, tagged_t w, unsigned tag, bool & failed, int * err) {
    if (!tag_is(w, tag) && !failed) {
        const unsigned long long t0 = global_ns();
        for (;;) {
            bool ok = false;
            for (int i = 0; i < 8 && !ok; i++) {
                w = ld_tag(p);
                ok = tag_is(w, tag);
            }
            if (ok) break;
            if (*(volatile int *) err || global_ns() - t0 > kWaitNs) {
                atomicCAS(err, 0, 21);
                failed = true;
                break;
            }
        }
    }
    return __uint_as_float((unsigned) w);
}
SB_DEV float ld_val(const tagged_t * p, unsigned tag, bool & failed, int * err) {
    return tag_val(p, ld_tag(p), tag, failed, err);
}

// Tags: version v of the residual stream (0 embedded, 2l+1 after layer l's o,
// 2l+2 after its down) and layer l's q|k|v, partials and hidden vector, in
// token `seq`. Distinct for 2^32 / (2 n_layer + 3) tokens.
SB_DEV unsigned tag_x(const MegaArgs & g, unsigned seq, int v) { return seq * (2u * g.n_layer + 3u) + (unsigned) v + 1u; }
SB_DEV unsigned tag_l(const MegaArgs & g, unsigned seq, int l) { return seq * ((unsigned) g.n_layer + 1u) + (unsigned) l + 1u; }

// ---------------------------------------------------------------- staging

// Stage the residual stream as the int8 activation: x read through L2 (other
// CTAs wrote it) and kept in xk (the epilogues of o and down add to it), the
// RMS norm (sum of squares in double, thread tid taking x[4 tid..4 tid+3] and
// every 2048 after, as tg_stage does), then the gather through perm_s.
SB_DEV void stage_x(const MegaArgs & g, unsigned tag, const int32_t * perm_s, const float * gain_s, ActS & a,
                    float * xk, double * red, bool & failed) {
    const int n = g.E, ng = n / kGroup, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int team = tid >> 3, sub = tid & 7, nteam = kConsThreads / 8;
    constexpr int kR = 4;   // n <= kR * 4 * 512
    tagged_t v[kR][4];
#pragma unroll
    for (int r = 0; r < kR; r++) {
        const int i = 4 * tid + r * 4 * kConsThreads;
#pragma unroll
        for (int c = 0; c < 4; c++) v[r][c] = i < n ? ld_tag(g.x + i + c) : 0ull;
    }
    double q = 0.0;
#pragma unroll
    for (int r = 0; r < kR; r++) {
        const int i = 4 * tid + r * 4 * kConsThreads;
        if (i < n) {
            float f[4];
#pragma unroll
            for (int c = 0; c < 4; c++) f[c] = tag_val(g.x + i + c, v[r][c], tag, failed, g.err);
            *reinterpret_cast<float4 *>(xk + i) = make_float4(f[0], f[1], f[2], f[3]);
            q += (double) f[0] * f[0] + (double) f[1] * f[1] + (double) f[2] * f[2] + (double) f[3] * f[3];
        }
    }
    float s = 1.0f;
    if (gain_s) {
        q = warp_sum_d(q);
        if (lane == 0) red[w] = q;
    }
    bar_sync(1, kConsThreads);
    if (gain_s) {
        double ss = 0.0;
        for (int k = 0; k < kConsWarps; k++) ss += red[k];
        s = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float) (ss / n), g.eps)));
    }
    for (int base = 0; base < ng; base += nteam) {
        const int grp = base + team;
        const int gg = grp < ng ? grp : 0;
        const int4 p4 = *reinterpret_cast<const int4 *>(perm_s + gg * kGroup + 4 * sub);
        const int pi[4] = {p4.x, p4.y, p4.z, p4.w};
        float vv[4];
#pragma unroll
        for (int k = 0; k < 4; k++)
            vv[k] = gain_s ? __fmul_rn(__fmul_rn(xk[pi[k]], s), gain_s[pi[k]]) : xk[pi[k]];
        quant_team_to(make_float4(vv[0], vv[1], vv[2], vv[3]), grp, sub, a, grp < ng);
    }
    bar_sync(1, kConsThreads);
}

// Stage the attention output for o: combine each head's chunk partials in
// chunk order (as k_attn's last chunk does), then gather through perm_s.
// cw: scratch of 2 * nh * nchunk + nh floats.
SB_DEV void stage_att(const MegaArgs & g, unsigned tag, int nchunk, const int32_t * perm_s, ActS & a, float * xin,
                      float * cw, bool & failed) {
    const int n = g.qd, ng = n / kGroup, tid = threadIdx.x, hd = g.hd, st = hd + 2, nhc = g.nh * nchunk;
    const int team = tid >> 3, sub = tid & 7, nteam = kConsThreads / 8;
    float * cm = cw, * cl = cw + nhc, * Lh = cl + nhc;
    // every load issued before the first is used: each thread's outputs of the
    // first kC chunks, then the (max, sum) pairs
    constexpr int kC = 4, kI = 4;   // first kC chunks of kI outputs per thread held in registers
    tagged_t ov[kI][kC];
#pragma unroll
    for (int r = 0; r < kI; r++) {
        const int i = tid + r * kConsThreads, h = i / hd, d = i - h * hd;
#pragma unroll
        for (int k = 0; k < kC; k++)
            ov[r][k] = i < n && k < nchunk ? ld_tag(g.part + ((size_t) h * g.max_chunks + k) * st + 2 + d) : 0ull;
    }
    for (int e = tid; e < nhc; e += kConsThreads) {
        const tagged_t * p = g.part + ((size_t) (e / nchunk) * g.max_chunks + e % nchunk) * st;
        const tagged_t m0 = ld_tag(p), l0 = ld_tag(p + 1);
        cm[e] = tag_val(p, m0, tag, failed, g.err);
        cl[e] = tag_val(p + 1, l0, tag, failed, g.err);
    }
    bar_sync(1, kConsThreads);
    if (tid < g.nh) {
        float * m = cm + tid * nchunk, * l = cl + tid * nchunk;
        float M = -INFINITY;
        for (int k = 0; k < nchunk; k++) M = fmaxf(M, m[k]);
        float L = 0.0f;
        for (int k = 0; k < nchunk; k++) {
            const float ek = expf(m[k] - M);
            L += l[k] * ek;
            m[k] = ek;                      // the chunk's weight from here on
        }
        Lh[tid] = L;
    }
    bar_sync(1, kConsThreads);
#pragma unroll
    for (int r = 0; r < kI; r++) {
        const int i = tid + r * kConsThreads;
        if (i < n) {
            const int h = i / hd, d = i - h * hd;
            const tagged_t * p = g.part + (size_t) h * g.max_chunks * st + 2 + d;
            float o = 0.0f;
#pragma unroll
            for (int k = 0; k < kC; k++)
                if (k < nchunk) o += tag_val(p + (size_t) k * st, ov[r][k], tag, failed, g.err) * cm[h * nchunk + k];
            for (int k = kC; k < nchunk; k++) o += ld_val(p + (size_t) k * st, tag, failed, g.err) * cm[h * nchunk + k];
            xin[i] = o / Lh[h];
        }
    }
    for (int i = tid + kI * kConsThreads; i < n; i += kConsThreads) {
        const int h = i / hd, d = i - h * hd;
        const tagged_t * p = g.part + (size_t) h * g.max_chunks * st + 2 + d;
        float o = 0.0f;
        for (int k = 0; k < nchunk; k++) o += ld_val(p + (size_t) k * st, tag, failed, g.err) * cm[h * nchunk + k];
        xin[i] = o / Lh[h];
    }
    bar_sync(1, kConsThreads);
    for (int base = 0; base < ng; base += nteam) {
        const int grp = base + team;
        const int gg = grp < ng ? grp : 0;
        const int4 p4 = *reinterpret_cast<const int4 *>(perm_s + gg * kGroup + 4 * sub);
        quant_team_to(make_float4(xin[p4.x], xin[p4.y], xin[p4.z], xin[p4.w]), grp, sub, a, grp < ng);
    }
    bar_sync(1, kConsThreads);
}

// Stage the hidden vector for down (already in its column order): a team of 8
// lanes per group of 32, every load of a batch issued before any is used.
SB_DEV void stage_hp(const MegaArgs & g, unsigned tag, ActS & a, bool & failed) {
    const int n = g.F, ng = n / kGroup, tid = threadIdx.x;
    const int team = tid >> 3, sub = tid & 7, nteam = kConsThreads / 8;
    constexpr int kR = 4;
    for (int base = 0; base < ng; base += kR * nteam) {
        tagged_t v[kR][4];
#pragma unroll
        for (int r = 0; r < kR; r++) {
            const int grp = base + r * nteam + team;
#pragma unroll
            for (int c = 0; c < 4; c++) v[r][c] = grp < ng ? ld_tag(g.hp + grp * kGroup + 4 * sub + c) : 0ull;
        }
#pragma unroll
        for (int r = 0; r < kR; r++) {
            const int g0 = base + r * nteam;
            if (g0 >= ng) break;
            const int grp = g0 + team;
            float f[4] = {0.f, 0.f, 0.f, 0.f};
            if (grp < ng)
#pragma unroll
                for (int c = 0; c < 4; c++) f[c] = tag_val(g.hp + grp * kGroup + 4 * sub + c, v[r][c], tag, failed, g.err);
            quant_team_to(make_float4(f[0], f[1], f[2], f[3]), grp, sub, a, grp < ng);
        }
    }
    bar_sync(1, kConsThreads);
}

// ---------------------------------------------------------------- attention

// Per-head RMS norm then RoPE by halved pairs, consumer threads (norm_rope of
// decode.cuh with a named barrier).
SB_DEV void mk_norm_rope(float * v, const float * w, float eps, int hd, const float * cs, const float * sn,
                         double * red) {
    const int tid = threadIdx.x;
    if (w) {
        const int lane = tid & 31, wp = tid >> 5;
        double s = 0.0;
        for (int i = tid; i < hd; i += kConsThreads) s += (double) v[i] * (double) v[i];
        s = warp_sum_d(s);
        if (lane == 0) red[wp] = s;
        bar_sync(1, kConsThreads);
        double ss = 0.0;
        for (int k = 0; k < kConsWarps; k++) ss += red[k];
        const float f = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float) (ss / hd), eps)));
        bar_sync(1, kConsThreads);
        for (int i = tid; i < hd; i += kConsThreads) v[i] = __fmul_rn(__fmul_rn(v[i], f), w[i]);
        bar_sync(1, kConsThreads);
    }
    const int half = hd / 2;
    for (int i = tid; i < half; i += kConsThreads) {
        const float a = v[i], b = v[i + half];
        // both products rounded, then the sum: no fused multiply-add, as the CPU
        // restatement computes it (sml/sml-run.c:363-366, built without contraction),
        // so keys are bit-equal before their fp16 rounding
        v[i] = __fsub_rn(__fmul_rn(a, cs[i]), __fmul_rn(b, sn[i]));
        v[i + half] = __fadd_rn(__fmul_rn(a, sn[i]), __fmul_rn(b, cs[i]));
    }
    bar_sync(1, kConsThreads);
}

// Shared-memory view of one attention item (k_attn's layout).
struct AttnSm {
    float * q, * kn, * vn, * cs, * sn, * sc;
    uint16_t * Ks, * Vs;
    int kst;
};
SB_DEV AttnSm attn_sm(float * sm, int hd, int chunk) {
    AttnSm a;
    a.q = sm; a.kn = sm + hd; a.vn = sm + 2 * hd; a.cs = sm + 3 * hd; a.sn = a.cs + hd / 2;
    a.sc = sm + 4 * hd;
    a.Ks = reinterpret_cast<uint16_t *>(sm + 4 * hd + chunk);
    a.Vs = a.Ks + (size_t) chunk * (hd + 4);
    a.kst = hd + 4;
    return a;
}

// The item's cached keys and values (earlier tokens: no dependence on this
// token's phases) and its RoPE row into shared memory.
SB_DEV void attn_load(const MegaArgs & g, const MegaLayer & y, int h, int c, int pos, const AttnSm & A) {
    const int hd = g.hd, tid = threadIdx.x, chunk = g.attn_chunk;
    const int t0 = c * chunk, t1 = min(pos + 1, t0 + chunk), nt = t1 - t0;
    const int kvh = h / (g.nh / g.nkv), per = hd / 8;
    constexpr int kB = 4;
    for (int b0 = 0; b0 < nt * per; b0 += kB * kConsThreads) {
        uint4 kv[kB], vv[kB];
#pragma unroll
        for (int r = 0; r < kB; r++) {
            const int idx = b0 + r * kConsThreads + tid;
            const int t = t0 + idx / per, part = idx % per;
            if (idx < nt * per && t != pos) {
                const size_t at = (size_t) t * g.kvd + (size_t) kvh * hd + part * 8;
                kv[r] = *reinterpret_cast<const uint4 *>(y.kc + at);
                vv[r] = *reinterpret_cast<const uint4 *>(y.vc + at);
            }
        }
#pragma unroll
        for (int r = 0; r < kB; r++) {
            const int idx = b0 + r * kConsThreads + tid;
            const int t = t0 + idx / per, part = idx % per;
            if (idx < nt * per && t != pos) {
                *reinterpret_cast<uint2 *>(A.Ks + (size_t) (t - t0) * A.kst + part * 8) = make_uint2(kv[r].x, kv[r].y);
                *reinterpret_cast<uint2 *>(A.Ks + (size_t) (t - t0) * A.kst + part * 8 + 4) = make_uint2(kv[r].z, kv[r].w);
                *reinterpret_cast<uint4 *>(A.Vs + (size_t) (t - t0) * hd + part * 8) = vv[r];
            }
        }
    }
    for (int i = tid; i < hd / 2; i += kConsThreads) {
        A.cs[i] = g.rcos[(size_t) pos * (hd / 2) + i];
        A.sn[i] = g.rsin[(size_t) pos * (hd / 2) + i];
    }
}

// The rest of the item once q|k|v exist: k_attn's computation; the item's
// partial (max, sum, unnormalized output) goes to part.
SB_DEV void attn_compute(const MegaArgs & g, const MegaLayer & y, int h, int c, int pos, unsigned tag,
                         const AttnSm & A, double * red, float * wred, bool & failed) {
    const int hd = g.hd, tid = threadIdx.x, chunk = g.attn_chunk;
    const int t0 = c * chunk, t1 = min(pos + 1, t0 + chunk), nt = t1 - t0;
    const int rep = g.nh / g.nkv, kvh = h / rep, kst = A.kst;
    for (int i = tid; i < 3 * hd; i += kConsThreads) {
        const int part = i / hd, d = i - part * hd;
        const tagged_t * p = g.qkv + (part == 0 ? h * hd : g.qd + (part - 1) * g.kvd + kvh * hd) + d;
        A.q[i] = ld_val(p, tag, failed, g.err);   // q | kn | vn are consecutive
    }
    bar_sync(1, kConsThreads);
    mk_norm_rope(A.q, y.qn, g.eps, hd, A.cs, A.sn, red);
    mk_norm_rope(A.kn, y.kn, g.eps, hd, A.cs, A.sn, red);
    const size_t at = (size_t) pos * g.kvd + (size_t) kvh * hd;
    const bool mine = pos >= t0 && pos < t1;
    for (int i = tid; i < hd; i += kConsThreads) {
        const uint16_t kh = f2h(A.kn[i]), vh = f2h(A.vn[i]);
        if (mine) { A.Ks[(size_t) (pos - t0) * kst + i] = kh; A.Vs[(size_t) (pos - t0) * hd + i] = vh; }
        if (h % rep == 0 && mine) { y.kc[at + i] = kh; y.vc[at + i] = vh; }
    }
    bar_sync(1, kConsThreads);
    const int lane = tid & 31, wp = tid >> 5;
    for (int base = 0; base < nt; base += kConsThreads / 2) {
        const int p = base + (tid >> 1), half = tid & 1;
        float s = 0.0f;
        if (p < nt) {
            const uint32_t * kr = reinterpret_cast<const uint32_t *>(A.Ks + (size_t) p * kst);
            for (int i = half; i < hd / 2; i += 2) {
                const uint32_t w2 = kr[i];
                s += A.q[2 * i] * h2f((uint16_t) (w2 & 0xffffu));
                s += A.q[2 * i + 1] * h2f((uint16_t) (w2 >> 16));
            }
        }
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (p < nt && half == 0) A.sc[p] = s * g.scale;
    }
    bar_sync(1, kConsThreads);
    float m = -INFINITY;
    for (int t = tid; t < nt; t += kConsThreads) m = fmaxf(m, A.sc[t]);
    m = warp_max(m);
    if (lane == 0) wred[wp] = m;
    bar_sync(1, kConsThreads);
    m = wred[0];
    for (int k = 1; k < kConsWarps; k++) m = fmaxf(m, wred[k]);
    bar_sync(1, kConsThreads);
    float l = 0.0f;
    for (int t = tid; t < nt; t += kConsThreads) { const float e = expf(A.sc[t] - m); A.sc[t] = e; l += e; }
    l = warp_sum(l);
    if (lane == 0) wred[wp] = l;
    bar_sync(1, kConsThreads);
    l = 0.0f;
    for (int k = 0; k < kConsWarps; k++) l += wred[k];
    tagged_t * P = g.part + ((size_t) h * g.max_chunks + c) * (hd + 2);
    for (int i = tid; i < hd; i += kConsThreads) {
        float o = 0.0f;
        for (int t = 0; t < nt; t++) o += A.sc[t] * h2f(A.Vs[(size_t) t * hd + i]);
        st_tag(P + 2 + i, o, tag);
    }
    if (tid == 0) { st_tag(P, m, tag); st_tag(P + 1, l, tag); }
    bar_sync(1, kConsThreads);
}

// ---------------------------------------------------------------- phases

// This CTA's share of a tiled matrix.
SB_DEV void cta_range(int ntiles, int & t0, int & t1) {
    t0 = (int) ((long) ntiles * blockIdx.x / gridDim.x);
    t1 = (int) ((long) ntiles * (blockIdx.x + 1) / gridDim.x);
}

// The matrix of phase ph (0 q|k|v, 2 o, 3 gate/up, 4 down, 5 head) of layer l.
SB_DEV const TT * phase_tt(const MegaArgs & g, int l, int ph) {
    if (ph == 5) return &g.head;
    const MegaLayer & y = g.L[l];
    return ph == 0 ? &y.qkv : ph == 2 ? &y.o : ph == 3 ? &y.gu : &y.dn;
}

// This CTA's tiles [i0, i1) of t (ring items k0..) against the staged
// activation a, with MODE's epilogue: q|k|v rows (+ bias), residual rows
// xk[r] + y (o, down), SiLU(gate)*up scattered (gate/up), logits and the
// running argmax (head). Ends with every consumer done (the next phase
// reuses the activation, the kept residual and the work area).
template <int MODE, int NB, int SIX>
SB_DEV void mk_tiles(const MegaArgs & g, const TT & t, int i0, int i1, int k0, const ActS & a, uint8_t * ring,
                     uint64_t * full, uint64_t * empty, const uint32_t * ioff, const float * bias, const float * xk,
                     tagged_t * out, unsigned tag, const int32_t * scatter, bool & failed, float & best_v,
                     int & best_i, int ph) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const TileGeom tg = tile_geom(t.cols, t.TR, NB, SIX, t.has_min);
    const int TR = t.TR, j = lane % TR, v = lane / TR, VS = 32 / TR;
    const int k1 = k0 + (i1 - i0);
    for (int k = k0 + (((warp - k0) % kConsWarps) + kConsWarps) % kConsWarps; k < k1; k += kConsWarps) {
        const int s = k & (kMaxStages - 1), i = i0 + (k - k0);
        const bool ok = !failed && mbar_wait(&full[s], (k / kMaxStages) & 1, g.err, 2);
        failed = !ok;
        if (k < k0 + kConsWarps) SB_MARK(g.trace, ph, 2);   // thread 0's first tile of the phase is resident
        float acc = 0.0f;
        if (ok) acc = tile_row<NB, SIX>(ring + ioff[s], tg, a, j, v, VS, t.has_min, t.mbias, g.err);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        for (int o = 16; o >= TR; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
        if (MODE == GM_FFN) {
            const float up = __shfl_down_sync(0xffffffffu, acc, TR / 2);
            const int idx = i * (TR / 2) + lane;
            if (lane < TR / 2 && idx < g.F && SB_CHECK(g.err, scatter[idx] >= 0 && scatter[idx] < g.F, 108))
                st_tag(out + scatter[idx], silu_mul(acc, up), tag);
            continue;
        }
        const int r = i * TR + lane;
        if (lane < TR && r < t.rows) {
            if (MODE == GM_QKV) {
                st_tag(out + r, bias ? acc + bias[r] : acc, tag);
            } else if (MODE == GM_O || MODE == GM_DOWN) {
                st_tag(out + r, xk[r] + acc, tag);
            } else if (MODE == GM_HEAD) {
                g.logits[r] = acc;
                if (acc > best_v || (acc == best_v && r < best_i)) { best_v = acc; best_i = r; }
            }
        }
    }
    bar_sync(1, kConsThreads);
    SB_MARK(g.trace, ph, 3);
}

template <int NB, int SIX>
__global__ void __launch_bounds__(kTgThreads, 1) k_token(const __grid_constant__ MegaArgs g) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], sbar;
    __shared__ uint32_t ioff[kMaxStages], isz[kMaxStages];   // ring offset and bytes held, per slot
    __shared__ double red[kConsWarps];
    __shared__ float wred[kConsWarps];
    __shared__ float am_v[kConsWarps];
    __shared__ int am_i[kConsWarps];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, G = gridDim.x;
    uint8_t * ring = smem + g.ring_off;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(&sbar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsWarps) {
        // ---------------- producer: this CTA's tiles of every phase, in phase order
        if (lane == 0) {
            const uint32_t R = g.ring_bytes;
            uint32_t head = 0, used = 0;
            int k = 0, oldest = 0;
            bool stop = false;
            for (int l = 0; l <= g.n_layer && !stop; l++) {
                for (int ph = 0; ph < 6 && !stop; ph++) {
                    if (ph == 1) continue;                            // attention: no tiles
                    if ((l == g.n_layer) != (ph == 5)) continue;      // the head after the last layer
                    const TT * tp = phase_tt(g, l, ph);
                    const uint8_t * src = tp->tiles;
                    const uint32_t tb = tp->tb;
                    int i0, i1;
                    cta_range(tp->ntiles, i0, i1);
#ifdef SB_TRACE
                    const int tph = l * 5 + ph + 1;   // the consumers' phase index
                    if (g.trace && blockIdx.x < kTraceCtas) g.trace[((size_t) tph * kTraceCtas + blockIdx.x) * 8 + 6] = global_ns();
#endif
                    for (int i = i0; i < i1; i++, k++) {
                        uint32_t at = head, need = tb;
                        if (at + tb > R) { need += R - at; at = 0; }   // the tail is skipped
                        // free the oldest items until this one fits and has a slot
                        while (used + need > R || k - oldest >= kMaxStages) {
                            const int so = oldest & (kMaxStages - 1);
                            if (!mbar_wait(&empty[so], (oldest / kMaxStages) & 1, g.err, 1)) { stop = true; break; }
                            used -= isz[so];
                            oldest++;
                        }
                        if (stop) break;
                        const int s = k & (kMaxStages - 1);
                        isz[s] = need;
                        ioff[s] = at;
                        used += need;
                        head = at + tb;
                        mbar_expect_tx(&full[s], tb);
                        bulk_g2s(ring + at, src + (size_t) i * tb, tb, &full[s]);
                    }
#ifdef SB_TRACE
                    if (g.trace && blockIdx.x < kTraceCtas) g.trace[((size_t) tph * kTraceCtas + blockIdx.x) * 8 + 7] = global_ns();
#endif
                }
            }
            // no copy may still be landing when the CTA exits
            for (int q = oldest; q < k; q++) mbar_wait(&full[q & (kMaxStages - 1)], (q / kMaxStages) & 1, g.err, 3);
        }
        return;
    }

    // ---------------- consumers
    bool failed = false;
    unsigned sphase = 0, passed = 0;
    int k = 0;   // ring items consumed so far (every warp counts every item)
    int ph = 0;  // trace: phases begun
    const int pos = *g.pos;
    const unsigned seq = *g.seq;
    const int nchunk = pos / g.attn_chunk + 1;
    float * xk = reinterpret_cast<float *>(smem);
    uint8_t * work = smem + g.work_off;
    float * xin = reinterpret_cast<float *>(smem + g.xin_off);
    const int nmax = g.E > g.qd ? g.E : g.qd;
    float * cw = xin + nmax;
    int32_t * perm_s = reinterpret_cast<int32_t *>(smem + g.stat_off);
    float * gain_s = reinterpret_cast<float *>(smem + g.stat_off + (size_t) nmax * 4);
    const AttnSm A = attn_sm(reinterpret_cast<float *>(work), g.hd, g.attn_chunk);
    // statics (column order, gain) of the next staged phase: one thread's bulk copies
    auto load_statics = [&](const int32_t * perm, int n, const float * gain) {
        if (threadIdx.x == 0) {
            mbar_expect_tx(&sbar, (uint32_t) n * 4 * (gain ? 2 : 1));
            bulk_g2s(perm_s, perm, (uint32_t) n * 4, &sbar);
            if (gain) bulk_g2s(gain_s, gain, (uint32_t) n * 4, &sbar);
        }
    };
    auto wait_statics = [&]() {
        if (!failed && !mbar_wait(&sbar, sphase & 1, g.err, 4)) failed = true;
        sphase++;
    };
    load_statics(g.L[0].qkv.perm, g.E, g.L[0].an);
    // embed: x[perm[i]] = row tok of the embedding, this CTA's share of the columns
    SB_MARK(g.trace, ph, 0);
    {
        const int tok = *g.tok;
        if (SB_CHECK(g.err, tok >= 0 && tok < g.emb.rows, 301)) {
            const int c0 = (int) ((long) g.E * blockIdx.x / G), c1 = (int) ((long) g.E * (blockIdx.x + 1) / G);
            const unsigned t0 = tag_x(g, seq, 0);
            for (int i = c0 + threadIdx.x; i < c1; i += kConsThreads)
                st_tag(g.x + g.emb.perm[i], dequant_at<NB, SIX>(g.emb, tok, i), t0);
        }
    }
    bar_arrive(g);
    bar_wait(g, ++passed, failed);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const int nitems = g.nh * nchunk;
    for (int l = 0; l < g.n_layer; l++) {
        const MegaLayer & y = g.L[l];
        const unsigned tl = tag_l(g, seq, l);
        int i0, i1;
        // q | k | v
        SB_MARK(g.trace, ++ph, 0);
        wait_statics();
        {
            ActS a = act_carve(work, g.E);
            stage_x(g, tag_x(g, seq, 2 * l), perm_s, gain_s, a, xk, red, failed);
            SB_MARK(g.trace, ph, 1);
            load_statics(y.o.perm, g.qd, nullptr);
            cta_range(y.qkv.ntiles, i0, i1);
            mk_tiles<GM_QKV, NB, SIX>(g, y.qkv, i0, i1, k, a, ring, full, empty, ioff, y.qkv_b, nullptr, g.qkv, tl, nullptr,
                                      failed, best_v, best_i, ph);
            k += i1 - i0;
        }
        bar_arrive(g);
        // attention: (head, chunk) items over the CTAs; the first item's cached
        // keys and values load while the others finish q|k|v
        if ((int) blockIdx.x < nitems) attn_load(g, y, blockIdx.x / nchunk, blockIdx.x % nchunk, pos, A);
        bar_wait(g, ++passed, failed);
        SB_MARK(g.trace, ++ph, 0);
        if ((int) blockIdx.x < nitems) SB_MARK(g.trace, ph, 1);
        for (int it = blockIdx.x; it < nitems; it += G) {
            if (it != (int) blockIdx.x) attn_load(g, y, it / nchunk, it % nchunk, pos, A);
            bar_sync(1, kConsThreads);
            attn_compute(g, y, it / nchunk, it % nchunk, pos, tl, A, red, wred, failed);
            SB_MARK(g.trace, ph, 3);
        }
        bar_arrive(g);
        bar_wait(g, ++passed, failed);
        // o (residual)
        SB_MARK(g.trace, ++ph, 0);
        wait_statics();
        {
            ActS a = act_carve(work, g.qd);
            stage_att(g, tl, nchunk, perm_s, a, xin, cw, failed);
            SB_MARK(g.trace, ph, 1);
            load_statics(y.gu.perm, g.E, y.fn);
            cta_range(y.o.ntiles, i0, i1);
            mk_tiles<GM_O, NB, SIX>(g, y.o, i0, i1, k, a, ring, full, empty, ioff, nullptr, xk, g.x, tag_x(g, seq, 2 * l + 1), nullptr,
                                    failed, best_v, best_i, ph);
            k += i1 - i0;
        }
        bar_arrive(g);
        bar_wait(g, ++passed, failed);
        // gate / up, SiLU, scattered into down's column order
        SB_MARK(g.trace, ++ph, 0);
        wait_statics();
        {
            ActS a = act_carve(work, g.E);
            stage_x(g, tag_x(g, seq, 2 * l + 1), perm_s, gain_s, a, xk, red, failed);
            SB_MARK(g.trace, ph, 1);
            if (l + 1 < g.n_layer) load_statics(g.L[l + 1].qkv.perm, g.E, g.L[l + 1].an);
            else load_statics(g.head.perm, g.E, g.out_norm);
            cta_range(y.gu.ntiles, i0, i1);
            mk_tiles<GM_FFN, NB, SIX>(g, y.gu, i0, i1, k, a, ring, full, empty, ioff, nullptr, nullptr, g.hp, tl, y.dn_iperm,
                                      failed, best_v, best_i, ph);
            k += i1 - i0;
        }
        bar_arrive(g);
        bar_wait(g, ++passed, failed);
        // down (residual), input already in its column order
        SB_MARK(g.trace, ++ph, 0);
        {
            ActS a = act_carve(work, g.F);
            stage_hp(g, tl, a, failed);
            SB_MARK(g.trace, ph, 1);
            cta_range(y.dn.ntiles, i0, i1);
            mk_tiles<GM_DOWN, NB, SIX>(g, y.dn, i0, i1, k, a, ring, full, empty, ioff, nullptr, xk, g.x, tag_x(g, seq, 2 * l + 2), nullptr,
                                       failed, best_v, best_i, ph);
            k += i1 - i0;
        }
        bar_arrive(g);
        bar_wait(g, ++passed, failed);
    }
    // head: logits and this CTA's argmax
    SB_MARK(g.trace, ++ph, 0);
    wait_statics();
    {
        ActS a = act_carve(work, g.E);
        stage_x(g, tag_x(g, seq, 2 * g.n_layer), perm_s, gain_s, a, xk, red, failed);
        SB_MARK(g.trace, ph, 1);
        int i0, i1;
        cta_range(g.head.ntiles, i0, i1);
        mk_tiles<GM_HEAD, NB, SIX>(g, g.head, i0, i1, k, a, ring, full, empty, ioff, nullptr, nullptr, nullptr, 0u, nullptr,
                                   failed, best_v, best_i, ph);
    }
    SB_MARK(g.trace, ph, 4);
    // greedy argmax, ties to the lower index (sml/sml-run.c:3539-3544); the
    // last CTA to finish writes the token and resets the counters
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best_v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, best_i, o);
        if (ov > best_v || (ov == best_v && oi < best_i)) { best_v = ov; best_i = oi; }
    }
    if (lane == 0) { am_v[warp] = best_v; am_i[warp] = best_i; }
    bar_sync(1, kConsThreads);
    if (threadIdx.x == 0) {
        float bv = am_v[0];
        int bi = am_i[0];
        for (int w = 1; w < kConsWarps; w++)
            if (am_v[w] > bv || (am_v[w] == bv && am_i[w] < bi)) { bv = am_v[w]; bi = am_i[w]; }
        g.am_val[blockIdx.x] = bv;
        g.am_idx[blockIdx.x] = bi;
        __threadfence();
        if (atomicAdd(g.am_cnt, 1u) == (unsigned) G - 1) {
            __threadfence();
            float fv = -INFINITY;
            int fi = 0x7fffffff;
            for (int b = 0; b < G; b++) {
                const float v2 = ((volatile float *) g.am_val)[b];
                const int ix = ((volatile int *) g.am_idx)[b];
                if (v2 > fv || (v2 == fv && ix < fi)) { fv = v2; fi = ix; }
            }
            *g.am_cnt = 0;
            *g.bar = 0;   // every CTA has passed its last barrier
            *g.seq = seq + 1;
            if (g.tlog) g.tlog[pos] = fi;
            *g.tok = fi;
            *g.pos = pos + 1;
        }
    }
    SB_MARK(g.trace, ph, 5);
}

}  // namespace sb
