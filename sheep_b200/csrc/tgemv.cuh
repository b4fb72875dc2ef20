// Streaming quantized GEMV over tile-major weights (tiles.h).
//
// One CTA per SM takes a contiguous range of tiles (TR whole rows each). A
// producer warp streams them into a ring of shared-memory stages with
// cp.async.bulk and mbarrier transaction counts -- it starts before the kernel
// waits on its predecessor, since weights never depend on it. Lane j of the
// producer owns stage j and issues its tiles, so the copies of a ring's worth
// of tiles leave in one warp instruction. Sixteen consumer warps stage the
// int8 activation (the mode's prologue: RMSNorm, gather, per-32
// quantization), then take whole tiles round-robin (tile k to warp k % 16):
// lane l owns row l % TR and every (32/TR)-th unit of it, so a lane's units are
// independent work and the warp reduces once per tile. Tile k lands in stage
// k % ns. mbarrier.try_wait.parity reports a phase done whenever the barrier's
// parity differs, so no waiter may run a phase ahead: with ns a multiple of 16
// a stage always has the same consumer warp, which takes it in order; a ring of
// 8 stages (wide tiles) has each waiter first see the stage's previous lap
// consumed (ring_wait).
//
// Arithmetic: the reference's, in the reference's float order (tile_exact
// below). Each group's dot is exact in integers (dp4a) whatever lanes compute
// it; the float epilogue then runs as the reference's vector kernels run it --
// eight accumulator chains per row (chain L takes groups 8k+L in k order, two
// fused multiply-adds per group) and their fixed horizontal sum, or the
// ladder's four chains, or the bit plane's single chain -- so a row's result
// equals the reference build's bit for bit (sml/sml-kernel.c:298-370,
// :572-718, :836-1005, :1036-1063).
#pragma once

#include "decode.cuh"
#include "tiles.h"

namespace sb {

constexpr int kConsWarps = 16;
constexpr int kConsThreads = kConsWarps * 32;
constexpr int kTgThreads = kConsThreads + 32;   // + one producer warp
constexpr int kMaxStages = 32;
// Dynamic shared memory a GEMV may use (the device allows 227 KB per block,
// less this file's static arrays).
constexpr size_t kSmemBudget = 225 * 1024;

// Tensor-parallel exchange of one GEMV: rows written into every peer's copy
// of the output buffer, then every CTA adds one to a counter per source rank
// in every peer (a system-scope release after a block barrier); and, before
// staging, a wait until each peer's counter has reached the count its event
// completes. The counters only grow: a token's raising kernels add c_tok in
// all (their CTA counts, summed on the host), so event e of the current token
// is complete at (tokens before it) * c_tok + the count up to e.
constexpr int kMaxTp = 8;
// Most groups of 32 hidden values one gate/up CTA quantizes for the down GEMV
// (their floats are kept in the column-order region of its shared memory, free
// once the input is staged: the input has at least this many values).
constexpr int kHqMaxGroups = 8;
struct TpX {
    int n, rank;                       // ranks; this one
    float * peer_out[kMaxTp];          // the output pointer as each peer maps it (NULL for this rank)
    unsigned * peer_cnt[kMaxTp];       // counter [rank] in each peer's counter array (NULL for this rank)
    const unsigned * cnt;              // this rank's counter array [n]: CTAs arrived per source rank
    const unsigned * tok_seq;          // tokens run so far, this one included (the embedding kernel counts)
    unsigned c_tok;                    // arrivals per token per source
    unsigned wait_count;               // arrivals, within a token, that complete the awaited event (0: none)
    int raise;                         // this kernel's CTAs arrive at the peers
    int * err;
};

// Wait, as one thread, until every peer's arrivals complete the awaited
// event (bounded: 2 s of the global timer, then an error code and on).
SB_DEV void tp_wait(const TpX & x) {
    if (x.n <= 1 || !x.wait_count) return;
    const unsigned want = (*x.tok_seq - 1u) * x.c_tok + x.wait_count;
    for (int p = 0; p < x.n; p++) {
        if (p == x.rank) continue;
        const unsigned * f = x.cnt + p;
        unsigned v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if ((int) (v - want) >= 0) continue;
        const unsigned long long t0 = global_ns();
        for (;;) {
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if ((int) (v - want) >= 0) break;
            if (global_ns() - t0 > kWaitNs) { if (x.err) atomicExch(x.err, 7); break; }
        }
    }
}

// After every thread of the CTA has stored its rows everywhere and passed a
// block barrier: one thread adds this CTA's arrival in every peer (release at
// system scope: the CTA's stores, ordered before it by the barrier, are seen
// before the count).
SB_DEV void tp_arrive(const TpX & x) {
    if (x.n <= 1 || !x.raise) return;
    for (int p = 0; p < x.n; p++)
        if (x.peer_cnt[p]) asm volatile("red.release.sys.global.add.u32 [%0], 1;" :: "l"(x.peer_cnt[p]) : "memory");
}

struct TGArgs {
    TT t;
    const float * in;        // input activation
    const float * norm_w;    // RMSNorm gain, NULL: none
    float eps;
    int in_permuted;         // `in` already in t.perm order
    const float * bias;      // per logical row (QKV: q|k|v concatenated); FFN: [gate bias | up bias]
    int ffn_f;               // FFN: hidden values this launch computes (rows / 2)
    int mode;                // GemvMode: the epilogue (one kernel serves every mode, so
                             // consecutive GEMVs of a token run the same code)
    int ffn_n;               // FFN: size of the output (the whole hidden vector; > ffn_f on a tensor-parallel rank)
    float * out;
    const int32_t * scatter; // FFN: write index of hidden value i
    float * am_val; int * am_idx; unsigned * am_cnt;
    int * tok; int * pos; int * tlog;
    int nstage;              // ring stages: a multiple of 16, or 8
    int x_smem;              // gathered input copied into shared memory first (else gathered from L2)
    int prefetch;            // L2 prefetch of this CTA's tiles before the wait
    int8_t * act_q; float * act_s; int32_t * act_sum;   // optional export (CTA 0)
    int * err;               // set if a bounded wait gave up
    unsigned long long * trace;   // trace build: per-CTA timestamps
    int launch_id;
    // The gate/up GEMV quantizing the hidden vector for the down GEMV: with
    // grp_tiles > 0 each CTA takes whole groups of 32 hidden values (tiles in
    // down's column order, grp_tiles tiles a group), keeps its values in shared
    // memory (the gathered input's column-order region) and writes their int8
    // codes, scales and scale * sums into hq in the
    // activation's shared-memory layout (ActS: codes in the slot order, then
    // xs[ng], then xsum[ng]). The down GEMV given in_act copies that block into
    // its shared memory with one bulk copy instead of reading the floats and
    // quantizing them after its wait. The codes are quant_lanes' own.
    int grp_tiles;
    uint8_t * hq;
    const uint8_t * in_act;
    // the next GEMV's tiles: this CTA prefetches the range its own index will
    // take there into L2, so the next kernel's bulk copies hit L2
    const uint8_t * next_tiles;
    int next_ntiles, next_grid;
    uint32_t next_tb;
    TpX tp;                  // tensor-parallel exchange (tp.n > 1)
};

// Shared memory: [act | perm | norm gain | input x | group dots | ring]. perm
// and the gain are static, so the producer bulk-loads them before the
// dependency wait; the input is read once, coalesced, after it (when it fits;
// wide inputs are gathered from L2 instead). The group dots are each consumer
// warp's scratch for the integer dots of its current tile (tile_exact).
struct StageLayout {
    uint32_t perm_off, w_off, x_off, d_off, ring_off;
};

// Integer dot arrays a width's epilogue needs per group: the main code, the
// bit plane (Q3, Q5, Q7: its own chain), the 2-bit plane of Q6/Q7 kept apart
// for rows whose groups are not whole 8-group blocks.
__host__ __device__ constexpr int dot_arrays(int nb) { return nb == 3 || nb == 5 || nb == 6 ? 2 : nb == 7 ? 3 : 1; }

// Bytes of every consumer warp's dot scratch for tiles of t.
__host__ __device__ inline uint32_t tg_dot_bytes(const TT & t) {
    if (t.nbits == 4) return 0u;   // tile_q4 keeps its dots in registers
    return (uint32_t) kConsWarps * dot_arrays(t.nbits) * t.TR * (t.cols / kGroup) * 4u;
}

__host__ __device__ inline StageLayout stage_layout(int n, int has_perm, int has_norm, int has_x, uint32_t dbytes) {
    StageLayout L;
    uint32_t off = (uint32_t) ((act_smem_bytes(n) + 127) / 128 * 128);
    L.perm_off = off;
    if (has_perm) off += (uint32_t) n * 4;
    L.w_off = off;
    if (has_norm) off += (uint32_t) n * 4;
    L.x_off = off;
    if (has_perm && has_x) off += (uint32_t) n * 4;
    L.d_off = (off + 15) / 16 * 16;
    off = L.d_off + dbytes;
    L.ring_off = (off + 127) / 128 * 128;
    return L;
}
__host__ __device__ inline size_t tg_ring_off(const TT & t, int in_permuted, int has_norm, int x_smem) {
    return stage_layout(t.cols, !in_permuted, has_norm, x_smem, tg_dot_bytes(t)).ring_off;
}

// Ring stages for tiles of tb bytes behind ring_off bytes of staging: the
// multiple of 16 nearest ~96 KB (16..32) when 16 fit the budget, else 8 if
// they fit; 0 otherwise. (Fewer than 8 would put four or more warps on one
// stage, where a parity wait can no longer tell its lap from an older one.)
__host__ __device__ inline int ring_stages(size_t ring_off, uint32_t tb) {
    if (ring_off >= kSmemBudget) return 0;
    const size_t fit = (kSmemBudget - ring_off) / tb;
    int ns = (int) ((96 * 1024) / tb) / kConsWarps * kConsWarps;
    ns = ns < kConsWarps ? kConsWarps : ns > kMaxStages ? kMaxStages : ns;
    while (ns > kConsWarps && (size_t) ns > fit) ns -= kConsWarps;
    if ((size_t) ns <= fit) return ns;
    return fit >= 8 ? 8 : 0;
}

// Staging layout and ring depth of one GEMV launch: the input copied into
// shared memory with a ring of at least 16 stages if that fits the budget,
// else gathered from L2 with 16 or 8 stages. False if not even 8 fit.
__host__ inline bool tg_plan(TGArgs & g) {
    const int hn = g.norm_w != nullptr;
    if (g.in_permuted) {
        g.x_smem = 0;
        g.nstage = ring_stages(tg_ring_off(g.t, 1, hn, 0), g.t.tb);
        return g.nstage > 0;
    }
    const int ns = ring_stages(tg_ring_off(g.t, 0, hn, 1), g.t.tb);
    if (ns >= kConsWarps) { g.x_smem = 1; g.nstage = ns; return true; }
    g.x_smem = 0;
    g.nstage = ring_stages(tg_ring_off(g.t, 0, hn, 0), g.t.tb);
    return g.nstage > 0;
}
__host__ inline size_t tg_smem(const TGArgs & g) {
    return tg_ring_off(g.t, g.in_permuted, g.norm_w != nullptr, g.x_smem) + (size_t) g.nstage * g.t.tb;
}

// Wait for tile k of the ring (stage k % ns, lap k / ns) as consumer warp
// k % 16. try_wait.parity reports a phase done whenever the barrier's parity
// differs from the one asked for, so the barrier must be at most one phase
// from the waiter's. With ns a multiple of 16 the stage's previous lap was this
// warp's own, so that holds. With ns = 8 two warps alternate on a stage: the
// waiter first sees the previous lap consumed (empty barrier: at most one
// phase behind, since its own lap before that is done), which puts the full
// barrier at this lap or just past it.
SB_DEV bool ring_wait(uint64_t * full, uint64_t * empty, int k, int ns, int * err) {
    const int s = k % ns, lap = k / ns;
    if (ns < kConsWarps && lap > 0 && !mbar_wait(&empty[s], (lap - 1) & 1, err, 2)) return false;
    return mbar_wait(&full[s], lap & 1, err, 2);
}

// Quantize groups of 32 with 8 lanes per group, 4 values per lane (4 groups
// per warp at a time): amax and sum by 3 shuffles inside the 8-lane team,
// s = amax/127, is = 1/s (0 if s = 0), q = clamp(rint(v*is), +-127) with IEEE
// division and round-to-nearest-even (sml/sml-kernel.c:89-109). The team's 32
// codes land as four 4-byte stores in the slot layout. Every lane of the warp
// runs the shuffles; `store` is false for a team past the last group.
SB_DEV void quant_team(float4 v, int grp, int sub, ActS & a, const TGArgs & g, bool ex, bool store) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 4; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = __fdiv_rn(amax, 127.0f);
    const float is = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    const float vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t word = 0;
    int sum = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) {
        int q = __float2int_rn(__fmul_rn(vv[b], is));
        q = q > 127 ? 127 : q < -127 ? -127 : q;
        sum += q;
        word |= ((uint32_t) (q & 0xff)) << (8 * b);
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (!store) return;
    *reinterpret_cast<uint32_t *>(a.q + act_slot_off(a.n, grp, 4 * sub)) = word;
    if (sub == 0) {
        a.xs[grp] = sc;
        a.xsum[grp] = sc * (float) sum;
    }
    if (ex) {
        *reinterpret_cast<uint32_t *>(g.act_q + grp * kGroup + 4 * sub) = word;
        if (sub == 0) { g.act_s[grp] = sc; g.act_sum[grp] = sum; }
    }
}

// quant_team with LPG lanes per group (4, 2 or 1), 32/LPG values per lane (v[k]
// holds the group's values (32/LPG)*sub + 4k .. +3): fewer shuffles and
// divisions per group than 8 lanes of 4. amax and the integer sum are exact
// whatever the lane split, so the codes, scale and sum are quant_team's (the
// reciprocal by __frcp_rn is the same IEEE value as 1.0f/s). A lane's codes
// land as 8-byte stores in the slot layout (8 consecutive values share one
// 16-byte slot row).
template <int LPG>
SB_DEV void quant_lanes(const float4 (&v)[8 / LPG], int grp, int sub, ActS & a, const TGArgs & g, bool ex, bool store) {
    constexpr int NV = 8 / LPG;   // float4s per lane
    float amax = 0.0f;
#pragma unroll
    for (int k = 0; k < NV; k++)
        amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v[k].x), fabsf(v[k].y)), fmaxf(fabsf(v[k].z), fabsf(v[k].w))));
#pragma unroll
    for (int o = LPG / 2; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = __fdiv_rn(amax, 127.0f);
    const float is = sc > 0.0f ? __frcp_rn(sc) : 0.0f;
    uint32_t w[NV];
    int sum = 0;
#pragma unroll
    for (int k = 0; k < NV; k++) {
        const float vv[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
        w[k] = 0u;
#pragma unroll
        for (int b = 0; b < 4; b++) {
            int q = __float2int_rn(__fmul_rn(vv[b], is));
            q = q > 127 ? 127 : q < -127 ? -127 : q;
            sum += q;
            w[k] |= ((uint32_t) (q & 0xff)) << (8 * b);
        }
    }
#pragma unroll
    for (int o = LPG / 2; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (!store) return;
#pragma unroll
    for (int k = 0; k < NV; k += 2)
        *reinterpret_cast<uint2 *>(a.q + act_slot_off(a.n, grp, 4 * NV * sub + 4 * k)) = make_uint2(w[k], w[k + 1]);
    if (sub == 0) {
        a.xs[grp] = sc;
        a.xsum[grp] = sc * (float) sum;
    }
    if (ex) {
        uint32_t * d = reinterpret_cast<uint32_t *>(g.act_q + grp * kGroup + 4 * NV * sub);
#pragma unroll
        for (int k = 0; k < NV; k++) d[k] = w[k];
        if (sub == 0) { g.act_s[grp] = sc; g.act_sum[grp] = sum; }
    }
}

// Quantize a team's 4 values of group grp into a (no export).
SB_DEV void quant_team_to(float4 v, int grp, int sub, ActS & a, bool store) {
    float amax = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
#pragma unroll
    for (int o = 4; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = __fdiv_rn(amax, 127.0f);
    const float is = sc > 0.0f ? __fdiv_rn(1.0f, sc) : 0.0f;
    const float vv[4] = {v.x, v.y, v.z, v.w};
    uint32_t word = 0;
    int sum = 0;
#pragma unroll
    for (int b = 0; b < 4; b++) {
        int q = __float2int_rn(__fmul_rn(vv[b], is));
        q = q > 127 ? 127 : q < -127 ? -127 : q;
        sum += q;
        word |= ((uint32_t) (q & 0xff)) << (8 * b);
    }
#pragma unroll
    for (int o = 4; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (!store) return;
    *reinterpret_cast<uint32_t *>(a.q + act_slot_off(a.n, grp, 4 * sub)) = word;
    if (sub == 0) {
        a.xs[grp] = sc;
        a.xsum[grp] = sc * (float) sum;
    }
}

// Stage the activation with the consumer threads only (named barrier 1).
// Gathered input: x is read into shared memory once, coalesced; the RMSNorm
// factor comes from a block reduction over it (sum in double, as
// sml/sml-run.c:147-152); teams of 8 lanes then quantize groups, reading
// x[perm[i]] and the gain from shared memory (both bulk-loaded by the producer
// before the wait; `statics` completes when they land). Pre-permuted input:
// one lane per group, reading its 32 values with eight 16-byte loads.
SB_DEV void tg_stage(const TGArgs & g, ActS & a, double * red, uint8_t * smem, const StageLayout & L,
                     uint64_t * statics, bool & failed) {
    const int n = g.t.cols, ng = n / kGroup, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int team = tid >> 3, sub = tid & 7, nteam = kConsThreads / 8;
    const bool ex = g.act_q && blockIdx.x == 0;
    if (g.in_permuted) {
        // every round's load issued before any group is quantized; one lane
        // per group, 128 bytes each
        constexpr int kLpg = 1, kNv = 8 / kLpg, kR = 1;   // rounds held in registers: n <= nlg * 32
        const int lg = tid / kLpg, ls = tid % kLpg, nlg = kConsThreads / kLpg;   // lane group, lane in it
        float4 v[kR][kNv];
#pragma unroll
        for (int r = 0; r < kR; r++) {
            const int grp = r * nlg + lg;
#pragma unroll
            for (int k = 0; k < kNv; k++)
                v[r][k] = grp < ng ? reinterpret_cast<const float4 *>(g.in + grp * kGroup + 4 * kNv * ls)[k]
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        SB_MARK(g.trace, g.launch_id, 5);   // thread 0's loads are issued
#pragma unroll
        for (int r = 0; r < kR; r++) {
            const int grp = r * nlg + lg;
            if (r * nlg < ng) quant_lanes<kLpg>(v[r], grp, ls, a, g, ex, grp < ng);
        }
        for (int base = kR * nlg; base < ng; base += nlg) {
            const int grp = base + lg;
            float4 w4[kNv];
#pragma unroll
            for (int k = 0; k < kNv; k++)
                w4[k] = grp < ng ? reinterpret_cast<const float4 *>(g.in + grp * kGroup + 4 * kNv * ls)[k]
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            quant_lanes<kLpg>(w4, grp, ls, a, g, ex, grp < ng);
        }
        bar_sync(1, kConsThreads);
        return;
    }
    float * xs = reinterpret_cast<float *>(smem + L.x_off);
    const float * xg = g.x_smem ? xs : g.in;   // where the gather reads x
    const int32_t * perm = reinterpret_cast<const int32_t *>(smem + L.perm_off);
    const float * gw = reinterpret_cast<const float *>(smem + L.w_off);
    double q = 0.0;
    if (g.x_smem || g.norm_w)
        for (int i = 4 * tid; i < n; i += 4 * kConsThreads) {
            const float4 f = *reinterpret_cast<const float4 *>(g.in + i);
            if (g.x_smem) *reinterpret_cast<float4 *>(xs + i) = f;
            q += (double) f.x * f.x + (double) f.y * f.y + (double) f.z * f.z + (double) f.w * f.w;
        }
    float s = 1.0f;
    if (g.norm_w) {
        q = warp_sum_d(q);
        if (lane == 0) red[w] = q;
    }
    SB_MARK(g.trace, g.launch_id, 5);   // thread 0's share of x is in
    bar_sync(1, kConsThreads);
    if (g.norm_w) {
        double ss = 0.0;
        for (int k = 0; k < kConsWarps; k++) ss += red[k];
        s = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float) (ss / n), g.eps)));
    }
    if (!failed && !mbar_wait(statics, 0, g.err, 4)) failed = true;
    if (!failed) {
        for (int base = 0; base < ng; base += nteam) {
            const int grp = base + team;
            const int gg = grp < ng ? grp : 0;   // a team past the end reads group 0 and stores nothing
            const int4 p4 = *reinterpret_cast<const int4 *>(perm + gg * kGroup + 4 * sub);
            const int pi[4] = {p4.x, p4.y, p4.z, p4.w};
            float vv[4];
#pragma unroll
            for (int k = 0; k < 4; k++)
                vv[k] = g.norm_w ? __fmul_rn(__fmul_rn(xg[pi[k]], s), gw[pi[k]]) : xg[pi[k]];
            quant_team(make_float4(vv[0], vv[1], vv[2], vv[3]), grp, sub, a, g, ex, grp < ng);
        }
    }
    bar_sync(1, kConsThreads);
}

// Integer dots of unit u of tile row j against the unit's activation slots.
template <int NB>
SB_DEV void tile_dots(const uint8_t * tile, const TileGeom & tg, int j, int u, const uint4 (&a)[4], int (&d)[4]) {
    int kinds[3], shifts[3];
    plane_kinds(NB, kinds, shifts);
    d[0] = d[1] = d[2] = d[3] = 0;
    const int at = u * tg.TR + j;
#pragma unroll
    for (int p = 0; p < 3; p++) {
        if (!kinds[p]) break;
        const uint8_t * sec = tile + tg.pl_off[p];
        const int sh = shifts[p];
        if (kinds[p] == 4) {
            const uint4 w0 = *reinterpret_cast<const uint4 *>(sec + 16 * at);
            const uint4 w1 = *reinterpret_cast<const uint4 *>(sec + tg.pl_sec[p] + 16 * at);
            const uint32_t x0[4] = {w0.x, w0.y, w0.z, w0.w}, x1[4] = {w1.x, w1.y, w1.z, w1.w};
            const uint32_t a0[4] = {a[0].x, a[0].y, a[0].z, a[0].w}, a1[4] = {a[1].x, a[1].y, a[1].z, a[1].w};
            const uint32_t a2[4] = {a[2].x, a[2].y, a[2].z, a[2].w}, a3[4] = {a[3].x, a[3].y, a[3].z, a[3].w};
            int s0 = 0, s1 = 0, s2 = 0, s3 = 0;
#pragma unroll
            for (int w = 0; w < 4; w++) {
                s0 = __dp4a((int) (x0[w] & 0x0f0f0f0fu), (int) a0[w], s0);
                s1 = __dp4a((int) ((x0[w] >> 4) & 0x0f0f0f0fu), (int) a1[w], s1);
                s2 = __dp4a((int) (x1[w] & 0x0f0f0f0fu), (int) a2[w], s2);
                s3 = __dp4a((int) ((x1[w] >> 4) & 0x0f0f0f0fu), (int) a3[w], s3);
            }
            d[0] += s0 << sh; d[1] += s1 << sh; d[2] += s2 << sh; d[3] += s3 << sh;
        } else if (kinds[p] == 2) {
            const uint4 w = *reinterpret_cast<const uint4 *>(sec + 16 * at);
            const uint32_t x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t ak[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
                int s = 0;
#pragma unroll
                for (int ww = 0; ww < 4; ww++) s = __dp4a((int) ((x[ww] >> (2 * k)) & 0x03030303u), (int) ak[ww], s);
                d[k] += s << sh;
            }
        } else {
            // 8 bytes: the unit's 16 columns of each of its 4 groups, 2 bytes each
            const uint2 w = *reinterpret_cast<const uint2 *>(sec + 8 * at);
            const uint32_t h[4] = {w.x & 0xffffu, w.x >> 16, w.y & 0xffffu, w.y >> 16};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t ak[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
                int s = 0;
#pragma unroll
                for (int ww = 0; ww < 4; ww++) s = __dp4a((int) nib_to_bytes((h[k] >> (4 * ww)) & 15u), (int) ak[ww], s);
                d[k] += s << sh;
            }
        }
    }
}

template <int SIX>
SB_DEV void tile_fields(const uint8_t * f, int (&v)[4]) {
    if (SIX) {
        const uint32_t b0 = f[0], b1 = f[1], b2 = f[2];
        v[0] = (int) (b0 & 63u);
        v[1] = (int) (((b0 >> 6) | (b1 << 2)) & 63u);
        v[2] = (int) (((b1 >> 4) | (b2 << 4)) & 63u);
        v[3] = (int) ((b2 >> 2) & 63u);
    } else {
        const uint32_t w = *reinterpret_cast<const uint32_t *>(f);
        v[0] = (int) (w & 255u); v[1] = (int) ((w >> 8) & 255u);
        v[2] = (int) ((w >> 16) & 255u); v[3] = (int) (w >> 24);
    }
}

// ---------------------------------------------------------------- exact epilogue
//
// tile_exact: the rows of one tile, each as the reference computes it.
//
// Phase A: the warp's lanes take the tile's units (lane l: row l % TR, units
// l / TR + k * (32 / TR), so a warp's reads are consecutive 16-byte words) and
// compute each unit's 4 group dots
// per dot array, exact in integers. The two halves of a group (units 2p and
// 2p+1) sit in lanes l and l ^ TR and are added by one shuffle; the even lane
// stores the 4 full dots into the warp's scratch D[array][row][group].
//
// Phase B: eight lanes per row (up to four rows per pass) run the reference's
// float epilogue over those dots:
//   flat   (matvec_flat4_l8 / il4 / il6 / flat6, sml/sml-kernel.c:572-1005):
//          lane L: acc = fma(d*sq, xs*dot, acc); acc = fma(md*(mq-bias), xs*sum,
//          acc) for groups 8k+L in k order; a 4-group tail in lanes 0-3;
//          then ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)) (+ (t0+t1)+(t2+t3));
//   ladder (sml_matvec_rows :298-370): lanes 0-3, groups 4p+L, the dot times
//          2^shift, sum (a0+a1)+(a2+a3);
//   bits1  (sml_matvec_bits1 :1036-1063): lane 0, every group whose bit word is
//          not zero, tot = fma(d*sq*xs, dot, tot).
// A width's result is y = 0 + its first pass, + later passes, as the
// reference's dispatch adds them into a zeroed y (sml/sml-run.c:612-680, :755).
// The row's value ends in lane 8*(row % 4) of its pass.

// Array of plane p's dot for width NB, and its factor when planes share one.
template <int NB> SB_DEV int plane_arr(int p) {
    switch (NB) {
    case 3: case 5: return p;          // main plane, bit plane
    case 6: return p == 0 ? 1 : 0;     // 2-bit plane apart, nibbles main
    case 7: return p;                  // nibbles, 2-bit, bit
    default: return 0;                 // Q2, Q4: one plane; Q8: lo + 16 hi
    }
}

template <int NB>
SB_DEV void tile_dots_exact(const uint8_t * tile, const TileGeom & tg, const ActS & a, int * D, int ng) {
    constexpr int ND = dot_arrays(NB);
    int kinds[3], shifts[3];
    plane_kinds(NB, kinds, shifts);
    const int lane = threadIdx.x & 31, TR = tg.TR, j = lane % TR, v = lane / TR, VS = 32 / TR;
    const int nit = (tg.U + VS - 1) / VS;
    for (int it = 0; it < nit; it++) {
        const int u = v + it * VS;
        const bool ok = u < tg.U;
        int dd[ND][4];
#pragma unroll
        for (int r = 0; r < ND; r++) dd[r][0] = dd[r][1] = dd[r][2] = dd[r][3] = 0;
        if (ok) {
            uint4 av[4];
#pragma unroll
            for (int k = 0; k < 4; k++) av[k] = *reinterpret_cast<const uint4 *>(a.q + k * (a.n >> 2) + 16 * u);
            const uint32_t a0[4] = {av[0].x, av[0].y, av[0].z, av[0].w}, a1[4] = {av[1].x, av[1].y, av[1].z, av[1].w};
            const uint32_t a2[4] = {av[2].x, av[2].y, av[2].z, av[2].w}, a3[4] = {av[3].x, av[3].y, av[3].z, av[3].w};
            const int at = u * TR + j;
#pragma unroll
            for (int p = 0; p < 3; p++) {
                if (!kinds[p]) break;
                const int r = plane_arr<NB>(p);
                const int f = (NB == 8 && p == 1) ? 4 : 0;   // Q8: hi nibbles x16 into the main dot
                const uint8_t * sec = tile + tg.pl_off[p];
                int s4[4] = {0, 0, 0, 0};
                if (kinds[p] == 4) {
                    const uint4 w0 = *reinterpret_cast<const uint4 *>(sec + 16 * at);
                    const uint4 w1 = *reinterpret_cast<const uint4 *>(sec + tg.pl_sec[p] + 16 * at);
                    const uint32_t x0[4] = {w0.x, w0.y, w0.z, w0.w}, x1[4] = {w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                    for (int w = 0; w < 4; w++) {
                        s4[0] = __dp4a((int) (x0[w] & 0x0f0f0f0fu), (int) a0[w], s4[0]);
                        s4[1] = __dp4a((int) ((x0[w] >> 4) & 0x0f0f0f0fu), (int) a1[w], s4[1]);
                        s4[2] = __dp4a((int) (x1[w] & 0x0f0f0f0fu), (int) a2[w], s4[2]);
                        s4[3] = __dp4a((int) ((x1[w] >> 4) & 0x0f0f0f0fu), (int) a3[w], s4[3]);
                    }
                } else if (kinds[p] == 2) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(sec + 16 * at);
                    const uint32_t x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int ww = 0; ww < 4; ww++) {
                        s4[0] = __dp4a((int) (x[ww] & 0x03030303u), (int) a0[ww], s4[0]);
                        s4[1] = __dp4a((int) ((x[ww] >> 2) & 0x03030303u), (int) a1[ww], s4[1]);
                        s4[2] = __dp4a((int) ((x[ww] >> 4) & 0x03030303u), (int) a2[ww], s4[2]);
                        s4[3] = __dp4a((int) ((x[ww] >> 6) & 0x03030303u), (int) a3[ww], s4[3]);
                    }
                } else {
                    const uint2 w = *reinterpret_cast<const uint2 *>(sec + 8 * at);
                    const uint32_t h[4] = {w.x & 0xffffu, w.x >> 16, w.y & 0xffffu, w.y >> 16};
                    const uint32_t * ak[4] = {a0, a1, a2, a3};
#pragma unroll
                    for (int k = 0; k < 4; k++)
#pragma unroll
                        for (int ww = 0; ww < 4; ww++)
                            s4[k] = __dp4a((int) nib_to_bytes((h[k] >> (4 * ww)) & 15u), (int) ak[k][ww], s4[k]);
                }
#pragma unroll
                for (int k = 0; k < 4; k++) dd[r][k] += s4[k] << f;
            }
        }
#pragma unroll
        for (int r = 0; r < ND; r++)
#pragma unroll
            for (int k = 0; k < 4; k++) dd[r][k] += __shfl_xor_sync(0xffffffffu, dd[r][k], TR);
        if (ok && !(v & 1)) {
#pragma unroll
            for (int r = 0; r < ND; r++)
                *reinterpret_cast<int4 *>(D + (r * TR + j) * ng + 4 * (u >> 1)) =
                    make_int4(dd[r][0], dd[r][1], dd[r][2], dd[r][3]);
        }
    }
}

// Group g's step d*sq and min md*(mq - bias) of tile row j, each a rounded
// product as the reference forms them (sml/sml-kernel.c:655-661).
// Field i (0..3) of a quad's packed step or min fields: a byte each, or 6 bits
// of a 3-byte little-endian word (sml/sml-kernel.h:65-96).
template <int SIX>
SB_DEV float tile_field1(const uint8_t * f, int i) {
    if (SIX) {
        const uint32_t b = (uint32_t) f[0] | ((uint32_t) f[1] << 8) | ((uint32_t) f[2] << 16);
        return (float) ((b >> (6 * i)) & 63u);
    }
    return (float) f[i];
}
template <int SIX>
SB_DEV float tile_step(const uint8_t * tile, const TileGeom & tg, int j, int g) {
    const float sq = tile_field1<SIX>(tile + tg.sq_off + ((g >> 2) * tg.TR + j) * tg.f_w, g & 3);
    return __fmul_rn(h2f(*reinterpret_cast<const uint16_t *>(tile + tg.sd_off + ((g >> 3) * tg.TR + j) * 2)), sq);
}
template <int SIX>
SB_DEV float tile_min(const uint8_t * tile, const TileGeom & tg, int j, int g, float mbias) {
    const float mq = tile_field1<SIX>(tile + tg.mq_off + ((g >> 2) * tg.TR + j) * tg.f_w, g & 3);
    return __fmul_rn(h2f(*reinterpret_cast<const uint16_t *>(tile + tg.md_off + ((g >> 3) * tg.TR + j) * 2)),
                     __fsub_rn(mq, mbias));
}

// dot of group g from arrays (flat: a + 16 b when b != NULL)
SB_DEV int dot_at(const int * da, const int * db, int g) { return db ? da[g] + 16 * db[g] : da[g]; }

// One group's two terms of the flat epilogue: step*(xs*dot) and min, xs*sum.
template <int SIX>
SB_DEV void flat_terms(const uint8_t * tile, const TileGeom & tg, const ActS & a, const int * da, const int * db,
                       int j, int g, bool with_min, float mbias, float & st, float & t1, float & mn, float & xm) {
    st = tile_step<SIX>(tile, tg, j, g);
    t1 = __fmul_rn(a.xs[g], (float) dot_at(da, db, g));
    mn = with_min ? tile_min<SIX>(tile, tg, j, g, mbias) : 0.0f;
    xm = with_min ? a.xsum[g] : 0.0f;
}

template <int SIX>
SB_DEV float chain_flat(const uint8_t * tile, const TileGeom & tg, const ActS & a, const int * da, const int * db,
                        int ng, int j, int L, bool with_min, float mbias) {
    const int nblk = ng >> 3;
    float acc = 0.0f, tac = 0.0f;
    int k = 0;
    // four steps' operands are loaded before their fused multiply-adds
    for (; k + 4 <= nblk; k += 4) {
        float st[4], t1[4], mn[4], xm[4];
#pragma unroll
        for (int u = 0; u < 4; u++) flat_terms<SIX>(tile, tg, a, da, db, j, 8 * (k + u) + L, with_min, mbias, st[u], t1[u], mn[u], xm[u]);
#pragma unroll
        for (int u = 0; u < 4; u++) {
            acc = __fmaf_rn(st[u], t1[u], acc);
            if (with_min) acc = __fmaf_rn(mn[u], xm[u], acc);
        }
    }
    for (; k < nblk; k++) {
        float st, t1, mn, xm;
        flat_terms<SIX>(tile, tg, a, da, db, j, 8 * k + L, with_min, mbias, st, t1, mn, xm);
        acc = __fmaf_rn(st, t1, acc);
        if (with_min) acc = __fmaf_rn(mn, xm, acc);
    }
    const bool tail = (ng & 7) != 0;
    if (tail && L < 4) {
        float st, t1, mn, xm;
        flat_terms<SIX>(tile, tg, a, da, db, j, 8 * nblk + L, with_min, mbias, st, t1, mn, xm);
        tac = __fmaf_rn(st, t1, tac);
        if (with_min) tac = __fmaf_rn(mn, xm, tac);
    }
    const float s = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4, 8));
    const float t = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 1, 8));
    float tot = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 2, 8));
    const float v = __fadd_rn(tac, __shfl_down_sync(0xffffffffu, tac, 1, 8));
    const float tt = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 8));
    if (tail) tot = __fadd_rn(tot, tt);
    return tot;
}

template <int SIX>
SB_DEV float chain_ladder(const uint8_t * tile, const TileGeom & tg, const ActS & a, const int * d, float mul,
                          int ng, int j, int L, bool with_min, float mbias) {
    float acc = 0.0f;
    if (L < 4)
        for (int p = 0; p < (ng >> 2); p++) {
            const int g = 4 * p + L;
            acc = __fmaf_rn(tile_step<SIX>(tile, tg, j, g), __fmul_rn(a.xs[g], __fmul_rn((float) d[g], mul)), acc);
            if (with_min) acc = __fmaf_rn(tile_min<SIX>(tile, tg, j, g, mbias), a.xsum[g], acc);
        }
    const float s = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 1, 8));
    return __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 2, 8));
}

// The bit plane's chain, lane 0 of the row: groups whose 32 bits are not all zero.
template <int SIX>
SB_DEV float chain_bits1(const uint8_t * tile, const TileGeom & tg, const ActS & a, const int * d, int plane,
                         int ng, int j, int L) {
    float tot = 0.0f;
    if (L == 0) {
        const uint8_t * sec = tile + tg.pl_off[plane];
        for (int g = 0; g < ng; g++) {
            const int u0 = 2 * (g >> 2), i = g & 3;
            const uint16_t b0 = *reinterpret_cast<const uint16_t *>(sec + (u0 * tg.TR + j) * 8 + 2 * i);
            const uint16_t b1 = *reinterpret_cast<const uint16_t *>(sec + ((u0 + 1) * tg.TR + j) * 8 + 2 * i);
            if (b0 | b1) tot = __fmaf_rn(__fmul_rn(tile_step<SIX>(tile, tg, j, g), a.xs[g]), (float) d[g], tot);
        }
    }
    return tot;
}

// Rows of one tile: returns row l's value in lane l < TR.
template <int NB, int SIX>
SB_DEV float tile_exact(const uint8_t * tile, const TileGeom & tg, const ActS & a, int * D, bool has_min, float mbias) {
    const int ng = a.n / kGroup, TR = tg.TR, lane = threadIdx.x & 31, jj = lane >> 3, L = lane & 7;
    tile_dots_exact<NB>(tile, tg, a, D, ng);
    __syncwarp();
    float mine = 0.0f;
    for (int r0 = 0; r0 < TR; r0 += 4) {
        const int j = r0 + jj < TR ? r0 + jj : TR - 1;   // lanes past the last row repeat it and are dropped
        const int * d0 = D + j * ng, * d1 = D + (TR + j) * ng, * d2 = D + (2 * TR + j) * ng;
        float y = 0.0f;
        switch (NB) {
        case 2: y = __fadd_rn(0.0f, chain_ladder<SIX>(tile, tg, a, d0, 1.0f, ng, j, L, has_min, mbias)); break;
        case 3: y = __fadd_rn(0.0f, chain_ladder<SIX>(tile, tg, a, d0, 1.0f, ng, j, L, has_min, mbias));
                y = __fadd_rn(y, __fmul_rn(chain_bits1<SIX>(tile, tg, a, d1, 1, ng, j, L), 4.0f)); break;
        case 5: y = __fadd_rn(0.0f, chain_flat<SIX>(tile, tg, a, d0, nullptr, ng, j, L, has_min, mbias));
                y = __fadd_rn(y, __fmul_rn(chain_bits1<SIX>(tile, tg, a, d1, 1, ng, j, L), 16.0f)); break;
        case 6: case 7:
            if ((ng & 7) == 0) {
                y = __fadd_rn(0.0f, chain_flat<SIX>(tile, tg, a, d0, d1, ng, j, L, has_min, mbias));
            } else {
                y = __fadd_rn(0.0f, chain_ladder<SIX>(tile, tg, a, d1, 16.0f, ng, j, L, has_min, mbias));
                y = __fadd_rn(y, chain_flat<SIX>(tile, tg, a, d0, nullptr, ng, j, L, false, mbias));
            }
            if (NB == 7) y = __fadd_rn(y, __fmul_rn(chain_bits1<SIX>(tile, tg, a, d2, 2, ng, j, L), 64.0f));
            break;
        default: y = __fadd_rn(0.0f, chain_flat<SIX>(tile, tg, a, d0, nullptr, ng, j, L, has_min, mbias)); break;
        }
        // row r0 + (lane - r0) takes the value from lane 8 * (lane - r0)
        const int src = lane - r0;
        const float got = __shfl_sync(0xffffffffu, y, (src >= 0 && src < 4 ? src : 0) * 8);
        if (src >= 0 && src < 4) mine = got;
    }
    return mine;
}

// ---------------------------------------------------------------- Q4 rows, one pass
//
// 4-bit tiles in the float order of tile_exact's flat epilogue (eight chains
// per row, chain L over groups 8k + L; the tree ((a0+a4)+(a1+a5))+((a2+a6)+
// (a3+a7)); a 4-group tail), with every group dot computed by the lane that
// uses it: no scratch, no second pass. Group g = 4p + i of row j: piece i/2 of
// units 2p and 2p+1 (groups 4p, 4p+1 in the low and high nibbles of piece 0,
// 4p+2, 4p+3 of piece 1); its 32 activation codes are 32 bytes at array i,
// offset 32p. A high-nibble group's dot is taken on the masked bytes (16x the
// code, unsigned) and shifted back down: exact, since it is a multiple of 16.

// Unsigned code bytes times signed activation bytes, accumulated (PTX dp4a.u32.s32).
SB_DEV int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// The integer dot of group g (= 4p + i) of the row whose unit-2p piece word is
// at pc, against activation words a0, a1.
SB_DEV int q4_dot(const uint8_t * pc, int TR, uint32_t mask, int dsh, const uint4 & a0, const uint4 & a1) {
    const uint4 c0 = *reinterpret_cast<const uint4 *>(pc);
    const uint4 c1 = *reinterpret_cast<const uint4 *>(pc + 16 * TR);
    int d = dp4a_us(c0.x & mask, a0.x, 0);
    d = dp4a_us(c0.y & mask, a0.y, d);
    d = dp4a_us(c0.z & mask, a0.z, d);
    d = dp4a_us(c0.w & mask, a0.w, d);
    d = dp4a_us(c1.x & mask, a1.x, d);
    d = dp4a_us(c1.y & mask, a1.y, d);
    d = dp4a_us(c1.z & mask, a1.z, d);
    d = dp4a_us(c1.w & mask, a1.w, d);
    return d >> dsh;
}

// tile_q4 (TR = 4, 8, 16): lane 4L + r runs chain L of rows r, r+4, ... (TR/4
// rows); a group's activation words are loaded once for them. A quarter warp
// (chains L, L+1 of one piece, four rows) reads four consecutive 16-byte words.
// Row j's value ends in lane j.
template <int SIX, int TR>
SB_DEV float tile_q4(const uint8_t * tile, const TileGeom & tg, const ActS & a, bool has_min, float mbias) {
    constexpr int R = TR / 4;
    const int lane = threadIdx.x & 31, r = lane & 3, L = lane >> 2, i = L & 3;
    const int n = a.n, nblk = (n / kGroup) >> 3;
    const uint32_t mask = (i & 1) ? 0xf0f0f0f0u : 0x0f0f0f0fu;
    const int dsh = (i & 1) ? 4 : 0;
    const uint8_t * pc0 = tile + tg.pl_off[0] + (i >> 1) * tg.pl_sec[0] + 16 * r;
    const int8_t * aq = a.q + i * (n >> 2);
    const uint32_t fw = tg.f_w;
    float acc[R];
#pragma unroll
    for (int m = 0; m < R; m++) acc[m] = 0.0f;
    // one chain step (group g) of every row the lane holds
    auto step = [&](int g, float (&ac)[R]) {
        const int p = g >> 2, k = g >> 3;
        const uint4 a0 = *reinterpret_cast<const uint4 *>(aq + 32 * p);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(aq + 32 * p + 16);
        const float xs = a.xs[g], xm = has_min ? a.xsum[g] : 0.0f;
#pragma unroll
        for (int m = 0; m < R; m++) {
            const int j = r + 4 * m;
            const int d = q4_dot(pc0 + 16 * (2 * p * TR + 4 * m), TR, mask, dsh, a0, a1);
            const float st = __fmul_rn(h2f(*reinterpret_cast<const uint16_t *>(tile + tg.sd_off + (k * TR + j) * 2)),
                                       tile_field1<SIX>(tile + tg.sq_off + (p * TR + j) * fw, i));
            ac[m] = __fmaf_rn(st, __fmul_rn(xs, (float) d), ac[m]);
            if (has_min) {
                const float mn = __fmul_rn(h2f(*reinterpret_cast<const uint16_t *>(tile + tg.md_off + (k * TR + j) * 2)),
                                           __fsub_rn(tile_field1<SIX>(tile + tg.mq_off + (p * TR + j) * fw, i), mbias));
                ac[m] = __fmaf_rn(mn, xm, ac[m]);
            }
        }
    };
    for (int k = 0; k < nblk; k++) step(8 * k + L, acc);
    float tac[R];
#pragma unroll
    for (int m = 0; m < R; m++) tac[m] = 0.0f;
    const bool tail = ((n / kGroup) & 7) != 0;
    if (tail && L < 4) step(8 * nblk + L, tac);
    float mine = 0.0f;
#pragma unroll
    for (int m = 0; m < R; m++) {
        // chain L + 4 is 16 lanes up, L + 1 four, L + 2 eight
        const float s = __fadd_rn(acc[m], __shfl_down_sync(0xffffffffu, acc[m], 16));
        const float t = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 4));
        float tot = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 8));
        const float v = __fadd_rn(tac[m], __shfl_down_sync(0xffffffffu, tac[m], 4));
        const float tt = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 8));
        if (tail) tot = __fadd_rn(tot, tt);
        // row r + 4m sits in lane r
        const float y = __shfl_sync(0xffffffffu, __fadd_rn(0.0f, tot), lane & 3);
        if ((lane >> 2) == m) mine = y;
    }
    return mine;
}

// tile_q4s (TR = 1, 2): a row's chains are short of lanes, so each takes S =
// 4/TR lanes: lane 8*TR*q + 8j + L computes step k0 + q of chain L of row j
// for each chunk of S steps (the next chunk's terms are formed while the
// current one is summed), and the chain's own lane (q = 0) adds the S steps in
// order, their terms fetched by shuffles. A quarter warp (the eight chains of
// one row and step) reads the four words of two pieces and two unit pairs.
// Row j's value ends in lane j.
template <int SIX, int TR>
SB_DEV float tile_q4s(const uint8_t * tile, const TileGeom & tg, const ActS & a, bool has_min, float mbias) {
    constexpr int S = 4 / TR;
    const int lane = threadIdx.x & 31, L = lane & 7, j = (lane >> 3) % TR, q = lane / (8 * TR), i = L & 3;
    const int n = a.n, ng = n / kGroup, nblk = ng >> 3;
    const uint32_t mask = (i & 1) ? 0xf0f0f0f0u : 0x0f0f0f0fu;
    const int dsh = (i & 1) ? 4 : 0;
    const uint8_t * pc0 = tile + tg.pl_off[0] + (i >> 1) * tg.pl_sec[0] + 16 * j;
    const int8_t * aq = a.q + i * (n >> 2);
    const uint32_t fw = tg.f_w;
    // the terms of group g of row j: step, xs * dot, min
    auto terms = [&](int g, float & st, float & t1, float & mn) {
        const int p = g >> 2, k = g >> 3;
        const uint4 a0 = *reinterpret_cast<const uint4 *>(aq + 32 * p);
        const uint4 a1 = *reinterpret_cast<const uint4 *>(aq + 32 * p + 16);
        const int d = q4_dot(pc0 + 16 * (2 * p * TR), TR, mask, dsh, a0, a1);
        st = __fmul_rn(h2f(*reinterpret_cast<const uint16_t *>(tile + tg.sd_off + (k * TR + j) * 2)),
                       tile_field1<SIX>(tile + tg.sq_off + (p * TR + j) * fw, i));
        t1 = __fmul_rn(a.xs[g], (float) d);
        mn = has_min ? __fmul_rn(h2f(*reinterpret_cast<const uint16_t *>(tile + tg.md_off + (k * TR + j) * 2)),
                                 __fsub_rn(tile_field1<SIX>(tile + tg.mq_off + (p * TR + j) * fw, i), mbias))
                     : 0.0f;
    };
    float acc = 0.0f;
    float st = 0.0f, t1 = 0.0f, mn = 0.0f;
    if (q < nblk) terms(8 * q + L, st, t1, mn);
    for (int k0 = 0; k0 < nblk; k0 += S) {
        const float cst = st, ct1 = t1, cmn = mn;
        if (k0 + S + q < nblk) terms(8 * (k0 + S + q) + L, st, t1, mn);
#pragma unroll
        for (int qq = 0; qq < S; qq++) {
            const int src = (lane & (8 * TR - 1)) + 8 * TR * qq;
            const float a_st = __shfl_sync(0xffffffffu, cst, src);
            const float a_t1 = __shfl_sync(0xffffffffu, ct1, src);
            const float a_mn = __shfl_sync(0xffffffffu, cmn, src);
            if (k0 + qq < nblk) {
                acc = __fmaf_rn(a_st, a_t1, acc);
                if (has_min) acc = __fmaf_rn(a_mn, a.xsum[8 * (k0 + qq) + L], acc);
            }
        }
    }
    const float s = __fadd_rn(acc, __shfl_down_sync(0xffffffffu, acc, 4));
    const float t = __fadd_rn(s, __shfl_down_sync(0xffffffffu, s, 1));
    float tot = __fadd_rn(t, __shfl_down_sync(0xffffffffu, t, 2));
    if (ng & 7) {
        float tac = 0.0f;
        if (q == 0 && L < 4) {
            const int g = 8 * nblk + L;
            float a_st, a_t1, a_mn;
            terms(g, a_st, a_t1, a_mn);
            tac = __fmaf_rn(a_st, a_t1, tac);
            if (has_min) tac = __fmaf_rn(a_mn, a.xsum[g], tac);
        }
        const float v = __fadd_rn(tac, __shfl_down_sync(0xffffffffu, tac, 1));
        tot = __fadd_rn(tot, __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2)));
    }
    // row j sits in lane 8j
    return __shfl_sync(0xffffffffu, __fadd_rn(0.0f, tot), 8 * (lane < TR ? lane : 0));
}

// 4-bit tiles take tile_q4 (no dot scratch: tg_dot_bytes is 0 for them);
// every other width tile_exact.
template <int NB, int SIX>
SB_DEV float tile_rows(const uint8_t * tile, const TileGeom & tg, const ActS & a, int * D, bool has_min, float mbias) {
    if constexpr (NB == 4) {
        switch (tg.TR) {
        case 16: return tile_q4<SIX, 16>(tile, tg, a, has_min, mbias);
        case 8: return tile_q4<SIX, 8>(tile, tg, a, has_min, mbias);
        case 4: return tile_q4<SIX, 4>(tile, tg, a, has_min, mbias);
        case 2: return tile_q4s<SIX, 2>(tile, tg, a, has_min, mbias);
        default: return tile_q4s<SIX, 1>(tile, tg, a, has_min, mbias);
        }
    } else {
        return tile_exact<NB, SIX>(tile, tg, a, D, has_min, mbias);
    }
}

template <int NB, int SIX>
// At most 88 registers a thread: a CTA's 17 warps fall 5/4/4/4 on the SM's four
// sub-partitions, and at 88 the busiest keeps room for two warps of the decode
// attention kernel (32 registers), so attention's CTAs start beside the q|k|v
// GEMV and stage their cached rows while it runs (96 registers left no room:
// attention waited for the GEMV's CTAs to leave; measured 1037 -> 1073 tok/s).
__global__ void __maxnreg__(88) k_tgemv(const __grid_constant__ TGArgs g) {
    const int MODE = g.mode;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages], statics, actbar;
    __shared__ double red[kConsWarps];
    __shared__ float am_v[kConsWarps];
    __shared__ int am_i[kConsWarps];
    pdl_launch_dependents();
    SB_MARK(g.trace, g.launch_id, 0);
    const TT & t = g.t;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int T = t.ntiles;
    // whole groups of hidden values per CTA when the gate/up GEMV quantizes for down
    const int gt = g.grp_tiles > 0 ? g.grp_tiles : 1, ngq = T / gt;
    const int t0 = (int) ((long) ngq * blockIdx.x / gridDim.x) * gt;
    const int t1 = (int) ((long) ngq * (blockIdx.x + 1) / gridDim.x) * gt;
    const int ns = g.nstage;
    const StageLayout SL = stage_layout(t.cols, !g.in_permuted, g.norm_w != nullptr, g.x_smem, tg_dot_bytes(t));
    uint8_t * ring = smem + SL.ring_off;
#ifdef SB_CHECKED
    uint32_t dsm;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(dsm));
    const size_t ring_end = dsm;
    if (!SB_CHECK(g.err, (ns == 8 || ns % kConsWarps == 0) && ns <= kMaxStages &&
                           SL.ring_off + (size_t) ns * t.tb <= dsm, 107)) return;
#else
    const size_t ring_end = ~(size_t) 0;
#endif
    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(&statics, 1);
        mbar_init(&actbar, 1);
        mbar_fence_init();
    }
    __syncthreads();

    if (warp == kConsWarps) {
        // ---------------- producer: weights never depend on the previous kernel
        if (lane == 0) {
            // the column order and the norm gain do not depend on the previous kernel
            const uint32_t sb = (g.in_permuted ? 0u : (uint32_t) t.cols * 4) + (g.norm_w ? (uint32_t) t.cols * 4 : 0u);
            mbar_expect_tx(&statics, sb);
            if (!g.in_permuted) bulk_g2s(smem + SL.perm_off, t.perm, (uint32_t) t.cols * 4, &statics);
            if (g.norm_w) bulk_g2s(smem + SL.w_off, g.norm_w, (uint32_t) t.cols * 4, &statics);
        }
        __syncwarp();
        // lane j < ns owns ring stage j and issues its tiles t0 + j, t0 + j + ns, ...:
        // one warp instruction issues the first lap's ns copies, ahead of the
        // L2 prefetches, which the copy engine would otherwise work through first
        const uint32_t tb = t.tb;
        if (lane < ns && t0 + lane < t1) {
            mbar_expect_tx(&full[lane], tb);
            bulk_g2s(ring + (size_t) lane * tb, t.tiles + (size_t) (t0 + lane) * tb, tb, &full[lane]);
        }
        __syncwarp();
        if (lane == 0) {
            // the tiles past the first lap, and the next kernel's share
            if (g.prefetch && t1 > t0 + ns) prefetch_l2(t.tiles + (size_t) (t0 + ns) * tb, (size_t) (t1 - t0 - ns) * tb);
            if (g.next_tiles && (int) blockIdx.x < g.next_grid) {
                const int n0 = (int) ((long) g.next_ntiles * blockIdx.x / g.next_grid);
                const int n1 = (int) ((long) g.next_ntiles * (blockIdx.x + 1) / g.next_grid);
                if (n1 > n0) prefetch_l2(g.next_tiles + (size_t) n0 * g.next_tb, (size_t) (n1 - n0) * g.next_tb);
            }
#ifdef SB_TRACE
            if (g.trace && blockIdx.x < kTraceCtas) g.trace[((size_t) g.launch_id * kTraceCtas + blockIdx.x) * 8 + 6] = global_ns();
#endif
        }
        __syncwarp();
        if (lane < ns) {
            const int s = lane;
            int lap = t0 + s < t1 ? 1 : 0;
            for (int i = t0 + s + ns; i < t1; i += ns, lap++) {
                if (!mbar_wait(&empty[s], (lap - 1) & 1, g.err, 1)) break;
                mbar_expect_tx(&full[s], tb);
                bulk_g2s(ring + (size_t) s * tb, t.tiles + (size_t) i * tb, tb, &full[s]);
            }
            // no copy may still be landing in shared memory when the CTA exits
            if (lap > 0) mbar_wait(&full[s], (lap - 1) & 1, g.err, 3);
        }
        __syncwarp();
        if (lane == 0) {
#ifdef SB_TRACE
            if (g.trace && blockIdx.x < kTraceCtas) g.trace[((size_t) g.launch_id * kTraceCtas + blockIdx.x) * 8 + 7] = global_ns();
#endif
            mbar_wait(&statics, 0, g.err, 5);
        }
        pdl_wait();
        return;
    }

    // ---------------- consumers
    // static epilogue data of the warp's first tile (the hidden vector's order,
    // the q|k|v and gate/up biases: uploaded weights, which no kernel writes)
    // is read before the dependency wait, so the tile's epilogue waits on no load
    int sc0 = 0;
    float gb0 = 0.0f, ub0 = 0.0f;
    if (MODE == GM_FFN) {
        const int idx = (t0 + warp) * (t.TR / 2) + lane;
        if (t0 + warp < t1 && lane < t.TR / 2 && idx < g.ffn_f) {
            sc0 = g.scatter[idx];
            if (g.bias) { gb0 = g.bias[idx]; ub0 = g.bias[g.ffn_f + idx]; }
        }
    } else if (MODE == GM_QKV) {
        const int r = (t0 + warp) * t.TR + lane;
        if (g.bias && t0 + warp < t1 && lane < t.TR && r < t.rows) gb0 = g.bias[r];
    }
    pdl_wait();
    SB_MARK(g.trace, g.launch_id, 1);
    // o / down add into the residual stream: the rows of the warp's first tile
    // are read now, so that add waits on no L2 round trip after the tile (each
    // row is this warp's alone; earlier kernels' writes are visible past the wait)
    float res0 = 0.0f;
    if (MODE == GM_O || MODE == GM_DOWN) {
        const int r = (t0 + warp) * t.TR + lane;
        if (t0 + warp < t1 && lane < t.TR && r < t.rows) res0 = g.out[r];
    }
    ActS a = act_carve(smem, t.cols);
    bool failed = false;   // after one wait gives up, the rest are skipped
    if (g.tp.n > 1 && g.tp.wait_count) {
        // the input's other rows come from the peers: wait for their event
        if (threadIdx.x == 0) tp_wait(g.tp);
        bar_sync(1, kConsThreads);
    }
    if (g.in_act) {
        // the input already quantized by the gate/up GEMV, in this layout: one copy
        const uint32_t ab = (uint32_t) t.cols + (uint32_t) (t.cols / kGroup) * 8u;
        if (threadIdx.x == 0) {
            mbar_expect_tx(&actbar, ab);
            bulk_g2s(smem, g.in_act, ab, &actbar);
        }
        if (!failed && !mbar_wait(&actbar, 0, g.err, 9)) failed = true;
    } else {
        tg_stage(g, a, red, smem, SL, &statics, failed);
    }
    SB_MARK(g.trace, g.launch_id, 2);
    const TileGeom tg = tile_geom(t.cols, t.TR, NB, SIX, t.has_min);
    const int TR = t.TR;
    // this warp's scratch for the group dots of its current tile
    int * D = reinterpret_cast<int *>(smem + SL.d_off) + (size_t) warp * (tg_dot_bytes(t) / kConsWarps / 4);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    for (int i = t0 + warp; i < t1; i += kConsWarps) {
        const int k = i - t0, s = k % ns;
        // one verdict for the warp: the tile's lanes meet in shuffles
        const bool ok = __all_sync(0xffffffffu, !failed && ring_wait(full, empty, k, ns, g.err));
        failed = !ok;
        if (k == 0) SB_MARK(g.trace, g.launch_id, 3);
        float acc = 0.0f;
        if (ok && SB_CHECK(g.err, tg.bytes == t.tb && (size_t) (s + 1) * t.tb + SL.ring_off <= ring_end, 106))
            acc = tile_rows<NB, SIX>(ring + (size_t) s * t.tb, tg, a, D, t.has_min, t.mbias);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (MODE == GM_FFN) {
            // rows 0..TR/2-1 of the tile are gate rows, TR/2..TR-1 the matching up rows
            const float up = __shfl_down_sync(0xffffffffu, acc, TR / 2);
            const int idx = i * (TR / 2) + lane;
            if (lane < TR / 2 && idx < g.ffn_f) {
                const bool first = k < kConsWarps;
                float gv = acc, uv = up;
                if (g.bias) {
                    gv = __fadd_rn(gv, first ? gb0 : g.bias[idx]);
                    uv = __fadd_rn(uv, first ? ub0 : g.bias[g.ffn_f + idx]);
                }
                const int sc = first ? sc0 : g.scatter[idx];
                if (SB_CHECK(g.err, sc >= 0 && sc < g.ffn_n, 108)) {
                    const float h = silu_mul(gv, uv);
                    g.out[sc] = h;
                    // the CTA's groups hold hidden positions [t0 TR/2, t1 TR/2)
                    // (kept where the column order lay: staging is over)
                    if (g.grp_tiles && SB_CHECK(g.err, !g.in_permuted && sc >= t0 * (TR / 2) && sc < t1 * (TR / 2), 109))
                        reinterpret_cast<float *>(smem + SL.perm_off)[sc - t0 * (TR / 2)] = h;
                    for (int p = 0; p < g.tp.n; p++)
                        if (g.tp.peer_out[p]) g.tp.peer_out[p][sc] = h;
                }
            }
            continue;
        }
        const int r = i * TR + lane;
        if (lane < TR && r < t.rows) {
            float y = acc;
            if (MODE == GM_QKV || MODE == GM_PLAIN) {
                if (g.bias) y = __fadd_rn(y, (MODE == GM_QKV && k < kConsWarps) ? gb0 : g.bias[r]);
                g.out[r] = y;
            } else if (MODE == GM_O || MODE == GM_DOWN) {
                y = __fadd_rn(k < kConsWarps ? res0 : g.out[r], y);
                g.out[r] = y;
            } else if (MODE == GM_HEAD) {
                g.out[r] = y;
                if (y > best_v || (y == best_v && r < best_i)) { best_v = y; best_i = r; }
            }
            for (int p = 0; p < g.tp.n; p++)
                if (g.tp.peer_out[p]) g.tp.peer_out[p][r] = y;
        }
    }

    if (MODE == GM_FFN && g.grp_tiles) {
        // every hidden value of the CTA's groups is in shared memory: their codes
        // for the down GEMV, one lane per group, quant_lanes as its staging would
        bar_sync(1, kConsThreads);
        const float * hq_vals = reinterpret_cast<const float *>(smem + SL.perm_off);
        const int F = g.ffn_n, ng = F / kGroup;
        ActS ga;
        ga.q = reinterpret_cast<int8_t *>(g.hq);
        ga.xs = reinterpret_cast<float *>(g.hq + F);
        ga.xsum = ga.xs + ng;
        ga.n = F;
        const int gq0 = t0 / g.grp_tiles, gq1 = t1 / g.grp_tiles;
        for (int grp = gq0 + (int) threadIdx.x; grp < gq1; grp += kConsThreads) {
            const float4 * src = reinterpret_cast<const float4 *>(hq_vals + (grp - gq0) * kGroup);
            float4 v[8];
#pragma unroll
            for (int k = 0; k < 8; k++) v[k] = src[k];
            quant_lanes<1>(v, grp, 0, ga, g, false, true);
        }
    }
    if (g.tp.n > 1 && g.tp.raise) {
        // every consumer's stores to the peers, then this CTA's arrival
        bar_sync(1, kConsThreads);
        if (threadIdx.x == 0) tp_arrive(g.tp);
    }
    bar_sync(1, kConsThreads);
    SB_MARK(g.trace, g.launch_id, 4);
    if (MODE == GM_HEAD && g.am_cnt) {
        // greedy argmax, ties to the lower index (sml/sml-run.c:3539-3544)
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
            if (atomicAdd(g.am_cnt, 1u) == gridDim.x - 1) {
                __threadfence();
                float fv = -INFINITY;
                int fi = 0x7fffffff;
                for (unsigned b = 0; b < gridDim.x; b++) {
                    const float v2 = ((volatile float *) g.am_val)[b];
                    const int ix = ((volatile int *) g.am_idx)[b];
                    if (v2 > fv || (v2 == fv && ix < fi)) { fv = v2; fi = ix; }
                }
                *g.am_cnt = 0;
                const int p = *g.pos;
                if (g.tlog) g.tlog[p] = fi;
                *g.tok = fi;
                *g.pos = p + 1;
            }
        }
    }
}

static __global__ void __launch_bounds__(kArgmaxThreads) k_tp_argmax(const float * logits, int V,
                                                                      const __grid_constant__ TpX x, int * tok,
                                                                      int * pos, int * tlog) {
    __shared__ float bv_s[kArgmaxThreads / 32];
    __shared__ int bi_s[kArgmaxThreads / 32];
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x == 0) tp_wait(x);
    __syncthreads();
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < V; i += blockDim.x) {
        const float v = logits[i];
        if (v > bv) { bv = v; bi = i; }   // increasing i: the first largest stays
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) { bv_s[threadIdx.x >> 5] = bv; bi_s[threadIdx.x >> 5] = bi; }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int) (blockDim.x >> 5); w++)
            if (bv_s[w] > bv || (bv_s[w] == bv && bi_s[w] < bi)) { bv = bv_s[w]; bi = bi_s[w]; }
        const int p = *pos;
        if (tlog) tlog[p] = bi;
        *tok = bi;
        *pos = p + 1;
    }
}

}  // namespace sb
