// Mixture-of-experts FFN on the device: router, top-k routing and dispatch,
// grouped expert GEMV (gate/up with SiLU, then down) and the weighted combine.
//
// The reference's layer (sml/sml-run.c:3071-3125 moe_ffn on the CPU;
// sml/sml-gpu-fwd.c:492-546 moe_ffn_dev with sml/sml-gpu-fast.cu:3356-3580 on
// its GPU) does, per token: fp32 router logits with double accumulation, the
// top-k experts (ties to the lower index), softmax weights, then for each
// chosen expert j: h = silu(gate_j x) * up_j x, t_j = down_j h, and
// y = sum_j w_j t_j in choice order. Here:
//
//   k_moe_router   one CTA per expert row: logits for every token; the last
//                  CTA to finish routes every token (one warp each) and builds
//                  the dispatch: slot ids (t*k + j) grouped by expert, cut into
//                  chunks of at most NT tokens of one expert.
//   k_moe_gemv     the tile ring of tgemv.cuh over work items (chunk, tile):
//                  the weights of a chunk's expert are read once for all of its
//                  tokens; each lane keeps NT row sums (one token per chunk:
//                  the reference's float order, tile_exact). GU mode fuses SiLU and
//                  scatters the hidden vector into the expert's down order; DN
//                  mode writes one output row per slot; PLAIN is a batched GEMV
//                  of one tensor over T input rows.
//   k_moe_comb     y[t] = sum_j w[t,j] * down rows of slot (t, j), in choice
//                  order, optionally added to a residual.
//
// Every row sum is finished by one warp in a fixed order, so results do not
// depend on timing or on how tokens fall into chunks.
#pragma once

#include "tgemv.cuh"

namespace sb {

constexpr int kMoeMaxExperts = 256;
constexpr int kMoeMaxK = 16;
constexpr int kRouterThreads = 256;

enum MoeMode { MG_GU = 0, MG_DN = 1, MG_PLAIN = 2 };

// Routing state, written by the router's last CTA and read by the GEMVs.
struct MoeRoute {
    float * logits;                  // [T][ne]
    int * sel;                       // [T][k] chosen experts
    float * w;                       // [T][k] their weights
    int * slots;                     // [T*k] slot ids grouped by expert, ascending within one
    int * ch_e, * ch_s0, * ch_n;     // per chunk: expert, first index into slots, tokens
    int * meta;                      // [0] chunks, [1] distinct experts chosen
    unsigned * cnt;                  // CTA completion counter, left at zero
};

struct MoeRouterArgs {
    const float * x;                 // [T][E] input rows
    const float * norm_w;            // RMSNorm gain applied first, or NULL
    float eps;
    float * xn;                      // [T][E] normalized rows (written when norm_w is set)
    const float * wr;                // [ne][E] router weights
    int T, E, ne, k, nt;             // nt: most tokens in one chunk
    unsigned flags;                  // bit 0: softmax over the chosen experts only
    int e_lo, e_hi;                  // experts this GPU holds: only their slots are dispatched
    const ExpfEntry * xtab;          // the host libm's expf (expf_libm.h), or NULL
    float xnear;
    MoeRoute r;
    int * err;
    unsigned long long * trace;
    int launch_id;
};

struct MoeGArgs {
    TT t;                            // shared geometry of every expert's tiles (t.tiles unused)
    const uint8_t * const * tiles;   // [expert] tile base
    const int32_t * const * perm;    // [expert] input gather (GU, PLAIN)
    const int32_t * const * scatter; // [expert] GU: where hidden value i goes (down's inverse order)
    const float * in;                // input rows
    int in_stride, in_div;           // floats per input row; input row = slot / in_div
    float * out;
    int out_stride;                  // floats per output row
    int ffn_f;                       // GU: hidden size
    const int * slots, * ch_e, * ch_s0, * ch_n, * meta;
    int nstage;
    int * err;
    unsigned long long * trace;
    int launch_id;
    // DN on a tensor-parallel engine: every output row also stored into each
    // peer's copy of `out`, then each CTA arrives at the peers (tgemv.cuh TpX)
    TpX tp;
};

// ---------------------------------------------------------------- routing

// Route one token with one warp (sml/sml-run.c:3009-3030, the plain softmax
// branch): k rounds of a warp argmax over the experts not yet taken, ties to
// the lower index; weights exp(l_j - l_0) / sum over the chosen (flags bit 0)
// or the softmax over every expert, sums in double; exp as the host libm
// rounds it when xtab is given (expf_libm.h), else rounded from double.
SB_DEV void route_warp(const float * lg, int ne, int k, unsigned flags, int * sel, float * w, int lane,
                       const ExpfEntry * xtab = nullptr, float xnear = 0.0f) {
    constexpr int kQ = kMoeMaxExperts / 32;
    float v[kQ];
#pragma unroll
    for (int q = 0; q < kQ; q++) {
        const int e = q * 32 + lane;
        v[q] = e < ne ? __ldcg(lg + e) : -INFINITY;
    }
    uint32_t taken = 0;
    int s[kMoeMaxK];
    float ls[kMoeMaxK];
    for (int j = 0; j < k; j++) {
        float bv = -INFINITY;
        int bi = 0x7fffffff;
#pragma unroll
        for (int q = 0; q < kQ; q++) {
            const int e = q * 32 + lane;
            if (e < ne && !((taken >> q) & 1u) && (bi == 0x7fffffff || v[q] > bv)) { bv = v[q]; bi = e; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (oi != 0x7fffffff && (bi == 0x7fffffff || ov > bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
        }
        s[j] = bi;
        ls[j] = bv;
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    }
    if (flags & 1u) {
        double sum = 0.0;
        float wf[kMoeMaxK];
        for (int j = 0; j < k; j++) { wf[j] = expf_libm(__fsub_rn(ls[j], ls[0]), xtab, xnear); sum += (double) wf[j]; }
        if (lane == 0)
            for (int j = 0; j < k; j++) { sel[j] = s[j]; w[j] = (float) ((double) wf[j] / sum); }
    } else {
        float mx = -INFINITY;
#pragma unroll
        for (int q = 0; q < kQ; q++) if (q * 32 + lane < ne) mx = fmaxf(mx, v[q]);
        mx = warp_max(mx);
        double sum = 0.0;
#pragma unroll
        for (int q = 0; q < kQ; q++) if (q * 32 + lane < ne) sum += (double) expf_libm(__fsub_rn(v[q], mx), xtab, xnear);
        sum = warp_sum_d(sum);
        if (lane == 0)
            for (int j = 0; j < k; j++) { sel[j] = s[j]; w[j] = (float) ((double) expf_libm(__fsub_rn(ls[j], mx), xtab, xnear) / sum); }
    }
}

// Exclusive prefix sums of a[0..n) (n <= 256) by one warp into out[0..n], out[n] = total.
SB_DEV void warp_scan_256(const int * a, int n, int * out, int lane) {
    int loc[8], tot = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int e = lane * 8 + i;
        loc[i] = tot;
        tot += e < n ? a[e] : 0;
    }
    int inc = tot;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    const int base = inc - tot;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int e = lane * 8 + i;
        if (e < n) out[e] = base + loc[i];
    }
    if (lane == 31) out[n] = inc;
}

// Dispatch by the last router CTA: count the slots of every expert, lay them
// out grouped by expert (ascending slot id within one), cut chunks of nt.
SB_DEV void moe_dispatch(const MoeRouterArgs & g) {
    __shared__ int cnt[kMoeMaxExperts], fill[kMoeMaxExperts];
    __shared__ int off[kMoeMaxExperts + 1], nch[kMoeMaxExperts], choff[kMoeMaxExperts + 1];
    const int tid = threadIdx.x, ne = g.ne, ns = g.T * g.k;
    for (int e = tid; e < ne; e += blockDim.x) { cnt[e] = 0; fill[e] = 0; }
    __syncthreads();
    // slots of experts held elsewhere (expert parallelism) are not dispatched here
    for (int s = tid; s < ns; s += blockDim.x) {
        const int e = g.r.sel[s];
        if (e >= g.e_lo && e < g.e_hi) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    for (int e = tid; e < ne; e += blockDim.x) nch[e] = (cnt[e] + g.nt - 1) / g.nt;
    __syncthreads();
    if (tid < 32) warp_scan_256(cnt, ne, off, tid);
    else if (tid < 64) warp_scan_256(nch, ne, choff, tid - 32);
    __syncthreads();
    for (int s = tid; s < ns; s += blockDim.x) {
        const int e = g.r.sel[s];
        if (e >= g.e_lo && e < g.e_hi) g.r.slots[off[e] + atomicAdd(&fill[e], 1)] = s;
    }
    __syncthreads();
    for (int e = tid; e < ne; e += blockDim.x) {
        int * l = g.r.slots + off[e];
        const int n = cnt[e];
        for (int a = 1; a < n; a++) {   // insertion sort: the lists are short
            const int v = l[a];
            int b = a - 1;
            while (b >= 0 && l[b] > v) { l[b + 1] = l[b]; b--; }
            l[b + 1] = v;
        }
        for (int c = 0; c < nch[e]; c++) {
            const int at = choff[e] + c;
            g.r.ch_e[at] = e;
            g.r.ch_s0[at] = off[e] + c * g.nt;
            g.r.ch_n[at] = n - c * g.nt < g.nt ? n - c * g.nt : g.nt;
        }
    }
    if (tid == 0) {
        int act = 0;
        for (int e = 0; e < ne; e++) act += cnt[e] > 0;
        g.r.meta[0] = choff[ne];
        g.r.meta[1] = act;
    }
}

// Router: CTA e computes logit e of every token (double accumulation, as
// sml/sml-run.c:3076-3081), warp w taking tokens w, w+8, ...; the last CTA to
// finish routes and dispatches. With a gain, each warp first RMS-normalizes
// its token (sum of squares in double, sml/sml-run.c:147-152); CTA 0 writes
// the normalized rows for the expert GEMVs.
static __global__ void __launch_bounds__(kRouterThreads) k_moe_router(const __grid_constant__ MoeRouterArgs g) {
    extern __shared__ __align__(16) float rsm[];   // [E] router row, then [E] gain
    __shared__ int last;
    pdl_launch_dependents();
    SB_MARK(g.trace, g.launch_id, 0);
    const int E = g.E, e = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float * wrow = rsm;
    float * gain = rsm + E;
    for (int i = 4 * tid; i < E; i += 4 * kRouterThreads) {
        *reinterpret_cast<float4 *>(wrow + i) = *reinterpret_cast<const float4 *>(g.wr + (size_t) e * E + i);
        if (g.norm_w) *reinterpret_cast<float4 *>(gain + i) = *reinterpret_cast<const float4 *>(g.norm_w + i);
    }
    __syncthreads();
    pdl_wait();
    for (int t = warp; t < g.T; t += kRouterThreads / 32) {
        const float * x = g.x + (size_t) t * E;
        float s = 1.0f;
        if (g.norm_w) {
            double q = 0.0;
            for (int i = 4 * lane; i < E; i += 128) {
                const float4 f = *reinterpret_cast<const float4 *>(x + i);
                q += (double) f.x * f.x + (double) f.y * f.y + (double) f.z * f.z + (double) f.w * f.w;
            }
            q = warp_sum_d(q);
            s = __fdiv_rn(1.0f, sqrtf(__fadd_rn((float) (q / E), g.eps)));
        }
        double acc = 0.0;
        for (int i = 4 * lane; i < E; i += 128) {
            float4 f = *reinterpret_cast<const float4 *>(x + i);
            if (g.norm_w) {
                f.x = __fmul_rn(__fmul_rn(f.x, s), gain[i]);
                f.y = __fmul_rn(__fmul_rn(f.y, s), gain[i + 1]);
                f.z = __fmul_rn(__fmul_rn(f.z, s), gain[i + 2]);
                f.w = __fmul_rn(__fmul_rn(f.w, s), gain[i + 3]);
                if (e == 0 && g.xn) *reinterpret_cast<float4 *>(g.xn + (size_t) t * E + i) = f;
            }
            acc += (double) wrow[i] * f.x + (double) wrow[i + 1] * f.y + (double) wrow[i + 2] * f.z +
                   (double) wrow[i + 3] * f.w;
        }
        acc = warp_sum_d(acc);
        if (lane == 0) g.r.logits[(size_t) t * g.ne + e] = (float) acc;
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        last = atomicAdd(g.r.cnt, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    SB_MARK(g.trace, g.launch_id, 1);
    for (int t = warp; t < g.T; t += kRouterThreads / 32)
        route_warp(g.r.logits + (size_t) t * g.ne, g.ne, g.k, g.flags, g.r.sel + (size_t) t * g.k,
                   g.r.w + (size_t) t * g.k, lane, g.xtab, g.xnear);
    __syncthreads();
    moe_dispatch(g);
    if (tid == 0) *g.r.cnt = 0;
    SB_MARK(g.trace, g.launch_id, 2);
}

// Routing alone over given logits (T tokens, one warp each).
static __global__ void k_moe_route(const float * lg, int T, int ne, int k, unsigned flags, int * sel, float * w) {
    const int t = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (t >= T) return;
    route_warp(lg + (size_t) t * ne, ne, k, flags, sel + (size_t) t * k, w + (size_t) t * k, threadIdx.x & 31);
}

// y[t][i] = sum_j w[t][j] * yk[t*k + j][i] in choice order from 0, each step
// one fused multiply-add as gcc contracts acc += w*t (sml/sml-run.c:3120),
// added to y[t][i] when resid (the layer's residual add, x + xb).
// On a tensor-parallel engine (tp.wait_count) the rows of the choices other
// GPUs hold arrive from them first: one thread of each block waits (bounded).
static __global__ void k_moe_comb(const float * yk, const float * w, int T, int k, int E, float * y, int resid,
                                  const __grid_constant__ TpX tp) {
    pdl_launch_dependents();
    pdl_wait();
    if (tp.n > 1 && tp.wait_count) {
        if (threadIdx.x == 0) tp_wait(tp);
        __syncthreads();
    }
    const int i = blockIdx.x * blockDim.x + threadIdx.x, t = blockIdx.y;
    if (i >= E || t >= T) return;
    float acc = 0.0f;
    for (int j = 0; j < k; j++)
        acc = __fmaf_rn(w[(size_t) t * k + j], yk[((size_t) t * k + j) * E + i], acc);
    float * o = y + (size_t) t * E + i;
    *o = resid ? __fadd_rn(*o, acc) : acc;
}

// ---------------------------------------------------------------- grouped GEMV

// The codes of unit u of tile row j as bytes (every plane's piece shifted into
// place): c[k][w] holds group k's columns 4w..4w+3 of the unit.
template <int NB>
SB_DEV void unit_codes(const uint8_t * tile, const TileGeom & tg, int j, int u, uint32_t (&c)[4][4]) {
    int kinds[3], shifts[3];
    plane_kinds(NB, kinds, shifts);
#pragma unroll
    for (int k = 0; k < 4; k++)
#pragma unroll
        for (int w = 0; w < 4; w++) c[k][w] = 0;
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
#pragma unroll
            for (int w = 0; w < 4; w++) {
                c[0][w] |= (x0[w] & 0x0f0f0f0fu) << sh;
                c[1][w] |= ((x0[w] >> 4) & 0x0f0f0f0fu) << sh;
                c[2][w] |= (x1[w] & 0x0f0f0f0fu) << sh;
                c[3][w] |= ((x1[w] >> 4) & 0x0f0f0f0fu) << sh;
            }
        } else if (kinds[p] == 2) {
            const uint4 w = *reinterpret_cast<const uint4 *>(sec + 16 * at);
            const uint32_t x[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int ww = 0; ww < 4; ww++) c[k][ww] |= ((x[ww] >> (2 * k)) & 0x03030303u) << sh;
        } else {
            const uint2 w = *reinterpret_cast<const uint2 *>(sec + 8 * at);
            const uint32_t h[4] = {w.x & 0xffffu, w.x >> 16, w.y & 0xffffu, w.y >> 16};
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int ww = 0; ww < 4; ww++) c[k][ww] |= nib_to_bytes((h[k] >> (4 * ww)) & 15u) << sh;
        }
    }
}


// Lane share of tile row j for up to NT activations at once (the activations
// of one chunk, act_b bytes apart): the codes and fields of a unit are read
// once and used for every token. The integers are exact; the float epilogue
// is summed per unit (lane l: row l % TR, units l / TR + k * (32 / TR)) and
// the lanes' shares are added by the caller -- another order than the
// reference's, within its rounding (the one-token path is exact: tile_exact).
template <int NB, int SIX, int NT>
SB_DEV void tile_row_nt(const uint8_t * tile, const TileGeom & tg, uint8_t * act0, uint32_t act_b, int n, int ntok,
                        int j, int u0, int step, bool has_min, float mbias, float (&acc)[NT]) {
#pragma unroll
    for (int tt = 0; tt < NT; tt++) acc[tt] = 0.0f;
    const int qn = n >> 2;
    for (int u = u0; u < tg.U; u += step) {
        uint32_t c[4][4];
        unit_codes<NB>(tile, tg, j, u, c);
        const int pq = u >> 1;
        int sq[4], mq[4];
        tile_fields<SIX>(tile + tg.sq_off + (pq * tg.TR + j) * tg.f_w, sq);
        const float sd = h2f(*reinterpret_cast<const uint16_t *>(tile + tg.sd_off + ((u >> 2) * tg.TR + j) * 2));
        const bool mins = has_min && (u & 1) == 0;
        float md = 0.0f;
        if (mins) {
            tile_fields<SIX>(tile + tg.mq_off + (pq * tg.TR + j) * tg.f_w, mq);
            md = h2f(*reinterpret_cast<const uint16_t *>(tile + tg.md_off + ((u >> 2) * tg.TR + j) * 2));
        }
#pragma unroll
        for (int tt = 0; tt < NT; tt++) {
            if (tt >= ntok) break;
            const uint8_t * ab = act0 + (size_t) tt * act_b;
            const int8_t * q = reinterpret_cast<const int8_t *>(ab);
            const float * xsv = reinterpret_cast<const float *>(ab + n);
            int d[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint4 a = *reinterpret_cast<const uint4 *>(q + k * qn + 16 * u);
                int s = dp4a_us(c[k][0], a.x, 0);
                s = dp4a_us(c[k][1], a.y, s);
                s = dp4a_us(c[k][2], a.z, s);
                d[k] = dp4a_us(c[k][3], a.w, s);
            }
            const float4 xs = *reinterpret_cast<const float4 *>(xsv + 4 * pq);
            float t1 = (float) sq[0] * xs.x * (float) d[0];
            t1 += (float) sq[1] * xs.y * (float) d[1];
            t1 += (float) sq[2] * xs.z * (float) d[2];
            t1 += (float) sq[3] * xs.w * (float) d[3];
            acc[tt] += sd * t1;
            if (mins) {
                const float4 xm = *reinterpret_cast<const float4 *>(xsv + (n >> 5) + 4 * pq);
                float t2 = ((float) mq[0] - mbias) * xm.x;
                t2 += ((float) mq[1] - mbias) * xm.y;
                t2 += ((float) mq[2] - mbias) * xm.z;
                t2 += ((float) mq[3] - mbias) * xm.w;
                acc[tt] += md * t2;
            }
        }
    }
}

// Stage the activations of one chunk (consumer threads, named barrier 1):
// (token, group) pairs go to teams of 8 lanes, every load of a batch issued
// before any quantization. Gathered modes read in[row][perm[i]].
template <int NT>
SB_DEV void moe_stage(const MoeGArgs & g, const int32_t * perm, const int (&slot)[NT], int ntok, uint8_t * act0,
                      uint32_t act_b) {
    const int n = g.t.cols, ng = n / kGroup, tid = threadIdx.x;
    const int team = tid >> 3, sub = tid & 7, nteam = kConsThreads / 8;
    const int pairs = ntok * ng;
    constexpr int kR = 8;
    for (int base = 0; base < pairs; base += kR * nteam) {
        float4 v[kR];
#pragma unroll
        for (int r = 0; r < kR; r++) {
            const int m = base + r * nteam + team;
            v[r] = make_float4(0.f, 0.f, 0.f, 0.f);
            if (m < pairs) {
                const int tt = m / ng, grp = m - tt * ng;
                int sl = slot[0];
#pragma unroll
                for (int q = 1; q < NT; q++) if (q == tt) sl = slot[q];
                const float * row = g.in + (size_t) (sl / g.in_div) * g.in_stride;
                if (perm) {
                    const int4 p4 = *reinterpret_cast<const int4 *>(perm + grp * kGroup + 4 * sub);
                    v[r] = make_float4(row[p4.x], row[p4.y], row[p4.z], row[p4.w]);
                } else {
                    v[r] = *reinterpret_cast<const float4 *>(row + grp * kGroup + 4 * sub);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kR; r++) {
            const int m0 = base + r * nteam;   // warp-uniform: teams of one warp share r
            if (m0 >= pairs) break;
            const int m = m0 + team;
            const int tt = m < pairs ? m / ng : 0, grp = m < pairs ? m - tt * ng : 0;
            ActS a = act_carve(act0 + (size_t) tt * act_b, n);
            quant_team_to(v[r], grp, sub, a, m < pairs);
        }
    }
    bar_sync(1, kConsThreads);
}

template <int MODE, int NB, int SIX, int NT>
__global__ void __launch_bounds__(kTgThreads, 1) k_moe_gemv(const __grid_constant__ MoeGArgs g) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full[kMaxStages], empty[kMaxStages];
    pdl_launch_dependents();
    SB_MARK(g.trace, g.launch_id, 0);
    const TT & t = g.t;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, ns = g.nstage, n = t.cols;
    const uint32_t act_b = (uint32_t) ((act_smem_bytes(n) + 127) / 128 * 128);
    // one token per chunk: the rows in the reference's float order (tile_exact),
    // each warp's group dots in a scratch after the activation
    const uint32_t dscr = NT == 1 ? (tg_dot_bytes(t) + 127) / 128 * 128 : 0u;
    int * D = reinterpret_cast<int *>(smem + (size_t) NT * act_b) + (size_t) warp * (tg_dot_bytes(t) / kConsWarps / 4);
    uint8_t * ring = smem + (size_t) NT * act_b + dscr;
    if (threadIdx.x == 0) {
        for (int s = 0; s < ns; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_fence_init();
    }
    __syncthreads();
    // which tiles this CTA reads depends on the routing: everyone waits first
    pdl_wait();
    const int ntl = t.ntiles;
    const long Q = (long) g.meta[0] * ntl;
    const int q0 = (int) (Q * blockIdx.x / gridDim.x), q1 = (int) (Q * (blockIdx.x + 1) / gridDim.x);

    if (warp == kConsWarps) {
        // lane j < ns owns ring stage j and issues items q0 + j, q0 + j + ns, ...
        if (lane < ns) {
            const int s = lane;
            const uint32_t tb = t.tb;
            int cur = -1, lap = 0;
            const uint8_t * base = nullptr;
            for (int q = q0 + s; q < q1; q += ns, lap++) {
                const int c = q / ntl, i = q - c * ntl;
                if (c != cur) { cur = c; base = g.tiles[g.ch_e[c]]; }
                if (lap > 0 && !mbar_wait(&empty[s], (lap - 1) & 1, g.err, 1)) break;
                mbar_expect_tx(&full[s], tb);
                bulk_g2s(ring + (size_t) s * tb, base + (size_t) i * tb, tb, &full[s]);
            }
            if (lap > 0) mbar_wait(&full[s], (lap - 1) & 1, g.err, 3);   // nothing may land after exit
        }
        return;
    }

    const TileGeom tg = tile_geom(n, t.TR, NB, SIX, t.has_min);
    const int TR = t.TR, j = lane % TR, v = lane / TR, VS = 32 / TR;
    bool failed = false;
    for (int q = q0; q < q1;) {
        const int c = q / ntl;
        const int qe = (c + 1) * ntl < q1 ? (c + 1) * ntl : q1;
        const int e = g.ch_e[c], ntok = g.ch_n[c], s0 = g.ch_s0[c];
        int slot[NT];
#pragma unroll
        for (int tt = 0; tt < NT; tt++) slot[tt] = tt < ntok ? g.slots[s0 + tt] : 0;
        moe_stage<NT>(g, MODE == MG_DN ? nullptr : g.perm[e], slot, ntok, smem, act_b);
        const int32_t * scat = MODE == MG_GU ? g.scatter[e] : nullptr;
        const int k0 = q - q0, k1 = qe - q0;
        for (int k = k0 + (((warp - k0) % kConsWarps) + kConsWarps) % kConsWarps; k < k1; k += kConsWarps) {
            const int s = k % ns, i = q0 + k - c * ntl;
            const bool ok = __all_sync(0xffffffffu, !failed && ring_wait(full, empty, k, ns, g.err));
            failed = !ok;
            float acc[NT];
            if (ok) {
                if (NT == 1) {
                    ActS a = act_carve(smem, n);
                    acc[0] = tile_rows<NB, SIX>(ring + (size_t) s * t.tb, tg, a, D, t.has_min, t.mbias);
                } else {
                    tile_row_nt<NB, SIX, NT>(ring + (size_t) s * t.tb, tg, smem, act_b, n, ntok, j, v, VS,
                                             t.has_min, t.mbias, acc);
                }
            } else {
#pragma unroll
                for (int tt = 0; tt < NT; tt++) acc[tt] = 0.0f;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
#pragma unroll
            for (int tt = 0; tt < NT; tt++) {
                if (tt >= ntok) break;
                float a = acc[tt];
                if (NT > 1)
                    for (int o = 16; o >= TR; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
                if (MODE == MG_GU) {
                    const float up = __shfl_down_sync(0xffffffffu, a, TR / 2);
                    const int idx = i * (TR / 2) + lane;
                    if (lane < TR / 2 && idx < g.ffn_f && SB_CHECK(g.err, scat[idx] >= 0 && scat[idx] < g.ffn_f, 110))
                        g.out[(size_t) slot[tt] * g.out_stride + scat[idx]] = silu_mul(a, up);
                } else {
                    const int r = i * TR + lane;
                    if (lane < TR && r < t.rows) {
                        const size_t at = (size_t) slot[tt] * g.out_stride + r;
                        g.out[at] = a;
                        for (int p = 0; p < g.tp.n; p++)
                            if (g.tp.peer_out[p]) g.tp.peer_out[p][at] = a;
                    }
                }
            }
        }
        bar_sync(1, kConsThreads);   // the chunk's activations are free again
        q = qe;
    }
    if (g.tp.n > 1 && g.tp.raise) {
        // every consumer's stores to the peers are ordered before this CTA's
        // arrival by the barrier of the last chunk (or there were none)
        bar_sync(1, kConsThreads);
        if (threadIdx.x == 0) tp_arrive(g.tp);
    }
    SB_MARK(g.trace, g.launch_id, 4);
}

// Launchers (explicitly instantiated in moe_gemv*.cu, one file per NT).
template <int MODE, int NB, int SIX, int NT>
cudaError_t moe_gemv_launch(const MoeGArgs & g, int grid, size_t smem, cudaStream_t st, bool pdl);

// The group-dot scratch of the one-token (exact) expert GEMV.
__host__ __device__ inline size_t moe_dot_smem(const TT & t, int nt) {
    return nt == 1 ? (tg_dot_bytes(t) + 127) / 128 * 128 : 0;
}

__host__ inline size_t moe_gemv_smem(const MoeGArgs & g, int nt) {
    return (size_t) nt * ((act_smem_bytes(g.t.cols) + 127) / 128 * 128) + moe_dot_smem(g.t, nt) +
           (size_t) g.nstage * g.t.tb;
}

}  // namespace sb
