// Host side of the mixture-of-experts FFN: upload of one layer's router and
// experts, the routing scratch, and the four launches of one layer.
//
// Expert e of layer L is blk.L.ffn_{gate,up,down}.e.weight (the loader's names,
// sml/sml-run.c:1675-1700); the router blk.L.ffn_gate_inp.weight is fp32 with
// n_expert x n_embd values. Every expert of a layer is tiled with the same
// geometry, so one TT describes them all and per-expert tables give the tile
// bases and column orders.
#pragma once

#include "moe.cuh"
#include "upload.h"

#include <cstdio>
#include <vector>

namespace sb {

struct MoeLayer {
    int E = 0, F = 0, ne = 0, k = 0;
    int e_lo = 0, e_hi = 0;                                // experts held on this GPU (all, unless expert-parallel)
    unsigned flags = 0;
    const float * router = nullptr;                        // [ne][E]
    TT gu{}, dn{};                                         // geometry (expert 0's tiles)
    const uint8_t * const * gu_tiles = nullptr;            // device tables, [ne] each
    const int32_t * const * gu_perm = nullptr;
    const uint8_t * const * dn_tiles = nullptr;
    const int32_t * const * dn_iperm = nullptr;
    uint64_t expert_file_bytes = 0;                        // gate + up + down of one expert, as stored
    uint64_t router_bytes = 0;
};

struct MoeScratch {
    int T = 0;
    float * xn = nullptr, * hp = nullptr, * yk = nullptr;
    MoeRoute r{};
    uint8_t * xb = nullptr;           // tensor-core path (moe_tc.cu): the chunks' fp16 B operands
    int tc_chunks = 0;                // chunks the B operands are sized for (0: no tensor-core path)
};

// The tensor-core path (moe_tc.cu) for calls of 16 or more rows: whether the
// layer's experts suit it (four-bit codes, 8-bit group fields, widths in
// multiples of 128), the most chunks T rows can make, the B-operand scratch
// for them, and its launches (gather, gate/up, down) after the router.
bool moe_tc_ok(const MoeLayer & m);
int moe_tc_chunks(const MoeLayer & m, int T);
size_t moe_tc_scratch(const MoeLayer & m, int T);
cudaError_t moe_tc_enqueue(const MoeLayer & m, const MoeScratch & s, const float * in, int T, int nch_max,
                           cudaStream_t st, bool pdl, int * err);
constexpr int kMoeTcRows = 16;        // rows per call from which the tensor-core path can run
// In the automatic choice the tensor cores take a call whose chosen rows are at
// least this many per expert on average (T k >= kMoeTcAuto E): below it the
// integer kernels are faster (configuration 2 measured: integer 190 / 369 us at
// 16 / 64 rows, the tensor cores 328 / 540; at 256 rows 963 against 793).
constexpr int kMoeTcAuto = 8;
enum MoeTc { MOE_TC_OFF = 0, MOE_TC_ON = 1, MOE_TC_AUTO = 2 };
constexpr int kMoeTcChunk = 64;       // most rows of one expert per chunk on it

inline uint64_t moe_rec_bytes(const ssf_rec * r) {
    uint64_t b = r->sd_n + r->sq_n + r->md_n + r->mq_n;
    for (int p = 0; p < SSF_MAX_LEVELS; p++) b += r->codes_n[p];
    return b;
}

// Why layer L's MoE cannot run here, or NULL.
inline const char * moe_unsupported(const ssf_file & f, int L) {
    const ssf_hdr * h = f.hdr;
    if (h->moe_flags & ~1u) return "sigmoid, grouped or sparsemixer expert routing";
    if (h->moe_scale != 0.0f) return "scaled expert weights";
    if (h->moe_groups > 1) return "grouped expert routing";
    const char * names[] = {"blk.%d.ffn_gate_shexp.weight", "blk.%d.ffn_up_shexp.weight",
                            "blk.%d.ffn_down_shexp.weight", "blk.%d.exp_probs_b.weight"};
    for (const char * n : names) if (ssf_findf(&f, n, L, 0)) return "shared experts or an expert bias";
    return nullptr;
}

// Shared memory of the grouped GEMV: eight staged activations, then the ring.
inline size_t moe_act_bytes(int cols) { return (act_smem_bytes(cols) + 127) / 128 * 128; }

// Rows per expert tile: the most (<= 16, even for gate/up pairs) whose tile
// stays under 12 KB and leaves room for a ring beside eight staged
// activations; 0 if not even the fewest rows fit.
inline int moe_pick_tr(int cols, int nbits, int six, int has_min, int even) {
    for (int tr = 16; tr >= (even ? 2 : 1); tr /= 2) {
        const uint32_t tb = tile_geom(cols, tr, nbits, six, has_min).bytes;
        if (tb <= 12288 && ring_stages(8 * moe_act_bytes(cols), tb) >= 2) return tr;
    }
    return 0;
}

// Upload layer L's router and experts [e_lo, e_hi) (all when e_hi <= 0); both
// arena passes run this. Every expert's shapes are checked; only the held ones
// are uploaded.
inline bool moe_upload(Arena & a, const ssf_file & f, int L, MoeLayer & m, char * why, int nwhy, int e_lo = 0,
                       int e_hi = 0) {
    const ssf_hdr * h = f.hdr;
    const int E = (int) h->n_embd;
    const ssf_rec * rt = ssf_findf(&f, "blk.%d.ffn_gate_inp.weight", L, 0);
    if (!rt) { snprintf(why, nwhy, "layer %d: no router", L); return false; }
    if (const char * u = moe_unsupported(f, L)) { snprintf(why, nwhy, "layer %d: %s", L, u); return false; }
    const uint64_t rn = (uint64_t) rt->rows * rt->cols;
    if (rt->kind != SSF_KIND_F32 || rn % E) { snprintf(why, nwhy, "layer %d: router is not fp32 n_embd wide", L); return false; }
    if (E % 64 || E > 8192) { snprintf(why, nwhy, "layer %d: n_embd %d (a multiple of 64, at most 8192)", L, E); return false; }
    m.E = E;
    m.ne = (int) (rn / E);
    if (m.ne < 1 || m.ne > kMoeMaxExperts) {
        snprintf(why, nwhy, "layer %d: %d experts (at most %d)", L, m.ne, kMoeMaxExperts);
        return false;
    }
    int k = (int) h->n_expert_used;
    if (k <= 0 || k > m.ne) k = m.ne;   // sml/sml-run.c:2928-2930
    if (k > kMoeMaxK) k = kMoeMaxK;
    m.k = k;
    m.flags = h->moe_flags;
    m.router = upload_f32(a, f, rt);
    m.router_bytes = rn * 4;
    m.e_lo = e_hi > 0 ? e_lo : 0;
    m.e_hi = e_hi > 0 ? (e_hi < m.ne ? e_hi : m.ne) : m.ne;
    if (m.e_lo < 0 || m.e_lo >= m.e_hi) { snprintf(why, nwhy, "layer %d: empty expert range", L); return false; }
    std::vector<const uint8_t *> gt(m.ne), dt(m.ne);
    std::vector<const int32_t *> gp(m.ne), di(m.ne);
    int gtr = 0, dtr = 0;
    // experts drawn on the device when the arena asks for it (sb_draw_experts)
    struct Drawing {
        Arena & a;
        explicit Drawing(Arena & a_) : a(a_) { a.drawing = a.draw_seed != 0; }
        ~Drawing() { a.drawing = false; }
    } drawing(a);
    for (int e = 0; e < m.ne; e++) {
        char nm[3][96];
        snprintf(nm[0], sizeof nm[0], "blk.%d.ffn_gate.%d.weight", L, e);
        snprintf(nm[1], sizeof nm[1], "blk.%d.ffn_up.%d.weight", L, e);
        snprintf(nm[2], sizeof nm[2], "blk.%d.ffn_down.%d.weight", L, e);
        const ssf_rec * g = ssf_find(&f, nm[0]), * u = ssf_find(&f, nm[1]), * d = ssf_find(&f, nm[2]);
        if (!g || !u || !d) { snprintf(why, nwhy, "layer %d: expert %d is incomplete or ungated", L, e); return false; }
        const int F = (int) g->rows;
        if ((int) g->cols != E || u->rows != g->rows || (int) d->rows != E || (int) d->cols != F || F % 64 ||
            (e > 0 && F != m.F)) {
            snprintf(why, nwhy, "layer %d: expert %d shapes do not match", L, e);
            return false;
        }
        m.F = F;
        if (e == 0) {
            gtr = moe_pick_tr(E, (int) g->nbits, f.scale6, g->mq_n != 0, 1);
            dtr = moe_pick_tr(F, (int) d->nbits, f.scale6, d->mq_n != 0, 0);
            if (!gtr || !dtr) { snprintf(why, nwhy, "layer %d: expert rows too wide for the tile ring", L); return false; }
            m.expert_file_bytes = moe_rec_bytes(g) + moe_rec_bytes(u) + moe_rec_bytes(d);
        }
        if (e < m.e_lo || e >= m.e_hi) {   // held by another GPU
            gt[e] = nullptr; gp[e] = nullptr; dt[e] = nullptr; di[e] = nullptr;
            continue;
        }
        TT tg, td;
        // gate / up interleaved: a tile of gtr rows holds gtr/2 gate rows then the same up rows
        if (!upload_tt(a, f, g, 2 * F, gtr, 0, 1, [&](int r) {
                const int hh = gtr / 2, ti = r / gtr, j = r % gtr, i = ti * hh + j % hh;
                return i >= F ? RowSrc{nullptr, 0} : RowSrc{j < hh ? g : u, i}; }, tg, why, nwhy) ||
            !upload_tt(a, f, d, E, dtr, 0, 0, [&](int r) { return RowSrc{r < E ? d : nullptr, r}; }, td, why, nwhy))
            return false;
        if (e == m.e_lo) { m.gu = tg; m.dn = td; }
        if (tg.nbits != m.gu.nbits || tg.has_min != m.gu.has_min || td.nbits != m.dn.nbits || td.has_min != m.dn.has_min) {
            snprintf(why, nwhy, "layer %d: experts differ in width or fields", L);
            return false;
        }
        gt[e] = tg.tiles; gp[e] = tg.perm; dt[e] = td.tiles; di[e] = td.iperm;
    }
    m.gu_tiles = (const uint8_t * const *) a.upload(gt.data(), gt.size() * sizeof(void *));
    m.gu_perm = (const int32_t * const *) a.upload(gp.data(), gp.size() * sizeof(void *));
    m.dn_tiles = (const uint8_t * const *) a.upload(dt.data(), dt.size() * sizeof(void *));
    m.dn_iperm = (const int32_t * const *) a.upload(di.data(), di.size() * sizeof(void *));
    return true;
}

// Scratch for up to T tokens through layers shaped like m (carved from the arena).
inline void moe_carve(Arena & a, const MoeLayer & m, int T, MoeScratch & s) {
    const size_t ns = (size_t) T * m.k;
    s.T = T;
    s.xn = (float *) a.carve((size_t) T * m.E * 4);
    s.hp = (float *) a.carve(ns * m.F * 4);
    s.yk = (float *) a.carve(ns * m.E * 4);
    s.r.logits = (float *) a.carve((size_t) T * m.ne * 4);
    s.r.sel = (int *) a.carve(ns * 4);
    s.r.w = (float *) a.carve(ns * 4);
    s.r.slots = (int *) a.carve(ns * 4);
    s.r.ch_e = (int *) a.carve(ns * 4);
    s.r.ch_s0 = (int *) a.carve(ns * 4);
    s.r.ch_n = (int *) a.carve(ns * 4);
    s.r.meta = (int *) a.carve(2 * 4);
    s.r.cnt = (unsigned *) a.carve(4);
    if (T >= kMoeTcRows && moe_tc_ok(m)) {
        s.tc_chunks = moe_tc_chunks(m, T);
        s.xb = (uint8_t *) a.carve(moe_tc_scratch(m, T));
    } else {
        s.tc_chunks = 0;
        s.xb = nullptr;
    }
}

// Ring stages of the grouped GEMV for nt staged activations.
inline int moe_stages(const TT & t, int nt) {
    return ring_stages((size_t) nt * moe_act_bytes(t.cols) + moe_dot_smem(t, nt), t.tb);
}

template <int NB, int SIX>
inline void moe_gemv_w(int mode, int nt, const MoeGArgs & g, int grid, size_t smem, cudaStream_t st, bool pdl,
                       cudaError_t * r) {
    if (nt == 1 && mode != MG_PLAIN) {
        *r = mode == MG_GU ? moe_gemv_launch<MG_GU, NB, SIX, 1>(g, grid, smem, st, pdl)
                           : moe_gemv_launch<MG_DN, NB, SIX, 1>(g, grid, smem, st, pdl);
    } else if (mode == MG_PLAIN && nt == 4) {
        *r = moe_gemv_launch<MG_PLAIN, NB, SIX, 4>(g, grid, smem, st, pdl);
    } else {
        *r = mode == MG_GU ? moe_gemv_launch<MG_GU, NB, SIX, 8>(g, grid, smem, st, pdl)
           : mode == MG_DN ? moe_gemv_launch<MG_DN, NB, SIX, 8>(g, grid, smem, st, pdl)
                           : moe_gemv_launch<MG_PLAIN, NB, SIX, 8>(g, grid, smem, st, pdl);
    }
}

// nt: tokens per chunk: 1 or 8 for the expert GEMVs, 8 or 4 for a batched
// PLAIN GEMV (4 when eight staged activations leave no room for the ring).
inline cudaError_t moe_gemv(int mode, int nt, const MoeGArgs & g, int grid, cudaStream_t st, bool pdl) {
    cudaError_t r = cudaErrorInvalidValue;
    if (mode == MG_PLAIN && nt != 4) nt = 8;
    SB_DISPATCH_QT(g.t.nbits, g.t.six, moe_gemv_w, mode, nt, g, grid, moe_gemv_smem(g, nt), st, pdl, &r);
    return r;
}

// The router over T rows (RMS-normalized by norm_w first when given): logits,
// each row's chosen experts and weights, and the dispatch of the slots whose
// expert lies in [e_lo, e_hi) in chunks of at most nt rows (none when the range
// is empty).
inline cudaError_t moe_router_launch(const MoeLayer & m, const MoeScratch & s, const float * x, int T,
                                     const float * norm_w, float eps, int nt, int e_lo, int e_hi, cudaStream_t st,
                                     bool pdl, int * err, unsigned long long * trace, int launch_id,
                                     const ExpfEntry * xtab, float xnear) {
    MoeRouterArgs r;
    memset(&r, 0, sizeof r);
    r.x = x; r.norm_w = norm_w; r.eps = eps; r.xn = norm_w ? s.xn : nullptr; r.wr = m.router;
    r.T = T; r.E = m.E; r.ne = m.ne; r.k = m.k; r.nt = nt; r.flags = m.flags; r.r = s.r;
    r.e_lo = e_lo; r.e_hi = e_hi;
    r.xtab = xtab; r.xnear = xnear;
    r.err = err; r.trace = trace; r.launch_id = launch_id;
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_moe_router, cudaFuncAttributeMaxDynamicSharedMemorySize, 2 * 8192 * 4);
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(m.ne);
    cfg.blockDim = dim3(kRouterThreads);
    cfg.dynamicSmemBytes = (size_t) m.E * 4 * (norm_w ? 2 : 1);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_moe_router, r);
}

// y[t] (+)= the choice-order combine of the per-choice outputs s.yk ([T*k][E]),
// after waiting for the peers' rows when tp is given.
inline cudaError_t moe_comb_launch(const MoeLayer & m, const MoeScratch & s, int T, float * y, int resid,
                                   cudaStream_t st, bool pdl, const TpX * tp = nullptr) {
    TpX none;
    memset(&none, 0, sizeof none);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((m.E + 255) / 256, T);
    cfg.blockDim = dim3(256);
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_moe_comb, (const float *) s.yk, (const float *) s.r.w, T, m.k, m.E, y, resid,
                              tp ? *tp : none);
}

// A tensor-parallel engine's exchange of an MoE layer's rows: the down GEMV
// stores each row into every rank's per-choice buffer (s.yk lies in the
// region the peers map) and its CTAs arrive at the peers; the combine waits
// for them. Each row is computed by the one GPU holding its expert.
struct MoePeerX {
    TpX dn, comb;
};

// Expert parallelism: the per-choice down outputs ([T*k][E]) are summed over
// the GPUs between the down GEMV and the combine. Each row is written by the one
// GPU holding its expert and is zero on the others, so the sum is exact and the
// combine then runs in choice order as on one GPU.
struct MoeExchange {
    cudaError_t (*sum)(void * ctx, float * buf, size_t n, cudaStream_t st);
    void * ctx;
};

// The launches of one MoE FFN over T <= s.T input rows x ([T][E]): router and
// routing (x RMS-normalized by norm_w first when given), gate/up, down, combine
// into y ([T][E]; added to it when resid). post(err, name) sees every launch.
// With ex (expert parallelism) the per-choice outputs are zeroed first and
// summed across GPUs before the combine. tc (MoeTc): ON runs the expert
// products of calls of kMoeTcRows rows or more on the tensor cores (moe_tc.cu)
// when the scratch was carved for it; AUTO only those with at least
// kMoeTcAuto chosen rows per expert on average.
template <class Post>
inline void moe_enqueue(const MoeLayer & m, const MoeScratch & s, const float * x, int T, const float * norm_w,
                        float eps, float * y, int resid, int nsm, cudaStream_t st, bool pdl, int * err,
                        unsigned long long * trace, int launch_id, Post post, const MoeExchange * ex = nullptr,
                        const ExpfEntry * xtab = nullptr, float xnear = 0.0f, int tc = MOE_TC_OFF,
                        const MoePeerX * px = nullptr) {
    const bool use_tc = tc != MOE_TC_OFF && s.tc_chunks > 0 && T >= kMoeTcRows &&
                        (tc == MOE_TC_ON || (long) T * m.k >= (long) kMoeTcAuto * m.ne);
    // one token per chunk at T = 1: a token never picks an expert twice
    const int nt = use_tc ? kMoeTcChunk : T == 1 ? 1 : 8;
    if (ex) post(cudaMemsetAsync(s.yk, 0, (size_t) T * m.k * m.E * 4, st), "moe.zero");
    post(moe_router_launch(m, s, x, T, norm_w, eps, nt, m.e_lo, m.e_hi, st, pdl, err, trace, launch_id, xtab, xnear),
         "moe.router");
    MoeGArgs g;
    memset(&g, 0, sizeof g);
    g.slots = s.r.slots; g.ch_e = s.r.ch_e; g.ch_s0 = s.r.ch_s0; g.ch_n = s.r.ch_n; g.meta = s.r.meta;
    g.err = err; g.trace = trace;
    if (use_tc) {
        post(moe_tc_enqueue(m, s, norm_w ? s.xn : x, T, s.tc_chunks, st, pdl, err), "moe.tensor_cores");
    } else {
        {
            MoeGArgs a = g;
            a.t = m.gu; a.tiles = m.gu_tiles; a.perm = m.gu_perm; a.scatter = m.dn_iperm;
            a.in = norm_w ? s.xn : x; a.in_stride = m.E; a.in_div = m.k;
            a.out = s.hp; a.out_stride = m.F; a.ffn_f = m.F;
            a.nstage = moe_stages(m.gu, nt);
            a.launch_id = launch_id + 1;
            post(moe_gemv(MG_GU, nt, a, nsm, st, pdl), "moe.gate_up");
        }
        {
            MoeGArgs a = g;
            a.t = m.dn; a.tiles = m.dn_tiles;
            a.in = s.hp; a.in_stride = m.F; a.in_div = 1;
            a.out = s.yk; a.out_stride = m.E;
            a.nstage = moe_stages(m.dn, nt);
            a.launch_id = launch_id + 2;
            if (px) a.tp = px->dn;
            post(moe_gemv(MG_DN, nt, a, nsm, st, pdl), "moe.down");
        }
    }
    if (ex) post(ex->sum(ex->ctx, s.yk, (size_t) T * m.k * m.E, st), "moe.exchange");
    post(moe_comb_launch(m, s, T, y, resid, st, pdl, px ? &px->comb : nullptr), "moe.combine");
}

}  // namespace sb
