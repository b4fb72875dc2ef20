// Host engine for the decode path: upload, plan, graph capture, step API.
//
// Replaces the reference's GPU host driver (sml/sml-gpu-fwd.c: gpu_setup :1789,
// gpu_forward :1643, graph_token :636, sml_gpu_open/step/prefill :2353-2412)
// with the Linux CUDA runtime: one arena for the model, one stream, one
// captured graph per token whose kernels chain by programmatic dependent
// launch, and the greedy choice made on the device so a generation loop is
// graph replays with no host round trip.
#include "decode.cuh"
#include "moe_host.h"
#include "tc_batch.h"
#include "tgemv.cuh"
#include "sheep_b200.h"
#include "ssf.h"
#include "upload.h"

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

using namespace sb;

static thread_local char g_err[512];

const char * sb_last_error(void) { return g_err; }

static bool ck(cudaError_t e, const char * what) {
    if (e == cudaSuccess) return true;
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return false;
}

struct LayerD {
    TT qkv, gateup, o, down;          // tiled: q|k|v rows; gate/up interleaved by 8 rows
    const float * an = nullptr, * fn = nullptr;
    const float * qkv_b = nullptr;    // q|k|v biases, or NULL
    const float * qn = nullptr, * kn = nullptr;
    const int32_t * down_iperm = nullptr;   // gate/up value i -> its place in down's column order
    bool moe = false;                 // mixture-of-experts FFN in place of gate/up/down
    MoeLayer ml;
};

// Tensor parallelism (tp > 1 ranks, one process per GPU): attention, q|k|v and
// o are replicated; gate/up, down and the head are split by rows. Rank r
// computes the hidden values of down's column positions [F r/tp, F (r+1)/tp)
// (whole groups of 32), down's rows [E r/tp, ..) and the head's rows
// [V r/tp, ..); each GEMV stores its rows into every rank's copy of the vector
// (peer pointers into each rank's exchange region, CUDA IPC) and its last CTA
// raises the event in every rank's flag array; the kernel that reads the whole
// vector waits for every peer's event first. Each row is still computed whole
// by one rank, in the same arithmetic, so the ranks' results equal one GPU's
// bit for bit. Events per token: hidden(l) = 2l, x(l) = 2l+1 after layer l's
// down, logits = 2 n_layer.
struct TpState {
    int n = 1, rank = 0;
    uint8_t * reg = nullptr;          // this rank's exchange region (cudaMalloc: IPC-exported)
    size_t reg_bytes = 0;
    void * peer[kMaxTp] = {};         // every rank's region as mapped here (this rank's = reg)
    size_t off_x = 0, off_hp = 0, off_lg = 0;   // vectors in the region (flags at 0)
    size_t off_yk = 0;                          // MoE layers: the per-choice rows [2][k][E] (by layer parity)
    unsigned * tok_seq = nullptr;
    std::vector<unsigned> cum;        // arrivals per token up to each event (tp_counts)
};

// Prompt reading on the tensor cores (sml_gpu_prompt_mode level 2; the
// reference's gpu_prefill, sml/sml-gpu-fwd.c:1418, with its tensor-core
// product sml_g_tcm3/tcm9): a prompt's tokens but the last go through in
// chunks of up to kPfChunk, every product the batched path's int8 arithmetic
// (tc_batch.cu: weights re-quantized once, made on first use), each token's
// keys and values written to the decode cache first (k_chunk_kv) and its
// attention then the decode kernel's own (k_attn_seq over (head, token)); the
// last token is stepped through the decode graph, so the logits returned are
// the decode arithmetic's over the cache the chunks filled.
constexpr int kPfChunk = 64;
struct PfGemm { TcPlan p; const int32_t * perm = nullptr; int rows = 0, cols = 0, split = 1; };
struct PfLayer { PfGemm qkv, o, gu, dn; };
struct PfState {
    bool tried = false, ok = false;
    Arena ar;
    std::vector<PfLayer> L;
    int Fp = 0, qkv_ld = 0;
    float * x = nullptr, * qkv = nullptr, * att = nullptr, * hid = nullptr, * xs = nullptr;
    uint8_t * xblk = nullptr;
    int * tok = nullptr, * h_tok = nullptr;
};

struct sb_engine {
    ssf_file f{};
    int n_layer = 0, E = 0, nh = 0, nkv = 0, hd = 0, qd = 0, kvd = 0, F = 0, V = 0, n_ctx = 0;
    float eps = 0.f, theta = 0.f, scale = 0.f;
    int six = 0, minneg = 0;
    Arena ar;
    std::vector<LayerD> L;
    QT emb{};                         // file layout: the embedding lookup reads rows
    TT head{};
    const float * out_norm = nullptr;
    // decode state
    float * x = nullptr, * qkv = nullptr, * att = nullptr, * hp = nullptr, * logits = nullptr;
    uint16_t * kc = nullptr, * vc = nullptr;
    float * rcos = nullptr, * rsin = nullptr;
    int * tok = nullptr, * pos = nullptr, * tlog = nullptr;
    float * am_val = nullptr;
    int * am_idx = nullptr;
    unsigned * am_cnt = nullptr;
    const ExpfEntry * xtab = nullptr;  // the host libm's expf corrections (expf_libm.h)
    float xnear = 0.0f;                // ... looked up within this midpoint distance
    MoeScratch ms;                    // routing scratch shared by every MoE layer (one token)
    uint8_t * hq = nullptr;           // down's input quantized by the gate/up GEMV (TGArgs.hq; one GPU)
    int * err = nullptr;              // bounded waits that gave up
    unsigned long long * trace = nullptr;   // trace build: [launch][cta][8] timestamps
    int n_launch_trace = 0;
    int nsm = 148;
    cudaStream_t st = nullptr;
    cudaGraphExec_t g_tok = nullptr;
    int launches = 0;
    int sync_mode = 0;                // SB_SYNC=1: eager launches, each synchronized and checked
    char cur[64] = {0};               // the kernel being enqueued (for sync-mode errors)
    bool failed = false;
    float * h_logits = nullptr;
    int * h_io = nullptr;
    uint64_t bytes_tok = 0;
    TpState tp;
    int prompt_level = 0;             // sml_gpu_prompt_mode: >= 2 reads prompts on the tensor cores
    PfState pf;
};

// ------------------------------------------------------------------ arena

static void * carve(sb_engine * e, size_t n) { return e->ar.carve(n); }
static const float * up_f32(sb_engine * e, const ssf_rec * r) { return upload_f32(e->ar, e->f, r); }


// ------------------------------------------------------------------ launch

// Count every launch; in sync mode (SB_SYNC=1) finish it and check its error
// flag before the next is enqueued.
static void after_launch(sb_engine * e, cudaError_t r) {
    e->launches++;
    if (e->sync_mode && !e->failed) {
        if (r == cudaSuccess) r = cudaStreamSynchronize(e->st);
        int err = 0;
        if (r == cudaSuccess) r = cudaMemcpy(&err, e->err, 4, cudaMemcpyDeviceToHost);
        if (r != cudaSuccess || err) {
            snprintf(g_err, sizeof g_err, "kernel %s: %s (check code %d)", e->cur,
                     r != cudaSuccess ? cudaGetErrorString(r) : "bounds check failed", err);
            e->failed = true;
        }
    }
}

template <typename... KArgs, typename... Args>
static cudaError_t launch(sb_engine * e, bool pdl, void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          Args &&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = e->st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    const cudaError_t r = cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
    after_launch(e, r);
    return r;
}

template <int NB, int SIX>
static void launch_embed(sb_engine * e, const QT & t) {
    launch(e, true, k_embed<NB, SIX>, dim3((t.cols + 255) / 256), dim3(256), 0, t, (const int *) e->tok, e->x, e->err,
           e->tp.tok_seq);
}

template <int NB, int SIX>
static void launch_tg_nb(sb_engine * e, int mode, const TGArgs & g0, int grid, size_t smem) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_tgemv<NB, SIX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kSmemBudget);
        attr = true;
    }
    TGArgs g = g0;
    g.mode = mode;
    launch(e, true, k_tgemv<NB, SIX>, dim3(grid), dim3(kTgThreads), smem, g);
}

static TGArgs tg_args(sb_engine * e, const TT & t, const float * in, const float * nw, float * out) {
    TGArgs g;
    memset(&g, 0, sizeof g);
    g.t = t;
    g.in = in;
    g.norm_w = nw;
    g.eps = e->eps;
    g.out = out;
    g.trace = e->trace;
    g.launch_id = e->launches;
    g.prefetch = 1;
    g.err = e->err;
    return g;
}

// The GEMV that follows `t` in the token (for the L2 prefetch one kernel ahead).
static void set_next(TGArgs & g, const TT * nt, int nsm) {
    if (!nt) return;
    g.next_tiles = nt->tiles;
    g.next_ntiles = nt->ntiles;
    g.next_grid = nt->ntiles < nsm ? nt->ntiles : nsm;
    g.next_tb = nt->tb;
}

// The exchange of one GEMV launch: `out` is this launch's output pointer in
// this rank's region (its rows go to the same offset in every peer's); raise:
// its CTAs arrive at the peers; wait_ev: the event (index into tp.cum) whose
// arrivals it waits for, -1 none.
static TpX make_tpx(sb_engine * e, bool raise, int wait_ev, float * out) {
    TpState & t = e->tp;
    TpX x;
    memset(&x, 0, sizeof x);
    if (t.n <= 1) return x;
    x.n = t.n; x.rank = t.rank;
    for (int p = 0; p < t.n; p++) {
        x.peer_out[p] = nullptr;
        x.peer_cnt[p] = nullptr;
        if (p == t.rank) continue;
        if (out) x.peer_out[p] = (float *) ((uint8_t *) t.peer[p] + ((uint8_t *) out - t.reg));
        if (raise) x.peer_cnt[p] = (unsigned *) t.peer[p] + t.rank;
    }
    x.cnt = (const unsigned *) t.reg;
    x.tok_seq = t.tok_seq;
    x.c_tok = t.cum.empty() ? 0u : t.cum.back();
    x.wait_count = wait_ev >= 0 ? t.cum[wait_ev] : 0u;
    x.raise = raise ? 1 : 0;
    x.err = e->err;
    return x;
}
static void set_tp(sb_engine * e, TGArgs & g, bool raise, int wait_ev, float * out) {
    if (e->tp.n > 1) g.tp = make_tpx(e, raise, wait_ev, out);
}

// Arrivals per token up to each event (hidden(l) = 2l, x(l) = 2l+1, logits =
// 2 n_layer): the raising kernels' CTA counts, in the order they run.
static void tp_counts(sb_engine * e) {
    TpState & t = e->tp;
    t.cum.clear();
    unsigned c = 0;
    auto grid = [&](const TT & tt) { return (unsigned) (tt.ntiles < e->nsm ? tt.ntiles : e->nsm); };
    for (const LayerD & y : e->L) {
        // an MoE layer: its expert down GEMV (grid nsm) raises x(l); its hidden event is empty
        if (!y.moe) c += grid(y.gateup);
        t.cum.push_back(c);
        c += y.moe ? (unsigned) e->nsm : grid(y.down);
        t.cum.push_back(c);
    }
    c += grid(e->head); t.cum.push_back(c);
}

// One GPU: the gate/up GEMV quantizes the hidden vector for the down GEMV (its
// CTAs take whole groups; TGArgs.grp_tiles) when the groups a CTA takes fit its
// buffer and the block copies in 16-byte units.
static bool hq_plan(const sb_engine * e, const TT & gu, int F) {
    if (!e->hq || e->tp.n > 1 || gu.TR < 2 || gu.TR > 16 || F % 32 || gu.cols < kHqMaxGroups * 32) return false;
    const int ng = F / 32, grid = gu.ntiles < e->nsm ? gu.ntiles : e->nsm;
    return gu.ntiles == ng * (64 / gu.TR) && (ng + grid - 1) / grid <= kHqMaxGroups && (F + ng * 8) % 16 == 0;
}
static void set_hq(sb_engine * e, TGArgs & ffn, TGArgs * down, const LayerD & y) {
    if (!hq_plan(e, y.gateup, e->F)) return;
    ffn.grp_tiles = 64 / y.gateup.TR;
    ffn.hq = e->hq;
    if (down) down->in_act = e->hq;
}

static void launch_tg(sb_engine * e, int mode, const TGArgs & g0) {
    const int grid = g0.t.ntiles < e->nsm ? g0.t.ntiles : e->nsm;
    TGArgs g = g0;
    if (!tg_plan(g)) {
        // not even the staged activation and a two-stage ring fit
        snprintf(g_err, sizeof g_err, "kernel %s: no shared-memory plan for tiles of %u bytes over %d columns",
                 e->cur, g.t.tb, g.t.cols);
        e->failed = true;
        return;
    }
    SB_DISPATCH_QT(g.t.nbits, g.t.six, launch_tg_nb, e, mode, g, grid, tg_smem(g));
}

// Decode attention of layer l (k_attn_seq, one CTA per query head).
static void launch_attn(sb_engine * e, int l) {
    const LayerD & y = e->L[l];
    AttnArgs a;
    memset(&a, 0, sizeof a);
    a.qkv = e->qkv; a.n_head = e->nh; a.n_kv = e->nkv; a.hd = e->hd; a.qd = e->qd; a.kvd = e->kvd;
    a.qn = y.qn; a.kn = y.kn; a.eps = e->eps;
    a.rcos = e->rcos; a.rsin = e->rsin;
    a.kc = e->kc + (size_t) l * e->n_ctx * e->kvd;
    a.vc = e->vc + (size_t) l * e->n_ctx * e->kvd;
    a.n_ctx = e->n_ctx; a.pos = e->pos; a.scale = e->scale;
    a.out = e->att; a.err = e->err; a.xtab = e->xtab; a.xnear = e->xnear;
    a.trace = e->trace; a.launch_id = e->launches;
    auto k = e->hd == 64 ? k_attn_seq<64> : e->hd == 128 ? k_attn_seq<128> : k_attn_seq<256>;
    launch(e, true, k, dim3(e->nh), dim3(kSeqThreads), attn_seq_smem_bytes(e->hd, e->n_ctx), a);
}

// One token: embed, every layer, head and argmax. Enqueued on e->st (captured).
static void enqueue_token(sb_engine * e) {
    snprintf(e->cur, sizeof e->cur, "embed");
    SB_DISPATCH_QT(e->emb.nbits, e->emb.six, launch_embed, e, e->emb);
    for (int l = 0; l < e->n_layer; l++) {
        const LayerD & y = e->L[l];
        snprintf(e->cur, sizeof e->cur, "L%d.qkv", l);
        {
            TGArgs g = tg_args(e, y.qkv, e->x, y.an, e->qkv);
            g.bias = y.qkv_b;
            set_next(g, &y.o, e->nsm);
            set_tp(e, g, false, l > 0 ? 2 * (l - 1) + 1 : -1, nullptr);   // x of the previous layer
            launch_tg(e, GM_QKV, g);
        }
        snprintf(e->cur, sizeof e->cur, "L%d.attn", l);
        launch_attn(e, l);
        snprintf(e->cur, sizeof e->cur, "L%d.o", l);
        {
            TGArgs g = tg_args(e, y.o, e->att, nullptr, e->x);
            set_next(g, y.moe ? nullptr : &y.gateup, e->nsm);
            launch_tg(e, GM_O, g);
        }
        if (y.moe) {
            // router on rmsnorm(x), experts, combine added to x (sml/sml-run.c:3503-3507)
            snprintf(e->cur, sizeof e->cur, "L%d.moe", l);
            // over GPUs: each row of a chosen expert is stored by the GPU holding it
            // into every GPU's per-choice buffer; the combine waits for them (event x(l))
            MoePeerX px;
            MoeScratch ms = e->ms;
            if (e->tp.n > 1) {
                ms.yk = e->ms.yk + (size_t) (l & 1) * y.ml.k * y.ml.E;
                px.dn = make_tpx(e, true, -1, ms.yk);
                px.comb = make_tpx(e, false, 2 * l + 1, nullptr);
            }
            moe_enqueue(y.ml, ms, e->x, 1, y.fn, e->eps, e->x, 1, e->nsm, e->st, true, e->err, e->trace,
                        e->launches, [&](cudaError_t r, const char *) { after_launch(e, r); }, nullptr, e->xtab,
                        e->xnear, MOE_TC_OFF, e->tp.n > 1 ? &px : nullptr);
            continue;
        }
        snprintf(e->cur, sizeof e->cur, "L%d.ffn", l);
        {
            TGArgs g = tg_args(e, y.gateup, e->x, y.fn, e->hp);
            g.ffn_f = y.gateup.rows / 2;
            g.ffn_n = e->F;
            g.scatter = y.down_iperm;
            set_next(g, &y.down, e->nsm);
            set_tp(e, g, true, -1, e->hp);
            set_hq(e, g, nullptr, y);
            launch_tg(e, GM_FFN, g);
        }
        snprintf(e->cur, sizeof e->cur, "L%d.down", l);
        {
            // a tensor-parallel rank's rows are x's rows [E r/tp, ..)
            float * xo = e->x + (size_t) e->E * e->tp.rank / e->tp.n;
            TGArgs g = tg_args(e, y.down, e->hp, nullptr, xo);
            g.in_permuted = 1;
            if (hq_plan(e, y.gateup, e->F)) g.in_act = e->hq;
            set_next(g, l + 1 < e->n_layer ? &e->L[l + 1].qkv : nullptr, e->nsm);
            set_tp(e, g, true, 2 * l, xo);
            launch_tg(e, GM_DOWN, g);
        }
    }
    snprintf(e->cur, sizeof e->cur, "head");
    float * lo = e->logits + (size_t) e->V * e->tp.rank / e->tp.n;
    TGArgs g = tg_args(e, e->head, e->x, e->out_norm, lo);
    g.prefetch = 0;   // larger than L2: streamed, not staged
    if (e->tp.n <= 1) {
        g.am_val = e->am_val; g.am_idx = e->am_idx; g.am_cnt = e->am_cnt;
        g.tok = e->tok; g.pos = e->pos; g.tlog = e->tlog;
    }
    set_tp(e, g, true, 2 * (e->n_layer - 1) + 1, lo);
    launch_tg(e, GM_HEAD, g);
    if (e->tp.n > 1) {
        // the greedy choice over every rank's logits
        snprintf(e->cur, sizeof e->cur, "argmax");
        TGArgs w;
        memset(&w, 0, sizeof w);
        set_tp(e, w, false, 2 * e->n_layer, nullptr);
        launch(e, true, k_tp_argmax, dim3(1), dim3(kArgmaxThreads), 0, (const float *) e->logits, e->V, w.tp,
               e->tok, e->pos, e->tlog);
    }
}

// ------------------------------------------------------------------ open

static void close_all(sb_engine * e) {
    if (e->g_tok) cudaGraphExecDestroy(e->g_tok);
    if (e->st) cudaStreamDestroy(e->st);
    for (int p = 0; p < e->tp.n; p++)
        if (p != e->tp.rank && e->tp.peer[p]) cudaIpcCloseMemHandle(e->tp.peer[p]);
    if (e->tp.reg) cudaFree(e->tp.reg);
    e->pf.ar.release();
    if (e->pf.h_tok) cudaFreeHost(e->pf.h_tok);
    e->ar.release();
    if (e->h_logits) cudaFreeHost(e->h_logits);
    if (e->h_io) cudaFreeHost(e->h_io);
    ssf_close(&e->f);
}

// Bytes one GEMV over t streams per launch (the tiles are exactly those bytes).
static uint64_t tt_bytes(const TT & t) { return (uint64_t) t.ntiles * t.tb; }

static bool build(sb_engine * e, char * why, int nwhy) {
    const ssf_file & f = e->f;
    e->bytes_tok = 0;
    const ssf_rec * er = ssf_find(&f, "token_embd.weight");
    if (!upload_qt(e->ar, f, er, e->emb, why, nwhy)) return false;
    const ssf_rec * hr = ssf_find(&f, "output.weight");
    if (!hr) hr = er;   // tied head (Qwen2.5): the embedding is streamed as the head
    const int min_tiles = 6 * e->nsm;
    constexpr int kTileCap = 12288;
    // in_perm: the input arrives in the tensor's column order (no gather);
    // has_norm: an RMSNorm gain is staged with it
    auto tr_for = [&](const ssf_rec * r, int rows, int even, int in_perm = 0, int has_norm = 1) {
        const int n = (int) r->cols, six = e->six, hm = r->mq_n != 0;
        int tr = pick_tr(rows, (int) tile_geom(n, 1, (int) r->nbits, six, hm).bytes, min_tiles, even, kTileCap);
        // short 4-bit rows: at least 4 a tile where a ring of 8 such tiles
        // fits, so tile_q4 keeps all 32 lanes of a warp busy (long rows keep
        // one or two a tile: more tiles in flight, tile_q4s splits the chains)
        if (r->nbits == 4 && tr < 4 && rows >= 4 && n <= 4096 &&
            ring_stages(stage_layout(n, !in_perm, has_norm, 0, 0).ring_off, tile_geom(n, 4, 4, six, hm).bytes) > 0)
            tr = 4;
        return tr;
    };
    const int tp = e->tp.n, rk = e->tp.rank;
    if ((int) hr->rows % tp || e->E % tp) { snprintf(why, nwhy, "vocab or width not divisible by %d ranks", tp); return false; }
    {
        // this rank's head rows [V r/tp, V (r+1)/tp)
        const int hn = (int) hr->rows / tp, h0 = hn * rk;
        if (!upload_tt(e->ar, f, hr, hn, tr_for(hr, hn, 0), min_tiles, 0,
                       [&](int v) { return RowSrc{v < hn ? hr : nullptr, h0 + v}; }, e->head, why, nwhy))
            return false;
    }
    e->bytes_tok += tt_bytes(e->head);
    e->out_norm = up_f32(e, ssf_find(&f, "output_norm.weight"));
    e->L.assign(e->n_layer, LayerD());
    const MoeLayer * moe0 = nullptr;
    for (int l = 0; l < e->n_layer; l++) {
        LayerD & y = e->L[l];
        auto R = [&](const char * fmt) { return ssf_findf(&f, fmt, l, 0); };
        if (!R("blk.%d.attn_norm.weight") || !R("blk.%d.ffn_norm.weight")) { snprintf(why, nwhy, "layer %d: missing norms", l); return false; }
        const ssf_rec * q = R("blk.%d.attn_q.weight"), * k = R("blk.%d.attn_k.weight"), * v = R("blk.%d.attn_v.weight");
        const ssf_rec * o = R("blk.%d.attn_output.weight"), * gt = R("blk.%d.ffn_gate.weight"), * up = R("blk.%d.ffn_up.weight");
        const ssf_rec * dn = R("blk.%d.ffn_down.weight");
        y.moe = R("blk.%d.ffn_gate_inp.weight") != nullptr;
        if (!q || !k || !v || !o || (!y.moe && (!gt || !up || !dn))) { snprintf(why, nwhy, "layer %d: missing projections", l); return false; }
        if ((int) q->rows != e->qd || (int) k->rows != e->kvd || (int) v->rows != e->kvd || (int) q->cols != e->E ||
            (int) o->rows != e->E || (int) o->cols != e->qd ||
            (!y.moe && ((int) gt->cols != e->E || gt->rows != up->rows || (int) dn->rows != e->E ||
                        dn->cols != gt->rows || gt->rows % 8))) {
            snprintf(why, nwhy, "layer %d: tensor shapes do not match the header", l);
            return false;
        }
        const int F = y.moe ? 0 : (int) gt->rows;
        e->F = F > e->F ? F : e->F;
        // q | k | v as one tensor (they share an input; sml/sml-run.c:1796 groups them)
        if (!upload_tt(e->ar, f, q, e->qd + 2 * e->kvd, tr_for(q, e->qd + 2 * e->kvd, 0), min_tiles, 0, [&](int r) {
                return r < e->qd ? RowSrc{q, r} : r < e->qd + e->kvd ? RowSrc{k, r - e->qd}
                     : r < e->qd + 2 * e->kvd ? RowSrc{v, r - e->qd - e->kvd} : RowSrc{nullptr, 0}; },
                       y.qkv, why, nwhy))
            return false;
        if (y.moe) {
            // over tp GPUs (expert parallelism inside the tensor-parallel engine):
            // this rank's experts [ne r / tp, ne (r + 1) / tp)
            int e_lo = 0, e_hi = 0;
            if (tp > 1) {
                const ssf_rec * rt = R("blk.%d.ffn_gate_inp.weight");
                const int ne = (int) ((uint64_t) rt->rows * rt->cols / e->E);
                if (ne < tp) { snprintf(why, nwhy, "layer %d: %d experts cannot spread over %d GPUs", l, ne, tp); return false; }
                e_lo = (int) ((long) ne * rk / tp);
                e_hi = (int) ((long) ne * (rk + 1) / tp);
            }
            if (!moe_upload(e->ar, f, l, y.ml, why, nwhy, e_lo, e_hi)) return false;
            if (moe0 && (y.ml.E != moe0->E || y.ml.F != moe0->F || y.ml.ne != moe0->ne || y.ml.k != moe0->k)) {
                snprintf(why, nwhy, "layer %d: MoE layers differ in shape", l);
                return false;
            }
            if (!moe0) moe0 = &y.ml;
        }
        // gate / up: a tile of TR rows holds TR/2 gate rows then the same TR/2 up rows
        if (!upload_tt(e->ar, f, o, e->E, tr_for(o, e->E, 0, 0, 0), min_tiles, 0, [&](int r) { return RowSrc{r < e->E ? o : nullptr, r}; },
                       y.o, why, nwhy))
            return false;
        if (!y.moe) {
            {
                // gate/up rows in down's column order (a tile of TR rows holds TR/2 gate rows
                // then the same TR/2 up rows): tile k yields hidden positions k TR/2 ..,
                // written at their place j of the permuted hidden vector, so consecutive
                // tiles give whole groups of down's input. Over tp GPUs this rank takes
                // the positions [F r/tp, F (r+1)/tp) -- whole groups -- and down's rows
                // [E r/tp, ..).
                if (F % (32 * tp)) { snprintf(why, nwhy, "layer %d: FFN %d not in whole groups per rank", l, F); return false; }
                const int fn = F / tp, j0 = fn * rk, en = e->E / tp, e0 = en * rk;
                const int32_t * dperm = (const int32_t *) (f.base + dn->perm_off);
                const int gtr = tr_for(gt, 2 * fn, 1);
                std::vector<int32_t> sc(fn);
                for (int m = 0; m < fn; m++) sc[m] = j0 + m;
                if (!upload_tt(e->ar, f, gt, 2 * fn, gtr, min_tiles, 1, [&](int r) {
                        const int h = gtr / 2, ti = r / gtr, j = r % gtr, m = ti * h + j % h;
                        return m >= fn ? RowSrc{nullptr, 0} : RowSrc{j < h ? gt : up, dperm[j0 + m]}; },
                               y.gateup, why, nwhy) ||
                    !upload_tt(e->ar, f, dn, en, tr_for(dn, en, 0, 1, 0), min_tiles, 0,
                               [&](int r) { return RowSrc{r < en ? dn : nullptr, e0 + r}; }, y.down, why, nwhy))
                    return false;
                y.down_iperm = (const int32_t *) e->ar.upload(sc.data(), sc.size() * 4);
            }
        }
        // per token: the router and the k chosen experts (as tiles)
        e->bytes_tok += tt_bytes(y.qkv) + tt_bytes(y.o) +
                        (y.moe ? y.ml.router_bytes + (uint64_t) y.ml.k * (tt_bytes(y.ml.gu) + tt_bytes(y.ml.dn)) / tp
                               : tt_bytes(y.gateup) + tt_bytes(y.down));
        y.an = up_f32(e, R("blk.%d.attn_norm.weight"));
        y.fn = up_f32(e, R("blk.%d.ffn_norm.weight"));
        const ssf_rec * qb = R("blk.%d.attn_q.bias"), * kb = R("blk.%d.attn_k.bias"), * vb = R("blk.%d.attn_v.bias");
        if (qb || kb || vb) {
            std::vector<float> b((size_t) e->qd + 2 * e->kvd, 0.0f);
            if (qb) memcpy(b.data(), f.base + qb->off, (size_t) e->qd * 4);
            if (kb) memcpy(b.data() + e->qd, f.base + kb->off, (size_t) e->kvd * 4);
            if (vb) memcpy(b.data() + e->qd + e->kvd, f.base + vb->off, (size_t) e->kvd * 4);
            y.qkv_b = (const float *) e->ar.upload(b.data(), b.size() * 4);
        }
        const ssf_rec * qn = R("blk.%d.attn_q_norm.weight"), * kn = R("blk.%d.attn_k_norm.weight");
        if ((qn && qn->rows * qn->cols != (uint32_t) e->hd) || (kn && kn->rows * kn->cols != (uint32_t) e->hd)) {
            snprintf(why, nwhy, "layer %d: Q/K norm over other than one head", l);
            return false;
        }
        y.qn = up_f32(e, qn);
        y.kn = up_f32(e, kn);
    }
    if (e->emb.cols != e->E || e->emb.rows != e->V || e->head.cols != e->E || e->head.rows != e->V / tp) {
        snprintf(why, nwhy, "embedding or head shape does not match the header");
        return false;
    }
    // decode state
    const size_t kv = (size_t) e->n_layer * e->n_ctx * e->kvd * 2;
    e->qkv = (float *) carve(e, (size_t) (e->qd + 2 * e->kvd) * 4);
    e->att = (float *) carve(e, (size_t) e->qd * 4);
    if (tp == 1) {
        e->x = (float *) carve(e, (size_t) e->E * 4);
        e->hp = (float *) carve(e, (size_t) (e->F > 0 ? e->F : 1) * 4);
        e->logits = (float *) carve(e, (size_t) e->V * 4);
        if (e->F > 0) e->hq = (uint8_t *) carve(e, (size_t) e->F + (size_t) (e->F / 32) * 8);
    } else {
        // the exchanged vectors live in the region the peers map: [flags | x | hidden | logits]
        TpState & t = e->tp;
        auto r256 = [](size_t v) { return (v + 255) / 256 * 256; };
        t.off_x = 256;
        t.off_hp = t.off_x + r256((size_t) e->E * 4);
        t.off_lg = t.off_hp + r256((size_t) (e->F > 0 ? e->F : 1) * 4);
        t.off_yk = t.off_lg + r256((size_t) e->V * 4);
        t.reg_bytes = t.off_yk + (moe0 ? r256((size_t) 2 * moe0->k * moe0->E * 4) : 0);
        if (t.reg) {
            e->x = (float *) (t.reg + t.off_x);
            e->hp = (float *) (t.reg + t.off_hp);
            e->logits = (float *) (t.reg + t.off_lg);
        }
        t.tok_seq = (unsigned *) carve(e, 4);
    }
    e->kc = (uint16_t *) carve(e, kv);
    e->vc = (uint16_t *) carve(e, kv);
    e->rcos = (float *) carve(e, (size_t) e->n_ctx * (e->hd / 2) * 4);
    e->rsin = (float *) carve(e, (size_t) e->n_ctx * (e->hd / 2) * 4);
    // tok and pos side by side: one 8-byte copy sets both
    e->tok = (int *) carve(e, 8);
    e->pos = e->tok + 1;
    e->tlog = (int *) carve(e, (size_t) (e->n_ctx + 1) * 4);
    e->am_val = (float *) carve(e, (size_t) 4 * e->nsm * 4);
    e->am_idx = (int *) carve(e, (size_t) 4 * e->nsm * 4);
    e->am_cnt = (unsigned *) carve(e, 4);
    {
        const ExpfTable & xt = expf_libm_table();
        if (xt.slots.empty()) { snprintf(why, nwhy, "this libm's expf differs from the rounded exponential too often"); return false; }
        e->xtab = (const ExpfEntry *) e->ar.upload(xt.slots.data(), xt.slots.size() * sizeof(ExpfEntry));
        e->xnear = xt.near;
    }
    e->err = (int *) carve(e, 4);
    if (moe0) moe_carve(e->ar, *moe0, 1, e->ms);
    // MoE layers over GPUs: the per-choice rows in the region the peers map, one
    // buffer per layer parity -- a peer writes the same buffer again only two
    // layers on, after waiting for an event this GPU raises after its combine
    if (moe0 && tp > 1 && e->tp.reg) e->ms.yk = (float *) (e->tp.reg + e->tp.off_yk);
#ifdef SB_TRACE
    e->n_launch_trace = 8 * e->n_layer + 8;
    e->trace = (unsigned long long *) carve(e, (size_t) e->n_launch_trace * kTraceCtas * 8 * 8);
#endif
    return true;
}


// Average duration of one kernel class of the token, each launch alone on the
// engine's stream (no programmatic overlap), timed by CUDA events, cycling
// over the layers so the weights come from HBM rather than L2 (a layer's
// gate/up is 16 MB, the 28 layers 445 MB). which: 0 q|k|v, 1 attention (at
// the engine's current position), 2 o, 3 gate/up, 4 down, 5 head. bytes_out: the file's bytes of the weights one launch reads.
// Leaves the decode state undefined: call it after generating, not between.
extern "C" int sb_time_kernel(sb_engine * e, int which, int reps, float * ms_avg, double * bytes_out) {
    if (!e || reps < 1 || e->sync_mode) return 0;
    if (which == 3 || which == 4)
        for (const LayerD & y : e->L) if (y.moe) return 0;   // no dense FFN to time
    const ssf_file & f = e->f;
    auto layer_bytes = [&](int l) -> double {
        auto R = [&](const char * fmt) { return ssf_findf(&f, fmt, l, 0); };
        switch (which) {
        case 0: return (double) (ssf_rec_bytes(R("blk.%d.attn_q.weight")) + ssf_rec_bytes(R("blk.%d.attn_k.weight")) +
                                 ssf_rec_bytes(R("blk.%d.attn_v.weight")));
        case 1: return (double) e->kvd * 2 * 2 * (e->n_ctx);   // an upper bound: the whole cache of one layer
        case 2: return (double) ssf_rec_bytes(R("blk.%d.attn_output.weight"));
        case 3: return (double) (ssf_rec_bytes(R("blk.%d.ffn_gate.weight")) + ssf_rec_bytes(R("blk.%d.ffn_up.weight")));
        case 4: return (double) ssf_rec_bytes(R("blk.%d.ffn_down.weight"));
        default: {
            const ssf_rec * h = ssf_find(&f, "output.weight");
            return (double) ssf_rec_bytes(h ? h : ssf_find(&f, "token_embd.weight"));
        }
        }
    };
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    double bytes = 0;
    auto one = [&](int r) {
        const int l = r % e->n_layer;
        const LayerD & y = e->L[l];
        TGArgs g;
        switch (which) {
        case 0: g = tg_args(e, y.qkv, e->x, y.an, e->qkv); g.bias = y.qkv_b; launch_tg(e, GM_QKV, g); break;
        case 1: launch_attn(e, l); break;
        case 2: g = tg_args(e, y.o, e->att, nullptr, e->x); launch_tg(e, GM_O, g); break;
        case 3: g = tg_args(e, y.gateup, e->x, y.fn, e->hp); g.ffn_f = y.gateup.rows / 2; g.ffn_n = e->F;
                g.scatter = y.down_iperm;
                set_hq(e, g, nullptr, y);
                launch_tg(e, GM_FFN, g); break;
        case 4: g = tg_args(e, y.down, e->hp, nullptr, e->x); g.in_permuted = 1;
                if (hq_plan(e, y.gateup, e->F)) g.in_act = e->hq;
                launch_tg(e, GM_DOWN, g); break;
        default: g = tg_args(e, e->head, e->x, e->out_norm, e->logits); g.prefetch = 0;
                 g.am_val = e->am_val; g.am_idx = e->am_idx; g.am_cnt = e->am_cnt;
                 g.tok = e->tok; g.pos = e->pos; g.tlog = nullptr; launch_tg(e, GM_HEAD, g); break;
        }
        bytes += layer_bytes(l);
    };
    for (int r = 0; r < 3; r++) one(r);   // warm-up
    bytes = 0;
    cudaStreamSynchronize(e->st);
    cudaEventRecord(a, e->st);
    for (int r = 0; r < reps; r++) one(r + 3);
    cudaEventRecord(b, e->st);
    const bool ok = ck(cudaStreamSynchronize(e->st), "time kernel");
    float ms = 0;
    cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (ms_avg) *ms_avg = ms / reps;
    if (bytes_out) *bytes_out = bytes / reps;
    return ok ? 1 : 0;
}

// Trace build: copy the per-CTA timestamps of the last token (launch x CTA x 8).
extern "C" int sb_trace(const sb_engine * e, unsigned long long * out, int cap) {
    if (!e->trace) return 0;
    const int n = e->n_launch_trace * kTraceCtas * 8;
    if (cap < n) return 0;
    cudaDeviceSynchronize();
    cudaMemcpy(out, e->trace, (size_t) n * 8, cudaMemcpyDeviceToHost);
    return e->n_launch_trace;
}

// Open, upload and plan (everything but the token graph). tp > 1: this rank's
// slices and its exchange region.
static sb_engine * open_engine(const char * path, int n_ctx, int tp, int rank, char * why, int nwhy) {
    g_err[0] = 0;
    if (tp < 1 || tp > kMaxTp || rank < 0 || rank >= tp) { snprintf(why, nwhy, "rank %d of %d", rank, tp); return nullptr; }
    sb_engine * e = new sb_engine();
    e->tp.n = tp;
    e->tp.rank = rank;
    if (!ssf_open(&e->f, path, why, nwhy)) { delete e; return nullptr; }
    const ssf_hdr * h = e->f.hdr;
    if (const char * u = ssf_unsupported(e->f)) {
        snprintf(why, nwhy, "%s: not on the GPU yet", u);
        close_all(e);
        delete e;
        return nullptr;
    }
    e->n_layer = (int) h->n_layer; e->E = (int) h->n_embd; e->nh = (int) h->n_head; e->nkv = (int) h->n_head_kv;
    e->V = (int) h->n_vocab; e->eps = h->rms_eps; e->theta = h->rope_theta;
    e->six = e->f.scale6; e->minneg = e->f.minneg;
    const ssf_rec * q0 = ssf_find(&e->f, "blk.0.attn_q.weight");
    e->hd = q0 && q0->rows % e->nh == 0 ? (int) q0->rows / e->nh : e->E / e->nh;
    e->qd = e->nh * e->hd;
    e->kvd = e->nkv * e->hd;
    e->scale = h->attn_scale != 0.0f ? h->attn_scale : 1.0f / sqrtf((float) e->hd);
    e->n_ctx = n_ctx > 0 ? n_ctx : 256;
    if (e->n_ctx < 64) e->n_ctx = 64;
    if (h->n_rot && (int) h->n_rot != e->hd) {
        snprintf(why, nwhy, "partial rotary: not on the GPU yet");
        close_all(e); delete e; return nullptr;
    }
    if (e->nh % e->nkv || e->hd % 64 || e->hd > 256) {
        snprintf(why, nwhy, "head layout %d/%d x %d not supported", e->nh, e->nkv, e->hd);
        close_all(e); delete e; return nullptr;
    }
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&e->nsm, cudaDevAttrMultiProcessorCount, dev);
    {
        // decode attention keeps a score per position in shared memory
        int optin = 0;
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        const size_t as = attn_seq_smem_bytes(e->hd, e->n_ctx);
        if (as + 1024 > (size_t) optin || (e->hd != 64 && e->hd != 128 && e->hd != 256) ||
            cudaFuncSetAttribute(e->hd == 64 ? k_attn_seq<64> : e->hd == 128 ? k_attn_seq<128> : k_attn_seq<256>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int) as) != cudaSuccess) {
            snprintf(why, nwhy, "head size %d at n_ctx %d: no decode attention for it (sizes 64, 128, 256; scores in shared memory)", e->hd, e->n_ctx);
            close_all(e); delete e; return nullptr;
        }
    }
    // MoE experts drawn on the device (sb_draw_experts) rather than read
    e->ar.draw_seed = draw_experts_seed();
    e->ar.minneg = e->minneg;
    // pass 1 sizes the arena (and the exchange region), pass 2 fills them
    if (!build(e, why, nwhy)) { close_all(e); delete e; return nullptr; }
    if (!e->ar.allocate()) {
        snprintf(why, nwhy, "cudaMalloc of %.2f GB for the model failed", e->ar.size / 1e9);
        close_all(e); delete e; return nullptr;
    }
    if (tp > 1 && (!ck(cudaMalloc(&e->tp.reg, e->tp.reg_bytes), "exchange region") ||
                   !ck(cudaMemset(e->tp.reg, 0, e->tp.reg_bytes), "exchange region"))) {
        snprintf(why, nwhy, "%s", g_err);
        close_all(e); delete e; return nullptr;
    }
    e->tp.peer[rank] = e->tp.reg;
    if (!build(e, why, nwhy)) { close_all(e); delete e; return nullptr; }
    upload_rope(e->rcos, e->rsin, e->n_ctx, e->hd, e->theta);
    if (!ck(cudaStreamCreateWithFlags(&e->st, cudaStreamNonBlocking), "stream") ||
        !ck(cudaMallocHost(&e->h_logits, (size_t) e->V * 4), "pinned logits") ||
        !ck(cudaMallocHost(&e->h_io, 64 * 4), "pinned io")) {
        snprintf(why, nwhy, "%s", g_err);
        close_all(e); delete e; return nullptr;
    }
    return e;
}

// Capture one token (SB_SYNC=1: no graph, every kernel synchronized and checked).
static bool capture(sb_engine * e) {
    if (e->tp.n > 1) tp_counts(e);
    const char * sm = getenv("SB_SYNC");
    e->sync_mode = sm && atoi(sm) != 0 && e->tp.n == 1;
    cudaGraph_t gr = nullptr;
    e->launches = 0;
    bool ok = true;
    if (!e->sync_mode) {
        ok = ck(cudaStreamBeginCapture(e->st, cudaStreamCaptureModeThreadLocal), "begin capture");
        if (ok) {
            enqueue_token(e);
            ok = ck(cudaStreamEndCapture(e->st, &gr), "end capture");
        }
        ok = ok && ck(cudaGraphInstantiateWithFlags(&e->g_tok, gr, 0), "instantiate");
        if (gr) cudaGraphDestroy(gr);
    }
    return ok && ck(cudaDeviceSynchronize(), "open") && !e->failed;
}

sb_engine * sb_open(const char * path, int n_ctx, char * why, int nwhy) {
    sb_engine * e = open_engine(path, n_ctx, 1, 0, why, nwhy);
    if (e && !capture(e)) {
        snprintf(why, nwhy, "%s", g_err);
        close_all(e); delete e; return nullptr;
    }
    return e;
}

sb_engine * sb_open_tp(const char * path, int n_ctx, int tp, int rank, char * why, int nwhy) {
    if (tp == 1) return sb_open(path, n_ctx, why, nwhy);
    return open_engine(path, n_ctx, tp, rank, why, nwhy);
}

int sb_tp_handle(const sb_engine * e, void * out) {
    if (!e || e->tp.n <= 1 || !out) return 0;
    cudaIpcMemHandle_t h;
    if (!ck(cudaIpcGetMemHandle(&h, e->tp.reg), "cudaIpcGetMemHandle")) return 0;
    static_assert(sizeof h == SB_TP_HANDLE_BYTES, "IPC handle size");
    memcpy(out, &h, sizeof h);
    return 1;
}

int sb_tp_connect(sb_engine * e, const void * handles, char * why, int nwhy) {
    if (!e || e->tp.n <= 1 || !handles || e->g_tok) { snprintf(why, nwhy, "not a tensor-parallel engine awaiting its peers"); return 0; }
    TpState & t = e->tp;
    for (int p = 0; p < t.n; p++) {
        if (p == t.rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, (const uint8_t *) handles + (size_t) p * SB_TP_HANDLE_BYTES, sizeof h);
        if (!ck(cudaIpcOpenMemHandle(&t.peer[p], h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle")) {
            snprintf(why, nwhy, "rank %d: %s", p, g_err);
            return 0;
        }
    }
    if (!capture(e)) { snprintf(why, nwhy, "%s", g_err); return 0; }
    return 1;
}

void sb_close(sb_engine * e) {
    if (!e) return;
    cudaStreamSynchronize(e->st);
    close_all(e);
    delete e;
}

void sb_info(const sb_engine * e, int * out) {
    out[0] = e->n_layer; out[1] = e->E; out[2] = e->nh; out[3] = e->nkv; out[4] = e->hd; out[5] = e->F;
    int ne = 0, k = 0;
    for (const LayerD & y : e->L) if (y.moe) { ne = y.ml.ne; k = y.ml.k; }
    out[6] = e->V; out[7] = e->n_ctx; out[8] = ne; out[9] = k;
    out[10] = (int) (e->bytes_tok & 0xffffffffu); out[11] = (int) (e->bytes_tok >> 32);
    out[12] = 0;
}

uint64_t sb_bytes_per_token(const sb_engine * e) { return e->bytes_tok; }
int sb_launches_per_token(const sb_engine * e) { return e->launches; }
const float * sb_device_logits(const sb_engine * e) { return e->logits; }

static bool set_tok_pos(sb_engine * e, int tok, int pos) {
    e->h_io[0] = tok;
    e->h_io[1] = pos;
    return ck(cudaMemcpyAsync(e->tok, &e->h_io[0], 8, cudaMemcpyHostToDevice, e->st), "tok and pos");
}

// One token through the captured graph, or eagerly with per-kernel checks.
static bool run_token(sb_engine * e) {
    if (!e->sync_mode) return ck(cudaGraphLaunch(e->g_tok, e->st), "graph launch");
    enqueue_token(e);
    return !e->failed;
}

// After a synchronize: the kernels' error flag (a bounded wait that gave up, a
// failed check) makes the call fail with its code.
static bool report_err(int err) {
    if (err) {
        snprintf(g_err, sizeof g_err, "a kernel reported error code %d (%s)", err,
                 err == 7 ? "a tensor-parallel peer's event did not arrive" : "a bounded wait or check");
        return false;
    }
    return true;
}
static bool check_err(sb_engine * e) {
    int err = 0;
    if (!ck(cudaMemcpy(&err, e->err, 4, cudaMemcpyDeviceToHost), "error flag")) return false;
    if (err) {
        snprintf(g_err, sizeof g_err, "a kernel reported error code %d (%s)", err,
                 err == 7 ? "a tensor-parallel peer's event did not arrive" : "a bounded wait or check");
        return false;
    }
    return true;
}

const float * sb_step(sb_engine * e, int tok, int pos) {
    if (!e || pos < 0 || pos >= e->n_ctx || tok < 0 || tok >= e->V) return nullptr;
    if (!set_tok_pos(e, tok, pos)) return nullptr;
    if (!run_token(e)) return nullptr;
    // the logits and the kernels' error flag come back with one synchronization
    if (!ck(cudaMemcpyAsync(e->h_logits, e->logits, (size_t) e->V * 4, cudaMemcpyDeviceToHost, e->st), "logits") ||
        !ck(cudaMemcpyAsync(&e->h_io[63], e->err, 4, cudaMemcpyDeviceToHost, e->st), "error flag"))
        return nullptr;
    if (!ck(cudaStreamSynchronize(e->st), "step") || !report_err(e->h_io[63])) return nullptr;
    return e->h_logits;
}

// ------------------------------------------------------------------ prompt chunks

static int pf_split(int tiles, int nsb, int nsm) {
    // superblock slices that fill the SMs: the fewest waves times the
    // superblocks a CTA walks (plus about two per CTA)
    int best = 1;
    double bc = 1e30;
    for (int sp = 1; sp <= nsb && sp <= kTcMaxSplit; sp++) {
        if (tc_split(nsb, sp) != sp) continue;
        const int per = (nsb + sp - 1) / sp, waves = (tiles * sp + nsm - 1) / nsm;
        const double cost = waves * (per + 2.0) + (sp > 1 ? 0.25 : 0.0);
        if (cost < bc - 1e-9) { bc = cost; best = sp; }
    }
    return best;
}

// One product of the chunk path: the tensors `recs` stacked (segments on 128
// rows), re-quantized for the tensor cores (sizing pass: carve only).
static bool pf_gemm(sb_engine * e, PfGemm & gm, const std::vector<const ssf_rec *> & recs, char * why, int nwhy) {
    Arena & ar = e->pf.ar;
    const ssf_rec * r0 = recs[0];
    int rows_pad = 0;
    for (const ssf_rec * r : recs) rows_pad += ((int) r->rows + 127) / 128 * 128;
    gm.rows = recs.size() == 1 ? (int) r0->rows : rows_pad;
    gm.cols = (int) r0->cols;
    QT meta;
    if (!upload_qt_meta(ar, e->f, r0, meta, why, nwhy)) return false;
    gm.perm = meta.perm;
    gm.p.rows_pad = rows_pad;
    gm.p.nsb = (gm.cols / SSF_GROUP + 7) / 8;
    gm.p.wblk = (uint8_t *) ar.carve((size_t) rows_pad * gm.p.nsb * 256);
    gm.p.s8 = (float *) ar.carve((size_t) gm.p.nsb * rows_pad * 4);
    gm.split = pf_split(rows_pad / 128, gm.p.nsb, e->nsm);
    if (!gm.p.wblk) return true;
    int off = 0;
    for (const ssf_rec * r : recs) {
        Arena tmp;
        QT t;
        bool ok = upload_qt(tmp, e->f, r, t, why, nwhy) && tmp.allocate() && upload_qt(tmp, e->f, r, t, why, nwhy);
        ok = ok && tc_requant(t, gm.p, off, e->st) == cudaSuccess && cudaStreamSynchronize(e->st) == cudaSuccess;
        tmp.release();
        if (!ok) { if (!why[0]) snprintf(why, nwhy, "%.64s: re-quantization failed", r->name); return false; }
        off += ((int) r->rows + 127) / 128 * 128;
    }
    return true;
}

static bool pf_layout(sb_engine * e, char * why, int nwhy) {
    PfState & P = e->pf;
    const ssf_file & f = e->f;
    P.L.assign(e->n_layer, PfLayer());
    for (int l = 0; l < e->n_layer; l++) {
        auto R = [&](const char * fmt) { return ssf_findf(&f, fmt, l, 0); };
        PfLayer & y = P.L[l];
        if (!pf_gemm(e, y.qkv, {R("blk.%d.attn_q.weight"), R("blk.%d.attn_k.weight"), R("blk.%d.attn_v.weight")}, why, nwhy) ||
            !pf_gemm(e, y.o, {R("blk.%d.attn_output.weight")}, why, nwhy) ||
            !pf_gemm(e, y.gu, {R("blk.%d.ffn_gate.weight"), R("blk.%d.ffn_up.weight")}, why, nwhy) ||
            !pf_gemm(e, y.dn, {R("blk.%d.ffn_down.weight")}, why, nwhy))
            return false;
    }
    P.Fp = (e->F + 127) / 128 * 128;
    P.qkv_ld = P.L[0].qkv.p.rows_pad;
    int wide = e->E > e->qd ? e->E : e->qd;
    wide = wide > e->F ? wide : e->F;
    const int nsb = (wide / SSF_GROUP + 7) / 8;
    P.x = (float *) P.ar.carve((size_t) kPfChunk * e->E * 4);
    P.qkv = (float *) P.ar.carve((size_t) kPfChunk * P.qkv_ld * 4);
    P.att = (float *) P.ar.carve((size_t) kPfChunk * e->qd * 4);
    P.hid = (float *) P.ar.carve((size_t) kPfChunk * 2 * P.Fp * 4);
    P.xblk = (uint8_t *) P.ar.carve((size_t) kPfChunk * nsb * 256);
    P.xs = (float *) P.ar.carve((size_t) nsb * kPfChunk * 4);
    P.tok = (int *) P.ar.carve((size_t) kPfChunk * 4);
    return true;
}

// Make the chunk path on first use: dense decoders on one GPU whose q|k|v
// segments need no padding (the fused product's rows are then the decode
// engine's q|k|v order, biases included).
static bool pf_ready(sb_engine * e) {
    PfState & P = e->pf;
    if (P.tried) return P.ok;
    P.tried = true;
    if (e->tp.n > 1 || e->qd % 128 || e->kvd % 128 || e->F <= 0) return false;
    for (const LayerD & y : e->L) if (y.moe) return false;
    char why[256] = {0};
    if (!pf_layout(e, why, sizeof why) || !P.ar.allocate() || !pf_layout(e, why, sizeof why) ||
        cudaMallocHost(&P.h_tok, kPfChunk * 4) != cudaSuccess) {
        P.ar.release();
        snprintf(g_err, sizeof g_err, "tensor-core prompt path unavailable: %s", why[0] ? why : "allocation failed");
        return false;
    }
    P.ok = true;
    return true;
}

template <int NB, int SIX>
static void pf_embed(sb_engine * e, int T) {
    k_embed_rows<NB, SIX><<<dim3((e->E + 255) / 256, T), 256, 0, e->st>>>(e->emb, e->pf.tok, e->pf.x, e->err);
}

// Positions pos0 .. pos0 + n - 1 of the prompt through the chunk path (the
// cache rows written; no logits).
static bool prefill_chunks(sb_engine * e, const int * ids, int pos0, int n) {
    PfState & P = e->pf;
    for (int c0 = 0; c0 < n; c0 += kPfChunk) {
        const int T = n - c0 < kPfChunk ? n - c0 : kPfChunk, Tp = tc_tokens_pad(T), N = tc_tile_n(T);
        if (!ck(cudaStreamSynchronize(e->st), "prefill")) return false;   // the staging buffer is reused
        memcpy(P.h_tok, ids + c0, (size_t) T * 4);
        if (!ck(cudaMemcpyAsync(P.tok, P.h_tok, (size_t) T * 4, cudaMemcpyHostToDevice, e->st), "prompt ids")) return false;
        SB_DISPATCH_QT(e->emb.nbits, e->emb.six, pf_embed, e, T);
        auto quant = [&](int mode, const PfGemm & gm, const float * x, int ldx, const float * gain, int up_off) {
            TcQuantArgs q;
            memset(&q, 0, sizeof q);
            q.x = x; q.ldx = ldx; q.up_off = up_off; q.perm = gm.perm; q.gain = gain; q.eps = e->eps;
            q.cols = gm.cols; q.T = T; q.T_pad = Tp; q.N = N; q.nsb = gm.p.nsb; q.xblk = P.xblk; q.xs = P.xs;
            return tc_quant(mode, q, e->st);
        };
        auto mma = [&](const PfGemm & gm, float * y, int ldy, const float * bias, int acc) {
            TcArgs a;
            memset(&a, 0, sizeof a);
            a.wblk = gm.p.wblk; a.s8 = gm.p.s8; a.xblk = P.xblk; a.xs = P.xs; a.y = y; a.ldy = ldy; a.bias = bias;
            a.accumulate = acc; a.rows = gm.rows; a.rows_pad = gm.p.rows_pad; a.nsb = gm.p.nsb; a.T = T; a.T_pad = Tp;
            a.split = gm.split; a.err = e->err;
            return tc_mma(a, e->st);
        };
        for (int l = 0; l < e->n_layer; l++) {
            const LayerD & y = e->L[l];
            const PfLayer & z = P.L[l];
            uint16_t * kc = e->kc + (size_t) l * e->n_ctx * e->kvd, * vc = e->vc + (size_t) l * e->n_ctx * e->kvd;
            cudaError_t r = quant(TQ_NORM, z.qkv, P.x, e->E, y.an, 0);
            if (r == cudaSuccess) r = mma(z.qkv, P.qkv, P.qkv_ld, y.qkv_b, 0);
            if (r == cudaSuccess) {
                auto kk = e->hd == 64 ? k_chunk_kv<64> : e->hd == 128 ? k_chunk_kv<128> : k_chunk_kv<256>;
                kk<<<dim3(e->nkv, T), 128, 0, e->st>>>(P.qkv, P.qkv_ld, e->qd, e->kvd, y.kn, e->eps, e->rcos, e->rsin,
                                                      kc, vc, pos0 + c0);
                r = cudaGetLastError();
            }
            if (r == cudaSuccess) {
                AttnArgs a;
                memset(&a, 0, sizeof a);
                a.qkv = P.qkv; a.qkv_ld = P.qkv_ld; a.n_head = e->nh; a.n_kv = e->nkv; a.hd = e->hd; a.qd = e->qd;
                a.kvd = e->kvd; a.qn = y.qn; a.kn = y.kn; a.eps = e->eps; a.rcos = e->rcos; a.rsin = e->rsin;
                a.kc = kc; a.vc = vc; a.n_ctx = e->n_ctx; a.pos = nullptr; a.pos_imm = pos0 + c0; a.scale = e->scale;
                a.out = P.att; a.out_ld = e->qd; a.err = e->err; a.xtab = e->xtab; a.xnear = e->xnear;
                auto ka = e->hd == 64 ? k_attn_seq<64> : e->hd == 128 ? k_attn_seq<128> : k_attn_seq<256>;
                ka<<<dim3(e->nh, T), kSeqThreads, attn_seq_smem_bytes(e->hd, e->n_ctx), e->st>>>(a);
                r = cudaGetLastError();
            }
            if (r == cudaSuccess) r = quant(TQ_PLAIN, z.o, P.att, e->qd, nullptr, 0);
            if (r == cudaSuccess) r = mma(z.o, P.x, e->E, nullptr, 1);
            if (r == cudaSuccess) r = quant(TQ_NORM, z.gu, P.x, e->E, y.fn, 0);
            if (r == cudaSuccess) r = mma(z.gu, P.hid, 2 * P.Fp, nullptr, 0);
            if (r == cudaSuccess) r = quant(TQ_SILU, z.dn, P.hid, 2 * P.Fp, nullptr, P.Fp);
            if (r == cudaSuccess) r = mma(z.dn, P.x, e->E, nullptr, 1);
            if (!ck(r, "prompt chunk")) return false;
        }
    }
    return true;
}

int sb_kv_rows(const sb_engine * e, int layer, int pos, uint16_t * k, uint16_t * v) {
    if (!e || layer < 0 || layer >= e->n_layer || pos < 0 || pos >= e->n_ctx || !k || !v) return 0;
    const size_t at = ((size_t) layer * e->n_ctx + pos) * e->kvd;
    return cudaMemcpy(k, e->kc + at, (size_t) e->kvd * 2, cudaMemcpyDeviceToHost) == cudaSuccess &&
           cudaMemcpy(v, e->vc + at, (size_t) e->kvd * 2, cudaMemcpyDeviceToHost) == cudaSuccess;
}

int sb_prompt_splits(sb_engine * e, int * out5) {
    if (!e || !out5 || !pf_ready(e)) return 0;
    const PfLayer & z = e->pf.L[0];
    out5[0] = z.qkv.split; out5[1] = z.o.split; out5[2] = z.gu.split; out5[3] = z.dn.split; out5[4] = 1;
    return 1;
}

int sb_set_prompt_mode(sb_engine * e, int level) {
    if (!e) return 0;
    e->prompt_level = level < 0 ? 0 : level > 2 ? 2 : level;
    return e->prompt_level;
}

const float * sb_prefill(sb_engine * e, const int * ids, int pos0, int n) {
    if (!e || n <= 0 || pos0 < 0 || pos0 + n > e->n_ctx) return nullptr;
    for (int i = 0; i < n; i++)
        if (ids[i] < 0 || ids[i] >= e->V) return nullptr;
    int i0 = 0;
    if (e->prompt_level >= 2 && n >= 2 && pf_ready(e)) {
        // every token but the last through the chunk path, then the last stepped
        if (!prefill_chunks(e, ids, pos0, n - 1)) return nullptr;
        i0 = n - 1;
    }
    for (int i = i0; i < n; i++) {
        if (ids[i] < 0 || ids[i] >= e->V) return nullptr;
        // each token's id must reach the device before its graph runs; every
        // staging slot is its own pinned word, reused only after a sync
        const int slot = 2 + (i % 30) * 2;
        e->h_io[slot] = ids[i];
        e->h_io[slot + 1] = pos0 + i;
        if (!ck(cudaMemcpyAsync(e->tok, &e->h_io[slot], 8, cudaMemcpyHostToDevice, e->st), "tok and pos") ||
            !run_token(e))
            return nullptr;
        if (i % 30 == 29) { if (!ck(cudaStreamSynchronize(e->st), "prefill") || !check_err(e)) return nullptr; }
    }
    if (!ck(cudaMemcpyAsync(e->h_logits, e->logits, (size_t) e->V * 4, cudaMemcpyDeviceToHost, e->st), "logits")) return nullptr;
    if (!ck(cudaStreamSynchronize(e->st), "prefill") || !check_err(e)) return nullptr;
    return e->h_logits;
}

// Greedy generation on the device: the prompt stepped from position 0, then
// nwarm + ngen tokens, each chosen on the GPU and fed back by graph replay. ms
// (if not NULL) times the last ngen replays by CUDA events on the stream.
static int generate(sb_engine * e, const int * prompt, int np, int nwarm, int ngen, int * out_ids, float * ms) {
    const int total = nwarm + ngen;
    if (!e || np < 1 || nwarm < 0 || ngen < 1 || np + total > e->n_ctx + 1) return 0;
    if (!sb_prefill(e, prompt, 0, np)) return 0;
    // the head of the last prompt token has written tok = argmax, pos = np and
    // tlog[np-1]; each replay reads them and writes the next
    for (int g = 0; g < nwarm; g++)
        if (!run_token(e)) return 0;
    cudaEvent_t a = nullptr, b = nullptr;
    if (ms) {
        if (!ck(cudaStreamSynchronize(e->st), "generate")) return 0;
        cudaEventCreate(&a);
        cudaEventCreate(&b);
        cudaEventRecord(a, e->st);
    }
    for (int g = 0; g + 1 < ngen; g++)
        if (!run_token(e)) return 0;
    if (ms) cudaEventRecord(b, e->st);
    if (!ck(cudaMemcpyAsync(out_ids, e->tlog + np - 1, (size_t) total * 4, cudaMemcpyDeviceToHost, e->st), "ids"))
        return 0;
    if (!ck(cudaStreamSynchronize(e->st), "generate") || !check_err(e)) return 0;
    if (ms) {
        cudaEventElapsedTime(ms, a, b);
        cudaEventDestroy(a);
        cudaEventDestroy(b);
    }
    return 1;
}

int sb_generate(sb_engine * e, const int * prompt, int np, int ngen, int * out_ids) {
    return generate(e, prompt, np, 0, ngen, out_ids, nullptr);
}

int sb_generate_timed(sb_engine * e, const int * prompt, int np, int nwarm, int ngen, int * out_ids, float * ms_out) {
    return generate(e, prompt, np, nwarm, ngen, out_ids, ms_out);
}

