// Batched serving on the GPU: n_seq conversations decode together, one token
// each per step and one read of the weights per step (the CPU's
// sml_forward_multi, sml/sml-run.c:2559-2604, driven by sml-batched,
// sml/sml-batched.c:43-146). Every product runs on the tensor cores with the
// reference's batched arithmetic (int8 re-quantized weights, per-256
// activations, tc_batch.cu); attention, the norms, RoPE and the greedy choice
// are each sequence's own (batch.cuh).
//
// Per step, one captured graph:
//   k_bembed
//   per layer: quant(norm) -> q|k|v GEMM (+ bias) -> k_battn
//              -> quant -> o GEMM (x +=) -> quant(norm) -> gate|up GEMM
//              -> quant(silu) -> down GEMM (x +=)
//   quant(norm) -> head GEMM -> k_bargmax (next token, position + 1)
// A mixture-of-experts layer replaces the gate|up/down products by the MoE
// FFN over the n_seq rows (moe_host.h: router with its RMSNorm, grouped
// gate/up and down GEMVs over the chosen experts' Q4 tiles, choice-order
// combine added to x), as the CPU's batched step runs moe_ffn per row
// (sml/sml-run.c:3182 moe_ffn_batch).
//
// HBM layout: the int8 weights as 32 KB (128 rows x 256 columns) blocks in the
// tensor cores' operand layout, q|k|v and gate|up each one tensor (segments
// padded to 128 rows); the KV cache in pages of 64 positions,
// [layer][page][kv head][64][hd] fp16, so a chunk of one head's positions is
// one contiguous copy. Each slot reads its positions through a page table
// ([slot][n_ctx / 64] page ids): fixed pages per slot for sb_batch_open
// (slot s owns pages s * maxp ..), or pages from a shared pool that
// sequences take as they grow and give back when freed (sb_batch_open_paged,
// sb_forward_seqs): continuous batching, where a sequence joins or leaves the
// step between any two steps and may run in any slot.
#include "batch.cuh"
#include "moe_host.h"
#include "tc_batch.h"
#include "sheep_b200.h"
#include "ssf.h"
#include "upload.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

using namespace sb;

static thread_local char g_berr[512];

const char * sb_batch_last_error(void) { return g_berr; }

static bool bck(cudaError_t e, const char * what) {
    if (e == cudaSuccess) return true;
    snprintf(g_berr, sizeof g_berr, "%s: %s", what, cudaGetErrorString(e));
    return false;
}

namespace {

// One product of the step: the re-quantized weights, the input's column order,
// and the number of superblock slices.
struct BGemm {
    TcPlan p;
    const int32_t * perm = nullptr;
    int rows = 0, cols = 0, split = 1;
    uint64_t file_bytes = 0;          // the file's bytes of the tensors (codes + fields)
};

struct BLayer {
    BGemm qkv, o, gu, dn;
    const float * an = nullptr, * fn = nullptr, * qkv_b = nullptr, * qn = nullptr, * kn = nullptr;
    bool moe = false;                 // MoE FFN in place of gate|up / down
    MoeLayer ml;
};

int round128(int n) { return (n + 127) / 128 * 128; }

// Slices of the superblocks so that the tiles fill the SMs: the fewest waves
// times the superblocks a CTA walks (plus a fixed cost per CTA of about two).
int pick_split(int tiles, int nsb, int nsm) {
    int best = 1;
    double bc = 1e30;
    for (int s = 1; s <= nsb && s <= kTcMaxSplit; s++) {
        if (tc_split(nsb, s) != s) continue;
        const int per = (nsb + s - 1) / s;
        const int waves = (tiles * s + nsm - 1) / nsm;
        const double cost = waves * (per + 2.0) + (s > 1 ? 0.25 : 0.0);
        if (cost < bc - 1e-9) { bc = cost; best = s; }
    }
    return best;
}

}  // namespace

struct sb_batch {
    ssf_file f{};
    int n_layer = 0, E = 0, nh = 0, nkv = 0, hd = 0, qd = 0, kvd = 0, F = 0, Fp = 0, V = 0, n_ctx = 0, B = 0;
    int qkv_rows = 0, koff = 0, voff = 0;
    float eps = 0.f, theta = 0.f, scale = 0.f;
    int nsm = 148, T_pad = 16, N = 16;
    Arena ar;
    std::vector<BLayer> L;
    QT emb{};
    BGemm head;
    const float * out_norm = nullptr;
    float * x = nullptr, * qkv = nullptr, * att = nullptr, * hid = nullptr, * logits = nullptr;
    uint16_t * kc = nullptr, * vc = nullptr;
    float * rcos = nullptr, * rsin = nullptr;
    int maxp = 0, n_pages = 0;        // pages of 64 positions a sequence can hold; pages in the cache
    int * pages = nullptr;            // device [B][maxp]: each slot's page table for the step
    int * h_pages = nullptr;          // pinned staging of the tables (paged handles)
    bool paged = false;               // sequences on pooled pages (sb_forward_seqs), not fixed slots
    std::vector<std::vector<int>> seq_pages;   // paged: each sequence's pages in position order
    std::vector<char> seq_live;
    std::vector<int> free_pages, free_seqs;
    int * tok = nullptr, * pos = nullptr, * tlog = nullptr;
    uint8_t * xblk = nullptr;
    float * xs = nullptr, * apart = nullptr;
    unsigned * acnt = nullptr;
    int attn_split = 1, attn_hg = 4, attn_groups = 1;
    int attn_t = 0;                   // k_battn_t with 1 or 2 n-tiles of 8 heads (hd 64, 128); 0: k_battn
    int * err = nullptr;
    cudaStream_t st = nullptr;
    cudaGraphExec_t g = nullptr;
    int launches = 0;
    int sync_mode = 0;
    bool failed = false;
    char cur[64] = {0};
    float * h_logits = nullptr;
    int * h_io = nullptr;             // [2][n_seq] staging of tokens and positions
    uint64_t bytes_file = 0, bytes_i8 = 0;
    MoeScratch ms;                    // routing scratch for n_seq rows, shared by the MoE layers
    uint64_t bytes_experts = 0;       // every MoE layer's experts and router, as stored
};

static void b_after(sb_batch * b, cudaError_t r) {
    b->launches++;
    if (r != cudaSuccess && !b->failed) {
        snprintf(g_berr, sizeof g_berr, "kernel %s: %s", b->cur, cudaGetErrorString(r));
        b->failed = true;
    }
    if (b->sync_mode && !b->failed) {
        r = cudaStreamSynchronize(b->st);
        int err = 0;
        if (r == cudaSuccess) r = cudaMemcpy(&err, b->err, 4, cudaMemcpyDeviceToHost);
        if (r != cudaSuccess || err) {
            snprintf(g_berr, sizeof g_berr, "kernel %s: %s (check code %d)", b->cur,
                     r != cudaSuccess ? cudaGetErrorString(r) : "a bounded wait or check failed", err);
            b->failed = true;
        }
    }
}

// ------------------------------------------------------------------ upload

// The plan of a GEMM whose rows are the tensors `recs` stacked, each segment
// starting on a multiple of 128 rows; the input's column order is the first
// tensor's, and every tensor must share it.
static bool b_gemm(sb_batch * b, BGemm & gm, const std::vector<const ssf_rec *> & recs, char * why, int nwhy) {
    const ssf_rec * r0 = recs[0];
    int rows_pad = 0;
    gm.rows = 0;
    gm.file_bytes = 0;
    for (const ssf_rec * r : recs) {
        if (r->cols != r0->cols || r->perm_off != r0->perm_off) {
            snprintf(why, nwhy, "%.64s: fused tensors differ in width or column order", r->name);
            return false;
        }
        rows_pad += round128((int) r->rows);
        gm.file_bytes += ssf_rec_bytes(r);
    }
    // a single tensor's product writes its own rows; a fused one every padded row
    gm.rows = recs.size() == 1 ? (int) r0->rows : rows_pad;
    gm.cols = (int) r0->cols;
    QT meta;
    if (!upload_qt_meta(b->ar, b->f, r0, meta, why, nwhy)) return false;
    gm.perm = meta.perm;
    gm.p.rows_pad = rows_pad;
    gm.p.nsb = (gm.cols / SSF_GROUP + 7) / 8;
    gm.p.wblk = (uint8_t *) b->ar.carve((size_t) rows_pad * gm.p.nsb * 256);
    gm.p.s8 = (float *) b->ar.carve((size_t) gm.p.nsb * rows_pad * 4);
    gm.split = pick_split((rows_pad / 128) * (b->T_pad / b->N), gm.p.nsb, b->nsm);
    b->bytes_file += gm.file_bytes;
    b->bytes_i8 += (uint64_t) rows_pad * gm.p.nsb * (256 + 4);
    if (!gm.p.wblk) return true;   // sizing pass
    // re-quantize each tensor into its segment from a temporary upload of its planes
    int off = 0;
    for (const ssf_rec * r : recs) {
        Arena tmp;
        QT t;
        if (!upload_qt(tmp, b->f, r, t, why, nwhy)) return false;
        if (!tmp.allocate()) { snprintf(why, nwhy, "cudaMalloc for the re-quantization failed"); return false; }
        bool ok = upload_qt(tmp, b->f, r, t, why, nwhy);
        ok = ok && tc_requant(t, gm.p, off, b->st) == cudaSuccess && cudaStreamSynchronize(b->st) == cudaSuccess;
        tmp.release();
        if (!ok) {
            if (!why[0]) snprintf(why, nwhy, "%.64s: re-quantization failed", r->name);
            return false;
        }
        off += round128((int) r->rows);
    }
    return true;
}

static const float * b_f32(sb_batch * b, const ssf_rec * r) { return upload_f32(b->ar, b->f, r); }

static bool b_build(sb_batch * b, char * why, int nwhy) {
    const ssf_file & f = b->f;
    b->bytes_file = b->bytes_i8 = 0;
    const ssf_rec * er = ssf_find(&f, "token_embd.weight");
    if (!upload_qt(b->ar, f, er, b->emb, why, nwhy)) return false;
    const ssf_rec * hr = ssf_find(&f, "output.weight");
    if (!b_gemm(b, b->head, {hr ? hr : er}, why, nwhy)) return false;
    b->out_norm = b_f32(b, ssf_find(&f, "output_norm.weight"));
    b->L.assign(b->n_layer, BLayer());
    b->F = 0;
    b->bytes_experts = 0;
    const MoeLayer * moe0 = nullptr;
    bool dense_seen = false;
    for (int l = 0; l < b->n_layer; l++) {
        BLayer & y = b->L[l];
        auto R = [&](const char * fmt) { return ssf_findf(&f, fmt, l, 0); };
        y.moe = R("blk.%d.ffn_gate_inp.weight") != nullptr;
        const ssf_rec * q = R("blk.%d.attn_q.weight"), * k = R("blk.%d.attn_k.weight"), * v = R("blk.%d.attn_v.weight");
        const ssf_rec * o = R("blk.%d.attn_output.weight"), * gt = R("blk.%d.ffn_gate.weight");
        const ssf_rec * up = R("blk.%d.ffn_up.weight"), * dn = R("blk.%d.ffn_down.weight");
        if (!q || !k || !v || !o || (!y.moe && (!gt || !up || !dn)) || !R("blk.%d.attn_norm.weight") ||
            !R("blk.%d.ffn_norm.weight")) {
            snprintf(why, nwhy, "layer %d: missing tensors", l);
            return false;
        }
        if ((int) q->rows != b->qd || (int) k->rows != b->kvd || (int) v->rows != b->kvd || (int) q->cols != b->E ||
            (int) o->rows != b->E || (int) o->cols != b->qd ||
            (!y.moe && ((int) gt->cols != b->E || gt->rows != up->rows || (int) dn->rows != b->E || dn->cols != gt->rows))) {
            snprintf(why, nwhy, "layer %d: tensor shapes do not match the header", l);
            return false;
        }
        if (!b_gemm(b, y.qkv, {q, k, v}, why, nwhy) || !b_gemm(b, y.o, {o}, why, nwhy)) return false;
        if (y.moe) {
            if (!moe_upload(b->ar, f, l, y.ml, why, nwhy)) return false;
            if (moe0 && (y.ml.E != moe0->E || y.ml.F != moe0->F || y.ml.ne != moe0->ne || y.ml.k != moe0->k)) {
                snprintf(why, nwhy, "layer %d: MoE shapes differ between layers", l);
                return false;
            }
            if (!moe0) moe0 = &y.ml;
            b->bytes_experts += (uint64_t) y.ml.ne * y.ml.expert_file_bytes + y.ml.router_bytes;
        } else {
            if (!dense_seen) b->F = (int) gt->rows;
            dense_seen = true;
            if ((int) gt->rows != b->F) { snprintf(why, nwhy, "layer %d: FFN widths differ", l); return false; }
            if (!b_gemm(b, y.gu, {gt, up}, why, nwhy) || !b_gemm(b, y.dn, {dn}, why, nwhy)) return false;
        }
        y.an = b_f32(b, R("blk.%d.attn_norm.weight"));
        y.fn = b_f32(b, R("blk.%d.ffn_norm.weight"));
        const ssf_rec * qb = R("blk.%d.attn_q.bias"), * kb = R("blk.%d.attn_k.bias"), * vb = R("blk.%d.attn_v.bias");
        if (qb || kb || vb) {
            // biases in the padded q | k | v row order of the fused product
            std::vector<float> bias((size_t) y.qkv.rows, 0.0f);
            if (qb) memcpy(bias.data(), f.base + qb->off, (size_t) b->qd * 4);
            if (kb) memcpy(bias.data() + b->koff, f.base + kb->off, (size_t) b->kvd * 4);
            if (vb) memcpy(bias.data() + b->voff, f.base + vb->off, (size_t) b->kvd * 4);
            y.qkv_b = (const float *) b->ar.upload(bias.data(), bias.size() * 4);
        }
        const ssf_rec * qn = R("blk.%d.attn_q_norm.weight"), * kn = R("blk.%d.attn_k_norm.weight");
        if ((qn && qn->rows * qn->cols != (uint32_t) b->hd) || (kn && kn->rows * kn->cols != (uint32_t) b->hd)) {
            snprintf(why, nwhy, "layer %d: Q/K norm over other than one head", l);
            return false;
        }
        y.qn = b_f32(b, qn);
        y.kn = b_f32(b, kn);
    }
    if (b->emb.cols != b->E || b->emb.rows != b->V || b->head.cols != b->E || (hr ? (int) hr->rows : b->V) != b->V) {
        snprintf(why, nwhy, "embedding or head shape does not match the header");
        return false;
    }
    b->Fp = round128(b->F);
    if (moe0) moe_carve(b->ar, *moe0, b->B, b->ms);
    // step state
    const int B = b->B, Tp = b->T_pad;
    int wide = b->E > b->qd ? b->E : b->qd;
    wide = wide > b->F ? wide : b->F;
    const int nsb_max = (wide / SSF_GROUP + 7) / 8;
    b->x = (float *) b->ar.carve((size_t) B * b->E * 4);
    b->qkv = (float *) b->ar.carve((size_t) B * b->qkv_rows * 4);
    b->att = (float *) b->ar.carve((size_t) B * b->qd * 4);
    b->hid = (float *) b->ar.carve((size_t) B * 2 * b->Fp * 4);
    b->logits = (float *) b->ar.carve((size_t) B * b->head.rows * 4);
    const size_t kv = (size_t) b->n_layer * b->n_pages * b->nkv * 64 * b->hd * 2;
    b->kc = (uint16_t *) b->ar.carve(kv);
    b->vc = (uint16_t *) b->ar.carve(kv);
    b->pages = (int *) b->ar.carve((size_t) B * b->maxp * 4);
    b->rcos = (float *) b->ar.carve((size_t) b->n_ctx * (b->hd / 2) * 4);
    b->rsin = (float *) b->ar.carve((size_t) b->n_ctx * (b->hd / 2) * 4);
    b->tok = (int *) b->ar.carve((size_t) B * 4);
    b->pos = (int *) b->ar.carve((size_t) B * 4);
    b->tlog = (int *) b->ar.carve((size_t) B * (b->n_ctx + 1) * 4);
    b->xblk = (uint8_t *) b->ar.carve((size_t) Tp * nsb_max * 256);
    b->xs = (float *) b->ar.carve((size_t) Tp * nsb_max * 4);
    // attention: head groups of attn_hg query heads; the positions of a
    // (sequence, group) split over attn_split CTAs so that the grid fills the
    // SMs' resident slots in whole waves (two CTAs per SM up to hd 128)
    const int rep = b->nh / b->nkv;
    // tensor-core attention for hd 64 and 128 (groups of 8 or 16 heads), CUDA cores for 256
    b->attn_t = b->hd <= 128 ? (rep <= 8 ? 1 : 2) : 0;
    b->attn_hg = b->attn_t ? 8 * b->attn_t : battn_hg(rep);
    b->attn_groups = (rep + b->attn_hg - 1) / b->attn_hg;
    {
        const int pairs = B * b->nkv * b->attn_groups, slots = (b->hd <= 128 ? 2 : 1) * b->nsm;
        double best = 1e30;
        for (int n = 1; n <= 16; n++) {
            const double cost = (double) ((pairs * n + slots - 1) / slots) / n + 0.02 * n;
            if (cost < best - 1e-9) { best = cost; b->attn_split = n; }
        }
    }
    b->apart = (float *) b->ar.carve((size_t) B * b->nkv * b->attn_groups * b->attn_split * b->attn_hg *
                                     (b->hd + 2) * 4);
    b->acnt = (unsigned *) b->ar.carve((size_t) B * b->nkv * b->attn_groups * 4);
    b->err = (int *) b->ar.carve(4);
    return true;
}

// ------------------------------------------------------------------ step

template <int NB, int SIX>
static void b_launch_embed(sb_batch * b) {
    k_bembed<NB, SIX><<<dim3((b->E + 255) / 256, b->B), 256, 0, b->st>>>(b->emb, b->tok, b->pos, b->x, b->E, b->err);
    b_after(b, cudaGetLastError());
}

static void b_quant(sb_batch * b, int mode, const BGemm & gm, const float * x, int ldx, const float * gain,
                    int up_off) {
    TcQuantArgs q;
    memset(&q, 0, sizeof q);
    q.x = x; q.ldx = ldx; q.up_off = up_off; q.perm = gm.perm; q.gain = gain; q.eps = b->eps;
    q.cols = gm.cols; q.T = b->B; q.T_pad = b->T_pad; q.N = b->N; q.nsb = gm.p.nsb;
    q.xblk = b->xblk; q.xs = b->xs;
    b_after(b, tc_quant(mode, q, b->st));
}

static void b_mma(sb_batch * b, const BGemm & gm, float * y, int ldy, const float * bias, int accumulate) {
    TcArgs a;
    memset(&a, 0, sizeof a);
    a.wblk = gm.p.wblk; a.s8 = gm.p.s8; a.xblk = b->xblk; a.xs = b->xs;
    a.y = y; a.ldy = ldy; a.bias = bias; a.accumulate = accumulate;
    a.rows = gm.rows; a.rows_pad = gm.p.rows_pad; a.nsb = gm.p.nsb; a.T = b->B; a.T_pad = b->T_pad;
    a.split = gm.split; a.err = b->err;
    b_after(b, tc_mma(a, b->st));
}

// Launch (or, with attr, set the shared-memory limit of) k_battn<hd, hg>.
static cudaError_t b_attn_launch(int hd, int hg, dim3 grid, size_t smem, cudaStream_t st, const BAttnArgs & a,
                                 bool attr) {
#define SB_BATTN(HD, HG)                                                                                   \
    if (hd == HD && hg == HG) {                                                                             \
        if (attr) return cudaFuncSetAttribute(k_battn<HD, HG>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                              (int) smem);                                                  \
        k_battn<HD, HG><<<grid, kBThreads, smem, st>>>(a);                                                  \
        return cudaGetLastError();                                                                          \
    }
    SB_BATTN(64, 4) SB_BATTN(64, 8) SB_BATTN(128, 4) SB_BATTN(128, 8) SB_BATTN(256, 4) SB_BATTN(256, 8)
#undef SB_BATTN
    return cudaErrorInvalidValue;
}

static void b_attn(sb_batch * b, const BLayer & y, int l) {
    BAttnArgs a;
    memset(&a, 0, sizeof a);
    a.qkv = b->qkv; a.ldq = b->qkv_rows; a.koff = b->koff; a.voff = b->voff;
    a.n_head = b->nh; a.n_kv = b->nkv; a.qn = y.qn; a.kn = y.kn; a.eps = b->eps;
    a.rcos = b->rcos; a.rsin = b->rsin;
    const size_t per_layer = (size_t) b->n_pages * b->nkv * 64 * b->hd;
    a.kc = b->kc + (size_t) l * per_layer;
    a.vc = b->vc + (size_t) l * per_layer;
    a.pages = b->pages; a.maxp = b->maxp; a.n_pages = b->n_pages;
    a.n_ctx = b->n_ctx; a.pos = b->pos; a.nsplit = b->attn_split; a.hgroups = b->attn_groups; a.scale = b->scale;
    a.part = b->apart; a.cnt = b->acnt; a.out = b->att; a.ldo = b->qd; a.err = b->err;
    const dim3 grid(b->attn_split, b->nkv * b->attn_groups, b->B);
    if (b->attn_t) {
        const size_t smem = battn_t_smem(b->hd, b->attn_t);
        if (b->hd == 64) {
            if (b->attn_t == 1) k_battn_t<64, 1><<<grid, kMThreads, smem, b->st>>>(a);
            else k_battn_t<64, 2><<<grid, kMThreads, smem, b->st>>>(a);
        } else {
            if (b->attn_t == 1) k_battn_t<128, 1><<<grid, kMThreads, smem, b->st>>>(a);
            else k_battn_t<128, 2><<<grid, kMThreads, smem, b->st>>>(a);
        }
        b_after(b, cudaGetLastError());
        return;
    }
    const size_t smem = battn_smem(b->hd, b->attn_hg);
    b_after(b, b_attn_launch(b->hd, b->attn_hg, grid, smem, b->st, a, false));
}

static void b_enqueue(sb_batch * b) {
    snprintf(b->cur, sizeof b->cur, "embed");
    SB_DISPATCH_QT(b->emb.nbits, b->emb.six, b_launch_embed, b);
    for (int l = 0; l < b->n_layer && !b->failed; l++) {
        const BLayer & y = b->L[l];
        snprintf(b->cur, sizeof b->cur, "L%d.qkv", l);
        b_quant(b, TQ_NORM, y.qkv, b->x, b->E, y.an, 0);
        b_mma(b, y.qkv, b->qkv, b->qkv_rows, y.qkv_b, 0);
        snprintf(b->cur, sizeof b->cur, "L%d.attn", l);
        b_attn(b, y, l);
        snprintf(b->cur, sizeof b->cur, "L%d.o", l);
        b_quant(b, TQ_PLAIN, y.o, b->att, b->qd, nullptr, 0);
        b_mma(b, y.o, b->x, b->E, nullptr, 1);
        if (y.moe) {
            // router on rmsnorm(x) per row, the chosen experts, combine added to x
            snprintf(b->cur, sizeof b->cur, "L%d.moe", l);
            moe_enqueue(y.ml, b->ms, b->x, b->B, y.fn, b->eps, b->x, 1, b->nsm, b->st, false, b->err, nullptr,
                        b->launches, [&](cudaError_t r, const char *) { b_after(b, r); }, nullptr, nullptr, 0.0f,
                        MOE_TC_ON);   // configuration 4 at 64 slots: 1160 tok/s here, 759 on the integer kernels
            continue;
        }
        snprintf(b->cur, sizeof b->cur, "L%d.ffn", l);
        b_quant(b, TQ_NORM, y.gu, b->x, b->E, y.fn, 0);
        b_mma(b, y.gu, b->hid, 2 * b->Fp, nullptr, 0);
        snprintf(b->cur, sizeof b->cur, "L%d.down", l);
        b_quant(b, TQ_SILU, y.dn, b->hid, 2 * b->Fp, nullptr, b->Fp);
        b_mma(b, y.dn, b->x, b->E, nullptr, 1);
    }
    snprintf(b->cur, sizeof b->cur, "head");
    b_quant(b, TQ_NORM, b->head, b->x, b->E, b->out_norm, 0);
    b_mma(b, b->head, b->logits, b->head.rows, nullptr, 0);
    snprintf(b->cur, sizeof b->cur, "argmax");
    k_bargmax<<<b->B, kArgThreads, 0, b->st>>>(b->logits, b->V, b->tok, b->pos, b->tlog, b->n_ctx);
    b_after(b, cudaGetLastError());
}

static void b_close_all(sb_batch * b) {
    if (b->g) cudaGraphExecDestroy(b->g);
    if (b->st) cudaStreamDestroy(b->st);
    b->ar.release();
    if (b->h_logits) cudaFreeHost(b->h_logits);
    if (b->h_io) cudaFreeHost(b->h_io);
    if (b->h_pages) cudaFreeHost(b->h_pages);
    ssf_close(&b->f);
}

static sb_batch * b_fail(sb_batch * b, char * why, int nwhy, const char * msg) {
    if (msg) snprintf(why, nwhy, "%s", msg);
    b_close_all(b);
    delete b;
    return nullptr;
}

// n_pages 0: fixed slots (slot s owns pages s * maxp ..); else a pool of that
// many pages for sequences (sb_seq_new / sb_forward_seqs).
static sb_batch * open_batch(const char * path, int n_seq, int n_ctx, int n_pages, char * why, int nwhy) {
    g_berr[0] = 0;
    if (why && nwhy) why[0] = 0;
    sb_batch * b = new sb_batch();
    if (n_seq < 1 || n_seq > kMaxBatchSeqs) return b_fail(b, why, nwhy, "n_seq out of range");
    if (n_pages < 0) return b_fail(b, why, nwhy, "n_pages out of range");
    if (!ssf_open(&b->f, path, why, nwhy)) { delete b; return nullptr; }
    const ssf_hdr * h = b->f.hdr;
    if (const char * u = ssf_unsupported(b->f)) {
        char msg[160];
        snprintf(msg, sizeof msg, "%s: not on the GPU yet", u);
        return b_fail(b, why, nwhy, msg);
    }
    b->n_layer = (int) h->n_layer; b->E = (int) h->n_embd; b->nh = (int) h->n_head; b->nkv = (int) h->n_head_kv;
    b->V = (int) h->n_vocab; b->eps = h->rms_eps; b->theta = h->rope_theta;
    const ssf_rec * q0 = ssf_find(&b->f, "blk.0.attn_q.weight");
    b->hd = q0 && q0->rows % b->nh == 0 ? (int) q0->rows / b->nh : b->E / b->nh;
    b->qd = b->nh * b->hd;
    b->kvd = b->nkv * b->hd;
    b->scale = h->attn_scale != 0.0f ? h->attn_scale : 1.0f / sqrtf((float) b->hd);
    b->n_ctx = n_ctx > 0 ? n_ctx : 256;
    b->B = n_seq;
    b->maxp = (b->n_ctx + 63) / 64;
    b->paged = n_pages > 0;
    b->n_pages = b->paged ? n_pages : n_seq * b->maxp;
    for (int p = b->n_pages - 1; b->paged && p >= 0; p--) b->free_pages.push_back(p);
    b->N = tc_tile_n(n_seq);
    b->T_pad = tc_tokens_pad(n_seq);
    b->qkv_rows = round128(b->qd) + 2 * round128(b->kvd);
    b->koff = round128(b->qd);
    b->voff = b->koff + round128(b->kvd);
    if (h->n_rot && (int) h->n_rot != b->hd) return b_fail(b, why, nwhy, "partial rotary: not on the GPU yet");
    if (b->nh % b->nkv || (b->hd != 64 && b->hd != 128 && b->hd != 256) || b->nh / b->nkv > kBMaxRep) {
        char msg[96];
        snprintf(msg, sizeof msg, "head layout %d/%d x %d not on the batched path", b->nh, b->nkv, b->hd);
        return b_fail(b, why, nwhy, msg);
    }
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&b->nsm, cudaDevAttrMultiProcessorCount, dev);
    if (!bck(cudaStreamCreateWithFlags(&b->st, cudaStreamNonBlocking), "stream"))
        return b_fail(b, why, nwhy, g_berr);
    // MoE experts drawn on the device (sb_draw_experts) rather than read
    b->ar.draw_seed = draw_experts_seed();
    b->ar.minneg = b->f.minneg;
    // pass 1 sizes the arena, pass 2 fills it (and re-quantizes every product's weights)
    if (!b_build(b, why, nwhy)) return b_fail(b, why, nwhy, nullptr);
    if (!b->ar.allocate()) {
        char msg[96];
        snprintf(msg, sizeof msg, "cudaMalloc of %.2f GB for the batched model failed", b->ar.size / 1e9);
        return b_fail(b, why, nwhy, msg);
    }
    if (!b_build(b, why, nwhy)) return b_fail(b, why, nwhy, nullptr);
    upload_rope(b->rcos, b->rsin, b->n_ctx, b->hd, b->theta);
    BAttnArgs none;
    memset(&none, 0, sizeof none);
    cudaError_t ar;
    if (b->attn_t) {
        void (*kt)(BAttnArgs) = b->hd == 64 ? (b->attn_t == 1 ? k_battn_t<64, 1> : k_battn_t<64, 2>)
                                            : (b->attn_t == 1 ? k_battn_t<128, 1> : k_battn_t<128, 2>);
        ar = cudaFuncSetAttribute(kt, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) battn_t_smem(b->hd, b->attn_t));
    } else {
        ar = b_attn_launch(b->hd, b->attn_hg, dim3(1), battn_smem(b->hd, b->attn_hg), b->st, none, true);
    }
    if (!bck(ar, "attention shared memory") || !bck(cudaMallocHost(&b->h_logits, (size_t) b->B * b->V * 4), "pinned logits") ||
        !bck(cudaMallocHost(&b->h_io, (size_t) 2 * b->B * 4), "pinned io"))
        return b_fail(b, why, nwhy, g_berr);
    std::vector<int> idle(b->B, -1);
    cudaMemcpy(b->pos, idle.data(), (size_t) b->B * 4, cudaMemcpyHostToDevice);
    {
        // fixed slots: slot s's positions 64c .. on page s * maxp + c; a paged
        // handle starts with empty tables (every step uploads its own)
        std::vector<int> tab((size_t) b->B * b->maxp, -1);
        for (int sl = 0; !b->paged && sl < b->B; sl++)
            for (int c = 0; c < b->maxp; c++) tab[(size_t) sl * b->maxp + c] = sl * b->maxp + c;
        if (!bck(cudaMemcpy(b->pages, tab.data(), tab.size() * 4, cudaMemcpyHostToDevice), "page tables") ||
            (b->paged && !bck(cudaMallocHost(&b->h_pages, tab.size() * 4), "pinned page tables")))
            return b_fail(b, why, nwhy, g_berr);
    }
    const char * sm = getenv("SB_SYNC");
    b->sync_mode = sm && atoi(sm) != 0;
    b->launches = 0;
    bool ok = true;
    if (!b->sync_mode) {
        cudaGraph_t gr = nullptr;
        ok = bck(cudaStreamBeginCapture(b->st, cudaStreamCaptureModeThreadLocal), "begin capture");
        if (ok) {
            b_enqueue(b);
            ok = bck(cudaStreamEndCapture(b->st, &gr), "end capture") && !b->failed;
        }
        ok = ok && bck(cudaGraphInstantiateWithFlags(&b->g, gr, 0), "instantiate");
        if (gr) cudaGraphDestroy(gr);
    }
    ok = ok && bck(cudaDeviceSynchronize(), "open") && !b->failed;
    if (!ok) return b_fail(b, why, nwhy, g_berr);
    return b;
}

extern "C" sb_batch * sb_batch_open(const char * path, int n_seq, int n_ctx, char * why, int nwhy) {
    return open_batch(path, n_seq, n_ctx, 0, why, nwhy);
}

extern "C" sb_batch * sb_batch_open_paged(const char * path, int n_slots, int n_ctx, int n_pages, char * why,
                                          int nwhy) {
    if (n_pages < 1) {
        if (why && nwhy) snprintf(why, nwhy, "n_pages must be at least 1");
        return nullptr;
    }
    return open_batch(path, n_slots, n_ctx, n_pages, why, nwhy);
}

extern "C" void sb_batch_close(sb_batch * b) {
    if (!b) return;
    cudaStreamSynchronize(b->st);
    b_close_all(b);
    delete b;
}

extern "C" void sb_batch_info(const sb_batch * b, int * out) {
    out[0] = b->B; out[1] = b->n_ctx; out[2] = b->V;
    const BLayer & y = b->L[0];
    out[3] = y.qkv.split; out[4] = y.o.split; out[5] = y.moe ? 0 : y.gu.split; out[6] = y.moe ? 0 : y.dn.split;
    out[7] = b->head.split;
    out[8] = (int) (b->bytes_file & 0xffffffffu); out[9] = (int) (b->bytes_file >> 32);
    out[10] = (int) (b->bytes_i8 & 0xffffffffu); out[11] = (int) (b->bytes_i8 >> 32);
    out[12] = b->launches;
    out[13] = b->N;
    out[14] = (int) (b->bytes_experts & 0xffffffffu); out[15] = (int) (b->bytes_experts >> 32);
}

// One step of every slot on the stream (graph replay or, with SB_SYNC=1, eager
// checked launches).
static bool b_run(sb_batch * b) {
    if (!b->sync_mode) return bck(cudaGraphLaunch(b->g, b->st), "graph launch");
    b->launches = 0;
    b_enqueue(b);
    return !b->failed;
}

static bool b_check_err(sb_batch * b, const char * what) {
    int err = 0;
    if (!bck(cudaMemcpy(&err, b->err, 4, cudaMemcpyDeviceToHost), what)) return false;
    if (err) {
        snprintf(g_berr, sizeof g_berr, "%s: device check %d failed", what, err);
        int zero = 0;
        cudaMemcpy(b->err, &zero, 4, cudaMemcpyHostToDevice);
        return false;
    }
    return true;
}

extern "C" const float * sb_forward_multi(sb_batch * b, const int * tokens, const int * pos) {
    g_berr[0] = 0;
    if (!b || !tokens || !pos) return nullptr;
    if (b->paged) { snprintf(g_berr, sizeof g_berr, "a paged handle runs sequences: sb_forward_seqs"); return nullptr; }
    for (int s = 0; s < b->B; s++) {
        if (pos[s] >= b->n_ctx || (pos[s] >= 0 && (tokens[s] < 0 || tokens[s] >= b->V))) {
            snprintf(g_berr, sizeof g_berr, "slot %d: token %d at position %d out of range", s, tokens[s], pos[s]);
            return nullptr;
        }
        b->h_io[s] = tokens[s];
        b->h_io[b->B + s] = pos[s] < 0 ? -1 : pos[s];
    }
    if (!bck(cudaMemcpyAsync(b->tok, b->h_io, (size_t) b->B * 4, cudaMemcpyHostToDevice, b->st), "tokens") ||
        !bck(cudaMemcpyAsync(b->pos, b->h_io + b->B, (size_t) b->B * 4, cudaMemcpyHostToDevice, b->st), "positions") ||
        !b_run(b) ||
        !bck(cudaMemcpyAsync(b->h_logits, b->logits, (size_t) b->B * b->V * 4, cudaMemcpyDeviceToHost, b->st), "logits") ||
        !bck(cudaStreamSynchronize(b->st), "step") || !b_check_err(b, "step"))
        return nullptr;
    return b->h_logits;
}

// Greedy generation for every slot on the device: prompts [n_seq][np] stepped
// from position 0, then nwarm + ngen tokens each, chosen on the GPU and fed
// back by graph replay. ids [n_seq][nwarm + ngen]. ms (if not NULL): the device
// time of the last ngen - 1 steps (CUDA events on the stream).
extern "C" int sb_batch_generate(sb_batch * b, const int * prompts, int np, int nwarm, int ngen, int * ids,
                                 float * ms) {
    g_berr[0] = 0;
    const int total = nwarm + ngen;
    if (!b || !prompts || !ids || np < 1 || nwarm < 0 || ngen < 1 || np + total - 1 > b->n_ctx || b->paged) {
        snprintf(g_berr, sizeof g_berr, "generate: bad arguments%s", b && b->paged ? " (a paged handle)" : "");
        return 0;
    }
    for (size_t i = 0; i < (size_t) b->B * np; i++)
        if (prompts[i] < 0 || prompts[i] >= b->V) { snprintf(g_berr, sizeof g_berr, "generate: bad prompt id"); return 0; }
    // every prompt step's tokens and positions staged once, pinned
    int * stage = nullptr;
    if (!bck(cudaMallocHost(&stage, (size_t) np * 2 * b->B * 4), "pinned prompts")) return 0;
    for (int i = 0; i < np; i++)
        for (int s = 0; s < b->B; s++) {
            stage[(size_t) i * 2 * b->B + s] = prompts[(size_t) s * np + i];
            stage[(size_t) i * 2 * b->B + b->B + s] = i;
        }
    bool ok = true;
    for (int i = 0; ok && i < np; i++) {
        ok = bck(cudaMemcpyAsync(b->tok, stage + (size_t) i * 2 * b->B, (size_t) b->B * 4, cudaMemcpyHostToDevice, b->st), "tokens") &&
             bck(cudaMemcpyAsync(b->pos, stage + (size_t) i * 2 * b->B + b->B, (size_t) b->B * 4, cudaMemcpyHostToDevice, b->st), "positions") &&
             b_run(b);
    }
    for (int g = 0; ok && g < nwarm; g++) ok = b_run(b);
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (ok && ms) {
        ok = bck(cudaStreamSynchronize(b->st), "generate");
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaEventRecord(e0, b->st);
    }
    for (int g = 0; ok && g + 1 < ngen; g++) ok = b_run(b);
    if (ok && ms) cudaEventRecord(e1, b->st);
    ok = ok && bck(cudaStreamSynchronize(b->st), "generate") && b_check_err(b, "generate");
    cudaFreeHost(stage);
    if (ok) {
        // slot s's ids sit at tlog[s][np .. np + total)
        std::vector<int> log((size_t) b->B * (b->n_ctx + 1));
        ok = bck(cudaMemcpy(log.data(), b->tlog, log.size() * 4, cudaMemcpyDeviceToHost), "ids");
        for (int s = 0; ok && s < b->B; s++)
            memcpy(ids + (size_t) s * total, log.data() + (size_t) s * (b->n_ctx + 1) + np, (size_t) total * 4);
    }
    if (e0) {
        if (ok) cudaEventElapsedTime(ms, e0, e1);
        cudaEventDestroy(e0);
        cudaEventDestroy(e1);
    }
    return ok ? 1 : 0;
}

extern "C" const float * sb_batch_device_logits(const sb_batch * b) { return b ? b->logits : nullptr; }

// The cached key and value rows of one slot at one position of one layer
// (host buffers of n_kv * hd fp16 each, head-major), for checks and export.
static bool kv_rows_at(const sb_batch * b, int layer, int page, int pos, uint16_t * k, uint16_t * v) {
    const size_t per_layer = (size_t) b->n_pages * b->nkv * 64 * b->hd;
    for (int h = 0; h < b->nkv; h++) {
        const size_t at = (size_t) layer * per_layer + (((size_t) page * b->nkv + h) * 64 + pos % 64) * b->hd;
        if (!bck(cudaMemcpy(k + (size_t) h * b->hd, b->kc + at, (size_t) b->hd * 2, cudaMemcpyDeviceToHost), "kv") ||
            !bck(cudaMemcpy(v + (size_t) h * b->hd, b->vc + at, (size_t) b->hd * 2, cudaMemcpyDeviceToHost), "kv"))
            return false;
    }
    return true;
}

extern "C" int sb_batch_kv(const sb_batch * b, int layer, int slot, int pos, uint16_t * k, uint16_t * v) {
    if (!b || b->paged || layer < 0 || layer >= b->n_layer || slot < 0 || slot >= b->B || pos < 0 || pos >= b->n_ctx ||
        !k || !v)
        return 0;
    return kv_rows_at(b, layer, slot * b->maxp + pos / 64, pos, k, v) ? 1 : 0;
}

// ------------------------------------------------------------------ sequences
// A paged handle serves sequences rather than slots: each sequence holds the
// pages its positions reached (taken from the pool when first needed), a
// step runs any set of live sequences in its slots (in any order), and a
// freed sequence's pages go back to the pool at once.

extern "C" int sb_seq_new(sb_batch * b) {
    g_berr[0] = 0;
    if (!b || !b->paged) { snprintf(g_berr, sizeof g_berr, "sb_seq_new: not a paged handle"); return -1; }
    int id;
    if (!b->free_seqs.empty()) {
        id = b->free_seqs.back();
        b->free_seqs.pop_back();
    } else {
        id = (int) b->seq_pages.size();
        b->seq_pages.emplace_back();
        b->seq_live.push_back(0);
    }
    b->seq_pages[id].clear();
    b->seq_live[id] = 1;
    return id;
}

static bool seq_ok(const sb_batch * b, int id) {
    return b && b->paged && id >= 0 && id < (int) b->seq_live.size() && b->seq_live[id];
}

// Keep the first n positions of a sequence: pages past them go back to the pool.
extern "C" int sb_seq_truncate(sb_batch * b, int id, int n) {
    g_berr[0] = 0;
    if (!seq_ok(b, id) || n < 0) { snprintf(g_berr, sizeof g_berr, "sb_seq_truncate: no such sequence"); return 0; }
    std::vector<int> & pg = b->seq_pages[id];
    const size_t keep = (size_t) (n + 63) / 64;
    while (pg.size() > keep) {
        b->free_pages.push_back(pg.back());
        pg.pop_back();
    }
    return 1;
}

extern "C" int sb_seq_free(sb_batch * b, int id) {
    if (!sb_seq_truncate(b, id, 0)) return 0;
    b->seq_live[id] = 0;
    b->free_seqs.push_back(id);
    return 1;
}

// out[0] pages in the pool, out[1] free pages, out[2] live sequences, out[3]
// positions a sequence may reach (n_ctx).
extern "C" void sb_batch_pages(const sb_batch * b, int * out) {
    int live = 0;
    for (char c : b->seq_live) live += c;
    out[0] = b->n_pages;
    out[1] = b->paged ? (int) b->free_pages.size() : 0;
    out[2] = live;
    out[3] = b->n_ctx;
}

extern "C" const float * sb_forward_seqs(sb_batch * b, const int * seqs, const int * tokens, const int * pos, int ns) {
    g_berr[0] = 0;
    if (!b || !b->paged || !seqs || !tokens || !pos || ns < 0 || ns > b->B) {
        snprintf(g_berr, sizeof g_berr, "sb_forward_seqs: bad arguments (a paged handle, 0..%d sequences)", b ? b->B : 0);
        return nullptr;
    }
    // every check and the pages the step needs before any state changes
    size_t need = 0;
    for (int s = 0; s < ns; s++) {
        if (!seq_ok(b, seqs[s])) { snprintf(g_berr, sizeof g_berr, "slot %d: sequence %d is not live", s, seqs[s]); return nullptr; }
        for (int r = 0; r < s; r++)
            if (seqs[r] == seqs[s]) { snprintf(g_berr, sizeof g_berr, "sequence %d in two slots", seqs[s]); return nullptr; }
        if (pos[s] < 0 || pos[s] >= b->n_ctx || tokens[s] < 0 || tokens[s] >= b->V) {
            snprintf(g_berr, sizeof g_berr, "slot %d: token %d at position %d out of range", s, tokens[s], pos[s]);
            return nullptr;
        }
        const size_t have = b->seq_pages[seqs[s]].size(), want = (size_t) pos[s] / 64 + 1;
        if (want > have) need += want - have;
    }
    if (need > b->free_pages.size()) {
        snprintf(g_berr, sizeof g_berr, "the step needs %zu more pages, %zu are free", need, b->free_pages.size());
        return nullptr;
    }
    for (int s = 0; s < ns; s++) {
        std::vector<int> & pg = b->seq_pages[seqs[s]];
        while (pg.size() < (size_t) pos[s] / 64 + 1) {
            pg.push_back(b->free_pages.back());
            b->free_pages.pop_back();
        }
    }
    for (int s = 0; s < b->B; s++) {
        int * row = b->h_pages + (size_t) s * b->maxp;
        for (int c = 0; c < b->maxp; c++) row[c] = -1;
        if (s < ns) {
            const std::vector<int> & pg = b->seq_pages[seqs[s]];
            for (size_t c = 0; c < pg.size(); c++) row[c] = pg[c];
        }
        b->h_io[s] = s < ns ? tokens[s] : 0;
        b->h_io[b->B + s] = s < ns ? pos[s] : -1;
    }
    if (!bck(cudaMemcpyAsync(b->pages, b->h_pages, (size_t) b->B * b->maxp * 4, cudaMemcpyHostToDevice, b->st), "page tables") ||
        !bck(cudaMemcpyAsync(b->tok, b->h_io, (size_t) b->B * 4, cudaMemcpyHostToDevice, b->st), "tokens") ||
        !bck(cudaMemcpyAsync(b->pos, b->h_io + b->B, (size_t) b->B * 4, cudaMemcpyHostToDevice, b->st), "positions") ||
        !b_run(b) ||
        !bck(cudaMemcpyAsync(b->h_logits, b->logits, (size_t) ns * b->V * 4, cudaMemcpyDeviceToHost, b->st), "logits") ||
        !bck(cudaStreamSynchronize(b->st), "step") || !b_check_err(b, "step"))
        return nullptr;
    return b->h_logits;
}

// The cached key and value rows of a sequence at one position of one layer.
extern "C" int sb_seq_kv(const sb_batch * b, int layer, int id, int pos, uint16_t * k, uint16_t * v) {
    if (!seq_ok(b, id) || layer < 0 || layer >= b->n_layer || pos < 0 || pos >= b->n_ctx || !k || !v ||
        (size_t) pos / 64 >= b->seq_pages[id].size())
        return 0;
    return kv_rows_at(b, layer, b->seq_pages[id][pos / 64], pos, k, v) ? 1 : 0;
}
