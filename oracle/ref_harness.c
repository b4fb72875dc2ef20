// TEST INFRASTRUCTURE ONLY -- the checker and the CPU baseline, never the product.
//
// A thin C harness linked against the reference engine's own, unchanged CPU
// sources (sml/sml-kernel.c, sml-run.c, sml-model.c, sml-pool.c), built by
// oracle/Makefile into oracle/_ref/libsmlref.so. It gives the tests and the
// bench flat entry points into the reference's real code path:
//
//   refh_open/refh_forward   sml_model_open + sml_ctx_init + sml_forward
//                            (sml/sml-run.c:1236, :3243), prompt stepped a token
//                            at a time as SML_SEQ_PROMPT=1 does (sml/sml-cli.c:481)
//   refh_quantize_act        sml_quantize_act (sml/sml-kernel.c:41)
//   refh_quantize_act_sb     sml_quantize_act_sb (sml/sml-kernel.c:116), the
//                            batched path's per-256 activation
//   refh_matvec              gather + quantize + the per-width dispatch of
//                            issue_rows_act (sml/sml-run.c:612-680), issued the
//                            way sml/sml-check.c:166-245 issues it
//   refh_dequant_row         the embedding-row dequant of sml_forward
//                            (sml/sml-run.c:3283-3330)
//   refh_moe_route           sml_moe_route (sml/sml-run.c:2925)
//   refh_forward_multi       sml_forward_multi (sml/sml-run.c:2559)
#include "sml-run.h"
#include "sml-kernel.h"
#include "sml-model.h"

#include <stdlib.h>
#include <string.h>

typedef struct {
    sml_model m;
    sml_ctx   c;
    int       have_ctx;
} refh;

void * refh_open(const char * path, int n_ctx, int threads, int with_ctx) {
    refh * h = (refh *) calloc(1, sizeof(refh));
    if (!h) return NULL;
    if (!sml_model_open(&h->m, path)) { free(h); return NULL; }
    if (with_ctx) {
        if (!sml_ctx_init(&h->c, &h->m, n_ctx, threads)) { sml_model_close(&h->m); free(h); return NULL; }
        h->have_ctx = 1;
    }
    return h;
}

void refh_close(void * p) {
    refh * h = (refh *) p;
    if (!h) return;
    if (h->have_ctx) sml_ctx_free(&h->c);
    sml_model_close(&h->m);
    free(h);
}

// Returns n_vocab and fills out[0..7] = n_layer, n_embd, n_head, n_head_kv,
// head_dim, n_ff, n_vocab, flags.
int refh_info(void * p, int * out) {
    refh * h = (refh *) p;
    const sml_hdr * hd = h->m.hdr;
    out[0] = (int) hd->n_layer; out[1] = (int) hd->n_embd; out[2] = (int) hd->n_head;
    out[3] = (int) hd->n_head_kv; out[4] = h->have_ctx ? h->c.head_dim : 0;
    out[5] = (int) hd->n_ff; out[6] = (int) hd->n_vocab; out[7] = (int) hd->flags;
    return (int) hd->n_vocab;
}

int refh_forward(void * p, int tok, int pos, float * logits) {
    refh * h = (refh *) p;
    if (!h->have_ctx || pos >= h->c.n_ctx) return 0;
    const float * lg = sml_forward(&h->c, tok, pos, 0);
    if (logits) memcpy(logits, lg, (size_t) h->m.hdr->n_vocab * sizeof(float));
    return sml_sample_greedy(lg, (int) h->m.hdr->n_vocab);
}

// Greedy decode: the prompt stepped token by token from position 0, then ngen
// tokens each fed back. ids_out gets the ngen generated ids; logits_out (if not
// NULL) gets ngen rows of n_vocab floats, row i being the logits that chose id i.
int refh_decode(void * p, const int * prompt, int np, int ngen, int * ids_out, float * logits_out) {
    refh * h = (refh *) p;
    if (!h->have_ctx || np < 1 || np + ngen > h->c.n_ctx + 1) return 0;
    const int nv = (int) h->m.hdr->n_vocab;
    const float * lg = NULL;
    for (int i = 0; i < np; i++) lg = sml_forward(&h->c, prompt[i], i, 0);
    int pos = np;
    for (int g = 0; g < ngen; g++) {
        const int t = sml_sample_greedy(lg, nv);
        ids_out[g] = t;
        if (logits_out) memcpy(logits_out + (size_t) g * nv, lg, (size_t) nv * sizeof(float));
        if (g + 1 < ngen) lg = sml_forward(&h->c, t, pos++, 0);
    }
    return 1;
}

void refh_quantize_act(const float * x, int n, int8_t * q, float * scale, int32_t * sums) {
    sml_act a = { q, scale, sums, n };
    sml_quantize_act(&a, x, n);
}

void refh_quantize_act_sb(const float * x, int n, int8_t * q, float * scale, int32_t * sums) {
    sml_act a = { q, scale, sums, n };
    sml_quantize_act_sb(&a, x, n);
}

// y[row0..row1) = W x for one tensor, x in the model's natural column order.
// Also returns the quantized activation it used when qx/qs/qsum are non-NULL.
int refh_matvec(void * p, const char * name, const float * x, float * y, int row0, int row1,
                int8_t * qx, float * qs, int32_t * qsum) {
    refh * h = (refh *) p;
    const sml_rec * r = sml_find(&h->m, name);
    if (!r || r->kind != SML_KIND_LADDER || r->layout != SML_LAYOUT_FLAT) return 0;
    const sml_model * m = &h->m;
    const int n = (int) r->cols, ng = n / SML_GROUP;
    float * xp = (float *) malloc((size_t) n * sizeof(float));
    sml_act a;
    a.q = (int8_t *) malloc((size_t) n);
    a.scale = (float *) malloc((size_t) ng * sizeof(float));
    a.sums = (int32_t *) malloc((size_t) ng * sizeof(int32_t));
    sml_gather(xp, x, (const int32_t *) sml_ptr(m, r->perm_off), n);
    sml_quantize_act(&a, xp, n);
    const uint16_t * sd = (const uint16_t *) sml_ptr(m, r->sd_off);
    const uint8_t  * sq = sml_ptr(m, r->sq_off);
    const uint16_t * md = r->mq_n ? (const uint16_t *) sml_ptr(m, r->md_off) : NULL;
    const uint8_t  * mq = r->mq_n ? sml_ptr(m, r->mq_off) : NULL;
    const uint8_t * p0 = sml_ptr(m, r->codes_off[0]);
    const uint8_t * p1 = r->codes_n[1] ? sml_ptr(m, r->codes_off[1]) : NULL;
    const uint8_t * p2 = r->codes_n[2] ? sml_ptr(m, r->codes_off[2]) : NULL;
    memset(y + row0, 0, (size_t) (row1 - row0) * sizeof(float));
    switch (r->nbits) {
    case 2: sml_matvec_rows(y, p0, sd, sq, md, mq, &a, row0, row1, n, 0, 0.0f); break;
    case 3: sml_matvec_rows(y, p0, sd, sq, md, mq, &a, row0, row1, n, 0, 0.0f);
            sml_matvec_bits1(y, p1, sd, sq, &a, 1, 0, row0, row1, n, 2); break;
    case 4: sml_matvec_rows_flat4(y, p0, sd, sq, md, mq, &a, row0, row1, n); break;
    case 5: sml_matvec_rows_flat4(y, p0, sd, sq, md, mq, &a, row0, row1, n);
            sml_matvec_bits1(y, p1, sd, sq, &a, 1, 0, row0, row1, n, 4); break;
    case 6: sml_matvec_rows_flat6(y, p1, p0, sd, sq, md, mq, &a, row0, row1, n); break;
    case 7: sml_matvec_rows_flat6(y, p0, p1, sd, sq, md, mq, &a, row0, row1, n);
            sml_matvec_bits1(y, p2, sd, sq, &a, 1, 0, row0, row1, n, 6); break;
    case 8: sml_matvec_rows_flat8(y, p0, p1, sd, sq, md, mq, &a, row0, row1, n); break;
    default: break;
    }
    if (qx) memcpy(qx, a.q, (size_t) n);
    if (qs) memcpy(qs, a.scale, (size_t) ng * sizeof(float));
    if (qsum) memcpy(qsum, a.sums, (size_t) ng * sizeof(int32_t));
    free(xp); free(a.q); free(a.scale); free(a.sums);
    return 1;
}

// One row of a flat tensor, dequantized by the reference's row functions, in
// the file's (permuted) column order.
int refh_dequant_row(void * p, const char * name, int row, float * out) {
    refh * h = (refh *) p;
    const sml_rec * r = sml_find(&h->m, name);
    if (!r || r->kind != SML_KIND_LADDER || r->layout != SML_LAYOUT_FLAT || row < 0 || row >= (int) r->rows)
        return 0;
    const sml_model * m = &h->m;
    const int n = (int) r->cols;
    const uint16_t * sd = (const uint16_t *) sml_ptr(m, r->sd_off);
    const uint8_t  * sq = sml_ptr(m, r->sq_off);
    const uint16_t * md = r->mq_n ? (const uint16_t *) sml_ptr(m, r->md_off) : NULL;
    const uint8_t  * mq = r->mq_n ? sml_ptr(m, r->mq_off) : NULL;
    const uint8_t * p0 = sml_ptr(m, r->codes_off[0]);
    const uint8_t * p1 = r->codes_n[1] ? sml_ptr(m, r->codes_off[1]) : NULL;
    const uint8_t * p2 = r->codes_n[2] ? sml_ptr(m, r->codes_off[2]) : NULL;
    switch (r->nbits) {
    case 2: { const uint8_t * pl[1] = { p0 }; sml_dequant_row(out, pl, 1, 1, sd, sq, md, mq, row, n); } break;
    case 3: { const uint8_t * pl[1] = { p0 }; sml_dequant_row(out, pl, 1, 1, sd, sq, md, mq, row, n);
              sml_dequant_bits1_add(out, p1, sd, sq, row, n, 2); } break;
    case 4: sml_dequant_row_flat4(out, p0, sd, sq, md, mq, row, n); break;
    case 5: sml_dequant_row_flat4(out, p0, sd, sq, md, mq, row, n);
            sml_dequant_bits1_add(out, p1, sd, sq, row, n, 4); break;
    case 6: sml_dequant_row_flat6(out, p1, p0, sd, sq, md, mq, row, n); break;
    case 7: sml_dequant_row_flat6(out, p0, p1, sd, sq, md, mq, row, n);
            sml_dequant_bits1_add(out, p2, sd, sq, row, n, 6); break;
    case 8: sml_dequant_row_flat8(out, p0, p1, sd, sq, md, mq, row, n); break;
    default: return 0;
    }
    return 1;
}

// Expert choice from router logits with the header's routing flags.
int refh_moe_route(const float * lg, int ne, int k, unsigned moe_flags, float moe_scale,
                   int * sel, float * w) {
    sml_hdr h;
    memset(&h, 0, sizeof h);
    h.n_expert_used = (uint32_t) k;
    h.moe_flags = moe_flags;
    h.moe_scale = moe_scale;
    sml_layer ly;
    memset(&ly, 0, sizeof ly);
    ly.n_exp = ne;
    float * sc = (float *) malloc((size_t) ne * sizeof(float));
    float * ch = (float *) malloc((size_t) ne * sizeof(float));
    const int got = sml_moe_route(&h, &ly, lg, sc, ch, sel, w);
    free(sc); free(ch);
    return got;
}

// Several sequences one step each (the sml-batched driver's call,
// sml/sml-batched.c:111). ctxs are refh handles opened with a context.
void refh_forward_multi(void ** hs, const int * toks, const int * pos, int ns, float * logits_out) {
    sml_ctx * cs[SML_MAX_BATCH];
    for (int i = 0; i < ns && i < SML_MAX_BATCH; i++) cs[i] = &((refh *) hs[i])->c;
    sml_forward_multi(cs, toks, pos, ns, 0, logits_out);
}

// Weight bytes one token streams, the reference's own counter.
unsigned long long refh_bytes_per_token(void * p) {
    return (unsigned long long) sml_bytes_at_depth(&((refh *) p)->m, 1);
}
