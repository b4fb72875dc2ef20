// Seeded synthetic SSF writer.
//
// There are no checkpoints on this machine, so every model the engine runs is
// written here from a seed: weights N(0, sigma) (RMSNorm gains 1), quantized by
// plain round-to-nearest onto the format's asymmetric two-level grid
//
//     w ~= code * (d * sq[g]) + md * (mq[g] - bias)
//
// with d, md fp16 per 256 weights and sq, mq one field per 32 weights (8-bit,
// or 6-bit packed four to three bytes in a v9 file). The grid only has to be
// valid: the engine and the CPU oracle read the same bytes. Plane packing
// follows the format rules (tooling/sml_format.py:392-446 pack_superblocks,
// pack_flat4, pack_bits1; plane order tooling/sml_quantize.py:106).
//
// Rows are generated in parallel from a counter-based stream keyed by
// (seed, tensor, row), so the file does not depend on the thread count.
#define _GNU_SOURCE
#include "ssf_gen.h"
#include "ssf.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>
#ifdef _OPENMP
#include <omp.h>
#endif

// ------------------------------------------------------------------ numbers

static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

typedef struct { uint64_t s; } rng_t;
static inline uint64_t rng_next(rng_t * r) { r->s += 0x9e3779b97f4a7c15ull; return mix64(r->s); }
static inline float rng_unit(rng_t * r) {              // (0, 1]
    return (float) ((rng_next(r) >> 40) + 1) * (1.0f / 16777216.0f);
}
// Two N(0,1) draws by Box-Muller.
static inline void rng_gauss2(rng_t * r, float * a, float * b) {
    const float u1 = rng_unit(r), u2 = rng_unit(r);
    const float rad = sqrtf(-2.0f * logf(u1));
    const float th = 6.28318530717958647f * u2;
    *a = rad * cosf(th);
    *b = rad * sinf(th);
}

// IEEE binary16 encode, round to nearest even (normal, subnormal, overflow).
uint16_t ssfgen_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = (int32_t) ((x >> 23) & 0xff);
    uint32_t m = x & 0x7fffffu;
    if (e == 0xff) return (uint16_t) (sign | 0x7c00u | (m ? 0x200u : 0u));
    int32_t he = e - 127 + 15;
    if (he >= 31) return (uint16_t) (sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return (uint16_t) sign;
        m |= 0x800000u;
        const uint32_t sh = (uint32_t) (14 - he);
        uint32_t v = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
        if (rem > half || (rem == half && (v & 1u))) v++;
        return (uint16_t) (sign | v);
    }
    uint32_t v = ((uint32_t) he << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (v & 1u))) v++;
    return (uint16_t) (sign | v);
}

float ssfgen_f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
    if (e == 0) {
        if (!m) bits = sign;
        else {
            e = 113;
            while (!(m & 0x400)) { m <<= 1; e--; }
            bits = sign | (e << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e + 112) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// ------------------------------------------------------------------ tensor list

enum { INIT_GAUSS = 0, INIT_ONES = 1 };

typedef struct {
    char name[SSF_NAME_LEN];
    int kind;                 // SSF_KIND_F32 / SSF_KIND_QUANT
    int rows, cols, nbits;
    int init;
    int perm_group;           // index into the perm list (quant only)
    int expert;               // a MoE expert's gate/up/down
    uint64_t stream;          // RNG stream id
    ssf_rec rec;
} tdesc;

typedef struct {
    tdesc * t;
    int n, cap;
    int * perm_cols;          // per perm group: its width
    uint64_t * perm_off;
    int n_perm, perm_cap;
} tlist;

static tdesc * add_t(tlist * L, const char * name, int kind, int rows, int cols, int nbits, int init) {
    if (L->n == L->cap) {
        L->cap = L->cap ? 2 * L->cap : 256;
        L->t = (tdesc *) realloc(L->t, (size_t) L->cap * sizeof(tdesc));
    }
    tdesc * d = &L->t[L->n];
    memset(d, 0, sizeof *d);
    snprintf(d->name, sizeof d->name, "%s", name);
    d->kind = kind; d->rows = rows; d->cols = cols; d->nbits = nbits; d->init = init;
    d->perm_group = -1;
    d->stream = (uint64_t) L->n + 1;
    L->n++;
    return d;
}

static int add_perm(tlist * L, int cols) {
    if (L->n_perm == L->perm_cap) {
        L->perm_cap = L->perm_cap ? 2 * L->perm_cap : 256;
        L->perm_cols = (int *) realloc(L->perm_cols, (size_t) L->perm_cap * sizeof(int));
        L->perm_off = (uint64_t *) realloc(L->perm_off, (size_t) L->perm_cap * sizeof(uint64_t));
    }
    L->perm_cols[L->n_perm] = cols;
    return L->n_perm++;
}

static tdesc * qt(tlist * L, const char * name, int rows, int cols, int nbits, int pg) {
    tdesc * d = add_t(L, name, SSF_KIND_QUANT, rows, cols, nbits, INIT_GAUSS);
    d->perm_group = pg;
    return d;
}

static void build_list(tlist * L, const ssfgen_spec * s) {
    char nm[SSF_NAME_LEN + 8];
    const int hd = (int) s->head_dim, E = (int) s->n_embd;
    const int qd = (int) s->n_head * hd, kvd = (int) s->n_head_kv * hd;
    const int pe = add_perm(L, E);
    qt(L, "token_embd.weight", (int) s->n_vocab, E, (int) s->emb_nbits, pe);
    add_t(L, "output_norm.weight", SSF_KIND_F32, 1, E, 0, INIT_ONES);
    if (!s->tied) qt(L, "output.weight", (int) s->n_vocab, E, (int) s->emb_nbits, add_perm(L, E));
    for (int l = 0; l < (int) s->n_layer; l++) {
#define NM(fmt) (snprintf(nm, sizeof nm, fmt, l), nm)
        add_t(L, NM("blk.%d.attn_norm.weight"), SSF_KIND_F32, 1, E, 0, INIT_ONES);
        const int pqkv = add_perm(L, E);
        qt(L, NM("blk.%d.attn_q.weight"), qd, E, (int) s->nbits, pqkv);
        qt(L, NM("blk.%d.attn_k.weight"), kvd, E, (int) s->nbits, pqkv);
        qt(L, NM("blk.%d.attn_v.weight"), kvd, E, (int) s->nbits, pqkv);
        if (s->qkv_bias) {
            add_t(L, NM("blk.%d.attn_q.bias"), SSF_KIND_F32, 1, qd, 0, INIT_GAUSS);
            add_t(L, NM("blk.%d.attn_k.bias"), SSF_KIND_F32, 1, kvd, 0, INIT_GAUSS);
            add_t(L, NM("blk.%d.attn_v.bias"), SSF_KIND_F32, 1, kvd, 0, INIT_GAUSS);
        }
        if (s->qk_norm) {
            add_t(L, NM("blk.%d.attn_q_norm.weight"), SSF_KIND_F32, 1, hd, 0, INIT_ONES);
            add_t(L, NM("blk.%d.attn_k_norm.weight"), SSF_KIND_F32, 1, hd, 0, INIT_ONES);
        }
        qt(L, NM("blk.%d.attn_output.weight"), E, qd, (int) s->nbits, add_perm(L, qd));
        add_t(L, NM("blk.%d.ffn_norm.weight"), SSF_KIND_F32, 1, E, 0, INIT_ONES);
        if (s->n_expert) {
            const int F = (int) s->expert_ff;
            add_t(L, NM("blk.%d.ffn_gate_inp.weight"), SSF_KIND_F32, (int) s->n_expert, E, 0, INIT_GAUSS);
            for (int e = 0; e < (int) s->n_expert; e++) {
                const int pgu = add_perm(L, E), pdn = add_perm(L, F);
                snprintf(nm, sizeof nm, "blk.%d.ffn_gate.%d.weight", l, e);
                qt(L, nm, F, E, (int) s->nbits, pgu)->expert = 1;
                snprintf(nm, sizeof nm, "blk.%d.ffn_up.%d.weight", l, e);
                qt(L, nm, F, E, (int) s->nbits, pgu)->expert = 1;
                snprintf(nm, sizeof nm, "blk.%d.ffn_down.%d.weight", l, e);
                qt(L, nm, E, F, (int) s->nbits, pdn)->expert = 1;
            }
        } else {
            const int F = (int) s->n_ff;
            const int pgu = add_perm(L, E);
            qt(L, NM("blk.%d.ffn_gate.weight"), F, E, (int) s->nbits, pgu);
            qt(L, NM("blk.%d.ffn_up.weight"), F, E, (int) s->nbits, pgu);
            qt(L, NM("blk.%d.ffn_down.weight"), E, F, (int) s->nbits, add_perm(L, F));
        }
#undef NM
    }
}

// ------------------------------------------------------------------ layout

static uint64_t align_up(uint64_t v, uint64_t a) { return (v + a - 1) / a * a; }

static uint64_t plane_row_bytes(int kind, int n) {
    return kind == 4 ? (uint64_t) n / 2 : kind == 2 ? (uint64_t) n / 4 : (uint64_t) n / 8;
}

static uint64_t place(uint64_t * cur, uint64_t n) {
    const uint64_t at = align_up(*cur, 256);
    *cur = at + n;
    return at;
}

static void layout(tlist * L, int six, uint64_t * end) {
    uint64_t cur = SSF_HEADER_BYTES + (uint64_t) L->n * sizeof(ssf_rec);
    for (int p = 0; p < L->n_perm; p++) L->perm_off[p] = place(&cur, (uint64_t) L->perm_cols[p] * 4);
    for (int i = 0; i < L->n; i++) {
        tdesc * d = &L->t[i];
        ssf_rec * r = &d->rec;
        memset(r, 0, sizeof *r);
        memcpy(r->name, d->name, SSF_NAME_LEN);
        r->kind = (uint32_t) d->kind;
        r->rows = (uint32_t) d->rows;
        r->cols = (uint32_t) d->cols;
        r->group = SSF_GROUP;
        if (d->kind == SSF_KIND_F32) {
            r->nbytes = (uint64_t) d->rows * d->cols * 4;
            r->off = place(&cur, r->nbytes);
            continue;
        }
        const int n = d->cols, ng = n / SSF_GROUP;
        r->layout = SSF_LAYOUT_FLAT;
        r->nbits = (uint32_t) d->nbits;
        r->perm_off = L->perm_off[d->perm_group];
        r->perm_n = (uint64_t) n * 4;
        r->sd_n = r->md_n = (uint64_t) d->rows * ssf_nscale(n) * 2;
        r->sq_n = r->mq_n = (uint64_t) d->rows * ssf_field_row_bytes(ng, six);
        r->sd_off = place(&cur, r->sd_n);
        r->sq_off = place(&cur, r->sq_n);
        r->md_off = place(&cur, r->md_n);
        r->mq_off = place(&cur, r->mq_n);
        int kinds[3], shifts[3];
        const int np = ssf_planes(d->nbits, kinds, shifts);
        for (int p = 0; p < np; p++) {
            r->codes_n[p] = (uint64_t) d->rows * plane_row_bytes(kinds[p], n);
            r->codes_off[p] = place(&cur, r->codes_n[p]);
        }
    }
    *end = align_up(cur, 256);
}

// ------------------------------------------------------------------ quantize

static int pwrite_all(int fd, const void * buf, uint64_t n, uint64_t off) {
    const uint8_t * p = (const uint8_t *) buf;
    while (n) {
        const ssize_t w = pwrite(fd, p, n > (1u << 30) ? (1u << 30) : (size_t) n, (off_t) off);
        if (w <= 0) return 0;
        p += w; n -= (uint64_t) w; off += (uint64_t) w;
    }
    return 1;
}

typedef struct {
    int six, minneg;
    float sigma;
    uint64_t seed;
    int direct;               // 1, 2: quantized tensors' ranges and codes drawn directly (quant_row);
                              // 2: MoE experts' bytes not written (holes of a sparse file)
} qctx;

// Quantize one row of n weights (already drawn) into its planes and fields.
// With rd (direct draws) w is not read: each group's range is drawn as
// [-sigma (1.6 + 0.8 u), sigma (1.6 + 0.8 v)] (about the extremes of 32
// normal draws), its fields follow from that range exactly as below, and its
// codes are uniform on [0, 2^nbits - 1]. Same layout and value scale, without
// drawing and rounding every weight: the ~130 GB configuration is written
// this way.
static void quant_row(const qctx * q, const float * w, int n, int nbits,
                      uint16_t * sd, uint8_t * sqf, uint16_t * md, uint8_t * mqf,
                      uint8_t * planes[3], uint8_t * codes_tmp, rng_t * rd) {
    const int ng = n / SSF_GROUP, nsb = ssf_nscale(n);
    const int nmax = (1 << nbits) - 1;
    const int fmax = q->six ? 63 : 255;
    const float mbias = q->six ? (q->minneg ? 63.0f : 31.0f) : 127.0f;
    int sqv[SSF_GPS], mqv[SSF_GPS];
    uint8_t * sq6 = NULL, * mq6 = NULL;
    for (int s = 0; s < nsb; s++) {
        const int g0 = s * SSF_GPS, g1 = g0 + SSF_GPS < ng ? g0 + SSF_GPS : ng;
        float step[SSF_GPS], mn[SSF_GPS], smax = 0.0f, mabs = 0.0f;
        for (int g = g0; g < g1; g++) {
            float lo, hi;
            if (rd) {
                lo = -q->sigma * (1.6f + 0.8f * rng_unit(rd));
                hi = q->sigma * (1.6f + 0.8f * rng_unit(rd));
            } else {
                lo = hi = w[g * SSF_GROUP];
                for (int j = 1; j < SSF_GROUP; j++) {
                    const float v = w[g * SSF_GROUP + j];
                    lo = v < lo ? v : lo; hi = v > hi ? v : hi;
                }
            }
            if (q->minneg && lo > 0.0f) lo = 0.0f;
            step[g - g0] = (hi - lo) / (float) nmax;
            mn[g - g0] = lo;
            smax = step[g - g0] > smax ? step[g - g0] : smax;
            mabs = fabsf(lo) > mabs ? fabsf(lo) : mabs;
        }
        const uint16_t d16 = ssfgen_f32_to_f16(smax / (float) fmax);
        const float dd = ssfgen_f16_to_f32(d16);
        const float mdiv = q->six ? (q->minneg ? 63.0f : 31.0f) : 127.0f;
        const uint16_t m16 = ssfgen_f32_to_f16(mabs / mdiv);
        const float mdd = ssfgen_f16_to_f32(m16);
        sd[s] = d16;
        md[s] = m16;
        for (int g = g0; g < g1; g++) {
            int sv = dd > 0.0f ? (int) lrintf(step[g - g0] / dd) : 0;
            // round up where rounding down would clip the group's top codes
            if (dd > 0.0f && (float) sv * dd < step[g - g0] && sv < fmax) sv++;
            sv = sv < 0 ? 0 : sv > fmax ? fmax : sv;
            int mv = mdd > 0.0f ? (int) lrintf(mn[g - g0] / mdd + mbias) : (int) mbias;
            mv = mv < 0 ? 0 : mv > fmax ? fmax : mv;
            sqv[g - g0] = sv;
            mqv[g - g0] = mv;
            const float es = dd * (float) sv, em = mdd * ((float) mv - mbias);
            if (rd) {
                for (int j = 0; j < SSF_GROUP; j += 8) {
                    const uint64_t b = rng_next(rd);
                    for (int k = 0; k < 8; k++) codes_tmp[g * SSF_GROUP + j + k] = (uint8_t) ((b >> (8 * k)) & (uint64_t) nmax);
                }
            } else for (int j = 0; j < SSF_GROUP; j++) {
                int c = es > 0.0f ? (int) lrintf((w[g * SSF_GROUP + j] - em) / es) : 0;
                c = c < 0 ? 0 : c > nmax ? nmax : c;
                codes_tmp[g * SSF_GROUP + j] = (uint8_t) c;
            }
            if (!q->six) { sqf[g] = (uint8_t) sv; mqf[g] = (uint8_t) mv; }
        }
        if (q->six) {
            // four groups to three bytes, in group order (tooling/sml_format.py:119-131)
            for (int g = g0; g < g1; g += 4) {
                sq6 = sqf + (g / 4) * 3;
                mq6 = mqf + (g / 4) * 3;
                const int * a = &sqv[g - g0], * b = &mqv[g - g0];
                sq6[0] = (uint8_t) (a[0] | (a[1] << 6));
                sq6[1] = (uint8_t) ((a[1] >> 2) | (a[2] << 4));
                sq6[2] = (uint8_t) ((a[2] >> 4) | (a[3] << 2));
                mq6[0] = (uint8_t) (b[0] | (b[1] << 6));
                mq6[1] = (uint8_t) ((b[1] >> 2) | (b[2] << 4));
                mq6[2] = (uint8_t) ((b[2] >> 4) | (b[3] << 2));
            }
        }
    }
    // planes
    int kinds[3], shifts[3];
    const int np = ssf_planes(nbits, kinds, shifts);
    for (int p = 0; p < np; p++) {
        uint8_t * dst = planes[p];
        const int kd = kinds[p], sh = shifts[p];
        if (kd == 4) {
            for (int qd = 0; qd < ng / 4; qd++)
                for (int half = 0; half < 2; half++)
                    for (int j = 0; j < SSF_GROUP; j++) {
                        const int ga = qd * 4 + half * 2;
                        const int lo = (codes_tmp[ga * SSF_GROUP + j] >> sh) & 15;
                        const int hi = (codes_tmp[(ga + 1) * SSF_GROUP + j] >> sh) & 15;
                        dst[qd * 64 + half * 32 + j] = (uint8_t) (lo | (hi << 4));
                    }
        } else if (kd == 2) {
            for (int pk = 0; pk < ng / 4; pk++)
                for (int j = 0; j < SSF_GROUP; j++) {
                    int b = 0;
                    for (int g = 0; g < 4; g++)
                        b |= ((codes_tmp[(pk * 4 + g) * SSF_GROUP + j] >> sh) & 3) << (2 * g);
                    dst[pk * 32 + j] = (uint8_t) b;
                }
        } else {
            for (int g = 0; g < ng; g++)
                for (int k = 0; k < 4; k++) {
                    int b = 0;
                    for (int j = 0; j < 8; j++)
                        b |= ((codes_tmp[g * SSF_GROUP + k * 8 + j] >> sh) & 1) << j;
                    dst[g * 4 + k] = (uint8_t) b;
                }
        }
    }
}

static void draw_row(const qctx * q, uint64_t stream, int row, float * w, int n, float sigma) {
    rng_t r = { mix64(q->seed * 0x100000001b3ull ^ (stream << 32) ^ (uint64_t) row) };
    for (int j = 0; j < n; j += 2) {
        float a, b;
        rng_gauss2(&r, &a, &b);
        w[j] = a * sigma;
        if (j + 1 < n) w[j + 1] = b * sigma;
    }
}

static int write_quant(int fd, const qctx * q, const tdesc * d) {
    const ssf_rec * r = &d->rec;
    const int n = d->cols, rows = d->rows, ng = n / SSF_GROUP, nsb = ssf_nscale(n);
    int kinds[3], shifts[3];
    const int np = ssf_planes(d->nbits, kinds, shifts);
    // rows are written in blocks so even a 151936-row head stays a few hundred MB
    const int block = 8192;
    const size_t frow = ssf_field_row_bytes(ng, q->six);
    uint16_t * sd = (uint16_t *) malloc((size_t) block * nsb * 2);
    uint16_t * md = (uint16_t *) malloc((size_t) block * nsb * 2);
    uint8_t * sqf = (uint8_t *) malloc((size_t) block * frow);
    uint8_t * mqf = (uint8_t *) malloc((size_t) block * frow);
    uint8_t * pl[3] = {0, 0, 0};
    for (int p = 0; p < np; p++) pl[p] = (uint8_t *) malloc((size_t) block * plane_row_bytes(kinds[p], n));
    int ok = sd && md && sqf && mqf;
    for (int r0 = 0; ok && r0 < rows; r0 += block) {
        const int r1 = r0 + block < rows ? r0 + block : rows;
#pragma omp parallel
        {
            float * w = (float *) malloc((size_t) n * sizeof(float));
            uint8_t * ct = (uint8_t *) malloc((size_t) n);
#pragma omp for schedule(static)
            for (int row = r0; row < r1; row++) {
                const int i = row - r0;
                uint8_t * planes[3];
                for (int p = 0; p < np; p++) planes[p] = pl[p] + (size_t) i * plane_row_bytes(kinds[p], n);
                rng_t rd = { mix64(q->seed * 0x100000001b3ull ^ 0x6469726563740000ull ^ (d->stream << 32) ^ (uint64_t) row) };
                if (!q->direct) draw_row(q, d->stream, row, w, n, q->sigma);
                quant_row(q, w, n, d->nbits, sd + (size_t) i * nsb, sqf + (size_t) i * frow,
                          md + (size_t) i * nsb, mqf + (size_t) i * frow, planes, ct, q->direct ? &rd : NULL);
            }
            free(w);
            free(ct);
        }
        const int nr = r1 - r0;
        ok = ok && pwrite_all(fd, sd, (uint64_t) nr * nsb * 2, r->sd_off + (uint64_t) r0 * nsb * 2);
        ok = ok && pwrite_all(fd, md, (uint64_t) nr * nsb * 2, r->md_off + (uint64_t) r0 * nsb * 2);
        ok = ok && pwrite_all(fd, sqf, (uint64_t) nr * frow, r->sq_off + (uint64_t) r0 * frow);
        ok = ok && pwrite_all(fd, mqf, (uint64_t) nr * frow, r->mq_off + (uint64_t) r0 * frow);
        for (int p = 0; p < np && ok; p++) {
            const uint64_t rb = plane_row_bytes(kinds[p], n);
            ok = pwrite_all(fd, pl[p], (uint64_t) nr * rb, r->codes_off[p] + (uint64_t) r0 * rb);
        }
    }
    free(sd); free(md); free(sqf); free(mqf);
    for (int p = 0; p < np; p++) free(pl[p]);
    return ok;
}

static int write_f32(int fd, const qctx * q, const tdesc * d) {
    const size_t cnt = (size_t) d->rows * d->cols;
    float * v = (float *) malloc(cnt * sizeof(float));
    if (!v) return 0;
    if (d->init == INIT_ONES) for (size_t i = 0; i < cnt; i++) v[i] = 1.0f;
    else for (int r = 0; r < d->rows; r++) draw_row(q, d->stream, r, v + (size_t) r * d->cols, d->cols, q->sigma);
    const int ok = pwrite_all(fd, v, cnt * 4, d->rec.off);
    free(v);
    return ok;
}

static int write_perm(int fd, const qctx * q, int p, int cols, uint64_t off, int mode) {
    int32_t * v = (int32_t *) malloc((size_t) cols * 4);
    if (!v) return 0;
    for (int i = 0; i < cols; i++) v[i] = i;
    if (mode == 1) {   // Fisher-Yates from the perm's own stream
        rng_t r = { mix64(q->seed ^ 0x7065726dull ^ ((uint64_t) p << 20)) };
        for (int i = cols - 1; i > 0; i--) {
            const int j = (int) (rng_next(&r) % (uint64_t) (i + 1));
            const int32_t t = v[i]; v[i] = v[j]; v[j] = t;
        }
    }
    const int ok = pwrite_all(fd, v, (uint64_t) cols * 4, off);
    free(v);
    return ok;
}

int ssfgen_write(const char * path, const ssfgen_spec * s, char * why, int nwhy) {
    const int E = (int) s->n_embd;
    const int qd = (int) (s->n_head * s->head_dim);
    const int F = (int) (s->n_expert ? s->expert_ff : s->n_ff);
    if (!s->n_layer || !E || !s->n_head || !s->n_head_kv || !s->head_dim || !F || !s->n_vocab ||
        s->n_head % s->n_head_kv || E % 128 || qd % 128 || F % 128 ||
        s->nbits < 2 || s->nbits > 8 || s->emb_nbits < 2 || s->emb_nbits > 8 ||
        (s->n_expert && (!s->n_expert_used || s->n_expert_used > s->n_expert))) {
        snprintf(why, (size_t) nwhy, "invalid model spec (widths must be multiples of 128, widths 2..8)");
        return 0;
    }
#ifdef _OPENMP
    if (s->threads > 0) omp_set_num_threads(s->threads);
#endif
    tlist L;
    memset(&L, 0, sizeof L);
    build_list(&L, s);
    const int six = s->scale6 != 0;
    uint64_t end = 0;
    layout(&L, six, &end);

    ssf_hdr h;
    memset(&h, 0, sizeof h);
    memcpy(h.magic, "SSF ", 4);
    h.version = 9;
    h.n_layer = s->n_layer; h.n_embd = s->n_embd; h.n_head = s->n_head; h.n_head_kv = s->n_head_kv;
    h.n_ff = (uint32_t) F; h.n_vocab = s->n_vocab; h.n_ctx_train = 32768;
    h.rope_theta = s->rope_theta; h.rms_eps = s->rms_eps;
    h.group = SSF_GROUP; h.n_levels = 1; h.level_bits[0] = 4;
    h.n_tensors = (uint64_t) L.n;
    h.table_off = SSF_HEADER_BYTES;
    h.flags = six ? (SSF_FLAG_SCALE6 | (s->minneg ? SSF_FLAG_MINNEG : 0u)) : 0u;
    h.n_expert_used = s->n_expert ? s->n_expert_used : 0;
    h.moe_flags = s->n_expert ? s->moe_flags : 0;

    const int fd = open(path, O_CREAT | O_TRUNC | O_WRONLY, 0644);
    if (fd < 0) { snprintf(why, (size_t) nwhy, "cannot create %s", path); return 0; }
    int ok = ftruncate(fd, (off_t) end) == 0;
    uint8_t * head = (uint8_t *) calloc(1, SSF_HEADER_BYTES);
    memcpy(head, &h, sizeof h);
    ok = ok && pwrite_all(fd, head, SSF_HEADER_BYTES, 0);
    free(head);
    for (int i = 0; ok && i < L.n; i++)
        ok = pwrite_all(fd, &L.t[i].rec, sizeof(ssf_rec), SSF_HEADER_BYTES + (uint64_t) i * sizeof(ssf_rec));
    const qctx q = { six, six && s->minneg, s->sigma > 0.0f ? s->sigma : 0.02f, s->seed, (int) s->direct };
    for (int p = 0; ok && p < L.n_perm; p++)
        ok = write_perm(fd, &q, p, L.perm_cols[p], L.perm_off[p], (int) s->perm_mode);
    for (int i = 0; ok && i < L.n; i++) {
        if (q.direct == 2 && L.t[i].expert) continue;   // left as a hole: drawn on the device at open
        ok = L.t[i].kind == SSF_KIND_F32 ? write_f32(fd, &q, &L.t[i]) : write_quant(fd, &q, &L.t[i]);
    }
    ok = (close(fd) == 0) && ok;
    free(L.t); free(L.perm_cols); free(L.perm_off);
    if (!ok) snprintf(why, (size_t) nwhy, "write to %s failed", path);
    return ok;
}
