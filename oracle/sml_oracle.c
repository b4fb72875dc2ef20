// TEST INFRASTRUCTURE ONLY -- a CPU restatement of the reference decode path,
// the checker for the CUDA engine. Not linked into the product.
//
// Each step cites the reference line it restates. Written as plain loops from
// the algorithm (codes unpacked to integers, one integer dot per group), with
// the reference's float operations in the reference's order: its vector
// kernels' accumulator chains and horizontal sums, the fused multiply-adds gcc
// forms from them under its default contraction (-ffp-contract=fast), the
// attention's chains, the SiLU's own exponential. The restatement therefore
// equals the reference build bit for bit (logits included), which the tests
// check against vectors the reference wrote.
#include "sml_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#define G 32

// ------------------------------------------------------------- format bits

#pragma pack(push, 1)
typedef struct {   // the 248-byte SSF record (sml/sml-model.h:83-103)
    char name[64];
    uint32_t kind, rows, cols, group;
    uint64_t off, nbytes, sd_off, sd_n, sq_off, sq_n, perm_off, perm_n, md_off, md_n, mq_off, mq_n;
    uint64_t codes_off[4], codes_n[4];
    uint32_t layout, nbits;
} rec_t;
#pragma pack(pop)

// sml/sml-kernel.c:14-39: binary16 -> binary32, exact
static float f16(uint16_t h) {
    const uint32_t s = (uint32_t) (h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 31u, m = h & 0x3ffu, b;
    if (!e) {
        if (!m) b = s;
        else { e = 113; while (!(m & 0x400u)) { m <<= 1; e--; } b = s | (e << 23) | ((m & 0x3ffu) << 13); }
    } else if (e == 31) b = s | 0x7f800000u | (m << 13);
    else b = s | ((e + 112) << 23) | (m << 13);
    float f; memcpy(&f, &b, 4); return f;
}

// sml/sml-run.c:76-96: binary32 -> binary16, round to nearest even (the KV cache)
static uint16_t to_f16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const int32_t e = (int32_t) ((x >> 23) & 0xff);
    uint32_t m = x & 0x7fffffu;
    if (e == 0xff) return (uint16_t) (sign | 0x7c00u | (m ? 0x200u : 0u));
    const int32_t he = e - 112;
    if (he >= 31) return (uint16_t) (sign | 0x7c00u);
    if (he <= 0) {
        if (he < -10) return (uint16_t) sign;
        m |= 0x800000u;
        const uint32_t sh = (uint32_t) (14 - he), half = 1u << (sh - 1);
        uint32_t v = m >> sh; const uint32_t rem = m & ((1u << sh) - 1u);
        if (rem > half || (rem == half && (v & 1u))) v++;
        return (uint16_t) (sign | v);
    }
    uint32_t v = ((uint32_t) he << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (v & 1u))) v++;
    return (uint16_t) (sign | v);
}

// sml/sml-kernel.h:65-96: a group's field, 8-bit or 6-bit (4 per 3 bytes)
static int field(const uint8_t * row, int g, int six) {
    if (!six) return row[g];
    const uint8_t * p = row + (g >> 2) * 3;
    const uint32_t b0 = p[0], b1 = p[1], b2 = p[2];
    switch (g & 3) {
    case 0: return (int) (b0 & 63u);
    case 1: return (int) (((b0 >> 6) | (b1 << 2)) & 63u);
    case 2: return (int) (((b1 >> 4) | (b2 << 4)) & 63u);
    default: return (int) ((b2 >> 2) & 63u);
    }
}

// ------------------------------------------------------------- activation

// sml/sml-kernel.c:89-109
void so_quantize_act(const float * x, int n, int8_t * q, float * scale, int32_t * sums) {
    for (int g = 0; g < n / G; g++) {
        float amax = 0.0f;
        for (int i = 0; i < G; i++) { const float v = fabsf(x[g * G + i]); if (v > amax) amax = v; }
        const float s = amax / 127.0f;
        const float is = s > 0.0f ? 1.0f / s : 0.0f;
        int32_t sum = 0;
        for (int i = 0; i < G; i++) {
            int v = (int) lrintf(x[g * G + i] * is);
            v = v > 127 ? 127 : v < -127 ? -127 : v;
            q[g * G + i] = (int8_t) v;
            sum += v;
        }
        scale[g] = s;
        sums[g] = sum;
    }
}

// sml/sml-kernel.c:161-189 (scalar arm of sml_quantize_act_sb)
void so_quantize_act_sb(const float * x, int n, int8_t * q, float * scale, int32_t * sums) {
    const int ng = n / G;
    for (int g0 = 0; g0 < ng; g0 += 8) {
        const int g1 = g0 + 8 < ng ? g0 + 8 : ng;
        float amax = 0.0f;
        for (int i = g0 * G; i < g1 * G; i++) { const float v = fabsf(x[i]); if (v > amax) amax = v; }
        const float s = amax / 127.0f;
        const float is = s > 0.0f ? 1.0f / s : 0.0f;
        for (int g = g0; g < g1; g++) {
            int32_t sum = 0;
            for (int i = 0; i < G; i++) {
                int v = (int) lrintf(x[g * G + i] * is);
                v = v > 127 ? 127 : v < -127 ? -127 : v;
                q[g * G + i] = (int8_t) v;
                sum += v;
            }
            scale[g] = s;
            sums[g] = sum;
        }
    }
}

// ------------------------------------------------------------- model

struct so_model {
    const uint8_t * base;
    size_t size;
    uint32_t n_layer, n_embd, n_head, n_kv, n_ff, n_vocab, flags, n_expert_used, moe_flags;
    float theta, eps;
    int six, minneg, hd, n_ctx, half;
    const rec_t * recs;
    uint64_t n_rec;
    uint16_t * kc, * vc;
    float * cos_t, * sin_t;
};

static const rec_t * find(const so_model * m, const char * name) {
    for (uint64_t i = 0; i < m->n_rec; i++)
        if (strncmp(m->recs[i].name, name, 64) == 0) return &m->recs[i];
    return NULL;
}
static const rec_t * findf(const so_model * m, const char * fmt, int a, int b) {
    char nm[80]; snprintf(nm, sizeof nm, fmt, a, b); return find(m, nm);
}
static const float * f32p(const so_model * m, const rec_t * r) {
    return r ? (const float *) (m->base + r->off) : NULL;
}

so_model * so_open(const char * path, int n_ctx) {
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return NULL;
    struct stat st;
    if (fstat(fd, &st)) { close(fd); return NULL; }
    void * b = mmap(NULL, (size_t) st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (b == MAP_FAILED) return NULL;
    so_model * m = (so_model *) calloc(1, sizeof *m);
    m->base = (const uint8_t *) b;
    m->size = (size_t) st.st_size;
    const uint8_t * h = m->base;
    // header fields at their HEADER_FMT offsets (tooling/sml_format.py:53-74)
    uint32_t u[8]; memcpy(u, h + 8, 28);
    m->n_layer = u[0]; m->n_embd = u[1]; m->n_head = u[2]; m->n_kv = u[3]; m->n_ff = u[4]; m->n_vocab = u[5];
    memcpy(&m->theta, h + 36, 4); memcpy(&m->eps, h + 40, 4);
    memcpy(&m->n_rec, h + 68, 8);
    uint64_t toff; memcpy(&toff, h + 76, 8);
    memcpy(&m->flags, h + 152, 4);
    memcpy(&m->n_expert_used, h + 168, 4); memcpy(&m->moe_flags, h + 172, 4);
    m->recs = (const rec_t *) (m->base + toff);
    m->six = (m->flags & 2u) != 0;
    m->minneg = m->six && (m->flags & 4u);
    const rec_t * q0 = findf(m, "blk.%d.attn_q.weight", 0, 0);
    m->hd = q0 ? (int) (q0->rows / m->n_head) : (int) (m->n_embd / m->n_head);
    m->n_ctx = n_ctx;
    m->half = m->hd / 2;
    const size_t kvd = (size_t) m->n_kv * m->hd;
    m->kc = (uint16_t *) calloc((size_t) m->n_layer * n_ctx * kvd, 2);
    m->vc = (uint16_t *) calloc((size_t) m->n_layer * n_ctx * kvd, 2);
    // RoPE tables, sml/sml-run.c:1383-1393
    m->cos_t = (float *) malloc((size_t) n_ctx * m->half * 4);
    m->sin_t = (float *) malloc((size_t) n_ctx * m->half * 4);
    for (int p = 0; p < n_ctx; p++)
        for (int i = 0; i < m->half; i++) {
            const float fr = powf(m->theta, -(float) i / (float) m->half);
            const float a = (float) p * fr;
            m->cos_t[(size_t) p * m->half + i] = cosf(a);
            m->sin_t[(size_t) p * m->half + i] = sinf(a);
        }
    return m;
}

void so_close(so_model * m) {
    if (!m) return;
    munmap((void *) m->base, m->size);
    free(m->kc); free(m->vc); free(m->cos_t); free(m->sin_t);
    free(m);
}

int so_info(const so_model * m, int * out) {
    out[0] = (int) m->n_layer; out[1] = (int) m->n_embd; out[2] = (int) m->n_head; out[3] = (int) m->n_kv;
    out[4] = m->hd; out[5] = (int) m->n_ff; out[6] = (int) m->n_vocab; out[7] = (int) m->flags;
    return (int) m->n_vocab;
}

// ------------------------------------------------------------- codes

// One row's codes as integers, permuted column order. Plane layouts:
//   nibble plane  sml/sml-kernel.c:2035-2046 (quad of 4 groups = 64 bytes;
//                 bytes 0-31 groups 4p|4p+1<<4, bytes 32-63 groups 4p+2|4p+3<<4)
//   2-bit plane   sml/sml-kernel.h:8-16 (128 weights in 32 bytes, group g in bits 2g)
//   1-bit plane   sml/sml-kernel.c:1986-1999 (4 bytes per group, bit j = weight j)
// and the per-width plane order of tooling/sml_quantize.py:106.
static void row_codes(const so_model * m, const rec_t * r, int row, uint8_t * c) {
    const int n = (int) r->cols;
    static const int kinds[9][3] = {{0},{0},{2},{2,1},{4},{4,1},{2,4},{4,2,1},{4,4}};
    static const int shifts[9][3] = {{0},{0},{0},{0,2},{0},{0,4},{4,0},{0,4,6},{0,4}};
    memset(c, 0, (size_t) n);
    for (int p = 0; p < 3; p++) {
        const int kd = kinds[r->nbits][p], sh = shifts[r->nbits][p];
        if (!kd) break;
        const uint8_t * pl = m->base + r->codes_off[p];
        for (int i = 0; i < n; i++) {
            const int g = i / G, j = i % G;
            int v;
            if (kd == 4) {
                const uint8_t b = pl[(size_t) row * (n / 2) + (g / 4) * 64 + ((g % 4) >= 2 ? 32 : 0) + j];
                v = (g & 1) ? (b >> 4) & 15 : b & 15;
            } else if (kd == 2) {
                const uint8_t b = pl[(size_t) row * (n / 4) + (g / 4) * 32 + j];
                v = (b >> (2 * (g % 4))) & 3;
            } else {
                const uint8_t b = pl[(size_t) row * (n / 8) + g * 4 + j / 8];
                v = (b >> (j % 8)) & 1;
            }
            c[i] = (uint8_t) (c[i] + (v << sh));
        }
    }
}

// Step and min of group g of a row: d*sq and md*(mq - bias), the bias 127 at
// 8 bits, 31 at 6 bits, 63 with MINNEG (sml/sml-kernel.c:246-250, 2146-2150).
static void group_grid(const so_model * m, const rec_t * r, int row, int g, float * step, float * mn) {
    const int n = (int) r->cols, ng = n / G, nsb = (ng + 7) / 8;
    const size_t frow = m->six ? (size_t) (ng / 4) * 3 : (size_t) ng;
    const uint16_t * sd = (const uint16_t *) (m->base + r->sd_off);
    const uint8_t * sq = m->base + r->sq_off;
    *step = f16(sd[(size_t) row * nsb + g / 8]) * (float) field(sq + row * frow, g, m->six);
    *mn = 0.0f;
    if (r->mq_n) {
        const uint16_t * md = (const uint16_t *) (m->base + r->md_off);
        const uint8_t * mq = m->base + r->mq_off;
        const float bias = m->six ? (m->minneg ? 63.0f : 31.0f) : 127.0f;
        *mn = f16(md[(size_t) row * nsb + g / 8]) * ((float) field(mq + row * frow, g, m->six) - bias);
    }
}

int so_codes_row(so_model * m, const char * name, int row, uint8_t * out) {
    const rec_t * r = find(m, name);
    if (!r || r->kind != 1 || r->layout != 1 || row < 0 || row >= (int) r->rows) return 0;
    row_codes(m, r, row, out);
    return 1;
}

// sml/sml-kernel.c:2134-2158: w = code * step + min
int so_dequant_row(so_model * m, const char * name, int row, float * out) {
    const rec_t * r = find(m, name);
    if (!r || r->kind != 1 || r->layout != 1 || row < 0 || row >= (int) r->rows) return 0;
    uint8_t * c = (uint8_t *) malloc(r->cols);
    row_codes(m, r, row, c);
    for (int g = 0; g < (int) r->cols / G; g++) {
        float st, mn;
        group_grid(m, r, row, g, &st, &mn);
        for (int j = 0; j < G; j++) out[g * G + j] = (float) c[g * G + j] * st + mn;
    }
    free(c);
    return 1;
}

// One plane's unsigned values of one row (permuted column order).
static void row_plane(const so_model * m, const rec_t * r, int row, int p, uint8_t * c) {
    static const int kinds[9][3] = {{0},{0},{2},{2,1},{4},{4,1},{2,4},{4,2,1},{4,4}};
    const int n = (int) r->cols, kd = kinds[r->nbits][p];
    const uint8_t * pl = m->base + r->codes_off[p];
    for (int i = 0; i < n; i++) {
        const int g = i / G, j = i % G;
        int v;
        if (kd == 4) {
            const uint8_t b = pl[(size_t) row * (n / 2) + (g / 4) * 64 + ((g % 4) >= 2 ? 32 : 0) + j];
            v = (g & 1) ? (b >> 4) & 15 : b & 15;
        } else if (kd == 2) {
            const uint8_t b = pl[(size_t) row * (n / 4) + (g / 4) * 32 + j];
            v = (b >> (2 * (g % 4))) & 3;
        } else {
            const uint8_t b = pl[(size_t) row * (n / 8) + g * 4 + j / 8];
            v = (b >> (j % 8)) & 1;
        }
        c[i] = (uint8_t) v;
    }
}

// The reference's float epilogues, each restated in its own order (a group's
// integer dot is exact whatever the order; the float sums are not):
//
// ep_flat -- matvec_flat4_l8 (sml/sml-kernel.c:572-718), which the decode
//   copy's sml_matvec_rows_il4/il6 (:836-905) and the fused 6-bit kernel
//   (:919-1005) repeat "in the same order" (:816): eight accumulators,
//   accumulator L taking groups 8k+L in k order, each group two fused
//   multiply-adds, acc = fma(d*sq, xs*dot, acc) then fma(md*(mq - bias), xs*sum,
//   acc) (gcc contracts the intrinsics' add(acc, mul(..)) under its default
//   -ffp-contract=fast); a 4-group tail in four more (:664-705); the horizontal
//   sum ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)), plus the tail's (t0+t1)+(t2+t3)
//   (:707-716).
// ep_ladder -- sml_matvec_rows (:298-370): four accumulators (groups 4p+L), the
//   dot scaled by 2^shift, the same two fused steps; sum (a0+a1)+(a2+a3).
// ep_bits1 -- sml_matvec_bits1 (:1036-1063): one scalar sum over the groups
//   whose bit word is not zero, tot = fma(d*sq*xs, dot, tot), no min term,
//   added to y as y + tot*2^shift.
static float ep_flat(const int32_t * d, int ng, const float * st, const float * mn, const float * xs,
                     const int32_t * sums) {
    const int nblk = ng / 8;
    float a[8] = {0}, t[4] = {0};
    for (int g = 0; g < ng; g++) {
        float * acc = g < nblk * 8 ? &a[g % 8] : &t[g % 4];
        *acc = fmaf(st[g], xs[g] * (float) d[g], *acc);
        if (mn) *acc = fmaf(mn[g], xs[g] * (float) sums[g], *acc);
    }
    float tot = ((a[0] + a[4]) + (a[1] + a[5])) + ((a[2] + a[6]) + (a[3] + a[7]));
    if (ng > nblk * 8) tot += (t[0] + t[1]) + (t[2] + t[3]);
    return tot;
}

static float ep_ladder(const int32_t * d, int ng, float mul, const float * st, const float * mn, const float * xs,
                       const int32_t * sums) {
    float a[4] = {0};
    for (int g = 0; g < ng; g++) {
        a[g % 4] = fmaf(st[g], xs[g] * ((float) d[g] * mul), a[g % 4]);
        if (mn) a[g % 4] = fmaf(mn[g], xs[g] * (float) sums[g], a[g % 4]);
    }
    return (a[0] + a[1]) + (a[2] + a[3]);
}

static float ep_bits1(const int32_t * d, const uint8_t * nz, int ng, const float * st, const float * xs) {
    float tot = 0.0f;
    for (int g = 0; g < ng; g++)
        if (nz[g]) tot = fmaf(st[g] * xs[g], (float) d[g], tot);
    return tot;
}

// y[row0..row1) = W x, x gathered through the tensor's column order and
// quantized per 32 (sml/sml-run.c:711-760), each width through the kernels
// the reference's decode dispatch picks (issue_rows_act, sml/sml-run.c:612-680):
// Q2 ladder; Q3 ladder + bit plane x4; Q4 flat; Q5 flat + bit plane x16; Q6 the
// fused flat form (two passes -- ladder x16 with the min, then flat without --
// when the groups are not whole 8-group blocks, :929-936); Q7 as Q6 + bit plane
// x64; Q8 flat over lo + 16 hi. y starts at 0 and each pass adds its sum.
static void matvec_rec(const so_model * m, const rec_t * r, const float * x, float * y, int row0, int row1) {
    const int n = (int) r->cols, ng = n / G, nb = (int) r->nbits;
    const int32_t * perm = (const int32_t *) (m->base + r->perm_off);
    float * xg = (float *) malloc((size_t) n * 4);
    int8_t * q = (int8_t *) malloc((size_t) n);
    float * xs = (float *) malloc((size_t) ng * 4);
    int32_t * sums = (int32_t *) malloc((size_t) ng * 4);
    for (int i = 0; i < n; i++) xg[i] = x[perm[i]];          // sml/sml-kernel.c:253-255
    so_quantize_act(xg, n, q, xs, sums);
    const int np = nb == 2 || nb == 4 ? 1 : nb == 7 ? 3 : 2;
#pragma omp parallel for schedule(static)
    for (int row = row0; row < row1; row++) {
        uint8_t * c = (uint8_t *) malloc((size_t) n * 3);
        int32_t * d = (int32_t *) malloc((size_t) ng * 3 * 4);
        float * st = (float *) malloc((size_t) ng * 4), * mn = (float *) malloc((size_t) ng * 4);
        uint8_t * nz = (uint8_t *) malloc((size_t) ng);
        for (int p = 0; p < np; p++) row_plane(m, r, row, p, c + (size_t) p * n);
        for (int p = 0; p < np; p++)
            for (int g = 0; g < ng; g++) {
                int32_t s = 0;
                for (int j = 0; j < G; j++) s += (int32_t) c[(size_t) p * n + g * G + j] * (int32_t) q[g * G + j];
                d[p * ng + g] = s;
            }
        for (int g = 0; g < ng; g++) {
            group_grid(m, r, row, g, &st[g], &mn[g]);
            nz[g] = 0;
            if (np > 1) for (int j = 0; j < G; j++) nz[g] |= c[(size_t) (np - 1) * n + g * G + j];
        }
        const float * mnp = r->mq_n ? mn : NULL;
        const int whole = ng % 8 == 0;
        float acc = 0.0f;
        int32_t * comb = (int32_t *) malloc((size_t) ng * 4);
        switch (nb) {
        case 2: acc = 0.0f + ep_ladder(d, ng, 1.0f, st, mnp, xs, sums); break;
        case 3: acc = 0.0f + ep_ladder(d, ng, 1.0f, st, mnp, xs, sums);
                acc = acc + ep_bits1(d + ng, nz, ng, st, xs) * 4.0f; break;
        case 4: acc = 0.0f + ep_flat(d, ng, st, mnp, xs, sums); break;
        case 5: acc = 0.0f + ep_flat(d, ng, st, mnp, xs, sums);
                acc = acc + ep_bits1(d + ng, nz, ng, st, xs) * 16.0f; break;
        case 6: case 7: {
            const int32_t * nib = nb == 6 ? d + ng : d, * two = nb == 6 ? d : d + ng;
            if (whole) {
                for (int g = 0; g < ng; g++) comb[g] = nib[g] + 16 * two[g];
                acc = 0.0f + ep_flat(comb, ng, st, mnp, xs, sums);
            } else {
                acc = 0.0f + ep_ladder(two, ng, 16.0f, st, mnp, xs, sums);
                acc = acc + ep_flat(nib, ng, st, NULL, xs, sums);
            }
            if (nb == 7) acc = acc + ep_bits1(d + 2 * ng, nz, ng, st, xs) * 64.0f;
            break;
        }
        default:
            for (int g = 0; g < ng; g++) comb[g] = d[g] + 16 * d[ng + g];
            acc = 0.0f + ep_flat(comb, ng, st, mnp, xs, sums);
            break;
        }
        y[row] = acc;
        free(comb); free(c); free(d); free(st); free(mn); free(nz);
    }
    free(xg); free(q); free(xs); free(sums);
}

// ------------------------------------------------------------- batched path

// The batched path's weights (sml_g_requant8, sml/sml-gpu-fast.cu:1804-1880):
// per row and 256-weight superblock, bound = the largest |w| its groups can
// take, max(|m|, |s*cmax + m|) with s = d*sq, m = md*(mq - bias) and s*cmax + m
// fused; s8 = bound/127; w8 = rint(fma(code, s*inv, m*inv)) with inv = 127/bound.
// Generalized from the reference's 4- and 6-bit codes with 8-bit fields to every
// width (cmax = 2^nbits - 1) and the file's min bias. w8: rows x (nsb * 256),
// zero past the last group; s8: rows x nsb.
int so_requant8(so_model * m, const char * name, int8_t * w8, float * s8) {
    const rec_t * r = find(m, name);
    if (!r || r->kind != 1 || r->layout != 1) return 0;
    const int n = (int) r->cols, ng = n / G, nsb = (ng + 7) / 8, K = nsb * 256;
    const float cmax = (float) ((1 << r->nbits) - 1);
#pragma omp parallel for schedule(static)
    for (int row = 0; row < (int) r->rows; row++) {
        uint8_t * c = (uint8_t *) malloc((size_t) n);
        row_codes(m, r, row, c);
        int8_t * wr = w8 + (size_t) row * K;
        memset(wr, 0, (size_t) K);
        for (int sb = 0; sb < nsb; sb++) {
            const int g0 = sb * 8, g1 = g0 + 8 < ng ? g0 + 8 : ng;
            float bound = 0.0f;
            for (int g = g0; g < g1; g++) {
                float st, mn;
                group_grid(m, r, row, g, &st, &mn);
                const float top = fmaf(st, cmax, mn);
                const float am = fabsf(mn), at = fabsf(top), b = am > at ? am : at;
                bound = b > bound ? b : bound;
            }
            s8[(size_t) row * nsb + sb] = bound / 127.0f;
            const float inv = bound > 0.0f ? 127.0f / bound : 0.0f;
            for (int g = g0; g < g1; g++) {
                float st, mn;
                group_grid(m, r, row, g, &st, &mn);
                const float ka = st * inv, kb = mn * inv;
                for (int j = 0; j < G; j++) wr[g * G + j] = (int8_t) rintf(fmaf((float) c[g * G + j], ka, kb));
            }
        }
        free(c);
    }
    return 1;
}

// The batched product for one activation row (sml_g_tcm3/tcm9 epilogue,
// sml/sml-gpu-fast.cu:2025-2031): the row gathered through the tensor's column
// order and quantized per 256 (one scale per superblock, sml_quantize_act_sb,
// sml/sml-kernel.c:164-189), then y[row] = sum over superblocks, in order, of
// fma(s8 * xs, dot(w8, xq), acc). With split > 1 (sml_g_tcm3 +
// sml_g_splitk_sum, sml/sml-gpu-fast.cu:1919-1921, 2057-2065) the superblocks
// are cut into runs of ceil(nsb / split), each run accumulated from zero as
// above, and y = ((0 + run 0) + run 1) + ...
static void sb_row(const int8_t * w8, const float * s8, const int32_t * perm, int n, int rows, const float * x,
                   int split, float * y) {
    const int ng = n / G, nsb = (ng + 7) / 8, K = nsb * 256, per = (nsb + split - 1) / split;
    int8_t * q = (int8_t *) calloc((size_t) K, 1);
    float * xs = (float *) malloc((size_t) nsb * 4), * xg = (float *) malloc((size_t) n * 4);
    for (int i = 0; i < n; i++) xg[i] = x[perm[i]];
    {
        // the per-256 activation (sml_quantize_act_sb); past n the codes stay 0
        float * gs = (float *) malloc((size_t) ng * 4);
        int32_t * gsum = (int32_t *) malloc((size_t) ng * 4);
        so_quantize_act_sb(xg, n, q, gs, gsum);
        for (int sb = 0; sb < nsb; sb++) xs[sb] = gs[sb * 8];
        free(gs); free(gsum);
    }
#pragma omp parallel for schedule(static)
    for (int row = 0; row < rows; row++) {
        const int8_t * wr = w8 + (size_t) row * K;
        float yv = 0.0f;
        for (int s0 = 0; s0 < nsb; s0 += per) {
            float acc = 0.0f;
            for (int sb = s0; sb < s0 + per && sb < nsb; sb++) {
                int32_t d = 0;
                for (int i = sb * 256; i < sb * 256 + 256; i++) d += (int32_t) wr[i] * (int32_t) q[i];
                acc = fmaf(s8[(size_t) row * nsb + sb] * xs[sb], (float) d, acc);
            }
            yv = per >= nsb ? acc : yv + acc;
        }
        y[row] = yv;
    }
    free(q); free(xs); free(xg);
}

// The batched product over T rows of X (T x cols) into Y (T x rows).
int so_gemm_sb_split(so_model * m, const char * name, const float * X, int T, int split, float * Y) {
    const rec_t * r = find(m, name);
    if (!r || r->kind != 1 || r->layout != 1 || T < 1 || split < 1) return 0;
    const int n = (int) r->cols, nsb = (n / G + 7) / 8, rows = (int) r->rows;
    int8_t * w8 = (int8_t *) malloc((size_t) rows * nsb * 256);
    float * s8 = (float *) malloc((size_t) rows * nsb * 4);
    so_requant8(m, name, w8, s8);
    const int32_t * perm = (const int32_t *) (m->base + r->perm_off);
    for (int t = 0; t < T; t++) sb_row(w8, s8, perm, n, rows, X + (size_t) t * n, split, Y + (size_t) t * rows);
    free(w8); free(s8);
    return 1;
}

int so_gemm_sb(so_model * m, const char * name, const float * X, int T, float * Y) {
    return so_gemm_sb_split(m, name, X, T, 1, Y);
}

static void matvec_f32(const float * w, int rows, int n, const float * x, float * y) {
    for (int i = 0; i < rows; i++) {                         // sml/sml-run.c:3076-3081
        double s = 0.0;
        for (int j = 0; j < n; j++) s += (double) w[(size_t) i * n + j] * x[j];
        y[i] = (float) s;
    }
}

int so_matvec(so_model * m, const char * name, const float * x, float * y, int row0, int row1) {
    const rec_t * r = find(m, name);
    if (!r || r->kind != 1 || r->layout != 1) return 0;
    matvec_rec(m, r, x, y, row0, row1);
    return 1;
}

// ------------------------------------------------------------- forward pieces

// sml/sml-run.c:147-152
static void rms_norm(float * out, const float * x, const float * w, int n, float eps) {
    double ss = 0.0;
    for (int i = 0; i < n; i++) ss += (double) x[i] * x[i];
    const float s = 1.0f / sqrtf((float) (ss / n) + eps);
    for (int i = 0; i < n; i++) out[i] = x[i] * s * w[i];
}

// sml/sml-run.c:339-375, halved pairs (i, i + half), as gcc's default
// contraction builds the two lines: x[i] = fma(a, cos, -(b*sin)),
// x[i + half] = fma(a, sin, b*cos) (the form the reference build's decode
// matches bit for bit; the other pairings do not).
static void rope(const so_model * m, float * v, int nh, int pos) {
    const float * cs = m->cos_t + (size_t) pos * m->half, * sn = m->sin_t + (size_t) pos * m->half;
    for (int h = 0; h < nh; h++) {
        float * x = v + (size_t) h * m->hd;
        for (int i = 0; i < m->half; i++) {
            const float a = x[i], b = x[i + m->half];
            x[i] = fmaf(a, cs[i], -(b * sn[i]));
            x[i + m->half] = fmaf(a, sn[i], b * cs[i]);
        }
    }
}

// sml/sml-run.c:295-325, one RMS norm per head sharing a head_dim weight
static void qk_norm(float * v, const float * w, int nh, int hd, float eps) {
    for (int h = 0; h < nh; h++) rms_norm(v + (size_t) h * hd, v + (size_t) h * hd, w, hd, eps);
}

// attn_row (sml/sml-run.c:180-266), the AVX2 arm's order: a position's score
// as eight fused multiply-add chains (chain l over dims l, l+8, ...), reduced
// ((c0+c4)+(c1+c5)) + ((c2+c6)+(c3+c7)) (sml_hsum256 :111-119), times 1/sqrt(hd);
// softmax with libm expf, the sum in position order, then times 1/sum
// (:280-288); the output per dim one fused multiply-add chain over the
// positions in order (:236-253; hd % 64 == 0, else the same per dim, :256-265).
static void attn_head(const so_model * m, const uint16_t * kc, const uint16_t * vc, int L, int h, int pos,
                      const float * q, float * out, float * sc) {
    const int hd = m->hd, kvd = (int) m->n_kv * hd, rep = (int) (m->n_head / m->n_kv);
    const size_t base = (size_t) L * m->n_ctx * kvd + (size_t) (h / rep) * hd;
    const float inv = 1.0f / sqrtf((float) hd);
    for (int t = 0; t <= pos; t++) {
        const uint16_t * k = kc + base + (size_t) t * kvd;
        float c[8] = {0};
        for (int i = 0; i < hd; i++) c[i % 8] = fmaf(q[i], f16(k[i]), c[i % 8]);
        const float s = ((c[0] + c[4]) + (c[1] + c[5])) + ((c[2] + c[6]) + (c[3] + c[7]));
        sc[t] = s * inv;
    }
    float mx = sc[0];
    for (int t = 1; t <= pos; t++) if (sc[t] > mx) mx = sc[t];
    float sum = 0.0f;
    for (int t = 0; t <= pos; t++) { sc[t] = expf(sc[t] - mx); sum += sc[t]; }
    const float is = 1.0f / sum;
    for (int t = 0; t <= pos; t++) sc[t] *= is;
    for (int i = 0; i < hd; i++) out[i] = 0.0f;
    for (int t = 0; t <= pos; t++) {
        const uint16_t * v = vc + base + (size_t) t * kvd;
        for (int i = 0; i < hd; i++) out[i] = fmaf(sc[t], f16(v[i]), out[i]);
    }
}

// The AVX2 arm's exp of silu_mul (sml_exp_ps, sml/sml-run.c:392-413): x clamped
// to [-88, 88], f = x*log2(e), r = f rounded to nearest even, 2^(f-r) by a
// degree-5 polynomial in Horner form (each step one fused multiply-add under
// gcc's contraction), times 2^r through the exponent field.
static float exp_ps1(float x) {
    x = fminf(fmaxf(x, -88.0f), 88.0f);
    const float f = x * 1.44269504088896341f;
    const float r = rintf(f);
    const float g = f - r;
    float p = 1.3697664e-3f;
    p = fmaf(p, g, 8.3013611e-3f);
    p = fmaf(p, g, 5.5826318e-2f);
    p = fmaf(p, g, 2.4022652e-1f);
    p = fmaf(p, g, 6.9314718e-1f);
    p = fmaf(p, g, 1.0f);
    uint32_t e = (uint32_t) ((int) r + 127) << 23;
    float s;
    memcpy(&s, &e, 4);
    return p * s;
}

// silu_mul (sml/sml-run.c:436-446): blocks of 8 through the vector exp,
// (g / (1 + exp(0 - g))) * u; a tail past the last block of 8 with libm expf.
static void silu_mul(float * g, const float * u, int n) {
    const int n8 = n / 8 * 8;
    for (int i = 0; i < n8; i++) g[i] = (g[i] / (1.0f + exp_ps1(0.0f - g[i]))) * u[i];
    for (int i = n8; i < n; i++) g[i] = (g[i] / (1.0f + expf(-g[i]))) * u[i];
}

// sml/sml-run.c:3009-3030: top-k on the logits (ties to the lower index), then
// softmax over the chosen (bit 0) or over all experts
int so_moe_route(const float * lg, int ne, int k, unsigned moe_flags, int * sel, float * w) {
    if (k <= 0 || k > ne) k = ne;
    if (k > 16) k = 16;
    for (int j = 0; j < k; j++) {
        int best = -1;
        for (int e = 0; e < ne; e++) {
            int taken = 0;
            for (int q = 0; q < j; q++) taken |= sel[q] == e;
            if (!taken && (best < 0 || lg[e] > lg[best])) best = e;
        }
        sel[j] = best;
    }
    if (moe_flags & 1u) {
        double sum = 0.0;
        for (int j = 0; j < k; j++) { w[j] = expf(lg[sel[j]] - lg[sel[0]]); sum += w[j]; }
        for (int j = 0; j < k; j++) w[j] = (float) (w[j] / sum);
    } else {
        float mx = lg[0];
        for (int e = 1; e < ne; e++) if (lg[e] > mx) mx = lg[e];
        double sum = 0.0;
        for (int e = 0; e < ne; e++) sum += expf(lg[e] - mx);
        for (int j = 0; j < k; j++) w[j] = (float) (expf(lg[sel[j]] - mx) / sum);
    }
    return k;
}

// sml/sml-run.c:3071-3125 (gated experts, no shared expert); the chosen
// experts and weights go to sel_out / w_out when they are not NULL
static int moe_ffn(so_model * m, int L, const float * xb, float * out, int * sel_out, float * w_out) {
    const int E = (int) m->n_embd;
    const rec_t * rt = findf(m, "blk.%d.ffn_gate_inp.weight", L, 0);
    const int ne = (int) ((uint64_t) rt->rows * rt->cols / E);
    float * lg = (float *) malloc((size_t) ne * 4);
    matvec_f32(f32p(m, rt), ne, E, xb, lg);
    int sel[16]; float w[16];
    const int k = so_moe_route(lg, ne, (int) m->n_expert_used, m->moe_flags, sel, w);
    for (int j = 0; j < k; j++) {
        if (sel_out) sel_out[j] = sel[j];
        if (w_out) w_out[j] = w[j];
    }
    const rec_t * u0 = findf(m, "blk.%d.ffn_up.%d.weight", L, 0);
    const int F = (int) u0->rows;
    float * g = (float *) malloc((size_t) F * 4), * u = (float *) malloc((size_t) F * 4);
    float * t = (float *) malloc((size_t) E * 4);
    for (int i = 0; i < E; i++) out[i] = 0.0f;
    for (int j = 0; j < k; j++) {
        matvec_rec(m, findf(m, "blk.%d.ffn_gate.%d.weight", L, sel[j]), xb, g, 0, F);
        matvec_rec(m, findf(m, "blk.%d.ffn_up.%d.weight", L, sel[j]), xb, u, 0, F);
        silu_mul(g, u, F);
        matvec_rec(m, findf(m, "blk.%d.ffn_down.%d.weight", L, sel[j]), g, t, 0, E);
        for (int i = 0; i < E; i++) out[i] = fmaf(w[j], t[i], out[i]);   // acc += w*t, contracted
    }
    free(lg); free(g); free(u); free(t);
    return k;
}

void so_moe_combine(int T, int k, int E, const float * w, const float * yk, float * y) {
    for (int t = 0; t < T; t++) {
        float * yt = y + (size_t) t * E;
        for (int i = 0; i < E; i++) yt[i] = 0.0f;
        for (int j = 0; j < k; j++)
            for (int i = 0; i < E; i++)
                yt[i] = fmaf(w[(size_t) t * k + j], yk[((size_t) t * k + j) * E + i], yt[i]);
    }
}

// One expert's FFN of layer L on one normalized row: down(silu(gate x) * up x)
// (the body of the choice loop of moe_ffn, sml/sml-run.c:3098-3121, before its
// weighting). 0 if the expert does not exist.
int so_moe_expert(so_model * m, int L, int e, const float * xb, float * out) {
    const rec_t * g = findf(m, "blk.%d.ffn_gate.%d.weight", L, e), * u = findf(m, "blk.%d.ffn_up.%d.weight", L, e);
    const rec_t * d = findf(m, "blk.%d.ffn_down.%d.weight", L, e);
    if (!g || !u || !d) return 0;
    const int F = (int) g->rows, E = (int) m->n_embd;
    float * gv = (float *) malloc((size_t) F * 4), * uv = (float *) malloc((size_t) F * 4);
    matvec_rec(m, g, xb, gv, 0, F);
    matvec_rec(m, u, xb, uv, 0, F);
    silu_mul(gv, uv, F);
    matvec_rec(m, d, gv, out, 0, E);
    free(gv); free(uv);
    return 1;
}

// The MoE FFN of layer L on one (already normalized) row: returns the experts
// per token, 0 if layer L has no router.
int so_moe_ffn(so_model * m, int L, const float * xb, float * out, int * sel, float * w) {
    if (L < 0 || L >= (int) m->n_layer || !findf(m, "blk.%d.ffn_gate_inp.weight", L, 0)) return 0;
    return moe_ffn(m, L, xb, out, sel, w);
}

static void add_bias(float * y, const float * b, int n) { if (b) for (int i = 0; i < n; i++) y[i] += b[i]; }

// The products of one step, by kind: 0 q/k/v, 1 o, 2 gate/up, 3 down, 4 head.
typedef void (*lin_fn)(void * ctx, so_model * m, const rec_t * r, int kind, const float * x, float * y);

static void lin_decode(void * ctx, so_model * m, const rec_t * r, int kind, const float * x, float * y) {
    (void) ctx; (void) kind;
    matvec_rec(m, r, x, y, 0, (int) r->rows);
}

// sml/sml-run.c:3243-3523, the dense / MoE decoder branch, over the caches kc/vc
static int forward_core(so_model * m, uint16_t * kc, uint16_t * vc, int tok, int pos, float * logits, lin_fn lin,
                        void * lctx) {
    if (pos >= m->n_ctx || tok < 0 || tok >= (int) m->n_vocab) return 0;
    const int E = (int) m->n_embd, hd = m->hd, nh = (int) m->n_head, nkv = (int) m->n_kv;
    const int qd = nh * hd, kvd = nkv * hd;
    const int wide = (int) (m->n_ff > (uint32_t) E ? m->n_ff : (uint32_t) E) > qd
                   ? (int) (m->n_ff > (uint32_t) E ? m->n_ff : (uint32_t) E) : qd;
    float * x = (float *) calloc((size_t) E, 4), * xb = (float *) calloc((size_t) wide, 4);
    float * q = (float *) malloc((size_t) qd * 4), * k = (float *) malloc((size_t) kvd * 4);
    float * v = (float *) malloc((size_t) kvd * 4), * att = (float *) malloc((size_t) qd * 4);
    float * hb = (float *) malloc((size_t) wide * 4), * hb2 = (float *) malloc((size_t) wide * 4);
    float * sc = (float *) malloc((size_t) m->n_ctx * 4);
    // embedding row, dequantized, scattered back through its perm (:3283-3338)
    const rec_t * emb = find(m, "token_embd.weight");
    so_dequant_row(m, "token_embd.weight", tok, xb);
    const int32_t * pe = (const int32_t *) (m->base + emb->perm_off);
    for (int i = 0; i < E; i++) x[pe[i]] = xb[i];
    for (int L = 0; L < (int) m->n_layer; L++) {
        rms_norm(xb, x, f32p(m, findf(m, "blk.%d.attn_norm.weight", L, 0)), E, m->eps);
        lin(lctx, m, findf(m, "blk.%d.attn_q.weight", L, 0), 0, xb, q);
        lin(lctx, m, findf(m, "blk.%d.attn_k.weight", L, 0), 0, xb, k);
        lin(lctx, m, findf(m, "blk.%d.attn_v.weight", L, 0), 0, xb, v);
        add_bias(q, f32p(m, findf(m, "blk.%d.attn_q.bias", L, 0)), qd);
        add_bias(k, f32p(m, findf(m, "blk.%d.attn_k.bias", L, 0)), kvd);
        add_bias(v, f32p(m, findf(m, "blk.%d.attn_v.bias", L, 0)), kvd);
        const float * qn = f32p(m, findf(m, "blk.%d.attn_q_norm.weight", L, 0));
        const float * kn = f32p(m, findf(m, "blk.%d.attn_k_norm.weight", L, 0));
        if (qn) qk_norm(q, qn, nh, hd, m->eps);
        if (kn) qk_norm(k, kn, nkv, hd, m->eps);
        rope(m, q, nh, pos);
        rope(m, k, nkv, pos);
        const size_t at = ((size_t) L * m->n_ctx + pos) * kvd;   // :3414-3415
        for (int i = 0; i < kvd; i++) { kc[at + i] = to_f16(k[i]); vc[at + i] = to_f16(v[i]); }
        for (int h = 0; h < nh; h++) attn_head(m, kc, vc, L, h, pos, q + (size_t) h * hd, att + (size_t) h * hd, sc);
        lin(lctx, m, findf(m, "blk.%d.attn_output.weight", L, 0), 1, att, hb2);
        for (int i = 0; i < E; i++) x[i] += hb2[i];
        rms_norm(xb, x, f32p(m, findf(m, "blk.%d.ffn_norm.weight", L, 0)), E, m->eps);
        if (findf(m, "blk.%d.ffn_gate_inp.weight", L, 0)) {
            moe_ffn(m, L, xb, hb2, NULL, NULL);
            for (int i = 0; i < E; i++) x[i] += hb2[i];
            continue;
        }
        const int F = (int) m->n_ff;
        lin(lctx, m, findf(m, "blk.%d.ffn_gate.weight", L, 0), 2, xb, hb);
        lin(lctx, m, findf(m, "blk.%d.ffn_up.weight", L, 0), 2, xb, hb2);
        silu_mul(hb, hb2, F);
        lin(lctx, m, findf(m, "blk.%d.ffn_down.weight", L, 0), 3, hb, xb);
        for (int i = 0; i < E; i++) x[i] += xb[i];
    }
    rms_norm(xb, x, f32p(m, find(m, "output_norm.weight")), E, m->eps);
    const rec_t * head = find(m, "output.weight");
    lin(lctx, m, head ? head : emb, 4, xb, logits);
    free(x); free(xb); free(q); free(k); free(v); free(att); free(hb); free(hb2); free(sc);
    int best = 0;                                                  // sml/sml-run.c:3539-3544
    for (int i = 1; i < (int) m->n_vocab; i++) if (logits[i] > logits[best]) best = i;
    return best;
}

int so_forward(so_model * m, int tok, int pos, float * logits) {
    return forward_core(m, m->kc, m->vc, tok, pos, logits, lin_decode, NULL);
}

int so_decode(so_model * m, const int * prompt, int np, int ngen, int * ids, float * logits) {
    const int nv = (int) m->n_vocab;
    float * lg = (float *) malloc((size_t) nv * 4);
    int t = 0;
    for (int i = 0; i < np; i++) t = so_forward(m, prompt[i], i, lg);
    for (int g = 0; g < ngen; g++) {
        ids[g] = t;
        if (logits) memcpy(logits + (size_t) g * nv, lg, (size_t) nv * 4);
        if (g + 1 < ngen) t = so_forward(m, t, np + g, lg);
    }
    free(lg);
    return 1;
}

// ------------------------------------------------------------- batched serving

// sml_forward_multi (sml/sml-run.c:2559-2604): ns sequences, one token each,
// each with its own cache and position. mode 0: every sequence through the
// decode arithmetic (SML_MULTI=exact); mode 1: every product on the batched
// path's arithmetic (so_gemm_sb_split with the splits set per kind, the
// re-quantized weights made once per tensor).
typedef struct { const rec_t * r; int8_t * w8; float * s8; } tc_cache_t;

struct so_batch {
    so_model * m;
    int ns, mode;
    int split[5];
    uint16_t * kc, * vc;
    tc_cache_t * cache;
    int ncache, capcache;
};

static void lin_batched(void * ctx, so_model * m, const rec_t * r, int kind, const float * x, float * y) {
    so_batch * b = (so_batch *) ctx;
    tc_cache_t * c = NULL;
    for (int i = 0; i < b->ncache; i++) if (b->cache[i].r == r) c = &b->cache[i];
    const int n = (int) r->cols, nsb = (n / G + 7) / 8;
    if (!c) {
        if (b->ncache == b->capcache) {
            b->capcache = b->capcache ? 2 * b->capcache : 64;
            b->cache = (tc_cache_t *) realloc(b->cache, (size_t) b->capcache * sizeof *b->cache);
        }
        c = &b->cache[b->ncache++];
        c->r = r;
        c->w8 = (int8_t *) malloc((size_t) r->rows * nsb * 256);
        c->s8 = (float *) malloc((size_t) r->rows * nsb * 4);
        char nm[65];
        memcpy(nm, r->name, 64);
        nm[64] = 0;
        so_requant8(m, nm, c->w8, c->s8);
    }
    sb_row(c->w8, c->s8, (const int32_t *) (m->base + r->perm_off), n, (int) r->rows, x, b->split[kind], y);
}

so_batch * so_batch_open(so_model * m, int ns, int mode) {
    so_batch * b = (so_batch *) calloc(1, sizeof *b);
    b->m = m;
    b->ns = ns;
    b->mode = mode;
    for (int k = 0; k < 5; k++) b->split[k] = 1;
    const size_t per = (size_t) m->n_layer * m->n_ctx * m->n_kv * m->hd;
    b->kc = (uint16_t *) calloc(per * ns, 2);
    b->vc = (uint16_t *) calloc(per * ns, 2);
    return b;
}

void so_batch_set_splits(so_batch * b, const int * split5) {
    for (int k = 0; k < 5; k++) b->split[k] = split5[k] > 0 ? split5[k] : 1;
}

int so_batch_step(so_batch * b, const int * tok, const int * pos, float * logits) {
    so_model * m = b->m;
    const size_t per = (size_t) m->n_layer * m->n_ctx * m->n_kv * m->hd;
    for (int s = 0; s < b->ns; s++)
        if (pos[s] >= m->n_ctx || (pos[s] >= 0 && (tok[s] < 0 || tok[s] >= (int) m->n_vocab))) return 0;
    for (int s = 0; s < b->ns; s++)
        if (pos[s] >= 0)
            forward_core(m, b->kc + per * s, b->vc + per * s, tok[s], pos[s], logits + (size_t) s * m->n_vocab,
                         b->mode ? lin_batched : lin_decode, b);
    return 1;
}

void so_batch_close(so_batch * b) {
    if (!b) return;
    for (int i = 0; i < b->ncache; i++) { free(b->cache[i].w8); free(b->cache[i].s8); }
    free(b->cache); free(b->kc); free(b->vc);
    free(b);
}

int so_batch_kv(const so_batch * b, int layer, int slot, int pos, uint16_t * k, uint16_t * v) {
    const so_model * m = b->m;
    if (layer < 0 || layer >= (int) m->n_layer || slot < 0 || slot >= b->ns || pos < 0 || pos >= m->n_ctx) return 0;
    const size_t kvd = (size_t) m->n_kv * m->hd, per = (size_t) m->n_layer * m->n_ctx * kvd;
    const size_t at = per * slot + ((size_t) layer * m->n_ctx + pos) * kvd;
    memcpy(k, b->kc + at, kvd * 2);
    memcpy(v, b->vc + at, kvd * 2);
    return 1;
}
