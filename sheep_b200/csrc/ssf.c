// SSF loader: mmap, then refuse anything malformed before a single byte of a
// payload is trusted. The acceptance rules follow the reference loader
// (sml/sml-model.c:24-75 record ranges, :174-260 header checks) so that a file
// one engine opens, the other opens too; only v8+ files are accepted here,
// because the flat layouts are what the GPU kernels read.
#define _GNU_SOURCE
#include "ssf.h"

#include <fcntl.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

static int fail(char * why, int nwhy, const char * fmt, ...) {
    if (why && nwhy > 0) {
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(why, (size_t) nwhy, fmt, ap);
        va_end(ap);
    }
    return 0;
}

static int inside(size_t size, uint64_t off, uint64_t n) {
    return off >= SSF_HEADER_BYTES && off <= (uint64_t) size && n <= (uint64_t) size - off;
}

int ssf_planes(int nbits, int kinds[3], int shifts[3]) {
    switch (nbits) {
    case 2: kinds[0] = 2; shifts[0] = 0; return 1;
    case 3: kinds[0] = 2; shifts[0] = 0; kinds[1] = 1; shifts[1] = 2; return 2;
    case 4: kinds[0] = 4; shifts[0] = 0; return 1;
    case 5: kinds[0] = 4; shifts[0] = 0; kinds[1] = 1; shifts[1] = 4; return 2;
    case 6: kinds[0] = 2; shifts[0] = 4; kinds[1] = 4; shifts[1] = 0; return 2;
    case 7: kinds[0] = 4; shifts[0] = 0; kinds[1] = 2; shifts[1] = 4; kinds[2] = 1; shifts[2] = 6; return 3;
    case 8: kinds[0] = 4; shifts[0] = 0; kinds[1] = 4; shifts[1] = 4; return 2;
    default: return 0;
    }
}

static uint64_t plane_row_bytes(int kind, int n) {
    return kind == 4 ? (uint64_t) n / 2 : kind == 2 ? (uint64_t) n / 4 : (uint64_t) n / 8;
}

static int check_rec(const ssf_file * f, const ssf_rec * r, char * why, int nwhy, uint64_t i) {
    const char * nm = r->name;
    if (!r->rows || !r->cols || r->rows > 0x7fffffffu || r->cols > 0x7fffffffu)
        return fail(why, nwhy, "tensor %llu (%.64s): invalid dimensions", (unsigned long long) i, nm);
    if (r->kind == SSF_KIND_F32) {
        const uint64_t cnt = (uint64_t) r->rows * r->cols;
        if (r->nbytes != cnt * 4 || !inside(f->size, r->off, r->nbytes))
            return fail(why, nwhy, "tensor %llu (%.64s): invalid f32 payload", (unsigned long long) i, nm);
        return 1;
    }
    if (r->kind != SSF_KIND_QUANT)
        return fail(why, nwhy, "tensor %llu (%.64s): unknown kind %u", (unsigned long long) i, nm, r->kind);
    if (r->layout > SSF_LAYOUT_FLAT || (r->layout == SSF_LAYOUT_FLAT && (r->nbits < 2 || r->nbits > 8)))
        return fail(why, nwhy, "tensor %llu (%.64s): invalid code layout", (unsigned long long) i, nm);
    const uint64_t offs[5] = {r->sd_off, r->sq_off, r->perm_off, r->md_off, r->mq_off};
    const uint64_t lens[5] = {r->sd_n, r->sq_n, r->perm_n, r->md_n, r->mq_n};
    for (int j = 0; j < 5; j++)
        if (lens[j] && !inside(f->size, offs[j], lens[j]))
            return fail(why, nwhy, "tensor %llu (%.64s): metadata exceeds file bounds", (unsigned long long) i, nm);
    for (int j = 0; j < SSF_MAX_LEVELS; j++)
        if (r->codes_n[j] && !inside(f->size, r->codes_off[j], r->codes_n[j]))
            return fail(why, nwhy, "tensor %llu (%.64s): codes exceed file bounds", (unsigned long long) i, nm);
    return 1;
}

int ssf_open(ssf_file * f, const char * path, char * why, int nwhy) {
    memset(f, 0, sizeof *f);
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(why, nwhy, "cannot open %s", path);
    struct stat st;
    if (fstat(fd, &st) != 0) { close(fd); return fail(why, nwhy, "cannot stat %s", path); }
    if ((size_t) st.st_size < SSF_HEADER_BYTES) {
        close(fd);
        return fail(why, nwhy, "%s is truncated (smaller than the SSF header)", path);
    }
    void * base = mmap(NULL, (size_t) st.st_size, PROT_READ, MAP_SHARED, fd, 0);
    close(fd);
    if (base == MAP_FAILED) return fail(why, nwhy, "cannot map %s", path);
    f->base = (const uint8_t *) base;
    f->size = (size_t) st.st_size;
    f->hdr = (const ssf_hdr *) f->base;
    const ssf_hdr * h = f->hdr;
    int ok = 1;
    if (memcmp(h->magic, "SSF ", 4) != 0) ok = fail(why, nwhy, "%s is not an .ssf file", path);
    else if (h->version > SSF_MAX_VERSION)
        ok = fail(why, nwhy, "%s is format v%u, this engine reads up to v%d", path, h->version, SSF_MAX_VERSION);
    else if (h->version < 8)
        ok = fail(why, nwhy, "%s is format v%u: only flat-layout files (v8+) run on the GPU", path, h->version);
    else if (!h->n_levels || h->n_levels > SSF_MAX_LEVELS || !h->n_tensors)
        ok = fail(why, nwhy, "%s has invalid level or tensor counts", path);
    else if ((h->flags & ~(SSF_FLAG_HADAMARD | SSF_FLAG_SCALE6 | SSF_FLAG_MINNEG | SSF_FLAG_EXACT)) ||
             ((h->flags & SSF_FLAG_MINNEG) && !(h->flags & SSF_FLAG_SCALE6)))
        ok = fail(why, nwhy, "%s has unsupported model flags", path);
    else if (h->table_off < SSF_HEADER_BYTES || h->table_off > f->size ||
             h->n_tensors > ((uint64_t) f->size - h->table_off) / sizeof(ssf_rec))
        ok = fail(why, nwhy, "%s has a tensor table outside file bounds", path);
    else if ((h->json_n && !inside(f->size, h->json_off, h->json_n)) ||
             (h->tok_n && !inside(f->size, h->tok_off, h->tok_n)))
        ok = fail(why, nwhy, "%s has metadata ranges outside the file", path);
    else if (h->group != SSF_GROUP)
        ok = fail(why, nwhy, "%s: group size %u, the kernels are built for %d", path, h->group, SSF_GROUP);
    if (!ok) { ssf_close(f); return 0; }
    f->recs = (const ssf_rec *) (f->base + h->table_off);
    f->scale6 = (h->flags & SSF_FLAG_SCALE6) != 0;
    f->minneg = f->scale6 && (h->flags & SSF_FLAG_MINNEG) != 0;
    for (uint64_t i = 0; i < h->n_tensors; i++) {
        if (!check_rec(f, &f->recs[i], why, nwhy, i)) { ssf_close(f); return 0; }
        const ssf_rec * r = &f->recs[i];
        if (r->kind == SSF_KIND_QUANT && r->layout == SSF_LAYOUT_FLAT) {
            // The shapes the code planes imply must be what the record stores.
            int kinds[3], shifts[3];
            const int np = ssf_planes((int) r->nbits, kinds, shifts);
            const int n = (int) r->cols, ng = n / SSF_GROUP;
            int bad = (n % 128) != 0;
            for (int p = 0; p < np && !bad; p++)
                bad = r->codes_n[p] != (uint64_t) r->rows * plane_row_bytes(kinds[p], n);
            bad = bad || r->perm_n != (uint64_t) n * 4
                      || r->sd_n != (uint64_t) r->rows * ssf_nscale(n) * 2
                      || r->sq_n != (uint64_t) r->rows * ssf_field_row_bytes(ng, f->scale6)
                      || (r->mq_n && (r->mq_n != r->sq_n || r->md_n != r->sd_n));
            if (bad) {
                fail(why, nwhy, "tensor %.64s: plane or field sizes do not match %ux%u Q%u",
                     r->name, r->rows, r->cols, r->nbits);
                ssf_close(f);
                return 0;
            }
        }
    }
    return 1;
}

void ssf_close(ssf_file * f) {
    if (f->base) munmap((void *) f->base, f->size);
    memset(f, 0, sizeof *f);
}

const ssf_rec * ssf_find(const ssf_file * f, const char * name) {
    for (uint64_t i = 0; i < f->hdr->n_tensors; i++)
        if (strncmp(f->recs[i].name, name, SSF_NAME_LEN) == 0) return &f->recs[i];
    return NULL;
}

const ssf_rec * ssf_findf(const ssf_file * f, const char * fmt, int a, int b) {
    char buf[SSF_NAME_LEN + 1];
    snprintf(buf, sizeof buf, fmt, a, b);
    return ssf_find(f, buf);
}
