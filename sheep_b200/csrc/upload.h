// Device arena and the upload of SSF flat tensors into it.
//
// Sizing runs the same code twice: once with no arena (only counting), then
// into one cudaMalloc of the counted size. Every array is 256-byte aligned and
// followed by 256 bytes of slack, so the 16-byte widening of L2 prefetch
// ranges and TMA-aligned copies never leave the allocation.
#pragma once

#include "qgemv.cuh"
#include "ssf.h"
#include "tiles.h"

#include <cmath>
#include <cstdio>
#include <cstring>
#include <unordered_map>
#include <utility>
#include <vector>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace sb {

// Tiles filled on the device instead of from the file (draw.cu): uniform code
// and field bytes, fixed superblock scales; false on a misaligned buffer or a
// failed launch.
bool draw_tiles(uint8_t * dev, size_t total, const TileGeom & g, int nbits, int six, int minneg, int has_min,
                uint64_t seed, float sigma);
// The seed set by sb_draw_experts (0: experts come from the file).
uint64_t draw_experts_seed();

struct Arena {
    uint8_t * base = nullptr;
    size_t used = 0, size = 0;
    std::unordered_map<uint64_t, std::pair<const int32_t *, const int32_t *>> perms;
    // while set, upload_tt draws tiles on the device (seeded by draw_seed and
    // the tiles' arena offset) instead of copying them from the file
    bool drawing = false;
    uint64_t draw_seed = 0;
    int minneg = 0;
    bool draw_failed = false;

    void * carve(size_t n) {
        const size_t at = (used + 255) / 256 * 256;
        used = at + (n + 15) / 16 * 16 + 256;
        return base ? base + at : nullptr;
    }
    void * upload(const void * src, size_t n) {
        void * d = carve(n);
        if (d && src && n) cudaMemcpy(d, src, n, cudaMemcpyHostToDevice);
        return d;
    }
    // Switch from counting to filling; returns false if cudaMalloc fails.
    bool allocate() {
        size = used;
        used = 0;
        perms.clear();
        if (cudaMalloc(&base, size) != cudaSuccess) { base = nullptr; return false; }
        cudaMemset(base, 0, size);
        return true;
    }
    void release() {
        if (base) cudaFree(base);
        base = nullptr;
        used = size = 0;
        perms.clear();
    }
};

inline const float * upload_f32(Arena & a, const ssf_file & f, const ssf_rec * r) {
    if (!r) return nullptr;
    return (const float *) a.upload(f.base + r->off, r->nbytes);
}

// The device view of one flat tensor; its permutation is shared with every
// tensor that names the same file offset (the reference shares an input's
// activation the same way, sml/sml-run.c:945-952).
inline bool upload_perm(Arena & a, const ssf_file & f, const ssf_rec * r, QT & t, char * why, int nwhy);

// Shape, field layout and column order of r, without its planes.
inline bool upload_qt_meta(Arena & a, const ssf_file & f, const ssf_rec * r, QT & t, char * why, int nwhy) {
    if (!r) { snprintf(why, nwhy, "missing tensor"); return false; }
    if (r->kind != SSF_KIND_QUANT || r->layout != SSF_LAYOUT_FLAT) {
        snprintf(why, nwhy, "%.64s: only flat quantized tensors run on the GPU", r->name);
        return false;
    }
    memset(&t, 0, sizeof t);
    t.rows = (int) r->rows;
    t.cols = (int) r->cols;
    t.nbits = (int) r->nbits;
    t.six = f.scale6;
    t.has_min = r->mq_n != 0;
    t.nsb = ssf_nscale(t.cols);
    t.frow = (int) ssf_field_row_bytes(t.cols / SSF_GROUP, f.scale6);
    t.mbias = f.scale6 ? (f.minneg ? 63.0f : 31.0f) : 127.0f;
    return upload_perm(a, f, r, t, why, nwhy);
}

inline bool upload_qt(Arena & a, const ssf_file & f, const ssf_rec * r, QT & t, char * why, int nwhy) {
    if (!r) { snprintf(why, nwhy, "missing tensor"); return false; }
    if (r->kind != SSF_KIND_QUANT || r->layout != SSF_LAYOUT_FLAT) {
        snprintf(why, nwhy, "%.64s: only flat quantized tensors run on the GPU", r->name);
        return false;
    }
    memset(&t, 0, sizeof t);
    t.rows = (int) r->rows;
    t.cols = (int) r->cols;
    t.nbits = (int) r->nbits;
    t.six = f.scale6;
    t.has_min = r->mq_n != 0;
    t.nsb = ssf_nscale(t.cols);
    t.frow = (int) ssf_field_row_bytes(t.cols / SSF_GROUP, f.scale6);
    t.mbias = f.scale6 ? (f.minneg ? 63.0f : 31.0f) : 127.0f;
    int kinds[3], shifts[3];
    const int np = ssf_planes(t.nbits, kinds, shifts);
    for (int p = 0; p < np; p++) t.pl[p] = (const uint8_t *) a.upload(f.base + r->codes_off[p], r->codes_n[p]);
    t.sd = (const uint16_t *) a.upload(f.base + r->sd_off, r->sd_n);
    t.sq = (const uint8_t *) a.upload(f.base + r->sq_off, r->sq_n);
    if (t.has_min) {
        t.md = (const uint16_t *) a.upload(f.base + r->md_off, r->md_n);
        t.mq = (const uint8_t *) a.upload(f.base + r->mq_off, r->mq_n);
    }
    return upload_perm(a, f, r, t, why, nwhy);
}

inline bool upload_perm(Arena & a, const ssf_file & f, const ssf_rec * r, QT & t, char * why, int nwhy) {
    auto it = a.perms.find(r->perm_off);
    if (it != a.perms.end()) {
        t.perm = it->second.first;
        t.iperm = it->second.second;
        return true;
    }
    const int32_t * p = (const int32_t *) (f.base + r->perm_off);
    std::vector<int32_t> inv(t.cols, -1);
    for (int i = 0; i < t.cols; i++) {
        if (p[i] < 0 || p[i] >= t.cols || inv[p[i]] >= 0) {
            snprintf(why, nwhy, "%.64s: column permutation is not a permutation", r->name);
            return false;
        }
        inv[p[i]] = i;
    }
    t.perm = (const int32_t *) a.upload(p, (size_t) t.cols * 4);
    t.iperm = (const int32_t *) a.upload(inv.data(), (size_t) t.cols * 4);
    a.perms[r->perm_off] = {t.perm, t.iperm};
    return true;
}

// ------------------------------------------------------------------ tiles

struct RowSrc {
    const ssf_rec * r;   // NULL: a padding row (zeros)
    int row;
};

inline size_t file_plane_row(int kind, int n) { return kind == 4 ? n / 2 : kind == 2 ? n / 4 : n / 8; }

// Copy row `row` of record r into row j of a tile (layout in tiles.h).
inline void fill_tile_row(uint8_t * tile, const TileGeom & tg, int j, const ssf_file & f, const ssf_rec * r,
                          int row, int six, int has_min) {
    const int n = (int) r->cols, ng = n / SSF_GROUP, TR = tg.TR;
    for (int p = 0; p < tg.np; p++) {
        const int kind = tg.pl_kind[p];
        const uint8_t * src = f.base + r->codes_off[p] + (size_t) row * file_plane_row(kind, n);
        uint8_t * dst = tile + tg.pl_off[p];
        for (int u = 0; u < tg.U; u++) {
            const int pq = u >> 1, c0 = (u & 1) * 16;
            const size_t at = (size_t) u * TR + j;
            if (kind == 4) {
                memcpy(dst + at * 16, src + 64 * pq + c0, 16);
                memcpy(dst + tg.pl_sec[p] + at * 16, src + 64 * pq + 32 + c0, 16);
            } else if (kind == 2) {
                memcpy(dst + at * 16, src + 32 * pq + c0, 16);
            } else {
                for (int k = 0; k < 4; k++) memcpy(dst + at * 8 + 2 * k, src + (4 * pq + k) * 4 + c0 / 8, 2);
            }
        }
    }
    const size_t frow = ssf_field_row_bytes(ng, six);
    const size_t nsb = (size_t) ssf_nscale(n);
    const uint8_t * sq = f.base + r->sq_off + (size_t) row * frow;
    const uint8_t * mq = f.base + r->mq_off + (size_t) row * frow;
    const uint8_t * sd = f.base + r->sd_off + (size_t) row * nsb * 2;
    const uint8_t * md = f.base + r->md_off + (size_t) row * nsb * 2;
    for (int pq = 0; pq < tg.P; pq++) {
        const size_t at = ((size_t) pq * TR + j) * tg.f_w;
        memcpy(tile + tg.sq_off + at, sq + (size_t) pq * tg.f_w, tg.f_w);
        if (has_min) memcpy(tile + tg.mq_off + at, mq + (size_t) pq * tg.f_w, tg.f_w);
    }
    for (int s = 0; s < tg.S; s++) {
        const size_t at = ((size_t) s * TR + j) * 2;
        memcpy(tile + tg.sd_off + at, sd + 2 * s, 2);
        if (has_min) memcpy(tile + tg.md_off + at, md + 2 * s, 2);
    }
}

// A tiled tensor of `rows` logical rows, each taken from src(v). Every part
// must share width, field layout, column count and column order (`first`).
// TR = 0 picks the rows per tile (pick_tr) for `min_tiles` tiles.
template <class F>
inline bool upload_tt(Arena & a, const ssf_file & f, const ssf_rec * first, int rows, int TR, int min_tiles,
                      int even, F src, TT & t, char * why, int nwhy) {
    QT q;
    if (!upload_qt_meta(a, f, first, q, why, nwhy)) return false;
    memset(&t, 0, sizeof t);
    t.rows = rows;
    t.cols = q.cols;
    t.nbits = q.nbits;
    t.six = q.six;
    t.has_min = q.has_min;
    t.mbias = q.mbias;
    t.perm = q.perm;
    t.iperm = q.iperm;
    const TileGeom g1 = tile_geom(t.cols, 1, t.nbits, t.six, t.has_min);
    t.TR = TR > 0 ? TR : pick_tr(rows, (int) g1.bytes, min_tiles, even);
    t.ntiles = (rows + t.TR - 1) / t.TR;
    const TileGeom tg = tile_geom(t.cols, t.TR, t.nbits, t.six, t.has_min);
    t.tb = tg.bytes;
    const size_t total = (size_t) t.ntiles * t.tb;
    uint8_t * dev = (uint8_t *) a.carve(total);
    t.tiles = dev;
    if (!dev) return true;   // sizing pass
    if (a.drawing) {
        if (!draw_tiles(dev, total, tg, t.nbits, t.six, a.minneg, t.has_min,
                        a.draw_seed ^ (uint64_t) (dev - a.base), 0.02f)) {
            snprintf(why, nwhy, "%.64s: drawing tiles on the device failed", first->name);
            a.draw_failed = true;
            return false;
        }
        return true;
    }
    std::vector<uint8_t> host(total, 0);
    bool bad = false;
#pragma omp parallel for schedule(dynamic, 16)
    for (int ti = 0; ti < t.ntiles; ti++) {
        for (int j = 0; j < t.TR; j++) {
            const RowSrc rs = src(ti * t.TR + j);
            if (!rs.r) continue;
            if ((int) rs.r->cols != t.cols || (int) rs.r->nbits != t.nbits || (rs.r->mq_n != 0) != (t.has_min != 0) ||
                rs.r->perm_off != first->perm_off) { bad = true; continue; }
            fill_tile_row(host.data() + (size_t) ti * t.tb, tg, j, f, rs.r, rs.row, t.six, t.has_min);
        }
    }
    if (bad) {
        snprintf(why, nwhy, "%.64s: fused tensors differ in width, fields or column order", first->name);
        return false;
    }
    cudaMemcpy(dev, host.data(), total, cudaMemcpyHostToDevice);
    return true;
}

// Features of a file the decode kernels do not implement (the reference's GPU
// open refuses by name the same way, sml/sml-gpu-fwd.c:1833-1840), or NULL.
inline const char * ssf_unsupported(const ssf_file & f) {
    const ssf_hdr * h = f.hdr;
    if (h->flags & SSF_FLAG_HADAMARD) return "Hadamard-rotated weights";
    if (h->flags & SSF_FLAG_EXACT) return "an exact-weight (f32) file";
    if (h->norm_type != 0) return "LayerNorm";
    if (h->rope_type != 0) return "interleaved RoPE";
    if (h->arch_bits) return "architecture flags beyond a plain decoder";
    if (h->logit_softcap != 0.0f || h->attn_softcap != 0.0f) return "soft-capping";
    if (h->n_swa) return "sliding-window attention";
    if (h->emb_scale != 0.0f || h->res_scale != 0.0f || h->logit_scale != 0.0f) return "embedding/residual/logit scales";
    if (h->clip_qkv != 0.0f) return "Q/K/V clamping";
    const char * names[] = {"position_embd.weight", "token_embd_norm.weight", "output.bias", "rope_freqs",
                            "attn_window", "attn_rope"};
    for (const char * n : names) if (ssf_find(&f, n)) return n;
    return nullptr;
}

// RoPE tables [n_ctx][hd/2] exactly as the CPU builds them (sml/sml-run.c:1383-1393).
inline void upload_rope(float * dcos, float * dsin, int n_ctx, int hd, float theta) {
    const int half = hd / 2;
    std::vector<float> c((size_t) n_ctx * half), s((size_t) n_ctx * half);
    for (int p = 0; p < n_ctx; p++)
        for (int i = 0; i < half; i++) {
            const float fr = powf(theta, -(float) i / (float) half);
            const float a = (float) p * fr;
            c[(size_t) p * half + i] = cosf(a);
            s[(size_t) p * half + i] = sinf(a);
        }
    cudaMemcpy(dcos, c.data(), c.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(dsin, s.data(), s.size() * 4, cudaMemcpyHostToDevice);
}

// Bytes of one record as the file stores it: codes and fields.
inline uint64_t ssf_rec_bytes(const ssf_rec * r) {
    uint64_t b = r->sd_n + r->sq_n + r->md_n + r->mq_n;
    for (int p = 0; p < SSF_MAX_LEVELS; p++) b += r->codes_n[p];
    return b;
}

}  // namespace sb
