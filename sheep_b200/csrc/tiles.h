// Tile-major weight layout for streaming GEMV.
//
// A tensor (or several tensors fused by rows) is cut into tiles of TR whole
// rows (TR = 1, 2, 4, 8 or 16, chosen per tensor so there are enough tiles to
// keep every SM busy and a tile stays near 8-16 KB). A tile holds every byte
// the GEMV needs for its rows, so ONE bulk copy brings it to shared memory.
// Sections, each padded to 16 bytes:
//
//   per code plane   nibble plane: piece 0 [U][TR] x 16 B, then piece 1 [U][TR] x 16 B
//                    2-bit plane:  [U][TR] x 16 B
//                    bit plane:    [U][TR] x 8 B
//   sq, mq           [U/2][TR] x (4 B at 8-bit fields, 3 B at 6-bit)
//   sd, md           [S][TR] x 2 B (fp16 per 256-weight superblock)
//
// A "unit" is 64 weights of a row: groups 4p..4p+3, columns c0..c0+15 with
// p = u/2, c0 = 16*(u%2). Nibble piece 0 is the file's bytes 64p+c0..+15 of
// the row (groups 4p and 4p+1), piece 1 the bytes 64p+32+c0..+15 (groups
// 4p+2 and 4p+3). In a warp, lane l takes row l % TR and units
// u = l / TR + k * (32 / TR); for a fixed k the lanes' pieces are consecutive
// 16-byte words, so shared-memory reads are free of bank conflicts.
//
// The bytes are the file's bytes, reordered, plus at most 15 bytes of padding
// per section.
#pragma once

#include <cstddef>
#include <cstdint>

namespace sb {

struct TileGeom {
    int TR, U, S, P;                 // rows, units per row, superblocks, unit pairs
    uint32_t pl_off[3], pl_sec[3];   // per plane: section offset, bytes of one piece array
    int pl_kind[3], pl_shift[3], np;
    uint32_t sq_off, mq_off, f_w;    // group fields: offset, bytes per (pair, row)
    uint32_t sd_off, md_off;         // superblock scales
    uint32_t bytes;                  // whole tile
};

// kinds: 4 nibble, 2 two-bit, 1 bit plane, in the width's plane order
// (tooling/sml_quantize.py:106)
__host__ __device__ inline int plane_kinds(int nbits, int * kinds, int * shifts) {
    int k[3] = {0, 0, 0}, s[3] = {0, 0, 0}, n = 0;
    switch (nbits) {
    case 2: k[0] = 2; n = 1; break;
    case 3: k[0] = 2; k[1] = 1; s[1] = 2; n = 2; break;
    case 4: k[0] = 4; n = 1; break;
    case 5: k[0] = 4; k[1] = 1; s[1] = 4; n = 2; break;
    case 6: k[0] = 2; s[0] = 4; k[1] = 4; n = 2; break;
    case 7: k[0] = 4; k[1] = 2; s[1] = 4; k[2] = 1; s[2] = 6; n = 3; break;
    case 8: k[0] = 4; k[1] = 4; s[1] = 4; n = 2; break;
    }
    for (int i = 0; i < 3; i++) { kinds[i] = k[i]; shifts[i] = s[i]; }
    return n;
}

__host__ __device__ inline uint32_t pad16(uint32_t v) { return (v + 15u) & ~15u; }

__host__ __device__ inline TileGeom tile_geom(int n, int TR, int nbits, int six, int has_min) {
    TileGeom g;
    g.TR = TR;
    g.U = n / 64;
    g.P = g.U / 2;
    g.S = (n + 255) / 256;
    g.np = plane_kinds(nbits, g.pl_kind, g.pl_shift);
    uint32_t off = 0;
    for (int p = 0; p < 3; p++) {
        g.pl_off[p] = off;
        g.pl_sec[p] = 0;
        if (p < g.np) {
            const int k = g.pl_kind[p];
            g.pl_sec[p] = (uint32_t) g.U * TR * (k == 1 ? 8 : 16);
            off += pad16(g.pl_sec[p] * (k == 4 ? 2 : 1));
        }
    }
    g.f_w = six ? 3u : 4u;
    g.sq_off = off;
    off += pad16((uint32_t) g.P * TR * g.f_w);
    g.mq_off = off;
    if (has_min) off += pad16((uint32_t) g.P * TR * g.f_w);
    g.sd_off = off;
    off += pad16((uint32_t) g.S * TR * 2);
    g.md_off = off;
    if (has_min) off += pad16((uint32_t) g.S * TR * 2);
    g.bytes = off;
    return g;
}

// Device view of a tiled (possibly fused) tensor.
struct TT {
    const uint8_t * tiles;
    int rows;          // logical rows (fused: all parts)
    int TR, ntiles;    // rows per tile, tiles (rows rounded up)
    int cols, nbits, six, has_min;
    uint32_t tb;       // bytes per tile
    float mbias;
    const int32_t * perm;   // input column order
    const int32_t * iperm;
};

// Rows per tile for a tensor of `rows` x `row_bytes`: as many as keep at least
// `min_tiles` tiles and a tile at most max_bytes (at least one row). `even`
// for fused gate/up tensors whose tiles pair rows.
__host__ __device__ inline int pick_tr(int rows, int row_bytes, int min_tiles, int even, int max_bytes = 12288) {
    int tr = 16;
    while (tr > (even ? 2 : 1) && (rows / tr < min_tiles || (long) tr * row_bytes > max_bytes)) tr /= 2;
    return tr;
}

}  // namespace sb
