// Expert weights drawn on the device.
//
// The Qwen3-235B-A22B-shaped configuration holds ~136 GB of Q4 weights, 97 %
// of them in its MoE experts. Its synthetic file (writer mode direct = 2)
// leaves the experts' bytes out, and an engine opened after
// sb_draw_experts(seed) fills their tiles here instead: every code plane and
// group-field byte uniform, the per-superblock scales fixed so that a weight
// code * (d * sq) + md * (mq - bias) spans about +-2 sigma, like the file's
// own draws. The tiles have the layout and size a file's experts would give,
// so the decode kernels read the same bytes per token; the values only have
// to be finite. Nothing compares these weights with a reference: parity at
// this shape runs on shallow files written in full.
#include <cuda_fp16.h>

#include "sheep_b200.h"
#include "tiles.h"
#include "upload.h"

namespace sb {

__host__ __device__ __forceinline__ uint64_t draw_mix(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// One thread per 16-byte word of the tiles: the word's offset inside its tile
// says which section it lies in (tile sections are 16-byte padded).
__global__ void k_draw_tiles(uint4 * t, uint64_t nwords, uint32_t tb, uint32_t sd_lo, uint32_t sd_hi,
                             uint32_t md_lo, uint32_t md_hi, uint64_t seed, float sd, float md) {
    const __half hs = __float2half_rn(sd), hm = __float2half_rn(md);
    const uint32_t ps = (uint32_t) __half_as_ushort(hs) * 0x10001u, pm = (uint32_t) __half_as_ushort(hm) * 0x10001u;
    for (uint64_t w = blockIdx.x * (uint64_t) blockDim.x + threadIdx.x; w < nwords;
         w += (uint64_t) gridDim.x * blockDim.x) {
        const uint32_t off = (uint32_t) ((w * 16) % tb);
        uint4 v;
        if (off >= sd_lo && off < sd_hi) {
            v = make_uint4(ps, ps, ps, ps);
        } else if (off >= md_lo && off < md_hi) {
            v = make_uint4(pm, pm, pm, pm);
        } else {
            const uint64_t a = draw_mix(seed + 2 * w), b = draw_mix(seed + 2 * w + 1);
            v = make_uint4((uint32_t) a, (uint32_t) (a >> 32), (uint32_t) b, (uint32_t) (b >> 32));
        }
        t[w] = v;
    }
}

bool draw_tiles(uint8_t * dev, size_t total, const TileGeom & g, int nbits, int six, int minneg, int has_min,
                uint64_t seed, float sigma) {
    if (total % 16 || g.bytes % 16 || (uintptr_t) dev % 16) return false;
    const float nmax = (float) ((1 << nbits) - 1), fmax = six ? 63.0f : 255.0f;
    const float mdiv = six ? (minneg ? 63.0f : 31.0f) : 127.0f;
    // steps up to 4 sigma / nmax over the group's codes, minimums within +-2 sigma
    const float sd = 4.0f * sigma / (nmax * fmax), md = 2.0f * sigma / mdiv;
    const uint32_t sd_hi = g.sd_off + pad16((uint32_t) g.S * g.TR * 2);
    const uint32_t md_hi = has_min ? g.md_off + pad16((uint32_t) g.S * g.TR * 2) : g.md_off;
    const uint64_t nwords = total / 16;
    const int grid = (int) ((nwords + 255) / 256 < 148u * 16u ? (nwords + 255) / 256 : 148u * 16u);
    k_draw_tiles<<<grid > 0 ? grid : 1, 256>>>((uint4 *) dev, nwords, g.bytes, g.sd_off, sd_hi, g.md_off, md_hi,
                                               draw_mix(seed), sd, md);
    return cudaGetLastError() == cudaSuccess;
}

}  // namespace sb

static uint64_t g_draw_seed = 0;

extern "C" void sb_draw_experts(uint64_t seed) { g_draw_seed = seed; }

namespace sb {
uint64_t draw_experts_seed() { return g_draw_seed; }
}  // namespace sb
