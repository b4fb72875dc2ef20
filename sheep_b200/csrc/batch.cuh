// Kernels of the batched decode step (sb_batch): B sequences advance one
// token each per step, each at its own position with its own fp16 KV cache.
// The products run on the tensor-core path (tc_batch.cu); this file holds the
// per-sequence work around them:
//
//   k_bembed    the B embedding rows, dequantized and scattered to natural order
//   k_battn     RoPE, the KV write and split-position attention, one CTA per
//               (run of positions, KV head, sequence) streaming 64-position
//               chunks through a bulk-copy ring with an online softmax, and
//               serving up to 8 query heads of the KV head, so each cached
//               byte is read once per step (GQA groups of <= 8)
//   k_bargmax   the greedy choice per sequence, fed back as its next token
//
// The CPU body these follow is sml_forward_multi / forward_slots
// (sml/sml-run.c:2559-2604, 2218), one sequence's arithmetic being
// sml_forward's (sml/sml-run.c:3243-3523).
#pragma once

#include "decode.cuh"

namespace sb {

constexpr int kBChunk = 64;      // positions per attention ring stage
constexpr int kBThreads = 256;
constexpr int kBMaxRep = 32;     // query heads per KV head
constexpr int kMaxBatchSeqs = 256;

// x[b][perm[i]] = dequant(emb[tok[b]], i); an idle slot (pos < 0) gets zeros.
template <int NB, int SIX>
__global__ void k_bembed(const __grid_constant__ QT t, const int * tok, const int * pos, float * x, int ldx,
                         int * err) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
    if (i >= t.cols) return;
    const int tk = tok[b];
    float v = 0.0f;
    if (pos[b] >= 0) {
        if (tk >= 0 && tk < t.rows) v = dequant_at<NB, SIX>(t, tk, i);
        else if (i == 0) atomicExch(err, 302);
    }
    x[(size_t) b * ldx + t.perm[i]] = v;
}

struct BAttnArgs {
    const float * qkv;       // [B][ldq]: query heads at 0, keys at koff, values at voff (before RoPE)
    int ldq, koff, voff;
    int n_head, n_kv;
    const float * qn, * kn;  // Q/K norm gains (hd long) or NULL
    float eps;
    const float * rcos, * rsin;   // [n_ctx][hd / 2]
    uint16_t * kc, * vc;     // this layer's cache pages: [n_pages][n_kv][kBChunk][hd] fp16
    int n_ctx;
    const int * pages;       // [B][maxp]: the page of each slot's positions 64c .. 64c + 63
    int maxp, n_pages;
    const int * pos;         // [B]; < 0: an idle slot
    int nsplit;              // CTAs sharing one (sequence, head group)'s positions
    int hgroups;             // head groups per KV head (ceil(rep / HG))
    float scale;             // 1/sqrt(hd)
    float * part;            // [B][n_kv * hgroups][nsplit][HG][hd + 2]: max, sum, weighted values
    unsigned * cnt;          // [B][n_kv * hgroups] arrivals, zero between steps
    float * out;             // [B][ldo] attention output (head-major)
    int ldo;
    int * err;
};

// Row of position t (of slot b, KV head kvh) in the paged cache, in units of
// hd halves: a page holds 64 consecutive positions of every KV head, so a
// chunk of 64 positions is one contiguous run of one head's rows. A slot whose
// table holds no page there (the host never launches one) records an error
// and reads page 0 instead, so every access stays inside the cache and the
// CTAs of the step still meet.
SB_DEV size_t kv_row(const BAttnArgs & g, int b, int kvh, int t) {
    int page = g.pages[(size_t) b * g.maxp + t / 64];
    if (page < 0 || page >= g.n_pages) {
        atomicExch(g.err, 215);
        page = 0;
    }
    return ((size_t) page * g.n_kv + kvh) * 64 + (t % 64);
}

// Ring stages of 64 positions' keys and values, and query heads per CTA.
__host__ __device__ constexpr int battn_stages(int hd) { return hd <= 128 ? 3 : 2; }
__host__ __device__ inline int battn_hg(int rep) { return rep <= 4 ? 4 : 8; }

// Shared memory of k_battn: the ring (reused at the end for the warps' sums),
// the group's rotated queries, the new key and value, the RoPE row, the scores.
__host__ __device__ inline size_t battn_smem(int hd, int hg) {
    const size_t ring = (size_t) battn_stages(hd) * 2 * kBChunk * hd * 2;
    const size_t ro = (size_t) (kBThreads / 32) * hg * hd * 4;
    return (ring > ro ? ring : ro) + (size_t) (hg * hd + 3 * hd) * 4 + (size_t) kBChunk * hg * 4 + 16;
}

// One CTA per (split of the positions, KV head x head group, sequence); the
// HG query heads of the group share every key and value the CTA reads.
//  1. thread 0 starts bulk copies of the split's first chunks of 64 positions
//     (keys and values contiguous in the cache layout) into a ring, while every
//     thread loads the group's queries and the new key/value and applies the
//     Q/K norms and RoPE (sml/sml-run.c:295-375);
//  2. per chunk, once it has landed: the chunk owning `pos` takes the new key
//     and value (fp16, round to nearest even; the head group 0 CTA also writes
//     them to the cache); scores by teams of 8 lanes (16 for hd 256) per
//     position, each lane 16-byte column pieces of the key row against 4 heads'
//     queries in registers, summed across the team; the online softmax per
//     head (running max and sum, expf; sml/sml-run.c:180-266 takes it over all
//     positions at once); weighted values, each warp a stride of positions and
//     each lane hd/32 columns, its running sums rescaled by the max's change;
//     then the stage is refilled with the chunk `stages` ahead;
//  3. the warps' sums added in warp order; one split alone writes the output,
//     several meet in `part` and the last to arrive combines them in split
//     order (flash-decoding partials).
template <int HD, int HG>
__global__ void __launch_bounds__(kBThreads, 2) k_battn(const __grid_constant__ BAttnArgs g) {
    constexpr int S = battn_stages(HD);
    constexpr int LPP = HD <= 128 ? 8 : 16;   // lanes per position in the scores
    constexpr int NCH = HD / 8;                // 16-byte pieces per key row
    constexpr int CPL = NCH / LPP;             // pieces per lane (1 or 2)
    constexpr int PPW = 32 / LPP;              // positions per warp step
    constexpr int DV = HD / 32;                // columns per lane in the weighted sum
    constexpr int NW = kBThreads / 32;
    constexpr size_t RING = (size_t) S * 2 * kBChunk * HD * 2;
    constexpr size_t RO = (size_t) NW * HG * HD * 4;
    extern __shared__ __align__(16) uint8_t bsm[];
    __shared__ __align__(8) uint64_t full[S];
    __shared__ double red[NW];
    __shared__ float hm[HG], hl[HG], ha[HG];
    __shared__ unsigned last_flag;
    const int split = blockIdx.x, gy = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rep = g.n_head / g.n_kv;
    const int kvh = gy / g.hgroups, h0 = (gy % g.hgroups) * HG, nh = min(HG, rep - h0);
    const int pos = g.pos[b];
    float * outb = g.out + (size_t) b * g.ldo + ((size_t) kvh * rep + h0) * HD;
    if (pos < 0) {
        if (split == 0)
            for (int i = tid; i < nh * HD; i += kBThreads) outb[i] = 0.0f;
        return;
    }
    if (pos >= g.n_ctx || rep > kBMaxRep) {
        if (tid == 0) atomicExch(g.err, 211);
        return;
    }
    const int nchunk = pos / kBChunk + 1;
    const int per = (nchunk + g.nsplit - 1) / g.nsplit;
    const int nact = (nchunk + per - 1) / per;   // splits with positions
    const int c0 = split * per, c1 = min(nchunk, c0 + per);
    if (c0 >= nchunk) return;
    const int nmine = c1 - c0;
    uint16_t * ring = reinterpret_cast<uint16_t *>(bsm);
    float * qs = reinterpret_cast<float *>(bsm + (RING > RO ? RING : RO));   // [HG][HD]
    float * kn = qs + HG * HD, * vn = kn + HD, * cs = vn + HD, * sn = cs + HD / 2;
    float * sc = sn + HD / 2;                                                // [kBChunk][HG]
    float * ro = reinterpret_cast<float *>(bsm);                             // [NW][HG][HD] at the end

    if (tid == 0) {
        for (int s = 0; s < S; s++) mbar_init(&full[s], 1);
        mbar_fence_init();
    }
    __syncthreads();
    auto issue = [&](int j) {   // chunk c0 + j into stage j % S
        const int t0 = (c0 + j) * kBChunk, nt = min(pos + 1, t0 + kBChunk) - t0;
        uint16_t * Ks = ring + (size_t) (j % S) * 2 * kBChunk * HD;
        const uint32_t bytes = (uint32_t) nt * HD * 2;
        mbar_expect_tx(&full[j % S], 2 * bytes);
        const size_t r0 = kv_row(g, b, kvh, t0);
        bulk_g2s(Ks, g.kc + r0 * HD, bytes, &full[j % S]);
        bulk_g2s(Ks + kBChunk * HD, g.vc + r0 * HD, bytes, &full[j % S]);
    };
    if (tid == 0)
        for (int j = 0; j < S && j < nmine; j++) issue(j);
    const float * qrow = g.qkv + (size_t) b * g.ldq;
    for (int i = tid; i < HD / 2; i += kBThreads) {
        cs[i] = g.rcos[(size_t) pos * (HD / 2) + i];
        sn[i] = g.rsin[(size_t) pos * (HD / 2) + i];
    }
    for (int i = tid; i < HG * HD; i += kBThreads)
        qs[i] = i < nh * HD ? qrow[((size_t) kvh * rep + h0) * HD + i] : 0.0f;
    for (int i = tid; i < HD; i += kBThreads) {
        kn[i] = qrow[g.koff + kvh * HD + i];
        vn[i] = qrow[g.voff + kvh * HD + i];
    }
    if (tid < HG) { hm[tid] = -INFINITY; hl[tid] = 0.0f; }
    __syncthreads();
    for (int h = 0; h < nh; h++) norm_rope(qs + h * HD, g.qn, g.eps, HD, cs, sn, red);
    norm_rope(kn, g.kn, g.eps, HD, cs, sn, red);

    float o[HG][DV];
#pragma unroll
    for (int h = 0; h < HG; h++)
#pragma unroll
        for (int d = 0; d < DV; d++) o[h][d] = 0.0f;
    const int team = lane / LPP, tl = lane % LPP;
    bool ok = true;
    for (int j = 0; j < nmine; j++) {
        const int c = c0 + j, t0 = c * kBChunk, nt = min(pos + 1, t0 + kBChunk) - t0;
        uint16_t * Ks = ring + (size_t) (j % S) * 2 * kBChunk * HD, * Vs = Ks + kBChunk * HD;
        ok = mbar_wait(&full[j % S], (uint32_t) (j / S) & 1u, g.err, 212) && ok;
        if (c == nchunk - 1 && ok) {
            const int r = pos - t0;
            const size_t rp = h0 == 0 ? kv_row(g, b, kvh, pos) : 0;
            for (int i = tid; i < HD; i += kBThreads) {
                const uint16_t kh = f2h(kn[i]), vh = f2h(vn[i]);
                Ks[r * HD + i] = kh;
                Vs[r * HD + i] = vh;
                if (h0 == 0) {
                    g.kc[rp * HD + i] = kh;
                    g.vc[rp * HD + i] = vh;
                }
            }
        }
        ok = __syncthreads_and(ok) != 0;   // one verdict for the whole CTA
        if (!ok) break;
        // ---- scores (sml/sml-run.c:180-235: dot * 1/sqrt(hd))
#pragma unroll
        for (int hg = 0; hg < HG; hg += 4) {
            float qr[4][CPL * 8];
#pragma unroll
            for (int h = 0; h < 4; h++)
#pragma unroll
                for (int k = 0; k < CPL; k++)
#pragma unroll
                    for (int jj = 0; jj < 8; jj++) qr[h][k * 8 + jj] = qs[(hg + h) * HD + (tl + k * LPP) * 8 + jj];
            for (int p0 = 0; p0 < nt; p0 += NW * PPW) {
                const int p = p0 + warp * PPW + team;
                float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                if (p < nt) {
#pragma unroll
                    for (int k = 0; k < CPL; k++) {
                        const uint4 w = *reinterpret_cast<const uint4 *>(Ks + p * HD + (tl + k * LPP) * 8);
                        const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                        for (int jj = 0; jj < 4; jj++) {
                            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wv[jj]));
#pragma unroll
                            for (int h = 0; h < 4; h++) {
                                s4[h] = fmaf(qr[h][k * 8 + 2 * jj], f.x, s4[h]);
                                s4[h] = fmaf(qr[h][k * 8 + 2 * jj + 1], f.y, s4[h]);
                            }
                        }
                    }
                }
#pragma unroll
                for (int off = LPP / 2; off; off >>= 1)
#pragma unroll
                    for (int h = 0; h < 4; h++) s4[h] += __shfl_xor_sync(0xffffffffu, s4[h], off);
                if (p < nt && tl == 0)
                    *reinterpret_cast<float4 *>(sc + p * HG + hg) =
                        make_float4(s4[0] * g.scale, s4[1] * g.scale, s4[2] * g.scale, s4[3] * g.scale);
            }
        }
        __syncthreads();
        // ---- online softmax, one warp per head
        if (warp < nh) {
            float mc = -INFINITY;
            for (int p = lane; p < nt; p += 32) mc = fmaxf(mc, sc[p * HG + warp]);
            mc = warp_max(mc);
            const float mo = hm[warp], mn = fmaxf(mo, mc);
            float l = 0.0f;
            for (int p = lane; p < nt; p += 32) {
                const float e = expf(sc[p * HG + warp] - mn);
                sc[p * HG + warp] = e;
                l += e;
            }
            l = warp_sum(l);
            if (lane == 0) {
                const float a = expf(mo - mn);
                ha[warp] = a;
                hl[warp] = hl[warp] * a + l;
                hm[warp] = mn;
            }
        }
        __syncthreads();
        // ---- weighted values
#pragma unroll
        for (int h = 0; h < HG; h++) {
            const float a = h < nh ? ha[h] : 0.0f;
#pragma unroll
            for (int d = 0; d < DV; d++) o[h][d] *= a;
        }
        for (int p = warp; p < nt; p += NW) {
            float v[DV];
            if constexpr (DV == 2) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(Vs + p * HD + lane * 2));
                v[0] = f.x; v[1] = f.y;
            } else {
#pragma unroll
                for (int d = 0; d < DV; d += 4) {
                    const uint2 w = *reinterpret_cast<const uint2 *>(Vs + p * HD + lane * DV + d);
                    const float2 f0 = __half22float2(*reinterpret_cast<const __half2 *>(&w.x));
                    const float2 f1 = __half22float2(*reinterpret_cast<const __half2 *>(&w.y));
                    v[d] = f0.x; v[d + 1] = f0.y; v[d + 2] = f1.x; v[d + 3] = f1.y;
                }
            }
#pragma unroll
            for (int hg = 0; hg < HG; hg += 4) {
                const float4 pr = *reinterpret_cast<const float4 *>(sc + p * HG + hg);
#pragma unroll
                for (int d = 0; d < DV; d++) {
                    o[hg][d] = fmaf(pr.x, v[d], o[hg][d]);
                    o[hg + 1][d] = fmaf(pr.y, v[d], o[hg + 1][d]);
                    o[hg + 2][d] = fmaf(pr.z, v[d], o[hg + 2][d]);
                    o[hg + 3][d] = fmaf(pr.w, v[d], o[hg + 3][d]);
                }
            }
        }
        __syncthreads();   // the stage and the scores are free
        if (tid == 0 && j + S < nmine) issue(j + S);
    }
    if (!ok) return;
    // ---- the warps' sums, in warp order (the ring is free: every copy landed)
#pragma unroll
    for (int h = 0; h < HG; h++)
#pragma unroll
        for (int d = 0; d < DV; d++) ro[(warp * HG + h) * HD + lane * DV + d] = o[h][d];
    __syncthreads();
    const size_t grp = (size_t) b * g.n_kv * g.hgroups + gy;
    float * pb = g.part + (grp * g.nsplit + split) * HG * (HD + 2);
    for (int i = tid; i < nh * HD; i += kBThreads) {
        const int h = i / HD, d = i % HD;
        float s = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) s += ro[(w * HG + h) * HD + d];
        if (nact == 1) outb[h * HD + d] = s / hl[h];
        else pb[h * (HD + 2) + 2 + d] = s;
    }
    if (nact == 1) return;
    if (tid < nh) {
        pb[tid * (HD + 2)] = hm[tid];
        pb[tid * (HD + 2) + 1] = hl[tid];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) last_flag = atomicAdd(&g.cnt[grp], 1u) == (unsigned) nact - 1;
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    // the last split combines every split of the group, in split order
    const float * P = g.part + grp * g.nsplit * HG * (HD + 2);
    const size_t sst = (size_t) HG * (HD + 2);
    for (int i = tid; i < nh * HD; i += kBThreads) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int k = 0; k < nact; k++) M = fmaxf(M, __ldcg(P + k * sst + h * (HD + 2)));
        float L = 0.0f, ov = 0.0f;
        for (int k = 0; k < nact; k++) {
            const float e = expf(__ldcg(P + k * sst + h * (HD + 2)) - M);
            L += __ldcg(P + k * sst + h * (HD + 2) + 1) * e;
            ov += __ldcg(P + k * sst + h * (HD + 2) + 2 + d) * e;
        }
        outb[h * HD + d] = ov / L;
    }
    if (tid == 0) g.cnt[grp] = 0;
}

// ---------------------------------------------------------------- attention on the tensor cores

// Warp-level f16 MMA (m16n8k16, fp32 accumulate), ldmatrix and 16-byte async
// copies (k_battn_t).
SB_DEV void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
                 "{%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
SB_DEV void ldsm4(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2, uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
SB_DEV void ldsm4t(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2, uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr) : "memory");
}
// 16 bytes global -> shared, bypassing L1; src_bytes 0 fills zeros.
SB_DEV void cp_async16(uint32_t dst, const void * src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" :: "r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
SB_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
SB_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" :: "n"(N) : "memory"); }
SB_DEV uint32_t pack_h2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}
// x = hi + lo in fp16 (hi = fp16(x), lo = fp16(x - hi)): two MMAs with the
// exact fp16 keys/values give the fp32 product to ~2^-22 of x.
SB_DEV void split_h2(float a, float b, uint32_t & hi, uint32_t & lo) {
    const __half2 h = __floats2half2_rn(a, b);
    const float2 f = __half22float2(h);
    hi = *reinterpret_cast<const uint32_t *>(&h);
    lo = pack_h2(a - f.x, b - f.y);
}

constexpr int kMChunk = 64;      // positions per ring stage
static_assert(kBChunk == 64 && kMChunk == 64, "a cache page holds one attention chunk of each KV head");
constexpr int kMStages = 3;
constexpr int kMThreads = 128;   // 4 warps, 16 positions of each chunk apiece


// Decode attention of a batch on the tensor cores (hd 64, 128). One CTA per
// (split of the positions, KV head x group of up to 16 query heads, sequence),
// 4 warps. Chunks of 64 positions stream into a 3-stage ring by 16-byte async
// copies into rows padded by 16 bytes (ldmatrix without bank conflicts; rows
// past the position are zero-filled). Decode has few query heads per KV head
// (configuration 3 has 4, configuration 0 6, configuration 4 16), so the
// products are turned over: M = the 16 positions of a warp, N = the CTA's
// heads in n-tiles of 8 (NH8 tiles) -- a KV head's 4 query heads fill half an
// n-tile, where as the 16-row M of a heads-by-positions product they filled a
// quarter, and the two products need half the MMAs:
//   scores  S^T[pos][head] = K Q^T: K rows by ldmatrix as the A fragment, Q^T
//           (hi + lo fp16 halves) as B fragments in registers;
//   softmax per head column: the 16 positions' max and sum by shuffles across
//           the fragment rows, the running state per head in every lane;
//   values  O^T[dim][head] += V^T P^T: V^T fragments by ldmatrix.trans, P^T
//           (hi + lo) as B fragments, turned from the score layout through a
//           small tile in shared memory.
// Rows past the position are masked. The 4 warps' (max, sum, O) merge at the
// end, then the splits as in k_battn.
template <int HD, int NH8>
__global__ void __launch_bounds__(kMThreads, 2) k_battn_t(const __grid_constant__ BAttnArgs g) {
    constexpr int HG = 8 * NH8;          // query heads of the CTA
    constexpr int RS = HD + 8;           // padded row, halves
    constexpr int KS = HD / 16;          // K steps of the scores
    constexpr int MT = HD / 16;          // m-tiles of the output (dims)
    constexpr int NW = kMThreads / 32;
    constexpr int PIECES = HD / 8;       // 16-byte pieces per row
    constexpr size_t STAGE = (size_t) 2 * kMChunk * RS;   // halves
    constexpr size_t RING = (size_t) kMStages * STAGE * 2;
    constexpr size_t COMB = (size_t) NW * HG * HD * 4;
    extern __shared__ __align__(16) uint8_t bsm[];
    __shared__ double red[NW];
    __shared__ float wm[NW][HG], wl[NW][HG];
    __shared__ float pt[NW][16][HG + 1];   // a warp's probabilities, [position][head]
    __shared__ unsigned last_flag;
    const int split = blockIdx.x, gy = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int gq = lane >> 2, tq = lane & 3;   // fragment row / column pair
    const int rep = g.n_head / g.n_kv;
    const int kvh = gy / g.hgroups, h0 = (gy % g.hgroups) * HG, nh = min(HG, rep - h0);
    const int pos = g.pos[b];
    float * outb = g.out + (size_t) b * g.ldo + ((size_t) kvh * rep + h0) * HD;
    if (pos < 0) {
        if (split == 0)
            for (int i = tid; i < nh * HD; i += kMThreads) outb[i] = 0.0f;
        return;
    }
    if (pos >= g.n_ctx || rep > kBMaxRep) {
        if (tid == 0) atomicExch(g.err, 214);
        return;
    }
    const int nchunk = pos / kMChunk + 1;
    const int per = (nchunk + g.nsplit - 1) / g.nsplit;
    const int nact = (nchunk + per - 1) / per;
    const int c0 = split * per, c1 = min(nchunk, c0 + per);
    if (c0 >= nchunk) return;
    const int nmine = c1 - c0;
    uint16_t * ring = reinterpret_cast<uint16_t *>(bsm);
    float * qs = reinterpret_cast<float *>(bsm + (RING > COMB ? RING : COMB));   // [HG][HD]
    float * kn = qs + HG * HD, * vn = kn + HD, * cs = vn + HD, * sn = cs + HD / 2;
    float * comb = reinterpret_cast<float *>(bsm);                              // [NW][HG][HD] at the end

    auto issue = [&](int j) {   // chunk c0 + j into stage j % kMStages
        const int t0 = (c0 + j) * kMChunk, nt = min(pos + 1, t0 + kMChunk) - t0;
        uint16_t * Ks = ring + (size_t) (j % kMStages) * STAGE;
        const size_t r0 = kv_row(g, b, kvh, t0);
        for (int i = tid; i < 2 * kMChunk * PIECES; i += kMThreads) {
            const int kv = i / (kMChunk * PIECES), rem = i % (kMChunk * PIECES);
            const int r = rem / PIECES, pc = rem % PIECES;
            const uint16_t * src = (kv ? g.vc : g.kc) + (r0 + min(r, nt - 1)) * HD + pc * 8;
            cp_async16(smem_u32(Ks + (size_t) kv * kMChunk * RS + r * RS + pc * 8), src, r < nt ? 16u : 0u);
        }
    };
#pragma unroll
    for (int j = 0; j < kMStages; j++) {
        if (j < nmine) issue(j);
        cp_async_commit();
    }
    const float * qrow = g.qkv + (size_t) b * g.ldq;
    for (int i = tid; i < HD / 2; i += kMThreads) {
        cs[i] = g.rcos[(size_t) pos * (HD / 2) + i];
        sn[i] = g.rsin[(size_t) pos * (HD / 2) + i];
    }
    for (int i = tid; i < HG * HD; i += kMThreads)
        qs[i] = i < nh * HD ? qrow[((size_t) kvh * rep + h0) * HD + i] : 0.0f;
    for (int i = tid; i < HD; i += kMThreads) {
        kn[i] = qrow[g.koff + kvh * HD + i];
        vn[i] = qrow[g.voff + kvh * HD + i];
    }
    __syncthreads();
    for (int h = 0; h < nh; h++) norm_rope(qs + h * HD, g.qn, g.eps, HD, cs, sn, red);
    norm_rope(kn, g.kn, g.eps, HD, cs, sn, red);
    // Q^T as B fragments: head gq of n-tile n, dims ks*16 + 2 tq (+1) and + 8 (+9)
    uint32_t qb[NH8][KS][2], qbl[NH8][KS][2];
#pragma unroll
    for (int n = 0; n < NH8; n++)
#pragma unroll
        for (int ks = 0; ks < KS; ks++)
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const float * q = qs + (n * 8 + gq) * HD + ks * 16 + 2 * tq + e * 8;
                split_h2(q[0], q[1], qb[n][ks][e], qbl[n][ks][e]);
            }
    // running state of heads n*8 + 2 tq (+1), the same in every lane of a column
    float mh[NH8][2], lh[NH8][2];
    float o[MT][NH8][4];
#pragma unroll
    for (int n = 0; n < NH8; n++) {
        mh[n][0] = mh[n][1] = -INFINITY;
        lh[n][0] = lh[n][1] = 0.0f;
#pragma unroll
        for (int m = 0; m < MT; m++)
#pragma unroll
            for (int e = 0; e < 4; e++) o[m][n][e] = 0.0f;
    }
    const int pw = warp * 16;   // the warp's positions in each chunk
    for (int j = 0; j < nmine; j++) {
        const int c = c0 + j, t0 = c * kMChunk, nt = min(pos + 1, t0 + kMChunk) - t0;
        uint16_t * Ks = ring + (size_t) (j % kMStages) * STAGE, * Vs = Ks + kMChunk * RS;
        cp_async_wait<kMStages - 1>();
        __syncthreads();
        if (c == nchunk - 1) {
            // the new key and value, fp16 round to nearest even, over the stale row
            const int r = pos - t0;
            const size_t rp = h0 == 0 ? kv_row(g, b, kvh, pos) : 0;
            for (int i = tid; i < HD; i += kMThreads) {
                const uint16_t kh = f2h(kn[i]), vh = f2h(vn[i]);
                Ks[r * RS + i] = kh;
                Vs[r * RS + i] = vh;
                if (h0 == 0) {
                    g.kc[rp * HD + i] = kh;
                    g.vc[rp * HD + i] = vh;
                }
            }
            __syncthreads();
        }
        if (pw < nt) {
            // ---- scores: rows gq, gq + 8 are positions pw + ..., columns heads
            float sc[NH8][4], sl[NH8][4];
#pragma unroll
            for (int n = 0; n < NH8; n++)
#pragma unroll
                for (int e = 0; e < 4; e++) sc[n][e] = sl[n][e] = 0.0f;
            const uint32_t kaddr = smem_u32(Ks + (pw + (lane & 15)) * RS + (lane >> 4) * 8);
#pragma unroll
            for (int ks = 0; ks < KS; ks++) {
                uint32_t a[4];
                ldsm4(kaddr + ks * 32, a[0], a[1], a[2], a[3]);
#pragma unroll
                for (int n = 0; n < NH8; n++) {
                    mma16816(sc[n], a, qb[n][ks][0], qb[n][ks][1]);
                    mma16816(sl[n], a, qbl[n][ks][0], qbl[n][ks][1]);
                }
            }
            const bool in0 = pw + gq < nt, in1 = pw + gq + 8 < nt;
#pragma unroll
            for (int n = 0; n < NH8; n++) {
#pragma unroll
                for (int hh = 0; hh < 2; hh++) {
                    // head n*8 + 2 tq + hh: its values at positions gq (e = hh) and gq + 8 (e = 2 + hh)
                    const float v0 = in0 ? (sc[n][hh] + sl[n][hh]) * g.scale : -INFINITY;
                    const float v1 = in1 ? (sc[n][2 + hh] + sl[n][2 + hh]) * g.scale : -INFINITY;
                    float mx = fmaxf(v0, v1);
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
                    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
                    const float mn = fmaxf(mh[n][hh], mx);
                    const float alpha = mh[n][hh] == -INFINITY ? 0.0f : expf(mh[n][hh] - mn);
                    const float p0 = v0 == -INFINITY ? 0.0f : expf(v0 - mn);
                    const float p1 = v1 == -INFINITY ? 0.0f : expf(v1 - mn);
                    float sum = p0 + p1;
                    sum += __shfl_xor_sync(0xffffffffu, sum, 4);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 8);
                    sum += __shfl_xor_sync(0xffffffffu, sum, 16);
                    lh[n][hh] = lh[n][hh] * alpha + sum;
                    mh[n][hh] = mn;
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        o[m][n][hh] *= alpha;
                        o[m][n][2 + hh] *= alpha;
                    }
                    pt[warp][gq][n * 8 + 2 * tq + hh] = p0;
                    pt[warp][gq + 8][n * 8 + 2 * tq + hh] = p1;
                }
            }
            __syncwarp();
            // ---- values: P^T (positions x heads) as B fragments: head gq, positions 2 tq (+1), + 8 (+9)
            uint32_t pb[NH8][2], pbl[NH8][2];
#pragma unroll
            for (int n = 0; n < NH8; n++) {
                split_h2(pt[warp][2 * tq][n * 8 + gq], pt[warp][2 * tq + 1][n * 8 + gq], pb[n][0], pbl[n][0]);
                split_h2(pt[warp][2 * tq + 8][n * 8 + gq], pt[warp][2 * tq + 9][n * 8 + gq], pb[n][1], pbl[n][1]);
            }
            __syncwarp();
            const uint32_t vaddr = smem_u32(Vs + (pw + ((lane >> 4) << 3) + (lane & 7)) * RS + ((lane >> 3) & 1) * 8);
#pragma unroll
            for (int m = 0; m < MT; m++) {
                uint32_t a[4];
                ldsm4t(vaddr + m * 32, a[0], a[1], a[2], a[3]);
#pragma unroll
                for (int n = 0; n < NH8; n++) mma16816(o[m][n], a, pb[n][0], pb[n][1]);
#pragma unroll
                for (int n = 0; n < NH8; n++) mma16816(o[m][n], a, pbl[n][0], pbl[n][1]);
            }
        }
        __syncthreads();   // the stage is free
        if (j + kMStages < nmine) issue(j + kMStages);
        cp_async_commit();
    }
    cp_async_wait<0>();
    __syncthreads();
    // ---- the warps' partial softmax states merge (the ring is free)
    if (gq == 0) {
#pragma unroll
        for (int n = 0; n < NH8; n++)
#pragma unroll
            for (int hh = 0; hh < 2; hh++) {
                wm[warp][n * 8 + 2 * tq + hh] = mh[n][hh];
                wl[warp][n * 8 + 2 * tq + hh] = lh[n][hh];
            }
    }
#pragma unroll
    for (int m = 0; m < MT; m++)
#pragma unroll
        for (int n = 0; n < NH8; n++)
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int d = m * 16 + gq + (e >> 1) * 8, h = n * 8 + 2 * tq + (e & 1);
                comb[(warp * HG + h) * HD + d] = o[m][n][e];
            }
    __syncthreads();
    const size_t grp = (size_t) b * g.n_kv * g.hgroups + gy;
    float * pbuf = g.part + (grp * g.nsplit + split) * HG * (HD + 2);
    for (int i = tid; i < nh * HD; i += kMThreads) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < NW; w++) M = fmaxf(M, wm[w][h]);
        float L = 0.0f, ov = 0.0f;
#pragma unroll
        for (int w = 0; w < NW; w++) {
            if (wm[w][h] == -INFINITY) continue;
            const float e = expf(wm[w][h] - M);
            L += wl[w][h] * e;
            ov += comb[(w * HG + h) * HD + d] * e;
        }
        if (nact == 1) outb[h * HD + d] = ov / L;
        else {
            pbuf[h * (HD + 2) + 2 + d] = ov;
            if (d == 0) { pbuf[h * (HD + 2)] = M; pbuf[h * (HD + 2) + 1] = L; }
        }
    }
    if (nact == 1) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) last_flag = atomicAdd(&g.cnt[grp], 1u) == (unsigned) nact - 1;
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    const float * P = g.part + grp * g.nsplit * HG * (HD + 2);
    const size_t sst = (size_t) HG * (HD + 2);
    for (int i = tid; i < nh * HD; i += kMThreads) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int k = 0; k < nact; k++) M = fmaxf(M, __ldcg(P + k * sst + h * (HD + 2)));
        float L = 0.0f, ov = 0.0f;
        for (int k = 0; k < nact; k++) {
            const float e = expf(__ldcg(P + k * sst + h * (HD + 2)) - M);
            L += __ldcg(P + k * sst + h * (HD + 2) + 1) * e;
            ov += __ldcg(P + k * sst + h * (HD + 2) + 2 + d) * e;
        }
        outb[h * HD + d] = ov / L;
    }
    if (tid == 0) g.cnt[grp] = 0;
}

__host__ __device__ inline size_t battn_t_smem(int hd, int nh8) {
    const size_t ring = (size_t) kMStages * 2 * kMChunk * (hd + 8) * 2;
    const size_t comb = (size_t) (kMThreads / 32) * 8 * nh8 * hd * 4;
    return (ring > comb ? ring : comb) + (size_t) (8 * nh8 * hd + 3 * hd) * 4 + 16;
}

// Greedy choice per sequence: the first index of the largest logit
// (sml/sml-run.c:3539-3544). It becomes the slot's next token, is logged at
// the slot's next position, and the position advances; idle slots stay idle.
constexpr int kArgThreads = 1024;
__global__ void __launch_bounds__(kArgThreads) k_bargmax(const float * logits, int V, int * tok, int * pos,
                                                         int * tlog, int n_ctx) {
    __shared__ float bv[kArgThreads / 32];
    __shared__ int bi[kArgThreads / 32];
    const int b = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float * l = logits + (size_t) b * V;
    float v = -INFINITY;
    int k = 0x7fffffff;
    for (int i = tid; i < V; i += kArgThreads) {
        const float x = l[i];
        if (x > v) { v = x; k = i; }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float v2 = __shfl_xor_sync(0xffffffffu, v, o);
        const int k2 = __shfl_xor_sync(0xffffffffu, k, o);
        if (v2 > v || (v2 == v && k2 < k)) { v = v2; k = k2; }
    }
    if (lane == 0) { bv[warp] = v; bi[warp] = k; }
    __syncthreads();
    if (tid == 0) {
        for (int w = 1; w < kArgThreads / 32; w++)
            if (bv[w] > v || (bv[w] == v && bi[w] < k)) { v = bv[w]; k = bi[w]; }
        if (k == 0x7fffffff) k = 0;
        const int p = pos[b];
        if (p >= 0) {
            tok[b] = k;
            if (tlog && p + 1 <= n_ctx) tlog[(size_t) b * (n_ctx + 1) + p + 1] = k;
            pos[b] = p + 1;
        }
    }
}

}  // namespace sb
