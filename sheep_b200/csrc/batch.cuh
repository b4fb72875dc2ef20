// Kernels of the batched decode step (sb_batch): B sequences advance one
// token each per step, each at its own position with its own fp16 KV cache.
// The products run on the tensor-core path (tc_batch.cu); this file holds the
// per-sequence work around them:
//
//   k_bembed    the B embedding rows, dequantized and scattered to natural order
//   k_battn     RoPE, the KV write and split-position attention, one CTA per
//               (128 positions, KV head, sequence) serving every query head
//               of the KV head's group, so each cached byte is read once
//   k_bargmax   the greedy choice per sequence, fed back as its next token
//
// The CPU body these follow is sml_forward_multi / forward_slots
// (sml/sml-run.c:2559-2604, 2218), one sequence's arithmetic being
// sml_forward's (sml/sml-run.c:3243-3523).
#pragma once

#include "decode.cuh"

namespace sb {

constexpr int kBChunk = 128;     // positions per attention CTA
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
    uint16_t * kc, * vc;     // this layer's cache: [B][n_kv][n_ctx][hd] fp16
    int n_ctx;
    const int * pos;         // [B]; < 0: an idle slot
    int max_chunks;
    float scale;             // 1/sqrt(hd)
    float * part;            // [B][n_kv][max_chunks][rep][hd + 2]: max, sum, weighted values
    unsigned * cnt;          // [B][n_kv] arrivals, zero between steps
    float * out;             // [B][ldo] attention output (head-major)
    int ldo;
    int * err;
};

// Shared memory of k_battn: the chunk's keys and values, the group's rotated
// queries, the new key and value, the RoPE row and the scores.
__host__ __device__ inline size_t battn_smem(int hd, int rep) {
    const int rp = (rep + 3) / 4 * 4;
    return (size_t) 2 * kBChunk * hd * 2 + (size_t) (rp * hd + 3 * hd) * 4 + (size_t) kBChunk * rp * 4 + 16;
}

// One CTA per (chunk of 128 positions, KV head, sequence).
//  1. one thread starts bulk copies of the chunk's keys and values (contiguous
//     in the cache layout) while every thread loads the group's queries and the
//     new key/value, applies the Q/K norms and RoPE (sml/sml-run.c:295-375);
//  2. the chunk owning `pos` writes the new key/value (fp16, round to nearest
//     even) into its copy and into the cache;
//  3. scores: a team of 8 lanes (16 for hd 256) per position, each lane 16 B
//     column pieces of the key row (a team reads 128 contiguous bytes) against
//     the queries of 4 heads held in registers, summed across the team;
//  4. per head, the max-subtracted softmax of the chunk (expf);
//  5. weighted values: each warp a stride of positions, each lane hd/32
//     columns, the 4 heads' weights of a position read as one float4; the
//     warps' sums added in warp order;
//  6. chunks meet in `part`; the last CTA of the (sequence, KV head) combines
//     them in chunk order (flash-decoding partials, as k_attn).
template <int HD>
__global__ void __launch_bounds__(kBThreads) k_battn(const __grid_constant__ BAttnArgs g) {
    constexpr int LPP = HD <= 128 ? 8 : 16;   // lanes per position in the scores
    constexpr int NCH = HD / 8;                // 16-byte pieces per key row
    constexpr int CPL = NCH / LPP;             // pieces per lane (1 or 2)
    constexpr int PPW = 32 / LPP;              // positions per warp step
    constexpr int DV = HD / 32;                // columns per lane in the weighted sum
    extern __shared__ __align__(16) uint8_t bsm[];
    __shared__ __align__(8) uint64_t bar;
    __shared__ double red[kBThreads / 32];
    __shared__ float hm[kBMaxRep], hl[kBMaxRep];
    __shared__ unsigned last_flag;
    const int c = blockIdx.x, kvh = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int rep = g.n_head / g.n_kv, rp = (rep + 3) / 4 * 4;
    const int pos = g.pos[b];
    float * outb = g.out + (size_t) b * g.ldo + (size_t) kvh * rep * HD;
    if (pos < 0) {
        if (c == 0)
            for (int i = tid; i < rep * HD; i += kBThreads) outb[i] = 0.0f;
        return;
    }
    if (pos >= g.n_ctx || rep > kBMaxRep) {
        if (tid == 0) atomicExch(g.err, 211);
        return;
    }
    const int nchunk = pos / kBChunk + 1;
    if (c >= nchunk) return;
    const int t0 = c * kBChunk, nt = min(pos + 1, t0 + kBChunk) - t0;
    uint16_t * Ks = reinterpret_cast<uint16_t *>(bsm);          // [kBChunk][HD]
    uint16_t * Vs = Ks + kBChunk * HD;                           // [kBChunk][HD]
    float * qs = reinterpret_cast<float *>(Vs + kBChunk * HD);   // [rp][HD]
    float * kn = qs + rp * HD, * vn = kn + HD, * cs = vn + HD, * sn = cs + HD / 2;
    float * sc = sn + HD / 2;                                    // [kBChunk][rp]
    float * ro = reinterpret_cast<float *>(bsm);                 // [8 warps][4][HD], over Ks after the scores
    const size_t row0 = ((size_t) b * g.n_kv + kvh) * g.n_ctx;

    if (tid == 0) {
        mbar_init(&bar, 1);
        mbar_fence_init();
    }
    __syncthreads();
    if (tid == 0) {
        const uint32_t bytes = (uint32_t) nt * HD * 2;
        mbar_expect_tx(&bar, 2 * bytes);
        bulk_g2s(Ks, g.kc + (row0 + t0) * HD, bytes, &bar);
        bulk_g2s(Vs, g.vc + (row0 + t0) * HD, bytes, &bar);
    }
    const float * qrow = g.qkv + (size_t) b * g.ldq;
    for (int i = tid; i < HD / 2; i += kBThreads) {
        cs[i] = g.rcos[(size_t) pos * (HD / 2) + i];
        sn[i] = g.rsin[(size_t) pos * (HD / 2) + i];
    }
    for (int i = tid; i < rp * HD; i += kBThreads)
        qs[i] = i < rep * HD ? qrow[(size_t) kvh * rep * HD + i] : 0.0f;
    for (int i = tid; i < HD; i += kBThreads) {
        kn[i] = qrow[g.koff + kvh * HD + i];
        vn[i] = qrow[g.voff + kvh * HD + i];
    }
    __syncthreads();
    for (int h = 0; h < rep; h++) norm_rope(qs + h * HD, g.qn, g.eps, HD, cs, sn, red);
    norm_rope(kn, g.kn, g.eps, HD, cs, sn, red);
    const bool landed = mbar_wait(&bar, 0, g.err, 212);
    if (pos < t0 + nt && landed) {
        const int r = pos - t0;
        for (int i = tid; i < HD; i += kBThreads) {
            const uint16_t kh = f2h(kn[i]), vh = f2h(vn[i]);
            Ks[r * HD + i] = kh;
            Vs[r * HD + i] = vh;
            g.kc[(row0 + pos) * HD + i] = kh;
            g.vc[(row0 + pos) * HD + i] = vh;
        }
    }
    __syncthreads();
    if (!landed) return;

    // ---- scores (sml/sml-run.c:180-235: dot * 1/sqrt(hd))
    const int team = lane / LPP, tl = lane % LPP;
    for (int hg = 0; hg < rp; hg += 4) {
        float qr[4][CPL * 8];
#pragma unroll
        for (int h = 0; h < 4; h++)
#pragma unroll
            for (int k = 0; k < CPL; k++)
#pragma unroll
                for (int j = 0; j < 8; j++) qr[h][k * 8 + j] = qs[(hg + h) * HD + (tl + k * LPP) * 8 + j];
        for (int p0 = 0; p0 < nt; p0 += (kBThreads / 32) * PPW) {
            const int p = p0 + warp * PPW + team;
            float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (p < nt) {
#pragma unroll
                for (int k = 0; k < CPL; k++) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(Ks + p * HD + (tl + k * LPP) * 8);
                    const uint32_t wv[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wv[j]));
#pragma unroll
                        for (int h = 0; h < 4; h++) {
                            s[h] = fmaf(qr[h][k * 8 + 2 * j], f.x, s[h]);
                            s[h] = fmaf(qr[h][k * 8 + 2 * j + 1], f.y, s[h]);
                        }
                    }
                }
            }
#pragma unroll
            for (int o = LPP / 2; o; o >>= 1)
#pragma unroll
                for (int h = 0; h < 4; h++) s[h] += __shfl_xor_sync(0xffffffffu, s[h], o);
            if (p < nt && tl == 0)
                *reinterpret_cast<float4 *>(sc + p * rp + hg) =
                    make_float4(s[0] * g.scale, s[1] * g.scale, s[2] * g.scale, s[3] * g.scale);
        }
    }
    __syncthreads();

    // ---- softmax of the chunk, per head (max-subtracted, expf)
    for (int h = warp; h < rep; h += kBThreads / 32) {
        float m = -INFINITY;
        for (int p = lane; p < nt; p += 32) m = fmaxf(m, sc[p * rp + h]);
        m = warp_max(m);
        float l = 0.0f;
        for (int p = lane; p < nt; p += 32) {
            const float e = expf(sc[p * rp + h] - m);
            sc[p * rp + h] = e;
            l += e;
        }
        l = warp_sum(l);
        if (lane == 0) { hm[h] = m; hl[h] = l; }
    }
    __syncthreads();

    // ---- weighted values
    float * pb = g.part + ((row0 / g.n_ctx) * g.max_chunks + c) * (size_t) rep * (HD + 2);
    for (int hg = 0; hg < rp; hg += 4) {
        float o[4][DV];
#pragma unroll
        for (int h = 0; h < 4; h++)
#pragma unroll
            for (int d = 0; d < DV; d++) o[h][d] = 0.0f;
        for (int p = warp; p < nt; p += kBThreads / 32) {
            const float4 pr = *reinterpret_cast<const float4 *>(sc + p * rp + hg);
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
            for (int d = 0; d < DV; d++) {
                o[0][d] = fmaf(pr.x, v[d], o[0][d]);
                o[1][d] = fmaf(pr.y, v[d], o[1][d]);
                o[2][d] = fmaf(pr.z, v[d], o[2][d]);
                o[3][d] = fmaf(pr.w, v[d], o[3][d]);
            }
        }
        __syncthreads();   // the keys (under ro) are no longer read; the previous group's sums are taken
#pragma unroll
        for (int h = 0; h < 4; h++)
#pragma unroll
            for (int d = 0; d < DV; d++) ro[(warp * 4 + h) * HD + lane * DV + d] = o[h][d];
        __syncthreads();
        for (int i = tid; i < 4 * HD; i += kBThreads) {
            const int h = i / HD, d = i % HD;
            if (hg + h >= rep) continue;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < kBThreads / 32; w++) s += ro[(w * 4 + h) * HD + d];
            if (nchunk == 1) outb[(hg + h) * HD + d] = s / hl[hg + h];
            else pb[(hg + h) * (HD + 2) + 2 + d] = s;
        }
    }
    if (nchunk == 1) return;
    if (tid < rep) {
        pb[tid * (HD + 2)] = hm[tid];
        pb[tid * (HD + 2) + 1] = hl[tid];
    }
    __threadfence();
    __syncthreads();
    unsigned * cnt = g.cnt + (size_t) b * g.n_kv + kvh;
    if (tid == 0) last_flag = atomicAdd(cnt, 1u) == (unsigned) nchunk - 1;
    __syncthreads();
    if (!last_flag) return;
    __threadfence();
    // the last chunk combines every chunk of the group, in chunk order
    const volatile float * P = g.part + (row0 / g.n_ctx) * g.max_chunks * (size_t) rep * (HD + 2);
    const size_t cst = (size_t) rep * (HD + 2);
    for (int i = tid; i < rep * HD; i += kBThreads) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int k = 0; k < nchunk; k++) M = fmaxf(M, P[k * cst + h * (HD + 2)]);
        float L = 0.0f, o = 0.0f;
        for (int k = 0; k < nchunk; k++) {
            const float e = expf(P[k * cst + h * (HD + 2)] - M);
            L += P[k * cst + h * (HD + 2) + 1] * e;
            o += P[k * cst + h * (HD + 2) + 2 + d] * e;
        }
        outb[h * HD + d] = o / L;
    }
    if (tid == 0) *cnt = 0;
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
