// Decode attention as a kernel-level C entry point: one token at position pos
// against an fp16 KV cache, device pointers in and out (the k_attn kernel of
// the decode graph: RoPE, the cache write at pos, chunked attention). Replaces
// the reference's sml_g_attn2 launch (sml/sml-gpu-fwd.c:346-356).
#include "decode.cuh"
#include "sheep_b200.h"

#include <cstdio>

using namespace sb;

static thread_local char g_attn_err[256];

extern "C" const char * sb_attn_last_error(void) { return g_attn_err; }

// Shape checks shared by the entry points; fills the kernel arguments except
// the scratch (partials, counters).
static bool attn_args(AttnArgs & a, const float * qkv, uint16_t * kc, uint16_t * vc, const float * rope_cos,
                      const float * rope_sin, const float * q_norm, const float * k_norm, float eps, int n_head,
                      int n_head_kv, int head_dim, int n_ctx, int pos, float scale, float * out, int & nchunk) {
    g_attn_err[0] = 0;
    if (!qkv || !kc || !vc || !rope_cos || !rope_sin || !out || n_head <= 0 || n_head_kv <= 0 ||
        n_head % n_head_kv || head_dim <= 0 || head_dim % 8 || head_dim > 256 || n_ctx <= 0 || pos < 0 ||
        pos >= n_ctx) {
        snprintf(g_attn_err, sizeof g_attn_err, "invalid attention arguments");
        return false;
    }
    memset(&a, 0, sizeof a);
    a.qkv = qkv; a.n_head = n_head; a.n_kv = n_head_kv; a.hd = head_dim;
    a.qd = n_head * head_dim; a.kvd = n_head_kv * head_dim;
    a.qn = q_norm; a.kn = k_norm; a.eps = eps;
    a.rcos = rope_cos; a.rsin = rope_sin;
    a.kc = kc; a.vc = vc; a.n_ctx = n_ctx;
    a.pos = nullptr; a.pos_imm = pos;
    a.chunk = head_dim <= 128 ? 64 : 32;
    a.scale = scale;
    a.out = out;
    nchunk = pos / a.chunk + 1;
    a.max_chunks = nchunk;
    return true;
}

// Launch with the scratch in place: part [n_head][nchunk][hd + 2] floats and
// cnt [n_head] counters, zero on entry and left zero on exit.
static bool attn_launch(AttnArgs & a, int nchunk, float * part, unsigned * cnt, cudaStream_t st) {
    a.part = part;
    a.cnt = cnt;
    k_attn<<<dim3(a.n_head, nchunk), kAttnThreads, attn_smem_bytes(a.hd, a.chunk), st>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) snprintf(g_attn_err, sizeof g_attn_err, "k_attn: %s", cudaGetErrorString(e));
    return e == cudaSuccess;
}

extern "C" int sb_attn_decode(const float * qkv, uint16_t * kc, uint16_t * vc, const float * rope_cos,
                              const float * rope_sin, const float * q_norm, const float * k_norm, float eps,
                              int n_head, int n_head_kv, int head_dim, int n_ctx, int pos, float scale, float * out,
                              void * stream) {
    AttnArgs a;
    int nchunk = 0;
    if (!attn_args(a, qkv, kc, vc, rope_cos, rope_sin, q_norm, k_norm, eps, n_head, n_head_kv, head_dim, n_ctx, pos,
                   scale, out, nchunk))
        return 0;
    const size_t part_bytes = (size_t) n_head * nchunk * (head_dim + 2) * sizeof(float);
    void * scratch = nullptr;
    cudaStream_t st = (cudaStream_t) stream;
    if (cudaMalloc(&scratch, part_bytes + (size_t) n_head * sizeof(unsigned)) != cudaSuccess) {
        snprintf(g_attn_err, sizeof g_attn_err, "cudaMalloc of the attention scratch failed");
        return 0;
    }
    unsigned * cnt = (unsigned *) ((char *) scratch + part_bytes);
    bool ok = cudaMemsetAsync(cnt, 0, (size_t) n_head * sizeof(unsigned), st) == cudaSuccess;
    ok = ok && attn_launch(a, nchunk, (float *) scratch, cnt, st);
    ok = cudaStreamSynchronize(st) == cudaSuccess && ok;
    cudaFree(scratch);
    return ok ? 1 : 0;
}
