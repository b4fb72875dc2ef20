// One MoE FFN layer of an SSF file as a C entry point (router, routing,
// experts, combine), and the routing alone.
//
// The reference runs this layer inside its forward pass (moe_ffn,
// sml/sml-run.c:3071-3125; moe_ffn_dev, sml/sml-gpu-fwd.c:492-546) and exposes
// the routing as sml_moe_route (sml/sml-run.h:304). Taking the layer out on its
// own gives the expert-GEMV path a boundary of its own, for a host that
// batches tokens by layer and for measurement at 1..256 tokens a step.
#include "moe_host.h"
#include "sheep_b200.h"
#include "ssf.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>

using namespace sb;

static thread_local char g_err[512];

extern "C" const char * sb_moe_last_error(void) { return g_err; }

// NCCL, loaded when an expert-parallel layer is opened (single-GPU users need
// no NCCL; in a process that already loaded one, dlopen returns that one).
struct NcclApi {
    ncclResult_t (*get_id)(ncclUniqueId *);
    ncclResult_t (*init_rank)(ncclComm_t *, int, ncclUniqueId, int);
    ncclResult_t (*all_reduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
    ncclResult_t (*destroy)(ncclComm_t);
    const char * (*error)(ncclResult_t);
};

static const NcclApi * nccl_api() {
    static NcclApi api;
    static int state = 0;   // 0 untried, 1 loaded, -1 unavailable
    if (state) return state > 0 ? &api : nullptr;
    state = -1;
    void * h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return nullptr;
    api.get_id = (ncclResult_t (*)(ncclUniqueId *)) dlsym(h, "ncclGetUniqueId");
    api.init_rank = (ncclResult_t (*)(ncclComm_t *, int, ncclUniqueId, int)) dlsym(h, "ncclCommInitRank");
    api.all_reduce = (ncclResult_t (*)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                       cudaStream_t)) dlsym(h, "ncclAllReduce");
    api.destroy = (ncclResult_t (*)(ncclComm_t)) dlsym(h, "ncclCommDestroy");
    api.error = (const char * (*)(ncclResult_t)) dlsym(h, "ncclGetErrorString");
    if (!api.get_id || !api.init_rank || !api.all_reduce || !api.destroy || !api.error) return nullptr;
    state = 1;
    return &api;
}

struct sb_moe {
    ssf_file f{};
    int world = 1, rank = 0;              // expert parallelism: this GPU holds experts [rank*ne/world, ...)
    ncclComm_t comm = nullptr;
    MoeExchange ex{};
    Arena ar;
    MoeLayer m;
    MoeScratch s;
    float * x = nullptr, * y = nullptr;   // device rows [T][E]
    int * err = nullptr;
    const ExpfEntry * xtab = nullptr;     // the host libm's expf corrections (expf_libm.h)
    float xnear = 0.0f;
    int nsm = 148, tmax = 0, layer = 0;
    int tc = MOE_TC_AUTO;                 // MoeTc: which calls run on the tensor cores (moe_tc.cu)
    cudaStream_t st = nullptr;
    void * flush = nullptr;               // timing: a buffer larger than L2, rewritten between runs
    size_t flush_n = 0;
};

static bool ck(cudaError_t e, const char * what) {
    if (e == cudaSuccess) return true;
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return false;
}

static void moe_free(sb_moe * h) {
    if (h->comm) nccl_api()->destroy(h->comm);
    if (h->st) cudaStreamDestroy(h->st);
    if (h->flush) cudaFree(h->flush);
    h->ar.release();
    ssf_close(&h->f);
    delete h;
}

static bool moe_build(sb_moe * h, char * why, int nwhy) {
    int e_lo = 0, e_hi = 0;
    if (h->world > 1) {
        const ssf_rec * rt = ssf_findf(&h->f, "blk.%d.ffn_gate_inp.weight", h->layer, 0);
        const int ne = rt ? (int) ((uint64_t) rt->rows * rt->cols / h->f.hdr->n_embd) : 0;
        if (ne < h->world) { snprintf(why, nwhy, "%d experts cannot spread over %d GPUs", ne, h->world); return false; }
        e_lo = (int) ((long) ne * h->rank / h->world);
        e_hi = (int) ((long) ne * (h->rank + 1) / h->world);
    }
    if (!moe_upload(h->ar, h->f, h->layer, h->m, why, nwhy, e_lo, e_hi)) return false;
    moe_carve(h->ar, h->m, h->tmax, h->s);
    h->x = (float *) h->ar.carve((size_t) h->tmax * h->m.E * 4);
    h->y = (float *) h->ar.carve((size_t) h->tmax * h->m.E * 4);
    h->err = (int *) h->ar.carve(4);
    const ExpfTable & xt = expf_libm_table();
    if (xt.slots.empty()) { snprintf(why, nwhy, "this libm's expf differs from the rounded exponential too often"); return false; }
    h->xtab = (const ExpfEntry *) h->ar.upload(xt.slots.data(), xt.slots.size() * sizeof(ExpfEntry));
    h->xnear = xt.near;
    return true;
}

static cudaError_t ep_sum(void * ctx, float * buf, size_t n, cudaStream_t st) {
    sb_moe * h = (sb_moe *) ctx;
    const ncclResult_t r = nccl_api()->all_reduce(buf, buf, n, ncclFloat, ncclSum, h->comm, st);
    if (r != ncclSuccess) {
        snprintf(g_err, sizeof g_err, "ncclAllReduce: %s", nccl_api()->error(r));
        return cudaErrorUnknown;
    }
    return cudaSuccess;
}

static sb_moe * moe_open(const char * path, int layer, int max_tokens, int world, int rank, const void * id,
                         char * why, int nwhy) {
    g_err[0] = 0;
    if (max_tokens < 1 || max_tokens > 4096) { snprintf(why, nwhy, "max_tokens must be 1..4096"); return nullptr; }
    if (world < 1 || world > 64 || rank < 0 || rank >= world || (world > 1 && !id)) {
        snprintf(why, nwhy, "world %d / rank %d / id", world, rank);
        return nullptr;
    }
    if (world > 1 && !nccl_api()) { snprintf(why, nwhy, "NCCL (libnccl.so.2) could not be loaded"); return nullptr; }
    sb_moe * h = new sb_moe();
    h->world = world;
    h->rank = rank;
    if (!ssf_open(&h->f, path, why, nwhy)) { delete h; return nullptr; }
    if (layer < 0 || layer >= (int) h->f.hdr->n_layer) {
        snprintf(why, nwhy, "layer %d out of range", layer);
        moe_free(h);
        return nullptr;
    }
    h->layer = layer;
    h->tmax = max_tokens;
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&h->nsm, cudaDevAttrMultiProcessorCount, dev);
    if (!moe_build(h, why, nwhy)) { moe_free(h); return nullptr; }
    if (!h->ar.allocate()) {
        snprintf(why, nwhy, "cudaMalloc of %.2f GB failed", h->ar.size / 1e9);
        moe_free(h);
        return nullptr;
    }
    if (!moe_build(h, why, nwhy)) { moe_free(h); return nullptr; }
    if (!ck(cudaStreamCreateWithFlags(&h->st, cudaStreamNonBlocking), "stream") ||
        !ck(cudaDeviceSynchronize(), "upload")) {
        snprintf(why, nwhy, "%s", g_err);
        moe_free(h);
        return nullptr;
    }
    if (world > 1) {
        ncclUniqueId uid;
        memcpy(&uid, id, sizeof uid);
        const ncclResult_t r = nccl_api()->init_rank(&h->comm, world, uid, rank);
        if (r != ncclSuccess) {
            snprintf(why, nwhy, "ncclCommInitRank: %s", nccl_api()->error(r));
            h->comm = nullptr;
            moe_free(h);
            return nullptr;
        }
        h->ex.sum = ep_sum;
        h->ex.ctx = h;
    }
    return h;
}

extern "C" sb_moe * sb_moe_open(const char * path, int layer, int max_tokens, char * why, int nwhy) {
    return moe_open(path, layer, max_tokens, 1, 0, nullptr, why, nwhy);
}

// Expert parallelism: `world` processes (one GPU each) call this with the same
// id; this one holds experts [rank*ne/world, (rank+1)*ne/world).
extern "C" sb_moe * sb_moe_open_ep(const char * path, int layer, int max_tokens, int world, int rank,
                                   const void * nccl_id, char * why, int nwhy) {
    return moe_open(path, layer, max_tokens, world, rank, nccl_id, why, nwhy);
}

extern "C" int sb_nccl_unique_id(void * id128) {
    g_err[0] = 0;
    const NcclApi * api = nccl_api();
    if (!api || !id128) { snprintf(g_err, sizeof g_err, "NCCL (libnccl.so.2) could not be loaded"); return 0; }
    ncclUniqueId uid;
    const ncclResult_t r = api->get_id(&uid);
    if (r != ncclSuccess) { snprintf(g_err, sizeof g_err, "ncclGetUniqueId: %s", api->error(r)); return 0; }
    memcpy(id128, &uid, sizeof uid);
    return 1;
}

extern "C" void sb_moe_close(sb_moe * h) {
    if (!h) return;
    cudaStreamSynchronize(h->st);
    moe_free(h);
}

// out: n_embd, expert hidden size, experts, experts per token, routing flags,
// max tokens, expert width (bits), bytes of one expert as stored (low, high 32
// bits), router bytes.
extern "C" void sb_moe_info(const sb_moe * h, int * out) {
    out[0] = h->m.E; out[1] = h->m.F; out[2] = h->m.ne; out[3] = h->m.k; out[4] = (int) h->m.flags;
    out[5] = h->tmax; out[6] = h->m.gu.nbits;
    out[7] = (int) (h->m.expert_file_bytes & 0xffffffffu); out[8] = (int) (h->m.expert_file_bytes >> 32);
    out[9] = (int) h->m.router_bytes;
    out[10] = h->world; out[11] = h->rank; out[12] = h->m.e_lo; out[13] = h->m.e_hi;
}

static bool enqueue(sb_moe * h, const float * x, int T, float * y, cudaStream_t st) {
    bool ok = true;
    moe_enqueue(h->m, h->s, x, T, nullptr, 0.0f, y, 0, h->nsm, st, true, h->err, nullptr, 0,
                [&](cudaError_t e, const char * name) {
                    if (ok && e != cudaSuccess) {
                        if (e != cudaErrorUnknown || !g_err[0]) ck(e, name);   // an NCCL failure set its own message
                        ok = false;
                    }
                },
                h->world > 1 ? &h->ex : nullptr, h->xtab, h->xnear, h->tc);
    return ok;
}

extern "C" int sb_moe_set_tensor_cores(sb_moe * h, int on) {
    if (!h) return 0;
    h->tc = on == 0 ? MOE_TC_OFF : on == 2 ? MOE_TC_AUTO : MOE_TC_ON;
    return h->s.tc_chunks > 0 ? 1 : 0;
}

extern "C" int sb_moe_forward(sb_moe * h, const float * x, int n_tok, float * y, void * stream) {
    g_err[0] = 0;
    if (!h || !x || !y || n_tok < 1 || n_tok > h->tmax) { snprintf(g_err, sizeof g_err, "invalid arguments"); return 0; }
    if (((uintptr_t) x | (uintptr_t) y) & 15) { snprintf(g_err, sizeof g_err, "x and y must be 16-byte aligned"); return 0; }
    return enqueue(h, x, n_tok, y, (cudaStream_t) stream) ? 1 : 0;
}

// Host rows in and out (copies inside); sel/w (n_tok x k) and n_active may be NULL.
extern "C" int sb_moe_forward_host(sb_moe * h, const float * x, int n_tok, float * y, int * sel, float * w,
                                   int * n_active) {
    g_err[0] = 0;
    if (!h || !x || !y || n_tok < 1 || n_tok > h->tmax) { snprintf(g_err, sizeof g_err, "invalid arguments"); return 0; }
    const size_t rb = (size_t) n_tok * h->m.E * 4, nk = (size_t) n_tok * h->m.k;
    int meta[2] = {0, 0}, err = 0;
    bool ok = ck(cudaMemcpyAsync(h->x, x, rb, cudaMemcpyHostToDevice, h->st), "copy in") &&
              enqueue(h, h->x, n_tok, h->y, h->st) &&
              ck(cudaMemcpyAsync(y, h->y, rb, cudaMemcpyDeviceToHost, h->st), "copy out") &&
              (!sel || ck(cudaMemcpyAsync(sel, h->s.r.sel, nk * 4, cudaMemcpyDeviceToHost, h->st), "sel")) &&
              (!w || ck(cudaMemcpyAsync(w, h->s.r.w, nk * 4, cudaMemcpyDeviceToHost, h->st), "w")) &&
              ck(cudaMemcpyAsync(meta, h->s.r.meta, 8, cudaMemcpyDeviceToHost, h->st), "meta") &&
              ck(cudaMemcpyAsync(&err, h->err, 4, cudaMemcpyDeviceToHost, h->st), "err") &&
              ck(cudaStreamSynchronize(h->st), "forward");
    if (ok && err) {
        snprintf(g_err, sizeof g_err, "a bounded wait gave up (code %d)", err);
        ok = false;
    }
    if (n_active) *n_active = meta[1];
    return ok ? 1 : 0;
}

// Device time of the layer over n_tok rows already on the device: reps runs,
// each preceded (outside its timing) by a rewrite of a buffer larger than L2, so
// every run reads its experts from HBM. ms_avg: mean CUDA-event time of one run;
// n_active: experts the routing chose (the same every run).
extern "C" int sb_moe_time(sb_moe * h, const float * x_host, int n_tok, int reps, float * ms_avg, int * n_active) {
    g_err[0] = 0;
    if (!h || !x_host || n_tok < 1 || n_tok > h->tmax || reps < 1) { snprintf(g_err, sizeof g_err, "invalid arguments"); return 0; }
    if (!h->flush) {
        h->flush_n = (size_t) 512 << 20;
        if (!ck(cudaMalloc(&h->flush, h->flush_n), "flush buffer")) { h->flush = nullptr; return 0; }
    }
    if (!ck(cudaMemcpy(h->x, x_host, (size_t) n_tok * h->m.E * 4, cudaMemcpyHostToDevice), "copy in")) return 0;
    cudaEvent_t a, b;
    cudaEventCreate(&a);
    cudaEventCreate(&b);
    bool ok = true;
    for (int r = 0; ok && r < 3; r++) ok = enqueue(h, h->x, n_tok, h->y, h->st);
    double total = 0.0;
    for (int r = 0; ok && r < reps; r++) {
        ok = ck(cudaMemsetAsync(h->flush, r & 0xff, h->flush_n, h->st), "flush") &&
             ck(cudaEventRecord(a, h->st), "event") && enqueue(h, h->x, n_tok, h->y, h->st) &&
             ck(cudaEventRecord(b, h->st), "event") && ck(cudaEventSynchronize(b), "run");
        float ms = 0.0f;
        if (ok) cudaEventElapsedTime(&ms, a, b);
        total += ms;
    }
    int meta[2] = {0, 0}, err = 0;
    ok = ok && ck(cudaMemcpy(meta, h->s.r.meta, 8, cudaMemcpyDeviceToHost), "meta") &&
         ck(cudaMemcpy(&err, h->err, 4, cudaMemcpyDeviceToHost), "err");
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (ok && err) { snprintf(g_err, sizeof g_err, "a bounded wait gave up (code %d)", err); ok = false; }
    if (ms_avg) *ms_avg = (float) (total / reps);
    if (n_active) *n_active = meta[1];
    return ok ? 1 : 0;
}

extern "C" int sb_moe_route(const float * logits, int n_tok, int n_expert, int k, unsigned flags, int * sel,
                            float * w, void * stream) {
    g_err[0] = 0;
    if (!logits || !sel || !w || n_tok < 1 || n_expert < 1 || n_expert > kMoeMaxExperts || k < 1 || k > n_expert ||
        k > kMoeMaxK || (flags & ~1u)) {
        snprintf(g_err, sizeof g_err, "invalid routing arguments");
        return 0;
    }
    const int per = 4;   // tokens (warps) per block
    k_moe_route<<<(n_tok + per - 1) / per, 32 * per, 0, (cudaStream_t) stream>>>(logits, n_tok, n_expert, k, flags, sel, w);
    return ck(cudaGetLastError(), "k_moe_route") ? 1 : 0;
}
