// One MoE FFN layer of an SSF file as a C entry point (router, routing,
// experts, combine), and the routing alone.
//
// The reference runs this layer inside its forward pass (moe_ffn,
// sml/sml-run.c:3071-3125; moe_ffn_dev, sml/sml-gpu-fwd.c:492-546) and exposes
// the routing as sml_moe_route (sml/sml-run.h:304). Taking the layer out on its
// own gives the expert-GEMV path a boundary of its own, for a host that
// batches tokens by layer and for measurement at 1..256 tokens a step.
#include "moe_a2a.h"
#include "moe_host.h"
#include "nccl_rt.h"
#include "sheep_b200.h"
#include "ssf.h"

#include <dlfcn.h>
#include <nccl.h>

#include <cstdio>
#include <cstring>

using namespace sb;

static thread_local char g_err[512];

extern "C" const char * sb_moe_last_error(void) { return g_err; }

const NcclApi * sb::nccl_api() {
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
    api.all_gather = (ncclResult_t (*)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t))
        dlsym(h, "ncclAllGather");
    api.send = (ncclResult_t (*)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t)) dlsym(h, "ncclSend");
    api.recv = (ncclResult_t (*)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t)) dlsym(h, "ncclRecv");
    api.group_start = (ncclResult_t (*)()) dlsym(h, "ncclGroupStart");
    api.group_end = (ncclResult_t (*)()) dlsym(h, "ncclGroupEnd");
    if (!api.get_id || !api.init_rank || !api.all_reduce || !api.destroy || !api.error || !api.all_gather ||
        !api.send || !api.recv || !api.group_start || !api.group_end)
        return nullptr;
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
    // all-to-all exchange (sb_moe_set_exchange 1): each rank passes its own tokens
    int a2a = 0;
    int * selpk = nullptr, * selall = nullptr, * h_selall = nullptr;   // [1 + tmax k] per rank: T, then sel
    float * sendbuf = nullptr, * yback = nullptr;                      // [tmax k][E]
    float * recvbuf = nullptr, * yrecv = nullptr, * hp2 = nullptr;     // [world tmax k][E], [..][F]
    int * d_plan = nullptr, * h_plan = nullptr;                        // send_tok, send_slot, slots, ch_e, ch_s0, ch_n, meta
    MoeA2aPlan plan;
};

static bool ck(cudaError_t e, const char * what) {
    if (e == cudaSuccess) return true;
    snprintf(g_err, sizeof g_err, "%s: %s", what, cudaGetErrorString(e));
    return false;
}

// Ints of the all-to-all plan staged per step: send_tok, send_slot [tmax k],
// slots, ch_e, ch_s0, ch_n [world tmax k], meta [2].
static size_t a2a_plan_ints(const sb_moe * h) {
    const size_t nk = (size_t) h->tmax * h->m.k;
    return 2 * nk + 4 * nk * h->world + 2;
}

static void moe_free(sb_moe * h) {
    if (h->comm) nccl_api()->destroy(h->comm);
    if (h->h_selall) cudaFreeHost(h->h_selall);
    if (h->h_plan) cudaFreeHost(h->h_plan);
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
    if (h->world > 1) {
        const size_t nk = (size_t) h->tmax * h->m.k, rows = nk * h->world;
        h->selpk = (int *) h->ar.carve((1 + nk) * 4);
        h->selall = (int *) h->ar.carve((1 + nk) * h->world * 4);
        h->sendbuf = (float *) h->ar.carve(nk * h->m.E * 4);
        h->yback = (float *) h->ar.carve(nk * h->m.E * 4);
        h->recvbuf = (float *) h->ar.carve(rows * h->m.E * 4);
        h->yrecv = (float *) h->ar.carve(rows * h->m.E * 4);
        h->hp2 = (float *) h->ar.carve(rows * h->m.F * 4);
        h->d_plan = (int *) h->ar.carve(a2a_plan_ints(h) * 4);
    }
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
        const size_t nk = (size_t) h->tmax * h->m.k;
        if (!ck(cudaMallocHost(&h->h_selall, (1 + nk) * world * 4), "pinned selections") ||
            !ck(cudaMallocHost(&h->h_plan, a2a_plan_ints(h) * 4), "pinned plan")) {
            snprintf(why, nwhy, "%s", g_err);
            moe_free(h);
            return nullptr;
        }
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

// ------------------------------------------------------------------ all-to-all

// dst[i] = src[idx[i]] (rows of E floats).
static __global__ void k_gather_rows(float * dst, const float * src, const int * idx, int n, int E) {
    const int r = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n && 4 * i < E)
        reinterpret_cast<float4 *>(dst + (size_t) r * E)[i] = reinterpret_cast<const float4 *>(src + (size_t) idx[r] * E)[i];
}

// dst[idx[i]] = src[i] (rows of E floats).
static __global__ void k_scatter_rows(float * dst, const float * src, const int * idx, int n, int E) {
    const int r = blockIdx.y, i = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < n && 4 * i < E)
        reinterpret_cast<float4 *>(dst + (size_t) idx[r] * E)[i] = reinterpret_cast<const float4 *>(src + (size_t) r * E)[i];
}

// [T, sel[0 .. T k), -1 ...] (1 + tmax k ints): this rank's part of the exchanged selections.
static __global__ void k_pack_sel(int * out, const int * sel, int T, int k, int tmax) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < 1 + tmax * k; i += gridDim.x * blockDim.x)
        out[i] = i == 0 ? T : i - 1 < T * k ? sel[i - 1] : -1;
}

static bool nck(ncclResult_t r, const char * what) {
    if (r == ncclSuccess) return true;
    snprintf(g_err, sizeof g_err, "%s: %s", what, nccl_api()->error(r));
    return false;
}

// Rows between ranks: rank d gets cnt_out[d] rows from out + off_out[d] and
// this rank gets cnt_in[d] rows from d into in + off_in[d] (rows of `width`
// floats); this rank's own share is a device copy.
static bool a2a_rows(sb_moe * h, const float * out, const std::vector<int> & cnt_out, const std::vector<int> & off_out,
                     float * in, const std::vector<int> & cnt_in, const std::vector<int> & off_in, int width,
                     cudaStream_t st) {
    const NcclApi * api = nccl_api();
    const int me = h->rank;
    if (cnt_out[me] &&
        !ck(cudaMemcpyAsync(in + (size_t) off_in[me] * width, out + (size_t) off_out[me] * width,
                            (size_t) cnt_out[me] * width * 4, cudaMemcpyDeviceToDevice, st), "own rows"))
        return false;
    if (!nck(api->group_start(), "ncclGroupStart")) return false;
    bool ok = true;
    for (int d = 0; d < h->world && ok; d++) {
        if (d == me) continue;
        if (cnt_out[d])
            ok = nck(api->send(out + (size_t) off_out[d] * width, (size_t) cnt_out[d] * width, ncclFloat, d, h->comm, st),
                     "ncclSend");
        if (ok && cnt_in[d])
            ok = nck(api->recv(in + (size_t) off_in[d] * width, (size_t) cnt_in[d] * width, ncclFloat, d, h->comm, st),
                     "ncclRecv");
    }
    return nck(api->group_end(), "ncclGroupEnd") && ok;
}

// One step of the layer with expert parallelism by all-to-all: this rank's own
// T rows routed here; every rank's choices exchanged (an all-gather), the rows
// sent to the ranks holding their experts, the experts run over the rows this
// rank received, the results sent back and combined in choice order. The host
// plans between the exchanges, so the call synchronizes with the device.
static bool a2a_forward(sb_moe * h, const float * x, int T, float * y, cudaStream_t st) {
    const MoeLayer & m = h->m;
    const int W = h->world, k = m.k, E = m.E, nt = 8;
    const size_t nk = (size_t) h->tmax * k, per = 1 + nk;
    if (!ck(moe_router_launch(m, h->s, x, T, nullptr, 0.0f, nt, 0, 0, st, false, h->err, nullptr, 0, h->xtab,
                              h->xnear), "moe.router"))
        return false;
    k_pack_sel<<<8, 256, 0, st>>>(h->selpk, h->s.r.sel, T, k, h->tmax);
    if (!ck(cudaGetLastError(), "pack") ||
        !nck(nccl_api()->all_gather(h->selpk, h->selall, per, ncclInt32, h->comm, st), "ncclAllGather") ||
        !ck(cudaMemcpyAsync(h->h_selall, h->selall, per * W * 4, cudaMemcpyDeviceToHost, st), "selections") ||
        !ck(cudaStreamSynchronize(st), "selections"))
        return false;
    std::vector<int> n_tok(W);
    std::vector<const int *> sel(W);
    for (int r = 0; r < W; r++) {
        n_tok[r] = h->h_selall[per * r];
        sel[r] = h->h_selall + per * r + 1;
        if (n_tok[r] < 0 || n_tok[r] > h->tmax) { snprintf(g_err, sizeof g_err, "rank %d sent %d rows", r, n_tok[r]); return false; }
    }
    MoeA2aPlan & p = h->plan;
    if (!moe_a2a_plan(W, h->rank, m.ne, k, nt, n_tok.data(), sel.data(), p)) {
        snprintf(g_err, sizeof g_err, "an exchanged choice names no expert");
        return false;
    }
    // the plan's arrays, staged in one copy
    const int ns = (int) p.send_tok.size(), nr = (int) p.recv_exp.size(), nch = (int) p.ch_e.size();
    int * hp = h->h_plan;
    int * send_tok = hp, * send_slot = hp + nk, * slots = hp + 2 * nk, * ch_e = slots + nk * W;
    int * ch_s0 = ch_e + nk * W, * ch_n = ch_s0 + nk * W, * meta = ch_n + nk * W;
    memcpy(send_tok, p.send_tok.data(), (size_t) ns * 4);
    memcpy(send_slot, p.send_slot.data(), (size_t) ns * 4);
    memcpy(slots, p.slots.data(), (size_t) nr * 4);
    memcpy(ch_e, p.ch_e.data(), (size_t) nch * 4);
    memcpy(ch_s0, p.ch_s0.data(), (size_t) nch * 4);
    memcpy(ch_n, p.ch_n.data(), (size_t) nch * 4);
    meta[0] = nch;
    meta[1] = p.distinct;
    int * dp = h->d_plan;
    if (!ck(cudaMemcpyAsync(dp, hp, a2a_plan_ints(h) * 4, cudaMemcpyHostToDevice, st), "plan")) return false;
    // dispatch: this rank's rows to the ranks holding their experts
    if (ns) {
        k_gather_rows<<<dim3((E / 4 + 127) / 128, ns), 128, 0, st>>>(h->sendbuf, x, dp, ns, E);
        if (!ck(cudaGetLastError(), "gather")) return false;
    }
    if (!a2a_rows(h, h->sendbuf, p.send_cnt, p.send_off, h->recvbuf, p.recv_cnt, p.recv_off, E, st)) return false;
    // this rank's experts over the rows it received (row = slot)
    if (nch) {
        MoeGArgs g;
        memset(&g, 0, sizeof g);
        g.slots = dp + 2 * nk; g.ch_e = g.slots + nk * W; g.ch_s0 = g.ch_e + nk * W; g.ch_n = g.ch_s0 + nk * W;
        g.meta = g.ch_n + nk * W;
        g.err = h->err;
        MoeGArgs a = g;
        a.t = m.gu; a.tiles = m.gu_tiles; a.perm = m.gu_perm; a.scatter = m.dn_iperm;
        a.in = h->recvbuf; a.in_stride = E; a.in_div = 1;
        a.out = h->hp2; a.out_stride = m.F; a.ffn_f = m.F;
        a.nstage = moe_stages(m.gu, nt);
        if (!ck(moe_gemv(MG_GU, nt, a, h->nsm, st, false), "moe.gate_up")) return false;
        a = g;
        a.t = m.dn; a.tiles = m.dn_tiles;
        a.in = h->hp2; a.in_stride = m.F; a.in_div = 1;
        a.out = h->yrecv; a.out_stride = E;
        a.nstage = moe_stages(m.dn, nt);
        if (!ck(moe_gemv(MG_DN, nt, a, h->nsm, st, false), "moe.down")) return false;
    }
    // combine: the results back to the tokens' ranks, into their slots, summed in choice order
    if (!a2a_rows(h, h->yrecv, p.recv_cnt, p.recv_off, h->yback, p.send_cnt, p.send_off, E, st)) return false;
    if (ns) {
        k_scatter_rows<<<dim3((E / 4 + 127) / 128, ns), 128, 0, st>>>(h->s.yk, h->yback, dp + nk, ns, E);
        if (!ck(cudaGetLastError(), "scatter")) return false;
    }
    return ck(moe_comb_launch(m, h->s, T, y, 0, st, false), "moe.combine") &&
           ck(cudaMemcpyAsync(h->s.r.meta, dp + 2 * nk + 4 * nk * W, 8, cudaMemcpyHostToDevice, st), "meta");
}

static bool enqueue(sb_moe * h, const float * x, int T, float * y, cudaStream_t st) {
    if (h->a2a) return a2a_forward(h, x, T, y, st);
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

extern "C" int sb_moe_a2a_plan(int world, int rank, int n_expert, int k, const int * n_tok, const int * sel,
                               int * send_cnt, int * recv_cnt, int * send_slot, int * recv_expert) {
    if (world < 1 || rank < 0 || rank >= world || n_expert < world || k < 1 || !n_tok || !sel) return -1;
    std::vector<const int *> rows(world);
    for (int r = 0, off = 0; r < world; r++) {
        if (n_tok[r] < 0) return -1;
        rows[r] = sel + off;
        off += n_tok[r] * k;
    }
    MoeA2aPlan p;
    if (!moe_a2a_plan(world, rank, n_expert, k, 8, n_tok, rows.data(), p)) return -1;
    for (int r = 0; r < world; r++) {
        if (send_cnt) send_cnt[r] = p.send_cnt[r];
        if (recv_cnt) recv_cnt[r] = p.recv_cnt[r];
    }
    if (send_slot) memcpy(send_slot, p.send_slot.data(), p.send_slot.size() * 4);
    if (recv_expert) memcpy(recv_expert, p.recv_exp.data(), p.recv_exp.size() * 4);
    return (int) p.ch_e.size();
}

extern "C" int sb_moe_set_exchange(sb_moe * h, int mode) {
    g_err[0] = 0;
    if (!h || mode < 0 || mode > 1 || (mode == 1 && h->world < 2)) {
        snprintf(g_err, sizeof g_err, "exchange %d: 0 (all-reduce) or 1 (all-to-all, expert-parallel handles)", mode);
        return 0;
    }
    h->a2a = mode;
    return 1;
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
