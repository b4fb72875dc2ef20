// A tensor set: every flat tensor of an SSF file on the device, addressable by
// name, for kernel-level entry points (GEMV microbench, parity tests, MoE
// layer). The decode engine holds its own copy in its own arena.
#include "moe_host.h"
#include "tc_batch.h"
#include "tgemv.cuh"
#include "sheep_b200.h"
#include "upload.h"

#include <cstdio>
#include <string>
#include <unordered_map>
#include <vector>

using namespace sb;

// A tiled tensor with one-entry tile and column-order tables: the form the
// grouped GEMV (moe.cuh, PLAIN mode) takes for a batch of vectors.
struct TTB {
    TT t;
    const uint8_t * const * tiles_tab;
    const int32_t * const * perm_tab;
};

constexpr int kMaxBatch = 4096;

struct sb_tset {
    ssf_file f{};
    Arena ar;
    std::unordered_map<std::string, QT> q;    // file layout (row dequant)
    std::unordered_map<std::string, TTB> tt;  // tiled (GEMV)
    std::unordered_map<std::string, const float *> f32;
    int * err = nullptr;
    // batch plan: identity slots, chunks of 8 vectors of the one "expert"
    int * slots = nullptr, * ch_e = nullptr, * ch_s0 = nullptr, * ch_n = nullptr, * meta = nullptr;
    // tensor-core batched path: per-tensor int8 re-quantization, made on first use
    std::unordered_map<std::string, TcPlan> tc;
    uint8_t * tc_x = nullptr;
    float * tc_xs = nullptr;
    size_t tc_x_cap = 0, tc_xs_cap = 0;
    int nsm = 148;
};

static bool tset_build(sb_tset * t, char * why, int nwhy) {
    t->q.clear();
    t->tt.clear();
    t->f32.clear();
    for (uint64_t i = 0; i < t->f.hdr->n_tensors; i++) {
        const ssf_rec * r = &t->f.recs[i];
        const std::string nm(r->name, strnlen(r->name, SSF_NAME_LEN));
        if (r->kind == SSF_KIND_F32) { t->f32[nm] = upload_f32(t->ar, t->f, r); continue; }
        if (r->layout != SSF_LAYOUT_FLAT) continue;
        QT qt;
        if (!upload_qt(t->ar, t->f, r, qt, why, nwhy)) return false;
        t->q[nm] = qt;
        TTB tb;
        if (!upload_tt(t->ar, t->f, r, (int) r->rows, 0, 6 * t->nsm, 0,
                       [&](int v) { return RowSrc{v < (int) r->rows ? r : nullptr, v}; }, tb.t, why, nwhy))
            return false;
        tb.tiles_tab = (const uint8_t * const *) t->ar.upload(&tb.t.tiles, sizeof(void *));
        tb.perm_tab = (const int32_t * const *) t->ar.upload(&tb.t.perm, sizeof(void *));
        t->tt[nm] = tb;
    }
    t->err = (int *) t->ar.carve(4);
    std::vector<int> ident(kMaxBatch);
    for (int i = 0; i < kMaxBatch; i++) ident[i] = i;
    t->slots = (int *) t->ar.upload(ident.data(), ident.size() * 4);
    const int nch = kMaxBatch / 8;
    t->ch_e = (int *) t->ar.carve((size_t) nch * 4);
    t->ch_s0 = (int *) t->ar.carve((size_t) nch * 4);
    t->ch_n = (int *) t->ar.carve((size_t) nch * 4);
    t->meta = (int *) t->ar.carve(8);
    return true;
}

extern "C" sb_tset * sb_tset_open(const char * path, char * why, int nwhy) {
    sb_tset * t = new sb_tset();
    if (!ssf_open(&t->f, path, why, nwhy)) { delete t; return nullptr; }
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&t->nsm, cudaDevAttrMultiProcessorCount, dev);
    if (!tset_build(t, why, nwhy) || !t->ar.allocate() || !tset_build(t, why, nwhy)) {
        if (!why[0]) snprintf(why, nwhy, "device allocation failed");
        t->ar.release();
        ssf_close(&t->f);
        delete t;
        return nullptr;
    }
    cudaDeviceSynchronize();
    return t;
}

extern "C" void sb_tset_close(sb_tset * t) {
    if (!t) return;
    cudaDeviceSynchronize();
    for (auto & kv : t->tc) { cudaFree(kv.second.wblk); cudaFree(kv.second.s8); }
    cudaFree(t->tc_x);
    cudaFree(t->tc_xs);
    t->ar.release();
    ssf_close(&t->f);
    delete t;
}

static const QT * find_qt(const sb_tset * t, const char * name) {
    auto it = t->q.find(name);
    return it == t->q.end() ? nullptr : &it->second;
}

extern "C" int sb_tset_shape(const sb_tset * t, const char * name, int * rows, int * cols, int * nbits) {
    const QT * q = find_qt(t, name);
    if (!q) return 0;
    if (rows) *rows = q->rows;
    if (cols) *cols = q->cols;
    if (nbits) *nbits = q->nbits;
    return 1;
}

extern "C" unsigned long long sb_tset_bytes(const sb_tset * t, const char * name) {
    const QT * q = find_qt(t, name);
    return q ? (unsigned long long) qt_row_bytes(*q) * (unsigned long long) q->rows : 0ull;
}

template <int NB, int SIX>
static void launch_plain(const TGArgs & g0, int grid, size_t smem, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_tgemv<NB, SIX>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kSmemBudget);
        attr = true;
    }
    TGArgs g = g0;
    g.mode = GM_PLAIN;
    k_tgemv<NB, SIX><<<grid, kTgThreads, smem, st>>>(g);
}

static const TTB * find_ttb(const sb_tset * t, const char * name) {
    auto it = t->tt.find(name);
    return it == t->tt.end() ? nullptr : &it->second;
}
static const TT * find_tt(const sb_tset * t, const char * name) {
    const TTB * b = find_ttb(t, name);
    return b ? &b->t : nullptr;
}

static TGArgs plain_args(const sb_tset * t, const TT & tt, const float * x, float * y) {
    TGArgs g;
    memset(&g, 0, sizeof g);
    g.t = tt;
    g.in = x;
    g.out = y;
    g.err = t->err;
    return g;
}

static bool run_plain(const sb_tset * t, const TGArgs & g0, cudaStream_t st) {
    TGArgs g = g0;
    if (!tg_plan(g)) return false;
    long grid = g.t.ntiles;
    if (grid > t->nsm) grid = t->nsm;
    SB_DISPATCH_QT(g.t.nbits, g.t.six, launch_plain, g, (int) grid, tg_smem(g), st);
    return true;
}

// The chunks of a batch of nb vectors: ceil(nb / nt) chunks of the one tensor.
static __global__ void k_batch_plan(int nb, int nt, int * ch_e, int * ch_s0, int * ch_n, int * meta) {
    const int nch = (nb + nt - 1) / nt;
    for (int c = threadIdx.x; c < nch; c += blockDim.x) {
        ch_e[c] = 0;
        ch_s0[c] = nt * c;
        ch_n[c] = nb - nt * c < nt ? nb - nt * c : nt;
    }
    if (threadIdx.x == 0) { meta[0] = nch; meta[1] = 1; }
}

// y[b] = W x[b] for nb > 1 vectors: the weights are read once per 8 vectors
// (per 4 for rows so wide that eight staged vectors leave no room for the
// ring), or once per vector if even that does not fit.
static bool run_batch(const sb_tset * t, const TTB & b, const float * x, int nb, float * y, cudaStream_t st) {
    const int nt = moe_stages(b.t, 8) ? 8 : moe_stages(b.t, 4) ? 4 : 0;
    if (!nt) {
        for (int i = 0; i < nb; i++)
            if (!run_plain(t, plain_args(t, b.t, x + (size_t) i * b.t.cols, y + (size_t) i * b.t.rows), st)) return false;
        return true;
    }
    k_batch_plan<<<1, 128, 0, st>>>(nb, nt, t->ch_e, t->ch_s0, t->ch_n, t->meta);
    MoeGArgs g;
    memset(&g, 0, sizeof g);
    g.t = b.t; g.tiles = b.tiles_tab; g.perm = b.perm_tab;
    g.in = x; g.in_stride = b.t.cols; g.in_div = 1;
    g.out = y; g.out_stride = b.t.rows;
    g.slots = t->slots; g.ch_e = t->ch_e; g.ch_s0 = t->ch_s0; g.ch_n = t->ch_n; g.meta = t->meta;
    g.nstage = moe_stages(b.t, nt);
    g.err = t->err;
    return moe_gemv(MG_PLAIN, nt, g, t->nsm, st, false) == cudaSuccess;
}

// y[b] = W x[b] for nb vectors on device pointers (x: nb x cols, y: nb x rows):
// one vector through the streaming GEMV, more through the batched one.
extern "C" int sb_tset_gemv_dev(sb_tset * t, const char * name, const float * x, int nb, float * y, void * stream) {
    const TTB * b = find_ttb(t, name);
    if (!b || nb < 1 || nb > kMaxBatch) return 0;
    const cudaStream_t st = (cudaStream_t) stream;
    const bool ok = nb == 1 ? run_plain(t, plain_args(t, b->t, x, y), st) : run_batch(t, *b, x, nb, y, st);
    return ok && cudaGetLastError() == cudaSuccess;
}

// The same with host buffers (copies included, synchronous).
extern "C" int sb_tset_gemv_host(sb_tset * t, const char * name, const float * x, int nb, float * y) {
    const TTB * b = find_ttb(t, name);
    if (!b || nb < 1 || nb > kMaxBatch) return 0;
    float * dx = nullptr, * dy = nullptr;
    bool ok = cudaMalloc(&dx, (size_t) nb * b->t.cols * 4) == cudaSuccess &&
              cudaMalloc(&dy, (size_t) nb * b->t.rows * 4) == cudaSuccess;
    int err = 0;
    if (ok) {
        cudaMemcpy(dx, x, (size_t) nb * b->t.cols * 4, cudaMemcpyHostToDevice);
        ok = sb_tset_gemv_dev(t, name, dx, nb, dy, nullptr) && cudaDeviceSynchronize() == cudaSuccess;
        cudaMemcpy(&err, t->err, 4, cudaMemcpyDeviceToHost);
        ok = ok && err == 0;
        if (ok) cudaMemcpy(y, dy, (size_t) nb * b->t.rows * 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(dx);
    cudaFree(dy);
    return ok ? 1 : 0;
}

// Mean device time of sb_tset_gemv_dev over nb host vectors (copied once),
// a buffer larger than L2 rewritten before each timed run so the weights come
// from HBM: CUDA events around each run.
extern "C" int sb_tset_time_gemv(sb_tset * t, const char * name, const float * x, int nb, int reps, float * ms_avg) {
    const TTB * b = find_ttb(t, name);
    if (!b || nb < 1 || nb > kMaxBatch || reps < 1) return 0;
    float * dx = nullptr, * dy = nullptr;
    void * flush = nullptr;
    const size_t flush_n = (size_t) 512 << 20;
    cudaStream_t st = nullptr;
    bool ok = cudaMalloc(&dx, (size_t) nb * b->t.cols * 4) == cudaSuccess &&
              cudaMalloc(&dy, (size_t) nb * b->t.rows * 4) == cudaSuccess &&
              cudaMalloc(&flush, flush_n) == cudaSuccess && cudaStreamCreate(&st) == cudaSuccess;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    double total = 0.0;
    if (ok) {
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaMemcpy(dx, x, (size_t) nb * b->t.cols * 4, cudaMemcpyHostToDevice);
        for (int r = 0; ok && r < 3; r++) ok = sb_tset_gemv_dev(t, name, dx, nb, dy, st);
        for (int r = 0; ok && r < reps; r++) {
            cudaMemsetAsync(flush, r & 0xff, flush_n, st);
            cudaEventRecord(e0, st);
            ok = sb_tset_gemv_dev(t, name, dx, nb, dy, st);
            cudaEventRecord(e1, st);
            ok = ok && cudaEventSynchronize(e1) == cudaSuccess;
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, e0, e1);
            total += ms;
        }
        int err = 0;
        cudaMemcpy(&err, t->err, 4, cudaMemcpyDeviceToHost);
        ok = ok && err == 0;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (st) cudaStreamDestroy(st);
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(flush);
    if (ms_avg) *ms_avg = (float) (total / reps);
    return ok ? 1 : 0;
}

// Host-buffer form for tests: y = W x, plus the int8 activation the kernel
// quantized (natural group order) when q/s/sums are not NULL.
static int matvec_host(sb_tset * t, const char * name, const float * x, int permuted, float * y, int8_t * qx,
                       float * qs, int32_t * qsum);

extern "C" int sb_tset_matvec(sb_tset * t, const char * name, const float * x, float * y, int8_t * qx, float * qs,
                              int32_t * qsum) {
    return matvec_host(t, name, x, 0, y, qx, qs, qsum);
}

// The same with x already in the tensor's column order (the staging the
// decode chain's down projection uses: no gather, one lane per group).
extern "C" int sb_tset_matvec_permuted(sb_tset * t, const char * name, const float * xp, float * y, int8_t * qx,
                                       float * qs, int32_t * qsum) {
    return matvec_host(t, name, xp, 1, y, qx, qs, qsum);
}

static int matvec_host(sb_tset * t, const char * name, const float * x, int permuted, float * y, int8_t * qx,
                       float * qs, int32_t * qsum) {
    const TT * q = find_tt(t, name);
    if (!q) return 0;
    const int n = q->cols, ng = n / SSF_GROUP;
    float * dx = nullptr, * dy = nullptr, * ds = nullptr;
    int8_t * dq = nullptr;
    int32_t * dsum = nullptr;
    bool ok = cudaMalloc(&dx, (size_t) n * 4) == cudaSuccess && cudaMalloc(&dy, (size_t) q->rows * 4) == cudaSuccess &&
              cudaMalloc(&dq, (size_t) n) == cudaSuccess && cudaMalloc(&ds, (size_t) ng * 4) == cudaSuccess &&
              cudaMalloc(&dsum, (size_t) ng * 4) == cudaSuccess;
    if (ok) {
        cudaMemcpy(dx, x, (size_t) n * 4, cudaMemcpyHostToDevice);
        TGArgs g = plain_args(t, *q, dx, dy);
        g.act_q = dq; g.act_s = ds; g.act_sum = dsum;
        g.in_permuted = permuted;
        ok = run_plain(t, g, (cudaStream_t) 0);
        int err = 0;
        ok = cudaDeviceSynchronize() == cudaSuccess && ok;
        cudaMemcpy(&err, t->err, 4, cudaMemcpyDeviceToHost);
        ok = ok && err == 0;
        if (ok) {
            cudaMemcpy(y, dy, (size_t) q->rows * 4, cudaMemcpyDeviceToHost);
            if (qx) cudaMemcpy(qx, dq, (size_t) n, cudaMemcpyDeviceToHost);
            if (qs) cudaMemcpy(qs, ds, (size_t) ng * 4, cudaMemcpyDeviceToHost);
            if (qsum) cudaMemcpy(qsum, dsum, (size_t) ng * 4, cudaMemcpyDeviceToHost);
        }
    }
    cudaFree(dx); cudaFree(dy); cudaFree(dq); cudaFree(ds); cudaFree(dsum);
    return ok ? 1 : 0;
}

template <int NB, int SIX>
static void launch_deq(const QT & q, const int * rows, int nrows, float * out) {
    k_dequant_rows<NB, SIX><<<dim3((q.cols + 255) / 256, nrows), 256>>>(q, rows, nrows, out);
}

// Rows of a tensor dequantized on the GPU (permuted column order), host buffers.
extern "C" int sb_tset_dequant_rows(sb_tset * t, const char * name, const int * rows, int nrows, float * out) {
    const QT * q = find_qt(t, name);
    if (!q || nrows < 1) return 0;
    for (int i = 0; i < nrows; i++) if (rows[i] < 0 || rows[i] >= q->rows) return 0;
    int * dr = nullptr;
    float * dout = nullptr;
    bool ok = cudaMalloc(&dr, (size_t) nrows * 4) == cudaSuccess &&
              cudaMalloc(&dout, (size_t) nrows * q->cols * 4) == cudaSuccess;
    if (ok) {
        cudaMemcpy(dr, rows, (size_t) nrows * 4, cudaMemcpyHostToDevice);
        SB_DISPATCH_QT(q->nbits, q->six, launch_deq, *q, dr, nrows, dout);
        ok = cudaDeviceSynchronize() == cudaSuccess;
        if (ok) cudaMemcpy(out, dout, (size_t) nrows * q->cols * 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(dr);
    cudaFree(dout);
    return ok ? 1 : 0;
}

// sml_gather + sml_quantize_act on the device (device pointers, perm may be NULL).
extern "C" int sb_quantize_act(const float * x, const int32_t * perm, int n, int8_t * q, float * s, int32_t * sums,
                               void * stream) {
    if (n <= 0 || n % SSF_GROUP) return 0;
    const int ng = n / SSF_GROUP;
    k_quant_act<<<(ng + 7) / 8, 256, 0, (cudaStream_t) stream>>>(x, perm, n, q, s, sums);
    return cudaGetLastError() == cudaSuccess;
}

// ------------------------------------------------------------------ tensor-core batched path

// The tensor's re-quantized form (made and kept on first use).
static const TcPlan * tc_plan(sb_tset * t, const char * name, const QT ** qo) {
    const QT * q = find_qt(t, name);
    if (!q) return nullptr;
    *qo = q;
    auto it = t->tc.find(name);
    if (it != t->tc.end()) return &it->second;
    TcPlan p;
    p.nsb = (q->cols / SSF_GROUP + 7) / 8;
    p.rows_pad = (q->rows + 127) / 128 * 128;
    if (cudaMalloc(&p.wblk, (size_t) p.rows_pad * p.nsb * 256) != cudaSuccess) return nullptr;
    if (cudaMalloc(&p.s8, (size_t) p.nsb * p.rows_pad * 4) != cudaSuccess) { cudaFree(p.wblk); return nullptr; }
    if (tc_requant(*q, p, 0, nullptr) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(p.wblk);
        cudaFree(p.s8);
        return nullptr;
    }
    return &t->tc.emplace(name, p).first->second;
}

// Grow a device buffer to at least n bytes (zeroed when grown; frees synchronize).
template <typename P>
static bool grow(P *& buf, size_t & cap, size_t n) {
    if (n <= cap) return true;
    cudaFree(buf);
    buf = nullptr;
    cap = 0;
    if (cudaMalloc(&buf, n) != cudaSuccess || cudaMemset(buf, 0, n) != cudaSuccess) return false;
    cap = n;
    return true;
}

// Scratch for the activations of T rows and the partial sums of `split` slices.
static bool tc_scratch(sb_tset * t, const TcPlan & p, int T, int split) {
    const int N = tc_tile_n(T), T_pad = tc_tokens_pad(T);
    (void) split;
    (void) N;
    return grow(t->tc_x, t->tc_x_cap, (size_t) T_pad * p.nsb * 256) &&
           grow(t->tc_xs, t->tc_xs_cap, (size_t) T_pad * p.nsb * 4);
}

extern "C" int sb_tset_gemm_tc(sb_tset * t, const char * name, const float * x, int nb, int split, float * y,
                               void * stream) {
    const QT * q = nullptr;
    if (!t || nb < 1 || nb > kMaxBatch || split < 1) return 0;
    const TcPlan * p = tc_plan(t, name, &q);
    if (!p || split != tc_split(p->nsb, split) || !tc_scratch(t, *p, nb, split)) return 0;
    const cudaStream_t st = (cudaStream_t) stream;
    TcQuantArgs qa;
    memset(&qa, 0, sizeof qa);
    qa.x = x; qa.ldx = q->cols; qa.perm = q->perm; qa.cols = q->cols; qa.T = nb; qa.T_pad = tc_tokens_pad(nb);
    qa.N = tc_tile_n(nb); qa.nsb = p->nsb; qa.xblk = t->tc_x; qa.xs = t->tc_xs;
    if (tc_quant(TQ_PLAIN, qa, st) != cudaSuccess) return 0;
    TcArgs a;
    memset(&a, 0, sizeof a);
    a.wblk = p->wblk; a.s8 = p->s8; a.xblk = t->tc_x; a.xs = t->tc_xs; a.y = y; a.ldy = q->rows;
    a.rows = q->rows; a.rows_pad = p->rows_pad; a.nsb = p->nsb; a.T = nb; a.T_pad = qa.T_pad; a.err = t->err;
    a.split = split;
    return tc_mma(a, st) == cudaSuccess;
}

extern "C" int sb_tset_gemm_tc_host(sb_tset * t, const char * name, const float * x, int nb, int split, float * y) {
    const QT * q = find_qt(t, name);
    if (!q || nb < 1 || nb > kMaxBatch) return 0;
    float * dx = nullptr, * dy = nullptr;
    bool ok = cudaMalloc(&dx, (size_t) nb * q->cols * 4) == cudaSuccess &&
              cudaMalloc(&dy, (size_t) nb * q->rows * 4) == cudaSuccess;
    int err = 0;
    if (ok) {
        cudaMemcpy(dx, x, (size_t) nb * q->cols * 4, cudaMemcpyHostToDevice);
        ok = sb_tset_gemm_tc(t, name, dx, nb, split, dy, nullptr) && cudaDeviceSynchronize() == cudaSuccess;
        cudaMemcpy(&err, t->err, 4, cudaMemcpyDeviceToHost);
        ok = ok && err == 0;
        if (ok) cudaMemcpy(y, dy, (size_t) nb * q->rows * 4, cudaMemcpyDeviceToHost);
    }
    cudaFree(dx);
    cudaFree(dy);
    return ok ? 1 : 0;
}

// Mean device time of sb_tset_gemm_tc (activation quantization + product; the
// weights' re-quantization, made once, is not timed) over nb host rows copied
// once, a buffer larger than L2 rewritten before each run.
extern "C" int sb_tset_time_gemm_tc(sb_tset * t, const char * name, const float * x, int nb, int split, int reps,
                                    float * ms_avg) {
    const QT * q = find_qt(t, name);
    if (!q || nb < 1 || nb > kMaxBatch || reps < 1) return 0;
    float * dx = nullptr, * dy = nullptr;
    void * flush = nullptr;
    const size_t flush_n = (size_t) 512 << 20;
    cudaStream_t st = nullptr;
    bool ok = cudaMalloc(&dx, (size_t) nb * q->cols * 4) == cudaSuccess &&
              cudaMalloc(&dy, (size_t) nb * q->rows * 4) == cudaSuccess &&
              cudaMalloc(&flush, flush_n) == cudaSuccess && cudaStreamCreate(&st) == cudaSuccess;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    double total = 0.0;
    if (ok) {
        cudaEventCreate(&e0);
        cudaEventCreate(&e1);
        cudaMemcpy(dx, x, (size_t) nb * q->cols * 4, cudaMemcpyHostToDevice);
        for (int r = 0; ok && r < 3; r++) ok = sb_tset_gemm_tc(t, name, dx, nb, split, dy, st);
        for (int r = 0; ok && r < reps; r++) {
            cudaMemsetAsync(flush, r & 0xff, flush_n, st);
            cudaEventRecord(e0, st);
            ok = sb_tset_gemm_tc(t, name, dx, nb, split, dy, st);
            cudaEventRecord(e1, st);
            ok = ok && cudaEventSynchronize(e1) == cudaSuccess;
            float ms = 0.0f;
            cudaEventElapsedTime(&ms, e0, e1);
            total += ms;
        }
        int err = 0;
        cudaMemcpy(&err, t->err, 4, cudaMemcpyDeviceToHost);
        ok = ok && err == 0;
    }
    if (e0) cudaEventDestroy(e0);
    if (e1) cudaEventDestroy(e1);
    if (st) cudaStreamDestroy(st);
    cudaFree(dx);
    cudaFree(dy);
    cudaFree(flush);
    if (ms_avg) *ms_avg = (float) (total / reps);
    return ok ? 1 : 0;
}

// The re-quantized weights in natural layout (host): w8 rows x (nsb * 256), s8 rows x nsb.
extern "C" int sb_tset_requant8_host(sb_tset * t, const char * name, int8_t * w8, float * s8) {
    const QT * q = nullptr;
    const TcPlan * p = tc_plan(t, name, &q);
    if (!p) return 0;
    const int nsb = p->nsb, K = nsb * 256;
    std::vector<uint8_t> blk((size_t) p->rows_pad * nsb * 256);
    std::vector<float> sc((size_t) nsb * p->rows_pad);
    if (cudaMemcpy(blk.data(), p->wblk, blk.size(), cudaMemcpyDeviceToHost) != cudaSuccess ||
        cudaMemcpy(sc.data(), p->s8, sc.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
        return 0;
    for (int r = 0; r < q->rows; r++)
        for (int sb = 0; sb < nsb; sb++) {
            s8[(size_t) r * nsb + sb] = sc[(size_t) sb * p->rows_pad + r];
            const uint8_t * b = blk.data() + ((size_t) (r >> 7) * nsb + sb) * 32768;
            for (int k = 0; k < 256; k++) w8[(size_t) r * K + sb * 256 + k] = (int8_t) b[tc_off(128, r & 127, k)];
        }
    return 1;
}
