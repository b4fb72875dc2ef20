// A tensor set: every flat tensor of an SSF file on the device, addressable by
// name, for kernel-level entry points (GEMV microbench, parity tests, MoE
// layer). The decode engine holds its own copy in its own arena.
#include "tgemv.cuh"
#include "sheep_b200.h"
#include "upload.h"

#include <cstdio>
#include <string>
#include <unordered_map>

using namespace sb;

struct sb_tset {
    ssf_file f{};
    Arena ar;
    std::unordered_map<std::string, QT> q;    // file layout (row dequant)
    std::unordered_map<std::string, TT> tt;   // tiled (GEMV)
    std::unordered_map<std::string, const float *> f32;
    int * err = nullptr;
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
        TT tt;
        if (!upload_tt(t->ar, t->f, r, (int) r->rows, 0, 6 * t->nsm, 0,
                       [&](int v) { return RowSrc{v < (int) r->rows ? r : nullptr, v}; }, tt, why, nwhy))
            return false;
        t->tt[nm] = tt;
    }
    t->err = (int *) t->ar.carve(4);
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
static void launch_plain(const TGArgs & g, int grid, size_t smem, cudaStream_t st) {
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(k_tgemv<GM_PLAIN, NB, SIX>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        attr = true;
    }
    k_tgemv<GM_PLAIN, NB, SIX><<<grid, kTgThreads, smem, st>>>(g);
}

static const TT * find_tt(const sb_tset * t, const char * name) {
    auto it = t->tt.find(name);
    return it == t->tt.end() ? nullptr : &it->second;
}

static TGArgs plain_args(const sb_tset * t, const TT & tt, const float * x, float * y) {
    TGArgs g;
    memset(&g, 0, sizeof g);
    g.t = tt;
    g.in = x;
    g.out = y;
    g.err = t->err;
    int ns = (int) ((96 * 1024) / tt.tb) / kConsWarps * kConsWarps;
    g.nstage = ns < kConsWarps ? kConsWarps : ns > kMaxStages ? kMaxStages : ns;
    return g;
}

static void run_plain(const sb_tset * t, const TGArgs & g, cudaStream_t st) {
    long grid = g.t.ntiles;
    if (grid > t->nsm) grid = t->nsm;
    const size_t smem = tg_ring_off(g.t.cols, g.in_permuted, g.norm_w != nullptr) + (size_t) g.nstage * g.t.tb;
    SB_DISPATCH_QT(g.t.nbits, g.t.six, launch_plain, g, (int) grid, smem, st);
}

// y[b] = W x[b] for nb vectors on device pointers (x: nb x cols, y: nb x rows).
extern "C" int sb_tset_gemv_dev(sb_tset * t, const char * name, const float * x, int nb, float * y, void * stream) {
    const TT * q = find_tt(t, name);
    if (!q || nb < 1) return 0;
    for (int b = 0; b < nb; b++)
        run_plain(t, plain_args(t, *q, x + (size_t) b * q->cols, y + (size_t) b * q->rows), (cudaStream_t) stream);
    return cudaGetLastError() == cudaSuccess;
}

// Host-buffer form for tests: y = W x, plus the int8 activation the kernel
// quantized (natural group order) when q/s/sums are not NULL.
extern "C" int sb_tset_matvec(sb_tset * t, const char * name, const float * x, float * y, int8_t * qx, float * qs,
                              int32_t * qsum) {
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
        run_plain(t, g, (cudaStream_t) 0);
        int err = 0;
        ok = cudaDeviceSynchronize() == cudaSuccess;
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
