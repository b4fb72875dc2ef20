// Decode attention for callers that cannot allocate device memory.
//
// Some callers of this library may not call cudaMalloc: a host that owns every
// device allocation up front and forbids allocation afterwards (a server with a
// fixed memory budget, an embedded pipeline), or one that enqueues work where an
// allocation would synchronize the device. sb_attn_decode allocates its chunk
// partials on every call; this variant takes them from a file-scope device
// array instead and calls no allocating routine.
//
// The array is kScratchBytes (1 MiB of partials plus 1 KiB of counters); every
// GPU that loads the library holds it until the process exits. Calls needing
// more -- n_head x chunks x (head_dim + 2) floats above 1 MiB (for example 32
// heads of 128 at positions past 4031), or more than 256 heads -- are rejected
// with an error. All calls share the one array, so calls that overlap
// on the GPU (other streams, other threads) race and give wrong results: issue
// them one after another on one stream.
//
// "Shared" means per device: each GPU has its own copy of the array, so calls
// on different devices do not race on it.
//
// In host code the array's name is not a device address; the address comes from
// cudaGetSymbolAddress once per device, with that device current. The first call
// on a device does that set-up and clears the counters (a cudaMemset, which
// synchronizes), so make the first call before any stream capture. The kernel
// leaves the counters at zero when it finishes, and the partials are written
// before they are read, so later calls need no clearing. The address and the
// cleared counters are kept for the life of the process: do not reset the
// device (cudaDeviceReset) after the first call -- a new context would hold a
// new copy of the array that this file has neither looked up nor cleared.
#include "decode.cuh"
#include "sheep_b200.h"

#include <cstdio>
#include <mutex>

using namespace sb;

namespace {

constexpr size_t kPartBytes = (size_t) 1 << 20;
constexpr int kMaxHeads = 256;
constexpr size_t kScratchBytes = kPartBytes + kMaxHeads * sizeof(unsigned);
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_attn_scratch[kScratchBytes];

std::mutex g_setup;
void * g_addr[kMaxDevices];
thread_local char g_err[256];   // per calling thread, as sb_attn_last_error

// The array's device address on the current device (set up on first use).
bool scratch_address(void ** out) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        snprintf(g_err, sizeof g_err, "no usable current device (%s)", cudaGetErrorString(e));
        return false;
    }
    std::lock_guard<std::mutex> lock(g_setup);
    if (!g_addr[dev]) {
        void * p = nullptr;
        e = cudaGetSymbolAddress(&p, g_attn_scratch);
        if (e != cudaSuccess || !p) {
            snprintf(g_err, sizeof g_err, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
            return false;
        }
        e = cudaMemset((char *) p + kPartBytes, 0, kMaxHeads * sizeof(unsigned));
        if (e != cudaSuccess) {
            snprintf(g_err, sizeof g_err, "clearing the counters: %s", cudaGetErrorString(e));
            return false;
        }
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return true;
}

}  // namespace

extern "C" const char * sb_attn_noalloc_last_error(void) { return g_err; }

extern "C" int sb_attn_decode_noalloc(const float * qkv, uint16_t * kc, uint16_t * vc, const float * rope_cos,
                                      const float * rope_sin, const float * q_norm, const float * k_norm, float eps,
                                      int n_head, int n_head_kv, int head_dim, int n_ctx, int pos, float scale,
                                      float * out, void * stream) {
    g_err[0] = 0;
    if (!qkv || !kc || !vc || !rope_cos || !rope_sin || !out || n_head <= 0 || n_head_kv <= 0 ||
        n_head % n_head_kv || head_dim <= 0 || head_dim % 8 || head_dim > 256 || n_ctx <= 0 || pos < 0 ||
        pos >= n_ctx) {
        snprintf(g_err, sizeof g_err, "invalid attention arguments");
        return 0;
    }
    AttnArgs a;
    memset(&a, 0, sizeof a);
    a.chunk = head_dim <= 128 ? 64 : 32;
    const int nchunk = pos / a.chunk + 1;
    const size_t need = (size_t) n_head * nchunk * (head_dim + 2) * sizeof(float);
    if (n_head > kMaxHeads || need > kPartBytes) {
        snprintf(g_err, sizeof g_err,
                 "needs %zu bytes of partials for %d heads: above the static scratch (%zu bytes, %d heads)",
                 need, n_head, kPartBytes, kMaxHeads);
        return 0;
    }
    void * base = nullptr;
    if (!scratch_address(&base)) return 0;
    a.qkv = qkv; a.n_head = n_head; a.n_kv = n_head_kv; a.hd = head_dim;
    a.qd = n_head * head_dim; a.kvd = n_head_kv * head_dim;
    a.qn = q_norm; a.kn = k_norm; a.eps = eps;
    a.rcos = rope_cos; a.rsin = rope_sin;
    a.kc = kc; a.vc = vc; a.n_ctx = n_ctx;
    a.pos = nullptr; a.pos_imm = pos;
    a.scale = scale;
    a.out = out;
    a.max_chunks = nchunk;
    a.part = (float *) base;
    a.cnt = (unsigned *) ((char *) base + kPartBytes);
    k_attn<<<dim3(n_head, nchunk), kAttnThreads, attn_smem_bytes(head_dim, a.chunk), (cudaStream_t) stream>>>(a);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        snprintf(g_err, sizeof g_err, "k_attn: %s", cudaGetErrorString(e));
        return 0;
    }
    return 1;
}
