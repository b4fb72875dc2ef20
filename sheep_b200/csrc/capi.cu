// The reference's C API (sml/sml-gpu.h) over one process-wide engine.
//
// Error behaviour follows sml/sml-gpu-fwd.c:2353-2434: open returns 1, or 0
// with a reason; prefill and step return NULL on any failure, including a
// position past n_ctx; nothing exits the process.
#include "sheep_b200.h"
#include "sml-gpu.h"
#include "ssf.h"

#include <cstdio>
#include <cstdlib>
#include <cuda_runtime.h>

static sb_engine * g_eng = nullptr;
static int g_prompt_level = 2;

extern "C" int sml_gpu_open(const char * path, int n_ctx, int threads, int gpu_layers, char * why, int nwhy) {
    (void) threads;
    (void) gpu_layers;
    if (g_eng) { sb_close(g_eng); g_eng = nullptr; }
    if (n_ctx <= 0) {
        const char * e = getenv("SML_CTX");
        n_ctx = e ? atoi(e) : 256;
    }
    if (n_ctx < 64) n_ctx = 64;
    char buf[256] = {0};
    g_eng = sb_open(path, n_ctx, buf, (int) sizeof buf);
    if (!g_eng) {
        if (why && nwhy > 0) snprintf(why, (size_t) nwhy, "%s", buf[0] ? buf : "this model cannot use the GPU path");
        return 0;
    }
    sb_set_prompt_mode(g_eng, g_prompt_level);
    return 1;
}

extern "C" const float * sml_gpu_prefill(const int * ids, int pos0, int n) {
    if (!g_eng) return nullptr;
    return sb_prefill(g_eng, ids, pos0, n);
}

extern "C" const float * sml_gpu_step(int tok, int pos) {
    if (!g_eng) return nullptr;
    return sb_step(g_eng, tok, pos);
}

extern "C" int sml_gpu_layers(int * of) {
    int info[16] = {0};
    if (g_eng) sb_info(g_eng, info);
    if (of) *of = info[0];
    return info[0];
}

// sml/sml-gpu-fwd.c:2420-2423: level >= 1 lets prompts be read in batches,
// >= 2 on the tensor cores. Here levels 0 and 1 step the prompt a token at a
// time through the decode path (exact: it writes what reading a token at a
// time writes); level 2, the default as in the reference, reads all but the
// last token in tensor-core chunks (the batched arithmetic).
extern "C" void sml_gpu_prompt_mode(int level) {
    g_prompt_level = level;
    if (g_eng) sb_set_prompt_mode(g_eng, level);
}

extern "C" int sml_gpu_decode_cpu(int on) {
    (void) on;
    return 0;
}

extern "C" void sml_gpu_set_middle(int layers, int (*fn)(float * rows, int pos0, int n)) {
    (void) layers;
    (void) fn;
}

// The process-wide engine behind the reference API, for callers that mix the
// two surfaces (the CLI, the bench's end-to-end leg).
extern "C" sb_engine * sml_gpu_engine(void) { return g_eng; }

extern "C" void sml_gpu_close(void) {
    if (g_eng) sb_close(g_eng);
    g_eng = nullptr;
}

// Open and validate an SSF file without a GPU (the loader's checks alone).
// Returns 1, or 0 with the reason in why.
extern "C" int sb_ssf_check(const char * path, char * why, int nwhy) {
    ssf_file f;
    if (!ssf_open(&f, path, why, nwhy)) return 0;
    ssf_close(&f);
    return 1;
}
