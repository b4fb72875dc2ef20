// The GPU forward pass as a library: the reference's C API, same names,
// argument meaning and error behaviour, implemented on an NVIDIA B200 (sm_100a)
// by libsheep_b200.so. One model and one KV cache per process; positions are
// absolute, so a prompt may continue a prefix the cache already holds. Every
// call returns NULL (or 0) on failure instead of ending the process.
//
// Replaces, entry point by entry point, sml/sml-gpu.h:11-34 of the reference
// (implemented there by sml/sml-gpu-fwd.c:2353-2434 under -DSML_GPU_LIB).
#pragma once

#ifdef __cplusplus
extern "C" {
#endif

// sml/sml-gpu.h:11 -- load the model on the GPU. Returns 1, or 0 with the
// reason in why. n_ctx <= 0 takes SML_CTX from the environment, else 256
// (at least 64). threads and gpu_layers are accepted for signature
// compatibility: every layer runs on the GPU and nothing runs on the CPU.
int sml_gpu_open(const char * path, int n_ctx, int threads, int gpu_layers, char * why, int nwhy);

// sml/sml-gpu.h:14 -- read ids[0..n) at positions pos0..pos0+n-1; logits of
// the last one, in library-owned host memory. NULL on failure, including
// pos0 + n > n_ctx.
const float * sml_gpu_prefill(const int * ids, int pos0, int n);

// sml/sml-gpu.h:17 -- one token at position pos; its logits (host memory).
// NULL on failure, including pos >= n_ctx.
const float * sml_gpu_step(int tok, int pos);

// sml/sml-gpu.h:20 -- layers on the card, and (in *of) of how many.
int sml_gpu_layers(int * of);

// sml/sml-gpu.h:26 -- how a prompt is read (sml/sml-gpu-fwd.c:2420-2423):
// 0 and 1 step every token through the decode graph (the decode arithmetic,
// bit for bit); 2, the default, reads all but the last token in chunks of 64
// on the tensor cores (int8 re-quantized weights, per-256 activations) and
// steps the last. Applies to the open model and to later opens.
void sml_gpu_prompt_mode(int level);

// sml/sml-gpu.h:28 -- no CPU decode exists in this engine: always returns 0.
int sml_gpu_decode_cpu(int on);

// sml/sml-gpu.h:34 -- no middle device: the whole model is on the GPU, so a
// middle stage is never called.
void sml_gpu_set_middle(int layers, int (*fn)(float * rows, int pos0, int n));

#ifdef __cplusplus
}
#endif
