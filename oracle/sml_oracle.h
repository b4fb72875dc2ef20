// TEST INFRASTRUCTURE ONLY. A plain-C restatement of the reference's decode
// path over SSF flat tensors, used by tests/ as the checker for the CUDA
// engine and pinned itself against the reference build (oracle/_ref) and the
// golden vectors in tests/golden/. Never linked into, or called by, the product.
#pragma once

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

// sml/sml-kernel.c:89-109 (scalar arm of sml_quantize_act)
void so_quantize_act(const float * x, int n, int8_t * q, float * scale, int32_t * sums);
// sml/sml-kernel.c:116-190 (sml_quantize_act_sb): one scale per 256 values
// (a partial last superblock on its own), written into each of its groups;
// codes and per-group sums as sml_quantize_act.
void so_quantize_act_sb(const float * x, int n, int8_t * q, float * scale, int32_t * sums);

typedef struct so_model so_model;

so_model * so_open(const char * path, int n_ctx);
void       so_close(so_model * m);
int        so_info(const so_model * m, int * out);   // same fields as refh_info

// y[row0..row1) of one named tensor for an activation x in natural order.
int so_matvec(so_model * m, const char * name, const float * x, float * y, int row0, int row1);
// One dequantized row (permuted column order).
int so_dequant_row(so_model * m, const char * name, int row, float * out);
// Unpacked integer codes of one row (permuted column order): bit-exact view of the planes.
int so_codes_row(so_model * m, const char * name, int row, uint8_t * out);

// Decode step: logits for token at absolute position pos (KV cache kept inside).
int so_forward(so_model * m, int tok, int pos, float * logits);
int so_decode(so_model * m, const int * prompt, int np, int ngen, int * ids, float * logits);

// sml/sml-run.c:2925-3040, the softmax-top-k branch (moe_flags bit 0 = renormalise)
int so_moe_route(const float * lg, int ne, int k, unsigned moe_flags, int * sel, float * w);
// sml/sml-run.c:3071-3125: the MoE FFN of layer L on one normalized row, with
// the chosen experts and weights (either may be NULL); returns k, 0 if layer L
// has no router.
int so_moe_ffn(so_model * m, int L, const float * xb, float * out, int * sel, float * w);
// The combine of moe_ffn (sml/sml-run.c:3120): for each of T rows, the k
// per-choice expert outputs yk [T][k][E] weighted by w [T][k] and summed in
// choice order into y [T][E] from 0, y = fma(w, yk, y).
void so_moe_combine(int T, int k, int E, const float * w, const float * yk, float * y);
// One expert's FFN output (unweighted) of layer L on a normalized row.
int so_moe_expert(so_model * m, int L, int e, const float * xb, float * out);
// The batched path: the int8 re-quantization of a tensor (w8: rows x nsb*256,
// s8: rows x nsb) and the product over T rows of X (sml_g_requant8 and the int8
// tiles' epilogue, sml/sml-gpu-fast.cu:1804-1880, 2025-2031).
int so_requant8(so_model * m, const char * name, int8_t * w8, float * s8);
int so_gemm_sb(so_model * m, const char * name, const float * X, int T, float * Y);
// The same with the superblocks cut into `split` runs summed in order (split-K).
int so_gemm_sb_split(so_model * m, const char * name, const float * X, int T, int split, float * Y);

// Batched serving (sml_forward_multi, sml/sml-run.c:2559-2604): ns sequences,
// each with its own KV cache. mode 0: each through the decode arithmetic;
// mode 1: every product with the batched path's arithmetic, superblock slices
// per kind (q|k|v, o, gate|up, down, head) from so_batch_set_splits. A step
// fills logits [ns][n_vocab] for the slots with pos >= 0 (the rest untouched)
// and returns 1, or 0 for a position or id out of range.
typedef struct so_batch so_batch;
so_batch * so_batch_open(so_model * m, int ns, int mode);
void so_batch_set_splits(so_batch * b, const int * split5);
int so_batch_step(so_batch * b, const int * tok, const int * pos, float * logits);
void so_batch_close(so_batch * b);
// Slot `slot`'s cached key and value rows at `pos` in `layer` (n_kv * hd fp16 each).
int so_batch_kv(const so_batch * b, int layer, int slot, int pos, uint16_t * k, uint16_t * v);

#ifdef __cplusplus
}
#endif
