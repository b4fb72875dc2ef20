// libsheep_b200.so: the B200 decode engine's C ABI beyond the reference's
// sml-gpu.h. Plain pointers and sizes only. "device" arguments are CUDA device
// pointers on the current device; "host" arguments are host memory.
#pragma once

#include <stdint.h>

#include "sml-gpu.h"

#ifdef __cplusplus
extern "C" {
#endif

// ------------------------------------------------------------------ engine
// A handle form of the sml-gpu.h API (several models per process, explicit
// n_ctx). Replaces the reference's gpu_setup / gpu_forward / graph_token
// (sml/sml-gpu-fwd.c:1789, :1643, :636).
typedef struct sb_engine sb_engine;

sb_engine * sb_open(const char * path, int n_ctx, char * why, int nwhy);
void        sb_close(sb_engine * e);

// Tensor-parallel decode over tp GPUs of one node, one process per GPU (the
// reference is single-device, cuDeviceGet(&dev, 0) at sml/sml-gpu-fwd.c:1877;
// this is the row-split GEMV with an exchange north of it): attention, q|k|v
// and o replicated on every rank; gate/up, down and the head split by rows;
// each GEMV stores its rows into every rank's copy of the vector over NVLink
// and raises a flag the consuming kernel waits on. A mixture-of-experts layer's
// experts are spread over the ranks ([ne r / tp, ne (r + 1) / tp) on rank r):
// the router runs on every rank, each runs the chosen experts it holds and its
// expert down GEMV stores every row into all ranks' per-choice buffer the same
// way; the combine, in choice order, waits for them. Results equal one GPU's bit
// for bit. Open on every rank (the current device is the rank's GPU), pass
// each rank's handle to every rank (rank order), then connect; every rank must
// then make the same calls in the same order (steps, prefill, generation).
#define SB_TP_HANDLE_BYTES 64
sb_engine * sb_open_tp(const char * path, int n_ctx, int tp, int rank, char * why, int nwhy);
int         sb_tp_handle(const sb_engine * e, void * out);   // SB_TP_HANDLE_BYTES of this rank's exchange region
int         sb_tp_connect(sb_engine * e, const void * handles, char * why, int nwhy);
// out[0..12]: n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, n_vocab,
// n_ctx, n_expert, n_expert_used, weight bytes per token (low, high 32 bits),
// 0 (reserved)
void        sb_info(const sb_engine * e, int * out);
uint64_t    sb_bytes_per_token(const sb_engine * e);
// sml/sml-gpu.h:17 semantics on a handle: logits in host memory, NULL on failure.
const float * sb_step(sb_engine * e, int tok, int pos);
// sml/sml-gpu.h:14 semantics on a handle. The prompt mode (sml_gpu_prompt_mode's
// levels, sml/sml-gpu-fwd.c:2420) decides how: 0 or 1 (the handle's default 0)
// step every token through the decode path; 2 reads all but the last in
// chunks of 64 on the tensor cores (int8 re-quantized weights made on first
// use, per-256 activations; attention the decode kernel's), then steps the last.
const float * sb_prefill(sb_engine * e, const int * ids, int pos0, int n);
int sb_set_prompt_mode(sb_engine * e, int level);   // returns the level set (0..2)
// The cached key and value rows of (layer, pos) (n_head_kv * head_dim fp16
// each), for checks; and the superblock slices of the tensor-core prompt
// products (q|k|v, o, gate|up, down, and 1 for the unused head).
int sb_kv_rows(const sb_engine * e, int layer, int pos, uint16_t * k, uint16_t * v);
int sb_prompt_splits(sb_engine * e, int * out5);
// Greedy decode with the choice made on the device (the reference's
// graph-replay benchmark loop, sml/sml-gpu-fwd.c:2626-2662): host prompt in,
// ngen host ids out. Returns 1, or 0 on failure.
int sb_generate(sb_engine * e, const int * prompt, int np, int ngen, int * out_ids);
// The same after nwarm untimed tokens: out_ids gets nwarm + ngen ids, ms_out
// the CUDA-event time of the generation loop after the warm-up. Each of the
// ngen tokens replays the token graph once; the first is chosen by the last
// warm-up (or prompt) replay, so ngen ids cost ngen - 1 timed replays.
int sb_generate_timed(sb_engine * e, const int * prompt, int np, int nwarm, int ngen, int * out_ids,
                      float * ms_out);
const float * sb_device_logits(const sb_engine * e);
int sb_launches_per_token(const sb_engine * e);
// Average duration (ms) of one kernel class of the token, each launch alone,
// timed by CUDA events, layers cycled so weights come from HBM; bytes_out =
// the weight bytes one launch reads. which: 0 q|k|v, 2 o, 3 gate/up, 4 down,
// 5 head. Leaves the decode state undefined (call after generating).
int sb_time_kernel(sb_engine * e, int which, int reps, float * ms_avg, double * bytes_out);
// Trace build only (-DSB_TRACE): per-CTA timestamps of the last token.
int sb_trace(const sb_engine * e, unsigned long long * out, int cap);
const char * sb_last_error(void);
// The engine behind sml_gpu_open, and its release.
sb_engine * sml_gpu_engine(void);
void sml_gpu_close(void);

// ------------------------------------------------------------------ tensors
// Every flat tensor of an SSF file on the device, by name. Kernel-level entry
// points over it replace the reference's per-kernel GPU bench and check
// drivers (sml/sml-gpu-bench.c:99-157, sml/sml-check.c:166-283).
typedef struct sb_tset sb_tset;

sb_tset * sb_tset_open(const char * path, char * why, int nwhy);
void      sb_tset_close(sb_tset * t);
int       sb_tset_shape(const sb_tset * t, const char * name, int * rows, int * cols, int * nbits);
// Weight bytes of the tensor (codes + fields): the bytes one GEMV streams.
unsigned long long sb_tset_bytes(const sb_tset * t, const char * name);
// y[b] = W x[b], nb vectors, device pointers (x nb x cols, y nb x rows),
// activation gathered through the tensor's perm and quantized per 32 inside.
// Replaces sml_g_mv3s / sml_g_qdmv2 (sml/sml-gpu-fast.cu:267-315).
// nb = 1 runs the streaming GEMV; nb > 1 (up to 4096) the batched one, which
// reads the weights once per 8 vectors.
int sb_tset_gemv_dev(sb_tset * t, const char * name, const float * x, int nb, float * y, void * stream);
// The same with host buffers (copies included, synchronous).
int sb_tset_gemv_host(sb_tset * t, const char * name, const float * x, int nb, float * y);
// Mean device time (CUDA events) of one sb_tset_gemv_dev over nb host vectors
// copied to the device once, a buffer larger than L2 rewritten before each run.
int sb_tset_time_gemv(sb_tset * t, const char * name, const float * x, int nb, int reps, float * ms_avg);
// The batched path on the tensor cores, with the reference's batched
// arithmetic (sml_g_requant8 + the int8 tiles, sml/sml-gpu-fast.cu:1804-1880,
// 2025-2031): the weights re-quantized once to int8 with one scale per row per
// 256 (kept on the device), x quantized per 256, int32 superblock dots from
// tcgen05, one float epilogue per superblock. Device pointers, nb <= 4096.
// split > 1 cuts the superblocks into that many equal runs whose sums are added
// in run order (the reference's split-K, sml_g_tcm3 + sml_g_splitk_sum,
// sml/sml-gpu-fast.cu:1907-2065); split must leave no run empty
// (ceil(nsb / ceil(nsb / split)) == split), else the call fails.
int sb_tset_gemm_tc(sb_tset * t, const char * name, const float * x, int nb, int split, float * y, void * stream);
int sb_tset_gemm_tc_host(sb_tset * t, const char * name, const float * x, int nb, int split, float * y);
int sb_tset_time_gemm_tc(sb_tset * t, const char * name, const float * x, int nb, int split, int reps, float * ms_avg);
// The re-quantized weights, host buffers: w8 rows x (nsb*256), s8 rows x nsb (nsb = ceil(cols/256)).
int sb_tset_requant8_host(sb_tset * t, const char * name, int8_t * w8, float * s8);
// Host-buffer form of one GEMV; q/s/sums (host, may be NULL) receive the int8
// activation the kernel used. Mirrors what sml-check writes
// (sml/sml-check.c:194-245).
int sb_tset_matvec(sb_tset * t, const char * name, const float * x, float * y, int8_t * q, float * s,
                   int32_t * sums);
// sb_tset_matvec with xp already in the tensor's column order (xp[i] =
// x[perm[i]]): the staging of the decode chain's down projection, whose input
// the gate/up epilogue writes in that order. The exported int8 activation is
// the per-32 quantization of xp.
int sb_tset_matvec_permuted(sb_tset * t, const char * name, const float * xp, float * y, int8_t * q, float * s,
                            int32_t * sums);
// Rows dequantized on the GPU, permuted column order (sml_dequant_row_flat*,
// sml/sml-kernel.c:2134-2260; the embedding path sml_g_embed,
// sml/sml-gpu-fast.cu:461). Host buffers.
int sb_tset_dequant_rows(sb_tset * t, const char * name, const int * rows, int nrows, float * out);

// sml_gather + sml_quantize_act (sml/sml-kernel.c:41, :253) on device
// pointers: q natural order (n bytes), s and sums per 32. perm may be NULL.
int sb_quantize_act(const float * x, const int32_t * perm, int n, int8_t * q, float * s, int32_t * sums,
                    void * stream);

// ------------------------------------------------------------------ attention
// One decode step of attention (the decode graph's k_attn kernel), device
// pointers: qkv = this token's [q (n_head*hd) | k (n_kv*hd) | v (n_kv*hd)]
// before RoPE; kc, vc = fp16 caches [n_ctx][n_kv*hd] (positions < pos are read,
// the token's roped key and its value are written at pos); rope_cos, rope_sin
// = [n_ctx][hd/2] tables; q_norm, k_norm = per-head RMS gains (hd) or NULL;
// out = [n_head*hd]. The chunk partials live in scratch the call allocates and
// frees. Synchronizes the stream; returns 1, or 0 (sb_attn_last_error()).
// Replaces the sml_g_attn2 launch (sml/sml-gpu-fwd.c:346-356; the kernel
// sml/sml-gpu-fast.cu:363-453).
int sb_attn_decode(const float * qkv, uint16_t * kc, uint16_t * vc, const float * rope_cos, const float * rope_sin,
                   const float * q_norm, const float * k_norm, float eps, int n_head, int n_head_kv, int head_dim,
                   int n_ctx, int pos, float scale, float * out, void * stream);
const char * sb_attn_last_error(void);
// sb_attn_decode for callers that cannot allocate device memory (a host that
// owns every allocation up front, or one that must not synchronize the device
// mid-stream): same arguments and results, but the chunk partials live in a
// static device array of 1 MiB (+ 256 counters) that every GPU loading the
// library holds until exit, and nothing is allocated. Rejects, with an error,
// calls needing more (n_head x chunks x (head_dim + 2) floats > 1 MiB, or > 256
// heads). All calls on one device share that device's array: calls that
// overlap on the GPU race. The first call on a device finds the array's address
// and clears the counters (synchronizing once), so make it before any stream
// capture, and do not reset the device afterwards. Asynchronous on `stream`.
// The error text is per calling thread. No counterpart in the reference: an
// addition of this library.
int sb_attn_decode_noalloc(const float * qkv, uint16_t * kc, uint16_t * vc, const float * rope_cos,
                           const float * rope_sin, const float * q_norm, const float * k_norm, float eps, int n_head,
                           int n_head_kv, int head_dim, int n_ctx, int pos, float scale, float * out, void * stream);
const char * sb_attn_noalloc_last_error(void);

// ------------------------------------------------------------------ MoE FFN
// One mixture-of-experts FFN layer of an SSF file on the current device:
// router (fp32, double accumulation), top-k routing with ties to the lower
// index and softmax weights (renormalized over the chosen experts when
// moe_flags bit 0 is set), each chosen expert's SwiGLU FFN, and the weighted
// sum in choice order -- per row, what moe_ffn does (sml/sml-run.c:3071-3125;
// on the reference's GPU moe_ffn_dev, sml/sml-gpu-fwd.c:492-546). Rows are
// the FFN's input (already normalized). Refused with a reason: routing other
// than flags 0/1, shared experts, an expert bias, scaled weights.
typedef struct sb_moe sb_moe;
sb_moe * sb_moe_open(const char * path, int layer, int max_tokens, char * why, int nwhy);
// Expert parallelism over `world` GPUs (one process each): every process calls
// sb_moe_open_ep with the same 128-byte NCCL id (made by one of them with
// sb_nccl_unique_id and shared by the host); this one holds experts
// [rank*ne/world, (rank+1)*ne/world). Every process passes all tokens; the
// router runs everywhere, each GPU runs the expert FFNs of the choices it holds,
// the per-choice outputs are summed over the GPUs (NCCL all-reduce; each row is
// one GPU's, zeros elsewhere, so the sum is exact) and combined in choice order
// on every GPU: y equals the single-GPU layer's bit for bit. NCCL is loaded at
// run time (libnccl.so.2); without it these return 0 / NULL with the reason.
sb_moe * sb_moe_open_ep(const char * path, int layer, int max_tokens, int world, int rank, const void * nccl_id,
                        char * why, int nwhy);
int sb_nccl_unique_id(void * id128);
// How an expert-parallel handle exchanges rows: 0 (the default) the all-reduce
// above; 1 all-to-all (the dispatch / combine of a token-sharded deployment):
// every process passes ITS OWN tokens (up to max_tokens, the same max_tokens on
// every process), routes them, and the processes exchange their choices (an
// all-gather), send each (token, choice) row to the GPU holding its expert
// (grouped ncclSend / ncclRecv), run their experts over the rows they received,
// send the results back and combine them in choice order: each process's y
// equals the single-GPU layer's rows for its tokens bit for bit. The host plans
// between the exchanges, so a call returns with the device synchronized.
// Returns 0 for a single-GPU handle.
int sb_moe_set_exchange(sb_moe * m, int mode);
// The all-to-all exchange's plan for one rank (host only; no GPU needed): from
// every rank's chosen experts (n_tok[world]; sel: the ranks' [n_tok[r]][k]
// choices concatenated) the rows this rank sends to and receives from each
// rank (send_cnt, recv_cnt [world]), the slot (token * k + choice) of each row
// it sends, grouped by destination in slot order (send_slot), and the expert of
// each row it receives, grouped by source (recv_expert). Any output may be
// NULL. Returns the chunks of at most 8 rows its experts run, -1 on bad input.
int sb_moe_a2a_plan(int world, int rank, int n_expert, int k, const int * n_tok, const int * sel, int * send_cnt,
                    int * recv_cnt, int * send_slot, int * recv_expert);
void sb_moe_close(sb_moe * m);
// out[14]: n_embd, expert hidden size, experts, experts per token, flags,
// max_tokens, expert width in bits, bytes of one expert as stored (low, high),
// router bytes, GPUs, rank, first and one-past-last expert held here.
void sb_moe_info(const sb_moe * m, int * out);
// y[n_tok][n_embd] from x[n_tok][n_embd], device pointers, asynchronous on
// `stream`. Calls on one handle must not overlap (they share its scratch).
int sb_moe_forward(sb_moe * m, const float * x, int n_tok, float * y, void * stream);
// The same with host rows (copies included, synchronous); sel and w
// (n_tok x k: chosen experts and weights) and n_active (distinct experts)
// may be NULL.
int sb_moe_forward_host(sb_moe * m, const float * x, int n_tok, float * y, int * sel, float * w, int * n_active);
// Mean device time (CUDA events) of one forward over rows already on the
// device, with a buffer larger than L2 rewritten before each timed run.
int sb_moe_time(sb_moe * m, const float * x_host, int n_tok, int reps, float * ms_avg, int * n_active);
// Which calls run the expert products on the tensor cores (tcgen05
// kind::f16: the experts' four-bit codes decoded to fp16 in shared memory,
// rows in fp16, fp32 sums; within about 1e-3 of the decode arithmetic):
// on = 1 every call of 16 or more rows, 0 none, 2 (the default) those whose
// chosen rows are at least 8 per expert on average (n_tok * k >= 8 * n_expert),
// where they are faster than the integer kernels. Fewer than 16 rows, and
// experts that are not four-bit codes with 8-bit group fields, always take the
// integer kernels. Returns 1 if the handle can use the tensor-core path
// (max_tokens >= 16 and suitable experts), else 0.
int sb_moe_set_tensor_cores(sb_moe * m, int on);
// Routing alone, device pointers: logits[n_tok][n_expert] -> sel, w
// [n_tok][k] (sml_moe_route, sml/sml-run.c:2925, for moe_flags 0 and 1).
int sb_moe_route(const float * logits, int n_tok, int n_expert, int k, unsigned flags, int * sel, float * w,
                 void * stream);
const char * sb_moe_last_error(void);

// ------------------------------------------------------------------ tensor cores
// C[M][N] (int32) = A[M][K] * B[N][K]^T on the 5th-generation tensor cores
// (tcgen05.mma kind::i8, accumulator in tensor memory): A and B signed 8-bit,
// row-major; M a multiple of 128, N one of 16/32/64/128/256, K a multiple of
// 32; device pointers, 16-byte aligned. *err (device) receives a code if a
// bounded wait gave up. Asynchronous on `stream`. The integer core of the
// batched path (the reference's int8 tiles, sml_g_tcm9, sml/sml-gpu-fast.cu:3149).
int sb_tc_imma(const int8_t * A, const int8_t * B, int32_t * C, int M, int N, int K, int * err, void * stream);
const char * sb_tc_last_error(void);
// Global-timer marks of the last batched tensor-core product, per CTA (8 words:
// start, first accumulator read, main loop done, slices added, stored, exit);
// filled only by the trace build (-DSB_TRACE), else returns 0.
int sb_tc_trace(unsigned long long * out, int cap_ctas);

// ------------------------------------------------------------------ batched serving
// n_seq conversations decoding together, one token each per step and one read
// of the weights per step: the GPU form of sml_forward_multi
// (sml/sml-run.c:2559-2604), driven like sml-batched (sml/sml-batched.c:43-146).
// Every product runs on the tensor cores with the batched arithmetic of
// sb_tset_gemm_tc; attention, norms, RoPE and the greedy choice are each
// sequence's own, over its own fp16 KV cache of n_ctx positions. Dense
// decoders only (an MoE file is refused with the reason in `why`).
typedef struct sb_batch sb_batch;
sb_batch * sb_batch_open(const char * path, int n_seq, int n_ctx, char * why, int nwhy);
void sb_batch_close(sb_batch * b);
// out (int[16]): [0] n_seq [1] n_ctx [2] n_vocab [3..7] superblock slices of
// the q|k|v, o, gate|up, down and head products [8,9] the file's weight bytes
// per step (lo, hi 32 bits) [10,11] the int8 weight bytes per step [12] kernel
// launches per step [13] tokens per tensor-core tile [14,15] every MoE
// layer's experts and router as stored (lo, hi 32 bits; 0 for a dense model;
// the gate|up and down splits read 0 when layer 0 is a MoE layer).
void sb_batch_info(const sb_batch * b, int * out);
// One token per slot: tokens[s] at absolute position pos[s] (pos[s] < 0 idles
// slot s: its logits are not meaningful). Host arrays of n_seq. Returns a host
// pointer to [n_seq][n_vocab] logits owned by the library, NULL on failure
// (positions >= n_ctx or ids out of range included). Replaces the reference's
// sml_forward_multi(cs, tokens, pos, ns, depth, logits_out).
const float * sb_forward_multi(sb_batch * b, const int * tokens, const int * pos);
// Greedy generation on the device: prompts [n_seq][np] stepped from position
// 0, then nwarm + ngen tokens per slot, each chosen on the GPU and fed back by
// graph replay; ids [n_seq][nwarm + ngen]. ms (if not NULL) receives the device
// time of the last ngen - 1 steps. np + nwarm + ngen - 1 <= n_ctx.
int sb_batch_generate(sb_batch * b, const int * prompts, int np, int nwarm, int ngen, int * ids, float * ms);
const float * sb_batch_device_logits(const sb_batch * b);
// The cached key and value rows of `slot` at `pos` in `layer`: n_kv * head_dim
// fp16 each (head-major), host buffers.
int sb_batch_kv(const sb_batch * b, int layer, int slot, int pos, uint16_t * k, uint16_t * v);
const char * sb_batch_last_error(void);

// Continuous batching over a paged KV cache. The reference's
// sml_forward_multi (sml/sml-run.c:2559-2604) takes one context per sequence
// (cs[b], each owning its cache and positions) for whichever conversations a
// step runs; sml-server's slots (sml/sml-server.c:1300-1330) pick the context a
// request continues. Here a sequence is the context: its cache lives in pages
// of 64 positions taken from one pool (n_pages per layer) as its positions
// reach them, and a step runs up to n_slots live sequences in any slots, so a
// sequence can join or leave between any two steps without moving its cache.
// The arithmetic per slot is sb_forward_multi's: a sequence's logits do not
// depend on its slot, its pages or the other sequences of the step.
sb_batch * sb_batch_open_paged(const char * path, int n_slots, int n_ctx, int n_pages, char * why, int nwhy);
// A new, empty sequence (its id), or -1. Ids of freed sequences are reused.
int sb_seq_new(sb_batch * b);
// Give every page of the sequence back to the pool; the id becomes free.
int sb_seq_free(sb_batch * b, int seq);
// Keep positions 0 .. n - 1 of the sequence; pages past them go back to the pool.
int sb_seq_truncate(sb_batch * b, int seq, int n);
// One step: slot s (s < ns <= n_slots) runs sequence seqs[s] with tokens[s] at
// absolute position pos[s] (continuing what the sequence holds); slots past ns
// idle. Pages the positions reach are taken from the pool first; a step whose
// sequences need more pages than are free fails without changing anything.
// Returns a host pointer to [ns][n_vocab] logits owned by the library, NULL on
// failure (a sequence not live or in two slots, ids or positions out of range).
const float * sb_forward_seqs(sb_batch * b, const int * seqs, const int * tokens, const int * pos, int ns);
// out (int[4]): pages in the pool, free pages, live sequences, n_ctx.
void sb_batch_pages(const sb_batch * b, int * out);
// The cached key and value rows of a sequence at `pos` in `layer` (as sb_batch_kv).
int sb_seq_kv(const sb_batch * b, int layer, int seq, int pos, uint16_t * k, uint16_t * v);

// ------------------------------------------------------------------ models
// Seeded synthetic SSF writer (the inputs every test and bench runs on; the
// reference builds SSF files offline, tooling/sml_quantize.py:596-651).
typedef struct {
    uint32_t n_layer, n_embd, n_head, n_head_kv, head_dim, n_ff, n_vocab;
    float    rope_theta, rms_eps;
    uint32_t tied, qkv_bias, qk_norm;
    uint32_t nbits, emb_nbits;
    uint32_t scale6, minneg;
    uint32_t n_expert, n_expert_used, moe_flags, expert_ff;
    uint32_t perm_mode;
    uint64_t seed;
    float    sigma;
    int      threads;
    // 0: every weight drawn N(0, sigma) and quantized; 1: quantized tensors'
    // group ranges and codes drawn directly from the seed (same layout and
    // value scale, several times faster); 2: as 1, but the MoE experts' bytes
    // are not written (the file is sparse there): an engine opened after
    // sb_draw_experts(seed) draws them on the device. For the ~130 GB
    // configuration, whose experts are 97 % of its bytes.
    uint32_t direct;
} ssfgen_spec;

int ssfgen_write(const char * path, const ssfgen_spec * s, char * why, int nwhy);

// Engines opened after this call (sb_open, sb_open_tp) fill their MoE experts'
// tiles on the device from `seed` instead of reading them from the file: for
// files written with direct = 2, which leave those bytes out. Code and field
// bytes uniform, superblock scales fixed (weights within about +-2 sigma); the
// tiles have the size and layout the file's experts would give. 0 restores
// reading from the file. A benchmark facility: such weights match no file.
void sb_draw_experts(uint64_t seed);

// The loader's validation alone, no GPU needed: 1, or 0 with the reason
// (the acceptance rules of sml/sml-model.c:24-75 and :174-260, v8+ files).
int sb_ssf_check(const char * path, char * why, int nwhy);

#ifdef __cplusplus
}
#endif
