// Host view of the batched tensor-core path (tc_batch.cu).
#pragma once

#include "qgemv.cuh"
#include "tc.cuh"

namespace sb {

// One tensor re-quantized for the tensor cores: A blocks of 32 KB per (128
// rows, 256 columns) in the core-matrix layout, and s8[sb][rows_pad].
struct TcPlan {
    uint8_t * wblk = nullptr;
    float * s8 = nullptr;
    int rows_pad = 0, nsb = 0;
};

struct TcArgs {
    const uint8_t * wblk;
    const float * s8;
    const uint8_t * xblk;     // B blocks of N x 256 per (N tokens, superblock)
    const float * xs;         // [sb][T_pad] activation scales
    float * y;                // y[t * ldy + r]
    const float * bias;       // per row, or NULL
    int accumulate;           // y += product (else y = product + bias)
    int ldy;
    int rows, rows_pad, nsb, T, T_pad;
    int split;                // slices of the superblocks (tc_split), 1..kTcMaxSplit
    int * err;
};

enum TcQuantMode { TQ_PLAIN = 0, TQ_NORM = 1, TQ_SILU = 2 };

// Rows of x into the B operand: x[t * ldx + perm[i]] (TQ_PLAIN), RMS-normalized
// with gain (TQ_NORM), or silu(x[t][perm i]) * x[t][up_off + perm i] (TQ_SILU).
struct TcQuantArgs {
    const float * x;
    int ldx, up_off;
    const int32_t * perm;
    const float * gain;
    float eps;
    int cols, T, T_pad, N, nsb;
    uint8_t * xblk;
    float * xs;
};

// Re-quantize t into rows [row_off, row_off + t.rows) of p (p allocated by the
// caller: rows_pad x nsb x 256 bytes, nsb x rows_pad floats; row_off a multiple of 128).
cudaError_t tc_requant(const QT & t, const TcPlan & p, int row_off, cudaStream_t st);
// Tokens per CTA for T rows of x (16, 32 or 64) and T rounded up to it. x
// blocks need T_pad x nsb x 256 bytes and nsb x T_pad scales.
int tc_tile_n(int T);
int tc_tokens_pad(int T);
cudaError_t tc_quant(int mode, const TcQuantArgs & a, cudaStream_t st);
// The number of non-empty slices when nsb superblocks are cut into `split`
// equal runs (a launch's split must be a value this returns, at most
// kTcMaxSplit: a tile's slices form one cluster whose partial tiles fit in the
// leader's shared memory).
constexpr int kTcMaxSplit = 7;
int tc_split(int nsb, int split);
cudaError_t tc_mma(const TcArgs & a, cudaStream_t st);
// y[T][rows] = W x[t] for x[T][cols] (device pointers): tc_quant + tc_mma.
cudaError_t tc_gemm(const QT & t, const TcPlan & p, const float * x, int T, uint8_t * xblk, float * xs, float * y,
                    int * err, cudaStream_t st);

}  // namespace sb
