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
    float * y;                // [T][rows]
    int rows, rows_pad, nsb, T, T_pad;
    int * err;
};

// Fill p (allocated by the caller: rows_pad x nsb x 256 bytes, nsb x rows_pad floats).
cudaError_t tc_requant(const QT & t, const TcPlan & p, cudaStream_t st);
// Tokens per CTA for T rows of x (16, 32 or 64); x blocks need T_pad x nsb x 256
// bytes and nsb x T_pad scales, T_pad = T rounded up to a multiple of it.
int tc_tile_n(int T);
// y[T][rows] = W x[t] for x[T][cols] (device pointers).
cudaError_t tc_gemm(const QT & t, const TcPlan & p, const float * x, int T, uint8_t * xblk, float * xs, float * y,
                    int * err, cudaStream_t st);

}  // namespace sb
