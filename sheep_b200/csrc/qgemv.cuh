// Quantized GEMV building blocks: the device view of an SSF flat tensor, the
// int8 activation as the kernels stage it in shared memory, activation
// quantization, and the per-row dot product for every flat width Q2..Q8.
//
// Arithmetic (the reference's, sml/sml-kernel.c:2027-2066 flat4, :1934-1983
// 2-bit planes, :1986-2005 bit planes, :2007-2018 Q8):
//
//   y[r] = sum_g  d[r,g/8]*sq[r,g] * xs[g] * dot(code[r,g,:], xq[g,:])
//               + md[r,g/8]*(mq[r,g] - bias) * xs[g] * sum(xq[g,:])
//
// with xq, xs, sums the per-32 int8 activation of sml_quantize_act
// (sml/sml-kernel.c:89-109). The integer dots are exact (dp4a); the float
// epilogue's order is the reference's in the decode GEMV (tgemv.cuh) and per
// unit in the batched GEMV (moe.cuh).
//
// Work unit: one lane takes 64 weights of a row -- groups 4p..4p+3, columns
// c0..c0+15 (c0 = 0 or 16) -- which is 2 x 16 bytes of the nibble plane,
// 16 bytes of a 2-bit plane, or 8 bytes of a bit plane, all 16-byte aligned.
#pragma once

#include "common.cuh"

namespace sb {

// Device view of one flat tensor. Planes and fields are the file's row-major
// arrays, uploaded as they are (each on its own 256-byte-aligned allocation).
struct QT {
    const uint8_t * pl[3];        // code planes in file order
    const uint16_t * sd;          // [rows][nsb] fp16 step scale
    const uint16_t * md;          // [rows][nsb] fp16 min scale
    const uint8_t * sq;           // [rows][frow] step fields
    const uint8_t * mq;           // [rows][frow] min fields
    const int32_t * perm;         // [cols] input gather
    const int32_t * iperm;        // [cols] inverse of perm
    int rows, cols, nbits, six, has_min, frow, nsb;
    float mbias;                  // 127 (8-bit), 31 (6-bit), 63 (6-bit MINNEG)
};

// Bytes of one row of every plane and field: the algorithmic bytes the GEMV
// streams per row.
__host__ __device__ inline size_t qt_row_bytes(const QT & t) {
    size_t b = 0;
    const int n = t.cols;
    switch (t.nbits) {
    case 2: b = n / 4; break;
    case 3: b = n / 4 + n / 8; break;
    case 4: b = n / 2; break;
    case 5: b = n / 2 + n / 8; break;
    case 6: b = n / 4 + n / 2; break;
    case 7: b = n / 2 + n / 4 + n / 8; break;
    case 8: b = n; break;
    }
    return b + (size_t) t.frow * (t.has_min ? 2 : 1) + (size_t) t.nsb * 2 * (t.has_min ? 2 : 1);
}

// ---------------------------------------------------------------- activation

// The int8 activation in shared memory, in the order the lanes read it: slot
// k (0..3) of unit u holds group 4*(u/2)+k, columns 16*(u%2)..+15, at byte
// k*(n/4) + 16u. One 16-byte load per slot, consecutive lanes on consecutive
// 16-byte words: no bank conflicts.
struct ActS {
    int8_t * q;        // n bytes, slot layout
    float * xs;        // [ng] group scale
    float * xsum;      // [ng] group scale * sum of the group's codes
    int n;
};

SB_DEV int act_slot_off(int n, int g, int j) {
    return (g & 3) * (n >> 2) + 16 * (2 * (g >> 2) + (j >> 4)) + (j & 15);
}

// Widths and field sizes as one switch, so every kernel instantiates all 14.
#define SB_DISPATCH_QT(nbits, six, FN, ...)                                        \
    do {                                                                           \
        switch ((nbits) * 2 + ((six) ? 1 : 0)) {                                   \
        case 4: FN<2, 0>(__VA_ARGS__); break;  case 5: FN<2, 1>(__VA_ARGS__); break; \
        case 6: FN<3, 0>(__VA_ARGS__); break;  case 7: FN<3, 1>(__VA_ARGS__); break; \
        case 8: FN<4, 0>(__VA_ARGS__); break;  case 9: FN<4, 1>(__VA_ARGS__); break; \
        case 10: FN<5, 0>(__VA_ARGS__); break; case 11: FN<5, 1>(__VA_ARGS__); break; \
        case 12: FN<6, 0>(__VA_ARGS__); break; case 13: FN<6, 1>(__VA_ARGS__); break; \
        case 14: FN<7, 0>(__VA_ARGS__); break; case 15: FN<7, 1>(__VA_ARGS__); break; \
        case 16: FN<8, 0>(__VA_ARGS__); break; case 17: FN<8, 1>(__VA_ARGS__); break; \
        default: break;                                                            \
        }                                                                          \
    } while (0)

}  // namespace sb
