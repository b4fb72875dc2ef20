// Definition of the grouped-GEMV launcher, included by the files that
// instantiate it (one per mode and chunk size, compiled in parallel).
#pragma once

#include "moe.cuh"

namespace sb {

template <int MODE, int NB, int SIX, int NT>
cudaError_t moe_gemv_launch(const MoeGArgs & g, int grid, size_t smem, cudaStream_t st, bool pdl) {
    static bool attr = false;
    if (!attr) {
        const cudaError_t e = cudaFuncSetAttribute(k_moe_gemv<MODE, NB, SIX, NT>,
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, (int) kSmemBudget);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kTgThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, k_moe_gemv<MODE, NB, SIX, NT>, g);
}

}  // namespace sb

#define SB_MOE_INST(MODE, NT)                                                                                 \
    namespace sb {                                                                                            \
    template cudaError_t moe_gemv_launch<MODE, 2, 0, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 2, 1, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 3, 0, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 3, 1, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 4, 0, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 4, 1, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 5, 0, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 5, 1, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 6, 0, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 6, 1, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 7, 0, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 7, 1, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 8, 0, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    template cudaError_t moe_gemv_launch<MODE, 8, 1, NT>(const MoeGArgs &, int, size_t, cudaStream_t, bool); \
    }
