// Grouped expert GEMV kernels: MG_GU, 1-token chunks, every flat width.
#include "moe_launch.cuh"

SB_MOE_INST(sb::MG_GU, 1)
