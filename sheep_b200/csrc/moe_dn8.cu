// Grouped expert GEMV kernels: MG_DN, 8-token chunks, every flat width.
#include "moe_launch.cuh"

SB_MOE_INST(sb::MG_DN, 8)
