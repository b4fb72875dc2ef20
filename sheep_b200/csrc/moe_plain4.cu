// Grouped GEMV kernels: MG_PLAIN, 4-vector chunks (wide rows), every flat width.
#include "moe_launch.cuh"

SB_MOE_INST(sb::MG_PLAIN, 4)
