// Expert-parallel MoE kernels (dispatch / grouped GEMM / combine).
#include "common.cuh"
#include "moe.h"
