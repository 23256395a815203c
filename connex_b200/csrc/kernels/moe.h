// Host entry points of the expert-parallel MoE kernels (moe.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
