// RL weight-sync kernels (multicast broadcast fused with cast + re-layout).
#include "common.cuh"
#include "comm.h"
