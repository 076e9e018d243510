// kernels.cuh — launch interfaces of the smaller kernels (quantizers).
#pragma once

#include "common.cuh"

namespace sg {

constexpr int Q8K_MAXV = 64;  // vectors per quantizer launch

struct Q8kArgs {
    const float *x;
    uint64_t ldx;   // floats between consecutive vectors
    uint32_t nb;    // 256-blocks per vector
    uint32_t nvec;  // <= Q8K_MAXV
    sg_q8k outs[Q8K_MAXV];
};

__global__ void q8k_quantize_kernel(const __grid_constant__ Q8kArgs a);
__global__ void quantize_q4k_kernel(const float *x, uint64_t nblocks, uint8_t *out);
__global__ void quantize_q6k_kernel(const float *x, uint64_t nblocks, uint8_t *out);

}  // namespace sg
