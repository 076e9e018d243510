// q8k.cu — Q8_K activation quantizer kernel (Q8K::quantize,
// quant_q8k.rs:73-121): one warp per 256-value block, exact (q8k_block.cuh).
#include "kernels.cuh"
#include "q8k_block.cuh"

namespace sg {

__global__ void __launch_bounds__(256) q8k_quantize_kernel(const __grid_constant__ Q8kArgs a) {
    // Programmatic dependent launch: let the next kernel (the GEMV that reads
    // this output) launch now, so its weight prefetch overlaps this kernel and
    // the one before it; then wait for the kernel that wrote x.
    asm volatile("griddepcontrol.launch_dependents;" :::);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31u;
    if (warp >= a.nb * a.nvec) return;
    const uint32_t vec = warp / a.nb, b = warp % a.nb;
    const sg_q8k &o = a.outs[vec];
    q8k_block(a.x + vec * a.ldx + (uint64_t)b * 256u, o.qs + (uint64_t)b * 256u, o.bsums + b * 16u, o.d + b, lane);
}

}  // namespace sg
