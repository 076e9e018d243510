// libm.cu — sg_libm_eval: the kernels' expf / sinf / cosf (glibc's functions,
// restated in glibc_math.h) over a strided range of float bit patterns, so a
// test can compare the device build with the host's glibc input by input.
#include "common.cuh"
#include "glibc_math.h"

namespace {

__global__ void libm_eval_kernel(int fn, uint64_t start, uint64_t stride, uint64_t count, float *out) {
    for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < count;
         i += (uint64_t)gridDim.x * blockDim.x) {
        const float x = __uint_as_float((uint32_t)(start + i * stride));
        out[i] = fn == 0 ? gm_expf(x) : fn == 1 ? gm_sinf(x) : gm_cosf(x);
    }
}

}  // namespace

extern "C" sg_status sg_libm_eval(int32_t fn, uint64_t start, uint64_t stride, uint64_t count, float *d_out,
                                  void *stream) {
    if (fn < 0 || fn > 2 || (count && !d_out)) return SG_ERR_INVALID;
    if (!count) return SG_OK;
    const uint64_t blocks = (count + 255) / 256;
    libm_eval_kernel<<<(unsigned)(blocks < 148 * 16 ? blocks : 148 * 16), 256, 0, (cudaStream_t)stream>>>(
        fn, start, stride, count, d_out);
    return cudaGetLastError() == cudaSuccess ? SG_OK : SG_ERR_CUDA;
}

extern "C" sg_status sg_binary_version(int32_t *out) {
    if (!out) return SG_ERR_INVALID;
    cudaFuncAttributes attr;
    if (cudaFuncGetAttributes(&attr, libm_eval_kernel) != cudaSuccess) return SG_ERR_CUDA;
    *out = attr.binaryVersion;
    return SG_OK;
}
