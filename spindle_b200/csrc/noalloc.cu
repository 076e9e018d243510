// noalloc.cu — sg_matvec_static: the matvec of sg_matvec_scratch without any
// allocation, for callers that cannot allocate device memory.
//
// Who needs it: hosts that drive the GPU through this C ABI but have no CUDA
// allocator of their own (a Rust or C engine that links only this library),
// code that must not call cudaMalloc on its path (it can synchronize the whole
// device and stall other streams mid-decode), and processes whose memory is
// fully reserved up front by another runtime's pool.  Such callers still own
// their inputs and outputs; only the Q8_K scratch moves into the library.
//
// The scratch is a file-scope device array of SG_NOALLOC_SCRATCH_BYTES bytes.
// Every GPU that loads the library holds it until the process exits.  Host
// code cannot use the array's name as a device address (it names a host-side
// stand-in), so the address is looked up once per device with
// cudaGetSymbolAddress, with that device current, on the first call made on
// that device.  That first call therefore does a little set-up work and
// should come before any stream capture.
//
// All calls share the one array and it keeps the last call's contents.  The
// quantizer overwrites every byte a call reads, so nothing has to start at
// zero; but two calls whose kernels overlap on the GPU (different streams,
// or different host threads) race on it and must be serialized by the caller.
#include <mutex>

#include "kernels.cuh"

namespace {

static __device__ __align__(256) uint8_t g_noalloc_scratch[SG_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
void *g_scratch_ptr[MAX_DEVICES] = {};
std::mutex g_scratch_mu;

// Device address of g_noalloc_scratch on the current device (looked up once).
sg_status scratch_address(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return SG_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return SG_ERR_CUDA;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return SG_OK;
}

}  // namespace

extern "C" sg_status sg_matvec_static(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx,
                                      float *d_out, uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1,
                                      void *stream) {
    if (!m) return SG_ERR_INVALID;
    if (sg_matvec_scratch_bytes(m->cols, n_vec) > SG_NOALLOC_SCRATCH_BYTES) return SG_ERR_NOALLOC_LIMIT;
    void *scratch = nullptr;
    const sg_status st = scratch_address(&scratch);
    if (st) return st;
    return sg_matvec_scratch(d_base, m, d_x, ldx, d_out, ldo, n_vec, r0, r1, scratch, SG_NOALLOC_SCRATCH_BYTES,
                             stream);
}
