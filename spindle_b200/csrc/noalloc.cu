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
// that device (and again on the first call after a device reset, which can
// move the array).  That first call therefore does a little set-up work and
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
struct ScratchSlot {
    unsigned long long ctx_id = 0;  // context the address belongs to (0 = none yet)
    void *ptr = nullptr;
};
ScratchSlot g_scratch[MAX_DEVICES];
std::mutex g_scratch_mu;

// The id of the current CUDA context (unique for the life of the process).
// A device reset or a new primary context reloads the library's module, so
// the array can move; the cached address is only reused under the same id.
// The driver calls come through cudaGetDriverEntryPoint, so the library keeps
// no link-time dependency on libcuda.
bool current_context_id(unsigned long long *id) {
    typedef int (*get_current_t)(void **);
    typedef int (*get_id_t)(void *, unsigned long long *);
    static get_current_t get_current = nullptr;
    static get_id_t get_id = nullptr;
    if (!get_current || !get_id) {
        void *f1 = nullptr, *f2 = nullptr;
        cudaDriverEntryPointQueryResult q1, q2;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
            q1 != cudaDriverEntryPointSuccess || !f1)
            return false;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
            q2 != cudaDriverEntryPointSuccess || !f2)
            return false;
        get_current = (get_current_t)f1;
        get_id = (get_id_t)f2;
    }
    void *ctx = nullptr;
    if (get_current(&ctx) != 0 || !ctx) return false;
    return get_id(ctx, id) == 0 && *id != 0;
}

// Device address of g_noalloc_scratch in the current device's context: looked
// up with cudaGetSymbolAddress once per device and context, with that device
// current (the first call on a device, or the first after a device reset).
sg_status scratch_address(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return SG_ERR_CUDA;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    unsigned long long id = 0;
    const bool have_ctx = current_context_id(&id);
    if (!have_ctx || g_scratch[dev].ctx_id != id || !g_scratch[dev].ptr) {
        // with no current context yet, this lookup makes the device's primary context current
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return SG_ERR_CUDA;
        if (!have_ctx && !current_context_id(&id)) return SG_ERR_CUDA;
        g_scratch[dev].ptr = p;
        g_scratch[dev].ctx_id = id;
    }
    *out = g_scratch[dev].ptr;
    return SG_OK;
}

}  // namespace

extern "C" sg_status sg_matvec_static(const uint8_t *d_base, const sg_mat *m, const float *d_x, uint64_t ldx,
                                      float *d_out, uint64_t ldo, uint64_t n_vec, uint64_t r0, uint64_t r1,
                                      void *stream) {
    if (!m) return SG_ERR_INVALID;
    const uint64_t qb = sg_q8k_bytes(m->cols);
    // a division, not n_vec * qb, so that no n_vec can wrap past the limit
    if (qb && n_vec > SG_NOALLOC_SCRATCH_BYTES / qb) return SG_ERR_NOALLOC_LIMIT;
    void *scratch = nullptr;
    const sg_status st = scratch_address(&scratch);
    if (st) return st;
    return sg_matvec_scratch(d_base, m, d_x, ldx, d_out, ldo, n_vec, r0, r1, scratch, SG_NOALLOC_SCRATCH_BYTES,
                             stream);
}
