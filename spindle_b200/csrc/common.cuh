// common.cuh — shared device helpers for the spindle-b200 kernels (sm_100a).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "spindle_gpu.h"

namespace sg {

// Device-side status word: bounded waits record where they gave up instead of
// hanging or trapping; the host reads it with sg_device_status().
enum : unsigned { DEV_OK = 0, DEV_TIMEOUT_TMA = 1, DEV_BAD_LAUNCH = 2, DEV_TIMEOUT_PEER = 3 };
extern __device__ unsigned g_dev_status;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint32_t dynamic_smem_size() {
    uint32_t v;
    asm volatile("mov.u32 %0, %%dynamic_smem_size;" : "=r"(v));
    return v;
}

__device__ __forceinline__ float half_at(const uint8_t *p) {
    // 2-byte aligned load; IEEE half -> float is exact (quant_q8k.rs:146-149).
    return __half2float(__ushort_as_half(*reinterpret_cast<const unsigned short *>(p)));
}

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) {
    return *reinterpret_cast<const uint32_t *>(p);
}

// 4 bytes at an even (possibly not 4-aligned) shared-memory offset.
__device__ __forceinline__ uint32_t lds32_u2(const uint8_t *base, uint32_t off) {
    uint32_t a = off & ~3u;
    uint32_t w0 = lds32(base + a), w1 = lds32(base + a + 4);
    return __funnelshift_r(w0, w1, (off & 3u) * 8u);
}

// ---- mbarrier + bulk copy (TMA engine, non-tensor form) -------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

// Waits for the phase with the given parity; gives up after ~limit_ns and
// returns false (the caller records the timeout and stops using the buffer).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    uint64_t t0 = globaltimer_ns();
    for (;;) {
        for (int i = 0; i < 64; i++)
            if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}

// Global -> shared bulk copy completing on `bar` (16-byte aligned addresses,
// size a multiple of 16), one destination CTA.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

constexpr uint64_t WAIT_LIMIT_NS = 2000000000ull;  // 2 s: far above any tile's latency

}  // namespace sg
