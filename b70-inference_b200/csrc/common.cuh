// Shared host/device helpers for the EXL3 B200 library: status codes, error text, launch checks, small PTX
// wrappers (mbarrier, bulk copy) used by several kernels.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

#include "../../include/exl3_b200.h"

namespace exl3 {

// ------------------------------------------------------------------------------------------------ host errors

// Last error text of the calling host thread (no global mutable state shared between threads).
void set_error(const char* fmt, ...);

#define EXL3_REQUIRE(cond, code, ...)          \
    do {                                       \
        if (!(cond)) {                         \
            ::exl3::set_error(__VA_ARGS__);    \
            return (code);                     \
        }                                      \
    } while (0)

#define EXL3_LAUNCH_CHECK(what)                                                              \
    do {                                                                                     \
        cudaError_t e_ = cudaGetLastError();                                                 \
        if (e_ != cudaSuccess) {                                                             \
            ::exl3::set_error("%s: launch failed: %s", what, cudaGetErrorString(e_));         \
            return EXL3_ERR_CUDA;                                                            \
        }                                                                                    \
    } while (0)

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Number of SMs of the current device (cached per device).
int num_sms();

// Device address of the library's sticky status word on the current device (see exl3_device_status).
int* device_status_ptr();

// The decode GEMVs' finisher wait for a split unit's other partials (exl3_set_finisher_wait), in ns.
uint64_t finisher_wait_ns();

// ------------------------------------------------------------------------------------------------ device helpers

constexpr uint32_t kMul1 = 0x83DCD12Du;
constexpr float kRsqrt128 = 0.08838834764831845f;
// Every device-side wait is bounded in time: a wait that has not completed after kWaitLimitNs of the global timer
// (100 ms; no wait of a healthy launch comes near it) gives up, the kernel records EXL3_ERR_TIMEOUT in its status
// word, lets its own copies in flight land and returns. kSpinLimit caps the polls as well, in case the timer stalls.
constexpr uint64_t kWaitLimitNs = 100ull * 1000 * 1000;
constexpr uint32_t kSpinLimit = 1u << 24;

__device__ __forceinline__ float h2f(__half h) { return __half2float(h); }

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier (shared::cta) ----
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: returns false when limit_ns of global time (or kSpinLimit polls) passed without completion. The
// fast path is one try_wait; the timer is read once per 32 polls after that.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 31) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
    }
    return false;
}
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---- 1D bulk copy global -> shared (TMA engine, no tensor map, no multicast) ----
// dst, src 16-byte aligned; bytes a multiple of 16. Completion is counted on the mbarrier as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Record a device-side failure (first writer wins) in a status word the host reads back.
__device__ __forceinline__ void report(int* status, int code) {
    if (status) atomicCAS(status, 0, code);
}

}  // namespace exl3
