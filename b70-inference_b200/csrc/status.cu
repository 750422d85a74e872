// Library plumbing: per-thread error text, SM count, and the device status word that bounded device waits write.
#include <stdarg.h>

#include <mutex>

#include <atomic>

#include "common.cuh"

namespace exl3 {

static thread_local char t_err[512] = {0};

void set_error(const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_err, sizeof(t_err), fmt, ap);
    va_end(ap);
}

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (cache[dev] == 0) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 148;
    }
    return cache[dev];
}

// Sticky device-side status (first failure wins); kernels receive its address as an argument.
static __device__ int g_device_status;

int* device_status_ptr() {
    static int* cache[64] = {nullptr};
    static std::mutex mu;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!cache[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_status) != cudaSuccess) return nullptr;
        cache[dev] = static_cast<int*>(p);
    }
    return cache[dev];
}

// A wait nothing completes: one thread initialises an mbarrier that expects one arrival and waits on it with the
// library's bounded wait and the given limit. The wait runs out, the kernel records EXL3_ERR_TIMEOUT and returns.
static __global__ void k_wait_probe(uint64_t limit_ns, int* status) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    mbar_init(&bar, 1);
    fence_barrier_init();
    if (!mbar_wait(&bar, 0, limit_ns)) report(status, EXL3_ERR_TIMEOUT);
}

static std::atomic<uint64_t> g_finisher_wait_ns{20000};
uint64_t finisher_wait_ns() { return g_finisher_wait_ns.load(std::memory_order_relaxed); }

}  // namespace exl3

extern "C" {

int exl3_set_finisher_wait(uint64_t wait_ns) {
    EXL3_REQUIRE(wait_ns <= exl3::kWaitLimitNs, EXL3_ERR_ARG, "exl3_set_finisher_wait: %llu ns above %llu",
                 (unsigned long long)wait_ns, (unsigned long long)exl3::kWaitLimitNs);
    exl3::g_finisher_wait_ns.store(wait_ns, std::memory_order_relaxed);
    return EXL3_OK;
}

int exl3_wait_probe(uint64_t limit_ns, void* stream) {
    EXL3_REQUIRE(limit_ns > 0 && limit_ns <= exl3::kWaitLimitNs, EXL3_ERR_ARG,
                 "exl3_wait_probe: limit %llu ns outside (0, %llu]", (unsigned long long)limit_ns,
                 (unsigned long long)exl3::kWaitLimitNs);
    int* status = exl3::device_status_ptr();
    EXL3_REQUIRE(status, EXL3_ERR_CUDA, "exl3_wait_probe: status word lookup failed");
    exl3::k_wait_probe<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, status);
    EXL3_LAUNCH_CHECK("exl3_wait_probe");
    return EXL3_OK;
}

int exl3_version(void) { return 100; }

const char* exl3_last_error(void) { return exl3::t_err; }

int exl3_device_status(int reset) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, exl3::g_device_status, sizeof(int)) != cudaSuccess) {
        exl3::set_error("exl3_device_status: %s", cudaGetErrorString(cudaGetLastError()));
        return EXL3_ERR_CUDA;
    }
    if (reset) {
        int z = 0;
        cudaMemcpyToSymbol(exl3::g_device_status, &z, sizeof(int));
    }
    return v;
}

}  // extern "C"
