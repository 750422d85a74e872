// exl3_gemv_noalloc: the dense decode GEMV with its scratch in a fixed, file-scope device array instead of a
// caller-provided workspace, for callers that cannot allocate device memory at all (an allocator-free host, a
// runtime that forbids allocation on its hot path). The kernels are exl3_gemv's (k_prep + k_gemv<EPI_LINEAR>); only
// where the scratch lives differs.
//
// Scratch (kNoAllocBytes = 1,845,248 bytes, 256-byte aligned): rotated input rows [8][kNoAllocMaxK] fp16 | their
// block sums [8][kNoAllocMaxK / 128] fp32 | tickets [kNoAllocMaxN / 128] int32 | split-unit partial slots
// [2 * kNoAllocMaxCtas][8][128] fp32.
// * Limits: M <= 8, k <= kNoAllocMaxK, n <= kNoAllocMaxN; the launch uses at most kNoAllocMaxCtas CTAs. Larger
//   shapes are rejected with EXL3_ERR_UNSUPPORTED.
// * Zero state: the tickets must be zero when the GEMV starts; the prep kernel of the same call zeroes them (and the
//   GEMV leaves them zero), so no initialisation by the caller is needed. The other regions are written before read.
// * The scratch is one per device and process: calls on the same device that may overlap (different streams,
//   threads or graphs in flight) race on it. Order them on one stream.
// * The symbol address is looked up once per device (cudaGetSymbolAddress) on the first call: make that first call
//   outside stream capture.
#include "gemv.cuh"

namespace exl3 {

constexpr int kNoAllocMaxK = 32768;
constexpr int kNoAllocMaxN = 65536;
constexpr int kNoAllocMaxCtas = 160;
constexpr size_t kNoAllocXf = (size_t)kMaxRows * kNoAllocMaxK * 2;
constexpr size_t kNoAllocXsum = (size_t)kMaxRows * (kNoAllocMaxK / 128) * 4;
constexpr size_t kNoAllocTickets = (size_t)(kNoAllocMaxN / 128) * 4;
constexpr size_t kNoAllocPartial = (size_t)2 * kNoAllocMaxCtas * unit_floats(EPI_LINEAR) * 4;
constexpr size_t kNoAllocBytes = kNoAllocXf + kNoAllocXsum + kNoAllocTickets + kNoAllocPartial;
static_assert(kNoAllocXf % 256 == 0 && kNoAllocXsum % 256 == 0 && kNoAllocTickets % 256 == 0, "region alignment");
static_assert(kNoAllocBytes == 1845248, "the documented scratch size");

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

// Device address of the scratch on the current device, resolved once per device.
static uint8_t* noalloc_scratch() {
    static uint8_t* addr[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    if (!addr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess) return nullptr;
        addr[dev] = static_cast<uint8_t*>(p);
    }
    return addr[dev];
}

}  // namespace exl3

using namespace exl3;

extern "C" {

int exl3_gemv_noalloc(const void* x, int x_dtype, int ldx, int M, const void* packed, const void* suh,
                      const void* svh, int k, int n, int K, int cb, void* y, int y_dtype, int ldy, void* stream) {
    EXL3_REQUIRE(cb == 2, EXL3_ERR_UNSUPPORTED, "exl3_gemv_noalloc: only the mul1 codebook (cb=2) is supported");
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_UNSUPPORTED, "exl3_gemv_noalloc: K=%d not in 1..8", K);
    EXL3_REQUIRE(M >= 0 && M <= kMaxRows, EXL3_ERR_ARG, "exl3_gemv_noalloc: M=%d rows (1..8 per call)", M);
    EXL3_REQUIRE(k > 0 && n > 0 && k % 128 == 0 && n % 128 == 0, EXL3_ERR_ARG,
                 "exl3_gemv_noalloc: k=%d, n=%d must be multiples of 128", k, n);
    EXL3_REQUIRE(k <= kNoAllocMaxK && n <= kNoAllocMaxN, EXL3_ERR_UNSUPPORTED,
                 "exl3_gemv_noalloc: k=%d, n=%d exceed the static scratch (k <= %d, n <= %d); use exl3_gemv", k, n,
                 kNoAllocMaxK, kNoAllocMaxN);
    EXL3_REQUIRE(x && packed && svh && y, EXL3_ERR_ARG, "exl3_gemv_noalloc: null pointer");
    EXL3_REQUIRE(aligned16(packed), EXL3_ERR_ARG, "exl3_gemv_noalloc: packed trellis must be 16-byte aligned");
    EXL3_REQUIRE(x_dtype == EXL3_F16 || x_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED,
                 "exl3_gemv_noalloc: x dtype %d", x_dtype);
    EXL3_REQUIRE(y_dtype == EXL3_F16 || y_dtype == EXL3_BF16 || y_dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED,
                 "exl3_gemv_noalloc: y dtype %d", y_dtype);
    EXL3_REQUIRE(ldx >= k && ldy >= n && ldx % 4 == 0 && ldy % 4 == 0, EXL3_ERR_ARG,
                 "exl3_gemv_noalloc: row strides ldx=%d ldy=%d", ldx, ldy);
    EXL3_REQUIRE((reinterpret_cast<uintptr_t>(x) & 7) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0,
                 EXL3_ERR_ARG, "exl3_gemv_noalloc: x must be 8-byte and y 16-byte aligned");
    if (M == 0) return EXL3_OK;
    uint8_t* ws = noalloc_scratch();
    EXL3_REQUIRE(ws, EXL3_ERR_CUDA, "exl3_gemv_noalloc: scratch symbol lookup failed: %s",
                 cudaGetErrorString(cudaGetLastError()));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    __half* xf = reinterpret_cast<__half*>(ws);
    float* xsum = reinterpret_cast<float*>(ws + kNoAllocXf);
    int* tickets = reinterpret_cast<int*>(ws + kNoAllocXf + kNoAllocXsum);

    PrepArgs pa = {};
    pa.x = x;
    pa.ldx = ldx;
    pa.x_bf16 = x_dtype == EXL3_BF16;
    pa.rows = M;
    pa.k = k;
    pa.suh = static_cast<const __half*>(suh);
    pa.xf = xf;
    pa.xsum = xsum;
    pa.zero = tickets;
    pa.n_zero = n / 128;
    int rc = launch_prep(pa, st, "exl3_gemv_noalloc");
    if (rc) return rc;

    GemvArgs a = {};
    a.tr = static_cast<const uint32_t*>(packed);
    a.svh = static_cast<const __half*>(svh);
    a.K = K;
    a.y = y;
    a.ldy = ldy;
    a.y_dtype = y_dtype;
    a.M = M;
    a.xf = xf;
    a.xsum = xsum;
    a.k = k;
    a.n = n;
    a.partial = reinterpret_cast<float*>(ws + kNoAllocXf + kNoAllocXsum + kNoAllocTickets);
    a.counters = tickets;
    a.status = device_status_ptr();
    GemvPlan pl = plan_gemv(EPI_LINEAR, (long long)(n / 128) * (k / 128), 0);
    if (pl.ctas > kNoAllocMaxCtas) pl.ctas = kNoAllocMaxCtas;
    return launch_gemv<EPI_LINEAR>(a, pl, st, "exl3_gemv_noalloc");
}

}  // extern "C"
