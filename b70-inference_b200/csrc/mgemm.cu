// exl3_mgemm: several EXL3 linears over pointer tables in one grouped launch (exllamav3's exl3_mgemm contract,
// glm/docs/ext-op-inventory.md:664-688,1104-1120): slot j computes C[j] = lin(A[j or 0], matrix q_j) (* w[j]), with
// q_j = indices[j] (or j), negative or filtered slots skipped, and with weights the slots of each token summed.
//
// Built from the grouped decode GEMV: a prep kernel turns the pointer tables into expert descriptors and an item
// table (one item per 8 rows of a slot) and rotates every slot's input rows with its matrix's input signs (xf order);
// k_gemv<EPI_DOWN> computes (w *) lin() per position into fp32 rows; an output kernel copies the slots into C, or
// sums each token's slots in slot order.
//
// Workspace: counters (8 ints) | descriptors [n_mats] | items [max_items] x 3 | row weights [P] | tickets
// [max_items][n/128] | xf rows [P][k] fp16 | their block sums [P][k/128] fp32 | fp32 rows [P][n] | split-unit
// partial slots, P = slots * m.
#include <type_traits>

#include "gemv.cuh"

namespace exl3 {

struct MgLayout {
    size_t desc, item_expert, item_start, item_cnt, pair_w, tickets, xf, xsum, ybuf, partial, total;
    int max_items, P, n_tickets;
};

inline MgLayout mg_layout(int slots, int m, int k, int n, int n_mats) {
    MgLayout L;
    const int ipr = (m + kMaxRows - 1) / kMaxRows;           // items per slot
    L.max_items = slots * ipr;
    L.P = slots * m;
    L.n_tickets = L.max_items * (n / 128);
    size_t o = 8 * 4;
    L.desc = align_up(o, 16); o = L.desc + (size_t)n_mats * sizeof(ExpertDesc);
    L.item_expert = align_up(o, 16); o = L.item_expert + (size_t)L.max_items * 4;
    L.item_start = o; o += (size_t)L.max_items * 4;
    L.item_cnt = o; o += (size_t)L.max_items * 4;
    L.pair_w = o; o += (size_t)L.P * 4;
    L.tickets = o; o += (size_t)L.n_tickets * 4;
    o = align_up(o, 256);
    L.xf = o; o += align_up((size_t)L.P * k * 2, 256);
    L.xsum = o; o += align_up((size_t)L.P * (k / 128) * 4, 256);
    L.ybuf = o; o += align_up((size_t)L.P * n * 4, 256);
    L.partial = o; o += partial_bytes(EPI_DOWN);
    L.total = o;
    return L;
}

// Matrix of slot j (-1: skipped): indices[j] or j, filtered to [min_index, max_index) and rebased when min_index >= 0.
__device__ __forceinline__ int slot_matrix(const int32_t* indices, int j, int n_mats, int min_index, int max_index) {
    int q = indices ? __ldg(indices + j) : j;
    if (min_index >= 0) q = (q >= min_index && q < max_index) ? q - min_index : -1;
    return (q >= 0 && q < n_mats) ? q : -1;
}

struct MgPrep {
    const void* A;
    int a_bf16, a_batches, lda;
    int m, k, n, slots, n_mats, min_index, max_index;
    const uint64_t* trellis;      // [n_mats] packed trellis addresses (exl3_pack)
    const uint64_t* suh;          // [n_mats] (entries may be 0: no input signs)
    const uint64_t* svh;          // [n_mats]
    const int32_t* K;             // [n_mats]
    const int32_t* indices;       // [slots] or null
    const float* weights;         // [slots] or null
    uint8_t* ws;
    MgLayout L;
};

constexpr int kMgThreads = 1024;

// CTA 0: descriptors, items, row weights, tickets, item count; then it lets the GEMV launch (whose producers read the
// item table before their griddepcontrol.wait). Other CTAs: rotated input rows of every position of a valid slot.
static __global__ void __launch_bounds__(kMgThreads) k_mg_prep(const MgPrep p) {
    __shared__ int scan[kMgThreads];
    pdl_wait();
    const int t = threadIdx.x;
    if (blockIdx.x == 0) {
        ExpertDesc* desc = reinterpret_cast<ExpertDesc*>(p.ws + p.L.desc);
        for (int i = t; i < p.n_mats; i += kMgThreads) {
            ExpertDesc d = {};
            d.tr[2] = reinterpret_cast<const uint32_t*>(p.trellis[i]);
            d.suh[2] = p.suh ? reinterpret_cast<const __half*>(p.suh[i]) : nullptr;
            d.svh[2] = reinterpret_cast<const __half*>(p.svh[i]);
            d.K[2] = p.K[i];
            desc[i] = d;
        }
        int* tickets = reinterpret_cast<int*>(p.ws + p.L.tickets);
        for (int i = t; i < p.L.n_tickets; i += kMgThreads) tickets[i] = 0;
        float* pw = reinterpret_cast<float*>(p.ws + p.L.pair_w);
        for (int i = t; i < p.L.P; i += kMgThreads) pw[i] = p.weights ? __ldg(p.weights + i / p.m) : 1.0f;
        int* ie = reinterpret_cast<int*>(p.ws + p.L.item_expert);
        int* is = reinterpret_cast<int*>(p.ws + p.L.item_start);
        int* ic = reinterpret_cast<int*>(p.ws + p.L.item_cnt);
        const int ipr = (p.m + kMaxRows - 1) / kMaxRows;
        int carry = 0;
        for (int j0 = 0; j0 < p.slots; j0 += kMgThreads) {
            const int j = j0 + t;
            const int q = j < p.slots ? slot_matrix(p.indices, j, p.n_mats, p.min_index, p.max_index) : -1;
            const int c = q >= 0 ? ipr : 0;
            scan[t] = c;
            __syncthreads();
            for (int o = 1; o < kMgThreads; o <<= 1) {        // inclusive scan
                const int add = t >= o ? scan[t - o] : 0;
                __syncthreads();
                scan[t] += add;
                __syncthreads();
            }
            const int base = carry + scan[t] - c;
            for (int i = 0; i < c; ++i) {
                ie[base + i] = q;
                is[base + i] = j * p.m + i * kMaxRows;
                ic[base + i] = min(kMaxRows, p.m - i * kMaxRows);
            }
            carry += scan[kMgThreads - 1];
            __syncthreads();
        }
        if (t == 0) reinterpret_cast<int*>(p.ws)[0] = carry;
        __threadfence();
        __syncthreads();
        pdl_trigger();
        return;
    }
    pdl_trigger();
    __half* xf = reinterpret_cast<__half*>(p.ws + p.L.xf);
    const int KB = p.k / 128, lane = t & 31;
    const long jobs = (long)p.L.P * KB;
    const long nw = (long)(gridDim.x - 1) * (kMgThreads / 32);
    for (long jb = (long)(blockIdx.x - 1) * (kMgThreads / 32) + (t >> 5); jb < jobs; jb += nw) {
        const int pos = (int)(jb / KB), kb = (int)(jb % KB);
        const int j = pos / p.m, r = pos % p.m;
        const int q = slot_matrix(p.indices, j, p.n_mats, p.min_index, p.max_index);
        if (q < 0) continue;                                  // warp-uniform
        const size_t xrow = ((size_t)(p.a_batches == 1 ? 0 : j) * p.m + r) * p.lda + (size_t)kb * 128;
        const __half* su = p.suh && p.suh[q] ? reinterpret_cast<const __half*>(p.suh[q]) + kb * 128 : nullptr;
        float v[4];
        if (p.a_bf16)
            rotated_block<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(p.A) + xrow, su, lane, v);
        else
            rotated_block<__half>(static_cast<const __half*>(p.A) + xrow, su, lane, v);
        store_xf_block(v, lane, xf + (size_t)pos * p.k + (size_t)kb * 128);
        const float bs = xf_block_sum(v);
        if (lane == 0) reinterpret_cast<float*>(p.ws + p.L.xsum)[(size_t)pos * KB + kb] = bs;
    }
}

// C from the fp32 rows: unweighted, C[j] = rows of slot j (valid slots only); weighted, C[t] = sum of token t's
// slots in slot order (stride = slots / num_tokens).
template <typename T>
static __global__ void __launch_bounds__(256) k_mg_out(const float* ybuf, const int32_t* indices, int slots, int m,
                                                       int n, int n_mats, int min_index, int max_index, int weighted,
                                                       int num_tokens, T* C, int ldc) {
    pdl_wait();
    pdl_trigger();
    const int n4 = n / 4;
    const int out_slots = weighted ? num_tokens : slots;
    const long total = (long)out_slots * m * n4;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (long)gridDim.x * blockDim.x) {
        const int c4 = (int)(i % n4);
        const long rowi = i / n4;
        const int r = (int)(rowi % m), s = (int)(rowi / m);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        if (weighted) {
            const int stride = slots / num_tokens;
            for (int j = s * stride; j < (s + 1) * stride; ++j) {
                if (slot_matrix(indices, j, n_mats, min_index, max_index) < 0) continue;
                const float4 v = __ldcg(reinterpret_cast<const float4*>(ybuf + ((size_t)j * m + r) * n) + c4);
                acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
        } else {
            if (slot_matrix(indices, s, n_mats, min_index, max_index) < 0) continue;
            acc = __ldcg(reinterpret_cast<const float4*>(ybuf + ((size_t)s * m + r) * n) + c4);
        }
        T* dst = C + ((size_t)s * m + r) * ldc + 4 * c4;
        if constexpr (std::is_same<T, float>::value) {
            *reinterpret_cast<float4*>(dst) = acc;
        } else {
            dst[0] = (T)acc.x; dst[1] = (T)acc.y; dst[2] = (T)acc.z; dst[3] = (T)acc.w;
        }
    }
}

}  // namespace exl3

using namespace exl3;

extern "C" {

size_t exl3_mgemm_workspace_size(int slots, int m, int k, int n, int n_mats) {
    if (slots <= 0 || m <= 0 || k <= 0 || n <= 0 || n_mats <= 0) return 0;
    return mg_layout(slots, m, k, n, n_mats).total;
}

int exl3_mgemm(const void* A, int a_dtype, int a_batches, int lda, int m, int k, int n, const uint64_t* trellis_ptrs,
               const uint64_t* suh_ptrs, const uint64_t* svh_ptrs, const int32_t* K_per_mat, int n_mats,
               const int32_t* indices, int slots, const float* weights, int num_tokens, int min_index, int max_index,
               void* C, int c_dtype, int ldc, void* workspace, size_t ws_bytes, void* stream) {
    EXL3_REQUIRE(A && trellis_ptrs && svh_ptrs && K_per_mat && C && n_mats > 0 && slots >= 0 && m >= 0, EXL3_ERR_ARG,
                 "exl3_mgemm: bad arguments");
    EXL3_REQUIRE(k > 0 && n > 0 && k % 128 == 0 && n % 128 == 0, EXL3_ERR_ARG,
                 "exl3_mgemm: k=%d, n=%d must be multiples of 128", k, n);
    EXL3_REQUIRE(a_batches == 1 || a_batches == slots, EXL3_ERR_ARG,
                 "exl3_mgemm: a_batches=%d must be 1 or the slot count %d", a_batches, slots);
    EXL3_REQUIRE(a_dtype == EXL3_F16 || a_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "exl3_mgemm: A dtype %d", a_dtype);
    EXL3_REQUIRE(c_dtype == EXL3_F16 || c_dtype == EXL3_BF16 || c_dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED,
                 "exl3_mgemm: C dtype %d", c_dtype);
    EXL3_REQUIRE(lda >= k && ldc >= n && (reinterpret_cast<uintptr_t>(A) & 7) == 0 && lda % 4 == 0, EXL3_ERR_ARG,
                 "exl3_mgemm: A rows must be 8-byte aligned (lda=%d), ldc=%d", lda, ldc);
    EXL3_REQUIRE(c_dtype != EXL3_F32 || ((reinterpret_cast<uintptr_t>(C) & 15) == 0 && ldc % 4 == 0), EXL3_ERR_ARG,
                 "exl3_mgemm: fp32 C must be 16-byte aligned with ldc %% 4 == 0");
    EXL3_REQUIRE(!weights || (num_tokens > 0 && slots % num_tokens == 0), EXL3_ERR_ARG,
                 "exl3_mgemm: %d slots do not split over %d tokens", slots, num_tokens);
    if (slots == 0 || m == 0) return EXL3_OK;
    const MgLayout L = mg_layout(slots, m, k, n, n_mats);
    EXL3_REQUIRE(workspace && ws_bytes >= L.total && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 EXL3_ERR_WORKSPACE, "exl3_mgemm: workspace %zu < %zu bytes (or not 256-byte aligned)", ws_bytes,
                 L.total);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    MgPrep pp = {};
    pp.A = A;
    pp.a_bf16 = a_dtype == EXL3_BF16;
    pp.a_batches = a_batches;
    pp.lda = lda;
    pp.m = m;
    pp.k = k;
    pp.n = n;
    pp.slots = slots;
    pp.n_mats = n_mats;
    pp.min_index = min_index;
    pp.max_index = max_index;
    pp.trellis = trellis_ptrs;
    pp.suh = suh_ptrs;
    pp.svh = svh_ptrs;
    pp.K = K_per_mat;
    pp.indices = indices;
    pp.weights = weights;
    pp.ws = ws;
    pp.L = L;
    {
        long rot_blocks = ((long)L.P * (k / 128) + 31) / 32;
        if (rot_blocks > 2L * num_sms()) rot_blocks = 2L * num_sms();
        if (rot_blocks < 1) rot_blocks = 1;
        cudaError_t e = launch_pdl(k_mg_prep, dim3((unsigned)(1 + rot_blocks)), dim3(kMgThreads), 0, st, pp);
        EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_mgemm: prep launch failed: %s", cudaGetErrorString(e));
    }
    GemvArgs a = {};
    a.experts = reinterpret_cast<const ExpertDesc*>(ws + L.desc);
    a.items.n_items = reinterpret_cast<const int*>(ws);
    a.items.item_expert = reinterpret_cast<const int*>(ws + L.item_expert);
    a.items.item_start = reinterpret_cast<const int*>(ws + L.item_start);
    a.items.item_cnt = reinterpret_cast<const int*>(ws + L.item_cnt);
    a.items.pair_w = reinterpret_cast<const float*>(ws + L.pair_w);
    a.ybuf = reinterpret_cast<float*>(ws + L.ybuf);
    a.ybuf_round_f16 = !weights && c_dtype == EXL3_F16;   // the fp16 linear's rounding for unweighted fp16 C
    a.xf = reinterpret_cast<const __half*>(ws + L.xf);
    a.xsum = reinterpret_cast<const float*>(ws + L.xsum);
    a.k = k;
    a.n = n;
    a.partial = reinterpret_cast<float*>(ws + L.partial);
    a.counters = reinterpret_cast<int*>(ws + L.tickets);
    a.status = device_status_ptr();
    const GemvPlan pl = plan_gemv(EPI_DOWN, (long long)L.max_items * (n / 128) * (k / 128), 0);
    int rc = launch_gemv<EPI_DOWN>(a, pl, st, "exl3_mgemm");
    if (rc) return rc;
    const float* ybuf = reinterpret_cast<const float*>(ws + L.ybuf);
    const long outs = (long)(weights ? num_tokens : slots) * m * (n / 4);
    long blocks = (outs + 255) / 256;
    if (blocks > 8L * num_sms()) blocks = 8L * num_sms();
    const dim3 grid((unsigned)(blocks > 0 ? blocks : 1));
    const int w = weights != nullptr;
    cudaError_t e;
    if (c_dtype == EXL3_F32)
        e = launch_pdl(k_mg_out<float>, grid, dim3(256), 0, st, ybuf, indices, slots, m, n, n_mats, min_index,
                       max_index, w, num_tokens, static_cast<float*>(C), ldc);
    else if (c_dtype == EXL3_F16)
        e = launch_pdl(k_mg_out<__half>, grid, dim3(256), 0, st, ybuf, indices, slots, m, n, n_mats, min_index,
                       max_index, w, num_tokens, static_cast<__half*>(C), ldc);
    else
        e = launch_pdl(k_mg_out<__nv_bfloat16>, grid, dim3(256), 0, st, ybuf, indices, slots, m, n, n_mats, min_index,
                       max_index, w, num_tokens, static_cast<__nv_bfloat16*>(C), ldc);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_mgemm: output launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

}  // extern "C"
