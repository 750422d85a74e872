// Expert-parallel token exchange over peer memory (NVLink / NVSwitch): the dispatch and combine steps of the
// expert-parallel MoE layer written as this library's own kernels, in place of two NCCL all-to-alls and their
// host-side glue per layer.
//
// Every rank holds one exchange buffer (exl3_ep_buffer_create: cudaMalloc'd, exported with a CUDA IPC handle) and maps
// its peers' buffers (exl3_ep_buffer_open). Layout of a buffer (W ranks, cap rows per rank and call, H hidden, k
// picks per row), identical on every rank:
//   control (8 KB): dispatch and combine flags [W][chunks] (slot [r][c] written by rank r's CTA for chunk c: the
//                   epoch of its last signal) and this rank's per-CTA call counters
//   recv_x   fp16 [W][cap][H]    row i of source rank r at [r][i]: written by rank r
//   recv_ids int32 [W][cap][k]   rank r's picks for row i rebased to this rank's experts (-1: another rank's)
//   recv_w   fp32 [W][cap][k]
//   back     fp32 [W][cap][H]    this rank's row i as computed by rank p's experts, at [p][i]: written by rank p
// Rows are cut into `chunks` contiguous chunks (the same on every rank); CTA (c, p) of a launch handles chunk c for
// peer p. No CTA waits for another CTA of its own launch and no atomics are involved:
// dispatch: CTA (c, p) of rank r writes chunk c of r's rows, with the picks rebased to p's expert range (a row's
//   activations only when it has a pick there; rows past the batch carry no picks), into recv[r] of peer p, fences
//   at system scope and stores the call's epoch into p's dispatch flag [r][c]; then it waits for its own flag [p][c]
//   (peer p's chunk c for this rank). The launch ends when every chunk of every peer has arrived (bounded waits:
//   100 ms, then EXL3_ERR_TIMEOUT in the status word).
// local experts: the grouped MoE kernels run on recv as one batch of W * cap rows.
// combine: CTA (c, r) of rank p writes the partial rows of chunk c received from r that had a pick on p into r's
//   back[p], fences, signals r's combine flag [p][c], and waits for the flags [q][c] of every rank q: this rank's
//   chunk-c rows are then complete; with the reduce fused, the W CTAs of chunk c then sum its rows:
// reduce: out[i] = sum over q in rank order of back[q][i] for the ranks q that row i picked (+ the shared expert's
//   row): a fixed order, so the result is bit-reproducible for a given world size.
// Every CTA counts its own calls (epochs), so the sequence is graph-capturable; every rank must make the same calls in
// the same order. The buffers are single-buffered: a rank's next dispatch can only start after its combine, which
// needs every peer's combine of the previous call, which follows that peer's use of its receive region.
#include "gemv.cuh"

namespace exl3 {

constexpr int kEpMaxRanks = 64;
constexpr int kEpThreads = 256;
constexpr int kEpMaxSlots = 512;    // W * chunks

struct EpCtl {
    uint32_t dflag[kEpMaxSlots];      // [source rank][chunk]: written by the peers
    uint32_t cflag[kEpMaxSlots];
    uint32_t d_epoch[kEpMaxSlots];    // [peer][chunk]: this rank's CTA calls
    uint32_t c_epoch[kEpMaxSlots];
};
constexpr size_t kEpCtlBytes = 8192;
static_assert(sizeof(EpCtl) <= kEpCtlBytes, "control block");

struct EpLayout {
    size_t recv_x, recv_ids, recv_w, back, total;
};
inline EpLayout ep_layout(int W, int cap, int H, int k) {
    EpLayout L;
    size_t o = kEpCtlBytes;
    L.recv_x = o; o += align_up((size_t)W * cap * H * 2, 256);
    L.recv_ids = o; o += align_up((size_t)W * cap * k * 4, 256);
    L.recv_w = o; o += align_up((size_t)W * cap * k * 4, 256);
    L.back = o; o += align_up((size_t)W * cap * H * 4, 256);
    L.total = o;
    return L;
}

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Wait (one thread) until flags[0], flags[stride], ..., flags[(n - 1) stride] all equal `epoch`; bounded by
// kWaitLimitNs of global time.
__device__ bool ep_wait_flags(const uint32_t* flags, int n, int stride, uint32_t epoch) {
    const uint64_t t0 = globaltimer_ns();
    for (int p = 0; p < n; ++p) {
        while (ld_acquire_sys(flags + (size_t)p * stride) != epoch) {
            if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
            __nanosleep(32);
        }
    }
    return true;
}

struct EpArgs {
    const uint64_t* peers;   // [W] exchange buffer addresses (this rank's own at [rank])
    uint8_t* local;          // this rank's buffer
    EpLayout L;
    int W, rank, cap, H, k, E, B;
    int x_bf16, ldx;
    const void* x;           // dispatch: [B][H] rows
    const int32_t* ids;      // dispatch: [B][k] global expert ids
    const float* w;          // dispatch: [B][k]
    const float* part;       // combine: [W][cap][H] local expert results on the received rows
    int* status;
};

// Whether row i of this rank picks an expert of rank p (ids global; per = E / W experts per rank).
__device__ __forceinline__ bool row_picks_rank(const int32_t* ids, int i, int k, int p, int per) {
    for (int j = 0; j < k; ++j) {
        const int e = ids[(size_t)i * k + j];
        if (e >= p * per && e < (p + 1) * per) return true;
    }
    return false;
}

// grid (chunks, W): CTA (c, p) sends rows [c * rpc, ...) of this rank to peer p and waits for peer p's chunk c.
__global__ void __launch_bounds__(kEpThreads) k_ep_dispatch(const EpArgs a) {
    pdl_wait();                                                 // ids and rows come from earlier kernels
    pdl_trigger();
    EpCtl* ctl = reinterpret_cast<EpCtl*>(a.local);
    const int c = blockIdx.x, p = blockIdx.y, nch = gridDim.x, per = a.E / a.W;
    const int rpc = (a.cap + nch - 1) / nch;
    const int i0 = c * rpc, i1 = min(a.cap, i0 + rpc);
    uint8_t* peer = reinterpret_cast<uint8_t*>(a.peers[p]);
    const size_t slot = (size_t)a.rank * a.cap;                // rows of this rank in the peer's recv arrays
    int32_t* rid = reinterpret_cast<int32_t*>(peer + a.L.recv_ids) + slot * a.k;
    float* rw = reinterpret_cast<float*>(peer + a.L.recv_w) + slot * a.k;
    uint4* rx = reinterpret_cast<uint4*>(peer + a.L.recv_x + slot * a.H * 2);
    const int vec = a.H / 8;                                    // 16-byte vectors per row
    for (int i = i0; i < i1; ++i) {
        const bool valid = i < a.B;
        const bool any = valid && row_picks_rank(a.ids, i, a.k, p, per);
        for (int j = threadIdx.x; j < a.k; j += blockDim.x) {
            int e = valid ? a.ids[(size_t)i * a.k + j] : -1;
            e = (e >= p * per && e < (p + 1) * per) ? e - p * per : -1;
            rid[(size_t)i * a.k + j] = e;
            rw[(size_t)i * a.k + j] = valid ? a.w[(size_t)i * a.k + j] : 0.f;
        }
        if (any) {
            const uint4* src = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.x) + (size_t)i * a.ldx * 2);
            for (int v = threadIdx.x; v < vec; v += blockDim.x) rx[(size_t)i * vec + v] = src[v];
        }
    }
    __syncthreads();                                            // the CTA's peer stores, then one thread fences
    if (threadIdx.x != 0) return;                               // them at system scope and signals
    const int my = p * nch + c;                                 // this CTA's counter; also its incoming flag slot
    const uint32_t epoch = ctl->d_epoch[my] + 1;
    asm volatile("fence.acq_rel.sys;" ::: "memory");
    st_release_sys(&reinterpret_cast<EpCtl*>(peer)->dflag[a.rank * nch + c], epoch);
    if (!ep_wait_flags(&ctl->dflag[my], 1, 0, epoch)) report(a.status, EXL3_ERR_TIMEOUT);
    ctl->d_epoch[my] = epoch;
}

// grid (chunks, W): CTA (c, r) returns the rows of chunk c received from rank r that had a pick here, signals r, and
// waits for every rank's chunk c of this rank's rows; with `out`, the W CTAs of chunk c then sum its rows (a
// fixed rank order) into out (+ shared), as k_ep_reduce does.
__global__ void __launch_bounds__(kEpThreads) k_ep_combine(const EpArgs a, const float* shared, float* out) {
    pdl_wait();
    pdl_trigger();
    __shared__ int ok;
    EpCtl* ctl = reinterpret_cast<EpCtl*>(a.local);
    const int c = blockIdx.x, r = blockIdx.y, nch = gridDim.x;
    const int rpc = (a.cap + nch - 1) / nch;
    const int i0 = c * rpc, i1 = min(a.cap, i0 + rpc);
    uint8_t* peer = reinterpret_cast<uint8_t*>(a.peers[r]);
    const int32_t* myids = reinterpret_cast<const int32_t*>(a.local + a.L.recv_ids) + (size_t)r * a.cap * a.k;
    float4* dst = reinterpret_cast<float4*>(peer + a.L.back) + ((size_t)a.rank * a.cap) * (a.H / 4);
    const float4* src = reinterpret_cast<const float4*>(a.part) + ((size_t)r * a.cap) * (a.H / 4);
    const int vec = a.H / 4;
    for (int i = i0; i < i1; ++i) {
        bool any = false;
        for (int j = 0; j < a.k; ++j) any |= myids[(size_t)i * a.k + j] >= 0;
        if (!any) continue;                                    // block-uniform
        for (int v = threadIdx.x; v < vec; v += blockDim.x) dst[(size_t)i * vec + v] = src[(size_t)i * vec + v];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const int my = r * nch + c;
        const uint32_t epoch = ctl->c_epoch[my] + 1;
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        st_release_sys(&reinterpret_cast<EpCtl*>(peer)->cflag[a.rank * nch + c], epoch);
        // every rank's partial rows of this rank's chunk c: flags [q][c], q = 0..W-1
        ok = ep_wait_flags(&ctl->cflag[c], a.W, nch, epoch);   // acquire loads: their rows are visible after
        if (!ok) report(a.status, EXL3_ERR_TIMEOUT);
        ctl->c_epoch[my] = epoch;
    }
    if (out == nullptr) return;
    __syncthreads();
    if (!ok) return;
    // this rank's rows of chunk c (below B), shared by the W CTAs of the chunk
    const int per = a.E / a.W;
    const int b1 = min(a.B, i1);
    const long total = (long)max(0, b1 - i0) * vec;
    const float4* back = reinterpret_cast<const float4*>(a.local + a.L.back);
    for (long t = (long)r * blockDim.x + threadIdx.x; t < total; t += (long)a.W * blockDim.x) {
        const int i = i0 + (int)(t / vec), v = (int)(t % vec);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int q = 0; q < a.W; ++q) {
            if (!row_picks_rank(a.ids, i, a.k, q, per)) continue;
            const float4 b = back[((size_t)q * a.cap + i) * vec + v];
            acc.x += b.x; acc.y += b.y; acc.z += b.z; acc.w += b.w;
        }
        if (shared) {
            const float4 sh = reinterpret_cast<const float4*>(shared)[(size_t)i * vec + v];
            acc.x += sh.x; acc.y += sh.y; acc.z += sh.z; acc.w += sh.w;
        }
        reinterpret_cast<float4*>(out)[(size_t)i * vec + v] = acc;
    }
}

// out[i][:] = sum over ranks p (in order) that row i picked of back[p][i][:] (+ shared[i][:]); one float4 per thread.
__global__ void __launch_bounds__(kEpThreads) k_ep_reduce(const EpArgs a, const float* shared, float* out) {
    pdl_wait();
    pdl_trigger();
    const int vec = a.H / 4, per = a.E / a.W;
    const long total = (long)a.B * vec;
    const float4* back = reinterpret_cast<const float4*>(a.local + a.L.back);
    for (long t = (long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += (long)gridDim.x * blockDim.x) {
        const int i = (int)(t / vec), v = (int)(t % vec);
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int p = 0; p < a.W; ++p) {
            if (!row_picks_rank(a.ids, i, a.k, p, per)) continue;
            const float4 b = back[((size_t)p * a.cap + i) * vec + v];
            acc.x += b.x; acc.y += b.y; acc.z += b.z; acc.w += b.w;
        }
        if (shared) {
            const float4 s = reinterpret_cast<const float4*>(shared)[(size_t)i * vec + v];
            acc.x += s.x; acc.y += s.y; acc.z += s.z; acc.w += s.w;
        }
        reinterpret_cast<float4*>(out)[(size_t)i * vec + v] = acc;
    }
}

static int ep_common(EpArgs& a, const uint64_t* peers, void* local, int W, int rank, int cap, int H, int k, int E,
                     int B, const char* what) {
    EXL3_REQUIRE(peers && local && W >= 1 && W <= kEpMaxRanks && rank >= 0 && rank < W, EXL3_ERR_ARG,
                 "%s: bad ranks (W=%d rank=%d)", what, W, rank);
    EXL3_REQUIRE(cap > 0 && B >= 0 && B <= cap && H > 0 && H % 8 == 0 && k > 0 && E > 0 && E % W == 0, EXL3_ERR_ARG,
                 "%s: bad shape (cap=%d B=%d H=%d k=%d E=%d W=%d)", what, cap, B, H, k, E, W);
    a.peers = peers;
    a.local = static_cast<uint8_t*>(local);
    a.L = ep_layout(W, cap, H, k);
    a.W = W;
    a.rank = rank;
    a.cap = cap;
    a.H = H;
    a.k = k;
    a.E = E;
    a.B = B;
    a.status = device_status_ptr();
    return EXL3_OK;
}

// Chunks per peer: about two CTAs per SM over all peers, at most one per row, and W * chunks flag slots at most.
// Depends only on (cap, W) and the GPU model, so every rank of a launch cuts its rows the same way.
static int ep_chunks(int cap, int W) {
    int c = (2 * num_sms() + W - 1) / W;
    if (c > cap) c = cap;
    if (c > kEpMaxSlots / W) c = kEpMaxSlots / W;
    return c < 1 ? 1 : c;
}

}  // namespace exl3

using namespace exl3;

extern "C" {

size_t exl3_ep_buffer_bytes(int W, int cap, int H, int topk) {
    if (W < 1 || W > kEpMaxRanks || cap <= 0 || H <= 0 || topk <= 0) return 0;
    return ep_layout(W, cap, H, topk).total;
}

int exl3_ep_recv_offsets(int W, int cap, int H, int topk, size_t* recv_x, size_t* recv_ids, size_t* recv_w) {
    EXL3_REQUIRE(W >= 1 && W <= kEpMaxRanks && cap > 0 && H > 0 && topk > 0 && recv_x && recv_ids && recv_w,
                 EXL3_ERR_ARG, "exl3_ep_recv_offsets: bad arguments");
    const EpLayout L = ep_layout(W, cap, H, topk);
    *recv_x = L.recv_x;
    *recv_ids = L.recv_ids;
    *recv_w = L.recv_w;
    return EXL3_OK;
}

int exl3_ep_buffer_create(size_t bytes, void** ptr, void* ipc_handle) {
    EXL3_REQUIRE(ptr && ipc_handle && bytes >= kEpCtlBytes, EXL3_ERR_ARG, "exl3_ep_buffer_create: bad arguments");
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_buffer_create: cudaMalloc(%zu): %s", bytes,
                 cudaGetErrorString(e));
    e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p);
    if (e != cudaSuccess) {
        cudaFree(p);
        set_error("exl3_ep_buffer_create: %s", cudaGetErrorString(e));
        return EXL3_ERR_CUDA;
    }
    *ptr = p;
    return EXL3_OK;
}

int exl3_ep_buffer_open(const void* ipc_handle, void** peer_ptr) {
    EXL3_REQUIRE(ipc_handle && peer_ptr, EXL3_ERR_ARG, "exl3_ep_buffer_open: bad arguments");
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    cudaError_t e = cudaIpcOpenMemHandle(peer_ptr, h, cudaIpcMemLazyEnablePeerAccess);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_buffer_open: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_ep_buffer_close(void* peer_ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(peer_ptr);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_buffer_close: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_ep_buffer_free(void* ptr) {
    cudaError_t e = cudaFree(ptr);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_buffer_free: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_ep_dispatch(const void* x, int x_dtype, int ldx, int B, const int32_t* ids, const float* w, int topk, int E,
                     int H, int W, int rank, int cap, const uint64_t* peers, void* local, void* stream) {
    EpArgs a = {};
    int rc = ep_common(a, peers, local, W, rank, cap, H, topk, E, B, "exl3_ep_dispatch");
    if (rc) return rc;
    EXL3_REQUIRE(B == 0 || (x && ids && w), EXL3_ERR_ARG, "exl3_ep_dispatch: null pointer");
    EXL3_REQUIRE(x_dtype == EXL3_F16 || x_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "exl3_ep_dispatch: x dtype");
    EXL3_REQUIRE(ldx >= H && ldx % 8 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0, EXL3_ERR_ARG,
                 "exl3_ep_dispatch: x rows must be 16-byte aligned (ldx=%d)", ldx);
    a.x = x;
    a.x_bf16 = x_dtype == EXL3_BF16;
    a.ldx = ldx;
    a.ids = ids;
    a.w = w;
    cudaError_t e = launch_pdl(k_ep_dispatch, dim3(ep_chunks(cap, W), W), dim3(kEpThreads), 0,
                               static_cast<cudaStream_t>(stream), a);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_dispatch: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_ep_combine(const float* part, int topk, int E, int H, int W, int rank, int cap, const uint64_t* peers,
                    void* local, void* stream) {
    EpArgs a = {};
    int rc = ep_common(a, peers, local, W, rank, cap, H, topk, E, cap, "exl3_ep_combine");
    if (rc) return rc;
    EXL3_REQUIRE(part && (reinterpret_cast<uintptr_t>(part) & 15) == 0 && H % 4 == 0, EXL3_ERR_ARG,
                 "exl3_ep_combine: part must be 16-byte aligned");
    a.part = part;
    cudaError_t e = launch_pdl(k_ep_combine, dim3(ep_chunks(cap, W), W), dim3(kEpThreads), 0,
                               static_cast<cudaStream_t>(stream), a, static_cast<const float*>(nullptr),
                               static_cast<float*>(nullptr));
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_combine: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_ep_combine_reduce(const float* part, const int32_t* ids, int B, int topk, int E, int H, int W, int rank,
                           int cap, const float* shared, const uint64_t* peers, void* local, float* out,
                           void* stream) {
    EpArgs a = {};
    int rc = ep_common(a, peers, local, W, rank, cap, H, topk, E, B, "exl3_ep_combine_reduce");
    if (rc) return rc;
    EXL3_REQUIRE(part && (reinterpret_cast<uintptr_t>(part) & 15) == 0 && H % 4 == 0, EXL3_ERR_ARG,
                 "exl3_ep_combine_reduce: part must be 16-byte aligned");
    EXL3_REQUIRE(out && (reinterpret_cast<uintptr_t>(out) & 15) == 0 && (B == 0 || ids) &&
                     (reinterpret_cast<uintptr_t>(shared) & 15) == 0,
                 EXL3_ERR_ARG, "exl3_ep_combine_reduce: out / shared must be 16-byte aligned, ids non-null");
    a.part = part;
    a.ids = ids;
    cudaError_t e = launch_pdl(k_ep_combine, dim3(ep_chunks(cap, W), W), dim3(kEpThreads), 0,
                               static_cast<cudaStream_t>(stream), a, shared, out);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_combine_reduce: launch failed: %s",
                 cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_ep_reduce(const int32_t* ids, int B, int topk, int E, int H, int W, int rank, int cap, const float* shared,
                   void* local, float* out, void* stream) {
    EpArgs a = {};
    int rc = ep_common(a, reinterpret_cast<const uint64_t*>(local), local, W, rank, cap, H, topk, E, B,
                       "exl3_ep_reduce");
    if (rc) return rc;
    EXL3_REQUIRE(out && (B == 0 || ids), EXL3_ERR_ARG, "exl3_ep_reduce: null pointer");
    if (B == 0) return EXL3_OK;
    a.ids = ids;
    const long total = (long)B * (H / 4);
    long blocks = (total + kEpThreads - 1) / kEpThreads;
    if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
    cudaError_t e = launch_pdl(k_ep_reduce, dim3((unsigned)blocks), dim3(kEpThreads), 0,
                               static_cast<cudaStream_t>(stream), a, shared, out);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_ep_reduce: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

}  // extern "C"
