// Fused EXL3 decode GEMV for B200 (sm_100a): one kernel per linear (or per grouped MoE projection) that
//   1. rotates its k-range of the input rows (fp16(x*suh) -> warp FWHT-128 -> fp16) into shared memory,
//   2. streams its k-range of trellis tile-rows from HBM into a shared-memory ring with TMA bulk copies
//      (cp.async.bulk, one elected producer thread, mbarrier transaction counts; no tensor maps, no multicast),
//   3. decodes every 16x16 tile in registers straight into the A fragment of an m16n8k16 MMA (the EXL3 position
//      order is that fragment's layout) and accumulates W_hat^T x in fp32 on the tensor cores (one MMA per tile
//      replaces 256 FMAs; batch rows ride along in the MMA's 8 columns, so rows 1..8 cost the same decode),
//   4. reduces the split-K partials of a cluster through distributed shared memory in a fixed order
//      (deterministic, no global scratch), and
//   5. runs the epilogue on the complete 128-column block: output Hadamard x svh (linear), the gated-MLP
//      activation + the down projection's input rotation (MoE gate|up), or Hadamard x svh x routing weight (down).
//
// Reference semantics: exllamav3 exl3_gemm (glm/docs/ext-op-inventory.md:498-557), the XPU GemvKernel/HadIn/HadOut
// (glm/xpu/csrc/exl3_esimd.h:283-338,444-580) and the MoE GateUp/Down kernels (glm/xpu/csrc/exl3_moe.n128.sycl:
// 136-383). Work partition and data movement are this file's own.
#pragma once

#include "common.cuh"
#include "hadamard.cuh"
#include "trellis.cuh"

namespace exl3 {

enum { EPI_LINEAR = 0, EPI_GATEUP = 1, EPI_DOWN = 2 };

constexpr int kTilesPerCta = 8;     // 128 output columns per matrix per CTA (one Hadamard block)
constexpr int kMaxRows = 8;         // MMA N dimension: input rows per CTA
constexpr int kStages = 6;          // shared-memory ring depth
constexpr int kMaxCluster = 8;      // split-K CTAs per cluster (portable cluster size)
constexpr int kStageTarget = 6144;  // bytes of trellis per ring stage (sets tile-rows per stage)

// Expert descriptor (device table, one entry per expert; the shared expert is an ordinary entry).
struct ExpertDesc {
    const uint32_t* tr[3];      // gate, up, down trellis words [k/16][n/16][8K]
    const __half* suh[3];       // input signs/scales
    const __half* svh[3];       // output signs/scales
    int K[3];
    int pad;
};

// Grouped work produced by the alignment kernel: item i covers pair positions [start, start + cnt) of expert e.
struct ItemTable {
    const int* n_items;      // [1]
    const int* item_expert;  // [max_items]
    const int* item_start;   // [max_items]
    const int* item_cnt;     // [max_items], 1..8
    const int* pair_tok;     // [pairs] token of a pair position
    const float* pair_w;     // [pairs] routing weight of a pair position
};

struct GemvArgs {
    // EPI_LINEAR: one matrix
    const uint32_t* tr;
    const __half* suh;
    const __half* svh;
    int K;
    const void* x;          // [M, k] fp16/bf16 rows, row stride ldx elements
    int ldx;
    int x_bf16;
    void* y;                // [M, n] rows, row stride ldy elements
    int ldy;
    int y_dtype;            // EXL3_F16 / EXL3_BF16 / EXL3_F32
    int M;
    // EPI_GATEUP / EPI_DOWN: grouped experts
    const ExpertDesc* experts;
    ItemTable items;
    __half* abuf;           // [pairs, I] fp16 Hadamard-domain activations
    float* ybuf;            // [pairs, H] fp32 weighted down outputs
    float act_limit;
    // shape of the matrices this launch runs (gate|up: k = H, n = I; down: k = I, n = H)
    int k, n;
    int split;              // CTAs per cluster along k
    int* status;
};

__host__ __device__ __forceinline__ int rows_per_stage(int row_stride) {
    int r = kStageTarget / row_stride;
    return r < 1 ? 1 : (r > 16 ? 16 : r);
}

// Dynamic shared memory layout of one CTA. It depends only on launch-wide values (so every CTA of a cluster has
// `red` at the same offset, which the distributed-shared-memory reduction relies on):
//   xs   [nmat][8 rows][xs_ld] fp16   rotated input rows of this CTA's k range (xs_ld = klen + 8: bank-conflict pad)
//   ring [kStages][kStageTarget]     trellis tile-rows in flight
//   red  [nmat][8][128] fp32         this CTA's split-K partial of the 128-column block
//   bars full[kStages], empty[kStages]
struct Smem {
    int xs_ld, xs_off, ring_off, red_off, bar_off, total;
};
__host__ __device__ __forceinline__ Smem smem_layout(int nmat, int klen_alloc) {
    Smem s;
    s.xs_ld = klen_alloc + 8;
    s.xs_off = 0;
    const int xs = nmat * kMaxRows * s.xs_ld * 2;
    s.ring_off = (xs + 127) & ~127;
    s.red_off = s.ring_off + kStages * kStageTarget;
    s.bar_off = s.red_off + nmat * kMaxRows * 128 * 4;
    s.total = s.bar_off + 2 * kStages * 8;
    return s;
}

__host__ __device__ __forceinline__ int klen_alloc_of(int k, int split) {
    const int KB = k / 128;
    return ((KB + split - 1) / split) * 128;
}

// One warp's pass over its tile column of one matrix; templated on the bit width.
template <int K>
__device__ __forceinline__ void consume(float d[4], const uint8_t* ring, int stage_bytes, int row_stride,
                                        int mat_off, int tile, int n_rows, int rps, uint64_t* full,
                                        uint64_t* empty, const __half* xs, int xs_ld, int Mi, int lane,
                                        bool& timed_out) {
    const LaneWords lw = lane_words<K>(lane);
    const int g = lane >> 2, q = lane & 3;
    const bool has_row = g < Mi;
    const __half* xrow = xs + (size_t)(has_row ? g : 0) * xs_ld + 2 * q;
    const int n_iter = (n_rows + rps - 1) / rps;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % kStages;
        if (!timed_out && !mbar_wait(&full[s], (it / kStages) & 1)) timed_out = true;
        if (!timed_out) {
            const uint8_t* base = ring + (size_t)s * stage_bytes + mat_off + tile * 32 * K;
            const int rr_end = min(rps, n_rows - it * rps);
            for (int rr = 0; rr < rr_end; ++rr) {
                const int r = it * rps + rr;
                uint32_t a[4];
                decode_frag<K>(reinterpret_cast<const uint32_t*>(base + (size_t)rr * row_stride), lw, a);
                uint32_t b0 = 0, b1 = 0;
                if (has_row) {
                    b0 = *reinterpret_cast<const uint32_t*>(xrow + 16 * r);
                    b1 = *reinterpret_cast<const uint32_t*>(xrow + 16 * r + 8);
                }
                mma_16816(d, a, b0, b1);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

__device__ __forceinline__ void consume_k(int K, float d[4], const uint8_t* ring, int stage_bytes, int row_stride,
                                          int mat_off, int tile, int n_rows, int rps, uint64_t* full,
                                          uint64_t* empty, const __half* xs, int xs_ld, int Mi, int lane, bool& to) {
#define EXL3_CONSUME(KK) \
    consume<KK>(d, ring, stage_bytes, row_stride, mat_off, tile, n_rows, rps, full, empty, xs, xs_ld, Mi, lane, to)
    switch (K) {
        case 1: EXL3_CONSUME(1); break;
        case 2: EXL3_CONSUME(2); break;
        case 3: EXL3_CONSUME(3); break;
        case 4: EXL3_CONSUME(4); break;
        case 5: EXL3_CONSUME(5); break;
        case 6: EXL3_CONSUME(6); break;
        case 7: EXL3_CONSUME(7); break;
        default: EXL3_CONSUME(8); break;
    }
#undef EXL3_CONSUME
}

__device__ __forceinline__ float silu_f(float g) { return g / (1.0f + expf(-g)); }

// Grid: blockIdx.x = unit * split + p, cluster (split, 1, 1). Block: (nmat*8 + 1) warps; the last is the producer.
template <int EPI, typename TIn>
__global__ void __launch_bounds__((EPI == EPI_GATEUP ? 17 : 9) * 32) k_gemv(const GemvArgs args) {
    constexpr int NMAT = EPI == EPI_GATEUP ? 2 : 1;
    constexpr int NCONS = NMAT * kTilesPerCta;     // consumer warps
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int P = args.split;
    const int p = blockIdx.x % P;
    const int unit = blockIdx.x / P;
    const int NB = args.n / 128;
    const int cb = unit % NB;

    // ---- work unit: matrices, rows ----
    const uint32_t* tr[NMAT];
    const __half* suh[NMAT];
    const __half* svh[NMAT];
    int Kb[NMAT];
    int Mi, s0 = 0, expert = 0;
    if constexpr (EPI == EPI_LINEAR) {
        tr[0] = args.tr; suh[0] = args.suh; svh[0] = args.svh; Kb[0] = args.K;
        Mi = args.M;
    } else {
        const int item = unit / NB;
        if (item >= *args.items.n_items) return;              // uniform over the cluster
        expert = args.items.item_expert[item];
        s0 = args.items.item_start[item];
        Mi = args.items.item_cnt[item];
        const ExpertDesc& ed = args.experts[expert];
        if constexpr (EPI == EPI_GATEUP) {
#pragma unroll
            for (int m = 0; m < 2; ++m) { tr[m] = ed.tr[m]; suh[m] = ed.suh[m]; svh[m] = ed.svh[m]; Kb[m] = ed.K[m]; }
        } else {
            tr[0] = ed.tr[2]; suh[0] = nullptr; svh[0] = ed.svh[2]; Kb[0] = ed.K[2];
        }
    }

    // ---- k range of this CTA (whole 128-blocks) ----
    const int KB = args.k / 128;
    const int kb0 = (p * KB) / P, kb1 = ((p + 1) * KB) / P;
    const int n_rows = (kb1 - kb0) * 8;                       // tile-rows
    const int r0 = kb0 * 8;
    const int TN = args.n / 16;

    int row_stride = 0, mat_off[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) { mat_off[m] = row_stride; row_stride += kTilesPerCta * 32 * Kb[m]; }
    const int rps = rows_per_stage(row_stride);
    const int stage_bytes = rps * row_stride;             // <= kStageTarget (row_stride <= 4096)
    const Smem L = smem_layout(NMAT, klen_alloc_of(args.k, P));
    const int xs_ld = L.xs_ld;
    __half* xs = reinterpret_cast<__half*>(smem + L.xs_off);
    uint8_t* ring = smem + L.ring_off;
    float* red = reinterpret_cast<float*>(smem + L.red_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* empty = full + kStages;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], NCONS); }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == NCONS) {
        // ---------------- producer: stream tile-rows into the ring ----------------
        if (lane == 0) {
            const int n_iter = (n_rows + rps - 1) / rps;
            bool to = false;
            int last_issue[kStages];
            for (int s = 0; s < kStages; ++s) last_issue[s] = -1;
            for (int it = 0; it < n_iter && !to; ++it) {
                const int s = it % kStages;
                if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1)) { to = true; break; }
                const int rows = min(rps, n_rows - it * rps);
                mbar_expect_tx(&full[s], rows * row_stride);
                uint8_t* dst = ring + (size_t)s * stage_bytes;
                for (int rr = 0; rr < rows; ++rr) {
                    const int rg = r0 + it * rps + rr;
#pragma unroll
                    for (int m = 0; m < NMAT; ++m) {
                        const uint32_t* src = tr[m] + ((size_t)rg * TN + (size_t)cb * kTilesPerCta) * (8 * Kb[m]);
                        bulk_g2s(dst + (size_t)rr * row_stride + mat_off[m], src, kTilesPerCta * 32 * Kb[m], &full[s]);
                    }
                }
                last_issue[s] = it;
            }
            if (to) report(args.status, EXL3_ERR_TIMEOUT);
            // every issued copy has landed before the CTA can retire its shared memory
            for (int s = 0; s < kStages; ++s)
                if (last_issue[s] >= 0 && !mbar_wait(&full[s], (last_issue[s] / kStages) & 1))
                    report(args.status, EXL3_ERR_TIMEOUT);
        }
    } else {
        // ---------------- consumers ----------------
        // 1. input rows -> shared memory (rotated unless already in the Hadamard domain)
        const int nblk = kb1 - kb0;
        const int jobs = NMAT * Mi * nblk;
        for (int j = warp; j < jobs; j += NCONS) {
            const int m = j / (Mi * nblk);
            const int row = (j / nblk) % Mi;
            const int kb = kb0 + j % nblk;
            __half* dst = xs + ((size_t)m * kMaxRows + row) * xs_ld + (kb - kb0) * 128;
            if constexpr (EPI == EPI_DOWN) {
                const __half* src = args.abuf + (size_t)(s0 + row) * args.k + kb * 128;
                *reinterpret_cast<uint2*>(dst + 4 * lane) = *reinterpret_cast<const uint2*>(src + 4 * lane);
            } else {
                size_t xrow;
                if constexpr (EPI == EPI_LINEAR) xrow = (size_t)row * args.ldx;
                else xrow = (size_t)args.items.pair_tok[s0 + row] * args.ldx;
                const __half* su = suh[m] ? suh[m] + kb * 128 : nullptr;
                if (args.x_bf16) {
                    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(args.x) + xrow + kb * 128;
                    had_in_block<__nv_bfloat16>(src, su, dst, lane);
                } else {
                    const __half* src = reinterpret_cast<const __half*>(args.x) + xrow + kb * 128;
                    had_in_block<__half>(src, su, dst, lane);
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(NCONS * 32) : "memory");

        // 2. main loop
        const int m = warp / kTilesPerCta, tile = warp % kTilesPerCta;
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        bool to = false;
        consume_k(Kb[m], d, ring, stage_bytes, row_stride, mat_off[m], tile, n_rows, rps, full, empty,
                  xs + (size_t)m * kMaxRows * xs_ld, xs_ld, Mi, lane, to);
        if (to) report(args.status, EXL3_ERR_TIMEOUT);

        // 3. partial tile -> red[m][row][col]: d = D[n][row] with n = g, g+8 and row = 2q, 2q+1
        const int g = lane >> 2, q = lane & 3;
        float* rm = red + (size_t)m * kMaxRows * 128;
        const int c0 = tile * 16 + g;
        rm[(2 * q) * 128 + c0] = d[0];
        rm[(2 * q + 1) * 128 + c0] = d[1];
        rm[(2 * q) * 128 + c0 + 8] = d[2];
        rm[(2 * q + 1) * 128 + c0 + 8] = d[3];
    }

    // ---- split-K reduction across the cluster (fixed order) + epilogue ----
    __syncwarp();
    if (P > 1) cluster_sync_all(); else __syncthreads();

    if (warp < kMaxRows) {
        const int row = p + warp * P;
        if (row < Mi) {
            float v[NMAT][4];
#pragma unroll
            for (int m = 0; m < NMAT; ++m) {
                v[m][0] = v[m][1] = v[m][2] = v[m][3] = 0.f;
                const float* src = red + ((size_t)m * kMaxRows + row) * 128 + 4 * lane;
                for (int c = 0; c < P; ++c) {
                    float4 t;
                    if (P > 1) t = ld_dsmem_f4(map_shared_rank(src, c));
                    else t = *reinterpret_cast<const float4*>(src);
                    v[m][0] += t.x; v[m][1] += t.y; v[m][2] += t.z; v[m][3] += t.w;
                }
                fwht128_warp(v[m], lane);
            }
            const int col = cb * 128 + 4 * lane;
            if constexpr (EPI == EPI_LINEAR) {
                float o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float sv = __half2float(svh[0][col + j]);
                    if (args.y_dtype == EXL3_F16)
                        o[j] = __half2float(__float2half_rn(__half2float(__float2half_rn(v[0][j] * kRsqrt128)) * sv));
                    else
                        o[j] = v[0][j] * kRsqrt128 * sv;
                }
                if (args.y_dtype == EXL3_F32) {
                    float* yp = reinterpret_cast<float*>(args.y) + (size_t)row * args.ldy + col;
                    *reinterpret_cast<float4*>(yp) = make_float4(o[0], o[1], o[2], o[3]);
                } else if (args.y_dtype == EXL3_F16) {
                    __half* yp = reinterpret_cast<__half*>(args.y) + (size_t)row * args.ldy + col;
                    __half2 h01 = __floats2half2_rn(o[0], o[1]), h23 = __floats2half2_rn(o[2], o[3]);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t*>(&h01);
                    u.y = *reinterpret_cast<uint32_t*>(&h23);
                    *reinterpret_cast<uint2*>(yp) = u;
                } else {
                    __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(args.y) + (size_t)row * args.ldy + col;
#pragma unroll
                    for (int j = 0; j < 4; ++j) yp[j] = __float2bfloat16_rn(o[j]);
                }
            } else if constexpr (EPI == EPI_GATEUP) {
                const ExpertDesc& ed = args.experts[expert];
                const float L = args.act_limit;
                float a[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    // gate/up outputs rounded to fp16 as the fp16 linear does: fp16(fp16(H(acc)*r) * svh)
                    float gg = __half2float(__float2half_rn(
                        __half2float(__float2half_rn(v[0][j] * kRsqrt128)) * __half2float(svh[0][col + j])));
                    float uu = __half2float(__float2half_rn(
                        __half2float(__float2half_rn(v[1][j] * kRsqrt128)) * __half2float(svh[1][col + j])));
                    float s = silu_f(gg);
                    if (L != 0.f) { s = fminf(s, L); uu = fminf(fmaxf(uu, -L), L); }
                    float act = __half2float(__float2half_rn(s * uu));
                    a[j] = __half2float(__float2half_rn(act * __half2float(ed.suh[2][col + j])));
                }
                fwht128_warp(a, lane);
                __half* dst = args.abuf + (size_t)(s0 + row) * args.n + col;
                __half2 h01 = __floats2half2_rn(a[0] * kRsqrt128, a[1] * kRsqrt128);
                __half2 h23 = __floats2half2_rn(a[2] * kRsqrt128, a[3] * kRsqrt128);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&h01);
                u.y = *reinterpret_cast<uint32_t*>(&h23);
                *reinterpret_cast<uint2*>(dst) = u;
            } else {
                const float w = args.items.pair_w[s0 + row];
                float o[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) o[j] = w * (v[0][j] * kRsqrt128 * __half2float(svh[0][col + j]));
                float* dst = args.ybuf + (size_t)(s0 + row) * args.n + col;
                *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
            }
        }
    }
    if (P > 1) cluster_sync_all();
}

}  // namespace exl3

// ------------------------------------------------------------------------------------------------ host launch

namespace exl3 {

// Split-K CTAs per cluster: enough CTAs for two waves of SMs, within the portable cluster size, at least the number
// that keeps the rotated-input buffer inside shared memory.
inline int choose_split(int units, int k, int nmat, int requested) {
    const int KB = k / 128;
    const int cap = KB < kMaxCluster ? KB : kMaxCluster;
    int P = requested > 0 ? requested : (2 * num_sms() + units - 1) / (units > 0 ? units : 1);
    if (P < 1) P = 1;
    if (P > cap) P = cap;
    while (P < cap && smem_layout(nmat, klen_alloc_of(k, P)).total > 200 * 1024) ++P;
    return P;
}

template <int EPI, typename TIn>
int launch_gemv(const GemvArgs& a, int units, cudaStream_t st, const char* what) {
    constexpr int NMAT = EPI == EPI_GATEUP ? 2 : 1;
    const Smem L = smem_layout(NMAT, klen_alloc_of(a.k, a.split));
    EXL3_REQUIRE(L.total <= 227 * 1024, EXL3_ERR_UNSUPPORTED, "%s: k=%d too large for split %d", what, a.k, a.split);
    auto kern = k_gemv<EPI, TIn>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && configured[dev] < L.total) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
            set_error("%s: cudaFuncSetAttribute: %s", what, cudaGetErrorString(cudaGetLastError()));
            return EXL3_ERR_CUDA;
        }
        configured[dev] = 227 * 1024;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(units * a.split, 1, 1);
    cfg.blockDim = dim3((NMAT * kTilesPerCta + 1) * 32, 1, 1);
    cfg.dynamicSmemBytes = L.total;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    if (a.split > 1) {
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = a.split;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
    if (e != cudaSuccess) {
        set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
        return EXL3_ERR_CUDA;
    }
    return EXL3_OK;
}

}  // namespace exl3
