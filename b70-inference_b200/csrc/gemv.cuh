// Fused EXL3 decode GEMV for B200 (sm_100a).
//
// Weights use the column-block-major trellis layout of this library ("packed"): for every 128-column block cb and
// tile-row r (16 input rows) the 8 tiles of that block are contiguous, [n/128][k/16][8 tiles][8K words]; a fused
// gate|up pair stores both matrices' 8 tiles per (cb, r), [I/128][H/16][gate 8 tiles | up 8 tiles]. It is a
// permutation of exllamav3's [k/16][n/16][16K] int16 trellis (same bytes), made once at load time (exl3_pack), so
// that the slice one CTA streams, (cb, tile-rows r0..r1), is ONE contiguous range: the producer moves it with a few
// large TMA bulk copies (cp.async.bulk, 8 KB stages, up to 128 KB in flight per CTA; no tensor maps, no multicast).
//
// Activations arrive pre-rotated in "xf" order (exl3 prep kernel, or the gate|up epilogue for the down projection):
// a = fp16(H(fp16(x*suh))/sqrt(128)) (exllamav3's roundings), stored per (row, 16-input tile-row) as 4 quads x 4 fp16
// {a[2q], a[2q+1], a[2q+8], a[2q+9]}: exactly the two registers of the m16n8k16 MMA B fragment of lane quad q.
//
// Decode (glm/docs/ext-op-inventory.md:559-574): the weight's 16-bit state times 0x83DCD12D, byte sum + 0x6400 by
// dp4a = fp16 bits of 1024 + bytesum, then fma.rn.f16x2 with the fp16 constants 0x1EEE / 0xC931: the reference's fp16
// weight, bit for bit, written straight into the MMA A fragment (the EXL3 position order is that fragment's layout:
// lane 4g+q owns positions 8l..8l+7, so no shuffles). One m16n8k16 MMA per 16x16 tile accumulates in fp32; batch
// rows ride in the MMA's 8 columns, so rows 1..8 cost the same decode. On sm_100 the legacy MMA issue cost per tile
// is what matters: one fp16 MMA per tile stays far from the tensor pipe's limit.
//
// One CTA = work unit (item x 128-column block x split-K part), made of KI independent k-groups; group ki streams a
// contiguous, block-aligned share of the CTA's tile-rows:
//   warp 0 of a group  (producer) streams its share into its part of the shared-memory ring;
//   warps 1..          consumers, one per tile group (TPW tiles of one matrix): decode, int8 MMAs, fold int32 -> fp32
//                      at every 128-block boundary with the block scales;
//   epilogue           fixed-order sum over the groups and over the cluster's split-K CTAs (distributed shared
//                      memory), then
//                      the output Hadamard x svh (linear), the gated-MLP activation + the down projection's input
//                      (MoE gate|up), or Hadamard x svh x routing weight (MoE down).
// Launched with programmatic stream serialization: the producer starts streaming weights while the previous kernel
// finishes; consumers execute griddepcontrol.wait before reading activations.
//
// Reference semantics: exllamav3 exl3_gemm (glm/docs/ext-op-inventory.md:498-557; its int8-activation GEMV,
// :539-549, uses the same byte-sum identity on dp4a), the XPU GemvKernel/HadIn/HadOut (glm/xpu/csrc/exl3_esimd.h:
// 283-338,444-580) and the MoE GateUp/Down kernels (glm/xpu/csrc/exl3_moe.n128.sycl:136-383). Work partition, the
// tensor-core byte sum, the packed layout and the data movement are this file's own.
#pragma once

#include "common.cuh"
#include "hadamard.cuh"
#include "trellis.cuh"

namespace exl3 {

enum { EPI_LINEAR = 0, EPI_GATEUP = 1, EPI_DOWN = 2 };

constexpr int kTilesPerCta = 8;     // 128 output columns per matrix per CTA (one Hadamard block)
constexpr int kMaxRows = 8;         // MMA N dimension: input rows per CTA
constexpr int kMaxCluster = 8;      // split-K CTAs per cluster (portable cluster size)
constexpr int kStageBytes = 8192;   // ring stage (one bulk copy)
constexpr int kMaxStages = 16;      // up to 128 KB in flight per CTA
constexpr int kMaxWarps = 28;       // warps of a one-CTA-per-SM launch (KI groups of 1 producer + tile-group consumers)

__host__ __device__ constexpr int tiles_per_warp(int) { return 2; }
__host__ __device__ constexpr int nmat_of(int epi) { return epi == EPI_GATEUP ? 2 : 1; }
__host__ __device__ constexpr int tile_groups(int epi) { return nmat_of(epi) * kTilesPerCta / tiles_per_warp(epi); }
// k-groups per CTA: independent pipelines (producer warp + one consumer warp per tile group), each streaming its own
// contiguous, block-aligned share of the CTA's tile-rows through its own part of the ring
__host__ __device__ constexpr int max_ki(int epi) { return kMaxWarps / (tile_groups(epi) + 1); }

// Expert descriptor (device table, one entry per expert; the shared expert is an ordinary entry).
// tr[0] = packed gate|up [I/128][H/16][8 gate tiles | 8 up tiles], tr[1] unused, tr[2] = packed down.
struct ExpertDesc {
    const uint32_t* tr[3];
    const __half* suh[3];       // input signs/scales (gate, up, down)
    const __half* svh[3];       // output signs/scales
    int K[3];
    int pad;
};

// Grouped work produced by the alignment kernel: item i covers pair positions [start, start + cnt) of expert e.
struct ItemTable {
    const int* n_items;      // [1]
    const int* item_expert;  // [max_items]
    const int* item_start;   // [max_items]
    const int* item_cnt;     // [max_items], 1..rows_max
    const int* pair_tok;     // [pairs] token of a pair position
    const float* pair_w;     // [pairs] routing weight of a pair position
};

struct GemvArgs {
    // EPI_LINEAR: one packed matrix
    const uint32_t* tr;
    const __half* svh;
    int K;
    void* y;                // [M, n] rows, row stride ldy elements
    int ldy;
    int y_dtype;            // EXL3_F16 / EXL3_BF16 / EXL3_F32
    int M;
    // EPI_GATEUP / EPI_DOWN: grouped experts
    const ExpertDesc* experts;
    ItemTable items;
    float* ybuf;            // [pairs, H] fp32 weighted down outputs
    float act_limit;
    // activations in xf order: input rows (linear: row m; gate|up: pair position x matrix; down: pair position)
    const __half* xf;       // [rows][nmat][k] (k in xf order within each tile-row)
    __half* xf_out;         // gate|up only: the down input in xf order [pairs][I]
    // shape of the matrices this launch runs (gate|up: k = H, n = I; down: k = I, n = H)
    int k, n;
    int split;              // CTAs per cluster along k
    int stages;             // ring stages (<= kMaxStages)
    int* status;
};

__host__ __device__ __forceinline__ int klen_alloc_of(int k, int split) {
    const int KB = k / 128;
    return ((KB + split - 1) / split) * 128;
}

// Dynamic shared memory: red [KI][nmat][8][128] fp32 at offset 0 (the same in every CTA of a cluster, read through
// distributed shared memory), bars full/empty [kMaxStages] each, then the ring [stages][kStageBytes].
struct Smem {
    int red_off, bar_off, ring_off, total;
};
__host__ __device__ __forceinline__ Smem smem_layout(int epi, int KI, int stages) {
    Smem s;
    s.red_off = 0;
    s.bar_off = KI * nmat_of(epi) * kMaxRows * 128 * 4;
    s.ring_off = (s.bar_off + 2 * kMaxStages * 8 + 127) & ~127;
    s.total = s.ring_off + stages * kStageBytes;
    return s;
}

// Optional per-CTA timeline for performance investigation: a harness that defines EXL3_TRACE before including this
// file provides `exl3_trace_point(slot)`, which records the global timer; otherwise the hooks compile to nothing.
#ifdef EXL3_TRACE
#define EXL3_TRACE_POINT(slot) exl3_trace_point(slot)
#else
#define EXL3_TRACE_POINT(slot)
#endif

// ---- programmatic dependent launch ----
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}

// Store one rotated 128-block (lane l holds k = 4l..4l+3) in xf order: tile-row r = l/4, quad q, slot idx with
// k16 = 2q -> 0, 2q+1 -> 1, 2q+8 -> 2, 2q+9 -> 3.
__device__ __forceinline__ void store_xf_block(const float v[4], int lane, __half* xf_blk) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int kl = 4 * lane + j;
        const int r = kl >> 4, k16 = kl & 15;
        const int qq = (k16 & 7) >> 1;
        const int idx = ((k16 >> 3) << 1) | (k16 & 1);
        xf_blk[r * 16 + qq * 4 + idx] = __float2half_rn(v[j]);
    }
}

// The lane's 4 rotated activations of one 128-block, as the fp16 values the reference computes (returned widened).
template <typename TIn>
__device__ __forceinline__ void rotated_block(const TIn* x, const __half* suh, int lane, float v[4]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float p = to_f32<TIn>(x[4 * lane + j]) * (suh ? __half2float(suh[4 * lane + j]) : 1.0f);
        v[j] = __half2float(__float2half_rn(p));
    }
    fwht128_warp(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = __half2float(__float2half_rn(v[j] * kRsqrt128));
}

// One consumer warp: its TPW tiles of one matrix over the group's tile-rows (all of every stage of the group).
// d[t] = D[16 n x 8 rows] of tile t: d[0], d[1] = (n = g, rows 2q, 2q+1), d[2], d[3] = (n = g + 8, rows 2q, 2q+1).
template <int K, int TPW>
__device__ __forceinline__ void consume(float d[TPW][4], const uint8_t* ring, int n_stages, int row_stride,
                                        int mat_off, int tile0, int n_rows, int rps, uint64_t* full,
                                        uint64_t* empty, const __half* xf_row, int xf_row_stride, int Mi, int lane,
                                        bool& timed_out) {
    const LaneWords lw = lane_words<K>(lane);
    const int g = lane >> 2, q = lane & 3;
    const bool has_row = g < Mi;
    // B fragment of tile-row r for this lane: 8 bytes at xf_row + g * stride + r * 16 + q * 4
    const uint2* bp = reinterpret_cast<const uint2*>(xf_row + (size_t)(has_row ? g : 0) * xf_row_stride + q * 4);
    uint2 bn = make_uint2(0, 0);
    if (has_row && n_rows > 0) bn = __ldg(bp);
    const int n_iter = (n_rows + rps - 1) / rps;
    int r = 0;
    for (int it = 0; it < n_iter; ++it) {
        const int s = it % n_stages;
        if (!timed_out && !mbar_wait(&full[s], (it / n_stages) & 1)) timed_out = true;
        if (!timed_out) {
            const int rows = min(rps, n_rows - it * rps);
            const uint8_t* base = ring + (size_t)s * kStageBytes + mat_off + tile0 * 32 * K;
            for (int rr = 0; rr < rows; ++rr, ++r, base += row_stride) {
                const uint2 b = bn;
                if (has_row && r + 1 < n_rows) bn = __ldg(bp + (size_t)(r + 1) * 4);   // next row's fragment
#pragma unroll
                for (int t = 0; t < TPW; ++t) {
                    uint32_t a[4];
                    decode_frag<K>(reinterpret_cast<const uint32_t*>(base + t * 32 * K), lw, a);
                    mma_16816(d[t], a, b.x, b.y);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
}

template <int TPW>
__device__ __forceinline__ void consume_k(int K, float d[TPW][4], const uint8_t* ring, int n_stages,
                                          int row_stride, int mat_off, int tile0, int n_rows, int rps,
                                          uint64_t* full, uint64_t* empty, const __half* xf_row, int xf_row_stride,
                                          int Mi, int lane, bool& to) {
#define EXL3_CONSUME(KK)                                                                                          \
    consume<KK, TPW>(d, ring, n_stages, row_stride, mat_off, tile0, n_rows, rps, full, empty, xf_row,             \
                     xf_row_stride, Mi, lane, to)
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

// Grid: blockIdx.x = unit * split + p, cluster (split, 1, 1). Block: KI groups of (1 producer + tile_groups(EPI)) warps.
template <int EPI>
__global__ void __launch_bounds__(kMaxWarps * 32, 1) k_gemv(const GemvArgs args) {
    constexpr int NMAT = nmat_of(EPI);
    constexpr int TPW = tiles_per_warp(EPI);
    constexpr int NTG = tile_groups(EPI);
    constexpr int TG_PER_MAT = NTG / NMAT;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KI = (int)(blockDim.x >> 5) / (NTG + 1);
    const int grp = warp / (NTG + 1), wig = warp % (NTG + 1);
    if (threadIdx.x == 0) EXL3_TRACE_POINT(0);
    pdl_trigger();
    const int P = args.split;
    const int p = blockIdx.x % P;
    const int unit = blockIdx.x / P;
    const int NB = args.n / 128;
    const int cb = unit % NB;
    const int KB = args.k / 128;

    // ---- work unit: packed weights, rows ----
    const uint8_t* wbase;
    const __half* svh[NMAT];
    int Kb[NMAT];
    int Mi, s0 = 0, expert = 0;
    if constexpr (EPI == EPI_LINEAR) {
        wbase = reinterpret_cast<const uint8_t*>(args.tr);
        svh[0] = args.svh;
        Kb[0] = args.K;
        Mi = args.M;
    } else {
        // the item table comes from the alignment kernel, complete before the kernel this one overlaps with
        const int item = unit / NB;
        if (item >= *args.items.n_items) return;              // uniform over the cluster
        expert = args.items.item_expert[item];
        s0 = args.items.item_start[item];
        Mi = args.items.item_cnt[item];
        const ExpertDesc& ed = args.experts[expert];
        if constexpr (EPI == EPI_GATEUP) {
            wbase = reinterpret_cast<const uint8_t*>(ed.tr[0]);
            svh[0] = ed.svh[0];
            svh[NMAT - 1] = ed.svh[1];
            Kb[0] = ed.K[0];
            Kb[NMAT - 1] = ed.K[1];
        } else {
            wbase = reinterpret_cast<const uint8_t*>(ed.tr[2]);
            svh[0] = ed.svh[2];
            Kb[0] = ed.K[2];
        }
    }
    int row_stride = 0, mat_off[NMAT];
#pragma unroll
    for (int m = 0; m < NMAT; ++m) { mat_off[m] = row_stride; row_stride += kTilesPerCta * 32 * Kb[m]; }

    // ---- k range of this CTA (whole 128-blocks), this group's contiguous share, its slice of the packed weights ----
    const int kb0 = (p * KB) / P, kb1 = ((p + 1) * KB) / P;
    const int per_grp = (kb1 - kb0 + KI - 1) / KI;             // blocks per group
    const int g_kb0 = min(kb1, kb0 + grp * per_grp), g_kb1 = min(kb1, g_kb0 + per_grp);
    const int n_rows = (g_kb1 - g_kb0) * 8;                    // this group's tile-rows
    const int rps = kStageBytes / row_stride;                 // tile-rows per stage (row_stride <= 4096)
    const int n_stages = args.stages / KI;                     // this group's ring stages
    const uint8_t* slice = wbase + ((size_t)cb * (KB * 8) + (size_t)g_kb0 * 8) * row_stride;

    const Smem L = smem_layout(EPI, KI, args.stages);
    float* red = reinterpret_cast<float*>(smem + L.red_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off) + grp * n_stages;
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.bar_off) + kMaxStages + grp * n_stages;
    uint8_t* ring = smem + L.ring_off + (size_t)grp * n_stages * kStageBytes;

    if (wig == 0 && lane == 0) {
        for (int s = 0; s < n_stages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], NTG); }
        fence_barrier_init();
    }
    __syncthreads();

    if (wig == 0) {
        // ---------------- producer: the slice, stage by stage ----------------
        if (lane == 0) {
            const int n_iter = (n_rows + rps - 1) / rps;
            bool to = false;
            int last_issue[kMaxStages];
            for (int s = 0; s < kMaxStages; ++s) last_issue[s] = -1;
            for (int it = 0; it < n_iter && !to; ++it) {
                const int s = it % n_stages;
                if (it >= n_stages && !mbar_wait(&empty[s], ((it / n_stages) - 1) & 1)) { to = true; break; }
                const uint32_t bytes = (uint32_t)(min(rps, n_rows - it * rps) * row_stride);
                mbar_expect_tx(&full[s], bytes);
                bulk_g2s(ring + (size_t)s * kStageBytes, slice + (size_t)it * rps * row_stride, bytes, &full[s]);
                last_issue[s] = it;
            }
            EXL3_TRACE_POINT(7);
            if (to) report(args.status, EXL3_ERR_TIMEOUT);
            // every issued copy has landed before the CTA can retire its shared memory
            for (int s = 0; s < n_stages; ++s)
                if (last_issue[s] >= 0 && !mbar_wait(&full[s], (last_issue[s] / n_stages) & 1))
                    report(args.status, EXL3_ERR_TIMEOUT);
        }
    } else {
        // ---------------- consumers ----------------
        const int tg = wig - 1;
        const int m = tg / TG_PER_MAT, tile0 = (tg % TG_PER_MAT) * TPW;
        const int g = lane >> 2, q = lane & 3;
        pdl_wait();                                           // activations come from the previous kernel
        if (threadIdx.x == 32) EXL3_TRACE_POINT(1);
        // xf rows: linear -> row m; gate|up -> pair position (s0 + row), matrix m; down -> pair position
        const size_t row_elems = (size_t)NMAT * args.k;
        const size_t row0 = (EPI == EPI_LINEAR) ? 0 : (size_t)s0;
        const __half* xf_row = args.xf + row0 * row_elems + (size_t)m * args.k + (size_t)g_kb0 * 128;
        float d[TPW][4];
#pragma unroll
        for (int t = 0; t < TPW; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) d[t][e] = 0.f;
        bool to = false;
        consume_k<TPW>(Kb[m], d, ring, n_stages, row_stride, mat_off[m], tile0, n_rows, rps, full, empty, xf_row,
                       (int)row_elems, Mi, lane, to);
        if (to) report(args.status, EXL3_ERR_TIMEOUT);
        if (lane == 0 && warp == 1) EXL3_TRACE_POINT(3);
        float* rm = red + ((size_t)grp * NMAT + m) * kMaxRows * 128;
#pragma unroll
        for (int t = 0; t < TPW; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int row = 2 * q + (e & 1);
                const int col = (tile0 + t) * 16 + g + ((e >> 1) << 3);
                rm[row * 128 + col] = d[t][e];
            }
    }

    // ---- reduction over ki and the cluster's split-K CTAs (fixed order) + epilogue ----
    __syncwarp();
    if (P > 1) cluster_sync_all(); else __syncthreads();
    if (threadIdx.x == 0) EXL3_TRACE_POINT(5);

    const int nwarps = blockDim.x >> 5;
    for (int row = p + warp * P; row < Mi; row += nwarps * P) {
        float v[NMAT][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            v[m][0] = v[m][1] = v[m][2] = v[m][3] = 0.f;
            for (int c = 0; c < P; ++c)
                for (int k2 = 0; k2 < KI; ++k2) {
                    const float* src = red + (((size_t)k2 * NMAT + m) * kMaxRows + row) * 128 + 4 * lane;
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
            const float Lc = args.act_limit;
            float a[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                // gate/up outputs rounded to fp16 as the fp16 linear does: fp16(fp16(H(acc)*r) * svh)
                float gg = __half2float(__float2half_rn(
                    __half2float(__float2half_rn(v[0][j] * kRsqrt128)) * __half2float(svh[0][col + j])));
                float uu = __half2float(__float2half_rn(
                    __half2float(__float2half_rn(v[NMAT - 1][j] * kRsqrt128)) *
                    __half2float(svh[NMAT - 1][col + j])));
                float sg = silu_f(gg);
                if (Lc != 0.f) { sg = fminf(sg, Lc); uu = fminf(fmaxf(uu, -Lc), Lc); }
                const float act = __half2float(__float2half_rn(sg * uu));
                a[j] = __half2float(__float2half_rn(act * __half2float(ed.suh[2][col + j])));
            }
            fwht128_warp(a, lane);
#pragma unroll
            for (int j = 0; j < 4; ++j) a[j] = a[j] * kRsqrt128;
            // the down projection's input block cb, straight into xf order
            store_xf_block(a, lane, args.xf_out + (size_t)(s0 + row) * args.n + (size_t)cb * 128);
        } else {
            const float w = args.items.pair_w[s0 + row];
            float o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) o[j] = w * (v[0][j] * kRsqrt128 * __half2float(svh[0][col + j]));
            float* dst = args.ybuf + (size_t)(s0 + row) * args.n + col;
            *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
    __syncwarp();
    if (P > 1) cluster_sync_all();
    if (threadIdx.x == 0) EXL3_TRACE_POINT(6);
}

// ------------------------------------------------------------------------------------------------ activation prep

// xf of input rows: job = (row, matrix, 128-block), one warp each. x rows are fp16/bf16 at row stride ldx; row_tok
// (optional) maps an xf row to its x row (MoE pair position -> token) and row_expert (optional) selects the suh of the
// picked expert's matrix; otherwise suh0 is shared by all rows.
struct PrepArgs {
    const void* x;
    int ldx;
    int x_bf16;
    int rows, nmat, k;
    const __half* suh0;
    const int* row_tok;
    const int* row_expert;
    const ExpertDesc* experts;
    const int* n_rows_dev;        // optional device count of valid rows (MoE: valid pair positions + shared rows)
    __half* xf;                   // [rows][nmat][k] in xf order
};

static __global__ void __launch_bounds__(256) k_prep(const PrepArgs a) {
    pdl_trigger();
    pdl_wait();
    const int KB = a.k / 128;
    const int lane = threadIdx.x & 31;
    const int rows = a.n_rows_dev ? min(a.rows, *a.n_rows_dev) : a.rows;
    const int jobs = rows * a.nmat * KB;
    for (int j = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < jobs; j += (gridDim.x * blockDim.x) >> 5) {
        const int row = j / (a.nmat * KB);
        const int m = (j / KB) % a.nmat;
        const int kb = j % KB;
        const __half* suh = a.suh0;
        size_t xrow = (size_t)row;
        if (a.row_tok) xrow = (size_t)a.row_tok[row];
        if (a.row_expert) suh = a.experts[a.row_expert[row]].suh[m];
        float v[4];
        const __half* su = suh ? suh + kb * 128 : nullptr;
        if (a.x_bf16)
            rotated_block<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(a.x) + xrow * a.ldx + kb * 128, su,
                                         lane, v);
        else
            rotated_block<__half>(reinterpret_cast<const __half*>(a.x) + xrow * a.ldx + kb * 128, su, lane, v);
        store_xf_block(v, lane, a.xf + ((size_t)row * a.nmat + m) * a.k + (size_t)kb * 128);
    }
}

// ------------------------------------------------------------------------------------------------ host launch

// Launch with programmatic stream serialization (the kernel may start while the previous one finishes).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              int cluster, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
    if (cluster > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = cluster;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Work decomposition: units = work items x column blocks. Grids with fewer units than SMs split k over a cluster;
// they and single-wave grids run KI = 3 consumer warps per tile group (one big CTA per SM, deep ring); larger grids
// run KI = 1 (several smaller CTAs per SM).
struct GemvPlan {
    int split, KI, stages, threads, smem;
};
inline GemvPlan plan_gemv(int epi, int units, int k, int row_stride_hint, int requested_split) {
    GemvPlan pl;
    const int sms = num_sms();
    const int KB = k / 128;
    const int cap = KB < kMaxCluster ? KB : kMaxCluster;
    int P = requested_split;
    if (P <= 0) {
        P = 1;
        while (P < cap && units * (P + 1) <= sms) ++P;
    }
    if (P > cap) P = cap;
    pl.split = P;
    // MoE grids are sized from an upper bound on items (the surplus CTAs exit at once), so up to 1.25 x SMs still
    // means about one working CTA per SM
    pl.KI = units * P * 4 > sms * 5 ? 1 : max_ki(epi);
    const int n_rows = klen_alloc_of(k, P) / 16;
    const long slice = (long)n_rows * row_stride_hint;
    int stages = (int)((slice + kStageBytes - 1) / kStageBytes);     // enough to hold the whole slice
    const int max_st = pl.KI == 1 ? 6 : kMaxStages;
    stages = stages > max_st ? max_st : stages;
    stages = (stages + pl.KI - 1) / pl.KI;                           // per group
    stages = stages < 2 ? 2 : stages;
    while (stages * pl.KI > kMaxStages) --stages;
    pl.stages = stages * pl.KI;
    pl.threads = pl.KI * (tile_groups(epi) + 1) * 32;
    pl.smem = smem_layout(epi, pl.KI, pl.stages).total;
    return pl;
}

template <int EPI>
int launch_gemv(GemvArgs a, int units, const GemvPlan& pl, cudaStream_t st, const char* what) {
    a.split = pl.split;
    a.stages = pl.stages;
    EXL3_REQUIRE(pl.smem <= 227 * 1024, EXL3_ERR_UNSUPPORTED, "%s: shared memory plan too large", what);
    auto kern = k_gemv<EPI>;
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
            set_error("%s: cudaFuncSetAttribute: %s", what, cudaGetErrorString(cudaGetLastError()));
            return EXL3_ERR_CUDA;
        }
        configured[dev] = 1;
    }
    cudaError_t e = launch_pdl(kern, dim3(units * pl.split), dim3(pl.threads), pl.smem, st, pl.split, a);
    if (e != cudaSuccess) {
        set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
        return EXL3_ERR_CUDA;
    }
    return EXL3_OK;
}

// pdl: overlap the prep kernel with its predecessor. The MoE path launches it without (pdl = 0): the GEMV that follows
// reads the alignment tables before its own griddepcontrol.wait, which is safe only if prep started after the
// alignment kernel completed.
inline int launch_prep(const PrepArgs& a, cudaStream_t st, const char* what, bool pdl) {
    const long jobs = (long)a.rows * a.nmat * (a.k / 128);
    long blocks = (jobs + 7) / 8;
    if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
    if (blocks < 1) blocks = 1;
    cudaError_t e;
    if (pdl) {
        e = launch_pdl(k_prep, dim3((unsigned)blocks), dim3(256), 0, st, 1, a);
    } else {
        k_prep<<<(unsigned)blocks, 256, 0, st>>>(a);
        e = cudaGetLastError();
    }
    if (e != cudaSuccess) {
        set_error("%s: prep launch failed: %s", what, cudaGetErrorString(e));
        return EXL3_ERR_CUDA;
    }
    return EXL3_OK;
}

}  // namespace exl3
