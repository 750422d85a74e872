// Fused EXL3 decode GEMV for B200 (sm_100a), persistent stream-K schedule.
//
// Weights use the column-block-major trellis layout of this library ("packed"): for every 128-column block cb and
// tile-row r (16 input rows) the 8 tiles of that block are contiguous, [n/128][k/16][8 tiles][8K words]; a fused
// gate|up pair stores both matrices' 8 tiles per (cb, r), [I/128][H/16][gate 8 tiles | up 8 tiles]. It is a
// permutation of exllamav3's [k/16][n/16][16K] int16 trellis (same bytes), made once at load time (exl3_pack), so
// that any run of k-blocks of one column block is ONE contiguous range: a producer moves it with large TMA bulk
// copies (cp.async.bulk, 8 KB stages; no tensor maps, no multicast).
//
// Schedule. A unit is (work item, 128-column block): the dense linear has n/128 units, a MoE launch one per
// (expert item, column block). The launch's work is units x k-blocks (128 input rows each), laid out unit-major and
// cut into equal contiguous ranges, one per CTA (one CTA per SM). In a CTA one producer warp streams the range through
// a 10-stage shared-memory ring to 20 consumer warps: five sub-groups of four warps take the stages in turn, the four
// warps of a sub-group covering all tiles of each tile-row; the shared ring keeps the sub-groups within a few
// stages of each other. At the end of each segment the consumers park their accumulators in one of two shared-memory
// slots and go on decoding; two epilogue warps sum them, reduce split units and run the epilogue. A CTA that covers a
// whole unit finishes it on the spot; units shared by several CTAs are reduced through global memory: the other
// contributors store their fp32 partials and take an atomic ticket, and the unit's first contributor, for which the
// unit is the last segment of its range, waits briefly for their count (they have the unit as the first segment of
// their ranges, so it is usually complete) and sums all partials in CTA order (a fixed order: results do not depend
// on timing). If the count does not complete within 20 us (exl3_set_finisher_wait) it publishes its own partial
// and takes a ticket too, and the contributor that completes the count finishes: no CTA waits long for one that may
// not be resident, so concurrent kernels cannot stall a launch. Units split over more than 4 CTAs always use the
// ticket. Every SM has work until the last k-block, whatever the number of units.
//
// Activations arrive pre-rotated in "xf" order (prep kernels, or the gate|up epilogue for the down projection):
// a = fp16(H(fp16(x*suh))/sqrt(128)) (exllamav3's roundings), stored per (row, 16-input tile-row) as 4 quads x 4 fp16
// {a[2q], a[2q+1], a[2q+8], a[2q+9]}: exactly the two registers of the m16n8k16 MMA B fragment of lane quad q.
//
// Decode (glm/docs/ext-op-inventory.md:559-574), fold form (glm/xpu/csrc/exl3_esimd.h:82-91): the weight's 16-bit
// state times 0x83DCD12D, byte sum + 0x6400 by dp4a = the fp16 bits of h = 1024 + bytesum (exact), packed two per
// register straight into the MMA A fragment (the EXL3 position order is that fragment's layout: lane 4g+q owns
// positions 8l..8l+7, so no shuffles). One m16n8k16 MMA per 16x16 tile accumulates D = sum_k h_k a_k in fp32; batch
// rows ride in the MMA's 8 columns, so rows 1..8 cost the same decode (the linear's 9..16-row calls issue a second
// MMA per decoded fragment for rows 9..16). The codebook's affine w = h c1 + c2 (fp16 constants 0x1EEE / 0xC931) is
// applied once per output in the epilogue, D' = c1 D + c2 S with S = sum_k a_k from the per-128-block activation sums
// the rotation kernels write: the product is the one of the unrounded affine (|w' - w| <= half an fp16 ulp of the
// reference's fp16 weight), one fp16 FMA per weight pair less than applying it to every weight. exl3_dequant keeps
// the rounded fp16 weights, bit for bit.
//
// Epilogues: the output Hadamard x svh (linear), the gated-MLP activation + the down projection's input rotation
// (MoE gate|up), or Hadamard x svh x routing weight (MoE down).
// Launched with programmatic stream serialization: producers start streaming weights while the previous kernel
// finishes; consumers execute griddepcontrol.wait before reading activations or touching the reduction state.
//
// Reference semantics: exllamav3 exl3_gemm (glm/docs/ext-op-inventory.md:498-557), the XPU GemvKernel/HadIn/HadOut
// (glm/xpu/csrc/exl3_esimd.h:283-338,444-580) and the MoE GateUp/Down kernels (glm/xpu/csrc/exl3_moe.n128.sycl:
// 136-383). Work partition, the packed layout and the data movement are this file's own.
#pragma once

#include "common.cuh"
#include "hadamard.cuh"
#include "trellis.cuh"

namespace exl3 {

enum { EPI_LINEAR = 0, EPI_GATEUP = 1, EPI_DOWN = 2 };

constexpr int kTilesPerMat = 8;     // 128 output columns per unit and matrix (one Hadamard block)
constexpr int kMaxRows = 8;         // MMA N dimension: input rows per row group of a unit
constexpr int kMaxRowGroups = 2;    // the linear GEMV's units take up to 2 row groups (16 rows, two MMAs per decoded
                                    // fragment); the MoE units take one
constexpr int kStageBytes = 8192;   // ring stage (one bulk copy)
constexpr int kStages = 10;         // ring stages per CTA (80 KB in flight; the rest of the 256 KB stays L1 for the
                                    // activation rows)
constexpr int kConsumers = 4;       // consumer warps that cover one tile-row (all tiles of all matrices)
constexpr int kSub = 5;             // consumer sub-groups; sub-group j takes ring stages j, j + kSub, ...
constexpr int kConsumerWarps = kSub * kConsumers;
constexpr int kEpilogueWarps = 2;   // reduce and finish units while the consumers decode the next segment
constexpr int kGemvThreads = (1 + kConsumerWarps + kEpilogueWarps) * 32;   // producer, consumers, epilogue
static_assert(kMaxRows % kEpilogueWarps == 0, "epilogue rows per warp");

__host__ __device__ constexpr int nmat_of(int epi) { return epi == EPI_GATEUP ? 2 : 1; }
__host__ __device__ constexpr int tiles_per_warp(int epi) { return nmat_of(epi) * kTilesPerMat / kConsumers; }
// floats of one unit's accumulators (also one partial slot): [nmat][kMaxRows * rg][128]
__host__ __device__ constexpr int unit_floats(int epi, int rg = 1) { return nmat_of(epi) * kMaxRows * rg * 128; }

// Expert descriptor (device table, one entry per expert; the shared expert is an ordinary entry).
// tr[0] = packed gate|up [I/128][H/16][8 gate tiles | 8 up tiles], tr[1] unused, tr[2] = packed down.
struct ExpertDesc {
    const uint32_t* tr[3];
    const __half* suh[3];       // input signs/scales (gate, up, down)
    const __half* svh[3];       // output signs/scales
    int K[3];
    int pad;
};

// Grouped work produced by the alignment step: item i covers pair positions [start, start + cnt) of expert e.
// Written by the preceding kernel before it triggers this launch; read with L2 loads.
struct ItemTable {
    const int* n_items;      // [1]
    const int* item_expert;  // [max_items]
    const int* item_start;   // [max_items]
    const int* item_cnt;     // [max_items], 1..kMaxRows
    const int* pair_src;     // [positions] gate|up activation row of a pair position
    const float* pair_w;     // [positions] routing weight of a pair position
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
    float* ybuf;            // [positions, H] fp32 weighted down outputs
    int ybuf_round_f16;     // down: round as the fp16 linear does, fp16(fp16(H(acc) / sqrt(128)) * svh), before the weight
    float act_limit;
    // activations in xf order: linear: [M][k]; gate|up: [rows][2][k] (row = pair_src of a position); down: [pos][k]
    const __half* xf;
    // sums of the fp16 activations per 128-block, in the same row order: [row][nmat][k / 128] fp32 (the fold's S)
    const float* xsum;
    __half* xf_out;         // gate|up only: the down input in xf order [positions][I]
    float* xsum_out;        // gate|up only: its block sums [positions][I / 128]
    // shape of the matrices this launch runs (gate|up: k = H, n = I; down: k = I, n = H)
    int k, n;
    float* partial;         // [2 gridDim.x][unit_floats] split-unit partial sums
    int* counters;          // [units] tickets, zero before the launch, left zero after it
    int* status;
    uint64_t head_wait_ns;  // a split unit's finisher waits this long for the other partials (set at launch)
};

// Dynamic shared memory: red [2][kSub][unit_floats] fp32 (per sub-group accumulators of two segments in flight),
// bars full/empty [kStages] + acc_full/acc_empty [2], the ticket flag, the ring [kStages][kStageBytes], then the
// descriptors of the CTA's first kMaxSeg segments.
constexpr int kMaxSeg = 64;
constexpr int kDescBytes = 128;     // >= sizeof(UnitInfo<any>)
struct Smem {
    int red_off, bar_off, flag_off, ring_off, desc_off, total;
};
__host__ __device__ __forceinline__ Smem smem_layout(int epi, int rg = 1) {
    Smem s;
    s.red_off = 0;
    s.bar_off = 2 * kSub * unit_floats(epi, rg) * 4;
    s.flag_off = s.bar_off + (2 * kStages + 4) * 8;
    s.ring_off = (s.flag_off + 16 + 127) & ~127;
    s.desc_off = s.ring_off + kStages * kStageBytes;
    s.total = s.desc_off + kMaxSeg * kDescBytes;
    return s;
}

// ---- programmatic dependent launch ----
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ void prefetch_l1(const void* p) {
    asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

// Acquire load at GPU scope (a ticket written by other CTAs with a fence before their atomic).
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Named barrier over the epilogue warps (id 1; 0 is __syncthreads, used once before the roles split).
__device__ __forceinline__ void epilogue_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kEpilogueWarps * 32) : "memory");
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

// Sum of one 128-block's values (lane l holds 4l..4l+3, already fp16-rounded) in a fixed association order; every
// lane gets lane 0's total.
__device__ __forceinline__ float xf_block_sum(const float v[4]) {
    float t = (v[0] + v[1]) + (v[2] + v[3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
    return __shfl_sync(0xFFFFFFFFu, t, 0);
}

// Sum of n per-block sums p[0..n) (lane-strided partial sums, then a fixed xor tree; lane 0's total to every lane).
__device__ __forceinline__ float xsum_total(const float* p, int n, int lane) {
    float t = 0.f;
    for (int b = lane; b < n; b += 32) t += __ldcg(p + b);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xFFFFFFFFu, t, o);
    return __shfl_sync(0xFFFFFFFFu, t, 0);
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

// One consumer warp over one segment: its TPW tiles of one matrix on every tile-row of the stages its sub-group owns
// (ring sequence numbers it with it % kSub == sub, visited directly), continuing the CTA's ring sequence at `it` and
// leaving it at the segment's end. The ring couples the sub-groups: one that falls behind holds the producer back, and
// the others then wait and leave it the issue slots. The B fragments of a stage's first kBatch tile-rows are loaded
// before the stage's full barrier is waited on, and each further row's fragment kBatch rows ahead. With RG row groups
// (the linear's 9..16-row calls) every decoded fragment feeds RG MMAs, one per group of 8 input rows.
// d[rg * TPW + t] = D[16 n x 8 rows] of tile t and row group rg: d[.][0], d[.][1] = (n = g, rows 2q, 2q+1),
// d[.][2], d[.][3] = (n = g + 8, rows 2q, 2q+1), rows counted inside the group.
template <int K, int TPW, int RG>
__device__ __forceinline__ void consume(float d[RG * TPW][4], const uint8_t* ring, int row_stride, int mat_off,
                                        int tile0, int n_rows, int rps, int sub, uint64_t* full, uint64_t* empty,
                                        const __half* const xf_row[RG], const bool has_row[RG], int lane, int& it,
                                        bool& timed_out) {
    constexpr int kBatch = RG > 1 ? 1 : (TPW >= 4 ? 2 : 4);   // B fragments in flight per group (registers: the
                                                              // 4-tile warps and the 2-group calls hold twice the
                                                              // accumulators)
    const LaneWords lw = lane_words<K>(lane);
    const int q = lane & 3;
    // B fragment of tile-row r for this lane and group: 8 bytes at xf_row[rg] + r * 16 + q * 4
    const uint2* bp[RG];
#pragma unroll
    for (int rg = 0; rg < RG; ++rg) bp[rg] = reinterpret_cast<const uint2*>(xf_row[rg] + q * 4);
    // a stage of a segment whose matrices share K holds RPS whole tile-rows of a compile-time stride: that case
    // runs fully unrolled with every row's B fragment loaded before the stage's barrier
    constexpr int RS = (TPW / 2) * kTilesPerMat * 32 * K;
    constexpr int RPS = kStageBytes / RS;
    constexpr int UNR = RG == 1 && RPS <= (TPW >= 4 ? 5 : 10) ? RPS : 0;
    const int nst = (n_rows + rps - 1) / rps, it_begin = it;
    for (int j = (sub - it % kSub + kSub) % kSub; j < nst; j += kSub) {
        it = it_begin + j;
        const int r0 = j * rps;
        const int s = it % kStages;
        const int rows = min(rps, n_rows - r0);
        if constexpr (UNR > 0) {
            if (row_stride == RS && rows == RPS) {
                uint2 bf[UNR > 0 ? UNR : 1][RG];
#pragma unroll
                for (int r = 0; r < UNR; ++r)
#pragma unroll
                    for (int rg = 0; rg < RG; ++rg)
                        bf[r][rg] = has_row[rg] ? __ldg(bp[rg] + (size_t)(r0 + r) * 4) : make_uint2(0, 0);
                if (!timed_out && !mbar_wait(&full[s], (it / kStages) & 1)) timed_out = true;
                if (!timed_out) {
                    const uint8_t* base = ring + (size_t)s * kStageBytes + mat_off + tile0 * 32 * K;
#pragma unroll
                    for (int r = 0; r < UNR; ++r) {
#pragma unroll
                        for (int t = 0; t < TPW; ++t) {
                            uint32_t a[4];
                            decode_frag_raw<K>(reinterpret_cast<const uint32_t*>(base + r * RS + t * 32 * K), lw, a);
#pragma unroll
                            for (int rg = 0; rg < RG; ++rg) mma_16816(d[rg * TPW + t], a, bf[r][rg].x, bf[r][rg].y);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[s]);
                continue;
            }
        }
        uint2 bq[kBatch][RG];
#pragma unroll
        for (int b = 0; b < kBatch; ++b)
#pragma unroll
            for (int rg = 0; rg < RG; ++rg)
                bq[b][rg] = (has_row[rg] && b < rows) ? __ldg(bp[rg] + (size_t)(r0 + b) * 4) : make_uint2(0, 0);
        if (!timed_out && !mbar_wait(&full[s], (it / kStages) & 1)) timed_out = true;
        if (!timed_out) {
            const uint8_t* base = ring + (size_t)s * kStageBytes + mat_off + tile0 * 32 * K;
            for (int rb = 0; rb < rows; rb += kBatch) {
#pragma unroll
                for (int b = 0; b < kBatch; ++b) {
                    if (rb + b < rows) {
                        uint2 bv[RG];
                        const int nx = rb + kBatch + b;            // the row this slot holds next
#pragma unroll
                        for (int rg = 0; rg < RG; ++rg) {
                            bv[rg] = bq[b][rg];
                            if (has_row[rg] && nx < rows) bq[b][rg] = __ldg(bp[rg] + (size_t)(r0 + nx) * 4);
                        }
#pragma unroll
                        for (int t = 0; t < TPW; ++t) {
                            uint32_t a[4];
                            decode_frag_raw<K>(reinterpret_cast<const uint32_t*>(base + t * 32 * K), lw, a);
#pragma unroll
                            for (int rg = 0; rg < RG; ++rg) mma_16816(d[rg * TPW + t], a, bv[rg].x, bv[rg].y);
                        }
                        base += row_stride;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
    }
    it = it_begin + nst;
}

template <int TPW, int RG>
__device__ __forceinline__ void consume_k(int K, float d[RG * TPW][4], const uint8_t* ring, int row_stride,
                                          int mat_off, int tile0, int n_rows, int rps, int sub, uint64_t* full,
                                          uint64_t* empty, const __half* const xf_row[RG], const bool has_row[RG],
                                          int lane, int& it, bool& to) {
#define EXL3_CONSUME(KK)                                                                                          \
    consume<KK, TPW, RG>(d, ring, row_stride, mat_off, tile0, n_rows, rps, sub, full, empty, xf_row, has_row,     \
                         lane, it, to)
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

// silu(g) = g / (1 + e^-g), fp32 with the fast exponential and division intrinsics (relative error ~1e-6, far below
// the fp16 rounding of the activation that follows; g -> -inf gives -0).
__device__ __forceinline__ float silu_f(float g) { return __fdividef(g, 1.0f + __expf(-g)); }

// What a unit needs: packed weights of its column block, bit widths, rows, and the activation row of each MMA
// column (linear: row g; gate|up: the pair's source row; down: the pair position).
template <int EPI>
struct UnitInfo {
    const uint8_t* w;           // packed weights of the unit's column block (k-block 0)
    int K[nmat_of(EPI)];
    int row_stride;             // bytes per tile-row of the block (all matrices)
    int Mi, s0, expert, cb;
    int xrow[kMaxRows];
};

template <int EPI>
__device__ __forceinline__ UnitInfo<EPI> unit_info(const GemvArgs& a, int u, int NB, int KB) {
    constexpr int NMAT = nmat_of(EPI);
    UnitInfo<EPI> ui;
    ui.cb = u % NB;
    const uint8_t* base;
    if constexpr (EPI == EPI_LINEAR) {
        base = reinterpret_cast<const uint8_t*>(a.tr);
        ui.K[0] = a.K;
        ui.Mi = a.M;
        ui.s0 = 0;
        ui.expert = 0;
    } else {
        const int item = u / NB;
        ui.expert = __ldcg(a.items.item_expert + item);
        ui.s0 = __ldcg(a.items.item_start + item);
        ui.Mi = __ldcg(a.items.item_cnt + item);
        const ExpertDesc& ed = a.experts[ui.expert];
        if constexpr (EPI == EPI_GATEUP) {
            base = reinterpret_cast<const uint8_t*>(ed.tr[0]);
            ui.K[0] = ed.K[0];
            ui.K[NMAT - 1] = ed.K[1];
        } else {
            base = reinterpret_cast<const uint8_t*>(ed.tr[2]);
            ui.K[0] = ed.K[2];
        }
    }
#pragma unroll
    for (int g = 0; g < kMaxRows; ++g) {
        int r = 0;
        if (g < ui.Mi) {
            if constexpr (EPI == EPI_LINEAR) r = g;
            else if constexpr (EPI == EPI_GATEUP) r = __ldcg(a.items.pair_src + ui.s0 + g);
            else r = ui.s0 + g;
        }
        ui.xrow[g] = r;
    }
    ui.row_stride = 0;
#pragma unroll
    for (int m = 0; m < NMAT; ++m) ui.row_stride += kTilesPerMat * 32 * ui.K[m];
    ui.w = base + (size_t)ui.cb * KB * 8 * ui.row_stride;
    return ui;
}

// Activation row of the unit's input row `row` (the linear's rows are the call's rows; up to 16 of them).
template <int EPI>
__device__ __forceinline__ int xrow_of(const UnitInfo<EPI>& ui, int row) {
    if constexpr (EPI == EPI_LINEAR) return row;
    else return ui.xrow[row];
}

// The epilogue operands of a unit for lane `lane` (columns cb * 128 + 4 lane ..+3) of epilogue warp ew: output
// scales of each matrix, the down projection's input signs (gate|up), the routing weights of the warp's rows (down).
// Loaded before the epilogue warps wait for the unit's accumulators, so that the dependent loads (expert descriptor,
// then its vectors) stay off the end of the launch.
template <int EPI>
struct EpiOperands {
    float sv[nmat_of(EPI)][4];
    float su_dn[4];                                           // gate|up: suh of the down projection
    float w[kMaxRows / kEpilogueWarps];                       // down: routing weights of rows ew, ew + kEpilogueWarps
    float c2s0[nmat_of(EPI)];                                 // c2 * S of row ew (the fold's term), per matrix
};

template <int EPI>
__device__ __forceinline__ EpiOperands<EPI> epi_operands(const GemvArgs& a, const UnitInfo<EPI>& ui, int ew, int lane) {
    constexpr int NMAT = nmat_of(EPI);
    EpiOperands<EPI> op;
    const int col = ui.cb * 128 + 4 * lane;
    const __half* svh[NMAT];
    if constexpr (EPI == EPI_LINEAR) {
        svh[0] = a.svh;
    } else {
        const ExpertDesc& ed = a.experts[ui.expert];
        if constexpr (EPI == EPI_GATEUP) {
            svh[0] = ed.svh[0];
            svh[NMAT - 1] = ed.svh[1];
#pragma unroll
            for (int j = 0; j < 4; ++j) op.su_dn[j] = __half2float(ed.suh[2][col + j]);
        } else {
            svh[0] = ed.svh[2];
        }
    }
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
#pragma unroll
        for (int j = 0; j < 4; ++j) op.sv[m][j] = __half2float(svh[m][col + j]);
    if constexpr (EPI == EPI_DOWN) {
#pragma unroll
        for (int i = 0; i < kMaxRows / kEpilogueWarps; ++i) {
            const int row = ew + i * kEpilogueWarps;
            op.w[i] = row < ui.Mi ? __ldcg(a.items.pair_w + ui.s0 + row) : 0.f;
        }
    }
    // the fold's activation sum of the warp's first row, before the accumulators are waited for (the other rows of
    // an item, rare in decode, load theirs in the epilogue)
#pragma unroll
    for (int m = 0; m < NMAT; ++m)
        op.c2s0[m] = ew < ui.Mi ? kMul1C2 * xsum_total(a.xsum + ((size_t)xrow_of(ui, ew) * NMAT + m) * (a.k / 128),
                                                       a.k / 128, lane)
                                : 0.f;
    return op;
}

// Epilogue of one unit from its summed accumulators red[nmat][kMaxRows * RG][128] (shared memory), one row per warp.
template <int EPI, int RG>
__device__ __forceinline__ void unit_epilogue(const GemvArgs& a, const UnitInfo<EPI>& ui, const float* red, int ew,
                                              int lane, const EpiOperands<EPI>& op) {
    constexpr int NMAT = nmat_of(EPI);
    constexpr int R = kMaxRows * RG;
    const int col = ui.cb * 128 + 4 * lane;
#pragma unroll(RG == 1 ? R / kEpilogueWarps : 1)
    for (int ri = 0; ri < R / kEpilogueWarps; ++ri) {
        const int row = ew + ri * kEpilogueWarps;
        if (row >= ui.Mi) break;
        float v[NMAT][4];
#pragma unroll
        for (int m = 0; m < NMAT; ++m) {
            // the codebook affine on the product: c1 * sum h a + c2 * sum a (S: the row's activation sum)
            const float* xs = a.xsum + ((size_t)xrow_of(ui, row) * NMAT + m) * (a.k / 128);
            const float c2s = ri == 0 ? op.c2s0[m] : kMul1C2 * xsum_total(xs, a.k / 128, lane);
            const float4 t = *reinterpret_cast<const float4*>(red + ((size_t)m * R + row) * 128 + 4 * lane);
            v[m][0] = fmaf(kMul1C1, t.x, c2s);
            v[m][1] = fmaf(kMul1C1, t.y, c2s);
            v[m][2] = fmaf(kMul1C1, t.z, c2s);
            v[m][3] = fmaf(kMul1C1, t.w, c2s);
            fwht128_warp(v[m], lane);
        }
        if constexpr (EPI == EPI_LINEAR) {
            float o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float sv = op.sv[0][j];
                if (a.y_dtype == EXL3_F16)
                    o[j] = __half2float(__float2half_rn(__half2float(__float2half_rn(v[0][j] * kRsqrt128)) * sv));
                else
                    o[j] = v[0][j] * kRsqrt128 * sv;
            }
            if (a.y_dtype == EXL3_F32) {
                float* yp = reinterpret_cast<float*>(a.y) + (size_t)row * a.ldy + col;
                *reinterpret_cast<float4*>(yp) = make_float4(o[0], o[1], o[2], o[3]);
            } else if (a.y_dtype == EXL3_F16) {
                __half* yp = reinterpret_cast<__half*>(a.y) + (size_t)row * a.ldy + col;
                __half2 h01 = __floats2half2_rn(o[0], o[1]), h23 = __floats2half2_rn(o[2], o[3]);
                uint2 u;
                u.x = *reinterpret_cast<uint32_t*>(&h01);
                u.y = *reinterpret_cast<uint32_t*>(&h23);
                *reinterpret_cast<uint2*>(yp) = u;
            } else {
                __nv_bfloat16* yp = reinterpret_cast<__nv_bfloat16*>(a.y) + (size_t)row * a.ldy + col;
#pragma unroll
                for (int j = 0; j < 4; ++j) yp[j] = __float2bfloat16_rn(o[j]);
            }
        } else if constexpr (EPI == EPI_GATEUP) {
            const float Lc = a.act_limit;
            float h[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                // gate/up outputs rounded to fp16 as the fp16 linear does: fp16(fp16(H(acc)*r) * svh)
                float gg = __half2float(__float2half_rn(__half2float(__float2half_rn(v[0][j] * kRsqrt128)) * op.sv[0][j]));
                float uu = __half2float(
                    __float2half_rn(__half2float(__float2half_rn(v[NMAT - 1][j] * kRsqrt128)) * op.sv[NMAT - 1][j]));
                float sg = silu_f(gg);
                if (Lc != 0.f) { sg = fminf(sg, Lc); uu = fminf(fmaxf(uu, -Lc), Lc); }
                const float act = __half2float(__float2half_rn(sg * uu));
                h[j] = __half2float(__float2half_rn(act * op.su_dn[j]));
            }
            fwht128_warp(h, lane);
#pragma unroll
            for (int j = 0; j < 4; ++j) h[j] = __half2float(__float2half_rn(h[j] * kRsqrt128));
            // the down projection's input block cb, straight into xf order, and its block sum
            store_xf_block(h, lane, a.xf_out + (size_t)(ui.s0 + row) * a.n + (size_t)ui.cb * 128);
            const float bs = xf_block_sum(h);
            if (lane == 0) a.xsum_out[(size_t)(ui.s0 + row) * (a.n / 128) + ui.cb] = bs;
        } else {
            const float w = op.w[ri];
            float o[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float sv = op.sv[0][j];
                o[j] = a.ybuf_round_f16
                           ? w * __half2float(__float2half_rn(__half2float(__float2half_rn(v[0][j] * kRsqrt128)) * sv))
                           : w * (v[0][j] * kRsqrt128 * sv);
            }
            float* dst = a.ybuf + (size_t)(ui.s0 + row) * a.n + col;
            *reinterpret_cast<float4*>(dst) = make_float4(o[0], o[1], o[2], o[3]);
        }
    }
}

// First k-block of CTA c's range, and the CTA that owns k-block x (the last CTA whose range starts at or before x;
// CTAs with empty ranges own nothing).
__device__ __forceinline__ long long range_start(long long c, long long T, long long G) { return c * T / G; }
__device__ __forceinline__ long long owner_of(long long x, long long T, long long G) { return ((x + 1) * G - 1) / T; }
// The CTA owning the first k-block after CTA c's range (contributors of one unit, in order).
__device__ __forceinline__ long long next_owner(long long c, long long T, long long G) {
    return owner_of(range_start(c + 1, T, G), T, G);
}

// Grid: persistent, at most one CTA per SM, each a contiguous range of the launch's k-blocks; block: 1 producer warp,
// kConsumerWarps consumer warps, kEpilogueWarps epilogue warps.
template <int EPI, int RG>
__global__ void __launch_bounds__(kGemvThreads, 1) k_gemv(const GemvArgs args) {
    static_assert(RG >= 1 && RG <= kMaxRowGroups && (RG == 1 || EPI == EPI_LINEAR), "row groups: linear only");
    constexpr int NMAT = nmat_of(EPI);
    constexpr int TPW = tiles_per_warp(EPI);
    constexpr int R = kMaxRows * RG;                            // input rows of a unit
    constexpr int UF = unit_floats(EPI, RG);
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();
    const int NB = args.n / 128, KB = args.k / 128;
    const long long G = gridDim.x;
    const long long ci = blockIdx.x;
    // units: the linear's column blocks, or (expert item, column block) pairs of the alignment step's table
    const int U = (EPI == EPI_LINEAR) ? NB : __ldcg(args.items.n_items) * NB;
    const long long T = (long long)U * KB;
    const long long r0 = range_start(ci, T, G), r1 = range_start(ci + 1, T, G);

    const Smem L = smem_layout(EPI, RG);
    float* red = reinterpret_cast<float*>(smem + L.red_off);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar_off);
    uint64_t* empty = full + kStages;
    uint64_t* acc_full = empty + kStages;                      // [2]: a segment's accumulators are in red[buf]
    uint64_t* acc_empty = acc_full + 2;                        // [2]: red[buf] may be overwritten
    volatile int* flag = reinterpret_cast<volatile int*>(smem + L.flag_off);
    uint8_t* ring = smem + L.ring_off;
    static_assert(sizeof(UnitInfo<EPI>) <= kDescBytes, "descriptor slot");
    UnitInfo<EPI>* descs = reinterpret_cast<UnitInfo<EPI>*>(smem + L.desc_off);

    // segments: the units the range touches; segment i = unit u0 + i, k-blocks [lo, hi). Their descriptors (dependent
    // table loads) are resolved once, one thread per segment, while the previous kernel may still be running.
    const long long u0 = r0 / KB;
    const int n_seg = r1 > r0 ? (int)((r1 - 1) / KB - u0 + 1) : 0;
    for (int i = threadIdx.x; i < n_seg && i < kMaxSeg; i += blockDim.x)
        descs[i] = unit_info<EPI>(args, (int)(u0 + i), NB, KB);
    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&full[s], 1); mbar_init(&empty[s], kConsumers); }
        for (int b = 0; b < 2; ++b) { mbar_init(&acc_full[b], kConsumerWarps); mbar_init(&acc_empty[b], kEpilogueWarps); }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ---------------- producer: the range, segment by segment, stage by stage ----------------
        if (lane == 0) {
            bool to = false;
            int it = 0;
            for (int i = 0; i < n_seg && !to; ++i) {
                const long long u = u0 + i;
                const int lo = i == 0 ? (int)(r0 - u * KB) : 0;
                const int hi = (int)min((long long)KB, r1 - u * KB);
                const UnitInfo<EPI> ui = i < kMaxSeg ? descs[i] : unit_info<EPI>(args, (int)u, NB, KB);
                const uint8_t* src = ui.w + (size_t)lo * 8 * ui.row_stride;
                const int n_rows = (hi - lo) * 8, rps = kStageBytes / ui.row_stride;
                for (int r = 0; r < n_rows; r += rps, ++it) {
                    const int s = it % kStages;
                    if (it >= kStages && !mbar_wait(&empty[s], ((it / kStages) - 1) & 1)) { to = true; break; }
                    const uint32_t bytes = (uint32_t)(min(rps, n_rows - r) * ui.row_stride);
                    mbar_expect_tx(&full[s], bytes);
                    bulk_g2s(ring + (size_t)s * kStageBytes, src + (size_t)r * ui.row_stride, bytes, &full[s]);
                }
            }
            if (to) report(args.status, EXL3_ERR_TIMEOUT);
            // every issued copy has landed before the CTA can retire its shared memory: stage s last held sequence
            // number s + kStages * floor((it - 1 - s) / kStages)
            for (int s = 0; s < kStages && s < it; ++s) {
                const int last = s + ((it - 1 - s) / kStages) * kStages;
                if (!mbar_wait(&full[s], (last / kStages) & 1)) report(args.status, EXL3_ERR_TIMEOUT);
            }
        }
        return;
    }

    if (warp <= kConsumerWarps) {
        // ---------------- consumers: decode + MMA, accumulators handed to the epilogue warps ----------------
        const int cw = warp - 1;
        const int sub = cw / kConsumers, cq = cw % kConsumers;
        const int m = (cq * TPW) / kTilesPerMat, tile0 = (cq * TPW) % kTilesPerMat;
        const int g = lane >> 2, q = lane & 3;
        pdl_wait();                                           // activations come from earlier kernels
        bool to = false;
        int it = 0;
        for (int i = 0; i < n_seg; ++i) {
            const long long u = u0 + i;
            const int lo = i == 0 ? (int)(r0 - u * KB) : 0;
            const int hi = (int)min((long long)KB, r1 - u * KB);
            const UnitInfo<EPI> ui = i < kMaxSeg ? descs[i] : unit_info<EPI>(args, (int)u, NB, KB);
            bool has_row[RG];
            const __half* xf_row[RG];
#pragma unroll
            for (int rg = 0; rg < RG; ++rg) {
                const int row = g + kMaxRows * rg;
                has_row[rg] = row < ui.Mi;
                const int xr = RG == 1 ? ui.xrow[g] : (has_row[rg] ? row : 0);
                xf_row[rg] = args.xf + (size_t)xr * NMAT * args.k + (size_t)m * args.k + (size_t)lo * 128;
            }
            int mat_off = 0;
#pragma unroll
            for (int mm = 0; mm < NMAT; ++mm)
                if (mm < m) mat_off += kTilesPerMat * 32 * ui.K[mm];
            float d[RG * TPW][4];
#pragma unroll
            for (int t = 0; t < RG * TPW; ++t)
#pragma unroll
                for (int e = 0; e < 4; ++e) d[t][e] = 0.f;
            consume_k<TPW, RG>(ui.K[m], d, ring, ui.row_stride, mat_off, tile0, (hi - lo) * 8,
                               kStageBytes / ui.row_stride, sub, full, empty, xf_row, has_row, lane, it, to);
            // hand the accumulators over: red[i & 1][sub], once the epilogue released segment i - 2's
            const int buf = i & 1;
            if (i >= 2 && !to && !mbar_wait(&acc_empty[buf], ((i >> 1) - 1) & 1)) to = true;
            float* rs = red + ((size_t)buf * kSub + sub) * UF;
#pragma unroll
            for (int rg = 0; rg < RG; ++rg)
#pragma unroll
                for (int t = 0; t < TPW; ++t)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int row = kMaxRows * rg + 2 * q + (e & 1);
                        const int col = (tile0 + t) * 16 + g + ((e >> 1) << 3);
                        rs[((size_t)m * R + row) * 128 + col] = d[rg * TPW + t][e];
                    }
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_full[buf]);
        }
        if (to) report(args.status, EXL3_ERR_TIMEOUT);
        return;
    }

    // ---------------- epilogue warps: sum the sub-groups, reduce split units, finish units ----------------
    // A unit split over n_c <= 4 CTAs is finished by its first contributor (the owner of its first k-block, for which
    // the unit is the last segment of its range): the others store their partials and take a ticket (a fence and an
    // atomic add whose result they read only at the end of the launch), usually long before, since the unit is the
    // first segment of their ranges; the finisher loads their partials into red[buf ^ 1] (no later segment of this
    // CTA uses it) while its own consumers are still decoding, or, if they are not all in yet, waits up to
    // head_wait_ns (exl3_set_finisher_wait, 20 us by default) once its own part is done, and after that publishes
    // its partial and takes a ticket as well; the contributor whose ticket completes the count then finishes (which
    // the others' tickets cannot do while the first contributor holds back its own). Units split over more than 4
    // CTAs always use the ticket. Every path sums the partials in CTA order, so the result does not depend on timing
    // or on the path.
    const int ew = warp - 1 - kConsumerWarps;
    const int et = ew * 32 + lane;
    pdl_wait();                                               // tickets and outputs belong to this launch from here
    bool to = false;
    // the partials of the unit's contributors summed in CTA order into rb (rows below Mi)
    auto sum_slots = [&](long long a0, long long a1, int Mi, float* rb) {
        int slots[4];                                         // partial slots of the first contributors, in order
        int nc = 0;
        for (long long c = owner_of(a0, T, G); nc < 4; c = next_owner(c, T, G)) {
            slots[nc++] = (int)(range_start(c, T, G) < a0 ? 2 * c + 1 : 2 * c);   // started before a0: 2nd slot
            if (range_start(c + 1, T, G) >= a1) break;
        }
        for (int e = et; e < UF / 4; e += kEpilogueWarps * 32) {
            if ((e / 32) % R >= Mi) continue;
            float4 p[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                p[j] = j < nc ? __ldcg(reinterpret_cast<const float4*>(args.partial + (size_t)slots[j] * UF) + e)
                              : make_float4(0.f, 0.f, 0.f, 0.f);
            float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int j = 0; j < 4; ++j) { acc.x += p[j].x; acc.y += p[j].y; acc.z += p[j].z; acc.w += p[j].w; }
            if (nc == 4) {                                    // units split over more than 4 CTAs: the rest in order
                long long c = owner_of(a0, T, G);
                for (int j = 0; j < 4; ++j) c = next_owner(c, T, G);
                for (;; c = next_owner(c, T, G)) {
                    if (range_start(c, T, G) >= a1) break;
                    const long long sl = range_start(c, T, G) < a0 ? 2 * c + 1 : 2 * c;
                    const float4 q = __ldcg(reinterpret_cast<const float4*>(args.partial + (size_t)sl * UF) + e);
                    acc.x += q.x; acc.y += q.y; acc.z += q.z; acc.w += q.w;
                }
            }
            reinterpret_cast<float4*>(rb)[e] = acc;
        }
    };
    // a published partial whose ticket is read at the end (at most one per CTA: its first segment); def_old is the
    // ticket of thread et == 0, def_u and def_nc are set in every epilogue thread
    bool has_def = false;
    int def_old = -1, def_nc = 0;
    long long def_u = 0;
    for (int i = 0; i < n_seg; ++i) {
        const long long u = u0 + i;
        const int lo = i == 0 ? (int)(r0 - u * KB) : 0;
        const int hi = (int)min((long long)KB, r1 - u * KB);
        const UnitInfo<EPI> ui = i < kMaxSeg ? descs[i] : unit_info<EPI>(args, (int)u, NB, KB);
        const EpiOperands<EPI> op = epi_operands<EPI>(args, ui, ew, lane);
        const int buf = i & 1;
        const bool whole = lo == 0 && hi == KB;
        const long long a0 = u * KB, a1 = a0 + KB;            // the unit's k-blocks [a0, a1)
        int n_c = 1;                                          // contributors (up to 4 counted, more = ticket path)
        bool more = false;
        if (!whole) {
            n_c = 0;
            for (long long c = owner_of(a0, T, G);; c = next_owner(c, T, G)) {
                ++n_c;
                if (range_start(c + 1, T, G) >= a1) break;
                if (n_c == 4) { more = true; break; }
            }
        }
        const bool head = !whole && !more && owner_of(a0, T, G) == ci;   // this CTA finishes the unit
        float* pf = red + (size_t)(buf ^ 1) * kSub * UF;
        bool ready = false;
        if (head) {
            if (et == 0) flag[1] = ld_acquire_gpu(args.counters + u) == n_c - 1;
            epilogue_sync();
            ready = flag[1] != 0;
            if (ready) {                                      // the others' partials, while the consumers finish
                long long c = next_owner(ci, T, G);
                for (int j = 1; j < n_c; ++j, c = next_owner(c, T, G)) {
                    const float4* src = reinterpret_cast<const float4*>(args.partial + (size_t)(2 * c) * UF);
                    for (int e = et; e < UF / 4; e += kEpilogueWarps * 32)
                        if ((e / 32) % R < ui.Mi) reinterpret_cast<float4*>(pf + (size_t)j * UF)[e] = __ldcg(src + e);
                }
            }
        }
        if (!to && !mbar_wait(&acc_full[buf], (i >> 1) & 1)) to = true;
        float* rb = red + (size_t)buf * kSub * UF;
        float4* slot = reinterpret_cast<float4*>(args.partial + (size_t)(i == 0 ? 2 * ci : 2 * ci + 1) * UF);
        // sub-group sums in sub-group order: into rb[0] (whole unit, or the finisher's own part), with the others'
        // partials in CTA order when they are already loaded, or into this CTA's partial slot
        for (int e = et; e < UF / 4; e += kEpilogueWarps * 32) {
            if ((e / 32) % R >= ui.Mi) continue;              // rows beyond the unit's
            float4 acc = reinterpret_cast<const float4*>(rb)[e];
#pragma unroll
            for (int j = 1; j < kSub; ++j) {
                const float4 v = reinterpret_cast<const float4*>(rb + (size_t)j * UF)[e];
                acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
            }
            if (ready) {
                float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (j == 0) p = acc;
                    else if (j < n_c) p = reinterpret_cast<const float4*>(pf + (size_t)j * UF)[e];
                    t.x += p.x; t.y += p.y; t.z += p.z; t.w += p.w;
                }
                reinterpret_cast<float4*>(rb)[e] = t;
            } else if (whole || head) {
                reinterpret_cast<float4*>(rb)[e] = acc;
            } else {
                slot[e] = acc;
            }
        }
        bool finish = whole || head;
        bool ticket = more || (!whole && !head && has_def);   // publish the partial, take a ticket and read it
        const bool publish = !whole && !more && !head && !has_def;   // publish, take a ticket, read it at the end
        if (head && !ready) {
            // the others are not all in yet: wait a short while for the count, then add their partials in CTA
            // order; if it does not complete (another kernel holds the SMs a contributor needs), publish this
            // partial too and take a ticket like the others: the last of them finishes the unit
            epilogue_sync();                                  // every thread has read flag[1] (ready) and rb
            if (et == 0) {
                const uint64_t t0 = globaltimer_ns();
                bool in = true;
                while (ld_acquire_gpu(args.counters + u) != n_c - 1) {
                    if (globaltimer_ns() - t0 > args.head_wait_ns) { in = false; break; }
                    __nanosleep(64);
                }
                flag[1] = in;
            }
            epilogue_sync();
            if (flag[1]) {
                for (int e = et; e < UF / 4; e += kEpilogueWarps * 32) {
                    if ((e / 32) % R >= ui.Mi) continue;
                    float4 t = make_float4(0.f, 0.f, 0.f, 0.f);
                    long long c = ci;
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float4 p = make_float4(0.f, 0.f, 0.f, 0.f);
                        if (j == 0) p = reinterpret_cast<const float4*>(rb)[e];
                        else if (j < n_c) {
                            c = next_owner(c, T, G);
                            p = __ldcg(reinterpret_cast<const float4*>(args.partial + (size_t)(2 * c) * UF) + e);
                        }
                        t.x += p.x; t.y += p.y; t.z += p.z; t.w += p.w;
                    }
                    reinterpret_cast<float4*>(rb)[e] = t;
                }
            } else {
                for (int e = et; e < UF / 4; e += kEpilogueWarps * 32)
                    if ((e / 32) % R < ui.Mi) slot[e] = reinterpret_cast<const float4*>(rb)[e];
                finish = false;
                ticket = true;
            }
        }
        if (finish && head && et == 0) args.counters[u] = 0;  // every other contributor has counted: left zero
        if (publish) {
            epilogue_sync();                                  // both warps' slot stores, then one fence and the add
            if (et == 0) {
                __threadfence();
                def_old = atomicAdd(args.counters + u, 1);    // read by this thread only, at the end
            }
            def_u = u;                                        // every epilogue thread: the unit and its count
            def_nc = n_c;
            has_def = true;
        }
        if (ticket) {
            // the partial is in this CTA's slot: one fence, then the ticket; the contributor that completes the
            // count sums every partial in CTA order
            __threadfence();
            epilogue_sync();
            if (et == 0) {
                int nseg = 1;
                for (long long c = owner_of(a0, T, G); range_start(c + 1, T, G) < a1; c = next_owner(c, T, G)) ++nseg;
                const int old = atomicAdd(args.counters + u, 1);
                const int last = old == nseg - 1;
                if (last) {
                    args.counters[u] = 0;                     // left zero for the next launch
                    __threadfence();
                }
                *flag = last;
            }
            epilogue_sync();
            finish = *flag != 0;
            if (finish) sum_slots(a0, a1, ui.Mi, rb);
        }
        if (finish) {
            epilogue_sync();
            unit_epilogue<EPI, RG>(args, ui, rb, ew, lane, op);
        }
        epilogue_sync();                                      // the flags and red[buf] are read: release them
        if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
    if (has_def) {
        // the first segment's ticket: its add completed the count only if the unit's first contributor gave up
        // waiting and counted itself; then this CTA finishes that unit (red[] is free: every segment is done)
        if (et == 0) {
            const int last = def_old == def_nc - 1;
            if (last) {
                args.counters[def_u] = 0;                     // left zero for the next launch
                __threadfence();
            }
            flag[0] = last;
        }
        epilogue_sync();
        if (flag[0]) {
            const int i0 = (int)(def_u - u0);
            const UnitInfo<EPI> ui = i0 < kMaxSeg ? descs[i0] : unit_info<EPI>(args, (int)def_u, NB, KB);
            const EpiOperands<EPI> op = epi_operands<EPI>(args, ui, ew, lane);
            sum_slots(def_u * KB, def_u * KB + KB, ui.Mi, red);
            epilogue_sync();
            unit_epilogue<EPI, RG>(args, ui, red, ew, lane, op);
        }
    }
    if (to) report(args.status, EXL3_ERR_TIMEOUT);
}

// ------------------------------------------------------------------------------------------------ activation prep

// xf of the dense linear's input rows: job = (row, 128-block), one warp each; also zeroes the GEMV's tickets.
struct PrepArgs {
    const void* x;
    int ldx;
    int x_bf16;
    int rows, k;
    const __half* suh;
    __half* xf;                   // [rows][k] in xf order
    float* xsum;                  // [rows][k / 128] block sums of the rotated rows
    int* zero;                    // tickets of the following GEMV
    int n_zero;
};

static __global__ void __launch_bounds__(256) k_prep(const PrepArgs a) {
    pdl_trigger();
    pdl_wait();
    const int gt = blockIdx.x * blockDim.x + threadIdx.x;
    for (int i = gt; i < a.n_zero; i += gridDim.x * blockDim.x) a.zero[i] = 0;
    const int KB = a.k / 128;
    const int lane = threadIdx.x & 31;
    const int jobs = a.rows * KB;
    for (int j = gt >> 5; j < jobs; j += (gridDim.x * blockDim.x) >> 5) {
        const int row = j / KB, kb = j % KB;
        float v[4];
        const __half* su = a.suh ? a.suh + kb * 128 : nullptr;
        if (a.x_bf16)
            rotated_block<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(a.x) + (size_t)row * a.ldx + kb * 128,
                                         su, lane, v);
        else
            rotated_block<__half>(reinterpret_cast<const __half*>(a.x) + (size_t)row * a.ldx + kb * 128, su, lane, v);
        store_xf_block(v, lane, a.xf + (size_t)row * a.k + (size_t)kb * 128);
        const float bs = xf_block_sum(v);
        if (lane == 0) a.xsum[(size_t)row * KB + kb] = bs;
    }
}

// ------------------------------------------------------------------------------------------------ host launch

// Launch with programmatic stream serialization (the kernel may start while the previous one finishes).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// Split-unit partial slots of a GEMV launch on the current device (workspace sizing): two per CTA.
inline int max_ctas() { return num_sms(); }
inline size_t partial_bytes(int epi, int rg = 1) { return (size_t)2 * max_ctas() * unit_floats(epi, rg) * 4; }

// Work decomposition: one CTA per SM, or fewer when the launch has fewer k-blocks; `ctas` > 0 overrides the count
// (tests, tuning).
struct GemvPlan {
    int ctas, smem;
};
inline GemvPlan plan_gemv(int epi, long long work_upper, int ctas, int rg = 1) {
    GemvPlan pl;
    const int sms = max_ctas();
    if (ctas <= 0) ctas = work_upper < sms ? (int)(work_upper < 1 ? 1 : work_upper) : sms;
    pl.ctas = ctas > sms ? sms : ctas;
    pl.smem = smem_layout(epi, rg).total;
    return pl;
}

template <int EPI, int RG = 1>
int launch_gemv(GemvArgs a, const GemvPlan& pl, cudaStream_t st, const char* what) {
    EXL3_REQUIRE(pl.smem <= 227 * 1024, EXL3_ERR_UNSUPPORTED, "%s: shared memory plan too large", what);
    auto kern = k_gemv<EPI, RG>;
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
    a.head_wait_ns = finisher_wait_ns();
    cudaError_t e = launch_pdl(kern, dim3(pl.ctas), dim3(kGemvThreads), pl.smem, st, a);
    if (e != cudaSuccess) {
        set_error("%s: launch failed: %s", what, cudaGetErrorString(e));
        return EXL3_ERR_CUDA;
    }
    return EXL3_OK;
}

inline int launch_prep(const PrepArgs& a, cudaStream_t st, const char* what) {
    const long jobs = (long)a.rows * (a.k / 128);
    long blocks = (jobs + 7) / 8;
    const long zb = (a.n_zero + 255) / 256;
    if (blocks < zb) blocks = zb;
    if (blocks > 4 * num_sms()) blocks = 4 * num_sms();
    if (blocks < 1) blocks = 1;
    cudaError_t e = launch_pdl(k_prep, dim3((unsigned)blocks), dim3(256), 0, st, a);
    if (e != cudaSuccess) {
        set_error("%s: prep launch failed: %s", what, cudaGetErrorString(e));
        return EXL3_ERR_CUDA;
    }
    return EXL3_OK;
}

}  // namespace exl3
