// EXL3 linears for prefill-sized batches on the 5th-generation tensor cores: the dense linear (any M) and the grouped
// MoE expert projections (rows grouped per expert by the alignment step).
//
// Shape of the contraction. The decoded weights are the MMA's A operand and live in TENSOR MEMORY; the rotated
// activation rows are the B operand in shared memory; the accumulator is D[feature][row] in tensor memory. A pair of
// CTAs (a 2-CTA cluster) runs one tile of 256 output features x up to 320 activation rows with
// tcgen05.mma.cta_group::2: CTA r decodes features [128 r, 128 r + 128) of the pair into its own TMEM lanes; the
// leader (rank 0) issues the MMAs for both. Per 16-deep k step the tile is two MMAs on the same decoded weights:
// rows 0..255 (N 256: CTA r supplies rows [128 r, 128 r + 128)) and, when the tile has more than 256 rows, rows
// 256..319 (N 64: CTA r supplies rows [256 + 32 r, 256 + 32 r + 32)). Each decoded weight thus serves up to 320
// rows, and the decoded weights never pass through shared memory: decoder warps write their fragments straight
// from registers with tcgen05.st; shared memory only carries the activations (TMA write + MMA read).
//
//   warp 0        TMA: the CTA's activation rows of the k-chunk ([160 rows][64 k] fp16 sub-tiles, 128-byte
//                 swizzle), completion counted on the leader's barrier (cp.async.bulk.tensor .cta_group::2);
//   warp 1        allocates the 512 TMEM columns of both CTAs; on the leader one lane issues the chunk's MMAs
//                 (M 256, K 16, A from TMEM) and commits each stage's release and, after the last chunk, the
//                 accumulators to both CTAs (tcgen05.commit multicast);
//   warp 2        bulk-copies the CTA's trellis tiles of the chunk into a ring;
//   warps 3..18   decode the trellis tiles (bit-exact fp16, register fragments) into the TMEM weight stage; after the
//                 main loop they run the epilogue, 128 rows at a time: TMEM -> shared memory [row][feature] fp32 ->
//                 output Hadamard per 128-feature block with warp shuffles -> the projection's epilogue.
// TMEM of each CTA: columns 0..319 the accumulators (lane = feature, column = activation row of the tile),
// 320..511 the weight ring (a k-chunk of 128 takes 64 columns: lane = feature, column c of a 16-deep step holds
// two k values).
//
// k order inside the contraction. tcgen05.st.16x256b stores a decoded fragment's registers {pair q, pair q + 4} of a
// 16-element k group into columns {2q, 2q + 1}; the MMA reads column c as k pair c. So every activation row is
// stored with the same fixed permutation inside each 16-element group: k pair p goes to pair slot
// (p < 4 ? 2p : 2p - 7). The rotation kernels below write rows in that order; the products are unchanged.
//
// Epilogues: linear (y = H(acc) * svh with the reference's fp16 roundings for fp16 y), MoE gate and up (the same
// fp16 output into the [2][positions][I] gate/up buffer; gate and up are separate pair tiles because the two
// matrices rotate the input with different signs), MoE down (routing weight x H(acc) * svh, fp32 rows). The
// activation between gate|up and down (SiLU * clamp, then the down input's rotation) is its own small kernel.
// All waits are bounded (EXL3_ERR_TIMEOUT in the device status word). No TMA multicast.
//
// Reference semantics: exl3_linear / ReconstructKernel + GEMM for M > 128 (glm/xpu/csrc/exl3_ops.sycl:539-555,
// 651-757; glm/docs/ext-op-inventory.md:597-612), the MoE prefill GateUpDpasKernel / DownDpasKernel
// (glm/xpu/csrc/exl3_moe.n128.sycl:422-690,868-916) and the expert math (glm/docs/ext-op-inventory.md:923-942).
#include "gemv.cuh"
#include "tc.cuh"

namespace exl3 {

#ifndef EXL3_TS_KS
#define EXL3_TS_KS 2
#endif
constexpr int TS_KS = EXL3_TS_KS;                             // 64-deep sub-chunks per k-chunk
constexpr int TS_BK = 64 * TS_KS;                             // k-chunk
constexpr int TS_N2 = 64;                                     // N of the second MMA (tile rows 256..319)
constexpr int TS_TILE_ROWS = 256 + TS_N2;                     // activation rows per pair tile
static_assert(TS_TILE_ROWS == kTcTileRows, "tile rows shared with the alignment step");
constexpr int TS_CROWS = 128 + TS_N2 / 2;                     // activation rows per CTA
constexpr int TS_DEC_WARPS = 16;
constexpr int TS_WARPS = 3 + TS_DEC_WARPS;
constexpr int TS_THREADS = TS_WARPS * 32;
constexpr int TS_SUB = TS_CROWS * 64 * 2;                     // one swizzled [160 rows][64 k] fp16 sub-tile
constexpr int TS_SUB2 = 128 * 64 * 2;                         // offset of the second MMA's rows in a sub-tile
constexpr int TS_B_STAGE = TS_KS * TS_SUB;
constexpr int TS_A_COL0 = 256 + TS_N2;                        // first TMEM column of the weight ring
constexpr int TS_A_COLS = TS_BK / 2;                          // TMEM columns of one weight stage
constexpr int TS_STAGES = (512 - TS_A_COL0) / TS_A_COLS;      // weight (and activation) stages
constexpr int TS_B_RING = TS_STAGES * TS_B_STAGE;             // activation ring (also the epilogue staging)
constexpr int TS_T_RING = 32 * 1024;                          // trellis ring
constexpr int TS_MAX_TSTAGES = 8;
constexpr int TS_TR = TS_BK / 16;                             // tile-rows per chunk
static_assert(TS_STAGES >= 2 && TS_SUB % 1024 == 0 && TS_SUB2 % 1024 == 0, "ring geometry");
static_assert(TS_B_RING >= 128 * 128 * 4, "epilogue staging [128 rows][128 features] fp32 fits the ring");

struct TsSmem {
    static constexpr int b0 = 0;
    static constexpr int t0 = TS_B_RING;
    static constexpr int bars = t0 + TS_T_RING;
    // b_full[S], a_full[S], empty[S], t_full[8], t_empty[8], acc_full
    static constexpr int n_bars = 3 * TS_STAGES + 2 * TS_MAX_TSTAGES + 1;
    static constexpr int tmem_slot = bars + n_bars * 8;
    static constexpr int total = tmem_slot + 16 + 1024;        // + slack for 1024-byte alignment of the base
};

// ---- cluster, TMA, tcgen05 wrappers ----
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
    return r;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on a barrier of either CTA of the pair (shared::cluster address). The data it publishes is tensor memory
// written with tcgen05.st and completed by tcgen05.wait::st + tcgen05.fence::before_thread_sync, read by the MMAs the
// leader issues after its wait; the default CTA-scope release suffices for that hand-off (a cluster-scope release is
// a full fence per arrival and costs about a microsecond).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 2D tile load into this CTA's shared memory; the transaction bytes complete on the barrier at `bar_cluster` (the
// leader CTA's barrier). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cluster) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[tmem] x B[smem desc]^T over both CTAs of the pair (M 256, N from idesc, K 16)
__device__ __forceinline__ void tc2_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n"
        ::"r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the barrier at this offset in both CTAs of the pair when the MMAs issued so far have completed.
__device__ __forceinline__ void tc2_commit_both(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"((uint16_t)3)
        : "memory");
}
// 16 TMEM lanes x 8 columns from the warp's registers: thread t -> lanes t/4 and t/4 + 8, columns 2(t%4), 2(t%4)+1
// (r0, r1 on the first lane, r2, r3 on the second).
__device__ __forceinline__ void tmem_st_16x256b(uint32_t taddr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    asm volatile("tcgen05.st.sync.aligned.16x256b.x1.b32 [%0], {%1, %2, %3, %4};" ::"r"(taddr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3)
                 : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (thread i <- lane base + i).
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t r[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Four fp16 values (8 bytes) widened to fp32.
__device__ __forceinline__ void unpack_h4(uint2 u, float v[4]) {
    const __half2 a = *reinterpret_cast<const __half2*>(&u.x), b = *reinterpret_cast<const __half2*>(&u.y);
    v[0] = __low2float(a);
    v[1] = __high2float(a);
    v[2] = __low2float(b);
    v[3] = __high2float(b);
}

// Shared-memory matrix descriptor of a [rows][64] fp16 sub-tile: canonical K-major layout, 128-byte swizzle, 8-row
// atoms 1024 bytes apart, sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_f16(int M, int N) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

struct TsArgs {
    // linear: one packed matrix [n/128][k/16][8 tiles][8K words], its svh
    const uint8_t* packed;
    const __half* svh;
    int K;
    // linear: y [M][ldy]; gate|up: the gate/up buffer [2][M][ldy] fp16 (M = positions, ldy = I)
    void* y;
    int ldy, y_dtype;
    int M, k, n;                  // rows (linear) or positions (grouped); k, n of the projection
    // grouped: alignment tables (items of <= 320 positions of one expert) and the expert table
    const int* n_items;
    const int* item_expert;
    const int* item_start;
    const int* item_cnt;
    const float* pair_w;          // down: routing weight of a position
    const ExpertDesc* experts;
    float* ybuf;                  // down: weighted rows [positions][n] fp32
    int* status;
};

// ------------------------------------------------------------------------------------------------ decode

// One decoder warp: lane quadrant q (TMEM lanes 32q..32q+31 = features of n-tiles 2q, 2q+1) and k-tile j of every
// 64-deep sub-chunk; per chunk it decodes 2 TS_KS tiles and stores each as one 16x256b block of the weight stage.
template <int K>
__device__ void ts_decoder_loop(uint8_t* smem, uint32_t tmem, int q, int j, int lane, bool has_cols, int nk,
                                int t_stages, uint32_t t_blk, uint64_t* t_full, uint64_t* t_empty, uint64_t* empty,
                                uint32_t lead_a_full, bool& to) {
    const LaneWords lw = lane_words<K>(lane);
    int ts = 0, s = 0;                                        // ring slots, advanced per chunk (no divisions)
    uint32_t tph = 0, eph = 1;                                // parity awaited on t_full[ts] / on empty[s]
    for (int kc = 0; kc < nk; ++kc) {
        bool ok = true;
        if (has_cols && !to) ok = mbar_wait(&t_full[ts], tph);
        if (ok && kc >= TS_STAGES && !to) ok = mbar_wait(&empty[s], eph);
        if (!__all_sync(0xFFFFFFFFu, ok)) to = true;
        if (has_cols && !to) {
            // all words of the chunk's tiles first, then the decodes, then the stores (the stores are ordered
            // asm statements; loads issued after one would wait for it)
            constexpr int NT = 2 * TS_KS;
            const uint32_t* tst = reinterpret_cast<const uint32_t*>(smem + TsSmem::t0 + (size_t)ts * t_blk);
            uint32_t w[NT][3];
#pragma unroll
            for (int t = 0; t < NT; ++t) {
                const uint32_t* tile = tst + ((j + 4 * (t >> 1)) * 8 + 2 * q + (t & 1)) * 8 * K;
                w[t][0] = tile[lw.i0];
                w[t][1] = tile[lw.i1];
                w[t][2] = K >= 3 ? tile[lw.i2] : 0u;          // K <= 2: the lane's bits span two words
            }
            uint32_t a[NT][4];
#pragma unroll
            for (int t = 0; t < NT; ++t) decode_frag_words<K>(w[t][0], w[t][1], w[t][2], lw.off, a[t]);
#pragma unroll
            for (int t = 0; t < NT; ++t)   // a = {n g, pair q'}, {n g+8, pair q'}, {n g, pair q'+4}, {n g+8, pair q'+4}
                tmem_st_16x256b(tmem + ((uint32_t)(32 * q + 16 * (t & 1)) << 16) +
                                    (uint32_t)(TS_A_COL0 + s * TS_A_COLS + (j + 4 * (t >> 1)) * 8),
                                a[t][0], a[t][2], a[t][1], a[t][3]);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
            mbar_arrive_cluster(lead_a_full + 8u * s);
            if (has_cols) mbar_arrive(&t_empty[ts]);
        }
        if (++ts == t_stages) { ts = 0; tph ^= 1u; }
        if (++s == TS_STAGES) { s = 0; eph ^= 1u; }
    }
}

__device__ void ts_decoder_dispatch(int K, uint8_t* smem, uint32_t tmem, int q, int j, int lane, bool has_cols,
                                    int nk, int t_stages, uint32_t t_blk, uint64_t* t_full, uint64_t* t_empty,
                                    uint64_t* empty, uint32_t lead_a_full, bool& to) {
#define EXL3_TS_DEC(KK) \
    ts_decoder_loop<KK>(smem, tmem, q, j, lane, has_cols, nk, t_stages, t_blk, t_full, t_empty, empty, lead_a_full, to)
    switch (K) {
        case 1: EXL3_TS_DEC(1); break;
        case 2: EXL3_TS_DEC(2); break;
        case 3: EXL3_TS_DEC(3); break;
        case 4: EXL3_TS_DEC(4); break;
        case 5: EXL3_TS_DEC(5); break;
        case 6: EXL3_TS_DEC(6); break;
        case 7: EXL3_TS_DEC(7); break;
        default: EXL3_TS_DEC(8); break;
    }
#undef EXL3_TS_DEC
}

// ------------------------------------------------------------------------------------------------ kernel

// Activation tensor maps of one launch: per matrix (gate|up: gate, up), boxes of 128 and of 32 rows.
struct TsMaps {
    CUtensorMap m[2][2];
};

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(TS_THREADS, 1)
    k_gemm_pair(const __grid_constant__ TsMaps maps, const TsArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_rank();
    pdl_trigger();

    // ---- the pair tile: activation rows [m0, m0 + rows), rows <= 320; this CTA's 128-feature column block cb ----
    int m0, rows, Kw = p.K, cb, mat = 0, expert = 0;
    const uint8_t* wsrc;                                      // the CTA's trellis, tile-row 0
    size_t row_stride;                                        // bytes between tile-rows in wsrc
    const __half* svh;
    if constexpr (EPI == TC_LINEAR) {
        m0 = blockIdx.y * TS_TILE_ROWS;
        rows = min(TS_TILE_ROWS, p.M - m0);
        cb = blockIdx.x;
        row_stride = (size_t)8 * 32 * Kw;
        wsrc = p.packed + (size_t)cb * (p.k / 16) * row_stride;
        svh = p.svh;
    } else {
        pdl_wait();                                           // the alignment tables come from an earlier kernel
        const int item = blockIdx.y;
        if (item >= __ldcg(p.n_items)) return;                // both CTAs of the pair: before any cluster barrier
        expert = __ldcg(p.item_expert + item);
        m0 = __ldcg(p.item_start + item);
        rows = __ldcg(p.item_cnt + item);
        const ExpertDesc& ed = p.experts[expert];
        if constexpr (EPI == TC_GATEUP) {
            const int npm = (p.n + 255) / 256;                // pairs per matrix
            const int pp = blockIdx.x >> 1;
            mat = pp / npm;
            cb = 2 * (pp % npm) + (int)rank;
            const int Kg = ed.K[0], Ku = ed.K[1];
            Kw = mat ? Ku : Kg;
            row_stride = (size_t)8 * 32 * (Kg + Ku);          // fused [I/128][H/16][8 gate | 8 up]
            wsrc = reinterpret_cast<const uint8_t*>(ed.tr[0]) + (size_t)cb * (p.k / 16) * row_stride +
                   (mat ? 8 * 32 * Kg : 0);
            svh = ed.svh[mat];
        } else {
            Kw = ed.K[2];
            cb = blockIdx.x;
            row_stride = (size_t)8 * 32 * Kw;
            wsrc = reinterpret_cast<const uint8_t*>(ed.tr[2]) + (size_t)cb * (p.k / 16) * row_stride;
            svh = ed.svh[2];
        }
    }
    const bool has_cols = (cb + 1) * 128 <= p.n;              // the last pair of an odd block count has one
    const bool has2 = rows > 256;                             // the second MMA (rows 256..319) is needed
    const int nk = p.k / TS_BK;
    const uint32_t t_blk = (uint32_t)(TS_TR * 8 * 32 * Kw);  // trellis bytes of one chunk
    int t_stages = TS_T_RING / (int)t_blk;
    if (t_stages > TS_MAX_TSTAGES) t_stages = TS_MAX_TSTAGES;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TsSmem::bars);
    uint64_t* b_full = bars;                                  // leader: activation stage landed (both CTAs)
    uint64_t* a_full = b_full + TS_STAGES;                    // leader: weight stage decoded (both CTAs)
    uint64_t* empty = a_full + TS_STAGES;                     // both: the stage's MMAs completed
    uint64_t* t_full = empty + TS_STAGES;
    uint64_t* t_empty = t_full + TS_MAX_TSTAGES;
    uint64_t* acc_full = t_empty + TS_MAX_TSTAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TsSmem::tmem_slot);

    if (threadIdx.x == 0) {
        for (int s = 0; s < TS_STAGES; ++s) {
            mbar_init(&b_full[s], 1);
            mbar_init(&a_full[s], 2 * TS_DEC_WARPS);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < t_stages; ++s) {
            mbar_init(&t_full[s], 1);
            mbar_init(&t_empty[s], TS_DEC_WARPS);
        }
        mbar_init(acc_full, 1);
        fence_barrier_init();
    }
    if (warp == 1) {                                          // TMEM: all 512 columns of both CTAs
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();                                           // barriers and TMEM ready in both CTAs
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t lead_b_full = map_to_rank(smem_u32(b_full), 0);
    const uint32_t lead_a_full = map_to_rank(smem_u32(a_full), 0);
    bool to = false;

    if (warp == 0) {
        // ---------------- activation rows (TMA) ----------------
        if constexpr (EPI == TC_LINEAR) pdl_wait();           // the rotated rows come from an earlier kernel
        if (lane == 0) {
            const CUtensorMap* map1 = &maps.m[EPI == TC_GATEUP ? mat : 0][0];
            const CUtensorMap* map2 = &maps.m[EPI == TC_GATEUP ? mat : 0][1];
            const int row1 = m0 + 128 * (int)rank, row2 = m0 + 256 + (TS_N2 / 2) * (int)rank;
            const uint32_t tx = 2u * TS_KS * (has2 ? TS_SUB : TS_SUB2);   // both CTAs' bytes of a stage
            int last[TS_STAGES];
            for (int s = 0; s < TS_STAGES; ++s) last[s] = -1;
            int s = 0;
            uint32_t eph = 1;
            for (int kc = 0; kc < nk; ++kc, s = s + 1 == TS_STAGES ? 0 : s + 1, eph ^= (s == 0)) {
                if (kc >= TS_STAGES && !mbar_wait(&empty[s], eph)) { to = true; break; }
                if (rank == 0) mbar_expect_tx(&b_full[s], tx);
                uint8_t* dst = smem + TsSmem::b0 + s * TS_B_STAGE;
#pragma unroll
                for (int si = 0; si < TS_KS; ++si) {
                    tma_load_2d_pair(dst + si * TS_SUB, map1, kc * TS_BK + si * 64, row1, lead_b_full + 8u * s);
                    if (has2)
                        tma_load_2d_pair(dst + si * TS_SUB + TS_SUB2, map2, kc * TS_BK + si * 64, row2,
                                         lead_b_full + 8u * s);
                }
                last[s] = kc;
            }
            if (rank == 0)                                    // both CTAs' copies landed before the pair may exit
                for (int s = 0; s < TS_STAGES; ++s)
                    if (last[s] >= 0 && !mbar_wait(&b_full[s], (last[s] / TS_STAGES) & 1)) to = true;
        }
    } else if (warp == 1) {
        // ---------------- MMA issue (leader, one lane) ----------------
        if (rank == 0 && lane == 0) {
            constexpr uint32_t idesc1 = tc_idesc_f16(256, 256), idesc2 = tc_idesc_f16(256, TS_N2);
            int s = 0;
            uint32_t ph = 0;
            for (int kc = 0; kc < nk; ++kc, s = s + 1 == TS_STAGES ? 0 : s + 1, ph ^= (s == 0)) {
                // no tcgen05 fence per chunk: the decoders complete their tensor-memory stores (tcgen05.wait::st)
                // before arriving, and a fence here would hold the MMAs until the queue drains every chunk
                if (!to && !mbar_wait(&a_full[s], ph)) to = true;
                if (!to && !mbar_wait(&b_full[s], ph)) to = true;
                if (!to) {
                    const uint32_t b_base = smem_u32(smem + TsSmem::b0 + s * TS_B_STAGE);
#pragma unroll
                    for (int kk = 0; kk < TS_BK / 16; ++kk) {
                        const uint32_t a_t = tmem + (uint32_t)(TS_A_COL0 + s * TS_A_COLS + kk * 8);
                        const uint32_t b_s = b_base + (kk >> 2) * TS_SUB + (kk & 3) * 32;
                        tc2_mma_ts(tmem, a_t, sw128_desc(b_s), idesc1, (kc | kk) != 0);
                        if (has2) tc2_mma_ts(tmem + 256, a_t, sw128_desc(b_s + TS_SUB2), idesc2, (kc | kk) != 0);
                    }
                }
                tc2_commit_both(&empty[s]);                   // both CTAs' stages are free once these completed
            }
            tc2_commit_both(acc_full);
        }
    } else if (warp == 2) {
        // ---------------- trellis tiles (bulk copies) ----------------
        if (lane == 0 && has_cols) {
            int last[TS_MAX_TSTAGES];
            for (int s = 0; s < TS_MAX_TSTAGES; ++s) last[s] = -1;
            const uint32_t tile_row_bytes = (uint32_t)(8 * 32 * Kw);
            int ts = 0;
            uint32_t eph = 1;
            for (int kc = 0; kc < nk; ++kc, ts = ts + 1 == t_stages ? 0 : ts + 1, eph ^= (ts == 0)) {
                if (kc >= t_stages && !mbar_wait(&t_empty[ts], eph)) { to = true; break; }
                mbar_expect_tx(&t_full[ts], t_blk);
                uint8_t* dst = smem + TsSmem::t0 + (size_t)ts * t_blk;
                if constexpr (EPI == TC_GATEUP) {
                    for (int tr = 0; tr < TS_TR; ++tr)
                        bulk_g2s(dst + tr * tile_row_bytes, wsrc + (size_t)(kc * TS_TR + tr) * row_stride,
                                 tile_row_bytes, &t_full[ts]);
                } else {
                    bulk_g2s(dst, wsrc + (size_t)kc * t_blk, t_blk, &t_full[ts]);
                }
                last[ts] = kc;
            }
            for (int s = 0; s < t_stages; ++s)
                if (last[s] >= 0 && !mbar_wait(&t_full[s], (last[s] / t_stages) & 1)) to = true;
        }
    } else {
        // ---------------- decoders, then the epilogue ----------------
        const int dw = warp - 3, q = warp & 3, j = dw >> 2;
        ts_decoder_dispatch(Kw, smem, tmem, q, j, lane, has_cols, nk, t_stages, t_blk, t_full, t_empty, empty,
                            lead_a_full, to);

        if constexpr (EPI == TC_LINEAR) pdl_wait();           // y may be in use by an earlier kernel until here
        if (!to && !mbar_wait(acc_full, 0)) to = true;
        if (!__all_sync(0xFFFFFFFFu, !to)) to = true;
        tc_fence_after();
        // 128 rows per pass: accumulator lanes 32q..32q+31 (features), columns 128 pass + 32j .. + 31 (rows) ->
        // staging [128 rows][128 features]
        float* stage = reinterpret_cast<float*>(smem + TsSmem::b0);
        const int col = cb * 128 + 4 * lane;                  // output feature of the projection
        // per-lane constants of the epilogue, loaded once: the lane's svh values and (down) the routing weights of
        // the warp's rows (row dw + 16 i in lane i)
        float sv[4] = {0.f, 0.f, 0.f, 0.f};
        float wrow = 0.f;
        if (has_cols) {
            const uint2 u = __ldg(reinterpret_cast<const uint2*>(svh + col));
            unpack_h4(u, sv);
        }
        if constexpr (EPI == TC_DOWN)
            if (dw + TS_DEC_WARPS * lane < rows) wrow = __ldcg(p.pair_w + m0 + dw + TS_DEC_WARPS * lane);
        for (int r0 = 0; r0 < rows; r0 += 128) {               // rows is uniform: every warp takes each barrier
            if (!to && r0 + 32 * j < rows) {
                uint32_t r[32];
                tc_ld32(tmem + ((uint32_t)(32 * q) << 16) + (uint32_t)(r0 + 32 * j), r);
#pragma unroll
                for (int c = 0; c < 32; ++c) stage[(32 * j + c) * 128 + 32 * q + lane] = __uint_as_float(r[c]);
            }
            asm volatile("bar.sync 1, %0;" ::"r"(TS_DEC_WARPS * 32) : "memory");
            for (int t = r0 + dw; t < min(rows, r0 + 128) && has_cols && !to; t += TS_DEC_WARPS) {
                const float4 s4 = *reinterpret_cast<const float4*>(stage + (t - r0) * 128 + 4 * lane);
                float v[4] = {s4.x, s4.y, s4.z, s4.w};
                fwht128_warp(v, lane);
                const int m = m0 + t;
                if constexpr (EPI == TC_DOWN) {
                    const float wgt = __shfl_sync(0xFFFFFFFFu, wrow, (t - dw) / TS_DEC_WARPS);
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) o[e] = wgt * (v[e] * kRsqrt128 * sv[e]);
                    *reinterpret_cast<float4*>(p.ybuf + (size_t)m * p.n + col) = make_float4(o[0], o[1], o[2], o[3]);
                } else {
                    const int ydt = EPI == TC_GATEUP ? EXL3_F16 : p.y_dtype;
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        if (ydt == EXL3_F16)
                            o[e] = __half2float(__float2half_rn(__half2float(__float2half_rn(v[e] * kRsqrt128)) * sv[e]));
                        else
                            o[e] = v[e] * kRsqrt128 * sv[e];
                    }
                    const size_t yrow = (EPI == TC_GATEUP ? (size_t)mat * p.M : 0) + (size_t)m;
                    if (ydt == EXL3_F32) {
                        *reinterpret_cast<float4*>(static_cast<float*>(p.y) + yrow * p.ldy + col) =
                            make_float4(o[0], o[1], o[2], o[3]);
                    } else if (ydt == EXL3_F16) {
                        __half2 h01 = __floats2half2_rn(o[0], o[1]), h23 = __floats2half2_rn(o[2], o[3]);
                        uint2 u;
                        u.x = *reinterpret_cast<uint32_t*>(&h01);
                        u.y = *reinterpret_cast<uint32_t*>(&h23);
                        *reinterpret_cast<uint2*>(static_cast<__half*>(p.y) + yrow * p.ldy + col) = u;
                    } else {
                        __nv_bfloat16* yp = static_cast<__nv_bfloat16*>(p.y) + yrow * p.ldy + col;
#pragma unroll
                        for (int e = 0; e < 4; ++e) yp[e] = __float2bfloat16_rn(o[e]);
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(TS_DEC_WARPS * 32) : "memory");
        }
    }
    if (to) report(p.status, EXL3_ERR_TIMEOUT);
    __syncwarp();
    tc_fence_before();
    cluster_sync();                                           // both CTAs done with TMEM and shared memory
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------ activation rows

// A 128-element block lives in a lane quad: lane i = lane % 4 holds elements 32 i .. 32 i + 31, so a warp works on 8
// blocks at once (8 consecutive blocks of one row) and only the last two of the seven Hadamard stages cross lanes.
constexpr int kQuadBlocks = 8;                                // blocks per warp (one per quad)
constexpr uint2 kOnes4 = {0x3C003C00u, 0x3C003C00u};          // four fp16 ones (a missing sign vector)

template <typename T>
__device__ __forceinline__ void unpack4(uint2 u, float* v) {
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) v[j] = to_f32<T>(e[j]);
}
// The lane's 32 consecutive 16-bit values (8-byte aligned) as 8 raw 8-byte words; `ones` when src is null.
__device__ __forceinline__ void load32_raw(const void* src, uint2 r[8]) {
    const uint2* p = reinterpret_cast<const uint2*>(src);
#pragma unroll
    for (int c = 0; c < 8; ++c) r[c] = p ? __ldg(p + c) : kOnes4;
}
__device__ __forceinline__ void load32_raw_cg(const void* src, uint2 r[8]) {
    const uint2* p = reinterpret_cast<const uint2*>(src);
#pragma unroll
    for (int c = 0; c < 8; ++c) r[c] = __ldcg(p + c);
}

// 128-point Walsh-Hadamard transform of a quad's block: stages h = 1 .. 16 inside the lane, h = 32 and 64 across
// the quad (lane xor 1, 2); the natural stage order with (a, b) -> (a + b, a - b) in fp32, as fwht128_warp.
__device__ __forceinline__ void fwht128_quad(float v[32], int lane) {
#pragma unroll
    for (int h = 1; h < 32; h <<= 1)
#pragma unroll
        for (int e = 0; e < 32; ++e)
            if ((e & h) == 0) {
                const float a = v[e], b = v[e + h];
                v[e] = a + b;
                v[e + h] = a - b;
            }
#pragma unroll
    for (int m = 1; m < 4; m <<= 1) {
        const float sgn = (lane & m) ? -1.0f : 1.0f;      // fma(v, -1, p) = p - v, fma(v, 1, p) = v + p
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = fmaf(v[e], sgn, __shfl_xor_sync(0xFFFFFFFFu, v[e], m));
    }
}

// xh = fp16(H(fp16(v * s)) / sqrt(128)) for the quad's block (v: the lane's 32 values, s: its 32 signs), stored at
// dst (the lane's 32 elements, 16-byte aligned) in the operand's k order: inside each 16-element group, k pair p goes
// to pair slot p < 4 ? 2p : 2p - 7, i.e. the group's pair words in the order 0 4 1 5 2 6 3 7. `store` is per lane;
// every lane of the warp must call this (the transform shuffles). The lanes' destinations are consecutive (lane l at
// lane 0's + 64 l bytes, lane 0 storing): the warp's 2 KB go through `stage` (the warp's 128 uint4 of shared memory,
// 16-byte chunks swizzled against bank conflicts) and out as four 512-byte contiguous stores.
__device__ __forceinline__ int stage_slot(int src, int c) { return 4 * src + (c ^ ((src >> 1) & 3)); }

__device__ __forceinline__ void rotate_store32(float v[32], const uint2 sraw[8], int lane, __half* dst, bool store,
                                               uint4* stage) {
#pragma unroll
    for (int c = 0; c < 8; ++c) {
        float sg[4];
        unpack4<__half>(sraw[c], sg);
#pragma unroll
        for (int j = 0; j < 4; ++j) v[4 * c + j] = __half2float(__float2half_rn(v[4 * c + j] * sg[j]));
    }
    fwht128_quad(v, lane);
    uint32_t w[16];
#pragma unroll
    for (int pp = 0; pp < 16; ++pp) {
        const __half2 h = __floats2half2_rn(v[2 * pp] * kRsqrt128, v[2 * pp + 1] * kRsqrt128);
        w[pp] = *reinterpret_cast<const uint32_t*>(&h);
    }
#pragma unroll
    for (int g = 0; g < 2; ++g) {
        const uint32_t* P = w + 8 * g;
        stage[stage_slot(lane, 2 * g)] = make_uint4(P[0], P[4], P[1], P[5]);
        stage[stage_slot(lane, 2 * g + 1)] = make_uint4(P[2], P[6], P[3], P[7]);
    }
    __syncwarp();
    const unsigned long long base = __shfl_sync(0xFFFFFFFFu, reinterpret_cast<unsigned long long>(dst), 0);
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const int src = 8 * g + (lane >> 2);                  // chunk 32 g + lane: chunk lane & 3 of lane src
        if (__shfl_sync(0xFFFFFFFFu, store, src))
            reinterpret_cast<uint4*>(base)[32 * g + lane] = stage[stage_slot(src, lane & 3)];
    }
    __syncwarp();                                             // the stage is reused by the warp's next job
}

// Rotated input rows of the dense linear, in the operand's k order: xh[m][k]. One warp per (row, 8 blocks).
template <typename T>
static __global__ void __launch_bounds__(256, 2) k_rotate_rows(const T* x, int ldx, int M, int k, const __half* suh,
                                                               __half* xh) {
    __shared__ uint4 s_stage[8][128];
    pdl_wait();
    pdl_trigger();
    const int KB = k / 128, lane = threadIdx.x & 31, i = lane & 3;
    const int nkg = (KB + kQuadBlocks - 1) / kQuadBlocks;
    const long njobs = (long)M * nkg;
    const long nw = ((long)gridDim.x * blockDim.x) >> 5;
    for (long job = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; job < njobs; job += nw) {
        const int row = (int)(job / nkg), kb = (int)(job % nkg) * kQuadBlocks + (lane >> 2);
        const bool act = kb < KB;
        const int off = (act ? kb : 0) * 128 + 32 * i;
        uint2 xr[8], sr[8];
        load32_raw(x + (size_t)row * ldx + off, xr);
        load32_raw(suh ? suh + off : nullptr, sr);
        float v[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) unpack4<T>(xr[c], v + 4 * c);
        rotate_store32(v, sr, lane, xh + (size_t)row * k + off, act, s_stage[threadIdx.x >> 5]);
    }
}

// Rotated gate and up input rows of every pair position, in the operand's k order: a_gu[mat][pos][H] =
// rot(x[token] * suh of the position's expert's matrix mat). One warp per (position, 8 blocks); the token's values
// are loaded once for both matrices.
template <typename T>
static __global__ void __launch_bounds__(256, 2) k_rotate_pairs(const T* x, int ldx, int H, int P, const int* n_pos,
                                                                const int* pair_tok, const int* pair_expert,
                                                                const ExpertDesc* experts, __half* a_gu) {
    __shared__ uint4 s_stage[8][128];
    pdl_wait();
    pdl_trigger();
    const int KB = H / 128, lane = threadIdx.x & 31, i = lane & 3;
    const int nkg = (KB + kQuadBlocks - 1) / kQuadBlocks;
    const long njobs = (long)min(P, __ldcg(n_pos)) * nkg;
    const long nw = ((long)gridDim.x * blockDim.x) >> 5;
    for (long job = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; job < njobs; job += nw) {
        const int pos = (int)(job / nkg), kb = (int)(job % nkg) * kQuadBlocks + (lane >> 2);
        const bool act = kb < KB;
        const int off = (act ? kb : 0) * 128 + 32 * i;
        const int tok = __ldcg(pair_tok + pos), e = __ldcg(pair_expert + pos);
        const __half* s0 = experts[e].suh[0];
        const __half* s1 = experts[e].suh[1];
        uint2 xr[8], gr[8], ur[8];
        load32_raw(x + (size_t)tok * ldx + off, xr);
        load32_raw(s0 ? s0 + off : nullptr, gr);
        load32_raw(s1 ? s1 + off : nullptr, ur);
        float v[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) unpack4<T>(xr[c], v + 4 * c);
        rotate_store32(v, gr, lane, a_gu + (size_t)pos * H + off, act, s_stage[threadIdx.x >> 5]);
#pragma unroll
        for (int c = 0; c < 8; ++c) unpack4<T>(xr[c], v + 4 * c);
        rotate_store32(v, ur, lane, a_gu + ((size_t)P + pos) * H + off, act, s_stage[threadIdx.x >> 5]);
    }
}

// The down projection's input rows from the gate and up outputs, in the operand's k order:
// a = fp16(min(silu(g), L) * clamp(u, -L, L)) (no clamp when L = 0), a_dn[pos] = fp16(H(fp16(a * suh_down)) / sqrt(128)).
// One warp per (position, 8 blocks).
static __global__ void __launch_bounds__(256, 2) k_act(const __half* gu, int I, int P, const int* n_pos,
                                                       const int* pair_expert, const ExpertDesc* experts,
                                                       float act_limit, __half* a_dn) {
    __shared__ uint4 s_stage[8][128];
    pdl_wait();
    pdl_trigger();
    const int KB = I / 128, lane = threadIdx.x & 31, i = lane & 3;
    const int nkg = (KB + kQuadBlocks - 1) / kQuadBlocks;
    const long njobs = (long)min(P, __ldcg(n_pos)) * nkg;
    const long nw = ((long)gridDim.x * blockDim.x) >> 5;
    for (long job = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; job < njobs; job += nw) {
        const int pos = (int)(job / nkg), kb = (int)(job % nkg) * kQuadBlocks + (lane >> 2);
        const bool act = kb < KB;
        const int off = (act ? kb : 0) * 128 + 32 * i;
        const __half* sd = experts[__ldcg(pair_expert + pos)].suh[2];
        uint2 gr[8], ur[8], sr[8];
        load32_raw_cg(gu + (size_t)pos * I + off, gr);
        load32_raw_cg(gu + ((size_t)P + pos) * I + off, ur);
        load32_raw(sd ? sd + off : nullptr, sr);
        float v[32];
#pragma unroll
        for (int c = 0; c < 8; ++c) {
            float g[4], u[4];
            unpack4<__half>(gr[c], g);
            unpack4<__half>(ur[c], u);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                float sg = silu_f(g[j]), uu = u[j];
                if (act_limit != 0.f) {
                    sg = fminf(sg, act_limit);
                    uu = fminf(fmaxf(uu, -act_limit), act_limit);
                }
                v[4 * c + j] = __half2float(__float2half_rn(sg * uu));
            }
        }
        rotate_store32(v, sr, lane, a_dn + (size_t)pos * I + off, act, s_stage[threadIdx.x >> 5]);
    }
}

// Grid of the element-wise kernels: one warp per job, up to 2 CTAs of 8 warps per SM resident.
static dim3 row_grid(long jobs) {
    long blocks = (jobs + 7) / 8;
    if (blocks > 4L * num_sms()) blocks = 4L * num_sms();
    if (blocks < 1) blocks = 1;
    return dim3((unsigned)blocks);
}

// ------------------------------------------------------------------------------------------------ host launch

using PFN_encode_tiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Tensor map of a row-major [rows][cols] fp16 matrix: boxes of 64 columns x box_rows rows, 128-byte swizzle (the
// MMA descriptors' layout), zero fill beyond the last row.
static int make_row_map(CUtensorMap* map, const __half* base, long rows, int cols, int box_rows, const char* what) {
    static PFN_encode_tiled encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        EXL3_REQUIRE(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
                         q == cudaDriverEntryPointSuccess && fn,
                     EXL3_ERR_CUDA, "%s: cuTensorMapEncodeTiled is not available", what);
        encode = reinterpret_cast<PFN_encode_tiled>(fn);
    }
    const cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    EXL3_REQUIRE(cr == CUDA_SUCCESS, EXL3_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)cr);
    return EXL3_OK;
}

// The two maps (128-row and 32-row boxes) of a [rows][cols] activation matrix.
static int make_maps(CUtensorMap m[2], const __half* base, long rows, int cols, const char* what) {
    int rc = make_row_map(&m[0], base, rows, cols, 128, what);
    return rc ? rc : make_row_map(&m[1], base, rows, cols, TS_N2 / 2, what);
}

template <int EPI>
static int launch_pair(const TsMaps& maps, const TsArgs& a, dim3 grid, cudaStream_t st, const char* what) {
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        EXL3_REQUIRE(cudaFuncSetAttribute(k_gemm_pair<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          TsSmem::total) == cudaSuccess,
                     EXL3_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", what, cudaGetErrorString(cudaGetLastError()));
        configured[dev] = 1;
    }
    cudaError_t e = launch_pdl(k_gemm_pair<EPI>, grid, dim3(TS_THREADS), TsSmem::total, st, maps, a);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return EXL3_OK;
}

int tc_moe_prefill(const TcMoeArgs& m, cudaStream_t st) {
    const char* what = "exl3_moe_prefill";
    cudaError_t e;
    const dim3 rg = row_grid((long)m.P * ((m.H / 128 + kQuadBlocks - 1) / kQuadBlocks));
    if (m.x_bf16)
        e = launch_pdl(k_rotate_pairs<__nv_bfloat16>, rg, dim3(256), 0, st,
                       static_cast<const __nv_bfloat16*>(m.x), m.ldx, m.H, m.P, m.n_pos, m.pair_tok, m.pair_expert,
                       m.experts, m.a_gu);
    else
        e = launch_pdl(k_rotate_pairs<__half>, rg, dim3(256), 0, st, static_cast<const __half*>(m.x), m.ldx, m.H,
                       m.P, m.n_pos, m.pair_tok, m.pair_expert, m.experts, m.a_gu);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "%s: rotate launch failed: %s", what, cudaGetErrorString(e));
    if (m.max_items == 0) return EXL3_OK;
    TsArgs a = {};
    a.n_items = m.n_items;
    a.item_expert = m.item_expert;
    a.item_start = m.item_start;
    a.item_cnt = m.item_cnt;
    a.pair_w = m.pair_w;
    a.experts = m.experts;
    a.ybuf = m.ybuf;
    a.status = device_status_ptr();
    a.M = m.P;
    TsMaps mgu, mdn;
    int rc = make_maps(mgu.m[0], m.a_gu, m.P, m.H, what);
    if (!rc) rc = make_maps(mgu.m[1], m.a_gu + (size_t)m.P * m.H, m.P, m.H, what);
    if (!rc) rc = make_maps(mdn.m[0], m.a_dn, m.P, m.I, what);
    if (rc) return rc;
    mdn.m[1][0] = mdn.m[0][0];
    mdn.m[1][1] = mdn.m[0][1];
    // gate and up: (I/256 rounded up) pairs per matrix, both matrices, into the gate/up buffer
    a.k = m.H;
    a.n = m.I;
    a.y = m.gu;
    a.ldy = m.I;
    rc = launch_pair<TC_GATEUP>(mgu, a, dim3(2 * 2 * ((m.I + 255) / 256), m.max_items), st, what);
    if (rc) return rc;
    e = launch_pdl(k_act, row_grid((long)m.P * ((m.I / 128 + kQuadBlocks - 1) / kQuadBlocks)), dim3(256), 0, st,
                   static_cast<const __half*>(m.gu), m.I, m.P, m.n_pos, m.pair_expert, m.experts, m.act_limit, m.a_dn);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "%s: activation launch failed: %s", what, cudaGetErrorString(e));
    a.k = m.I;
    a.n = m.H;
    a.y = nullptr;
    return launch_pair<TC_DOWN>(mdn, a, dim3(2 * ((m.H + 255) / 256), m.max_items), st, what);
}

}  // namespace exl3

using namespace exl3;

extern "C" {

size_t exl3_gemm_tc_workspace_size(int M, int k) {
    if (M <= 0 || k <= 0) return 0;
    return align_up((size_t)M * k * 2, 256);
}

int exl3_gemm_tc(const void* x, int x_dtype, int ldx, int M, const void* packed, const void* suh, const void* svh,
                 int k, int n, int K, int cb, void* y, int y_dtype, int ldy, void* workspace, size_t ws_bytes,
                 void* stream) {
    EXL3_REQUIRE(cb == 2, EXL3_ERR_UNSUPPORTED, "exl3_gemm_tc: only the mul1 codebook (cb=2) is supported");
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_UNSUPPORTED, "exl3_gemm_tc: K=%d not in 1..8", K);
    EXL3_REQUIRE(M >= 0 && k > 0 && n > 0 && k % 128 == 0 && n % 128 == 0, EXL3_ERR_ARG,
                 "exl3_gemm_tc: k=%d, n=%d must be multiples of 128", k, n);
    EXL3_REQUIRE(x && packed && svh && y, EXL3_ERR_ARG, "exl3_gemm_tc: null pointer");
    EXL3_REQUIRE(aligned16(packed) && aligned16(y), EXL3_ERR_ARG, "exl3_gemm_tc: packed and y must be 16-byte aligned");
    EXL3_REQUIRE((!suh || (reinterpret_cast<uintptr_t>(suh) & 7) == 0) && (reinterpret_cast<uintptr_t>(svh) & 7) == 0,
                 EXL3_ERR_ARG, "exl3_gemm_tc: suh and svh must be 8-byte aligned");
    EXL3_REQUIRE(x_dtype == EXL3_F16 || x_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "exl3_gemm_tc: x dtype %d",
                 x_dtype);
    EXL3_REQUIRE(y_dtype == EXL3_F16 || y_dtype == EXL3_BF16 || y_dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED,
                 "exl3_gemm_tc: y dtype %d", y_dtype);
    EXL3_REQUIRE(ldx >= k && ldy >= n && ldx % 4 == 0 && ldy % 4 == 0, EXL3_ERR_ARG,
                 "exl3_gemm_tc: row strides ldx=%d ldy=%d", ldx, ldy);
    EXL3_REQUIRE((reinterpret_cast<uintptr_t>(x) & 7) == 0, EXL3_ERR_ARG, "exl3_gemm_tc: x must be 8-byte aligned");
    if (M == 0) return EXL3_OK;
    const size_t need = exl3_gemm_tc_workspace_size(M, k);
    EXL3_REQUIRE(workspace && ws_bytes >= need && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 EXL3_ERR_WORKSPACE, "exl3_gemm_tc: workspace %zu < %zu bytes (or not 256-byte aligned)", ws_bytes,
                 need);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    __half* xh = static_cast<__half*>(workspace);
    {
        const dim3 rg = row_grid((long)M * ((k / 128 + kQuadBlocks - 1) / kQuadBlocks));
        const __half* s = static_cast<const __half*>(suh);
        cudaError_t e;
        if (x_dtype == EXL3_BF16)
            e = launch_pdl(k_rotate_rows<__nv_bfloat16>, rg, dim3(256), 0, st, static_cast<const __nv_bfloat16*>(x),
                           ldx, M, k, s, xh);
        else
            e = launch_pdl(k_rotate_rows<__half>, rg, dim3(256), 0, st, static_cast<const __half*>(x), ldx, M, k, s,
                           xh);
        EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_gemm_tc: rotate launch failed: %s", cudaGetErrorString(e));
    }
    TsMaps maps;
    int rc = make_maps(maps.m[0], xh, M, k, "exl3_gemm_tc");
    if (rc) return rc;
    maps.m[1][0] = maps.m[0][0];
    maps.m[1][1] = maps.m[0][1];
    TsArgs a = {};
    a.packed = static_cast<const uint8_t*>(packed);
    a.svh = static_cast<const __half*>(svh);
    a.K = K;
    a.y = y;
    a.ldy = ldy;
    a.y_dtype = y_dtype;
    a.M = M;
    a.k = k;
    a.n = n;
    a.status = device_status_ptr();
    return launch_pair<TC_LINEAR>(maps, a, dim3(2 * ((n + 255) / 256), (M + TS_TILE_ROWS - 1) / TS_TILE_ROWS), st,
                                  "exl3_gemm_tc");
}

}  // extern "C"
