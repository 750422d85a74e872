// EXL3 linears for prefill-sized batches on the 5th-generation tensor cores (tcgen05, TMEM accumulators): the dense
// linear (any M) and the grouped MoE expert projections (rows grouped per expert by the alignment step).
//
// Weights are decoded from the packed trellis (exl3_pack / exl3_pack_gateup layouts) to the reference's fp16 values
// bit for bit, written into shared memory in the canonical K-major swizzled layout and multiplied with
// tcgen05.mma kind::f16, fp32 accumulation in tensor memory. One CTA computes a 256-row x 256-column tile over the
// whole k range, in k-chunks of TC_BK (32: 64-byte rows with the 64-byte swizzle, so that the rings are deep):
//   warp 0        TMA: the chunk's rotated activation tile(s) [256 rows][TC_BK] fp16 (one per matrix), swizzled;
//   warp 1        allocates the 512 TMEM columns, then one elected lane issues the chunk's MMAs (M 128, K 16) and
//                 commits each stage's release and, after the last chunk, the accumulators;
//   warp 2        bulk-copies the chunk's trellis tiles into a ring;
//   warps 3..18   decode the trellis tiles into the B stage [256 columns][TC_BK]; after the main loop they run the
//                 epilogue: TMEM -> registers -> shared memory (XOR-swizzled rows) -> output Hadamard per 128-column
//                 block with warp shuffles -> the epilogue of the projection.
// Epilogues: linear (y = H(acc) * svh), MoE gate|up (the tile's 256 columns are the fused gate and up blocks of one
// column block; two activation matrices, four 128 x 128 accumulators; SiLU * clamp, then the down input's
// rotation, stored as the down projection's activation rows), MoE down (routing weight x H(acc) * svh, fp32 rows).
// All waits are bounded (EXL3_ERR_TIMEOUT in the device status word). No multicast, no clusters.
//
// Reference semantics: exl3_linear / ReconstructKernel + GEMM for M > 128 (glm/xpu/csrc/exl3_ops.sycl:539-555,
// 651-757; glm/docs/ext-op-inventory.md:597-612), the MoE prefill GateUpDpasKernel / DownDpasKernel
// (glm/xpu/csrc/exl3_moe.n128.sycl:422-690,868-916) and the expert math (glm/docs/ext-op-inventory.md:923-942).
#include "gemv.cuh"
#include "tc.cuh"

namespace exl3 {

#ifndef EXL3_TC_BK
#define EXL3_TC_BK 64
#endif
// k-chunk of 64 (128-byte rows, 128-byte swizzle) or 32 (64-byte rows, 64-byte swizzle)
constexpr int TC_BM = 256, TC_BN = 256, TC_BK = EXL3_TC_BK;
constexpr int TC_ROWB = TC_BK * 2;                            // bytes of one tile row
constexpr int TC_ATOM = 8 * TC_ROWB;                          // swizzle atom: 8 rows
constexpr int TC_DEC_WARPS = 16;
constexpr int TC_WARPS = 3 + TC_DEC_WARPS;
constexpr int TC_THREADS = TC_WARPS * 32;
constexpr int TC_TILE_BYTES = TC_BM * TC_BK * 2;              // one activation tile (and the B stage)
constexpr int TC_AB_REGION = 192 * 1024;                      // activation ring + B ring
constexpr int TC_T_RING = 32 * 1024;                          // trellis ring bytes
constexpr int TC_MAX_TSTAGES = 8;
constexpr int TC_TR = TC_BK / 16;                             // tile-rows per chunk
constexpr int TC_TPW = 2 * TC_TR * 8 / TC_DEC_WARPS;          // trellis tiles per decoder warp per chunk
constexpr int TC_MAX_ASTAGES = 8, TC_MAX_BSTAGES = 8;

__host__ __device__ constexpr int tc_nmat(int epi) { return epi == TC_GATEUP ? 2 : 1; }
// ring depths: gate|up (two activation tiles per stage) 2 + 2 stages, linear / down 3 + 3; the 192 KB of both
// rings (free once the accumulators are complete) also hold the epilogue's 128 KB staging
__host__ __device__ constexpr int tc_b_stages(int epi) { return epi == TC_GATEUP ? 2 : 3; }
__host__ __device__ constexpr int tc_a_stages(int epi) {
    return (TC_AB_REGION - tc_b_stages(epi) * TC_TILE_BYTES) / (tc_nmat(epi) * TC_TILE_BYTES);
}

struct TcSmem {
    static constexpr int a0 = 0;                               // activation ring then B ring (1024-aligned)
    static constexpr int t0 = TC_AB_REGION;
    static constexpr int bars = t0 + TC_T_RING;
    // a_full[], a_empty[], b_full[], b_empty[], t_full[8], t_empty[8], acc_full
    static constexpr int n_bars = 2 * TC_MAX_ASTAGES + 2 * TC_MAX_BSTAGES + 2 * TC_MAX_TSTAGES + 1;
    static constexpr int tmem_slot = bars + n_bars * 8;
    static constexpr int total = tmem_slot + 16 + 1024;        // + slack for 1024-byte alignment of the base
};

// ---- tcgen05 / TMA wrappers ----
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
        ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
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

// Shared-memory matrix descriptor: canonical K-major layout with the 128-byte (TC_BK 64) or 64-byte (TC_BK 32)
// swizzle (8-row atoms, TC_ATOM bytes apart), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw_desc(uint32_t saddr) {
    constexpr uint64_t layout = TC_BK == 64 ? 2 : 4;          // SWIZZLE_128B : SWIZZLE_64B
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(TC_ATOM >> 4) << 32) |
           ((uint64_t)1 << 46) | (layout << 61);
}
// Instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_f16(int M, int N) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Byte offset of element (row, k) of a [rows][TC_BK] fp16 tile in the swizzled K-major layout: 16-byte chunk c of
// a row lands at c ^ (row & 7) (128-byte swizzle) or c ^ ((row >> 1) & 3) (64-byte swizzle).
__device__ __forceinline__ uint32_t sw_off(int row, int k) {
    const int x = TC_BK == 64 ? (row & 7) : ((row >> 1) & 3);
    return (uint32_t)((row >> 3) * TC_ATOM + (row & 7) * TC_ROWB + ((((k >> 3) ^ x)) << 4) + (k & 7) * 2);
}

struct TcArgs {
    // linear: one packed matrix [n/128][k/16][8 tiles][8K words], its svh, y rows
    const uint8_t* packed;
    const __half* svh;
    int K;
    void* y;
    int ldy, y_dtype;
    int M, k, n;                  // linear: M rows; grouped: k, n of the launch's projection
    // grouped: alignment tables (items of <= 256 rows of one expert) and the expert table
    const int* n_items;
    const int* item_expert;
    const int* item_start;
    const int* item_cnt;
    const float* pair_w;          // down: routing weight of a pair position
    const ExpertDesc* experts;
    float act_limit;
    __half* a_dn;                 // gate|up: the down projection's activation rows [positions][I]
    float* ybuf;                  // down: weighted rows [positions][H]
    int* status;
};

// ------------------------------------------------------------------------------------------------ decode

// Per-thread constant addressing of the decode: for each of the warp's TC_TPW tiles of a chunk, the tile's byte offset in
// a trellis stage and the four swizzled byte offsets in a B stage that receive the lane's fragment registers
// {n, k..k+1}, {n + 8, k..}, {n, k + 8..}, {n + 8, k + 8..} (n = tile column + g, k = tile row + 2q).
// Linear / down: a stage holds two column blocks [cb][TC_TR tile-rows][8 tiles][32K bytes] of one matrix; warp dw
// takes tiles TC_TPW dw ... Gate|up: a stage holds TC_TR tile-rows of the fused block, each [8 gate tiles (Kg) |
// 8 up tiles (Ku)]; warps 0-7 take the gate tiles, 8-15 the up tiles, and B rows 0-127 / 128-255 are gate / up.
struct TcDecodeMap {
    uint32_t tile[TC_TPW];
    uint32_t st[TC_TPW][4];
};

__device__ __forceinline__ TcDecodeMap tc_decode_map(int epi, int dw, int lane, int Kg, int Ku) {
    TcDecodeMap mp;
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int j = 0; j < TC_TPW; ++j) {
        int n0, k0;
        if (epi == TC_GATEUP) {
            const int mat = dw >> 3, idx = (dw & 7) * TC_TPW + j;    // 0 .. 8 TC_TR - 1 within the matrix
            const int tr = idx >> 3, t = idx & 7;
            const int row_stride = 8 * 32 * Kg + 8 * 32 * Ku;
            mp.tile[j] = (uint32_t)(tr * row_stride + (mat ? 8 * 32 * Kg : 0) + t * 32 * (mat ? Ku : Kg));
            n0 = mat * 128 + t * 16 + g;
            k0 = tr * 16 + 2 * q;
        } else {
            const int ti = dw * TC_TPW + j;
            const int cb = ti / (8 * TC_TR), tr = (ti >> 3) % TC_TR, t = ti & 7;
            mp.tile[j] = (uint32_t)(((cb * TC_TR + tr) * 8 + t) * 32 * Ku);
            n0 = cb * 128 + t * 16 + g;
            k0 = tr * 16 + 2 * q;
        }
        mp.st[j][0] = sw_off(n0, k0);
        mp.st[j][1] = sw_off(n0 + 8, k0);
        mp.st[j][2] = sw_off(n0, k0 + 8);
        mp.st[j][3] = sw_off(n0 + 8, k0 + 8);
    }
    return mp;
}

template <int K>
__device__ __forceinline__ void tc_decode_chunk(const uint8_t* tst, uint8_t* bst, const TcDecodeMap& mp,
                                                const LaneWords& lw) {
#pragma unroll
    for (int j = 0; j < TC_TPW; ++j) {
        uint32_t a[4];
        decode_frag<K>(reinterpret_cast<const uint32_t*>(tst + mp.tile[j]), lw, a);
#pragma unroll
        for (int r = 0; r < 4; ++r) *reinterpret_cast<uint32_t*>(bst + mp.st[j][r]) = a[r];
    }
}

template <int K>
__device__ void tc_decoder_loop(const TcDecodeMap& mp, uint8_t* smem, uint8_t* bring, int bst, int t_stages,
                                int t_stage_bytes, uint64_t* t_full, uint64_t* t_empty, uint64_t* b_full,
                                uint64_t* b_empty, int nk, int lane, bool& to) {
    const LaneWords lw = lane_words<K>(lane);
    for (int kc = 0; kc < nk; ++kc) {
        const int ts = kc % t_stages, s = kc % bst;
        if (!to && !mbar_wait(&t_full[ts], (kc / t_stages) & 1)) to = true;
        if (kc >= bst && !to && !mbar_wait(&b_empty[s], ((kc / bst) - 1) & 1)) to = true;
        if (!to)
            tc_decode_chunk<K>(smem + TcSmem::t0 + (size_t)ts * t_stage_bytes, bring + s * TC_TILE_BYTES, mp, lw);
        fence_proxy_async();                                  // generic-proxy writes -> the tensor core's reads
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&t_empty[ts]);
            mbar_arrive(&b_full[s]);
        }
    }
}

__device__ void tc_decoder_dispatch(int K, const TcDecodeMap& mp, uint8_t* smem, uint8_t* bring, int bst,
                                    int t_stages, int t_stage_bytes, uint64_t* t_full, uint64_t* t_empty,
                                    uint64_t* b_full, uint64_t* b_empty, int nk, int lane, bool& to) {
#define EXL3_TC_DEC(KK)                                                                                         \
    tc_decoder_loop<KK>(mp, smem, bring, bst, t_stages, t_stage_bytes, t_full, t_empty, b_full, b_empty, nk, lane, \
                        to)
    switch (K) {
        case 1: EXL3_TC_DEC(1); break;
        case 2: EXL3_TC_DEC(2); break;
        case 3: EXL3_TC_DEC(3); break;
        case 4: EXL3_TC_DEC(4); break;
        case 5: EXL3_TC_DEC(5); break;
        case 6: EXL3_TC_DEC(6); break;
        case 7: EXL3_TC_DEC(7); break;
        default: EXL3_TC_DEC(8); break;
    }
#undef EXL3_TC_DEC
}

// ------------------------------------------------------------------------------------------------ kernel

template <int EPI>
__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(const __grid_constant__ CUtensorMap amap0,
                                                           const __grid_constant__ CUtensorMap amap1,
                                                           const TcArgs p) {
    constexpr int NMAT = tc_nmat(EPI);
    constexpr int AST = tc_a_stages(EPI);
    constexpr int BST = tc_b_stages(EPI);
    constexpr int A_STAGE = NMAT * TC_TILE_BYTES;
    static_assert(AST <= TC_MAX_ASTAGES && BST <= TC_MAX_BSTAGES && AST * A_STAGE + BST * TC_TILE_BYTES <= TC_AB_REGION,
                  "rings");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    pdl_trigger();

    // ---- the tile: rows [m0, m0 + rows) of the activation matrices, output columns from n0 ----
    int m0, rows, n0, Ku = p.K, Kg = p.K, expert = 0;
    const uint8_t* wmat;                                      // packed weights of the tile's first column block
    size_t cb_bytes;                                          // bytes of one column block (all k)
    const __half* svh0;
    const __half* svh1 = nullptr;
    if constexpr (EPI == TC_LINEAR) {
        m0 = blockIdx.y * TC_BM;
        rows = min(TC_BM, p.M - m0);
        n0 = blockIdx.x * TC_BN;
        cb_bytes = (size_t)(p.k / 16) * 8 * 32 * Ku;
        wmat = p.packed + (size_t)(n0 / 128) * cb_bytes;
        svh0 = p.svh;
    } else {
        pdl_wait();                                           // the alignment tables come from an earlier kernel
        const int item = blockIdx.y;
        if (item >= __ldcg(p.n_items)) return;                // before any barrier or TMEM allocation
        expert = __ldcg(p.item_expert + item);
        m0 = __ldcg(p.item_start + item);
        rows = __ldcg(p.item_cnt + item);
        const ExpertDesc& ed = p.experts[expert];
        if constexpr (EPI == TC_GATEUP) {
            Kg = ed.K[0];
            Ku = ed.K[1];
            n0 = blockIdx.x * 128;                            // output column block of gate and up
            cb_bytes = (size_t)(p.k / 16) * (8 * 32 * Kg + 8 * 32 * Ku);
            wmat = reinterpret_cast<const uint8_t*>(ed.tr[0]) + (size_t)blockIdx.x * cb_bytes;
            svh0 = ed.svh[0];
            svh1 = ed.svh[1];
        } else {
            Ku = ed.K[2];
            Kg = Ku;
            n0 = blockIdx.x * TC_BN;
            cb_bytes = (size_t)(p.k / 16) * 8 * 32 * Ku;
            wmat = reinterpret_cast<const uint8_t*>(ed.tr[2]) + (size_t)(n0 / 128) * cb_bytes;
            svh0 = ed.svh[2];
        }
    }
    const int nk = p.k / TC_BK;
    // trellis stage: linear / down two column blocks x 4 tile-rows x 8 tiles; gate|up 4 fused tile-rows
    const int t_stage_bytes = EPI == TC_GATEUP ? TC_TR * (8 * 32 * Kg + 8 * 32 * Ku) : 2 * TC_TR * 8 * 32 * Ku;
    int t_stages = TC_T_RING / t_stage_bytes;
    if (t_stages > TC_MAX_TSTAGES) t_stages = TC_MAX_TSTAGES;

    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::bars);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + TC_MAX_ASTAGES;
    uint64_t* b_full = a_empty + TC_MAX_ASTAGES;
    uint64_t* b_empty = b_full + TC_MAX_BSTAGES;
    uint64_t* t_full = b_empty + TC_MAX_BSTAGES;
    uint8_t* bring = smem + TcSmem::a0 + AST * A_STAGE;           // B ring after the activation ring
    uint64_t* t_empty = t_full + TC_MAX_TSTAGES;
    uint64_t* acc_full = t_empty + TC_MAX_TSTAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::tmem_slot);

    if (threadIdx.x == 0) {
        for (int s = 0; s < AST; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < BST; ++s) {
            mbar_init(&b_full[s], TC_DEC_WARPS);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < t_stages; ++s) {
            mbar_init(&t_full[s], 1);
            mbar_init(&t_empty[s], TC_DEC_WARPS);
        }
        mbar_init(acc_full, 1);
        fence_barrier_init();
    }
    if (warp == 1) {                                          // TMEM: all 512 columns (four 128 x 128 fp32 blocks)
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(tmem_slot))
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    bool to = false;

    if (warp == 0) {
        // ---------------- activation tiles (TMA) ----------------
        pdl_wait();                                           // the rotated activations come from an earlier kernel
        if (lane == 0) {
            int last_s[TC_MAX_ASTAGES];
            for (int s = 0; s < TC_MAX_ASTAGES; ++s) last_s[s] = -1;
            for (int kc = 0; kc < nk && !to; ++kc) {
                const int s = kc % AST;
                if (kc >= AST && !mbar_wait(&a_empty[s], ((kc / AST) - 1) & 1)) { to = true; break; }
                mbar_expect_tx(&a_full[s], A_STAGE);
                uint8_t* dst = smem + TcSmem::a0 + s * A_STAGE;
                tma_load_2d(dst, &amap0, kc * TC_BK, m0, &a_full[s]);
                if constexpr (NMAT == 2) tma_load_2d(dst + TC_TILE_BYTES, &amap1, kc * TC_BK, m0, &a_full[s]);
                last_s[s] = kc;
            }
            for (int s = 0; s < AST; ++s)                     // copies landed before the CTA may exit
                if (last_s[s] >= 0 && !mbar_wait(&a_full[s], (last_s[s] / AST) & 1)) to = true;
        }
    } else if (warp == 1) {
        // ---------------- MMA issue (one lane) ----------------
        if (lane == 0) {
            for (int kc = 0; kc < nk; ++kc) {
                const int sa = kc % AST, sb = kc % BST;
                if (!to && !mbar_wait(&a_full[sa], (kc / AST) & 1)) to = true;
                if (!to && !mbar_wait(&b_full[sb], (kc / BST) & 1)) to = true;
                tc_fence_after();
                if (!to) {
                    const uint32_t a_base = smem_u32(smem + TcSmem::a0 + sa * A_STAGE);
                    const uint32_t b_base = smem_u32(bring + sb * TC_TILE_BYTES);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk) {
                        const uint32_t acc = (kc | kk) != 0;
                        if constexpr (EPI == TC_GATEUP) {
                            // accumulator (mat, j) at TMEM column (2 mat + j) * 128: activation tile of the matrix,
                            // row half j; B rows of the matrix (gate 0-127, up 128-255)
#pragma unroll
                            for (int mat = 0; mat < 2; ++mat)
#pragma unroll
                                for (int j = 0; j < 2; ++j)
                                    tc_mma_f16(tmem + (2 * mat + j) * 128,
                                               sw_desc(a_base + mat * TC_TILE_BYTES + j * (TC_TILE_BYTES / 2) +
                                                       kk * 32),
                                               sw_desc(b_base + mat * (TC_TILE_BYTES / 2) + kk * 32),
                                               tc_idesc_f16(128, 128), acc);
                        } else {
#pragma unroll
                            for (int j = 0; j < 2; ++j)
                                tc_mma_f16(tmem + j * TC_BN, sw_desc(a_base + j * (TC_TILE_BYTES / 2) + kk * 32),
                                           sw_desc(b_base + kk * 32), tc_idesc_f16(128, TC_BN), acc);
                        }
                    }
                }
                tc_commit(&a_empty[sa]);                      // the stages are free once these MMAs completed
                tc_commit(&b_empty[sb]);
            }
            tc_commit(acc_full);
        }
    } else if (warp == 2) {
        // ---------------- trellis tiles (bulk copies) ----------------
        if (lane == 0) {
            int last[TC_MAX_TSTAGES];
            for (int s = 0; s < TC_MAX_TSTAGES; ++s) last[s] = -1;
            // column blocks present (the last tile of a linear or down projection may have 1); gate|up: one fused block
            const int nbv = EPI == TC_GATEUP ? 1 : min(2, (p.n - n0) / 128);
            const uint32_t blk = (uint32_t)(t_stage_bytes / (EPI == TC_GATEUP ? 1 : 2));
            for (int kc = 0; kc < nk && !to; ++kc) {
                const int ts = kc % t_stages;
                if (kc >= t_stages && !mbar_wait(&t_empty[ts], ((kc / t_stages) - 1) & 1)) { to = true; break; }
                mbar_expect_tx(&t_full[ts], blk * (uint32_t)nbv);
                uint8_t* dst = smem + TcSmem::t0 + (size_t)ts * t_stage_bytes;
                for (int b = 0; b < nbv; ++b)
                    bulk_g2s(dst + b * blk, wmat + (size_t)b * cb_bytes + (size_t)kc * blk, blk, &t_full[ts]);
                last[ts] = kc;
            }
            for (int s = 0; s < t_stages; ++s)
                if (last[s] >= 0 && !mbar_wait(&t_full[s], (last[s] / t_stages) & 1)) to = true;
        }
    } else {
        // ---------------- decoders, then the epilogue ----------------
        const int dw = warp - 3;
        const TcDecodeMap mp = tc_decode_map(EPI, dw, lane, Kg, Ku);
        const int Kw = (EPI == TC_GATEUP && dw < 8) ? Kg : Ku;
        tc_decoder_dispatch(Kw, mp, smem, bring, BST, t_stages, t_stage_bytes, t_full, t_empty, b_full, b_empty, nk,
                            lane, to);

        pdl_wait();                                           // outputs may be in use by an earlier kernel until here
        if (!to && !mbar_wait(acc_full, 0)) to = true;
        tc_fence_after();
        // the four 128 x 128 accumulator blocks: block bi at TMEM column 128 bi. Linear / down: bi = 2 j + b
        // (row half j, column block b); gate|up: bi = 2 mat + j. The four warps of a TMEM lane quadrant each load
        // one block; staging [2][128 rows][128 cols] fp32 in the activation + B rings (free after the main loop), columns
        // XOR-swizzled by the row. Pass 0: blocks of row half 0, pass 1: row half 1.
        const int quad = warp & 3, bi = dw >> 2;              // warps 3..18: quad covers 0..3 four times
        const int bj = EPI == TC_GATEUP ? (bi & 1) : (bi >> 1);   // row half of block bi
        const int bslot = EPI == TC_GATEUP ? (bi >> 1) : (bi & 1); // staging slot: column block, or gate / up
        float* stage = reinterpret_cast<float*>(smem + TcSmem::a0);
        for (int pass = 0; pass < 2; ++pass) {
            if (bj == pass) {
                float* st = stage + (size_t)bslot * 128 * 128;
                const int row = quad * 32 + lane;             // accumulator row = TMEM lane
#pragma unroll
                for (int c0 = 0; c0 < 128; c0 += 32) {
                    uint32_t r[32];
                    tc_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(bi * 128 + c0), r);
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        st[row * 128 + ((c0 + c) ^ (row & 31))] = __uint_as_float(r[c]);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(TC_DEC_WARPS * 32) : "memory");
            if constexpr (EPI == TC_GATEUP) {
                // row r of this half: gate and up blocks -> act -> the down input's rotation, into a_dn
                const __half* suh_d = p.experts[expert].suh[2];
                for (int row = dw; row < 128; row += TC_DEC_WARPS) {
                    const int rr = pass * 128 + row;
                    if (rr >= rows) continue;
                    float gv[4], uv[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        gv[e] = stage[row * 128 + ((4 * lane + e) ^ (row & 31))];
                        uv[e] = stage[128 * 128 + row * 128 + ((4 * lane + e) ^ (row & 31))];
                    }
                    fwht128_warp(gv, lane);
                    fwht128_warp(uv, lane);
                    const int col = n0 + 4 * lane;            // column of I
                    float h[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float gg = __half2float(__float2half_rn(
                            __half2float(__float2half_rn(gv[e] * kRsqrt128)) * __half2float(svh0[col + e])));
                        float uu = __half2float(__float2half_rn(
                            __half2float(__float2half_rn(uv[e] * kRsqrt128)) * __half2float(svh1[col + e])));
                        float sg = silu_f(gg);
                        if (p.act_limit != 0.f) {
                            sg = fminf(sg, p.act_limit);
                            uu = fminf(fmaxf(uu, -p.act_limit), p.act_limit);
                        }
                        const float act = __half2float(__float2half_rn(sg * uu));
                        h[e] = __half2float(__float2half_rn(act * __half2float(suh_d[col + e])));
                    }
                    fwht128_warp(h, lane);
                    __half2 h01 = __floats2half2_rn(h[0] * kRsqrt128, h[1] * kRsqrt128);
                    __half2 h23 = __floats2half2_rn(h[2] * kRsqrt128, h[3] * kRsqrt128);
                    uint2 u;
                    u.x = *reinterpret_cast<uint32_t*>(&h01);
                    u.y = *reinterpret_cast<uint32_t*>(&h23);
                    *reinterpret_cast<uint2*>(p.a_dn + (size_t)(m0 + rr) * p.n + col) = u;
                }
            } else {
                // 2 column blocks x 128 rows over 16 warps, one row at a time
                for (int rb = dw; rb < 2 * 128; rb += TC_DEC_WARPS) {
                    const int b = rb >> 7, row = rb & 127;
                    const int rr = pass * 128 + row;
                    const int col = n0 + b * 128 + 4 * lane;
                    if (rr >= rows || col >= p.n) continue;
                    const float* src = stage + (size_t)b * 128 * 128 + row * 128;
                    float v[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[e] = src[(4 * lane + e) ^ (row & 31)];
                    fwht128_warp(v, lane);
                    if constexpr (EPI == TC_DOWN) {
                        const float wgt = __ldcg(p.pair_w + m0 + rr);
                        float o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) o[e] = wgt * (v[e] * kRsqrt128 * __half2float(svh0[col + e]));
                        *reinterpret_cast<float4*>(p.ybuf + (size_t)(m0 + rr) * p.n + col) =
                            make_float4(o[0], o[1], o[2], o[3]);
                    } else {
                        const int m = m0 + rr;
                        float o[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float sv = __half2float(svh0[col + e]);
                            if (p.y_dtype == EXL3_F16)
                                o[e] = __half2float(
                                    __float2half_rn(__half2float(__float2half_rn(v[e] * kRsqrt128)) * sv));
                            else
                                o[e] = v[e] * kRsqrt128 * sv;
                        }
                        if (p.y_dtype == EXL3_F32) {
                            *reinterpret_cast<float4*>(static_cast<float*>(p.y) + (size_t)m * p.ldy + col) =
                                make_float4(o[0], o[1], o[2], o[3]);
                        } else if (p.y_dtype == EXL3_F16) {
                            __half2 h01 = __floats2half2_rn(o[0], o[1]), h23 = __floats2half2_rn(o[2], o[3]);
                            uint2 u;
                            u.x = *reinterpret_cast<uint32_t*>(&h01);
                            u.y = *reinterpret_cast<uint32_t*>(&h23);
                            *reinterpret_cast<uint2*>(static_cast<__half*>(p.y) + (size_t)m * p.ldy + col) = u;
                        } else {
                            __nv_bfloat16* yp = static_cast<__nv_bfloat16*>(p.y) + (size_t)m * p.ldy + col;
#pragma unroll
                            for (int e = 0; e < 4; ++e) yp[e] = __float2bfloat16_rn(o[e]);
                        }
                    }
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(TC_DEC_WARPS * 32) : "memory");
        }
    }
    if (to) report(p.status, EXL3_ERR_TIMEOUT);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
    }
}

// ------------------------------------------------------------------------------------------------ activation rows

// Rotated input rows in plain row-major order: xh[m][k] = fp16(H(fp16(x * suh)) / sqrt(128)) per 128-block.
static __global__ void __launch_bounds__(256) k_rotate_rows(const void* x, int ldx, int x_bf16, int M, int k,
                                                            const __half* suh, __half* xh) {
    pdl_wait();
    pdl_trigger();
    const int KB = k / 128, lane = threadIdx.x & 31;
    for (long j = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < (long)M * KB;
         j += ((long)gridDim.x * blockDim.x) >> 5) {
        const int row = (int)(j / KB), kb = (int)(j % KB);
        float v[4];
        const __half* su = suh ? suh + kb * 128 : nullptr;
        if (x_bf16)
            rotated_block<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x) + (size_t)row * ldx + kb * 128, su,
                                         lane, v);
        else
            rotated_block<__half>(static_cast<const __half*>(x) + (size_t)row * ldx + kb * 128, su, lane, v);
        __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&h01);
        u.y = *reinterpret_cast<uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(xh + (size_t)row * k + kb * 128 + 4 * lane) = u;
    }
}

// Rotated gate and up input rows of every pair position, row-major: a_gu[mat][pos][H] = rot(x[token] * suh of the
// position's expert's matrix mat). Positions beyond the count in use are skipped.
static __global__ void __launch_bounds__(256) k_rotate_pairs(const void* x, int ldx, int x_bf16, int H, int P,
                                                             const int* n_pos, const int* pair_tok,
                                                             const int* pair_expert, const ExpertDesc* experts,
                                                             __half* a_gu) {
    pdl_wait();
    pdl_trigger();
    const int KB = H / 128, lane = threadIdx.x & 31;
    const int np = min(P, __ldcg(n_pos));
    for (long j = ((long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; j < (long)np * 2 * KB;
         j += ((long)gridDim.x * blockDim.x) >> 5) {
        const int pos = (int)(j / (2 * KB)), mat = (int)((j / KB) % 2), kb = (int)(j % KB);
        const int tok = __ldcg(pair_tok + pos), e = __ldcg(pair_expert + pos);
        const __half* suh = experts[e].suh[mat];
        const __half* su = suh ? suh + kb * 128 : nullptr;
        float v[4];
        if (x_bf16)
            rotated_block<__nv_bfloat16>(static_cast<const __nv_bfloat16*>(x) + (size_t)tok * ldx + kb * 128, su,
                                         lane, v);
        else
            rotated_block<__half>(static_cast<const __half*>(x) + (size_t)tok * ldx + kb * 128, su, lane, v);
        __half2 h01 = __floats2half2_rn(v[0], v[1]), h23 = __floats2half2_rn(v[2], v[3]);
        uint2 u;
        u.x = *reinterpret_cast<uint32_t*>(&h01);
        u.y = *reinterpret_cast<uint32_t*>(&h23);
        *reinterpret_cast<uint2*>(a_gu + ((size_t)mat * P + pos) * H + kb * 128 + 4 * lane) = u;
    }
}

// ------------------------------------------------------------------------------------------------ host launch

using PFN_encode_tiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// Tensor map of a row-major [rows][cols] fp16 matrix: boxes of TC_BK columns x 256 rows, swizzled as the MMA
// descriptors expect, zero fill.
static int make_row_map(CUtensorMap* map, const __half* base, long rows, int cols, const char* what) {
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
    const cuuint32_t box[2] = {TC_BK, TC_BM};
    const cuuint32_t estr[2] = {1, 1};
    CUresult cr = encode(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE,
                         TC_BK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    EXL3_REQUIRE(cr == CUDA_SUCCESS, EXL3_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed (%d)", what, (int)cr);
    return EXL3_OK;
}

template <int EPI>
static int launch_tc(const CUtensorMap& m0, const CUtensorMap& m1, const TcArgs& a, dim3 grid, cudaStream_t st,
                     const char* what) {
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        EXL3_REQUIRE(cudaFuncSetAttribute(k_gemm_tc<EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          TcSmem::total) == cudaSuccess,
                     EXL3_ERR_CUDA, "%s: cudaFuncSetAttribute: %s", what, cudaGetErrorString(cudaGetLastError()));
        configured[dev] = 1;
    }
    cudaError_t e = launch_pdl(k_gemm_tc<EPI>, grid, dim3(TC_THREADS), TcSmem::total, st, m0, m1, a);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return EXL3_OK;
}

int tc_moe_prefill(const TcMoeArgs& m, cudaStream_t st) {
    const char* what = "exl3_moe_prefill";
    {
        const long jobs = (long)m.P * 2 * (m.H / 128);
        long blocks = (jobs + 7) / 8;
        if (blocks > 8L * num_sms()) blocks = 8L * num_sms();
        cudaError_t e = launch_pdl(k_rotate_pairs, dim3((unsigned)blocks), dim3(256), 0, st, m.x, m.ldx, m.x_bf16,
                                   m.H, m.P, m.n_pos, m.pair_tok, m.pair_expert, m.experts, m.a_gu);
        EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "%s: rotate launch failed: %s", what, cudaGetErrorString(e));
    }
    if (m.max_items == 0) return EXL3_OK;
    TcArgs a = {};
    a.n_items = m.n_items;
    a.item_expert = m.item_expert;
    a.item_start = m.item_start;
    a.item_cnt = m.item_cnt;
    a.pair_w = m.pair_w;
    a.experts = m.experts;
    a.act_limit = m.act_limit;
    a.a_dn = m.a_dn;
    a.ybuf = m.ybuf;
    a.status = device_status_ptr();
    CUtensorMap mg, mu, md;
    int rc = make_row_map(&mg, m.a_gu, m.P, m.H, what);
    if (!rc) rc = make_row_map(&mu, m.a_gu + (size_t)m.P * m.H, m.P, m.H, what);
    if (!rc) rc = make_row_map(&md, m.a_dn, m.P, m.I, what);
    if (rc) return rc;
    a.k = m.H;
    a.n = m.I;
    rc = launch_tc<TC_GATEUP>(mg, mu, a, dim3(m.I / 128, m.max_items), st, what);
    if (rc) return rc;
    a.k = m.I;
    a.n = m.H;
    return launch_tc<TC_DOWN>(md, md, a, dim3((m.H + TC_BN - 1) / TC_BN, m.max_items), st, what);
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
        const long jobs = (long)M * (k / 128);
        long blocks = (jobs + 7) / 8;
        if (blocks > 8L * num_sms()) blocks = 8L * num_sms();
        cudaError_t e = launch_pdl(k_rotate_rows, dim3((unsigned)blocks), dim3(256), 0, st, x, ldx,
                                   (int)(x_dtype == EXL3_BF16), M, k, static_cast<const __half*>(suh), xh);
        EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_gemm_tc: rotate launch failed: %s", cudaGetErrorString(e));
    }
    CUtensorMap map;
    int rc = make_row_map(&map, xh, M, k, "exl3_gemm_tc");
    if (rc) return rc;
    TcArgs a = {};
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
    return launch_tc<TC_LINEAR>(map, map, a, dim3((n + TC_BN - 1) / TC_BN, (M + TC_BM - 1) / TC_BM), st,
                                "exl3_gemm_tc");
}

}  // extern "C"
