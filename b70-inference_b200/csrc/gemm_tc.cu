// EXL3 linear for prefill-sized batches on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
// y[M][n] = Had(Had(x * suh) @ W_hat) * svh, W_hat decoded from the packed trellis (exl3_pack layout) to the
// reference's fp16 weights bit for bit, multiplied on tcgen05 kind::f16 with fp32 accumulation in tensor memory.
//
// One CTA computes a TC_BM x TC_BN output tile (TC_BM / 128 accumulators of TC_BN fp32 columns = all 512 TMEM
// columns) over the whole k range, in k-chunks of 64:
//   warp 0        TMA: the chunk's rotated activation tile [TC_BM rows][64] fp16, 128-byte swizzle, into a ring;
//   warp 1        allocates TMEM, then one elected lane issues (TC_BM / 128) x 4 tcgen05.mma (M 128, N TC_BN, K 16)
//                 per chunk and commits each stage's release and, after the last chunk, the accumulators;
//   warp 2        bulk-copies the chunk's trellis tiles (TC_BN / 128 column blocks x 4 tile-rows x 8 tiles);
//   warps 3..18   decode the trellis tiles (same register decode as the GEMV: one lane, eight positions of a tile)
//                 into the B stage [TC_BN columns][64] fp16 in the canonical K-major 128-byte-swizzled layout; after
//                 the main loop the same warps run the epilogue: TMEM -> registers -> shared memory (XOR-swizzled
//                 rows) -> output Hadamard per 128-column block with warp shuffles -> x svh -> y.
// All waits are bounded (EXL3_ERR_TIMEOUT in the device status word). No multicast, no clusters.
//
// Reference semantics: exl3_linear / ReconstructKernel + GEMM for M > 128 (glm/xpu/csrc/exl3_ops.sycl:539-555,
// 651-757; glm/docs/ext-op-inventory.md:597-612) and the DPAS small-batch kernel (glm/xpu/csrc/exl3_esimd.h:582-862).
#include "gemv.cuh"

namespace exl3 {

#ifndef EXL3_TC_BM
#define EXL3_TC_BM 256
#define EXL3_TC_BN 256
#define EXL3_TC_ASTAGES 4
#define EXL3_TC_BSTAGES 2
#endif
constexpr int TC_BM = EXL3_TC_BM, TC_BN = EXL3_TC_BN, TC_BK = 64;
constexpr int TC_ACC = TC_BM / 128;                            // 128-row accumulators (TMEM: TC_ACC x TC_BN columns)
constexpr int TC_NB = TC_BN / 128;                             // 128-column blocks per tile
static_assert(TC_ACC * TC_BN == 512, "the accumulators fill the 512 TMEM columns");
constexpr int TC_DEC_WARPS = 16;
constexpr int TC_WARPS = 3 + TC_DEC_WARPS;
constexpr int TC_THREADS = TC_WARPS * 32;
constexpr int TC_A_BYTES = TC_BM * TC_BK * 2;
constexpr int TC_B_BYTES = TC_BN * TC_BK * 2;
constexpr int TC_A_STAGES = EXL3_TC_ASTAGES, TC_B_STAGES = EXL3_TC_BSTAGES;
constexpr int TC_T_RING = 32 * 1024;                          // trellis ring bytes
constexpr int TC_MAX_TSTAGES = 8;
constexpr int TC_TILES = (TC_BN / 16) * (TC_BK / 16);         // trellis tiles per chunk

struct TcSmem {
    static constexpr int a0 = 0;                               // A[3] (1024-aligned)
    static constexpr int b0 = TC_A_STAGES * TC_A_BYTES;        // B[2]
    static constexpr int t0 = b0 + TC_B_STAGES * TC_B_BYTES;   // trellis ring
    static constexpr int bars = t0 + TC_T_RING;
    // a_full[3], a_empty[3], b_full[2], b_empty[2], t_full[8], t_empty[8], acc_full
    static constexpr int n_bars = 2 * TC_A_STAGES + 2 * TC_B_STAGES + 2 * TC_MAX_TSTAGES + 1;
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

// Shared-memory matrix descriptor: canonical K-major layout with the 128-byte swizzle (8-row atoms of 128 bytes,
// atoms 1024 bytes apart), sm100 descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor, kind::f16: fp16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t tc_idesc_f16(int M, int N) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Byte offset of element (row, k) of a [rows][64] fp16 tile in the 128-byte-swizzled K-major layout.
__device__ __forceinline__ uint32_t sw128_off(int row, int k) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7))) << 4) + (k & 7) * 2);
}

struct TcArgs {
    const uint8_t* packed;     // [n/128][k/16][8 tiles][8K words]
    const __half* svh;
    void* y;
    int ldy, y_dtype;
    int M, k, n, K;
    int t_stages, t_stage_bytes;
    int* status;
};

// Per-thread constant addressing of the decode: for each of the warp's tiles in a chunk, the tile's byte
// offset in a trellis stage and the four swizzled byte offsets in a B stage that receive the lane's fragment
// registers {n, k..k+1}, {n + 8, k..}, {n, k + 8..}, {n + 8, k + 8..} (n = tile column + g, k = tile row + 2q).
constexpr int TC_TPW = TC_TILES / TC_DEC_WARPS;
struct TcDecodeMap {
    uint32_t tile[TC_TPW];
    uint32_t st[TC_TPW][4];
};

template <int K>
__device__ __forceinline__ TcDecodeMap tc_decode_map(int dw, int lane) {
    TcDecodeMap mp;
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int j = 0; j < TC_TPW; ++j) {
        const int ti = dw * TC_TPW + j;
        const int cb = ti >> 5, tr = (ti >> 3) & 3, t = ti & 7;   // column block, tile-row, tile
        mp.tile[j] = (uint32_t)(((cb * 4 + tr) * 8 + t) * 32 * K);
        const int n0 = cb * 128 + t * 16 + g, k0 = tr * 16 + 2 * q;
        mp.st[j][0] = sw128_off(n0, k0);
        mp.st[j][1] = sw128_off(n0 + 8, k0);
        mp.st[j][2] = sw128_off(n0, k0 + 8);
        mp.st[j][3] = sw128_off(n0 + 8, k0 + 8);
    }
    return mp;
}

// Decode one chunk's trellis tiles of this warp into the swizzled B stage.
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
__device__ void tc_decoder_loop(const TcArgs& p, uint8_t* smem, uint64_t* t_full, uint64_t* t_empty,
                                uint64_t* b_full, uint64_t* b_empty, int nk, int dw, int lane, bool& to) {
    const TcDecodeMap mp = tc_decode_map<K>(dw, lane);
    const LaneWords lw = lane_words<K>(lane);
    for (int kc = 0; kc < nk; ++kc) {
        const int ts = kc % p.t_stages, s = kc % TC_B_STAGES;
        if (!to && !mbar_wait(&t_full[ts], (kc / p.t_stages) & 1)) to = true;
        if (kc >= TC_B_STAGES && !to && !mbar_wait(&b_empty[s], ((kc / TC_B_STAGES) - 1) & 1)) to = true;
        if (!to)
            tc_decode_chunk<K>(smem + TcSmem::t0 + (size_t)ts * p.t_stage_bytes, smem + TcSmem::b0 + s * TC_B_BYTES,
                               mp, lw);
        fence_proxy_async();                                  // generic-proxy writes -> the tensor core's reads
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&t_empty[ts]);
            mbar_arrive(&b_full[s]);
        }
    }
}

__global__ void __launch_bounds__(TC_THREADS, 1) k_gemm_tc(const __grid_constant__ CUtensorMap amap,
                                                           const TcArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + TcSmem::bars);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + TC_A_STAGES;
    uint64_t* b_full = a_empty + TC_A_STAGES;
    uint64_t* b_empty = b_full + TC_B_STAGES;
    uint64_t* t_full = b_empty + TC_B_STAGES;
    uint64_t* t_empty = t_full + TC_MAX_TSTAGES;
    uint64_t* acc_full = t_empty + TC_MAX_TSTAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + TcSmem::tmem_slot);
    const int n0 = blockIdx.x * TC_BN, m0 = blockIdx.y * TC_BM;
    const int nk = p.k / TC_BK;
    pdl_trigger();

    if (threadIdx.x == 0) {
        for (int s = 0; s < TC_A_STAGES; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], 1);
        }
        for (int s = 0; s < TC_B_STAGES; ++s) {
            mbar_init(&b_full[s], TC_DEC_WARPS);
            mbar_init(&b_empty[s], 1);
        }
        for (int s = 0; s < p.t_stages; ++s) {
            mbar_init(&t_full[s], 1);
            mbar_init(&t_empty[s], TC_DEC_WARPS);
        }
        mbar_init(acc_full, 1);
        fence_barrier_init();
    }
    if (warp == 1) {                                          // TMEM: 512 columns = four 128 x 128 fp32 accumulators
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
        pdl_wait();                                           // the rotated activations come from the previous kernel
        if (lane == 0) {
            int last_s[TC_A_STAGES];
            for (int s = 0; s < TC_A_STAGES; ++s) last_s[s] = -1;
            for (int kc = 0; kc < nk && !to; ++kc) {
                const int s = kc % TC_A_STAGES;
                if (kc >= TC_A_STAGES && !mbar_wait(&a_empty[s], ((kc / TC_A_STAGES) - 1) & 1)) { to = true; break; }
                mbar_expect_tx(&a_full[s], TC_A_BYTES);
#pragma unroll
                for (int h = 0; h < (TC_BM + 255) / 256; ++h)  // boxes of 256 rows
                    tma_load_2d(smem + TcSmem::a0 + s * TC_A_BYTES + h * (TC_A_BYTES * 256 / TC_BM), &amap,
                                kc * TC_BK, m0 + h * 256, &a_full[s]);
                last_s[s] = kc;
            }
            for (int s = 0; s < TC_A_STAGES; ++s)             // copies landed before the CTA may exit
                if (last_s[s] >= 0 && !mbar_wait(&a_full[s], (last_s[s] / TC_A_STAGES) & 1)) to = true;
        }
    } else if (warp == 1) {
        // ---------------- MMA issue (one lane) ----------------
        if (lane == 0) {
            constexpr uint32_t idesc = tc_idesc_f16(128, TC_BN);
            for (int kc = 0; kc < nk; ++kc) {
                const int sa = kc % TC_A_STAGES, sb = kc % TC_B_STAGES;
                if (!to && !mbar_wait(&a_full[sa], (kc / TC_A_STAGES) & 1)) to = true;
                if (!to && !mbar_wait(&b_full[sb], (kc / TC_B_STAGES) & 1)) to = true;
                tc_fence_after();
                if (!to) {
                    const uint32_t a_base = smem_u32(smem + TcSmem::a0 + sa * TC_A_BYTES);
                    const uint32_t b_base = smem_u32(smem + TcSmem::b0 + sb * TC_B_BYTES);
#pragma unroll
                    for (int kk = 0; kk < TC_BK / 16; ++kk)
#pragma unroll
                        for (int j = 0; j < TC_ACC; ++j)
                            tc_mma_f16(tmem + j * TC_BN, sw128_desc(a_base + j * (TC_A_BYTES / TC_ACC) + kk * 32),
                                       sw128_desc(b_base + kk * 32), idesc, (kc | kk) != 0);
                }
                tc_commit(&a_empty[sa]);                      // the stages are free once these MMAs completed
                tc_commit(&b_empty[sb]);
            }
            tc_commit(acc_full);
        }
    } else if (warp == 2) {
        // ---------------- trellis tiles (bulk copies) ----------------
        if (lane == 0) {
            const size_t block_bytes = (size_t)(p.k / 16) * 8 * 32 * p.K;       // one 128-column block, all k
            int last[TC_MAX_TSTAGES];
            for (int s = 0; s < TC_MAX_TSTAGES; ++s) last[s] = -1;
            for (int kc = 0; kc < nk && !to; ++kc) {
                const int ts = kc % p.t_stages;
                if (kc >= p.t_stages && !mbar_wait(&t_empty[ts], ((kc / p.t_stages) - 1) & 1)) { to = true; break; }
                const uint32_t blk = (uint32_t)(p.t_stage_bytes / TC_NB);           // a block's 4 tile-rows
                const int nbv = min(TC_NB, (p.n - n0) / 128);    // column blocks present (last tile may be partial)
                mbar_expect_tx(&t_full[ts], blk * (uint32_t)nbv);
                uint8_t* dst = smem + TcSmem::t0 + (size_t)ts * p.t_stage_bytes;
                for (int b = 0; b < nbv; ++b) {
                    const uint8_t* src = p.packed + (size_t)(n0 / 128 + b) * block_bytes + (size_t)kc * blk;
                    bulk_g2s(dst + b * blk, src, blk, &t_full[ts]);
                }
                last[ts] = kc;
            }
            for (int s = 0; s < p.t_stages; ++s)
                if (last[s] >= 0 && !mbar_wait(&t_full[s], (last[s] / p.t_stages) & 1)) to = true;
        }
    } else {
        // ---------------- decoders, then the epilogue ----------------
        const int dw = warp - 3;
        switch (p.K) {
            case 1: tc_decoder_loop<1>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
            case 2: tc_decoder_loop<2>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
            case 3: tc_decoder_loop<3>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
            case 4: tc_decoder_loop<4>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
            case 5: tc_decoder_loop<5>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
            case 6: tc_decoder_loop<6>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
            case 7: tc_decoder_loop<7>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
            default: tc_decoder_loop<8>(p, smem, t_full, t_empty, b_full, b_empty, nk, dw, lane, to); break;
        }
        pdl_wait();                                           // y may be in use by an earlier kernel until here
        if (!to && !mbar_wait(acc_full, 0)) to = true;
        tc_fence_after();
        // TMEM lane quadrant of this warp; the four warps of a quadrant take one 128 x 128 block each:
        // block bi = accumulator bi / TC_NB, column block bi % TC_NB
        const int quad = warp & 3, bi = dw >> 2;              // warps 3..18: quad covers 0..3 four times
        static_assert(TC_ACC * TC_NB == 4, "four 128 x 128 blocks per tile");
        // staging: [2][128 rows][128 cols] fp32 in the A stages (free after the main loop), columns XOR-swizzled
        // by the row; blocks 0, 1 then 2, 3
        for (int pass = 0; pass < 2; ++pass) {
            if ((bi >> 1) == pass) {
                float* st = reinterpret_cast<float*>(smem + TcSmem::a0) + (size_t)(bi & 1) * 128 * 128;
                const int row = quad * 32 + lane;             // accumulator row = TMEM lane
                const uint32_t col0 = (uint32_t)((bi / TC_NB) * TC_BN + (bi % TC_NB) * 128);
#pragma unroll
                for (int c0 = 0; c0 < 128; c0 += 32) {
                    uint32_t r[32];
                    tc_ld32(tmem + ((uint32_t)(quad * 32) << 16) + col0 + (uint32_t)c0, r);
#pragma unroll
                    for (int c = 0; c < 32; ++c)
                        st[row * 128 + ((c0 + c) ^ (row & 31))] = __uint_as_float(r[c]);
                }
            }
            asm volatile("bar.sync 1, %0;" ::"r"(TC_DEC_WARPS * 32) : "memory");
            // 2 accumulators x 128 rows over 16 warps, one row at a time
            for (int rb = dw; rb < 2 * 128; rb += TC_DEC_WARPS) {
                const int jj = rb >> 7, row = rb & 127;
                const float* src = reinterpret_cast<const float*>(smem + TcSmem::a0) + (size_t)jj * 128 * 128 +
                                   row * 128;
                float v[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) v[e] = src[(4 * lane + e) ^ (row & 31)];
                fwht128_warp(v, lane);
                const int blk = pass * 2 + jj;
                const int m = m0 + (blk / TC_NB) * 128 + row;
                const int col = n0 + (blk % TC_NB) * 128 + 4 * lane;
                if (m < p.M && col < p.n) {
                    float o[4];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float sv = __half2float(p.svh[col + e]);
                        if (p.y_dtype == EXL3_F16)
                            o[e] = __half2float(__float2half_rn(__half2float(__float2half_rn(v[e] * kRsqrt128)) * sv));
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

using PFN_encode_tiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                      const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                      CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

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

    // rotated activations, row-major fp16
    {
        const long jobs = (long)M * (k / 128);
        long blocks = (jobs + 7) / 8;
        if (blocks > 8L * num_sms()) blocks = 8L * num_sms();
        cudaError_t e = launch_pdl(k_rotate_rows, dim3((unsigned)blocks), dim3(256), 0, st, x, ldx,
                                   (int)(x_dtype == EXL3_BF16), M, k, static_cast<const __half*>(suh), xh);
        EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_gemm_tc: rotate launch failed: %s", cudaGetErrorString(e));
    }
    // tensor map of xh: [M][k] fp16, box 64 x 256, 128-byte swizzle, zero fill beyond M
    CUtensorMap map;
    const cuuint64_t dims[2] = {(cuuint64_t)k, (cuuint64_t)M};
    const cuuint64_t strides[1] = {(cuuint64_t)k * 2};
    const cuuint32_t box[2] = {TC_BK, TC_BM < 256 ? TC_BM : 256};  // TC_BM / 256 boxes per stage
    const cuuint32_t estr[2] = {1, 1};
    // the driver entry point through the runtime (no link-time dependency on libcuda)
    static PFN_encode_tiled encode = nullptr;
    if (!encode) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        EXL3_REQUIRE(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
                         q == cudaDriverEntryPointSuccess && fn,
                     EXL3_ERR_CUDA, "exl3_gemm_tc: cuTensorMapEncodeTiled is not available");
        encode = reinterpret_cast<PFN_encode_tiled>(fn);
    }
    CUresult cr = encode(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, xh, dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    EXL3_REQUIRE(cr == CUDA_SUCCESS, EXL3_ERR_CUDA, "exl3_gemm_tc: cuTensorMapEncodeTiled failed (%d)", (int)cr);

    TcArgs a = {};
    a.packed = static_cast<const uint8_t*>(packed);
    a.svh = static_cast<const __half*>(svh);
    a.y = y;
    a.ldy = ldy;
    a.y_dtype = y_dtype;
    a.M = M;
    a.k = k;
    a.n = n;
    a.K = K;
    a.t_stage_bytes = TC_NB * 4 * 8 * 32 * K;                // column blocks x 4 tile-rows x 8 tiles
    a.t_stages = TC_T_RING / a.t_stage_bytes;
    if (a.t_stages > TC_MAX_TSTAGES) a.t_stages = TC_MAX_TSTAGES;
    a.status = device_status_ptr();

    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        EXL3_REQUIRE(cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, TcSmem::total) ==
                         cudaSuccess,
                     EXL3_ERR_CUDA, "exl3_gemm_tc: cudaFuncSetAttribute: %s",
                     cudaGetErrorString(cudaGetLastError()));
        configured[dev] = 1;
    }
    const dim3 grid((n + TC_BN - 1) / TC_BN, (M + TC_BM - 1) / TC_BM);
    cudaError_t e = launch_pdl(k_gemm_tc, grid, dim3(TC_THREADS), TcSmem::total, st, map, a);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_gemm_tc: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

}  // extern "C"
