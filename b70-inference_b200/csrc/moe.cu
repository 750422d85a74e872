// MoE decode path: top-k router with residency bias, the prepare step (token/expert alignment + rotated activation
// rows), grouped gate|up and down GEMVs (gemv.cuh), and the fixed-order combine.
//
// Workspace layout of exl3_moe_decode and its phases (int32 words unless noted; P = pairs + shared rows):
//   [0] n_items  [1] n_valid (routed pair positions)  [2] positions in use (+ shared rows)  [3..7] reserved
//   item_expert[max_items] item_start[max_items] item_cnt[max_items]
//   pair_tok[P] pair_expert[P] pair_of[pairs] pair_w[P] (fp32) pair_src[P]
//   tickets[max_items * max(H, I) / 128] (GEMV split-unit counters)
//   then, 256-byte aligned: gate|up input rows in xf order fp16 [P][2][H] (row = routed pair index, or pairs + m for
//   the shared expert's row of token m), down input rows in xf order fp16 [P][I] (by position), the block sums of
//   both (fp32 [P][2][H/128], [P][I/128]), ybuf fp32 [P][H], GEMV split-unit partial slots.
#include <type_traits>

#include "gemv.cuh"
#include "tc.cuh"

namespace exl3 {

// Rows per GEMV work item: the MMA's N (8), or fewer when the batch is smaller.
inline int item_rows(int M) { return M < 8 ? (M > 0 ? M : 1) : 8; }

struct WsLayout {
    size_t item_expert, item_start, item_cnt, pair_tok, pair_expert, pair_of, pair_w, pair_src, tickets, seg_cnt,
        xf_gu, xf_dn, xsum_gu, xsum_dn, ybuf, partial, total;
    int max_items, p_max, n_tickets;
};

constexpr int kAlignSegPairs = 8192;                            // pairs per CTA of the multi-CTA alignment

inline WsLayout ws_layout(int M, int topk, int E, int H, int I, int shared, int chunk) {
    WsLayout L;
    const int npairs = M * topk;
    const int active = npairs < E ? npairs : E;
    // sum over active experts of ceil(count / chunk) <= (pairs + active (chunk - 1)) / chunk
    L.max_items = (npairs + active * (chunk - 1)) / chunk + (shared ? (M + chunk - 1) / chunk : 0);
    L.p_max = npairs + (shared ? M : 0);
    L.n_tickets = L.max_items * ((H > I ? H : I) / 128);
    size_t o = 8 * 4;
    L.item_expert = o; o += (size_t)L.max_items * 4;
    L.item_start = o; o += (size_t)L.max_items * 4;
    L.item_cnt = o; o += (size_t)L.max_items * 4;
    L.pair_tok = o; o += (size_t)L.p_max * 4;
    L.pair_expert = o; o += (size_t)L.p_max * 4;
    L.pair_of = o; o += (size_t)npairs * 4;
    L.pair_w = o; o += (size_t)L.p_max * 4;
    L.pair_src = o; o += (size_t)L.p_max * 4;
    L.tickets = o; o += (size_t)L.n_tickets * 4;
    L.seg_cnt = o; o += (size_t)((npairs + kAlignSegPairs - 1) / kAlignSegPairs) * E * 4;   // multi-CTA alignment
    o = align_up(o, 256);
    L.xf_gu = o; o += align_up((size_t)L.p_max * 2 * H * 2, 256);
    L.xf_dn = o; o += align_up((size_t)L.p_max * I * 2, 256);
    L.xsum_gu = o; o += align_up((size_t)L.p_max * 2 * (H / 128) * 4, 256);
    L.xsum_dn = o; o += align_up((size_t)L.p_max * (I / 128) * 4, 256);
    L.ybuf = o; o += align_up((size_t)L.p_max * H * 4, 256);
    L.partial = o; o += partial_bytes(EPI_GATEUP);
    L.total = o;
    return L;
}

// ------------------------------------------------------------------------------------------------ router

__device__ __forceinline__ uint32_t ordered_bits(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// Max-reduction key: higher score first, then lower expert index.
__device__ __forceinline__ uint64_t pack_key(float key, int e) {
    if (isnan(key)) key = -INFINITY;
    return ((uint64_t)ordered_bits(key) << 32) | (uint32_t)(0xFFFFFFFFu - (uint32_t)e);
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
    return v;
}
__device__ __forceinline__ uint64_t warp_max_u64(uint64_t v) {
#pragma unroll
    for (int m = 16; m > 0; m >>= 1) {
        uint64_t o = __shfl_xor_sync(0xFFFFFFFFu, v, m);
        v = o > v ? o : v;
    }
    return v;
}

constexpr int kRouteWarps = 4;                        // rows per CTA, one warp each
constexpr int kRouteMaxE = 1024;
constexpr int kRouteMaxK = 32;

__device__ __forceinline__ float route_score(float v, int kind) {
    if (kind == EXL3_ROUTE_SIGMOID) return (float)(1.0 / (1.0 + exp(-(double)v)));
    if (kind == EXL3_ROUTE_SQRT_SOFTPLUS) {
        const double d = (double)v;
        return (float)sqrt(d > 20.0 ? d : log1p(exp(d)));
    }
    return v;
}

// One warp per row. Scores in fp64 rounded once to fp32; selection key = order-preserving bits of the biased
// score, ties to the lowest expert index. Each lane keeps its four best keys (experts lane, lane + 32, ...) sorted in
// registers; a pick is the row's best head by two warp max reductions (key bits, then the negated index among the
// lanes holding that key), and only the lane that owned it pops its head (rescanning its experts for the next four
// once its list runs out). The picks' weights are evaluated in parallel, one lane per pick, and summed in slot order.
// Code stays compact (loops, not unrolled expert scans): a router runs once per layer from a cold instruction cache.
struct RouteParams {
    int E, kind, k;
    const float* bias;
    const float* res;
    const float* mul;
    float scale;
    int renorm;
    void* ids;
    int ids64;
    float* w;
    void* want;
};

// A lane's best keys, best first; key 0 (below every real key: ordered_bits(-inf) > 0) = empty slot.
struct LaneTop4 {
    uint32_t c0, c1, c2, c3;
    int e0, e1, e2, e3;
};

// Insert (kv, e) scanned in ascending e: a key equal to a listed one goes after it (the lower index wins the tie).
__device__ __forceinline__ void top4_insert(LaneTop4& t, uint32_t kv, int e) {
    if (kv <= t.c3) return;
    if (kv > t.c2) {
        t.c3 = t.c2; t.e3 = t.e2;
        if (kv > t.c1) {
            t.c2 = t.c1; t.e2 = t.e1;
            if (kv > t.c0) { t.c1 = t.c0; t.e1 = t.e0; t.c0 = kv; t.e0 = e; }
            else { t.c1 = kv; t.e1 = e; }
        } else {
            t.c2 = kv; t.e2 = e;
        }
    } else {
        t.c3 = kv; t.e3 = e;
    }
}

// The lane's four best keys among its experts (bit j of `live`: expert lane + 32 j) that rank below (kl, el) when
// `below`.
template <int NPL>
__device__ __forceinline__ LaneTop4 top4_fill(const uint32_t (&kh)[NPL], uint32_t live, int lane, bool below,
                                              uint32_t kl, int el) {
    LaneTop4 t = {0u, 0u, 0u, 0u, -1, -1, -1, -1};
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = lane + 32 * j;
        const uint32_t kv = kh[j];
        if (((live >> j) & 1u) && (!below || kv < kl || (kv == kl && e > el))) top4_insert(t, kv, e);
    }
    return t;
}

// k argmax passes over the lane's keys; lane p < k returns pick p.
template <int NPL>
__device__ __forceinline__ int select_topk(const uint32_t (&kh)[NPL], uint32_t live, int k, int lane) {
    LaneTop4 t = top4_fill<NPL>(kh, live, lane, false, 0u, 0);
    int pick = -1;
    for (int p = 0; p < k; ++p) {
        const uint32_t top = __reduce_max_sync(0xFFFFFFFFu, t.c0);
        const uint32_t cand = (t.e0 >= 0 && t.c0 == top) ? 0xFFFFFFFFu - (uint32_t)t.e0 : 0u;
        const int e = (int)(0xFFFFFFFFu - __reduce_max_sync(0xFFFFFFFFu, cand));
        if (lane == p) pick = e;
        const bool own = (e & 31) == lane;
        const uint32_t kl = t.c0;
        if (own) {                                            // the owner pops its head
            t.c0 = t.c1; t.e0 = t.e1; t.c1 = t.c2; t.e1 = t.e2; t.c2 = t.c3; t.e2 = t.e3; t.c3 = 0u; t.e3 = -1;
        }
        // rare (a lane held more than four of the picks so far): its next four, behind a warp-uniform branch
        if (__any_sync(0xFFFFFFFFu, own && t.e0 < 0) && own) t = top4_fill<NPL>(kh, live, lane, true, kl, e);
    }
    return pick;
}

__device__ __forceinline__ uint32_t key_bits(float kv) { return ordered_bits(isnan(kv) ? -INFINITY : kv); }

// s_sc: the warp's shared-memory row of kRouteMaxE scores. NPL = experts per lane (E <= 32 NPL).
template <int NPL>
__device__ void route_row(const float* __restrict__ l, int row, const RouteParams& rp, int lane,
                          float* __restrict__ s_sc) {
    const int E = rp.E, kind = rp.kind, k = rp.k;
    const float* __restrict__ bias = rp.bias;
    const float* __restrict__ res = rp.res;
    const float* __restrict__ mul = rp.mul;
    // every global load of the row issued before any is used
    float v[NPL], bv[NPL], rv[NPL], mv[NPL];
    uint32_t valid = 0;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        const int e = lane + 32 * j;
        const bool ok = e < E;
        valid |= (ok ? 1u : 0u) << j;
        v[j] = ok ? l[e] : -INFINITY;
        bv[j] = (ok && bias) ? bias[e] : 0.f;
        rv[j] = (ok && res) ? res[e] : 0.f;
        mv[j] = (ok && mul) ? mul[e] : 1.f;
    }
    float lmax = -INFINITY;
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
        lmax = fmaxf(lmax, v[j]);
        if ((valid >> j) & 1u) s_sc[lane + 32 * j] = v[j];
    }
    __syncwarp();
    float sc[NPL];
    if (kind != EXL3_ROUTE_SOFTMAX) {                         // fp64 score functions: a compact loop in place
#pragma unroll 2
        for (int e = lane; e < E; e += 32) s_sc[e] = route_score(s_sc[e], kind);
        __syncwarp();
#pragma unroll
        for (int j = 0; j < NPL; ++j) sc[j] = ((valid >> j) & 1u) ? s_sc[lane + 32 * j] : -INFINITY;
    } else {
#pragma unroll
        for (int j = 0; j < NPL; ++j) sc[j] = v[j];
    }
    double denom = 1.0, dmax = 0.0;
    if (kind == EXL3_ROUTE_SOFTMAX) {
        // softmax denominator, only for the weights: fp32 exponentials of the fp32 differences to the row maximum,
        // four partial sums per lane, lanes summed in fp64 (relative error a few 1e-7, which renormalised weights do
        // not see; the picks' own probabilities are evaluated in fp64)
        const float fmax = warp_max(lmax);
        dmax = (double)fmax;
        float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < NPL; ++j)
            if ((valid >> j) & 1u) part[j & 3] += expf(sc[j] - fmax);
        double tot = (double)((part[0] + part[1]) + (part[2] + part[3]));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) tot += __shfl_xor_sync(0xFFFFFFFFu, tot, o);
        denom = tot;
    }

    for (int pass = 0; pass < 2; ++pass) {
        if (pass == 1 && !rp.want) break;
        uint32_t kh[NPL];
#pragma unroll
        for (int j = 0; j < NPL; ++j) {
            float kv = sc[j];
            if (pass == 0 && mul) kv = kv * mv[j];
            if (bias) kv = kv + bv[j];
            if (pass == 0 && res) kv = kv + rv[j];
            kh[j] = key_bits(kv);
        }
        const int pick = select_topk<NPL>(kh, valid, k, lane);
        if (pass == 0) {
            // weights from the unbiased score, summed over the picks in slot order
            float wv = 0.f;
            if (lane < k)
                wv = kind == EXL3_ROUTE_SOFTMAX ? (float)(exp((double)s_sc[pick] - dmax) / denom) : s_sc[pick];
            float tot = 0.f;
            for (int j = 0; j < k; ++j) tot += __shfl_sync(0xFFFFFFFFu, wv, j);
            if (lane < k) {
                float o;
                if (kind == EXL3_ROUTE_SOFTMAX) o = rp.renorm ? wv / (tot + 1e-20f) : wv;
                else o = wv * rp.scale / (tot + 1e-20f);
                rp.w[(size_t)row * k + lane] = o;
                if (rp.ids64) static_cast<int64_t*>(rp.ids)[(size_t)row * k + lane] = pick;
                else static_cast<int32_t*>(rp.ids)[(size_t)row * k + lane] = pick;
            }
        } else if (lane < k) {
            if (rp.ids64) static_cast<int64_t*>(rp.want)[(size_t)row * k + lane] = pick;
            else static_cast<int32_t*>(rp.want)[(size_t)row * k + lane] = pick;
        }
    }
    __syncwarp();
}

// Experts per lane of a row of E experts (a compiled instance of route_row).
inline int route_npl(int E) { return E <= 128 ? 4 : E <= 256 ? 8 : E <= 512 ? 16 : 32; }

__device__ __forceinline__ void route_row_any(const float* __restrict__ l, int row, const RouteParams& rp, int lane,
                                              float* sc) {
    if (rp.E <= 128) route_row<4>(l, row, rp, lane, sc);
    else if (rp.E <= 256) route_row<8>(l, row, rp, lane, sc);
    else if (rp.E <= 512) route_row<16>(l, row, rp, lane, sc);
    else route_row<32>(l, row, rp, lane, sc);
}

template <int NPL>
__global__ void __launch_bounds__(kRouteWarps * 32) k_route(const float* __restrict__ logits, int ld, int R,
                                                            const RouteParams rp) {
    __shared__ float s_score[kRouteWarps][kRouteMaxE];
    pdl_wait();                                               // logits may come from the previous kernel
    const int lane = threadIdx.x & 31, wr = threadIdx.x >> 5;
    const int row = blockIdx.x * kRouteWarps + wr;
    if (row >= R) return;
    route_row<NPL>(logits + (size_t)row * ld, row, rp, lane, s_score[wr]);
}

// Router from the hidden states (the router GEMV fused into the launch): CTAs split the experts, one warp per expert
// computes its logits for every row (fp32 FMA dot over fp16 pairs, lane-strided, then a warp reduction; rounded to
// fp16 as the reference's routing GEMV does, glm/docs/ext-op-inventory.md:980-1004) into the workspace; the CTA that
// finishes last (atomic ticket, left at zero for the next call) routes every row. With a second router (gate_t1, the
// next layer's), one GEMV computes both layers' logits over the same hidden states, [R][E0 + E1], and the last CTA also
// routes the next layer's rows: the reference's layer-ahead prediction in one launch
// (dsv41/xpu/csrc/dsv_moe_glue.sycl:442-520 route_fused / GemvH; glm/xpu/glm_xpu/moe_patch.py:74-84).
constexpr int kRhWarps = 8;
constexpr int kRhRouteWarps = 8;                      // routing warps of the last CTA (static shared memory: 32 KB)
constexpr int kRhMaxRows = 64;

template <typename T>
__global__ void __launch_bounds__(kRhWarps * 32) k_route_hidden(const T* __restrict__ hidden, int ldh, int R, int H,
                                                                const __half* __restrict__ gate_t,
                                                                const __half* __restrict__ gate_t1, float* lg,
                                                                __half* logits_out, unsigned int* ticket,
                                                                const RouteParams rp, const RouteParams rp1) {
    __shared__ float s_score[kRhRouteWarps][kRouteMaxE];
    __shared__ int s_last;
    pdl_wait();                                               // hidden states come from the previous kernel
    const int lane = threadIdx.x & 31, wr = threadIdx.x >> 5;
    const int E0 = rp.E, E = rp.E + (gate_t1 ? rp1.E : 0);   // logits row stride: both routers' experts
    for (int e = blockIdx.x * kRhWarps + wr; e < E; e += gridDim.x * kRhWarps) {
        const __half2* g = reinterpret_cast<const __half2*>(e < E0 ? gate_t + (size_t)e * H
                                                                   : gate_t1 + (size_t)(e - E0) * H);
        for (int r0 = 0; r0 < R; r0 += 8) {
            float acc[8];
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) acc[rr] = 0.f;
            for (int c = lane; c < H / 2; c += 32) {
                const float2 gv = __half22float2(g[c]);
#pragma unroll
                for (int rr = 0; rr < 8; ++rr) {
                    if (r0 + rr < R) {
                        const T* xp = hidden + (size_t)(r0 + rr) * ldh + 2 * c;
                        acc[rr] = fmaf(to_f32<T>(xp[0]), gv.x, acc[rr]);
                        acc[rr] = fmaf(to_f32<T>(xp[1]), gv.y, acc[rr]);
                    }
                }
            }
#pragma unroll
            for (int rr = 0; rr < 8; ++rr) {
                float v = acc[rr];
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
                if (lane == 0 && r0 + rr < R) {
                    const __half h = __float2half_rn(v);
                    lg[(size_t)(r0 + rr) * E + e] = __half2float(h);
                    if (logits_out && e < E0) logits_out[(size_t)(r0 + rr) * E0 + e] = h;
                }
            }
        }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicInc(ticket, gridDim.x - 1) == gridDim.x - 1;
    __syncthreads();
    pdl_trigger();
    if (!s_last) return;
    __threadfence();
    if (wr >= kRhRouteWarps) return;
    for (int row = wr; row < R; row += kRhRouteWarps) {
        route_row_any(lg + (size_t)row * E, row, rp, lane, s_score[wr]);
        if (gate_t1) route_row_any(lg + (size_t)row * E + E0, row, rp1, lane, s_score[wr]);
    }
}

// Router logits for many rows (prefill batches): logits[r][e] = fp16(hidden[r] . gate_t[e]) on the tensor cores
// (mma.sync m16n8k16, fp16 operands, fp32 accumulation; bf16 hidden states converted to fp16 while staged), the same
// faithful fp16 rounding as the fused router's GEMV. CTA tile 64 rows x 64 experts, four warps of 32 x 32, 32-deep
// k chunks staged through shared memory (padded rows: conflict-free ldmatrix), the next chunk loaded into registers
// while the current one is multiplied.
constexpr int kRlTile = 64, kRlK = 32, kRlPad = 40;

__device__ __forceinline__ void ldsm_x4(uint32_t r[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

template <typename T>
__device__ __forceinline__ uint4 rl_load(const T* src, bool ok) {
    if (!ok) return make_uint4(0, 0, 0, 0);
    const uint4 v = *reinterpret_cast<const uint4*>(src);
    if constexpr (sizeof(T) == 2 && !std::is_same<T, __half>::value) {   // bf16 -> fp16, 8 values
        const __nv_bfloat162* b = reinterpret_cast<const __nv_bfloat162*>(&v);
        uint4 o;
        __half2* h = reinterpret_cast<__half2*>(&o);
#pragma unroll
        for (int j = 0; j < 4; ++j) h[j] = __float22half2_rn(__bfloat1622float2(b[j]));
        return o;
    }
    return v;
}

template <typename T>
__global__ void __launch_bounds__(128) k_router_logits(const T* __restrict__ hidden, int ldh, int R, int H,
                                                       const __half* __restrict__ gate_t, int E, float* logits,
                                                       __half* logits_f16) {
    __shared__ __align__(16) __half As[kRlTile][kRlPad];
    __shared__ __align__(16) __half Bs[kRlTile][kRlPad];
    pdl_wait();
    pdl_trigger();
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int m_blk = blockIdx.x * kRlTile, n_blk = blockIdx.y * kRlTile;
    const int wm = (warp >> 1) * 32, wn = (warp & 1) * 32;
    float acc[2][4][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][j][e] = 0.f;
    // staging: 64 rows x 4 uint4 per tile, two uint4 per thread for each of A and B
    uint4 ra[2], rb[2];
    auto load = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int idx = tid + j * 128, row = idx >> 2, c = (idx & 3) * 8;
            ra[j] = rl_load<T>(hidden + (size_t)(m_blk + row) * ldh + k0 + c, m_blk + row < R);
            rb[j] = rl_load<__half>(gate_t + (size_t)(n_blk + row) * H + k0 + c, n_blk + row < E);
        }
    };
    auto store = [&]() {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int idx = tid + j * 128, row = idx >> 2, c = (idx & 3) * 8;
            *reinterpret_cast<uint4*>(&As[row][c]) = ra[j];
            *reinterpret_cast<uint4*>(&Bs[row][c]) = rb[j];
        }
    };
    load(0);
    for (int k0 = 0; k0 < H; k0 += kRlK) {
        __syncthreads();
        store();
        __syncthreads();
        if (k0 + kRlK < H) load(k0 + kRlK);
#pragma unroll
        for (int kk = 0; kk < kRlK; kk += 16) {
            uint32_t a[2][4], b[2][4];
#pragma unroll
            for (int i = 0; i < 2; ++i)
                ldsm_x4(a[i], &As[wm + i * 16 + (lane & 15)][kk + (lane >> 4) * 8]);
#pragma unroll
            for (int j = 0; j < 2; ++j)
                ldsm_x4(b[j], &Bs[wn + j * 16 + (lane & 7) + ((lane >> 4) << 3)][kk + ((lane >> 3) & 1) * 8]);
#pragma unroll
            for (int i = 0; i < 2; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) mma_16816(acc[i][j], a[i], b[j >> 1][(j & 1) * 2], b[j >> 1][(j & 1) * 2 + 1]);
        }
    }
    const int g = lane >> 2, q = lane & 3;
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int m = m_blk + wm + i * 16 + g + ((e >> 1) << 3), n = n_blk + wn + j * 8 + 2 * q + (e & 1);
                if (m < R && n < E) {
                    const __half h = __float2half_rn(acc[i][j][e]);
                    logits[(size_t)m * E + n] = __half2float(h);
                    if (logits_f16) logits_f16[(size_t)m * E + n] = h;
                }
            }
}

// ------------------------------------------------------------------------------------------------ align

constexpr int kAlignThreads = 1024;
constexpr int kAlignWarps = kAlignThreads / 32;

// Exclusive prefix sum over the CTA (one value per thread); *total receives the sum of all values.
__device__ __forceinline__ int block_excl_scan(int v, int* scan, int* total) {
    const int t = threadIdx.x;
    scan[t] = v;
    __syncthreads();
    for (int o = 1; o < kAlignThreads; o <<= 1) {
        const int add = t >= o ? scan[t - o] : 0;
        __syncthreads();
        scan[t] += add;
        __syncthreads();
    }
    const int incl = scan[t];
    *total = scan[kAlignThreads - 1];
    __syncthreads();
    return incl - v;
}

struct AlignOut {
    int* ws_i;
    int* item_expert;
    int* item_start;
    int* item_cnt;
    int* pair_tok;
    int* pair_expert;
    int* pair_of;
    float* pair_w;
    int* pair_src;
};

// Stable placement of the pairs [a0, a1) of one warp: cnt_w[e] is the warp's next position for expert e (experts
// ascending, pair index ascending within an expert). Deterministic, unlike an atomic fill
// (glm/xpu/csrc/exl3_moe.n128.sycl:693-734 fills positions in atomic order).
__device__ void place_pairs(const int32_t* __restrict__ ids, const float* __restrict__ w, int topk, int E, int a0,
                            int a1, int* cnt_w, const AlignOut& o) {
    const int lane = threadIdx.x & 31;
    for (int base = a0; base < a1; base += 32) {
        const int i = base + lane;
        const bool act = i < a1;
        const unsigned amask = __ballot_sync(0xFFFFFFFFu, act);
        if (act) {
            const int e = ids[i];
            const bool valid = e >= 0 && e < E;
            const unsigned peers = __match_any_sync(amask, valid ? e : -1);
            const unsigned before = peers & ((1u << lane) - 1u);
            if (valid) {
                const int pos = cnt_w[e] + __popc(before);
                o.pair_tok[pos] = i / topk;
                o.pair_expert[pos] = e;
                o.pair_w[pos] = w[i];
                o.pair_src[pos] = i;
                o.pair_of[i] = pos;
            } else {
                o.pair_of[i] = -1;
            }
            __syncwarp(amask);
            if (valid && before == 0) cnt_w[e] += __popc(peers);
            __syncwarp(amask);
        }
    }
}

// Item table and counters (thread t = expert t holds its count `total` and first position `start`): ceil(count /
// chunk) items per active expert in expert order, then the shared expert's rows (expert id E, weight 1) at positions
// n_valid + m. Every thread of the CTA calls this (it scans).
__device__ void write_items(int total, int start, int n_valid, int E, int M, int npairs, int shared, int chunk,
                            const AlignOut& o, int* scan) {
    const int t = threadIdx.x;
    const int nch = t < E ? (total + chunk - 1) / chunk : 0;
    int n_routed_items = 0;
    const int ibase = block_excl_scan(nch, scan, &n_routed_items);
    const int shared_items = shared ? (M + chunk - 1) / chunk : 0;
    if (t == 0) {
        o.ws_i[0] = n_routed_items + shared_items;
        o.ws_i[1] = n_valid;
        o.ws_i[2] = n_valid + (shared ? M : 0);
    }
    if (t < E)
        for (int c = 0; c < nch; ++c) {
            o.item_expert[ibase + c] = t;
            o.item_start[ibase + c] = start + c * chunk;
            o.item_cnt[ibase + c] = min(chunk, total - c * chunk);
        }
    if (shared) {
        for (int m = t; m < M; m += kAlignThreads) {
            o.pair_tok[n_valid + m] = m;
            o.pair_expert[n_valid + m] = E;
            o.pair_w[n_valid + m] = 1.0f;
            o.pair_src[n_valid + m] = npairs + m;
        }
        for (int c = t; c < shared_items; c += kAlignThreads) {
            o.item_expert[n_routed_items + c] = E;
            o.item_start[n_routed_items + c] = n_valid + c * chunk;
            o.item_cnt[n_routed_items + c] = min(chunk, M - c * chunk);
        }
    }
}

// One CTA. Pairs are split into 32 contiguous warp segments; per-(warp, expert) counts give every pair a stable
// position (experts ascending, pair index ascending within an expert). pair_src[position] = the routed pair index
// (the gate|up activation row), npairs + m for shared rows.
__device__ void align_cta(const int32_t* __restrict__ ids, const float* __restrict__ w, int npairs, int topk, int E,
                          int M, int shared, int chunk, const AlignOut& o, int* sm) {
    int* cnt = sm;                             // [kAlignWarps][E]
    int* scan = sm + kAlignWarps * E;          // [kAlignThreads]
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    for (int i = t; i < kAlignWarps * E; i += kAlignThreads) cnt[i] = 0;
    __syncthreads();
    const int seg = (npairs + kAlignWarps - 1) / kAlignWarps;
    const int a0 = min(npairs, warp * seg), a1 = min(npairs, a0 + seg);
    for (int i = a0 + lane; i < a1; i += 32) {
        const int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(&cnt[warp * E + e], 1);
    }
    __syncthreads();
    int total = 0;
    if (t < E)
        for (int ww = 0; ww < kAlignWarps; ++ww) total += cnt[ww * E + t];
    int n_valid = 0;
    const int start = block_excl_scan(total, scan, &n_valid);
    if (t < E) {
        int run = start;
        for (int ww = 0; ww < kAlignWarps; ++ww) {
            const int c = cnt[ww * E + t];
            cnt[ww * E + t] = run;
            run += c;
        }
    }
    write_items(total, start, n_valid, E, M, npairs, shared, chunk, o, scan);
    __syncthreads();
    place_pairs(ids, w, topk, E, a0, a1, cnt + warp * E, o);
}

// Alignment of at most kAlignSmallPairs pairs by all warps of the CTA (decode batches): the same tables as
// align_cta from warp votes, without block-wide scans. Every lane holds the experts of pairs lane and lane + 32; the
// warp of pair i counts by ballot the valid pairs ranked before it (smaller expert, or the same expert and a smaller
// index: its position), the pairs of its expert, and whether it is the expert's first pair, which then writes the
// expert's items after those of all smaller experts. sm: 3 kAlignSmallPairs ints of shared memory.
constexpr int kAlignSmallPairs = 64;

__device__ void align_small(const int32_t* __restrict__ ids, const float* __restrict__ w, int npairs, int topk, int E,
                            int M, int shared, int chunk, const AlignOut& o, int* sm) {
    int* s_nch = sm;
    int* s_pos = sm + kAlignSmallPairs;
    int* s_cnt = sm + 2 * kAlignSmallPairs;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    int ej[2];
    bool vj[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int j = lane + 32 * h;
        ej[h] = j < npairs ? ids[j] : -1;
        vj[h] = ej[h] >= 0 && ej[h] < E;
    }
    for (int i = warp; i < npairs; i += nw) {
        const int ei = __shfl_sync(0xFFFFFFFFu, i < 32 ? ej[0] : ej[1], i & 31);
        const bool vi = ei >= 0 && ei < E;
        int pos = 0, cnt = 0;
        bool first = true;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = lane + 32 * h;
            const bool same = vj[h] && ej[h] == ei;
            pos += __popc(__ballot_sync(0xFFFFFFFFu, vj[h] && (ej[h] < ei || (same && j < i))));
            cnt += __popc(__ballot_sync(0xFFFFFFFFu, same));
            if (__ballot_sync(0xFFFFFFFFu, same && j < i)) first = false;
        }
        if (lane == 0) {
            s_nch[i] = (vi && first) ? (cnt + chunk - 1) / chunk : 0;
            s_pos[i] = vi ? pos : -1;
            s_cnt[i] = cnt;
        }
    }
    __syncthreads();
    int nch_j[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) nch_j[h] = lane + 32 * h < npairs ? s_nch[lane + 32 * h] : 0;
    const int n_valid = __popc(__ballot_sync(0xFFFFFFFFu, vj[0])) + __popc(__ballot_sync(0xFFFFFFFFu, vj[1]));
    const int n_routed_items = (int)__reduce_add_sync(0xFFFFFFFFu, (unsigned)(nch_j[0] + nch_j[1]));
    const int shared_items = shared ? (M + chunk - 1) / chunk : 0;
    for (int i = warp; i < npairs; i += nw) {
        const int ei = __shfl_sync(0xFFFFFFFFu, i < 32 ? ej[0] : ej[1], i & 31);
        const int pos = s_pos[i], nch = s_nch[i], cnt = s_cnt[i];
        if (lane == 0) {
            o.pair_of[i] = pos;
            if (pos >= 0) {
                o.pair_tok[pos] = i / topk;
                o.pair_expert[pos] = ei;
                o.pair_w[pos] = w[i];
                o.pair_src[pos] = i;
            }
        }
        if (nch) {                                            // warp-uniform: the expert's first pair
            const unsigned below = (vj[0] && ej[0] < ei ? nch_j[0] : 0) + (vj[1] && ej[1] < ei ? nch_j[1] : 0);
            const int ibase = (int)__reduce_add_sync(0xFFFFFFFFu, below);
            for (int c = lane; c < nch; c += 32) {
                o.item_expert[ibase + c] = ei;
                o.item_start[ibase + c] = pos + c * chunk;
                o.item_cnt[ibase + c] = min(chunk, cnt - c * chunk);
            }
        }
    }
    if (warp == 0) {
        if (lane == 0) {
            o.ws_i[0] = n_routed_items + shared_items;
            o.ws_i[1] = n_valid;
            o.ws_i[2] = n_valid + (shared ? M : 0);
        }
        if (shared) {
            for (int m = lane; m < M; m += 32) {
                o.pair_tok[n_valid + m] = m;
                o.pair_expert[n_valid + m] = E;
                o.pair_w[n_valid + m] = 1.0f;
                o.pair_src[n_valid + m] = npairs + m;
            }
            for (int c = lane; c < shared_items; c += 32) {
                o.item_expert[n_routed_items + c] = E;
                o.item_start[n_routed_items + c] = n_valid + c * chunk;
                o.item_cnt[n_routed_items + c] = min(chunk, M - c * chunk);
            }
        }
    }
}

// Multi-CTA alignment of large pair counts (prefill), the same tables as align_cta: segments of kAlignSeg pairs,
// pass 1 counts per (segment, expert), pass 2 gives each segment its offsets from those counts and places its pairs.
constexpr int kAlignSeg = kAlignSegPairs;

__global__ void __launch_bounds__(kAlignThreads) k_align_count(const int32_t* __restrict__ ids, int npairs, int E,
                                                               int* __restrict__ seg_cnt) {
    extern __shared__ int h[];                                // [E]
    pdl_wait();
    pdl_trigger();
    for (int e = threadIdx.x; e < E; e += kAlignThreads) h[e] = 0;
    __syncthreads();
    const int a0 = blockIdx.x * kAlignSeg, a1 = min(npairs, a0 + kAlignSeg);
    for (int i = a0 + threadIdx.x; i < a1; i += kAlignThreads) {
        const int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(&h[e], 1);
    }
    __syncthreads();
    for (int e = threadIdx.x; e < E; e += kAlignThreads) seg_cnt[(size_t)blockIdx.x * E + e] = h[e];
}

__global__ void __launch_bounds__(kAlignThreads) k_align_place(const int32_t* __restrict__ ids,
                                                               const float* __restrict__ w, int npairs, int topk,
                                                               int E, int M, int shared, int chunk,
                                                               const int* __restrict__ seg_cnt, const AlignOut o) {
    extern __shared__ int sm[];
    int* cnt = sm;                             // [kAlignWarps][E]
    int* scan = sm + kAlignWarps * E;          // [kAlignThreads]
    pdl_wait();
    pdl_trigger();
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, sg = blockIdx.x;
    int total = 0, before = 0;
    if (t < E)
        for (int ss = 0; ss < (int)gridDim.x; ++ss) {
            const int c = __ldcg(seg_cnt + (size_t)ss * E + t);
            total += c;
            if (ss < sg) before += c;
        }
    int n_valid = 0;
    const int start = block_excl_scan(total, scan, &n_valid);
    for (int i = t; i < kAlignWarps * E; i += kAlignThreads) cnt[i] = 0;
    __syncthreads();
    const int s0 = sg * kAlignSeg, s1 = min(npairs, s0 + kAlignSeg);
    const int wseg = (s1 - s0 + kAlignWarps - 1) / kAlignWarps;
    const int a0 = min(s1, s0 + warp * wseg), a1 = min(s1, a0 + wseg);
    for (int i = a0 + lane; i < a1; i += 32) {
        const int e = ids[i];
        if (e >= 0 && e < E) atomicAdd(&cnt[warp * E + e], 1);
    }
    __syncthreads();
    if (t < E) {
        int run = start + before;
        for (int ww = 0; ww < kAlignWarps; ++ww) {
            const int c = cnt[ww * E + t];
            cnt[ww * E + t] = run;
            run += c;
        }
    }
    if (sg == 0) write_items(total, start, n_valid, E, M, npairs, shared, chunk, o, scan);
    __syncthreads();
    place_pairs(ids, w, topk, E, a0, a1, cnt + warp * E, o);
}

__global__ void __launch_bounds__(kAlignThreads) k_align(const int32_t* __restrict__ ids, const float* __restrict__ w,
                                                         int npairs, int topk, int E, int M, int shared, int chunk,
                                                         const AlignOut o) {
    extern __shared__ int sm[];
    pdl_wait();
    if (npairs <= kAlignSmallPairs) {
        align_small(ids, w, npairs, topk, E, M, shared, chunk, o, sm);
    } else {
        align_cta(ids, w, npairs, topk, E, M, shared, chunk, o, sm);
    }
}

// ------------------------------------------------------------------------------------------------ prepare

// CTA 0 aligns (tables, tickets zeroed) and only then lets the gate|up GEMV launch: that kernel's producers read the
// item table before their own griddepcontrol.wait. The other CTAs rotate the activation rows of every routed pair
// (row = pair index: token i / topk, the picked expert's gate and up input signs) and of the shared expert's rows,
// one warp per (row, matrix, 128-block); they need only ids, so they run beside the alignment.
struct PrepareArgs {
    const void* x;
    int ldx, x_bf16;
    const int32_t* ids;
    const float* w;
    int M, topk, E, shared, H, chunk;
    const ExpertDesc* experts;
    AlignOut o;
    int* tickets;
    int n_tickets;
    __half* xf;                  // [P][2][H]
    float* xsum;                 // [P][2][H / 128] block sums of the rotated rows
};

__global__ void __launch_bounds__(kAlignThreads) k_prepare(const PrepareArgs a) {
    extern __shared__ int sm[];
    pdl_wait();                                               // ids (router) and x come from earlier kernels
    const int npairs = a.M * a.topk;
    if (blockIdx.x == 0) {
        for (int i = threadIdx.x; i < a.n_tickets; i += kAlignThreads) a.tickets[i] = 0;
        if (npairs <= kAlignSmallPairs) align_small(a.ids, a.w, npairs, a.topk, a.E, a.M, a.shared, a.chunk, a.o, sm);
        else align_cta(a.ids, a.w, npairs, a.topk, a.E, a.M, a.shared, a.chunk, a.o, sm);
        __threadfence();
        __syncthreads();
        pdl_trigger();
        return;
    }
    pdl_trigger();
    const int KB = a.H / 128;
    const int lane = threadIdx.x & 31;
    const int rows = npairs + (a.shared ? a.M : 0);
    const int jobs = rows * 2 * KB;
    const int nw = (gridDim.x - 1) * (kAlignThreads / 32);
    for (int j = (blockIdx.x - 1) * (kAlignThreads / 32) + (threadIdx.x >> 5); j < jobs; j += nw) {
        const int row = j / (2 * KB), mat = (j / KB) % 2, kb = j % KB;
        int tok, e;
        if (row < npairs) {
            e = a.ids[row];
            if (e < 0 || e >= a.E) continue;                  // never read: the pair has no position
            tok = row / a.topk;
        } else {
            tok = row - npairs;
            e = a.E;
        }
        const __half* suh = a.experts[e].suh[mat];
        const __half* su = suh ? suh + kb * 128 : nullptr;
        float v[4];
        if (a.x_bf16)
            rotated_block<__nv_bfloat16>(
                reinterpret_cast<const __nv_bfloat16*>(a.x) + (size_t)tok * a.ldx + kb * 128, su, lane, v);
        else
            rotated_block<__half>(reinterpret_cast<const __half*>(a.x) + (size_t)tok * a.ldx + kb * 128, su, lane, v);
        store_xf_block(v, lane, a.xf + ((size_t)row * 2 + mat) * a.H + (size_t)kb * 128);
        const float bs = xf_block_sum(v);
        if (lane == 0) a.xsum[((size_t)row * 2 + mat) * KB + kb] = bs;
    }
}

// ------------------------------------------------------------------------------------------------ combine

// out[m][h] = sum_j ybuf[pair_of[m*topk + j]][h] (+ ybuf[n_valid + m][h] for the shared expert), slot order.
template <typename TOut>
__global__ void k_combine(const float* __restrict__ ybuf, const int* __restrict__ pair_of, const int* ws_i, int M,
                          int H, int topk, int shared, TOut* out) {
    pdl_wait();                                               // ybuf comes from the down kernel
    const int idx = blockIdx.x * blockDim.x + threadIdx.x;     // one float4 of one row
    const int per_row = H / 4;
    if (idx >= M * per_row) return;
    const int m = idx / per_row, c = (idx % per_row) * 4;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < topk; ++j) {
        const int pos = pair_of[m * topk + j];
        if (pos < 0) continue;
        const float4 v = *reinterpret_cast<const float4*>(ybuf + (size_t)pos * H + c);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if (shared) {
        const float4 v = *reinterpret_cast<const float4*>(ybuf + (size_t)(ws_i[1] + m) * H + c);
        acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
    if constexpr (sizeof(TOut) == 4) {
        *reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + (size_t)m * H + c) = acc;
    } else {
        __half* o = reinterpret_cast<__half*>(out) + (size_t)m * H + c;
        o[0] = __float2half_rn(acc.x); o[1] = __float2half_rn(acc.y);
        o[2] = __float2half_rn(acc.z); o[3] = __float2half_rn(acc.w);
    }
}

// ------------------------------------------------------------------------------------------------ host side

static AlignOut align_out(uint8_t* ws, const WsLayout& L) {
    AlignOut o;
    o.ws_i = reinterpret_cast<int*>(ws);
    o.item_expert = reinterpret_cast<int*>(ws + L.item_expert);
    o.item_start = reinterpret_cast<int*>(ws + L.item_start);
    o.item_cnt = reinterpret_cast<int*>(ws + L.item_cnt);
    o.pair_tok = reinterpret_cast<int*>(ws + L.pair_tok);
    o.pair_expert = reinterpret_cast<int*>(ws + L.pair_expert);
    o.pair_of = reinterpret_cast<int*>(ws + L.pair_of);
    o.pair_w = reinterpret_cast<float*>(ws + L.pair_w);
    o.pair_src = reinterpret_cast<int*>(ws + L.pair_src);
    return o;
}

template <typename Kern>
static int set_max_smem_once(Kern kern, int* configured, const char* what) {
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !configured[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess) {
            set_error("%s: cudaFuncSetAttribute: %s", what, cudaGetErrorString(cudaGetLastError()));
            return EXL3_ERR_CUDA;
        }
        configured[dev] = 1;
    }
    return EXL3_OK;
}

static size_t align_smem(int E) { return (size_t)(kAlignWarps * E + kAlignThreads) * 4; }

static int launch_align_multi(const int32_t* ids, const float* w, int M, int topk, int E, int shared, int chunk,
                              uint8_t* ws, const WsLayout& L, cudaStream_t st);

// The alignment kernels: one CTA up to kAlignSeg pairs, the two-pass multi-CTA version beyond.
static int launch_align(const int32_t* ids, const float* w, int M, int topk, int E, int shared, int chunk,
                        uint8_t* ws, const WsLayout& L, cudaStream_t st) {
    if (M * topk > kAlignSeg) return launch_align_multi(ids, w, M, topk, E, shared, chunk, ws, L, st);
    const size_t smem = align_smem(E);
    EXL3_REQUIRE(smem <= 227 * 1024, EXL3_ERR_UNSUPPORTED, "moe align: E=%d too large", E);
    static int configured[64] = {0};
    int rc = set_max_smem_once(k_align, configured, "moe align");
    if (rc) return rc;
    cudaError_t e = launch_pdl(k_align, dim3(1), dim3(kAlignThreads), smem, st, ids, w, M * topk, topk, E, M, shared,
                               chunk, align_out(ws, L));
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "moe align: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

// Alignment of a large batch over several CTAs (per-segment counts in the workspace's seg_cnt region).
static int launch_align_multi(const int32_t* ids, const float* w, int M, int topk, int E, int shared, int chunk,
                              uint8_t* ws, const WsLayout& L, cudaStream_t st) {
    const int npairs = M * topk;
    const int nseg = (npairs + kAlignSeg - 1) / kAlignSeg;
    int* seg_cnt = reinterpret_cast<int*>(ws + L.seg_cnt);
    const size_t smem = align_smem(E);
    EXL3_REQUIRE(smem <= 227 * 1024, EXL3_ERR_UNSUPPORTED, "moe align: E=%d too large", E);
    static int configured[64] = {0};
    int rc = set_max_smem_once(k_align_place, configured, "moe align");
    if (rc) return rc;
    cudaError_t e = launch_pdl(k_align_count, dim3(nseg), dim3(kAlignThreads), (size_t)E * 4, st, ids, npairs, E,
                               seg_cnt);
    if (e == cudaSuccess)
        e = launch_pdl(k_align_place, dim3(nseg), dim3(kAlignThreads), smem, st, ids, w, npairs, topk, E, M, shared,
                       chunk, static_cast<const int*>(seg_cnt), align_out(ws, L));
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "moe align: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

static int moe_check(int M, int topk, const exl3_expert* experts, int E, int H, int I, int n_ctas,
                     const char* what) {
    EXL3_REQUIRE(experts && M >= 0 && topk > 0 && E > 0, EXL3_ERR_ARG, "%s: bad arguments", what);
    EXL3_REQUIRE(E <= 1024, EXL3_ERR_UNSUPPORTED, "%s: E=%d > 1024", what, E);
    EXL3_REQUIRE(H % 128 == 0 && I % 128 == 0 && H > 0 && I > 0, EXL3_ERR_ARG,
                 "%s: H=%d, I=%d must be multiples of 128", what, H, I);
    EXL3_REQUIRE(n_ctas >= 0, EXL3_ERR_ARG, "%s: n_ctas=%d", what, n_ctas);
    return EXL3_OK;
}

static int ws_check(void* workspace, size_t ws_bytes, const WsLayout& L, const char* what) {
    EXL3_REQUIRE(workspace && ws_bytes >= L.total && aligned16(workspace), EXL3_ERR_WORKSPACE,
                 "%s: workspace %zu < %zu bytes (or not 16-byte aligned)", what, ws_bytes, L.total);
    return EXL3_OK;
}

static int run_prepare(const void* x, int x_dtype, int ldx, int M, const int32_t* ids, const float* w, int topk,
                       const exl3_expert* experts, int E, int shared, int H, int I, void* workspace,
                       size_t ws_bytes, cudaStream_t st) {
    int rc = moe_check(M, topk, experts, E, H, I, 0, "exl3_moe_prepare");
    if (rc || M == 0) return rc;
    EXL3_REQUIRE(x && ids && w, EXL3_ERR_ARG, "exl3_moe_prepare: null pointer");
    EXL3_REQUIRE(x_dtype == EXL3_F16 || x_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "exl3_moe_prepare: x dtype");
    EXL3_REQUIRE(ldx >= H && ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 7) == 0, EXL3_ERR_ARG,
                 "exl3_moe_prepare: x rows must be 8-byte aligned (ldx=%d)", ldx);
    const WsLayout L = ws_layout(M, topk, E, H, I, shared, item_rows(M));
    rc = ws_check(workspace, ws_bytes, L, "exl3_moe_prepare");
    if (rc) return rc;
    const size_t smem = align_smem(E);
    EXL3_REQUIRE(smem <= 227 * 1024, EXL3_ERR_UNSUPPORTED, "exl3_moe_prepare: E=%d too large", E);
    static int configured[64] = {0};
    rc = set_max_smem_once(k_prepare, configured, "exl3_moe_prepare");
    if (rc) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    PrepareArgs a = {};
    a.x = x;
    a.ldx = ldx;
    a.x_bf16 = x_dtype == EXL3_BF16;
    a.ids = ids;
    a.w = w;
    a.M = M;
    a.topk = topk;
    a.E = E;
    a.shared = shared;
    a.H = H;
    a.chunk = item_rows(M);
    a.experts = reinterpret_cast<const ExpertDesc*>(experts);
    a.o = align_out(ws, L);
    a.tickets = reinterpret_cast<int*>(ws + L.tickets);
    a.n_tickets = L.n_tickets;
    a.xf = reinterpret_cast<__half*>(ws + L.xf_gu);
    a.xsum = reinterpret_cast<float*>(ws + L.xsum_gu);
    const long jobs = (long)L.p_max * 2 * (H / 128);
    long ctas = (jobs + kAlignWarps - 1) / kAlignWarps;
    if (ctas > 2 * num_sms()) ctas = 2 * num_sms();
    cudaError_t e = launch_pdl(k_prepare, dim3((unsigned)(1 + ctas)), dim3(kAlignThreads), smem, st, a);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_moe_prepare: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

static GemvArgs moe_args(const exl3_expert* experts, float act_limit, uint8_t* ws, const WsLayout& L) {
    GemvArgs a = {};
    a.experts = reinterpret_cast<const ExpertDesc*>(experts);
    a.items.n_items = reinterpret_cast<const int*>(ws);
    a.items.item_expert = reinterpret_cast<const int*>(ws + L.item_expert);
    a.items.item_start = reinterpret_cast<const int*>(ws + L.item_start);
    a.items.item_cnt = reinterpret_cast<const int*>(ws + L.item_cnt);
    a.items.pair_src = reinterpret_cast<const int*>(ws + L.pair_src);
    a.items.pair_w = reinterpret_cast<const float*>(ws + L.pair_w);
    a.ybuf = reinterpret_cast<float*>(ws + L.ybuf);
    a.act_limit = act_limit;
    a.partial = reinterpret_cast<float*>(ws + L.partial);
    a.counters = reinterpret_cast<int*>(ws + L.tickets);
    a.status = device_status_ptr();
    return a;
}

static int run_gateup(int M, int topk, const exl3_expert* experts, int E, int shared, int H, int I,
                      float act_limit, void* workspace, size_t ws_bytes, int n_ctas, cudaStream_t st) {
    int rc = moe_check(M, topk, experts, E, H, I, n_ctas, "exl3_moe_gateup");
    if (rc || M == 0) return rc;
    const WsLayout L = ws_layout(M, topk, E, H, I, shared, item_rows(M));
    rc = ws_check(workspace, ws_bytes, L, "exl3_moe_gateup");
    if (rc) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    GemvArgs a = moe_args(experts, act_limit, ws, L);
    a.xf = reinterpret_cast<const __half*>(ws + L.xf_gu);
    a.xsum = reinterpret_cast<const float*>(ws + L.xsum_gu);
    a.xf_out = reinterpret_cast<__half*>(ws + L.xf_dn);
    a.xsum_out = reinterpret_cast<float*>(ws + L.xsum_dn);
    a.k = H;
    a.n = I;
    const GemvPlan pl = plan_gemv(EPI_GATEUP, (long long)L.max_items * (I / 128) * (H / 128), n_ctas);
    return launch_gemv<EPI_GATEUP>(a, pl, st, "exl3_moe_gateup");
}

static int run_down(int M, int topk, const exl3_expert* experts, int E, int shared, int H, int I, void* workspace,
                    size_t ws_bytes, int n_ctas, cudaStream_t st) {
    int rc = moe_check(M, topk, experts, E, H, I, n_ctas, "exl3_moe_down");
    if (rc || M == 0) return rc;
    const WsLayout L = ws_layout(M, topk, E, H, I, shared, item_rows(M));
    rc = ws_check(workspace, ws_bytes, L, "exl3_moe_down");
    if (rc) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    GemvArgs a = moe_args(experts, 0.f, ws, L);
    a.xf = reinterpret_cast<const __half*>(ws + L.xf_dn);
    a.xsum = reinterpret_cast<const float*>(ws + L.xsum_dn);
    a.k = I;
    a.n = H;
    const GemvPlan pl = plan_gemv(EPI_DOWN, (long long)L.max_items * (H / 128) * (I / 128), n_ctas);
    return launch_gemv<EPI_DOWN>(a, pl, st, "exl3_moe_down");
}

static int run_combine(int M, int topk, int E, int shared, int H, int I, void* out, int out_dtype, void* workspace,
                       size_t ws_bytes, cudaStream_t st) {
    EXL3_REQUIRE(out && M >= 0 && topk > 0 && E > 0 && H % 128 == 0 && I % 128 == 0, EXL3_ERR_ARG,
                 "exl3_moe_combine: bad arguments");
    EXL3_REQUIRE(out_dtype == EXL3_F16 || out_dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED, "exl3_moe_combine: out dtype");
    if (M == 0) return EXL3_OK;
    const WsLayout L = ws_layout(M, topk, E, H, I, shared, item_rows(M));
    int rc = ws_check(workspace, ws_bytes, L, "exl3_moe_combine");
    if (rc) return rc;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const float* ybuf = reinterpret_cast<const float*>(ws + L.ybuf);
    const int* pair_of = reinterpret_cast<const int*>(ws + L.pair_of);
    const int* wi = reinterpret_cast<const int*>(ws);
    const int n4 = M * (H / 4);
    const dim3 grid((n4 + 255) / 256);
    cudaError_t e;
    if (out_dtype == EXL3_F32)
        e = launch_pdl(k_combine<float>, grid, dim3(256), 0, st, ybuf, pair_of, wi, M, H, topk, shared,
                       static_cast<float*>(out));
    else
        e = launch_pdl(k_combine<__half>, grid, dim3(256), 0, st, ybuf, pair_of, wi, M, H, topk, shared,
                       static_cast<__half*>(out));
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_moe_combine: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

// ------------------------------------------------------------------------------------------------ prefill

// Workspace of exl3_moe_prefill: the alignment tables of ws_layout (items of <= kTcTileRows positions), then the
// rotated gate/up input rows [2][P][H] fp16, the gate/up outputs [2][P][I] fp16, the down projection's input rows
// [P][I] fp16 and the weighted rows [P][H] fp32.
struct PrefillLayout {
    WsLayout t;
    size_t a_gu, gu, a_dn, ybuf, total;
};
constexpr int kPrefillItemRows = kTcTileRows;
inline PrefillLayout prefill_layout(int M, int topk, int E, int H, int I, int shared) {
    PrefillLayout L;
    L.t = ws_layout(M, topk, E, H, I, shared, kPrefillItemRows);
    size_t o = L.t.xf_gu;
    L.a_gu = o; o += align_up((size_t)2 * L.t.p_max * H * 2, 256);
    L.gu = o; o += align_up((size_t)2 * L.t.p_max * I * 2, 256);
    L.a_dn = o; o += align_up((size_t)L.t.p_max * I * 2, 256);
    L.ybuf = o; o += (size_t)L.t.p_max * H * 4;
    L.total = o;
    return L;
}

}  // namespace exl3

using namespace exl3;

extern "C" {

size_t exl3_moe_prefill_workspace_size(int M, int topk, int E, int H, int I, int shared) {
    if (M <= 0 || topk <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
    return prefill_layout(M, topk, E, H, I, shared).total;
}

int exl3_moe_prefill(const void* x, int x_dtype, int ldx, int M, const int32_t* ids, const float* w, int topk,
                     const exl3_expert* experts, int E, int shared, int H, int I, float act_limit, void* out,
                     int out_dtype, void* workspace, size_t ws_bytes, void* stream) {
    int rc = moe_check(M, topk, experts, E, H, I, 0, "exl3_moe_prefill");
    if (rc) return rc;
    EXL3_REQUIRE(x && ids && w && out, EXL3_ERR_ARG, "exl3_moe_prefill: null pointer");
    EXL3_REQUIRE(x_dtype == EXL3_F16 || x_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "exl3_moe_prefill: x dtype");
    EXL3_REQUIRE(out_dtype == EXL3_F16 || out_dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED, "exl3_moe_prefill: out dtype");
    EXL3_REQUIRE(ldx >= H && ldx % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 7) == 0, EXL3_ERR_ARG,
                 "exl3_moe_prefill: x rows must be 8-byte aligned (ldx=%d)", ldx);
    if (M == 0) return EXL3_OK;
    const PrefillLayout L = prefill_layout(M, topk, E, H, I, shared);
    EXL3_REQUIRE(workspace && ws_bytes >= L.total && (reinterpret_cast<uintptr_t>(workspace) & 255) == 0,
                 EXL3_ERR_WORKSPACE, "exl3_moe_prefill: workspace %zu < %zu bytes (or not 256-byte aligned)",
                 ws_bytes, L.total);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    rc = launch_align(ids, w, M, topk, E, shared, kPrefillItemRows, ws, L.t, st);
    if (rc) return rc;
    TcMoeArgs m = {};
    m.x = x;
    m.ldx = ldx;
    m.x_bf16 = x_dtype == EXL3_BF16;
    m.H = H;
    m.I = I;
    m.P = L.t.p_max;
    m.max_items = L.t.max_items;
    m.n_items = reinterpret_cast<const int*>(ws);
    m.item_expert = reinterpret_cast<const int*>(ws + L.t.item_expert);
    m.item_start = reinterpret_cast<const int*>(ws + L.t.item_start);
    m.item_cnt = reinterpret_cast<const int*>(ws + L.t.item_cnt);
    m.n_pos = reinterpret_cast<const int*>(ws) + 2;
    m.pair_tok = reinterpret_cast<const int*>(ws + L.t.pair_tok);
    m.pair_expert = reinterpret_cast<const int*>(ws + L.t.pair_expert);
    m.pair_w = reinterpret_cast<const float*>(ws + L.t.pair_w);
    m.experts = reinterpret_cast<const ExpertDesc*>(experts);
    m.act_limit = act_limit;
    m.a_gu = reinterpret_cast<__half*>(ws + L.a_gu);
    m.gu = reinterpret_cast<__half*>(ws + L.gu);
    m.a_dn = reinterpret_cast<__half*>(ws + L.a_dn);
    m.ybuf = reinterpret_cast<float*>(ws + L.ybuf);
    rc = tc_moe_prefill(m, st);
    if (rc) return rc;
    const float* ybuf = m.ybuf;
    const int* pair_of = reinterpret_cast<const int*>(ws + L.t.pair_of);
    const int* wi = reinterpret_cast<const int*>(ws);
    const dim3 grid((M * (H / 4) + 255) / 256);
    cudaError_t e;
    if (out_dtype == EXL3_F32)
        e = launch_pdl(k_combine<float>, grid, dim3(256), 0, st, ybuf, pair_of, wi, M, H, topk, shared,
                       static_cast<float*>(out));
    else
        e = launch_pdl(k_combine<__half>, grid, dim3(256), 0, st, ybuf, pair_of, wi, M, H, topk, shared,
                       static_cast<__half*>(out));
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_moe_prefill: combine launch failed: %s",
                 cudaGetErrorString(e));
    return EXL3_OK;
}


int exl3_route(const float* logits, int ld, int R, int E, int kind, int k, const float* bias, const float* res,
               const float* mul, float scale, int renorm, void* ids, int ids64, float* w, void* want,
               void* stream) {
    EXL3_REQUIRE(logits && ids && w && R >= 0 && E > 0 && ld >= E, EXL3_ERR_ARG, "exl3_route: bad arguments");
    EXL3_REQUIRE(E <= kRouteMaxE, EXL3_ERR_UNSUPPORTED, "exl3_route: E=%d > %d", E, kRouteMaxE);
    EXL3_REQUIRE(k >= 1 && k <= kRouteMaxK && k <= E, EXL3_ERR_ARG, "exl3_route: k=%d", k);
    EXL3_REQUIRE(kind >= 0 && kind <= 2, EXL3_ERR_ARG, "exl3_route: kind=%d", kind);
    if (R == 0) return EXL3_OK;
    const RouteParams rp = {E, kind, k, bias, res, mul, scale, renorm, ids, ids64, w, want};
    const dim3 grid((R + kRouteWarps - 1) / kRouteWarps), block(kRouteWarps * 32);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e;
    switch (route_npl(E)) {
        case 4: e = launch_pdl(k_route<4>, grid, block, 0, st, logits, ld, R, rp); break;
        case 8: e = launch_pdl(k_route<8>, grid, block, 0, st, logits, ld, R, rp); break;
        case 16: e = launch_pdl(k_route<16>, grid, block, 0, st, logits, ld, R, rp); break;
        default: e = launch_pdl(k_route<32>, grid, block, 0, st, logits, ld, R, rp); break;
    }
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_route: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

size_t exl3_route_hidden_workspace_size(int R, int E) {
    if (R <= 0 || E <= 0) return 0;
    return 256 + align_up((size_t)R * E * 4, 256);
}

static int route_hidden_launch(const void* hidden, int h_dtype, int ldh, int R, int H, const void* gate_t,
                               const void* gate_t1, const RouteParams& rp, const RouteParams& rp1, void* logits_out,
                               void* workspace, size_t ws_bytes, void* stream, const char* what) {
    const int E = rp.E + (gate_t1 ? rp1.E : 0);
    EXL3_REQUIRE(hidden && gate_t && rp.ids && rp.w && R >= 0 && rp.E > 0 && H > 0 && H % 2 == 0 && ldh >= H,
                 EXL3_ERR_ARG, "%s: bad arguments", what);
    EXL3_REQUIRE(rp.E <= kRouteMaxE && (!gate_t1 || rp1.E <= kRouteMaxE), EXL3_ERR_UNSUPPORTED, "%s: E > %d", what,
                 kRouteMaxE);
    EXL3_REQUIRE(R <= kRhMaxRows, EXL3_ERR_UNSUPPORTED,
                 "%s: R=%d > %d rows (compute the logits with exl3_router_logits and call exl3_route)", what, R,
                 kRhMaxRows);
    EXL3_REQUIRE(rp.k >= 1 && rp.k <= kRouteMaxK && rp.k <= rp.E, EXL3_ERR_ARG, "%s: k=%d", what, rp.k);
    EXL3_REQUIRE(rp.kind >= 0 && rp.kind <= 2, EXL3_ERR_ARG, "%s: kind=%d", what, rp.kind);
    if (gate_t1) {
        EXL3_REQUIRE(rp1.ids && rp1.w && rp1.E > 0 && rp1.k >= 1 && rp1.k <= kRouteMaxK && rp1.k <= rp1.E &&
                         rp1.kind >= 0 && rp1.kind <= 2 && (reinterpret_cast<uintptr_t>(gate_t1) & 3) == 0,
                     EXL3_ERR_ARG, "%s: bad next-layer router arguments", what);
    }
    EXL3_REQUIRE(h_dtype == EXL3_F16 || h_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "%s: dtype %d", what, h_dtype);
    EXL3_REQUIRE((reinterpret_cast<uintptr_t>(gate_t) & 3) == 0, EXL3_ERR_ARG, "%s: gate_t must be 4-byte aligned",
                 what);
    if (R == 0) return EXL3_OK;
    EXL3_REQUIRE(workspace && ws_bytes >= exl3_route_hidden_workspace_size(R, E), EXL3_ERR_WORKSPACE,
                 "%s: workspace %zu < %zu bytes", what, ws_bytes, exl3_route_hidden_workspace_size(R, E));
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    unsigned int* ticket = reinterpret_cast<unsigned int*>(ws);
    float* lg = reinterpret_cast<float*>(ws + 256);
    const dim3 grid((E + kRhWarps - 1) / kRhWarps);
    cudaError_t e;
    if (h_dtype == EXL3_BF16)
        e = launch_pdl(k_route_hidden<__nv_bfloat16>, grid, dim3(kRhWarps * 32), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const __nv_bfloat16*>(hidden), ldh, R, H, static_cast<const __half*>(gate_t),
                       static_cast<const __half*>(gate_t1), lg, static_cast<__half*>(logits_out), ticket, rp, rp1);
    else
        e = launch_pdl(k_route_hidden<__half>, grid, dim3(kRhWarps * 32), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const __half*>(hidden), ldh, R, H, static_cast<const __half*>(gate_t),
                       static_cast<const __half*>(gate_t1), lg, static_cast<__half*>(logits_out), ticket, rp, rp1);
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_router_logits(const void* hidden, int h_dtype, int ldh, int R, int H, const void* gate_t, int E,
                       float* logits, void* logits_f16, void* stream) {
    EXL3_REQUIRE(hidden && gate_t && logits && R >= 0 && E > 0 && H > 0 && H % kRlK == 0 && ldh >= H && ldh % 8 == 0,
                 EXL3_ERR_ARG, "exl3_router_logits: bad arguments (H %% 32 == 0, ldh %% 8 == 0)");
    EXL3_REQUIRE(h_dtype == EXL3_F16 || h_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "exl3_router_logits: dtype %d",
                 h_dtype);
    EXL3_REQUIRE(aligned16(hidden) && aligned16(gate_t), EXL3_ERR_ARG,
                 "exl3_router_logits: hidden and gate_t must be 16-byte aligned");
    if (R == 0) return EXL3_OK;
    const dim3 grid((R + kRlTile - 1) / kRlTile, (E + kRlTile - 1) / kRlTile);
    cudaError_t e;
    if (h_dtype == EXL3_BF16)
        e = launch_pdl(k_router_logits<__nv_bfloat16>, grid, dim3(128), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const __nv_bfloat16*>(hidden), ldh, R, H, static_cast<const __half*>(gate_t), E,
                       logits, static_cast<__half*>(logits_f16));
    else
        e = launch_pdl(k_router_logits<__half>, grid, dim3(128), 0, static_cast<cudaStream_t>(stream),
                       static_cast<const __half*>(hidden), ldh, R, H, static_cast<const __half*>(gate_t), E, logits,
                       static_cast<__half*>(logits_f16));
    EXL3_REQUIRE(e == cudaSuccess, EXL3_ERR_CUDA, "exl3_router_logits: launch failed: %s", cudaGetErrorString(e));
    return EXL3_OK;
}

int exl3_route_hidden(const void* hidden, int h_dtype, int ldh, int R, int H, const void* gate_t, int E, int kind,
                      int k, const float* bias, const float* res, const float* mul, float scale, int renorm, void* ids,
                      int ids64, float* w, void* want, void* logits_out, void* workspace, size_t ws_bytes,
                      void* stream) {
    const RouteParams rp = {E, kind, k, bias, res, mul, scale, renorm, ids, ids64, w, want};
    const RouteParams none = {};
    return route_hidden_launch(hidden, h_dtype, ldh, R, H, gate_t, nullptr, rp, none, logits_out, workspace, ws_bytes,
                               stream, "exl3_route_hidden");
}

int exl3_route_hidden_pair(const void* hidden, int h_dtype, int ldh, int R, int H, const void* gate_t, int E,
                           int kind, int k, const float* bias, const float* res, const float* mul, float scale,
                           int renorm, void* ids, int ids64, float* w, void* want, void* logits_out,
                           const void* gate_t1, int E1, int kind1, int k1, const float* bias1, const float* mul1,
                           float scale1, int renorm1, void* ids1, int ids1_64, float* w1, void* workspace,
                           size_t ws_bytes, void* stream) {
    EXL3_REQUIRE(gate_t1, EXL3_ERR_ARG, "exl3_route_hidden_pair: gate_t1 is null");
    const RouteParams rp = {E, kind, k, bias, res, mul, scale, renorm, ids, ids64, w, want};
    const RouteParams rp1 = {E1, kind1, k1, bias1, nullptr, mul1, scale1, renorm1, ids1, ids1_64, w1, nullptr};
    return route_hidden_launch(hidden, h_dtype, ldh, R, H, gate_t, gate_t1, rp, rp1, logits_out, workspace, ws_bytes,
                               stream, "exl3_route_hidden_pair");
}

size_t exl3_moe_workspace_size(int M, int topk, int E, int H, int I, int shared) {
    if (M <= 0 || topk <= 0 || E <= 0 || H <= 0 || I <= 0) return 0;
    return ws_layout(M, topk, E, H, I, shared, item_rows(M)).total;
}

int exl3_moe_align(const int32_t* ids, const float* w, int M, int topk, int E, int shared, int chunk,
                   void* workspace, size_t ws_bytes, void* stream) {
    EXL3_REQUIRE(ids && w && M > 0 && topk > 0 && E > 0 && chunk > 0, EXL3_ERR_ARG, "exl3_moe_align: bad arguments");
    EXL3_REQUIRE(E <= 1024, EXL3_ERR_UNSUPPORTED, "exl3_moe_align: E=%d > 1024", E);
    const WsLayout L = ws_layout(M, topk, E, 128, 128, shared, chunk);
    EXL3_REQUIRE(workspace && ws_bytes >= L.xf_gu, EXL3_ERR_WORKSPACE, "exl3_moe_align: workspace %zu < %zu",
                 ws_bytes, L.xf_gu);
    return launch_align(ids, w, M, topk, E, shared, chunk, static_cast<uint8_t*>(workspace), L,
                        static_cast<cudaStream_t>(stream));
}

int exl3_moe_prepare(const void* x, int x_dtype, int ldx, int M, const int32_t* ids, const float* w, int topk,
                     const exl3_expert* experts, int E, int shared, int H, int I, void* workspace, size_t ws_bytes,
                     void* stream) {
    return run_prepare(x, x_dtype, ldx, M, ids, w, topk, experts, E, shared, H, I, workspace, ws_bytes,
                       static_cast<cudaStream_t>(stream));
}

int exl3_moe_gateup(int M, int topk, const exl3_expert* experts, int E, int shared, int H, int I, float act_limit,
                    void* workspace, size_t ws_bytes, int n_ctas, void* stream) {
    return run_gateup(M, topk, experts, E, shared, H, I, act_limit, workspace, ws_bytes, n_ctas,
                      static_cast<cudaStream_t>(stream));
}

int exl3_moe_down(int M, int topk, const exl3_expert* experts, int E, int shared, int H, int I, void* workspace,
                  size_t ws_bytes, int n_ctas, void* stream) {
    return run_down(M, topk, experts, E, shared, H, I, workspace, ws_bytes, n_ctas,
                    static_cast<cudaStream_t>(stream));
}

int exl3_moe_combine(int M, int topk, int E, int shared, int H, int I, void* out, int out_dtype, void* workspace,
                     size_t ws_bytes, void* stream) {
    return run_combine(M, topk, E, shared, H, I, out, out_dtype, workspace, ws_bytes,
                       static_cast<cudaStream_t>(stream));
}

int exl3_moe_decode(const void* x, int x_dtype, int ldx, int M, const int32_t* ids, const float* w, int topk,
                    const exl3_expert* experts, int E, int shared, int H, int I, float act_limit, void* out,
                    int out_dtype, void* workspace, size_t ws_bytes, int n_ctas, void* stream) {
    int rc = moe_check(M, topk, experts, E, H, I, n_ctas, "exl3_moe_decode");
    if (rc) return rc;
    EXL3_REQUIRE(out, EXL3_ERR_ARG, "exl3_moe_decode: null out");
    EXL3_REQUIRE(out_dtype == EXL3_F16 || out_dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED, "exl3_moe_decode: out dtype");
    if (M == 0) return EXL3_OK;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    rc = run_prepare(x, x_dtype, ldx, M, ids, w, topk, experts, E, shared, H, I, workspace, ws_bytes, st);
    if (rc) return rc;
    rc = run_gateup(M, topk, experts, E, shared, H, I, act_limit, workspace, ws_bytes, n_ctas, st);
    if (rc) return rc;
    rc = run_down(M, topk, experts, E, shared, H, I, workspace, ws_bytes, n_ctas, st);
    if (rc) return rc;
    return run_combine(M, topk, E, shared, H, I, out, out_dtype, workspace, ws_bytes, st);
}

}  // extern "C"
