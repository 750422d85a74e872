// Dense EXL3 linear entry points: trellis dequantisation, blockwise Hadamard, the SiLU gate and the fused decode
// GEMV (exl3_gemv). Reference semantics are cited per entry in include/exl3_b200.h.
#include "gemv.cuh"

namespace exl3 {

// ------------------------------------------------------------------------------------------------ dequant

// Grid (k/16, ceil(n_slice/16 / 8)), 8 warps: warp w decodes tile (blockIdx.x, tile column n0/16 + 8*blockIdx.y + w)
// in registers, stages it in shared memory as a row-major 16x16 block and writes 16 rows of 16 fp16 (one 16-byte
// store per lane).
template <int K>
__global__ void __launch_bounds__(256) k_dequant(const uint32_t* __restrict__ tr, int TN, int n0t, int n_tiles,
                                                 __half* __restrict__ w, int ldw) {
    __shared__ __align__(16) __half tile_s[8][16][16 + 8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tk = blockIdx.x;
    const int tj = blockIdx.y * 8 + warp;             // tile column inside the slice
    if (tj >= n_tiles) return;
    const uint32_t* t = tr + ((size_t)tk * TN + n0t + tj) * (8 * K);
    const LaneWords lw = lane_words<K>(lane);
    uint32_t st[8];
    lane_states<K>(__ldg(t + lw.i0), __ldg(t + lw.i1), __ldg(t + lw.i2), lw.off, st);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const uint32_t h2 = mul1_pair(st[i], st[i + 1]);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int pos = 8 * lane + i + u;
            tile_s[warp][tile_row(pos)][tile_col(pos)] =
                __ushort_as_half(static_cast<unsigned short>((h2 >> (16 * u)) & 0xFFFFu));
        }
    }
    __syncwarp();
    const int r = lane >> 1, c = (lane & 1) * 8;
    uint4 v;
    v.x = *reinterpret_cast<const uint32_t*>(&tile_s[warp][r][c + 0]);
    v.y = *reinterpret_cast<const uint32_t*>(&tile_s[warp][r][c + 2]);
    v.z = *reinterpret_cast<const uint32_t*>(&tile_s[warp][r][c + 4]);
    v.w = *reinterpret_cast<const uint32_t*>(&tile_s[warp][r][c + 6]);
    *reinterpret_cast<uint4*>(w + (size_t)(tk * 16 + r) * ldw + tj * 16 + c) = v;
}

// ------------------------------------------------------------------------------------------------ Hadamard

// One warp per (row, 128-block). F16: pre product rounded to fp16, butterfly fp32, *r, round, post product rounded.
template <typename T>
__global__ void __launch_bounds__(256) k_had(const T* in, T* out, int rows, int cols, const __half* pre,
                                             const __half* post, float r) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    const int nb = cols / 128;
    if (warp >= rows * nb) return;
    const int row = warp / nb, b = warp % nb;
    const size_t base = (size_t)row * cols + b * 128 + 4 * lane;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float x = to_f32<T>(in[base + j]);
        if (pre) {
            x *= __half2float(pre[b * 128 + 4 * lane + j]);
            if constexpr (sizeof(T) == 2) x = __half2float(__float2half_rn(x));
        }
        v[j] = x;
    }
    fwht128_warp(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float y = v[j] * r;
        if constexpr (sizeof(T) == 2) {
            y = __half2float(__float2half_rn(y));
            if (!pre && post) y = __half2float(__float2half_rn(y * __half2float(post[b * 128 + 4 * lane + j])));
            out[base + j] = __float2half_rn(y);
        } else {
            if (!pre && post) y = y * __half2float(post[b * 128 + 4 * lane + j]);
            reinterpret_cast<float*>(out)[base + j] = y;
        }
    }
}

// ------------------------------------------------------------------------------------------------ activation

__global__ void k_silu_mul(const __half* g, const __half* u, __half* z, int64_t count, float L) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    const float gg = __half2float(g[i]);
    float uu = __half2float(u[i]);
    float s = gg / (1.0f + expf(-gg));
    if (L != 0.f) { s = fminf(s, L); uu = fminf(fmaxf(uu, -L), L); }
    z[i] = __float2half_rn(s * uu);
}

// ------------------------------------------------------------------------------------------------ packing

// exllamav3 [k/16][n/16][8K words] -> column-block-major [n/128][k/16][mats x 8 tiles][8K words]. The 8 tiles of one
// (tile-row, 128-column block) are contiguous on both sides, so the permutation moves whole chunks: one warp per
// destination chunk copies the chunk of every matrix (gate then up for a fused pair) with 16-byte loads.
__global__ void __launch_bounds__(256) k_pack(const uint4* __restrict__ a, const uint4* __restrict__ b, int R,
                                              int NB, int Ka, int Kb, uint4* __restrict__ out) {
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (warp >= R * NB) return;
    const int cb = warp / R, r = warp % R;
    const int ca = 16 * Ka, cbn = 16 * Kb;            // uint4 per chunk (8 tiles x 32K bytes / 16)
    uint4* dst = out + (size_t)warp * (ca + cbn);
    const uint4* sa = a + ((size_t)r * NB + cb) * ca;
    for (int i = lane; i < ca; i += 32) dst[i] = __ldg(sa + i);
    if (b) {
        const uint4* sb = b + ((size_t)r * NB + cb) * cbn;
        for (int i = lane; i < cbn; i += 32) dst[ca + i] = __ldg(sb + i);
    }
}

}  // namespace exl3

using namespace exl3;

extern "C" {

int exl3_pack(const void* trellis, int k, int n, int K, void* out, void* stream) {
    EXL3_REQUIRE(trellis && out && k > 0 && n > 0 && k % 16 == 0 && n % 128 == 0, EXL3_ERR_ARG,
                 "exl3_pack: k=%d must be a multiple of 16 and n=%d of 128", k, n);
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_UNSUPPORTED, "exl3_pack: K=%d not in 1..8", K);
    EXL3_REQUIRE(aligned16(trellis) && aligned16(out) && trellis != out, EXL3_ERR_ARG,
                 "exl3_pack: 16-byte aligned, non-overlapping buffers required");
    const int R = k / 16, NB = n / 128;
    const long warps = (long)R * NB;
    k_pack<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(trellis), nullptr, R, NB, K, 0, static_cast<uint4*>(out));
    EXL3_LAUNCH_CHECK("exl3_pack");
    return EXL3_OK;
}

int exl3_pack_gateup(const void* gate, const void* up, int H, int I, int Kg, int Ku, void* out, void* stream) {
    EXL3_REQUIRE(gate && up && out && H > 0 && I > 0 && H % 16 == 0 && I % 128 == 0, EXL3_ERR_ARG,
                 "exl3_pack_gateup: H=%d must be a multiple of 16 and I=%d of 128", H, I);
    EXL3_REQUIRE(Kg >= 1 && Kg <= 8 && Ku >= 1 && Ku <= 8, EXL3_ERR_UNSUPPORTED, "exl3_pack_gateup: K out of 1..8");
    EXL3_REQUIRE(aligned16(gate) && aligned16(up) && aligned16(out), EXL3_ERR_ARG,
                 "exl3_pack_gateup: 16-byte aligned buffers required");
    const int R = H / 16, NB = I / 128;
    const long warps = (long)R * NB;
    k_pack<<<(unsigned)((warps * 32 + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint4*>(gate), static_cast<const uint4*>(up), R, NB, Kg, Ku, static_cast<uint4*>(out));
    EXL3_LAUNCH_CHECK("exl3_pack_gateup");
    return EXL3_OK;
}

// Workspace of exl3_gemv: rotated input rows [M][k] fp16 | tickets [n/128] int32 | split-unit partial slots.
struct GemvWs {
    size_t xf, xsum, tickets, partial, total;
};
// rotated rows [M][k] fp16 | their block sums [M][k / 128] fp32 | tickets [n / 128] | split-unit partial slots
static GemvWs gemv_ws(int M, int k, int n) {
    GemvWs w;
    w.xf = 0;
    w.xsum = align_up((size_t)M * k * 2, 256);
    w.tickets = align_up(w.xsum + (size_t)M * (k / 128) * 4, 256);
    w.partial = align_up(w.tickets + (size_t)(n / 128) * 4, 256);
    w.total = w.partial + partial_bytes(EPI_LINEAR, M > kMaxRows ? 2 : 1);
    return w;
}

size_t exl3_gemv_workspace_size(int M, int k, int n) {
    if (M <= 0 || k <= 0 || n <= 0) return 0;
    return gemv_ws(M, k, n).total;
}

int exl3_dequant(const void* trellis, int k, int n, int K, int cb, int n0, int n_slice, void* w, int ldw,
                 void* stream) {
    EXL3_REQUIRE(cb == 2, EXL3_ERR_UNSUPPORTED, "exl3_dequant: only the mul1 codebook (cb=2) is supported");
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_UNSUPPORTED, "exl3_dequant: K=%d not in 1..8", K);
    EXL3_REQUIRE(trellis && w && k > 0 && n > 0 && k % 16 == 0 && n % 16 == 0, EXL3_ERR_ARG,
                 "exl3_dequant: bad shape k=%d n=%d", k, n);
    EXL3_REQUIRE(n0 >= 0 && n_slice > 0 && n0 % 16 == 0 && n_slice % 16 == 0 && n0 + n_slice <= n, EXL3_ERR_ARG,
                 "exl3_dequant: bad slice n0=%d n_slice=%d of n=%d", n0, n_slice, n);
    EXL3_REQUIRE(ldw >= n_slice && ldw % 8 == 0 && aligned16(w), EXL3_ERR_ARG,
                 "exl3_dequant: output needs 16-byte aligned rows (ldw=%d)", ldw);
    EXL3_REQUIRE(aligned16(trellis), EXL3_ERR_ARG, "exl3_dequant: trellis must be 16-byte aligned");
    const int n_tiles = n_slice / 16;
    dim3 grid(k / 16, (n_tiles + 7) / 8);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const uint32_t* tr = static_cast<const uint32_t*>(trellis);
    __half* wp = static_cast<__half*>(w);
    switch (K) {
        case 1: k_dequant<1><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
        case 2: k_dequant<2><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
        case 3: k_dequant<3><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
        case 4: k_dequant<4><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
        case 5: k_dequant<5><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
        case 6: k_dequant<6><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
        case 7: k_dequant<7><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
        default: k_dequant<8><<<grid, 256, 0, st>>>(tr, n / 16, n0 / 16, n_tiles, wp, ldw); break;
    }
    EXL3_LAUNCH_CHECK("exl3_dequant");
    return EXL3_OK;
}

int exl3_had_r_128(const void* in, void* out, int dtype, int rows, int cols, const void* pre, const void* post,
                   float scale, void* stream) {
    EXL3_REQUIRE(in && out && rows >= 0 && cols > 0 && cols % 128 == 0, EXL3_ERR_ARG,
                 "exl3_had_r_128: cols=%d must be a positive multiple of 128", cols);
    EXL3_REQUIRE(dtype == EXL3_F16 || dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED, "exl3_had_r_128: dtype %d", dtype);
    if (rows == 0) return EXL3_OK;
    const float r = static_cast<float>(static_cast<double>(scale) * 0.08838834764831845);
    const int64_t warps = (int64_t)rows * (cols / 128);
    const int blocks = (int)((warps * 32 + 255) / 256);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (dtype == EXL3_F16)
        k_had<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(in), static_cast<__half*>(out), rows, cols,
                                              static_cast<const __half*>(pre), static_cast<const __half*>(post), r);
    else
        k_had<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(in), static_cast<float*>(out), rows, cols,
                                             static_cast<const __half*>(pre), static_cast<const __half*>(post), r);
    EXL3_LAUNCH_CHECK("exl3_had_r_128");
    return EXL3_OK;
}

int exl3_silu_mul(const void* g, const void* u, void* z, int64_t count, float act_limit, void* stream) {
    EXL3_REQUIRE(g && u && z && count >= 0, EXL3_ERR_ARG, "exl3_silu_mul: bad arguments");
    if (count == 0) return EXL3_OK;
    k_silu_mul<<<(unsigned)((count + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __half*>(g), static_cast<const __half*>(u), static_cast<__half*>(z), count, act_limit);
    EXL3_LAUNCH_CHECK("exl3_silu_mul");
    return EXL3_OK;
}

int exl3_gemv(const void* x, int x_dtype, int ldx, int M, const void* packed, const void* suh, const void* svh,
              int k, int n, int K, int cb, void* y, int y_dtype, int ldy, void* workspace, size_t ws_bytes,
              int n_ctas, void* stream) {
    EXL3_REQUIRE(cb == 2, EXL3_ERR_UNSUPPORTED, "exl3_gemv: only the mul1 codebook (cb=2) is supported");
    EXL3_REQUIRE(K >= 1 && K <= 8, EXL3_ERR_UNSUPPORTED, "exl3_gemv: K=%d not in 1..8", K);
    EXL3_REQUIRE(M >= 0 && M <= kMaxRows * kMaxRowGroups, EXL3_ERR_ARG, "exl3_gemv: M=%d rows (1..16 per call)", M);
    EXL3_REQUIRE(k > 0 && n > 0 && k % 128 == 0 && n % 128 == 0, EXL3_ERR_ARG,
                 "exl3_gemv: k=%d, n=%d must be multiples of 128", k, n);
    EXL3_REQUIRE(x && packed && svh && y, EXL3_ERR_ARG, "exl3_gemv: null pointer");
    EXL3_REQUIRE(aligned16(packed), EXL3_ERR_ARG, "exl3_gemv: packed trellis must be 16-byte aligned");
    EXL3_REQUIRE(x_dtype == EXL3_F16 || x_dtype == EXL3_BF16, EXL3_ERR_UNSUPPORTED, "exl3_gemv: x dtype %d", x_dtype);
    EXL3_REQUIRE(y_dtype == EXL3_F16 || y_dtype == EXL3_BF16 || y_dtype == EXL3_F32, EXL3_ERR_UNSUPPORTED,
                 "exl3_gemv: y dtype %d", y_dtype);
    EXL3_REQUIRE(ldx >= k && ldy >= n && ldx % 4 == 0 && ldy % 4 == 0, EXL3_ERR_ARG,
                 "exl3_gemv: row strides ldx=%d ldy=%d", ldx, ldy);
    EXL3_REQUIRE((reinterpret_cast<uintptr_t>(x) & 7) == 0 && (reinterpret_cast<uintptr_t>(y) & 15) == 0,
                 EXL3_ERR_ARG, "exl3_gemv: x must be 8-byte and y 16-byte aligned");
    EXL3_REQUIRE(n_ctas >= 0, EXL3_ERR_ARG, "exl3_gemv: n_ctas=%d", n_ctas);
    if (M == 0) return EXL3_OK;
    const GemvWs W = gemv_ws(M, k, n);
    EXL3_REQUIRE(workspace && ws_bytes >= W.total && aligned16(workspace), EXL3_ERR_WORKSPACE,
                 "exl3_gemv: workspace %zu < %zu bytes (or not 16-byte aligned)", ws_bytes, W.total);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    __half* xf = reinterpret_cast<__half*>(ws + W.xf);
    int* tickets = reinterpret_cast<int*>(ws + W.tickets);

    PrepArgs pa = {};
    pa.x = x;
    pa.ldx = ldx;
    pa.x_bf16 = x_dtype == EXL3_BF16;
    pa.rows = M;
    pa.k = k;
    pa.suh = static_cast<const __half*>(suh);
    pa.xf = xf;
    pa.xsum = reinterpret_cast<float*>(ws + W.xsum);
    pa.zero = tickets;
    pa.n_zero = n / 128;
    int rc = launch_prep(pa, st, "exl3_gemv");
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
    a.xsum = reinterpret_cast<const float*>(ws + W.xsum);
    a.k = k;
    a.n = n;
    a.partial = reinterpret_cast<float*>(ws + W.partial);
    a.counters = tickets;
    a.status = device_status_ptr();
    if (M > kMaxRows) {                                       // 9..16 rows: two MMAs per decoded fragment
        const GemvPlan pl = plan_gemv(EPI_LINEAR, (long long)(n / 128) * (k / 128), n_ctas, 2);
        return launch_gemv<EPI_LINEAR, 2>(a, pl, st, "exl3_gemv");
    }
    const GemvPlan pl = plan_gemv(EPI_LINEAR, (long long)(n / 128) * (k / 128), n_ctas);
    return launch_gemv<EPI_LINEAR>(a, pl, st, "exl3_gemv");
}

}  // extern "C"
