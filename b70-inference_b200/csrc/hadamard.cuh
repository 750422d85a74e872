// 128-point Walsh-Hadamard transform (natural Sylvester order) across one warp: lane l holds v[4l .. 4l+3].
// Stages run h = 1, 2, 4, ..., 64, each (a, b) -> (a + b, a - b) in fp32, the order of the reference's
// fwht128 (glm/xpu/csrc/exl3_esimd.h:210-221) and exllamav3's had_r_128 (4-point in registers, then xor
// shuffles; glm/docs/ext-op-inventory.md:576-595). Same stage order => the same fp32 roundings as the CPU oracle.
#pragma once

#include "common.cuh"

namespace exl3 {

__device__ __forceinline__ void fwht128_warp(float v[4], int lane) {
    // h = 1, 2 inside the lane
    float a0 = v[0] + v[1], a1 = v[0] - v[1], a2 = v[2] + v[3], a3 = v[2] - v[3];
    v[0] = a0 + a2;
    v[1] = a1 + a3;
    v[2] = a0 - a2;
    v[3] = a1 - a3;
    // h = 4 .. 64 across lanes: partner = lane ^ (h / 4). The butterfly is one fma with a +-1 factor:
    // fma(v, -1, p) = p - v and fma(v, 1, p) = v + p, each rounded once, as the subtraction / addition.
#pragma unroll
    for (int m = 1; m < 32; m <<= 1) {
        const float sgn = (lane & m) ? -1.0f : 1.0f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float p = __shfl_xor_sync(0xFFFFFFFFu, v[j], m);
            v[j] = fmaf(v[j], sgn, p);
        }
    }
}

// xh[0..127] = fp16( FWHT( fp16(x * suh) ) / sqrt(128) ) for one 128-block; x/suh/xh are this lane's 4 elements.
template <typename TIn>
__device__ __forceinline__ void had_in_block(const TIn* x, const __half* suh, __half* xh, int lane) {
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float p = to_f32<TIn>(x[4 * lane + j]) * (suh ? __half2float(suh[4 * lane + j]) : 1.0f);
        v[j] = __half2float(__float2half_rn(p));
    }
    fwht128_warp(v, lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) xh[4 * lane + j] = __float2half_rn(v[j] * kRsqrt128);
}

}  // namespace exl3
