// EXL3 trellis tile format and the mul1 codebook, decoded in registers.
//
// A 16x16 tile of K-bit weights is a ring of 256*K bits stored as 8*K little-endian uint32 words, read MSB-first
// (bit b is bit 31 - b%32 of word b/32). Ring position t (0..255) owns the 16-bit window of stream bits
// [(t+1)K - 16, (t+1)K), circular inside the tile, and lands on tile row (input dim) 8((t>>1)&1) + 2((t>>3)&3) +
// (t&1), column (output dim) (t>>5) + 8((t>>2)&1) (reference: glm/xpu/csrc/exl3_esimd.h:4-8,117-149;
// glm/docs/ext-op-inventory.md:698-733).
//
// That position order is the register layout of an m16n8k16 MMA A fragment for A = W^T (rows = output columns):
// lane l = 4g + q owns positions 8l .. 8l+7, i.e. (n = g, g+8) x (k = 2q, 2q+1, 2q+8, 2q+9). Positions 8l..8l+7
// are K*8 consecutive stream bits, so each lane decodes its own fragment from at most three words.
//
// mul1 codebook (glm/docs/ext-op-inventory.md:559-574): x = state * 0x83DCD12D (mod 2^32);
// h = fp16 bits (0x6400 + bytesum(x)) = 1024 + bytesum exactly; w = fma(h, 0x1EEE, 0xC931) in fp16 (one rounding).
#pragma once

#include "common.cuh"

namespace exl3 {

// Per-lane constants of the fragment decode for bit width K: which three tile words hold the lane's bits and the
// left shift that puts the first window's MSB at bit 63 of the (hi:lo) pair.
struct LaneWords {
    uint32_t i0, i1, i2;   // word indices inside the tile (mod 8K)
    uint32_t off;          // bit offset of the first window inside word i0
};

template <int K>
__device__ __forceinline__ LaneWords lane_words(int lane) {
    constexpr int RING = 256 * K;
    constexpr int W = 8 * K;
    int b = (8 * lane + 1) * K - 16;        // first bit of position 8*lane's window
    b = (b + RING) % RING;
    int w0 = b >> 5;
    LaneWords lw;
    lw.i0 = w0;
    lw.i1 = (w0 + 1) % W;
    lw.i2 = (w0 + 2) % W;
    lw.off = b & 31;
    return lw;
}

// The eight 16-bit states of the lane's positions, from the three words (w0, w1, w2) = words i0, i1, i2.
template <int K>
__device__ __forceinline__ void lane_states(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t off, uint32_t st[8]) {
    // hi:mid = stream bits [b, b + 64) of the lane, MSB first; lo3 = bits [b + 64, b + 96) (only K >= 7 needs it)
    const uint32_t hi = __funnelshift_l(w1, w0, off);
    const uint32_t mid = __funnelshift_l(w2, w1, off);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int s = 48 - i * K;   // right shift of the 64-bit (hi:mid) that aligns window i at bit 0
        uint32_t v;
        if (s >= 32 && (K % 2 == 0) && s - 32 < 16) {
            // even K: the windows inside hi sit at few bit offsets mod 8; shift once per offset (the shifted copies
            // are shared between windows) and take the window's two bytes with a zero-filling byte permute
            const int r = s - 32, sh = r & 7, b = (r - sh) >> 3;
            v = __byte_perm(sh ? hi >> sh : hi, 0u, (uint32_t)(b | ((b + 1) << 4) | 0x4400));
        } else if (s >= 32) {
            // window at bit r = s - 32 of hi: shifted up against bit 31 (a constant left shift, which issues on its
            // own pipe), then down by 16 (one ALU op instead of a shift and a mask)
            v = (s - 32 == 16) ? (hi >> 16) : ((hi << (48 - s)) >> 16);
        } else if (s >= 16) {
            v = __funnelshift_r(mid, hi, s) & 0xFFFFu;
        } else if (s >= 0) {
            v = (mid << (16 - s)) >> 16;
        } else {
            const uint32_t lo3 = w2 << off;                  // bits [b + 64, b + 96) (only the top ones are used)
            v = __funnelshift_r(lo3, mid, s + 32) & 0xFFFFu;
        }
        st[i] = v;
    }
}

// mul1 codebook for two states -> half2 {w(a), w(b)}, bit-exact with the reference decode.
__device__ __forceinline__ uint32_t mul1_pair(uint32_t sa, uint32_t sb) {
    const uint32_t xa = sa * kMul1;
    const uint32_t xb = sb * kMul1;
    const uint32_t ha = __dp4a(xa, 0x01010101u, 0x6400u);   // fp16 bits of 1024 + bytesum (< 2048: exact)
    const uint32_t hb = __dp4a(xb, 0x01010101u, 0x6400u);
    // {lo: ha, hi: hb}: both < 2^16, so a shift-and-add (off the ALU pipe) packs them
    const uint32_t h2 = ha + (hb << 16);
    uint32_t r;
    // fma in fp16x2 with the fp16 constants 0x1EEE (0.00676727294921875) and 0xC931 (-10.3828125): single rounding
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(h2), "r"(0x1EEE1EEEu), "r"(0xC931C931u));
    return r;
}

__device__ __forceinline__ __half mul1_one(uint32_t s) {
    uint32_t r = mul1_pair(s, s);
    return __ushort_as_half(static_cast<unsigned short>(r & 0xFFFFu));
}

// The codebook without its affine ("fold" form, the reference's decode_mul1_raw, glm/xpu/csrc/exl3_esimd.h:82-91):
// h = fp16 bits of 1024 + bytesum(state * 0x83DCD12D), exact in fp16, for two states packed as half2. The affine
// w = fp16(h * c1 + c2) is then applied to the dot product instead of to every weight:
//   sum_k a_k * (h_k * c1 + c2) = c1 * sum_k a_k h_k + c2 * sum_k a_k,
// i.e. the product uses the unrounded w' = h c1 + c2 (|w' - w| <= half an fp16 ulp of w) and needs the sum of the
// activations, which the kernels that rotate the activations provide per 128-block. Saves the fp16 FMA per pair.
constexpr float kMul1C1 = 0.00676727294921875f;     // fp16 0x1EEE
constexpr float kMul1C2 = -10.3828125f;             // fp16 0xC931
__device__ __forceinline__ uint32_t mul1_raw_pair(uint32_t sa, uint32_t sb) {
    const uint32_t ha = __dp4a(sa * kMul1, 0x01010101u, 0x6400u);
    const uint32_t hb = __dp4a(sb * kMul1, 0x01010101u, 0x6400u);
    return ha + (hb << 16);
}

// Decode the lane's A fragment (4 x half2) of one tile from its three words (tile words lw.i0, lw.i1, lw.i2).
// Register order follows the m16n8k16 A layout: {pos0,pos1} {pos4,pos5} {pos2,pos3} {pos6,pos7}.
template <int K>
__device__ __forceinline__ void decode_frag_words(uint32_t w0, uint32_t w1, uint32_t w2, uint32_t off, uint32_t a[4]) {
    uint32_t st[8];
    lane_states<K>(w0, w1, w2, off, st);
    a[0] = mul1_pair(st[0], st[1]);
    a[1] = mul1_pair(st[4], st[5]);
    a[2] = mul1_pair(st[2], st[3]);
    a[3] = mul1_pair(st[6], st[7]);
}

// The same fragment in the fold form: h values (1024 + bytesum) instead of weights.
template <int K>
__device__ __forceinline__ void decode_frag_raw(const uint32_t* tile, const LaneWords& lw, uint32_t a[4]) {
    uint32_t st[8];
    lane_states<K>(tile[lw.i0], tile[lw.i1], tile[lw.i2], lw.off, st);
    a[0] = mul1_raw_pair(st[0], st[1]);
    a[1] = mul1_raw_pair(st[4], st[5]);
    a[2] = mul1_raw_pair(st[2], st[3]);
    a[3] = mul1_raw_pair(st[6], st[7]);
}

// Decode the lane's A fragment of one tile whose words start at `tile` (shared or global memory).
template <int K>
__device__ __forceinline__ void decode_frag(const uint32_t* tile, const LaneWords& lw, uint32_t a[4]) {
    decode_frag_words<K>(tile[lw.i0], tile[lw.i1], tile[lw.i2], lw.off, a);
}

// D[16x8] += A[16x16] * B[16x8], fp16 inputs, fp32 accumulators.
__device__ __forceinline__ void mma_16816(float d[4], const uint32_t a[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};\n"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Position t -> (row k, col n) inside a tile.
__host__ __device__ __forceinline__ int tile_row(int t) { return 8 * ((t >> 1) & 1) + 2 * ((t >> 3) & 3) + (t & 1); }
__host__ __device__ __forceinline__ int tile_col(int t) { return (t >> 5) + 8 * ((t >> 2) & 1); }

}  // namespace exl3
