// Host-side interface between the MoE orchestration (moe.cu) and the tcgen05 grouped expert projections
// (gemm_tc.cu).
#pragma once

#include "gemv.cuh"

namespace exl3 {

enum { TC_LINEAR = 0, TC_GATEUP = 1, TC_DOWN = 2 };

// Activation rows of one tensor-core tile (a pair of SMs): the MoE prefill groups each expert's positions into items
// of at most this many rows.
constexpr int kTcTileRows = 320;

// The MoE prefill path after alignment: rotated gate/up input rows of every pair position, the grouped gate and up
// projections on the tensor cores, SiLU * clamp + the down input's rotation, and the grouped down projection
// (x routing weight) on the tensor cores. Items hold at most kTcTileRows positions of one expert.
struct TcMoeArgs {
    const void* x;
    int ldx, x_bf16;
    int H, I;
    int P;                        // positions (pairs + shared rows): rows of a_gu / a_dn / ybuf
    int max_items;
    const int* n_items;
    const int* item_expert;
    const int* item_start;
    const int* item_cnt;
    const int* n_pos;             // positions in use
    const int* pair_tok;
    const int* pair_expert;
    const float* pair_w;
    const ExpertDesc* experts;
    float act_limit;
    __half* a_gu;                 // [2][P][H] fp16, rotated input rows (operand k order)
    __half* gu;                   // [2][P][I] fp16, gate and up outputs
    __half* a_dn;                 // [P][I] fp16, rotated down input rows (operand k order)
    float* ybuf;                  // [P][H] fp32
};

int tc_moe_prefill(const TcMoeArgs& m, cudaStream_t st);

}  // namespace exl3
