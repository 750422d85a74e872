"""B200-native EXL3 trellis path: dequant-fused GEMV / grouped MoE linears and the routed-expert top-k with
residency bias, behind the reference's BC_LinearEXL3 / BlockSparseMLP API. CUDA kernels live in ../csrc and are
reached through the C ABI of libexl3_b200.so (include/exl3_b200.h)."""
from . import _lib, torch_ops
from .exllama_patch import install
from .ops import (BC_GatedMLP, BC_LinearEXL3, det_quant_weight, exl3_gemm, exl3_gemv, exl3_reconstruct, had_r_128,
                  reconstruct, reconstruct_slice, route, routing_ds3_nogroup, silu_mul)
from .moe import (BlockSparseMLP, Expert, ExpertTable, Exl3Matrix, ROUTE_SIGMOID, ROUTE_SOFTMAX, ROUTE_SQRT_SOFTPLUS,
                  moe_align, moe_forward)

__all__ = ["BC_GatedMLP", "BC_LinearEXL3", "BlockSparseMLP", "Expert", "ExpertTable", "Exl3Matrix", "ROUTE_SIGMOID",
           "ROUTE_SOFTMAX", "ROUTE_SQRT_SOFTPLUS", "det_quant_weight", "exl3_gemm", "exl3_gemv", "exl3_reconstruct",
           "had_r_128", "moe_align", "moe_forward", "reconstruct", "reconstruct_slice", "route", "routing_ds3_nogroup",
           "silu_mul", "_lib", "install", "torch_ops"]
