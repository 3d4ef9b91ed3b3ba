"""tabinfer_b200 -- B200 backend for TabInfer's quantized-GEMV hot path.

The product is libtabinfer_b200.so (hand-written sm_100a CUDA behind the C ABI
in include/tabinfer_b200.h).  This package is the host-side mirror of the
reference's operator interface for that path (models/qwen3.js linearQ /
gemvQ / gemvDP4A / rmsnormQ / gateUpSiluDP4 / attnPrepQ8 / attentionQ8 /
argmaxKernel, the ternary WebGPU layout quantizeTernaryBf16 / gemvTern /
gateupTern, and native/crates/n2-kernels tern::{pack_ternary,
quantize_act, gemv_tern}), taking torch CUDA tensors as device buffers.
Errors raise TabInferError, as the reference throws.
"""
from .ops import (  # noqa: F401
    TabInferError, Context, default_context,
    quantize_int4_bf16, convert_bf16_f16, quant_q8, rmsnorm_q8, gemv_q, gemv_dp4, gemv_dp4_multi, linear_q,
    gemv_dp4a, gemv_dp4a_multi, gate_up_silu_dp4a, gemv_mma, gemv_mma_multi, gate_up_silu_mma, gemv_q_norm, gemm_q,
    requant_int3, quant_int3, moe_router, moe_ffn_int3,
    gate_up_silu_dp4, pack_ternary, quantize_act, quantize_wasm, gemv_tern, linear_tern,
    quantize_tern_bf16, gemv_tern_wgsl, gemv_tern_wgsl_dp4a_multi, gate_up_silu_tern, gate_up_silu_tern_dp4a,
    gemm_tern, gemm_dp4, gemm_dp4_f16, linear_tern_wgsl,
    attn_prep_q8, kv_quant_write, attention_decode_q8, attention_prefill_q8, argmax,
    logit_mask, gumbel_noise, sample_argmax, GumbelSeeds, rmsnorm, embed_gather,
)
from .qwen3 import Qwen3, QWEN3_1_7B, QWEN3_0_6B  # noqa: F401,E402
from .moe_ep import MoeEP  # noqa: F401,E402
