"""ctypes binding of libtabinfer_b200.so (the C ABI in include/tabinfer_b200.h).

The library is loaded from this package directory (built in-tree by
tabinfer_b200/csrc/build.py).  There is no fallback: if the shared library is
missing or fails to load, importing this module raises.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtabinfer_b200.so")

P = ctypes.c_void_p
I64 = ctypes.c_int64
I32 = ctypes.c_int
F32 = ctypes.c_float

# name -> argtypes (restype int status unless noted)
SIGNATURES = {
    "tb_version": [],
    "tb_ctx_create": [I32, ctypes.POINTER(P)],
    "tb_ctx_destroy": [P],
    "tb_ctx_set_stream": [P, P],
    "tb_ctx_get_stream": [P],
    "tb_ctx_set_pdl": [P, I32],
    "tb_last_error": [P],
    "tb_ctx_synchronize": [P],
    "tb_ctx_device_error": [P, ctypes.POINTER(I32)],
    "tb_batch_begin": [P],
    "tb_batch_end": [P, ctypes.POINTER(P)],
    "tb_batch_submit": [P, P],
    "tb_batch_destroy": [P],
    "tb_copy_h2d": [P, P, P, ctypes.c_size_t],
    "tb_copy_d2h": [P, P, P, ctypes.c_size_t],
    "tb_attn_prefill_q8": [P, P, P, P, P, P, P, I64, I64, I64, I64, I64],
    "tb_logit_mask": [P, P, P, I64, I64],
    "tb_gumbel_noise": [P, P, I64, I64, ctypes.c_uint32, F32],
    "tb_sample_argmax": [P, P, I64, I64, P, ctypes.c_uint32, F32, P],
    "tb_bin_check": [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t],
    "tb_bin_open": [P, ctypes.c_char_p, ctypes.POINTER(P)],
    "tb_bin_close": [P],
    "tb_bin_blob_bytes": [P],
    "tb_bin_count": [P],
    "tb_bin_info": [P, I32, P],
    "tb_bin_find": [P, ctypes.c_char_p, P],
    "tb_quant_int4_g32": [P, P, P, P, I64, I64],
    "tb_quant_q8": [P, P, P, P, P, I64, I64],
    "tb_rmsnorm_q8": [P, P, P, F32, P, P, P, I64, I64],
    "tb_gemv_int4_q8": [P, P, P, P, P, P, I64, I64, I32, I32],
    "tb_gemv_int4_f32": [P, P, P, P, P, I64, I64, I32, I32],
    "tb_linear_int4": [P, P, P, P, P, I64, I64, I64, I32],
    "tb_gateup_silu_int4_q8": [P, P, P, P, P, P, P, P, I64, I64, I32],
    "tb_gemv_int4_q8_multi": [P, I32, P, P, P, P, P, P, I64, I32, I32],
    "tb_gemv_int4_dp4a": [P, P, P, P, F32, P, P, I64, I64, I32, I32],
    "tb_gemv_int4_dp4a_multi": [P, I32, P, P, P, P, P, P, F32, I64, I32, I32],
    "tb_gemv_int4_mma": [P, P, P, P, F32, P, P, I64, I64, I32, I32],
    "tb_gemv_int4_mma_multi": [P, I32, P, P, P, P, P, P, F32, I64, I32, I32],
    "tb_gateup_silu_int4_mma": [P, P, P, P, F32, P, P, P, P, I64, I64, I32],
    "tb_gemv_tern_wgsl_mma": [P, P, P, P, F32, P, P, I64, I64, I32, I32],
    "tb_gateup_silu_tern_wgsl_mma": [P, P, P, P, F32, P, P, P, P, I64, I64, I32],
    "tb_gateup_silu_int4_dp4a": [P, P, P, P, F32, P, P, P, P, I64, I64, I32],
    "tb_gemv_int4_f32_norm": [P, P, P, P, F32, P, P, I64, I64, I32, I32],
    "tb_pack_tern_q2g64": [P, P, P, P, I64, I64],
    "tb_quant_tern_wgsl_bf16": [P, P, P, P, I64, I64, P],
    "tb_gemv_tern_wgsl_q8": [P, P, P, P, P, P, I64, I64, I32, I32],
    "tb_gemv_tern_wgsl_dp4a_multi": [P, I32, P, P, P, P, P, P, F32, I64, I32, I32],
    "tb_gateup_silu_tern_wgsl_q8": [P, P, P, P, P, P, P, P, I64, I64, I32],
    "tb_gateup_silu_tern_wgsl_dp4a": [P, P, P, P, F32, P, P, P, P, I64, I64, I32],
    "tb_gemm_tern_wgsl": [P, P, P, P, P, P, I64, I64, I64, I32],
    "tb_gemm_int4_q8": [P, P, P, P, P, P, I64, I64, I64, I32],
    "tb_gemm_dp4": [P, P, P, P, P, P, I64, I64, I64, I32, I32],
    "tb_gemm_dp4_warp": [P, P, P, P, P, P, I64, I64, I64, I32, I32],
    "tb_linear_tern_wgsl": [P, P, P, P, P, I64, I64, I64, I32],
    "tb_quant_act_q8": [P, P, P, P, P, I64, I64],
    "tb_quantize_wasm": [P, P, P, P, I64, P, I64],
    "tb_gemv_tern_q2g64": [P, P, P, P, P, P, I64, I64, I32],
    "tb_linear_tern": [P, P, P, P, P, I64, I64, I64],
    "tb_attn_prep_q8": [P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, F32, F32],
    "tb_kv_quant_write": [P, P, P, P, P, P, P, I64, I64, I64, I64],
    "tb_attn_decode_q8": [P, P, P, P, P, P, P, I64, I64, I64, I64, I32],
    "tb_attn_decode_q8_noalloc": [P, P, P, P, P, P, P, I64, I64, I64, I64, I32],
    "tb_argmax": [P, P, I64, I64, P, I64],
    "tb_rmsnorm": [P, P, P, P, I64, I64, F32],
    "tb_embed_gather": [P, P, I64, P, P, I64, I64],
    "tb_attn_prep_q8_batch": [P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, P, F32, F32],
    "tb_attn_decode_q8_batch": [P, P, P, P, P, P, P, I64, I64, P, I64, I64, I64, I64, I32],
    "tb_convert_bf16_f16": [P, P, P, I64],
    "tb_gemm_int4_g32": [P, P, P, I32, P, P, I64, I64, I64, I32],
    "tb_requant_int4_int3": [P, P, P, P, P, I64, I64],
    "tb_moe_router": [P, P, P, P, P, I64, I64, I64],
    "tb_moe_ffn_int3": [P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64],
    "tb_moe_ffn_int3_g": [P, P, P, P, P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I32],
    "tb_quant_int3_bf16": [P, P, P, P, I64, I64, I32],
    "tb_moe_ep_create": [P, ctypes.c_int, ctypes.c_int, I64, I64, I64, I64, I64, P],
    "tb_moe_ep_destroy": [P],
    "tb_moe_ep_handle": [P, P],
    "tb_moe_ep_connect": [P, P],
    "tb_moe_ep_set_experts": [P, P, P, P, P, P, P],
    "tb_moe_ep_forward": [P, P, P, P, P, I64],
    "tb_qwen3_shard": [P, I32, ctypes.POINTER(I64), ctypes.POINTER(I64), ctypes.POINTER(I64), ctypes.POINTER(I64)],
    "tb_qwen3_create": [P, P, ctypes.POINTER(P)],
    "tb_qwen3_destroy": [P],
    "tb_qwen3_set_weight": [P, I32, I32, P, I64, I64],
    "tb_qwen3_set_weight_q": [P, I32, I32, I32, P, P, I64, I64],
    "tb_qwen3_prefill": [P, I32, P, I64, I64],
    "tb_qwen3_weight_format": [P, I32, I32],
    "tb_qwen3_kv": [P, I32, ctypes.POINTER(P), ctypes.POINTER(P), ctypes.POINTER(P), ctypes.POINTER(P)],
    "tb_qwen3_io": [P, ctypes.POINTER(P), ctypes.POINTER(P), ctypes.POINTER(P)],
    "tb_nccl_unique_id": [P],
    "tb_qwen3_tp_init": [P, P],
    "tb_qwen3_set_step_mode": [P, ctypes.c_int],
    "tb_qwen3_step_kind": [P],
    "tb_qwen3_step_layers": [P],
    "tb_qwen3_step_trace": [P, P],
    "tb_qwen3_tp_handle": [P, P],
    "tb_qwen3_tp_connect": [P, P],
    "tb_qwen3_tp_reset": [P],
    "tb_qwen3_decode_step": [P],
    "tb_qwen3_launches_per_step": [P, ctypes.POINTER(I32), ctypes.POINTER(I32)],
}


class Qwen3Config(ctypes.Structure):
    """tb_qwen3_config (include/tabinfer_b200.h)."""
    _fields_ = [("hidden", ctypes.c_int32), ("layers", ctypes.c_int32), ("n_heads", ctypes.c_int32),
                ("n_kv_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32), ("intermediate", ctypes.c_int32),
                ("vocab", ctypes.c_int32), ("rope_theta", ctypes.c_float), ("rms_eps", ctypes.c_float),
                ("max_seq", ctypes.c_int32), ("batch", ctypes.c_int32), ("tp_size", ctypes.c_int32),
                ("tp_rank", ctypes.c_int32), ("ternary", ctypes.c_int32)]


# weight kinds (TB_QW_*)
QW_EMBED, QW_LM_HEAD, QW_FINAL_NORM, QW_Q, QW_K, QW_V, QW_O, QW_GATE, QW_UP, QW_DOWN, \
    QW_LN_ATTN, QW_LN_MLP, QW_Q_NORM, QW_K_NORM = range(14)
# formats of pre-quantized weights (TB_QW_FMT_*)
QW_FMT_INT4, QW_FMT_TERN, QW_FMT_F16 = 0, 1, 2
# how the decode step runs (TB_QW_STEP_*)
QW_STEP_AUTO, QW_STEP_KERNELS, QW_STEP_PERSISTENT = 0, 1, 2
RESTYPES = {
    "tb_bin_blob_bytes": I64,
    "tb_last_error": ctypes.c_char_p,
    "tb_ctx_get_stream": P,
    "tb_moe_ep_destroy": None,
}


class BinTensor(ctypes.Structure):
    """tb_bin_tensor (include/tabinfer_b200.h)"""
    _fields_ = [("name", ctypes.c_char_p), ("kind", ctypes.c_int), ("N", I64), ("K", I64), ("ndim", ctypes.c_int),
                ("shape", I64 * 4), ("data", P), ("bytes", I64), ("scales", P), ("scales_bytes", I64),
                ("blob_offset", I64)]


BIN_TERN, BIN_EMBED_F16, BIN_F32 = 0, 1, 2


def load(path=LIB_PATH):
    if not os.path.exists(path):
        raise ImportError(
            "libtabinfer_b200.so not found at %s; build it with "
            "`python -c 'import __graft_entry__ as g; g.build()'` (nvcc, sm_100a)" % path)
    lib = ctypes.CDLL(path)
    for name, args in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = RESTYPES.get(name, ctypes.c_int)
    return lib


def header_symbols(header=None):
    """Function names declared TB_API in include/*.h."""
    import re
    inc = os.path.join(os.path.dirname(HERE), "include")
    names = []
    for fn in sorted(os.listdir(inc)):
        if fn.endswith(".h"):
            txt = open(os.path.join(inc, fn)).read()
            names += re.findall(r"TB_API\s+[\w\s\*]+?\b(tb_\w+)\s*\(", txt)
    return names


LIB = load()
