"""ctypes bindings of include/ammon_b200.h (libammon_b200.so).

The library is loaded from this package directory; there is no fallback. Importing
this module does not touch a GPU: only calls do.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libammon_b200.so")

AB_OK = 0
AB_ERR_VALIDATION = 1
AB_ERR_CUDA = 2
AB_ERR_ARGUMENT = 3
AB_ERR_DEVICE = 4
AB_ERR_NCCL = 5

AB_F32, AB_BF16, AB_U32 = 0, 1, 2


class Tensor_t(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int32), ("rank", C.c_int32),
                ("dims", C.c_uint32 * 4)]


class DecodeStep_t(C.Structure):
    _fields_ = [("token", C.c_uint32), ("position", C.c_uint32)]


class AttentionWeights_t(C.Structure):
    _fields_ = [("norm", Tensor_t), ("query", Tensor_t), ("key", Tensor_t), ("value", Tensor_t),
                ("output", Tensor_t)]


class SwigluWeights_t(C.Structure):
    _fields_ = [("norm", Tensor_t), ("gate", Tensor_t), ("up", Tensor_t), ("down", Tensor_t)]


class LlamaConfig_t(C.Structure):
    _fields_ = [("dim", C.c_uint32), ("layers", C.c_uint32), ("heads", C.c_uint32),
                ("kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("hidden", C.c_uint32),
                ("vocab", C.c_uint32), ("seq", C.c_uint32), ("batch", C.c_uint32),
                ("rope_theta", C.c_float), ("norm_eps", C.c_float), ("dtype", C.c_int32)]


VOCAB_FN = C.CFUNCTYPE(C.c_uint32, C.c_void_p)
SEQ_FN = C.CFUNCTYPE(C.c_uint32, C.c_void_p)
STEP_FN = C.CFUNCTYPE(C.c_int, C.c_void_p, C.c_uint32, C.c_uint32,
                      C.POINTER(C.POINTER(C.c_float)))


class Model_t(C.Structure):
    _fields_ = [("self", C.c_void_p), ("vocab_size", VOCAB_FN), ("max_seq_len", SEQ_FN),
                ("step", STEP_FN)]


P = C.c_void_p
PP = C.POINTER(C.c_void_p)
T = Tensor_t
u32, i32, u64, f32 = C.c_uint32, C.c_int32, C.c_uint64, C.c_float

SIGNATURES = {
    "ab_last_error": (C.c_char_p, []),
    "ab_runtime_create": (C.c_int, [i32, PP]),
    "ab_runtime_destroy": (C.c_int, [P]),
    "ab_runtime_synchronize": (C.c_int, [P]),
    "ab_runtime_stream": (P, [P]),
    "ab_runtime_sm_count": (C.c_int, [P, C.POINTER(i32)]),
    "ab_runtime_set_wait_limit": (C.c_int, [P, u32]),
    "ab_host_register": (C.c_int, [P, u64]),
    "ab_host_unregister": (C.c_int, [P]),
    "ab_runtime_wait_limit": (C.c_int, [P, C.POINTER(u32)]),
    "ab_tensor_zeros": (C.c_int, [P, i32, i32, C.POINTER(u32), C.POINTER(T)]),
    "ab_tensor_free": (C.c_int, [P, C.POINTER(T)]),
    "ab_tensor_write": (C.c_int, [P, T, P, u64]),
    "ab_tensor_read": (C.c_int, [P, T, P, u64]),
    "ab_tensor_fill_normal": (C.c_int, [P, T, u64, u64, f32, f32]),
    "ab_tensor_narrow": (C.c_int, [T, u32, u32, C.POINTER(T)]),
    "ab_tensor_reshape": (C.c_int, [T, i32, C.POINTER(u32), C.POINTER(T)]),
    "ab_step_parcel": (C.c_int, [P, u32, C.POINTER(T)]),
    "ab_step_deposit": (C.c_int, [P, T, C.POINTER(DecodeStep_t), u32]),
    "ab_scheme_create": (C.c_int, [P, PP]),
    "ab_scheme_destroy": (C.c_int, [P]),
    "ab_scheme_submit": (C.c_int, [P]),
    "ab_scheme_node_count": (C.c_int, [P, C.POINTER(u32)]),
    "ab_scheme_replay_stats": (C.c_int, [P, C.POINTER(u32), C.POINTER(u32)]),
    "ab_scheme_use_graph": (C.c_int, [P, i32]),
    "ab_scheme_time_nodes": (C.c_int, [P, u32, C.POINTER(f32), u32]),
    "ab_scheme_node_label": (C.c_int, [P, u32, C.c_char_p, u32]),
    "ab_kernel_embed": (C.c_int, [P, T, T, T]),
    "ab_kernel_gemv": (C.c_int, [P, T, T, T, T]),
    "ab_kernel_rmsnorm": (C.c_int, [P, T, T, T]),
    "ab_kernel_rmsnorm_inplace": (C.c_int, [P, T, T]),
    "ab_kernel_rope": (C.c_int, [P, T, T, T, f32]),
    "ab_kernel_rope_store": (C.c_int, [P, T, T, T, T, f32]),
    "ab_kernel_cache_store": (C.c_int, [P, T, T, T]),
    "ab_kernel_attention_partial": (C.c_int, [P, T, T, T, T, T]),
    "ab_kernel_attention_combine": (C.c_int, [P, T, T, T]),
    "ab_kernel_attention": (C.c_int, [P, T, T, T, T, T, T]),
    "ab_kernel_attention_decode": (C.c_int, [P, T, T, T, T, T]),
    "ab_kernel_swiglu": (C.c_int, [P, T, T]),
    "ab_tensor_add_into": (C.c_int, [P, T, T, T]),
    "ab_tensor_matmul_into": (C.c_int, [P, T, T, T]),
    "ab_embedding_record": (C.c_int, [P, T, T, T]),
    "ab_rmsnorm_record": (C.c_int, [P, T, T, T]),
    "ab_rmsnorm_record_inplace": (C.c_int, [P, T, T]),
    "ab_linear_record": (C.c_int, [P, T, T, T]),
    "ab_kvcache_create": (C.c_int, [P, u32, u32, u32, u32, i32, u32, PP]),
    "ab_kvcache_layer": (C.c_int, [P, u32, C.POINTER(T), C.POINTER(T)]),
    "ab_kvcache_zero": (C.c_int, [P]),
    "ab_kvcache_destroy": (C.c_int, [P]),
    "ab_attention_block_create": (C.c_int, [P, u32, u32, u32, u32, f32, PP]),
    "ab_attention_block_record": (C.c_int, [P, P, T, C.POINTER(AttentionWeights_t), T, T, T]),
    "ab_attention_block_destroy": (C.c_int, [P]),
    "ab_swiglu_block_create": (C.c_int, [P, u32, u32, u32, PP]),
    "ab_swiglu_block_record": (C.c_int, [P, P, T, C.POINTER(SwigluWeights_t)]),
    "ab_swiglu_block_destroy": (C.c_int, [P]),
    "ab_attention_decode_noalloc": (C.c_int, [P, T, T, T, T, T]),
    "ab_attention_decode_noalloc_status": (C.c_int, [P, C.POINTER(u32)]),
    "ab_sample_argmax": (i32, [C.POINTER(f32), u32]),
    "ab_generate_tokens": (C.c_int, [C.POINTER(Model_t), C.POINTER(i32), u32, u32, i32, i32,
                                     C.POINTER(i32), u32, C.POINTER(u32), C.POINTER(C.c_double)]),
    "ab_bpe_from_path": (C.c_int, [C.c_char_p, u32, PP]),
    "ab_bpe_from_parts": (C.c_int, [C.POINTER(C.c_char_p), C.POINTER(u32), C.POINTER(f32), u32,
                                    u32, PP]),
    "ab_bpe_info": (C.c_int, [P, C.POINTER(u32), C.POINTER(u32)]),
    "ab_bpe_encode": (C.c_int, [P, C.c_char_p, C.c_size_t, i32, i32, C.POINTER(i32), u32,
                                C.POINTER(u32)]),
    "ab_bpe_decode": (C.c_int, [P, i32, i32, C.c_char_p, u32, C.POINTER(u32)]),
    "ab_bpe_destroy": (C.c_int, [P]),
    "ab_llama_create": (C.c_int, [P, C.POINTER(LlamaConfig_t), PP]),
    "ab_llama_init_synthetic": (C.c_int, [P, u64, f32]),
    "ab_llama_weight": (C.c_int, [P, i32, u32, C.POINTER(T)]),
    "ab_llama_cache": (C.c_int, [P, PP]),
    "ab_llama_step": (C.c_int, [P, C.POINTER(DecodeStep_t), u32, C.POINTER(f32),
                                C.POINTER(i32)]),
    "ab_llama_decode_device": (C.c_int, [P, C.POINTER(DecodeStep_t), u32, u32,
                                         C.POINTER(i32)]),
    "ab_llama_prefill": (C.c_int, [P, u32, C.POINTER(i32), u32, u32, C.POINTER(f32),
                                   C.POINTER(i32)]),
    "ab_llama_prefill_rows": (C.c_int, [P, u32]),
    "ab_llama_prefill_launches": (C.c_int, [P, C.POINTER(u32)]),
    "ab_llama_prefill_scheme": (C.c_int, [P, u32, u32, i32, PP]),
    "ab_llama_generate_tokens": (C.c_int, [P, C.POINTER(i32), u32, u32, i32, i32,
                                           C.POINTER(i32), u32, C.POINTER(u32),
                                           C.POINTER(C.c_double)]),
    "ab_llama_scheme": (C.c_int, [P, PP]),
    "ab_llama_step_trace": (C.c_int, [P, C.POINTER(C.c_uint64), u32, C.POINTER(u32),
                                      C.POINTER(u32)]),
    "ab_llama_logits": (C.c_int, [P, C.POINTER(T)]),
    "ab_llama_reset": (C.c_int, [P]),
    "ab_llama_as_model": (C.c_int, [P, C.POINTER(Model_t)]),
    "ab_llama_destroy": (C.c_int, [P]),
    "ab_comm_unique_id": (C.c_int, [C.POINTER(C.c_uint8)]),
    "ab_comm_create": (C.c_int, [P, C.POINTER(C.c_uint8), i32, i32, PP]),
    "ab_comm_create_timeout": (C.c_int, [P, C.POINTER(C.c_uint8), i32, i32, u32, PP]),
    "ab_comm_loopback_reduce": (C.c_int, [P, u32, u32, u32, C.POINTER(C.c_float)]),
    "ab_comm_rank": (C.c_int, [P, C.POINTER(i32), C.POINTER(i32)]),
    "ab_comm_abort": (C.c_int, [P]),
    "ab_comm_destroy": (C.c_int, [P]),
    "ab_comm_last_error": (C.c_char_p, []),
    "ab_llama_create_tp": (C.c_int, [P, C.POINTER(LlamaConfig_t), P, PP]),
    "ab_llama2c_config": (C.c_int, [C.c_char_p, C.c_uint32, C.c_int32, C.c_float,
                                    C.POINTER(LlamaConfig_t)]),
    "ab_llama_load_llama2c": (C.c_int, [P, C.c_char_p, C.c_int32, C.c_uint32, C.c_float, P,
                                        C.POINTER(LlamaConfig_t), PP]),
}

COMM_ID_BYTES = 128

_lib = None


def lib():
    """Load libammon_b200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m ammon_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def header_symbols(path=None):
    """Function names declared in include/ammon_b200.h."""
    import re

    path = path or os.path.join(os.path.dirname(HERE), "include", "ammon_b200.h")
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ab_[a-z0-9_]+)\s*\(", text)) -
                  {n for n in re.findall(r"\(\*(ab_[a-z0-9_]+)\)", text)})
