"""ctypes binding of libmoestream_cuda.so (the C ABI declared in include/moestream_cuda.h).

There is no fallback: if the CUDA library is missing or cannot be loaded, every entry
point raises.  Build it with ``python -m moe_stream_b200.build``.
"""
from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "libmoestream_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "moestream_cuda.h")

MS_OK = 0
STATUS = {0: "ok", 1: "invalid argument", 2: "out of device memory", 3: "CUDA error", 4: "NCCL error",
          5: "device wait timed out", 6: "unsupported tensor type", 7: "shape mismatch", 8: "I/O error",
          9: "malformed GGUF", 10: "call out of order", 11: "out-of-range index seen on the device"}

ARCH_GPT_OSS, ARCH_QWEN_MOE = 0, 1


class MsError(RuntimeError):
    def __init__(self, status: int, msg: str):
        super().__init__(f"{STATUS.get(status, status)}: {msg}")
        self.status = status


class ModelConfig(C.Structure):
    _fields_ = [("arch", C.c_int), ("hidden", C.c_int), ("layers", C.c_int), ("heads", C.c_int),
                ("kv_heads", C.c_int), ("head_dim", C.c_int), ("rot_dim", C.c_int), ("experts", C.c_int),
                ("top_k", C.c_int), ("inter", C.c_int), ("vocab", C.c_int), ("rope_theta", C.c_float),
                ("eps", C.c_float), ("sliding_window", C.c_int), ("norm_topk_prob", C.c_int),
                ("max_seq_len", C.c_int), ("ep_rank", C.c_int), ("ep_size", C.c_int), ("attn_splits", C.c_int),
                ("attn_interval", C.c_int), ("ssm_groups", C.c_int), ("ssm_state", C.c_int),
                ("ssm_dt_rank", C.c_int), ("ssm_inner", C.c_int), ("ssm_conv", C.c_int)]


class AttnLayer(C.Structure):
    """ms_attn_layer: one attention half-layer in device memory (device pointers as ints)."""
    _fields_ = [("hidden", C.c_int), ("heads", C.c_int), ("kv_heads", C.c_int), ("head_dim", C.c_int),
                ("rot_dim", C.c_int), ("eps", C.c_float), ("window", C.c_int), ("cap", C.c_int),
                ("attn_norm", C.c_void_p), ("wqkv", C.c_void_p), ("bqkv", C.c_void_p), ("wo", C.c_void_p),
                ("bo", C.c_void_p), ("sinks", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("k_cache", C.c_void_p), ("v_cache", C.c_void_p), ("cos_t", C.c_void_p), ("sin_t", C.c_void_p),
                ("q_gate", C.c_int)]


class DeltaNetLayer(C.Structure):
    """ms_deltanet_layer: one Gated DeltaNet layer in device memory (device pointers as ints)."""
    _fields_ = [("hidden", C.c_int), ("n_k_heads", C.c_int), ("head_k_dim", C.c_int), ("n_v_heads", C.c_int),
                ("head_v_dim", C.c_int), ("conv_kernel", C.c_int), ("eps", C.c_float),
                ("qkv_q", C.c_int), ("qkv", C.c_void_p), ("gate_q", C.c_int), ("gate", C.c_void_p),
                ("ba_q", C.c_int), ("ba", C.c_void_p), ("out_q", C.c_int), ("out", C.c_void_p),
                ("conv1d", C.c_void_p), ("ssm_a", C.c_void_p), ("dt_bias", C.c_void_p), ("norm", C.c_void_p)]


_lib = None
_vp, _i, _f = C.c_void_p, C.c_int, C.c_float
_ip = C.POINTER(C.c_int32)
_fp = C.POINTER(C.c_float)

# name -> (restype, argtypes)
_SIGS = {
    "ms_abi_version": (C.c_int, []),
    "ms_status_string": (C.c_char_p, [C.c_int]),
    "ms_ctx_create": (C.c_int, [C.c_int, C.POINTER(_vp)]),
    "ms_ctx_destroy": (C.c_int, [_vp]),
    "ms_ctx_set_stream": (C.c_int, [_vp, _vp]),
    "ms_ctx_use_own_stream": (C.c_int, [_vp]),
    "ms_sync": (C.c_int, [_vp]),
    "ms_last_error": (C.c_char_p, [_vp]),
    "ms_ctx_error_flags": (C.c_int, [_vp, C.POINTER(C.c_uint32), C.c_int]),
    "ms_ctx_sm_count": (C.c_int, [_vp]),
    "ms_malloc": (C.c_int, [_vp, C.c_size_t, C.POINTER(_vp)]),
    "ms_free": (C.c_int, [_vp, _vp]),
    "ms_memcpy_h2d": (C.c_int, [_vp, _vp, _vp, C.c_size_t]),
    "ms_memcpy_d2h": (C.c_int, [_vp, _vp, _vp, C.c_size_t]),
    "ms_dequantize": (C.c_int, [_vp, _i, _vp, C.c_int64, _vp]),
    "ms_rms_norm": (C.c_int, [_vp, _vp, _vp, _vp, _i, _i, _f]),
    "ms_gemv": (C.c_int, [_vp, _i, _vp, _i, _i, _vp, _vp, _vp]),
    "ms_router_topk": (C.c_int, [_vp, _vp, _vp, _f, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "ms_moe_mxfp4_decode": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp, _vp]),
    "ms_moe_mxfp4_decode_noalloc": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp,
                                              _vp, _vp]),
    "ms_mxfp4_packed_bytes": (C.c_int, [_i, _i, _i, C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
    "ms_mxfp4_pack_experts": (C.c_int, [_vp, _vp, _vp, _vp, _i, _i, _i, _vp, _vp]),
    "ms_moe_mxfp4_decode_packed": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _vp, _vp,
                                             _vp]),
    "ms_moe_mxfp4_prefill_packed": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i, _vp, _i, _vp,
                                              _vp, _vp, _i]),
    "ms_rope": (C.c_int, [_vp, _vp, _vp, _vp, _i, _i, _i, _i, _vp]),
    "ms_sample": (C.c_int, [_vp, _vp, _i, _vp, C.c_float, C.c_float, C.c_float, C.c_float, _vp, _vp]),
    "ms_attn_layer_decode": (C.c_int, [_vp, C.POINTER(AttnLayer), _i, _vp]),
    "ms_deltanet_decode": (C.c_int, [_vp, C.POINTER(DeltaNetLayer), _vp, _vp, _vp, _vp]),
    "ms_shared_expert": (C.c_int, [_vp, _i, _vp, _vp, _i, _vp, _vp, _i, _i, _vp, _vp]),
    "ms_nccl_unique_id": (C.c_int, [_vp, _vp, C.c_size_t]),
    "ms_model_init_ep": (C.c_int, [_vp, _vp, C.c_size_t]),
    "ms_model_ep_handle": (C.c_int, [_vp, _vp, C.c_size_t]),
    "ms_model_ep_connect": (C.c_int, [_vp, _vp, C.c_size_t]),
    "ms_model_create": (C.c_int, [_vp, C.POINTER(ModelConfig), C.POINTER(_vp)]),
    "ms_model_set_tensor": (C.c_int, [_vp, C.c_char_p, _i, _i, C.POINTER(C.c_int64), _vp, C.c_size_t]),
    "ms_model_finalize": (C.c_int, [_vp]),
    "ms_model_open_gguf": (C.c_int, [_vp, C.c_char_p, _i, _i, _i, C.POINTER(_vp)]),
    "ms_model_open_gguf_tiered": (C.c_int, [_vp, C.c_char_p, _i, _i, C.POINTER(_vp)]),
    "ms_model_set_expert_tier": (C.c_int, [_vp, _i]),
    "ms_model_set_dynamic_k": (C.c_int, [_vp, _i, _i, _i, _i]),
    "ms_model_set_router_stats": (C.c_int, [_vp, _i]),
    "ms_model_router_stats": (C.c_int, [_vp, _fp, _ip]),
    "ms_model_router_totals": (C.c_int, [_vp, _vp, _vp, _vp, _vp, _i, C.POINTER(C.c_int)]),
    "ms_model_expert_tier_stats": (C.c_int, [_vp, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)]),
    "ms_model_get_config": (C.c_int, [_vp, C.POINTER(ModelConfig)]),
    "ms_model_destroy": (C.c_int, [_vp]),
    "ms_model_forward": (C.c_int, [_vp, _ip, _i, _fp]),
    "ms_model_decode_step": (C.c_int, [_vp, C.c_int32, _ip]),
    "ms_model_generate": (C.c_int, [_vp, _ip, _i, _i, _ip, C.POINTER(C.c_int)]),
    "ms_model_decode_steps_device": (C.c_int, [_vp, _i]),
    "ms_model_batch_open": (C.c_int, [_vp, _i]),
    "ms_model_batch_close": (C.c_int, [_vp]),
    "ms_model_batch_clear": (C.c_int, [_vp]),
    "ms_model_batch_forward": (C.c_int, [_vp, _ip, _i, _ip]),
    "ms_model_batch_decode_steps_device": (C.c_int, [_vp, _i]),
    "ms_model_batch_next_tokens": (C.c_int, [_vp, _ip]),
    "ms_model_batch_token_log": (C.c_int, [_vp, _ip, _i, C.POINTER(C.c_int)]),
    "ms_model_batch_last_logits": (C.c_int, [_vp, _fp]),
    "ms_model_batch_kernels_per_step": (C.c_int, [_vp]),
    "ms_model_batch_profile_step": (C.c_int, [_vp, _fp, _i, C.POINTER(C.c_int)]),
    "ms_model_token_log": (C.c_int, [_vp, _ip, _i, C.POINTER(C.c_int)]),
    "ms_model_clear_cache": (C.c_int, [_vp]),
    "ms_model_seq_len": (C.c_int, [_vp, C.POINTER(C.c_int)]),
    "ms_model_last_hidden": (C.c_int, [_vp, _fp]),
    "ms_model_last_routing": (C.c_int, [_vp, _i, _ip, _fp]),
    "ms_model_last_logits": (C.c_int, [_vp, _fp]),
    "ms_model_set_trace": (C.c_int, [_vp, _i]),
    "ms_model_set_prefill": (C.c_int, [_vp, _i]),
    "ms_model_set_exact": (C.c_int, [_vp, _i]),
    "ms_model_set_sampling": (C.c_int, [_vp, _i, C.c_float, C.c_float, C.c_float, C.c_uint64]),
    "ms_model_layer_trace": (C.c_int, [_vp, _fp, _fp]),
    "ms_model_set_graph": (C.c_int, [_vp, _i]),
    "ms_model_kernels_per_step": (C.c_int, [_vp]),
    "ms_model_profile_step": (C.c_int, [_vp, _fp, _i, C.POINTER(C.c_int)]),
}


def header_symbols() -> list:
    """Every function the public header declares."""
    src = open(HEADER).read()
    return re.findall(r"^MS_API\s+[\w\s\*]+?\b(ms_\w+)\s*\(", src, flags=re.M)


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: build it with `python -m moe_stream_b200.build`")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, ctx=None) -> None:
    if status != MS_OK:
        msg = lib().ms_last_error(ctx).decode() if ctx else ""
        raise MsError(status, msg)
