"""ctypes binding of libqxcuda.so (the C ABI declared in include/qxcuda.h).

The library is required: importing this module on a machine where it is
missing raises immediately, so no call can silently fall back to a CPU path.
"""
from __future__ import annotations

import ctypes as C
import os

PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(PKG, "libqxcuda.so")

# qxc_status
OK, ERR_INVALID_ARG, ERR_POSITION, ERR_NONFINITE, ERR_CUDA, ERR_NCCL, ERR_TIMEOUT, ERR_UNSUPPORTED, \
    ERR_OUT_OF_MEMORY = range(9)
# qxc_model / qxc_dtype
MODEL_GRANITE, MODEL_QWEN3 = 0, 1
F32, BF16, F16 = 0, 1, 2
DECODE_NO_ADVANCE, DECODE_NATIVE_EXP, DECODE_PINNED_EXP = 0x1, 0x2, 0x4
VERIFY_PER_TOKEN = 0x8
HASH_AUTO, HASH_PER_CHUNK, HASH_PER_SLOT = 0, 1, 2
PEER_HANDLE_BYTES = 64


class KvDesc(C.Structure):
    _fields_ = [("model", C.c_int32), ("layers", C.c_int32), ("sequences", C.c_int32), ("capacity", C.c_int32),
                ("key_dtype", C.c_int32), ("value_dtype", C.c_int32), ("first_position", C.c_int32)]


class DecodeArgs(C.Structure):
    _fields_ = [("layer_begin", C.c_int32), ("layer_count", C.c_int32), ("seq_count", C.c_int32),
                ("seq_ids", C.POINTER(C.c_int32)), ("positions", C.POINTER(C.c_int32)),
                ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p),
                ("q_rot_out", C.c_void_p), ("q_norm", C.c_void_p), ("k_norm", C.c_void_p),
                ("q_dtype", C.c_int32), ("in_dtype", C.c_int32), ("out_dtype", C.c_int32),
                ("flags", C.c_int32), ("split", C.c_int32)]


class PrefillArgs(C.Structure):
    _fields_ = [("seq", C.c_int32), ("layer", C.c_int32), ("length", C.c_int32), ("q", C.c_void_p),
                ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p), ("in_dtype", C.c_int32),
                ("out_dtype", C.c_int32), ("flags", C.c_int32)]


class PartialArgs(C.Structure):
    _fields_ = [("seq", C.c_int32), ("layer", C.c_int32), ("position", C.c_int32), ("append", C.c_int32),
                ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("q_norm", C.c_void_p),
                ("k_norm", C.c_void_p), ("partials", C.c_void_p), ("q_dtype", C.c_int32),
                ("in_dtype", C.c_int32), ("flags", C.c_int32), ("split", C.c_int32)]


class VerifyArgs(C.Structure):
    """qxc_verify_args (K speculative tokens of one sequence)."""
    _fields_ = [("seq", C.c_int32), ("layer_begin", C.c_int32), ("layer_count", C.c_int32), ("start", C.c_int32),
                ("tokens", C.c_int32), ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p),
                ("q_norm", C.c_void_p), ("k_norm", C.c_void_p), ("q_dtype", C.c_int32), ("in_dtype", C.c_int32),
                ("out_dtype", C.c_int32), ("flags", C.c_int32), ("split", C.c_int32)]


class Q4Matrix(C.Structure):
    """qxc_q4_matrix: row-major Q4, group 32 (device codes and FP16 scales)."""
    _fields_ = [("rows", C.c_int32), ("cols", C.c_int32), ("codes", C.c_void_p), ("scales", C.c_void_p)]


class LayerArgs(C.Structure):
    """qxc_layer_args (the attention sub-layer of a Granite layer with Q4 weights)."""
    _fields_ = [("seq", C.c_int32), ("layer", C.c_int32), ("position", C.c_int32), ("hidden_in", C.c_void_p),
                ("hidden_out", C.c_void_p), ("input_norm", C.c_void_p), ("q_proj", Q4Matrix), ("k_proj", Q4Matrix),
                ("v_proj", Q4Matrix), ("o_proj", Q4Matrix), ("attention_out", C.c_void_p), ("flags", C.c_int32),
                ("split", C.c_int32)]


class LayerWeights(C.Structure):
    """qxc_layer_weights (one layer's RMSNorm weight and Q4 q/k/v/o)."""
    _fields_ = [("input_norm", C.c_void_p), ("q_proj", Q4Matrix), ("k_proj", Q4Matrix), ("v_proj", Q4Matrix),
                ("o_proj", Q4Matrix)]


class StackArgs(C.Structure):
    """qxc_stack_args (the attention sub-layers of consecutive layers, one token)."""
    _fields_ = [("seq", C.c_int32), ("layer_begin", C.c_int32), ("layer_count", C.c_int32),
                ("position", C.c_int32), ("hidden_in", C.c_void_p), ("hidden_out", C.c_void_p),
                ("layers", C.POINTER(LayerWeights)), ("flags", C.c_int32), ("split", C.c_int32)]


class KvPaging(C.Structure):
    """qxc_kv_paging (paged arena: rows per page, physical pages per layer)."""
    _fields_ = [("page_size", C.c_int32), ("pool_pages", C.c_int32)]


class VerificationHashArgs(C.Structure):
    """qxc_verification_hash_args (per-token state roots and KV slot leaves)."""
    _fields_ = [("seq", C.c_int32), ("token", C.c_int32), ("residuals", C.c_void_p),
                ("residual_stride", C.c_int64), ("checkpoint_interval", C.c_int32), ("digests", C.c_void_p)]


class StaticDecodeArgs(C.Structure):
    """qxc_static_decode_args (allocation-free Granite decode)."""
    _fields_ = [("key_cache", C.c_void_p), ("value_cache", C.c_void_p), ("capacity", C.c_int32),
                ("key_dtype", C.c_int32), ("value_dtype", C.c_int32), ("position", C.c_int32),
                ("q", C.c_void_p), ("k", C.c_void_p), ("v", C.c_void_p), ("out", C.c_void_p),
                ("q_dtype", C.c_int32), ("in_dtype", C.c_int32), ("out_dtype", C.c_int32),
                ("flags", C.c_int32), ("split", C.c_int32), ("device_error", C.c_void_p)]


_lib = None


def load() -> C.CDLL:
    """Load libqxcuda.so (raises if it has not been built)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: build it with `python -m qx_b200.build` "
                           "(qx_b200 has no CPU fallback)")
    lib = C.CDLL(LIB_PATH)
    vp, i32, pp = C.c_void_p, C.c_int32, C.POINTER(C.c_void_p)
    sig = {
        "qxc_abi_version": (C.c_int, []),
        "qxc_status_string": (C.c_char_p, [C.c_int]),
        "qxc_init": (C.c_int, [C.c_int, pp]),
        "qxc_destroy": (None, [vp]),
        "qxc_set_stream": (C.c_int, [vp, vp]),
        "qxc_get_stream": (vp, [vp]),
        "qxc_sync": (C.c_int, [vp]),
        "qxc_last_error": (C.c_char_p, [vp]),
        "qxc_launch_count": (C.c_uint64, [vp]),
        "qxc_last_split": (C.c_int32, [vp]),
        "qxc_auto_split": (C.c_int32, [C.c_int32, C.POINTER(C.c_int32), C.c_int32, C.c_int32, C.c_int32, C.c_int32]),
        "qxc_kv_bytes": (C.c_int, [C.POINTER(KvDesc), C.POINTER(C.c_size_t), C.POINTER(C.c_size_t)]),
        "qxc_kv_create": (C.c_int, [vp, C.POINTER(KvDesc), pp]),
        "qxc_kv_create_paged": (C.c_int, [vp, C.POINTER(KvDesc), C.POINTER(KvPaging), pp]),
        "qxc_kv_paged_bytes": (C.c_int, [C.POINTER(KvDesc), C.POINTER(KvPaging), C.POINTER(C.c_size_t),
                                         C.POINTER(C.c_size_t)]),
        "qxc_kv_page_stats": (C.c_int, [vp, i32, C.POINTER(i32), C.POINTER(i32)]),
        "qxc_kv_trim": (C.c_int, [vp, i32]),
        "qxc_kv_pool_buffer": (C.c_int, [vp, i32, pp, C.POINTER(C.c_size_t)]),
        "qxc_kv_destroy": (None, [vp]),
        "qxc_kv_len": (C.c_int, [vp, i32, C.POINTER(i32)]),
        "qxc_kv_reset": (C.c_int, [vp, i32]),
        "qxc_kv_set_len": (C.c_int, [vp, i32, i32]),
        "qxc_kv_checkpoint": (C.c_int, [vp, i32, C.POINTER(i32)]),
        "qxc_kv_rollback": (C.c_int, [vp, i32, i32]),
        "qxc_kv_commit": (C.c_int, [vp, i32, i32, i32]),
        "qxc_kv_key_buffer": (C.c_int, [vp, i32, i32, pp, C.POINTER(C.c_size_t)]),
        "qxc_kv_value_buffer": (C.c_int, [vp, i32, i32, pp, C.POINTER(C.c_size_t)]),
        "qxc_kv_read": (C.c_int, [vp, i32, i32, i32, i32, vp, vp]),
        "qxc_kv_write": (C.c_int, [vp, i32, i32, i32, i32, vp, vp]),
        "qxc_decode": (C.c_int, [vp, vp, C.POINTER(DecodeArgs)]),
        "qxc_decode_host": (C.c_int, [vp, vp, C.POINTER(DecodeArgs)]),
        "qxc_granite_attention_decode": (C.c_int, [vp, vp, vp, vp, vp, i32, vp]),
        "qxc_apply_granite_rope": (C.c_int, [vp, vp, vp, i32]),
        "qxc_prefill": (C.c_int, [vp, vp, C.POINTER(PrefillArgs)]),
        "qxc_decode_partials": (C.c_int, [vp, vp, C.POINTER(PartialArgs)]),
        "qxc_decode_verify": (C.c_int, [vp, vp, C.POINTER(VerifyArgs)]),
        "qxc_q4_mat_vec": (C.c_int, [vp, C.POINTER(Q4Matrix), vp, vp, vp]),
        "qxc_attention_layer": (C.c_int, [vp, vp, C.POINTER(LayerArgs)]),
        "qxc_attention_stack": (C.c_int, [vp, vp, C.POINTER(StackArgs)]),
        "qxc_lse_merge": (C.c_int, [vp, i32, i32, vp, vp, i32]),
        "qxc_peer_group_create": (C.c_int, [vp, i32, i32, pp]),
        "qxc_peer_group_destroy": (None, [vp]),
        "qxc_peer_group_handle": (C.c_int, [vp, vp]),
        "qxc_peer_group_base": (C.c_int, [vp, pp]),
        "qxc_peer_group_open": (C.c_int, [vp, i32, vp]),
        "qxc_peer_group_set_peer": (C.c_int, [vp, i32, vp]),
        "qxc_exchange_merge": (C.c_int, [vp, vp, i32, vp, vp, i32]),
        "qxc_decode_exchange": (C.c_int, [vp, vp, C.POINTER(PartialArgs), vp, vp, i32]),
        "qxc_verification_hashes": (C.c_int, [vp, vp, C.POINTER(VerificationHashArgs)]),
        "qxc_kv_slot_hashes": (C.c_int, [vp, vp, i32, i32, i32, i32, i32, vp, i32]),
        "qxc_blake3_compress_rate": (C.c_int, [vp, C.POINTER(C.c_double)]),
        "qxc_consensus_math_conformance": (C.c_int, [vp, vp, C.c_int32, vp]),
        "qxc_granite_decode_static_scratch": (C.c_int, [C.POINTER(StaticDecodeArgs), vp, C.c_char_p, C.c_size_t]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def header_symbols(header: str | None = None) -> list[str]:
    """Every function name declared in include/*.h (for the export check)."""
    import re
    inc = os.path.join(os.path.dirname(PKG), "include")
    names = []
    for f in sorted(os.listdir(inc)) if header is None else [header]:
        if f.endswith(".h"):
            text = open(os.path.join(inc, f)).read()
            text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
            names += re.findall(r"\b(qxc_\w+)\s*\(", text)
    return sorted(set(names))
