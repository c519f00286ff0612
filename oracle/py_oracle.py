"""ctypes binding of the CPU oracle (oracle/libqx_oracle.so).

TEST INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference arm, as the checker or the timed CPU
baseline. The product package qx_b200 never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libqx_oracle.so")

F32, BF16, F16 = 0, 1, 2
OK, ERR_INVALID_ARG, ERR_POSITION, ERR_NONFINITE = 0, 1, 2, 3

_lib = None


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (gcc only)."""
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(
        os.path.getmtime(os.path.join(HERE, f)) for f in ("qx_oracle.c", "qx_oracle.h", "Makefile")
    ):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        _lib = C.CDLL(LIB_PATH)
        fp, ip, vp = C.POINTER(C.c_float), C.POINTER(C.c_int), C.c_void_p
        u16p = C.POINTER(C.c_uint16)
        _lib.qxo_exp_f32.argtypes = [C.c_float, fp]
        _lib.qxo_rsqrt_f32.argtypes = [C.c_float, fp]
        _lib.qxo_sin_cos_f32.argtypes = [C.c_float, fp, fp]
        _lib.qxo_granite_rope_sin_cos.argtypes = [C.c_uint32, C.c_uint32, fp, fp]
        _lib.qxo_granite_rope_pair.argtypes = [C.c_uint32, C.c_uint32, C.c_float, C.c_float, fp, fp]
        _lib.qxo_granite_inverse_frequency_bits.argtypes = [C.c_uint32]
        _lib.qxo_granite_inverse_frequency_bits.restype = C.c_uint32
        _lib.qxo_reduce_simd32.argtypes = [fp]
        _lib.qxo_reduce_simd32.restype = C.c_float
        for name in ("qxo_exp_worst_relative_error", "qxo_rsqrt_worst_relative_error",
                     "qxo_rope_worst_absolute_error"):
            getattr(_lib, name).restype = C.c_float
        _lib.qxo_rotate_heads.argtypes = [fp, C.c_int, C.c_uint32]
        _lib.qxo_granite_attention_decode.argtypes = [fp, fp, fp, C.c_int, vp, vp, C.c_int, C.c_int, ip,
                                                      C.c_int, C.c_int, fp]
        _lib.qxo_granite_attention_decode_many.argtypes = [
            C.c_int, C.POINTER(fp), C.POINTER(fp), C.POINTER(fp), ip, C.POINTER(vp), C.POINTER(vp),
            C.c_int, C.c_int, ip, C.c_int, C.c_int, C.POINTER(fp), C.c_int, ip]
        _lib.qxo_granite_prefill.argtypes = [vp, vp, vp, C.c_int, C.c_int, vp, vp, C.c_int, fp, C.c_int]
        _lib.qxo_qwen_qk_norm_rope.argtypes = [u16p, u16p, fp, fp, C.c_uint32, C.c_int, u16p, u16p]
        _lib.qxo_qwen_rope_table.argtypes = [C.c_uint32, fp, fp]
        _lib.qxo_qwen_gqa_attention.argtypes = [u16p, u16p, u16p, C.c_int, C.c_int, fp, u16p, C.c_int]
        _lib.qxo_f32_to_bf16.argtypes = [C.c_float]
        _lib.qxo_f32_to_bf16.restype = C.c_uint16
        u8p = C.POINTER(C.c_uint8)
        _lib.qxo_rms_norm_simd.argtypes = [fp, fp, fp]
        _lib.qxo_q4_quantize.argtypes = [fp, C.c_int, C.c_int, u8p, u16p]
        _lib.qxo_q4_mat_vec_simd32.argtypes = [u8p, u16p, C.c_int, C.c_int, fp, fp]
        _lib.qxo_granite_attention_layer.argtypes = [fp, fp, u8p, u16p, u8p, u16p, u8p, u16p, u8p, u16p, C.c_int,
                                                     fp, fp, ip, C.c_int, C.c_int, fp, fp]
        _lib.qxo_cpu_rotate_heads.argtypes = [fp, C.c_int, C.c_uint32]
        _lib.qxo_blake3_single_chunk.argtypes = [vp, C.c_size_t, u8p]
        _lib.qxo_chunk_tree_hash.argtypes = [vp, C.c_size_t, C.c_char_p, C.c_char_p, u8p]
        _lib.qxo_kv_leaf_hash.argtypes = [C.c_uint16, C.c_uint32, vp, C.c_size_t, vp, C.c_size_t, u8p]
    return _lib


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u16(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint16))


def _vp(a):
    return C.c_void_p(a.ctypes.data)


def exp_f32(x: float):
    out = C.c_float()
    return out.value if lib().qxo_exp_f32(x, C.byref(out)) else None


def rsqrt_f32(x: float):
    out = C.c_float()
    return out.value if lib().qxo_rsqrt_f32(x, C.byref(out)) else None


def granite_rope_sin_cos(position: int, pair: int):
    s, c = C.c_float(), C.c_float()
    return (s.value, c.value) if lib().qxo_granite_rope_sin_cos(position, pair, C.byref(s), C.byref(c)) else None


def reduce_simd32(lanes) -> float:
    a = np.ascontiguousarray(lanes, dtype=np.float32)
    return lib().qxo_reduce_simd32(_fp(a))


def kv_np_dtype(dtype: int):
    return np.float32 if dtype == F32 else np.uint16


class KvCache:
    """Oracle twin of qx_runtime::KvCache (crates/qx-runtime/src/lib.rs:350-432)."""

    def __init__(self, max_context: int, key_dtype: int = F32, value_dtype: int = F32,
                 kv_heads: int = 8, head_dim: int = 64):
        self.max_context = max_context
        self.key_dtype, self.value_dtype = key_dtype, value_dtype
        self.keys = np.zeros((max_context, kv_heads, head_dim), kv_np_dtype(key_dtype))
        self.values = np.zeros((max_context, kv_heads, head_dim), kv_np_dtype(value_dtype))
        self.length = C.c_int(0)

    def __len__(self):
        return self.length.value

    def reset(self):
        self.length.value = 0


def granite_attention_decode(q, k, v, position: int, cache: KvCache, hierarchical: bool = False):
    """Returns (status, output[16*64])."""
    q = np.ascontiguousarray(q, np.float32).reshape(-1)
    k = np.ascontiguousarray(k, np.float32).reshape(-1)
    v = np.ascontiguousarray(v, np.float32).reshape(-1)
    out = np.zeros(1024, np.float32)
    st = lib().qxo_granite_attention_decode(_fp(q), _fp(k), _fp(v), position, _vp(cache.keys), _vp(cache.values),
                                            cache.key_dtype, cache.value_dtype, C.byref(cache.length),
                                            cache.max_context, int(hierarchical), _fp(out))
    return st, out


def granite_decode_many(qs, ks, vs, positions, caches, threads=1, hierarchical=False):
    """Decode one token on many independent caches (OpenMP-free pthread pool)."""
    n = len(caches)
    FP = C.POINTER(C.c_float)
    qarr = (FP * n)(*[_fp(a) for a in qs])
    karr = (FP * n)(*[_fp(a) for a in ks])
    varr = (FP * n)(*[_fp(a) for a in vs])
    outs = [np.zeros(1024, np.float32) for _ in range(n)]
    oarr = (FP * n)(*[_fp(a) for a in outs])
    kc = (C.c_void_p * n)(*[c.keys.ctypes.data for c in caches])
    vc = (C.c_void_p * n)(*[c.values.ctypes.data for c in caches])
    lens = (C.c_int * n)(*[c.length.value for c in caches])
    pos = (C.c_int * n)(*positions)
    sts = (C.c_int * n)()
    worst = lib().qxo_granite_attention_decode_many(n, qarr, karr, varr, pos, kc, vc, caches[0].key_dtype,
                                                    caches[0].value_dtype, lens, caches[0].max_context,
                                                    int(hierarchical), oarr, threads, sts)
    for c, l in zip(caches, lens):
        c.length.value = l
    return worst, outs


def granite_prefill(q, k, v, in_dtype: int, kv_dtype: int, threads: int = 1):
    """q:[L,16,64], k,v:[L,8,64] (uint16 bf16 bits or f32). Returns (status, keys, values, out[L,16,64])."""
    L = q.shape[0]
    keys = np.zeros((L, 8, 64), kv_np_dtype(kv_dtype))
    values = np.zeros((L, 8, 64), kv_np_dtype(kv_dtype))
    out = np.zeros((L, 16, 64), np.float32)
    st = lib().qxo_granite_prefill(_vp(np.ascontiguousarray(q)), _vp(np.ascontiguousarray(k)),
                                   _vp(np.ascontiguousarray(v)), in_dtype, L, _vp(keys), _vp(values), kv_dtype,
                                   _fp(out), threads)
    return st, keys, values, out


def qwen_qk_norm_rope(q_bits, k_bits, q_norm, k_norm, position: int, dtype: int = BF16):
    q_bits = np.ascontiguousarray(q_bits, np.uint16).reshape(-1)
    k_bits = np.ascontiguousarray(k_bits, np.uint16).reshape(-1)
    qn = np.ascontiguousarray(q_norm, np.float32)
    kn = np.ascontiguousarray(k_norm, np.float32)
    qo = np.zeros_like(q_bits)
    ko = np.zeros_like(k_bits)
    lib().qxo_qwen_qk_norm_rope(_u16(q_bits), _u16(k_bits), _fp(qn), _fp(kn), position, dtype, _u16(qo), _u16(ko))
    return qo, ko


def qwen_rope_table(position: int):
    c = np.zeros(64, np.float32)
    s = np.zeros(64, np.float32)
    lib().qxo_qwen_rope_table(position, _fp(c), _fp(s))
    return c, s


def qwen_gqa_attention(q_bits, key_cache_bits, value_cache_bits, context: int, dtype: int = BF16, threads: int = 1):
    q_bits = np.ascontiguousarray(q_bits, np.uint16).reshape(-1)
    kc = np.ascontiguousarray(key_cache_bits, np.uint16)
    vc = np.ascontiguousarray(value_cache_bits, np.uint16)
    out = np.zeros(32 * 128, np.float32)
    bits = np.zeros(32 * 128, np.uint16)
    lib().qxo_qwen_gqa_attention(_u16(q_bits), _u16(kc), _u16(vc), context, dtype, _fp(out), _u16(bits), threads)
    return out, bits


def qwen_decode(q_bits, k_bits, v_bits, q_norm, k_norm, key_cache, value_cache, position: int,
                dtype: int = BF16, threads: int = 1):
    """One Qwen decode step: QK-norm+RoPE, store into slot `position`, attend over position+1 rows
    (qx-runtime-v2 lib.rs:904-1024 stage order). Caches are [capacity,4,128] uint16 and updated in place."""
    qr, kr = qwen_qk_norm_rope(q_bits, k_bits, q_norm, k_norm, position, dtype)
    key_cache[position] = kr.reshape(4, 128)
    value_cache[position] = np.asarray(v_bits, np.uint16).reshape(4, 128)
    out, bits = qwen_gqa_attention(qr, key_cache[: position + 1], value_cache[: position + 1], position + 1, dtype,
                                   threads)
    return qr, kr, out, bits


# ---- attention sub-layer with Q4 projections (qx-runtime-v2 CpuQ4Reference::step) ----
def _u8(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint8))


def rms_norm_simd(x, weight):
    """cpu_rms_norm_simd over HIDDEN = 1024 -> (status 1 ok, normalized)."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(weight, np.float32)
    out = np.zeros(1024, np.float32)
    st = lib().qxo_rms_norm_simd(_fp(x), _fp(w), _fp(out))
    return st, out


class Q4Matrix:
    """Q4, group 32, row-major: codes [rows][cols/32][16] u8, scales
    [rows][cols/32] FP16 bits (QuantizedTensor::quantize)."""

    def __init__(self, weights: np.ndarray):
        w = np.ascontiguousarray(weights, np.float32)
        self.rows, self.cols = w.shape
        self.codes = np.zeros((self.rows, self.cols // 32, 16), np.uint8)
        self.scales = np.zeros((self.rows, self.cols // 32), np.uint16)
        lib().qxo_q4_quantize(_fp(w), self.rows, self.cols, _u8(self.codes), _u16(self.scales))

    def mat_vec(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.rows, np.float32)
        lib().qxo_q4_mat_vec_simd32(_u8(self.codes), _u16(self.scales), self.rows, self.cols, _fp(x), _fp(out))
        return out


def granite_attention_layer(hidden, input_norm, qp: Q4Matrix, kp: Q4Matrix, vp: Q4Matrix, op: Q4Matrix,
                            position: int, cache: KvCache, cpu_twin: bool = False):
    """(status 0 ok, hidden out [1024], attention [1024]) for one layer at
    `position`: the V2 GPU stage's arithmetic, or with cpu_twin the V2 CPU
    twin CpuQ4Reference::step (no-fma RoPE, hierarchical attention, <= 512)."""
    h = np.ascontiguousarray(hidden, np.float32)
    w = np.ascontiguousarray(input_norm, np.float32)
    out = np.zeros(1024, np.float32)
    att = np.zeros(1024, np.float32)
    st = lib().qxo_granite_attention_layer(_fp(h), _fp(w), _u8(qp.codes), _u16(qp.scales), _u8(kp.codes),
                                           _u16(kp.scales), _u8(vp.codes), _u16(vp.scales), _u8(op.codes),
                                           _u16(op.scales), position, _fp(cache.keys), _fp(cache.values),
                                           C.byref(cache.length), cache.max_context, int(bool(cpu_twin)), _fp(out),
                                           _fp(att))
    return st, out, att


# ---- KV-slot commitments (qx-commit state.rs) -----------------------------------------
def blake3_single_chunk(data: bytes) -> bytes:
    out = np.zeros(32, np.uint8)
    buf = np.frombuffer(bytes(data), np.uint8) if data else np.zeros(1, np.uint8)
    assert lib().qxo_blake3_single_chunk(buf.ctypes.data, len(data), _u8(out)) == 1
    return out.tobytes()


def chunk_tree_hash(data: bytes, leaf_domain: bytes, tree_domain: bytes) -> bytes:
    out = np.zeros(32, np.uint8)
    buf = np.frombuffer(bytes(data), np.uint8)
    assert lib().qxo_chunk_tree_hash(buf.ctypes.data, len(data), leaf_domain, tree_domain, _u8(out)) == 1
    return out.tobytes()


def kv_leaf_hash(layer: int, token: int, key: bytes, value: bytes) -> bytes:
    """kv_leaf_hash_v1: the 32-byte commitment of one (layer, token) K/V slot."""
    out = np.zeros(32, np.uint8)
    kb, vb = np.frombuffer(bytes(key), np.uint8), np.frombuffer(bytes(value), np.uint8)
    assert lib().qxo_kv_leaf_hash(layer, token, kb.ctypes.data, len(key), vb.ctypes.data, len(value), _u8(out)) == 1
    return out.tobytes()


def state_hash(residual: bytes) -> bytes:
    """state_hash_v1 (qx-commit state.rs:253-257): the chunk tree of a
    residual snapshot under QX:STATE:CHUNK:V1 / QX:STATE:V1."""
    return chunk_tree_hash(residual, b"QX:STATE:CHUNK:V1", b"QX:STATE:V1")


def verification_hashes(residuals: bytes, residual_stride: int, checkpoint_interval: int, layers: int,
                        key_rows, value_rows, token: int) -> bytes:
    """The bytes encode_verification_hashes writes for one token
    (kernels/verification_hash.metal:428-522): per position p in 0..layers,
    32 bytes of state root (p == 0, p % interval == 0 or p == layers; else
    zeros) then 32 bytes of kv_leaf_hash_v1(p - 1, token, ...) (zeros at
    p == 0). key_rows[l] / value_rows[l] are layer l's row bytes."""
    out = bytearray()
    for p in range(layers + 1):
        if p == 0 or p % checkpoint_interval == 0 or p == layers:
            out += state_hash(residuals[p * residual_stride:(p + 1) * residual_stride])
        else:
            out += bytes(32)
        out += bytes(32) if p == 0 else kv_leaf_hash(p - 1, token, key_rows[p - 1], value_rows[p - 1])
    return bytes(out)
