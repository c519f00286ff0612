"""Python host API over libqxcuda, mirroring the reference's operator and
KV-cache interfaces for the attention path (names, argument meaning and
error behaviour follow blasrodri/qx):

  KvCache, granite_attention_decode, apply_granite_rope
      crates/qx-runtime/src/lib.rs:350-452
  ExecutionPlan.granite_with_kv_precision / kv_bytes / kv_key_bytes / kv_value_bytes
      crates/qx-runtime-v2/src/lib.rs:6566-6656
  KvArena.key_buffer / value_buffer, checkpoint / rollback / commit
      crates/qx-runtime-v2/src/lib.rs:6837-6860, 3265-3310

Errors the reference returns as `Err(String)` raise QxError carrying the
C status code and the same message text. Device tensors are passed as
torch tensors (or raw integer device pointers); every computation runs in
libqxcuda's CUDA kernels.
"""
from __future__ import annotations

import ctypes as C
import enum
import weakref
from dataclasses import dataclass

import numpy as np

from . import _lib
from ._lib import BF16, F16, F32, HASH_AUTO, HASH_PER_CHUNK, HASH_PER_SLOT, MODEL_GRANITE, MODEL_QWEN3  # noqa: F401

HIDDEN, ATTENTION_HEADS, KV_HEADS, HEAD_DIM, MAX_CONTEXT, LAYERS = 1024, 16, 8, 64, 4096, 24  # qx-model lib.rs:9-17
ATTENTION_MULTIPLIER = 0.015625  # qx-model lib.rs:20


class QxError(RuntimeError):
    def __init__(self, status: int, message: str):
        super().__init__(message)
        self.status = status


def _check(lib, ctx_handle, status: int):
    if status != _lib.OK:
        msg = lib.qxc_last_error(ctx_handle).decode() if ctx_handle else ""
        raise QxError(status, msg or lib.qxc_status_string(status).decode())


def _ptr(x) -> int | None:
    if x is None:
        return None
    if isinstance(x, int):
        return x
    if hasattr(x, "data_ptr"):
        return x.data_ptr()
    if isinstance(x, np.ndarray):
        return x.ctypes.data
    raise TypeError(f"cannot take a pointer of {type(x)}")


class Context:
    """qxc_ctx: one per host thread; owns (or borrows) a CUDA stream."""

    def __init__(self, device: int = 0):
        self.lib = _lib.load()
        h = C.c_void_p()
        st = self.lib.qxc_init(device, C.byref(h))
        if st != _lib.OK:
            raise QxError(st, f"qxc_init({device}) failed: {self.lib.qxc_status_string(st).decode()}")
        self.handle = h
        self.device = device
        self._arenas = weakref.WeakSet()  # destroyed before the context

    def close(self):
        if self.handle:
            for a in list(self._arenas):
                a.close()
            self.lib.qxc_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def check(self, status: int):
        _check(self.lib, self.handle, status)

    CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy: the implicitly synchronising default stream

    def set_stream(self, stream) -> None:
        """Borrow a CUDA stream: a torch.cuda.Stream or a raw handle. torch's
        default stream (handle 0) maps to cudaStreamLegacy so work stays
        ordered with torch; None restores the context's own stream."""
        if stream is None:
            self.check(self.lib.qxc_set_stream(self.handle, None))
            return
        raw = getattr(stream, "cuda_stream", stream)
        raw = raw or self.CUDA_STREAM_LEGACY
        self.check(self.lib.qxc_set_stream(self.handle, C.c_void_p(raw)))

    @property
    def stream(self) -> int:
        return self.lib.qxc_get_stream(self.handle) or 0

    def sync(self) -> None:
        self.check(self.lib.qxc_sync(self.handle))

    @property
    def launch_count(self) -> int:
        return int(self.lib.qxc_launch_count(self.handle))

    @property
    def last_split(self) -> int:
        """Cache positions per split chosen by the last decode call."""
        return int(self.lib.qxc_last_split(self.handle))

    def blake3_compress_rate(self) -> float:
        """BLAKE3 block compressions per second with no memory traffic (the
        ceiling the hash kernels are measured against); synchronous."""
        r = C.c_double()
        self.check(self.lib.qxc_blake3_compress_rate(self.handle, C.byref(r)))
        return r.value

    def run_consensus_math_conformance(self, inputs) -> list:
        """Raw bits [exp, rsqrt, rope sin, rope cos] of the device's pinned
        math per input (qx-metal/src/lib.rs:9622, the Metal context's
        conformance dispatch); the RoPE position is the input truncated to
        u32 and the pair its index mod 32. Quiet NaN bits where the CPU
        function returns None."""
        x = np.ascontiguousarray(inputs, dtype=np.float32)
        out = np.zeros((x.size, 4), dtype=np.uint32)
        self.check(self.lib.qxc_consensus_math_conformance(
            self.handle, x.ctypes.data_as(C.c_void_p), int(x.size), out.ctypes.data_as(C.c_void_p)))
        return [tuple(int(v) for v in row) for row in out]

    def lse_merge(self, model: int, n_parts: int, partials, out, out_dtype: int = F32) -> None:
        self.check(self.lib.qxc_lse_merge(self.handle, model, n_parts, _ptr(partials), _ptr(out), out_dtype))


class PeerGroup:
    """qxc_peer_group: this rank's area for the NVLink exchange of a KV-length
    split (qxc_exchange_merge). Attach every other rank's area with open()
    (a CUDA IPC handle from another process) or set_peer() (another group of
    this process); qx_b200.distributed.open_peer_group does it for a
    torch.distributed job."""

    def __init__(self, ctx: Context, rank: int, world: int):
        self.ctx, self.lib = ctx, ctx.lib
        h = C.c_void_p()
        ctx.check(self.lib.qxc_peer_group_create(ctx.handle, rank, world, C.byref(h)))
        self.handle, self.rank, self.world = h, rank, world

    def close(self):
        if getattr(self, "handle", None):
            if self.ctx.handle:
                self.lib.qxc_peer_group_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def ipc_handle(self) -> bytes:
        buf = C.create_string_buffer(_lib.PEER_HANDLE_BYTES)
        self.ctx.check(self.lib.qxc_peer_group_handle(self.handle, buf))
        return buf.raw

    def base(self) -> int:
        p = C.c_void_p()
        self.ctx.check(self.lib.qxc_peer_group_base(self.handle, C.byref(p)))
        return p.value

    def open(self, peer: int, ipc_handle: bytes) -> None:
        buf = C.create_string_buffer(bytes(ipc_handle), _lib.PEER_HANDLE_BYTES)
        self.ctx.check(self.lib.qxc_peer_group_open(self.handle, peer, buf))

    def set_peer(self, peer: int, base: int) -> None:
        self.ctx.check(self.lib.qxc_peer_group_set_peer(self.handle, peer, C.c_void_p(base)))

    def exchange_merge(self, model: int, partials, out, out_dtype: int = F32) -> None:
        """Push this rank's partials [q_heads][head_dim + 2] to every rank and
        merge all ranks' into out [q_heads][head_dim] (device tensors)."""
        self.ctx.check(self.lib.qxc_exchange_merge(self.ctx.handle, self.handle, model, _ptr(partials), _ptr(out),
                                                   out_dtype))


_default_ctx: Context | None = None


def default_context() -> Context:
    global _default_ctx
    if _default_ctx is None:
        _default_ctx = Context(0)
    return _default_ctx


def model_shape(model: int):
    """(query heads, kv heads, head dim)"""
    return (32, 4, 128) if model == MODEL_QWEN3 else (16, 8, 64)


def _np_dtype(dtype: int):
    return np.float32 if dtype == F32 else np.uint16


class KvArena:
    """qxc_kv: KV caches of `sequences` x `layers` in one device allocation,
    each [capacity][kv_heads][head_dim] (the reference's position-major layout)."""

    def __init__(self, ctx: Context, model: int = MODEL_GRANITE, layers: int = 1, sequences: int = 1,
                 capacity: int = MAX_CONTEXT, key_dtype: int = F32, value_dtype: int | None = None,
                 first_position: int = 0, page_size: int = 0, pool_pages: int = 0):
        """page_size > 0 makes a paged arena (qxc_kv_create_paged): per layer
        `pool_pages` pages of `page_size` rows shared by all sequences,
        mapped on demand; `capacity` is then the longest sequence."""
        self.ctx, self.lib = ctx, ctx.lib
        value_dtype = key_dtype if value_dtype is None else value_dtype
        self.desc = _lib.KvDesc(model, layers, sequences, capacity, key_dtype, value_dtype, first_position)
        h = C.c_void_p()
        if page_size:
            self.paging = _lib.KvPaging(page_size, pool_pages)
            ctx.check(self.lib.qxc_kv_create_paged(ctx.handle, C.byref(self.desc), C.byref(self.paging), C.byref(h)))
        else:
            self.paging = None
            ctx.check(self.lib.qxc_kv_create(ctx.handle, C.byref(self.desc), C.byref(h)))
        self.handle = h
        ctx._arenas.add(self)
        self.model, self.layers, self.sequences, self.capacity = model, layers, sequences, capacity
        self.key_dtype, self.value_dtype, self.first_position = key_dtype, value_dtype, first_position
        self.hq, self.hkv, self.d = model_shape(model)

    def close(self):
        if getattr(self, "handle", None):
            if self.ctx.handle:  # a closed context already destroyed its arenas
                self.lib.qxc_kv_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # cursors
    def len(self, seq: int = 0) -> int:
        n = C.c_int32()
        self.ctx.check(self.lib.qxc_kv_len(self.handle, seq, C.byref(n)))
        return n.value

    def reset(self, seq: int = -1) -> None:
        self.ctx.check(self.lib.qxc_kv_reset(self.handle, seq))

    def page_stats(self, seq: int = -1) -> tuple[int, int]:
        """(pages mapped by `seq`, or by all sequences when seq < 0; pages free)."""
        m, f = C.c_int32(), C.c_int32()
        self.ctx.check(self.lib.qxc_kv_page_stats(self.handle, seq, C.byref(m), C.byref(f)))
        return m.value, f.value

    def pool_tensor(self, key: bool = True):
        """Zero-copy torch view [layers][pool_pages][page_size][kv_heads][head_dim]
        of a paged arena's key (or value) pool (int16 for 16-bit storage)."""
        import torch
        p, n = C.c_void_p(), C.c_size_t()
        self.ctx.check(self.lib.qxc_kv_pool_buffer(self.handle, 1 if key else 0, C.byref(p), C.byref(n)))
        dt = self.key_dtype if key else self.value_dtype
        shape = (self.layers, self.paging.pool_pages, self.paging.page_size, self.hkv, self.d)

        class _View:
            __cuda_array_interface__ = {"shape": shape, "typestr": "<f4" if dt == F32 else "<i2",
                                        "data": (p.value, False), "version": 3, "strides": None}
        return torch.as_tensor(_View(), device=f"cuda:{self.ctx.device}")

    def trim(self, seq: int) -> None:
        """Return the pages of `seq` past its length to the pool (qxc_kv_trim)."""
        self.ctx.check(self.lib.qxc_kv_trim(self.handle, seq))

    def set_len(self, seq: int, length: int) -> None:
        self.ctx.check(self.lib.qxc_kv_set_len(self.handle, seq, length))

    def checkpoint(self, seq: int = 0) -> int:
        n = C.c_int32()
        self.ctx.check(self.lib.qxc_kv_checkpoint(self.handle, seq, C.byref(n)))
        return n.value

    def rollback(self, seq: int, sequence_len: int) -> None:
        self.ctx.check(self.lib.qxc_kv_rollback(self.handle, seq, sequence_len))

    def commit(self, seq: int, sequence_len: int, accepted_prefix: int) -> None:
        self.ctx.check(self.lib.qxc_kv_commit(self.handle, seq, sequence_len, accepted_prefix))

    # views and copies
    def key_buffer(self, seq: int, layer: int):
        p, n = C.c_void_p(), C.c_size_t()
        self.ctx.check(self.lib.qxc_kv_key_buffer(self.handle, seq, layer, C.byref(p), C.byref(n)))
        return p.value, n.value

    def value_buffer(self, seq: int, layer: int):
        p, n = C.c_void_p(), C.c_size_t()
        self.ctx.check(self.lib.qxc_kv_value_buffer(self.handle, seq, layer, C.byref(p), C.byref(n)))
        return p.value, n.value

    def tensor(self, seq: int, layer: int, key: bool = True):
        """Zero-copy torch view [capacity][kv_heads][head_dim] of one cache
        (int16 for 16-bit storage), through __cuda_array_interface__."""
        import torch
        ptr, nbytes = self.key_buffer(seq, layer) if key else self.value_buffer(seq, layer)
        dt = self.key_dtype if key else self.value_dtype
        typestr = "<f4" if dt == F32 else "<i2"

        class _View:
            __cuda_array_interface__ = {"shape": (self.capacity, self.hkv, self.d), "typestr": typestr,
                                        "data": (ptr, False), "version": 3, "strides": None}
        return torch.as_tensor(_View(), device=f"cuda:{self.ctx.device}")

    def read(self, seq: int, layer: int, begin: int, count: int):
        k = np.zeros((count, self.hkv, self.d), _np_dtype(self.key_dtype))
        v = np.zeros((count, self.hkv, self.d), _np_dtype(self.value_dtype))
        self.ctx.check(self.lib.qxc_kv_read(self.handle, seq, layer, begin, count, k.ctypes.data, v.ctypes.data))
        return k, v

    def write(self, seq: int, layer: int, begin: int, keys: np.ndarray | None, values: np.ndarray | None):
        count = (keys if keys is not None else values).shape[0]
        if keys is not None:
            keys = np.ascontiguousarray(keys, _np_dtype(self.key_dtype))
        if values is not None:
            values = np.ascontiguousarray(values, _np_dtype(self.value_dtype))
        self.ctx.check(self.lib.qxc_kv_write(self.handle, seq, layer, begin, count,
                                             None if keys is None else keys.ctypes.data,
                                             None if values is None else values.ctypes.data))

    # compute
    def _decode_args(self, q, k, v, out, positions, layer_begin, layer_count, seq_ids, q_dtype, in_dtype,
                     out_dtype, flags, split, q_rot_out, q_norm, k_norm):
        n = len(positions)
        pos = (C.c_int32 * n)(*[int(x) for x in positions])
        ids = (C.c_int32 * n)(*[int(x) for x in seq_ids]) if seq_ids is not None else None
        a = _lib.DecodeArgs(layer_begin, layer_count, n, ids, pos, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                            _ptr(q_rot_out), _ptr(q_norm), _ptr(k_norm), q_dtype, in_dtype, out_dtype, flags,
                            split)
        a._keep = (pos, ids)
        return a

    def decode(self, q, k, v, out, positions, layer_begin: int = 0, layer_count: int | None = None, seq_ids=None,
               q_dtype: int | None = None, in_dtype: int | None = None, out_dtype: int = F32, flags: int = 0,
               split: int = 0, q_rot_out=None, q_norm=None, k_norm=None) -> None:
        """Asynchronous decode step on device tensors (qxc_decode)."""
        layer_count = self.layers - layer_begin if layer_count is None else layer_count
        dflt = self.key_dtype if self.model == MODEL_QWEN3 else F32
        a = self._decode_args(q, k, v, out, positions, layer_begin, layer_count, seq_ids,
                              dflt if q_dtype is None else q_dtype, dflt if in_dtype is None else in_dtype,
                              out_dtype, flags, split, q_rot_out, q_norm, k_norm)
        self.ctx.check(self.lib.qxc_decode(self.ctx.handle, self.handle, C.byref(a)))

    def decode_verify(self, q, k, v, out, start: int, tokens: int, seq: int = 0, layer_begin: int = 0,
                      layer_count: int | None = None, q_dtype: int | None = None, in_dtype: int | None = None,
                      out_dtype: int = F32, flags: int = 0, split: int = 0, q_norm=None, k_norm=None) -> None:
        """K speculative tokens of one sequence in one call (qxc_decode_verify):
        rows start..start+tokens-1 appended, token t attending [0, start + t].
        q/out [tokens][layer_count][Hq*D], k/v [tokens][layer_count][Hkv*D] on
        the device; the reference's batched verifier attention stage."""
        layer_count = self.layers - layer_begin if layer_count is None else layer_count
        dflt = self.key_dtype if self.model == MODEL_QWEN3 else F32
        a = _lib.VerifyArgs(seq, layer_begin, layer_count, start, tokens, _ptr(q), _ptr(k), _ptr(v), _ptr(out),
                            _ptr(q_norm), _ptr(k_norm), dflt if q_dtype is None else q_dtype,
                            dflt if in_dtype is None else in_dtype, out_dtype, flags, split)
        self.ctx.check(self.lib.qxc_decode_verify(self.ctx.handle, self.handle, C.byref(a)))

    def attention_layer(self, hidden_in, hidden_out, input_norm, q_proj: "Q4Weights", k_proj: "Q4Weights",
                        v_proj: "Q4Weights", o_proj: "Q4Weights", position: int, seq: int = 0, layer: int = 0,
                        attention_out=None, flags: int = 0, split: int = 0) -> None:
        """The attention sub-layer of a Granite layer with Q4 weights for one
        token (qxc_attention_layer): RMSNorm, Q4 q/k/v, RoPE + append +
        attention, Q4 o-projection, residual; device tensors."""
        a = _lib.LayerArgs(seq, layer, position, _ptr(hidden_in), _ptr(hidden_out), _ptr(input_norm),
                           q_proj.ref(), k_proj.ref(), v_proj.ref(), o_proj.ref(), _ptr(attention_out), flags, split)
        self.ctx.check(self.lib.qxc_attention_layer(self.ctx.handle, self.handle, C.byref(a)))

    def attention_stack(self, hidden_in, hidden_out, layers, position: int, seq: int = 0, layer_begin: int = 0,
                        flags: int = 0, split: int = 0) -> None:
        """The attention sub-layers of len(layers) consecutive layers for one
        token (qxc_attention_stack, PreparedAttentionStack::encode): each
        entry of `layers` is a dict with "norm" (device [1024]) and "q", "k",
        "v", "o" (Q4Weights); hidden_out receives the last layer's output."""
        ws = (_lib.LayerWeights * len(layers))()
        for i, w in enumerate(layers):
            ws[i] = _lib.LayerWeights(_ptr(w["norm"]), w["q"].ref(), w["k"].ref(), w["v"].ref(), w["o"].ref())
        a = _lib.StackArgs(seq, layer_begin, len(layers), position, _ptr(hidden_in), _ptr(hidden_out), ws, flags,
                           split)
        self.ctx.check(self.lib.qxc_attention_stack(self.ctx.handle, self.handle, C.byref(a)))

    def verification_hashes(self, token: int, residuals, residual_stride: int, checkpoint_interval: int, digests,
                            seq: int = 0) -> None:
        """Per-token commitments (qxc_verification_hashes): digests[p] = state
        root of residual snapshot p (checkpoint positions, else zeros) || KV
        slot leaf of layer p-1 (zeros at p = 0), p in 0..layers; device
        tensors, the reference's encode_verification_hashes stage."""
        a = _lib.VerificationHashArgs(seq, token, _ptr(residuals), residual_stride, checkpoint_interval,
                                      _ptr(digests))
        self.ctx.check(self.lib.qxc_verification_hashes(self.ctx.handle, self.handle, C.byref(a)))

    def slot_hashes(self, digests, layer_begin: int, layer_count: int, token_begin: int, token_count: int,
                    seq: int = 0, layout: int = 0) -> None:
        """kv_leaf_hash_v1 of every (layer, token) slot of the range into the
        device tensor digests [layer_count][token_count][32]
        (qxc_kv_slot_hashes; layout: HASH_AUTO, HASH_PER_CHUNK or HASH_PER_SLOT)."""
        self.ctx.check(self.lib.qxc_kv_slot_hashes(self.ctx.handle, self.handle, seq, layer_begin, layer_count,
                                                   token_begin, token_count, _ptr(digests), layout))

    def decode_host(self, q: np.ndarray, k: np.ndarray, v: np.ndarray, positions, layer_begin: int = 0,
                    layer_count: int | None = None, seq_ids=None, q_dtype: int | None = None,
                    in_dtype: int | None = None, out_dtype: int = F32, flags: int = 0, split: int = 0,
                    out: np.ndarray | None = None, q_norm=None, k_norm=None) -> np.ndarray:
        """Synchronous decode step on host arrays (qxc_decode_host)."""
        layer_count = self.layers - layer_begin if layer_count is None else layer_count
        dflt = self.key_dtype if self.model == MODEL_QWEN3 else F32
        q_dtype = dflt if q_dtype is None else q_dtype
        in_dtype = dflt if in_dtype is None else in_dtype
        units = len(positions) * layer_count
        if out is None:
            out = np.zeros((units, self.hq * self.d), _np_dtype(out_dtype))
        q = np.ascontiguousarray(q, _np_dtype(q_dtype))
        k = np.ascontiguousarray(k, _np_dtype(in_dtype))
        v = np.ascontiguousarray(v, _np_dtype(in_dtype))
        a = self._decode_args(q, k, v, out, positions, layer_begin, layer_count, seq_ids, q_dtype, in_dtype,
                              out_dtype, flags, split, None, q_norm, k_norm)
        self.ctx.check(self.lib.qxc_decode_host(self.ctx.handle, self.handle, C.byref(a)))
        return out

    def prefill(self, q, k, v, out, length: int, seq: int = 0, layer: int = 0, out_dtype: int = F32,
                flags: int = 0) -> None:
        a = _lib.PrefillArgs(seq, layer, length, _ptr(q), _ptr(k), _ptr(v), _ptr(out), BF16, out_dtype, flags)
        self.ctx.check(self.lib.qxc_prefill(self.ctx.handle, self.handle, C.byref(a)))

    def decode_partials(self, q, k, v, partials, position: int, append: bool, seq: int = 0, layer: int = 0,
                        q_dtype: int | None = None, in_dtype: int | None = None, flags: int = 0, split: int = 0,
                        q_norm=None, k_norm=None) -> None:
        dflt = self.key_dtype if self.model == MODEL_QWEN3 else F32
        a = _lib.PartialArgs(seq, layer, position, int(bool(append)), _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm),
                             _ptr(k_norm), _ptr(partials), dflt if q_dtype is None else q_dtype,
                             dflt if in_dtype is None else in_dtype, flags, split)
        self.ctx.check(self.lib.qxc_decode_partials(self.ctx.handle, self.handle, C.byref(a)))


    def decode_exchange(self, q, k, v, out, position: int, append: bool, group: "PeerGroup", seq: int = 0,
                        layer: int = 0, out_dtype: int = F32, q_dtype: int | None = None,
                        in_dtype: int | None = None, flags: int = 0, split: int = 0, q_norm=None,
                        k_norm=None) -> None:
        """This rank's part of a KV-length split decode, exchanged with every
        rank over NVLink inside the split merge kernel (qxc_decode_exchange):
        out [q_heads][head_dim] holds the merged attention of all ranks."""
        dflt = self.key_dtype if self.model == MODEL_QWEN3 else F32
        a = _lib.PartialArgs(seq, layer, position, int(bool(append)), _ptr(q), _ptr(k), _ptr(v), _ptr(q_norm),
                             _ptr(k_norm), None, dflt if q_dtype is None else q_dtype,
                             dflt if in_dtype is None else in_dtype, flags, split)
        self.ctx.check(self.lib.qxc_decode_exchange(self.ctx.handle, self.handle, C.byref(a), group.handle,
                                                    _ptr(out), out_dtype))


# ---- qx-runtime (V1) mirror ---------------------------------------------------
class KvCache:
    """qx_runtime::KvCache (crates/qx-runtime/src/lib.rs:350-432): a static
    single-sequence fp32 Granite cache, resident on the GPU."""

    def __init__(self, max_context: int, ctx: Context | None = None):
        self.ctx = ctx or default_context()
        self.max_context = max_context
        self.arena = KvArena(self.ctx, MODEL_GRANITE, 1, 1, max_context, F32, F32)

    def __len__(self) -> int:
        return self.arena.len(0)

    def len(self) -> int:
        return self.arena.len(0)

    def is_empty(self) -> bool:
        return self.len() == 0

    def reset(self) -> None:
        self.arena.reset(0)

    def token(self, position: int):
        """Rotated key and value rows of one committed position (KvCache::token :417-431)."""
        if position >= self.len():
            raise QxError(_lib.ERR_POSITION,
                          f"KV position {position} is outside committed length {self.len()}")
        k, v = self.arena.read(0, 0, position, 1)
        return k.reshape(-1), v.reshape(-1)


def granite_attention_decode(query, key, value, position: int, cache: KvCache) -> np.ndarray:
    """qx_runtime::granite_attention_decode (crates/qx-runtime/src/lib.rs:444-452):
    RoPE q/k at `position`, append k/v (position must equal cache length),
    attend over the cache; returns the [1024] f32 output."""
    q = np.ascontiguousarray(query, np.float32).reshape(-1)
    k = np.ascontiguousarray(key, np.float32).reshape(-1)
    v = np.ascontiguousarray(value, np.float32).reshape(-1)
    if q.size != HIDDEN or k.size != KV_HEADS * HEAD_DIM or v.size != KV_HEADS * HEAD_DIM:
        raise QxError(_lib.ERR_INVALID_ARG, "query must hold 1024 and key/value 512 f32 values")
    out = np.zeros(HIDDEN, np.float32)
    ctx = cache.ctx
    ctx.check(ctx.lib.qxc_granite_attention_decode(ctx.handle, cache.arena.handle, q.ctypes.data, k.ctypes.data,
                                                   v.ctypes.data, int(position), out.ctypes.data))
    return out


def apply_granite_rope(query: np.ndarray, key: np.ndarray, position: int, ctx: Context | None = None) -> None:
    """qx_runtime::apply_granite_rope (crates/qx-runtime/src/lib.rs:434-442), in place."""
    ctx = ctx or default_context()
    if query.dtype != np.float32 or key.dtype != np.float32 or query.size != HIDDEN or key.size != 512:
        raise QxError(_lib.ERR_INVALID_ARG, "query f32[1024] and key f32[512] required")
    if not (query.flags.c_contiguous and key.flags.c_contiguous):
        raise QxError(_lib.ERR_INVALID_ARG, "arrays must be contiguous")
    ctx.check(ctx.lib.qxc_apply_granite_rope(ctx.handle, query.ctypes.data, key.ctypes.data, int(position)))


# ---- qx-runtime-v2 KV plan mirror ------------------------------------------------
class KvPrecision(enum.Enum):
    """qx_format::KvPrecision (crates/qx-format/src/lib.rs:136-141) plus bf16 for B200."""
    Fp32 = (F32, F32)
    Fp32KFp16V = (F32, F16)
    Fp16KFp32V = (F16, F32)
    Fp16 = (F16, F16)
    Bf16 = (BF16, BF16)


@dataclass
class ExecutionPlan:
    """KV part of qx_runtime_v2::ExecutionPlan (crates/qx-runtime-v2/src/lib.rs:6566-6656)."""
    context: int
    kv_precision: KvPrecision
    kv_bytes: int
    layers: int = LAYERS

    @staticmethod
    def granite(context: int) -> "ExecutionPlan":
        return ExecutionPlan.granite_with_kv_precision(context, KvPrecision.Fp32)

    @staticmethod
    def granite_with_kv_precision(context: int, precision: KvPrecision, sequences: int = 1) -> "ExecutionPlan":
        lib = _lib.load()
        kd, vd = precision.value
        desc = _lib.KvDesc(MODEL_GRANITE, LAYERS, sequences, context, kd, vd, 0)
        kb, vb = C.c_size_t(), C.c_size_t()
        st = lib.qxc_kv_bytes(C.byref(desc), C.byref(kb), C.byref(vb))
        if st != _lib.OK:
            raise QxError(st, f"context {context} must be in 1..=4096")
        plan = ExecutionPlan(context, precision, kb.value + vb.value)
        plan._key, plan._value = kb.value, vb.value
        return plan

    def kv_key_bytes(self) -> int:
        return self._key

    def kv_value_bytes(self) -> int:
        return self._value

    def allocate(self, ctx: Context, sequences: int = 1) -> KvArena:
        """GpuRuntimeBuffers::new's KV allocation (qx-runtime-v2 lib.rs:6774-6811)."""
        kd, vd = self.kv_precision.value
        return KvArena(ctx, MODEL_GRANITE, self.layers, sequences, self.context, kd, vd)


class Q4Weights:
    """A Q4 matrix on the device in the reference's row-major group-32 layout
    (qx-quant QuantizedTensor): `codes` [rows][cols/32][16] uint8 and
    `scales` [rows][cols/32] FP16 bits, as torch tensors (or anything with
    __cuda_array_interface__ / data_ptr())."""

    def __init__(self, codes, scales, rows: int, cols: int):
        self.codes, self.scales, self.rows, self.cols = codes, scales, rows, cols

    def ref(self) -> "_lib.Q4Matrix":
        return _lib.Q4Matrix(self.rows, self.cols, _ptr(self.codes), _ptr(self.scales))


def q4_mat_vec(ctx: "Context", w: Q4Weights, x, y, rms_weight=None) -> None:
    """y = W x, or W rms_norm(x, rms_weight) (qxc_q4_mat_vec); device tensors."""
    m = w.ref()
    ctx.check(ctx.lib.qxc_q4_mat_vec(ctx.handle, C.byref(m), _ptr(x), _ptr(rms_weight), _ptr(y)))
