"""GPU test of qxc_granite_decode_static_scratch, the decode entry point that
allocates nothing at call time.

It exists for callers that own all device memory themselves (a runtime that
plans one arena before generation and forbids allocation afterwards, or a
host with its own memory pool), so the library may not cudaMalloc the
split-KV scratch behind their back; that scratch lives in a static device
array instead. These tests call it through the C ABI on caches held in
caller-owned torch memory and check it against the CPU oracle (outputs within
the KV type's gate, the appended row bit-exact) and against the regular
qxc_decode, on two decode steps in a row, for every KV precision it accepts
and for split counts the regular path never merges inside the decode kernel
(it hands more than 8 to a separate merge kernel). This file is named to be
collected last.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import as_kv, granite_inputs, normwise
from qx_b200 import BF16, F16, F32, MODEL_GRANITE, KvArena
from qx_b200 import _lib
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu

PAIRS = [(F32, F32), (F32, F16), (F16, F32), (F16, F16), (BF16, BF16)]


def _tol(kd, vd):
    return 1e-5 if kd == F32 and vd == F32 else 2e-2


def _static_decode(lib, kc, vc, kd, vd, capacity, position, q, k, v, out, stream, split=0, err=None):
    a = _lib.StaticDecodeArgs(kc.data_ptr(), vc.data_ptr(), capacity, kd, vd, position, q.data_ptr(),
                              k.data_ptr(), v.data_ptr(), out.data_ptr(), F32, F32, F32, 0, split,
                              err.data_ptr() if err is not None else None)
    msg = C.create_string_buffer(256)
    st = lib.qxc_granite_decode_static_scratch(C.byref(a), C.c_void_p(stream), msg, len(msg))
    return st, msg.value.decode()


def _torch_cache(capacity, dtype, rows):
    """A caller-owned cache tensor [capacity][8][64] holding `rows` (f32 or
    16-bit patterns, as the arena stores them)."""
    import torch
    t = torch.zeros(capacity, 8, 64, dtype=torch.float32 if dtype == F32 else torch.int16, device="cuda")
    bits = as_kv(rows, dtype)
    t[:rows.shape[0]] = torch.from_numpy(bits if dtype == F32 else bits.view(np.int16)).cuda()
    return t


def _row_bits(t, pos, dtype):
    x = t[pos].cpu().numpy()
    return x.view(np.uint32) if dtype == F32 else x.view(np.uint16)


def _oracle_row_bits(rows, dtype):
    return rows.view(np.uint32) if dtype == F32 else rows.view(np.uint16)


@pytest.mark.parametrize("kd,vd", PAIRS)
@pytest.mark.parametrize("prefix,split", [(1500, 0), (700, 64), (1918, 64), (4094, 0)])
def test_static_scratch_decode_matches_oracle(gpu_ctx, oracle, kd, vd, prefix, split):
    """Two calls in a row on the shared static scratch: outputs within the
    KV type's gate of the oracle and equal to qxc_decode's, new rows
    bit-exact. (700, 64) gives 11 splits and (1918, 64) 30 (the most the
    array holds), both merged inside the decode kernel."""
    import torch
    lib = _lib.load()
    torch.cuda.set_device(0)
    capacity = 4096
    _, _, _, kc, vc = granite_inputs(0x7700 + prefix + 16 * kd + vd, prefix, capacity)
    oc = oracle.KvCache(capacity, kd, vd)
    oc.keys[:prefix], oc.values[:prefix] = as_kv(kc, kd), as_kv(vc, vd)
    oc.length.value = prefix
    # the regular path: arena + qxc_decode, with the same split
    arena = KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, capacity, kd, vd)
    arena.write(0, 0, 0, as_kv(kc, kd), as_kv(vc, vd))
    arena.set_len(0, prefix)
    # the allocation-free path: the caller owns the cache tensors
    key_cache = _torch_cache(capacity, kd, kc)
    value_cache = _torch_cache(capacity, vd, vc)
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for step in range(2):
        pos = prefix + step
        qn = syn.normal(0x7800 + step + prefix, (1024,))
        kn = syn.normal(0x7900 + step + prefix, (512,))
        vn = syn.normal(0x7A00 + step + prefix, (512,))
        st, ref = oracle.granite_attention_decode(qn, kn, vn, pos, oc)
        assert st == 0
        q, k, v = (torch.from_numpy(x).cuda() for x in (qn, kn, vn))
        reg = torch.zeros(1, 1024, device="cuda")
        if kd == vd and kd in (BF16, F16):
            # 16-bit Granite runs on the tensor-core kernel in qxc_decode; the
            # static path keeps the CUDA-core kernel (same gate, other roundings)
            arena.decode(q.view(1, -1), k.view(1, -1), v.view(1, -1), reg, [pos])
        else:
            arena.decode(q.view(1, -1), k.view(1, -1), v.view(1, -1), reg, [pos], split=split)
        gpu_ctx.sync()
        out = torch.zeros(1024, device="cuda")
        st, msg = _static_decode(lib, key_cache, value_cache, kd, vd, capacity, pos, q, k, v, out, stream,
                                 split=split, err=err)
        assert st == _lib.OK, msg
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert normwise(got, ref) <= _tol(kd, vd), (kd, vd, prefix, split, step)
        assert normwise(got, reg.cpu().numpy()[0]) <= _tol(kd, vd)
        if kd == F32 and vd == F32:
            assert normwise(got, reg.cpu().numpy()[0]) <= 1e-6
        assert int(err.item()) == 0
        assert np.array_equal(_row_bits(key_cache, pos, kd), _oracle_row_bits(oc.keys[pos], kd))
        assert np.array_equal(_row_bits(value_cache, pos, vd), _oracle_row_bits(oc.values[pos], vd))
    arena.close()


def test_static_scratch_rejects_requests_beyond_its_size(gpu_ctx):
    import torch
    lib = _lib.load()
    torch.cuda.set_device(0)
    capacity = 4096
    key_cache = torch.zeros(capacity, 8, 64, device="cuda")
    value_cache = torch.zeros(capacity, 8, 64, device="cuda")
    q = torch.zeros(1024, device="cuda")
    kv = torch.zeros(512, device="cuda")
    out = torch.full((1024,), 7.0, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    # 64-position splits over 4096 slots need 64 x 8 partial sets: too many
    st, msg = _static_decode(lib, key_cache, value_cache, F32, F32, capacity, capacity - 1, q, kv, kv, out, stream,
                             split=64)
    assert st == _lib.ERR_INVALID_ARG
    assert "exceeds the static scratch" in msg
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched
    st, msg = _static_decode(lib, key_cache, value_cache, F32, F32, capacity, capacity - 1, q, kv, kv, out, stream)
    assert st == _lib.OK, msg
    torch.cuda.synchronize()
    assert torch.all(out == 0.0)
