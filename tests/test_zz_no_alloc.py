"""GPU test of qxc_granite_decode_static_scratch, the decode entry point that
allocates nothing at call time.

It exists for callers that own all device memory themselves (a runtime that
plans one arena before generation and forbids allocation afterwards, or a
host with its own memory pool), so the library may not cudaMalloc the
split-KV scratch behind their back; that scratch lives in a static device
array instead. This test calls it through the C ABI on a cache held in
caller-owned torch memory and checks it against the regular qxc_decode, on
two decode steps in a row. This file is named to be collected last.
"""
import ctypes as C

import numpy as np
import pytest

from helpers import granite_inputs, normwise
from qx_b200 import F32, MODEL_GRANITE, KvArena
from qx_b200 import _lib
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def _static_decode(lib, kc, vc, capacity, position, q, k, v, out, stream, split=0, err=None):
    a = _lib.StaticDecodeArgs(kc.data_ptr(), vc.data_ptr(), capacity, F32, F32, position, q.data_ptr(),
                              k.data_ptr(), v.data_ptr(), out.data_ptr(), F32, F32, F32, 0, split,
                              err.data_ptr() if err is not None else None)
    msg = C.create_string_buffer(256)
    st = lib.qxc_granite_decode_static_scratch(C.byref(a), C.c_void_p(stream), msg, len(msg))
    return st, msg.value.decode()


def test_static_scratch_decode_matches_regular_decode(gpu_ctx):
    import torch
    lib = _lib.load()
    torch.cuda.set_device(0)
    capacity, prefix = 2048, 1500
    _, _, _, kc, vc = granite_inputs(0x7700, prefix, capacity)
    # regular path: arena + qxc_decode
    arena = KvArena(gpu_ctx, MODEL_GRANITE, 1, 1, capacity, F32, F32)
    arena.write(0, 0, 0, kc, vc)
    arena.set_len(0, prefix)
    # allocation-free path: the caller owns the cache tensors
    key_cache = torch.zeros(capacity, 8, 64, device="cuda")
    value_cache = torch.zeros(capacity, 8, 64, device="cuda")
    key_cache[:prefix] = torch.from_numpy(kc).cuda()
    value_cache[:prefix] = torch.from_numpy(vc).cuda()
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for step in range(2):  # two calls in a row on the same static scratch
        pos = prefix + step
        q = torch.from_numpy(syn.normal(0x7800 + step, (1024,))).cuda()
        k = torch.from_numpy(syn.normal(0x7900 + step, (512,))).cuda()
        v = torch.from_numpy(syn.normal(0x7A00 + step, (512,))).cuda()
        ref = torch.zeros(1, 1024, device="cuda")
        arena.decode(q.view(1, -1), k.view(1, -1), v.view(1, -1), ref, [pos])
        gpu_ctx.sync()
        out = torch.zeros(1024, device="cuda")
        st, msg = _static_decode(lib, key_cache, value_cache, capacity, pos, q, k, v, out, stream, err=err)
        assert st == _lib.OK, msg
        torch.cuda.synchronize()
        assert normwise(out.cpu().numpy(), ref.cpu().numpy()[0]) <= 1e-5
        assert int(err.item()) == 0
        gk, gv = arena.read(0, 0, pos, 1)
        assert np.array_equal(key_cache[pos].cpu().numpy(), gk[0])
        assert np.array_equal(value_cache[pos].cpu().numpy(), gv[0])


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
    st, msg = _static_decode(lib, key_cache, value_cache, capacity, capacity - 1, q, kv, kv, out, stream, split=64)
    assert st == _lib.ERR_INVALID_ARG
    assert "exceeds the static scratch" in msg
    torch.cuda.synchronize()
    assert torch.all(out == 7.0)  # nothing was launched
    st, msg = _static_decode(lib, key_cache, value_cache, capacity, capacity - 1, q, kv, kv, out, stream)
    assert st == _lib.OK, msg
    torch.cuda.synchronize()
    assert torch.all(out == 0.0)
