"""CPU tests of the C ABI boundary: the library loads, exports every symbol
include/*.h declares, and its host-only logic (KV byte plan, argument
checks) behaves like the reference. No call here touches a GPU."""
import ctypes as C

import pytest

from qx_b200 import _lib
from qx_b200.runtime import ExecutionPlan, KvPrecision, QxError


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.load()
    names = _lib.header_symbols()
    assert len(names) >= 25
    missing = [n for n in names if not hasattr(lib, n)]
    assert missing == []
    assert lib.qxc_abi_version() == 1


def test_status_strings():
    lib = _lib.load()
    assert lib.qxc_status_string(_lib.ERR_POSITION) == b"KV position error"
    assert lib.qxc_status_string(_lib.OK) == b"ok"


def test_kv_precision_is_a_first_class_memory_plan_dimension():
    # qx-runtime-v2 lib.rs:7203-7221 (expected values read from the reference test)
    import json, os
    kats = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "consensus_math_kats.json")))
    want = kats["kv_bytes_context_512"]
    fp32 = ExecutionPlan.granite_with_kv_precision(512, KvPrecision.Fp32)
    asym = ExecutionPlan.granite_with_kv_precision(512, KvPrecision.Fp32KFp16V)
    fp16 = ExecutionPlan.granite_with_kv_precision(512, KvPrecision.Fp16)
    assert fp32.kv_bytes == want["fp32"] == 50_331_648
    assert asym.kv_bytes == want["asymmetric"]
    assert fp16.kv_bytes == want["fp16"]
    assert fp32.kv_key_bytes() == asym.kv_key_bytes()
    assert asym.kv_value_bytes() * 2 == fp32.kv_value_bytes()
    assert fp16.kv_bytes * 2 == fp32.kv_bytes


@pytest.mark.parametrize("context", [0, 4097])
def test_context_must_be_in_range(context):
    with pytest.raises(QxError) as e:
        ExecutionPlan.granite(context)
    assert "must be in 1..=4096" in str(e.value)


def test_kv_bytes_rejects_bad_descriptors():
    lib = _lib.load()
    kb, vb = C.c_size_t(), C.c_size_t()
    bad = [
        _lib.KvDesc(7, 1, 1, 16, 0, 0, 0),            # unknown model
        _lib.KvDesc(0, 0, 1, 16, 0, 0, 0),            # no layers
        _lib.KvDesc(1, 1, 1, 16, _lib.F32, _lib.F32, 0),  # Qwen needs 16-bit KV
        _lib.KvDesc(0, 1, 1, 16, 9, 0, 0),            # unknown dtype
    ]
    for d in bad:
        assert lib.qxc_kv_bytes(C.byref(d), C.byref(kb), C.byref(vb)) != _lib.OK
    ok = _lib.KvDesc(1, 48, 1, 32768, _lib.BF16, _lib.BF16, 0)
    assert lib.qxc_kv_bytes(C.byref(ok), C.byref(kb), C.byref(vb)) == _lib.OK
    assert kb.value == vb.value == 48 * 32768 * 4 * 128 * 2


def test_null_arguments_are_rejected_without_a_gpu():
    lib = _lib.load()
    assert lib.qxc_init(0, None) == _lib.ERR_INVALID_ARG
    assert lib.qxc_sync(None) == _lib.ERR_INVALID_ARG
    assert lib.qxc_decode(None, None, None) == _lib.ERR_INVALID_ARG


def _auto_split(slots, attend, units, max_splits, tile):
    lib = _lib.load()
    a = (C.c_int32 * len(attend))(*attend)
    return lib.qxc_auto_split(slots, a, len(attend), units, max_splits, tile)


def test_automatic_split_keeps_the_measured_optima():
    """qxc_auto_split is the decode calls' own split choice (host only).
    Each case pins a split that a sweep on a B200 found best: config 1 at
    2048 rows (384 CTAs in one wave of 444 slots), config 3 at 896 (148 CTAs
    for 148 slots), the Q4 layer's one-layer decode at 256, config 0 at 64."""
    assert [_auto_split(444, [n], 24 * 8, 1024, 64) for n in (4033, 4064, 4096)] == [2048] * 3
    assert _auto_split(148, [32768], 4, 1024, 128) == 896
    assert _auto_split(444, [4064], 8, 1024, 64) == 256
    assert _auto_split(444, [512], 8, 1024, 64) == 64


def test_automatic_split_leaves_large_batches_unsplit():
    """A batch whose unsplit work fills the slots at least twice per longest
    item runs unsplit: config 4's 256 sequences and its first 8 (measured
    62.1k and 54.4k tok/s unsplit against 48.1k and 45.1k split). Its first
    4 still split."""
    from qx_b200 import synthetic as syn
    lengths = [int(x) for x in syn.uniform_int(0x51580400, 256, 128, 4096)]
    top = lambda xs: -(-max(xs) // 128) * 128  # noqa: E731
    assert _auto_split(148, lengths, 24 * 4, 1024, 128) == top(lengths)
    assert _auto_split(148, lengths[:8], 24 * 4, 1024, 128) == top(lengths[:8])
    assert _auto_split(148, lengths[:4], 24 * 4, 1024, 128) < top(lengths[:4])


def test_automatic_split_rejects_bad_arguments():
    assert _auto_split(0, [5], 1, 1, 64) == 0
    assert _auto_split(148, [0], 1, 1, 64) == 0
    assert _auto_split(148, [100], 0, 1, 64) == 0


def test_every_declared_entry_point_has_a_python_signature():
    """The ctypes mirror declares argument and result types for every
    function include/*.h declares, so no call goes through ctypes' default
    int conversion of pointers and sizes."""
    lib = _lib.load()
    untyped = [n for n in _lib.header_symbols() if getattr(lib, n).argtypes is None]
    assert untyped == []
