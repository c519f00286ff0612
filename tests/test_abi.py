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
