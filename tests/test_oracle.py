"""CPU tests of the oracle against the reference's own known answers
(crates/qx-consensus-math/src/lib.rs:213-330, crates/qx-runtime/src/lib.rs:2873-2902)."""
import json
import os
import struct

import numpy as np
import pytest

from helpers import normwise
from qx_b200 import synthetic as syn

HERE = os.path.dirname(os.path.abspath(__file__))
KATS = json.load(open(os.path.join(HERE, "golden", "consensus_math_kats.json")))


def bits(f: float) -> int:
    return struct.unpack("<I", struct.pack("<f", f))[0]


def test_inverse_frequency_table(oracle):
    lib = oracle.lib()
    assert [lib.qxo_granite_inverse_frequency_bits(i) for i in range(32)] == KATS["granite_inverse_frequency_bits"]


def test_exp_golden_bits(oracle):
    got = [bits(oracle.exp_f32(x)) for x in KATS["exp"]["inputs"]]
    assert got == KATS["exp"]["bits"]


def test_rsqrt_golden_bits(oracle):
    got = [bits(oracle.rsqrt_f32(x)) for x in KATS["rsqrt"]["inputs"]]
    assert got == KATS["rsqrt"]["bits"]


def test_rope_sin_cos_golden_bits(oracle):
    for case in KATS["granite_rope_sin_cos"]:
        s, c = oracle.granite_rope_sin_cos(case["position"], case["pair"])
        assert (bits(s), bits(c)) == (case["sine_bits"], case["cosine_bits"])


def test_error_bounds(oracle):
    lib = oracle.lib()
    b = KATS["error_bounds"]
    assert lib.qxo_exp_worst_relative_error() <= b["exp_worst_relative"]
    assert lib.qxo_rsqrt_worst_relative_error() <= b["rsqrt_worst_relative"]
    assert lib.qxo_rope_worst_absolute_error() <= b["rope_worst_absolute"]


def test_special_values(oracle):
    # special_values_are_rejected_or_clamped (qx-consensus-math lib.rs:256-264)
    assert oracle.exp_f32(-100.0) == 0.0
    assert oracle.exp_f32(100.0) == np.finfo(np.float32).max
    assert oracle.exp_f32(float("nan")) is None
    assert oracle.rsqrt_f32(0.0) is None
    assert oracle.rsqrt_f32(-1.0) is None
    assert oracle.granite_rope_sin_cos(5000, 0) is None  # angle > 4096


def test_reduce_simd32_order(oracle):
    lanes = np.array([1e8] + [1.0] * 31, np.float32)
    # the tree order (16,8,4,2,1) differs from a sequential sum here
    t = lanes.astype(np.float32).copy()
    for off in (16, 8, 4, 2, 1):
        t[:off] = t[:off] + t[off:2 * off]
    assert oracle.reduce_simd32(lanes) == t[0]


def test_grouped_query_attention_uses_the_matching_kv_head(oracle):
    cache = oracle.KvCache(4)
    q = np.zeros(1024, np.float32)
    k = np.zeros(512, np.float32)
    v = np.zeros(512, np.float32)
    for h in range(8):
        v[h * 64:(h + 1) * 64] = h + 1
    st, out = oracle.granite_attention_decode(q, k, v, 0, cache)
    assert st == oracle.OK and len(cache) == 1
    for qh in range(16):
        assert np.all(out[qh * 64:(qh + 1) * 64] == qh // 2 + 1)


def test_kv_cache_rejects_non_sequential_positions(oracle):
    cache = oracle.KvCache(2)
    z = np.zeros(1024, np.float32)
    st, _ = oracle.granite_attention_decode(z, z[:512], z[:512], 1, cache)
    assert st == oracle.ERR_POSITION and len(cache) == 0


def test_kv_cache_rejects_full_cache(oracle):
    cache = oracle.KvCache(1)
    z = np.zeros(1024, np.float32)
    assert oracle.granite_attention_decode(z, z[:512], z[:512], 0, cache)[0] == oracle.OK
    assert oracle.granite_attention_decode(z, z[:512], z[:512], 1, cache)[0] == oracle.ERR_POSITION


def test_hierarchical_matches_plain_closely(oracle):
    from helpers import granite_inputs, normwise
    q, k, v, kc, vc = granite_inputs(0x51580000, 300, 512)
    outs = []
    for hier in (False, True):
        c = oracle.KvCache(512)
        c.keys[:300], c.values[:300] = kc, vc
        c.length.value = 300
        st, o = oracle.granite_attention_decode(q, k, v, 300, c, hierarchical=hier)
        assert st == 0
        outs.append(o)
    assert normwise(outs[1], outs[0]) < 1e-5


def test_hierarchical_rejects_beyond_512(oracle):
    q, k, v = (np.zeros(n, np.float32) for n in (1024, 512, 512))
    c = oracle.KvCache(600)
    c.length.value = 512
    st, _ = oracle.granite_attention_decode(q, k, v, 512, c, hierarchical=True)
    assert st == oracle.ERR_INVALID_ARG  # the reference slices partials[..17] and panics


def test_prefill_equals_iterated_decode(oracle):
    from qx_b200 import synthetic as syn
    L = 70
    q = syn.to_bf16_bits(syn.normal(1, (L, 16, 64), 0.5))
    k = syn.to_bf16_bits(syn.normal(2, (L, 8, 64), 0.5))
    v = syn.to_bf16_bits(syn.normal(3, (L, 8, 64), 0.5))
    st, kc, vc, out = oracle.granite_prefill(q, k, v, oracle.BF16, oracle.BF16, threads=4)
    assert st == 0
    cache = oracle.KvCache(L, oracle.BF16, oracle.BF16)
    for p in range(L):
        st, o = oracle.granite_attention_decode(syn.bf16_bits_to_f32(q[p]), syn.bf16_bits_to_f32(k[p]),
                                                syn.bf16_bits_to_f32(v[p]), p, cache)
        assert st == 0
        assert np.array_equal(o, out[p].reshape(-1))
    assert np.array_equal(cache.keys, kc) and np.array_equal(cache.values, vc)


def test_qwen_oracle_f16_matches_written_reference_shape(oracle):
    from qx_b200 import synthetic as syn
    q = syn.to_f16_bits(syn.normal(5, (32, 128)))
    k = syn.to_f16_bits(syn.normal(6, (4, 128)))
    ones = np.ones(128, np.float32)
    qo, ko = oracle.qwen_qk_norm_rope(q, k, ones, ones, 37, oracle.F16)
    # RMS-normalised rows have unit RMS before rotation; rotation keeps the norm
    qf = qo.view(np.float16).astype(np.float32).reshape(32, 128)
    assert np.allclose(np.sqrt((qf ** 2).mean(axis=1)), 1.0, atol=3e-3)
    kc = syn.to_f16_bits(syn.normal(7, (64, 4, 128)))
    vc = syn.to_f16_bits(syn.normal(8, (64, 4, 128)))
    out, _ = oracle.qwen_gqa_attention(qo, kc, vc, 64, oracle.F16)
    assert np.all(np.isfinite(out))


@pytest.mark.parametrize("threads", [1, 3])
def test_decode_many_threads_identical(oracle, threads):
    from helpers import granite_inputs
    caches, qs, ks, vs = [], [], [], []
    for u in range(5):
        q, k, v, kc, vc = granite_inputs(100 + u, 40 + u, 64)
        c = oracle.KvCache(64)
        c.keys[:40 + u], c.values[:40 + u] = kc, vc
        c.length.value = 40 + u
        caches.append(c)
        qs.append(q), ks.append(k), vs.append(v)
    worst, outs = oracle.granite_decode_many(qs, ks, vs, [40 + u for u in range(5)], caches, threads=threads)
    assert worst == 0
    for u in range(5):
        c = oracle.KvCache(64)
        _, _, _, kc, vc = granite_inputs(100 + u, 40 + u, 64)
        c.keys[:40 + u], c.values[:40 + u] = kc, vc
        c.length.value = 40 + u
        st, o = oracle.granite_attention_decode(qs[u], ks[u], vs[u], 40 + u, c)
        assert np.array_equal(o, outs[u])


# ---- the Q4 attention sub-layer (qx-runtime-v2 CpuQ4Reference::step) ----------------
def test_q4_quantizer_follows_pack_scaled(oracle):
    """qx-quant QuantizedTensor::quantize / pack_scaled: scale = max|x|/7
    as FP16, codes round-half-away(x / scale) clamped to [-7, 7] + 7."""
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((6, 96)) * 0.1).astype(np.float32)
    w[2, 32:64] = 0.0  # an all-zero group takes scale 1.0
    m = oracle.Q4Matrix(w)
    scales = m.scales.view(np.float16).astype(np.float32)
    for r in range(6):
        for g in range(3):
            grp = w[r, g * 32:(g + 1) * 32]
            mx = np.abs(grp).max()
            expect = np.float32(np.float16(mx / np.float32(7.0))) if mx > 0 else np.float32(1.0)
            assert scales[r, g] == expect
            lo = m.codes[r, g] & 0xF
            hi = m.codes[r, g] >> 4
            codes = np.empty(32, np.int32)
            codes[0::2], codes[1::2] = lo, hi
            q = grp / scales[r, g]
            ref = np.clip(np.sign(q) * np.floor(np.abs(q) + 0.5), -7, 7).astype(np.int32) + 7
            assert np.array_equal(codes, ref)


def test_q4_mat_vec_and_rms_against_float64(oracle):
    rng = np.random.default_rng(6)
    m = oracle.Q4Matrix((rng.standard_normal((40, 1024)) * 0.05).astype(np.float32))
    x = rng.standard_normal(1024).astype(np.float32)
    scales = m.scales.view(np.float16).astype(np.float64)
    codes = np.empty((40, 1024), np.float64)
    for g in range(32):
        for i in range(32):
            c = (m.codes[:, g, i // 2] >> ((i & 1) * 4)) & 0xF
            codes[:, g * 32 + i] = (c.astype(np.float64) - 7.0) * scales[:, g]
    y = m.mat_vec(x)
    assert np.abs(y - codes @ x.astype(np.float64)).max() <= 1e-5 * np.abs(codes @ x).max()
    w = (1.0 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    st, xn = oracle.rms_norm_simd(x, w)
    assert st == 1
    ref = x.astype(np.float64) / np.sqrt((x.astype(np.float64) ** 2).mean() + 1e-6) * w
    assert np.abs(xn - ref).max() <= 2e-6 * np.abs(ref).max()


def test_attention_layer_oracle_composes_its_parts(oracle):
    """granite_attention_layer = rms -> q/k/v -> decode -> o -> fma residual."""
    rng = np.random.default_rng(7)
    W = [oracle.Q4Matrix((rng.standard_normal(s) * 0.05).astype(np.float32))
         for s in ((1024, 1024), (512, 1024), (512, 1024), (1024, 1024))]
    norm = (1.0 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    h = rng.standard_normal(1024).astype(np.float32)
    c1, c2 = oracle.KvCache(8), oracle.KvCache(8)
    st, out, att = oracle.granite_attention_layer(h, norm, *W, 0, c1)
    assert st == 0
    _, xn = oracle.rms_norm_simd(h, norm)
    q, k, v = W[0].mat_vec(xn), W[1].mat_vec(xn), W[2].mat_vec(xn)
    st2, att2 = oracle.granite_attention_decode(q, k, v, 0, c2)
    assert st2 == 0 and np.array_equal(att, att2)
    o = W[3].mat_vec(att2)
    assert np.array_equal(out, (np.float32(0.22) * o.astype(np.float64) + h).astype(np.float32)) or \
        np.abs(out - (0.22 * o.astype(np.float64) + h)).max() <= 1e-6


def test_cpu_rotate_heads_is_the_no_fma_pair(oracle):
    """cpu_rotate_heads (qx-runtime-v2 lib.rs:4957-4970): left*cos - right*sin
    and left*sin + right*cos, each product and sum rounded on its own (float32
    numpy arithmetic rounds every operation), with the pinned sin/cos."""
    import ctypes as C
    x = syn.normal(0x9100, (24 * 64,))
    for position in (0, 1, 7, 511, 4095):
        got = x.copy()
        assert oracle.lib().qxo_cpu_rotate_heads(oracle._fp(got), 24, position) == 0
        s = np.zeros(32, np.float32)
        c = np.zeros(32, np.float32)
        for pair in range(32):
            ss, cc = C.c_float(), C.c_float()
            assert oracle.lib().qxo_granite_rope_sin_cos(position, pair, C.byref(ss), C.byref(cc)) == 1
            s[pair], c[pair] = ss.value, cc.value
        h = x.reshape(24, 64)
        left, right = h[:, :32], h[:, 32:]
        exp = np.concatenate([left * c - right * s, left * s + right * c], axis=1).reshape(-1)
        assert np.array_equal(got.view(np.uint32), exp.view(np.uint32))
        # rotate_heads (fma) differs from it in the last bits only
        fma = x.copy()
        assert oracle.lib().qxo_rotate_heads(oracle._fp(fma), 24, position) == 0
        assert np.abs(fma - got).max() <= 4e-7 * np.abs(x).max() * 4


def test_attention_layer_cpu_twin(oracle):
    """The V2 CPU twin (CpuQ4Reference::step) against the V2 GPU stage's form:
    the value rows are bit-identical (no RoPE on v), the key rows differ only
    by the RoPE rounding, outputs agree within 1e-5 normwise over 40 steps;
    the twin stops past 512 positions, as the reference's partials slice."""
    rng = np.random.default_rng(11)
    W = [oracle.Q4Matrix((rng.standard_normal(s) * 0.05).astype(np.float32))
         for s in ((1024, 1024), (512, 1024), (512, 1024), (1024, 1024))]
    norm = (1.0 + 0.1 * rng.standard_normal(1024)).astype(np.float32)
    cap, prefix = 520, 470
    kc = syn.normal(0x9200, (prefix, 8, 64))
    vc = syn.normal(0x9201, (prefix, 8, 64))
    gpu_form, twin = oracle.KvCache(cap), oracle.KvCache(cap)
    for c in (gpu_form, twin):
        c.keys[:prefix], c.values[:prefix] = kc, vc
        c.length.value = prefix
    worst = 0.0
    for t in range(42):
        h = syn.normal(0x9300 + t, (1024,))
        st, out, att = oracle.granite_attention_layer(h, norm, *W, prefix + t, gpu_form)
        st2, out2, att2 = oracle.granite_attention_layer(h, norm, *W, prefix + t, twin, cpu_twin=True)
        assert st == 0 and st2 == 0
        worst = max(worst, normwise(att2, att), normwise(out2, out))
    assert worst <= 1e-5
    n = prefix + 42
    assert np.array_equal(twin.values[:n].view(np.uint32), gpu_form.values[:n].view(np.uint32))
    assert not np.array_equal(twin.keys[prefix:n], gpu_form.keys[prefix:n])
    assert np.abs(twin.keys[:n] - gpu_form.keys[:n]).max() <= 1e-5
    # position 512 makes the twin attend over 513 rows: its 16 x 32 value chunks end at 512
    st, _, _ = oracle.granite_attention_layer(syn.normal(1, (1024,)), norm, *W, n, twin, cpu_twin=True)
    assert st == oracle.ERR_INVALID_ARG


# ---- KV-slot commitments (qx-commit state.rs:213-251, :334-368) ----------------------
def _blake3_ref():
    import blake3  # the blake3 crate's official Python binding: the reference's own hash library
    return lambda data: blake3.blake3(data).digest()


def _hash_domain(b3, domain, fields):
    """qx-commit hash.rs hash_domain for Blake3V1: domain, then u64 LE length + bytes per field."""
    import struct
    return b3(domain + b"".join(struct.pack("<Q", len(f)) + f for f in fields))


def _tree_ref(b3, data, leaf_domain, tree_domain):
    """qx-commit chunk_tree_hash (state.rs:213-251) over 256-byte chunks."""
    import struct
    leaves = [_hash_domain(b3, leaf_domain, [struct.pack("<I", i), data[i * 256:(i + 1) * 256]])
              for i in range((len(data) + 255) // 256)]
    cap = 1
    while cap < len(leaves):
        cap *= 2
    leaves += [_hash_domain(b3, b"QX:MERKLE:EMPTY:V1", [tree_domain])] * (cap - len(leaves))
    while len(leaves) > 1:
        leaves = [b3(leaves[2 * i] + leaves[2 * i + 1]) for i in range(len(leaves) // 2)]
    return leaves[0]


def _kv_leaf_ref(b3, layer, token, key, value):
    """qx-commit kv_leaf_hash_v1 (state.rs:334-368)."""
    import struct
    kr = _tree_ref(b3, key, b"QX:KV:KEY:CHUNK:V1", b"QX:KV:KEY:TREE:V1")
    vr = _tree_ref(b3, value, b"QX:KV:VALUE:CHUNK:V1", b"QX:KV:VALUE:TREE:V1")
    return _hash_domain(b3, b"QX:KV:V1", [struct.pack("<H", layer), struct.pack("<I", token), kr, vr])


@pytest.mark.parametrize("n", [0, 1, 63, 64, 65, 127, 128, 129, 300, 1023, 1024])
def test_blake3_restatement_matches_the_blake3_crate(oracle, n):
    b3 = _blake3_ref()
    data = bytes((i * 7 + 3) % 251 for i in range(n))
    assert oracle.blake3_single_chunk(data) == b3(data)


@pytest.mark.parametrize("key_len,value_len", [(2048, 2048), (1024, 1024), (1024, 2048), (300, 700), (256, 1)])
def test_kv_leaf_hash_matches_qx_commit(oracle, key_len, value_len):
    b3 = _blake3_ref()
    rng = np.random.default_rng(key_len * 7 + value_len)
    key = rng.integers(0, 256, key_len, dtype=np.uint8).tobytes()
    value = rng.integers(0, 256, value_len, dtype=np.uint8).tobytes()
    assert oracle.kv_leaf_hash(3, 4095, key, value) == _kv_leaf_ref(b3, 3, 4095, key, value)
    # the coordinates are committed (qx-commit state.rs:375-387)
    assert oracle.kv_leaf_hash(3, 4095, key, value) != oracle.kv_leaf_hash(4, 4095, key, value)
    assert oracle.kv_leaf_hash(3, 4095, key, value) != oracle.kv_leaf_hash(3, 4094, key, value)


@pytest.mark.parametrize("n", [256, 1024, 4096, 3000])
def test_state_hash_matches_qx_commit(oracle, n):
    b3 = _blake3_ref()
    data = np.random.default_rng(n).integers(0, 256, n, dtype=np.uint8).tobytes()
    assert oracle.state_hash(data) == _tree_ref(b3, data, b"QX:STATE:CHUNK:V1", b"QX:STATE:V1")


def test_verification_hashes_reference_golden_case(oracle):
    """The reference's verification_hash_matches_cpu_golden_oracle case
    (qx-metal lib.rs:15531-15604): one layer, checkpoint interval 1, token 11;
    snapshot 0 and 1 hold the same residual; the expected bytes are the CPU
    state_hash_v1 / kv_leaf_hash_v1, restated here on the blake3 package."""
    b3 = _blake3_ref()
    residual = (np.arange(1024, dtype=np.float32) * np.float32(0.125) - np.float32(64.0)).tobytes()
    key = (np.arange(512, dtype=np.float32) * np.float32(-0.25) + np.float32(3.0)).tobytes()
    value = (np.arange(512, dtype=np.float32) / np.float32(17.0)).tobytes()
    out = oracle.verification_hashes(residual + residual, len(residual), 1, 1, [key], [value], 11)
    state = _tree_ref(b3, residual, b"QX:STATE:CHUNK:V1", b"QX:STATE:V1")
    assert len(out) == 128
    assert out[:32] == state and out[32:64] == bytes(32)
    assert out[64:96] == state and out[96:128] == _kv_leaf_ref(b3, 0, 11, key, value)


def test_verification_hashes_checkpoint_positions(oracle):
    """Positions that are not checkpoints carry a zero state root
    (verification_hash.metal:446-459)."""
    rng = np.random.default_rng(5)
    layers, stride = 6, 512
    res = rng.integers(0, 256, (layers + 1) * stride, dtype=np.uint8).tobytes()
    keys = [rng.integers(0, 256, 1024, dtype=np.uint8).tobytes() for _ in range(layers)]
    vals = [rng.integers(0, 256, 1024, dtype=np.uint8).tobytes() for _ in range(layers)]
    out = oracle.verification_hashes(res, stride, 4, layers, keys, vals, 7)
    for p in range(layers + 1):
        state = out[64 * p:64 * p + 32]
        if p in (0, 4, 6):
            assert state == oracle.state_hash(res[p * stride:(p + 1) * stride])
        else:
            assert state == bytes(32)
