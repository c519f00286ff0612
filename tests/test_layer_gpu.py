"""The attention sub-layer with Q4 projections (qxc_q4_mat_vec,
qxc_attention_layer) against the oracle.

qxc_attention_layer computes the V2 GPU stage (qx-runtime-v2
encode_attention_layer, lib.rs:6916-6994): RMSNorm, Q4 q/k/v, the fma RoPE
of the Metal kernel qx_v2_rope_kv (the same operations as V1's
rotate_heads), attention, Q4 o-projection, fma residual. The oracle's
default layer restates exactly that: the RMSNorm and Q4 mat-vec keep the
reference's lane order, so q/k/v, the appended rows and the projections are
bit-exact, and the outputs, which pass through the attention, are within the
fp32 gate (1e-5 normwise).

The V2 CPU twin CpuQ4Reference::step (lib.rs:4680-4706) rotates without fma
(cpu_rotate_heads) and attends with hierarchical sums up to 512 positions;
against it the value rows are bit-exact, the key rows differ in the RoPE's
last bits, and the outputs stay within the same 1e-5 gate and the
reference's own V2 gate (0.01 absolute, tools/qx-bench/src/main.rs:11064-11076).
"""
import sys
import os

import numpy as np
import pytest

from helpers import normwise
from qx_b200 import BF16, F32, MODEL_GRANITE, KvArena, Q4Weights, QxError, q4_mat_vec
from qx_b200 import synthetic as syn

pytestmark = pytest.mark.gpu


def q4(oracle, rows, cols, seed, scale=0.05):
    m = oracle.Q4Matrix((syn.normal(seed, (rows, cols)) * scale).astype(np.float32))
    return m


def dev_q4(m):
    import torch
    return Q4Weights(torch.from_numpy(m.codes).cuda(), torch.from_numpy(m.scales.view(np.int16)).cuda(), m.rows,
                     m.cols)


@pytest.mark.parametrize("rows,cols", [(1, 32), (7, 96), (512, 1024), (1024, 1024), (33, 4096)])
def test_q4_mat_vec_bit_exact(gpu_ctx, oracle, rows, cols):
    import torch
    m = q4(oracle, rows, cols, 0x8100 + rows + cols)
    x = syn.normal(0x8200 + cols, (cols,))
    y = torch.zeros(rows, device="cuda")
    q4_mat_vec(gpu_ctx, dev_q4(m), torch.from_numpy(x).cuda(), y)
    gpu_ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), m.mat_vec(x).view(np.uint32))


def test_rms_then_q4_bit_exact(gpu_ctx, oracle):
    import torch
    m = q4(oracle, 512, 1024, 0x8300)
    x = syn.normal(0x8301, (1024,)) * 3.0
    w = (1.0 + 0.1 * syn.normal(0x8302, (1024,))).astype(np.float32)
    st, xn = oracle.rms_norm_simd(x, w)
    assert st == 1
    y = torch.zeros(512, device="cuda")
    q4_mat_vec(gpu_ctx, dev_q4(m), torch.from_numpy(x).cuda(), y, rms_weight=torch.from_numpy(w).cuda())
    gpu_ctx.sync()
    assert np.array_equal(y.cpu().numpy().view(np.uint32), m.mat_vec(xn).view(np.uint32))


def layer_setup(gpu_ctx, oracle, layers, prefix, cap):
    import torch
    W = []
    for l in range(layers):
        W.append(dict(norm=(1.0 + 0.1 * syn.normal(0x8400 + l, (1024,))).astype(np.float32),
                      q=q4(oracle, 1024, 1024, 0x8410 + l), k=q4(oracle, 512, 1024, 0x8420 + l),
                      v=q4(oracle, 512, 1024, 0x8430 + l), o=q4(oracle, 1024, 1024, 0x8440 + l)))
    kc = syn.normal(0x8450, (layers, prefix, 8, 64))
    vc = syn.normal(0x8451, (layers, prefix, 8, 64))
    arena = KvArena(gpu_ctx, MODEL_GRANITE, layers, 1, cap, F32, F32)
    caches = []
    for l in range(layers):
        c = oracle.KvCache(cap)
        if prefix:
            arena.write(0, l, 0, kc[l], vc[l])
            c.keys[:prefix], c.values[:prefix] = kc[l], vc[l]
            c.length.value = prefix
        caches.append(c)
    arena.set_len(0, prefix)
    dW = [dict(norm=torch.from_numpy(w["norm"]).cuda(), q=dev_q4(w["q"]), k=dev_q4(w["k"]), v=dev_q4(w["v"]),
               o=dev_q4(w["o"])) for w in W]
    return W, dW, arena, caches


@pytest.mark.parametrize("prefix", [0, 1, 300])
def test_attention_layer_matches_oracle(gpu_ctx, oracle, prefix):
    """Every layer fed the oracle's input for that layer: q/k/v and so every
    cache row bit-exact; each layer's output within 1e-5."""
    import torch
    layers, tokens, cap = 2, 3, 320
    W, dW, arena, caches = layer_setup(gpu_ctx, oracle, layers, prefix, cap)
    for t in range(tokens):
        ref = syn.normal(0x8460 + t, (1024,))
        for l in range(layers):
            inp = ref
            st, ref, att_ref = oracle.granite_attention_layer(inp, W[l]["norm"], W[l]["q"], W[l]["k"], W[l]["v"],
                                                              W[l]["o"], prefix + t, caches[l])
            assert st == 0
            out = torch.zeros(1024, device="cuda")
            att = torch.zeros(1024, device="cuda")
            arena.attention_layer(torch.from_numpy(inp).cuda(), out, dW[l]["norm"], dW[l]["q"], dW[l]["k"],
                                  dW[l]["v"], dW[l]["o"], prefix + t, layer=l, attention_out=att,
                                  flags=1 if l + 1 < layers else 0)
            gpu_ctx.sync()
            assert normwise(att.cpu().numpy(), att_ref) <= 1e-5
            assert normwise(out.cpu().numpy(), ref) <= 1e-5
            # the reference's V2 gate (tools/qx-bench/src/main.rs:11064-11076)
            assert np.abs(att.cpu().numpy() - att_ref).max() <= 0.01
    assert arena.len(0) == prefix + tokens
    for l in range(layers):
        gk, gv = arena.read(0, l, 0, prefix + tokens)
        assert np.array_equal(gk.view(np.uint32), caches[l].keys[:prefix + tokens].view(np.uint32))
        assert np.array_equal(gv.view(np.uint32), caches[l].values[:prefix + tokens].view(np.uint32))


def test_attention_layers_chained(gpu_ctx, oracle):
    """The GPU's own hidden states through a 4-layer stack for 4 tokens:
    within 1e-5 of the oracle's stack."""
    import torch
    layers, tokens, prefix, cap = 4, 4, 200, 256
    W, dW, arena, caches = layer_setup(gpu_ctx, oracle, layers, prefix, cap)
    for t in range(tokens):
        h = syn.normal(0x8470 + t, (1024,))
        ref, cur = h.copy(), torch.from_numpy(h).cuda()
        for l in range(layers):
            st, ref, _ = oracle.granite_attention_layer(ref, W[l]["norm"], W[l]["q"], W[l]["k"], W[l]["v"],
                                                        W[l]["o"], prefix + t, caches[l])
            assert st == 0
            nxt = torch.zeros(1024, device="cuda")
            arena.attention_layer(cur, nxt, dW[l]["norm"], dW[l]["q"], dW[l]["k"], dW[l]["v"], dW[l]["o"],
                                  prefix + t, layer=l, flags=1 if l + 1 < layers else 0)
            cur = nxt
        gpu_ctx.sync()
        assert normwise(cur.cpu().numpy(), ref) <= 1e-5
    assert arena.len(0) == prefix + tokens


def test_attention_layer_against_cpu_twin(gpu_ctx, oracle):
    """qxc_attention_layer against the V2 CPU twin (CpuQ4Reference::step's
    attention part), up to the twin's 512 positions."""
    import torch
    layers, prefix, cap = 1, 490, 512
    W, dW, arena, caches = layer_setup(gpu_ctx, oracle, layers, prefix, cap)
    twin = caches[0]
    for t in range(cap - prefix):
        h = syn.normal(0x8480 + t, (1024,))
        st, ref, att_ref = oracle.granite_attention_layer(h, W[0]["norm"], W[0]["q"], W[0]["k"], W[0]["v"],
                                                          W[0]["o"], prefix + t, twin, cpu_twin=True)
        assert st == 0
        out = torch.zeros(1024, device="cuda")
        att = torch.zeros(1024, device="cuda")
        arena.attention_layer(torch.from_numpy(h).cuda(), out, dW[0]["norm"], dW[0]["q"], dW[0]["k"], dW[0]["v"],
                              dW[0]["o"], prefix + t, layer=0, attention_out=att)
        gpu_ctx.sync()
        a, o = att.cpu().numpy(), out.cpu().numpy()
        assert normwise(a, att_ref) <= 1e-5 and normwise(o, ref) <= 1e-5, t
        assert np.abs(a - att_ref).max() <= 0.01
    gk, gv = arena.read(0, 0, 0, cap)
    assert np.array_equal(gv.view(np.uint32), twin.values[:cap].view(np.uint32))
    assert np.abs(gk - twin.keys[:cap]).max() <= 1e-5


# ---- qxc_attention_stack: every layer of a stack in one persistent launch -------------
def _stack_ref(oracle, W, caches, h, position, layers):
    ref = h.copy()
    for l in range(layers):
        st, ref, _ = oracle.granite_attention_layer(ref, W[l]["norm"], W[l]["q"], W[l]["k"], W[l]["v"], W[l]["o"],
                                                    position, caches[l])
        assert st == 0
    return ref


@pytest.mark.parametrize("prefix", [0, 1, 63, 64, 255, 256, 700])
def test_attention_stack_matches_oracle(gpu_ctx, oracle, prefix):
    """4 layers per launch, 3 tokens: the last hidden state within 1e-5 of the
    oracle's chain; layer 0's appended rows bit-exact (its input is the
    oracle's), the deeper layers' within the attention's rounding."""
    import torch
    layers, tokens, cap = 4, 3, 1024
    W, dW, arena, caches = layer_setup(gpu_ctx, oracle, layers, prefix, cap)
    for t in range(tokens):
        h = syn.normal(0x8490 + t + prefix, (1024,))
        ref = _stack_ref(oracle, W, caches, h, prefix + t, layers)
        out = torch.zeros(1024, device="cuda")
        before = gpu_ctx.launch_count
        arena.attention_stack(torch.from_numpy(h).cuda(), out, dW, prefix + t)
        gpu_ctx.sync()
        assert gpu_ctx.launch_count - before == 1
        assert normwise(out.cpu().numpy(), ref) <= 1e-5, (prefix, t)
    assert arena.len(0) == prefix + tokens
    n = prefix + tokens
    gk, gv = arena.read(0, 0, 0, n)
    assert np.array_equal(gk.view(np.uint32), caches[0].keys[:n].view(np.uint32))
    assert np.array_equal(gv.view(np.uint32), caches[0].values[:n].view(np.uint32))
    for l in range(1, layers):
        gk, gv = arena.read(0, l, 0, n)
        assert np.abs(gk - caches[l].keys[:n]).max() <= 1e-4 and np.abs(gv - caches[l].values[:n]).max() <= 1e-4


def test_attention_stack_one_layer_calls_bit_exact_rows(gpu_ctx, oracle):
    """One-layer stack calls fed the oracle's input of each layer: q/k/v and
    so every appended row bit-exact, every output within 1e-5."""
    import torch
    layers, tokens, prefix, cap = 2, 3, 300, 320
    W, dW, arena, caches = layer_setup(gpu_ctx, oracle, layers, prefix, cap)
    for t in range(tokens):
        ref = syn.normal(0x84A0 + t, (1024,))
        for l in range(layers):
            inp = ref
            st, ref, _ = oracle.granite_attention_layer(inp, W[l]["norm"], W[l]["q"], W[l]["k"], W[l]["v"],
                                                        W[l]["o"], prefix + t, caches[l])
            assert st == 0
            out = torch.zeros(1024, device="cuda")
            arena.attention_stack(torch.from_numpy(inp).cuda(), out, [dW[l]], prefix + t, layer_begin=l,
                                  flags=1 if l + 1 < layers else 0)
            gpu_ctx.sync()
            assert normwise(out.cpu().numpy(), ref) <= 1e-5
    for l in range(layers):
        gk, gv = arena.read(0, l, 0, prefix + tokens)
        assert np.array_equal(gk.view(np.uint32), caches[l].keys[:prefix + tokens].view(np.uint32))
        assert np.array_equal(gv.view(np.uint32), caches[l].values[:prefix + tokens].view(np.uint32))


def test_attention_stack_bench_shape(gpu_ctx, oracle):
    """The bench's shape: 24 layers at context 4096 (16 items of 256 rows per
    kv head), the last two positions, against the oracle's 24-layer chain."""
    import torch
    layers, cap, prefix = 24, 4096, 4094
    W, dW, arena, caches = layer_setup(gpu_ctx, oracle, layers, prefix, cap)
    for t in range(2):
        h = syn.normal(0x84B0 + t, (1024,))
        ref = _stack_ref(oracle, W, caches, h, prefix + t, layers)
        out = torch.zeros(1024, device="cuda")
        arena.attention_stack(torch.from_numpy(h).cuda(), out, dW, prefix + t)
        gpu_ctx.sync()
        assert normwise(out.cpu().numpy(), ref) <= 1e-5, t
    assert arena.len(0) == cap


def test_attention_stack_beyond_one_launch_and_per_layer_path(gpu_ctx, oracle):
    """34 layers: two launches (32 + 2) chained through the context, against
    the oracle's chain; and a stack on a bf16 arena, which runs
    qxc_attention_layer per layer: identical to calling it layer by layer."""
    import torch
    from helpers import as_kv
    layers, cap, prefix = 34, 128, 100
    W3, dW3, _, _ = layer_setup(gpu_ctx, oracle, 3, 0, cap)
    W = [W3[l % 3] for l in range(layers)]
    dW = [dW3[l % 3] for l in range(layers)]
    arena = KvArena(gpu_ctx, MODEL_GRANITE, layers, 1, cap, F32, F32)
    caches = []
    for l in range(layers):
        kc, vc = syn.normal(0x84D0 + l, (prefix, 8, 64)), syn.normal(0x84E0 + l, (prefix, 8, 64))
        arena.write(0, l, 0, kc, vc)
        c = oracle.KvCache(cap)
        c.keys[:prefix], c.values[:prefix] = kc, vc
        c.length.value = prefix
        caches.append(c)
    arena.set_len(0, prefix)
    h = syn.normal(0x84C0, (1024,))
    ref = _stack_ref(oracle, W, caches, h, prefix, layers)
    out = torch.zeros(1024, device="cuda")
    before = gpu_ctx.launch_count
    arena.attention_stack(torch.from_numpy(h).cuda(), out, dW, prefix)
    gpu_ctx.sync()
    assert gpu_ctx.launch_count - before == 2
    assert normwise(out.cpu().numpy(), ref) <= 1e-5
    # the per-layer path on two bf16 arenas holding the same rows
    a16, b16 = (KvArena(gpu_ctx, MODEL_GRANITE, 3, 1, cap, BF16, BF16) for _ in range(2))
    for a in (a16, b16):
        for l in range(3):
            a.write(0, l, 0, as_kv(syn.normal(0x84D0 + l, (prefix, 8, 64)), BF16),
                    as_kv(syn.normal(0x84E0 + l, (prefix, 8, 64)), BF16))
        a.set_len(0, prefix)
    hin = torch.from_numpy(h).cuda()
    out16 = torch.zeros(1024, device="cuda")
    a16.attention_stack(hin, out16, dW3, prefix)
    cur = hin
    for l in range(3):
        nxt = torch.zeros(1024, device="cuda")
        b16.attention_layer(cur, nxt, dW3[l]["norm"], dW3[l]["q"], dW3[l]["k"], dW3[l]["v"], dW3[l]["o"], prefix,
                            layer=l, flags=1 if l < 2 else 0)
        cur = nxt
    gpu_ctx.sync()
    assert torch.equal(out16, cur)
    assert a16.len(0) == prefix + 1 and b16.len(0) == prefix + 1
    for l in range(3):
        assert all(np.array_equal(x, y) for x, y in zip(a16.read(0, l, 0, prefix + 1), b16.read(0, l, 0, prefix + 1)))


def test_attention_stack_rejects(gpu_ctx, oracle):
    import torch
    W, dW, arena, caches = layer_setup(gpu_ctx, oracle, 2, 10, 64)
    h = torch.zeros(1024, device="cuda")
    with pytest.raises(QxError, match="does not follow cache length"):
        arena.attention_stack(h, h, dW, 11)
    with pytest.raises(QxError, match="split"):
        arena.attention_stack(h, h, dW, 10, split=96)
    with pytest.raises(QxError, match="outside the arena"):
        arena.attention_stack(h, h, dW + dW, 10)
    assert arena.len(0) == 10
