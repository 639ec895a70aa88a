"""Each fused decode kernel alone, on Qwen3-0.6B shapes and weights, against
the oracle's ops (model/cpu.rs restated): the kernel reads and writes the
state's buffers exactly as in the decode step's graph (tb200_enqueue_op).

Tolerance: 1e-4 relative + 1e-4 absolute — f32 accumulation in another
order than the reference's 8-lane dot."""

import numpy as np
import pytest

import titania_b200 as tb
from oracle import oracle as orc
from titania_b200 import synth
from titania_b200.model import (OP_ATTENTION, OP_ATTENTION_O, OP_DOWN, OP_GATE_UP, OP_GATE_UP_SUM, OP_LM_HEAD, OP_O,
                                OP_QKV, Weights)

from conftest import close

pytestmark = pytest.mark.gpu

REL, ABS = 1e-4, 1e-4


@pytest.fixture(scope="module")
def setup(b200):
    path = synth.cached_model("qwen3-0.6b", seed=0)
    m = tb.Model.load(path, b200)
    w = Weights.open(path + "/model.safetensors")
    return m, w


def t(w, name):
    x = w.read(name)
    return np.asarray(x.data).reshape(x.shape)


def rmsnorm(x, g, eps=1e-6):
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    orc.rmsnorm(y, np.ascontiguousarray(g), eps)
    return y


def matmul(wt, x):
    out = np.zeros(wt.shape[0], dtype=np.float32)
    orc.matmul(out, np.ascontiguousarray(wt), np.ascontiguousarray(x, dtype=np.float32))
    return out


@pytest.mark.parametrize("layer", [0, 27])
def test_qkv(setup, layer):
    m, w = setup
    st = m.state(64)
    x = np.random.default_rng(layer).standard_normal(1024, dtype=np.float32)
    st.write("x", x)
    m.enqueue_op(st, OP_QKV, layer)
    p = f"model.layers.{layer}"
    xb = rmsnorm(x, t(w, f"{p}.input_layernorm.weight"))
    exp = np.concatenate([matmul(t(w, f"{p}.self_attn.{n}_proj.weight"), xb) for n in "qkv"])
    close(st.read("qkv"), exp, REL, ABS)


@pytest.mark.parametrize("layer", [0, 13])
def test_o_proj_residual(setup, layer):
    m, w = setup
    st = m.state(64)
    rng = np.random.default_rng(100 + layer)
    att = rng.standard_normal(2048, dtype=np.float32)
    x = rng.standard_normal(1024, dtype=np.float32)
    st.write("att", att)
    st.write("x", x)
    m.enqueue_op(st, OP_O, layer)
    exp = x + matmul(t(w, f"model.layers.{layer}.self_attn.o_proj.weight"), att)
    close(st.read("x"), exp, REL, ABS)


@pytest.mark.parametrize("layer", [0, 27])
def test_gate_up_silu(setup, layer):
    m, w = setup
    st = m.state(64)
    x = np.random.default_rng(200 + layer).standard_normal(1024, dtype=np.float32)
    st.write("x", x)
    m.enqueue_op(st, OP_GATE_UP, layer)
    p = f"model.layers.{layer}"
    xb = rmsnorm(x, t(w, f"{p}.post_attention_layernorm.weight"))
    g = matmul(t(w, f"{p}.mlp.gate_proj.weight"), xb)
    u = matmul(t(w, f"{p}.mlp.up_proj.weight"), xb)
    orc.silu_mul(g, u)
    close(st.read("h"), g, REL, ABS)
    assert np.array_equal(st.read("x2"), x)  # the residual DOWN adds back


def test_gate_up_sum_of_partials(setup):
    """GATE_UP_SUM: x + (the o_proj partials summed over kv groups), then as GATE_UP."""
    m, w = setup
    st = m.state(64)
    rng = np.random.default_rng(250)
    x = rng.standard_normal(1024, dtype=np.float32)
    part = rng.standard_normal(8 * 1024, dtype=np.float32)
    st.write("x", x)
    st.write("part", part)
    m.enqueue_op(st, OP_GATE_UP_SUM, 5)
    xs = x + part.reshape(8, 1024).sum(axis=0, dtype=np.float32)
    close(st.read("x2"), xs, REL, ABS)
    p = "model.layers.5"
    xb = rmsnorm(xs, t(w, f"{p}.post_attention_layernorm.weight"))
    g = matmul(t(w, f"{p}.mlp.gate_proj.weight"), xb)
    u = matmul(t(w, f"{p}.mlp.up_proj.weight"), xb)
    orc.silu_mul(g, u)
    close(st.read("h"), g, REL, ABS)


@pytest.mark.parametrize("layer", [0, 27])
def test_down_residual(setup, layer):
    m, w = setup
    st = m.state(64)
    rng = np.random.default_rng(300 + layer)
    h = rng.standard_normal(3072, dtype=np.float32)
    x = rng.standard_normal(1024, dtype=np.float32)
    st.write("h", h)
    st.write("x2", x)  # DOWN adds the residual GATE_UP stored
    m.enqueue_op(st, OP_DOWN, layer)
    exp = x + matmul(t(w, f"model.layers.{layer}.mlp.down_proj.weight"), h)
    close(st.read("x"), exp, REL, ABS)


def test_lm_head_and_greedy(setup):
    m, w = setup
    st = m.state(64)
    x = np.random.default_rng(400).standard_normal(1024, dtype=np.float32)
    st.write("x", x)
    st.set_position(1, 5)
    m.enqueue_op(st, OP_LM_HEAD, 0)
    exp = matmul(t(w, "model.embed_tokens.weight"), rmsnorm(x, t(w, "model.norm.weight")))
    got = st.read("logits")
    close(got, exp, REL, ABS)
    assert int(np.argmax(got)) == orc.sample_greedy(exp)


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_attention_over_positions(setup, kv):
    """QK-norm, RoPE, cache append and attention, position by position up to
    150 (three 64-position splits), against the oracle's ops on f32 caches."""
    m, w = setup
    layer = 3
    max_len = 160
    st = m.state(max_len, kv=kv)
    p = f"model.layers.{layer}"
    qn, kn = t(w, f"{p}.self_attn.q_norm.weight"), t(w, f"{p}.self_attn.k_norm.weight")
    table = orc.rope_table(max_len, 128, 1e6)
    kc = np.zeros(max_len * 1024, dtype=np.float32)
    vc = np.zeros(max_len * 1024, dtype=np.float32)
    rng = np.random.default_rng(500)
    tol = (REL, ABS) if kv == "f32" else (2e-2, 2e-2)
    for pos in range(151):
        qkv = rng.standard_normal(4096, dtype=np.float32)
        st.write("qkv", qkv)
        st.set_position(1, pos)
        m.enqueue_op(st, OP_ATTENTION, layer)
        q, k, v = qkv[:2048].copy(), qkv[2048:3072].copy(), qkv[3072:].copy()
        orc.rmsnorm(q, qn, 1e-6)
        orc.rmsnorm(k, kn, 1e-6)
        orc.rope(q, table, pos, 16, 128)
        orc.rope(k, table, pos, 8, 128)
        if kv == "bf16":  # the cache rounds k and v
            from titania_b200.synth import f32_to_bf16_bits
            k = (f32_to_bf16_bits(k).astype(np.uint32) << 16).view(np.float32)
            v = (f32_to_bf16_bits(v).astype(np.uint32) << 16).view(np.float32)
        kc[pos * 1024:(pos + 1) * 1024] = k
        vc[pos * 1024:(pos + 1) * 1024] = v
        if pos in (0, 1, 47, 63, 64, 65, 100, 127, 128, 150):
            exp = np.zeros(2048, dtype=np.float32)
            orc.attention(exp, q, kc, vc, pos, 16, 128, 8)
            close(st.read("att"), exp, *tol)
            close(st.read_kv(layer, 0, pos), k, *tol)


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_attention_o_over_positions(setup, kv):
    """ATTENTION_O for every position of the short-context path (0..63): the
    per-group o_proj partials against o_proj applied to the oracle's
    attention, column block by column block."""
    m, w = setup
    layer = 9
    st = m.state(64, kv=kv)
    p = f"model.layers.{layer}"
    qn, kn = t(w, f"{p}.self_attn.q_norm.weight"), t(w, f"{p}.self_attn.k_norm.weight")
    wo = t(w, f"{p}.self_attn.o_proj.weight")
    table = orc.rope_table(64, 128, 1e6)
    kc = np.zeros(64 * 1024, dtype=np.float32)
    vc = np.zeros(64 * 1024, dtype=np.float32)
    rng = np.random.default_rng(600)
    tol = (REL, ABS) if kv == "f32" else (2e-2, 2e-2)
    for pos in range(64):
        qkv = rng.standard_normal(4096, dtype=np.float32)
        st.write("qkv", qkv)
        st.set_position(1, pos)
        m.enqueue_op(st, OP_ATTENTION_O, layer)
        q, k, v = qkv[:2048].copy(), qkv[2048:3072].copy(), qkv[3072:].copy()
        orc.rmsnorm(q, qn, 1e-6)
        orc.rmsnorm(k, kn, 1e-6)
        orc.rope(q, table, pos, 16, 128)
        orc.rope(k, table, pos, 8, 128)
        if kv == "bf16":
            from titania_b200.synth import f32_to_bf16_bits
            k = (f32_to_bf16_bits(k).astype(np.uint32) << 16).view(np.float32)
            v = (f32_to_bf16_bits(v).astype(np.uint32) << 16).view(np.float32)
        kc[pos * 1024:(pos + 1) * 1024] = k
        vc[pos * 1024:(pos + 1) * 1024] = v
        if pos in (0, 1, 2, 15, 31, 47, 62, 63):
            att = np.zeros(2048, dtype=np.float32)
            orc.attention(att, q, kc, vc, pos, 16, 128, 8)
            part = st.read("part").reshape(8, 1024)
            for g in range(8):
                exp = matmul(np.ascontiguousarray(wo[:, g * 256:(g + 1) * 256]), att[g * 256:(g + 1) * 256])
                close(part[g], exp, *tol)
            close(st.read_kv(layer, 1, pos), v, *tol)
