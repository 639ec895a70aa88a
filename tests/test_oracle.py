"""The CPU oracle against the golden fixtures (an independent numpy
restatement of model/cpu.rs and model/model.rs; see tests/golden/gen_golden.py).
Everything here must match bit for bit."""

import os

import numpy as np
import pytest

from oracle import oracle as orc

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def same_bits(a, b):
    a = np.asarray(a, dtype=np.float32)
    b = np.asarray(b, dtype=np.float32)
    assert a.shape == b.shape
    diff = np.flatnonzero(a.view(np.uint32) != b.view(np.uint32))
    assert diff.size == 0, f"{diff.size} elements differ, first at {diff[0]}: {a[diff[0]]} vs {b[diff[0]]}"


def test_elementwise(golden_ops):
    g = golden_ops
    x, y = g["add/x"].copy(), g["add/y"].copy()
    orc.add(x, y)
    same_bits(x, g["add/out"])
    orc.silu_mul(x, y)
    same_bits(x, g["silu_mul/out"])


def test_embed(golden_ops):
    g = golden_ops
    out = np.zeros(3 * 128, dtype=np.float32)
    orc.embed(out, g["embed/table"], g["embed/tokens"])
    same_bits(out, g["embed/out"])


@pytest.mark.parametrize("shape", [(24, 256, 1), (5, 64, 3), (9, 384, 16), (24, 128, 19)])
def test_matmul(golden_ops, shape):
    rows, cols, n = shape
    key = f"matmul/{rows}x{cols}x{n}"
    out = np.zeros(n * rows, dtype=np.float32)
    orc.matmul(out, golden_ops[key + "/w"], golden_ops[key + "/x"])
    same_bits(out, golden_ops[key + "/out"])


def test_matmul_chunking_is_bit_identical(golden_ops):
    """cpu.rs:60-76: a batch computes the same dot per (row, token) as one token at a time."""
    w, x = golden_ops["matmul/24x128x19/w"], golden_ops["matmul/24x128x19/x"]
    whole = np.zeros(19 * 24, dtype=np.float32)
    orc.matmul(whole, w, x)
    for t in range(19):
        one = np.zeros(24, dtype=np.float32)
        orc.matmul(one, w, x[t * 128:(t + 1) * 128].copy())
        same_bits(one, whole[t * 24:(t + 1) * 24])


@pytest.mark.parametrize("shape", [(3, 128), (1, 1024), (9, 64)])
def test_rmsnorm(golden_ops, shape):
    rows, dim = shape
    key = f"rmsnorm/{rows}x{dim}"
    x = golden_ops[key + "/x"].copy()
    orc.rmsnorm(x, golden_ops[key + "/w"], 1e-6)
    same_bits(x, golden_ops[key + "/out"])


@pytest.mark.parametrize("n", [1, 3])
def test_rope(golden_ops, n):
    key = f"rope/{n}"
    x = golden_ops[key + "/x"].copy()
    orc.rope(x, golden_ops[key + "/table"], 37, 4, 128)
    same_bits(x, golden_ops[key + "/out"])


@pytest.mark.parametrize("case", [(0, 1), (6, 1), (32, 1), (39, 1), (0, 5), (30, 10)])
def test_attention(golden_ops, case):
    pos, n = case
    key = f"attention/{pos}_{n}"
    q = golden_ops[key + "/q"]
    out = np.zeros_like(q)
    orc.attention(out, q, golden_ops[key + "/k"], golden_ops[key + "/v"], pos, 4, 64, 2)
    same_bits(out, golden_ops[key + "/out"])


def test_attention_thread_count_invariant(golden_ops):
    key = "attention/30_10"
    outs = []
    for threads in (1, 3):
        orc.set_threads(threads)
        out = np.zeros_like(golden_ops[key + "/q"])
        orc.attention(out, golden_ops[key + "/q"], golden_ops[key + "/k"], golden_ops[key + "/v"], 30, 4, 64, 2)
        outs.append(out)
    orc.set_threads(os.cpu_count() or 1)
    same_bits(outs[0], outs[1])


def test_rope_table(golden_ops):
    same_bits(orc.rope_table(40, 128, 1e6), golden_ops["rope_table/128x40"])
    same_bits(orc.rope_table(8, 64, 10000.0), golden_ops["rope_table/64x8_theta1e4"])


def test_matmul_shape_mismatch_panics():
    out = np.zeros(10, dtype=np.float32)
    with pytest.raises(orc.OracleError):
        orc.matmul(out, np.zeros((3, 4), dtype=np.uint16), np.zeros(8, dtype=np.float32))


def test_greedy_total_order():
    logits = np.array([0.5, 2.0, -1.0, 2.0, np.float32(-0.0)], dtype=np.float32)
    assert orc.sample_greedy(logits) == 1  # ties go to the lowest id
    assert orc.sample_greedy(np.array([-0.0, 0.0], dtype=np.float32)) == 1  # +0 > -0 under total_cmp


def test_tiny_model_forward_and_greedy(tiny_model_dir):
    g = dict(np.load(os.path.join(ROOT, "tests", "golden", "tiny_model.npz")))
    m = orc.Model(tiny_model_dir)
    prompt = g["prompt"].tolist()
    steps = len(g["tokens"])
    st = m.state(len(prompt) + steps + 1)
    logits = m.forward(st, prompt, 0)
    pos = len(prompt)
    for i in range(steps):
        same_bits(logits, g["logits"][i])
        t = orc.sample_greedy(logits)
        assert t == int(g["tokens"][i])
        logits = m.forward(st, [t], pos)
        pos += 1
    same_bits(logits, g["final_logits"])
    kv_dim = m.num_key_value_heads * m.head_dim
    same_bits(st.kv(1, 0, pos * kv_dim), g["k_cache_l1"])
    same_bits(st.kv(1, 1, pos * kv_dim), g["v_cache_l1"])


def test_prefill_chunking_matches_token_by_token(tiny_model_dir):
    """model.rs:83-91: the prompt split into BATCH-sized chunks or fed token by
    token gives the same logits bit for bit."""
    m = orc.Model(tiny_model_dir)
    prompt = list(range(70))
    a = m.forward(m.state(80), prompt, 0)
    st = m.state(80)
    for p, t in enumerate(prompt):
        b = m.forward(st, [t], p)
    same_bits(a, b)


def test_forward_past_max_len_panics(tiny_model_dir):
    m = orc.Model(tiny_model_dir)
    with pytest.raises(orc.OracleError, match="past the end"):
        m.forward(m.state(4), [1, 2, 3, 4, 5], 0)
