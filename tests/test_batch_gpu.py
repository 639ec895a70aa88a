"""The many-token and many-sequence paths on the B200 against the oracle
(model/cpu.rs and model/model.rs restated):

- the tensor-core contraction, through the Device trait's matmul over
  several tokens (model/cpu.rs:49-77), at the reference's op tolerance
  (model/titania.rs:263: 1e-5 + 1e-4 |e|) and at Qwen3 shapes;
- prompts (Model::forward with n >= 2 tokens) through the tensor-core path,
  including prompts longer than one pass, continued by single-token steps;
- decode steps of many sequences at once, each sequence against its own
  oracle run (the parity bar: logits rel 2e-2 / abs 1e-2, greedy tokens
  identical)."""

import numpy as np
import pytest

import titania_b200 as tb
from oracle import oracle as orc
from titania_b200 import synth

from conftest import close

pytestmark = pytest.mark.gpu

REL_OP, ABS_OP = 1e-4, 1e-5  # model/titania.rs:263
REL, ABS = 2e-2, 1e-2        # logits, north star


def bf16_normal(rng, shape, std=0.02):
    return synth.f32_to_bf16_bits(rng.normal(0.0, std, size=shape).astype(np.float32)).reshape(shape)


def buf(dev, values):
    b = dev.alloc(values.size)
    dev.write(b, values)
    return b


@pytest.mark.parametrize("rows,cols,n", [
    (5, 64, 3), (100, 72, 2), (300, 520, 130),             # ragged: partial tiles in rows, columns and tokens
    (2048, 1024, 2), (4096, 1024, 64), (1024, 2048, 65),    # q|k|v, o_proj (split-K)
    (6144, 1024, 7), (1024, 3072, 200), (3072, 1024, 256),  # gate|up, down, up
    (151936, 1024, 64),                                     # lm_head over a batch
])
def test_matmul_tokens(b200, rows, cols, n):
    rng = np.random.default_rng(rows * 31 + cols * 7 + n)
    w = bf16_normal(rng, (rows, cols))
    x = rng.standard_normal(n * cols, dtype=np.float32)
    exp = np.zeros(n * rows, dtype=np.float32)
    orc.matmul(exp, w, x)
    out = b200.alloc(n * rows)
    b200.matmul(out, b200.upload(tb.Tensor([rows, cols], w)), buf(b200, x))
    close(b200.read(out), exp, REL_OP, ABS_OP)


def test_matmul_tokens_repeat_is_deterministic(b200):
    """Split-K partials are summed in split order: identical results."""
    rng = np.random.default_rng(5)
    w = b200.upload(tb.Tensor([1024, 3072], bf16_normal(rng, (1024, 3072))))
    x = buf(b200, rng.standard_normal(64 * 3072, dtype=np.float32))
    outs = []
    for _ in range(3):
        out = b200.alloc(64 * 1024)
        b200.matmul(out, w, x)
        outs.append(b200.read(out))
    assert np.array_equal(outs[0], outs[1]) and np.array_equal(outs[0], outs[2])


@pytest.fixture(scope="module")
def tiny(b200, tiny_model_dir):
    return tb.Model.load(tiny_model_dir, b200), orc.Model(tiny_model_dir)


@pytest.mark.parametrize("kv", ["f32", "bf16"])
@pytest.mark.parametrize("n", [2, 9, 64, 200, 1100])
def test_tiny_prompt(tiny, kv, n):
    """A prompt through the tensor-core path (1100 tokens: two passes), then
    single-token steps from the same cache."""
    m, ref = tiny
    prompt = synth.prompt_tokens(n, 1024, seed=100 + n)
    max_len = n + 8
    rs = ref.state(max_len)
    exp = ref.forward(rs, prompt, 0)
    st = m.state(max_len, kv=kv)
    got = m.forward(st, prompt, 0)
    close(got, exp, REL, ABS)
    assert int(np.argmax(got)) == int(np.argmax(exp))
    pos = n
    t = int(np.argmax(exp))
    for _ in range(4):
        exp = ref.forward(rs, [t], pos)
        got = m.forward(st, [t], pos)
        close(got, exp, REL, ABS)
        assert int(np.argmax(got)) == int(np.argmax(exp))
        t = int(np.argmax(exp))
        pos += 1


def test_tiny_prompt_continues_a_prompt(tiny):
    """Two prompt calls on one sequence (the second attends to the first's cache)."""
    m, ref = tiny
    a = synth.prompt_tokens(37, 1024, seed=1)
    b = synth.prompt_tokens(70, 1024, seed=2)
    rs = ref.state(128)
    ref.forward(rs, a, 0)
    exp = ref.forward(rs, b, len(a))
    st = m.state(128)
    m.forward(st, a, 0)
    got = m.forward(st, b, len(a))
    close(got, exp, REL, ABS)
    npos, kv_dim = len(a) + len(b), 2 * 128
    k_ref = rs.kv(1, 0, npos * kv_dim).reshape(npos, kv_dim)
    for p in (0, len(a), npos - 1):
        close(st.read_kv(1, 0, p), k_ref[p], 1e-4, 1e-4)


def _tiny_batch(m, ref, kv, prompts, steps):
    n = len(prompts)
    max_len = max(len(p) for p in prompts) + steps + 4
    bs = m.batch_state(n, max_len, kv=kv)
    first, positions = [], []
    for i, p in enumerate(prompts):
        first.append(m.forward_seq(bs, i, p, 0, logits=False))
        positions.append(len(p))
    expected = [orc.greedy_generate(ref, p, steps + 1, max_len=max_len) for p in prompts]
    return bs, first, positions, expected


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_tiny_batch_generate(tiny, kv):
    """Five sequences of different lengths decoded together on the device."""
    m, ref = tiny
    prompts = [synth.prompt_tokens(k, 1024, seed=k) for k in (3, 9, 1, 17, 40)]
    steps = 8
    bs, first, positions, expected = _tiny_batch(m, ref, kv, prompts, steps)
    for i in range(len(prompts)):
        assert first[i] == expected[i][0][0]
    out = m.generate_batch(bs, first, positions, steps)
    for i in range(len(prompts)):
        assert [first[i]] + out[:, i].tolist() == expected[i][0][:steps + 1], f"sequence {i}"


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_tiny_batch_long_contexts(tiny, kv):
    """Few sequences with long contexts: the decode attention splits each
    context into parts and combines them (contexts of 1 to 5 parts)."""
    m, ref = tiny
    prompts = [synth.prompt_tokens(k, 1024, seed=200 + k) for k in (150, 300, 20)]
    steps = 4
    bs = m.batch_state(len(prompts), 400, kv=kv)
    first = [m.forward_seq(bs, i, p, 0, logits=False) for i, p in enumerate(prompts)]
    expected = [orc.greedy_generate(ref, p, steps + 1, max_len=400) for p in prompts]
    tokens, positions = list(first), [len(p) for p in prompts]
    for step in range(steps):
        logits, nxt = m.forward_batch(bs, tokens, positions)
        for i in range(len(prompts)):
            close(logits[i], expected[i][1][step + 1], REL, ABS)
            assert int(nxt[i]) == expected[i][0][step + 1]
        tokens, positions = nxt.tolist(), [p + 1 for p in positions]


def test_tiny_batch_forward_logits(tiny):
    """One step of every sequence at once returns each sequence's logits."""
    m, ref = tiny
    prompts = [synth.prompt_tokens(k, 1024, seed=50 + k) for k in (4, 12, 2)]
    bs, first, positions, expected = _tiny_batch(m, ref, "f32", prompts, 3)
    tokens = list(first)
    for step in range(3):
        logits, nxt = m.forward_batch(bs, tokens, positions)
        for i in range(len(prompts)):
            close(logits[i], expected[i][1][step + 1], REL, ABS)
            assert int(nxt[i]) == expected[i][0][step + 1]
        tokens = nxt.tolist()
        positions = [p + 1 for p in positions]


@pytest.mark.parametrize("heads,kv_heads", [(2, 2), (8, 2)])
@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_tiny_batch_group_sizes(b200, heads, kv_heads, kv):
    """1 and 4 query heads per kv head (the tensor-core decode attention
    takes 1 and 2; 4 runs on the CUDA cores), prompt and batched decode."""
    import os
    from conftest import ROOT
    cfg = dict(synth.TINY, num_attention_heads=heads, num_key_value_heads=kv_heads)
    d = os.path.join(ROOT, "_build", f"tiny-h{heads}-kv{kv_heads}")
    synth.write_model(d, cfg, seed=5)
    m, ref = tb.Model.load(d, b200), orc.Model(d)
    prompts = [synth.prompt_tokens(k, 1024, seed=300 + k) for k in (70, 5, 130)]
    steps = 3
    bs = m.batch_state(len(prompts), 160, kv=kv)
    first = [m.forward_seq(bs, i, p, 0, logits=False) for i, p in enumerate(prompts)]
    expected = [orc.greedy_generate(ref, p, steps + 1, max_len=160) for p in prompts]
    assert first == [e[0][0] for e in expected]
    tokens, positions = list(first), [len(p) for p in prompts]
    for step in range(steps):
        logits, nxt = m.forward_batch(bs, tokens, positions)
        for i in range(len(prompts)):
            close(logits[i], expected[i][1][step + 1], REL, ABS)
            assert int(nxt[i]) == expected[i][0][step + 1]
        tokens, positions = nxt.tolist(), [p + 1 for p in positions]


def test_batch_state_bounds(tiny):
    m, _ = tiny
    bs = m.batch_state(3, 16)
    with pytest.raises(tb.DeviceError, match="not in this state"):
        m.forward_seq(bs, 3, [1, 2], 0)
    with pytest.raises(tb.DeviceError, match="past the end"):
        m.generate_batch(bs, [1, 1, 1], [10, 10, 10], 7)
    with pytest.raises(tb.DeviceError, match="vocabulary"):
        m.forward_batch(bs, [1, 1024, 1], [0, 0, 0])
    with pytest.raises(tb.DeviceError, match="one-sequence"):
        m.generate(bs, 1, 0, 2)


@pytest.fixture(scope="module")
def qwen06b():
    return synth.cached_model("qwen3-0.6b", seed=0)


@pytest.mark.parametrize("kv,abs_", [("f32", ABS), ("bf16", 1.5e-2)])
def test_qwen3_0_6b_batch(b200, qwen06b, kv, abs_):
    """Four Qwen3-0.6B sequences (16-token prompts, as BASELINE config 0)
    decoded together for 8 greedy steps, each against its own oracle run."""
    m = tb.Model.load(qwen06b, b200)
    ref = orc.Model(qwen06b)
    prompts = [synth.prompt_tokens(16, 151936, seed=s) for s in (1, 2, 3, 4)]
    steps = 8
    expected = [orc.greedy_generate(ref, p, steps + 1, max_len=32) for p in prompts]
    bs = m.batch_state(len(prompts), 32, kv=kv)
    first = [m.forward_seq(bs, i, p, 0, logits=False) for i, p in enumerate(prompts)]
    assert first == [e[0][0] for e in expected]
    tokens, positions = list(first), [16] * len(prompts)
    for step in range(steps):
        logits, nxt = m.forward_batch(bs, tokens, positions)
        for i in range(len(prompts)):
            close(logits[i], expected[i][1][step + 1], REL, abs_)
            assert int(nxt[i]) == expected[i][0][step + 1], f"sequence {i} step {step}"
        tokens = nxt.tolist()
        positions = [p + 1 for p in positions]


def test_qwen3_0_6b_long_prompt(b200, qwen06b):
    """A 300-token prompt (three token tiles per contraction) on 0.6B shapes."""
    m = tb.Model.load(qwen06b, b200)
    ref = orc.Model(qwen06b)
    prompt = synth.prompt_tokens(300, 151936, seed=9)
    rs = ref.state(320)
    exp = ref.forward(rs, prompt, 0)
    st = m.state(320)
    got = m.forward(st, prompt, 0)
    close(got, exp, REL, ABS)
    assert int(np.argmax(got)) == int(np.argmax(exp))


@pytest.mark.parametrize("kv", ["bf16"])
def test_tiny_batch_many_sequences_long_contexts(tiny, kv):
    """Enough sequences that each (token, kv head) gets one CTA over its whole
    context (148 x 2 kv heads >= two CTAs per SM), with contexts of 5 to 7
    32-position chunks: the decode attention reuses its staging ring and its
    two warp pairs walk alternate chunks. Every sequence against its own
    oracle run."""
    m, ref = tiny
    rng = np.random.default_rng(31)
    n = 148
    lengths = [int(x) for x in rng.integers(140, 215, size=n)]
    prompts = [synth.prompt_tokens(k, 1024, seed=4000 + i) for i, k in enumerate(lengths)]
    steps = 3
    max_len = max(lengths) + steps + 4
    bs = m.batch_state(n, max_len, kv=kv)
    first = [m.forward_seq(bs, i, p, 0, logits=False) for i, p in enumerate(prompts)]
    expected = [orc.greedy_generate(ref, p, steps + 1, max_len=max_len) for p in prompts]
    assert first == [e[0][0] for e in expected]
    tokens, positions = list(first), list(lengths)
    for step in range(steps):
        logits, nxt = m.forward_batch(bs, tokens, positions)
        for i in range(n):
            close(logits[i], expected[i][1][step + 1], REL, 1.5e-2)
            assert int(nxt[i]) == expected[i][0][step + 1], f"sequence {i} step {step}"
        tokens, positions = nxt.tolist(), [p + 1 for p in positions]


@pytest.mark.slow
def test_config3_prompt_2048_two_layers(b200):
    """BASELINE config 3's prompt length: 2048 uniform ids in two passes of the
    tensor-core path, causal attention on the tensor cores over a bf16 cache,
    on two layers of Qwen3-0.6B (every matrix its real shape) against the
    oracle; then one single-token step over the 2048 cached positions."""
    path = synth.cached_model("qwen3-0.6b-2l", seed=0)
    m = tb.Model.load(path, b200)
    ref = orc.Model(path)
    prompt = synth.prompt_tokens(2048, 151936, seed=12)
    rs = ref.state(2050)
    exp = ref.forward(rs, prompt, 0)
    st = m.state(2050, kv="bf16")
    got = m.forward(st, prompt, 0)
    close(got, exp, REL, 1.5e-2)
    t = int(np.argmax(exp))
    assert int(np.argmax(got)) == t
    exp = ref.forward(rs, [t], 2048)
    got = m.forward(st, [t], 2048)
    close(got, exp, REL, 1.5e-2)
    assert int(np.argmax(got)) == int(np.argmax(exp))
