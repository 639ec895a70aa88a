"""Each Device op on the B200 against the oracle (model/cpu.rs restated),
with the reference's own op-test inputs, shapes and tolerance
(model/titania.rs:259-370: |a - e| <= 1e-5 + 1e-4 |e|), then on Qwen3-0.6B
shapes (the per-op sweep configuration)."""

import numpy as np
import pytest

import titania_b200 as tb
from oracle import oracle as orc

from conftest import close

pytestmark = pytest.mark.gpu

REL, ABS = 1e-4, 1e-5  # model/titania.rs:263


def buf(dev, values):
    b = dev.alloc(values.size)
    dev.write(b, values)
    return b


def test_elementwise(b200, golden_ops):
    g = golden_ops
    x, y = buf(b200, g["add/x"]), buf(b200, g["add/y"])
    b200.add(x, y)
    assert np.array_equal(b200.read(x), g["add/out"])  # same order: bit-exact
    b200.silu_mul(x, y)
    close(b200.read(x), g["silu_mul/out"], REL, ABS)
    dst = buf(b200, g["copy/dst_in"])
    src = buf(b200, g["silu_mul/out"])
    b200.copy(dst, 7, src, 5, 300 - 5)
    assert np.array_equal(b200.read(dst), g["copy/out"])


def test_resize(b200, golden_ops):
    x = buf(b200, np.resize(golden_ops["add/x"], 300).astype(np.float32))
    y = buf(b200, golden_ops["add/y"][:100].copy())
    b200.resize(x, 100)
    b200.add(x, y)
    exp = golden_ops["add/x"][:100] + golden_ops["add/y"][:100]
    assert np.array_equal(b200.read(x), exp)
    b200.resize(x, 300)
    assert len(b200.read(x)) == 300
    with pytest.raises(tb.DeviceError, match="can't hold"):
        b200.resize(x, 301)


def test_embed(b200, golden_ops):
    g = golden_ops
    table = b200.upload(tb.Tensor([10, 128], g["embed/table"]))
    out = b200.alloc(3 * 128)
    b200.embed(out, table, g["embed/tokens"])
    assert np.array_equal(b200.read(out), g["embed/out"])
    with pytest.raises(tb.DeviceError, match="past the table"):
        b200.embed(out, table, [3, 10, 0])


@pytest.mark.parametrize("shape", [(24, 256, 1), (5, 64, 3), (9, 384, 16), (24, 128, 19)])
def test_matmul(b200, golden_ops, shape):
    rows, cols, n = shape
    key = f"matmul/{rows}x{cols}x{n}"
    w = b200.upload(tb.Tensor([rows, cols], golden_ops[key + "/w"]))
    x = buf(b200, golden_ops[key + "/x"])
    out = b200.alloc(n * rows)
    b200.matmul(out, w, x)
    close(b200.read(out), golden_ops[key + "/out"], REL, ABS)


@pytest.mark.parametrize("shape", [(3, 128), (1, 1024), (9, 64)])
def test_rmsnorm(b200, golden_ops, shape):
    rows, dim = shape
    key = f"rmsnorm/{rows}x{dim}"
    x = buf(b200, golden_ops[key + "/x"])
    b200.rmsnorm(x, b200.upload(tb.Tensor([dim], golden_ops[key + "/w"])), 1e-6)
    close(b200.read(x), golden_ops[key + "/out"], REL, ABS)


@pytest.mark.parametrize("n", [1, 3])
def test_rope(b200, golden_ops, n):
    key = f"rope/{n}"
    x = buf(b200, golden_ops[key + "/x"])
    table = buf(b200, golden_ops[key + "/table"])
    b200.rope(x, table, 37, 4, 128)
    assert np.array_equal(b200.read(x), golden_ops[key + "/out"])  # same order: bit-exact
    with pytest.raises(tb.DeviceError, match="past the end of the table"):
        b200.rope(x, table, 40 - n + 1, 4, 128)


@pytest.mark.parametrize("case", [(0, 1), (6, 1), (32, 1), (39, 1), (0, 5), (30, 10)])
def test_attention(b200, golden_ops, case):
    pos, n = case
    key = f"attention/{pos}_{n}"
    q = buf(b200, golden_ops[key + "/q"])
    k = buf(b200, golden_ops[key + "/k"])
    v = buf(b200, golden_ops[key + "/v"])
    out = b200.alloc(n * 4 * 64)
    b200.attention(out, q, k, v, pos, 4, 64, 2)
    close(b200.read(out), golden_ops[key + "/out"], REL, ABS)


def test_argmax(b200):
    rng = np.random.default_rng(0)
    x = rng.standard_normal(151936).astype(np.float32)
    x[77777] = 9.0
    x[99999] = 9.0  # tie: the lower index wins
    b = buf(b200, x)
    assert b200.argmax(b) == 77777 == orc.sample_greedy(x)


# ---- Qwen3-0.6B shapes (bf16 W ~ N(0, 0.02), f32 x ~ N(0, 1), batch 1) -------

def bf16_normal(rng, shape, std=0.02):
    from titania_b200.synth import f32_to_bf16_bits
    return f32_to_bf16_bits(rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(std)).reshape(
        shape)


@pytest.mark.parametrize("rows,cols", [(2048, 1024), (1024, 1024), (1024, 2048), (3072, 1024), (1024, 3072),
                                       (151936, 1024)])
def test_matmul_qwen3_shapes(b200, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    w = bf16_normal(rng, (rows, cols))
    x = rng.standard_normal(cols, dtype=np.float32)
    exp = np.zeros(rows, dtype=np.float32)
    orc.matmul(exp, w, x)
    out = b200.alloc(rows)
    b200.matmul(out, b200.upload(tb.Tensor([rows, cols], w)), buf(b200, x))
    close(b200.read(out), exp, REL, ABS)


def test_norm_rope_silu_qwen3_shapes(b200):
    rng = np.random.default_rng(3)
    ones = np.full(1024, 0x3F80, np.uint16)
    x = rng.standard_normal(1024, dtype=np.float32)
    exp = x.copy()
    orc.rmsnorm(exp, ones, 1e-6)
    d = buf(b200, x)
    b200.rmsnorm(d, b200.upload(tb.Tensor([1024], ones)), 1e-6)
    close(b200.read(d), exp, REL, ABS)
    # per-head QK-norm: 16 heads x 128
    q = rng.standard_normal(16 * 128, dtype=np.float32)
    w = bf16_normal(rng, (128,), 1.0)
    exp = q.copy()
    orc.rmsnorm(exp, w, 1e-6)
    d = buf(b200, q)
    b200.rmsnorm(d, b200.upload(tb.Tensor([128], w)), 1e-6)
    close(b200.read(d), exp, REL, ABS)
    # RoPE, 16 + 8 heads, across positions 0..4095
    table = orc.rope_table(4096, 128, 1e6)
    tdev = buf(b200, table)
    for heads in (16, 8):
        for pos in (0, 1, 1000, 4095):
            x = rng.standard_normal(heads * 128, dtype=np.float32)
            exp = x.copy()
            orc.rope(exp, table, pos, heads, 128)
            d = buf(b200, x)
            b200.rope(d, tdev, pos, heads, 128)
            assert np.array_equal(b200.read(d), exp)
    g = rng.standard_normal(3072, dtype=np.float32)
    u = rng.standard_normal(3072, dtype=np.float32)
    exp = g.copy()
    orc.silu_mul(exp, u)
    dg = buf(b200, g)
    b200.silu_mul(dg, buf(b200, u))
    close(b200.read(dg), exp, REL, ABS)


@pytest.mark.parametrize("ctx", [512, 4096])
def test_attention_qwen3_decode(b200, ctx):
    """16 q / 8 kv heads, head_dim 128, one token at position ctx-1."""
    rng = np.random.default_rng(ctx)
    kv = ctx * 8 * 128
    q = rng.standard_normal(16 * 128, dtype=np.float32)
    k = rng.standard_normal(kv, dtype=np.float32)
    v = rng.standard_normal(kv, dtype=np.float32)
    exp = np.zeros_like(q)
    orc.attention(exp, q, k, v, ctx - 1, 16, 128, 8)
    out = b200.alloc(q.size)
    b200.attention(out, buf(b200, q), buf(b200, k), buf(b200, v), ctx - 1, 16, 128, 8)
    close(b200.read(out), exp, REL, ABS)


def test_contract_violations_raise(b200):
    w = b200.upload(tb.Tensor([4, 8], np.zeros(32, np.uint16)))
    x = b200.alloc(12)
    out = b200.alloc(4)
    with pytest.raises(tb.DeviceError, match="whole number"):
        b200.matmul(out, w, x)
    with pytest.raises(tb.DeviceError):
        b200.write(out, np.zeros(5, np.float32))
    with pytest.raises(tb.DeviceError, match="out of range"):
        b200.copy(out, 2, x, 0, 3)
