"""Decode attention over a bf16 cache (tb200_attention_cache, the kernel the
batched decode step runs) against the oracle's attention (model/cpu.rs:
113-149), on BASELINE config 2: 16 query heads / 8 kv heads, head_dim 128,
K and V ~ N(0, 1) rounded to bf16, queries ~ N(0, 1), contexts of 512, 4096
and 32768 positions at batch 1 and 64.

The kernel multiplies exact products (q split into three bf16 planes, bf16
K/V) with f32 accumulation and a base-2 online softmax, so its results stay
within 2e-4 of the oracle's sequential f32 sums; the bound below is 1e-3."""

import numpy as np
import pytest

from conftest import close

pytestmark = pytest.mark.gpu

HQ, HKV, D = 16, 8, 128
TOL = 1e-3


def _cache_bits(batch, max_len, seed):
    """[batch, 2, HKV, max_len, D] bf16 bits of N(0, 1) values, generated in
    chunks (the 32768 x 64 case holds 4.3 G values)."""
    from titania_b200.synth import f32_to_bf16_bits

    out = np.empty((batch, 2, HKV, max_len, D), dtype=np.uint16)
    flat = out.reshape(-1)
    rng = np.random.Generator(np.random.PCG64(seed))
    step = 1 << 26
    buf = np.empty(step, dtype=np.float32)
    for s in range(0, flat.size, step):
        k = min(step, flat.size - s)
        rng.standard_normal(out=buf[:k], dtype=np.float32)
        flat[s:s + k] = f32_to_bf16_bits(buf[:k])
    return out


def _oracle(q, bits, b, pos):
    """The oracle's attention for sequence b at position pos (caches as f32,
    [position][kv head][head_dim], the reference's layout)."""
    from oracle import oracle as orc

    kv = (bits[b, :, :, :pos + 1, :].astype(np.uint32) << 16).view(np.float32)
    kc = np.ascontiguousarray(kv[0].transpose(1, 0, 2)).reshape(-1)
    vc = np.ascontiguousarray(kv[1].transpose(1, 0, 2)).reshape(-1)
    out = np.zeros(HQ * D, dtype=np.float32)
    orc.attention(out, np.ascontiguousarray(q), kc, vc, pos, HQ, D, HKV)
    return out


@pytest.mark.parametrize("ctx", [512, 4096, 32768])
@pytest.mark.parametrize("batch", [1, 64])
def test_config2_attention(b200, ctx, batch):
    from titania_b200 import Tensor

    bits = _cache_bits(batch, ctx, seed=ctx + batch)
    cache = b200.upload(Tensor(list(bits.shape), bits))
    rng = np.random.default_rng(7 + ctx + batch)
    q = rng.standard_normal((batch, HQ * D), dtype=np.float32)
    qb, ob = b200.alloc(q.size), b200.alloc(q.size)
    b200.write(qb, q.reshape(-1))
    positions = [ctx - 1] * batch
    b200.attention_cache(ob, qb, cache, positions, HQ)
    got = b200.read(ob).reshape(batch, HQ * D)
    check = range(batch) if ctx <= 4096 else sorted({0, batch // 2, batch - 1})
    for b in check:
        close(got[b], _oracle(q[b], bits, b, ctx - 1), TOL, TOL)


def test_ragged_positions_and_repeated_calls(b200):
    """Sequences at different positions in one call (each attends only to
    its own prefix), and a second call with other positions reuses the
    device's workspace."""
    from titania_b200 import Tensor

    batch, max_len = 5, 700
    bits = _cache_bits(batch, max_len, seed=3)
    cache = b200.upload(Tensor(list(bits.shape), bits))
    rng = np.random.default_rng(11)
    q = rng.standard_normal((batch, HQ * D), dtype=np.float32)
    qb, ob = b200.alloc(q.size), b200.alloc(q.size)
    b200.write(qb, q.reshape(-1))
    for positions in ([0, 1, 63, 64, 699], [699, 300, 2, 31, 32]):
        b200.attention_cache(ob, qb, cache, positions, HQ)
        got = b200.read(ob).reshape(batch, HQ * D)
        for b, p in enumerate(positions):
            close(got[b], _oracle(q[b], bits, b, p), TOL, TOL)


def test_rejects_bad_arguments(b200):
    from titania_b200 import DeviceError, Tensor

    bits = np.zeros((2, 2, HKV, 16, D), dtype=np.uint16)
    cache = b200.upload(Tensor(list(bits.shape), bits))
    qb, ob = b200.alloc(2 * HQ * D), b200.alloc(2 * HQ * D)
    with pytest.raises(DeviceError, match="past the end"):
        b200.attention_cache(ob, qb, cache, [3, 16], HQ)
    with pytest.raises(DeviceError, match="different number"):
        b200.attention_cache(ob, qb, cache, [3], HQ)
    with pytest.raises(DeviceError, match="multiple"):
        b200.attention_cache(ob, qb, cache, [3, 4], 12)
