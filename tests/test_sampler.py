"""Sampler::sample (model/sampler.rs:21-77): top-k, top-p and temperature with
the reference's xorshift64* generator.

CPU: the oracle's C restatement (oracle.cpp orc_sample) against the host
Sampler (titania_b200.model.Sampler, sums accumulated sequentially as the
reference's): identical tokens and generator states, top_k from 1 to 64 and
the CLI's default of 20 (cli/run.rs:142).
GPU: the device sampler (tb200_sampler_*) against the oracle: identical tokens
and identical generator states, draw after draw."""

import numpy as np
import pytest

from oracle import oracle as orc


def _cases(rng, n):
    for _ in range(n):
        vocab = int(rng.integers(8, 5000))
        x = (rng.standard_normal(vocab) * 3).astype(np.float32)
        yield vocab, x, float(rng.choice([0.0, 0.5, 0.7, 1.3])), float(rng.choice([0.5, 0.8, 1.0]))


def test_oracle_sampler_matches_numpy_restatement():
    from titania_b200.model import Sampler
    rng = np.random.default_rng(7)
    for vocab, x, temperature, top_p in _cases(rng, 300):
        top_k = int(rng.choice([int(rng.integers(1, 65)), 20]))
        seed = int(rng.integers(0, 2**63))
        a, b = orc.Sampler(temperature, top_k, top_p, seed), Sampler(temperature, top_k, top_p, seed)
        for _ in range(4):
            assert a.sample(x) == b.sample(x)
        assert a.state.value == b._rng


def test_host_sampler_top_k_20_near_ties():
    """top_k 20 with probabilities that need exact sequential sums: many
    near-equal logits, where a pairwise (blocked) sum can round differently
    and move the sampled token."""
    from titania_b200.model import Sampler
    rng = np.random.default_rng(11)
    for trial in range(300):
        x = (np.float32(5.0) + rng.standard_normal(4096).astype(np.float32) * np.float32(1e-3)).astype(np.float32)
        seed = int(rng.integers(1, 2**63))
        a, b = orc.Sampler(0.8, 20, 0.95, seed), Sampler(0.8, 20, 0.95, seed)
        for _ in range(3):
            assert a.sample(x) == b.sample(x)


def test_oracle_sampler_rules():
    """Temperature 0 is the greedy choice; top_k 1 always returns the best
    logit; the generator starts at max(seed, 1) and advances only when
    sampling at a temperature."""
    x = np.array([0.5, 2.0, 2.0, -1.0, 1.5], dtype=np.float32)
    g = orc.Sampler(0.0, 20, 0.8, 0)
    assert g.sample(x) == 1 and g.state.value == 1  # tie 1/2 -> lowest id; no draw at T = 0
    s = orc.Sampler(0.7, 1, 0.8, 5)
    assert all(s.sample(x) == 1 for _ in range(5))
    assert s.state.value != 5


# ---- on the GPU ----------------------------------------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("vocab,rows", [(151936, 1), (151936, 4), (1024, 3), (5000, 2), (7, 1)])
@pytest.mark.parametrize("temperature,top_k,top_p", [(0.0, 20, 0.8), (0.7, 20, 0.8), (1.0, 64, 1.0),
                                                     (1.3, 5, 0.5), (0.7, 1, 0.8)])
def test_device_sampler_matches_oracle(b200, vocab, rows, temperature, top_k, top_p):
    import titania_b200 as tb
    rng = np.random.default_rng(vocab * 7 + rows * 13 + top_k)
    seeds = [int(s) for s in rng.integers(0, 2**63, size=rows)]
    seeds[0] = 0  # the reference clamps the seed to 1
    ds = tb.DeviceSampler(b200, rows, vocab, temperature, top_k, top_p, seeds)
    refs = [orc.Sampler(temperature, top_k, top_p, s) for s in seeds]
    buf = b200.alloc(rows * vocab)
    for step in range(12):
        x = (rng.standard_normal((rows, vocab)) * (1 + step % 3)).astype(np.float32)
        if step % 4 == 3:
            x = np.round(x).astype(np.float32)  # many exact ties
        b200.write(buf, x.reshape(-1))
        got = ds.sample(buf)
        exp = [refs[i].sample(x[i]) for i in range(rows)]
        assert got.tolist() == exp, f"step {step}"
    assert ds.states().tolist() == [r.state.value for r in refs]
    ds.close()


@pytest.mark.gpu
def test_device_sampler_arguments(b200):
    import titania_b200 as tb
    with pytest.raises(tb.DeviceError, match="top_k"):
        tb.DeviceSampler(b200, 1, 151936, 0.7, 65, 0.8, [1])
    ds = tb.DeviceSampler(b200, 2, 100, 0.7, 20, 0.8, [1, 2])
    with pytest.raises(tb.DeviceError, match="fewer"):
        ds.sample(b200.alloc(150))
    ds.close()
