"""tb200_decode_persistent: greedy decode with one persistent kernel per step
(every phase of the step in one launch, phases exchanging tagged vectors),
against the oracle and against the fused path, on the seeded tiny checkpoint."""

import numpy as np
import pytest

from conftest import close

REL, ABS = 2e-2, 1e-2


@pytest.mark.gpu
def test_persistent_decode_against_oracle_and_fused_path(tiny_model_dir):
    import titania_b200 as tb
    from oracle import oracle as orc
    from titania_b200 import synth

    P, S = 9, 8
    prompt = synth.prompt_tokens(P, synth.TINY["vocab_size"], seed=3)
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(tiny_model_dir), prompt, S + 4)
    dev = tb.B200(0)
    m = tb.Model.load(tiny_model_dir, dev)

    fused = m.state(40)
    first = int(np.argmax(m.forward(fused, prompt, 0)))
    assert first == ref_tokens[0]
    fused_tokens = m.generate(fused, first, P, S)

    st = m.state(40)
    m.forward(st, prompt, 0)
    toks, logits = m.decode_persistent(st, first, P, S, logits=True)
    assert toks == fused_tokens == ref_tokens[1:S + 1]
    for i in range(S):
        close(logits[i], ref_logits[i + 1], REL, ABS)
    # the fused path continues from the cache the persistent kernel wrote
    assert m.generate(st, toks[-1], P + S, 3) == ref_tokens[S + 1:S + 4]


@pytest.mark.gpu
def test_persistent_decode_rejects_what_it_does_not_run(tiny_model_dir):
    import titania_b200 as tb
    from titania_b200 import _lib, synth

    dev = tb.B200(0)
    m = tb.Model.load(tiny_model_dir, dev)
    prompt = synth.prompt_tokens(4, synth.TINY["vocab_size"], seed=5)
    bf = m.state(32, kv="bf16")
    m.forward(bf, prompt, 0)
    with pytest.raises(_lib.DeviceError) as e:
        m.decode_persistent(bf, 1, 4, 2)
    assert e.value.code == _lib.TB200_ERR_ARG and "f32 cache" in str(e.value)
    st = m.state(128)
    m.forward(st, prompt, 0)
    with pytest.raises(_lib.DeviceError) as e:
        m.decode_persistent(st, 1, 60, 8)  # positions past 64
    assert e.value.code == _lib.TB200_ERR_ARG and "64 positions" in str(e.value)
