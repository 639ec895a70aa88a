"""The persistent single-token step (TB200_DECODE_PERSISTENT: one kernel per
launch runs every phase of every step, the phases exchanging tagged vectors)
against the oracle and against the fused path.

Shapes are chosen so that every branch of the kernel runs: the tiny model
(few rows per CTA, inputs narrower than 256 columns), two layers of
Qwen3-0.6B (every matrix at its real per-CTA row count; the lm_head's last
ring stage has three rows and takes the column-split branch), two layers of
Qwen3-4B (hidden 2560, FFN 9728: the smaller ring slots, batched polls of
the 9728-wide input, down_proj in three-row stages split by columns over
the warps, layers streamed without L2 prefetch), and a model with four
query heads per kv head and more than eight residual rows per CTA. Contexts
past 256 positions take the split attention (members of a kv group
exchange partial softmax results)."""

import os

import numpy as np
import pytest

from conftest import ROOT, close

pytestmark = pytest.mark.gpu

REL, ABS = 2e-2, 1e-2  # the north star's logit bound against the oracle


def _load(name):
    import titania_b200 as tb
    from titania_b200 import synth

    return synth.cached_model(name, seed=0), tb


@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_tiny_against_oracle_and_fused_path(b200, tiny_model_dir, kv):
    import titania_b200 as tb
    from oracle import oracle as orc
    from titania_b200 import synth

    P, S = 9, 8
    prompt = synth.prompt_tokens(P, synth.TINY["vocab_size"], seed=3)
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(tiny_model_dir), prompt, S + 4)
    m = tb.Model.load(tiny_model_dir, b200)

    fused = m.state(40, kv=kv, decode="fused")
    first = int(np.argmax(m.forward(fused, prompt, 0)))
    assert first == ref_tokens[0]
    fused_tokens = m.generate(fused, first, P, S)

    st = m.state(40, kv=kv)
    assert st.decode == "persistent"  # the default where the model allows it
    m.forward(st, prompt, 0)
    toks, logits = m.decode_persistent(st, first, P, S, logits=True)
    assert toks == fused_tokens == ref_tokens[1:S + 1]
    for i in range(S):
        close(logits[i], ref_logits[i + 1], REL, ABS)
    # the fused path continues from the cache the persistent kernel wrote
    st.decode = "fused"
    assert m.generate(st, toks[-1], P + S, 3) == ref_tokens[S + 1:S + 4]


@pytest.mark.parametrize("name", ["qwen3-0.6b-2l", "qwen3-4b-2l", "wide-gqa4"])
def test_every_branch_against_fused_path_and_oracle(b200, name):
    """Logits of every step within 1e-4 of the fused path's (f32 cache: the
    two differ only in summation order) and within the north-star bound of
    the oracle's; tokens identical; one launch of many steps gives the same
    tokens as one launch per step."""
    import titania_b200 as tb
    from oracle import oracle as orc
    from titania_b200 import synth

    path = synth.cached_model(name, seed=0)
    cfg = synth.CONFIGS[name]
    P, S = 12, 6
    prompt = synth.prompt_tokens(P, cfg["vocab_size"], seed=4)
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(path), prompt, S + 1, max_len=32)
    m = tb.Model.load(path, b200)

    fused = m.state(32, decode="fused")
    first = int(np.argmax(m.forward(fused, prompt, 0)))
    assert first == ref_tokens[0]
    fused_logits = []
    tok = first
    for i in range(S):
        lg = m.forward(fused, [tok], P + i)
        fused_logits.append(lg.copy())
        tok = int(np.argmax(lg))

    st = m.state(32, decode="persistent")
    m.forward(st, prompt, 0)
    toks, logits = m.decode_persistent(st, first, P, S, logits=True)
    assert toks == ref_tokens[1:S + 1]
    for i in range(S):
        close(logits[i], fused_logits[i], 1e-4, 1e-4)
        close(logits[i], ref_logits[i + 1], REL, ABS)

    st2 = m.state(32)
    m.forward(st2, prompt, 0)
    assert m.generate(st2, first, P, S) == toks


LONG_MODELS = {  # name: changes to the tiny checkpoint
    "tiny": None,
    "wide-ffn": dict(intermediate_size=3328),                              # the wide kernel
    "gqa4": dict(num_attention_heads=8),                                   # four query heads per kv head
    "gqa4-wide": dict(num_attention_heads=8, intermediate_size=3328),      # both
}


@pytest.mark.parametrize("model", list(LONG_MODELS))
@pytest.mark.parametrize("kv", ["f32", "bf16"])
def test_long_context_split_attention(b200, tiny_model_dir, kv, model):
    """A 1100-token prompt (the tensor-core prompt path), then greedy steps
    past 1100 positions: the members of each kv group attend to their share
    of the context and merge partials. Against the oracle, on the narrow
    kernel (tiny) and the wide one (an FFN of 3328 columns, 74 members per
    kv group; its down_proj stages of one or two rows split by columns),
    each with two and with four query heads per kv head (the merge then
    runs in two quarters of the threads instead of four)."""
    import titania_b200 as tb
    from oracle import oracle as orc
    from titania_b200 import synth

    d = tiny_model_dir
    if LONG_MODELS[model]:
        d = os.path.join(ROOT, "_build", "long-" + model)
        synth.write_model(d, dict(synth.TINY, **LONG_MODELS[model]), seed=6)
    P, S = 1100, 6
    prompt = synth.prompt_tokens(P, synth.TINY["vocab_size"], seed=8)
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(d), prompt, S + 1, max_len=P + S + 2)
    m = tb.Model.load(d, b200)
    st = m.state(P + S + 2, kv=kv)
    assert st.decode == "persistent"
    first = int(np.argmax(m.forward(st, prompt, 0)))
    assert first == ref_tokens[0]
    toks, logits = m.decode_persistent(st, first, P, S, logits=True)
    assert toks == ref_tokens[1:S + 1]
    tol = (1e-3, 1e-3) if kv == "f32" else (REL, ABS)
    for i in range(S):
        close(logits[i], ref_logits[i + 1], *tol)
    # many steps in one launch cross from the positions the prompt wrote into
    # those this launch appends
    st2 = m.state(P + S + 2, kv=kv)
    m.forward(st2, prompt, 0)
    assert m.generate(st2, first, P, S) == toks


def test_modes_and_rejection(b200, tiny_model_dir):
    """A model the persistent kernel cannot run (FFN wider than 10240) keeps
    the fused path by default and refuses the persistent one with a reason;
    unknown modes are refused."""
    import titania_b200 as tb
    from titania_b200 import _lib, synth

    m = tb.Model.load(tiny_model_dir, b200)
    st = m.state(16)
    with pytest.raises(ValueError):
        st.decode = "fast"
    with pytest.raises(_lib.DeviceError) as e:
        _lib.call("tb200_state_set_decode", st._h, 7)
    assert e.value.code == _lib.TB200_ERR_ARG

    wide = dict(synth.TINY, intermediate_size=10496, num_hidden_layers=1)
    d = os.path.join(ROOT, "_build", "wide-ffn")
    synth.write_model(d, wide, seed=2)
    mw = tb.Model.load(d, b200)
    sw = mw.state(16)
    assert sw.decode == "fused"
    with pytest.raises(_lib.DeviceError) as e:
        sw.decode = "persistent"
    assert e.value.code == _lib.TB200_ERR_ARG and "10240" in str(e.value)
    with pytest.raises(_lib.DeviceError) as e:
        mw.decode_persistent(sw, 1, 0, 2)
    assert e.value.code == _lib.TB200_ERR_ARG
    # the fused path still decodes it
    prompt = synth.prompt_tokens(4, wide["vocab_size"], seed=1)
    first = mw.forward(sw, prompt, 0, logits=False)
    assert len(mw.generate(sw, first, 4, 3)) == 3


def test_logits_into_page_locked_memory(b200, tiny_model_dir):
    """A single-token forward whose logits buffer is page-locked host memory
    gets them written by the persistent kernel itself (no copy after it):
    the same bits as through a pageable buffer, step after step."""
    torch = pytest.importorskip("torch")
    import titania_b200 as tb
    from titania_b200 import synth

    m = tb.Model.load(tiny_model_dir, b200)
    prompt = synth.prompt_tokens(9, synth.TINY["vocab_size"], seed=3)
    pinned = torch.empty(synth.TINY["vocab_size"], dtype=torch.float32, pin_memory=True).numpy()
    a, b = m.state(32), m.state(32)
    tok_a = int(np.argmax(m.forward(a, prompt, 0)))
    tok_b = int(np.argmax(m.forward(b, prompt, 0)))
    for i in range(4):
        la = m.forward(a, [tok_a], 9 + i).copy()  # pageable: copied after the kernel
        m.forward(b, [tok_b], 9 + i, out=pinned)  # page-locked: written by the kernel
        assert np.array_equal(la, pinned), i
        tok_a, tok_b = int(np.argmax(la)), int(np.argmax(pinned))
        assert tok_a == tok_b
