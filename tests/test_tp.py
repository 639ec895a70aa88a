"""Tensor parallelism (titania_b200.tp): the sharding rule and the data flow
on the CPU (two gloo ranks running the numpy restatement of
model/model.rs on their shards, partial sums added with all_reduce), then
the library on two GPUs against the oracle.

The reference has no multi-GPU path; the bar is the single-GPU one: logits
within rel 2e-2 / abs 1e-2 of the oracle and identical greedy tokens (the
partial sums are added in a different order, so results are close, not
bitwise equal)."""

import os
import sys

import numpy as np
import pytest

from conftest import ROOT, close

sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))

REL, ABS = 2e-2, 1e-2


def test_shard_rule_reassembles(tiny_model_dir):
    """Every rank's slices, put back together, are the whole tensor."""
    from titania_b200.model import Config, Weights, tensor_names
    from titania_b200.tp import shard_config, shard_tensor
    c = Config.load(os.path.join(tiny_model_dir, "config.json"))
    w = Weights.open(os.path.join(tiny_model_dir, "model.safetensors"))
    world = 2
    lc = shard_config(c, world)
    assert (lc.num_attention_heads, lc.num_key_value_heads, lc.intermediate_size) == (2, 1, 256)
    for name, _ in tensor_names(c):
        t = w.read(name)
        full = t.data.reshape(t.shape)
        parts = [shard_tensor(c, name, t.shape, t.data, r, world) for r in range(world)]
        arrs = [p[1].reshape(p[0]) for p in parts]
        if name.endswith(("o_proj.weight", "down_proj.weight")):
            back = np.concatenate(arrs, axis=1)
        elif name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight", "gate_proj.weight", "up_proj.weight")):
            back = np.concatenate(arrs, axis=0)
        else:
            assert all(np.array_equal(a, full) for a in arrs), name  # replicated
            continue
        assert np.array_equal(back, full), name


def test_shard_rule_rejects_uneven():
    from titania_b200.model import Config
    from titania_b200 import synth
    from titania_b200.tp import shard_config
    c = Config(**synth.TINY)
    with pytest.raises(ValueError):
        shard_config(c, 4)  # 2 kv heads over 4 ranks


def _np_tp_rank(rank, world, port, model_dir, prompt, q):
    """One gloo rank: the numpy restatement of model.rs's forward on this
    rank's shards, with the o_proj and down_proj partial sums all-reduced."""
    import torch
    import torch.distributed as dist

    import gen_golden as g
    from titania_b200.model import Config
    from titania_b200.tp import shard_config, shard_tensor
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        m = g.NpModel(model_dir)
        c = Config.load(os.path.join(model_dir, "config.json"))
        lc = shard_config(c, world)
        t = {k: shard_tensor(c, k, v.shape, v.reshape(-1), rank, world) for k, v in m.t.items()}
        t = {k: s[1].reshape(s[0]) for k, s in t.items()}
        hd = c.head_dim()
        H, eps = c.hidden_size, np.float32(c.rms_norm_eps)
        nh, nkv = lc.num_attention_heads, lc.num_key_value_heads
        n = len(prompt)
        table = g.np_rope_table(n, hd, np.float32(c.rope_theta))
        kv_dim = nkv * hd

        def allreduce(v):
            x = torch.from_numpy(v.copy())
            dist.all_reduce(x)
            return x.numpy()

        x = g.bf16(t["model.embed_tokens.weight"][prompt]).reshape(-1).copy()
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}"
            xb = g.np_rmsnorm(x, t[f"{p}.input_layernorm.weight"], eps)
            qv = g.np_matmul(t[f"{p}.self_attn.q_proj.weight"], xb)
            kv = g.np_matmul(t[f"{p}.self_attn.k_proj.weight"], xb)
            vv = g.np_matmul(t[f"{p}.self_attn.v_proj.weight"], xb)
            qv = g.np_rmsnorm(qv, t[f"{p}.self_attn.q_norm.weight"], eps)
            kv = g.np_rmsnorm(kv, t[f"{p}.self_attn.k_norm.weight"], eps)
            qv = g.np_rope(qv, table, 0, nh, hd)
            kv = g.np_rope(kv, table, 0, nkv, hd)
            kc = np.zeros(n * kv_dim, np.float32)
            vc = np.zeros(n * kv_dim, np.float32)
            kc[:] = kv
            vc[:] = vv
            att = g.np_attention(qv, kc, vc, 0, nh, hd, nkv)
            x = x + allreduce(g.np_matmul(t[f"{p}.self_attn.o_proj.weight"], att))
            xb = g.np_rmsnorm(x, t[f"{p}.post_attention_layernorm.weight"], eps)
            gg = g.np_matmul(t[f"{p}.mlp.gate_proj.weight"], xb)
            uu = g.np_matmul(t[f"{p}.mlp.up_proj.weight"], xb)
            x = x + allreduce(g.np_matmul(t[f"{p}.mlp.down_proj.weight"], g.np_silu_mul(gg, uu)))
        xl = g.np_rmsnorm(x[(n - 1) * H:n * H], t["model.norm.weight"], eps)
        logits = g.np_matmul(t["model.embed_tokens.weight"], xl)
        q.put((rank, logits))
        dist.destroy_process_group()
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_tp_data_flow_gloo(tiny_model_dir):
    """Two CPU ranks (gloo) compute the tiny model's prompt logits from their
    shards; the all-reduced result matches the unsharded restatement."""
    import multiprocessing as mp
    import socket

    import gen_golden as g
    from titania_b200 import synth
    prompt = synth.prompt_tokens(9, 1024, seed=3)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_np_tp_rank, args=(r, 2, port, tiny_model_dir, prompt, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert all(not isinstance(v, str) for v in out.values()), out
    m = g.NpModel(tiny_model_dir)
    kv = [[np.zeros(len(prompt) * 256, np.float32), np.zeros(len(prompt) * 256, np.float32)] for _ in range(2)]
    exp = m.forward(kv, prompt, 0, len(prompt))
    for r in range(2):
        close(out[r], exp, 1e-5, 1e-5)


# ---- on two GPUs -------------------------------------------------------------

def _gpu_tp_rank(rank, world, port, model_dir, prompt, steps, kv, q, late=0.0, decode=None):
    # No NVLink multicast (NVLS) in tests: a rank that dies bound to a
    # multicast object can fault the other ranks' GPUs.
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    import torch
    import torch.distributed as dist

    import titania_b200 as tb
    from titania_b200.tp import TPGroup, load_tp_model
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        dev = tb.B200(rank)
        uid = [TPGroup.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        group = TPGroup(dev, rank, world, uid[0])
        m = load_tp_model(model_dir, dev, group)
        peer = m.tp_peer_exchange
        st = m.state(len(prompt) + steps + 2, kv=kv, decode=decode)
        logits = [m.forward(st, prompt, 0)]
        if late:
            # The last rank starts its first single-token step `late` seconds
            # after the others: their kernels wait a bounded second for its
            # partial sums and report TB200_ERR_TIMEOUT; no rank hangs.
            import time
            if rank == world - 1:
                time.sleep(late)
            tok = int(np.argmax(logits[-1]))
            code = 0
            try:
                m.forward(st, [tok], len(prompt))
            except tb.DeviceError as e:
                code = e.code
            q.put((rank, (peer, code)))
            del st, m
            group.close()
            dist.destroy_process_group()
            return
        toks = [int(np.argmax(logits[-1]))]
        pos = len(prompt)
        for _ in range(steps):
            logits.append(m.forward(st, [toks[-1]], pos))
            toks.append(int(np.argmax(logits[-1])))
            pos += 1
        # the device-side loop and the batched path agree with the host loop
        st2 = m.state(len(prompt) + steps + 2, kv=kv, decode=decode)
        first = m.forward(st2, prompt, 0, logits=False)
        gen = [first] + m.generate(st2, first, len(prompt), steps)
        bs = m.batch_state(2, len(prompt) + steps + 2, kv=kv)
        bfirst = [m.forward_seq(bs, i, prompt, 0, logits=False) for i in range(2)]
        bgen = m.generate_batch(bs, bfirst, [len(prompt)] * 2, steps)
        q.put((rank, (np.stack(logits), toks, gen, [bfirst] + bgen.tolist(), peer, st.decode)))
        del st, st2, bs, m
        group.close()
        dist.destroy_process_group()
    except Exception as e:
        import traceback
        q.put((rank, traceback.format_exc()))


def _run_tp(model_dir, prompt, steps, kv, world=2, late=0.0, decode=None):
    import multiprocessing as mp
    import socket
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gpu_tp_rank, args=(r, world, port, model_dir, prompt, steps, kv, q, late, decode))
             for r in range(world)]
    for p in procs:
        p.start()
    try:
        out = dict(q.get(timeout=600) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():  # a rank stuck in a collective: end it (its GPU work ends with it)
                p.terminate()
                p.join(timeout=30)
    for r, v in out.items():
        assert not isinstance(v, str), f"rank {r}:\n{v}"
    return out


def _two_gpus():
    try:
        import torch
        return torch.cuda.device_count() >= 2
    except Exception:
        return False


@pytest.mark.gpu
def test_tp1_group_load_against_oracle(tiny_model_dir):
    """load_tp_model (checkpoint windows straight to the device) with a
    one-rank group, on one GPU: the logits after a prompt match the oracle
    and the greedy token is the oracle's."""
    import titania_b200 as tb
    from oracle import oracle as orc
    from titania_b200 import synth
    from titania_b200.tp import TPGroup, load_tp_model
    prompt = synth.prompt_tokens(9, 1024, seed=3)
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(tiny_model_dir), prompt, 2)
    dev = tb.B200(0)
    group = TPGroup(dev, 0, 1, TPGroup.unique_id())
    try:
        m = load_tp_model(tiny_model_dir, dev, group)
        st = m.state(32)
        logits = m.forward(st, prompt, 0)
        close(logits, ref_logits[0], REL, ABS)
        assert int(np.argmax(logits)) == ref_tokens[0]
        del st, m
    finally:
        group.close()


@pytest.mark.gpu
@pytest.mark.parametrize("kv", ["f32", "bf16"])
@pytest.mark.parametrize("plen", [9, 70])
def test_tp2_tiny_against_oracle(tiny_model_dir, kv, plen):
    """Two ranks against the oracle: single-token steps on the persistent
    kernel (the default; o_proj and down_proj partials by peer stores),
    prompts and the batched path with NCCL."""
    if not _two_gpus():
        pytest.skip("needs two GPUs")
    from oracle import oracle as orc
    from titania_b200 import synth
    prompt = synth.prompt_tokens(plen, 1024, seed=3)
    steps = 6
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(tiny_model_dir), prompt, steps + 1, max_len=plen + 16)
    out = _run_tp(tiny_model_dir, prompt, steps, kv)
    for r, (logits, toks, gen, bgen, peer, decode) in out.items():
        assert peer, f"rank {r}: the partial sums should go by peer stores on distinct GPUs"
        assert decode == "persistent", f"rank {r}: tensor-parallel single-token steps run the persistent kernel"
        for i in range(steps + 1):
            close(logits[i], ref_logits[i], REL, ABS)
        assert toks == ref_tokens, f"rank {r}"
        assert gen == ref_tokens, f"rank {r}: device loop"
        assert [row[0] for row in bgen] == ref_tokens and [row[1] for row in bgen] == ref_tokens, f"rank {r}: batch"


@pytest.mark.gpu
@pytest.mark.parametrize("plen", [9, 70])
def test_tp2_tiny_fused_path_against_oracle(tiny_model_dir, plen):
    """The fused single-token graphs at TP2 (what a state runs when it asks
    for them): with a 9-token prompt the short-context graph (attention +
    o_proj per kv group, NCCL for those partials, peer stores for
    down_proj); past 64 positions every partial sum goes by peer stores."""
    if not _two_gpus():
        pytest.skip("needs two GPUs")
    from oracle import oracle as orc
    from titania_b200 import synth
    prompt = synth.prompt_tokens(plen, 1024, seed=3)
    steps = 6
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(tiny_model_dir), prompt, steps + 1, max_len=plen + 16)
    out = _run_tp(tiny_model_dir, prompt, steps, "f32", decode="fused")
    for r, (logits, toks, gen, bgen, peer, decode) in out.items():
        assert peer and decode == "fused", f"rank {r}"
        for i in range(steps + 1):
            close(logits[i], ref_logits[i], REL, ABS)
        assert toks == ref_tokens and gen == ref_tokens, f"rank {r}"


@pytest.mark.gpu
def test_tp2_qwen3_0_6b_against_oracle():
    if not _two_gpus():
        pytest.skip("needs two GPUs")
    from oracle import oracle as orc
    from titania_b200 import synth
    d = synth.cached_model("qwen3-0.6b", seed=0)
    prompt = synth.prompt_tokens(16, 151936, seed=1)
    steps = 8
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(d), prompt, steps + 1, max_len=64)
    out = _run_tp(d, prompt, steps, "f32")
    for r, (logits, toks, gen, bgen, peer, decode) in out.items():
        assert decode == "persistent"
        for i in range(steps + 1):
            close(logits[i], ref_logits[i], REL, ABS)
        assert toks == ref_tokens and gen == ref_tokens, f"rank {r}"


@pytest.mark.gpu
def test_tp2_qwen3_4b_two_layers_against_oracle():
    """Two layers of Qwen3-4B over two ranks (each: 4 kv heads, 4864 FFN
    columns, the wide persistent kernel with o_proj and down_proj partials
    exchanged by peer stores) against the oracle."""
    if not _two_gpus():
        pytest.skip("needs two GPUs")
    from oracle import oracle as orc
    from titania_b200 import synth
    d = synth.cached_model("qwen3-4b-2l", seed=0)
    prompt = synth.prompt_tokens(12, 151936, seed=5)
    steps = 4
    ref_tokens, ref_logits = orc.greedy_generate(orc.Model(d), prompt, steps + 1, max_len=32)
    out = _run_tp(d, prompt, steps, "f32")
    for r, (logits, toks, gen, bgen, peer, decode) in out.items():
        assert peer and decode == "persistent", f"rank {r}"
        for i in range(steps + 1):
            close(logits[i], ref_logits[i], REL, ABS)
        assert toks == ref_tokens and gen == ref_tokens, f"rank {r}"


@pytest.mark.gpu
@pytest.mark.parametrize("decode", ["persistent", "fused"])
def test_tp2_late_rank_times_out_without_hanging(tiny_model_dir, decode):
    """A rank that starts its step three seconds late: the other rank's
    kernels give up their bounded wait for its partial sums after a second
    and the call reports TB200_ERR_TIMEOUT; the late rank then finds the
    other's words or flags written and finishes; both processes end
    normally."""
    if not _two_gpus():
        pytest.skip("needs two GPUs")
    from titania_b200 import _lib, synth
    prompt = synth.prompt_tokens(70, 1024, seed=4)  # past 64 positions: no NCCL in the fused step
    out = _run_tp(tiny_model_dir, prompt, 1, "f32", late=3.0, decode=decode)
    assert out[0] == (True, _lib.TB200_ERR_TIMEOUT), out
    assert out[1][0] is True


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_rule_reassembles_at_4_and_8_ranks(tmp_path, world):
    """The sharding rule at the tensor-parallel widths of the scaling run, on a
    small model with 8 kv heads (as Qwen3-4B): every rank's slices put back
    together are the whole tensor, and the per-rank shapes divide evenly."""
    from titania_b200 import synth
    from titania_b200.model import Config, Weights, tensor_names
    from titania_b200.tp import shard_config, shard_tensor
    cfg = dict(synth.TINY, num_attention_heads=16, num_key_value_heads=8, intermediate_size=1024)
    d = str(tmp_path / "tiny-kv8")
    synth.write_model(d, cfg, seed=9)
    c = Config.load(os.path.join(d, "config.json"))
    w = Weights.open(os.path.join(d, "model.safetensors"))
    lc = shard_config(c, world)
    assert lc.num_key_value_heads * world == 8 and lc.num_attention_heads * world == 16
    assert lc.intermediate_size * world == 1024
    for name, _ in tensor_names(c):
        t = w.read(name)
        full = t.data.reshape(t.shape)
        arrs = [p[1].reshape(p[0]) for p in (shard_tensor(c, name, t.shape, t.data, r, world) for r in range(world))]
        if name.endswith(("o_proj.weight", "down_proj.weight")):
            back = np.concatenate(arrs, axis=1)
        elif name.endswith(("q_proj.weight", "k_proj.weight", "v_proj.weight", "gate_proj.weight", "up_proj.weight")):
            back = np.concatenate(arrs, axis=0)
        else:
            assert all(np.array_equal(a, full) for a in arrs), name
            continue
        assert np.array_equal(back, full), name


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_qwen3_4b_shards_fit_the_kernels(world):
    """Config 4 at TP 1-8: per-rank widths are multiples of the kernels' 64-column
    blocks and 16-row tiles, and a kv head keeps whole query groups."""
    from titania_b200 import synth
    from titania_b200.model import Config
    from titania_b200.tp import shard_config
    lc = shard_config(Config(**synth.QWEN3_4B), world)
    hd = lc.head_dim()
    widths = [lc.hidden_size, lc.intermediate_size, lc.num_attention_heads * hd, lc.num_key_value_heads * hd]
    assert all(x % 64 == 0 for x in widths), widths
    assert lc.num_attention_heads % lc.num_key_value_heads == 0
    assert (lc.num_attention_heads // lc.num_key_value_heads) in (1, 2, 4, 8)
