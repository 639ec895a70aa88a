"""Benchmark: Qwen3-0.6B greedy decode on B200 at batch 1
and batch 64 (config 3).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

One step is one decoded token. The workload replays config 0's generation
(16-token prompt, then 32 greedy steps, so the context runs 16..48) as many
times as the step count needs; K steps therefore cover K/32 generations.
Weights are seeded random-init bf16 (no real checkpoint offline).

`value` is device-timed tok/s with everything resident in HBM; `e2e` is the
same metric through the public forward call with host buffers: each step
copies its token and position in and the logits (vocab_size f32) and greedy
token out, as Model::forward + Sampler do in the reference loop.

`--impl reference` times the CPU restatement of the reference path (the
reference itself is Rust and cannot be built here) on the host cores.
With N > 1 (torchrun), every rank runs its own batch-1 decode stream
(replicas); value is the sum of tokens over the max time across ranks.

The `bs64` object: config 3's batched decode (64 sequences, each prefilled
with 1024 ids through the tensor-core prompt path, then 128 greedy steps of
all sequences at once, bf16 K/V cache), device-timed, with its own e2e
(one tb200_forward_batch call per step, tokens in and greedy tokens out).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Qwen3-0.6B decode tok/s (bs1, bs64) + achieved HBM GB/s vs 8 TB/s peak"
PROMPT = 16
GEN = 32  # greedy steps per generation (config 0)
NOMINAL_HBM_GBS = 8000.0


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def model_bytes(c, kv_bytes=4):
    """Algorithmic bytes of one batch-1 decode step: every weight once (tied
    lm_head counted once as the head; the embedding row is 2*H bytes) plus
    the K/V read at the step's context (kv_bytes per element)."""
    H, F, L, V = c["hidden_size"], c["intermediate_size"], c["num_hidden_layers"], c["vocab_size"]
    D, Hq, Hkv = c["head_dim"], c["num_attention_heads"], c["num_key_value_heads"]
    q_dim, kv_dim = Hq * D, Hkv * D
    linear = L * (H * (q_dim + 2 * kv_dim) + q_dim * H + 3 * H * F) * 2
    norms = (L * (2 * H + 2 * D) + H) * 2
    head = V * H * 2
    return linear + norms + head + 2 * H, 2 * L * kv_dim * kv_bytes  # (weights, kv bytes per context position)


class Clocks:
    """Samples SM clocks and throttle reasons with nvidia-smi during a region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def _query(self):
        try:
            r = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                "--format=csv,noheader,nounits"], capture_output=True, text=True, timeout=20)
            return [ln for ln in r.stdout.splitlines() if ln.strip()]
        except (OSError, subprocess.SubprocessError):
            return []

    def __enter__(self):
        # One sample just before the region and one just after it (a timed
        # region shorter than the sampling period would otherwise have none),
        # and a 100 ms stream in between.
        self.before = self._query()
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc:
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [ln for ln in out.splitlines() if ln.strip()]
        self.lines = self.before + self.lines + self._query()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def busy(torch, us=300):
    """Keeps the GPU busy for about `us` microseconds (a spin kernel on the
    current stream), so that the host has enqueued the next timed work before
    the GPU reaches it and the events time the device alone."""
    torch.cuda._sleep(int(us * 2000))


def timed_calls(torch, stream, fn, reps, flush=None):
    """Device durations (s) of `fn` (which only enqueues work on `stream`),
    one per repetition; `flush` (a buffer larger than L2) is rewritten before
    each, so no repetition finds its inputs in L2."""
    ts = []
    with torch.cuda.stream(stream):
        for _ in range(reps):
            busy(torch)
            if flush is not None:
                flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            ts.append((e0, e1))
    torch.cuda.synchronize()
    return [a.elapsed_time(b) * 1e-3 for a, b in ts]


def timeline(tr, names, end_tag=None):
    """Splits a traced decode step into consecutive segments, one per launch
    (or phase of the persistent kernel), ordered by when its last CTA
    finished: a segment runs from the previous unit's last DONE to this
    one's, the first from the step's earliest record. The segments add up to
    the step; per op they are summed over layers (us). Also the median over
    CTAs of each unit's own INPUT -> DONE time, averaged over its layers."""
    tr = tr[tr["ns"] > 0]
    t0 = int(tr["ns"].min())
    done = {}
    work = {}
    for tag in np.unique(tr["tag"]):
        r = tr[tr["tag"] == tag]
        d = r[r["event"] == 4]
        if not d.size:
            continue
        done[int(tag)] = int(d["ns"].max())
        i = r[r["event"] == 2]
        if i.size:
            by = {int(x["cta"]): int(x["ns"]) for x in i}
            w = [int(x["ns"]) - by[int(x["cta"])] for x in d if int(x["cta"]) in by]
            if w:
                work[int(tag)] = float(np.median(w))
    seg, comp, cnt = {}, {}, {}
    prev = t0
    for tag, t in sorted(done.items(), key=lambda kv: kv[1]):
        name = names.get(tag >> 16, str(tag >> 16))
        seg[name] = seg.get(name, 0.0) + (t - prev) / 1e3
        if tag in work:
            comp[name] = comp.get(name, 0.0) + work[tag] / 1e3
            cnt[name] = cnt.get(name, 0) + 1
        prev = t
    return {"step_us": (prev - t0) / 1e3,
            "segments_us": {k: round(v, 2) for k, v in seg.items()},
            "own_work_us_per_launch": {k: round(comp[k] / cnt[k], 3) for k in comp}}


PERSIST_NAMES = {32: "q|k|v", 33: "attention + o_proj partials + residual", 34: "gate|up + silu", 35: "down + residual",
                 36: "lm_head + argmax", 38: "token"}
FUSED_NAMES = {0: "embed", 1: "q|k|v", 2: "attention", 3: "o_proj", 4: "gate|up", 5: "down", 6: "lm_head",
               7: "attention + o_proj", 8: "gate|up (+o partials)"}
BATCH_NAMES = {16: "embed", 17: "rmsnorm (tp)", 18: "q|k|v (tcgen05)", 20: "attention", 21: "o_proj (tcgen05)",
               22: "rmsnorm 2 (tp)", 23: "gate|up (tcgen05)", 24: "down (tcgen05)", 25: "final norm (tp)",
               26: "lm_head (tcgen05)", 27: "argmax"}


def step_trace(m, st, first, decode, prompt=PROMPT):
    """One traced single-token step at position prompt + 16 (the middle of
    config 0's contexts) on the given path."""
    prev = st.decode
    st.decode = decode
    m.decode_enqueue(st, first, prompt, 16)
    st.trace_start(1 << 22)
    m.decode_enqueue(st, first, prompt + 16, 1)
    tr = st.trace_stop()
    st.decode = prev
    return timeline(tr, PERSIST_NAMES if decode == "persistent" else FUSED_NAMES)


def run_attn_sweep(tb, dev, torch, peak):
    """GQA decode attention (16 query / 8 kv heads,
    head_dim 128) over a bf16 cache, contexts 512 / 4096 / 32768 at batch 1
    and 64, through tb200_attention_cache. Each call is timed alone on the
    device with L2 flushed before it; bytes = the K and V read."""
    stream = torch.cuda.ExternalStream(dev.stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    rng = np.random.default_rng(0)
    from titania_b200.synth import f32_to_bf16_bits
    block = f32_to_bf16_bits(rng.standard_normal(1 << 24, dtype=np.float32))
    out = []
    for batch in (1, 64):
        shape = (batch, 2, 8, 32768, 128)
        bits = np.resize(block, int(np.prod(shape))).reshape(shape)  # K, V ~ N(0, 1) in bf16 (a 16M-value block tiled)
        cache = dev.upload(tb.Tensor(list(shape), bits))
        del bits
        q, o = dev.alloc(batch * 2048), dev.alloc(batch * 2048)
        dev.write(q, rng.standard_normal(batch * 2048, dtype=np.float32))
        for ctx in (512, 4096, 32768):
            pos = [ctx - 1] * batch
            for _ in range(3):
                dev.attention_cache(o, q, cache, pos, 16)
            dev.sync()
            t = statistics.median(timed_calls(torch, stream, lambda: dev.attention_cache(o, q, cache, pos, 16), 20,
                                              flush))
            nbytes = batch * ctx * 8 * 128 * 2 * 2 + 2 * batch * 2048 * 4
            out.append({"ctx": ctx, "batch": batch, "us": t * 1e6, "gbs": nbytes / t / 1e9,
                        "frac_of_measured": nbytes / t / 1e9 / peak})
        del cache, q, o
    dev.sync()
    return {"workload": "config 2: GQA decode attention, 16 q / 8 kv heads, head_dim 128, bf16 K/V ~N(0,1)",
            "op": "tb200_attention_cache (tensor-core decode attention + planes -> f32)",
            "l2": "256 MB written before every timed call", "timing": "median of 20 calls, CUDA events",
            "peak_gbs": peak, "points": out}


def run_op_sweep(tb, dev, torch):
    """BASELINE config 1, the ops besides the fused matvecs, one trait call
    each (model/cpu.rs:85-111, 151-155): RMSNorm over 1024 and per head over
    128 (16 + 8 heads), RoPE on 16 + 8 heads x 128 at position 4095, SiLU-mul
    over 3072; and the matvecs of Qwen3-0.6B's shapes through the trait's
    matmul at batch 1. Each timed alone on the device after an L2 flush."""
    from titania_b200 import synth
    stream = torch.cuda.ExternalStream(dev.stream)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    rng = np.random.default_rng(1)

    def buf(n, std=1.0):
        b = dev.alloc(n)
        dev.write(b, (rng.standard_normal(n, dtype=np.float32) * std).astype(np.float32))
        return b

    def weight(shape, std=0.02):
        return dev.upload(tb.Tensor(list(shape), synth.f32_to_bf16_bits(
            rng.standard_normal(int(np.prod(shape)), dtype=np.float32) * np.float32(std))))

    ones1024 = dev.upload(tb.Tensor([1024], np.full(1024, 0x3F80, dtype=np.uint16)))
    ones128 = dev.upload(tb.Tensor([128], np.full(128, 0x3F80, dtype=np.uint16)))
    x = buf(1024)
    heads = buf(24 * 128)
    table = dev.alloc(4096 * 128)
    tab = np.empty(4096 * 128, dtype=np.float32)
    _lib_call = tb._lib.call
    _lib_call("tb200_rope_table", 4096, 128, np.float32(1e6).item(), tab.ctypes.data_as(tb._lib.F32P))
    dev.write(table, tab)
    g, u = buf(3072), buf(3072)
    ops = {
        "rmsnorm 1024": (lambda: dev.rmsnorm(x, ones1024, 1e-6), 1024 * 4 * 2 + 1024 * 2),
        "rmsnorm per head 24 x 128": (lambda: dev.rmsnorm(heads, ones128, 1e-6), 24 * 128 * 4 * 2 + 128 * 2),
        "rope 24 heads x 128 at 4095": (lambda: dev.rope(heads, table, 4095, 24, 128), 24 * 128 * 4 * 2 + 128 * 4),
        "silu_mul 3072": (lambda: dev.silu_mul(g, u), 3072 * 4 * 3),
    }
    for name, (rows, cols) in (("q", (2048, 1024)), ("k", (1024, 1024)), ("v", (1024, 1024)), ("o", (1024, 2048)),
                               ("gate", (3072, 1024)), ("up", (3072, 1024)), ("down", (1024, 3072)),
                               ("lm_head", (151936, 1024))):
        w = weight((rows, cols))
        xin, xo = buf(cols), dev.alloc(rows)
        ops[f"matmul {name} {rows}x{cols}"] = ((lambda w=w, xin=xin, xo=xo: dev.matmul(xo, w, xin)),
                                               rows * cols * 2 + cols * 4 + rows * 4)
    res = {}
    for name, (fn, nbytes) in ops.items():
        fn()
        dev.sync()
        t = statistics.median(timed_calls(torch, stream, fn, 20, flush))
        res[name] = {"us": t * 1e6, "gbs": nbytes / t / 1e9, "bytes": nbytes}
    dev.sync()
    return {"workload": "config 1: per-op sweep on Qwen3-0.6B shapes (trait ops, batch 1)",
            "l2": "256 MB written before every timed call", "timing": "median of 20 calls, CUDA events",
            "ops": res}


def run_prefill(tb, m, dev, cfg, torch):
    """BASELINE config 3's prompt: 2048 uniform token ids at batch 1 through
    Model::forward (the tensor-core path, passes of up to 1024 tokens).
    FLOPs: 2 x the linear parameters x tokens (the lm_head only for the last
    token) + causal attention 2 x 2 x head_dim x T^2 / 2 per head and layer."""
    from titania_b200 import synth
    T = 2048
    prompt = synth.prompt_tokens(T, cfg["vocab_size"], seed=3)
    st = m.state(T + 1, kv="bf16")
    stream = torch.cuda.ExternalStream(dev.stream)
    m.forward(st, prompt, 0, logits=False)
    times = []
    for _ in range(3):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        m.forward(st, prompt, 0, logits=False)
        e1.record(stream)
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1) * 1e-3)
    t = min(times)
    H, F, L, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["num_hidden_layers"], cfg["head_dim"]
    q_dim, kv_dim = cfg["num_attention_heads"] * D, cfg["num_key_value_heads"] * D
    linear = L * (H * (q_dim + 2 * kv_dim) + q_dim * H + 3 * H * F)
    flops = 2.0 * linear * T + 2.0 * H * cfg["vocab_size"] + L * cfg["num_attention_heads"] * 2.0 * D * T * T
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            pk = json.load(fh)
        peak_tf, kind = float(pk["bf16_tflops_sustained"]), "measured sustained"
    except Exception:
        peak_tf, kind = 1400.0, "fallback sustained"
    del st
    return {"workload": "config 3 prefill: 2048 uniform ids, batch 1, bf16 cache", "seconds": t,
            "tok_s": T / t, "tflops": flops / t / 1e12, "flops": flops, "peak_tflops": peak_tf, "peak_kind": kind,
            "frac_of_peak": flops / t / 1e12 / peak_tf,
            "timing": "CUDA events around Model::forward (host orchestration included), best of 3"}


def run_trait_path(tb, dev, path, cfg, torch):
    """The literal drop-in: Model::forward_batch issued one Device-trait call
    at a time (titania_b200.OpModel, about 594 calls per token), greedy
    decode of config 0 after the 16-token prompt, host wall clock."""
    from titania_b200 import synth
    om = tb.OpModel.load(path, dev)
    prompt = synth.prompt_tokens(PROMPT, cfg["vocab_size"], seed=1)
    st = om.state(PROMPT + GEN + 1)
    logits = om.forward(st, prompt, 0)
    tok, pos = int(np.argmax(logits)), PROMPT
    n = 0
    for _ in range(2):  # warm-up
        logits = om.forward(st, [tok], pos)
        tok, pos = int(np.argmax(logits)), pos + 1
    t0 = time.perf_counter()
    while n < 12:
        logits = om.forward(st, [tok], pos)
        tok, pos, n = int(np.argmax(logits)), pos + 1, n + 1
    secs = time.perf_counter() - t0
    del om, st
    return {"value": n / secs, "unit": "tok/s", "steps": n,
            "path": "OpModel: one C-ABI Device call per op (model/model.rs:93-149), logits read every step"}


BS64_SEQS, BS64_CTX, BS64_GEN = 64, 1024, 128  # config 3's batched decode


def run_bs64(args, tb, m, dev, cfg, torch, world):
    """Config 3's batched decode: 64 sequences, each prefilled with 1024
    uniform token ids through the tensor-core prompt path, then 128 greedy
    steps of all 64 at once (contexts 1024..1151), replayed; bf16 K/V cache
    (the north star's; the bs1 line keeps the reference's f32)."""
    from titania_b200 import synth
    V = cfg["vocab_size"]
    max_len = BS64_CTX + BS64_GEN
    bs = m.batch_state(BS64_SEQS, max_len, kv="bf16")
    t0 = time.perf_counter()
    first = [m.forward_seq(bs, i, synth.prompt_tokens(BS64_CTX, V, seed=1000 + i), 0, logits=False)
             for i in range(BS64_SEQS)]
    prefill_s = time.perf_counter() - t0
    pos = [BS64_CTX] * BS64_SEQS
    stream = torch.cuda.ExternalStream(dev.stream)
    gens = max(1, args.bs64_gens)
    m.decode_batch_enqueue(bs, first, pos, BS64_GEN)  # warm-up generation
    dev.sync()
    if world > 1:
        torch.distributed.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(dev.ordinal) as clk:
        e0.record(stream)
        for _ in range(gens):
            m.decode_batch_enqueue(bs, first, pos, BS64_GEN)
        e1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
    secs = e0.elapsed_time(e1) * 1e-3
    steps = gens * BS64_GEN

    # e2e: one public call per step, host tokens and positions in, greedy
    # tokens out (no logits: 64 x 608 KB per step is the sampler's business)
    def e2e(k):
        toks, p = list(first), list(pos)
        for i in range(k):
            if i % BS64_GEN == 0:
                toks, p = list(first), list(pos)
            _, nxt = m.forward_batch(bs, toks, p, logits=False)
            toks, p = nxt, [x + 1 for x in p]
    e2e(4)
    dev.sync()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    e2e(steps)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_secs = f0.elapsed_time(f1) * 1e-3
    if world > 1:
        t = torch.tensor([secs, e2e_secs], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        secs, e2e_secs = t.tolist()

    # One traced step (every kernel records its CTAs' events): per kernel, the
    # segment from the previous kernel's last CTA to its own (they add up to
    # the step) and the CTAs' median own work.
    try:
        bs.trace_start(1 << 22)
        m.decode_batch_enqueue(bs, first, pos, 1)
        step_timeline = timeline(bs.trace_stop(), BATCH_NAMES)
    except Exception as e:  # secondary: report it, keep the measurement
        step_timeline = {"error": f"{type(e).__name__}: {e}"[:300]}

    weights, kv_per_pos = model_bytes(cfg, kv_bytes=2)
    mean_ctx = BS64_CTX + (BS64_GEN + 1) / 2
    step_bytes = weights + BS64_SEQS * kv_per_pos * mean_ctx
    peak, peak_kind = peaks()
    L = cfg["num_hidden_layers"]
    return {
        "value": world * steps * BS64_SEQS / secs, "unit": "tok/s", "steps": steps,
        "ms_per_step": secs / steps * 1e3,
        "config": {"workload": "qwen3-0.6b bs64 greedy decode (config 3: 64 sequences x 1024-token prompt, "
                               "128 steps, replayed)", "batch": BS64_SEQS, "ctx": [BS64_CTX, max_len - 1],
                   "kv_cache": "bf16", "prefill_seconds": prefill_s,
                   "l2": "no flush needed: each step reads ~9 GB (weights + K/V), > 126 MB L2"},
        "hbm": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes * steps / secs / 1e9,
                "frac_of_8tbs": step_bytes * steps / secs / 1e9 / NOMINAL_HBM_GBS,
                "frac_of_measured": step_bytes * steps / secs / 1e9 / peak, "peak_gbs": peak,
                "peak_kind": peak_kind},
        "e2e": {"value": world * steps * BS64_SEQS / e2e_secs, "unit": "tok/s",
                "h2d_bytes_per_step": BS64_SEQS * (4 + 8) + 3 * 4, "d2h_bytes_per_step": BS64_SEQS * 4 + 4},
        "gpu_launches": steps * (1 + 8 * L + 3),
        "clocks": clk.summary(),
        "step_timeline": step_timeline,
    }


def cached_model_all_ranks(name, rank, world, torch):
    """The seeded checkpoint, written once (rank 0) while the others wait."""
    from titania_b200 import synth
    if rank == 0:
        path = synth.cached_model(name, seed=0)
    if world > 1:
        torch.distributed.barrier()
    return synth.cached_model(name, seed=0) if rank != 0 else path


TP_CTX, TP_GEN, TP_BATCH = 2048, 32, 256  # config 4


def run_tp(args, rank, world, torch):
    """Config 4: Qwen3-4B-shaped random-init weights, tensor-parallel over the
    `world` GPUs of this node (one rank per GPU; world 1 is the single-GPU
    baseline). bs1: a 2048-token prompt, then TP_GEN greedy steps (contexts
    2048..2079), replayed, on the state's default single-token path (the
    persistent kernel: o_proj and down_proj partials to every rank by peer
    stores over NVLink); bs256: 256 sequences, each prefilled with 2048 ids,
    then TP_GEN steps of all at once (bf16 K/V; NCCL all-reduces captured in
    the decode graphs). Device time, max over ranks."""
    import titania_b200 as tb
    from titania_b200 import synth
    from titania_b200.tp import TPGroup, load_tp_model
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = tb.B200(local)
    path = cached_model_all_ranks("qwen3-4b", rank, world, torch)
    cfg = dict(synth.QWEN3_4B)
    uid = [TPGroup.unique_id() if rank == 0 else None]
    if world > 1:
        torch.distributed.broadcast_object_list(uid, src=0)
    group = TPGroup(dev, rank, world, uid[0])
    m = load_tp_model(path, dev, group)
    stream = torch.cuda.ExternalStream(dev.stream)
    V = cfg["vocab_size"]

    def timed(fn, warm):
        fn(warm)
        dev.sync()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        steps = fn(None)
        e1.record(stream)
        dev.sync()
        torch.cuda.synchronize()
        secs = e0.elapsed_time(e1) * 1e-3
        if world > 1:
            t = torch.tensor([secs], dtype=torch.float64, device="cuda")
            torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
            secs = t.item()
        return steps, secs

    weights, kv_per_pos = model_bytes(cfg, kv_bytes=2)
    weights32, kv_per_pos32 = model_bytes(cfg, kv_bytes=4)
    out = {"model": "Qwen3-4B architecture (random-init bf16)", "tp": world, "ctx": [TP_CTX, TP_CTX + TP_GEN - 1]}

    # bs1 (f32 cache, as the reference)
    st = m.state(TP_CTX + TP_GEN + 1)
    first = m.forward(st, synth.prompt_tokens(TP_CTX, V, seed=7), 0, logits=False)

    def bs1(warm):
        n = 1 if warm else max(1, args.tp_gens)
        for _ in range(n):
            m.decode_enqueue(st, first, TP_CTX, TP_GEN)
        return n * TP_GEN
    steps, secs = timed(bs1, True)
    step_bytes = weights32 + kv_per_pos32 * (TP_CTX + TP_GEN / 2)
    out["bs1"] = {"tok_s": steps / secs, "ms_per_step": secs / steps * 1e3, "kv_cache": "f32", "decode": st.decode,
                  "hbm_frac_of_8tbs_x_n": step_bytes * steps / secs / (NOMINAL_HBM_GBS * 1e9 * world)}
    if st.decode == "persistent":  # where a step goes (every rank traces alike; rank 0's is reported)
        out["bs1"]["step_timeline"] = step_trace(m, st, first, "persistent", prompt=TP_CTX)
    del st

    # bs256 (bf16 cache)
    if args.tp_batch > 0:
        B = args.tp_batch
        bs = m.batch_state(B, TP_CTX + TP_GEN, kv="bf16")
        t0 = time.perf_counter()
        bfirst = [m.forward_seq(bs, i, synth.prompt_tokens(TP_CTX, V, seed=2000 + i), 0, logits=False)
                  for i in range(B)]
        prefill_s = time.perf_counter() - t0
        pos = [TP_CTX] * B

        def bsn(warm):
            n = 1 if warm else max(1, args.tp_gens)
            for _ in range(n):
                m.decode_batch_enqueue(bs, bfirst, pos, TP_GEN)
            return n * TP_GEN
        steps, secs = timed(bsn, True)
        step_bytes = weights + B * kv_per_pos * (TP_CTX + TP_GEN / 2)
        out[f"bs{B}"] = {"tok_s": steps * B / secs, "ms_per_step": secs / steps * 1e3, "kv_cache": "bf16",
                         "prefill_seconds": prefill_s,
                         "hbm_frac_of_8tbs_x_n": step_bytes * steps / secs / (NOMINAL_HBM_GBS * 1e9 * world)}
        del bs
    del m
    group.close()
    return out


def measure_load(dev, path, reps=2):
    """Checkpoint load throughput, file already in the page cache: the
    library's direct safetensors path (tb200_upload_safetensors, what
    Model.load uses) against per-tensor Weights.read + upload (the
    reference's Model::load shape, model/model.rs:251-254). Host wall clock
    from the call to every byte on the device; best of `reps` after a first
    call (reported as `first_seconds`: for the direct path it also page-locks
    the device's staging buffers, which later loads reuse)."""
    from titania_b200.model import Config, Weights, load_weights, tensor_names, upload_checkpoint
    c = Config.load(os.path.join(path, "config.json"))
    f = os.path.join(path, "model.safetensors")
    w = Weights.open(f)
    nbytes = sum(w.entries[n]["data_offsets"][1] - w.entries[n]["data_offsets"][0]
                 for n, _ in tensor_names(c) if w.contains(n))
    out = {"bytes": nbytes, "page_cache": "warm"}
    for kind, fn in (("direct", lambda: upload_checkpoint(dev, c, f)),
                     ("per_tensor", lambda: load_weights(dev, c, Weights.open(f)))):
        times = []
        for i in range(reps + 1):
            t0 = time.perf_counter()
            ws = fn()
            dev.sync()
            times.append(time.perf_counter() - t0)
            del ws
        best = min(times[1:])
        out[kind] = {"seconds": best, "gbs": nbytes / best / 1e9, "first_seconds": times[0]}
    return out


def run_ours(args, rank, world, torch):
    import titania_b200 as tb
    from titania_b200 import synth

    dev = tb.B200(int(os.environ.get("LOCAL_RANK", rank)) if world > 1 else 0)
    torch.cuda.set_device(dev.ordinal)
    cfg = dict(synth.QWEN3_0_6B)
    path = cached_model_all_ranks("qwen3-0.6b", rank, world, torch)
    m = tb.Model.load(path, dev)
    load = measure_load(dev, path) if world == 1 else None
    prompt = synth.prompt_tokens(PROMPT, cfg["vocab_size"], seed=1)
    st = m.state(PROMPT + GEN + 1)  # the default single-token path: the persistent kernel where the model allows it
    decode = st.decode
    first = m.forward(st, prompt, 0, logits=False)  # prefill: K/V for positions 0..15

    K, W = args.steps, args.warmup
    gens = lambda k: [(GEN if i + GEN <= k else k - i) for i in range(0, k, GEN)]
    stream = torch.cuda.ExternalStream(dev.stream)
    weights, kv_per_pos = model_bytes(cfg)
    ctx_of = lambda i: PROMPT + 1 + (i % GEN)  # context of step i of a generation

    def device_rate(state, k):
        """K greedy steps (config 0's generation replayed) on `state`'s path,
        device time; also each launch's own events (one launch is one
        generation on the persistent path)."""
        for g in gens(W):
            m.decode_enqueue(state, first, PROMPT, g)
        dev.sync()
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        per = []
        with Clocks(dev.ordinal) as clk:
            e0.record(stream)
            for g in gens(k):
                a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                a.record(stream)
                m.decode_enqueue(state, first, PROMPT, g)
                b.record(stream)
                per.append((a, b, g))
            e1.record(stream)
            dev.sync()
            torch.cuda.synchronize()
        launches = [(a.elapsed_time(b) * 1e-3, g) for a, b, g in per]
        return e0.elapsed_time(e1) * 1e-3, launches, clk.summary()

    secs, launches, clocks = device_rate(st, K)
    if world > 1:
        torch.distributed.barrier()

    # e2e: the public forward call with host buffers (pinned), one token per call
    logits = torch.empty(cfg["vocab_size"], dtype=torch.float32, pin_memory=True).numpy()
    def e2e_steps(k):
        tok, pos, done = first, PROMPT, 0
        while done < k:
            m.forward(st, [tok], pos, out=logits)
            tok, pos, done = m.last_token, pos + 1, done + 1
            if pos == PROMPT + GEN:
                tok, pos = first, PROMPT
    e2e_steps(W)
    dev.sync()
    if world > 1:
        torch.distributed.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record(stream)
    e2e_steps(K)
    f1.record(stream)
    torch.cuda.synchronize()
    e2e_secs = f0.elapsed_time(f1) * 1e-3

    if world > 1:
        t = torch.tensor([secs, e2e_secs], dtype=torch.float64, device="cuda")
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        secs, e2e_secs = t.tolist()

    step_bytes = weights + kv_per_pos * (sum(ctx_of(i) for i in range(K)) / K)
    peak, peak_kind = peaks()
    persistent = decode == "persistent"
    result = {
        "metric": METRIC,
        "value": world * K / secs,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": secs / K * 1e3,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded random-init Qwen3-0.6B bf16 weights (N(0,0.02), norms 1.0), "
                "16 uniform prompt ids",
        "config": {"workload": "qwen3-0.6b bs1 greedy decode (config 0: 16-token prompt + 32 steps, replayed)",
                   "model": "Qwen3-0.6B architecture", "batch": 1, "ctx": [PROMPT + 1, PROMPT + GEN],
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "weights": "bf16", "activations": "f32", "kv_cache": "f32 (the reference's; bf16 optional)",
                   "l2": "no flush needed: each step streams 1.19 GB of weights, > 126 MB L2",
                   "decode": decode,
                   "launch": ("one persistent cooperative kernel (one CTA per SM) per 32-step generation"
                              if persistent else "one CUDA graph per step, programmatic dependent launch")},
        "hbm": {"bytes_per_step": step_bytes, "achieved_gbs": step_bytes * K / secs / 1e9,
                "frac_of_8tbs": step_bytes * K / secs / 1e9 / NOMINAL_HBM_GBS,
                "frac_of_measured": step_bytes * K / secs / 1e9 / peak, "peak_gbs": peak, "peak_kind": peak_kind},
        "e2e": {"value": world * K / e2e_secs, "unit": "tok/s", "h2d_bytes_per_step": 8,
                "d2h_bytes_per_step": cfg["vocab_size"] * 4 + 16},
        "gpu_launches": (2 * len(gens(K)) if persistent
                         else K * (2 + 5 * cfg["num_hidden_layers"]) + len(gens(K))),
        "clocks": clocks,
    }
    if rank == 0 and world == 1:
        # The dominant kernel of the step: on the persistent path the step
        # kernel itself (each launch runs a whole generation), timed by its own
        # events inside the timed region; bytes = every step's weights + K/V.
        lt = sum(t for t, _ in launches)
        lbytes, i = 0.0, 0
        for _, g in launches:
            lbytes += sum(weights + kv_per_pos * ctx_of(j) for j in range(g))
        traffic = None
        try:
            with open(os.path.join(ROOT, "profiles", "traffic.json")) as fh:
                tj = json.load(fh)
            if persistent and tj.get("persistent step"):
                # captured on a one-step launch; a timed launch runs its generation's steps
                traffic = tj["persistent step"] * sum(g for _, g in launches) / len(launches)
        except Exception:
            pass
        result["roofline"] = {
            "bound": "hbm", "kernel": ("tb::persist::step_kernel (the whole decode step)" if persistent
                                       else "the fused step's kernels (one graph)"),
            "achieved": lbytes / lt / 1e9, "peak": peak, "unit": "GB/s", "frac": lbytes / lt / 1e9 / peak,
            "peak_kind": peak_kind, "traffic": traffic,
            "algorithmic_bytes_per_launch": lbytes / len(launches), "avg_launch_us": lt / len(launches) * 1e6,
            "launches": len(launches), "steps_per_launch": sum(g for _, g in launches) / len(launches),
            "traffic_note": "ncu dram read+write of a one-step launch (profiles/traffic.json), times the steps "
                            "per timed launch"}
        # Where a step goes: the traced step cut into consecutive segments
        # (they add up to the step), on both single-token paths.
        try:
            result["step_timeline"] = step_trace(m, st, first, decode)
            if persistent:
                fst = m.state(PROMPT + GEN + 1, decode="fused")
                fsecs, _, _ = device_rate(fst, min(K, 256))
                result["fused"] = {"value": min(K, 256) / fsecs, "unit": "tok/s",
                                   "ms_per_step": fsecs / min(K, 256) * 1e3,
                                   "step_timeline": step_trace(m, fst, first, "fused")}
                del fst
        except Exception as e:
            result["step_timeline"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if not args.no_bs64:
        result["bs64"] = run_bs64(args, tb, m, dev, cfg, torch, world)
    if rank == 0 and world == 1 and not args.no_sweeps:
        for key, fn in (("attn_sweep", lambda: run_attn_sweep(tb, dev, torch, peak)),
                        ("op_sweep", lambda: run_op_sweep(tb, dev, torch)),
                        ("prefill", lambda: run_prefill(tb, m, dev, cfg, torch)),
                        ("trait_path", lambda: run_trait_path(tb, dev, path, cfg, torch))):
            try:
                result[key] = fn()
            except Exception as e:  # secondary sections: report, keep the headline line
                result[key] = {"error": f"{type(e).__name__}: {e}"[:300]}
    if load is not None:
        result["load"] = load
    if rank == 0 and world == 1 and not args.no_cpu:
        result["cpu_baseline"] = cpu_baseline(path, prompt, budget_s=args.cpu_seconds)
    if args.tp4b or (world > 1 and not args.no_tp):
        del st, m
        try:
            result["tp4b"] = run_tp(args, rank, world, torch)
        except Exception as e:  # config 4 is a secondary section: report it, keep the headline line
            result["tp4b"] = {"error": f"{type(e).__name__}: {e}"[:300]}
    return result


def cpu_oracle(path):
    from oracle import oracle as orc
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    orc.set_threads(threads)
    return orc, orc.Model(path), threads


def cpu_decode_rate(orc, ref, prompt, budget_s, min_steps=3, max_steps=None):
    """Times the oracle (CPU restatement of the reference path) decoding
    greedily after the prompt, for about budget_s seconds."""
    st = ref.state(PROMPT + GEN + 1)
    logits = ref.forward(st, prompt, 0)
    first = orc.sample_greedy(logits)
    n, t0, tok, pos = 0, time.perf_counter(), first, PROMPT
    while True:
        logits = ref.forward(st, [tok], pos)
        tok, pos, n = orc.sample_greedy(logits), pos + 1, n + 1
        if pos == PROMPT + GEN:
            tok, pos = first, PROMPT
        el = time.perf_counter() - t0
        if (n >= min_steps and el >= budget_s) or (max_steps and n >= max_steps):
            break
    return n / el, n


def cpu_baseline(path, prompt, budget_s):
    orc, ref, threads = cpu_oracle(path)
    rate, n = cpu_decode_rate(orc, ref, prompt, budget_s)
    return {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"{n} greedy decode steps of config 0 (ctx 17..48) after the 16-token prompt, "
                      f"oracle/oracle.cpp (C++ restatement of model/cpu.rs + model/model.rs), "
                      f"OpenMP over matvec rows and attention heads as the reference uses rayon"}


def run_reference(args):
    from titania_b200 import synth
    path = synth.cached_model("qwen3-0.6b", seed=0)
    prompt = synth.prompt_tokens(PROMPT, synth.QWEN3_0_6B["vocab_size"], seed=1)
    orc, ref, threads = cpu_oracle(path)
    w = max(1, min(args.warmup, 3))  # untimed warm-up steps
    cpu_decode_rate(orc, ref, prompt, 0.0, min_steps=w, max_steps=w)
    # then K steps, bounded to ~2 minutes of CPU work
    rate, n = cpu_decode_rate(orc, ref, prompt, 120.0, min_steps=min(args.steps, 3), max_steps=args.steps)
    return {
        "impl": "reference",
        "metric": METRIC, "value": rate, "unit": "tok/s", "n_gpus": 0, "steps": n, "warmup": args.warmup,
        "ms_per_step": 1e3 / rate, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "f32 activations, bf16 weights, f32 KV",
        "data": "synthetic: seeded random-init Qwen3-0.6B bf16 weights, 16 uniform prompt ids",
        "config": {"workload": "qwen3-0.6b bs1 greedy decode (config 0: 16-token prompt + 32 steps, replayed)",
                   "model": "Qwen3-0.6B architecture", "batch": 1, "ctx": [PROMPT + 1, PROMPT + GEN]},
        "cpu_baseline": {"value": rate, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": f"{n} greedy decode steps (at most {args.steps}, bounded to ~120 s), "
                                   "oracle/oracle.cpp restating model/cpu.rs + model/model.rs; the Rust "
                                   "reference needs cargo and crates.io, absent offline"},
        "e2e": {"value": rate, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def profile_op(args):
    """A small case for ncu: loads the model and launches one fused kernel
    `--launches` times (layers cycling), nothing else on the GPU besides set-up."""
    import titania_b200 as tb
    from titania_b200 import synth
    from titania_b200.model import OP_ATTENTION, OP_DOWN, OP_GATE_UP, OP_LM_HEAD, OP_O, OP_QKV
    ops = {"qkv": OP_QKV, "attention": OP_ATTENTION, "o": OP_O, "gate_up": OP_GATE_UP, "down": OP_DOWN,
           "lm_head": OP_LM_HEAD}
    dev = tb.B200(0)
    m = tb.Model.load(synth.cached_model("qwen3-0.6b", seed=0), dev)
    st = m.state(PROMPT + GEN + 1)
    for i in range(args.launches):
        st.set_position(1, PROMPT + (i % GEN))
        m.enqueue_op(st, ops[args.profile_op], i % 28)
    dev.sync()
    print(json.dumps({"profile_op": args.profile_op, "launches": args.launches}))


def profile_persistent(args):
    """For ncu: the persistent single-token step on Qwen3-0.6B (f32 cache):
    the 16-token prompt, then `--launches` one-step launches at context 17
    (capture the last with `-k regex:step_kernel -s <launches - 1> -c 1`)."""
    import titania_b200 as tb
    from titania_b200 import synth
    dev = tb.B200(0)
    m = tb.Model.load(synth.cached_model("qwen3-0.6b", seed=0), dev)
    st = m.state(PROMPT + GEN + 1)
    first = m.forward(st, synth.prompt_tokens(PROMPT, synth.QWEN3_0_6B["vocab_size"], seed=1), 0, logits=False)
    for _ in range(args.launches):
        m.decode_enqueue(st, first, PROMPT, 1)
    dev.sync()
    print(json.dumps({"profile_persistent": st.decode, "launches": args.launches}))


def profile_prefill(args):
    """For ncu: config 3's 2048-token prompt at batch 1 (bf16 cache),
    `--launches` times."""
    import titania_b200 as tb
    from titania_b200 import synth
    dev = tb.B200(0)
    m = tb.Model.load(synth.cached_model("qwen3-0.6b", seed=0), dev)
    st = m.state(2049, kv="bf16")
    prompt = synth.prompt_tokens(2048, synth.QWEN3_0_6B["vocab_size"], seed=3)
    for _ in range(args.launches):
        m.forward(st, prompt, 0, logits=False)
    dev.sync()
    print(json.dumps({"profile_prefill": 2048, "launches": args.launches}))


def profile_bs64(args):
    """For ncu: config 3's prefill (`--profile-seqs` sequences x
    `--profile-ctx` tokens, one pass of 228 kernels each at the defaults), then
    `--launches` batched decode steps (228 kernels each). Smaller sequence
    counts and contexts keep full captures to a few GB on the device."""
    import titania_b200 as tb
    from titania_b200 import synth
    dev = tb.B200(0)
    m = tb.Model.load(synth.cached_model("qwen3-0.6b", seed=0), dev)
    V = synth.QWEN3_0_6B["vocab_size"]
    n, ctx = args.profile_seqs, args.profile_ctx
    bs = m.batch_state(n, ctx + BS64_GEN, kv="bf16")
    first = [m.forward_seq(bs, i, synth.prompt_tokens(ctx, V, seed=1000 + i), 0, logits=False) for i in range(n)]
    m.decode_batch_enqueue(bs, first, [ctx] * n, 1)  # builds the step graph
    dev.sync()
    # Only the decode steps are profiled (ncu --profile-from-start off).
    _profiler(True)
    m.decode_batch_enqueue(bs, first, [ctx] * n, args.launches)
    dev.sync()
    _profiler(False)
    print(json.dumps({"profile_bs64": True, "seqs": n, "ctx": ctx, "steps": args.launches}))


def _profiler(on):
    """cudaProfilerStart / Stop (context-wide) through PyTorch's CUDA runtime."""
    import torch
    rt = torch.cuda.cudart()
    (rt.cudaProfilerStart if on else rt.cudaProfilerStop)()


GEMM_SHAPES = [(151936, 1024, 64), (6144, 1024, 64), (4096, 1024, 64), (1024, 2048, 64), (1024, 3072, 64),
               (151936, 1024, 1), (6144, 1024, 512)]


def profile_gemm(args):
    """For ncu: the tensor-core contraction (through the trait matmul over
    several tokens) at the batched decode's shapes, `--launches` times each."""
    import titania_b200 as tb
    from titania_b200 import synth
    dev = tb.B200(0)
    rng = np.random.default_rng(0)
    for rows, cols, n in GEMM_SHAPES:
        w = dev.upload(tb.Tensor([rows, cols], synth.f32_to_bf16_bits(
            rng.normal(0, 0.02, size=(rows, cols)).astype(np.float32)).reshape(rows, cols)))
        x = dev.alloc(n * cols)
        dev.write(x, rng.standard_normal(n * cols, dtype=np.float32))
        out = dev.alloc(n * rows)
        dev.matmul(out, w, x)  # first use: plans, tensor maps
        dev.sync()
        _profiler(True)
        for _ in range(args.launches):
            dev.matmul(out, w, x)
        dev.sync()
        _profiler(False)
    dev.sync()
    print(json.dumps({"profile_gemm": GEMM_SHAPES, "launches": args.launches}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=4096)
    ap.add_argument("--warmup", type=int, default=64)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-sweeps", action="store_true",
                    help="skip the config 1/2/3 sections (op sweep, attention sweep, prefill) and the trait path")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--cpu-seconds", type=float, default=15.0)
    ap.add_argument("--no-bs64", action="store_true", help="skip the batch-64 decode (config 3)")
    ap.add_argument("--bs64-gens", type=int, default=2, help="timed 128-step generations of the bs64 decode")
    ap.add_argument("--tp4b", action="store_true",
                    help="also run config 4 (Qwen3-4B, tensor-parallel over the ranks; default when N > 1)")
    ap.add_argument("--no-tp", action="store_true", help="skip config 4 when N > 1")
    ap.add_argument("--tp-gens", type=int, default=2, help="timed 32-step generations of config 4")
    ap.add_argument("--tp-batch", type=int, default=TP_BATCH, help="config 4's large batch (0: skip it)")
    ap.add_argument("--profile-op", choices=["qkv", "attention", "o", "gate_up", "down", "lm_head"],
                    help="small case for ncu: launch one fused kernel only")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--profile-bs64", action="store_true",
                    help="small case for ncu: the bs64 prefill, then --launches batched decode steps")
    ap.add_argument("--profile-seqs", type=int, default=BS64_SEQS)
    ap.add_argument("--profile-ctx", type=int, default=BS64_CTX)
    ap.add_argument("--profile-persistent", action="store_true",
                    help="small case for ncu: --launches one-step launches of the persistent decode kernel")
    ap.add_argument("--profile-prefill", action="store_true",
                    help="small case for ncu: --launches passes of config 3's 2048-token prompt")
    ap.add_argument("--profile-gemm", action="store_true",
                    help="small case for ncu: the tensor-core contraction at the batched shapes")
    args = ap.parse_args()
    if args.profile_gemm:
        profile_gemm(args)
        return
    if args.profile_persistent:
        profile_persistent(args)
        return
    if args.profile_prefill:
        profile_prefill(args)
        return
    if args.profile_op:
        profile_op(args)
        return
    if args.profile_bs64:
        profile_bs64(args)
        return
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)), flush=True)
        return

    import torch
    if world > 1:
        import datetime
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        res = run_ours(args, rank, world, torch)
        if rank == 0:
            print(json.dumps(res), flush=True)
    finally:
        if world > 1:
            torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
