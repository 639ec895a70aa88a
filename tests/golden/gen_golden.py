"""Generates the golden fixtures in this directory from an independent numpy
restatement of the Titania reference CPU path.

The reference (penberg/titania, Rust) ships no golden vectors and cannot be
built here, so these fixtures are produced by a second restatement of its
arithmetic, written separately from the C++ oracle (oracle/oracle.cpp):
vectorised numpy with explicit sequential loops wherever the reference's
summation order matters, and glibc's expf/powf/sinf/cosf called through
ctypes (numpy's own exp differs from glibc in the last bit). The CPU test
suite then checks the C++ oracle against these fixtures bit for bit.

Cases follow the reference's op tests (model/titania.rs:268-370): the same
xorshift32 input generator (:231-241), bf16 truncation for weights
(:243-249), shapes and positions. A seeded two-layer model with Qwen3's head
geometry adds an end-to-end forward/greedy fixture.

Run from the repository root:  python tests/golden/gen_golden.py
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from titania_b200 import synth  # noqa: E402

F = np.float32
_libm = ctypes.CDLL("libm.so.6")
for _name in ("expf", "sinf", "cosf"):
    getattr(_libm, _name).restype = ctypes.c_float
    getattr(_libm, _name).argtypes = [ctypes.c_float]
_libm.powf.restype = ctypes.c_float
_libm.powf.argtypes = [ctypes.c_float, ctypes.c_float]


def _vec(fn, a):
    a = np.asarray(a, dtype=F)
    return np.array([fn(float(v)) for v in a.ravel()], dtype=F).reshape(a.shape)


def expf(a):
    return _vec(_libm.expf, a)


# --- the reference's test input generator (model/titania.rs:231-249) --------

def numbers(n: int, seed: int) -> np.ndarray:
    state = (seed * 2654435761) & 0xFFFFFFFF
    state = max(state, 1)
    out = np.empty(n, dtype=F)
    for i in range(n):
        state ^= (state << 13) & 0xFFFFFFFF
        state ^= state >> 17
        state ^= (state << 5) & 0xFFFFFFFF
        out[i] = F(state >> 8) / F(1 << 23) - F(1.0)
    return out


def tensor(shape, seed):
    x = numbers(int(np.prod(shape)), seed)
    return (x.view(np.uint32) >> 16).astype(np.uint16).reshape(shape)


def bf16(bits):
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(F)


# --- numpy restatement of model/cpu.rs ---------------------------------------

def dot_rows(w, x):
    """cpu.rs:167-177 for every row of w at once: eight running sums in
    order, summed in order, plus the ragged tail."""
    wf = bf16(w)
    rows, cols = wf.shape
    done = cols // 8 * 8
    acc = np.zeros((rows, 8), dtype=F)
    for c in range(0, done, 8):
        acc += wf[:, c:c + 8] * x[c:c + 8]
    rest = np.full(rows, -0.0, dtype=F)
    for c in range(done, cols):
        rest = rest + wf[:, c] * x[c]
    s = np.full(rows, -0.0, dtype=F)
    for i in range(8):
        s = s + acc[:, i]
    return s + rest


def np_matmul(w, x):
    rows, cols = w.shape
    n = x.size // cols
    out = np.empty(n * rows, dtype=F)
    for t in range(n):
        out[t * rows:(t + 1) * rows] = dot_rows(w, x[t * cols:(t + 1) * cols])
    return out


def np_rmsnorm(x, w, eps):
    dim = w.size
    rows = x.reshape(-1, dim).copy()
    ss = np.full(rows.shape[0], -0.0, dtype=F)
    for i in range(dim):
        ss = ss + rows[:, i] * rows[:, i]
    ms = ss / F(dim)
    scale = F(1.0) / np.sqrt(ms + F(eps))
    rows *= scale[:, None] * bf16(w)[None, :]
    return rows.reshape(-1)


def np_rope(x, table, pos, n_heads, head_dim):
    half = head_dim // 2
    x = x.reshape(-1, n_heads, head_dim).copy()
    for t in range(x.shape[0]):
        ang = table[(pos + t) * head_dim:(pos + t + 1) * head_dim].reshape(half, 2)
        c, s = ang[:, 0], ang[:, 1]
        a, b = x[t, :, :half].copy(), x[t, :, half:].copy()
        x[t, :, :half] = a * c - b * s
        x[t, :, half:] = b * c + a * s
    return x.reshape(-1)


def np_softmax(v):
    mx = F(-np.inf)
    for s in v:
        mx = max(mx, s)
    e = expf(v - mx)
    total = F(0.0)
    for s in e:
        total = F(total + s)
    return e / total


def np_attention(q, k_cache, v_cache, pos, n_heads, head_dim, n_kv_heads):
    group = n_heads // n_kv_heads
    kv_dim = n_kv_heads * head_dim
    scale = F(1.0) / np.sqrt(F(head_dim))
    items = q.size // head_dim
    out = np.empty_like(q)
    K = k_cache.reshape(-1, kv_dim)
    V = v_cache.reshape(-1, kv_dim)
    for i in range(items):
        token, head = divmod(i, n_heads)
        length = pos + token + 1
        kv = head // group * head_dim
        qh = q[i * head_dim:(i + 1) * head_dim]
        s = np.full(length, -0.0, dtype=F)
        for d in range(head_dim):
            s = s + qh[d] * K[:length, kv + d]
        p = np_softmax(scale * s)
        o = np.zeros(head_dim, dtype=F)
        for t in range(length):
            o = o + p[t] * V[t, kv:kv + head_dim]
        out[i * head_dim:(i + 1) * head_dim] = o
    return out


def np_silu_mul(g, u):
    return g / (F(1.0) + expf(-g)) * u


def np_rope_table(max_len, head_dim, theta):
    half = head_dim // 2
    freq = np.array([F(1.0) / F(_libm.powf(float(theta), float(F(2 * i) / F(head_dim)))) for i in range(half)],
                    dtype=F)
    out = np.empty((max_len, half, 2), dtype=F)
    for pos in range(max_len):
        a = F(pos) * freq
        out[pos, :, 0] = _vec(_libm.cosf, a)
        out[pos, :, 1] = _vec(_libm.sinf, a)
    return out.reshape(-1)


def total_key(v):
    b = np.asarray(v, dtype=F).view(np.int32).astype(np.int64)
    return np.where(b < 0, b ^ 0x7FFFFFFF, b)


def np_greedy(logits):
    k = total_key(logits)
    return int(np.flatnonzero(k == k.max())[0])


# --- numpy restatement of model/model.rs forward ----------------------------

class NpModel:
    def __init__(self, path):
        with open(os.path.join(path, "config.json")) as fh:
            c = json.load(fh)
        self.c = c
        self.hd = c.get("head_dim") or c["hidden_size"] // c["num_attention_heads"]
        with open(os.path.join(path, "model.safetensors"), "rb") as fh:
            blob = fh.read()
        n = int.from_bytes(blob[:8], "little")
        header = json.loads(blob[8:8 + n])
        self.t = {}
        for name, e in header.items():
            if name == "__metadata__":
                continue
            a, b = e["data_offsets"]
            self.t[name] = np.frombuffer(blob[8 + n + a:8 + n + b], dtype="<u2").reshape(e["shape"])

    def forward(self, kv, tokens, pos, max_len):
        c, hd = self.c, self.hd
        H, eps = c["hidden_size"], F(c["rms_norm_eps"])
        nh, nkv = c["num_attention_heads"], c["num_key_value_heads"]
        kv_dim = nkv * hd
        table = np_rope_table(max_len, hd, F(c["rope_theta"]))
        logits = None
        for b0 in range(0, len(tokens), 64):
            batch = tokens[b0:b0 + 64]
            p0 = pos + b0
            n = len(batch)
            x = bf16(self.t["model.embed_tokens.weight"][batch]).reshape(-1).copy()
            for i in range(c["num_hidden_layers"]):
                p = f"model.layers.{i}"
                xb = np_rmsnorm(x, self.t[f"{p}.input_layernorm.weight"], eps)
                q = np_matmul(self.t[f"{p}.self_attn.q_proj.weight"], xb)
                k = np_matmul(self.t[f"{p}.self_attn.k_proj.weight"], xb)
                v = np_matmul(self.t[f"{p}.self_attn.v_proj.weight"], xb)
                q = np_rmsnorm(q, self.t[f"{p}.self_attn.q_norm.weight"], eps)
                k = np_rmsnorm(k, self.t[f"{p}.self_attn.k_norm.weight"], eps)
                q = np_rope(q, table, p0, nh, hd)
                k = np_rope(k, table, p0, nkv, hd)
                kv[i][0][p0 * kv_dim:(p0 + n) * kv_dim] = k
                kv[i][1][p0 * kv_dim:(p0 + n) * kv_dim] = v
                att = np_attention(q, kv[i][0], kv[i][1], p0, nh, hd, nkv)
                x = x + np_matmul(self.t[f"{p}.self_attn.o_proj.weight"], att)
                xb = np_rmsnorm(x, self.t[f"{p}.post_attention_layernorm.weight"], eps)
                g = np_matmul(self.t[f"{p}.mlp.gate_proj.weight"], xb)
                u = np_matmul(self.t[f"{p}.mlp.up_proj.weight"], xb)
                x = x + np_matmul(self.t[f"{p}.mlp.down_proj.weight"], np_silu_mul(g, u))
            xl = np_rmsnorm(x[(n - 1) * H:n * H], self.t["model.norm.weight"], eps)
            logits = np_matmul(self.t.get("lm_head.weight", self.t["model.embed_tokens.weight"]), xl)
        return logits


def op_cases():
    """The reference's op tests (model/titania.rs:268-370), with outputs."""
    g = {}
    n = 300
    x, y = numbers(n, 1), numbers(n, 2)
    g["add/x"], g["add/y"] = x, y
    xa = x + y
    g["add/out"] = xa
    g["silu_mul/out"] = np_silu_mul(xa, y)
    dst = numbers(n + 10, 3)
    g["copy/dst_in"] = dst.copy()
    dst[7:7 + n - 5] = g["silu_mul/out"][5:n]
    g["copy/out"] = dst
    table = tensor((10, 128), 4)
    g["embed/table"] = table
    g["embed/tokens"] = np.array([3, 9, 0], dtype=np.uint32)
    g["embed/out"] = bf16(table[[3, 9, 0]]).reshape(-1)
    for rows, cols, nt in [(24, 256, 1), (5, 64, 3), (9, 384, 16), (24, 128, 19)]:
        key = f"matmul/{rows}x{cols}x{nt}"
        w, xm = tensor((rows, cols), 6), numbers(nt * cols, 7)
        g[key + "/w"], g[key + "/x"], g[key + "/out"] = w, xm, np_matmul(w, xm)
    for rows, dim in [(3, 128), (1, 1024), (9, 64)]:
        key = f"rmsnorm/{rows}x{dim}"
        w, xr = tensor((dim,), 9), numbers(rows * dim, 10)
        g[key + "/w"], g[key + "/x"], g[key + "/out"] = w, xr, np_rmsnorm(xr, w, 1e-6)
    for nt in [1, 3]:
        key = f"rope/{nt}"
        xr, tb = numbers(nt * 4 * 128, 11), numbers(40 * 128, 16)
        g[key + "/x"], g[key + "/table"], g[key + "/out"] = xr, tb, np_rope(xr, tb, 37, 4, 128)
    nh, hd, nkv, max_len = 4, 64, 2, 40
    for pos, nt in [(0, 1), (6, 1), (32, 1), (39, 1), (0, 5), (30, 10)]:
        key = f"attention/{pos}_{nt}"
        kvl = max_len * nkv * hd
        q, k, v = numbers(nt * nh * hd, 12), numbers(kvl, 13), numbers(kvl, 14)
        g[key + "/q"], g[key + "/k"], g[key + "/v"] = q, k, v
        g[key + "/out"] = np_attention(q, k, v, pos, nh, hd, nkv)
    g["rope_table/128x40"] = np_rope_table(40, 128, F(1e6))
    g["rope_table/64x8_theta1e4"] = np_rope_table(8, 64, F(10000.0))
    return g


TINY_SEED = 7
TINY_PROMPT = 9
TINY_STEPS = 6


def tiny_model_case(model_dir):
    m = NpModel(model_dir)
    vocab = m.c["vocab_size"]
    prompt = synth.prompt_tokens(TINY_PROMPT, vocab, seed=3)
    max_len = TINY_PROMPT + TINY_STEPS + 1
    kv_dim = m.c["num_key_value_heads"] * m.hd
    kv = [[np.zeros(max_len * kv_dim, F), np.zeros(max_len * kv_dim, F)] for _ in range(m.c["num_hidden_layers"])]
    logits = m.forward(kv, prompt, 0, max_len)
    toks, all_logits, pos = [], [], len(prompt)
    for _ in range(TINY_STEPS):
        t = np_greedy(logits)
        toks.append(t)
        all_logits.append(logits)
        logits = m.forward(kv, [t], pos, max_len)
        pos += 1
    return {
        "prompt": np.array(prompt, dtype=np.uint32),
        "tokens": np.array(toks, dtype=np.uint32),
        "logits": np.stack(all_logits),
        "final_logits": logits,
        "k_cache_l1": kv[1][0][:pos * kv_dim],
        "v_cache_l1": kv[1][1][:pos * kv_dim],
    }


def main():
    g = op_cases()
    np.savez_compressed(os.path.join(HERE, "ops.npz"), **g)
    tiny_dir = os.path.join(ROOT, "_build", "golden-tiny")
    sha = synth.write_model(tiny_dir, synth.TINY, seed=TINY_SEED)
    case = tiny_model_case(tiny_dir)
    np.savez_compressed(os.path.join(HERE, "tiny_model.npz"), **case)
    with open(os.path.join(HERE, "tiny_model.json"), "w") as fh:
        json.dump({"config": "tiny", "seed": TINY_SEED, "sha256": sha, "prompt_len": TINY_PROMPT,
                   "steps": TINY_STEPS, "prompt_seed": 3}, fh, indent=2)
    with open(os.path.join(HERE, "ops.npz"), "rb") as fh:
        print("ops.npz", hashlib.sha256(fh.read()).hexdigest()[:16], len(g), "arrays")
    print("tiny model sha256", sha, "tokens", case["tokens"].tolist())


if __name__ == "__main__":
    main()
