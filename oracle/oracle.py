"""ctypes wrapper for the CPU oracle (liboracle.so) — TEST INFRASTRUCTURE ONLY.

The oracle restates the Titania reference CPU device (model/cpu.rs) and model
forward pass (model/model.rs) in C++; see oracle.cpp's header for what it
follows and why its parity is unpinned against the running reference. Only
the tests, `__graft_entry__.smoke()` and bench.py's CPU-baseline leg use it,
as the checker or the timed CPU baseline; the product never does.

Op functions work on numpy arrays in place, mirroring the `Device` trait's
argument meaning (model/device.rs:9-89): f32 activation arrays for buffers,
uint16 bf16-bit arrays (with a shape) for weights.
"""

from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None

f32p = ctypes.POINTER(ctypes.c_float)
u16p = ctypes.POINTER(ctypes.c_uint16)
u32p = ctypes.POINTER(ctypes.c_uint32)
sz = ctypes.c_size_t


class OracleError(RuntimeError):
    """A reference panic (assertion failure) inside the oracle."""


def build() -> str:
    """Builds liboracle.so with the committed Makefile if it is missing or stale."""
    src = os.path.join(_HERE, "oracle.cpp")
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-C", _HERE, "liboracle.so"], check=True, capture_output=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(_LIB_PATH)
        L.orc_last_error.restype = ctypes.c_char_p
        L.orc_set_threads.argtypes = [ctypes.c_int]
        L.orc_max_threads.restype = ctypes.c_int
        L.orc_embed.argtypes = [f32p, sz, u16p, sz, u32p, sz]
        L.orc_matmul.argtypes = [f32p, sz, u16p, sz, sz, f32p, sz]
        L.orc_add.argtypes = [f32p, f32p, sz]
        L.orc_rmsnorm.argtypes = [f32p, sz, u16p, sz, ctypes.c_float]
        L.orc_rope.argtypes = [f32p, sz, f32p, sz, sz, sz]
        L.orc_attention.argtypes = [f32p, f32p, sz, f32p, f32p, sz, sz, sz, sz]
        L.orc_silu_mul.argtypes = [f32p, f32p, sz]
        L.orc_rope_table.argtypes = [f32p, sz, sz, ctypes.c_float]
        L.orc_sample_greedy.argtypes = [f32p, sz]
        L.orc_sample_greedy.restype = ctypes.c_uint32
        L.orc_sample.argtypes = [f32p, sz, ctypes.c_float, sz, ctypes.c_float, ctypes.POINTER(ctypes.c_uint64)]
        L.orc_sample.restype = ctypes.c_uint32
        L.orc_model_load.argtypes = [ctypes.c_char_p]
        L.orc_model_load.restype = ctypes.c_void_p
        L.orc_model_free.argtypes = [ctypes.c_void_p]
        L.orc_model_dims.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_size_t)]
        L.orc_state_new.argtypes = [ctypes.c_void_p, sz]
        L.orc_state_new.restype = ctypes.c_void_p
        L.orc_state_free.argtypes = [ctypes.c_void_p]
        L.orc_forward.argtypes = [ctypes.c_void_p, ctypes.c_void_p, u32p, sz, sz, f32p]
        L.orc_state_kv.argtypes = [ctypes.c_void_p, sz, ctypes.c_int, f32p, sz]
        _lib = L
    return _lib


def _p(a, t):
    return a.ctypes.data_as(t)


def _check(rc):
    if rc != 0:
        raise OracleError(lib().orc_last_error().decode())


def _f32(a):
    assert a.dtype == np.float32 and a.flags.c_contiguous
    return _p(a, f32p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return lib().orc_max_threads()


# --- Device ops (model/cpu.rs:38-155), in place on numpy arrays -------------

def embed(out, table, tokens):
    tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
    _check(lib().orc_embed(_f32(out), out.size, _p(table, u16p), table.shape[1], _p(tokens, u32p), tokens.size))


def matmul(out, w, x):
    _check(lib().orc_matmul(_f32(out), out.size, _p(w, u16p), w.shape[0], w.shape[1], _f32(x), x.size))


def add(x, y):
    assert x.size == y.size
    _check(lib().orc_add(_f32(x), _f32(y), x.size))


def rmsnorm(x, weight, eps):
    _check(lib().orc_rmsnorm(_f32(x), x.size, _p(weight, u16p), weight.size, ctypes.c_float(eps)))


def rope(x, table, pos, n_heads, head_dim):
    _check(lib().orc_rope(_f32(x), x.size, _f32(table), pos, n_heads, head_dim))


def attention(out, q, k_cache, v_cache, pos, n_heads, head_dim, n_kv_heads):
    _check(lib().orc_attention(_f32(out), _f32(q), q.size, _f32(k_cache), _f32(v_cache), pos, n_heads, head_dim,
                               n_kv_heads))


def silu_mul(gate, up):
    assert gate.size == up.size
    _check(lib().orc_silu_mul(_f32(gate), _f32(up), gate.size))


def rope_table(max_len, head_dim, theta):
    out = np.empty(max_len * head_dim, dtype=np.float32)
    _check(lib().orc_rope_table(_f32(out), max_len, head_dim, ctypes.c_float(theta)))
    return out


class Sampler:
    """model/sampler.rs:12-77 restated in C (oracle.cpp orc_sample): top-k,
    top-p and temperature with the reference's xorshift64* state."""

    def __init__(self, temperature: float, top_k: int, top_p: float, seed: int):
        self.temperature, self.top_k, self.top_p = float(temperature), int(top_k), float(top_p)
        self.state = ctypes.c_uint64(max(int(seed), 1) & 0xFFFFFFFFFFFFFFFF)

    def sample(self, logits) -> int:
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        return int(lib().orc_sample(_f32(logits), logits.size, self.temperature, self.top_k, self.top_p,
                                    ctypes.byref(self.state)))


def sample_greedy(logits) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    return int(lib().orc_sample_greedy(_f32(logits), logits.size))


# --- Model (model/model.rs) --------------------------------------------------

class Model:
    """The reference `Model<Cpu>` loaded from a checkpoint directory."""

    def __init__(self, path: str):
        h = lib().orc_model_load(path.encode())
        if not h:
            raise OracleError(lib().orc_last_error().decode())
        self._h = h
        dims = (ctypes.c_size_t * 7)()
        lib().orc_model_dims(h, dims)
        (self.hidden_size, self.intermediate_size, self.num_hidden_layers, self.num_attention_heads,
         self.num_key_value_heads, self.head_dim, self.vocab_size) = list(dims)

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_model_free(self._h)
            self._h = None

    def state(self, max_len: int) -> "State":
        return State(self, max_len)

    def forward(self, state: "State", tokens, pos: int) -> np.ndarray:
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        out = np.empty(self.vocab_size, dtype=np.float32)
        _check(lib().orc_forward(self._h, state._h, _p(tokens, u32p), tokens.size, pos, _f32(out)))
        return out


class State:
    def __init__(self, model: Model, max_len: int):
        h = lib().orc_state_new(model._h, max_len)
        if not h:
            raise OracleError(lib().orc_last_error().decode())
        self._h = h
        self.model = model
        self.max_len = max_len

    def __del__(self):
        if getattr(self, "_h", None):
            lib().orc_state_free(self._h)
            self._h = None

    def kv(self, layer: int, which: int, length: int) -> np.ndarray:
        out = np.empty(length, dtype=np.float32)
        _check(lib().orc_state_kv(self._h, layer, which, _f32(out), length))
        return out


def greedy_generate(model: Model, prompt, steps: int, max_len: int | None = None):
    """Feeds `prompt`, then `steps` greedy tokens (model/chat.rs:149-196 with
    temperature 0). Returns (tokens, logits per generated step)."""
    max_len = max_len or (len(prompt) + steps + 1)
    st = model.state(max_len)
    logits = model.forward(st, prompt, 0)
    pos = len(prompt)
    toks, all_logits = [], []
    for _ in range(steps):
        t = sample_greedy(logits)
        toks.append(t)
        all_logits.append(logits)
        logits = model.forward(st, [t], pos)
        pos += 1
    return toks, all_logits
