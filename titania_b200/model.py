"""The model side of the reference's `model` crate, over the B200 device.

- `Config` and `Weights` read a Hugging Face checkpoint directory as
  model/config.rs:10-35 and model/weights.rs:35-81 do.
- `OpModel`/`OpState` replay Model::forward (model/model.rs:83-149) one
  `Device` call at a time: the literal drop-in, generic over any object with
  the trait's methods.
- `Model`/`State` are the fast path on a `B200`: the same forward pass as a
  few fused kernels per layer, replayed from a CUDA graph, with a bf16
  key/value cache and greedy sampling on the device.
- `Sampler` restates model/sampler.rs for the host side.
"""

from __future__ import annotations

import ctypes
import json
import os
import sys

import numpy as np

from . import _lib
from ._lib import call
from .device import B200, Tensor

BATCH = 64  # model/model.rs:8

# The fused kernels of a decode step (include/titania_b200.h TB200_OP_*).
OP_EMBED, OP_QKV, OP_ATTENTION, OP_O, OP_GATE_UP, OP_DOWN, OP_LM_HEAD, OP_ATTENTION_O, OP_GATE_UP_SUM = range(9)
ATTN_O_MAX_CTX = 64  # positions below this run attention and o_proj fused


class Config:
    """config.json fields (model/config.rs:10-25)."""

    FIELDS = ("hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
              "num_key_value_heads", "rms_norm_eps", "rope_theta", "vocab_size")

    def __init__(self, **kw):
        for f in self.FIELDS:
            if f not in kw:
                raise ValueError(f"config.json: missing field `{f}`")
        self.hidden_size = int(kw["hidden_size"])
        self.intermediate_size = int(kw["intermediate_size"])
        self.num_hidden_layers = int(kw["num_hidden_layers"])
        self.num_attention_heads = int(kw["num_attention_heads"])
        self.num_key_value_heads = int(kw["num_key_value_heads"])
        self._head_dim = kw.get("head_dim")
        self.rms_norm_eps = float(np.float32(kw["rms_norm_eps"]))
        self.rope_theta = float(np.float32(kw["rope_theta"]))
        self.vocab_size = int(kw["vocab_size"])
        self.tie_word_embeddings = bool(kw.get("tie_word_embeddings", False))

    @classmethod
    def load(cls, path: str) -> "Config":
        with open(path) as fh:
            return cls(**json.load(fh))

    def head_dim(self) -> int:
        """model/config.rs:32-35"""
        return int(self._head_dim) if self._head_dim else self.hidden_size // self.num_attention_heads

    def to_c(self) -> _lib.Config:
        return _lib.Config(self.hidden_size, self.intermediate_size, self.num_hidden_layers,
                           self.num_attention_heads, self.num_key_value_heads, self.head_dim(),
                           self.rms_norm_eps, self.rope_theta, self.vocab_size, int(self.tie_word_embeddings))


class Weights:
    """A safetensors file (model/weights.rs:21-81), memory-mapped."""

    def __init__(self, path: str):
        with open(path, "rb") as fh:
            n = int.from_bytes(fh.read(8), "little")
            header = json.loads(fh.read(n))
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        self._start = 8 + n
        self.entries = {k: v for k, v in header.items() if k != "__metadata__"}

    @classmethod
    def open(cls, path: str) -> "Weights":
        return cls(path)

    def contains(self, name: str) -> bool:
        return name in self.entries

    def read(self, name: str) -> Tensor:
        e = self.entries.get(name)
        if e is None:
            raise KeyError(f"missing tensor '{name}'")
        if e["dtype"] != "BF16":
            raise ValueError(f"tensor '{name}' is {e['dtype']}, expected BF16")
        a, b = e["data_offsets"]
        data = self._map[self._start + a:self._start + b].view("<u2")
        return Tensor(e["shape"], data)


def tensor_names(c: Config) -> list[tuple[str, bool]]:
    """(name, required) for every tensor Model::load reads (model/model.rs:46-72)."""
    out = []
    for i in range(c.num_hidden_layers):
        p = f"model.layers.{i}"
        out += [(f"{p}.input_layernorm.weight", True), (f"{p}.self_attn.q_proj.weight", True),
                (f"{p}.self_attn.k_proj.weight", True), (f"{p}.self_attn.v_proj.weight", True),
                (f"{p}.self_attn.o_proj.weight", True), (f"{p}.self_attn.q_norm.weight", False),
                (f"{p}.self_attn.k_norm.weight", False), (f"{p}.post_attention_layernorm.weight", True),
                (f"{p}.mlp.gate_proj.weight", True), (f"{p}.mlp.up_proj.weight", True),
                (f"{p}.mlp.down_proj.weight", True)]
    if not c.tie_word_embeddings:
        out.append(("lm_head.weight", True))
    out += [("model.embed_tokens.weight", True), ("model.norm.weight", True)]
    return out


def load_weights(device, c: Config, w: Weights) -> dict:
    """Uploads every tensor of the checkpoint to `device` (Model::load)."""
    up = {}
    for name, required in tensor_names(c):
        if w.contains(name):
            up[name] = device.upload(w.read(name))
        elif required:
            raise KeyError(f"missing tensor '{name}'")
    return up


def upload_checkpoint(device: B200, c: Config, path: str) -> dict:
    """Model::load's reads and uploads (model/model.rs:42-72, 251-254) in one
    library call: every tensor goes from the safetensors file at `path` to
    device memory with no host-side conversion (tb200_upload_safetensors).
    A missing required tensor raises KeyError as Weights::read fails."""
    names = tensor_names(c)
    ws = device.upload_safetensors(path, [n for n, _ in names])
    up = {}
    for (name, required), w in zip(names, ws):
        if w is not None:
            up[name] = w
        elif required:
            raise KeyError(f"missing tensor '{name}'")
    return up


def rope_table(max_len: int, head_dim: int, theta: float) -> np.ndarray:
    """model/model.rs:239-250, computed by the library on the host with the
    platform libm, as the reference computes it."""
    out = np.empty(int(max_len) * int(head_dim), dtype=np.float32)
    call("tb200_rope_table", int(max_len), int(head_dim), ctypes.c_float(theta), out.ctypes.data_as(_lib.F32P))
    return out


# ---- the generic model: one Device call per op -----------------------------

class OpState:
    """State (model/model.rs:156-233) on any device."""

    def __init__(self, model: "OpModel", max_len: int, table=None):
        c, d = model.config, model.device
        q_dim, kv_dim = c.num_attention_heads * c.head_dim(), c.num_key_value_heads * c.head_dim()
        self.widths = [c.hidden_size, c.hidden_size, q_dim, kv_dim, kv_dim, q_dim, c.intermediate_size,
                       c.intermediate_size]
        (self.x, self.xb, self.q, self.k, self.v, self.att, self.gate, self.up) = [
            d.alloc(BATCH * w) for w in self.widths]
        table = rope_table(max_len, c.head_dim(), c.rope_theta) if table is None else table
        self.rope = d.alloc(table.size)
        d.write(self.rope, table)
        self.logits = d.alloc(c.vocab_size)
        self.k_cache = [d.alloc(max_len * kv_dim) for _ in range(c.num_hidden_layers)]
        self.v_cache = [d.alloc(max_len * kv_dim) for _ in range(c.num_hidden_layers)]
        self.max_len = max_len

    def batch(self, device, n: int):
        if n > BATCH:
            raise ValueError(f"a batch of {n} tokens is more than {BATCH}")
        for buf, w in zip((self.x, self.xb, self.q, self.k, self.v, self.att, self.gate, self.up), self.widths):
            device.resize(buf, n * w)


class OpModel:
    """Model<D> (model/model.rs:11-149) driving `device` one trait call at a time."""

    def __init__(self, config: Config, device, weights: dict):
        self.config, self.device, self.w = config, device, weights

    @classmethod
    def load(cls, path: str, device) -> "OpModel":
        c = Config.load(os.path.join(path, "config.json"))
        return cls(c, device, load_weights(device, c, Weights.open(os.path.join(path, "model.safetensors"))))

    def state(self, max_len: int, table=None) -> OpState:
        return OpState(self, max_len, table)

    def forward(self, state: OpState, tokens, pos: int) -> np.ndarray:
        tokens = list(tokens)
        if not tokens:
            raise ValueError("no tokens to run")
        if pos + len(tokens) > state.max_len:
            raise ValueError("tokens past the end of the cache")
        logits = None
        for i in range(0, len(tokens), BATCH):
            logits = self._forward_batch(state, tokens[i:i + BATCH], pos + i)
        return logits

    def _forward_batch(self, s: OpState, tokens, pos: int) -> np.ndarray:
        c, d, w = self.config, self.device, self.w
        n, eps, hd = len(tokens), c.rms_norm_eps, c.head_dim()
        kv_dim = c.num_key_value_heads * hd
        s.batch(d, n)
        d.embed(s.x, w["model.embed_tokens.weight"], tokens)
        for i in range(c.num_hidden_layers):
            p = f"model.layers.{i}"
            d.copy(s.xb, 0, s.x, 0, n * c.hidden_size)
            d.rmsnorm(s.xb, w[f"{p}.input_layernorm.weight"], eps)
            d.matmul(s.q, w[f"{p}.self_attn.q_proj.weight"], s.xb)
            d.matmul(s.k, w[f"{p}.self_attn.k_proj.weight"], s.xb)
            d.matmul(s.v, w[f"{p}.self_attn.v_proj.weight"], s.xb)
            if f"{p}.self_attn.q_norm.weight" in w:
                d.rmsnorm(s.q, w[f"{p}.self_attn.q_norm.weight"], eps)
            if f"{p}.self_attn.k_norm.weight" in w:
                d.rmsnorm(s.k, w[f"{p}.self_attn.k_norm.weight"], eps)
            d.rope(s.q, s.rope, pos, c.num_attention_heads, hd)
            d.rope(s.k, s.rope, pos, c.num_key_value_heads, hd)
            d.copy(s.k_cache[i], pos * kv_dim, s.k, 0, n * kv_dim)
            d.copy(s.v_cache[i], pos * kv_dim, s.v, 0, n * kv_dim)
            d.attention(s.att, s.q, s.k_cache[i], s.v_cache[i], pos, c.num_attention_heads, hd,
                        c.num_key_value_heads)
            d.matmul(s.xb, w[f"{p}.self_attn.o_proj.weight"], s.att)
            d.add(s.x, s.xb)
            d.copy(s.xb, 0, s.x, 0, n * c.hidden_size)
            d.rmsnorm(s.xb, w[f"{p}.post_attention_layernorm.weight"], eps)
            d.matmul(s.gate, w[f"{p}.mlp.gate_proj.weight"], s.xb)
            d.matmul(s.up, w[f"{p}.mlp.up_proj.weight"], s.xb)
            d.silu_mul(s.gate, s.up)
            d.matmul(s.xb, w[f"{p}.mlp.down_proj.weight"], s.gate)
            d.add(s.x, s.xb)
        d.resize(s.xb, c.hidden_size)
        d.copy(s.xb, 0, s.x, (n - 1) * c.hidden_size, c.hidden_size)
        d.rmsnorm(s.xb, w["model.norm.weight"], eps)
        d.matmul(s.logits, w.get("lm_head.weight", w["model.embed_tokens.weight"]), s.xb)
        return d.read(s.logits)


# ---- the fused fast path -------------------------------------------------------

class Model:
    """Model<B200> with the fused decode path (no trait counterpart in the
    reference; its forward pass computes what model/model.rs:93-149 does)."""

    def __init__(self, config: Config, device: B200, weights: dict, tp=None):
        self.config, self.device, self.weights, self.tp = config, device, weights, tp
        h = ctypes.c_void_p()
        cfg = config.to_c()
        call("tb200_model_create", device._h, ctypes.byref(cfg), ctypes.byref(h))
        self._h = h.value
        for name, wt in weights.items():
            call("tb200_model_bind", self._h, name.encode(), wt._h)
        if tp is not None:  # a tensor-parallel rank (titania_b200.tp): partial sums are reduced over the group
            call("tb200_model_set_tp", self._h, tp._h)
        call("tb200_model_finalize", self._h)

    @classmethod
    def load(cls, path: str, device: B200) -> "Model":
        """Model::load (model/model.rs:40-77)."""
        c = Config.load(os.path.join(path, "config.json"))
        return cls(c, device, upload_checkpoint(device, c, os.path.join(path, "model.safetensors")))

    def __del__(self):
        if getattr(self, "_h", None) and not sys.is_finalizing():
            _lib.lib().tb200_model_free(self._h)
        self._h = None

    @property
    def tp_peer_exchange(self) -> bool:
        """Whether this tensor-parallel rank's single-token steps add the
        o_proj / down_proj partial sums by peer stores over NVLink (the
        persistent kernel, and the fused graphs' flags); else the fused graphs
        with NCCL."""
        return bool(_lib.lib().tb200_model_tp_peer_exchange(self._h))

    def state(self, max_len: int, kv: str = "f32", decode: str | None = None) -> "State":
        return State(self, max_len, kv, decode)

    def forward(self, state: "State", tokens, pos: int, logits: bool = True, out=None):
        """Model::forward (model/model.rs:83-91): the logits for the token after
        the last of `tokens` (a float32 array of vocab_size, written into `out`
        when given), or, with logits=False, only the greedy next token."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        nxt = ctypes.c_uint32()
        if logits and out is None:
            out = np.empty(self.config.vocab_size, dtype=np.float32)
        if logits:
            assert out.dtype == np.float32 and out.size == self.config.vocab_size and out.flags.c_contiguous
        call("tb200_forward", self._h, state._h, t.ctypes.data_as(_lib.U32P), t.size, int(pos),
             out.ctypes.data_as(_lib.F32P) if logits else None, ctypes.byref(nxt))
        self.last_token = int(nxt.value)
        return out if logits else self.last_token

    def generate(self, state: "State", token: int, pos: int, steps: int) -> list[int]:
        """Greedy decoding on the device: feeds `token` at `pos`, then each
        chosen token; returns the `steps` chosen tokens."""
        out = np.empty(steps, dtype=np.uint32)
        call("tb200_generate", self._h, state._h, int(token), int(pos), int(steps), out.ctypes.data_as(_lib.U32P))
        return out.tolist()

    def decode_persistent(self, state: "State", token: int, pos: int, steps: int, logits: bool = False):
        """`generate` through the persistent kernel whatever the state's
        decode mode: the `steps` chosen tokens, and with logits=True also
        their [steps][vocab] logits (one launch per step then)."""
        out = np.empty(steps, dtype=np.uint32)
        lg = np.empty((steps, self.config.vocab_size), dtype=np.float32) if logits else None
        call("tb200_decode_persistent", self._h, state._h, int(token), int(pos), int(steps),
             out.ctypes.data_as(_lib.U32P), lg.ctypes.data_as(_lib.F32P) if logits else None)
        return (out.tolist(), lg) if logits else out.tolist()

    def decode_enqueue(self, state: "State", token: int, pos: int, steps: int) -> None:
        """Enqueues `steps` greedy steps from `token` at `pos` without waiting
        or copying back (for timing)."""
        call("tb200_decode_enqueue", self._h, state._h, int(token), int(pos), int(steps))

    def enqueue_op(self, state: "State", op: int, layer: int = 0) -> None:
        """Enqueues one fused kernel of the decode step (TB200_OP_*)."""
        call("tb200_enqueue_op", self._h, state._h, int(op), int(layer))

    # ---- many sequences ----------------------------------------------------

    def batch_state(self, n_seqs: int, max_len: int, kv: str = "f32") -> "BatchState":
        return BatchState(self, n_seqs, max_len, kv)

    def forward_seq(self, state: "BatchState", seq: int, tokens, pos: int, logits: bool = True, out=None):
        """Model::forward for sequence `seq` of a many-sequence state."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        nxt = ctypes.c_uint32()
        if logits and out is None:
            out = np.empty(self.config.vocab_size, dtype=np.float32)
        call("tb200_forward_seq", self._h, state._h, int(seq), t.ctypes.data_as(_lib.U32P), t.size, int(pos),
             out.ctypes.data_as(_lib.F32P) if logits else None, ctypes.byref(nxt))
        self.last_token = int(nxt.value)
        return out if logits else self.last_token

    def forward_batch(self, state: "BatchState", tokens, positions, logits: bool = True, out=None):
        """One decode step of every sequence (token i of sequence i at
        positions[i]). Returns (logits [n_seqs][vocab] or None, next tokens)."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uintp)
        n = state.n_seqs
        assert t.size == n and p.size == n
        if logits and out is None:
            out = np.empty((n, self.config.vocab_size), dtype=np.float32)
        nxt = np.empty(n, dtype=np.uint32)
        call("tb200_forward_batch", self._h, state._h, t.ctypes.data_as(_lib.U32P), p.ctypes.data_as(_lib.SZP),
             out.ctypes.data_as(_lib.F32P) if logits else None, nxt.ctypes.data_as(_lib.U32P))
        return (out if logits else None), nxt

    def generate_batch(self, state: "BatchState", tokens, positions, steps: int) -> np.ndarray:
        """Greedy decoding of every sequence on the device; [steps][n_seqs]."""
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uintp)
        out = np.empty((steps, state.n_seqs), dtype=np.uint32)
        call("tb200_generate_batch", self._h, state._h, t.ctypes.data_as(_lib.U32P), p.ctypes.data_as(_lib.SZP),
             int(steps), out.ctypes.data_as(_lib.U32P))
        return out

    def decode_batch_enqueue(self, state: "BatchState", tokens, positions, steps: int) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        p = np.ascontiguousarray(positions, dtype=np.uintp)
        call("tb200_decode_batch_enqueue", self._h, state._h, t.ctypes.data_as(_lib.U32P),
             p.ctypes.data_as(_lib.SZP), int(steps))


KV_TYPES = {"bf16": 0, "f32": 1}
DECODE_MODES = {"fused": 0, "persistent": 1}


class State:
    """State (model/model.rs:156-211) of the fused path. The key/value cache
    holds f32 like the reference (default) or bf16, which halves the bytes
    attention reads at long contexts at the cost of rounding K and V."""

    def __init__(self, model: Model, max_len: int, kv: str = "f32", decode: str | None = None):
        if kv not in KV_TYPES:
            raise ValueError(f"kv must be one of {sorted(KV_TYPES)}")
        h = ctypes.c_void_p()
        call("tb200_state_new", model._h, int(max_len), KV_TYPES[kv], ctypes.byref(h))
        self._h = h.value
        self.model = model
        self.max_len = max_len
        self.kv = kv
        if decode is not None:
            self.decode = decode

    @property
    def decode(self) -> str:
        """What single-token steps run: "persistent" (one kernel per launch,
        the default where the model allows it) or "fused" (2 + 5 * layers
        kernels per step from a CUDA graph)."""
        return {v: k for k, v in DECODE_MODES.items()}[_lib.lib().tb200_state_decode(self._h)]

    @decode.setter
    def decode(self, mode: str) -> None:
        if mode not in DECODE_MODES:
            raise ValueError(f"decode must be one of {sorted(DECODE_MODES)}")
        call("tb200_state_set_decode", self._h, DECODE_MODES[mode])

    def __del__(self):
        if getattr(self, "_h", None) and not sys.is_finalizing():
            _lib.lib().tb200_state_free(self._h)
        self._h = None

    TRACE_DTYPE = np.dtype([("tag", "<u4"), ("cta", "<u4"), ("event", "<u4"), ("sm", "<u4"), ("ns", "<u8")])

    def trace_start(self, capacity: int = 1 << 20) -> None:
        """Starts recording the kernels' device-side trace events."""
        call("tb200_trace_start", self._h, int(capacity))
        self._trace_cap = int(capacity)

    def trace_stop(self) -> np.ndarray:
        """Stops tracing; returns the records (tag = op << 16 | layer, cta,
        event, sm, ns) as a numpy structured array."""
        out = np.zeros(self._trace_cap, dtype=self.TRACE_DTYPE)
        n = ctypes.c_size_t()
        call("tb200_trace_stop", self._h, out.ctypes.data_as(ctypes.c_void_p), out.size, ctypes.byref(n))
        out = out[:min(n.value, out.size)]
        return out[out["ns"] != 0]

    BUFFERS = {"x": 0, "qkv": 1, "att": 2, "h": 3, "logits": 4, "x2": 5, "part": 6}

    def _buf_len(self, name):
        c = self.model.config
        d = c.head_dim()
        return {"x": c.hidden_size, "qkv": (c.num_attention_heads + 2 * c.num_key_value_heads) * d,
                "att": c.num_attention_heads * d, "h": c.intermediate_size, "logits": c.vocab_size,
                "x2": c.hidden_size, "part": c.num_key_value_heads * c.hidden_size}[name]

    def read(self, name: str) -> np.ndarray:
        """A copy of one of the fused path's activation buffers."""
        out = np.empty(self._buf_len(name), dtype=np.float32)
        call("tb200_state_read", self._h, self.BUFFERS[name], out.ctypes.data_as(_lib.F32P), out.size)
        return out

    def write(self, name: str, data) -> None:
        a = np.ascontiguousarray(data, dtype=np.float32)
        call("tb200_state_write", self._h, self.BUFFERS[name], a.ctypes.data_as(_lib.F32P), a.size)

    def set_position(self, token: int, pos: int) -> None:
        call("tb200_state_set_position", self._h, int(token), int(pos))

    def read_kv(self, layer: int, which: int, pos: int) -> np.ndarray:
        c = self.model.config
        out = np.empty(c.num_key_value_heads * c.head_dim(), dtype=np.float32)
        call("tb200_state_read_kv", self._h, int(layer), int(which), int(pos), out.ctypes.data_as(_lib.F32P))
        return out


class BatchState:
    """`n_seqs` independent sequences, each with its own key/value cache of
    `max_len` positions (what n_seqs separate State::new would hold), run
    together by Model.forward_batch / generate_batch."""

    def __init__(self, model: Model, n_seqs: int, max_len: int, kv: str = "f32"):
        if kv not in KV_TYPES:
            raise ValueError(f"kv must be one of {sorted(KV_TYPES)}")
        h = ctypes.c_void_p()
        call("tb200_batch_state_new", model._h, int(n_seqs), int(max_len), KV_TYPES[kv], ctypes.byref(h))
        self._h = h.value
        self.model = model
        self.n_seqs = n_seqs
        self.max_len = max_len
        self.kv = kv

    def __del__(self):
        if getattr(self, "_h", None) and not sys.is_finalizing():
            _lib.lib().tb200_state_free(self._h)
        self._h = None

    def read_kv(self, seq: int, layer: int, which: int, pos: int) -> np.ndarray:
        c = self.model.config
        out = np.empty(c.num_key_value_heads * c.head_dim(), dtype=np.float32)
        call("tb200_batch_read_kv", self._h, int(seq), int(layer), int(which), int(pos),
             out.ctypes.data_as(_lib.F32P))
        return out

    def trace_start(self, capacity: int = 1 << 20) -> None:
        """Records the batched decode step's kernels (TB200_TRACE_OP_* tags)."""
        call("tb200_trace_start", self._h, int(capacity))
        self._trace_cap = int(capacity)

    def trace_stop(self) -> np.ndarray:
        out = np.zeros(self._trace_cap, dtype=State.TRACE_DTYPE)
        n = ctypes.c_size_t()
        call("tb200_trace_stop", self._h, out.ctypes.data_as(ctypes.c_void_p), out.size, ctypes.byref(n))
        out = out[:min(n.value, out.size)]
        return out[out["ns"] != 0]


class DeviceSampler:
    """model/sampler.rs:12-77 on the B200 (tb200_sampler_*): top-k, top-p and
    temperature over `rows` rows of `vocab` logits in a device buffer, with one
    xorshift64* state per row kept in device memory (row i starts at
    max(seeds[i], 1)). Exact logit ties go to the lowest token id."""

    def __init__(self, dev: B200, rows: int, vocab: int, temperature: float, top_k: int, top_p: float, seeds):
        seeds = [int(x) & 0xFFFFFFFFFFFFFFFF for x in seeds]
        if len(seeds) != rows:
            raise ValueError("one seed per row")
        self._dev, self.rows, self.vocab = dev, int(rows), int(vocab)
        arr = (ctypes.c_uint64 * rows)(*seeds)
        h = ctypes.c_void_p()
        call("tb200_sampler_new", dev._h, rows, vocab, float(temperature), int(top_k), float(top_p), arr,
             ctypes.byref(h))
        self._h = h.value

    def sample(self, logits) -> np.ndarray:
        """One token per row of `logits` (a device Buffer of rows x vocab f32)."""
        out = np.zeros(self.rows, dtype=np.uint32)
        call("tb200_sample", self._h, logits._h, out.ctypes.data_as(_lib.U32P))
        return out

    def states(self) -> np.ndarray:
        out = (ctypes.c_uint64 * self.rows)()
        call("tb200_sampler_state", self._h, out)
        return np.array(list(out), dtype=np.uint64)

    def close(self) -> None:
        if getattr(self, "_h", None) and not sys.is_finalizing():
            _lib.lib().tb200_sampler_free(self._h)
        self._h = None

    __del__ = close


def _libm_expf():
    """The platform libm's expf, which Rust's f32::exp calls on Linux."""
    import ctypes.util
    libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
    f = libm.expf
    f.restype = ctypes.c_float
    f.argtypes = [ctypes.c_float]
    return f


_expf = _libm_expf()


class Sampler:
    """model/sampler.rs: top-k, then top-p, at a temperature; temperature 0 is
    greedy (ties to the lowest token id)."""

    def __init__(self, temperature: float, top_k: int, top_p: float, seed: int):
        self.temperature, self.top_k, self.top_p = np.float32(temperature), int(top_k), np.float32(top_p)
        self._rng = max(int(seed), 1) & 0xFFFFFFFFFFFFFFFF

    def _next_f32(self) -> np.float32:
        x = self._rng
        x ^= x >> 12
        x ^= (x << 25) & 0xFFFFFFFFFFFFFFFF
        x ^= x >> 27
        self._rng = x
        v = (x * 0x2545F4914F6CDD1D) & 0xFFFFFFFFFFFFFFFF
        return np.float32(v >> 40) / np.float32(1 << 24)

    def sample(self, logits) -> int:
        logits = np.asarray(logits, dtype=np.float32)
        b = logits.view(np.int32).astype(np.int64)
        key = np.where(b < 0, b ^ 0x7FFFFFFF, b)
        k = min(max(self.top_k, 1), logits.size)
        order = np.lexsort((np.arange(logits.size), -key))[:k]
        if self.temperature == 0:
            return int(order[0])
        # sampler.rs:35-50 in its order, in f32: exp through the platform libm
        # (as Rust's f32::exp), the sum of the probabilities accumulated
        # sequentially, then each divided by it while the running total is
        # below top_p.
        cand = logits[order]
        mx = np.float32(cand[0])
        probs = [np.float32(_expf(float((np.float32(c) - mx) / self.temperature))) for c in cand]
        total = np.float32(0)
        for p in probs:
            total = np.float32(total + p)
        cum, n = np.float32(0), 0
        for i in range(len(probs)):
            probs[i] = np.float32(probs[i] / total)
            if cum < self.top_p:
                cum = np.float32(cum + probs[i])
                n += 1
        r = np.float32(self._next_f32() * cum)
        for tok, p in zip(order[:n], probs[:n]):
            r = np.float32(r - p)
            if r <= 0:
                return int(tok)
        return int(order[n - 1])
