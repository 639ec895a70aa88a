"""Tensor parallelism over the GPUs of one node (no counterpart in the
reference): one process per GPU, each holding one rank's share of the model.

Rank r of `world` holds, per layer (Megatron-style):
  q_proj / k_proj / v_proj   rows of its num_key_value_heads/world kv heads and
                             their query heads (GQA groups stay on one rank);
  o_proj                     the matching input columns (a partial sum of the
                             hidden vector);
  gate_proj / up_proj        rows r*F/world .. (r+1)*F/world;
  down_proj                  the matching input columns (a partial sum);
and all norms, the embedding and lm_head whole. The library adds the partial
sums over the group before they join the residual stream, so every rank
computes the same logits and greedy tokens: single-token steps exchange them
by peer stores over NVLink (the persistent kernel; when every rank has its own
GPU), prompts and the batched path by NCCL all-reduce. Greedy steps without
logits split the lm_head by vocabulary over the ranks.

`shard_config` / `shard_tensor` are the sharding rule (pure numpy, tested on
the CPU); `TPGroup` is the NCCL group; `load_tp_model` builds a rank's model.
"""

from __future__ import annotations

import ctypes

import numpy as np

from . import _lib
from ._lib import call

ID_BYTES = 128


def check_shardable(c, world: int) -> None:
    """The split must keep whole GQA groups and 8-aligned FFN slices."""
    if world < 1:
        raise ValueError("world size must be at least 1")
    if c.num_key_value_heads % world or c.num_attention_heads % world:
        raise ValueError(f"{c.num_key_value_heads} kv heads / {c.num_attention_heads} heads do not split over {world}")
    if c.intermediate_size % world or (c.intermediate_size // world) % 8:
        raise ValueError(f"intermediate size {c.intermediate_size} does not split into 8-aligned slices over {world}")


def shard_config(c, world: int):
    """The config rank r's model is built with: local head and FFN counts."""
    from .model import Config
    check_shardable(c, world)
    d = dict(hidden_size=c.hidden_size, intermediate_size=c.intermediate_size // world,
             num_hidden_layers=c.num_hidden_layers, num_attention_heads=c.num_attention_heads // world,
             num_key_value_heads=c.num_key_value_heads // world, head_dim=c.head_dim(),
             rms_norm_eps=c.rms_norm_eps, rope_theta=c.rope_theta, vocab_size=c.vocab_size,
             tie_word_embeddings=c.tie_word_embeddings)
    return Config(**d)


def shard_window(c, name: str, shape, rank: int, world: int):
    """Rank `rank`'s block of checkpoint tensor `name` of `shape`, as
    (row0, rows, col0, cols), or None when every rank holds it whole."""
    d = c.head_dim()
    q_rows = c.num_attention_heads // world * d
    kv_rows = c.num_key_value_heads // world * d
    f = c.intermediate_size // world
    if name.endswith(("q_proj.weight",)):
        return rank * q_rows, q_rows, 0, shape[1]
    if name.endswith(("k_proj.weight", "v_proj.weight")):
        return rank * kv_rows, kv_rows, 0, shape[1]
    if name.endswith("o_proj.weight"):
        return 0, shape[0], rank * q_rows, q_rows
    if name.endswith(("gate_proj.weight", "up_proj.weight")):
        return rank * f, f, 0, shape[1]
    if name.endswith("down_proj.weight"):
        return 0, shape[0], rank * f, f
    return None


def shard_tensor(c, name: str, shape, data: np.ndarray, rank: int, world: int):
    """Rank `rank`'s part of checkpoint tensor `name` (shape, bf16 bits)."""
    shape = list(shape)
    a = np.asarray(data).reshape(shape)
    w = shard_window(c, name, shape, rank, world)
    if w is not None:
        r0, nr, c0, nc = w
        a = a[r0:r0 + nr, c0:c0 + nc]
    a = np.ascontiguousarray(a)
    return list(a.shape), a.reshape(-1)


def _nccl_after_torch() -> None:
    """The library opens NCCL as libnccl.so.2 the first time a group needs
    it. PyTorch links its own (newer) libnccl.so.2, and the dynamic linker
    resolves a library by that name to whichever copy the process loaded
    first: if the system's older NCCL came first, `import torch` afterwards
    fails on a missing NCCL symbol. Importing torch (when installed) before
    the first NCCL call makes both use PyTorch's copy."""
    try:
        import torch  # noqa: F401
    except ImportError:
        pass


class TPGroup:
    """An NCCL group of `world` ranks, this process being `rank` on `device`.
    Every rank passes the same 128-byte id, made once by `unique_id()`."""

    def __init__(self, device, rank: int, world: int, uid: bytes):
        if len(uid) != ID_BYTES:
            raise ValueError(f"group id is {ID_BYTES} bytes")
        _nccl_after_torch()
        h = ctypes.c_void_p()
        call("tb200_tp_init", device._h, int(rank), int(world), uid, ID_BYTES, ctypes.byref(h))
        self._h = h.value
        self.device, self.rank, self.world = device, rank, world

    @staticmethod
    def unique_id() -> bytes:
        _nccl_after_torch()
        buf = ctypes.create_string_buffer(ID_BYTES)
        call("tb200_tp_unique_id", buf, ID_BYTES)
        return buf.raw

    def allreduce(self, buf) -> None:
        call("tb200_tp_allreduce", self._h, buf._h)

    def close(self) -> None:
        if getattr(self, "_h", None):
            _lib.lib().tb200_tp_free(self._h)
            self._h = None


def load_tp_model(path: str, device, group: TPGroup):
    """Model::load of rank `group.rank`'s share of the checkpoint at `path`."""
    import os

    from .model import Config, Model, Weights, tensor_names
    c = Config.load(os.path.join(path, "config.json"))
    local = shard_config(c, group.world)
    f = os.path.join(path, "model.safetensors")
    w = Weights.open(f)  # the header, for the shapes the windows are cut from
    names = [(n, req) for n, req in tensor_names(c) if w.contains(n) or req]
    for n, req in names:
        if not w.contains(n):
            raise KeyError(f"missing tensor '{n}'")
    wins = [shard_window(c, n, w.entries[n]["shape"], group.rank, group.world) for n, _ in names]
    ws = device.upload_safetensors(f, [n for n, _ in names], windows=wins)
    return Model(local, device, dict(zip([n for n, _ in names], ws)), tp=group)
