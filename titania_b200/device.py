"""The `Device` trait (model/device.rs:9-89) implemented on a B200.

`B200` has the trait's methods with the trait's names and argument meaning;
`Buffer` and `Weight` are handles to device memory like Titania's
(model/titania.rs:43-55). Activations cross to the host only through
`read`, `write` and `embed`'s token ids, as in the reference. A violated
contract raises `DeviceError` where the reference panics.
"""

from __future__ import annotations

import ctypes
import os
import sys

import numpy as np

from . import _lib
from ._lib import DeviceError, call, lib


class Tensor:
    """A bf16 tensor on the host: its shape and raw bf16 bits
    (model/weights.rs:14-17)."""

    __slots__ = ("shape", "data")

    def __init__(self, shape, data):
        self.shape = list(int(s) for s in shape)
        self.data = np.ascontiguousarray(data, dtype=np.uint16).reshape(-1)
        if self.data.size != int(np.prod(self.shape)):
            raise ValueError(f"tensor of shape {self.shape} given {self.data.size} values")


class Weight:
    """Device::Weight: a bf16 tensor in device memory."""

    __slots__ = ("_h", "shape", "_dev")

    def __init__(self, handle, shape, dev):
        self._h, self.shape, self._dev = handle, list(shape), dev

    def __del__(self):
        if self._h and self._dev is not None and self._dev._h and not sys.is_finalizing():
            lib().tb200_free_weight(self._dev._h, self._h)
        self._h = None


class Buffer:
    """Device::Buffer: f32 activations in device memory."""

    __slots__ = ("_h", "_dev")

    def __init__(self, handle, dev):
        self._h, self._dev = handle, dev

    def __len__(self):
        return int(lib().tb200_buffer_len(self._h))

    def __del__(self):
        if self._h and self._dev is not None and self._dev._h and not sys.is_finalizing():
            lib().tb200_free_buffer(self._dev._h, self._h)
        self._h = None


def safetensors_entry(path: str, name: str):
    """(dtype, shape, file offset, bytes) of tensor `name` in the safetensors
    file at `path` as the library parses its header, or None when the file
    has no such tensor. Host only: needs no GPU."""
    found = ctypes.c_int()
    dtype = ctypes.create_string_buffer(64)
    shape = (ctypes.c_size_t * 16)()
    ndim = ctypes.c_size_t()
    off, nbytes = ctypes.c_uint64(), ctypes.c_uint64()
    call("tb200_safetensors_entry", os.fsencode(path), name.encode(), ctypes.byref(found), dtype, len(dtype), shape,
         16, ctypes.byref(ndim), ctypes.byref(off), ctypes.byref(nbytes))
    if not found.value:
        return None
    return dtype.value.decode(), [int(shape[i]) for i in range(ndim.value)], int(off.value), int(nbytes.value)


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_lib.F32P)


class B200:
    """A B200 GPU running the model's operations (one CUDA device)."""

    def __init__(self, ordinal: int = 0):
        h = ctypes.c_void_p()
        call("tb200_device_open", int(ordinal), ctypes.byref(h))
        self._h = h.value
        self.ordinal = ordinal

    def close(self):
        if getattr(self, "_h", None):
            lib().tb200_device_close(self._h)
            self._h = None

    def __del__(self):
        # Handles created on this device free themselves while it is open;
        # the device itself is left to process exit (as the reference never
        # frees a device).
        pass

    @property
    def stream(self) -> int:
        """The cudaStream_t every operation is enqueued on."""
        return int(lib().tb200_device_stream(self._h) or 0)

    @property
    def sms(self) -> int:
        return int(lib().tb200_device_sms(self._h))

    def sync(self):
        call("tb200_sync", self._h)

    # ---- the trait -----------------------------------------------------------

    def upload(self, tensor: Tensor) -> Weight:
        shape = (ctypes.c_size_t * len(tensor.shape))(*tensor.shape)
        h = ctypes.c_void_p()
        call("tb200_upload", self._h, tensor.data.ctypes.data_as(_lib.U16P), shape, len(tensor.shape),
             ctypes.byref(h))
        return Weight(h.value, tensor.shape, self)

    def upload_safetensors(self, path: str, names, threads: int = 0, windows=None) -> list:
        """Weights::read + upload for every name in `names` at once, straight
        from the safetensors file at `path` to device memory (no host-side
        conversion; reads overlapped with copies on `threads` host threads,
        0 = automatic). Returns one Weight per name, or None where the file
        has no such tensor; a tensor that is not BF16 raises as
        Weights::read fails (model/weights.rs:61-81). `windows`, if given,
        holds per name None (the tensor whole) or (row0, rows, col0, cols):
        that block of a matrix, packed (a tensor-parallel rank's share)."""
        names = [str(n) for n in names]
        arr = (ctypes.c_char_p * max(1, len(names)))(*[n.encode() for n in names])
        out = (ctypes.c_void_p * max(1, len(names)))()
        if windows is None:
            call("tb200_upload_safetensors", self._h, os.fsencode(path), arr, len(names), int(threads), out)
        else:
            if len(windows) != len(names):
                raise ValueError(f"{len(windows)} windows for {len(names)} tensors")
            win = (_lib.Window * max(1, len(names)))(*[_lib.Window(*(w or (0, 0, 0, 0))) for w in windows])
            call("tb200_upload_safetensors_windows", self._h, os.fsencode(path), arr, win, len(names),
                 int(threads), out)
        res = []
        shape, ndim = (ctypes.c_size_t * 16)(), ctypes.c_size_t()
        for i in range(len(names)):
            if out[i]:
                call("tb200_weight_shape", out[i], shape, 16, ctypes.byref(ndim))
                res.append(Weight(out[i], shape[:ndim.value], self))
            else:
                res.append(None)
        return res

    def alloc(self, length: int) -> Buffer:
        h = ctypes.c_void_p()
        call("tb200_alloc", self._h, int(length), ctypes.byref(h))
        return Buffer(h.value, self)

    def resize(self, buf: Buffer, length: int) -> None:
        call("tb200_resize", self._h, buf._h, int(length))

    def read(self, buf: Buffer) -> np.ndarray:
        out = np.empty(len(buf), dtype=np.float32)
        call("tb200_read", self._h, buf._h, out.ctypes.data_as(_lib.F32P), out.size)
        return out

    def write(self, buf: Buffer, data) -> None:
        a, p = _f32(data)
        call("tb200_write", self._h, buf._h, p, a.size)

    def copy(self, dst: Buffer, dst_offset: int, src: Buffer, src_offset: int, length: int) -> None:
        call("tb200_copy", self._h, dst._h, int(dst_offset), src._h, int(src_offset), int(length))

    def embed(self, out: Buffer, table: Weight, tokens) -> None:
        t = np.ascontiguousarray(tokens, dtype=np.uint32)
        call("tb200_embed", self._h, out._h, table._h, t.ctypes.data_as(_lib.U32P), t.size)

    def matmul(self, out: Buffer, w: Weight, x: Buffer) -> None:
        call("tb200_matmul", self._h, out._h, w._h, x._h)

    def add(self, x: Buffer, y: Buffer) -> None:
        call("tb200_add", self._h, x._h, y._h)

    def rmsnorm(self, x: Buffer, weight: Weight, eps: float) -> None:
        call("tb200_rmsnorm", self._h, x._h, weight._h, ctypes.c_float(eps))

    def rope(self, x: Buffer, table: Buffer, pos: int, n_heads: int, head_dim: int) -> None:
        call("tb200_rope", self._h, x._h, table._h, int(pos), int(n_heads), int(head_dim))

    def attention(self, out: Buffer, q: Buffer, k_cache: Buffer, v_cache: Buffer, pos: int, n_heads: int,
                  head_dim: int, n_kv_heads: int) -> None:
        call("tb200_attention", self._h, out._h, q._h, k_cache._h, v_cache._h, int(pos), int(n_heads),
             int(head_dim), int(n_kv_heads))

    def silu_mul(self, gate: Buffer, up: Buffer) -> None:
        call("tb200_silu_mul", self._h, gate._h, up._h)

    # ---- beyond the trait ---------------------------------------------------

    def argmax(self, logits: Buffer) -> int:
        """Greedy choice (model/sampler.rs:31-33) computed on the device."""
        out = ctypes.c_uint32()
        call("tb200_argmax", self._h, logits._h, ctypes.byref(out))
        return int(out.value)

    def attention_cache(self, out: Buffer, q: Buffer, cache: Weight, positions, n_heads: int) -> None:
        """Decode attention over a bf16 cache in the model path's layout
        (`cache` of shape [batch, 2, n_kv_heads, max_len, 128]): for each
        sequence b, the query q[b] (n_heads x 128, after QK-norm and RoPE) at
        positions[b] attends to cached positions 0..positions[b]
        (Device::attention, model/cpu.rs:113-149, one token per sequence)."""
        pos = np.ascontiguousarray(positions, dtype=np.uint64)
        call("tb200_attention_cache", self._h, out._h, q._h, cache._h, pos.ctypes.data_as(_lib.SZP), pos.size,
             int(n_heads))


__all__ = ["B200", "Buffer", "Weight", "Tensor", "DeviceError"]
