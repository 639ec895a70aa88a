"""Loads libtitania_b200.so and declares the C ABI of include/titania_b200.h.

There is no fallback: if the library is missing or cannot be loaded, every
use raises. Build it with `python -m titania_b200.build`.
"""

from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "libtitania_b200.so")

TB200_OK, TB200_ERR_ARG, TB200_ERR_CUDA, TB200_ERR_TIMEOUT, TB200_ERR_IO, TB200_ERR_FORMAT = 0, 1, 2, 3, 4, 5


class DeviceError(RuntimeError):
    """A nonzero status from the library: the reference would have panicked
    (TB200_ERR_ARG), or CUDA / a kernel-side wait failed."""

    def __init__(self, code: int, message: str):
        super().__init__(message)
        self.code = code


class Window(ctypes.Structure):
    """tb200_window: rows [row0, row0 + rows) x columns [col0, col0 + cols)."""

    _fields_ = [("row0", ctypes.c_size_t), ("rows", ctypes.c_size_t), ("col0", ctypes.c_size_t),
                ("cols", ctypes.c_size_t)]


class Config(ctypes.Structure):
    _fields_ = [
        ("hidden_size", ctypes.c_size_t),
        ("intermediate_size", ctypes.c_size_t),
        ("num_hidden_layers", ctypes.c_size_t),
        ("num_attention_heads", ctypes.c_size_t),
        ("num_key_value_heads", ctypes.c_size_t),
        ("head_dim", ctypes.c_size_t),
        ("rms_norm_eps", ctypes.c_float),
        ("rope_theta", ctypes.c_float),
        ("vocab_size", ctypes.c_size_t),
        ("tie_word_embeddings", ctypes.c_int),
    ]


P = ctypes.c_void_p
SZ = ctypes.c_size_t
PP = ctypes.POINTER(ctypes.c_void_p)
F32P = ctypes.POINTER(ctypes.c_float)
U16P = ctypes.POINTER(ctypes.c_uint16)
U32P = ctypes.POINTER(ctypes.c_uint32)
SZP = ctypes.POINTER(ctypes.c_size_t)

# name: (restype, argtypes); every int-returning function is a status.
SIGNATURES = {
    "tb200_last_error": (ctypes.c_char_p, []),
    "tb200_device_open": (ctypes.c_int, [ctypes.c_int, PP]),
    "tb200_device_close": (ctypes.c_int, [P]),
    "tb200_sync": (ctypes.c_int, [P]),
    "tb200_device_stream": (ctypes.c_void_p, [P]),
    "tb200_device_sms": (ctypes.c_int, [P]),
    "tb200_rope_table": (ctypes.c_int, [SZ, SZ, ctypes.c_float, F32P]),
    "tb200_upload": (ctypes.c_int, [P, U16P, SZP, SZ, PP]),
    "tb200_upload_safetensors": (ctypes.c_int, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p), SZ, ctypes.c_int,
                                                PP]),
    "tb200_weight_shape": (ctypes.c_int, [P, SZP, SZ, SZP]),
    "tb200_upload_safetensors_windows": (ctypes.c_int, [P, ctypes.c_char_p, ctypes.POINTER(ctypes.c_char_p),
                                                        ctypes.POINTER(Window), SZ, ctypes.c_int, PP]),
    "tb200_safetensors_entry": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int),
                                               ctypes.c_char_p, SZ, SZP, SZ, SZP, ctypes.POINTER(ctypes.c_uint64),
                                               ctypes.POINTER(ctypes.c_uint64)]),
    "tb200_alloc": (ctypes.c_int, [P, SZ, PP]),
    "tb200_resize": (ctypes.c_int, [P, P, SZ]),
    "tb200_buffer_len": (ctypes.c_size_t, [P]),
    "tb200_read": (ctypes.c_int, [P, P, F32P, SZ]),
    "tb200_write": (ctypes.c_int, [P, P, F32P, SZ]),
    "tb200_copy": (ctypes.c_int, [P, P, SZ, P, SZ, SZ]),
    "tb200_embed": (ctypes.c_int, [P, P, P, U32P, SZ]),
    "tb200_matmul": (ctypes.c_int, [P, P, P, P]),
    "tb200_add": (ctypes.c_int, [P, P, P]),
    "tb200_rmsnorm": (ctypes.c_int, [P, P, P, ctypes.c_float]),
    "tb200_rope": (ctypes.c_int, [P, P, P, SZ, SZ, SZ]),
    "tb200_attention": (ctypes.c_int, [P, P, P, P, P, SZ, SZ, SZ, SZ]),
    "tb200_attention_cache": (ctypes.c_int, [P, P, P, P, SZP, SZ, SZ]),
    "tb200_silu_mul": (ctypes.c_int, [P, P, P]),
    "tb200_free_buffer": (ctypes.c_int, [P, P]),
    "tb200_free_weight": (ctypes.c_int, [P, P]),
    "tb200_argmax": (ctypes.c_int, [P, P, U32P]),
    "tb200_argmax_noalloc": (ctypes.c_int, [P, SZ, P, P]),
    "tb200_sampler_new": (ctypes.c_int, [P, SZ, SZ, ctypes.c_float, SZ, ctypes.c_float,
                                         ctypes.POINTER(ctypes.c_uint64), PP]),
    "tb200_sampler_free": (ctypes.c_int, [P]),
    "tb200_sample": (ctypes.c_int, [P, P, U32P]),
    "tb200_sample_enqueue": (ctypes.c_int, [P, P]),
    "tb200_sampler_state": (ctypes.c_int, [P, ctypes.POINTER(ctypes.c_uint64)]),
    "tb200_model_create": (ctypes.c_int, [P, ctypes.POINTER(Config), PP]),
    "tb200_model_bind": (ctypes.c_int, [P, ctypes.c_char_p, P]),
    "tb200_model_finalize": (ctypes.c_int, [P]),
    "tb200_model_free": (ctypes.c_int, [P]),
    "tb200_state_new": (ctypes.c_int, [P, SZ, ctypes.c_int, PP]),
    "tb200_state_free": (ctypes.c_int, [P]),
    "tb200_forward": (ctypes.c_int, [P, P, U32P, SZ, SZ, F32P, U32P]),
    "tb200_batch_state_new": (ctypes.c_int, [P, SZ, SZ, ctypes.c_int, PP]),
    "tb200_tp_unique_id": (ctypes.c_int, [ctypes.c_char_p, SZ]),
    "tb200_tp_init": (ctypes.c_int, [P, ctypes.c_int, ctypes.c_int, ctypes.c_char_p, SZ, PP]),
    "tb200_tp_free": (ctypes.c_int, [P]),
    "tb200_tp_rank": (ctypes.c_int, [P]),
    "tb200_tp_world": (ctypes.c_int, [P]),
    "tb200_tp_allreduce": (ctypes.c_int, [P, P]),
    "tb200_model_set_tp": (ctypes.c_int, [P, P]),
    "tb200_model_tp_peer_exchange": (ctypes.c_int, [P]),
    "tb200_state_seqs": (SZ, [P]),
    "tb200_forward_seq": (ctypes.c_int, [P, P, SZ, U32P, SZ, SZ, F32P, U32P]),
    "tb200_forward_batch": (ctypes.c_int, [P, P, U32P, SZP, F32P, U32P]),
    "tb200_generate_batch": (ctypes.c_int, [P, P, U32P, SZP, SZ, U32P]),
    "tb200_decode_batch_enqueue": (ctypes.c_int, [P, P, U32P, SZP, SZ]),
    "tb200_batch_read_kv": (ctypes.c_int, [P, SZ, SZ, ctypes.c_int, SZ, F32P]),
    "tb200_generate": (ctypes.c_int, [P, P, ctypes.c_uint32, SZ, SZ, U32P]),
    "tb200_decode_persistent": (ctypes.c_int, [P, P, ctypes.c_uint32, SZ, SZ, U32P, F32P]),
    "tb200_decode_enqueue": (ctypes.c_int, [P, P, ctypes.c_uint32, SZ, SZ]),
    "tb200_state_set_decode": (ctypes.c_int, [P, ctypes.c_int]),
    "tb200_state_decode": (ctypes.c_int, [P]),
    "tb200_enqueue_op": (ctypes.c_int, [P, P, ctypes.c_int, SZ]),
    "tb200_trace_start": (ctypes.c_int, [P, SZ]),
    "tb200_trace_stop": (ctypes.c_int, [P, P, SZ, SZP]),
    "tb200_state_read": (ctypes.c_int, [P, ctypes.c_int, F32P, SZ]),
    "tb200_state_write": (ctypes.c_int, [P, ctypes.c_int, F32P, SZ]),
    "tb200_state_set_position": (ctypes.c_int, [P, ctypes.c_uint32, SZ]),
    "tb200_state_read_kv": (ctypes.c_int, [P, SZ, ctypes.c_int, SZ, F32P]),
}

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded library, with every entry point declared."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m titania_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(rc: int) -> None:
    if rc != TB200_OK:
        raise DeviceError(rc, lib().tb200_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib(), name)(*args))
