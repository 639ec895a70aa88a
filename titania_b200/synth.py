"""Seeded random-init Qwen3-shaped checkpoints in the Hugging Face layout.

The reference loads `config.json` + `model.safetensors` from a directory
(model/model.rs:40-77, model/config.rs:28-30, model/weights.rs:35-81) using
the tensor names of model/model.rs:48-72. Real Qwen3 weights are not
available offline, so benchmarks and parity runs use checkpoints written
here: linear and embedding weights ~N(0, 0.02) rounded to bf16
(round-to-nearest-even), every norm weight 1.0, tied embeddings.

Generation is deterministic for a given (config, seed): one numpy PCG64
stream per tensor, derived from the seed and the tensor's index.
"""

from __future__ import annotations

import hashlib
import json
import os
import struct

import numpy as np

# Qwen3-0.6B and Qwen3-4B architecture fields, as their config.json states them.
QWEN3_0_6B = dict(
    hidden_size=1024, intermediate_size=3072, num_hidden_layers=28, num_attention_heads=16,
    num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-06, rope_theta=1000000.0,
    vocab_size=151936, tie_word_embeddings=True,
)
QWEN3_4B = dict(
    hidden_size=2560, intermediate_size=9728, num_hidden_layers=36, num_attention_heads=32,
    num_key_value_heads=8, head_dim=128, rms_norm_eps=1e-06, rope_theta=1000000.0,
    vocab_size=151936, tie_word_embeddings=True,
)
# A two-layer model with the real head geometry, small enough for the CPU
# oracle to run in well under a second per token.
TINY = dict(
    hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
    num_key_value_heads=2, head_dim=128, rms_norm_eps=1e-06, rope_theta=1000000.0,
    vocab_size=1024, tie_word_embeddings=True,
)
# Two layers of Qwen3-0.6B (every matrix its real shape, lm_head included):
# the single-token kernels see the real per-CTA row counts at a fraction of
# the oracle's time.
QWEN3_0_6B_2L = dict(QWEN3_0_6B, num_hidden_layers=2)
# Two layers of Qwen3-4B (its widths: hidden 2560, FFN 9728, 32 query heads
# over 8 kv heads), for the single-token kernels' wide-input branches.
QWEN3_4B_2L = dict(QWEN3_4B, num_hidden_layers=2)
# Two layers with four query heads per kv head (Qwen3-4B's grouping) and a
# hidden size that gives every CTA more than eight residual rows.
WIDE_GQA4 = dict(
    hidden_size=1536, intermediate_size=2048, num_hidden_layers=2, num_attention_heads=16,
    num_key_value_heads=4, head_dim=128, rms_norm_eps=1e-06, rope_theta=1000000.0,
    vocab_size=4096, tie_word_embeddings=True,
)
CONFIGS = {"qwen3-0.6b": QWEN3_0_6B, "qwen3-4b": QWEN3_4B, "tiny": TINY, "qwen3-0.6b-2l": QWEN3_0_6B_2L,
           "qwen3-4b-2l": QWEN3_4B_2L, "wide-gqa4": WIDE_GQA4}


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Rounds f32 to bf16 (round to nearest, ties to even) and returns the bits."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    return ((u + rounding) >> 16).astype(np.uint16)


def tensor_list(c: dict) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) for every tensor, in the order of model/model.rs:48-72."""
    h, f, d = c["hidden_size"], c["intermediate_size"], c["head_dim"]
    q_dim, kv_dim = c["num_attention_heads"] * d, c["num_key_value_heads"] * d
    out = [("model.embed_tokens.weight", (c["vocab_size"], h), "normal")]
    for i in range(c["num_hidden_layers"]):
        p = f"model.layers.{i}"
        out += [
            (f"{p}.input_layernorm.weight", (h,), "ones"),
            (f"{p}.self_attn.q_proj.weight", (q_dim, h), "normal"),
            (f"{p}.self_attn.k_proj.weight", (kv_dim, h), "normal"),
            (f"{p}.self_attn.v_proj.weight", (kv_dim, h), "normal"),
            (f"{p}.self_attn.o_proj.weight", (h, q_dim), "normal"),
            (f"{p}.self_attn.q_norm.weight", (d,), "ones"),
            (f"{p}.self_attn.k_norm.weight", (d,), "ones"),
            (f"{p}.post_attention_layernorm.weight", (h,), "ones"),
            (f"{p}.mlp.gate_proj.weight", (f, h), "normal"),
            (f"{p}.mlp.up_proj.weight", (f, h), "normal"),
            (f"{p}.mlp.down_proj.weight", (h, f), "normal"),
        ]
    out.append(("model.norm.weight", (h,), "ones"))
    if not c.get("tie_word_embeddings", False):
        out.append(("lm_head.weight", (c["vocab_size"], h), "normal"))
    return out


def _chunks(shape, init, seed, index, std, buf, bits):
    """Yields the tensor's bf16 bytes in chunks, reusing the scratch arrays."""
    n = int(np.prod(shape))
    if init == "ones":
        yield np.full(n, 0x3F80, dtype=np.uint16).tobytes()
        return
    rng = np.random.Generator(np.random.PCG64([seed, index]))
    step = buf.size
    for s in range(0, n, step):
        k = min(step, n - s)
        v = buf[:k]
        rng.standard_normal(out=v, dtype=np.float32)
        v *= np.float32(std)
        u = v.view(np.uint32)
        b = bits[:k]
        np.right_shift(u, 16, out=b)
        np.bitwise_and(b, 1, out=b)
        b += np.uint32(0x7FFF)
        b += u
        b >>= 16
        yield b.astype(np.uint16).tobytes()


def write_model(dirpath: str, config: dict, seed: int = 0, std: float = 0.02) -> str:
    """Writes config.json and model.safetensors into `dirpath`; returns the
    sha256 of the safetensors file."""
    os.makedirs(dirpath, exist_ok=True)
    tensors = tensor_list(config)
    header, offset = {}, 0
    for name, shape, _ in tensors:
        nbytes = int(np.prod(shape)) * 2
        header[name] = {"dtype": "BF16", "shape": list(shape), "data_offsets": [offset, offset + nbytes]}
        offset += nbytes
    header["__metadata__"] = {"format": "pt", "generator": f"titania_b200.synth seed={seed} std={std}"}
    hbytes = json.dumps(header, separators=(",", ":")).encode()
    hbytes += b" " * ((-len(hbytes)) % 8)
    h = hashlib.sha256()
    tmp = os.path.join(dirpath, f"model.safetensors.{os.getpid()}.tmp")  # concurrent writers never share it
    with open(tmp, "wb") as fh:
        pre = struct.pack("<Q", len(hbytes)) + hbytes
        fh.write(pre)
        h.update(pre)
        buf = np.empty(1 << 22, dtype=np.float32)
        bits = np.empty(1 << 22, dtype=np.uint32)
        for index, (name, shape, init) in enumerate(tensors):
            for data in _chunks(shape, init, seed, index, std, buf, bits):
                fh.write(data)
                h.update(data)
    os.replace(tmp, os.path.join(dirpath, "model.safetensors"))
    cfg = dict(config)
    cfg["architectures"] = ["Qwen3ForCausalLM"]
    cfg["torch_dtype"] = "bfloat16"
    with open(os.path.join(dirpath, "config.json"), "w") as fh:
        json.dump(cfg, fh, indent=2)
    digest = h.hexdigest()
    with open(os.path.join(dirpath, "SHA256"), "w") as fh:
        fh.write(digest + "\n")
    return digest


def cached_model(name: str, seed: int = 0, root: str | None = None) -> str:
    """Returns a directory holding the seeded checkpoint `name`, writing it on
    first use."""
    root = root or os.environ.get("TITANIA_B200_MODELS") or os.path.join(
        os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "_build", "models")
    d = os.path.join(root, f"{name}-seed{seed}")
    if not (os.path.exists(os.path.join(d, "SHA256")) and os.path.exists(os.path.join(d, "model.safetensors"))):
        write_model(d, CONFIGS[name], seed)
    return d


def prompt_tokens(n: int, vocab: int, seed: int = 1) -> list[int]:
    """`n` token ids uniform in [0, vocab) from a seeded stream separate from
    the weights'."""
    rng = np.random.Generator(np.random.PCG64([seed, 0xA11CE]))
    return [int(t) for t in rng.integers(0, vocab, size=n)]
