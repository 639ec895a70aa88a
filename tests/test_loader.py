"""The safetensors fast path (tb200_upload_safetensors, tb200_safetensors_entry)
against model/weights.rs:35-81 read as Python does it.

CPU: the library's header parser against `json` on the same files (the
checkpoint the other tests use and hand-written headers with every JSON form a
header may hold), and its errors. GPU: the bytes on the device are the file's,
for tensors spanning several staging pieces and at file offsets that are not
16-byte aligned, with 1..16 host threads; a model loaded this way computes
bit-identical logits to one loaded tensor by tensor.
"""

import json
import os
import struct

import numpy as np
import pytest

from titania_b200 import _lib
from titania_b200.device import safetensors_entry

PIECE = 8 << 20  # the loader's staging piece (bytes)


def write_raw(path, header: bytes, data: bytes = b"", pad: int = 0):
    """A file with an 8-byte header length, `header` (+ `pad` spaces) and `data`."""
    h = header + b" " * pad
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(h)) + h + data)
    return str(path)


def write_tensors(path, tensors, metadata=None):
    """tensors: list of (name, dtype, shape, raw bytes), laid out back to back
    in the given order with no alignment padding."""
    header, blobs, off = {}, [], 0
    if metadata is not None:
        header["__metadata__"] = metadata
    for name, dtype, shape, raw in tensors:
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    return write_raw(path, json.dumps(header).encode(), b"".join(blobs))


def bf16_bits(rng, shape):
    return rng.integers(0, 1 << 16, size=shape, dtype=np.uint16) & np.uint16(0x7F7F)  # finite values


# ---- CPU: the header parser --------------------------------------------------

def test_entries_match_json(tiny_model_dir):
    f = os.path.join(tiny_model_dir, "model.safetensors")
    with open(f, "rb") as fh:
        n = struct.unpack("<Q", fh.read(8))[0]
        header = json.loads(fh.read(n))
    names = [k for k in header if k != "__metadata__"]
    assert len(names) > 10
    for name in names:
        e = header[name]
        dtype, shape, off, nbytes = safetensors_entry(f, name)
        assert (dtype, shape) == (e["dtype"], e["shape"]), name
        assert off == 8 + n + e["data_offsets"][0], name
        assert nbytes == e["data_offsets"][1] - e["data_offsets"][0], name
    assert safetensors_entry(f, "model.layers.99.mlp.up_proj.weight") is None


def test_header_forms(tmp_path):
    """Field order, unknown fields of every JSON type, escapes, metadata
    anywhere, whitespace and the spaces safetensors pads the header with."""
    header = (b'{\n  "a\\"b\\\\c" : {"shape": [2, 3], "extra": {"x": [1, -2.5e+3, true, false, null, "s"]},'
              b' "data_offsets": [0, 12], "dtype": "BF16"},\r\n'
              b' "__metadata__": {"format": "pt", "nested": {"k": [0.5, {}]}},\t'
              b'"caf\\u00e9\\ud83d\\ude00/\\n" :{"dtype":"F32","data_offsets":[12,20],"shape":[2]},'
              b'"scalar": {"dtype": "BF16", "shape": [], "data_offsets": [20, 22]}}')
    f = write_raw(tmp_path / "forms.safetensors", header, bytes(22), pad=5)
    start = 8 + len(header) + 5
    assert safetensors_entry(f, 'a"b\\c') == ("BF16", [2, 3], start, 12)
    assert safetensors_entry(f, "café\U0001F600/\n") == ("F32", [2], start + 12, 8)
    assert safetensors_entry(f, "scalar") == ("BF16", [], start + 20, 2)
    assert safetensors_entry(f, "__metadata__") is None
    assert safetensors_entry(f, "a") is None


def test_empty_header_object(tmp_path):
    f = write_raw(tmp_path / "empty.safetensors", b"{}", pad=6)
    assert safetensors_entry(f, "x") is None


@pytest.mark.parametrize("header", [
    b"[]",                                                              # not an object
    b'{"t": {"shape": [1], "data_offsets": [0, 2]}}',                    # missing dtype
    b'{"t": {"dtype": "BF16", "data_offsets": [0, 2]}}',                 # missing shape
    b'{"t": {"dtype": "BF16", "shape": [1]}}',                           # missing data_offsets
    b'{"t": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2, 4]}}',  # three offsets
    b'{"t": {"dtype": "BF16", "shape": [-1], "data_offsets": [0, 2]}}',  # negative dimension
    b'{"t": {"dtype": "BF16", "shape": [1.0], "data_offsets": [0, 2]}}',  # fractional dimension
    b'{"t": {"dtype": "BF16", "shape": [01], "data_offsets": [0, 2]}}',  # leading zero
    b'{"t": {"dtype": "BF16", "shape": [99999999999999999999], "data_offsets": [0, 2]}}',  # > u64
    b'{"t": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}} x',  # bytes after the object
    b'{"t": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}',    # unterminated object
    b'{"t": {"dtype": "BF16, "shape": [1], "data_offsets": [0, 2]}}',    # broken string
    b'{"t\\ud800": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}}',  # unpaired surrogate
    b'{"t": {"dtype": "BF16", "shape": [1], "data_offsets": [0, 2]}, "u": tru}',  # bad literal
])
def test_header_errors(tmp_path, header):
    f = write_raw(tmp_path / "bad.safetensors", header, bytes(4))
    with pytest.raises(_lib.DeviceError) as e:
        safetensors_entry(f, "t")
    assert e.value.code == _lib.TB200_ERR_FORMAT, str(e.value)


def test_header_longer_than_file(tmp_path):
    f = tmp_path / "short.safetensors"
    f.write_bytes(struct.pack("<Q", 1000) + b"{}")
    with pytest.raises(_lib.DeviceError) as e:
        safetensors_entry(str(f), "t")
    assert e.value.code == _lib.TB200_ERR_FORMAT and "header length 1000" in str(e.value)


def test_unreadable_files(tmp_path):
    with pytest.raises(_lib.DeviceError) as e:
        safetensors_entry(str(tmp_path / "nonexistent.safetensors"), "t")
    assert e.value.code == _lib.TB200_ERR_IO
    f = tmp_path / "tiny.safetensors"
    f.write_bytes(b"\x02\x00\x00")  # shorter than the length field: read_exact fails
    with pytest.raises(_lib.DeviceError) as e:
        safetensors_entry(str(f), "t")
    assert e.value.code == _lib.TB200_ERR_IO and "end of file" in str(e.value)


class _StubDevice:
    """Answers upload_safetensors from a set of present names (no GPU)."""

    def __init__(self, present):
        self.present, self.asked = set(present), None

    def upload_safetensors(self, path, names, threads=0):
        self.asked = list(names)
        return [f"w:{n}" if n in self.present else None for n in names]


def test_upload_checkpoint_names_and_optional_tensors():
    """Model::load's tensor list (model/model.rs:46-72): q_norm / k_norm are
    optional, everything else is required; a tied model reads no lm_head."""
    from titania_b200.model import Config, tensor_names, upload_checkpoint

    c = Config(**dict(synth_cfg(), tie_word_embeddings=True))
    names = [n for n, _ in tensor_names(c)]
    optional = {n for n, req in tensor_names(c) if not req}
    assert "lm_head.weight" not in names
    assert optional == {f"model.layers.{i}.self_attn.{k}_norm.weight" for i in range(2) for k in "qk"}
    dev = _StubDevice(set(names) - optional)
    up = upload_checkpoint(dev, c, "unused")
    assert dev.asked == names and set(up) == set(names) - optional
    untied = Config(**dict(synth_cfg(), tie_word_embeddings=False))
    assert "lm_head.weight" in [n for n, _ in tensor_names(untied)]


def test_upload_checkpoint_missing_required_tensor():
    from titania_b200.model import Config, tensor_names, upload_checkpoint

    c = Config(**dict(synth_cfg(), tie_word_embeddings=True))
    names = [n for n, _ in tensor_names(c)]
    with pytest.raises(KeyError, match="missing tensor 'model.layers.1.mlp.down_proj.weight'"):
        upload_checkpoint(_StubDevice(set(names) - {"model.layers.1.mlp.down_proj.weight"}), c, "unused")


def synth_cfg():
    from titania_b200 import synth

    return dict(synth.TINY, num_hidden_layers=2)


# ---- GPU: the bytes on the device ------------------------------------------

def device_bits(dev, w):
    """The bf16 bits of a 2-D weight, read back exactly through Device::embed
    (bf16 -> f32 is a shift)."""
    import titania_b200 as tb

    rows, cols = w.shape
    out = dev.alloc(rows * cols)
    dev.embed(out, w, np.arange(rows, dtype=np.uint32))
    return (dev.read(out).view(np.uint32) >> 16).astype(np.uint16).reshape(rows, cols)


@pytest.mark.gpu
@pytest.mark.parametrize("threads", [0, 1, 3, 16])
def test_pieces_and_unaligned_offsets(b200, tmp_path, threads):
    rng = np.random.default_rng(5)
    odd = bf16_bits(rng, (3, 5))          # 30 bytes: everything after it starts off 16-byte alignment
    big = bf16_bits(rng, (4200, 2048))    # 17.2 MB: three staging pieces
    mid = bf16_bits(rng, (7, 9))
    f = write_tensors(tmp_path / "t.safetensors", [
        ("odd", "BF16", odd.shape, odd.tobytes()),
        ("skip", "F32", (3,), np.arange(3, dtype=np.float32).tobytes()),
        ("big", "BF16", big.shape, big.tobytes()),
        ("empty", "BF16", (0, 8), b""),
        ("mid", "BF16", mid.shape, mid.tobytes()),
    ], metadata={"format": "pt"})
    assert big.nbytes > PIECE and safetensors_entry(f, "big")[2] % 16 != 0
    ws = b200.upload_safetensors(f, ["big", "nope", "odd", "empty", "mid"], threads=threads)
    assert ws[1] is None
    assert ws[3].shape == [0, 8]
    for w, ref in ((ws[0], big), (ws[2], odd), (ws[4], mid)):
        assert w.shape == list(ref.shape)
        np.testing.assert_array_equal(device_bits(b200, w), ref)


@pytest.mark.gpu
def test_norm_vectors_match_per_tensor_upload(b200, tiny_model_dir):
    """1-D tensors (norm weights): rmsnorm with the fast-path weight equals,
    bit for bit, rmsnorm with the same tensor uploaded by Device::upload."""
    from titania_b200.model import Weights

    f = os.path.join(tiny_model_dir, "model.safetensors")
    w = Weights.open(f)
    names = [n for n, e in w.entries.items() if len(e["shape"]) == 1]
    assert names
    fast = b200.upload_safetensors(f, names)
    rng = np.random.default_rng(3)
    for name, wf in zip(names, fast):
        ws = b200.upload(w.read(name))
        dim = wf.shape[0]
        x = rng.standard_normal(4 * dim).astype(np.float32)
        a, b = b200.alloc(x.size), b200.alloc(x.size)
        b200.write(a, x)
        b200.write(b, x)
        b200.rmsnorm(a, wf, 1e-6)
        b200.rmsnorm(b, ws, 1e-6)
        np.testing.assert_array_equal(b200.read(a), b200.read(b), err_msg=name)


@pytest.mark.gpu
def test_matrices_match_file(b200, tiny_model_dir):
    from titania_b200.model import Weights

    f = os.path.join(tiny_model_dir, "model.safetensors")
    w = Weights.open(f)
    names = [n for n, e in w.entries.items() if len(e["shape"]) == 2]
    for name, wf in zip(names, b200.upload_safetensors(f, names, threads=4)):
        np.testing.assert_array_equal(device_bits(b200, wf), w.read(name).data.reshape(wf.shape), err_msg=name)


@pytest.mark.gpu
def test_upload_errors(b200, tmp_path):
    rng = np.random.default_rng(1)
    ok = bf16_bits(rng, (4, 4))
    f = write_tensors(tmp_path / "e.safetensors", [("ok", "BF16", ok.shape, ok.tobytes()),
                                                   ("f", "F32", (2,), bytes(8))])
    with pytest.raises(_lib.DeviceError) as e:  # Weights::read's dtype check
        b200.upload_safetensors(f, ["ok", "f"])
    assert e.value.code == _lib.TB200_ERR_FORMAT and "tensor 'f' is F32, expected BF16" in str(e.value)
    bad = write_raw(tmp_path / "o.safetensors",  # offsets past the end of the data
                    b'{"t": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 8]}}', bytes(6))
    with pytest.raises(_lib.DeviceError) as e:
        b200.upload_safetensors(bad, ["t"])
    assert e.value.code == _lib.TB200_ERR_FORMAT and "outside" in str(e.value)
    size = write_raw(tmp_path / "s.safetensors",  # 6 bytes for a shape of 4 elements
                     b'{"t": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 6]}}', bytes(6))
    with pytest.raises(_lib.DeviceError) as e:
        b200.upload_safetensors(size, ["t"])
    assert e.value.code == _lib.TB200_ERR_FORMAT
    with pytest.raises(_lib.DeviceError) as e:
        b200.upload_safetensors(str(tmp_path / "missing.safetensors"), ["t"])
    assert e.value.code == _lib.TB200_ERR_IO
    with pytest.raises(_lib.DeviceError) as e:
        b200.upload_safetensors(f, ["ok"], threads=17)
    assert e.value.code == _lib.TB200_ERR_ARG
    # the device is still usable and the good tensor loads
    (w,) = b200.upload_safetensors(f, ["ok"])
    np.testing.assert_array_equal(device_bits(b200, w), ok)


@pytest.mark.gpu
def test_model_load_direct_equals_per_tensor(b200, tiny_model_dir):
    import titania_b200 as tb
    from titania_b200 import synth
    from titania_b200.model import Config, Weights, load_weights, upload_checkpoint

    c = Config.load(os.path.join(tiny_model_dir, "config.json"))
    f = os.path.join(tiny_model_dir, "model.safetensors")
    fast = tb.Model(c, b200, upload_checkpoint(b200, c, f))
    slow = tb.Model(c, b200, load_weights(b200, c, Weights.open(f)))
    prompt = synth.prompt_tokens(6, synth.TINY["vocab_size"], seed=4)
    la = fast.forward(fast.state(16), prompt, 0)
    lb = slow.forward(slow.state(16), prompt, 0)
    np.testing.assert_array_equal(la, lb)


# ---- windows: a tensor-parallel rank's share -------------------------------

@pytest.mark.gpu
@pytest.mark.parametrize("world", [1, 2])
def test_windows_match_the_shard_rule(b200, tiny_model_dir, world):
    """Every rank's windows hold exactly the bytes titania_b200.tp.shard_tensor
    cuts from the file: row blocks (q/k/v/gate/up), column blocks (o/down),
    and whole tensors (norms, embedding)."""
    from titania_b200.model import Config, Weights, tensor_names
    from titania_b200.tp import shard_tensor, shard_window

    c = Config.load(os.path.join(tiny_model_dir, "config.json"))
    f = os.path.join(tiny_model_dir, "model.safetensors")
    w = Weights.open(f)
    names = [n for n, _ in tensor_names(c) if w.contains(n)]
    for rank in range(world):
        wins = [shard_window(c, n, w.entries[n]["shape"], rank, world) for n in names]
        assert any(x is not None and x[3] < w.entries[n]["shape"][1] for x, n in zip(wins, names)) == (world > 1)
        for name, wt in zip(names, b200.upload_safetensors(f, names, windows=wins)):
            t = w.read(name)
            shape, data = shard_tensor(c, name, t.shape, t.data, rank, world)
            assert wt.shape == shape, name
            if len(shape) == 2:
                np.testing.assert_array_equal(device_bits(b200, wt), data.reshape(shape), err_msg=f"{name} rank {rank}")


@pytest.mark.gpu
@pytest.mark.parametrize("threads", [1, 4])
def test_windows_across_staging_pieces(b200, tmp_path, threads):
    rng = np.random.default_rng(9)
    head = bf16_bits(rng, (1, 7))                 # 14 bytes: the matrix starts off 16-byte alignment
    m = bf16_bits(rng, (1200, 4000))              # 9.6 MB: more than one staging piece
    f = write_tensors(tmp_path / "w.safetensors", [("head", "BF16", head.shape, head.tobytes()),
                                                   ("m", "BF16", m.shape, m.tobytes())])
    cases = [(5, 1190, 1000, 2000),   # column window, rows in two pieces
             (3, 1100, 0, 4000),      # whole rows: one run
             (0, 1200, 3999, 1),      # the last column
             (1199, 1, 0, 1),         # one element
             (0, 0, 0, 0)]            # whole
    ws = b200.upload_safetensors(f, ["m"] * len(cases), threads=threads,
                                 windows=[None if x == (0, 0, 0, 0) else x for x in cases])
    for (r0, nr, c0, nc), wt in zip(cases, ws):
        ref = m if nr == 0 else m[r0:r0 + nr, c0:c0 + nc]
        np.testing.assert_array_equal(device_bits(b200, wt), ref, err_msg=str((r0, nr, c0, nc)))


@pytest.mark.gpu
def test_window_errors(b200, tmp_path):
    rng = np.random.default_rng(2)
    m = bf16_bits(rng, (6, 10))
    v = bf16_bits(rng, (10,))
    f = write_tensors(tmp_path / "we.safetensors", [("m", "BF16", m.shape, m.tobytes()),
                                                    ("v", "BF16", v.shape, v.tobytes())])
    for names, wins, what in ((["m"], [(4, 3, 0, 10)], "outside"), (["m"], [(0, 6, 8, 3)], "outside"),
                              (["m"], [(0, 0, 0, 5)], "empty window"), (["v"], [(0, 1, 0, 5)], "needs a matrix")):
        with pytest.raises(_lib.DeviceError) as e:
            b200.upload_safetensors(f, names, windows=wins)
        assert e.value.code == _lib.TB200_ERR_ARG and what in str(e.value), str(e.value)
    with pytest.raises(ValueError):
        b200.upload_safetensors(f, ["m", "v"], windows=[None])
    (wv,) = b200.upload_safetensors(f, ["v"], windows=[None])  # a vector whole is fine
    assert wv.shape == [10]


def test_shard_window_agrees_with_shard_tensor(tiny_model_dir):
    """The window rule and the numpy slicing are one rule (CPU)."""
    from titania_b200.model import Config, Weights, tensor_names
    from titania_b200.tp import shard_tensor, shard_window

    c = Config.load(os.path.join(tiny_model_dir, "config.json"))
    w = Weights.open(os.path.join(tiny_model_dir, "model.safetensors"))
    for world in (1, 2):
        for rank in range(world):
            for name, _ in tensor_names(c):
                if not w.contains(name):
                    continue
                t = w.read(name)
                shape, data = shard_tensor(c, name, t.shape, t.data, rank, world)
                win = shard_window(c, name, t.shape, rank, world)
                full = t.data.reshape(t.shape)
                if win is None:
                    assert shape == t.shape
                else:
                    r0, nr, c0, nc = win
                    np.testing.assert_array_equal(full[r0:r0 + nr, c0:c0 + nc].reshape(-1), data)
