"""tb200_argmax_noalloc against tb200_argmax, through the C ABI.

The no-allocation entry point exists for callers that cannot allocate
device memory — a caller whose GPU memory belongs to another allocator, or
one that keeps cudaMalloc/cudaFree out of its per-token loop because those
calls can synchronize the device. It must choose exactly the token the
existing entry point chooses, on consecutive calls that reuse its static
scratch, and refuse inputs larger than that scratch can serve. Collected
last so that a failure here stops a run only after every other test ran."""

import ctypes

import numpy as np
import pytest

import titania_b200 as tb
from titania_b200 import _lib

pytestmark = pytest.mark.gpu

MAX_LOGITS = 4096 * 2048


def argmax_noalloc(torch, logits_ptr, n, out_ptr):
    stream = torch.cuda.current_stream().cuda_stream
    rc = _lib.lib().tb200_argmax_noalloc(ctypes.c_void_p(logits_ptr), n, ctypes.c_void_p(out_ptr),
                                         ctypes.c_void_p(stream))
    _lib.check(rc)


def test_noalloc_argmax_matches_argmax_on_consecutive_calls():
    torch = pytest.importorskip("torch")
    dev = tb.B200(0)
    rng = np.random.default_rng(7)
    cases = []
    for n, tie in ((151936, True), (151936, False), (5000, True)):
        x = rng.standard_normal(n).astype(np.float32)
        if tie:  # equal maxima: both entry points take the lowest index
            x[n // 3] = x[2 * n // 3] = np.float32(9.5)
        cases.append(x)
    # the maximum in the last, partial tile (151936 is not a multiple of the tile)
    last = rng.standard_normal(151936).astype(np.float32)
    last[-1] = np.float32(12.0)
    cases.append(last)
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    for x in cases:  # consecutive calls share and reuse the scratch
        logits = torch.from_numpy(x).to("cuda")
        argmax_noalloc(torch, logits.data_ptr(), logits.numel(), out.data_ptr())
        torch.cuda.synchronize()
        buf = dev.alloc(x.size)
        dev.write(buf, x)
        got = int(out.item())
        assert got == dev.argmax(buf)
        assert got == int(np.argmax(x))  # numpy: the first index of the maximum


def test_noalloc_argmax_rejects_inputs_beyond_its_scratch():
    torch = pytest.importorskip("torch")
    logits = torch.zeros(16, dtype=torch.float32, device="cuda")
    out = torch.zeros(1, dtype=torch.int32, device="cuda")
    # the length is checked before anything reads the logits
    with pytest.raises(tb.DeviceError, match="exceed the maximum"):
        argmax_noalloc(torch, logits.data_ptr(), MAX_LOGITS + 1, out.data_ptr())
    with pytest.raises(tb.DeviceError, match="no logits"):
        argmax_noalloc(torch, logits.data_ptr(), 0, out.data_ptr())
