"""cs_softmax_noalloc: the one-shot entry point that allocates no device memory.

It serves callers whose own allocator owns the GPU's memory (serving engines,
frameworks with a caching allocator) and that therefore cannot let a library
call cudaMalloc. Its status word comes from a static device array instead of
the per-device buffer cs_softmax_batched allocates. These tests call it
through the C ABI twice in a row, on the same status slot, and compare each
result with cs_softmax_batched on the same input within the parity tests'
tolerance. The file is named to be collected last, and it also passes alone in
a fresh process.
"""
import ctypes

import numpy as np
import pytest
import torch

import causal_softmax as cs
from gpu_helpers import ABS_TOL, from_dev, sentinel_like, to_dev

pytestmark = pytest.mark.gpu

SLOTS = 64
ERR_ARG = -16


def _half(bits: np.ndarray) -> np.ndarray:
    return bits.view(np.float16).astype(np.float32)


def _batched(kernel, d_in, d_out, batch, rows, cols, pitch, row_offset, scale):
    rc = cs.lib().cs_softmax_batched(cs.kernel_id(kernel), d_in.data_ptr(), d_out.data_ptr(), batch,
                                     rows * pitch, rows, cols, pitch, row_offset, scale, None)
    assert rc == 0, cs.lib().cs_last_error_detail()


def _noalloc(kernel, d_in, d_out, batch, rows, cols, pitch, row_offset, scale, slot, want_status=True):
    word = ctypes.c_uint32(0xFFFFFFFF)
    rc = cs.lib().cs_softmax_noalloc(cs.kernel_id(kernel), d_in.data_ptr(), d_out.data_ptr(), batch,
                                     rows * pitch, rows, cols, pitch, row_offset, scale, slot,
                                     ctypes.byref(word) if want_status else None, None)
    return rc, word.value


@pytest.mark.parametrize("kernel,batch,rows,cols,row_offset,scale", [
    ("auto", 3, 700, 700, 0, 0.0883883),
    ("pipeline", 1, 4096, 4096, 0, 0.0883883),
    ("tma", 2, 96, 1037, 900, 1.0),
    ("online", 2, 300, 9000, 8000, 0.125),
    ("baseline", 4, 257, 257, 0, 0.5),
    ("warp", 8, 32, 32, 0, 1.0),
])
def test_two_calls_match_batched(kernel, batch, rows, cols, row_offset, scale):
    pitch = cs.padded_pitch(cols)
    slot = 5
    for call, seed in enumerate((11, 12)):
        x = cs.generate(2, seed, batch=batch, rows=rows, cols=cols, first_row=row_offset)
        d_in = to_dev(x)
        ref = sentinel_like(d_in)
        out = sentinel_like(d_in)
        _batched(kernel, d_in, ref, batch, rows, cols, pitch, row_offset, scale)
        rc, status = _noalloc(kernel, d_in, out, batch, rows, cols, pitch, row_offset, scale, slot)
        assert rc == 0, (call, cs.lib().cs_last_error_detail())
        assert status == 0, (call, status)
        torch.cuda.synchronize()
        a, b = from_dev(out), from_dev(ref)
        assert np.array_equal(a == 0, b == 0), call
        err = np.abs(_half(a) - _half(b))
        assert float(err.max()) <= ABS_TOL, (call, float(err.max()))


def test_without_status_and_each_slot_edge():
    rows = cols = 512
    pitch = cs.padded_pitch(cols)
    x = cs.generate(1, 3, batch=1, rows=rows, cols=cols)
    d_in = to_dev(x)
    ref = sentinel_like(d_in)
    _batched("auto", d_in, ref, 1, rows, cols, pitch, 0, 1.0)
    for slot in (0, SLOTS - 1):
        out = sentinel_like(d_in)
        rc, _ = _noalloc("auto", d_in, out, 1, rows, cols, pitch, 0, 1.0, slot, want_status=False)
        assert rc == 0, cs.lib().cs_last_error_detail()
        torch.cuda.synchronize()
        err = np.abs(_half(from_dev(out)) - _half(from_dev(ref)))
        assert float(err.max()) <= ABS_TOL


def test_rejects_slots_outside_the_static_array():
    rows = cols = 64
    pitch = cs.padded_pitch(cols)
    d_in = to_dev(cs.generate(1, 4, batch=1, rows=rows, cols=cols))
    out = sentinel_like(d_in)
    for slot in (SLOTS, -1, 1 << 30):
        rc, _ = _noalloc("auto", d_in, out, 1, rows, cols, pitch, 0, 1.0, slot)
        assert rc == ERR_ARG
        assert b"static status array holds 64 words" in cs.lib().cs_last_error_detail()
    torch.cuda.synchronize()
    assert np.all(from_dev(out) == 0xFB00)
