"""dfl_verify_qmm_w4g64_noalloc (fixed device scratch, no workspace) against
dfl_verify_qmm_w4g64 (caller workspace), both called through the C ABI.

Calls in a row on one stream share the library's scratch array.  Both entry
points run the same kernel with the same stream-K split and reduce split-K
partials in a fixed order, so each no-allocation result must equal the
workspace entry point's bit for bit; the first shape is also checked against
the oracle within the qmm tests' tolerance (|y - ref| <= 1e-2 + 2e-2 |ref|).
The shapes split K across CTAs at both tile heights (16 and 32 rows), so the
partial slots of both layouts are written, consumed and cleared in the
shared array, and the 16-row shape runs again after the 32-row one.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from conftest import bf16_to_np_bits, to_dev_bf16, to_dev_u32
from oracle import bf16 as obf16
from oracle import qmm as oqmm

pytestmark = pytest.mark.gpu

ATOL = 1e-2
RTOL = 2e-2


def _inputs(dev, seed, m, k, n):
    rng = np.random.default_rng(seed)
    w_q, s, b = oqmm.synth_weights(rng, n, k)
    x = oqmm.synth_x(rng, m, k)
    return (to_dev_bf16(x, dev), to_dev_u32(w_q, dev), to_dev_bf16(s, dev), to_dev_bf16(b, dev))


def _with_workspace(lib, dev, x, w, s, b, m, k, n, stream):
    import torch

    st = ctypes.c_int(-1)
    nbytes = lib.dfl_verify_qmm_workspace_bytes(m, k, n, ctypes.byref(st))
    assert st.value == 0
    ws = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    rc = lib.dfl_verify_qmm_w4g64(x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(),
                                  y.data_ptr(), ws.data_ptr(), nbytes, m, k, n, stream)
    assert rc == 0, lib.dfl_status_string(rc)
    return y


def _no_alloc(lib, dev, x, w, s, b, m, k, n, stream):
    import torch

    y = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    rc = lib.dfl_verify_qmm_w4g64_noalloc(x.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(),
                                          y.data_ptr(), m, k, n, stream)
    assert rc == 0, lib.dfl_status_string(rc)
    return y


def _assert_equal(y, ref, what):
    a, b = bf16_to_np_bits(y), bf16_to_np_bits(ref)
    assert np.array_equal(a, b), f"{what}: {int((a != b).sum())} of {a.size} outputs differ"


def test_no_alloc_matches_workspace_entry_two_calls_in_a_row(pkg, dev):
    import torch

    lib = pkg._lib.load()
    stream = torch.cuda.current_stream(dev).cuda_stream
    # split-K at 16 rows; split-K at 32 rows; 32 rows with an N tail
    shapes = [(16, 5120, 6144), (32, 5120, 6144), (32, 1024, 1000)]
    inputs = [_inputs(dev, 100 + i, *shp) for i, shp in enumerate(shapes)]
    refs = [_with_workspace(lib, dev, *inp, *shp, stream) for inp, shp in zip(inputs, shapes)]
    outs = [_no_alloc(lib, dev, *inp, *shp, stream) for inp, shp in zip(inputs, shapes)]
    # and the 16-row shape again, after the 32-row calls used the same scratch
    again = _no_alloc(lib, dev, *inputs[0], *shapes[0], stream)
    torch.cuda.synchronize(dev)
    for (m, k, n), y, ref in zip(shapes, outs, refs):
        _assert_equal(y, ref, f"{m}x{k}x{n}")
    _assert_equal(again, refs[0], "repeat of 16x5120x6144")
    # the first shape against the oracle
    rng = np.random.default_rng(100)
    w_q, s, b = oqmm.synth_weights(rng, 6144, 5120)
    x = oqmm.synth_x(rng, 16, 5120)
    y_ref = oqmm.qmm(x, w_q, s, b)
    _assert_close_np(outs[0], y_ref, "oracle 16x5120x6144")
    err = ctypes.c_int(-1)
    assert lib.dfl_get_device_error(ctypes.byref(err)) == 0 and err.value == 0


def _assert_close_np(y, ref_bits, what):
    yv = obf16.to_f32(bf16_to_np_bits(y)).astype(np.float64)
    rv = obf16.to_f32(np.asarray(ref_bits)).astype(np.float64)
    err = np.abs(yv - rv)
    bad = err > ATOL + RTOL * np.abs(rv)
    assert not bad.any(), f"{what}: {int(bad.sum())} outside tolerance, max err {err.max():.4g}"


def test_no_alloc_rejects_bad_arguments(pkg, dev):
    lib = pkg._lib.load()
    assert lib.dfl_verify_qmm_w4g64_noalloc(None, None, None, None, None, 16, 100, 64, None) == 2
    assert lib.dfl_verify_qmm_w4g64_noalloc(None, None, None, None, None, 16, 128, 64, None) == 1
