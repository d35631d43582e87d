"""The entry point that allocates nothing (qs_argmax_rows_static).

It exists for callers that cannot call cudaMalloc when they sample: code
running inside a memory pool or allocator it does not own, plugins whose host
framework forbids allocation on the decode path, processes that keep their
device footprint fixed after start-up.  It must return exactly what the
regular entry point returns for temperature 0 (penalties, then the lowest
index of the largest logit), call after call, although every call reuses the
same fixed working memory inside the library.

This file is collected last so that a run stopping at its first failure has
already run every other test.
"""
import ctypes as C

import numpy as np
import pytest

from qwen600_engine_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def _batch(seed, dtype, B=96, V=W.VOCAB, window=64):
    g = np.random.default_rng(seed)
    x = g.normal(0.0, 3.0, size=(B, V)).astype(np.float32)
    for r in range(0, B, 7):               # exact duplicate maxima: lowest index must win
        m = int(np.argmax(x[r]))
        x[r, (m + 12345) % V] = x[r, m]
    hist = g.integers(0, V, size=(B, window)).astype(np.int32)
    hist[:, :min(4, window)] = np.argmax(x, axis=1)[:, None]   # penalise each row's maximum, repeatedly
    counts = g.integers(1, 4, size=(B, window)).astype(np.float32)
    count = np.full(B, window, np.int32)
    logits = W.to_bf16_bits(x) if dtype == "bf16" else x
    return logits, hist, counts, count


def _dev(torch, logits, hist, counts, count, dtype):
    if dtype == "bf16":
        x = torch.from_numpy(logits.view(np.int16)).cuda().view(torch.bfloat16)
    else:
        x = torch.from_numpy(logits).cuda()
    return (x, torch.from_numpy(hist).cuda(), torch.from_numpy(counts).cuda(),
            torch.from_numpy(count).cuda())


def _static_call(torch, x, h, c, n, pen):
    from qwen600_engine_b200 import _lib
    B, V = x.shape
    out = torch.full((B,), -7, dtype=torch.int32, device="cuda")
    code = _lib.QS_BF16 if x.dtype == torch.bfloat16 else _lib.QS_F32
    rc = _lib.lib.qs_argmax_rows_static(
        x.data_ptr(), code, B, V, h.data_ptr(), c.data_ptr(), n.data_ptr(), h.shape[1],
        C.c_float(pen[0]), C.c_float(pen[1]), C.c_float(pen[2]), out.data_ptr(),
        torch.cuda.current_stream().cuda_stream)
    _lib.check(rc)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def _regular_call(torch, x, h, c, n, pen):
    from qwen600_engine_b200.sampler import Sampler
    B, V = x.shape
    s = Sampler(0.0, 1.0, 0.0, 0, pen[0], pen[1], pen[2], h.shape[1], 1, max_batch=B, vocab=V)
    rng = torch.ones(B, dtype=torch.int64, device="cuda")
    out = s.sample_rows(x, h, c, n, rng)
    torch.cuda.synchronize()
    s.free()
    return out.cpu().numpy()


def test_static_entry_matches_regular_entry_on_consecutive_calls():
    torch = _torch()
    pen = (1.3, 0.4, 0.25)
    # calls in a row, different data, dtype, batch and window, reusing the
    # fixed memory: a large call first, then smaller ones, so that results or
    # window tables a larger call left behind would show
    cases = ((101, "bf16", 96, 64), (202, "f32", 96, 64), (303, "bf16", 5, 3), (404, "f32", 7, 0))
    for seed, dtype, B, window in cases:
        d = _dev(torch, *_batch(seed, dtype, B=B, window=window), dtype)
        got = _static_call(torch, *d, pen)
        want = _regular_call(torch, *d, pen)
        np.testing.assert_array_equal(got, want, err_msg=f"seed {seed} ({dtype}, B={B}, window={window})")
        assert (got >= 0).all()


def test_static_entry_allocates_no_device_memory():
    torch = _torch()
    pen = (1.2, 0.0, 0.0)
    d = _dev(torch, *_batch(505, "bf16", B=64, window=32), "bf16")
    _static_call(torch, *d, pen)            # set-up: the array's address is looked up once
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(3):
        _static_call(torch, *d, pen)
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, f"device memory in use grew by {free0 - free1} bytes"


def test_static_entry_rejects_sizes_beyond_its_memory():
    torch = _torch()
    from qwen600_engine_b200 import _lib
    x = torch.zeros((1025, 16), device="cuda")
    h = torch.zeros((1025, 4), dtype=torch.int32, device="cuda")
    c = torch.zeros((1025, 4), device="cuda")
    n = torch.zeros(1025, dtype=torch.int32, device="cuda")
    out = torch.zeros(1025, dtype=torch.int32, device="cuda")
    rc = _lib.lib.qs_argmax_rows_static(x.data_ptr(), _lib.QS_F32, 1025, 16, h.data_ptr(),
                                        c.data_ptr(), n.data_ptr(), 4, C.c_float(1.1),
                                        C.c_float(0.0), C.c_float(0.0), out.data_ptr(), None)
    assert rc == _lib.QS_ERR_UNSUPPORTED
    assert b"batch" in _lib.lib.qs_last_error()
    rc = _lib.lib.qs_argmax_rows_static(x.data_ptr(), _lib.QS_F32, 4, 16, h.data_ptr(),
                                        c.data_ptr(), n.data_ptr(), 129, C.c_float(1.1),
                                        C.c_float(0.0), C.c_float(0.0), out.data_ptr(), None)
    assert rc == _lib.QS_ERR_UNSUPPORTED
