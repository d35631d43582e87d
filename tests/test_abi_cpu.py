"""The C-ABI library loads and exports every entry point include/*.h
declares; argument checks that need no GPU return the documented codes."""
import ctypes as C
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        txt = open(h).read()
        names |= set(re.findall(r"QS_API\s+[\w\s\*]+?\b(qs_\w+)\s*\(", txt))
    return sorted(names)


def test_header_declares_entry_points():
    names = _declared()
    assert "qs_build_sampler" in names and "qs_sample" in names and len(names) >= 13


def test_library_exports_every_declared_symbol():
    from qwen600_engine_b200 import _lib
    for n in _declared():
        assert hasattr(_lib.lib, n), n
    assert set(_lib.EXPORTS) >= set(_declared())
    assert _lib.lib.qs_max_vocab() >= 151936


def test_argument_errors_without_gpu():
    from qwen600_engine_b200 import _lib
    L = _lib.lib
    h = C.c_void_p()
    p = _lib.Params(0.6, 0.95, 0.05, 20, 1.1, 0.0, 0.0)
    assert L.qs_build_sampler(None, C.byref(p), 1, 151936, 64, 1, 0) == _lib.QS_ERR_INVALID
    assert L.qs_build_sampler(C.byref(h), None, 1, 151936, 64, 1, 0) == _lib.QS_ERR_INVALID
    assert L.qs_build_sampler(C.byref(h), C.byref(p), 0, 151936, 64, 1, 0) == _lib.QS_ERR_INVALID
    assert L.qs_build_sampler(C.byref(h), C.byref(p), 1, 10 ** 7, 64, 1, 0) == _lib.QS_ERR_UNSUPPORTED
    assert L.qs_build_sampler(C.byref(h), C.byref(p), 1, 151936, 10 ** 6, 1, 0) == _lib.QS_ERR_UNSUPPORTED
    assert b"max_batch" in L.qs_last_error() or b"window" in L.qs_last_error()
    assert L.qs_free_sampler(None) == _lib.QS_OK
    assert L.qs_set_params(None, C.byref(p)) == _lib.QS_ERR_INVALID
    assert L.qs_sample(None, None, 0, 1, None, None, 0) == _lib.QS_ERR_INVALID


def test_python_mirror_of_reference_api():
    from qwen600_engine_b200 import sampler as S
    cfg = S.SamplingConfig()
    d = cfg.to_dict()
    # defaults of python/qwen_engine/qwen_inference.py:52-62
    assert (cfg.temperature, cfg.top_k, cfg.top_p, cfg.min_p) == (0.6, 20, 0.95, 0.05)
    assert (cfg.repetition_penalty, cfg.penalty_window, d["seed"]) == (1.1, 64, -1)
    for fn in ("build_sampler", "sample", "reset_sampler_history", "free_sampler"):
        assert callable(getattr(S, fn))
