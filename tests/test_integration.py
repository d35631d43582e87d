"""The sampler as a drop-in for the reference's decode loops.

* CPU: the reference's own main.cu and python/bindings.cu, with their sampler
  include switched to integration/qs_sampler_compat.h, compile for sm_100a
  (integration/patch_reference.py; needs a reference tree, named by the
  QWEN600_REF environment variable or found beside the repository).
* GPU: a decode loop written against the reference's interface
  (integration/decode_demo.cu: main.cu's loop shape -- prompt tokens fed,
  sample() at every position, prefill included -- over a stub forward())
  draws exactly the tokens the reference's own Samplers draw on the same
  logits, with host fp32 logits (sample()) and with device bf16 logits
  (sample_device()).
"""
import ctypes as C
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INTEG = os.path.join(ROOT, "integration")
DEMO = os.path.join(INTEG, "libqs_decode_demo.so")
V = 151936


def _ref_tree():
    cand = os.environ.get("QWEN600_REF") or os.path.join(os.path.dirname(ROOT), "reference")
    return cand if os.path.isfile(os.path.join(cand, "sampler.h")) else None


def test_reference_loops_compile_against_the_c_abi():
    ref = _ref_tree()
    if ref is None:
        pytest.skip("no reference tree (set QWEN600_REF)")
    sys.path.insert(0, INTEG)
    import patch_reference
    res = patch_reference.compile_all(ref)
    for name, (rc, err) in res.items():
        assert rc == 0, f"{name} does not compile on the C ABI:\n{err}"


def test_demo_library_exports_the_loop():
    if not os.path.exists(DEMO):
        pytest.skip("integration library not built")
    lib = C.CDLL(DEMO)
    assert hasattr(lib, "qs_demo_decode")


def _demo(n_steps, prompt, p, window, seed, device_logits):
    lib = C.CDLL(DEMO)
    f = lib.qs_demo_decode
    f.restype = C.c_int
    f.argtypes = [C.c_int, C.POINTER(C.c_int), C.c_int, C.c_float, C.c_float, C.c_float, C.c_int,
                  C.c_float, C.c_float, C.c_float, C.c_int, C.c_ulonglong, C.c_int,
                  C.POINTER(C.c_int), C.POINTER(C.c_uint16)]
    pr = np.ascontiguousarray(prompt, dtype=np.int32)
    toks = np.zeros(n_steps, np.int32)
    logits = np.zeros((n_steps, V), np.uint16)
    rc = f(n_steps, pr.ctypes.data_as(C.POINTER(C.c_int)), len(pr), p.temperature, p.topp, p.minp,
           int(p.top_k), p.repetition_penalty, p.frequency_penalty, p.presence_penalty, window, seed,
           device_logits, toks.ctypes.data_as(C.POINTER(C.c_int)), logits.ctypes.data_as(C.POINTER(C.c_uint16)))
    assert rc == 0
    return toks, logits


@pytest.mark.gpu
@pytest.mark.parametrize("device_logits", [0, 1])
@pytest.mark.parametrize("pi", [0, 1])
def test_decode_loop_matches_reference_sampler(ref_sampler, device_logits, pi):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen600_engine_b200 import workloads as W
    params = [W.SamplingParams(0.6, 0.95, 0.05, 20, 1.1, 0.0, 0.0),       # the reference's defaults
              W.SamplingParams(0.8, 0.9, 0.0, 50, 1.2, 0.4, 0.3)][pi]
    window, seed = 16, 1234 + pi
    prompt = [101, 2024, 77, 151935, 5, 60000]
    n = 28
    toks, logits = _demo(n, prompt, params, window, seed, device_logits)
    # the reference's Sampler driven the same way: one sample() per position
    sess = ref_sampler.session(params, 1, window, [seed])
    want = np.zeros(n, np.int32)
    for pos in range(n):
        x = (logits[pos].astype(np.uint32) << 16).view(np.float32).reshape(1, V)
        want[pos] = sess.step(x)[0]
    sess.free()
    np.testing.assert_array_equal(toks, want)
    # the loop fed its own samples back after the prompt
    assert len(set(toks[len(prompt):].tolist())) > 1
