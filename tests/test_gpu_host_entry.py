"""qs_sample_rows_host: every buffer on the host, the logits staged over the
handle's copy streams.  Tokens and advanced RNG states must equal those of
the device entry qs_sample_rows on the same inputs, and the handle's own RNG
states must be untouched."""
import numpy as np
import pytest

from qwen600_engine_b200 import workloads as W

from test_gpu_parity import make_sampler, run_gpu, torch_mod

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("make", [lambda: W.topk_bf16(B=96, seed=21), lambda: W.nucleus_f32(B=16, seed=22)])
def test_host_entry_matches_device_entry(make):
    torch = torch_mod()
    wl = make()
    g = run_gpu(wl)
    s = make_sampler(wl)
    rng_before = s.rng_state.copy()
    if wl.dtype == "bf16":
        x = torch.from_numpy(wl.logits.view(np.int16)).view(torch.bfloat16).pin_memory()
    else:
        x = torch.from_numpy(np.ascontiguousarray(wl.logits)).pin_memory()
    rng = torch.from_numpy(wl.rng.view(np.int64).copy()).pin_memory()
    hist = counts = count = None
    if wl.window > 0:
        hist = torch.from_numpy(wl.hist.astype(np.int32)).pin_memory()
        counts = torch.from_numpy(wl.hist_counts.astype(np.float32)).pin_memory()
        count = torch.from_numpy(wl.hist_count.astype(np.int32)).pin_memory()
    tok = s.sample_rows_host(x, hist, counts, count, rng)
    np.testing.assert_array_equal(tok.numpy(), g["tokens"])
    np.testing.assert_array_equal(rng.numpy().view(np.uint64), g["rng"])
    np.testing.assert_array_equal(s.rng_state, rng_before)
    s.free()
