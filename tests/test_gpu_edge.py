"""Edge cases of the CUDA sampler against the oracle: small and unaligned
vocabularies (scalar tail loads), top-k above the kernel's segment count (the
row goes to the exact pass), duplicate maxima, repeated and out-of-range
window ids, non-finite logits (no fault, valid output), argument errors."""
import numpy as np
import pytest

from qwen600_engine_b200 import workloads as W

from test_gpu_parity import compare, run_gpu, torch_mod

pytestmark = pytest.mark.gpu


def small(V, dtype, params, B=16, seed=0, W_=16, dist="normal"):
    g = np.random.default_rng(seed)
    if dist == "normal":
        x = g.normal(0, 2.0, size=(B, V)).astype(np.float32)
    else:
        x = (3.0 * g.gumbel(size=(B, V))).astype(np.float32)
    logits = W.to_bf16_bits(x) if dtype == "bf16" else x
    ids = g.integers(-3, V + 3, size=B * W_) if W_ else np.zeros(0)   # a few out of range
    wl = W._full_window(B, W_, ids, seed + 100, f"small_{V}_{dtype}", params, logits, dtype)
    return wl


PARAMS = [
    W.SamplingParams(0.8, 0.9, 0.05, 20, 1.3, 0.2, 0.1),
    W.SamplingParams(1.0, 0.5, 0.0, 0, 1.0, 0.0, 0.0),
    W.SamplingParams(0.0, 1.0, 0.0, 0, 1.2, 0.0, 0.0),
    W.SamplingParams(0.6, 1.0, 0.1, 3, 1.0, 0.0, 0.5),
]


@pytest.mark.parametrize("V", [1000, 1003, 4099])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("pi", range(len(PARAMS)))
def test_small_vocab(oracle, V, dtype, pi):
    wl = small(V, dtype, PARAMS[pi], seed=V + pi)
    o = oracle.sample_workload(wl, debug=True, cand_cap=64)
    g = run_gpu(wl)
    compare(wl, g, o)


def test_topk_above_segment_count(oracle):
    # V = 3000 bf16 has 12 segments; k = 40 > 12 makes the kernel select its
    # candidate threshold over elements instead of segment maxima
    wl = small(3000, "bf16", W.SamplingParams(0.9, 0.99, 0.0, 40, 1.1, 0.0, 0.0), seed=3,
               dist="gumbel")
    o = oracle.sample_workload(wl, debug=True, cand_cap=64)
    g = run_gpu(wl)
    compare(wl, g, o)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("pi", [0, 1])
def test_first_segment_running_maximum(oracle, dtype, pi):
    """Rows whose first 256 elements rise, fall, stay flat or hold one spike:
    the first segment has no earlier segment to bound its stash threshold,
    so each of its elements is held against the running maximum before it."""
    V, B = 4096, 8
    g = np.random.default_rng(7 + pi)
    x = g.normal(0, 2.0, size=(B, V)).astype(np.float32)
    ramp = np.linspace(-10, 10, 256, dtype=np.float32)
    x[0, :256] = ramp             # every element a new running maximum
    x[1, :256] = ramp[::-1]       # the first element the maximum of the segment
    x[2, :256] = -30.0
    x[2, 0] = 5.0
    x[3, :256] = -30.0
    x[3, 255] = 12.0
    x[4, :256] = 0.3 * ramp       # a ramp inside the significance gap
    x[5, :256] = 0.0              # ties all along
    x[6, 0] = 40.0                # an early spike that dominates the row
    x[7, 100:110] = 15.0
    logits = W.to_bf16_bits(x) if dtype == "bf16" else x
    ids = g.integers(0, V, size=B * 16)
    wl = W._full_window(B, 16, ids, 300 + pi, f"first_segment_{dtype}_{pi}", PARAMS[pi], logits, dtype)
    o = oracle.sample_workload(wl, debug=True, cand_cap=64)
    gg = run_gpu(wl)
    compare(wl, gg, o)


def test_large_topk_full_vocab(oracle):
    wl = W.topk_bf16(B=8, seed=12)
    wl.params = W.SamplingParams(1.0, 0.999, 0.0, 1000, 1.15, 0.0, 0.0)
    o = oracle.sample_workload(wl, debug=True, cand_cap=64)
    g = run_gpu(wl)
    compare(wl, g, o)


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_non_finite_logits_do_not_fault(dtype):
    torch = torch_mod()
    V, B = 2048, 6
    g = np.random.default_rng(5)
    x = g.normal(0, 1.0, size=(B, V)).astype(np.float32)
    x[0, 17] = np.inf
    x[1, :] = -np.inf
    x[2, 100] = np.nan
    x[3, 5] = -np.inf
    x[4, [3, 9]] = np.inf
    logits = W.to_bf16_bits(x) if dtype == "bf16" else x
    for p in (W.SamplingParams(0.7, 0.9, 0.05, 20, 1.0, 0.0, 0.0),
              W.SamplingParams(0.0, 1.0, 0.0, 0, 1.0, 0.0, 0.0),
              W.SamplingParams(1.0, 0.9, 0.0, 0, 1.0, 0.0, 0.0)):
        wl = W._full_window(B, 0, np.zeros(0), 9, "nonfinite", p, logits, dtype)
        out = run_gpu(wl)
        assert ((out["tokens"] >= -1) & (out["tokens"] < V)).all()
    torch.cuda.synchronize()
    # the device is still healthy: a finite batch samples exactly
    wl = small(V, dtype, PARAMS[0], seed=77)
    run_gpu(wl)


def test_argument_errors_on_gpu():
    torch = torch_mod()
    from qwen600_engine_b200.sampler import Sampler, SamplerError
    s = Sampler(0.7, 0.9, 0.0, 50, 1.0, 0.0, 0.0, 0, 1, max_batch=4, vocab=4000)
    x = torch.zeros((4, 4000), device="cuda")
    rng = torch.ones(4, dtype=torch.int64, device="cuda")
    with pytest.raises(SamplerError):
        s.sample_rows(torch.zeros((4, 3999), device="cuda"), rng=rng)    # vocab mismatch
    with pytest.raises(SamplerError):
        s.sample_rows(torch.zeros((5, 4000), device="cuda"),
                      rng=torch.ones(5, dtype=torch.int64, device="cuda"))   # batch > max
    with pytest.raises(SamplerError):
        s.sample_rows(x.to(torch.float16), rng=rng)                      # dtype
    s.set_params(top_k=1500)                                             # any top-k samples
    toks = s.sample_rows(x, rng=rng).cpu().numpy()
    assert ((toks >= 0) & (toks < 4000)).all()
    s.free()


def test_write_penalized_bit_exact(oracle):
    """QS_FLAG_WRITE_PENALIZED writes the penalised fp32 logits back in place,
    as the reference's sample() leaves them after its penalty loop
    (sampler.h:114-141).  Zipf windows repeat tokens many times, with
    repetition, frequency and presence penalties all on, so each penalised
    token replays the whole per-occurrence sequence; every one of the V
    entries must equal the oracle's bit for bit (the north star allows 1 ulp)."""
    from qwen600_engine_b200.sampler import QS_FLAG_WRITE_PENALIZED
    wl = W.nucleus_f32(B=16, seed=31)
    x0 = wl.logits.copy()
    g = run_gpu(wl, flags=QS_FLAG_WRITE_PENALIZED)
    after = g["logits_after"].cpu().numpy()
    # the oracle at temperature 0 stops after the penalties, so its mutated
    # rows are the penalised logits alone
    pen_only = W.SamplingParams(0.0, 1.0, 0.0, 0, wl.params.repetition_penalty,
                                wl.params.frequency_penalty, wl.params.presence_penalty)
    o = oracle.sample_rows(pen_only, x0, wl.hist, wl.hist_counts, wl.hist_count,
                           wl.rng.copy(), want_mutated=True)
    want = o["mutated"]
    changed = (want.view(np.uint32) != x0.view(np.uint32)).sum()
    assert changed > 16 * 50, "the windows should penalise many tokens"
    diff = np.nonzero(after.view(np.uint32) != want.view(np.uint32))
    assert diff[0].size == 0, (
        f"{diff[0].size} penalised logits differ, first at row {diff[0][0]} token {diff[1][0]}: "
        f"{after[diff[0][0], diff[1][0]]!r} != {want[diff[0][0], diff[1][0]]!r}")


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_greedy_nan_first_logit(oracle, dtype):
    """sample_argmax (sampler.h:100-111) starts from logits[0] with a strict
    '>': a NaN there wins, anywhere else it never does."""
    V, B = 3000, 5
    g = np.random.default_rng(11)
    x = g.normal(0, 1.0, size=(B, V)).astype(np.float32)
    x[0, 0] = np.nan                  # reference: token 0
    x[1, 0] = np.nan
    x[1, 7] = 50.0                    # still token 0
    x[2, 5] = np.nan                  # skipped: the argmax of the rest
    x[3, 0] = -np.inf
    x[3, 1:] = np.nan                 # token 0
    x[4, 10] = np.nan
    x[4, 11] = 9.0
    logits = W.to_bf16_bits(x) if dtype == "bf16" else x
    p = W.SamplingParams(0.0, 1.0, 0.0, 0, 1.0, 0.0, 0.0)
    wl = W._full_window(B, 0, np.zeros(0), 5, "greedy_nan", p, logits, dtype)
    o = oracle.sample_workload(wl)
    gg = run_gpu(wl)
    np.testing.assert_array_equal(gg["tokens"], o["tokens"])
    assert gg["tokens"][0] == 0 and gg["tokens"][1] == 0 and gg["tokens"][3] == 0
