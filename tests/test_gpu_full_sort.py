"""Rows sampled without top-k whose min-p / top-p cut lies beyond the row
kernel's candidate buffer: the exact full-sort pass (qs_sort.cu) against the
oracle.  The reference sorts the whole vocabulary with a stable qsort
(sampler.h:216-217, compare_prob_desc :67-73), so equal probabilities keep
index order; flat bf16 rows hold thousands of equal probabilities and check
that order through the sampled token and the candidate list."""
import numpy as np
import pytest

from qwen600_engine_b200 import workloads as W

from test_gpu_parity import check_candidates, compare, run_gpu, torch_mod

pytestmark = pytest.mark.gpu


def flat(V, dtype, params, B=4, scale=1.0, seed=0, W_=0):
    g = np.random.default_rng(seed)
    x = g.normal(0.0, scale, size=(B, V)).astype(np.float32)
    logits = W.to_bf16_bits(x) if dtype == "bf16" else x
    ids = g.integers(0, V, size=B * W_) if W_ else np.zeros(0)
    return W._full_window(B, W_, ids, seed + 50, f"flat_{V}_{dtype}", params, logits, dtype)


NUCLEUS = [
    W.SamplingParams(1.0, 0.9, 0.0, 0, 1.0, 0.0, 0.0),     # top-p cut deep in the row
    W.SamplingParams(1.3, 1.0, 0.02, 0, 1.0, 0.0, 0.0),    # min-p keeps thousands, no top-p
    W.SamplingParams(1.0, 1.0, 0.0, 0, 1.0, 0.0, 0.0),     # neither: the whole vocabulary
    W.SamplingParams(0.9, 0.95, 0.01, 0, 1.2, 0.3, 0.2),   # both, with penalties
]


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
@pytest.mark.parametrize("pi", range(len(NUCLEUS)))
def test_full_sort_full_vocab(oracle, dtype, pi):
    p = NUCLEUS[pi]
    wl = flat(W.VOCAB, dtype, p, B=4, scale=0.7 if dtype == "bf16" else 1.0, seed=pi,
              W_=32 if p.repetition_penalty != 1.0 else 0)
    o = oracle.sample_workload(wl, debug=True, cand_cap=64)
    g = run_gpu(wl, cand_cap=64)
    compare(wl, g, o)
    for r in range(wl.batch):
        od = o["debug"][r]
        assert g["debug"]["n_final"][r] == od["n_final"]
        assert g["debug"]["renorm_sum"][r] == np.float32(od["renorm_sum"]), f"row {r}: renormalising sum"
        n = min(od["n_final"], 64)
        check_candidates(g["cand_index"][r], g["cand_prob"][r], od["cand_index"], od["cand_prob"],
                         n, True, f"row {r}")


@pytest.mark.parametrize("V", [1003, 4099])
@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_full_sort_small_vocab(oracle, V, dtype):
    for pi, p in enumerate(NUCLEUS):
        wl = flat(V, dtype, p, B=6, scale=0.3, seed=10 + pi, W_=8)
        o = oracle.sample_workload(wl, debug=True, cand_cap=64)
        g = run_gpu(wl)
        compare(wl, g, o)


def test_full_sort_against_reference(ref_sampler):
    """The compiled reference itself on flat bf16 rows (heavy ties)."""
    p = NUCLEUS[0]
    wl = flat(W.VOCAB, "bf16", p, B=3, scale=0.5, seed=21)
    o = ref_sampler.sample_workload(wl, want_probindex=True)
    g = run_gpu(wl, cand_cap=64)
    np.testing.assert_array_equal(g["tokens"], o["tokens"])
    np.testing.assert_array_equal(g["rng"], o["rng"])
    # the reference's sorted array after sampling: its first 64 ids in order
    np.testing.assert_array_equal(g["cand_index"], o["index"][:, :64])


@pytest.mark.parametrize("k", [1000, 4000])
def test_index_ties_topk_overflow(oracle, k):
    """Top-k beyond the candidate buffer under QS_FLAG_INDEX_TIES (ties in
    index order): the full sort takes the first k.  fp32 normal rows hold no
    equal probabilities, so the reference's order is the same."""
    torch_mod()
    from qwen600_engine_b200.sampler import QS_FLAG_INDEX_TIES
    p = W.SamplingParams(1.0, 0.97, 0.0, k, 1.0, 0.0, 0.0)
    wl = flat(W.VOCAB, "f32", p, B=4, seed=33)
    o = oracle.sample_workload(wl, debug=True, cand_cap=64)
    g = run_gpu(wl, flags=QS_FLAG_INDEX_TIES, cand_cap=64)
    compare(wl, g, o)
    assert (g["tokens"] >= 0).all()
