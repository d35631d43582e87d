"""CPU checks of the oracle (oracle/sampler_oracle.c): it is pinned against
the reference's own sampler.h, both through the committed golden vectors
(tests/golden/reference_vectors.npz, produced by the reference) and, where
oracle/_ref is built, by direct comparison on further seeded inputs."""
import hashlib
import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))
import make_golden  # noqa: E402

from qwen600_engine_b200 import workloads as W  # noqa: E402

GOLD = np.load(os.path.join(HERE, "golden", "reference_vectors.npz"))


def _digest(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def _cases():
    names = list(GOLD["names"])
    return list(zip(names, make_golden.golden_cases()))


@pytest.mark.parametrize("name,wl", _cases(), ids=[n for n, _ in _cases()])
def test_oracle_reproduces_reference_golden(oracle, name, wl):
    assert _digest(wl.logits) == str(GOLD[f"{name}/input_sha"]), "input generator changed"
    res = oracle.sample_workload(wl, want_mutated=True, debug=True, cand_cap=make_golden.NPI)
    np.testing.assert_array_equal(res["tokens"], GOLD[f"{name}/tokens"])
    np.testing.assert_array_equal(res["rng"], GOLD[f"{name}/rng"])
    for r, d in enumerate(res["debug"]):
        if d["greedy"]:
            continue
        np.testing.assert_array_equal(d["cand_index"], GOLD[f"{name}/pi_index"][r])
        np.testing.assert_array_equal(d["cand_prob"].view(np.uint32),
                                      GOLD[f"{name}/pi_prob"][r].view(np.uint32))
    for r in range(wl.batch):
        assert _digest(res["mutated"][r]) == str(GOLD[f"{name}/mutated_sha"][r])


def test_rng_matches_python_xorshift(oracle):
    def step(x):
        M = (1 << 64) - 1
        x ^= x >> 12
        x ^= (x << 25) & M
        x ^= x >> 27
        return x, ((x * 0x2545F4914F6CDD1D) & M) >> 32
    for seed in (1, 2, 12345, 2 ** 63 + 17):
        x = seed
        v, st = oracle.random_f32(seed)
        x, u = step(x)
        assert st == x
        assert v == np.float32((u >> 8) / 16777216.0)


@pytest.mark.parametrize("maker,kw", [
    (W.single_row, {"seed": 7}), (W.topk_bf16, {"B": 24, "seed": 41}),
    (W.nucleus_f32, {"B": 3, "seed": 9}), (W.greedy_bf16, {"B": 16, "seed": 5}),
])
def test_oracle_matches_compiled_reference(oracle, ref_sampler, maker, kw):
    wl = maker(**kw)
    a = ref_sampler.sample_workload(wl, want_mutated=True)
    b = oracle.sample_workload(wl, want_mutated=True)
    np.testing.assert_array_equal(a["tokens"], b["tokens"])
    np.testing.assert_array_equal(a["rng"], b["rng"])
    assert np.array_equal(a["mutated"].view(np.uint32), b["mutated"].view(np.uint32))


def test_oracle_small_vocab_semantics(oracle):
    # hand-checked 6-token row: penalties then greedy argmax (lowest index on ties)
    p = W.SamplingParams(0.0, 1.0, 0.0, 0, 2.0, 0.5, 0.25)
    x = np.array([[3.0, 6.0, 6.0, -1.0, 0.0, 5.0]], np.float32)
    hist = np.array([[1, 1, 3, 9]], np.int32)     # 9 is out of range: skipped
    cnt = np.array([[2.0, 2.0, 1.0, 1.0]], np.float32)
    res = oracle.sample_rows(p, x, hist, cnt, np.array([4], np.int32),
                             np.array([1], np.uint64), want_mutated=True)
    # token 1: 6 /2 -1 -.25 = 1.75; /2 -1 -.25 = -0.375 ; token 3: -1*2 -.5 -.25 = -2.75
    np.testing.assert_allclose(res["mutated"][0], [3.0, -0.375, 6.0, -2.75, 0.0, 5.0])
    assert res["tokens"][0] == 2
    assert res["rng"][0] == 1  # greedy draws no uniform
