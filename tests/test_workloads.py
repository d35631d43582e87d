import numpy as np

from qwen600_engine_b200 import workloads as W


def test_bf16_round_trip_and_rounding():
    x = np.array([1.0, -2.5, 3.14159, 1e-40, np.inf, -np.inf, 65504.0], np.float32)
    b = W.to_bf16_bits(x)
    w = W.widen_bf16(b)
    assert w[0] == 1.0 and w[1] == -2.5 and np.isinf(w[4]) and np.isinf(w[5])
    # round to nearest even on the 16 dropped bits
    u = np.array([0x3F808000, 0x3F818000, 0x3F808001], np.uint32).view(np.float32)
    assert list(W.to_bf16_bits(u)) == [0x3F80, 0x3F82, 0x3F81]


def test_generators_are_deterministic_and_shaped():
    a = W.topk_bf16(B=4, V=1000)
    b = W.topk_bf16(B=4, V=1000)
    assert a.logits.dtype == np.uint16 and a.logits.shape == (4, 1000)
    assert np.array_equal(a.logits, b.logits) and np.array_equal(a.hist, b.hist)
    assert list(a.rng) == [4, 5, 6, 7]
    n = W.nucleus_f32(B=2, V=5000)
    assert n.hist.shape == (2, 128) and n.hist.max() < 5000 and n.hist.min() >= 0
    # token_counts per slot = multiplicity of the slot's token in the window
    for r in range(2):
        ids, cnt = np.unique(n.hist[r], return_counts=True)
        m = dict(zip(ids, cnt))
        assert all(n.hist_counts[r, i] == m[n.hist[r, i]] for i in range(128))
    g = W.greedy_bf16(B=200, V=3000)
    for r in g.extra["tie_rows"]:
        w = W.widen_bf16(g.logits[r])
        assert (w == w.max()).sum() >= 2
