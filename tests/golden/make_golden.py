"""Generates tests/golden/reference_vectors.npz from the reference's own
sampler.h (compiled by oracle/Makefile into oracle/_ref/libref_sampler.so).

The inputs are not stored (a full-vocabulary fp32 row is 600 KB); they are
regenerated from seeds by qwen600_engine_b200.workloads and by the small
recipes below, and each case stores a SHA-256 of its input batch so that a
change in the generators is detected instead of silently comparing other
data.  Stored per row: the sampled token, the advanced xorshift64* state, the
first 64 (prob, index) entries of the reference's scratch array after
sample() (its final candidate order, renormalised over the kept prefix) and a
hash of the logits as sample() left them (penalised and temperature-scaled
in place).

Run (needs oracle/_ref/libref_sampler.so, built from the reference tree by
`make -C oracle REF=<reference tree>`):
    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from qwen600_engine_b200 import workloads as W  # noqa: E402

OUT = os.path.join(HERE, "reference_vectors.npz")
NPI = 64  # scratch entries kept per row


def digest(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def edge_workloads():
    """Hand-made rows: ties everywhere, duplicate maxima, penalised maxima."""
    V = W.VOCAB
    cases = []
    # all logits equal: every probability ties; k = 20
    x = np.zeros((2, V), np.float32)
    x[1] = -3.25
    cases.append(W._full_window(2, 0, np.zeros(0), 11, "all_equal_topk", W.SamplingParams(
        1.0, 0.9, 0.0, 20, 1.0, 0.0, 0.0), x, "f32"))
    # two exact maxima far apart, greedy and sampled
    x = np.full((2, V), -1.0, np.float32)
    x[:, [777, 150000]] = 9.0
    x[:, 5] = 8.5
    cases.append(W._full_window(2, 0, np.zeros(0), 12, "dup_max_greedy", W.SamplingParams(
        0.0, 1.0, 0.0, 0, 1.0, 0.0, 0.0), x, "f32"))
    cases.append(W._full_window(2, 0, np.zeros(0), 13, "dup_max_topk", W.SamplingParams(
        0.9, 0.99, 0.0, 5, 1.0, 0.0, 0.0), x.copy(), "f32"))
    # penalised maximum with repeats in the window, negative and positive logits
    g = np.random.default_rng(14)
    x = g.normal(0, 1.5, size=(4, V)).astype(np.float32)
    ids = np.tile(np.array([10, 20, 10, 30, 10, 40, 20, 50] * 4, np.int64), 4)
    x[:, 10] = 7.0
    x[:, 20] = -0.5
    x[:, 30] = 0.0
    cases.append(W._full_window(4, 32, ids, 14, "penalty_repeats", W.SamplingParams(
        0.7, 0.8, 0.02, 40, 1.3, 0.4, 0.25), x, "f32"))
    # bf16 plateau: many exact ties near the top
    g = np.random.default_rng(15)
    x = np.round(g.normal(0, 2.0, size=(4, V)) * 4) / 4
    b = W.to_bf16_bits(x.astype(np.float32))
    cases.append(W._full_window(4, 0, np.zeros(0), 15, "bf16_plateau", W.SamplingParams(
        0.5, 0.97, 0.0, 50, 1.0, 0.0, 0.0), b, "bf16"))
    return cases


def golden_cases():
    cases = [W.single_row(seed=s) for s in (1, 2, 3)]
    cases += [W.greedy_bf16(B=8), W.nucleus_f32(B=4), W.topk_bf16(B=8)]
    cases += edge_workloads()
    return cases


def main():
    from oracle.oracle import RefSampler
    ref = RefSampler()
    store = {}
    names = []
    for wl in golden_cases():
        key = f"{wl.name}_{wl.batch}"
        if key in names:
            key = key + "_" + str(int(wl.rng[0]))
        names.append(key)
        res = ref.sample_workload(wl, want_mutated=True, want_probindex=True)
        store[f"{key}/input_sha"] = np.array(digest(wl.logits))
        store[f"{key}/tokens"] = res["tokens"]
        store[f"{key}/rng"] = res["rng"]
        store[f"{key}/pi_prob"] = res["prob"][:, :NPI].copy()
        store[f"{key}/pi_index"] = res["index"][:, :NPI].copy()
        store[f"{key}/mutated_sha"] = np.array([digest(m) for m in res["mutated"]])
    store["names"] = np.array(names)
    np.savez_compressed(OUT, **store)
    print(f"wrote {OUT}: {len(names)} cases")


if __name__ == "__main__":
    main()
