"""GPU parity of the CUDA sampler against the CPU oracle (itself pinned to the
reference's sampler.h) on seeded inputs, through the C ABI.

Tolerances (north star): greedy tokens and top-k candidate sets bit-exact;
penalised logits within 1 ulp (the kernels use the same IEEE operations, so
bit-exact is asserted); probabilities within 1e-6 absolute; sampled tokens
equal on >= 99.9% of rows, a mismatch allowed only where the uniform lies
within 1e-6 of a CDF boundary.  The softmax denominator is reproduced
bit-for-bit (the reference's sequential fp32 sum), so the tests assert
exact equality of sums and tokens and report any deviation.
"""
import hashlib
import os
import sys

import numpy as np
import pytest

from qwen600_engine_b200 import workloads as W

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

PROB_TOL = 1e-6


def torch_mod():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch


def dev_inputs(wl):
    torch = torch_mod()
    if wl.dtype == "bf16":
        x = torch.from_numpy(wl.logits.view(np.int16)).cuda().view(torch.bfloat16)
    else:
        x = torch.from_numpy(np.ascontiguousarray(wl.logits)).cuda()
    d = {"logits": x,
         "rng": torch.from_numpy(wl.rng.view(np.int64).copy()).cuda()}
    if wl.window > 0:
        d["hist"] = torch.from_numpy(wl.hist.astype(np.int32)).cuda()
        d["hist_counts"] = torch.from_numpy(wl.hist_counts.astype(np.float32)).cuda()
        d["hist_count"] = torch.from_numpy(wl.hist_count.astype(np.int32)).cuda()
    return d


def make_sampler(wl, window=None):
    from qwen600_engine_b200.sampler import Sampler
    p = wl.params
    return Sampler(p.temperature, p.topp, p.minp, p.top_k, p.repetition_penalty,
                   p.frequency_penalty, p.presence_penalty,
                   wl.window if window is None else window, 1,
                   max_batch=wl.batch, vocab=wl.vocab)


def run_gpu(wl, flags=0, probs=False, cand_cap=0):
    torch = torch_mod()
    s = make_sampler(wl)
    d = dev_inputs(wl)
    res = s.sample_rows(d["logits"], d.get("hist"), d.get("hist_counts"), d.get("hist_count"),
                        d["rng"], debug=True, probs=probs, cand_cap=cand_cap, flags=flags)
    torch.cuda.synchronize()
    out = {"tokens": res["tokens"].cpu().numpy(),
           "rng": d["rng"].cpu().numpy().view(np.uint64),
           "debug": res["debug"], "logits_after": d["logits"]}
    if probs:
        out["probs"] = res["probs"].cpu().numpy()
    if cand_cap:
        out["cand_index"] = res["cand_index"].cpu().numpy()
        out["cand_prob"] = res["cand_prob"].cpu().numpy()
    s.free()
    return out


def cdf_boundary_gap(row_dbg_o):
    """Distance of the oracle's uniform to its nearest CDF boundary."""
    n = row_dbg_o["n_final"]
    p = row_dbg_o["cand_prob"][:n]
    c = np.float32(0)
    best = np.inf
    for v in p:
        c = np.float32(c + v)
        best = min(best, abs(float(row_dbg_o["r"]) - float(c)))
    return best


def compare(wl, g, o, *, allow_boundary=True):
    """Assert GPU results match the oracle's; returns mismatch statistics."""
    B = wl.batch
    ot = o["tokens"]
    gt = g["tokens"]
    np.testing.assert_array_equal(g["rng"], o["rng"], err_msg="xorshift states differ")
    bad = np.nonzero(gt != ot)[0]
    dbg = g["debug"]
    for r in range(B):
        od = o["debug"][r]
        if od["greedy"]:
            assert dbg["greedy"][r] == 1
            continue
        assert dbg["max_logit"][r] == np.float32(od["max"]), f"row {r}: max differs"
        assert dbg["r"][r] == np.float32(od["r"]), f"row {r}: uniform differs"
        assert dbg["sum"][r] == np.float32(od["sum"]), (
            f"row {r}: softmax sum {dbg['sum'][r]!r} != reference {od['sum']!r}")
        if r not in bad:
            assert dbg["n_final"][r] == od["n_final"], f"row {r}: n_final differs"
            assert dbg["n_minp"][r] == od["n_minp"], f"row {r}: n_minp differs"
    agree = 1.0 - len(bad) / max(B, 1)
    for r in bad:
        gap = cdf_boundary_gap(o["debug"][r])
        assert allow_boundary and gap < 1e-6, (
            f"row {r}: token {gt[r]} != reference {ot[r]} and the uniform is {gap:.3g} from a "
            f"CDF boundary (exact_ties={dbg['exact_ties'][r]})")
    assert agree >= 0.999 or len(bad) == 0
    return {"rows": B, "mismatch": len(bad), "exact_ties": int(dbg["exact_ties"].sum()),
            "sum_fallback_mean": float(dbg["sum_fallback"].mean())}


def check_candidates(g_idx, g_prob, o_idx, o_prob, n, exact, what):
    """Candidate order [0, n): probabilities bit-exact; token ids identical
    when the reference's tie arrangement was reproduced (exact), else equal
    as sets inside every group of equal probability that is not cut by the
    list's end."""
    np.testing.assert_array_equal(g_prob[:n].view(np.uint32), o_prob[:n].view(np.uint32),
                                  err_msg=f"{what}: candidate probabilities")
    if exact:
        np.testing.assert_array_equal(g_idx[:n], o_idx[:n], err_msg=f"{what}: candidate order")
        return
    last = o_prob[n - 1]
    for v in np.unique(o_prob[:n]):
        if v == last:
            continue
        gi = set(g_idx[:n][g_prob[:n] == v].tolist())
        oi = set(o_idx[:n][o_prob[:n] == v].tolist())
        assert gi == oi, f"{what}: ids with probability {v!r} differ"


def oracle_run(oracle, wl, cap=64):
    return oracle.sample_workload(wl, debug=True, cand_cap=max(cap, 1))


def stack_single_rows(seeds):
    rows = [W.single_row(seed=s) for s in seeds]
    wl = rows[0]
    wl.logits = np.concatenate([w.logits for w in rows])
    wl.hist = np.concatenate([w.hist for w in rows])
    wl.hist_counts = np.concatenate([w.hist_counts for w in rows])
    wl.hist_count = np.concatenate([w.hist_count for w in rows])
    wl.hist_pos = np.concatenate([w.hist_pos for w in rows])
    wl.rng = np.array([s for s in seeds], dtype=np.uint64)
    return wl


CASES = {
    "single_row_x24": lambda: stack_single_rows(range(1, 25)),
    "greedy_bf16_256": lambda: W.greedy_bf16(B=256),
    "nucleus_f32_24": lambda: W.nucleus_f32(B=24),
    "topk_bf16_192": lambda: W.topk_bf16(B=192),
    # the measured configurations at their full batch: batch 64 full-vocabulary
    # nucleus (fp32, Zipf windows with frequency / presence penalties) and the
    # benchmark's batch 1024 top-k (bf16), where the tie pass queues ~4% of rows
    "nucleus_f32_64_full": lambda: W.nucleus_f32(B=64),
    "topk_bf16_1024_full": lambda: W.topk_bf16(B=1024),
    # batches of 256 rows and more take the persistent streaming kernel
    # (bf16 above; fp32 here, with Zipf windows and frequency / presence
    # penalties)
    "nucleus_f32_320_streamed": lambda: W.nucleus_f32(B=320, seed=31),
    "greedy_f32_300_streamed": lambda: _greedy_f32(300),
    # top k above the tie replay's shared-memory sort (1024): every such row
    # is queued and its k entries sorted in global memory
    "topk3000_bf16_12": lambda: _large_k(W.topk_bf16(B=12, seed=41), (0.7, 1.0, 0.0, 3000, 1.15, 0.0, 0.0)),
    "topk1500_f32_16": lambda: _large_k(_normal_f32(16, 43, 1.5), (0.35, 0.9, 0.0, 1500, 1.2, 0.5, 0.3)),
    "topk2000_bf16_256_streamed": lambda: _large_k(W.topk_bf16(B=256, seed=45),
                                                   (2.0, 0.97, 0.0, 2000, 1.1, 0.0, 0.0)),
    "topk5000_ties_f32_8": lambda: _large_k(_rounded_f32(8, 47), (1.0, 0.98, 0.01, 5000, 1.0, 0.0, 0.0)),
}


def _large_k(wl, params):
    wl.params = W.SamplingParams(*params)
    return wl


def _normal_f32(B, seed, scale):
    wl = W.nucleus_f32(B=B, seed=seed)
    g = np.random.default_rng(seed)
    wl.logits = (scale * g.standard_normal(wl.logits.shape)).astype(np.float32)
    return wl


def _rounded_f32(B, seed):
    """Logits rounded to multiples of 0.5 (thousands of exact ties at every
    rank), the first row all equal."""
    wl = W.nucleus_f32(B=B, seed=seed)
    g = np.random.default_rng(seed)
    wl.logits = np.round(2.0 * g.standard_normal(wl.logits.shape)).astype(np.float32) * np.float32(0.5)
    wl.logits[0] = 0.0
    return wl


def _greedy_f32(B):
    """Greedy fp32 rows with penalties: the streaming kernel's argmax path
    with window substitutions, exact duplicate maxima and a NaN at index 0."""
    wl = W.nucleus_f32(B=B, seed=37)
    wl.params = W.SamplingParams(0.0, 1.0, 0.0, 0, 1.3, 0.4, 0.25)
    x = wl.logits
    for r in range(0, B, 5):
        m = int(np.argmax(x[r]))
        x[r, (m + 777) % x.shape[1]] = x[r, m]
    x[7, 0] = np.float32("nan")
    return wl


@pytest.mark.parametrize("name", list(CASES))
def test_parity_full_vocab(oracle, name):
    wl = CASES[name]()
    o = oracle_run(oracle, wl)
    g = run_gpu(wl)
    stats = compare(wl, g, o)
    print(name, stats)


def test_golden_vectors_on_gpu():
    """The CUDA path against outputs of the reference itself (committed)."""
    import make_golden
    gold = np.load(os.path.join(HERE, "golden", "reference_vectors.npz"))
    for name, wl in zip(list(gold["names"]), make_golden.golden_cases()):
        assert hashlib.sha256(np.ascontiguousarray(wl.logits).tobytes()).hexdigest() == \
            str(gold[f"{name}/input_sha"])
        g = run_gpu(wl, cand_cap=make_golden.NPI)
        np.testing.assert_array_equal(g["tokens"], gold[f"{name}/tokens"], err_msg=name)
        np.testing.assert_array_equal(g["rng"], gold[f"{name}/rng"], err_msg=name)
        for r in range(wl.batch):
            if g["debug"]["greedy"][r]:
                continue
            n = min(int(g["debug"]["n_final"][r]), make_golden.NPI)
            check_candidates(g["cand_index"][r], g["cand_prob"][r], gold[f"{name}/pi_index"][r],
                             gold[f"{name}/pi_prob"][r], n, bool(g["debug"]["exact_ties"][r]),
                             f"{name} row {r}")


@pytest.mark.parametrize("name", ["single_row_x24", "topk_bf16_192", "nucleus_f32_24", "topk3000_bf16_12",
                                  "topk5000_ties_f32_8"])
def test_probabilities_and_candidates(oracle, name):
    wl = CASES[name]()
    rows = min(wl.batch, 6)
    sub = W.Workload(wl.name, wl.params, wl.logits[:rows].copy(), wl.dtype, wl.hist[:rows],
                     wl.hist_counts[:rows], wl.hist_count[:rows], wl.hist_pos[:rows],
                     wl.rng[:rows].copy(), wl.window)
    o = oracle.sample_workload(sub, debug=True, cand_cap=64, want_probs=True)
    g = run_gpu(sub, probs=True, cand_cap=64)
    for r in range(rows):
        od = o["debug"][r]
        diff = np.abs(g["probs"][r] - od["probs"]).max()
        assert diff <= PROB_TOL, f"row {r}: max |p - p_ref| = {diff:.3g}"
        n = min(od["n_final"], 64)
        check_candidates(g["cand_index"][r], g["cand_prob"][r], od["cand_index"], od["cand_prob"],
                         n, bool(g["debug"]["exact_ties"][r]), f"row {r}")
