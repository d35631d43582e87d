"""Multi-step sampling with history, as the reference's decode loop drives it
(main.cu:136-139): every step samples each row and sample() updates the
row's window ring, its count / position and the cumulative token counts
(sampler.h:257-267); bindings.cu:213-239 rewrites parameters and the RNG
state between steps and reset_state clears the history (sampler.h:346-354).

The CPU test pins the oracle's stateless entry (explicit window, counts and
RNG) against the reference's own persistent Samplers by replaying the
history update on the host.  The GPU test drives the library's stateful
API (qs_sample on device bf16 logits and qs_sample_host on host fp32
logits) against the same reference Samplers, step by step.
"""
import numpy as np
import pytest

from qwen600_engine_b200 import workloads as W

V = W.VOCAB
PARAMS = W.SamplingParams(0.8, 0.95, 0.05, 20, 1.3, 0.2, 0.1)
PARAMS2 = W.SamplingParams(1.1, 0.9, 0.0, 40, 1.1, 0.0, 0.3)


def step_logits(g, B, prev, dtype="bf16"):
    """Gumbel rows with the previous tokens pushed up, so that penalties
    decide draws.  bf16-representable values (the device path reads bf16)."""
    x = (3.0 * g.gumbel(size=(B, V))).astype(np.float32)
    for r in range(B):
        for t in prev[r][-6:]:
            x[r, t] = np.float32(x[r].max() + g.uniform(-0.5, 1.5))
    bits = W.to_bf16_bits(x)
    return bits, W.widen_bf16(bits)


class HostHistory:
    """The reference's per-row history update (sampler.h:257-267) on the host."""

    def __init__(self, B, window):
        self.W = window
        self.ring = np.zeros((B, window), np.int32)
        self.count = np.zeros(B, np.int32)
        self.pos = np.zeros(B, np.int32)
        self.tc = [dict() for _ in range(B)]

    def slot_counts(self):
        hc = np.zeros(self.ring.shape, np.float32)
        for r in range(self.ring.shape[0]):
            for i in range(self.W):
                hc[r, i] = self.tc[r].get(int(self.ring[r, i]), 0.0)
        return hc

    def record(self, tokens):
        for r, t in enumerate(tokens):
            t = int(t)
            self.tc[r][t] = self.tc[r].get(t, 0.0) + 1.0
            self.ring[r, self.pos[r]] = t
            self.pos[r] = (self.pos[r] + 1) % self.W
            self.count[r] = min(self.count[r] + 1, self.W)

    def reset(self):
        # sampler.h:346-354 zeroes count, position and counts; slot contents stay
        self.count[:] = 0
        self.pos[:] = 0
        self.tc = [dict() for _ in self.tc]


def test_oracle_replay_matches_reference_session(oracle, ref_sampler):
    B, Wn, steps = 3, 8, 12
    seeds = [11, 12, 13]
    sess = ref_sampler.session(PARAMS, B, Wn, seeds)
    hh = HostHistory(B, Wn)
    rng = np.array(seeds, np.uint64)
    g = np.random.default_rng(7)
    prev = [[] for _ in range(B)]
    params = PARAMS
    for s in range(steps):
        if s == 6:
            params = PARAMS2
            sess.set_params(params)
        if s == 9:
            sess.reset()
            hh.reset()
        _, x = step_logits(g, B, prev)
        want = sess.step(x)
        o = oracle.sample_rows(params, x, hh.ring, hh.slot_counts(), hh.count, rng)
        np.testing.assert_array_equal(o["tokens"], want, err_msg=f"step {s}")
        rng = o["rng"]
        hh.record(want)
        for r in range(B):
            prev[r].append(int(want[r]))
    for r in range(B):
        st = sess.state(r)
        assert st["rng"] == int(rng[r])
        assert st["count"] == hh.count[r] and st["pos"] == hh.pos[r]
        np.testing.assert_array_equal(st["ring"], hh.ring[r])
    sess.free()


@pytest.mark.gpu
def test_stateful_api_matches_reference_session(ref_sampler):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen600_engine_b200.sampler import Sampler
    B, Wn, steps, seed = 4, 8, 14, 21
    dev = Sampler(PARAMS.temperature, PARAMS.topp, PARAMS.minp, PARAMS.top_k,
                  PARAMS.repetition_penalty, PARAMS.frequency_penalty, PARAMS.presence_penalty,
                  Wn, seed, max_batch=B)
    host = Sampler(PARAMS.temperature, PARAMS.topp, PARAMS.minp, PARAMS.top_k,
                   PARAMS.repetition_penalty, PARAMS.frequency_penalty, PARAMS.presence_penalty,
                   Wn, seed, max_batch=B)
    # the library seeds row r with seed + r; the reference runs one Sampler per row
    sess = ref_sampler.session(PARAMS, B, Wn, [seed + r for r in range(B)])
    g = np.random.default_rng(8)
    prev = [[] for _ in range(B)]
    for s in range(steps):
        if s == 5:
            dev.set_params(**PARAMS2.__dict__)
            host.set_params(**PARAMS2.__dict__)
            sess.set_params(PARAMS2)
        if s == 8:
            new = [1234567 + 7 * r for r in range(B)]
            dev.rng_state = new
            host.rng_state = new
            for r in range(B):
                sess.set_rng(r, new[r])
        if s == 11:
            dev.reset_history()
            host.reset_history()
            sess.reset()
        bits, x = step_logits(g, B, prev)
        want = sess.step(x)
        xt = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
        got = dev.sample(xt).cpu().numpy()
        got_h = host.sample_host(x)
        np.testing.assert_array_equal(got, want, err_msg=f"device path, step {s}")
        np.testing.assert_array_equal(got_h, want, err_msg=f"host path, step {s}")
        for r in range(B):
            prev[r].append(int(want[r]))
    rng_ref = np.array([sess.state(r)["rng"] for r in range(B)], np.uint64)
    np.testing.assert_array_equal(dev.rng_state, rng_ref)
    np.testing.assert_array_equal(host.rng_state, rng_ref)
    dev.free()
    host.free()
    sess.free()
