"""The decode tail before sampling (qwen_model.cuh:710-723): final RMSNorm and
the lm_head projection on tcgen05 tensor cores, then sampling.

The reference computes the projection with cublasGemmEx (bf16 in and out,
fp32 accumulation), whose summation order is its own, so the logits are
checked against the exact product: every logit within one bf16 ulp of it
plus the fp32 accumulation bound, and nearly all equal to it rounded to bf16
(a difference needs the exact value within accumulation error of a bf16
rounding boundary, or products that cancel to nearly zero).  The sampled tokens are
checked exactly: the reference's own sampler.h run on the logits this kernel
emitted must draw the same tokens."""
import numpy as np
import pytest

from qwen600_engine_b200 import workloads as W

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.backends.cuda.matmul.allow_tf32 = False
    return torch


def _inputs(torch, B, D, V, seed, norm_weight=True):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    h = torch.randn((B, D), generator=g, device="cuda").to(torch.bfloat16)
    w = (0.02 * torch.randn((V, D), generator=g, device="cuda")).to(torch.bfloat16)
    nw = (1.0 + 0.1 * torch.randn((D,), generator=g, device="cuda")).to(torch.bfloat16) if norm_weight else None
    return h, w, nw


def _ulp_bf16(x):
    """One bf16 ulp at |x| (fp32 tensor)."""
    import torch
    a = x.abs().clamp_min(2.0 ** -126)
    e = torch.floor(torch.log2(a))
    return torch.pow(2.0, e - 7)


def _check_norm(torch, h, nw, normed):
    x = h.double()
    ms = (x * x).mean(dim=1, keepdim=True)
    ref = x / torch.sqrt(ms + 1e-6)
    if nw is not None:
        ref = ref * nw.double()
    got = normed.double()
    ulp = _ulp_bf16(ref.float()).double()
    assert ((got - ref).abs() <= 1.01 * ulp).all(), "RMSNorm off by more than one bf16 ulp"
    exact = (got == ref.to(torch.bfloat16).double()).float().mean().item()
    assert exact > 0.99, f"RMSNorm: only {exact:.4f} of values round like the exact value"


def _check_logits(torch, normed, w, logits):
    """Each logit within one bf16 ulp of the exact product plus the fp32
    accumulation bound K * 2^-24 * sum|a_k b_k| (which matters where the
    products cancel to nearly zero)."""
    ref = (normed.double() @ w.double().t())
    acc = normed.shape[1] * 2.0 ** -24 * (normed.double().abs() @ w.double().abs().t())
    got = logits.double()
    ulp = _ulp_bf16(ref.float()).double()
    diff = (got - ref).abs()
    assert (diff <= 1.01 * ulp + acc).all(), f"logit off by {float((diff / (ulp + acc)).max()):.2f} tolerances"
    same = (logits == ref.to(torch.bfloat16)).float().mean().item()
    assert same > 0.995, f"only {same:.5f} of logits equal the exact product rounded to bf16"
    # the reference's own route: cuBLAS bf16 GEMM with fp32 accumulation
    cub = torch.matmul(normed, w.t())
    d2 = (cub.double() - got).abs()
    assert (d2 <= 2.02 * ulp + 2 * acc).all()


# The launch picks its tile width from the vocabulary size (208 for the whole
# Qwen3 vocabulary on 148 SMs, 176 for half of it, 144 for a quarter, 128 for
# small vocabularies): the cases cover every width.
@pytest.mark.parametrize("B,D,V", [(128, 1024, W.VOCAB), (5, 64, 1003), (130, 1024, 4096), (1, 1024, 151936),
                                   (96, 1024, 75968), (128, 1024, 37984), (7, 1024, 18992)])
def test_rmsnorm_and_logits(B, D, V):
    torch = _torch()
    from qwen600_engine_b200.sampler import lm_head
    h, w, nw = _inputs(torch, B, D, V, seed=B * 7 + V)
    normed, logits = lm_head(h, w, nw)
    torch.cuda.synchronize()
    _check_norm(torch, h, nw, normed)
    _check_logits(torch, normed, w, logits)


def test_norm_weight_none_is_ones():
    torch = _torch()
    from qwen600_engine_b200.sampler import lm_head
    h, w, _ = _inputs(torch, 16, 1024, 2048, seed=3, norm_weight=False)
    n1, l1 = lm_head(h, w, None)
    n2, l2 = lm_head(h, w, torch.ones(1024, dtype=torch.bfloat16, device="cuda"))
    assert torch.equal(n1, n2) and torch.equal(l1, l2)


def test_lm_head_sample_matches_reference_sampler_on_emitted_logits(ref_sampler):
    """Three decode steps of 128 rows through RMSNorm + lm_head + sample()
    with history, against the reference's Samplers fed the same logits."""
    torch = _torch()
    from qwen600_engine_b200.sampler import Sampler
    B, D = 128, 1024
    p = W.SamplingParams(0.6, 0.95, 0.05, 20, 1.1, 0.0, 0.0)   # the reference's defaults
    seed = 42
    s = Sampler(p.temperature, p.topp, p.minp, p.top_k, p.repetition_penalty,
                p.frequency_penalty, p.presence_penalty, 64, seed, max_batch=B)
    sess = ref_sampler.session(p, B, 64, [seed + r for r in range(B)])
    _, w, nw = _inputs(torch, 1, D, W.VOCAB, seed=11)
    for step in range(3):
        h, _, _ = _inputs(torch, B, D, 8, seed=100 + step, norm_weight=False)
        tok = s.lm_head_sample(h, w, nw)
        torch.cuda.synchronize()
        s.lm_head_status()
        logits = s.lm_head_logits(B)
        x = logits.float().cpu().numpy()
        want = sess.step(x, n_threads=8)
        np.testing.assert_array_equal(tok.cpu().numpy(), want, err_msg=f"step {step}")
    rng_ref = np.array([sess.state(r)["rng"] for r in range(B)], np.uint64)
    np.testing.assert_array_equal(s.rng_state, rng_ref)
    s.free()
    sess.free()


@pytest.mark.parametrize("B,V,params", [
    (128, W.VOCAB, (0.6, 0.95, 0.05, 20, 1.1, 0.5, 0.3)),   # penalised window tokens, tile 208
    (130, 37984, (0.8, 0.9, 0.0, 0, 1.2, 0.0, 0.0)),        # two 128-row launches, tile 144, no top-k
    (7, 4096, (0.0, 1.0, 0.0, 0, 1.3, 0.0, 0.2)),           # greedy rows, tile 128
])
def test_lm_head_sample_epilogue_maxima_match_streamed(B, V, params):
    """qs_lm_head_sample takes the rows' segment maxima from the lm_head
    epilogue and reads only the window's segments from the logits; sampling
    the same logits with qs_sample (which streams them) must give the same
    tokens and RNG states, step after step (the scan zeroes the epilogue's
    buffer for the next call, and the sampled tokens enter the windows)."""
    torch = _torch()
    from qwen600_engine_b200.sampler import Sampler
    D = 1024
    p = W.SamplingParams(*params)

    def make():
        return Sampler(p.temperature, p.topp, p.minp, p.top_k, p.repetition_penalty, p.frequency_penalty,
                       p.presence_penalty, 64, 5, max_batch=B, vocab=V)
    fused, plain = make(), make()
    _, w, nw = _inputs(torch, 1, D, V, seed=21)
    for step in range(4):
        h, _, _ = _inputs(torch, B, D, 8, seed=300 + step, norm_weight=False)
        tok = fused.lm_head_sample(h, w, nw)
        torch.cuda.synchronize()
        fused.lm_head_status()
        logits = fused.lm_head_logits(B).clone()
        want = plain.sample(logits)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(tok.cpu().numpy(), want.cpu().numpy(), err_msg=f"step {step}")
    np.testing.assert_array_equal(fused.rng_state, plain.rng_state)
    fused.free()
    plain.free()


def test_lm_head_argument_errors():
    torch = _torch()
    from qwen600_engine_b200.sampler import SamplerError, lm_head
    h = torch.zeros((4, 100), dtype=torch.bfloat16, device="cuda")
    w = torch.zeros((64, 100), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(SamplerError):
        lm_head(h, w)   # hidden_dim not a multiple of 64


def test_lm_head_gives_up_cleanly_when_its_waits_run_out():
    """A wait limit of a few nanoseconds (the test hook) makes the pipeline
    waits run out: the kernel raises its error flag, lets the copies and MMAs
    it issued complete, frees its TMEM and returns.  The error is reported,
    the context stays usable, and the next launch with the default limit
    computes the right logits."""
    torch = _torch()
    from qwen600_engine_b200 import _lib
    from qwen600_engine_b200.sampler import SamplerError, lm_head
    h, w, nw = _inputs(torch, 128, 1024, W.VOCAB, seed=77)
    normed_ok, logits_ok = lm_head(h, w, nw)
    torch.cuda.synchronize()
    gave_up = False
    _lib.check(_lib.lib.qs_lm_head_set_wait_limit(1))
    try:
        for _ in range(3):
            try:
                lm_head(h, w, nw)
            except SamplerError as e:
                assert "gave up" in str(e)
                gave_up = True
                break
    finally:
        _lib.check(_lib.lib.qs_lm_head_set_wait_limit(0))
    torch.cuda.synchronize()
    assert gave_up, "no wait ran out under a 1 ns limit"
    normed, logits = lm_head(h, w, nw)
    torch.cuda.synchronize()
    assert torch.equal(normed, normed_ok) and torch.equal(logits, logits_ok)
