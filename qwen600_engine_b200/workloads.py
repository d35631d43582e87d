"""Seeded synthetic sampling workloads.

The reference publishes no sampler benchmark data, so every workload here is
synthetic: logit rows over the Qwen3-0.6B vocabulary (V = 151936, reference
config.h:52) with the distributions, penalty windows and sampling parameters
of the five measured configurations, plus a small-V variant of each for quick
parity checks.  numpy PCG64 generators are seeded per workload; row r's
xorshift64* state is ``base_seed + r`` (never 0, the generator's fixed point).

bf16 rows are produced by rounding fp32 draws to bfloat16 (round to nearest
even) and are returned as uint16 bit patterns; ``widen_bf16`` gives the exact
fp32 values the reference sampler would see after its bf16->fp32 convert
(qwen_model.cuh:635-643).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional

import numpy as np

VOCAB = 151936


@dataclass
class SamplingParams:
    """The reference Sampler's parameter fields (sampler.h:23-31)."""

    temperature: float = 0.6
    topp: float = 0.95
    minp: float = 0.05
    top_k: int = 20
    repetition_penalty: float = 1.1
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0


@dataclass
class Workload:
    name: str
    params: SamplingParams
    logits: np.ndarray          # [B, V] float32, or uint16 bf16 bit patterns
    dtype: str                  # "f32" | "bf16"
    hist: np.ndarray            # [B, W] int32 ring contents (storage order)
    hist_counts: np.ndarray     # [B, W] float32 token_counts of each slot's token
    hist_count: np.ndarray      # [B] int32 valid slots
    hist_pos: np.ndarray        # [B] int32 next ring write slot
    rng: np.ndarray             # [B] uint64 xorshift64* states
    window: int
    extra: dict = field(default_factory=dict)

    @property
    def batch(self) -> int:
        return int(self.logits.shape[0])

    @property
    def vocab(self) -> int:
        return int(self.logits.shape[1])

    def logits_f32(self) -> np.ndarray:
        return widen_bf16(self.logits) if self.dtype == "bf16" else self.logits


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bfloat16 bit patterns, round to nearest even (NaN kept NaN)."""
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounding = ((u >> 16) & 1) + np.uint32(0x7FFF)
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(x)
    if nan.any():
        out[nan] = 0x7FC0
    return out


def widen_bf16(b: np.ndarray) -> np.ndarray:
    return (b.astype(np.uint32) << 16).view(np.float32)


def _counts_from_window(hist: np.ndarray, count: np.ndarray) -> np.ndarray:
    """token_counts value per slot = multiplicity of that token in the valid
    part of the window (a history produced by sampling since the last reset)."""
    B, W = hist.shape
    out = np.zeros((B, W), dtype=np.float32)
    for r in range(B):
        n = int(count[r])
        ids, inv, cnt = np.unique(hist[r, :n], return_inverse=True, return_counts=True)
        out[r, :n] = cnt[inv].astype(np.float32)
    return out


def _rng_states(seed: int, B: int) -> np.ndarray:
    return (np.uint64(seed) + np.arange(B, dtype=np.uint64)).astype(np.uint64)


def _full_window(B: int, W: int, ids: np.ndarray, seed: int, name: str,
                 params: SamplingParams, logits: np.ndarray, dtype: str,
                 extra: Optional[dict] = None) -> Workload:
    hist = ids.astype(np.int32).reshape(B, W) if W > 0 else np.zeros((B, 0), np.int32)
    count = np.full(B, W, dtype=np.int32)
    pos = np.zeros(B, dtype=np.int32)
    counts = _counts_from_window(hist, count) if W > 0 else np.zeros((B, 0), np.float32)
    return Workload(name, params, logits, dtype, hist, counts, count, pos,
                    _rng_states(seed, B), W, extra or {})


def single_row(V: int = VOCAB, seed: int = 1) -> Workload:
    """Batch 1, fp32 N(0, 2.5^2) plus 8 spikes at +12 on distinct random
    indices; 64-token uniform history; T .6, k 20, p .95, min-p .05, rp 1.1."""
    g = np.random.default_rng(seed)
    x = g.normal(0.0, 2.5, size=(1, V)).astype(np.float32)
    spikes = g.choice(V, size=min(8, V), replace=False)
    x[0, spikes] = 12.0
    ids = g.integers(0, V, size=64)
    p = SamplingParams(0.6, 0.95, 0.05, 20, 1.1, 0.0, 0.0)
    return _full_window(1, 64, ids, seed, "single_row", p, x, "f32",
                        {"spikes": spikes})


def greedy_bf16(B: int = 256, V: int = VOCAB, seed: int = 2) -> Workload:
    """Greedy argmax, bf16 N(0, 3^2); in 1% of rows (at least one) the row max
    is copied to a second random index so that ties must resolve to the
    lowest index."""
    g = np.random.default_rng(seed)
    x = g.normal(0.0, 3.0, size=(B, V)).astype(np.float32)
    b = to_bf16_bits(x)
    n_tie = max(1, B // 100)
    tie_rows = g.choice(B, size=n_tie, replace=False)
    for r in tie_rows:
        w = widen_bf16(b[r])
        m = int(np.argmax(w))
        j = int(g.integers(0, V))
        while j == m:
            j = int(g.integers(0, V))
        b[r, j] = b[r, m]
    p = SamplingParams(0.0, 1.0, 0.0, 0, 1.0, 0.0, 0.0)
    return _full_window(B, 0, np.zeros(0), seed, "greedy_bf16", p, b, "bf16",
                        {"tie_rows": tie_rows})


def _zipf_ids(g: np.random.Generator, n: int, s: float, V: int) -> np.ndarray:
    out = np.empty(n, dtype=np.int64)
    k = 0
    while k < n:
        z = g.zipf(s, size=2 * (n - k))
        z = z[z <= V]
        take = min(len(z), n - k)
        out[k:k + take] = z[:take]
        k += take
    return out - 1


def nucleus_f32(B: int = 64, V: int = VOCAB, seed: int = 3) -> Workload:
    """fp32 2*Student-t(3); 128-token Zipf(1.1) history (many repeats);
    rp 1.2, freq .5, presence .3; top-k off, top-p .9, min-p 0, T .8."""
    g = np.random.default_rng(seed)
    x = (2.0 * g.standard_t(3.0, size=(B, V))).astype(np.float32)
    ids = _zipf_ids(g, B * 128, 1.1, V)
    p = SamplingParams(0.8, 0.9, 0.0, 0, 1.2, 0.5, 0.3)
    return _full_window(B, 128, ids, seed, "nucleus_f32", p, x, "f32")


def topk_bf16(B: int = 1024, V: int = VOCAB, seed: int = 4,
              row_offset: float = 8.0) -> Workload:
    """bf16 4*Gumbel(0,1) plus a per-row offset drawn U[-8, 8]; 64-token
    uniform history; T .7, k 50, p .95, min-p .1, rp 1.15."""
    g = np.random.default_rng(seed)
    off = g.uniform(-row_offset, row_offset, size=(B, 1)).astype(np.float32)
    x = (4.0 * g.gumbel(0.0, 1.0, size=(B, V))).astype(np.float32) + off
    b = to_bf16_bits(x)
    ids = g.integers(0, V, size=B * 64)
    p = SamplingParams(0.7, 0.95, 0.1, 50, 1.15, 0.0, 0.0)
    return _full_window(B, 64, ids, seed, "topk_bf16", p, b, "bf16")


WORKLOADS = {
    "single_row": single_row,
    "greedy_bf16": greedy_bf16,
    "nucleus_f32": nucleus_f32,
    "topk_bf16": topk_bf16,
}
