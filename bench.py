#!/usr/bin/env python
"""Benchmark: sampled rows/s of the B200 token sampler.

Workload (one step = one batch of rows through the whole sampler):
  top-k sampling over bf16 logit rows of the Qwen3-0.6B vocabulary
  (V = 151936), 1024 rows per GPU drawn 4*Gumbel(0,1) plus a per-row offset
  U[-8, 8]; a 64-token window per row drawn uniformly over V; temperature 0.7,
  top-k 50, top-p 0.95, min-p 0.1, repetition penalty 1.15.  Synthetic data
  (the reference publishes no sampler dataset); rows are independent, so
  with N GPUs each rank samples its own 1024 rows (weak scaling) and the
  tokens are gathered to rank 0 on a side stream.

Reported (one JSON line on rank 0):
  value       rows/s of the whole job, logits already in HBM, device time
              (CUDA events on the launching stream, max over ranks); two
              distinct logit buffers (2 x 311 MB, above the 126 MB L2) are
              used in turn so that every step streams its rows from HBM.
  e2e         rows/s through the C ABI with host buffers: each step copies
              its logits, window and RNG states from pinned host memory and
              reads the tokens back.
  roofline    the row kernel's streaming pass: its algorithmic bytes per
              launch (the bf16 logits it must read, 303,872 B per row) over
              its average launch time, against MEASURED_PEAKS.json's HBM copy
              bandwidth.
  cpu_baseline  the reference's own sampler.h (oracle/_ref, compiled from the
              reference tree) on this host's cores, on a bounded sample.

`--impl reference` times that CPU sampler as the job itself (rank 0 only).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

V = 151936
WINDOW = 64
PARAMS = dict(temperature=0.7, topp=0.95, minp=0.1, top_k=50, repetition_penalty=1.15,
              frequency_penalty=0.0, presence_penalty=0.0)
METRIC = "sampled rows/sec @V=151936 (B=1/64/1024), % of HBM roofline, 1/2/4/8 GPU"
WORKLOAD = ("top-k sampling, bf16 logits 4*Gumbel+U[-8,8] per row, V=151936, 1024 rows/GPU, "
            "64-token uniform window, T=0.7 k=50 p=0.95 min-p=0.1 rep=1.15")
ROW_BYTES = V * 2            # logits the streaming pass must read per row (bf16)
STEP_ROW_BYTES = V * 2 + WINDOW * 4   # plus the window ids


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed
    region (read only)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.proc = None
        self.lines = []
        self.t = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100", "-i", str(self.gpu)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for ln in self.proc.stdout:
            self.lines.append(ln.strip())

    def __exit__(self, *a):
        if self.proc:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def cpu_model() -> str:
    try:
        for ln in open("/proc/cpuinfo"):
            if ln.startswith("model name"):
                return ln.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def reference_runner():
    """The reference's own sampler.h (oracle/_ref) over all host threads, or
    the oracle port on one thread where that build is absent.  Returns
    (run(params, x_f32, hist, counts, count, pos, rng) -> tokens, kind,
    threads)."""
    threads = os.cpu_count() or 1
    try:
        from oracle.oracle import RefSampler
        ref = RefSampler()

        def run(params, x, hist, counts, count, pos, rng):
            return ref.sample_rows(params, x, hist, counts, count, pos, rng.copy(),
                                   n_threads=threads)["tokens"]
        return run, "reference", threads
    except Exception:
        from oracle.oracle import Oracle
        o = Oracle()

        def run(params, x, hist, counts, count, pos, rng):
            return o.sample_rows(params, x, hist, counts, count, rng.copy())["tokens"]
        return run, "port", 1


def cpu_leg(params, x, hist, counts, count, rng, gpu_tokens=None, target_s: float = 10.0):
    """The CPU baseline on a bounded sample: the reference sampler on the same
    rows the GPU sampled (fp32 logits as the reference reads them, the same
    windows and initial RNG states), repeated until about `target_s` of wall
    time; its tokens are also compared with the GPU's (parity of the bench's
    own rows)."""
    import numpy as np
    run, kind, threads = reference_runner()
    B = x.shape[0]
    pos = np.zeros(B, np.int32)
    t0 = time.perf_counter()
    toks = run(params, x, hist, counts, count, pos, rng)
    dt = time.perf_counter() - t0
    reps = max(1, min(64, int(target_s / max(dt, 1e-6))))
    t0 = time.perf_counter()
    for _ in range(reps):
        run(params, x, hist, counts, count, pos, rng)
    dt = time.perf_counter() - t0
    out = {"value": reps * B / dt, "unit": "rows/s", "cores": threads, "kind": kind,
           "cpu_model": cpu_model(),
           "sample": f"the same {B} rows the GPU sampled x {reps} passes, {dt:.1f} s on {threads} host threads"}
    if gpu_tokens is not None:
        gt = np.asarray(gpu_tokens)
        out["parity"] = {"rows": int(B), "tokens_equal": int((gt == toks).sum()),
                         "checker": kind}
    return out


def run_reference_arm(args):
    """The reference's own CPU sampler as the job: every step samples the whole
    batch of the benchmark configuration (1024 rows per GPU of the run) on all
    host threads.  Rank 0 alone runs; other ranks exit."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np

    from qwen600_engine_b200 import workloads as W
    run, kind, threads = reference_runner()
    rows = args.batch * max(args.gpus, 1)
    import torch
    # the benchmark workload drawn on the host (make_inputs' recipe on the CPU
    # generator), widened to fp32 outside the timing: the reference reads fp32
    logits, hist, counts, count, rng = make_inputs(torch, rows, 4, torch.device("cpu"))
    x = logits.float().numpy()
    h, c, n = hist.numpy(), counts.numpy(), count.numpy()
    pos = np.zeros(rows, np.int32)
    st = rng.numpy().view(np.uint64)
    params = W.SamplingParams(**PARAMS)

    def one(i):
        run(params, x, h, c, n, pos, st)
    for i in range(args.warmup):
        one(i)
    t0 = time.perf_counter()
    for i in range(args.steps):
        one(i)
    dt = time.perf_counter() - t0
    v = rows * args.steps / dt
    line = {"metric": METRIC, "value": v, "unit": "rows/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * dt / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": {"workload": WORKLOAD, "global_batch": rows, "rows_per_gpu": args.batch,
                       "vocab": V, "window": WINDOW},
            "cpu_baseline": {"value": v, "unit": "rows/s", "cores": threads, "kind": kind,
                             "cpu_model": cpu_model(),
                             "sample": f"the whole batch of {rows} rows per step x {args.steps} steps"},
            "e2e": {"value": v, "unit": "rows/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def measure_lm_head(torch, dev, B=128, K=1024, iters=20):
    """RMSNorm + lm_head (qs_lm_head) at configuration 5, and the same plus
    sampling (qs_lm_head_sample with history): CUDA events over `iters`
    launches alternating two W copies (622 MB, larger than L2)."""
    from qwen600_engine_b200 import _lib
    from qwen600_engine_b200.sampler import Sampler
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    h = torch.randn((B, K), generator=g, device=dev).to(torch.bfloat16)
    ws = [(0.02 * torch.randn((V, K), generator=g, device=dev)).to(torch.bfloat16) for _ in range(2)]
    normed = torch.empty((B, K), dtype=torch.bfloat16, device=dev)
    logits = torch.empty((B, V), dtype=torch.bfloat16, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream()

    def one(i):
        _lib.check(_lib.lib.qs_lm_head(h.data_ptr(), None, ws[i % 2].data_ptr(), B, K, V,
                                       normed.data_ptr(), logits.data_ptr(), err.data_ptr(),
                                       st.cuda_stream))
    for i in range(3):
        one(i)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(st)
    for i in range(iters):
        one(i)
    b.record(st)
    torch.cuda.synchronize()
    us = 1e3 * a.elapsed_time(b) / iters
    s = Sampler(0.6, 0.95, 0.05, 20, 1.1, 0.0, 0.0, 64, 1, max_batch=B, device=dev.index or 0)
    for i in range(3):
        s.lm_head_sample(h, ws[i % 2])
    torch.cuda.synchronize()
    a.record(st)
    for i in range(iters):
        s.lm_head_sample(h, ws[i % 2])
    b.record(st)
    torch.cuda.synchronize()
    us_s = 1e3 * a.elapsed_time(b) / iters
    s.lm_head_status()
    s.free()
    hbm, kind = peaks()
    byts = V * K * 2 + B * V * 2 + 2 * B * K * 2
    flops = 2.0 * B * K * V
    return {"config": f"hidden [{B},{K}] bf16 -> RMSNorm -> W [{V},{K}] bf16 (random N(0,0.02^2)), fp32 accumulate, bf16 logits",
            "us_per_launch": us, "achieved_GBps": byts / (us * 1e-6) / 1e9, "peak_GBps": hbm,
            "frac": byts / (us * 1e-6) / 1e9 / hbm, "algorithmic_bytes": byts,
            "tflops": flops / (us * 1e-6) / 1e12, "error_flag": int(err.item()),
            "with_sampling_us": us_s, "sampling_rows_per_s": B / (us_s * 1e-6),
            "note": "random weights give flat logits (std 0.64): every row takes the dense softmax "
                    "path and ~16% of rows the tie-order pass"}


def measure_lm_head_sharded(torch, dev, rank, world, B=128, K=1024, iters=20):
    """The decode tail of configuration 5 on `world` GPUs, vocabulary-sharded
    (shard.VocabShardedLmHead): each rank streams its slice of W, stores each
    row's logits into the rank that samples it, then samples its row block
    (64-token windows, temperature 0.6, top-k 20, top-p 0.95, min-p 0.05,
    repetition penalty 1.1).  CUDA events per rank, the slowest rank's time;
    slice copies used in turn so that together they exceed L2."""
    from qwen600_engine_b200 import shard
    from qwen600_engine_b200.sampler import Sampler
    c0, n = shard.vocab_shard(rank, world, V)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    h = torch.randn((B, K), generator=g, device=dev).to(torch.bfloat16)
    ncopy = max(2, -(-300_000_000 // (n * K * 2)))
    gw = torch.Generator(device=dev)
    gw.manual_seed(6 + rank)
    ws = [(0.02 * torch.randn((n, K), generator=gw, device=dev)).to(torch.bfloat16) for _ in range(ncopy)]
    head = shard.VocabShardedLmHead(ws[0], c0, V, B, rank=rank, world=world)
    a_, b_ = shard.row_block(rank, world, B)
    rows_n = b_ - a_
    s = Sampler(0.6, 0.95, 0.05, 20, 1.1, 0.0, 0.0, 64, 1, max_batch=max(rows_n, 1), device=dev.index or 0)
    hist = torch.randint(0, V, (max(rows_n, 1), 64), generator=g, device=dev, dtype=torch.int32)
    cnt = torch.full((max(rows_n, 1),), 64, device=dev, dtype=torch.int32)
    rng = torch.arange(max(rows_n, 1), device=dev, dtype=torch.int64) + 1 + a_
    tok = torch.empty(max(rows_n, 1), dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream()

    def one(i, sample):
        rows = head(h, weight=ws[i % ncopy])
        if sample and rows_n:
            s.sample_rows(rows, hist[:rows_n], None, cnt[:rows_n], rng[:rows_n], out=tok[:rows_n])

    res = {}
    for sample in (False, True):
        for i in range(3):
            one(i, sample)
        torch.cuda.synchronize()
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(st)
        for i in range(iters):
            one(i, sample)
        ev1.record(st)
        torch.cuda.synchronize()
        res[sample] = shard.max_over_ranks(1e3 * ev0.elapsed_time(ev1) / iters, device=dev)
    head.status()
    head.close()
    s.free()
    byts = V * K * 2 + B * V * 2
    return {"config": f"hidden [{B},{K}] bf16 replicated -> RMSNorm -> W [{V},{K}] bf16 split by vocabulary "
                      f"over {world} GPUs ({n} rows each), logits rows stored to their sampling GPU over NVLink",
            "us_per_step": res[False], "with_sampling_us": res[True],
            "rows_per_s_with_sampling": B / (res[True] * 1e-6),
            "whole_job_GBps": byts / (res[False] * 1e-6) / 1e9,
            "note": "max over ranks of CUDA-event time; the step includes the completion handshake "
                    "(device-side flag words over NVLink, qs_shard_handshake)"}


def _wl_to_dev(torch, wl, dev):
    """A workload's logits, window and RNG states as device tensors."""
    import numpy as np
    if wl.dtype == "bf16":
        x = torch.from_numpy(wl.logits.view(np.int16)).to(dev).view(torch.bfloat16)
    else:
        x = torch.from_numpy(np.ascontiguousarray(wl.logits)).to(dev)
    d = {"x": x, "rng": torch.from_numpy(wl.rng.view(np.int64).copy()).to(dev)}
    if wl.window > 0:
        d["hist"] = torch.from_numpy(wl.hist.astype(np.int32)).to(dev)
        d["counts"] = torch.from_numpy(wl.hist_counts.astype(np.float32)).to(dev)
        d["count"] = torch.from_numpy(wl.hist_count.astype(np.int32)).to(dev)
    else:
        d["hist"] = d["counts"] = d["count"] = None
    return d


def _stack(wls):
    """One workload holding the rows of several (same parameters)."""
    import numpy as np
    from qwen600_engine_b200 import workloads as W
    w0 = wls[0]
    return W.Workload(w0.name, w0.params, np.concatenate([w.logits for w in wls]), w0.dtype,
                      np.concatenate([w.hist for w in wls]), np.concatenate([w.hist_counts for w in wls]),
                      np.concatenate([w.hist_count for w in wls]), np.concatenate([w.hist_pos for w in wls]),
                      np.concatenate([w.rng for w in wls]), w0.window)


def _sampler_for(wl, B, dev):
    from qwen600_engine_b200.sampler import Sampler
    p = wl.params
    return Sampler(p.temperature, p.topp, p.minp, p.top_k, p.repetition_penalty,
                   p.frequency_penalty, p.presence_penalty, wl.window, 1, max_batch=B,
                   vocab=wl.vocab, device=dev.index or 0)


def _kernel_split(s, run_pass, steps):
    """Per-kernel CUDA-event times of `steps` more steps (a separate pass)."""
    import torch
    s.profile(True)
    s.profile_reset()
    run_pass()
    torch.cuda.synchronize()
    pr = s.profile_read()
    s.profile(False)
    return {"stream_ms": pr["stream_ms"] / steps, "finish_ms": pr["finish_ms"] / steps,
            "ties_ms": pr["ties_ms"] / steps, "emit_ms": pr["emit_ms"] / steps}


def measure_configs(torch, dev, steps: int, warmup: int, cpu: bool = True):
    """The other configurations of the headline metric, each on one GPU with
    its own synthetic inputs (qwen600_engine_b200.workloads), timed with CUDA
    events on the launching stream over distinct input buffers whose total
    exceeds L2, and checked against the reference sampler on the same rows:

      1  batch 1, fp32 N(0, 2.5^2) + 8 spikes at +12, 64-token window, k 20:
         latency of one sampling call (256 distinct rows, each sampled once
         in the timed pass; its tokens are the parity tokens)
      2  batch 256, bf16 N(0, 3^2) with duplicate maxima, greedy
      3  batch 64, fp32 2*Student-t(3), 128-token Zipf window with frequency
         and presence penalties, top-k off, top-p 0.9 (full-vocabulary nucleus)
    """
    import numpy as np
    from qwen600_engine_b200 import workloads as W
    hbm, peak_kind = peaks()
    st = torch.cuda.current_stream()
    out = {}

    def ev_time(fn, n):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(st)
        for i in range(n):
            fn(i)
        b.record(st)
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    def roofline(B, row_bytes, ms, bound):
        ach = B * row_bytes / (ms * 1e-3) / 1e9
        return {"bound": bound, "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm,
                "algorithmic_bytes_per_step": B * row_bytes, "peak_source": peak_kind}

    # ---- configuration 1: one row per call
    rows = _stack([W.single_row(seed=s_) for s_ in range(1, 257)])
    d = _wl_to_dev(torch, rows, dev)
    s = _sampler_for(rows, 1, dev)
    toks = torch.empty(rows.batch, dtype=torch.int32, device=dev)
    rng_w = d["rng"].clone()

    def c1(i, rng=d["rng"]):
        j = i % rows.batch
        s.sample_rows(d["x"][j:j + 1], d["hist"][j:j + 1], d["counts"][j:j + 1], d["count"][j:j + 1],
                      rng[j:j + 1], out=toks[j:j + 1])
    for i in range(max(warmup, 3)):
        c1(i, rng_w)
    torch.cuda.synchronize()
    ms = ev_time(c1, rows.batch)
    gpu_t = toks.cpu().numpy()
    ks = _kernel_split(s, lambda: [c1(i, rng_w) for i in range(64)], 64)
    s.free()
    ent = {"workload": "batch 1, fp32 N(0,2.5^2) + 8 spikes at +12 (256 distinct rows in turn, 155 MB), "
                       "64-token window, T=0.6 k=20 p=0.95 min-p=0.05 rep=1.1",
           "us_per_row": 1e3 * ms, "rows_per_s": 1e3 / ms,
           "roofline": roofline(1, V * 4 + 64 * 4, ms, "latency (one row)"), "kernel_ms_per_call": ks}
    if cpu:
        ent["cpu_baseline"] = cpu_leg(rows.params, rows.logits, rows.hist, rows.hist_counts, rows.hist_count,
                                      rows.rng, gpu_t, target_s=3.0)
    out["1"] = ent
    del d

    # ---- configurations 2 and 3: whole batches, buffers used in turn
    for name, mk, nbuf, row_bytes, label in (
            ("2", lambda sd: W.greedy_bf16(B=256, seed=sd), 4, V * 2,
             "batch 256, bf16 N(0,3^2), 1% rows with duplicate maxima, greedy (4 buffers in turn, 311 MB)"),
            ("3", lambda sd: W.nucleus_f32(B=64, seed=sd), 8, V * 4 + 128 * 4,
             "batch 64, fp32 2*Student-t(3), 128-token Zipf(1.1) window, rep 1.2 freq 0.5 pres 0.3, "
             "top-k off, top-p 0.9, T 0.8 (8 buffers in turn, 311 MB)")):
        seed0 = int(name)
        wls = [mk(seed0 + 100 * k) for k in range(nbuf)]
        ds = [_wl_to_dev(torch, w, dev) for w in wls]
        B = wls[0].batch
        s = _sampler_for(wls[0], B, dev)
        toks = torch.empty(B, dtype=torch.int32, device=dev)
        rng0 = ds[0]["rng"].clone()
        s.sample_rows(ds[0]["x"], ds[0]["hist"], ds[0]["counts"], ds[0]["count"], rng0, out=toks)
        gpu_t = toks.cpu().numpy()
        rng_w = ds[0]["rng"].clone()

        def cn(i):
            dd = ds[i % nbuf]
            s.sample_rows(dd["x"], dd["hist"], dd["counts"], dd["count"], rng_w, out=toks)
        for i in range(max(warmup, 3)):
            cn(i)
        torch.cuda.synchronize()
        ms = ev_time(cn, steps)
        ks = _kernel_split(s, lambda: [cn(i) for i in range(steps)], steps)
        s.free()
        ent = {"workload": label, "batch": B, "ms_per_step": ms, "rows_per_s": B / (ms * 1e-3),
               "roofline": roofline(B, row_bytes, ms, "hbm"), "kernel_ms_per_step": ks}
        if cpu:
            w0 = wls[0]
            ent["cpu_baseline"] = cpu_leg(w0.params, w0.logits_f32(), w0.hist if w0.window else None,
                                          w0.hist_counts if w0.window else None,
                                          w0.hist_count if w0.window else None, w0.rng, gpu_t,
                                          target_s=3.0)
        out[name] = ent
        del ds
    torch.cuda.empty_cache()
    return out


def make_inputs(torch, B, seed, device):
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    u = torch.rand((B, V), generator=g, device=device, dtype=torch.float32).clamp_(1e-12, 1 - 1e-7)
    off = (torch.rand((B, 1), generator=g, device=device) * 16.0 - 8.0)
    logits = (4.0 * (-torch.log(-torch.log(u))) + off).to(torch.bfloat16)
    del u
    hist = torch.randint(0, V, (B, WINDOW), generator=g, device=device, dtype=torch.int32)
    counts = torch.ones((B, WINDOW), device=device, dtype=torch.float32)
    count = torch.full((B,), WINDOW, device=device, dtype=torch.int32)
    rng = (torch.arange(B, device=device, dtype=torch.int64) + seed * 1000003 + 1)
    return logits, hist, counts, count, rng


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--batch", type=int, default=1024, help="rows per GPU")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-configs", dest="configs", action="store_false",
                    help="skip configurations 1-3 (batch 1 fp32, batch 256 greedy, batch 64 nucleus)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--no-lm-head", dest="lm_head", action="store_false",
                    help="skip the RMSNorm + lm_head measurement")
    ap.add_argument("--only-lm-head", action="store_true",
                    help="one GPU: run only the decode-tail measurement (configuration 5) and print it")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.only_lm_head:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps({"lm_head": measure_lm_head(torch, torch.device("cuda", 0))}), flush=True)
        return 0

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import numpy as np

    from qwen600_engine_b200 import shard
    from qwen600_engine_b200.sampler import Sampler

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    B = args.batch

    bufs = [make_inputs(torch, B, 4 + 7919 * rank + 104729 * i, dev) for i in range(2)]
    hist, counts, count = bufs[0][1], bufs[0][2], bufs[0][3]
    # this rank's block of the world x B batch keeps the global rows' RNG streams
    a, b = shard.row_block(rank, world, world * B)
    rng = torch.from_numpy(shard.row_seeds(4, a, b).view(np.int64)).to(dev)
    toks = [torch.empty(B, dtype=torch.int32, device=dev) for _ in range(2)]
    # tokens to rank 0 without a collective: peer copies into rank 0's buffer
    # and the device-side flag handshake (shard.TokenGather)
    tg = shard.TokenGather(world * B, rank=rank, world=world, device=dev) if world > 1 else None
    # two independent batches in flight, each with its own handle (scratch)
    # and stream: batch i runs on handle/stream i % 2, so one batch's
    # latency-bound passes (finishing, tie replay) overlap the next batch's
    # HBM-bound streaming pass.  The one-batch-at-a-time latency is measured
    # too (handle 0 alone on the launching stream).
    ss = [Sampler(PARAMS["temperature"], PARAMS["topp"], PARAMS["minp"], PARAMS["top_k"],
                  PARAMS["repetition_penalty"], PARAMS["frequency_penalty"],
                  PARAMS["presence_penalty"], WINDOW, 1, max_batch=B, vocab=V, device=local)
          for _ in range(2)]
    s = ss[0]
    main_stream = torch.cuda.current_stream()
    streams = [main_stream, torch.cuda.Stream()]
    rngs = [rng, rng.clone()]
    gstream = torch.cuda.Stream() if world > 1 else None
    gdone = [torch.cuda.Event(), torch.cuda.Event()]

    def step(i, nflight=2):
        j = i % 2
        k = i % nflight
        st = streams[k]
        if world > 1 and i >= 2:
            st.wait_event(gdone[j])
        with torch.cuda.stream(st):
            ss[k].sample_rows(bufs[j][0], hist, counts, count, rngs[k], out=toks[j], stream=st)
        if world > 1:
            ev = torch.cuda.Event()
            ev.record(st)
            with torch.cuda.stream(gstream):
                gstream.wait_event(ev)
                tg(toks[j], stream=gstream)
                gdone[j].record(gstream)

    def join():
        for st in streams[1:]:
            main_stream.wait_stream(st)
        if gstream is not None:
            main_stream.wait_stream(gstream)

    def sync_all():
        join()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    rng_init = rng.clone()
    for i in range(max(args.warmup, 2)):
        step(i)
    sync_all()

    def timed(nflight):
        # device time on the launching stream; the other stream starts after t0
        # and the launching stream waits for it before t1
        p0 = [h.profile_read()["launches"] for h in ss]
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(main_stream)
        for st in streams[1:]:
            st.wait_stream(main_stream)
        for i in range(args.steps):
            step(i, nflight)
        join()
        t1.record(main_stream)
        torch.cuda.synchronize()
        nl = sum(int(h.profile_read()["launches"] - a) for h, a in zip(ss, p0))
        return t0.elapsed_time(t1), nl

    # ---- one batch at a time (latency per batch)
    ms1, _ = timed(1)
    sync_all()
    if world > 1:
        ms1 = shard.max_over_ranks(ms1, device=dev)
    latency_ms = ms1 / args.steps
    # ---- timed region: two batches in flight (throughput)
    with ClockSampler(local) as clk:
        ms, launches = timed(2)
    if tg is not None:
        launches += args.steps  # one handshake kernel per step
    sync_all()
    if world > 1:
        ms = shard.max_over_ranks(ms, device=dev)
    ms_step = ms / args.steps
    value = world * B / (ms_step / 1e3)

    # ---- per-kernel timing of the same steps (separate pass, one batch at a
    # time on handle 0, events around each kernel)
    s.profile(True)
    s.profile_reset()
    for i in range(args.steps):
        step(i, 1)
    sync_all()
    pr = s.profile_read()
    s.profile(False)
    kms = {"stream_ms": pr["stream_ms"] / args.steps, "finish_ms": pr["finish_ms"] / args.steps,
           "ties_ms": pr["ties_ms"] / args.steps, "emit_ms": pr["emit_ms"] / args.steps}
    row_ms = pr["stream_ms"] / max(pr["row_launches"], 1)  # the streaming pass: every logit once
    hbm, peak_kind = peaks()
    stream_ach = B * ROW_BYTES / (row_ms / 1e3) / 1e9
    step_ach = B * STEP_ROW_BYTES / (ms_step / 1e3) / 1e9
    traffic = None
    tfile = os.path.join(ROOT, "profiles", "launches_topk_bf16_b1024.md")
    if os.path.exists(tfile):
        for ln in open(tfile):
            if ln.startswith("dram_bytes_per_step_B1024:"):
                try:
                    traffic = float(ln.split(":", 1)[1].split()[0])
                except ValueError:
                    pass

    # ---- the GPU's tokens for buffer 0 from the initial RNG states: checked
    # against the reference in the CPU-baseline leg below
    parity_tokens = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rng_p = rng_init.clone()
        tok_p = torch.empty(B, dtype=torch.int32, device=dev)
        s.sample_rows(bufs[0][0], hist, counts, count, rng_p, out=tok_p)
        parity_tokens = tok_p.cpu().numpy()

    # ---- end to end through the C ABI with host buffers
    e2e = None
    if args.e2e_steps > 0:
        h_logits = [bufs[i][0].cpu().pin_memory() for i in range(2)]
        h_hist, h_counts, h_count = hist.cpu().pin_memory(), counts.cpu().pin_memory(), count.cpu().pin_memory()
        h_rng = rng.cpu().pin_memory()
        h_tok = torch.empty(B, dtype=torch.int32).pin_memory()

        def e2e_step(i):
            # the C ABI's host-buffer entry: logits, window and RNG states in,
            # tokens and advanced states out, all through host memory
            s.sample_rows_host(h_logits[i % 2], h_hist, h_counts, h_count, h_rng, out=h_tok,
                               stream=main_stream, synchronize=False)

        e2e_step(0)
        sync_all()
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        a.record(main_stream)
        for i in range(args.e2e_steps):
            e2e_step(i)
        b.record(main_stream)
        torch.cuda.synchronize()
        ems = a.elapsed_time(b)
        if world > 1:
            ems = shard.max_over_ranks(ems, device=dev)
        h2d = (bufs[0][0].numel() * 2 + hist.numel() * 4 + counts.numel() * 4 + count.numel() * 4
               + rng.numel() * 8)
        e2e = {"value": world * B / (ems / args.e2e_steps / 1e3), "unit": "rows/s",
               "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(B * (4 + 8)),
               "steps": args.e2e_steps,
               "path": "pinned host -> qs_sample_rows_host (C ABI; tokens and RNG states back) -> host"}

    # ---- the decode tail (final RMSNorm + lm_head, hidden [128, 1024] bf16):
    # 128 hidden rows x W [151936, 1024] bf16, two weight copies used in turn
    lmh = None
    if rank == 0 and world == 1 and args.lm_head:
        lmh = measure_lm_head(torch, dev)
    if world > 1 and args.lm_head:
        lmh = measure_lm_head_sharded(torch, dev, rank, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            from qwen600_engine_b200 import workloads as W
            cpu = cpu_leg(W.SamplingParams(**PARAMS), bufs[0][0].float().cpu().numpy(),
                          hist.cpu().numpy(), counts.cpu().numpy(), count.cpu().numpy(),
                          rng_init.cpu().numpy().view(np.uint64), parity_tokens)
        except Exception as exc:  # report, do not fail the GPU measurement
            cpu = {"value": None, "error": str(exc)}

    configs = None
    if rank == 0 and world == 1 and args.configs:
        configs = measure_configs(torch, dev, steps=max(args.steps, 20), warmup=args.warmup,
                                  cpu=not args.no_cpu_baseline)

    if tg is not None:
        tg.status()
        tg.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": value, "unit": "rows/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
        "batches_in_flight": 2, "latency_ms_per_batch": latency_ms,
        "rows_per_s_one_batch_in_flight": world * B / (latency_ms / 1e3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": WORKLOAD, "global_batch": world * B, "rows_per_gpu": B,
                   "vocab": V, "window": WINDOW, "seq_len": None,
                   "parallelism": f"row-sharded x{world}, tokens copied to rank 0 over NVLink with a device-side "
                                  "handshake (no NCCL in the timed region); per GPU two independent batches in "
                                  "flight (two handles, two streams)",
                   "l2": "inputs larger than L2: two 311 MB logit buffers used in turn"},
        "e2e": e2e,
        "roofline": {"bound": "hbm", "achieved": step_ach, "peak": hbm, "unit": "GB/s",
                     "frac": step_ach / hbm, "traffic": traffic, "peak_source": peak_kind,
                     "kernel": "the sampling step (streaming, finishing, tie-replay and emit kernels)",
                     "algorithmic_bytes_per_step": B * STEP_ROW_BYTES,
                     "row_kernel": {"kernel": "qs::wide::row_stream_kernel<bf16> (the streaming pass)",
                                    "kernel_ms": row_ms, "achieved": stream_ach, "frac": stream_ach / hbm,
                                    "algorithmic_bytes_per_launch": B * ROW_BYTES}},
        "kernel_ms_per_step": kms,
        "tie_clusters": int(pr.get("tie_clusters", 0)),
        "dominant_kernel": max(kms, key=kms.get).replace("_ms", ""),
        "cpu_baseline": cpu,
        "lm_head": lmh,
        "configs": configs,
        "clocks": clk.summary(),
        "gpu_launches": launches,
    }
    print(json.dumps(line), flush=True)
    for h in ss:
        h.free()
    return 0


if __name__ == "__main__":
    sys.exit(main())
