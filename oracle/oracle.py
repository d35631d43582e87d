"""ctypes bindings to the CPU checkers — TEST INFRASTRUCTURE ONLY.

* ``Oracle``     — this project's C restatement of the reference sampler
                   (oracle/sampler_oracle.c, run-time V, intermediates).
* ``RefSampler`` — the reference's own sampler.h compiled from its tree
                   (oracle/_ref/libref_sampler.so; V fixed at 151936).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module.
"""
from __future__ import annotations

import ctypes as C
import os
from typing import Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_sampler.so")


class _Params(C.Structure):
    _fields_ = [("temperature", C.c_float), ("topp", C.c_float), ("minp", C.c_float),
                ("top_k", C.c_int), ("repetition_penalty", C.c_float),
                ("frequency_penalty", C.c_float), ("presence_penalty", C.c_float)]


class _Debug(C.Structure):
    _fields_ = [("greedy", C.c_int), ("token", C.c_int), ("n_topk", C.c_int),
                ("n_minp", C.c_int), ("n_final", C.c_int), ("max_logit", C.c_float),
                ("sum", C.c_float), ("r", C.c_float), ("renorm_sum", C.c_float),
                ("probs", C.POINTER(C.c_float)), ("cand_index", C.POINTER(C.c_int)),
                ("cand_prob", C.POINTER(C.c_float)), ("cand_cap", C.c_int)]


def _ptr(a: Optional[np.ndarray], ct):
    if a is None:
        return None
    return a.ctypes.data_as(C.POINTER(ct))


def _params(p) -> _Params:
    return _Params(p.temperature, p.topp, p.minp, int(p.top_k), p.repetition_penalty,
                   p.frequency_penalty, p.presence_penalty)


def build(quiet: bool = True) -> None:
    """Compile the oracle (and oracle/_ref where the reference tree exists)."""
    import subprocess
    subprocess.run(["make", "-s", "-C", HERE], check=True,
                   stdout=subprocess.DEVNULL if quiet else None)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            build()
        self.lib = C.CDLL(path)
        L = self.lib
        L.qso_sample_rows.restype = C.c_int
        L.qso_sample_rows.argtypes = [C.POINTER(_Params), C.POINTER(C.c_float), C.c_int, C.c_int,
                                      C.POINTER(C.c_int), C.POINTER(C.c_float), C.POINTER(C.c_int),
                                      C.c_int, C.POINTER(C.c_uint64), C.POINTER(C.c_int),
                                      C.POINTER(C.c_float), C.POINTER(_Debug)]
        L.qso_random_u32.restype = C.c_uint
        L.qso_random_u32.argtypes = [C.POINTER(C.c_uint64)]
        L.qso_random_f32.restype = C.c_float
        L.qso_random_f32.argtypes = [C.POINTER(C.c_uint64)]

    def random_f32(self, state: int):
        s = C.c_uint64(state)
        v = self.lib.qso_random_f32(C.byref(s))
        return v, s.value

    def sample_rows(self, params, logits_f32: np.ndarray, hist=None, hist_counts=None,
                    hist_count=None, rng=None, want_mutated=False, debug=False,
                    cand_cap: int = 0, want_probs: bool = False):
        """Returns dict(tokens, rng, mutated?, debug?) for a [B, V] fp32 batch."""
        x = np.ascontiguousarray(logits_f32, dtype=np.float32)
        B, V = x.shape
        W = 0 if hist is None else int(hist.shape[1])
        hist = None if hist is None else np.ascontiguousarray(hist, dtype=np.int32)
        hc = None if hist_counts is None else np.ascontiguousarray(hist_counts, dtype=np.float32)
        cnt = None if hist_count is None else np.ascontiguousarray(hist_count, dtype=np.int32)
        st = np.ascontiguousarray(rng if rng is not None else np.ones(B, np.uint64),
                                  dtype=np.uint64).copy()
        out = np.zeros(B, dtype=np.int32)
        mut = np.zeros_like(x) if want_mutated else None
        dbg = None
        keep = []
        if debug:
            dbg = (_Debug * B)()
            for r in range(B):
                if want_probs:
                    pr = np.zeros(V, np.float32)
                    keep.append(pr)
                    dbg[r].probs = _ptr(pr, C.c_float)
                if cand_cap:
                    ci = np.zeros(cand_cap, np.int32)
                    cp = np.zeros(cand_cap, np.float32)
                    keep += [ci, cp]
                    dbg[r].cand_index = _ptr(ci, C.c_int)
                    dbg[r].cand_prob = _ptr(cp, C.c_float)
                    dbg[r].cand_cap = cand_cap
        rc = self.lib.qso_sample_rows(C.byref(_params(params)), _ptr(x, C.c_float), B, V,
                                      _ptr(hist, C.c_int), _ptr(hc, C.c_float), _ptr(cnt, C.c_int),
                                      W, _ptr(st, C.c_uint64), _ptr(out, C.c_int),
                                      _ptr(mut, C.c_float), dbg)
        if rc != 0:
            raise RuntimeError(f"oracle failed: {rc}")
        res = {"tokens": out, "rng": st}
        if want_mutated:
            res["mutated"] = mut
        if debug:
            rows = []
            k = 0
            for r in range(B):
                d = dbg[r]
                row = {"greedy": d.greedy, "token": d.token, "n_topk": d.n_topk,
                       "n_minp": d.n_minp, "n_final": d.n_final, "max": d.max_logit,
                       "sum": d.sum, "r": d.r, "renorm_sum": d.renorm_sum}
                if want_probs:
                    row["probs"] = keep[k]
                    k += 1
                if cand_cap:
                    row["cand_index"] = keep[k]
                    row["cand_prob"] = keep[k + 1]
                    k += 2
                rows.append(row)
            res["debug"] = rows
        return res

    def sample_workload(self, wl, **kw):
        return self.sample_rows(wl.params, wl.logits_f32(), wl.hist, wl.hist_counts,
                                wl.hist_count, wl.rng, **kw)


class RefSampler:
    """The reference's own sampler.h (compiled from the reference tree)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.lib = C.CDLL(path)
        L = self.lib
        L.ref_vocab_size.restype = C.c_int
        L.ref_sample_rows.restype = C.c_int
        L.ref_sample_rows.argtypes = [C.POINTER(C.c_float), C.c_int, C.c_int, C.POINTER(C.c_int),
                                      C.POINTER(C.c_float), C.POINTER(C.c_int), C.POINTER(C.c_int),
                                      C.c_int, C.c_float, C.c_float, C.c_float, C.c_int, C.c_float,
                                      C.c_float, C.c_float, C.POINTER(C.c_uint64),
                                      C.POINTER(C.c_int), C.POINTER(C.c_float), C.c_void_p,
                                      C.c_int]
        L.ref_session_create.restype = C.c_void_p
        L.ref_session_create.argtypes = [C.c_int, C.c_float, C.c_float, C.c_float, C.c_int,
                                         C.c_float, C.c_float, C.c_float, C.c_int,
                                         C.POINTER(C.c_uint64)]
        L.ref_session_step.restype = C.c_int
        L.ref_session_step.argtypes = [C.c_void_p, C.POINTER(C.c_float), C.c_int,
                                       C.POINTER(C.c_int), C.POINTER(C.c_float), C.c_int]
        L.ref_session_set_params.argtypes = [C.c_void_p, C.c_float, C.c_float, C.c_float, C.c_int,
                                             C.c_float, C.c_float, C.c_float]
        L.ref_session_state.argtypes = [C.c_void_p, C.c_int, C.POINTER(C.c_uint64),
                                        C.POINTER(C.c_int), C.POINTER(C.c_int),
                                        C.POINTER(C.c_int), C.c_int]
        L.ref_session_token_count.restype = C.c_float
        L.ref_session_token_count.argtypes = [C.c_void_p, C.c_int, C.c_int]
        L.ref_session_reset.argtypes = [C.c_void_p]
        L.ref_session_free.argtypes = [C.c_void_p]
        L.ref_session_set_rng.argtypes = [C.c_void_p, C.c_int, C.c_uint64]
        self.vocab = L.ref_vocab_size()

    def session(self, params, batch: int, window: int, seeds) -> "RefSession":
        return RefSession(self, params, batch, window, seeds)

    def sample_rows(self, params, logits_f32, hist=None, hist_counts=None, hist_count=None,
                    hist_pos=None, rng=None, want_mutated=False, want_probindex=False,
                    n_threads: int = 1):
        x = np.ascontiguousarray(logits_f32, dtype=np.float32)
        B, V = x.shape
        W = 0 if hist is None else int(hist.shape[1])
        hist = None if hist is None else np.ascontiguousarray(hist, dtype=np.int32)
        hc = None if hist_counts is None else np.ascontiguousarray(hist_counts, dtype=np.float32)
        cnt = None if hist_count is None else np.ascontiguousarray(hist_count, dtype=np.int32)
        pos = None if hist_pos is None else np.ascontiguousarray(hist_pos, dtype=np.int32)
        st = np.ascontiguousarray(rng if rng is not None else np.ones(B, np.uint64),
                                  dtype=np.uint64).copy()
        out = np.zeros(B, dtype=np.int32)
        mut = np.zeros_like(x) if want_mutated else None
        pi = np.zeros((B, V, 2), dtype=np.int32) if want_probindex else None
        rc = self.lib.ref_sample_rows(_ptr(x, C.c_float), B, V, _ptr(hist, C.c_int),
                                      _ptr(hc, C.c_float), _ptr(cnt, C.c_int), _ptr(pos, C.c_int),
                                      W, params.temperature, params.topp, params.minp,
                                      int(params.top_k), params.repetition_penalty,
                                      params.frequency_penalty, params.presence_penalty,
                                      _ptr(st, C.c_uint64), _ptr(out, C.c_int),
                                      _ptr(mut, C.c_float),
                                      None if pi is None else pi.ctypes.data_as(C.c_void_p),
                                      n_threads)
        if rc != 0:
            raise RuntimeError(f"reference sampler rejected the call: {rc}")
        res = {"tokens": out, "rng": st}
        if want_mutated:
            res["mutated"] = mut
        if want_probindex:
            res["prob"] = pi[..., 0].copy().view(np.float32)
            res["index"] = pi[..., 1].copy()
        return res

    def sample_workload(self, wl, **kw):
        return self.sample_rows(wl.params, wl.logits_f32(), wl.hist, wl.hist_counts,
                                wl.hist_count, wl.hist_pos, wl.rng, **kw)


class RefSession:
    """``batch`` persistent reference Samplers driven step by step, as
    main.cu's decode loop drives one (main.cu:136-139): each step samples every
    row and the reference updates the row's history itself (sampler.h:257-267)."""

    def __init__(self, ref: RefSampler, params, batch: int, window: int, seeds):
        self.ref = ref
        self.batch = int(batch)
        self.window = int(window)
        sd = np.ascontiguousarray(np.asarray(seeds, dtype=np.uint64).reshape(-1))
        if sd.shape[0] != self.batch:
            raise ValueError("one seed per row")
        self.h = ref.lib.ref_session_create(self.batch, params.temperature, params.topp,
                                            params.minp, int(params.top_k),
                                            params.repetition_penalty, params.frequency_penalty,
                                            params.presence_penalty, self.window,
                                            _ptr(sd, C.c_uint64))

    def step(self, logits_f32: np.ndarray, n_threads: int = 1) -> np.ndarray:
        x = np.ascontiguousarray(logits_f32, dtype=np.float32)
        out = np.zeros(self.batch, dtype=np.int32)
        rc = self.ref.lib.ref_session_step(self.h, _ptr(x, C.c_float), int(x.shape[1]),
                                           _ptr(out, C.c_int), None, n_threads)
        if rc != 0:
            raise RuntimeError(f"reference session rejected the step: {rc}")
        return out

    def set_params(self, params) -> None:
        self.ref.lib.ref_session_set_params(self.h, params.temperature, params.topp, params.minp,
                                            int(params.top_k), params.repetition_penalty,
                                            params.frequency_penalty, params.presence_penalty)

    def set_rng(self, r: int, state: int) -> None:
        self.ref.lib.ref_session_set_rng(self.h, int(r), C.c_uint64(int(state)))

    def state(self, r: int):
        rng = C.c_uint64()
        cnt = C.c_int()
        pos = C.c_int()
        ring = np.zeros(max(self.window, 1), dtype=np.int32)
        self.ref.lib.ref_session_state(self.h, int(r), C.byref(rng), C.byref(cnt), C.byref(pos),
                                       _ptr(ring, C.c_int), self.window)
        return {"rng": int(rng.value), "count": cnt.value, "pos": pos.value,
                "ring": ring[:self.window].copy()}

    def token_count(self, r: int, token: int) -> float:
        return float(self.ref.lib.ref_session_token_count(self.h, int(r), int(token)))

    def reset(self) -> None:
        self.ref.lib.ref_session_reset(self.h)

    def free(self) -> None:
        if self.h:
            self.ref.lib.ref_session_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def ref_available() -> bool:
    return os.path.exists(REF_SO)
