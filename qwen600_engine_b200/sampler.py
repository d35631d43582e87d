"""Host-side mirror of the reference sampler interface, over the C ABI.

Reference interface (KennethWang1221/qwen600_engine):
  * sampler.h:21-43      ``Sampler`` fields (temperature, topp, minp, top_k,
                         repetition/frequency/presence penalty, window, rng)
  * sampler.h:277-327    ``build_sampler(...)``
  * sampler.h:165-270    ``sample(sampler, logits) -> token``
  * sampler.h:346-354    ``reset_sampler_history(sampler)``
  * sampler.h:330-343    ``free_sampler(sampler)``
  * python/qwen_engine/qwen_inference.py:22-72  ``SamplingConfig``
  * python/bindings.cu:213-239  parameter updates between calls

Differences a caller sees: a ``Sampler`` here is batched (``max_batch``
independent sequences, row r seeded ``rng_seed + r``), logits live on the GPU
(torch tensors, fp32 or bf16, shape [B, V] or [V]) and errors raise
``SamplerError`` instead of exiting the process.  Device memory and streams
come from PyTorch; all computation runs in the CUDA library.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Any, Dict, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import (QS_BF16, QS_F32, QS_FLAG_INDEX_TIES, QS_FLAG_WRITE_PENALIZED, Params,
                   RowDebug, SamplerError, check)

VOCAB_SIZE = 151936  # reference config.h:52


@dataclass
class SamplingConfig:
    """Same fields and defaults as the reference's SamplingConfig
    (python/qwen_engine/qwen_inference.py:22-72)."""

    temperature: float = 0.6
    top_k: int = 20
    top_p: float = 0.95
    min_p: float = 0.05
    repetition_penalty: float = 1.1
    frequency_penalty: float = 0.0
    presence_penalty: float = 0.0
    penalty_window: int = 64
    max_tokens: int = 512
    seed: Optional[int] = None
    reasoning_mode: int = 0

    def to_dict(self) -> Dict[str, Any]:
        return {
            "temperature": self.temperature, "top_k": self.top_k, "top_p": self.top_p,
            "min_p": self.min_p, "repetition_penalty": self.repetition_penalty,
            "frequency_penalty": self.frequency_penalty,
            "presence_penalty": self.presence_penalty, "penalty_window": self.penalty_window,
            "max_tokens": self.max_tokens, "seed": self.seed if self.seed is not None else -1,
            "reasoning_mode": self.reasoning_mode,
        }


def _torch():
    import torch
    return torch


def _dtype_code(t) -> int:
    torch = _torch()
    if t.dtype == torch.float32:
        return QS_F32
    if t.dtype == torch.bfloat16:
        return QS_BF16
    raise SamplerError(_lib.QS_ERR_INVALID, f"logits dtype {t.dtype} (want float32 or bfloat16)")


def _stream_handle(stream) -> Optional[int]:
    torch = _torch()
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _ptr(t) -> Optional[int]:
    return None if t is None else int(t.data_ptr())


class Sampler:
    """A batch of ``max_batch`` independent reference samplers on one GPU."""

    _FIELDS = ("temperature", "topp", "minp", "top_k", "repetition_penalty",
               "frequency_penalty", "presence_penalty")

    def __init__(self, temperature=0.6, topp=0.95, minp=0.05, top_k=20,
                 repetition_penalty=1.1, frequency_penalty=0.0, presence_penalty=0.0,
                 penalty_window_size=64, rng_seed=1, *, max_batch: int = 1,
                 vocab: int = VOCAB_SIZE, device: int = 0):
        p = Params(float(temperature), float(topp), float(minp), int(top_k),
                   float(repetition_penalty), float(frequency_penalty), float(presence_penalty))
        h = C.c_void_p()
        check(_lib.lib.qs_build_sampler(C.byref(h), C.byref(p), int(max_batch), int(vocab),
                                        int(max(penalty_window_size, 0)),
                                        C.c_ulonglong(int(rng_seed) & 0xFFFFFFFFFFFFFFFF),
                                        int(device)))
        self._h = h
        self.max_batch = int(max_batch)
        self.vocab = int(vocab)
        self.window = int(max(penalty_window_size, 0))
        self.device = int(device)

    # -- parameter fields, written like bindings.cu:213-235 writes Sampler fields
    def _params(self) -> Params:
        p = Params()
        check(_lib.lib.qs_get_params(self._h, C.byref(p)))
        return p

    def __getattr__(self, name):
        if name in Sampler._FIELDS:
            return getattr(self._params(), name)
        raise AttributeError(name)

    def __setattr__(self, name, value):
        if name in Sampler._FIELDS:
            p = self._params()
            setattr(p, name, int(value) if name == "top_k" else float(value))
            check(_lib.lib.qs_set_params(self._h, C.byref(p)))
        else:
            object.__setattr__(self, name, value)

    def set_params(self, **kw) -> None:
        p = self._params()
        for k, v in kw.items():
            if k not in Sampler._FIELDS:
                raise KeyError(k)
            setattr(p, k, int(v) if k == "top_k" else float(v))
        check(_lib.lib.qs_set_params(self._h, C.byref(p)))

    @property
    def rng_state(self) -> np.ndarray:
        out = np.zeros(self.max_batch, dtype=np.uint64)
        check(_lib.lib.qs_get_rng_state(self._h, out.ctypes.data_as(C.POINTER(C.c_ulonglong)),
                                        self.max_batch))
        return out

    @rng_state.setter
    def rng_state(self, states: Sequence[int]) -> None:
        arr = np.ascontiguousarray(np.asarray(states, dtype=np.uint64).reshape(-1))
        check(_lib.lib.qs_set_rng_state(self._h, arr.ctypes.data_as(C.POINTER(C.c_ulonglong)),
                                        int(arr.shape[0])))

    # -- sampling
    def sample(self, logits, out=None, *, flags: int = 0, stream=None):
        """Stateful sample() over the rows of ``logits`` ([B, V] or [V] device
        tensor); returns int32 tokens [B] on the device."""
        torch = _torch()
        x = logits if logits.dim() == 2 else logits.view(1, -1)
        if not x.is_cuda or not x.is_contiguous():
            raise SamplerError(_lib.QS_ERR_INVALID, "logits must be a contiguous CUDA tensor")
        B = int(x.shape[0])
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=x.device)
        check(_lib.lib.qs_sample(self._h, _ptr(x), _dtype_code(x), B, _ptr(out),
                                 _stream_handle(stream), int(flags)))
        return out

    def sample_host(self, logits: np.ndarray, *, flags: int = 0) -> np.ndarray:
        """Host-buffer entry (fp32 numpy [B, V]); returns numpy int32 tokens."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        if x.ndim == 1:
            x = x.reshape(1, -1)
        out = np.zeros(x.shape[0], dtype=np.int32)
        check(_lib.lib.qs_sample_host(self._h, x.ctypes.data, int(x.shape[0]), out.ctypes.data,
                                      int(flags)))
        return out

    def sample_rows_host(self, logits, hist=None, hist_counts=None, hist_count=None, rng=None,
                         out=None, *, flags: int = 0, stream=None, synchronize: bool = True):
        """sample_rows with host (CPU, ideally pinned) tensors: logits [B, V]
        float32/bfloat16, the caller's window, rng int64 [B] (advanced in
        place); returns int32 tokens [B] on the host.  The copies and the
        sampling are enqueued on ``stream``; with ``synchronize`` the call
        waits for them."""
        torch = _torch()
        x = logits if logits.dim() == 2 else logits.view(1, -1)
        if x.is_cuda or not x.is_contiguous():
            raise SamplerError(_lib.QS_ERR_INVALID, "logits must be a contiguous host tensor")
        if rng is None or rng.is_cuda:
            raise SamplerError(_lib.QS_ERR_INVALID, "rng states must be a host tensor (int64 [B])")
        B, V = int(x.shape[0]), int(x.shape[1])
        if out is None:
            out = torch.empty(B, dtype=torch.int32)
        W = 0 if hist is None else int(hist.shape[1])
        check(_lib.lib.qs_sample_rows_host(
            self._h, _ptr(x), _dtype_code(x), B, V, _ptr(hist), _ptr(hist_counts), _ptr(hist_count), W,
            _ptr(rng), _ptr(out), _stream_handle(stream), int(flags)))
        if synchronize:
            (stream if stream is not None else torch.cuda.current_stream()).synchronize()
        return out

    def sample_rows(self, logits, hist=None, hist_counts=None, hist_count=None, rng=None,
                    out=None, *, debug: bool = False, probs: bool = False, cand_cap: int = 0,
                    flags: int = 0, stream=None):
        """Stateless batched sampling with caller history (device tensors).
        Returns tokens, or a dict with tokens and the requested diagnostics."""
        torch = _torch()
        x = logits if logits.dim() == 2 else logits.view(1, -1)
        B, V = int(x.shape[0]), int(x.shape[1])
        dev = x.device
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=dev)
        if rng is None:
            raise SamplerError(_lib.QS_ERR_INVALID, "rng states tensor (uint64/int64 [B]) required")
        W = 0 if hist is None else int(hist.shape[1])
        dbg = torch.zeros((B, C.sizeof(RowDebug) // 4), dtype=torch.int32, device=dev) if debug else None
        pr = torch.empty((B, V), dtype=torch.float32, device=dev) if probs else None
        ci = torch.full((B, cand_cap), -1, dtype=torch.int32, device=dev) if cand_cap else None
        cp = torch.zeros((B, cand_cap), dtype=torch.float32, device=dev) if cand_cap else None
        check(_lib.lib.qs_sample_rows_debug(
            self._h, _ptr(x), _dtype_code(x), B, V, _ptr(hist), _ptr(hist_counts),
            _ptr(hist_count), W, _ptr(rng), _ptr(out), _ptr(dbg), _ptr(pr), _ptr(ci), _ptr(cp),
            int(cand_cap), _stream_handle(stream), int(flags)))
        if not (debug or probs or cand_cap):
            return out
        res = {"tokens": out}
        if debug:
            res["debug"] = decode_debug(dbg)
        if probs:
            res["probs"] = pr
        if cand_cap:
            res["cand_index"] = ci
            res["cand_prob"] = cp
        return res

    # -- kernel timing (for benchmarks)
    def lm_head_sample(self, hidden, weight, norm_weight=None, out=None, *, flags: int = 0,
                       stream=None):
        """Final RMSNorm + lm_head + stateful sample() for the rows of
        ``hidden`` (bf16 [B, hidden_dim] device tensor; ``weight`` bf16
        [vocab, hidden_dim]); returns int32 tokens [B] on the device."""
        torch = _torch()
        h = hidden if hidden.dim() == 2 else hidden.view(1, -1)
        for t in (h, weight) + ((norm_weight,) if norm_weight is not None else ()):
            if not t.is_cuda or not t.is_contiguous() or t.dtype != torch.bfloat16:
                raise SamplerError(_lib.QS_ERR_INVALID, "hidden, weight and norm_weight must be "
                                   "contiguous bf16 CUDA tensors")
        B = int(h.shape[0])
        if out is None:
            out = torch.empty(B, dtype=torch.int32, device=h.device)
        check(_lib.lib.qs_lm_head_sample(self._h, _ptr(h), _ptr(norm_weight), _ptr(weight), B,
                                         int(h.shape[1]), _ptr(out), _stream_handle(stream),
                                         int(flags)))
        return out

    def lm_head_logits(self, batch: int):
        """The bf16 logits [batch, vocab] the last lm_head_sample produced (a
        view of the handle's workspace)."""
        torch = _torch()
        p = C.c_void_p()
        check(_lib.lib.qs_lm_head_logits(self._h, C.byref(p)))
        if not p.value:
            raise SamplerError(_lib.QS_ERR_INVALID, "no lm_head call yet")
        return _wrap_device(p.value, (int(batch), self.vocab), torch.bfloat16, self.device)

    def lm_head_status(self, stream=None) -> None:
        check(_lib.lib.qs_lm_head_status(self._h, _stream_handle(stream)))

    def profile(self, on: bool = True) -> None:
        check(_lib.lib.qs_profile_enable(self._h, 1 if on else 0))

    def profile_reset(self) -> None:
        check(_lib.lib.qs_profile_reset(self._h))

    def profile_read(self) -> Dict[str, float]:
        p = _lib.Profile()
        check(_lib.lib.qs_profile_read(self._h, C.byref(p)))
        return {f: getattr(p, f) for f, _ in _lib.Profile._fields_}

    def profile_phases(self, on: bool = True) -> None:
        """Per-row clock64() phase stamps of the row kernel and the tie replay
        (kernel tuning)."""
        check(_lib.lib.qs_profile_phases(self._h, 1 if on else 0))

    def profile_phases_read(self, which: int, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.int64)
        check(_lib.lib.qs_profile_phases_read(self._h, int(which),
                                              out.ctypes.data_as(C.POINTER(C.c_longlong)), int(n)))
        return out

    def reset_history(self) -> None:
        check(_lib.lib.qs_reset_sampler_history(self._h))

    def free(self) -> None:
        h = self.__dict__.get("_h")
        if h is not None and h.value:
            check(_lib.lib.qs_free_sampler(h))
            object.__setattr__(self, "_h", C.c_void_p())

    def __del__(self):
        try:
            self.free()
        except Exception:
            pass


def _wrap_device(ptr: int, shape, dtype, device: int):
    """A torch tensor over device memory the library owns (no copy)."""
    torch = _torch()
    n = 1
    for d in shape:
        n *= int(d)
    itemsize = torch.empty((), dtype=dtype).element_size()

    class _Mem:
        __cuda_array_interface__ = {"shape": (n * itemsize,), "typestr": "|u1",
                                    "data": (int(ptr), False), "version": 3}
    with torch.cuda.device(device):
        raw = torch.as_tensor(_Mem(), device=f"cuda:{device}")
    return raw.view(dtype).view(*shape)


def lm_head(hidden, weight, norm_weight=None, *, stream=None):
    """Final RMSNorm + lm_head (qwen_model.cuh:710-723) for bf16 device
    tensors; returns (normed [B, hidden_dim], logits [B, vocab]) bf16."""
    torch = _torch()
    h = hidden if hidden.dim() == 2 else hidden.view(1, -1)
    B, D = int(h.shape[0]), int(h.shape[1])
    Vv = int(weight.shape[0])
    normed = torch.empty((B, D), dtype=torch.bfloat16, device=h.device)
    logits = torch.empty((B, Vv), dtype=torch.bfloat16, device=h.device)
    err = torch.zeros(1, dtype=torch.int32, device=h.device)
    check(_lib.lib.qs_lm_head(_ptr(h), _ptr(norm_weight), _ptr(weight), B, D, Vv, _ptr(normed),
                              _ptr(logits), _ptr(err), _stream_handle(stream)))
    if int(err.item()) != 0:
        raise SamplerError(_lib.QS_ERR_CUDA, "lm_head kernel gave up waiting on its pipeline")
    return normed, logits


def decode_debug(dbg) -> Dict[str, np.ndarray]:
    """Per-row diagnostics tensor ([B, 12] int32 view of qs_row_debug) -> dict
    of numpy columns."""
    a = dbg.cpu().numpy()
    out = {}
    for j, (name, ct) in enumerate(RowDebug._fields_):
        col = np.ascontiguousarray(a[:, j])
        out[name] = col.view(np.float32) if ct is C.c_float else col
    return out


# ------------------------------------------------------------------ functions
def build_sampler(temperature, topp, minp, top_k, repetition_penalty, frequency_penalty,
                  presence_penalty, penalty_window_size, rng_seed, *, max_batch: int = 1,
                  vocab: int = VOCAB_SIZE, device: int = 0) -> Sampler:
    """build_sampler (sampler.h:277-327): top_k outside [0, vocab] becomes
    vocab (a full sort), as sampler.h:292 does."""
    tk = int(top_k) if 0 <= int(top_k) <= vocab else vocab
    return Sampler(temperature, topp, minp, tk, repetition_penalty, frequency_penalty,
                   presence_penalty, penalty_window_size, rng_seed, max_batch=max_batch,
                   vocab=vocab, device=device)


def sample(sampler: Sampler, logits, *, flags: int = 0):
    """sample() (sampler.h:165-270) for the rows of a device tensor; a 1-D
    logits vector returns a Python int like the reference."""
    toks = sampler.sample(logits, flags=flags)
    if logits.dim() == 1:
        return int(toks[0].item())
    return toks


def reset_sampler_history(sampler: Sampler) -> None:
    sampler.reset_history()


def free_sampler(sampler: Sampler) -> None:
    sampler.free()


__all__ = ["Sampler", "SamplingConfig", "build_sampler", "sample", "reset_sampler_history",
           "free_sampler", "decode_debug", "SamplerError", "QS_F32", "QS_BF16",
           "QS_FLAG_WRITE_PENALIZED", "QS_FLAG_INDEX_TIES", "VOCAB_SIZE"]
