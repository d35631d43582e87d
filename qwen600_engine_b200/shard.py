"""Row sharding across GPUs, one process per GPU.

Every row is an independent sampler (the reference keeps one ``Sampler`` per
sequence, sampler.h:165, and ``sample()`` touches nothing else), so a batch
splits into contiguous row blocks with no exchange while sampling.  Row r
keeps the RNG stream it has on one GPU (seed + r, counted over the whole
batch), so the sharded job draws exactly what the single-GPU job draws.  The
tokens go to one rank either with a collective (``gather_rows``, any
per-row tensor) or with no collective at all (``TokenGather``: peer copies
into rank 0's buffer and a device-side flag handshake), plus the
max-over-ranks of the timed region.

The functions take a torch.distributed process group (NCCL on GPUs, gloo in
the CPU tests) and plain tensors; nothing above ``VocabShardedLmHead``
depends on the sampler library.

The decode tail (final RMSNorm + lm_head, qwen_model.cuh:710-723) shards the
other way: splitting its rows would make every GPU stream the whole 311 MB
weight, so ``VocabShardedLmHead`` splits the vocabulary (``vocab_shard``).
Each GPU computes its slice of every row's logits and stores each row segment
straight into the buffer of the GPU that samples that row (peer stores over
NVLink inside the lm_head kernel).  A small kernel after it completes the
call on the device (``qs_shard_handshake``): it publishes the call's epoch
into every GPU's flag words and waits, bounded, for every GPU's; then each
GPU holds whole rows of its ``row_block`` and samples them as above.
"""
import ctypes as C
from typing import List, Optional, Tuple

import numpy as np


def row_block(rank: int, world: int, batch: int) -> Tuple[int, int]:
    """Rows [start, stop) of ``rank``: contiguous blocks of ceil(batch / world)
    rows (the last ones shorter or empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    per = -(-batch // world)
    start = min(rank * per, batch)
    return start, min(start + per, batch)


def row_seeds(seed: int, start: int, stop: int) -> np.ndarray:
    """xorshift64* states of rows [start, stop) of a batch seeded with
    ``seed``: seed + r for global row r (never 0, the generator's fixed point)."""
    s = (np.arange(start, stop, dtype=np.uint64) + np.uint64(seed & 0xFFFFFFFFFFFFFFFF))
    s[s == 0] = 1
    return s


def gather_rows(local, batch: int, world: int, rank: int, dst: int = 0, group=None):
    """Gathers every rank's row block of a per-row tensor (first dimension =
    rows, blocks as ``row_block``) into the whole batch on ``dst``; other
    ranks get None.  Blocks are padded to a common length for the collective."""
    import torch
    import torch.distributed as dist
    per = -(-batch // world)
    start, stop = row_block(rank, world, batch)
    n = stop - start
    if local.shape[0] != n:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its block has {n}")
    pad = torch.zeros((per,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    pad[:n] = local
    parts: Optional[List] = None
    if rank == dst:
        parts = [torch.empty_like(pad) for _ in range(world)]
    dist.gather(pad, gather_list=parts, dst=dst, group=group)
    if rank != dst:
        return None
    out = []
    for r in range(world):
        a, b = row_block(r, world, batch)
        out.append(parts[r][:b - a])
    return torch.cat(out, dim=0)


class TokenGather:
    """Gathers every rank's int32 tokens (its ``row_block``) to rank 0 without
    a collective: each rank copies its block straight into rank 0's buffer
    (device memory mapped through CUDA IPC; over NVLink), then the ranks run
    the device-side flag handshake (``qs_shard_handshake``, bounded: a rank
    that never arrives raises the error flag instead of hanging the others).
    Two buffer slots alternate, so a call's tokens stay readable on rank 0
    until the call after next.  The buffers are mapped once, at
    construction; every rank must construct and ``close`` together."""

    def __init__(self, batch: int, *, rank: int, world: int, device, group=None):
        import torch
        import torch.distributed as dist
        from . import _lib
        from .sampler import _wrap_device
        if world > 8:
            raise ValueError("at most 8 ranks")
        self.lib = _lib.lib
        self.batch, self.rank, self.world, self.group = int(batch), rank, world, group
        self.per = max(1, -(-self.batch // world))
        self.device = torch.device(device)
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        slot = world * self.per * 4
        self.flag_off = -(-(2 * slot) // 256) * 256
        hb = self.lib.qs_ipc_handle_bytes()
        handle = (C.c_ubyte * hb)()
        own = C.c_void_p()
        _lib.check(self.lib.qs_ipc_alloc(self.flag_off + 256, C.byref(own), handle))
        self._own = own.value
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine, group=group)
        ptrs, self._peers = [], []
        for r in range(world):
            if r == rank:
                ptrs.append(self._own)
                continue
            h = (C.c_ubyte * hb).from_buffer_copy(bytes(parts[r].cpu().tolist()))
            q = C.c_void_p()
            _lib.check(self.lib.qs_ipc_open(h, C.byref(q)))
            self._peers.append(q.value)
            ptrs.append(q.value)
        self._bufs = (C.c_void_p * world)(*ptrs)
        self._root = ptrs[0]  # rank 0's two slots as seen from this rank (a peer mapping elsewhere)
        self._view = _wrap_device(self._own, (2, world * self.per), torch.int32, dev) if rank == 0 else None
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = 0
        self.calls = 0
        self.wait_limit_ns = 2_000_000_000

    def __call__(self, tokens, stream=None):
        """Copies this rank's tokens into rank 0's current slot and completes
        the call; rank 0 gets the whole batch's tokens (a view of that slot,
        valid for the next call as well), other ranks None."""
        import torch
        from . import _lib
        from .sampler import _ptr, _stream_handle
        a, b = row_block(self.rank, self.world, self.batch)
        if tokens.shape[0] != b - a:
            raise ValueError(f"rank {self.rank} holds {tokens.shape[0]} rows, its block has {b - a}")
        j = self.calls % 2
        self.calls += 1
        if b > a:
            if not tokens.is_contiguous() or tokens.dtype != torch.int32:
                raise ValueError("tokens must be a contiguous int32 CUDA tensor")
            dst = self._root + (j * self.world * self.per + a) * 4
            _lib.check(self.lib.qs_copy_async(C.c_void_p(dst), _ptr(tokens), (b - a) * 4,
                                              _stream_handle(stream)))
        self.epoch = self.epoch % 0xFFFFFFFF + 1
        _lib.check(self.lib.qs_shard_handshake(self._bufs, self.world, self.rank, self.flag_off, self.epoch,
                                               self.wait_limit_ns, _ptr(self.err), _stream_handle(stream)))
        return self._view[j, :self.batch] if self.rank == 0 else None

    def status(self) -> None:
        """Raises if a handshake gave up waiting for a rank."""
        from . import _lib
        if int(self.err.item()) != 0:
            raise _lib.SamplerError(_lib.QS_ERR_CUDA, "token gather: a rank did not arrive in time")

    def close(self) -> None:
        import torch
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        self._view = None
        for p in self._peers:
            self.lib.qs_ipc_close(C.c_void_p(p))
        self._peers = []
        dist.barrier(group=self.group)
        self.lib.qs_ipc_free(C.c_void_p(self._own))
        self._own = None


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The largest of every rank's ``value`` (the timed region of a multi-GPU
    step is the slowest rank's)."""
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def vocab_shard(rank: int, world: int, vocab: int, align: int = 8) -> Tuple[int, int]:
    """Columns [col0, col0 + cols) of the vocabulary held by ``rank``:
    contiguous slices of ceil(vocab / world) rounded up to ``align`` columns
    (the last ones shorter or empty)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank outside [0, world)")
    per = -(-vocab // world)
    per = -(-per // align) * align
    col0 = min(rank * per, vocab)
    return col0, min(col0 + per, vocab) - col0


class VocabShardedLmHead:
    """The decode tail on ``world`` GPUs, one process each, vocabulary-sharded.

    ``weight_shard`` is this rank's rows [col0, col0 + cols) of the tied
    lm_head / embedding weight (bf16 [cols, hidden_dim] on this rank's GPU;
    ``vocab_shard`` gives the split).  Each call takes the same final hidden
    rows on every rank, computes this rank's slice of every row's logits
    (``qs_lm_head_shard``) and returns this rank's ``row_block`` of whole
    logit rows, bit-identical to the single-GPU ``lm_head``.  The row buffers
    are mapped between the processes once, at construction (CUDA IPC; every
    rank must construct and ``close`` together, since both exchange over the
    process group).  Each call ends with the device-side handshake, so no
    collective runs per call; every rank must have read its rows of one call
    before any rank makes the next (in a decode loop the token exchange
    between steps orders this)."""

    def __init__(self, weight_shard, col0: int, vocab: int, max_batch: int, *, rank: int, world: int,
                 group=None):
        import torch
        import torch.distributed as dist
        from . import _lib
        from .sampler import _wrap_device
        if weight_shard.dtype != torch.bfloat16 or weight_shard.dim() != 2 or not weight_shard.is_cuda:
            raise ValueError("weight_shard must be a bf16 [cols, hidden_dim] CUDA tensor")
        if world > 8:
            raise ValueError("at most 8 ranks")
        self.lib = _lib.lib
        self.weight = weight_shard.contiguous()
        self.col0, self.cols = int(col0), int(self.weight.shape[0])
        self.vocab, self.max_batch = int(vocab), int(max_batch)
        self.rank, self.world, self.group = rank, world, group
        self.device = self.weight.device
        self.hidden_dim = int(self.weight.shape[1])
        self.rows_cap = -(-self.max_batch // world)
        # the rows, then one 32-bit flag word per rank (written by that rank)
        self.flag_off = -(-(self.rows_cap * self.vocab * 2) // 256) * 256
        nbytes = self.flag_off + 256
        hb = self.lib.qs_ipc_handle_bytes()
        handle = (C.c_ubyte * hb)()
        own = C.c_void_p()
        _lib.check(self.lib.qs_ipc_alloc(nbytes, C.byref(own), handle))
        self._own = own.value
        self._peers: List[int] = []
        mine = torch.tensor(list(bytes(handle)), dtype=torch.uint8, device=self.device)
        parts = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(parts, mine, group=group)
        ptrs = []
        for r in range(world):
            if r == rank:
                ptrs.append(self._own)
                continue
            h = (C.c_ubyte * hb).from_buffer_copy(bytes(parts[r].cpu().tolist()))
            q = C.c_void_p()
            _lib.check(self.lib.qs_ipc_open(h, C.byref(q)))
            self._peers.append(q.value)
            ptrs.append(q.value)
        self._dst = (C.c_void_p * world)(*ptrs)
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        self.rows = _wrap_device(self._own, (self.rows_cap, self.vocab), torch.bfloat16, dev)
        self.normed = torch.empty((self.max_batch, self.hidden_dim), dtype=torch.bfloat16, device=self.device)
        self.err = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.epoch = 0
        self.wait_limit_ns = 2_000_000_000

    def __call__(self, hidden, norm_weight=None, stream=None, weight=None):
        """This rank's rows [start, stop) of ``row_block(rank, world, B)`` as a
        bf16 [stop - start, vocab] view of its row buffer (valid until the
        next call).  ``weight`` replaces the shard for this call (same shape)."""
        from . import _lib
        from .sampler import _ptr, _stream_handle
        B = int(hidden.shape[0])
        if B > self.max_batch or int(hidden.shape[1]) != self.hidden_dim:
            raise ValueError("hidden must be [B <= max_batch, hidden_dim]")
        per = max(1, -(-B // self.world))
        w = self.weight if weight is None else weight
        if tuple(w.shape) != tuple(self.weight.shape) or w.dtype != self.weight.dtype:
            raise ValueError("weight must have the shard's shape and dtype")
        _lib.check(self.lib.qs_lm_head_shard(_ptr(hidden), _ptr(norm_weight), _ptr(w), B,
                                             self.hidden_dim, self.vocab, self.col0, self.cols,
                                             _ptr(self.normed), self._dst, self.world, per,
                                             _ptr(self.err), _stream_handle(stream)))
        # every rank's stores have landed once every rank has published this
        # call's epoch (after its kernel) into this rank's flags
        self.epoch = self.epoch % 0xFFFFFFFF + 1  # 1, 2, ..., never 0 (the words' initial value)
        _lib.check(self.lib.qs_shard_handshake(self._dst, self.world, self.rank, self.flag_off, self.epoch,
                                               self.wait_limit_ns, _ptr(self.err), _stream_handle(stream)))
        start, stop = row_block(self.rank, self.world, B)
        return self.rows[:stop - start]

    def status(self) -> None:
        """Raises if a kernel gave up waiting on its own pipeline."""
        from . import _lib
        if int(self.err.item()) != 0:
            raise _lib.SamplerError(_lib.QS_ERR_CUDA, "lm_head kernel gave up waiting on its pipeline")

    def close(self) -> None:
        """Unmaps the peers' buffers, then (after every rank has) frees this
        rank's own."""
        import torch
        import torch.distributed as dist
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        for p in self._peers:
            self.lib.qs_ipc_close(C.c_void_p(p))
        self._peers = []
        dist.barrier(group=self.group)
        self.rows = None
        self.lib.qs_ipc_free(C.c_void_p(self._own))
        self._own = None
