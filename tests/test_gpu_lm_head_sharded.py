"""Vocabulary-sharded decode tail on two GPUs (one process each, NCCL for
set-up only): each rank computes its slice of every row's logits and copies
row segments into the rank that samples the row (bulk copies over NVLink
inside the lm_head kernel), then the ranks complete the call with a
device-side flag handshake.  Each rank's whole rows must equal the
single-GPU lm_head's bit for bit, and sampling them must give the
single-GPU tokens.  Needs two GPUs; skipped otherwise.  The handshake's own
cases run on one GPU: a flag word already published passes at once, and a
flag that nothing sets makes the bounded wait give up with the error flag
raised."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _rank_main(rank, world, port, B, V, K, out_path):
    import datetime
    import torch
    import torch.distributed as dist
    from qwen600_engine_b200 import shard
    from qwen600_engine_b200.sampler import Sampler, lm_head
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    head = None
    try:
        dev = torch.device("cuda", rank)
        g = torch.Generator(device=dev).manual_seed(11)
        W = (0.02 * torch.randn(V, K, generator=g, device=dev)).to(torch.bfloat16)
        h = torch.randn(B, K, generator=g, device=dev).to(torch.bfloat16)
        nw = (1.0 + 0.1 * torch.randn(K, generator=g, device=dev)).to(torch.bfloat16)
        _, full = lm_head(h, W, nw)
        c0, n = shard.vocab_shard(rank, world, V)
        head = shard.VocabShardedLmHead(W[c0:c0 + n], c0, V, B, rank=rank, world=world)
        a, b = shard.row_block(rank, world, B)
        res = {}
        for call in range(2):  # the row buffers are reused across calls
            rows = head(h, nw)
            torch.cuda.synchronize()
            head.status()
            res[f"equal{call}"] = bool(torch.equal(rows.view(torch.int16), full[a:b].view(torch.int16)))
        # sampling the rows this rank owns gives the single-GPU tokens
        s = Sampler(temperature=0.6, topp=0.95, minp=0.05, top_k=20, repetition_penalty=1.0,
                    penalty_window_size=0, max_batch=max(1, b - a), vocab=V, device=rank)
        rng = torch.from_numpy(shard.row_seeds(77, a, b).view(np.int64)).to(dev)
        rng2 = rng.clone()
        t_sharded = s.sample_rows(rows, rng=rng)
        t_full = s.sample_rows(full[a:b].contiguous(), rng=rng2)
        torch.cuda.synchronize()
        res["tokens_equal"] = bool(torch.equal(t_sharded, t_full))
        s.free()
        np.save(out_path + f".{rank}.npy", np.array([res["equal0"], res["equal1"], res["tokens_equal"]]))
    finally:
        if head is not None:
            head.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("B,V", [(128, 151936), (100, 20008)])
def test_two_gpu_vocab_sharded_lm_head(tmp_path, B, V):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    out = str(tmp_path / "r")
    mp.start_processes(_rank_main, args=(2, _free_port(), B, V, 1024, out), nprocs=2,
                       start_method="spawn")
    for r in range(2):
        got = np.load(out + f".{r}.npy")
        assert got[0] and got[1], f"rank {r}: rows differ from the single-GPU lm_head"
        assert got[2], f"rank {r}: tokens differ"


def _gather_main(rank, world, port, B, out_path):
    import datetime
    import torch
    import torch.distributed as dist
    from qwen600_engine_b200 import shard
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    tg = None
    try:
        dev = torch.device("cuda", rank)
        tg = shard.TokenGather(B, rank=rank, world=world, device=dev)
        a, b = shard.row_block(rank, world, B)
        ok = []
        for call in range(3):  # both slots, then the first again
            toks = (torch.arange(a, b, dtype=torch.int32, device=dev) * 7 + 1000 * call)
            got = tg(toks)
            want = shard.gather_rows(toks, B, world, rank)  # NCCL (blocks padded to a common length)
            torch.cuda.synchronize()
            if rank == 0:
                ok.append(bool(torch.equal(got, want)))
        tg.status()
        np.save(out_path + f".{rank}.npy", np.array(ok if rank == 0 else [True]))
    finally:
        if tg is not None:
            tg.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [2048, 101])
def test_two_gpu_token_gather_without_collective(tmp_path, B):
    """shard.TokenGather: each rank copies its tokens into rank 0's buffer
    over NVLink and the device handshake completes the call; rank 0's result
    equals NCCL's gather, on three calls in a row (both buffer slots)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    out = str(tmp_path / "g")
    mp.start_processes(_gather_main, args=(2, _free_port(), B, out), nprocs=2, start_method="spawn")
    assert np.load(out + ".0.npy").all(), "gathered tokens differ from NCCL's gather"
    assert np.load(out + ".1.npy").all()


def test_handshake_on_one_gpu():
    """The handshake kernel against flag words set by the host (no second
    kernel to wait for): with the peer's word already at the epoch the call
    completes and leaves the error flag clear; with a word that nothing sets
    the wait runs out after its limit and raises the error flag; the context
    stays usable."""
    import ctypes as C
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from qwen600_engine_b200 import _lib
    lib = _lib.lib
    bufs = [torch.zeros(64, dtype=torch.int32, device="cuda") for _ in range(2)]
    ptrs = (C.c_void_p * 2)(*[b.data_ptr() for b in bufs])
    err = torch.zeros(1, dtype=torch.int32, device="cuda")
    # rank 0 of 2; its own word 1 (rank 1's) already holds epoch 3
    bufs[0][1] = 3
    torch.cuda.synchronize()
    _lib.check(lib.qs_shard_handshake(ptrs, 2, 0, 0, 3, 10_000_000, C.c_void_p(err.data_ptr()), None))
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    assert int(bufs[0][0].item()) == 3 and int(bufs[1][0].item()) == 3  # published to both ranks
    # epoch 4: rank 1's word stays at 3, so the wait gives up after 10 ms
    _lib.check(lib.qs_shard_handshake(ptrs, 2, 0, 0, 4, 10_000_000, C.c_void_p(err.data_ptr()), None))
    torch.cuda.synchronize()
    assert int(err.item()) == 1
    assert int(bufs[1][0].item()) == 4
    x = torch.arange(10, device="cuda").sum()
    assert int(x.item()) == 45
