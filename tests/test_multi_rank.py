"""The multi-GPU path's host logic with world_size 2 on CPU (gloo): rows are
split into blocks, each rank samples its block with the global rows' RNG
streams, and rank 0 gathers tokens and RNG states.  The gathered result must
equal the single-process result (the oracle stands in for each rank's
sampler; the split and the collectives are what is tested)."""
import os
import socket

import numpy as np
import pytest

from qwen600_engine_b200 import shard


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _workload(B, V=4096, seed=5):
    from qwen600_engine_b200 import workloads as W
    g = np.random.default_rng(seed)
    x = (3.0 * g.gumbel(size=(B, V))).astype(np.float32)
    hist = g.integers(0, V, size=(B, 16)).astype(np.int32)
    counts = g.integers(1, 3, size=(B, 16)).astype(np.float32)
    cnt = np.full(B, 16, np.int32)
    p = W.SamplingParams(0.8, 0.95, 0.05, 20, 1.2, 0.1, 0.05)
    return p, x, hist, counts, cnt


def _rank_main(rank, world, port, B, seed, out_path):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle.oracle import Oracle
        p, x, hist, counts, cnt = _workload(B)
        a, b = shard.row_block(rank, world, B)
        rng = shard.row_seeds(seed, a, b)
        o = Oracle().sample_rows(p, x[a:b], hist[a:b], counts[a:b], cnt[a:b], rng)
        toks = shard.gather_rows(torch.from_numpy(o["tokens"].astype(np.int32)), B, world, rank)
        states = shard.gather_rows(torch.from_numpy(o["rng"].view(np.int64)), B, world, rank)
        slowest = shard.max_over_ranks(1.5 + rank)
        if rank == 0:
            np.savez(out_path, tokens=toks.numpy(), rng=states.numpy().view(np.uint64),
                     slowest=slowest)
        else:
            assert toks is None and states is None
    finally:
        dist.destroy_process_group()


def test_row_blocks_cover_the_batch():
    for B in (0, 1, 7, 10, 1024):
        for G in (1, 2, 3, 4, 8):
            blocks = [shard.row_block(r, G, B) for r in range(G)]
            assert blocks[0][0] == 0 and blocks[-1][1] == B
            for (a0, b0), (a1, b1) in zip(blocks, blocks[1:]):
                assert b0 == a1 and a0 <= b0
    np.testing.assert_array_equal(shard.row_seeds(5, 2, 5), np.array([7, 8, 9], np.uint64))
    assert shard.row_seeds(2**64 - 1, 1, 2)[0] == 1  # wraps past the fixed point 0


@pytest.mark.parametrize("B", [10, 11])
def test_two_ranks_gather_equals_one_process(tmp_path, B):
    import torch.multiprocessing as mp
    from oracle.oracle import Oracle
    seed = 1000
    out = str(tmp_path / "rank0.npz")
    mp.start_processes(_rank_main, args=(2, _free_port(), B, seed, out), nprocs=2,
                       start_method="spawn")
    got = np.load(out)
    p, x, hist, counts, cnt = _workload(B)
    want = Oracle().sample_rows(p, x, hist, counts, cnt, shard.row_seeds(seed, 0, B))
    np.testing.assert_array_equal(got["tokens"], want["tokens"])
    np.testing.assert_array_equal(got["rng"], want["rng"])
    assert float(got["slowest"]) == 2.5


def test_vocab_shards_cover_the_vocabulary():
    for V in (8, 4096, 20008, 151936):
        for G in (1, 2, 3, 4, 8):
            sh = [shard.vocab_shard(r, G, V) for r in range(G)]
            assert sh[0][0] == 0 and sh[-1][0] + sh[-1][1] == V
            for (c0, n0), (c1, n1) in zip(sh, sh[1:]):
                assert c0 + n0 == c1 and c1 % 8 == 0 and n0 >= 0
            assert all(n % 8 == 0 for _, n in sh[:-1])


def _vocab_rank_main(rank, world, port, B, V, K, out_path):
    """Each rank computes its vocabulary slice of every row's logits; the
    slices are exchanged and each rank keeps whole rows of its row block --
    the data movement the sharded lm_head kernel does with peer stores."""
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(3)
        W = torch.randn(V, K, generator=g)
        h = torch.randn(B, K, generator=g)
        c0, n = shard.vocab_shard(rank, world, V)
        part = (h @ W[c0:c0 + n].T).to(torch.bfloat16).float()
        width = max(shard.vocab_shard(r, world, V)[1] for r in range(world))
        pad = torch.zeros(B, width)
        pad[:, :n] = part
        parts = [torch.empty_like(pad) for _ in range(world)]
        dist.all_gather(parts, pad)
        a, b = shard.row_block(rank, world, B)
        rows = torch.empty(b - a, V)
        for r in range(world):
            rc0, rn = shard.vocab_shard(r, world, V)
            rows[:, rc0:rc0 + rn] = parts[r][a:b, :rn]
        full = (h @ W.T).to(torch.bfloat16).float()[a:b]
        np.save(out_path + f".{rank}.npy", np.array([torch.equal(rows, full)]))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("B", [6, 7])
def test_two_ranks_vocab_slices_rebuild_rows(tmp_path, B):
    import torch.multiprocessing as mp
    out = str(tmp_path / "v")
    mp.start_processes(_vocab_rank_main, args=(2, _free_port(), B, 1000, 64, out), nprocs=2,
                       start_method="spawn")
    for r in range(2):
        assert bool(np.load(out + f".{r}.npy")[0])
