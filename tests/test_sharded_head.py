"""Host logic of the vocab-sharded LM head (clusterlm_b200.sharded_head) under a 2-rank gloo group on CPU: shard
boundaries, and the combination of per-rank maxima and chunk sums gathered over the group, which must give the whole
rows' statistics exactly (the device kernels behind them are covered by the GPU test)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from clusterlm_b200.sharded_head import (CHUNK, combine_kept, combine_max, merge_argmax, shard_bounds, verify_decisions,
                                         verify_decisions_t)


def test_shard_bounds_cover_the_vocabulary_at_chunk_boundaries():
    for V in (128256, 151936, 65536, 16384 * 3 + 5):
        for world in (1, 2, 3, 4, 8):
            chunks = (V + CHUNK - 1) // CHUNK
            if world > chunks:
                with pytest.raises(ValueError):
                    shard_bounds(V, world)
                continue
            b = shard_bounds(V, world)
            assert b[0][0] == 0 and b[-1][1] == V
            for (a0, a1), (c0, _) in zip(b, b[1:]):
                assert a1 == c0 and a0 % CHUNK == 0 and a1 > a0
            sizes = [(b1 - b0 + CHUNK - 1) // CHUNK for b0, b1 in b]
            assert max(sizes) - min(sizes) <= 1


def test_merge_argmax_and_verify_decisions():
    assert merge_argmax([1.0, 3.0, 3.0], [5, 70000, 140000]) == 70000
    assert merge_argmax([2.0, 2.0], [9, 3]) == 3
    # all accepted: uniforms 0, 1, 2 consumed, the final sample uses the fourth
    assert verify_decisions([0.5, 0.5, 0.5], [0.25, 0.25, 0.25], [0.1, 0.2, 0.3, 0.4]) == (3, 3)
    # q = 0 rejects without drawing (sampling.cpp:113)
    assert verify_decisions([0.5, 0.5], [0.25, 0.0], [0.1, 0.2, 0.3]) == (1, 1)
    # p / q below the uniform rejects; the resample takes the next uniform
    assert verify_decisions([0.1, 0.5], [0.5, 0.5], [0.9, 0.2, 0.3]) == (0, 1)


def test_tensor_decisions_equal_the_walk():
    rng = np.random.default_rng(9)
    for case in range(400):
        k = int(rng.integers(1, 9))
        p = rng.random(k) * rng.choice([0.0, 1.0], k, p=[0.1, 0.9])
        q = rng.random(k) * rng.choice([0.0, 1.0], k, p=[0.15, 0.85])
        if case % 5 == 0:
            q = p * rng.uniform(0.5, 1.5, k)  # mostly accepted windows
        u = rng.random(k + 1)
        a, n = verify_decisions_t(torch.from_numpy(p), torch.from_numpy(q), torch.from_numpy(u))
        assert (int(a), int(n)) == verify_decisions(p.tolist(), q.tolist(), u.tolist()), (p, q, u)


def _chunk_stats(row):
    """(max, double sum of exp(l - max)) of each chunk, in one fixed order per chunk (a stand-in for the device
    chunk kernel)."""
    out = []
    for c in range(0, row.size, CHUNK):
        ch = row[c:c + CHUNK]
        m = float(max(ch.max(), np.float32(-3.4028235e38)))
        out.append((m, float(np.sum(np.exp(ch.astype(np.float64) - m)))))
    return out


def _factor(m, M):
    return float(np.exp(np.float64(np.float32(m) - np.float32(M))))


def _rank(rank, world, port, V, rows, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        logits = np.random.default_rng(3).standard_normal((rows, V)).astype(np.float32) * 3
        v0, v1 = shard_bounds(V, world)[rank]
        mine = logits[:, v0:v1]
        counts = [(b1 - b0 + CHUNK - 1) // CHUNK for b0, b1 in shard_bounds(V, world)]
        # the maxima of the shards combine exactly in any order
        local = torch.from_numpy(mine.max(axis=1).copy())
        out = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(out, local)
        assert np.array_equal(combine_max(torch.stack(out)).numpy(), logits.max(axis=1))
        # the chunk statistics, padded to the widest rank, gathered, combined in column order
        cm = np.full((rows, max(counts)), -3.0e38)
        cs = np.zeros((rows, max(counts)))
        for i in range(rows):
            for c, (m, sm) in enumerate(_chunk_stats(mine[i])):
                cm[i, c], cs[i, c] = m, sm
        gm = [torch.empty((rows, max(counts)), dtype=torch.float64) for _ in range(world)]
        gs = [torch.empty((rows, max(counts)), dtype=torch.float64) for _ in range(world)]
        dist.all_gather(gm, torch.from_numpy(cm))
        dist.all_gather(gs, torch.from_numpy(cs))
        got = combine_kept([g.tolist() for g in gm], [g.tolist() for g in gs], counts, _factor)
        for i in range(rows):
            whole = _chunk_stats(logits[i])
            M = max(m for m, _ in whole)
            a = 0.0
            for m, sm in whole:
                a += sm * _factor(m, M)
            assert got[i] == (M, a)
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        q.put((rank, repr(e)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,V", [(2, 128256), (3, 151936)])
def test_gathered_statistics_equal_whole_rows(world, V):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, V, 3, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {r: "ok" for r in range(world)}, res
