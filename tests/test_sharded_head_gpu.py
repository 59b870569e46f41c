"""The vocab-sharded LM head on 2 GPUs (NCCL): each rank holds half of a Q4_K head's rows; its distribution columns,
the speculative acceptance, the stochastic draft sample and the argmax over the sharded rows must equal the
single-GPU kernels on the gathered logits bit for bit (clm_b200_distribution_rows, clm_b200_accept_logits,
sample_from, argmax), and the sharded logits must match an unsharded head within 1e-5 (the split-K order
differs)."""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

V, H, Q = 128256, 512, 4


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device(f"cuda:{rank}"))
    try:
        from clusterlm_b200.runtime import (Context, Matrix, accept_logits, argmax_token, distribution, encode,
                                            generate_weights, sample_from)
        from clusterlm_b200.sharded_head import ShardedHead, shard_bounds

        dev = torch.device(f"cuda:{rank}")
        ctx = Context(rank)
        v0, v1 = shard_bounds(V, world)[rank]
        w = generate_weights(ctx, 0, 1001, v0 * H, (v1 - v0) * H, 0.02)
        head = ShardedHead(ctx, "q4_k", encode(ctx, "q4_k", w), V, H)
        g = torch.Generator().manual_seed(11)
        x = (torch.randn((2 * Q, H), generator=g) * 3).to(dev)
        Ls = head.logits(x)
        full = torch.empty((world, 2 * Q, max(b1 - b0 for b0, b1 in shard_bounds(V, world))), device=dev)
        pad = torch.zeros_like(full[0])
        pad[:, :Ls.shape[1]] = Ls
        dist.all_gather_into_tensor(full, pad)
        Lf = torch.cat([full[r, :, :b1 - b0] for r, (b0, b1) in enumerate(shard_bounds(V, world))], dim=1).contiguous()
        # against an unsharded head over the same weights
        whole = Matrix(ctx, "q4_k", encode(ctx, "q4_k", generate_weights(ctx, 0, 1001, 0, V * H, 0.02)), V, H)
        Lw = whole.matmul_rows(x)
        rel = ((Lw - Lf).abs().max() / Lw.abs().max()).item()
        assert rel < 1e-5, rel
        for T in (1.0, 0.7):
            gm, kp = head.stats(Ls, T)
            P = head.probs(Ls, gm, kp, T)
            Pw = distribution(ctx, Lf, T)
            assert torch.equal(P, Pw[:, v0:v1]), T
        # acceptance: target rows 0..Q, draft rows Q..2Q-1 (k = Q - 1), drafts taken near the top of each row
        tgt, drf = Ls[:Q].contiguous(), Ls[Q:2 * Q - 1].contiguous()
        tgt_f, drf_f = Lf[:Q].contiguous(), Lf[Q:2 * Q - 1].contiguous()
        for case in range(12):
            T = 1.0 if case % 2 == 0 else 0.7
            drafts = [int(torch.topk(tgt_f[j], 3).indices[case % 3]) for j in range(Q - 1)]
            dd = torch.tensor([drafts], dtype=torch.int32, device=dev)
            one_hot = case % 3 == 2
            a, n = head.accept(tgt, None if one_hot else drf, drafts, T, seed=5, counter_base=case)
            a, n = int(a), int(n)
            ar, nr = accept_logits(ctx, tgt_f.view(1, Q, V), None if one_hot else drf_f.view(1, Q - 1, V), dd, T,
                                   seed=5, counter_base=case)
            assert (a, n) == (int(ar.item()), int(nr.item())), (case, a, n, int(ar.item()), int(nr.item()))
        # one stochastic draft and the argmax
        u = torch.tensor([0.37], dtype=torch.float64, device=dev)
        tok, qrow = head.draft_sample(Ls[:1].contiguous(), 1.0, u)
        assert int(tok) == int(sample_from(ctx, distribution(ctx, Lf[:1].contiguous(), 1.0), u).item())
        assert head.argmax(Ls) == argmax_token(ctx, Lf).tolist()
        head.close()
        whole.close()
        torch.cuda.synchronize()
        ctx.close()
        q.put((rank, "ok"))
    except Exception as e:  # noqa: BLE001
        import traceback

        q.put((rank, traceback.format_exc()[-1500:]))
    finally:
        dist.destroy_process_group()


def test_sharded_head_equals_unsharded_on_two_gpus():
    import torch
    import torch.multiprocessing as mp

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert res == {0: "ok", 1: "ok"}, res
