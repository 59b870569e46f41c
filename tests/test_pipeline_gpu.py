"""Stage pipeline across GPUs (clm_b200_link_* / clm_b200_pipe_*), one process per GPU.

Parity: a pipeline split of a small Llama-shaped model over 2 GPUs, several sequences in flight, emits exactly the
tokens of the whole-model engine's speculative rounds (greedy acceptance and stochastic acceptance at T = 1 with
the same Philox keys); the split stages are bitwise equal to the whole model, so the tokens must be identical.
Failure: a link wait that nothing satisfies ends with CLM_DEADLINE_EXCEEDED on the host (no GPU fault).
Tests that need two GPUs skip on a one-GPU host.
"""
import os
import socket
from datetime import timedelta

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GEO = dict(n_layers=4, hidden=256, n_heads=2, n_kv_heads=1, head_dim=128, ffn=512, vocab=512)
Q, ROUNDS, SESSIONS, MAXW, MAXCTX = 4, 10, 3, 8, 256


def _geo():
    from clusterlm_b200.engine import LlamaGeometry

    return LlamaGeometry(quant="q4_k", **GEO)


def _prompts():
    rng = np.random.default_rng(21)
    return [rng.integers(0, GEO["vocab"], 11 + 5 * s).astype(np.int32) for s in range(SESSIONS)]


def _two_gpus():
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _whole_model_tokens(ctx, temperature, seed):
    from clusterlm_b200.engine import ROLE_WHOLE, Engine

    geo = _geo()
    e = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, MAXCTX, MAXW, SESSIONS)
    e.generate_weights(seed=0, stddev=0.02)
    e.prepare()
    out = {}
    for s, prompt in enumerate(_prompts()):
        e.open_session(s + 1)
        e.spec_begin(s + 1, prompt, Q, temperature=temperature, seed=seed)
        out[s + 1] = [list(e.spec_round(s + 1, Q, temperature, seed)) for _ in range(ROUNDS)]
    e.close()
    return out


def _pipe_worker(rank, world, port, plan_text, temperature, seed, out):
    import torch
    import torch.distributed as dist

    from clusterlm_b200.pipeline import StagePipeline, parse_plan
    from clusterlm_b200.runtime import Context

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        torch.cuda.set_device(rank)
        ctx = Context(rank)
        geo = _geo()

        def gather(obj):
            res = [None] * world
            dist.all_gather_object(res, obj)
            return res

        p = StagePipeline(ctx, geo, parse_plan(plan_text, geo.n_layers), rank, MAXCTX, SESSIONS, gather,
                          max_window=MAXW, timeout_s=20.0)
        dev = torch.device(f"cuda:{rank}")
        toks = torch.zeros((ROUNDS, SESSIONS, Q + 1), dtype=torch.int32, device=dev)
        cnt = torch.zeros((ROUNDS, SESSIONS), dtype=torch.int32, device=dev)
        torch.cuda.synchronize(dev)
        for s, prompt in enumerate(_prompts()):
            p.open_session(s + 1)
            row = p.prefill(s + 1, prompt)
            p.begin(s + 1, row, Q, temperature, seed)
        for r in range(ROUNDS):
            for s in range(SESSIONS):
                p.round(s + 1, Q, temperature, seed, toks[r, s], cnt[r, s])
        p.status()
        if p.is_tail:
            # a tail replica writes the tokens of its own sessions only
            t, c = toks.cpu().numpy(), cnt.cpu().numpy()
            out[f"tail{rank}"] = {s + 1: [list(t[r, s, :c[r, s]]) for r in range(ROUNDS)] for s in range(SESSIONS)
                                  if p.owner(s + 1) == p.tail_index}
        p.close(dist.barrier)
        ctx.close()
        out[rank] = "ok"
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("temperature, seed", [(0.0, 0), (1.0, 5)])
def test_two_stage_pipeline_equals_whole_model(ctx, temperature, seed):
    _two_gpus()
    import torch.multiprocessing as mp

    want = _whole_model_tokens(ctx, temperature, seed)
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_pipe_worker, args=(2, _free_port(), "0-3@g0,3-4@g1", temperature, seed, out), nprocs=2, join=True)
    assert out[0] == "ok" and out[1] == "ok"
    got = out["tail1"]
    for s in want:
        assert got[s] == want[s], f"session {s}"
    # every round emits 1..q tokens
    assert all(1 <= len(r) <= Q for s in got for r in got[s])


@pytest.mark.parametrize("plan_text, temperature, seed", [("0-2@g0,2-3@g1,3-4@g2,3-4@g3", 1.0, 5),
                                                          ("0-4@g0,4-4@g1,4-4@g2", 0.0, 0)])
def test_tail_replicas_equal_whole_model(ctx, plan_text, temperature, seed):
    """Tail replicas (clm_b200_pipe_relay): each tail GPU runs the sessions s with s % replicas == its index and
    passes the others' records and tokens on; every session's tokens equal the whole model's."""
    import torch

    from clusterlm_b200.pipeline import parse_plan, tail_replicas

    world = len(plan_text.split(","))
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    want = _whole_model_tokens(ctx, temperature, seed)
    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_pipe_worker, args=(world, _free_port(), plan_text, temperature, seed, out), nprocs=world, join=True)
    assert all(out[r] == "ok" for r in range(world))
    k = tail_replicas(parse_plan(plan_text, GEO["n_layers"]))
    got = {}
    for r in range(world - k, world):
        mine = out[f"tail{r}"]
        assert set(mine) == {s for s in want if s % k == r - (world - k)}
        got.update(mine)
    assert got == want


def _timeout_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist

    from clusterlm_b200._native import ClmError
    from clusterlm_b200.pipeline import StagePipeline, parse_plan
    from clusterlm_b200.runtime import Context

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        torch.cuda.set_device(rank)
        ctx = Context(rank)
        geo = _geo()

        def gather(obj):
            res = [None] * world
            dist.all_gather_object(res, obj)
            return res

        p = StagePipeline(ctx, geo, parse_plan("0-2@g0,2-4@g1", geo.n_layers), rank, MAXCTX, 1, gather,
                          max_window=MAXW, timeout_s=0.5)
        p.open_session(1)
        code = None
        if p.is_tail:
            # the prefix never sends: the tail's input wait runs out and the host sees the status
            p.round(1, Q)
            try:
                p.status()
            except ClmError as e:
                code = e.name
        p.close(dist.barrier)
        ctx.close()
        out[rank] = code
    finally:
        dist.destroy_process_group()


def test_link_wait_times_out_with_status():
    _two_gpus()
    import torch.multiprocessing as mp

    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_timeout_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    assert out[1] == "kDeadlineExceeded"
    assert out[0] is None


def test_link_refuses_one_gpu_and_mismatched_ends(ctx):
    from clusterlm_b200._native import ClmError
    from clusterlm_b200.engine import LINK_RECV, LINK_SEND, Link

    a = Link(ctx, LINK_SEND, 4, 1024)
    b = Link(ctx, LINK_RECV, 4, 1024)
    with pytest.raises(ClmError, match="same GPU"):
        a.connect(b.export())
    c = Link(ctx, LINK_SEND, 4, 1024)
    with pytest.raises(ClmError, match="same direction"):
        a.connect(c.export())
    d = Link(ctx, LINK_RECV, 8, 1024)
    with pytest.raises(ClmError, match="disagree"):
        a.connect(d.export())
    with pytest.raises(ClmError, match="not a link handle"):
        a.connect(bytes(128))
    with pytest.raises(ClmError):
        Link(ctx, LINK_SEND, 0, 1024)
    for l in (a, b, c, d):
        l.close()


def test_pipe_calls_need_attachment(ctx):
    from clusterlm_b200._native import ClmError
    from clusterlm_b200.engine import ROLE_PREFIX, ROLE_WHOLE, Engine, LINK_RECV, LINK_SEND, Link

    geo = _geo()
    e = Engine(ctx, geo, 0, 2, ROLE_PREFIX, MAXCTX, MAXW, 1)
    e.generate_weights(0, 0.02)
    e.prepare()
    e.open_session(1)
    with pytest.raises(ClmError, match="not attached"):
        e.pipe_round(1, Q)
    w = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, MAXCTX, MAXW, 1)
    w.generate_weights(0, 0.02)
    w.prepare()
    a, b = Link(ctx, LINK_RECV, 2, 64), Link(ctx, LINK_SEND, 2, 64)
    with pytest.raises(ClmError, match="whole-model"):
        w.pipe_attach(a, b)
    with pytest.raises(ClmError, match="not connected"):
        e.pipe_attach(a, b)
    e.close()
    w.close()
    a.close()
    b.close()
