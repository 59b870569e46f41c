"""Host logic of the stage pipeline (clusterlm_b200/pipeline.py) on CPU: plan text (ClusterPlan::parse rules,
orchestrator/coordinator/src/coordinator.cpp:54-110), byte-balanced stage planning, link wiring, and the call
sequence of every rank under torch.distributed (gloo, world sizes 2 and 3) with stand-in engines and links."""
import os
import socket

import pytest

from clusterlm_b200.engine import LLAMA3_8B, LLAMA3_70B, ROLE_MIDDLE, ROLE_PREFIX, ROLE_TAIL, LlamaGeometry
from clusterlm_b200.pipeline import (StagePipeline, StagePlan, format_plan, link_peers, parse_plan, plan_stages,
                                     role_of, stage_costs, wire)


def test_parse_plan_accepts_reference_form():
    st = parse_plan("0-10@g0,10-20@g1,20-32@2", 32)
    assert st == [StagePlan(0, 10, 0), StagePlan(10, 20, 1), StagePlan(20, 32, 2)]
    assert format_plan(st) == "0-10@g0,10-20@g1,20-32@g2"
    # only the tail may be empty (ClusterPlan::validate)
    assert parse_plan("0-32@g0,32-32@g1", 32)[1] == StagePlan(32, 32, 1)


@pytest.mark.parametrize("text, msg", [
    ("0-32@g0", "prefix and a tail"),
    ("0-10@g0,10-30@g1", "end at layer 32"),
    ("0-10@g0,11-32@g1", "contiguous"),
    ("0-0@g0,0-32@g1", "contiguous"),
    ("0-10g0,10-32@g1", "BEGIN-END@OWNER"),
    ("0-x@g0,10-32@g1", "bad layer range"),
    ("0-10@father,10-32@g1", "bad owner"),
    ("0-10@g1,10-32@g1", "own GPU"),
])
def test_parse_plan_rejects(text, msg):
    with pytest.raises(ValueError, match=msg):
        parse_plan(text, 32)


@pytest.mark.parametrize("world", [2, 3, 4, 8])
def test_plan_stages_balances_bytes(world):
    geo, q, ctx = LLAMA3_8B, 4, 4096
    plan = plan_stages(geo, world, q, ctx)
    assert len(plan) == world
    assert plan[0].begin == 0 and plan[-1].end == geo.n_layers
    assert all(a.end == b.begin for a, b in zip(plan, plan[1:]))
    assert all(s.end > s.begin for s in plan[:-1])
    layer, tail = stage_costs(geo, q, ctx)
    costs = [(s.end - s.begin) * layer + (tail if i == world - 1 else 0) for i, s in enumerate(plan)]
    # optimal: no single-layer move between neighbours lowers the maximum
    top = max(costs)
    for i in range(world - 1):
        for d in (-1, 1):
            c = list(costs)
            c[i] += d * layer
            c[i + 1] -= d * layer
            n_i = plan[i].end - plan[i].begin + d
            if n_i >= 1 and (plan[i + 1].end - plan[i + 1].begin - d) >= (0 if i + 1 == world - 1 else 1):
                assert max(c) >= top - 1e-6
    # the tail carries the head and the MTP drafts, so it gets fewer layers than the prefix
    assert plan[-1].end - plan[-1].begin < plan[0].end - plan[0].begin


def test_plan_stages_70b_eight_gpus():
    plan = plan_stages(LLAMA3_70B, 8, 8, 8192)
    assert [s.gpu for s in plan] == list(range(8))
    assert sum(s.end - s.begin for s in plan) == 80


def test_roles_and_ring():
    assert [role_of(r, 4) for r in range(4)] == [ROLE_PREFIX, ROLE_MIDDLE, ROLE_MIDDLE, ROLE_TAIL]
    assert [link_peers(r, 3) for r in range(3)] == [(2, 1), (0, 2), (1, 0)]
    g = [(b"in0", b"out0"), (b"in1", b"out1"), (b"in2", b"out2")]
    # rank r's receiving end maps the sender's output end; its sending end maps the receiver's input end
    assert wire(0, 3, g) == (b"out2", b"in1")
    assert wire(1, 3, g) == (b"out0", b"in2")
    assert wire(2, 3, g) == (b"out1", b"in0")


# ---- gloo: every rank's StagePipeline with stand-in engines and links ----

class FakeLink:
    def __init__(self, ctx, end, slots, payload, timeout_s):
        self.end, self.slots, self.payload, self.peer, self.closed = end, slots, payload, None, False
        self.rank = ctx.rank

    def export(self):
        return f"r{self.rank}-{'recv' if self.end else 'send'}-{self.slots}-{self.payload}".encode()

    def connect(self, h):
        self.peer = h

    def close(self):
        self.closed = True


class FakeEngine:
    def __init__(self, ctx, geo, begin, end, role, max_context, max_window, sessions):
        self.log = ctx.log
        self.log.append(("create", begin, end, role, max_context, max_window, sessions))

    def generate_weights(self, seed, stddev):
        self.log.append(("weights", seed))

    def prepare(self):
        self.log.append(("prepare",))

    def pipe_attach(self, a, b):
        self.log.append(("attach", a.peer, b.peer))

    def open_session(self, s):
        self.log.append(("open", s))

    def pipe_prefill(self, s, q, tokens, stream):
        self.log.append(("prefill", s, q, None if tokens is None else list(tokens)))

    def pipe_begin(self, s, row, q, T, seed, stream):
        self.log.append(("begin", s, row, q))

    def pipe_round(self, s, q, T, seed, d_tokens, d_count, stream):
        self.log.append(("round", s, q))

    def pipe_status(self, stream):
        self.log.append(("status",))

    def close(self):
        self.log.append(("close",))


class FakeCtx:
    def __init__(self, rank):
        self.rank, self.log = rank, []

    def synchronize(self):
        self.log.append(("sync",))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        geo = LlamaGeometry(6, 256, 4, 2, 128, 512, 512)
        plan = plan_stages(geo, world, 4, 64)

        def gather(obj):
            res = [None] * world
            dist.all_gather_object(res, obj)
            return res

        ctx = FakeCtx(rank)
        p = StagePipeline(ctx, geo, plan, rank, 256, 2, gather, max_window=16, engine_factory=FakeEngine,
                          link_factory=FakeLink)
        prompt = list(range(37))
        for s in (1, 2):
            p.open_session(s)
            row = p.prefill(s, prompt)
            p.begin(s, row, 4)
        for _ in range(3):
            for s in (1, 2):
                p.round(s, 4)
        p.close(dist.barrier)
        out[rank] = (ctx.log, p.link_in.peer, p.link_out.peer, p.link_in.closed and p.link_out.closed, row,
                     p.link_in.export(), p.link_out.export())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 3])
def test_pipeline_ranks_gloo(world):
    import torch.multiprocessing as mp

    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
    logs = {r: out[r] for r in range(world)}
    for r in range(world):
        log, peer_in, peer_out, closed, row, own_in, own_out = logs[r]
        src, dst = (r - 1) % world, (r + 1) % world
        # ring wiring: input from the previous stage's sending end, output to the next stage's receiving end
        assert peer_in.startswith(f"r{src}-send".encode()) and peer_out.startswith(f"r{dst}-recv".encode())
        # both ends of a link agree on slots and payload size
        assert own_out.split(b"-")[2:] == logs[dst][5].split(b"-")[2:]
        assert own_in.split(b"-")[2:] == logs[src][6].split(b"-")[2:]
        assert closed
        assert row == (37 - 1) % 16
        kinds = [e[0] for e in log]
        role = role_of(r, world)
        assert kinds[:4] == ["create", "weights", "prepare", "attach"]
        assert log[0][3] == role
        prefills = [e for e in log if e[0] == "prefill"]
        # chunks of max_window: 16, 16, 5 per session; only the prefix passes tokens
        assert [e[2] for e in prefills] == [16, 16, 5, 16, 16, 5]
        assert all((e[3] is not None) == (role == ROLE_PREFIX) for e in prefills)
        if role == ROLE_PREFIX:
            assert prefills[0][3] == list(range(16)) and prefills[2][3] == list(range(32, 37))
        begins = [e for e in log if e[0] == "begin"]
        assert len(begins) == (2 if role == ROLE_TAIL else 0)
        assert [e[1] for e in log if e[0] == "round"] == [1, 2] * 3
        # close protocol: drain this stage, wait for every rank, then release
        assert kinds[-2:] == ["sync", "close"]
    # the same prefill / round sequence on every rank
    seqs = [[(e[0], e[1], e[2]) for e in logs[r][0] if e[0] in ("prefill", "round")] for r in range(world)]
    assert all(s == seqs[0] for s in seqs)
    # the tail -> prefix link carries window tokens, the others boundary records
    assert int(logs[world - 1][6].split(b"-")[3]) == (16 + 1) * 4
    assert int(logs[0][6].split(b"-")[3]) == 16 * (2 * 256 + 1) * 4
