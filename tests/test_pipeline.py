"""Host logic of the stage pipeline (clusterlm_b200/pipeline.py) on CPU: plan text (ClusterPlan::parse rules,
orchestrator/coordinator/src/coordinator.cpp:54-110), byte-balanced stage planning, link wiring, and the call
sequence of every rank under torch.distributed (gloo, world sizes 2 and 3) with stand-in engines and links."""
import os
import socket

import pytest

from clusterlm_b200.engine import LLAMA3_8B, LLAMA3_70B, ROLE_MIDDLE, ROLE_PREFIX, ROLE_TAIL, LlamaGeometry
from clusterlm_b200.pipeline import (StagePipeline, StagePlan, format_plan, link_peers, parse_plan, plan_stages,
                                     role_of, stage_costs, tail_replicas, wire)


def test_parse_plan_accepts_reference_form():
    st = parse_plan("0-10@g0,10-20@g1,20-32@2", 32)
    assert st == [StagePlan(0, 10, 0), StagePlan(10, 20, 1), StagePlan(20, 32, 2)]
    assert format_plan(st) == "0-10@g0,10-20@g1,20-32@g2"
    # only the tail may be empty (ClusterPlan::validate)
    assert parse_plan("0-32@g0,32-32@g1", 32)[1] == StagePlan(32, 32, 1)
    # tail replicas: trailing items with one range
    st = parse_plan("0-8@g0,8-20@g1,20-32@g2,20-32@g3,20-32@g4", 32)
    assert tail_replicas(st) == 3 and tail_replicas(parse_plan("0-8@g0,8-32@g1", 32)) == 1
    assert tail_replicas(parse_plan("0-32@g0,32-32@g1,32-32@g2", 32)) == 2


@pytest.mark.parametrize("text, msg", [
    ("0-32@g0", "prefix and a tail"),
    ("0-10@g0,10-30@g1", "end at layer 32"),
    ("0-10@g0,11-32@g1", "contiguous"),
    ("0-0@g0,0-32@g1", "contiguous"),
    ("0-10g0,10-32@g1", "BEGIN-END@OWNER"),
    ("0-x@g0,10-32@g1", "bad layer range"),
    ("0-10@father,10-32@g1", "bad owner"),
    ("0-10@g1,10-32@g1", "own GPU"),
    ("32-32@g0,32-32@g1", "prefix before its tail replicas"),
    ("0-10@g0,10-20@g1,32-32@g2,32-32@g3", "contiguous"),
    ("0-10@g0,10-10@g1,10-32@g2,10-32@g3", "contiguous"),
])
def test_parse_plan_rejects(text, msg):
    with pytest.raises(ValueError, match=msg):
        parse_plan(text, 32)


def _stage_loads(plan, geo, q, ctx, sessions):
    """Bytes each stage streams while every session runs one round (replicas: their busiest share)."""
    layer, tail = stage_costs(geo, q, ctx)
    r = tail_replicas(plan)
    n = len(plan) - r
    loads = [sessions * (s.end - s.begin) * layer for s in plan[:n]]
    return loads + [-(-sessions // r) * ((s.end - s.begin) * layer + tail) for s in plan[n:]]


@pytest.mark.parametrize("world", [2, 3, 4, 5, 8])
def test_plan_stages_balances_bytes(world):
    geo, q, ctx = LLAMA3_8B, 4, 4096
    plan = plan_stages(geo, world, q, ctx)
    assert len(plan) == world and [s.gpu for s in plan] == list(range(world))
    r = tail_replicas(plan)
    n = world - r
    assert plan[0].begin == 0 and plan[-1].end == geo.n_layers
    assert all(a.end == b.begin for a, b in zip(plan[:n], plan[1:n + 1]))
    assert all(s.end > s.begin for s in plan[:n])
    assert all((s.begin, s.end) == (plan[-1].begin, plan[-1].end) for s in plan[n:])
    layer, _ = stage_costs(geo, q, ctx)
    costs = _stage_loads(plan, geo, q, ctx, world)
    top = max(costs)
    # no other replica count does better (each count's own split is optimal among contiguous splits)
    for rr in range(1, world):
        assert max(_stage_loads(plan_stages(geo, world, q, ctx, tails=rr), geo, q, ctx, world)) >= top - 1e-3
    # optimal for its replica count: no single-layer move between neighbouring stages lowers the maximum
    sizes = [s.end - s.begin for s in plan[:n]] + [plan[-1].end - plan[-1].begin]
    for i in range(n):
        for d in (-1, 1):
            sz = list(sizes)
            sz[i] += d
            sz[i + 1] -= d
            if min(sz[:n]) < 1 or sz[n] < 0:
                continue
            bounds = [0]
            for x in sz[:n]:
                bounds.append(bounds[-1] + x)
            moved = [StagePlan(bounds[j], bounds[j + 1], j) for j in range(n)]
            moved += [StagePlan(bounds[n], geo.n_layers, j) for j in range(n, world)]
            assert max(_stage_loads(moved, geo, q, ctx, world)) >= top - 1e-3
    if r == 1:
        # the tail carries the head and the MTP drafts, so it gets fewer layers than the prefix
        assert plan[-1].end - plan[-1].begin < plan[0].end - plan[0].begin
    # 2 and 4 GPUs keep a single tail; 8 GPUs share the tail's head and drafts among replicas
    assert (r == 1) if world in (2, 4) else True
    if world == 8:
        assert r > 1 and top < 0.6 * max(_stage_loads(plan_stages(geo, 8, q, ctx, tails=1), geo, q, ctx, 8))


def test_plan_stages_70b_eight_gpus():
    plan = plan_stages(LLAMA3_70B, 8, 8, 8192)
    assert [s.gpu for s in plan] == list(range(8))
    n = len(plan) - tail_replicas(plan)
    assert sum(s.end - s.begin for s in plan[:n]) + plan[-1].end - plan[-1].begin == 80


def test_roles_and_ring():
    assert [role_of(r, 4) for r in range(4)] == [ROLE_PREFIX, ROLE_MIDDLE, ROLE_MIDDLE, ROLE_TAIL]
    assert [role_of(r, 4, 2) for r in range(4)] == [ROLE_PREFIX, ROLE_MIDDLE, ROLE_TAIL, ROLE_TAIL]
    # one tail: the ring prefix -> ... -> tail -> prefix
    assert [link_peers(r, 3) for r in range(3)] == [([2], [1]), ([0], [2]), ([1], [0])]
    # replicas 3 and 4: the stage before them feeds both, both feed the prefix
    assert [link_peers(r, 5, 2) for r in range(5)] == [([3, 4], [1]), ([0], [2]), ([1], [3, 4]), ([2], [0]),
                                                       ([2], [0])]
    # the prefix itself before the replicas
    assert [link_peers(r, 3, 2) for r in range(3)] == [([1, 2], [1, 2]), ([0], [0]), ([0], [0])]
    g = [{("in", 2): b"in0", ("out", 1): b"out0"}, {("in", 0): b"in1", ("out", 2): b"out1"},
         {("in", 1): b"in2", ("out", 0): b"out2"}]
    # rank r's receiving end maps the sender's output end; its sending end maps the receiver's input end
    assert wire(0, 3, g) == ({2: b"out2"}, {1: b"in1"})
    assert wire(1, 3, g) == ({0: b"out0"}, {2: b"in2"})
    assert wire(2, 3, g) == ({1: b"out1"}, {0: b"in0"})


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

    def pipe_attach_session(self, s, a, b):
        self.log.append(("attach_session", s, None if a is None else a.peer, None if b is None else b.peer))

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


def _worker(rank, world, port, plan_text, out):
    import torch.distributed as dist

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        geo = LlamaGeometry(6, 256, 4, 2, 128, 512, 512)
        plan = parse_plan(plan_text, geo.n_layers) if plan_text else plan_stages(geo, world, 4, 64)

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
        links = {("in", k): (l.export(), l.peer, l.closed) for k, l in p.links_in.items()}
        links.update({("out", k): (l.export(), l.peer, l.closed) for k, l in p.links_out.items()})
        out[rank] = (ctx.log, links, row, p.tail_index)
    finally:
        dist.destroy_process_group()


def _replay(logs, world, tails):
    """Replays every rank's calls over FIFO links and returns the largest number of messages any link held.  A
    message is (kind, session); a call receives on the link its role and session name (the prefix from the
    session's replica, a replica from the stage before the replicas, others from the previous stage) and sends on
    the matching one.  Fails on a message of the wrong kind or session, on a call that could never run (deadlock)
    or on messages left over beyond the next windows of sessions 1 and 2."""
    first = world - tails

    def src(r, s):
        return first + s % tails if r == 0 else first - 1 if r >= first else r - 1

    def dst(r, s):
        return 0 if r >= first else first + s % tails if r == first - 1 else r + 1

    ops = []
    for r in range(world):
        role = logs[r][0][0][3]
        seq = []
        for e in logs[r][0]:
            s = e[1] if e[0] in ("prefill", "begin", "round") else None
            if e[0] == "prefill":
                seq.append(("pre" if role != ROLE_PREFIX else None, ("pre", s) if role != ROLE_TAIL else None, s))
            elif e[0] == "begin":
                seq.append((None, ("tok", s), s))
            elif e[0] == "round":
                seq.append(("tok" if role == ROLE_PREFIX else "rec", ("tok", s) if role == ROLE_TAIL else ("rec", s), s))
        ops.append(seq)
    inbox = {}
    at = [0] * world
    peak = 0
    while any(at[r] < len(ops[r]) for r in range(world)):
        moved = False
        for r in range(world):
            if at[r] == len(ops[r]):
                continue
            want, send, s = ops[r][at[r]]
            if want is not None:
                box = inbox.setdefault((src(r, s), r), [])
                if not box:
                    continue
                msg = box.pop(0)
                assert msg == (want, s), f"rank {r} call {at[r]} wanted {(want, s)}, got {msg}"
            if send is not None:
                box = inbox.setdefault((r, dst(r, s)), [])
                box.append(send)
                peak = max(peak, len(box))
            at[r] += 1
            moved = True
        assert moved, f"deadlock: calls done {at} of {[len(o) for o in ops]}, inboxes {inbox}"
    left = sorted(m for b in inbox.values() for m in b)
    # only the next windows the last rounds drafted wait at the prefix, one per session
    assert left == [("tok", 1), ("tok", 2)], f"messages left over: {inbox}"
    assert all(k[1] == 0 for k, b in inbox.items() if b)
    return peak


@pytest.mark.parametrize("world, plan_text", [(2, None), (3, None), (4, "0-3@g0,3-5@g1,5-6@g2,5-6@g3"),
                                              (4, "0-4@g0,4-6@g1,6-6@g2,6-6@g3"), (3, "0-6@g0,6-6@g1,6-6@g2")])
def test_pipeline_ranks_gloo(world, plan_text):
    import torch.multiprocessing as mp

    mgr = mp.Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _free_port(), plan_text, out), nprocs=world, join=True)
    logs = {r: out[r] for r in range(world)}
    tails = 1 if plan_text is None else tail_replicas(parse_plan(plan_text, 6))
    for r in range(world):
        log, links, row, tail_index = logs[r]
        ins, outs = link_peers(r, world, tails)
        assert sorted(k for k in links if k[0] == "in") == [("in", x) for x in ins]
        assert sorted(k for k in links if k[0] == "out") == [("out", x) for x in outs]
        for (end, peer), (own, connected, closed) in links.items():
            # a receiving end maps the sender's output end and vice versa; both ends agree on slots and payload
            other = logs[peer][1][("out" if end == "in" else "in", r)][0]
            assert connected == other and closed
            assert own.split(b"-")[2:] == other.split(b"-")[2:]
            # replicas send window tokens, every other stage boundary records
            sender = peer if end == "in" else r
            assert int(own.split(b"-")[3]) == ((16 + 1) * 4 if sender >= world - tails else 16 * (2 * 256 + 1) * 4)
        assert row == (37 - 1) % 16
        kinds = [e[0] for e in log]
        role = role_of(r, world, tails)
        assert kinds[:4] == ["create", "weights", "prepare", "attach"]
        assert log[0][3] == role
        assert tail_index == (r - (world - tails) if role == ROLE_TAIL else None)
        # a tail replica runs the sessions s with s % tails == its index, and no other
        own = [1, 2] if role != ROLE_TAIL else [s for s in (1, 2) if s % tails == tail_index]
        assert [e[1] for e in log if e[0] == "open"] == own
        # stages with several links bind every session to its replica's link
        binds = [e for e in log if e[0] == "attach_session"]
        if len(ins) > 1 or len(outs) > 1:
            for s in own:
                replica = world - tails + s % tails
                want_in = links[("in", replica)][1] if ("in", replica) in links else None
                want_out = links[("out", replica)][1] if ("out", replica) in links else None
                assert ("attach_session", s, want_in, want_out) in binds
        else:
            assert not binds
        prefills = [e for e in log if e[0] == "prefill"]
        # chunks of max_window: 16, 16, 5 per session; only the prefix passes tokens
        assert [e[2] for e in prefills] == [16, 16, 5] * len(own)
        assert [e[1] for e in prefills] == [s for s in own for _ in range(3)]
        assert all((e[3] is not None) == (role == ROLE_PREFIX) for e in prefills)
        if role == ROLE_PREFIX:
            assert prefills[0][3] == list(range(16)) and prefills[2][3] == list(range(32, 37))
        begins = [e for e in log if e[0] == "begin"]
        assert [e[1] for e in begins] == (own if role == ROLE_TAIL else [])
        assert [e[1] for e in log if e[0] == "round"] == [s for s in [1, 2] * 3 if s in own]
        # close protocol: drain this stage, wait for every rank, then release
        assert kinds[-2:] == ["sync", "close"]
    # the same prefill / round sequence on every rank that is not a tail replica
    seqs = [[(e[0], e[1], e[2]) for e in logs[r][0] if e[0] in ("prefill", "round")]
            for r in range(world - tails)]
    assert all(s == seqs[0] for s in seqs)
    # every message reaches the stage that expects it, in order, within the link's slots (sessions + 1)
    assert _replay(logs, world, tails) <= 3
