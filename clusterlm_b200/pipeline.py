"""Speculative stage pipeline across the GPUs of one node (one process per GPU).

The reference runs a speculative round stage by stage: the Father's prefix, the Nodes' middle stages and the
Father's tail, joined by RunWindow / StageResult messages over TCP (orchestrator/coordinator/src/
coordinator.cpp:736-832), with the drafter on the tail and a CommitWindow fan-out after acceptance
(coordinator.cpp:836-892).  Here every stage is a b200 engine on its own GPU and the hops are device links
(clm_b200_link_*): records go stage to stage, the tail accepts, commits, drafts the next window with its MTP head
and sends the window's tokens back to the prefix; each message carries the commit count of the session's previous
round, so no stage needs a host round trip.  Several sequences are in flight so that every stage is busy.

Plans use the reference's text form (ClusterPlan::parse, coordinator.cpp:54-95): "BEGIN-END@OWNER,...", in pipeline
order, contiguous, ending at the last layer, only the tail may be empty; an owner here is a GPU of the node
("g3" or "3") rather than a Node index or "father".  One extension: the plan may end in k > 1 items with the same
range (e.g. "...,27-32@g5,32-32@g6,32-32@g7"), k tail replicas.  Replica j runs the sessions s with s % k == j:
the stage before the replicas has a link to each and sends every session's records to its replica, and the prefix
has a link from each and takes every session's window tokens from its replica (clm_b200_pipe_attach_session).
The tail's LM head and MTP draft steps, which no layer split can shrink, are then shared by k GPUs.
"""
from __future__ import annotations

import dataclasses
from typing import Callable, Sequence

from .engine import LINK_RECV, LINK_SEND, ROLE_MIDDLE, ROLE_PREFIX, ROLE_TAIL, Engine, LlamaGeometry, Link

BYTES_PER_WEIGHT = {"q4_k": 144 / 256, "q8_0": 34 / 32}


@dataclasses.dataclass(frozen=True)
class StagePlan:
    begin: int
    end: int
    gpu: int

    def describe(self) -> str:
        return f"{self.begin}-{self.end}@g{self.gpu}"


def parse_plan(text: str, n_layers: int) -> list[StagePlan]:
    """ClusterPlan::parse + validate (coordinator.cpp:54-110) for GPU owners."""
    stages = []
    for item in text.split(","):
        at, dash = item.find("@"), item.find("-")
        if at < 0 or dash < 0 or dash > at:
            raise ValueError(f"plan item '{item}' is not BEGIN-END@OWNER")
        try:
            begin, end = int(item[:dash]), int(item[dash + 1:at])
        except ValueError:
            raise ValueError(f"bad layer range in '{item}'") from None
        owner = item[at + 1:]
        try:
            gpu = int(owner[1:] if owner.startswith("g") else owner)
        except ValueError:
            raise ValueError(f"bad owner in '{item}' (a GPU of this node: gK)") from None
        stages.append(StagePlan(begin, end, gpu))
    if len(stages) < 2:
        raise ValueError("a plan needs at least a prefix and a tail")
    if stages[-1].end != n_layers:
        raise ValueError(f"plan must end at layer {n_layers}")
    k = tail_replicas(stages)
    if k == len(stages):
        raise ValueError("a plan needs a prefix before its tail replicas")
    expect = 0
    for i, s in enumerate(stages[:len(stages) - k + 1]):
        if s.begin != expect or (s.end <= s.begin and i != len(stages) - k):
            raise ValueError("stage ranges must be contiguous and non-empty")
        expect = s.end
    if len({s.gpu for s in stages}) != len(stages):
        raise ValueError("every stage needs its own GPU")
    return stages


def tail_replicas(stages: Sequence[StagePlan]) -> int:
    """Number k of tail replicas: the trailing plan items with the last item's layer range."""
    k = 1
    while k < len(stages) and (stages[-1 - k].begin, stages[-1 - k].end) == (stages[-1].begin, stages[-1].end):
        k += 1
    return k


def format_plan(stages: Sequence[StagePlan]) -> str:
    return ",".join(s.describe() for s in stages)


def stage_costs(geo: LlamaGeometry, q: int, context: int) -> tuple[float, float]:
    """(bytes one layer streams per round, extra bytes of the tail per round): layer weights plus the layer's KV
    of every session's context; the tail adds the LM head and q-1 MTP draft steps (MTP block + LM head each)."""
    bw = BYTES_PER_WEIGHT[geo.quant]
    H, F, V = geo.hidden, geo.ffn, geo.vocab
    qd, kvd = geo.n_heads * geo.head_dim, geo.n_kv_heads * geo.head_dim
    layer = (H * (qd + 2 * kvd) + qd * H + 3 * F * H) * bw + 2 * context * kvd * 2
    head = V * H * bw
    mtp = 3 * F * H * bw if geo.mtp else 0.0
    tail = head + (q - 1) * (mtp + head)
    return layer, tail


def plan_stages(geo: LlamaGeometry, world: int, q: int, context: int, tails: int | None = None,
                sessions: int | None = None) -> list[StagePlan]:
    """Contiguous layer ranges for `world` GPUs minimising the largest byte stream of a stage while each of
    `sessions` sequences in flight (default `world`) runs one round (every stage but the tail holds at least one
    layer).  The last `tails` GPUs are tail replicas with one range; the busiest runs ceil(sessions / tails) of the
    sessions.  By default the replica count (1 .. world-1) with the smallest largest stream, the fewest on ties."""
    L = geo.n_layers
    if world < 2:
        raise ValueError("a pipeline needs at least two stages")
    if world - 1 > L:
        raise ValueError("more stages than layers")
    if tails is not None and not 1 <= tails <= world - 1:
        raise ValueError("tail replicas must leave at least the prefix")
    S = sessions or world
    layer, tail = stage_costs(geo, q, context)
    layer *= S
    INF = float("inf")
    # best[i][k]: smallest max cost placing layers [0, k) on stages [0, i) (all non-empty)
    best = [[INF] * (L + 1) for _ in range(world)]
    cut = [[0] * (L + 1) for _ in range(world)]
    best[0][0] = 0.0
    for i in range(1, world):
        for k in range(i, L + 1):
            for j in range(i - 1, k):
                c = max(best[i - 1][j], (k - j) * layer)
                if c < best[i][k]:
                    best[i][k], cut[i][k] = c, j
    # the tail replicas take the rest (possibly nothing); the busiest runs ceil(S / r) sessions
    choice, top = None, INF
    for r in ([tails] if tails else range(1, world)):
        n = world - r  # stages before the tail replicas
        busiest = -(-S // r)
        for k in range(n, L + 1):
            c = max(best[n][k], busiest * ((L - k) * layer / S + tail))
            if choice is None or c < top - 1e-9 * top:
                top, choice = c, (r, k)
    r, end = choice
    n = world - r
    bounds = [end]
    for i in range(n, 0, -1):
        bounds.append(cut[i][bounds[-1]])
    bounds = bounds[::-1]
    return ([StagePlan(bounds[i], bounds[i + 1], i) for i in range(n)] +
            [StagePlan(end, L, n + j) for j in range(r)])


def role_of(rank: int, world: int, tails: int = 1) -> int:
    return ROLE_PREFIX if rank == 0 else ROLE_TAIL if rank >= world - tails else ROLE_MIDDLE


def link_peers(rank: int, world: int, tails: int = 1) -> tuple[list[int], list[int]]:
    """(ranks this rank receives from, ranks it sends to).  Stages pass records forward; the stage before the
    tail replicas sends to every replica, and every replica sends window tokens back to the prefix (with one tail:
    the ring prefix -> ... -> tail -> prefix)."""
    first = world - tails  # the first tail replica
    last = first - 1       # the stage before the replicas
    ins = list(range(first, world)) if rank == 0 else [last] if rank >= first else [rank - 1]
    outs = [0] if rank >= first else list(range(first, world)) if rank == last else [rank + 1]
    return ins, outs


def wire(rank: int, world: int, gathered: Sequence[dict], tails: int = 1) -> tuple[dict, dict]:
    """Given every rank's exported link ends ({("in", src): handle, ("out", dst): handle}), the handles this rank's
    links connect to: {src: the sender's output end} and {dst: the receiver's input end}."""
    ins, outs = link_peers(rank, world, tails)
    return ({src: gathered[src][("out", rank)] for src in ins}, {dst: gathered[dst][("in", rank)] for dst in outs})


class StagePipeline:
    """This rank's stage of a speculative pipeline: engine, links and the per-round calls.

    Every rank must make the same calls (prefill chunks, rounds) for the same sessions in the same order; a tail
    replica makes them only for its own sessions (`owner`).  `all_gather` exchanges one picklable object per rank
    (torch.distributed.all_gather_object in practice); `engine_factory` / `link_factory` default to the device
    classes (host-logic tests pass stand-ins)."""

    def __init__(self, ctx, geo: LlamaGeometry, plan: Sequence[StagePlan], rank: int, max_context: int,
                 sessions: int, all_gather: Callable[[object], list], max_window: int = 16, slots: int = 0,
                 timeout_s: float = 30.0, weight_seed: int = 0, stddev: float = 0.02,
                 engine_factory=Engine, link_factory=Link):
        self.rank, self.world = rank, len(plan)
        self.tails = tail_replicas(plan)
        self.role = role_of(rank, self.world, self.tails)
        self.first_tail = self.world - self.tails
        # this rank's place among the tail replicas (0 .. tails-1), or None
        self.tail_index = rank - self.first_tail if self.role == ROLE_TAIL else None
        self.max_window = max_window
        self.ctx = ctx
        st = plan[rank]
        self.engine = engine_factory(ctx, geo, st.begin, st.end, self.role, max_context, max_window, sessions)
        self.engine.generate_weights(seed=weight_seed, stddev=stddev)
        self.engine.prepare()
        fpp = 2 * geo.hidden + 1
        rec = max_window * fpp * 4
        tok = (max_window + 1) * 4
        # a slot per sequence in flight (plus one), so no sender ever waits on a credit in steady state
        slots = slots or sessions + 1
        ins, outs = link_peers(rank, self.world, self.tails)
        # replicas send window tokens, every other stage boundary records
        self.links_in = {src: link_factory(ctx, LINK_RECV, slots, tok if src >= self.first_tail else rec, timeout_s)
                         for src in ins}
        self.links_out = {dst: link_factory(ctx, LINK_SEND, slots, tok if self.role == ROLE_TAIL else rec, timeout_s)
                          for dst in outs}
        mine = {("in", src): l.export() for src, l in self.links_in.items()}
        mine.update({("out", dst): l.export() for dst, l in self.links_out.items()})
        peer_in, peer_out = wire(rank, self.world, all_gather(mine), self.tails)
        for src, l in self.links_in.items():
            l.connect(peer_in[src])
        for dst, l in self.links_out.items():
            l.connect(peer_out[dst])
        self.link_in, self.link_out = self.links_in[ins[0]], self.links_out[outs[0]]
        self.engine.pipe_attach(self.link_in, self.link_out)

    @property
    def is_tail(self) -> bool:
        return self.role == ROLE_TAIL

    def owner(self, session: int) -> int:
        """The tail replica (0 .. tails-1) that runs `session`'s head, acceptance and drafts."""
        return session % self.tails

    def runs(self, session: int) -> bool:
        """Whether this rank runs `session` (every stage does; a tail replica only its own sessions)."""
        return self.tail_index is None or self.owner(session) == self.tail_index

    def open_session(self, session: int):
        if not self.runs(session):
            return
        self.engine.open_session(session)
        if len(self.links_in) > 1 or len(self.links_out) > 1:
            replica = self.first_tail + self.owner(session)
            self.engine.pipe_attach_session(session, self.links_in.get(replica), self.links_out.get(replica))

    def prefill(self, session: int, prompt: Sequence[int], stream=None) -> int:
        """Runs the prompt through this stage in chunks of max_window; returns the last chunk's final row."""
        n = len(prompt)
        off = 0
        while off < n:
            q = min(self.max_window, n - off)
            if self.runs(session):
                self.engine.pipe_prefill(session, q, prompt[off:off + q] if self.role == ROLE_PREFIX else None,
                                         stream)
            off += q
        return (n - 1) % self.max_window

    def begin(self, session: int, row: int, q: int, temperature: float = 0.0, seed: int = 0, stream=None):
        if self.is_tail and self.runs(session):
            self.engine.pipe_begin(session, row, q, temperature, seed, stream)

    def round(self, session: int, q: int, temperature: float = 0.0, seed: int = 0, d_tokens=None, d_count=None,
              stream=None):
        """One round of `session` on this stage (a tail replica: its own sessions only, which alone write
        d_tokens / d_count)."""
        if self.runs(session):
            self.engine.pipe_round(session, q, temperature, seed, d_tokens, d_count, stream)

    def status(self, stream=None):
        self.engine.pipe_status(stream)

    def close(self, barrier: Callable[[], None]):
        """Waits for this stage's work, then for every rank (`barrier`), before any link memory is released: a
        peer may still be storing into this rank's inbox until its own stream has drained."""
        self.ctx.synchronize()
        barrier()
        self.engine.close()
        for l in list(self.links_in.values()) + list(self.links_out.values()):
            l.close()
        barrier()
