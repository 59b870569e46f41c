"""Vocabulary-sharded LM head: the head's rows, its softmax statistics, draft sampling and speculative acceptance
split by vocabulary over the GPUs of a process group, with results identical to the unsharded path.

The reference computes the head and distribution() over whole rows on one process
(runtime/domain/src/reference_domain.cpp:577-585, runtime/domain/src/sampling.cpp:51-131).  Here rank r holds the
head rows [v0_r, v1_r) (shard boundaries at multiples of the 16,384-column statistics chunk) and:

  * computes its columns of the logits (clm_b200_matmul_rows over its shard of the head);
  * computes, in one pass over its logits, each 16,384-column chunk's maximum and the double sum of
    exp(double(l - chunk max) / T) (clm_b200_shard_stats, the same device code as the whole-row statistics);
  * all-gathers these chunk statistics, and every rank combines them in column order (clm_b200_shard_combine): the
    row maximum, and the kept sum as the chunk sums times exp(double(chunk max - max) / T) added one after another
    from 0.0, exactly as the whole-row statistics combine their chunks, so max and kept equal the whole row's bit
    for bit;
  * evaluates any probability it owns as float(exp(double(l - max) / T) / kept), the whole-row value;
  * runs verify_speculative (sampling.cpp:103-131) with p(d) / q(d) at the draft tokens taken from their owning
    ranks (an all-reduce of a k-vector), the accept decisions in IEEE double exactly as the reference's walk, and
    the residual / bonus row gathered to full rows for sample_from (clm_b200_sample_rows).

Everything stays on the device: the maxima, chunk sums and decisions are tensors combined where they lie, so a
window's acceptance is a fixed sequence of kernels and collectives with no host synchronisation.

The uniforms are the device path's Philox draws (counter (draw, sequence 0, counter_base)), one per test with q > 0
and one for the final sample, in the reference's order.  Collectives go through torch.distributed (NCCL between
GPUs); every rank makes the same calls in the same order.
"""
from __future__ import annotations

import ctypes as C

import torch
import torch.distributed as dist

from .runtime import Context, Matrix, philox_uniforms, sample_from
from ._native import call
from .runtime import _ptr, _stream

CHUNK = 16384  # statistics chunk (columns) of the device distribution kernels


def shard_bounds(vocab: int, world: int) -> list[tuple[int, int]]:
    """Contiguous column ranges [v0, v1) per rank: whole 16,384-column chunks spread as evenly as possible."""
    chunks = (vocab + CHUNK - 1) // CHUNK
    if world > chunks:
        raise ValueError(f"{world} shards need at least {world} statistics chunks; the vocabulary has {chunks}")
    out = []
    for r in range(world):
        c0, c1 = r * chunks // world, (r + 1) * chunks // world
        out.append((c0 * CHUNK, min(vocab, c1 * CHUNK)))
    return out


def combine_max(gathered: torch.Tensor) -> torch.Tensor:
    """Row maxima from the ranks' shard maxima ([world][rows]); the maximum is exact in any order."""
    return gathered.max(dim=0).values


def combine_kept(chunk_max, chunk_sum, counts, factor):
    """The whole rows' (max, kept) from the ranks' chunk statistics (chunk_max[r][row][c], chunk_sum[r][row][c],
    counts[r] chunks of rank r) in column order: max over every chunk, then kept = sum of chunk_sum * factor(chunk
    max, max) added one after another from 0.0 (factor: exp(double(m_c - max) / T) in the device code)."""
    rows = len(chunk_max[0])
    out = []
    for i in range(rows):
        M = max(chunk_max[r][i][c] for r, n in enumerate(counts) for c in range(n))
        a = 0.0
        for r, n in enumerate(counts):
            for c in range(n):
                a += chunk_sum[r][i][c] * factor(chunk_max[r][i][c], M)
        out.append((M, a))
    return out


def merge_argmax(values, indices):
    """(value, index) per rank -> the maximum, lowest index on ties (argmax_token, sampling.cpp:44-49)."""
    best_v, best_i = None, None
    for v, i in zip(values, indices):
        if best_v is None or v > best_v or (v == best_v and i < best_i):
            best_v, best_i = v, i
    return best_i


def verify_decisions(p_d, q_d, uniforms):
    """The accept / reject walk of verify_speculative (sampling.cpp:107-117) on the draft probabilities: returns
    (accepted drafts, index of the uniform the final sample uses)."""
    n = 0
    for j, (p, q) in enumerate(zip(p_d, q_d)):
        if q > 0.0:
            u = uniforms[n]
            n += 1
            if u < min(1.0, p / q):
                continue
        return j, n
    return len(p_d), n


def verify_decisions_t(p_d: torch.Tensor, q_d: torch.Tensor, uniforms: torch.Tensor):
    """verify_decisions on float64 tensors, where they lie (0-d int64 results, no host synchronisation): draft j is
    tested with the uniform after the tests of drafts 0..j-1 that had q > 0, and passes when q > 0 and
    u < min(1, p / q) (IEEE double division and comparison, as the reference's walk)."""
    k = p_d.shape[0]
    tests = q_d > 0.0
    before = torch.cumsum(tests.to(torch.int64), 0)  # tests up to and including j
    u = uniforms[before - tests.to(torch.int64)]
    ratio = torch.where(tests, p_d / torch.where(tests, q_d, torch.ones_like(q_d)), torch.zeros_like(p_d))
    ok = tests & (u < torch.clamp(ratio, max=1.0))
    a = torch.cumprod(ok.to(torch.int64), 0).sum()
    n = torch.where(a < k, before[a.clamp(max=k - 1)], before[k - 1])
    return a, n


class ShardedHead:
    """One rank's shard of a vocab-sharded LM head (Q4_K / Q8_0 rows [v0, v1) of a [vocab][hidden] head)."""

    def __init__(self, ctx: Context, quant: str, shard_bytes: torch.Tensor, vocab: int, hidden: int,
                 group=None):
        self.ctx, self.vocab, self.hidden, self.group = ctx, vocab, hidden, group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.bounds = shard_bounds(vocab, self.world)
        self.v0, self.v1 = self.bounds[self.rank]
        self.n = self.v1 - self.v0
        self.counts = [(b1 - b0 + CHUNK - 1) // CHUNK for b0, b1 in self.bounds]
        self.dev = torch.device(f"cuda:{ctx.device}")
        self.head = Matrix(ctx, quant, shard_bytes, self.n, hidden)

    def close(self):
        self.head.close()

    # ---- logits and statistics
    def logits(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's columns of the logits of rows x (q, hidden) (normalised head inputs)."""
        return self.head.matmul_rows(x)

    def _all_gather(self, t: torch.Tensor) -> list[torch.Tensor]:
        out = [torch.empty_like(t) for _ in range(self.world)]
        dist.all_gather(out, t.contiguous(), group=self.group)
        return out

    def stats(self, L: torch.Tensor, temperature: float):
        """(max, kept) of the whole rows: float32 and float64 device tensors of len(L) rows."""
        rows = L.shape[0]
        cmax = max(self.counts)
        cm = torch.full((rows, cmax), -3.0e38, dtype=torch.float32, device=self.dev)
        cs = torch.zeros((rows, cmax), dtype=torch.float64, device=self.dev)
        mine_m = torch.empty((rows, self.counts[self.rank]), dtype=torch.float32, device=self.dev)
        mine_s = torch.empty((rows, self.counts[self.rank]), dtype=torch.float64, device=self.dev)
        call("clm_b200_shard_stats", self.ctx.h, _ptr(L), rows, self.n, self.v0, temperature, _ptr(mine_m),
             _ptr(mine_s), _stream())
        cm[:, :mine_m.shape[1]] = mine_m
        cs[:, :mine_s.shape[1]] = mine_s
        gm = torch.empty((self.world, rows, cmax), dtype=torch.float32, device=self.dev)
        gs = torch.empty((self.world, rows, cmax), dtype=torch.float64, device=self.dev)
        dist.all_gather_into_tensor(gm, cm, group=self.group)
        dist.all_gather_into_tensor(gs, cs, group=self.group)
        gmax = torch.empty(rows, dtype=torch.float32, device=self.dev)
        kept = torch.empty(rows, dtype=torch.float64, device=self.dev)
        counts = (C.c_uint32 * self.world)(*self.counts)
        call("clm_b200_shard_combine", self.ctx.h, _ptr(gm), _ptr(gs), self.world, counts, rows, cmax, temperature,
             _ptr(gmax), _ptr(kept), _stream())
        return gmax, kept

    def probs(self, L: torch.Tensor, gmax: torch.Tensor, kept: torch.Tensor, temperature: float) -> torch.Tensor:
        out = torch.empty_like(L)
        call("clm_b200_shard_probs", self.ctx.h, _ptr(L), L.shape[0], self.n, temperature, _ptr(gmax), _ptr(kept),
             _ptr(out), _stream())
        return out

    def gather_row(self, row: torch.Tensor) -> torch.Tensor:
        """A full row (vocab,) on every rank from the ranks' column shards."""
        width = max(b1 - b0 for b0, b1 in self.bounds)
        pad = torch.zeros(width, dtype=row.dtype, device=self.dev)
        pad[:self.n] = row
        parts = torch.empty((self.world, width), dtype=row.dtype, device=self.dev)
        dist.all_gather_into_tensor(parts, pad, group=self.group)
        return torch.cat([parts[r, :b1 - b0] for r, (b0, b1) in enumerate(self.bounds)])

    def owned(self, rows: torch.Tensor, cols: torch.Tensor) -> torch.Tensor:
        """rows[j][cols[j] - v0] where this rank owns column cols[j], summed over the ranks (each entry has one owner,
        the others add 0.0): the values at the given columns of the whole rows, in float64, on every rank."""
        idx = cols.to(torch.int64) - self.v0
        mine = (idx >= 0) & (idx < self.n)
        vals = rows.gather(1, idx.clamp(0, self.n - 1).view(-1, 1)).view(-1).double()
        vals = torch.where(mine, vals, torch.zeros_like(vals))
        dist.all_reduce(vals, op=dist.ReduceOp.SUM, group=self.group)
        return vals

    # ---- sampling
    def argmax(self, L: torch.Tensor) -> list[int]:
        """argmax of every row over the whole vocabulary (lowest index on ties)."""
        v, i = L.max(dim=1)  # torch returns the first maximal index of the shard
        vals = torch.stack(self._all_gather(v.float())).cpu()
        idx = torch.stack(self._all_gather((i + self.v0).to(torch.int64))).cpu()
        return [merge_argmax(vals[:, r].tolist(), idx[:, r].tolist()) for r in range(L.shape[0])]

    def sample_row(self, full_row: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
        """sample_from(full_row, u) on the device (bit-identical to the reference's serial walk): a 0-d int32 tensor."""
        return sample_from(self.ctx, full_row.view(1, -1).contiguous(), u.view(1))[0]

    def accept(self, target_logits: torch.Tensor, draft_logits: torch.Tensor | None, drafts, temperature: float,
               seed: int, counter_base: int):
        """verify_speculative over the sharded rows of one sequence: target_logits (k+1, vocab shard), draft_logits
        (k, vocab shard) or None (one-hot drafts), drafts (k,) token ids; returns (accepted drafts, next token) as
        0-d device tensors.  Nothing waits for the host: every step is a kernel or a collective on the stream."""
        k = len(drafts)
        d = torch.as_tensor(drafts, dtype=torch.int64).to(self.dev, non_blocking=True)
        us = philox_uniforms(self.ctx, seed, 0, counter_base & 0xFFFFFFFF, counter_base >> 32, k + 1)
        gm, kp = self.stats(target_logits, temperature)
        P = self.probs(target_logits, gm, kp, temperature)
        p_d = self.owned(P[:k], d)
        Q = None
        if draft_logits is not None:
            qm, qk = self.stats(draft_logits, temperature)
            Q = self.probs(draft_logits, qm, qk, temperature)
            q_d = self.owned(Q, d)
        else:
            q_d = torch.ones(k, dtype=torch.float64, device=self.dev)
        a, n = verify_decisions_t(p_d, q_d, us)
        # the final sample: P[k] when every draft passed, else the residual max(P[a] - Q[a], 0) (P[a] when it has
        # no mass anywhere in the vocabulary)
        Pa = P.index_select(0, a.view(1)).view(-1)
        ar = a.clamp(max=k - 1).view(1)
        if Q is not None:
            Qa = Q.index_select(0, ar).view(-1).double()
        else:
            cols = torch.arange(self.v0, self.v1, device=self.dev)
            Qa = (cols == d.index_select(0, ar)).double()
        r = (Pa.double() - Qa).clamp_min(0.0)
        mass = (r > 0).any().to(torch.float32).view(1)
        dist.all_reduce(mass, op=dist.ReduceOp.MAX, group=self.group)
        row = torch.where((a < k) & (mass[0] > 0), r.float(), Pa)
        return a, self.sample_row(self.gather_row(row), us[n])

    def draft_sample(self, logits: torch.Tensor, temperature: float, u: torch.Tensor):
        """One stochastic MTP draft from one sharded logits row (1, vocab shard): sample_from(distribution(row, T),
        u); returns the token (0-d device tensor) and this rank's shard of the distribution (the Q row of the later
        verification)."""
        gm, kp = self.stats(logits, temperature)
        Q = self.probs(logits, gm, kp, temperature)
        return self.sample_row(self.gather_row(Q[0]), u), Q[0]
