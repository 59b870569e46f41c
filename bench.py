"""Benchmark: accepted tok/s of 8B-shape Q4_K speculative decoding (q = 4) on B200, plus verify-window HBM GB/s.

Workload (one "step" = one speculative round): Llama-3-8B-shaped decoder (32 layers, d_model 4096, 32/8 heads x
128, FFN 14336 SwiGLU, vocab 128,256, RoPE theta 5e5) with random-init weights N(0, 0.02) (counter-based
generator) quantised to GGUF Q4_K, a one-layer MTP draft head, context filled with 4096 seeded random tokens
(prefill), q = 4 linear windows, batch 1, stochastic acceptance at temperature 1 (Philox draws).  A round is:
MTP draft of 3 tokens -> 4-row verify window over all 32 layers + LM head -> rejection-sampling acceptance ->
commit of accepted + 1 positions, all device-resident in one CUDA graph.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

value        emitted tokens / device time of the K timed rounds (inputs resident in HBM)
e2e          the same through clm_b200_spec_round (host API: round parameters host->device, emitted tokens
             device->host, synchronised every round)
roofline     the verify window (32 layers + head, q = 4): algorithmic bytes / event-timed window duration
cpu_baseline the oracle's refmath-order CPU restatement on this host's cores, a bounded sample (one decoder
             layer at context 4096 + the LM head + one MTP step, q = 4) extrapolated to a round
wide_window  128 window rows (8 sequences x 16 tree nodes) through the tcgen05 tensor-core GEMM over one 8B layer's
             Q8_0 matrices: TFLOP/s against the measured bf16 tensor peak
prefill      a 4096-token prompt in 256-row windows through the engine (tcgen05 path): tokens/s, GEMM TFLOP/s
tree_window  C4: a 16-node draft tree at context 4096 in Q8_0, batch 1 (GEMV chain) and batch 8 (eight sessions'
             trees in one 128-row window, clm_b200_run_batch_window): window time and HBM / tensor rooflines
c5_stage     C5 per GPU: a middle stage of 10 layers of the 70B shape (Q4_K), q = 8 windows of boundary records at
             context 8192, four sessions: window time and HBM roofline
With N > 1 (torchrun, one process per GPU) the model is split into N pipeline stages (layer ranges balanced by
the bytes each stage streams per round; the tail holds the LM head and the MTP drafter), joined by device links
over NVLink, with N sequences in flight (--inflight) so that every stage is busy: weak scaling (each GPU streams
about one model's worth of bytes per N rounds).  value = emitted tokens of all sequences / max-over-ranks device
time; the roofline is the per-GPU HBM stream of the timed rounds.
"""
from __future__ import annotations

import argparse
import dataclasses
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

Q = 4
CONTEXT = 4096
TEMPERATURE = 1.0
SEED = 0
METRIC = "accepted tok/s, 8B-shape Q4_K spec decode q=4"

# algorithmic bytes of one q = 4 verify window (weights of 32 layers + LM head, KV of 4096 positions)
def round_bytes(geo, context, q=Q):
    """Algorithmic bytes of one speculative round: the verify window plus q-1 MTP draft steps (MTP block + head)."""
    total, _, _ = window_bytes(geo, context)
    H, F, V = geo.hidden, geo.ffn, geo.vocab
    return total + (q - 1) * (3 * F * H + V * H) * 144 // 256


def window_bytes(geo, context):
    H, qd, kvd, F, V = geo.hidden, geo.n_heads * geo.head_dim, geo.n_kv_heads * geo.head_dim, geo.ffn, geo.vocab
    per_layer = (qd * H + 2 * kvd * H + H * qd + 3 * F * H) * 144 // 256
    head = V * H * 144 // 256
    kv = geo.n_layers * 2 * context * kvd * 2
    return geo.n_layers * per_layer + head + kv, geo.n_layers * per_layer + head, kv


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.lines = []
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.dev}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "50"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()
        # nvidia-smi needs a moment before its first line: start timing only once it is sampling
        t0 = time.time()
        while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
            time.sleep(0.01)
        self.lines.clear()

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=5)
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [x.strip() for x in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(world, value, device):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(world, value, device):
    if world == 1:
        return value
    import torch
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# --------------------------------------------------------------------------- CPU side (oracle)

@dataclasses.dataclass(frozen=True)
class Shape:
    """The decoder shape of the workload (the GPU arm asserts it equals clusterlm_b200.engine.LLAMA3_8B).  Kept here
    so that the reference arm never imports clusterlm_b200, which loads the CUDA library."""
    n_layers: int = 32
    hidden: int = 4096
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 14336
    vocab: int = 128256
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5


SHAPE_8B = Shape()


def bench_config(n_gpus: int, context: int, inflight: int = 1) -> dict:
    """The workload description both arms print as `config` (identical for the same N)."""
    return {"workload": f"llama3-8b-shape q4_k spec decode q={Q} ctx={context} mtp=1-layer T={TEMPERATURE:g}",
            "q": Q, "context": context, "temperature": TEMPERATURE, "batch": 1,
            "weights": "random-init N(0, 0.02) quantised to Q4_K", "parallelism": "single" if n_gpus == 1 else
            f"pp{n_gpus}", "inflight": inflight,
            "l2": "inputs larger than L2 (4.8 GB of weights streamed per round)"}


class CpuRounds:
    """Speculative rounds of the workload on the host cores: the oracle's restatement of the reference's refmath
    order (f32 dot products in ascending order over Q4_K rows decoded one at a time) for the decoder layers, the LM
    head and the MTP head, and its restatement of distribution / sample_from / verify_speculative for the draft
    sampling and the acceptance.  A round is what the GPU arm's round is: 3 MTP drafts (each: the MTP block, the
    head, distribution and a Philox-drawn sample), the 4-row verify window over all 32 layers and the head,
    distribution of the 4 target rows and rejection-sampling acceptance, then the commit (the context grows by the
    emitted tokens).  Weights come from the same counter-based generator as the GPU engine (seed 0, N(0, 0.02),
    Q4_K); the KV context of 4096 positions holds seeded N(0, 1) values (a CPU prefill of 4096 tokens through
    32 layers would take hours)."""

    def __init__(self, threads: int, shape: Shape = SHAPE_8B, context: int = CONTEXT, max_rounds: int = 64):
        import concurrent.futures as cf

        import numpy as np

        from oracle.oracle_py import LlamaDims, Oracle

        self.np, self.o, self.g, self.threads = np, Oracle(), shape, threads
        g, o = shape, self.o
        H, qd, kvd, F, V = g.hidden, g.n_heads * g.head_dim, g.n_kv_heads * g.head_dim, g.ffn, g.vocab
        t0 = time.perf_counter()
        pool = cf.ThreadPoolExecutor(max_workers=threads)

        def gen(tid, n):  # generate + encode in chunks of whole superblocks on all threads (ctypes drops the GIL)
            chunk = 1 << 22
            parts = list(pool.map(lambda f: o.encode("q4_k", o.gen_weights(SEED, tid, f, min(chunk, n - f), 0.02)),
                                  range(0, n, chunk)))
            return np.concatenate(parts)

        self.layers = []
        for L in range(g.n_layers):
            i = 16 * L
            self.layers.append((np.concatenate([gen(i, qd * H), gen(i + 1, kvd * H), gen(i + 2, kvd * H)]),
                                gen(i + 3, H * qd), np.concatenate([gen(i + 4, F * H), gen(i + 5, F * H)]),
                                gen(i + 6, H * F)))
        self.head = gen(1001, V * H)
        self.mtp = (np.concatenate([gen(1002, F * H), gen(1003, F * H)]), gen(1004, H * F))
        pool.shutdown()
        self.ones = np.ones(H, np.float32)
        self.dims = LlamaDims(H, g.n_heads, g.n_kv_heads, g.head_dim, F, g.rope_theta, g.rms_eps)
        rng = np.random.default_rng(4096)
        cap = context + (Q + 1) * max_rounds + 8
        self.kc = [np.zeros((cap, kvd), np.float32) for _ in range(g.n_layers)]
        self.vc = [np.zeros((cap, kvd), np.float32) for _ in range(g.n_layers)]
        for L in range(g.n_layers):
            self.kc[L][:context] = rng.standard_normal((context, kvd), dtype=np.float32)
            self.vc[L][:context] = rng.standard_normal((context, kvd), dtype=np.float32)
        self.pos, self.cap = context, cap
        self.next_token = int(rng.integers(0, V))
        self.round_no = 0
        self.setup_s = time.perf_counter() - t0
        self.parts = {}

    def embed(self, tokens):
        o, g = self.o, self.g
        rows = [o.decode("q4_k", o.encode("q4_k", o.gen_weights(SEED, 1000, int(t) * g.hidden, g.hidden, 0.02)),
                         g.hidden) for t in tokens]
        return self.np.stack(rows).astype(self.np.float32)

    def head_logits(self, h):
        o, g = self.o, self.g
        x = self.np.stack([o.rmsnorm(r, self.ones, g.rms_eps) for r in h])
        return o.matmul_rows_quant("q4_k", self.head, g.vocab, g.hidden, x, self.threads)

    def mtp_logits(self, prev: int):
        np, o, g = self.np, self.o, self.g
        x = self.embed([prev])
        xn = o.rmsnorm(x[0], self.ones, g.rms_eps)[None]
        y = o.matmul_rows_quant("q4_k", self.mtp[0], 2 * g.ffn, g.hidden, xn, self.threads)[0]
        with np.errstate(over="ignore"):
            a = (y[:g.ffn] / (np.float32(1.0) + np.exp(-y[:g.ffn])) * y[g.ffn:]).astype(np.float32)
        d = o.matmul_rows_quant("q4_k", self.mtp[1], g.hidden, g.ffn, a[None], self.threads)[0]
        return self.head_logits((x[0] + d)[None])[0]

    def round(self) -> int:
        """One speculative round; returns the emitted tokens (accepted drafts + 1)."""
        np, o, g = self.np, self.o, self.g
        if self.pos + Q + 1 > self.cap:
            raise RuntimeError("CpuRounds: context capacity reached")
        r = self.round_no
        t0 = time.perf_counter()
        win, dprobs = [self.next_token], []
        for j in range(Q - 1):  # MTP drafts, sampled at T = 1
            p = o.distribution(self.mtp_logits(win[-1]), TEMPERATURE)
            dprobs.append(p)
            win.append(o.sample_from(p, o.philox_uniform(SEED, j, 1, r & 0xFFFFFFFF, r >> 32)))
        t1 = time.perf_counter()
        h = self.embed(win)
        for L, (wqkv, wo, wgu, wd) in enumerate(self.layers):
            o.llama_layer(self.dims, "q4_k", wqkv, wo, wgu, wd, self.ones, self.ones, self.kc[L], self.vc[L],
                          self.pos, h, None, self.threads)
        logits = self.head_logits(h)
        t2 = time.perf_counter()
        P = np.stack([o.distribution(row, TEMPERATURE) for row in logits])
        us = np.array([o.philox_uniform(SEED, n, 0, r & 0xFFFFFFFF, r >> 32) for n in range(Q)])
        acc, nxt, _ = o.verify(P, np.array(win[1:], np.int32), np.stack(dprobs), us)
        t3 = time.perf_counter()
        self.pos += acc + 1  # commit: the accepted window rows stay in the caches
        self.next_token = int(nxt)
        self.round_no += 1
        self.parts = {"draft_s": t1 - t0, "window_s": t2 - t1, "accept_s": t3 - t2}
        return acc + 1

    def sample_text(self, rounds: int, emitted: int) -> str:
        p = self.parts
        return (f"oracle port (refmath-order f32 dot products over Q4_K rows decoded one at a time; double-precision "
                f"distribution / verify_speculative), {self.threads} threads: {rounds} full speculative rounds "
                f"(3 MTP drafts, 32-layer q={Q} window + LM head, acceptance, commit) from context {CONTEXT}, "
                f"{emitted} tokens emitted; last round draft {p.get('draft_s', 0):.2f} s, window "
                f"{p.get('window_s', 0):.2f} s, acceptance {p.get('accept_s', 0):.2f} s; weights generated in "
                f"{self.setup_s:.1f} s (untimed)")


def run_reference(args, world, rank):
    """The reference arm: ClusterLM has no Llama-family CPU code of its own (its llama path is the un-vendored
    llama.cpp), so this runs the oracle's restatement of its refmath-order math on all host threads: W untimed and
    K timed full speculative rounds (CpuRounds), tokens counted from its own acceptance."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    cpu = CpuRounds(threads, max_rounds=args.warmup + args.steps + 2)
    for _ in range(args.warmup):
        cpu.round()
    t0 = time.perf_counter()
    emitted = sum(cpu.round() for _ in range(args.steps))
    sec = time.perf_counter() - t0
    value = emitted / sec
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": sec / args.steps * 1e3,
        "ms_per_round": sec / args.steps * 1e3, "emitted_per_round": emitted / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": bench_config(args.gpus, CONTEXT, args.inflight or args.gpus if args.gpus > 1 else 1),
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": threads, "kind": "port",
                         "sample": cpu.sample_text(args.steps, emitted)},
        "e2e": {"value": value, "unit": "tok/s", "ms_per_round": sec / args.steps * 1e3, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------- GPU side

def profile_case(args) -> bool:
    return args.layers != 32 or args.context != CONTEXT


# acceptance micro-workload: 64 sequences x q = 8 (k = 7 drafts) x vocab 151,936, target logits ~ N(0, 3^2), draft
# logits = target + N(0, 0.5^2), drafts sampled from the draft distribution, Philox seed 0, T = 1
C2_B, C2_Q, C2_V = 64, 8, 151936


def acceptance_micro(ctx, dev, peak, with_cpu):
    """clm_b200_accept_logits on the acceptance micro-workload, device-resident inputs, event-timed."""
    import numpy as np
    import torch

    from clusterlm_b200.runtime import accept_logits

    g = torch.Generator(device=dev).manual_seed(0)
    k = C2_Q - 1
    tl = torch.randn((C2_B, C2_Q, C2_V), generator=g, device=dev) * 3.0
    dl = tl[:, :k] + torch.randn((C2_B, k, C2_V), generator=g, device=dev) * 0.5
    drafts = torch.multinomial(torch.softmax(dl.reshape(-1, C2_V), dim=-1), 1, generator=g).reshape(C2_B, k)
    drafts = drafts.to(torch.int32).contiguous()
    for _ in range(3):
        accept_logits(ctx, tl, dl, drafts, 1.0, seed=0, counter_base=0)
    torch.cuda.synchronize(dev)
    n = 10
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for i in range(n):
        acc, nxt = accept_logits(ctx, tl, dl, drafts, 1.0, seed=0, counter_base=i)
    s1.record()
    torch.cuda.synchronize(dev)
    sec = s0.elapsed_time(s1) / 1e3 / n
    # logits read once plus the residual sample's two rows per sequence
    algo = (C2_B * (C2_Q + k) + 2 * C2_B) * C2_V * 4
    out = {"config": f"{C2_B} sequences x q={C2_Q} (k={k}) x vocab {C2_V}, logits N(0,3^2), drafts +N(0,0.5^2), "
                     "Philox seed 0, T=1",
           "ms_per_call": sec * 1e3, "sequences_per_s": C2_B / sec,
           "accepted_mean": float(acc.float().mean().item()),
           "roofline": {"bound": "hbm", "algorithmic_bytes": algo, "achieved": algo / sec / 1e9, "peak": peak,
                        "unit": "GB/s", "frac": algo / sec / 1e9 / peak}}
    if with_cpu:
        from oracle.oracle_py import Oracle

        orc = Oracle()
        t0 = time.perf_counter()
        t = tl[0].cpu().numpy()
        d = dl[0].cpu().numpy()
        P = np.stack([orc.distribution(r, 1.0) for r in t])
        Q = np.stack([orc.distribution(r, 1.0) for r in d])
        us = np.array([orc.philox_uniform(0, j, 0, 0, 0) for j in range(k + 1)])
        orc.verify(P, drafts[0].cpu().numpy(), Q, us)
        one = time.perf_counter() - t0
        out["cpu_baseline"] = {"value": 1.0 / one, "unit": "sequences/s", "cores": 1, "kind": "port",
                               "sample": "oracle distribution (stable sort, double) + verify_speculative, one "
                                         f"sequence ({C2_Q + k} rows) timed ({one:.2f} s)"}
    del tl, dl
    return out


# tree-window micro-workload: the 8B shape in Q8_0 with a 16-node draft tree (root; 4 children; 2 children each;
# 3 nodes at depth 3, so 16 = max_window nodes), context 4096, batch 1 (one sequence per window)
C4_PARENTS = [-1, 0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 6, 7]


C4_BATCH = 8


def tree_micro(ctx, dev, peak, context):
    """C4: 16-node tree verification windows (Q8_0 8B shape, context `context` per sequence).
    batch 1: one sequence's tree through clm_b200_run_tree_window_device (the GEMV chain), event-timed on the
    engine's stream.  batch 8: eight sequences' trees in ONE window through clm_b200_run_batch_window (128 rows:
    tcgen05 GEMMs, each weight matrix read once; per-sequence RoPE/KV and attention; a CUDA graph per session
    set), timed by events on the engine stream around the host call."""
    import numpy as np
    import torch

    from clusterlm_b200.engine import LLAMA3_8B, ROLE_WHOLE, Engine

    geo = dataclasses.replace(LLAMA3_8B, quant="q8_0")
    q = len(C4_PARENTS)
    wmax = C4_BATCH * q
    eng = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, context + 64, wmax, C4_BATCH)
    eng.generate_weights(seed=SEED, stddev=0.02)
    eng.prepare()
    eng.open_session(1)
    rng = np.random.default_rng(77)
    eng.spec_begin(1, rng.integers(0, geo.vocab, context).astype(np.int32), 4)
    stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    parents = torch.tensor(C4_PARENTS, dtype=torch.int32, device=dev)
    toks = torch.from_numpy(rng.integers(0, geo.vocab, q).astype(np.int32)).to(dev)
    logits = torch.empty((q, geo.vocab), dtype=torch.float32, device=dev)
    pos = eng.position(1)
    times = []
    for i in range(8):
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        eng.run_tree_window_device(1, pos, parents, toks, logits, stream.cuda_stream)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        eng.abort(1)
        if i >= 3:
            times.append(s0.elapsed_time(s1) / 1e3)
    sec = statistics.median(times)
    # batch 8: sessions 2..8 prefilled in wmax-row windows (device tokens), then one 128-row window per call
    pre_out = torch.empty((wmax, geo.vocab), dtype=torch.float32, device=dev)
    for b in range(2, C4_BATCH + 1):
        eng.open_session(b)
        prompt = torch.from_numpy(rng.integers(0, geo.vocab, context).astype(np.int32)).to(dev)
        for off in range(0, context, wmax):
            n = min(wmax, context - off)
            eng.run_window_device(b, off, prompt[off:off + n], pre_out[:n], stream.cuda_stream)
            eng.commit(b, n)
    ids = list(range(1, C4_BATCH + 1))
    bases = [eng.position(b) for b in ids]
    btoks = rng.integers(0, geo.vocab, (C4_BATCH, q)).astype(np.int32)
    btimes, bwall = [], []
    for i in range(6):
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        s0.record(stream)
        eng.run_batch_window(ids, bases, btoks, C4_PARENTS, logits=False)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        t1 = time.perf_counter()
        for b in ids:
            eng.abort(b)
        if i >= 2:
            btimes.append(s0.elapsed_time(s1) / 1e3)
            bwall.append(t1 - t0)
    bsec = statistics.median(btimes)
    for b in ids:
        eng.close_session(b)
    eng.close()
    H, qd, kvd, F, V = geo.hidden, geo.n_heads * geo.head_dim, geo.n_kv_heads * geo.head_dim, geo.ffn, geo.vocab
    params = geo.n_layers * (qd * H + 2 * kvd * H + H * qd + 3 * F * H) + V * H
    weights = params * 34 // 32
    kv = geo.n_layers * 2 * context * kvd * 2
    algo = weights + kv
    balgo = weights + C4_BATCH * kv
    bflops = 2.0 * C4_BATCH * q * params
    tpeak, tkind = load_tensor_peak()
    return {"config": f"8B-shape Q8_0, 16-node draft tree (parents {C4_PARENTS}), context {context}",
            "ms_per_window": sec * 1e3, "windows_per_s": 1.0 / sec,
            "roofline": {"bound": "hbm", "algorithmic_bytes": algo, "weight_bytes": weights, "kv_bytes": kv,
                         "achieved": algo / sec / 1e9, "peak": peak, "unit": "GB/s", "frac": algo / sec / 1e9 / peak},
            "batch8": {"config": f"{C4_BATCH} sequences x {q}-node trees = {C4_BATCH * q} rows in one window "
                                 "(clm_b200_run_batch_window), no logits read back",
                       "ms_per_window": bsec * 1e3, "host_ms_per_call": statistics.median(bwall) * 1e3,
                       "tree_nodes_per_s": C4_BATCH * q / bsec,
                       "roofline": {"bound": "hbm", "algorithmic_bytes": balgo, "achieved": balgo / bsec / 1e9,
                                    "peak": peak, "unit": "GB/s", "frac": balgo / bsec / 1e9 / peak},
                       "tensor": {"gemm_flops": bflops, "achieved": bflops / bsec / 1e12, "peak": tpeak,
                                  "unit": "TFLOP/s", "frac": bflops / bsec / 1e12 / tpeak, "peak_kind": tkind}}}


# C5: one middle stage of the 70B shape in an 8-stage plan (10 of 80 layers, Q4_K), q = 8, batch 4, context 8192
C5_LAYERS, C5_Q, C5_BATCH, C5_CONTEXT = 10, 8, 4, 8192


def c5_micro(ctx, dev, peak):
    """C5 per GPU: a middle stage holding 10 layers of the 70B shape (Q4_K) with four sessions at context 8192.
    Each verify window (q = 8 boundary records in, records out, clm_b200_run_window_device) is event-timed on the
    engine stream and dropped; batch 4 is one window over the four sessions (32 rows,
    clm_b200_run_batch_window_device), which streams the stage's weights once."""
    import numpy as np
    import torch

    from clusterlm_b200.engine import LLAMA3_70B, ROLE_MIDDLE, Engine

    geo = LLAMA3_70B
    H = geo.hidden
    fpp = 2 * H + 1
    eng = Engine(ctx, geo, 30, 30 + C5_LAYERS, ROLE_MIDDLE, C5_CONTEXT + 64, 32, C5_BATCH)
    eng.generate_weights(seed=SEED, stddev=0.02)
    eng.prepare()
    stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    gen = torch.Generator(device=dev).manual_seed(55)
    rows = C5_BATCH * C5_Q
    rec = torch.zeros((rows, fpp), dtype=torch.float32, device=dev)
    rec[:, :H] = torch.randn((rows, H), generator=gen, device=dev)
    rec[:, 2 * H] = 1.0
    out = torch.empty((rows, fpp), dtype=torch.float32, device=dev)
    for b in range(1, C5_BATCH + 1):
        eng.open_session(b)
        for off in range(0, C5_CONTEXT, 16):
            eng.run_window_device(b, off, d_out=out[:16], stream=stream.cuda_stream, d_records=rec[:16])
            eng.commit(b, 16)
    times = []
    for i in range(6):
        per = []
        for b in range(1, C5_BATCH + 1):
            torch.cuda.synchronize(dev)
            s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s0.record(stream)
            eng.run_window_device(b, C5_CONTEXT, d_out=out[:C5_Q], stream=stream.cuda_stream, d_records=rec[:C5_Q])
            s1.record(stream)
            torch.cuda.synchronize(dev)
            eng.abort(b)
            per.append(s0.elapsed_time(s1) / 1e3)
        if i >= 2:
            times.extend(per)
    batch = []
    ids = list(range(1, C5_BATCH + 1))
    for i in range(6):
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        eng.run_batch_window_device(ids, [C5_CONTEXT] * C5_BATCH, C5_Q, d_records=rec, d_out=out,
                                    stream=stream.cuda_stream)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        for b in ids:
            eng.abort(b)
        if i >= 2:
            batch.append(s0.elapsed_time(s1) / 1e3)
    del rec, out
    torch.cuda.synchronize(dev)
    for b in range(1, C5_BATCH + 1):
        eng.close_session(b)
    eng.close()
    sec = statistics.median(times)
    bsec = statistics.median(batch)
    qd, kvd, F = geo.n_heads * geo.head_dim, geo.n_kv_heads * geo.head_dim, geo.ffn
    params = C5_LAYERS * ((qd + 2 * kvd) * H + H * qd + 3 * F * H)
    weights = params * 144 // 256
    kv = C5_LAYERS * 2 * C5_CONTEXT * kvd * 2
    algo = weights + kv
    balgo = weights + C5_BATCH * kv  # the batch streams the weights once and every session's KV
    return {"config": f"70B-shape middle stage: layers 30-39 of 80 (Q4_K), q={C5_Q} boundary records in and out, "
                      f"context {C5_CONTEXT}, {C5_BATCH} sessions",
            "ms_per_window": sec * 1e3, "batch4_ms": bsec * 1e3, "batch4_separate_ms": C5_BATCH * sec * 1e3,
            "roofline": {"bound": "hbm", "algorithmic_bytes": algo, "weight_bytes": weights, "kv_bytes": kv,
                         "achieved": algo / sec / 1e9, "peak": peak, "unit": "GB/s", "frac": algo / sec / 1e9 / peak},
            "batch4_roofline": {"bound": "hbm", "algorithmic_bytes": balgo, "achieved": balgo / bsec / 1e9,
                                "peak": peak, "unit": "GB/s", "frac": balgo / bsec / 1e9 / peak}}


def load_tensor_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    return 1590.0, "fallback"


def wide_micro(ctx, dev):
    """The C4 batch's weight stream as one wide window: 8 sequences x 16 tree nodes = 128 rows through the
    tcgen05 GEMM (clm_b200_matmul_rows with 128 positions) over one 8B-shape decoder layer's matrices in Q8_0
    (qkv, o, gate|up, down), event-timed back to back with device-resident inputs; 32 layers extrapolated."""
    import torch

    from clusterlm_b200.runtime import Matrix, generate_weights, encode

    rows_q = 128
    shapes = {"qkv": (6144, 4096), "o": (4096, 4096), "gate|up": (28672, 4096), "down": (4096, 14336)}
    mats, xs, ys = [], [], []
    for tid, (name, (r, c)) in enumerate(shapes.items()):
        w = generate_weights(ctx, SEED, 900 + tid, 0, r * c, 0.02)
        mats.append(Matrix(ctx, "q8_0", encode(ctx, "q8_0", w), r, c))
        del w
        xs.append(torch.randn((rows_q, c), device=dev, generator=torch.Generator(device=dev).manual_seed(tid)))
        ys.append(torch.empty((rows_q, r), device=dev))
    torch.cuda.synchronize(dev)
    for _ in range(3):
        for m, x, y in zip(mats, xs, ys):
            m.matmul_rows(x, y)
    torch.cuda.synchronize(dev)
    n = 10
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for _ in range(n):
        for m, x, y in zip(mats, xs, ys):
            m.matmul_rows(x, y)
    s1.record()
    torch.cuda.synchronize(dev)
    sec = s0.elapsed_time(s1) / 1e3 / n
    for m in mats:
        m.close()
    params = sum(r * c for r, c in shapes.values())
    flops = 2.0 * rows_q * params
    peak, kind = load_tensor_peak()
    tf = flops / sec / 1e12
    return {"config": "one 8B-shape decoder layer (qkv 6144x4096, o 4096^2, gate|up 28672x4096, down 4096x14336), "
                      "Q8_0, 128 window rows (8 sequences x 16 tree nodes), x f32 in, y f32 out",
            "ms_per_layer": sec * 1e3, "ms_per_32_layers": 32 * sec * 1e3,
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_kind": kind, "flops_per_layer": flops,
                         "weight_gbs": params * 34 / 32 / sec / 1e9}}


PREFILL_CHUNK = 256


def prefill_micro(eng, geo, dev, stream, context, rng):
    """Prefill of a `context`-token prompt in 256-row windows (the tcgen05 GEMM path of the engine) on session 2 of
    the bench engine: each window is event-timed on the engine stream and committed.  Tensor roofline over the
    GEMM flops (every window row through every layer matrix and the head); the time also holds the attention and
    the elementwise steps."""
    import numpy as np
    import torch

    ch = PREFILL_CHUNK
    n = context - context % ch
    prompt = torch.from_numpy(rng.integers(0, geo.vocab, max(n, ch)).astype(np.int32)).to(dev)
    out = torch.empty((ch, geo.vocab), dtype=torch.float32, device=dev)
    eng.open_session(2)
    for _ in range(3):  # eager, graph capture, replay
        eng.run_window_device(2, 0, prompt[:ch], out, stream.cuda_stream)
        torch.cuda.synchronize(dev)
        eng.abort(2)
    times = []
    for off in range(0, n, ch):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        eng.run_window_device(2, off, prompt[off:off + ch], out, stream.cuda_stream)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        eng.commit(2, ch)
        times.append(s0.elapsed_time(s1) / 1e3)
    eng.close_session(2)
    if not times:
        return None
    sec = sum(times)
    H, F, V = geo.hidden, geo.ffn, geo.vocab
    qd, kvd = geo.n_heads * geo.head_dim, geo.n_kv_heads * geo.head_dim
    params = geo.n_layers * ((qd + 2 * kvd) * H + H * qd + 2 * F * H + H * F) + V * H
    flops = 2.0 * n * params
    peak, kind = load_tensor_peak()
    tf = flops / sec / 1e12
    return {"config": f"{n}-token prompt in {ch}-row windows through the engine (tcgen05 GEMMs, paged fp16 KV), "
                      f"{geo.quant} {geo.n_layers}-layer 8B shape, logits for every row",
            "tok_s": n / sec, "ms_per_window": 1e3 * sec / len(times),
            "ms_first_window": 1e3 * times[0], "ms_last_window": 1e3 * times[-1],
            "roofline": {"bound": "tensor", "achieved": tf, "peak": peak, "unit": "TFLOP/s", "frac": tf / peak,
                         "peak_kind": kind, "gemm_flops": flops}}


# DRAM bytes (read + write) of one verify window (q = 4, context 4096), keyed by layer count: an ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum, caches not flushed between kernels) of every kernel of one window
# of `bench.py --micro window --layers 8`; 32 layers = the head and embedding kernels + 4 x the 8 layers' kernels.
# The capture and its command are summarised under profiles/.
WINDOW_TRAFFIC: dict = {8: 1530851840, 32: 5100370688}


def c1_fixture():
    """C1 (the reference's own fixture model, 4-stage plan, q = 4, ScriptedDrafter corruption 0.3, 32 new tokens):
    the reference's ReferenceDomain pipeline (its own compiled CPU code, 1 thread per stage) against the b200
    pipeline (the product's C++ backend behind the same ExecutionDomain interface), both driven in one process by
    the drop-in parity driver built from the reference sources.  None when the driver is not built."""
    import tempfile

    exe = os.path.join(ROOT, "oracle", "_ref", "backend_parity")
    if not os.path.exists(exe):
        return None
    with tempfile.TemporaryDirectory() as d:
        r = subprocess.run([exe, d, "--bench"], capture_output=True, text=True, timeout=600)
    for ln in r.stdout.splitlines():
        if ln.startswith("{"):
            o = json.loads(ln)
            o["config"] = ("clusterlm-fixture default spec (16 layers, H 64, hc 4, 32 experts top-4, V 256), plan "
                           "0-4|4-10|10-13|13-16 in one process, q=4, ScriptedDrafter corruption 0.3, 32 new tokens")
            o["parity_failures"] = r.returncode
            return o
    return {"error": (r.stdout + r.stderr)[-300:]}


def run_b200(args, world, rank, local):
    import numpy as np
    import torch

    from clusterlm_b200.engine import LLAMA3_8B, ROLE_WHOLE, Engine
    from clusterlm_b200.runtime import Context

    torch.cuda.set_device(local)
    dev = torch.device(f"cuda:{local}")
    assert all(getattr(LLAMA3_8B, f.name) == getattr(SHAPE_8B, f.name) for f in dataclasses.fields(Shape))
    geo = LLAMA3_8B if args.layers == LLAMA3_8B.n_layers else dataclasses.replace(LLAMA3_8B, n_layers=args.layers)
    context = args.context
    ctx = Context(local)
    n_rounds = args.warmup + args.steps
    max_ctx = context + (n_rounds + 8) * (Q + 1) + 64
    # windows of up to 256 rows: the prompt is prefilled in 256-row windows on the tensor-core path (the profile
    # case keeps 16-row prefill windows, so its launch list matches the recorded ncu skip counts)
    wmax = 16 if profile_case(args) else PREFILL_CHUNK
    # sessions: 1 the device-resident rounds, 3 the same rounds through the host API (same prompt and seed, so the
    # same emitted tokens), 2 the prefill measurement
    eng = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, max_ctx, wmax, 3)
    eng.generate_weights(seed=SEED, stddev=0.02)
    eng.prepare()
    rng = np.random.default_rng(1234 + rank)
    prompt = rng.integers(0, geo.vocab, context).astype(np.int32)
    t0 = time.perf_counter()
    for sid in (1, 3):
        eng.open_session(sid)
        eng.spec_begin(sid, prompt, Q, temperature=TEMPERATURE, seed=SEED)
    prefill_s = (time.perf_counter() - t0) / 2
    stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    counts = torch.zeros(n_rounds, dtype=torch.int32, device=dev)
    toks = torch.zeros((n_rounds, Q + 1), dtype=torch.int32, device=dev)
    for i in range(args.warmup):
        eng.spec_round_device(1, Q, TEMPERATURE, SEED, toks[i], counts[i], stream.cuda_stream)
    torch.cuda.synchronize(dev)
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    start.record(stream)
    for i in range(args.warmup, n_rounds):
        eng.spec_round_device(1, Q, TEMPERATURE, SEED, toks[i], counts[i], stream.cuda_stream)
    end.record(stream)
    torch.cuda.synchronize(dev)
    clk = clocks.stop()
    launches = eng.last_launches()
    elapsed = start.elapsed_time(end) / 1e3
    emitted = int(counts[args.warmup:].sum().item())
    elapsed_max = max_over_ranks(world, elapsed, dev)
    emitted_all = sum_over_ranks(world, emitted, dev)
    value = emitted_all / elapsed_max

    # e2e: the same W + K rounds on session 3 through the host API (round parameters host -> device and the emitted
    # tokens device -> host every round, synchronised); the K rounds after the warm-up are timed on the host
    barrier(world)
    torch.cuda.synchronize(dev)
    host_tokens = []
    for _ in range(args.warmup):
        host_tokens.append(eng.spec_round(3, Q, TEMPERATURE, SEED))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        host_tokens.append(eng.spec_round(3, Q, TEMPERATURE, SEED))
    e2e_s = time.perf_counter() - t0
    e_emitted = sum(t.size for t in host_tokens[args.warmup:])
    dev_tokens = [toks[i, :int(counts[i])].cpu().numpy() for i in range(n_rounds)]
    e2e_same = all(np.array_equal(a, b) for a, b in zip(host_tokens, dev_tokens))
    e2e_s = max_over_ranks(world, e2e_s, dev)
    e2e_value = sum_over_ranks(world, e_emitted, dev) / e2e_s
    eng.close_session(3)

    # verify-window roofline: one q = 4 window through the public window call, event-timed
    total_b, weight_b, kv_b = window_bytes(geo, context)
    pos = eng.position(1)
    wt = []
    wtoks = torch.from_numpy(rng.integers(0, geo.vocab, Q).astype(np.int32)).to(dev)
    wlogits = torch.empty((Q, geo.vocab), dtype=torch.float32, device=dev)
    for i in range(8):
        torch.cuda.synchronize(dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        eng.run_window_device(1, pos, wtoks, wlogits, stream.cuda_stream)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        eng.abort(1)
        if i >= 3:
            wt.append(s0.elapsed_time(s1) / 1e3)
    window_s = statistics.median(wt)
    peak, peak_kind = load_peaks()
    achieved = total_b / window_s / 1e9
    eng.close_session(1)
    prefill = prefill_micro(eng, geo, dev, stream, context, rng) if (world == 1 and wmax > 16) else None
    eng.close()
    micro = acceptance_micro(ctx, dev, peak, not args.no_cpu) if (world == 1 and not profile_case(args)) else None
    tree = tree_micro(ctx, dev, peak, context) if (world == 1 and not profile_case(args)) else None
    wide = wide_micro(ctx, dev) if (world == 1 and not profile_case(args)) else None
    c5 = c5_micro(ctx, dev, peak) if (world == 1 and not profile_case(args)) else None
    ctx.close()

    if rank != 0:
        return
    profile = profile_case(args)
    cpu, c1 = None, None
    if world == 1 and not args.no_cpu and not profile:
        cr = CpuRounds(os.cpu_count() or 1, max_rounds=4)
        cr.round()  # untimed
        t0 = time.perf_counter()
        n_cpu = 2
        cpu_emitted = sum(cr.round() for _ in range(n_cpu))
        cpu_s = time.perf_counter() - t0
        cpu = {"value": cpu_emitted / cpu_s, "unit": "tok/s", "cores": cr.threads, "kind": "port",
               "ms_per_round": cpu_s / n_cpu * 1e3, "sample": cr.sample_text(n_cpu, cpu_emitted)}
        del cr
        c1 = c1_fixture()
    config = bench_config(world, context)
    if profile:
        config["workload"] += f" PROFILE CASE ({geo.n_layers} layers)"
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_max / args.steps * 1e3,
        "ms_per_round": elapsed_max / args.steps * 1e3, "emitted_per_round": emitted / args.steps,
        "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_k weights, fp16 operands, f32 accumulate",
        "data": "synthetic (random-init N(0,0.02) weights, seeded random context tokens)",
        "config": config,
        "prefill_s": round(prefill_s, 2),
        "e2e": {"value": e2e_value, "unit": "tok/s", "ms_per_round": e2e_s / args.steps * 1e3,
                "rounds": args.steps, "same_tokens_as_device_rounds": bool(e2e_same),
                "h2d_bytes_per_step": 16, "d2h_bytes_per_step": (Q + 1) * 4 + 4},
        "gpu_launches": launches * args.steps,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": WINDOW_TRAFFIC.get(geo.n_layers), "peak_kind": peak_kind,
                     "kernel": f"verify window q=4 ({geo.n_layers} layers + head)",
                     "algorithmic_bytes": total_b, "weight_bytes": weight_b, "kv_bytes": kv_b,
                     "window_ms": window_s * 1e3},
        "clocks": clk,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    if c1:
        line["c1_fixture"] = c1
    if micro:
        line["acceptance_micro"] = micro
    if tree:
        line["tree_window"] = tree
    if wide:
        line["wide_window"] = wide
    if prefill:
        line["prefill"] = prefill
    if c5:
        line["c5_stage"] = c5
    print(json.dumps(line), flush=True)


def sharded_head_micro(ctx, dev, world, rank, steps=20):
    """The vocab-sharded LM head on the N GPUs of the pipeline job (NCCL): the 8B head (128,256 x 4,096, Q4_K)
    split by vocabulary, one q = 4 verify window per step: the shard logits, the global statistics of the target
    and draft rows and the speculative acceptance over the shards.  Event-timed on each rank, max over ranks;
    rank 0 also times the unsharded head and clm_b200_accept_logits on its own GPU."""
    import numpy as np
    import torch

    from clusterlm_b200.engine import LLAMA3_8B
    from clusterlm_b200.runtime import Matrix, accept_logits, encode, generate_weights
    from clusterlm_b200.sharded_head import ShardedHead, shard_bounds

    V, H = LLAMA3_8B.vocab, LLAMA3_8B.hidden
    v0, v1 = shard_bounds(V, world)[rank]
    head = ShardedHead(ctx, "q4_k", encode(ctx, "q4_k", generate_weights(ctx, SEED, 1001, v0 * H, (v1 - v0) * H, 0.02)),
                       V, H)
    g = torch.Generator().manual_seed(3)
    x = (torch.randn((2 * Q - 1, H), generator=g)).to(dev)
    drafts = [int(d) for d in np.random.default_rng(4).integers(0, V, Q - 1)]

    def step(i):
        L = head.logits(x)
        return head.accept(L[:Q].contiguous(), L[Q:].contiguous(), drafts, TEMPERATURE, seed=SEED, counter_base=i)

    for i in range(3):
        step(i)
    torch.cuda.synchronize(dev)
    barrier(world)
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s0.record()
    for i in range(steps):
        step(i)
    s1.record()
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(world, s0.elapsed_time(s1) / steps, dev)
    head.close()
    out = {"config": f"8B head {V} x {H} Q4_K split by vocabulary over {world} GPUs ({v1 - v0} columns on rank "
                     f"{rank}), q={Q} window, T={TEMPERATURE:g}, stochastic drafts; logits + global max / kept "
                     "(NCCL all-gathers in column order) + acceptance", "ms_per_window": ms}
    if rank == 0:
        whole = Matrix(ctx, "q4_k", encode(ctx, "q4_k", generate_weights(ctx, SEED, 1001, 0, V * H, 0.02)), V, H)
        dd = torch.tensor([drafts], dtype=torch.int32, device=dev)

        def one(i):
            L = whole.matmul_rows(x)
            return accept_logits(ctx, L[:Q].reshape(1, Q, V), L[Q:].reshape(1, Q - 1, V), dd, TEMPERATURE, seed=SEED,
                                 counter_base=i)

        for i in range(3):
            one(i)
        torch.cuda.synchronize(dev)
        s0.record()
        for i in range(steps):
            one(i)
        s1.record()
        torch.cuda.synchronize(dev)
        out["unsharded_ms_per_window"] = s0.elapsed_time(s1) / steps
        whole.close()
    return out


def run_pipeline(args, world, rank, local):
    """N > 1: the stage pipeline (clusterlm_b200.pipeline) with `inflight` sequences."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from clusterlm_b200.engine import LLAMA3_8B
    from clusterlm_b200.pipeline import StagePipeline, format_plan, parse_plan, plan_stages
    from clusterlm_b200.runtime import Context

    dev = torch.device(f"cuda:{local}")
    geo = LLAMA3_8B if args.layers == LLAMA3_8B.n_layers else dataclasses.replace(LLAMA3_8B, n_layers=args.layers)
    context = args.context
    S = args.inflight or world
    plan = parse_plan(args.plan, geo.n_layers) if args.plan else plan_stages(geo, world, Q, context, sessions=S)
    e2e_n = args.steps  # the e2e leg runs as many rounds as the timed loop
    max_ctx = context + (args.warmup + args.steps + 8) * (Q + 1) + 64
    ctx = Context(local)

    def gather(obj):
        res = [None] * world
        dist.all_gather_object(res, obj)
        return res

    # sessions 1..S, S sequences in flight.  The e2e leg continues the same sessions through the host API: a stage's
    # inbound link is one FIFO for all sessions and the tail sends every session's next window at the end of its
    # round, so a fresh session's first window would queue behind the timed sessions' last ones
    pipe = StagePipeline(ctx, geo, plan, rank, max_ctx, S, gather, max_window=16, timeout_s=60.0, weight_seed=SEED)
    stream = torch.cuda.ExternalStream(pipe.engine.stream(), device=dev)
    t0 = time.perf_counter()
    for s in range(S):
        prompt = np.random.default_rng(1234 + s).integers(0, geo.vocab, context).astype(np.int32)
        pipe.open_session(s + 1)
        row = pipe.prefill(s + 1, prompt)
        pipe.begin(s + 1, row, Q, TEMPERATURE, SEED)
    pipe.status()
    barrier(world)
    prefill_s = max_over_ranks(world, time.perf_counter() - t0, dev)
    n_rounds = args.warmup + args.steps
    toks = torch.zeros((n_rounds, S, Q + 1), dtype=torch.int32, device=dev)
    cnt = torch.zeros((n_rounds, S), dtype=torch.int32, device=dev)
    torch.cuda.synchronize(dev)
    for k in range(args.warmup):
        for s in range(S):
            pipe.round(s + 1, Q, TEMPERATURE, SEED, toks[k, s], cnt[k, s])
    pipe.status()
    barrier(world)
    clocks = ClockSampler(local)
    clocks.start()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for k in range(args.warmup, n_rounds):
        for s in range(S):
            pipe.round(s + 1, Q, TEMPERATURE, SEED, toks[k, s], cnt[k, s])
    end.record(stream)
    pipe.status()
    clk = clocks.stop()
    launches = pipe.engine.last_launches() * args.steps * sum(pipe.runs(s + 1) for s in range(S))
    elapsed = start.elapsed_time(end) / 1e3
    emitted = int(cnt[args.warmup:].sum().item()) if pipe.is_tail else 0
    elapsed_max = max_over_ranks(world, elapsed, dev)
    emitted_all = sum_over_ranks(world, emitted, dev)
    launches_all = sum_over_ranks(world, launches, dev)
    value = emitted_all / elapsed_max

    # e2e: as many further rounds of the same sessions with the emitted tokens read back to pinned host memory every
    # round (the tail) and the round parameters copied host -> device every round (every stage), timed on the host,
    # max over ranks
    host = torch.zeros((n_rounds, S, Q + 1), dtype=torch.int32).pin_memory()
    hcnt = torch.zeros((n_rounds, S), dtype=torch.int32).pin_memory()
    e_toks = torch.zeros((S, Q + 1), dtype=torch.int32, device=dev)
    e_cnt = torch.zeros(S, dtype=torch.int32, device=dev)

    def host_rounds(k0, k1):
        with torch.cuda.stream(stream):
            for k in range(k0, k1):
                for s in range(S):
                    pipe.round(s + 1, Q, TEMPERATURE, SEED, e_toks[s], e_cnt[s], stream.cuda_stream)
                    if pipe.is_tail:
                        host[k, s].copy_(e_toks[s], non_blocking=True)
                        hcnt[k, s].copy_(e_cnt[s], non_blocking=True)
        stream.synchronize()

    host_rounds(0, args.warmup)
    torch.cuda.synchronize(dev)
    barrier(world)
    t0 = time.perf_counter()
    host_rounds(args.warmup, n_rounds)
    e2e_s = max_over_ranks(world, time.perf_counter() - t0, dev)
    e2e_emitted = sum_over_ranks(world, int(hcnt[args.warmup:].sum().item()) if pipe.is_tail else 0, dev)
    pipe.status()
    # torch buffers used on the engine's stream are released while that stream still exists (the pinned host
    # allocator records an event on it when a buffer is freed)
    del host, hcnt, e_toks, e_cnt, toks, cnt
    torch.cuda.synchronize(dev)
    pipe.close(lambda: barrier(world))
    sharded = sharded_head_micro(ctx, dev, world, rank) if not profile_case(args) else None
    ctx.close()
    if rank != 0:
        return
    peak, peak_kind = load_peaks()
    per_gpu = S * args.steps * round_bytes(geo, context) / world / elapsed_max / 1e9
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_max / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "q4_k weights, fp16 operands, f32 accumulate",
        "data": "synthetic (random-init N(0,0.02) weights, seeded random context tokens)",
        "config": bench_config(world, context, S),
        "plan": format_plan(plan), "tail_replicas": pipe.tails, "step": f"one round of each of the {S} sequences",
        "ms_per_round": elapsed_max / (args.steps * S) * 1e3, "emitted_per_round": emitted_all / (args.steps * S),
        "prefill_s": round(prefill_s, 2),
        "e2e": {"value": e2e_emitted / e2e_s, "unit": "tok/s", "ms_per_round": e2e_s / (e2e_n * S) * 1e3,
                "rounds": e2e_n, "sessions": "the device-timed sessions' next rounds",
                "emitted_per_round": e2e_emitted / (e2e_n * S),
                "h2d_bytes_per_step": 16 * S * world,
                "d2h_bytes_per_step": ((Q + 1) * 4 + 4) * S},
        "gpu_launches": int(launches_all),
        "roofline": {"bound": "hbm", "achieved": per_gpu, "peak": peak, "unit": "GB/s", "frac": per_gpu / peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": "pipeline rounds, per GPU (all stages' weights + KV + MTP drafts / N / device time)",
                     "algorithmic_bytes_per_round": round_bytes(geo, context)},
        "clocks": clk,
    }
    if sharded:
        line["sharded_head"] = sharded
    print(json.dumps(line), flush=True)


def window_micro(ctx, dev, args):
    """The C3 verify window alone: an 8B-shape Q4_K engine with `--layers` decoder layers, the `--context` prompt
    prefilled in 256-row windows, then `--warmup` untimed and `--steps` (at most 50) event-timed q = 4 windows on
    the engine stream, each aborted after it runs.  A small command for launch lists and DRAM-traffic captures of
    one window's kernels (the prefill's launches come first)."""
    import numpy as np
    import torch

    from clusterlm_b200.engine import LLAMA3_8B, ROLE_WHOLE, Engine

    geo = LLAMA3_8B if args.layers == LLAMA3_8B.n_layers else dataclasses.replace(LLAMA3_8B, n_layers=args.layers)
    context = args.context
    eng = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, context + 64, PREFILL_CHUNK, 1)
    eng.generate_weights(seed=SEED, stddev=0.02)
    eng.prepare()
    eng.open_session(1)
    stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
    rng = np.random.default_rng(1)
    prompt = torch.from_numpy(rng.integers(0, geo.vocab, context).astype(np.int32)).to(dev)
    out = torch.empty((PREFILL_CHUNK, geo.vocab), dtype=torch.float32, device=dev)
    for off in range(0, context, PREFILL_CHUNK):
        n = min(PREFILL_CHUNK, context - off)
        eng.run_window_device(1, off, prompt[off:off + n], out[:n], stream.cuda_stream)
        eng.commit(1, n)
    toks = torch.from_numpy(rng.integers(0, geo.vocab, Q).astype(np.int32)).to(dev)
    logits = torch.empty((Q, geo.vocab), dtype=torch.float32, device=dev)
    times = []
    for i in range(args.warmup + min(args.steps, 50)):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        eng.run_window_device(1, context, toks, logits, stream.cuda_stream)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        eng.abort(1)
        if i >= args.warmup:
            times.append(s0.elapsed_time(s1) / 1e3)
    eng.close()
    sec = statistics.median(times)
    total_b, weight_b, kv_b = window_bytes(geo, context)
    peak, kind = load_peaks()
    return {"config": f"8B-shape Q4_K verify window, q={Q}, {geo.n_layers} layers + head, context {context}",
            "ms_per_window": sec * 1e3, "windows": len(times),
            "roofline": {"bound": "hbm", "algorithmic_bytes": total_b, "weight_bytes": weight_b, "kv_bytes": kv_b,
                         "achieved": total_b / sec / 1e9, "peak": peak, "unit": "GB/s",
                         "frac": total_b / sec / 1e9 / peak, "peak_kind": kind}}


def run_micro(args):
    """One micro-benchmark alone on cuda:0 (a small command for profiler captures); prints its JSON object."""
    import torch

    from clusterlm_b200.runtime import Context

    torch.cuda.set_device(0)
    dev = torch.device("cuda:0")
    ctx = Context(0)
    peak, _ = load_peaks()
    if args.micro == "wide":
        obj = wide_micro(ctx, dev)
    elif args.micro == "prefill":
        import numpy as np

        from clusterlm_b200.engine import LLAMA3_8B, ROLE_WHOLE, Engine

        geo = LLAMA3_8B if args.layers == LLAMA3_8B.n_layers else dataclasses.replace(LLAMA3_8B, n_layers=args.layers)
        eng = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, args.context + 64, PREFILL_CHUNK, 2)
        eng.generate_weights(seed=SEED, stddev=0.02)
        eng.prepare()
        stream = torch.cuda.ExternalStream(eng.stream(), device=dev)
        obj = prefill_micro(eng, geo, dev, stream, args.context, np.random.default_rng(5)) or {}
        eng.close()
    elif args.micro == "tree":
        obj = tree_micro(ctx, dev, peak, args.context)
    elif args.micro == "window":
        obj = window_micro(ctx, dev, args)
    elif args.micro == "c5":
        obj = c5_micro(ctx, dev, peak)
    else:
        obj = acceptance_micro(ctx, dev, peak, False)
    ctx.close()
    print(json.dumps({"micro": args.micro, **obj}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    # smaller cases for profiler captures (the line is then marked PROFILE CASE and is not a bench result)
    ap.add_argument("--context", type=int, default=CONTEXT, help="prefilled context (profiling)")
    ap.add_argument("--layers", type=int, default=32, help="decoder layers of the 8B shape (profiling)")
    ap.add_argument("--inflight", type=int, default=0, help="sequences in flight with N > 1 (default N)")
    ap.add_argument("--plan", default="", help="stage plan BEGIN-END@gK,... with N > 1 (default: byte-balanced)")
    ap.add_argument("--micro", default="", choices=["", "wide", "accept", "prefill", "tree", "c5", "window"],
                    help="run one micro-benchmark alone and print its object (profiling)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    world, rank, local = dist_setup()
    try:
        if args.impl == "reference":
            run_reference(args, world, rank)
        elif args.micro:
            run_micro(args)
        elif world > 1:
            run_pipeline(args, world, rank, local)
        else:
            run_b200(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
