"""Llama-shaped engine on the B200 through the C ABI, against the oracle model (identical generated weights).

Tolerances: logits and hidden states within 2e-2 of the reference scale (max |diff| / max |ref|), the
north-star bound for fp16 operands with f32 accumulation against the f32 oracle.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.dirname(__file__))

SMALL = dict(n_layers=2, hidden=256, n_heads=2, n_kv_heads=1, head_dim=128, ffn=512, vocab=512)


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


def small_geo(quant="q4_k", **kw):
    from clusterlm_b200.engine import LlamaGeometry

    d = dict(SMALL)
    d.update(kw)
    return LlamaGeometry(quant=quant, **d)


def make_engine(ctx, geo, role=3, lb=0, le=None, max_context=256, max_window=8, sessions=2):
    from clusterlm_b200.engine import Engine

    e = Engine(ctx, geo, lb, geo.n_layers if le is None else le, role, max_context, max_window, sessions)
    e.generate_weights(seed=0, stddev=0.02)
    e.prepare()
    return e


@pytest.mark.parametrize("quant", ["q4_k", "q8_0"])
def test_windows_match_oracle(ctx, oracle, quant):
    from llama_oracle import LlamaOracle

    geo = small_geo(quant)
    e = make_engine(ctx, geo)
    m = LlamaOracle(oracle, geo)
    e.open_session(1)
    rng = np.random.default_rng(0)
    toks = rng.integers(0, geo.vocab, 40).astype(np.int32)
    pos = 0
    # prefill 8, then windows of 4 committing 4, 2, 1, 3 positions (the rest are rejected drafts)
    plan = [(8, 8), (4, 4), (4, 2), (4, 1), (3, 3), (5, 2)]
    for q, keep in plan:
        w = toks[pos:pos + q]
        got = e.run_window(1, pos, tokens=w)
        want = m.window(w, pos)
        assert rel(got, want) < 2e-2, (q, keep, rel(got, want))
        e.commit(1, keep)
        pos += keep
    assert e.position(1) == pos
    e.close()


def test_split_stages_equal_whole_model_bitwise(ctx):
    """tests/domain/test_split_equivalence.cpp:52 pattern: any layer split gives identical logits."""
    from clusterlm_b200.engine import ROLE_MIDDLE, ROLE_PREFIX, ROLE_TAIL

    geo = small_geo(n_layers=3)
    whole = make_engine(ctx, geo)
    stages = [make_engine(ctx, geo, ROLE_PREFIX, 0, 1), make_engine(ctx, geo, ROLE_MIDDLE, 1, 2),
              make_engine(ctx, geo, ROLE_TAIL, 2, 3)]
    whole.open_session(7)
    for s in stages:
        s.open_session(7)
    rng = np.random.default_rng(1)
    pos = 0
    for q, keep in [(8, 8), (4, 3), (4, 4), (2, 1)]:
        toks = rng.integers(0, geo.vocab, q).astype(np.int32)
        want = whole.run_window(7, pos, tokens=toks)
        rec = stages[0].run_window(7, pos, tokens=toks)
        rec = stages[1].run_window(7, pos, records=rec)
        got = stages[2].run_window(7, pos, records=rec)
        assert np.array_equal(got, want)
        whole.commit(7, keep)
        for s in stages:
            s.commit(7, keep)
        pos += keep
    for s in stages + [whole]:
        s.close()


def test_abort_keeps_committed_state(ctx):
    geo = small_geo()
    e = make_engine(ctx, geo)
    e.open_session(1)
    rng = np.random.default_rng(2)
    prompt = rng.integers(0, geo.vocab, 8)
    e.run_window(1, 0, tokens=prompt)
    e.commit(1, 8)
    w = rng.integers(0, geo.vocab, 4)
    first = e.run_window(1, 8, tokens=w)
    e.abort(1)
    e.run_window(1, 8, tokens=rng.integers(0, geo.vocab, 4))  # a different window in between
    e.abort(1)
    again = e.run_window(1, 8, tokens=w)
    assert np.array_equal(first, again)
    e.close()


def test_engine_refusals(ctx):
    from clusterlm_b200 import ClmError

    geo = small_geo()
    e = make_engine(ctx, geo, max_context=32, max_window=8, sessions=1)
    with pytest.raises(ClmError) as ex:
        e.run_window(1, 0, tokens=[1, 2])
    assert ex.value.name == "kNotFound"
    e.open_session(1)
    with pytest.raises(ClmError) as ex:
        e.open_session(2)
    assert ex.value.name == "kResourceExhausted"
    with pytest.raises(ClmError) as ex:
        e.run_window(1, 3, tokens=[1, 2])
    assert ex.value.name == "kFailedPrecondition"
    with pytest.raises(ClmError) as ex:
        e.run_window(1, 0, tokens=[1] * 9)
    assert ex.value.name == "kResourceExhausted"
    with pytest.raises(ClmError) as ex:
        e.run_window(1, 0, tokens=[geo.vocab])
    assert ex.value.name == "kInvalidArgument"
    e.run_window(1, 0, tokens=[1, 2, 3])
    with pytest.raises(ClmError) as ex:
        e.run_window(1, 0, tokens=[1])
    assert ex.value.name == "kFailedPrecondition"
    with pytest.raises(ClmError) as ex:
        e.commit(1, 4)
    assert ex.value.name == "kInvalidArgument"
    e.commit(1, 3)
    for _ in range(3):
        e.run_window(1, e.position(1), tokens=[1] * 8)
        e.commit(1, 8)
    with pytest.raises(ClmError) as ex:
        e.run_window(1, 27, tokens=[1] * 8)
    assert ex.value.name == "kResourceExhausted"
    e.close()


def test_mtp_draft_matches_oracle(ctx, oracle):
    from llama_oracle import LlamaOracle

    geo = small_geo()
    e = make_engine(ctx, geo)
    m = LlamaOracle(oracle, geo, layers=[])
    toks, logits = e.mtp_draft(17, 3, want_logits=True)
    prev = 17
    for j in range(3):
        want = m.mtp_logits(prev)
        assert rel(logits[j], want) < 2e-2
        assert toks[j] == int(np.argmax(logits[j]))
        prev = int(toks[j])
    e.close()


def test_greedy_speculative_equals_plain_greedy(ctx):
    """Speculative decoding with greedy acceptance emits exactly the greedy sequence (q = 1..4)."""
    geo = small_geo()
    rng = np.random.default_rng(3)
    prompt = rng.integers(0, geo.vocab, 12)
    seqs = {}
    for q in (1, 2, 4):
        e = make_engine(ctx, geo, max_context=256, max_window=8)
        e.open_session(1)
        e.spec_begin(1, prompt, q)
        out = []
        while len(out) < 40:
            out += list(e.spec_round(1, q))
        seqs[q] = out[:40]
        assert e.position(1) == 12 + len(out)
        e.close()
    assert seqs[1] == seqs[2] == seqs[4]


def test_stochastic_rounds_are_reproducible_and_advance(ctx):
    geo = small_geo()
    rng = np.random.default_rng(4)
    prompt = rng.integers(0, geo.vocab, 10)
    runs = []
    for _ in range(2):
        e = make_engine(ctx, geo)
        e.open_session(1)
        e.spec_begin(1, prompt, 4, temperature=1.0, seed=11)
        out, counts = [], []
        for _ in range(12):
            r = e.spec_round(1, 4, temperature=1.0, seed=11)
            assert 1 <= r.size <= 4
            counts.append(r.size)
            out += list(r)
        assert e.position(1) == 10 + sum(counts)
        runs.append(out)
        e.close()
    assert runs[0] == runs[1]


@pytest.mark.slow
def test_llama8b_first_layer_matches_oracle(ctx, oracle):
    """Full-size 8B-shape Q4_K: a prefix stage holding layer 0, one q = 4 window, against the oracle."""
    from clusterlm_b200.engine import LLAMA3_8B, ROLE_PREFIX, Engine
    from llama_oracle import LlamaOracle

    geo = LLAMA3_8B
    e = Engine(ctx, geo, 0, 1, ROLE_PREFIX, 64, 4, 1)
    e.generate_weights(seed=0, stddev=0.02)
    e.prepare()
    e.open_session(1)
    toks = np.array([1, 500, 128000, 77], np.int32)
    rec = e.run_window(1, 0, tokens=toks)
    m = LlamaOracle(oracle, geo, layers=[0], max_ctx=64, threads=os.cpu_count() or 8)
    h = m.run_layers(m.embed(toks), 0)
    H = geo.hidden
    assert rel(rec[:, :H], h) < 2e-2
    assert np.all(rec[:, H:2 * H] == 0) and np.all(rec[:, 2 * H] == 1)
    e.close()


@pytest.mark.parametrize("heads", [(8, 4), (16, 4)])
def test_flow_window_matches_chain_and_oracle(ctx, oracle, monkeypatch, heads):
    """The dataflow window kernel (one cooperative launch per window, the default for windows of <= 16 rows) computes
    the same windows as the per-kernel chain (CLM_B200_FLOW=0): multi-page contexts split over several CTAs per kv
    head, so every combine path runs, at q = 1..16 (one and two column tiles); GQA groups of 2 (two kv heads share
    a W_o input chunk) and 4 (one chunk per kv head)."""
    from llama_oracle import LlamaOracle

    geo = small_geo(n_layers=2, hidden=1024, n_heads=heads[0], n_kv_heads=heads[1], ffn=2048, vocab=1024)
    monkeypatch.setenv("CLM_B200_FLOW", "1")
    fl = make_engine(ctx, geo, max_context=512, max_window=16)
    monkeypatch.setenv("CLM_B200_FLOW", "0")
    ch = make_engine(ctx, geo, max_context=512, max_window=16)
    m = LlamaOracle(oracle, geo, max_ctx=512)
    rng = np.random.default_rng(5)
    toks = rng.integers(0, geo.vocab, 400).astype(np.int32)
    for e in (fl, ch):
        e.open_session(1)
    pos = 0
    plan = [(16, 16)] * 20 + [(4, 2), (4, 4), (3, 1), (12, 5), (1, 1), (8, 3)]
    for q, keep in plan:
        w = toks[pos:pos + q]
        a = fl.run_window(1, pos, tokens=w)
        n_fl = fl.last_launches()
        b = ch.run_window(1, pos, tokens=w)
        n_ch = ch.last_launches()
        assert n_fl < n_ch, (n_fl, n_ch)  # the dataflow kernel really ran
        # the two attention schedules round the fp16 probabilities against different running maxima
        assert rel(a, b) < 5e-3, (q, pos, rel(a, b))
        assert rel(a, m.window(w, pos)) < 2e-2
        fl.commit(1, keep)
        ch.commit(1, keep)
        pos += keep
    # repeated windows (CUDA graph replays) give identical logits
    w = toks[pos:pos + 4]
    first = fl.run_window(1, pos, tokens=w)
    fl.abort(1)
    for _ in range(3):
        again = fl.run_window(1, pos, tokens=w)
        fl.abort(1)
        assert np.array_equal(first, again)
    fl.close()
    ch.close()


def _tree16():
    # root 0; children 1..4 of 0; two children each of 1..4 (5..12); one child each of 5, 6, 7 (13, 14, 15)
    parents = [-1, 0, 0, 0, 0, 1, 1, 2, 2, 3, 3, 4, 4, 5, 6, 7]
    return np.array(parents, np.int32)


@pytest.mark.parametrize("quant", ["q4_k", "q8_0"])
def test_tree_window_matches_oracle_and_path_commit(ctx, oracle, quant):
    """A 16-node draft tree (4, 2, 1 branching): every node attends to the committed context and its ancestors and
    is rotated at base + depth; committing a root-to-leaf path compacts its KV rows, so the next linear window sees
    exactly the context a linear run of that path would have produced."""
    from llama_oracle import LlamaOracle

    geo = small_geo(quant)
    e = make_engine(ctx, geo, max_context=256, max_window=16)
    m = LlamaOracle(oracle, geo)
    e.open_session(1)
    rng = np.random.default_rng(3)
    pos = 0
    pre = rng.integers(0, geo.vocab, 12).astype(np.int32)
    assert rel(e.run_window(1, pos, tokens=pre), m.window(pre, pos)) < 2e-2
    e.commit(1, 12)
    pos = 12
    parents = _tree16()
    toks = rng.integers(0, geo.vocab, 16).astype(np.int32)
    got = e.run_tree_window(1, pos, parents, tokens=toks)
    want = m.logits(m.run_layers(m.embed(toks), pos, parent=parents))
    assert rel(got, want) < 2e-2, rel(got, want)
    path = [0, 2, 7, 15]
    e.commit_path(1, path)
    for L in m.layers:  # the oracle keeps the same rows
        m.kc[L][pos:pos + 4] = m.kc[L][[pos + i for i in path]]
        m.vc[L][pos:pos + 4] = m.vc[L][[pos + i for i in path]]
    pos += 4
    assert e.position(1) == pos
    nxt = rng.integers(0, geo.vocab, 4).astype(np.int32)
    assert rel(e.run_window(1, pos, tokens=nxt), m.window(nxt, pos)) < 2e-2


def test_tree_window_refusals(ctx):
    from clusterlm_b200 import ClmError

    geo = small_geo()
    e = make_engine(ctx, geo, max_context=64, max_window=16)
    e.open_session(1)
    toks = np.zeros(4, np.int32)
    with pytest.raises(ClmError):
        e.run_tree_window(1, 0, [-1, 0, 3, 1], tokens=toks)  # parent after the node
    e.run_tree_window(1, 0, [-1, 0, 0, 1], tokens=toks)
    with pytest.raises(ClmError):
        e.commit(1, 2)  # a tree is committed by path
    with pytest.raises(ClmError):
        e.commit_path(1, [0, 2, 3])  # 3's parent is 1, not 2
    e.commit_path(1, [0, 1, 3])
    assert e.position(1) == 3


def test_tree_window_device_equals_host_and_guards_parents(ctx):
    """The device-buffer tree window gives the host variant's logits bit for bit; a parent that is not -1 or an
    earlier node is replaced on the device and the commit reports CLM_INVALID_ARGUMENT."""
    import torch

    from clusterlm_b200 import ClmError

    geo = small_geo("q8_0")
    e = make_engine(ctx, geo, max_context=256, max_window=16)
    e.open_session(1)
    rng = np.random.default_rng(9)
    pre = rng.integers(0, geo.vocab, 16).astype(np.int32)
    e.run_window(1, 0, tokens=pre)
    e.commit(1, 16)
    parents = np.array(_tree16(), np.int32)
    toks = rng.integers(0, geo.vocab, 16).astype(np.int32)
    want = e.run_tree_window(1, 16, parents, tokens=toks)
    e.abort(1)
    dev = torch.device("cuda:0")
    out = torch.empty((16, geo.vocab), dtype=torch.float32, device=dev)
    e.run_tree_window_device(1, 16, torch.from_numpy(parents).to(dev), torch.from_numpy(toks).to(dev), out)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), want)
    e.commit_path(1, [0, 1])
    bad = parents.copy()
    bad[5] = 9  # a later node
    e.run_tree_window_device(1, 18, torch.from_numpy(bad).to(dev), torch.from_numpy(toks).to(dev), out)
    with pytest.raises(ClmError, match="earlier node"):
        e.commit_path(1, [0])
    assert e.position(1) == 18
    e.close()


@pytest.mark.parametrize("role", [1, 3])  # middle stage (records in and out), whole model (tokens in, logits out)
def test_batched_gemv_window_equals_separate_windows(ctx, role):
    """clm_b200_run_batch_window_device: four sessions' 8-row windows in one 32-row window on the q-row GEMV chain
    (every matrix streamed once) give each session the outputs of its own window, at different committed positions,
    and the KV rows each session commits are the ones its later windows read."""
    import torch

    from clusterlm_b200.engine import ROLE_MIDDLE, ROLE_WHOLE

    geo = small_geo(n_layers=2, hidden=512, n_heads=8, n_kv_heads=2, ffn=1024)
    role = ROLE_MIDDLE if role == 1 else ROLE_WHOLE
    e = make_engine(ctx, geo, role, 0, 2, max_context=256, max_window=32, sessions=4)
    dev = torch.device("cuda:0")
    fpp = 2 * geo.hidden + 1
    gen = torch.Generator(device=dev).manual_seed(9)
    rng = np.random.default_rng(9)
    n, q = 4, 8
    ids = [11, 12, 13, 14]

    def inputs(rows):
        if role == ROLE_WHOLE:
            return dict(d_tokens=torch.from_numpy(rng.integers(0, geo.vocab, rows).astype(np.int32)).to(dev))
        rec = torch.zeros((rows, fpp), dtype=torch.float32, device=dev)
        rec[:, :geo.hidden] = torch.randn((rows, geo.hidden), generator=gen, device=dev)
        rec[:, 2 * geo.hidden] = 1.0
        return dict(d_records=rec)

    width = geo.vocab if role == ROLE_WHOLE else fpp
    pos = {}
    for b, s in enumerate(ids):  # different context lengths
        e.open_session(s)
        L = [9, 16, 23, 5][b]
        out = torch.empty((L, width), device=dev)
        e.run_window_device(s, 0, d_out=out, **inputs(L))
        e.commit(s, L)
        pos[s] = L
    for rnd in range(2):
        inp = inputs(n * q)
        key = "d_tokens" if role == ROLE_WHOLE else "d_records"
        want = []
        for b, s in enumerate(ids):
            o = torch.empty((q, width), device=dev)
            e.run_window_device(s, pos[s], d_out=o, **{key: inp[key][b * q:(b + 1) * q].contiguous()})
            torch.cuda.synchronize()
            e.abort(s)
            want.append(o)
        got = torch.empty((n * q, width), device=dev)
        e.run_batch_window_device(ids, [pos[s] for s in ids], q, d_out=got, **inp)
        torch.cuda.synchronize()
        for b in range(n):
            # the 32-row GEMV adds each row's products in another order than the 8-row one (single-superblock units,
            # other split-K segments), and the fp16 rounding of every layer's inputs turns such last-bit differences
            # into ~1e-3 of the scale by the logits: a quarter of the oracle bound of these tests (2e-2)
            w, g = want[b].cpu().numpy(), got[b * q:(b + 1) * q].cpu().numpy()
            assert rel(g, w) < 5e-3, (rnd, b, rel(g, w))
        for b, s in enumerate(ids):
            keep = [8, 3, 5, 1][(b + rnd) % 4]
            e.commit(s, keep)
            pos[s] += keep
    e.close()
