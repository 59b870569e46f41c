"""The clusterlm-fixture family on the B200 against the REFERENCE (golden vectors and the compiled reference).

The model files are written by the reference's own fixture generator (via oracle/_ref) into a temporary
directory; objects are read through the reference's CanonicalModelStore and bound to the device engines.
The golden windows were produced by the reference's ReferenceDomain pipeline (tests/golden/make_golden.py).
"""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
BOUNDS = [0, 4, 10, 13, 16]


@pytest.fixture(scope="module")
def store(reference):
    from oracle.oracle_py import ModelStore

    d = tempfile.mkdtemp(prefix="clm_fixture_")
    reference.write_fixture(d, seed=0x434C4D31)
    s = ModelStore(reference, d)
    s.dir = d
    yield s
    s.close()


def geometry(store):
    from clusterlm_b200.engine import FixtureGeometry

    g = dict(store.geometry)
    g.pop("mtp_layers")
    return FixtureGeometry(layer_kinds=tuple(int(k) for k in store.layer_kinds), **g)


def object_names(geo, lb, le, role):
    from clusterlm_b200.engine import ROLE_PREFIX, ROLE_TAIL, ROLE_WHOLE

    names = []
    if role in (ROLE_PREFIX, ROLE_WHOLE):
        names += ["token_embd", "ple_lookup"]
    for L in range(lb, le):
        names += [f"blk.{L}.dense", f"blk.{L}.shared"] + [f"blk.{L}.exp.{e}" for e in range(geo.n_experts)]
    if role in (ROLE_TAIL, ROLE_WHOLE):
        names += ["output_head", "mtp_drafter", "token_embd"]
    return names


def make_stage(ctx, store, lb, le, role, max_context=256, max_window=8, sessions=2):
    from clusterlm_b200.engine import FixtureEngine

    geo = geometry(store)
    e = FixtureEngine(ctx, geo, lb, le, role, max_context, max_window, sessions)
    for n in dict.fromkeys(object_names(geo, lb, le, role)):
        q, b = store.object(n)
        e.set_object(n, q, b)
    e.prepare()
    return e


def make_pipeline(ctx, store, bounds=BOUNDS):
    from clusterlm_b200.engine import ROLE_MIDDLE, ROLE_PREFIX, ROLE_TAIL

    n = len(bounds) - 1
    roles = [ROLE_PREFIX] + [ROLE_MIDDLE] * (n - 2) + [ROLE_TAIL]
    return [make_stage(ctx, store, bounds[i], bounds[i + 1], roles[i]) for i in range(n)]


def run_pipeline(stages, session, base, tokens):
    rec = stages[0].run_window(session, base, tokens=tokens)
    outs = [rec]
    for s in stages[1:-1]:
        rec = s.run_window(session, base, records=rec)
        outs.append(rec)
    return stages[-1].run_window(session, base, records=rec), outs


def rel(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("tag", ["greedy", "spec"])
def test_pipeline_replays_reference_windows(ctx, store, tag):
    """The reference's 4-stage pipeline windows (prefill, then q = 1 or q = 4 scripted:0.3 windows with their
    commits) replayed on four device stages: stage records and logits match the reference."""
    g = np.load(os.path.join(GOLDEN, "fixture.npz"))
    stages = make_pipeline(ctx, store)
    for s in stages:
        s.open_session(1)
    toks, acc, logits, recs = g[f"{tag}_tokens"], g[f"{tag}_accepted"], g[f"{tag}_logits"], g[f"{tag}_stages"]
    base, worst, exact, total = 0, 0.0, 0, 0
    for w in range(toks.shape[0]):
        t = toks[w][toks[w] >= 0]
        q = t.size
        got, outs = run_pipeline(stages, 1, base, t)
        want = logits[w][:q]
        worst = max(worst, rel(got, want))
        exact += int((got == want).sum())
        total += want.size
        for si, r in enumerate(outs):
            assert rel(r, recs[w][si][:q]) < 1e-4, (w, si)
        # the same greedy decisions as the reference
        assert np.array_equal(got.argmax(1), want.argmax(1))
        for s in stages:
            s.commit(1, int(acc[w]))
        base += int(acc[w])
    assert worst < 1e-4, worst
    print(f"fixture {tag}: max rel diff {worst:.2e}, bit-exact logits {exact}/{total}")
    for s in stages:
        s.close()


def test_whole_model_greedy_generation_matches_reference(ctx, store):
    """Father-only greedy generation (q = 1) on one whole-model engine reproduces the reference continuation."""
    from clusterlm_b200.engine import ROLE_WHOLE

    g = np.load(os.path.join(GOLDEN, "fixture.npz"))
    e = make_stage(ctx, store, 0, 16, ROLE_WHOLE)
    e.open_session(3)
    prompt = g["prompt"]
    base = 0
    for off in range(0, prompt.size, 8):
        chunk = prompt[off:off + 8]
        logits = e.run_window(3, base, tokens=chunk)
        e.commit(3, chunk.size)
        base += chunk.size
    nxt = int(logits[-1].argmax())
    out = []
    while len(out) < 32:
        out.append(nxt)
        logits = e.run_window(3, base, tokens=[nxt])
        e.commit(3, 1)
        base += 1
        nxt = int(logits[0].argmax())
    assert out == list(g["greedy_generated"])
    e.close()


def test_mtp_fixture_drafter_matches_reference(ctx, store):
    from clusterlm_b200.engine import ROLE_TAIL

    g = np.load(os.path.join(GOLDEN, "fixture.npz"))
    e = make_stage(ctx, store, 13, 16, ROLE_TAIL)
    for prev in range(0, 256, 5):
        toks, logits = e.mtp_draft(prev, 1, want_logits=True)
        assert toks[0] == g["mtp_step"][prev], prev
        if prev < 8:
            assert rel(logits[0], g["mtp_logits_0_7"][prev]) < 1e-5
    # chained drafting: d_{i+1} = step(d_i)
    toks = e.mtp_draft(17, 4)
    prev = 17
    for t in toks:
        assert t == g["mtp_step"][prev]
        prev = int(t)
    e.close()


def test_committing_fewer_positions_equals_running_only_those(ctx, store):
    """tests/domain/test_domain_lifecycle.cpp:357: a window of q committed with n < q leaves the same state as
    a window of only the first n positions (recurrent snapshot[n-1], PLE history, KV)."""
    from clusterlm_b200.engine import ROLE_WHOLE

    a = make_stage(ctx, store, 0, 16, ROLE_WHOLE)
    b = make_stage(ctx, store, 0, 16, ROLE_WHOLE)
    rng = np.random.default_rng(5)
    prompt = rng.integers(0, 256, 8)
    for e in (a, b):
        e.open_session(1)
        e.run_window(1, 0, tokens=prompt)
        e.commit(1, 8)
    w = rng.integers(0, 256, 6)
    a.run_window(1, 8, tokens=w)
    a.commit(1, 3)
    b.run_window(1, 8, tokens=w[:3])
    b.commit(1, 3)
    nxt = rng.integers(0, 256, 4)
    assert np.array_equal(a.run_window(1, 11, tokens=nxt), b.run_window(1, 11, tokens=nxt))
    a.close()
    b.close()


def test_fixture_role_rules_and_refusals(ctx, store):
    from clusterlm_b200 import ClmError
    from clusterlm_b200.engine import ROLE_MIDDLE, ROLE_PREFIX, ROLE_TAIL, FixtureEngine

    geo = geometry(store)
    with pytest.raises(ClmError) as e:
        FixtureEngine(ctx, geo, 0, 2, ROLE_PREFIX, 64, 4)  # must contain the PLE layer (2)
    assert e.value.name == "kInvalidArgument"
    with pytest.raises(ClmError):
        FixtureEngine(ctx, geo, 2, 6, ROLE_MIDDLE, 64, 4)  # middle may not contain the PLE layer
    with pytest.raises(ClmError):
        FixtureEngine(ctx, geo, 10, 15, ROLE_TAIL, 64, 4)  # tail must end at the last layer
    eng = FixtureEngine(ctx, geo, 4, 10, ROLE_MIDDLE, 64, 4)
    with pytest.raises(ClmError) as e:
        eng.prepare()  # objects missing
    assert e.value.name == "kNotFound"
    q, b = store.object("blk.4.dense")
    with pytest.raises(ClmError) as e:
        eng.set_object("blk.4.dense", q, b[:-4])
    assert e.value.name == "kDataLoss"
    with pytest.raises(ClmError) as e:
        eng.set_object("blk.99.dense", q, b)
    assert e.value.name == "kNotFound"
    eng.close()
