"""Wide verify windows (17..256 rows: prefill chunks and large draft trees) through the C ABI: tensor-core GEMMs
with the RoPE/KV, residual-norm and SwiGLU steps between them, against the oracle model (identical generated
weights) and against the <= 16-row GEMV chain on the same cache.

Tolerances: logits within 2e-2 of the reference scale (max |diff| / max |ref|), the north-star bound for fp16
operands with f32 accumulation against the f32 oracle.
"""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

sys.path.insert(0, os.path.dirname(__file__))

from test_llama_gpu import make_engine, rel, small_geo  # noqa: E402


@pytest.mark.parametrize("quant", ["q4_k", "q8_0"])
def test_wide_windows_match_oracle(ctx, oracle, quant):
    """A 200-row prefill chunk, then linear windows alternating between the tensor-core path (> 16 rows) and the
    GEMV chain (<= 16 rows) on one KV cache, each compared with the oracle and partly committed."""
    from llama_oracle import LlamaOracle

    geo = small_geo(quant)
    e = make_engine(ctx, geo, max_context=1024, max_window=256, sessions=1)
    m = LlamaOracle(oracle, geo, max_ctx=1024)
    e.open_session(1)
    rng = np.random.default_rng(11)
    toks = rng.integers(0, geo.vocab, 900).astype(np.int32)
    pos = 0
    plan = [(200, 200), (4, 3), (64, 40), (17, 17), (16, 9), (256, 100), (33, 1), (8, 8)]
    for q, keep in plan:
        w = toks[pos:pos + q]
        got = e.run_window(1, pos, tokens=w)
        assert got.shape == (q, geo.vocab)
        want = m.window(w, pos)
        assert rel(got, want) < 2e-2, (q, pos, rel(got, want))
        e.commit(1, keep)
        pos += keep
    assert e.position(1) == pos
    e.close()


def test_wide_window_more_head_tiles_than_sms(ctx, oracle):
    """256 rows x 16 query heads over 4 kv heads: 4 x 64 (kv head, 16-row tile) pairs, more than the SMs, so the
    attention runs one split per pair; the context spans several pages."""
    from llama_oracle import LlamaOracle

    geo = small_geo("q4_k", n_layers=1, hidden=1024, n_heads=16, n_kv_heads=4, ffn=1024, vocab=1024)
    e = make_engine(ctx, geo, max_context=1024, max_window=256, sessions=1)
    m = LlamaOracle(oracle, geo, max_ctx=1024)
    e.open_session(1)
    rng = np.random.default_rng(12)
    toks = rng.integers(0, geo.vocab, 600).astype(np.int32)
    pos = 0
    for q, keep in [(256, 256), (256, 200), (5, 5)]:
        w = toks[pos:pos + q]
        got = e.run_window(1, pos, tokens=w)
        assert rel(got, m.window(w, pos)) < 2e-2, (q, pos)
        e.commit(1, keep)
        pos += keep
    e.close()


def test_wide_prefill_equals_narrow_prefill(ctx, oracle):
    """The same 240-token prompt prefilled as one wide window and as fifteen 16-row windows: the next decode
    windows agree with each other and with the oracle."""
    from llama_oracle import LlamaOracle

    geo = small_geo("q4_k")
    wide = make_engine(ctx, geo, max_context=512, max_window=256, sessions=1)
    narrow = make_engine(ctx, geo, max_context=512, max_window=16, sessions=1)
    m = LlamaOracle(oracle, geo, max_ctx=512)
    rng = np.random.default_rng(13)
    prompt = rng.integers(0, geo.vocab, 240).astype(np.int32)
    wide.open_session(1)
    narrow.open_session(1)
    a_pre = wide.run_window(1, 0, tokens=prompt)
    wide.commit(1, 240)
    b_rows = []
    for off in range(0, 240, 16):
        b_rows.append(narrow.run_window(1, off, tokens=prompt[off:off + 16]))
        narrow.commit(1, 16)
    b_pre = np.concatenate(b_rows)
    want = m.window(prompt, 0)
    assert rel(a_pre, want) < 2e-2 and rel(b_pre, want) < 2e-2
    nxt = rng.integers(0, geo.vocab, 4).astype(np.int32)
    a = wide.run_window(1, 240, tokens=nxt)
    b = narrow.run_window(1, 240, tokens=nxt)
    want = m.window(nxt, 240)
    assert rel(a, want) < 2e-2 and rel(b, want) < 2e-2
    assert rel(a, b) < 2e-2
    wide.close()
    narrow.close()


def _tree(n, seed):
    rng = np.random.default_rng(seed)
    parents = [-1] + [int(rng.integers(max(0, i - 8), i)) for i in range(1, n)]
    return np.array(parents, np.int32)


def test_wide_tree_window_matches_oracle_and_path_commit(ctx, oracle):
    """A 96-node draft tree on the tensor-core path: each node attends to the committed context and its ancestors,
    rotated at base + depth; committing a root-to-leaf path compacts its KV rows for the next window."""
    from llama_oracle import LlamaOracle

    geo = small_geo("q8_0")
    e = make_engine(ctx, geo, max_context=512, max_window=128, sessions=1)
    m = LlamaOracle(oracle, geo, max_ctx=512)
    e.open_session(1)
    rng = np.random.default_rng(14)
    pre = rng.integers(0, geo.vocab, 70).astype(np.int32)
    assert rel(e.run_window(1, 0, tokens=pre), m.window(pre, 0)) < 2e-2
    e.commit(1, 70)
    pos = 70
    parents = _tree(96, 15)
    toks = rng.integers(0, geo.vocab, 96).astype(np.int32)
    got = e.run_tree_window(1, pos, parents, tokens=toks)
    want = m.logits(m.run_layers(m.embed(toks), pos, parent=parents))
    assert rel(got, want) < 2e-2, rel(got, want)
    leaf = 95
    path = []
    while leaf >= 0:
        path.append(leaf)
        leaf = int(parents[leaf])
    path = path[::-1]
    e.commit_path(1, path)
    for L in m.layers:
        m.kc[L][pos:pos + len(path)] = m.kc[L][[pos + i for i in path]]
        m.vc[L][pos:pos + len(path)] = m.vc[L][[pos + i for i in path]]
    pos += len(path)
    assert e.position(1) == pos
    nxt = rng.integers(0, geo.vocab, 20).astype(np.int32)
    assert rel(e.run_window(1, pos, tokens=nxt), m.window(nxt, pos)) < 2e-2
    e.close()


def test_batch_tree_window_matches_per_session_trees(ctx, oracle):
    """Four sessions at different committed positions verify a 16-node tree each in ONE window (64 rows on the
    tensor-core path, every weight matrix read once): each session's logits match its own oracle and its own
    single-session tree window (the GEMV chain); each then commits a different root-to-leaf path, continues
    linearly, and a linear batch runs at the new positions."""
    from llama_oracle import LlamaOracle
    from test_llama_gpu import _tree16

    geo = small_geo("q8_0")
    e = make_engine(ctx, geo, max_context=256, max_window=64, sessions=4)
    ref = make_engine(ctx, geo, max_context=256, max_window=16, sessions=4)
    oracles = [LlamaOracle(oracle, geo) for _ in range(4)]
    rng = np.random.default_rng(21)
    pos = []
    for b in range(4):
        n = 3 + 4 * b  # at most 16: the reference engine's windows
        pre = rng.integers(0, geo.vocab, n).astype(np.int32)
        for eng in (e, ref):
            eng.open_session(b + 1)
            eng.run_window(b + 1, 0, tokens=pre)
            eng.commit(b + 1, n)
        oracles[b].window(pre, 0)
        pos.append(n)
    parents = _tree16()
    toks = rng.integers(0, geo.vocab, (4, 16)).astype(np.int32)
    got = e.run_batch_window([1, 2, 3, 4], pos, toks, parents)
    for b in range(4):
        m = oracles[b]
        want = m.logits(m.run_layers(m.embed(toks[b]), pos[b], parent=parents))
        assert rel(got[b], want) < 2e-2, (b, rel(got[b], want))
        alone = ref.run_tree_window(b + 1, pos[b], parents, tokens=toks[b])
        assert rel(got[b], alone) < 2e-2, (b, rel(got[b], alone))
        ref.abort(b + 1)
    paths = [[0, 1, 5, 13], [0, 2, 7, 15], [0, 3, 9], [0, 4]]
    for b in range(4):
        e.commit_path(b + 1, paths[b])
        m = oracles[b]
        for L in m.layers:
            m.kc[L][pos[b]:pos[b] + len(paths[b])] = m.kc[L][[pos[b] + i for i in paths[b]]]
            m.vc[L][pos[b]:pos[b] + len(paths[b])] = m.vc[L][[pos[b] + i for i in paths[b]]]
        pos[b] += len(paths[b])
        assert e.position(b + 1) == pos[b]
        nxt = rng.integers(0, geo.vocab, 3).astype(np.int32)
        assert rel(e.run_window(b + 1, pos[b], tokens=nxt), m.window(nxt, pos[b])) < 2e-2
        e.commit(b + 1, 3)
        pos[b] += 3
    lin = rng.integers(0, geo.vocab, (4, 8)).astype(np.int32)
    got = e.run_batch_window([1, 2, 3, 4], pos, lin)
    for b in range(4):
        assert rel(got[b], oracles[b].window(lin[b], pos[b])) < 2e-2
        e.commit(b + 1, 8)
        assert e.position(b + 1) == pos[b] + 8
    e.close()
    ref.close()


def test_batch_window_refusals(ctx):
    from clusterlm_b200 import ClmError

    geo = small_geo("q4_k")
    e = make_engine(ctx, geo, max_context=64, max_window=32, sessions=3)
    for s in (1, 2, 3):
        e.open_session(s)
    toks = np.ones((3, 16), np.int32)
    with pytest.raises(ClmError) as ex:  # 48 rows > max_window
        e.run_batch_window([1, 2, 3], [0, 0, 0], toks)
    assert ex.value.name == "kResourceExhausted"
    with pytest.raises(ClmError) as ex:
        e.run_batch_window([1, 1], [0, 0], toks[:2])
    assert ex.value.name == "kInvalidArgument"
    with pytest.raises(ClmError) as ex:  # 16 rows in all: one window per session instead
        e.run_batch_window([1, 2], [0, 0], toks[:2, :8])
    assert ex.value.name == "kOutOfRange"
    with pytest.raises(ClmError) as ex:  # base != committed position
        e.run_batch_window([1, 2], [0, 3], toks[:2])
    assert ex.value.name == "kFailedPrecondition"
    got = e.run_batch_window([1, 2], [0, 0], toks[:2])
    assert np.allclose(got[0], got[1], rtol=1e-6, atol=1e-6)  # same tokens, same empty context
    with pytest.raises(ClmError) as ex:  # windows outstanding
        e.run_batch_window([1, 2], [0, 0], toks[:2])
    assert ex.value.name == "kFailedPrecondition"
    e.abort(1)
    e.abort(2)
    e.close()
