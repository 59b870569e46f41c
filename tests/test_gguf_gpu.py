"""A Llama GGUF file bound to the engine (clm_b200_llama_load_tensors through clusterlm_b200.gguf_file): the file
holds the same encoded tensors as the counter-based generator (written by gguf-py in llama.cpp's tensor names), so
an engine loaded from it must compute bit-identical windows, MTP drafts and stage records to an engine with
generated weights."""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

gguf = pytest.importorskip("gguf")

sys.path.insert(0, os.path.dirname(__file__))

from test_llama_gpu import small_geo  # noqa: E402


def _write_model(path, oracle, geo, head_id=1001, tie_head=False, q6k_down0=False):
    """tie_head: no output.weight (the head shares token_embd.weight); head_id: generator tensor of output.weight;
    q6k_down0: blk.0.ffn_down.weight stored as (random) Q6_K blocks."""
    from llama_oracle import LlamaOracle

    m = LlamaOracle(oracle, geo, layers=[])
    qt = {"q4_k": gguf.GGMLQuantizationType.Q4_K, "q8_0": gguf.GGMLQuantizationType.Q8_0}[geo.quant]
    row_bytes = (lambda cols: cols // 256 * 144) if geo.quant == "q4_k" else (lambda cols: cols // 32 * 34)
    H, qd, kvd, F, V = geo.hidden, geo.n_heads * geo.head_dim, geo.n_kv_heads * geo.head_dim, geo.ffn, geo.vocab
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_block_count(geo.n_layers)
    w.add_embedding_length(H)
    w.add_head_count(geo.n_heads)
    w.add_head_count_kv(geo.n_kv_heads)
    w.add_feed_forward_length(F)
    w.add_rope_freq_base(geo.rope_theta)
    w.add_layer_norm_rms_eps(geo.rms_eps)

    def mat(name, tid, rows, cols):
        w.add_tensor(name, np.asarray(m.enc(tid, rows * cols), np.uint8).reshape(rows, row_bytes(cols)), raw_dtype=qt)

    ones = np.ones(H, np.float32)
    mat("token_embd.weight", 1000, V, H)
    for L in range(geo.n_layers):
        b = f"blk.{L}."
        mat(b + "attn_q.weight", 16 * L + 0, qd, H)
        mat(b + "attn_k.weight", 16 * L + 1, kvd, H)
        mat(b + "attn_v.weight", 16 * L + 2, kvd, H)
        mat(b + "attn_output.weight", 16 * L + 3, H, qd)
        mat(b + "ffn_gate.weight", 16 * L + 4, F, H)
        mat(b + "ffn_up.weight", 16 * L + 5, F, H)
        if q6k_down0 and L == 0:
            blocks = np.random.default_rng(3).integers(0, 256, (H, F // 256 * 210), dtype=np.uint8)
            w.add_tensor(b + "ffn_down.weight", blocks, raw_dtype=gguf.GGMLQuantizationType.Q6_K)
        else:
            mat(b + "ffn_down.weight", 16 * L + 6, H, F)
        w.add_tensor(b + "attn_norm.weight", ones)
        w.add_tensor(b + "ffn_norm.weight", ones)
    w.add_tensor("output_norm.weight", ones)
    if not tie_head:
        mat("output.weight", head_id, V, H)
    mat("mtp.ffn_gate.weight", 1002, F, H)
    mat("mtp.ffn_up.weight", 1003, F, H)
    mat("mtp.ffn_down.weight", 1004, H, F)
    w.add_tensor("mtp.ffn_norm.weight", ones)
    w.add_tensor("mtp.output_norm.weight", ones)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


@pytest.mark.parametrize("quant", ["q4_k", "q8_0"])
def test_gguf_engine_equals_generated_engine(ctx, oracle, tmp_path, quant):
    from clusterlm_b200.engine import ROLE_PREFIX, ROLE_WHOLE, Engine
    from clusterlm_b200.gguf_file import GGUFFile, llama_geometry

    geo = small_geo(quant)
    path = tmp_path / "model.gguf"
    _write_model(path, oracle, geo)
    fg = llama_geometry(GGUFFile(str(path)))
    assert (fg.n_layers, fg.hidden, fg.n_heads, fg.n_kv_heads, fg.ffn, fg.vocab, fg.quant, fg.mtp) == (
        geo.n_layers, geo.hidden, geo.n_heads, geo.n_kv_heads, geo.ffn, geo.vocab, geo.quant, True)
    engines = []
    for role, le, source in [(ROLE_WHOLE, geo.n_layers, "gen"), (ROLE_WHOLE, geo.n_layers, "gguf"),
                             (ROLE_PREFIX, 1, "gen"), (ROLE_PREFIX, 1, "gguf")]:
        e = Engine(ctx, geo, 0, le, role, 256, 16, 1)
        if source == "gen":
            e.generate_weights(seed=0, stddev=0.02)
        else:
            e.load_gguf(str(path))
        e.prepare()
        e.open_session(1)
        engines.append(e)
    rng = np.random.default_rng(9)
    toks = rng.integers(0, geo.vocab, 40).astype(np.int32)
    pos = 0
    for q, keep in [(16, 16), (4, 3), (8, 8)]:
        w = toks[pos:pos + q]
        outs = [e.run_window(1, pos, tokens=w) for e in engines]
        assert np.array_equal(outs[0], outs[1])  # logits
        assert np.array_equal(outs[2], outs[3])  # stage records
        for e in engines:
            e.commit(1, keep)
        pos += keep
    ta, la = engines[0].mtp_draft(int(toks[0]), 3, temperature=0.0, want_logits=True)
    tb, lb = engines[1].mtp_draft(int(toks[0]), 3, temperature=0.0, want_logits=True)
    assert np.array_equal(ta, tb) and np.array_equal(la, lb)
    for e in engines:
        e.close()


def test_gguf_refusals(ctx, oracle, tmp_path):
    from clusterlm_b200 import ClmError
    from clusterlm_b200.engine import ROLE_WHOLE, Engine

    geo = small_geo("q4_k")
    path = tmp_path / "model.gguf"
    _write_model(path, oracle, geo)
    other = small_geo("q8_0")  # the file's matrices are Q4_K
    e = Engine(ctx, other, 0, other.n_layers, ROLE_WHOLE, 64, 4, 1)
    with pytest.raises(ClmError) as ex:
        e.load_gguf(str(path))
    assert ex.value.name == "kUnimplemented"
    e.close()
    wider = small_geo("q4_k", n_layers=3)  # a layer the file does not hold
    e = Engine(ctx, wider, 0, wider.n_layers, ROLE_WHOLE, 64, 4, 1)
    with pytest.raises(ClmError) as ex:
        e.load_gguf(str(path))
    assert ex.value.name == "kNotFound" and "blk.2." in str(ex.value)
    e.close()


def test_gguf_tied_head_and_unsupported_type(ctx, oracle, tmp_path):
    """A file without output.weight uses token_embd.weight as its head (llama.cpp's tied embedding): it computes the
    same logits as a file whose output.weight holds the embedding's bytes.  A stage matrix in a ggml type the engine
    does not bind (Q6_K here) is refused by name with CLM_UNIMPLEMENTED."""
    from clusterlm_b200 import ClmError
    from clusterlm_b200.engine import ROLE_WHOLE, Engine

    geo = small_geo("q4_k")
    tied, explicit, q6k = tmp_path / "tied.gguf", tmp_path / "explicit.gguf", tmp_path / "q6k.gguf"
    _write_model(tied, oracle, geo, tie_head=True)
    _write_model(explicit, oracle, geo, head_id=1000)
    _write_model(q6k, oracle, geo, q6k_down0=True)
    outs = []
    for path in (tied, explicit):
        e = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, 64, 8, 1)
        e.load_gguf(str(path))
        e.prepare()
        e.open_session(1)
        outs.append(e.run_window(1, 0, tokens=np.arange(5, dtype=np.int32)))
        e.close()
    assert np.array_equal(outs[0], outs[1])
    e = Engine(ctx, geo, 0, geo.n_layers, ROLE_WHOLE, 64, 8, 1)
    with pytest.raises(ClmError, match="blk.0.ffn_down.weight is in ggml type 14") as ex:
        e.load_gguf(str(q6k))
    assert ex.value.name == "kUnimplemented"
    e.close()
