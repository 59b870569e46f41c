"""The oracle (CPU restatement) pinned against the reference's golden vectors and the compiled reference."""
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    return np.load(os.path.join(GOLDEN, name))


def test_half_conversions_match_reference_golden(oracle):
    g = load("codec.npz")
    got = np.array([oracle.half_to_float(int(h)) for h in g["h2f_in"]], np.float32)
    same = (got.view(np.uint32) == g["h2f_out"].view(np.uint32)) | (np.isnan(got) & np.isnan(g["h2f_out"]))
    assert same.all()
    got = np.array([oracle.float_to_half(float(f)) for f in g["f2h_in"]], np.uint16)
    assert np.array_equal(got, g["f2h_out"])
    # tests/gguf/test_ggml_types.cpp:76 known answers
    assert oracle.float_to_half(1.0) == 0x3C00 and oracle.float_to_half(-2.0) == 0xC000
    assert oracle.float_to_half(65504.0) == 0x7BFF and oracle.float_to_half(1e10) == 0x7C00
    assert oracle.float_to_half(1.0 + 1.0 / 2048.0) == 0x3C00 and oracle.float_to_half(1.0 + 3.0 / 2048.0) == 0x3C02


@pytest.mark.parametrize("quant,key", [("q8_0", "q8_0"), ("q8_0-fixture", "q8f")])
def test_q8_codecs_match_reference_golden(oracle, quant, key):
    g = load("codec.npz")
    enc = oracle.encode(quant, g["q8_in"])
    assert np.array_equal(enc, g[f"{key}_bytes"])
    dec = oracle.decode(quant, g[f"{key}_bytes"], g["q8_in"].size)
    assert np.array_equal(dec.view(np.uint32), g[f"{key}_decoded"].view(np.uint32))


def test_q8_fixture_hand_block(oracle):
    # tests/objects/test_manifest.cpp:220 hand-built block: scale 0.5, q = i - 16
    blk = np.zeros(36, np.uint8)
    blk[:4] = np.frombuffer(np.float32(0.5).tobytes(), np.uint8)
    blk[4:] = (np.arange(32) - 16).astype(np.int8).view(np.uint8)
    out = oracle.decode("q8_0-fixture", blk, 32)
    assert np.array_equal(out, 0.5 * (np.arange(32) - 16).astype(np.float32))
    with pytest.raises(ValueError):
        oracle.decode("q8_0-fixture", blk[:35], 32)


def test_q4k_decode_matches_gguf_py_golden(oracle):
    g = load("codec.npz")
    assert np.array_equal(oracle.encode("q4_k", g["q4k_in"]), g["q4k_bytes"])  # encoder is deterministic
    dec = oracle.decode("q4_k", g["q4k_bytes"], g["q4k_in"].size)
    assert np.array_equal(dec.view(np.uint32), g["q4k_decoded_gguf"].view(np.uint32))
    assert oracle.tensor_bytes("q4_k", 256) == 144 and oracle.tensor_bytes("q4_k", 255) == 0
    err = np.abs(dec - g["q4k_in"]).reshape(-1, 32)
    rng = g["q4k_in"].reshape(-1, 32)
    span = np.maximum(rng.max(1), 0) - np.minimum(rng.min(1), 0)
    assert (err.max(1) <= span / 15 * 0.75 + 1e-6).all()  # half a step plus 6-bit scale error


def test_philox_known_answers(oracle):
    g = load("philox.npz")
    for c, k, o in zip(g["kat_ctr"], g["kat_key"], g["kat_out"]):
        assert np.array_equal(oracle.philox(c, k), o)
    u = np.array([oracle.philox_uniform(int(g["uniform_seed"]), i, 7, 9, 11) for i in range(256)])
    assert np.array_equal(u, g["uniforms"])
    assert np.array_equal(oracle.gen_weights(0, 3, 1000, 4096, 0.02), g["gen_weights"])


def test_sampling_matches_reference_golden(oracle):
    g = load("sampling.npz")
    for r, a in zip(g["logits"], g["argmax"]):
        assert oracle.argmax(r) == a
    for pi, p in enumerate(g["dist_params"]):
        for r, want in zip(g["logits"], g["dist"][pi]):
            got = oracle.distribution(r, float(p[0]), int(p[1]), float(p[2]))
            assert np.array_equal(got, want), p
    for probs, u, want in zip(g["sample_probs"], g["sample_uniforms"], g["sample_out"]):
        assert oracle.sample_from(probs, u) == want
    for b in range(g["verify_drafts"].shape[0]):
        a, n, _ = oracle.verify(g["verify_P"][b], g["verify_drafts"][b], g["verify_Q"][b], g["verify_uniforms"][b])
        assert (a, n) == (g["verify_accepted"][b], g["verify_next"][b])
        a, n, _ = oracle.verify(g["verify_P"][b], g["verify_drafts"][b], None, g["verify_uniforms"][b])
        assert (a, n) == (g["verify_accepted_onehot"][b], g["verify_next_onehot"][b])


def test_scripted_drafter_matches_reference(oracle, reference):
    ref_seq = np.random.default_rng(5).integers(0, 256, 100).astype(np.int32)
    for c in range(0, 60, 3):
        for rate in (0.0, 0.3, 1.0):
            assert np.array_equal(oracle.scripted_draft(ref_seq, 256, 1, rate, c, 3),
                                  reference.scripted_draft(ref_seq, 256, 1, rate, c, 3))


def test_oracle_matches_reference_on_random_inputs(oracle, reference):
    rng = np.random.default_rng(7)
    v = (rng.standard_normal(32 * 50) * 3).astype(np.float32)
    for q in ("q8_0", "q8_0-fixture"):
        assert np.array_equal(oracle.encode(q, v), reference.encode(q, v))
    w = rng.standard_normal((33, 70)).astype(np.float32)
    x = rng.standard_normal((5, 70)).astype(np.float32)
    assert np.array_equal(oracle.matmul_rows(w, x), reference.matmul_rows(w, x))
    V = 3000
    for T, k, p in [(1.0, 0, 1.0), (0.5, 7, 1.0), (2.0, 0, 0.3)]:
        lg = (rng.standard_normal(V) * 4).astype(np.float32)
        assert np.array_equal(oracle.distribution(lg, T, k, p), reference.distribution(lg, T, k, p))


def test_matmul_rows_quant_equals_decode_then_matmul(oracle):
    rng = np.random.default_rng(3)
    rows, cols = 32, 512
    w = (rng.standard_normal(rows * cols) * 0.02).astype(np.float32)
    x = rng.standard_normal((3, cols)).astype(np.float32)
    for q in ("q8_0", "q4_k"):
        enc = oracle.encode(q, w)
        dec = oracle.decode(q, enc, w.size).reshape(rows, cols)
        want = oracle.matmul_rows(dec, x)
        for threads in (1, 4):
            got = oracle.matmul_rows_quant(q, enc, rows, cols, x, threads)
            assert np.array_equal(got, want)


def test_fixture_golden_is_self_consistent():
    g = load("fixture.npz")
    # greedy windows: every generated token is the argmax of the previous position's logits
    toks, acc, logits = g["spec_tokens"], g["spec_accepted"], g["spec_logits"]
    assert acc.min() >= 1
    # speculative generation with the scripted drafter reproduces the greedy continuation exactly
    assert np.array_equal(g["spec_generated"], g["greedy_generated"])
    assert logits.shape[-1] == 256
