"""GGUF container reader (clusterlm_b200.gguf_file) against files written by gguf-py, the reference implementation
of the format in ggml's tree: metadata, tensor table, aligned data offsets and tensor bytes, the llama geometry
read from the metadata, and refusals of broken files.  No GPU."""
import numpy as np
import pytest

gguf = pytest.importorskip("gguf")

from clusterlm_b200.gguf_file import GGUFFile, llama_geometry  # noqa: E402


def _write(path, alignment=None):
    w = gguf.GGUFWriter(str(path), "llama")
    if alignment:
        w.add_custom_alignment(alignment)
    w.add_block_count(2)
    w.add_embedding_length(256)
    w.add_head_count(2)
    w.add_head_count_kv(1)
    w.add_feed_forward_length(512)
    w.add_rope_freq_base(500000.0)
    w.add_layer_norm_rms_eps(1e-5)
    w.add_array("tokenizer.ggml.tokens", ["a", "bc", "def"])
    rng = np.random.default_rng(0)
    t = {
        "token_embd.weight": (rng.integers(0, 256, (512, 144), dtype=np.uint8), gguf.GGMLQuantizationType.Q4_K),
        "blk.0.attn_q.weight": (rng.integers(0, 256, (256, 144), dtype=np.uint8), gguf.GGMLQuantizationType.Q4_K),
        "blk.0.attn_k.weight": (rng.integers(0, 256, (128, 8 * 34), dtype=np.uint8), gguf.GGMLQuantizationType.Q8_0),
        "blk.0.attn_norm.weight": (rng.standard_normal(256).astype(np.float32), None),
    }
    for name, (a, qt) in t.items():
        if qt is None:
            w.add_tensor(name, a)
        else:
            w.add_tensor(name, a, raw_dtype=qt)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return t


@pytest.mark.parametrize("alignment", [None, 64])
def test_reader_matches_gguf_py(tmp_path, alignment):
    path = tmp_path / "m.gguf"
    t = _write(path, alignment)
    f = GGUFFile(str(path))
    ref = gguf.GGUFReader(str(path))
    assert f.version == 3
    assert f.kv["llama.block_count"] == 2 and f.kv["tokenizer.ggml.tokens"] == ["a", "bc", "def"]
    assert set(f.tensors) == set(t)
    for rt in ref.tensors:
        info = f.tensors[rt.name]
        assert f.data_start + info.offset == rt.data_offset
        assert info.nbytes == rt.n_bytes
        assert list(info.dims) == [int(x) for x in rt.shape]
    for name, (a, _) in t.items():
        assert np.array_equal(np.asarray(f.data(name)), a.reshape(-1).view(np.uint8))
    assert f.tensors["blk.0.attn_q.weight"].dims == (256, 256)
    assert f.tensors["blk.0.attn_k.weight"].dims == (256, 128)
    g = llama_geometry(f)
    assert (g.n_layers, g.hidden, g.n_heads, g.n_kv_heads, g.head_dim, g.ffn, g.vocab) == (2, 256, 2, 1, 128, 512, 512)
    assert g.quant == "q4_k" and not g.mtp and g.rope_theta == 500000.0


def test_reader_refuses_broken_files(tmp_path):
    path = tmp_path / "m.gguf"
    _write(path)
    raw = path.read_bytes()
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"GGUX" + raw[4:])
    with pytest.raises(ValueError, match="not a GGUF"):
        GGUFFile(str(bad))
    bad.write_bytes(raw[:4] + (1).to_bytes(4, "little") + raw[8:])
    with pytest.raises(ValueError, match="version 1"):
        GGUFFile(str(bad))
    bad.write_bytes(raw[:200])
    with pytest.raises(ValueError, match="truncated"):
        GGUFFile(str(bad))
    bad.write_bytes(raw[:-1000])
    with pytest.raises(ValueError, match="past the end"):
        GGUFFile(str(bad)).data("blk.0.attn_norm.weight")


def test_geometry_refuses_rope_frequency_scaling(tmp_path):
    """Llama 3.1+ files carry RoPE frequency factors (rope_freqs.weight) or a rope.scaling.type; the engine's RoPE is
    the unscaled theta^(-2i/hd) rotation, so such files are refused instead of running with other logits."""
    from clusterlm_b200 import ClmError

    path = tmp_path / "freqs.gguf"
    w = gguf.GGUFWriter(str(path), "llama")
    w.add_block_count(1)
    w.add_embedding_length(256)
    w.add_head_count(2)
    w.add_feed_forward_length(512)
    rng = np.random.default_rng(1)
    w.add_tensor("token_embd.weight", rng.integers(0, 256, (512, 144), dtype=np.uint8),
                 raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.add_tensor("blk.0.attn_q.weight", rng.integers(0, 256, (256, 144), dtype=np.uint8),
                 raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.add_tensor("rope_freqs.weight", np.ones(64, np.float32))
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ClmError, match="rope_freqs") as ex:
        llama_geometry(GGUFFile(str(path)))
    assert ex.value.name == "kUnimplemented"

    path2 = tmp_path / "scaled.gguf"
    w = gguf.GGUFWriter(str(path2), "llama")
    w.add_block_count(1)
    w.add_embedding_length(256)
    w.add_head_count(2)
    w.add_feed_forward_length(512)
    w.add_string("llama.rope.scaling.type", "linear")
    w.add_tensor("token_embd.weight", rng.integers(0, 256, (512, 144), dtype=np.uint8),
                 raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.add_tensor("blk.0.attn_q.weight", rng.integers(0, 256, (256, 144), dtype=np.uint8),
                 raw_dtype=gguf.GGMLQuantizationType.Q4_K)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with pytest.raises(ClmError, match="scaling 'linear'"):
        llama_geometry(GGUFFile(str(path2)))
