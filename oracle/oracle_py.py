"""ctypes bindings to the CPU checkers (TEST INFRASTRUCTURE ONLY).

`Oracle` wraps liboracle.so (this project's C restatement, oracle.c); `Reference` wraps
_ref/libclm_ref.so (the reference's own code compiled in place, via ref_shim.cpp).  Both take and return
numpy arrays.  The product package never imports this module.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libclm_ref.so")

F32 = np.float32
_fp = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
_dp = np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS")
_i32p = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
_u32p = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
_u64p = np.ctypeslib.ndpointer(dtype=np.uint64, flags="C_CONTIGUOUS")
_u8p = np.ctypeslib.ndpointer(dtype=np.uint8, flags="C_CONTIGUOUS")

QUANTS = {"f32": 0, "q8_0-fixture": 1, "q8_0": 2, "q4_k": 3}


def build(reference_root: str | None = None) -> None:
    """Compile liboracle.so, and (when the reference sources are present) _ref/libclm_ref.so and the
    drop-in parity driver _ref/backend_parity (needs libclm_b200.so built first)."""
    targets = ["oracle"]
    root = reference_root or os.environ.get("CLM_REFERENCE_ROOT", "")
    if root and os.path.isdir(os.path.join(root, "runtime", "domain")):
        targets += ["ref", "parity"]
    subprocess.run(["make", "-s", "-C", HERE, f"REFERENCE_ROOT={root}", "-j8", *targets], check=True)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class Oracle:
    def __init__(self, path: str = ORACLE_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: run oracle.oracle_py.build()")
        L = self.L = C.CDLL(path)
        L.orc_half_to_float.restype = C.c_float
        L.orc_half_to_float.argtypes = [C.c_uint16]
        L.orc_float_to_half.restype = C.c_uint16
        L.orc_float_to_half.argtypes = [C.c_float]
        L.orc_tensor_bytes.restype = C.c_uint64
        L.orc_tensor_bytes.argtypes = [C.c_int, C.c_uint64]
        L.orc_decode_tensor.restype = C.c_int
        L.orc_decode_tensor.argtypes = [C.c_int, _u8p, C.c_uint64, _fp, C.c_uint64]
        for fn in ("orc_encode_q8_fixture", "orc_encode_q8_0", "orc_encode_q4_k"):
            getattr(L, fn).restype = C.c_int
            getattr(L, fn).argtypes = [_fp, C.c_uint64, _u8p]
        L.orc_matmul_rows.argtypes = [_fp, C.c_uint64, C.c_uint64, _fp, C.c_uint64, _fp]
        L.orc_matmul_rows_quant.restype = C.c_int
        L.orc_matmul_rows_quant.argtypes = [C.c_int, _u8p, C.c_uint64, C.c_uint64, _fp, C.c_uint64, _fp, C.c_int]
        L.orc_philox4x32_10.argtypes = [_u32p, _u32p, _u32p]
        L.orc_philox_uniform.restype = C.c_double
        L.orc_philox_uniform.argtypes = [C.c_uint64, C.c_uint32, C.c_uint32, C.c_uint32, C.c_uint32]
        L.orc_mix_seed.restype = C.c_uint64
        L.orc_mix_seed.argtypes = [C.c_uint64, C.c_uint64]
        L.orc_argmax.restype = C.c_int32
        L.orc_argmax.argtypes = [_fp, C.c_uint64]
        L.orc_distribution.argtypes = [_fp, C.c_uint64, C.c_float, C.c_uint32, C.c_float, _fp]
        L.orc_sample_from.restype = C.c_int32
        L.orc_sample_from.argtypes = [_fp, C.c_uint64, C.c_double]
        L.orc_verify_speculative.argtypes = [_fp, _i32p, C.c_void_p, C.c_uint32, C.c_uint64, _dp,
                                             C.POINTER(C.c_uint32), C.POINTER(C.c_int32), C.POINTER(C.c_uint32)]
        L.orc_mtp_fixture_step.restype = C.c_int32
        L.orc_mtp_fixture_step.argtypes = [_fp, _fp, _fp, C.c_uint32, C.c_uint32, C.c_int32]
        L.orc_scripted_draft.argtypes = [_i32p, C.c_uint64, C.c_uint32, C.c_uint64, C.c_double, C.c_uint64,
                                         C.c_uint32, _i32p]
        L.orc_gen_weights.argtypes = [C.c_uint64, C.c_uint32, C.c_uint64, C.c_uint64, C.c_float, _fp]
        L.orc_rmsnorm.argtypes = [_fp, _fp, C.c_uint64, C.c_float, _fp]
        L.orc_silu.restype = C.c_float
        L.orc_silu.argtypes = [C.c_float]
        L.orc_llama_kv_rows.restype = C.c_int
        L.orc_llama_kv_rows.argtypes = [C.c_void_p, C.c_int, _u8p, _fp, _fp, C.c_uint64, C.c_uint32, _fp, _fp, C.c_int]
        L.orc_llama_layer.restype = C.c_int
        L.orc_llama_layer.argtypes = [C.c_void_p, C.c_int, _u8p, _u8p, _u8p, _u8p, _fp, _fp, _fp, _fp,
                                      C.c_uint64, C.c_uint32, C.c_void_p, _fp, C.c_int]

    # codecs
    def half_to_float(self, h: int) -> float:
        return self.L.orc_half_to_float(h)

    def float_to_half(self, f: float) -> int:
        return self.L.orc_float_to_half(f)

    def tensor_bytes(self, quant: str, n: int) -> int:
        return self.L.orc_tensor_bytes(QUANTS[quant], n)

    def decode(self, quant: str, data: np.ndarray, n: int) -> np.ndarray:
        out = np.zeros(n, F32)
        data = _c(data, np.uint8)
        st = self.L.orc_decode_tensor(QUANTS[quant], data, data.size, out, n)
        if st:
            raise ValueError(f"decode failed with code {st}")
        return out

    def encode(self, quant: str, v: np.ndarray) -> np.ndarray:
        v = _c(v, F32).ravel()
        out = np.zeros(self.tensor_bytes(quant, v.size), np.uint8)
        fn = {"q8_0-fixture": self.L.orc_encode_q8_fixture, "q8_0": self.L.orc_encode_q8_0,
              "q4_k": self.L.orc_encode_q4_k}[quant]
        if fn(v, v.size, out):
            raise ValueError("encode failed")
        return out

    # math
    def matmul_rows(self, w: np.ndarray, x: np.ndarray) -> np.ndarray:
        w = _c(w, F32)
        x = _c(x, F32)
        rows, cols = w.shape
        pos = x.shape[0]
        y = np.zeros((pos, rows), F32)
        self.L.orc_matmul_rows(w, rows, cols, x, pos, y)
        return y

    def matmul_rows_quant(self, quant: str, wbytes: np.ndarray, rows: int, cols: int, x: np.ndarray,
                          threads: int = 1) -> np.ndarray:
        x = _c(x, F32)
        pos = x.shape[0]
        y = np.zeros((pos, rows), F32)
        st = self.L.orc_matmul_rows_quant(QUANTS[quant], _c(wbytes, np.uint8), rows, cols, x, pos, y, threads)
        if st:
            raise ValueError(f"matmul_rows_quant failed with code {st}")
        return y

    # rng
    def philox(self, ctr, key) -> np.ndarray:
        out = np.zeros(4, np.uint32)
        self.L.orc_philox4x32_10(_c(ctr, np.uint32), _c(key, np.uint32), out)
        return out

    def philox_uniform(self, key: int, c0: int, c1: int, c2: int, c3: int) -> float:
        return self.L.orc_philox_uniform(key, c0, c1, c2, c3)

    def mix_seed(self, a: int, b: int) -> int:
        return self.L.orc_mix_seed(a, b)

    # sampling
    def argmax(self, logits) -> int:
        logits = _c(logits, F32)
        return self.L.orc_argmax(logits, logits.size)

    def distribution(self, logits, temperature=1.0, top_k=0, top_p=1.0) -> np.ndarray:
        logits = _c(logits, F32)
        out = np.zeros_like(logits)
        self.L.orc_distribution(logits, logits.size, temperature, top_k, top_p, out)
        return out

    def sample_from(self, probs, u: float) -> int:
        probs = _c(probs, F32)
        return self.L.orc_sample_from(probs, probs.size, u)

    def verify(self, target, drafts, draft_probs, uniforms):
        """One sequence: target (k+1, V), drafts (k,), draft_probs (k, V) or None, uniforms (>= k+1,)."""
        target = _c(target, F32)
        drafts = _c(drafts, np.int32)
        k = drafts.size
        V = target.shape[1]
        dp = None if draft_probs is None else _c(draft_probs, F32)
        acc, nxt, used = C.c_uint32(), C.c_int32(), C.c_uint32()
        self.L.orc_verify_speculative(target, drafts, None if dp is None else dp.ctypes.data, k, V,
                                      _c(uniforms, np.float64), C.byref(acc), C.byref(nxt), C.byref(used))
        return acc.value, nxt.value, used.value

    def mtp_step(self, embd, norm, head, prev: int) -> int:
        V, H = head.shape
        return self.L.orc_mtp_fixture_step(_c(embd, F32), _c(norm, F32), _c(head, F32), H, V, prev)

    def scripted_draft(self, ref, vocab, seed, rate, committed_len, count) -> np.ndarray:
        ref = _c(ref, np.int32)
        out = np.zeros(count, np.int32)
        self.L.orc_scripted_draft(ref, ref.size, vocab, seed, rate, committed_len, count, out)
        return out

    def rmsnorm(self, x, w, eps: float) -> np.ndarray:
        x = _c(x, F32)
        out = np.zeros_like(x)
        self.L.orc_rmsnorm(x, _c(w, F32), x.size, eps, out)
        return out

    def llama_layer(self, dims: "LlamaDims", quant: str, wqkv, wo, wgu, wd, attn_norm, ffn_norm, kcache, vcache,
                    base: int, h, parent=None, threads: int = 8) -> None:
        """In place on h (q, H) and the caches (max_ctx, kvd)."""
        par = None if parent is None else _c(parent, np.int32)
        st = self.L.orc_llama_layer(C.byref(dims), QUANTS[quant], wqkv, wo, wgu, wd, _c(attn_norm, F32),
                                    _c(ffn_norm, F32), kcache, vcache, base, h.shape[0],
                                    None if par is None else par.ctypes.data, h, threads)
        if st:
            raise RuntimeError(f"orc_llama_layer failed with code {st}")

    def llama_kv_rows(self, dims: "LlamaDims", quant: str, wqkv, attn_norm, kcache, vcache, base: int, h,
                      threads: int = 8) -> None:
        """The K / V rows of positions base..base+len(h)-1 into the caches (max_ctx, kvd), in place."""
        st = self.L.orc_llama_kv_rows(C.byref(dims), QUANTS[quant], wqkv, _c(attn_norm, F32), _c(h, F32), base,
                                      h.shape[0], kcache, vcache, threads)
        if st:
            raise RuntimeError(f"orc_llama_kv_rows failed with code {st}")

    def gen_weights(self, seed: int, tensor_id: int, first: int, n: int, stddev: float) -> np.ndarray:
        out = np.zeros(n, F32)
        self.L.orc_gen_weights(seed, tensor_id, first, n, stddev, out)
        return out


class LlamaDims(C.Structure):
    _fields_ = [("hidden", C.c_uint32), ("n_heads", C.c_uint32), ("n_kv_heads", C.c_uint32),
                ("head_dim", C.c_uint32), ("ffn", C.c_uint32), ("rope_theta", C.c_float), ("rms_eps", C.c_float)]


class Reference:
    """The reference's own compiled code (ref_shim.cpp over the unmodified sources)."""

    def __init__(self, path: str = REF_SO):
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} missing: the reference was not compiled here")
        L = self.L = C.CDLL(path)
        L.ref_last_error.restype = C.c_char_p
        L.ref_half_to_float.restype = C.c_float
        L.ref_half_to_float.argtypes = [C.c_uint16]
        L.ref_float_to_half.restype = C.c_uint16
        L.ref_float_to_half.argtypes = [C.c_float]
        L.ref_tensor_bytes.restype = C.c_uint64
        L.ref_tensor_bytes.argtypes = [C.c_int, C.c_uint64]
        L.ref_decode_tensor.restype = C.c_int
        L.ref_decode_tensor.argtypes = [C.c_int, _u8p, C.c_uint64, _fp, C.c_uint64]
        L.ref_encode.restype = C.c_int
        L.ref_encode.argtypes = [C.c_int, _fp, C.c_uint64, _u8p, C.c_uint64]
        L.ref_matmul_rows.argtypes = [_fp, C.c_uint64, C.c_uint64, _fp, C.c_uint64, _fp]
        L.ref_rng_uniforms.argtypes = [C.c_uint64, C.c_uint64, _dp]
        L.ref_mix_seed.restype = C.c_uint64
        L.ref_mix_seed.argtypes = [C.c_uint64, C.c_uint64]
        L.ref_argmax.restype = C.c_int32
        L.ref_argmax.argtypes = [_fp, C.c_uint64]
        L.ref_distribution.argtypes = [_fp, C.c_uint64, C.c_float, C.c_uint32, C.c_float, _fp]
        L.ref_sample_from.restype = C.c_int32
        L.ref_sample_from.argtypes = [_fp, C.c_uint64, C.c_uint64]
        L.ref_verify_speculative.argtypes = [_fp, _i32p, C.c_void_p, C.c_uint32, C.c_uint32, C.c_uint64, _u64p,
                                             _u32p, _i32p]
        L.ref_scripted_draft.argtypes = [_i32p, C.c_uint64, C.c_uint32, C.c_uint64, C.c_double, C.c_uint64,
                                         C.c_uint32, _i32p]
        L.ref_write_fixture.restype = C.c_int
        L.ref_write_fixture.argtypes = [C.c_char_p, C.c_int, C.c_uint32, C.c_uint64]
        L.ref_store_open.restype = C.c_void_p
        L.ref_store_open.argtypes = [C.c_char_p]
        L.ref_store_close.argtypes = [C.c_void_p]
        L.ref_store_object.restype = C.c_int
        L.ref_store_object.argtypes = [C.c_void_p, C.c_char_p, C.c_void_p, C.c_uint64, C.POINTER(C.c_int),
                                       C.POINTER(C.c_uint64)]
        L.ref_store_geometry.restype = C.c_int
        L.ref_store_geometry.argtypes = [C.c_void_p, _u32p, _u8p, C.c_uint32]
        L.ref_pipeline_create.restype = C.c_void_p
        L.ref_pipeline_create.argtypes = [C.c_char_p, _u32p, C.c_uint32, C.c_uint32, C.c_uint32]
        L.ref_pipeline_destroy.argtypes = [C.c_void_p]
        L.ref_pipeline_run.restype = C.c_int
        L.ref_pipeline_run.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint64, _i32p, C.c_uint32, _fp,
                                       C.c_void_p]
        L.ref_pipeline_commit.restype = C.c_int
        L.ref_pipeline_commit.argtypes = [C.c_void_p, C.c_uint64, C.c_uint64, C.c_uint32]
        L.ref_pipeline_abort.restype = C.c_int
        L.ref_pipeline_abort.argtypes = [C.c_void_p, C.c_uint64]
        L.ref_pipeline_mtp_step.restype = C.c_int32
        L.ref_pipeline_mtp_step.argtypes = [C.c_void_p, C.c_int32]
        L.ref_pipeline_mtp_logits.restype = C.c_int
        L.ref_pipeline_mtp_logits.argtypes = [C.c_void_p, C.c_int32, _fp]

    def err(self) -> str:
        return self.L.ref_last_error().decode()

    def decode(self, quant: str, data: np.ndarray, n: int) -> np.ndarray:
        out = np.zeros(n, F32)
        data = _c(data, np.uint8)
        st = self.L.ref_decode_tensor(QUANTS[quant], data, data.size, out, n)
        if st:
            raise ValueError(self.err())
        return out

    def encode(self, quant: str, v: np.ndarray) -> np.ndarray:
        v = _c(v, F32).ravel()
        out = np.zeros(self.L.ref_tensor_bytes(QUANTS[quant], v.size), np.uint8)
        if self.L.ref_encode(QUANTS[quant], v, v.size, out, out.size):
            raise ValueError(self.err())
        return out

    def matmul_rows(self, w, x):
        w = _c(w, F32)
        x = _c(x, F32)
        y = np.zeros((x.shape[0], w.shape[0]), F32)
        self.L.ref_matmul_rows(w, w.shape[0], w.shape[1], x, x.shape[0], y)
        return y

    def uniforms(self, seed: int, n: int) -> np.ndarray:
        out = np.zeros(n, np.float64)
        self.L.ref_rng_uniforms(seed, n, out)
        return out

    def distribution(self, logits, temperature=1.0, top_k=0, top_p=1.0):
        logits = _c(logits, F32)
        out = np.zeros_like(logits)
        self.L.ref_distribution(logits, logits.size, temperature, top_k, top_p, out)
        return out

    def verify(self, target, drafts, draft_probs, seeds):
        """target (B, k+1, V), drafts (B, k), draft_probs (B, k, V) or None, seeds (B,) -> (accepted, next)."""
        target = _c(target, F32)
        drafts = _c(drafts, np.int32)
        B, k = drafts.shape
        V = target.shape[2]
        dp = None if draft_probs is None else _c(draft_probs, F32)
        acc = np.zeros(B, np.uint32)
        nxt = np.zeros(B, np.int32)
        self.L.ref_verify_speculative(target, drafts, None if dp is None else dp.ctypes.data, B, k, V,
                                      _c(seeds, np.uint64), acc, nxt)
        return acc, nxt

    def scripted_draft(self, ref, vocab, seed, rate, committed_len, count):
        ref = _c(ref, np.int32)
        out = np.zeros(count, np.int32)
        self.L.ref_scripted_draft(ref, ref.size, vocab, seed, rate, committed_len, count, out)
        return out

    def write_fixture(self, d: str, tiny: bool = False, layers: int = 0, seed: int = 0x434C4D31) -> None:
        if self.L.ref_write_fixture(d.encode(), int(tiny), layers, seed):
            raise RuntimeError(self.err())


class ModelStore:
    """The reference's CanonicalModelStore over a fixture model directory: geometry and object bytes."""

    NAMES = {0: "f32", 1: "q8_0-fixture", 2: "q8_0"}

    def __init__(self, ref: Reference, model_dir: str):
        self.ref = ref
        self.h = ref.L.ref_store_open(model_dir.encode())
        if not self.h:
            raise RuntimeError(ref.err())
        dims = np.zeros(15, np.uint32)
        kinds = np.zeros(1024, np.uint8)
        ref.L.ref_store_geometry(self.h, dims, kinds, kinds.size)
        keys = ["n_layers", "hidden", "residual_streams", "n_experts", "n_active_experts", "expert_ff",
                "shared_expert_ff", "n_heads", "n_kv_heads", "head_dim", "vocab", "ple_layer", "ple_ngram",
                "ple_rows", "mtp_layers"]
        self.geometry = {k: int(v) for k, v in zip(keys, dims)}
        self.layer_kinds = kinds[: self.geometry["n_layers"]].copy()

    def object(self, name: str):
        """(quant name, bytes) of a provisioned object."""
        q, n = C.c_int(), C.c_uint64()
        if self.ref.L.ref_store_object(self.h, name.encode(), None, 0, C.byref(q), C.byref(n)):
            raise KeyError(self.ref.err())
        buf = np.zeros(n.value, np.uint8)
        self.ref.L.ref_store_object(self.h, name.encode(), buf.ctypes.data, buf.size, C.byref(q), C.byref(n))
        return self.NAMES[q.value], buf

    def close(self):
        if self.h:
            self.ref.L.ref_store_close(self.h)
            self.h = None


class RefPipeline:
    """ReferenceDomain stages over a fixture model directory (tests/domain/pipeline_harness.hpp pattern)."""

    def __init__(self, ref: Reference, model_dir: str, bounds, max_context=256, max_window=8, vocab=256,
                 floats_per_position=0):
        self.ref = ref
        b = np.asarray(bounds, np.uint32)
        self.h = ref.L.ref_pipeline_create(model_dir.encode(), b, b.size, max_context, max_window)
        if not self.h:
            raise RuntimeError(ref.err())
        self.vocab = vocab
        self.nstages = b.size - 1
        self.fpp = floats_per_position

    def close(self):
        if self.h:
            self.ref.L.ref_pipeline_destroy(self.h)
            self.h = None

    def run(self, window_id, base, state, tokens, want_stages=False):
        tokens = _c(tokens, np.int32)
        q = tokens.size
        logits = np.zeros((q, self.vocab), F32)
        stage_out = np.zeros((self.nstages - 1, q, self.fpp), F32) if want_stages else None
        st = self.ref.L.ref_pipeline_run(self.h, window_id, base, state, tokens, q, logits,
                                         None if stage_out is None else stage_out.ctypes.data)
        if st:
            raise RuntimeError(self.ref.err())
        return (logits, stage_out) if want_stages else logits

    def commit(self, window_id, state, accepted):
        if self.ref.L.ref_pipeline_commit(self.h, window_id, state, accepted):
            raise RuntimeError(self.ref.err())

    def abort(self, window_id):
        if self.ref.L.ref_pipeline_abort(self.h, window_id):
            raise RuntimeError(self.ref.err())

    def mtp_step(self, prev: int) -> int:
        return self.ref.L.ref_pipeline_mtp_step(self.h, prev)

    def mtp_logits(self, prev: int) -> np.ndarray:
        out = np.zeros(self.vocab, F32)
        self.ref.L.ref_pipeline_mtp_logits(self.h, prev, out)
        return out
