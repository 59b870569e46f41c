"""Python face of the engine ABI (clm_b200_llama_create and friends) with host numpy buffers.

Mirrors the ExecutionDomain flow of the reference (runtime/domain/include/clusterlm/domain/
execution_domain.hpp:143-174): create -> (weights) -> prepare -> open_session -> run_window -> commit /
abort.  Admission rules (epochs, window ids) belong to the caller's ledger; the engine checks positions.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np

from ._native import LINK_HANDLE_BYTES, QUANTS, call

_vp = C.c_void_p

ROLE_PREFIX, ROLE_MIDDLE, ROLE_TAIL, ROLE_WHOLE = 0, 1, 2, 3


class _Geometry(C.Structure):
    _fields_ = [("n_layers", C.c_uint32), ("hidden", C.c_uint32), ("n_heads", C.c_uint32),
                ("n_kv_heads", C.c_uint32), ("head_dim", C.c_uint32), ("ffn", C.c_uint32), ("vocab", C.c_uint32),
                ("rope_theta", C.c_float), ("rms_eps", C.c_float), ("quant", C.c_int), ("mtp", C.c_uint32)]


class _Spec(C.Structure):
    _fields_ = [("layer_begin", C.c_uint32), ("layer_end", C.c_uint32), ("role", C.c_int),
                ("max_context", C.c_uint32), ("max_window", C.c_uint32), ("max_sessions", C.c_uint32)]


class _SpecParams(C.Structure):
    _fields_ = [("q", C.c_uint32), ("temperature", C.c_float), ("seed", C.c_uint64)]


@dataclass
class LlamaGeometry:
    n_layers: int
    hidden: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    ffn: int
    vocab: int
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5
    quant: str = "q4_k"
    mtp: bool = True

    def c(self) -> _Geometry:
        return _Geometry(self.n_layers, self.hidden, self.n_heads, self.n_kv_heads, self.head_dim, self.ffn,
                         self.vocab, self.rope_theta, self.rms_eps, QUANTS[self.quant], int(self.mtp))


LLAMA3_8B = LlamaGeometry(32, 4096, 32, 8, 128, 14336, 128256)
LLAMA3_70B = LlamaGeometry(80, 8192, 64, 8, 128, 28672, 128256)


def _i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def _f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


class _FixGeometry(C.Structure):
    _fields_ = [(n, C.c_uint32) for n in ("n_layers", "hidden", "residual_streams", "n_experts", "n_active_experts",
                                          "expert_ff", "shared_expert_ff", "n_heads", "n_kv_heads", "head_dim",
                                          "vocab", "ple_layer", "ple_ngram", "ple_rows")] + [("layer_kinds", _vp)]


@dataclass
class FixtureGeometry:
    """ModelGeometry of the clusterlm-fixture family (runtime/objects/include/clusterlm/objects/geometry.hpp)."""
    n_layers: int
    hidden: int
    residual_streams: int
    n_experts: int
    n_active_experts: int
    expert_ff: int
    shared_expert_ff: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    ple_layer: int
    ple_ngram: int
    ple_rows: int
    layer_kinds: tuple

    @property
    def floats_per_position(self) -> int:
        return self.residual_streams * self.hidden + self.hidden + self.residual_streams


class Engine:
    def __init__(self, ctx, geometry: LlamaGeometry, layer_begin: int, layer_end: int, role: int,
                 max_context: int, max_window: int, max_sessions: int = 1):
        self.ctx, self.geo, self.role = ctx, geometry, role
        self.max_window = max_window
        self._g = geometry.c()
        self._s = _Spec(layer_begin, layer_end, role, max_context, max_window, max_sessions)
        h = _vp()
        call("clm_b200_llama_create", ctx.h, C.byref(self._g), C.byref(self._s), C.byref(h))
        self.h = h
        self.fpp = 2 * geometry.hidden + 1
        self.vocab = geometry.vocab

    def close(self):
        if self.h:
            call("clm_b200_engine_destroy", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def generate_weights(self, seed: int = 0, stddev: float = 0.02):
        call("clm_b200_engine_generate_weights", self.h, seed, stddev)

    def load_gguf(self, path: str):
        """Binds this stage's weights from a GGUF file (clusterlm_b200.gguf_file; llama.cpp tensor names)."""
        from .gguf_file import GGUFFile, load_into

        load_into(self, GGUFFile(path))

    def prepare(self):
        call("clm_b200_engine_prepare", self.h)

    def info(self):
        w, s, f = C.c_uint64(), C.c_uint64(), C.c_uint32()
        call("clm_b200_engine_info", self.h, C.byref(w), C.byref(s), C.byref(f))
        return {"weight_bytes": w.value, "state_bytes_per_session": s.value, "floats_per_position": f.value}

    def open_session(self, session: int):
        call("clm_b200_session_open", self.h, session)

    def close_session(self, session: int):
        call("clm_b200_session_close", self.h, session)

    def last_launches(self) -> int:
        v = C.c_uint64()
        call("clm_b200_engine_last_launches", self.h, C.byref(v))
        return v.value

    def stream(self) -> int:
        v = _vp()
        call("clm_b200_ctx_stream", self.ctx.h, C.byref(v))
        return v.value or 0

    def position(self, session: int) -> int:
        v = C.c_uint64()
        call("clm_b200_session_position", self.h, session, C.byref(v))
        return v.value

    def run_window(self, session: int, base: int, tokens=None, records=None):
        """Returns logits (q, vocab) for tail/whole stages, records (q, floats_per_position) otherwise."""
        fpp = self.fpp
        if tokens is not None:
            tokens = _i32(tokens)
            q = tokens.size
        else:
            records = _f32(records)
            q = records.shape[0]
        has_head = self.role in (ROLE_TAIL, ROLE_WHOLE)
        out = np.zeros((q, self.vocab if has_head else fpp), np.float32)
        call("clm_b200_run_window", self.h, session, base, q,
             None if tokens is None else tokens.ctypes.data_as(_vp),
             None if records is None else records.ctypes.data_as(_vp),
             None if has_head else out.ctypes.data_as(_vp), out.ctypes.data_as(_vp) if has_head else None)
        return out

    def run_window_device(self, session: int, base: int, d_tokens=None, d_out=None, stream=None, d_records=None):
        """Device-buffer window (torch CUDA tensors): tokens or records in; logits or records out."""
        q = (d_tokens if d_tokens is not None else d_records).shape[0]
        has_head = self.role in (ROLE_TAIL, ROLE_WHOLE)
        call("clm_b200_run_window_device", self.h, session, base, q,
             None if d_tokens is None else _vp(d_tokens.data_ptr()),
             None if d_records is None else _vp(d_records.data_ptr()),
             None if has_head else _vp(d_out.data_ptr()), _vp(d_out.data_ptr()) if has_head else None,
             None if stream is None else _vp(stream))

    def run_tree_window(self, session: int, base: int, parents, tokens=None, records=None):
        """Tree window: node i's parent is parents[i] (an earlier node or -1); logits or records per node."""
        parents = _i32(parents)
        fpp = self.fpp
        if tokens is not None:
            tokens = _i32(tokens)
        else:
            records = _f32(records)
        q = parents.size
        has_head = self.role in (ROLE_TAIL, ROLE_WHOLE)
        out = np.zeros((q, self.vocab if has_head else fpp), np.float32)
        call("clm_b200_run_tree_window", self.h, session, base, q, parents.ctypes.data_as(_vp),
             None if tokens is None else tokens.ctypes.data_as(_vp),
             None if records is None else records.ctypes.data_as(_vp),
             None if has_head else out.ctypes.data_as(_vp), out.ctypes.data_as(_vp) if has_head else None)
        return out

    def run_batch_window(self, sessions, bases, tokens, parents=None, logits=True):
        """One window over several sessions (clm_b200_run_batch_window): tokens (n, q), shared tree parents (q,) or
        None for linear windows; returns logits (n, q, vocab), or None with logits=False (no device-to-host copy)."""
        ids = np.ascontiguousarray(sessions, dtype=np.uint64)
        bs = np.ascontiguousarray(bases, dtype=np.uint64)
        tokens = _i32(tokens)
        n, q = tokens.shape
        out = np.zeros((n, q, self.vocab), np.float32) if logits else None
        par = None if parents is None else _i32(parents)
        call("clm_b200_run_batch_window", self.h, n, ids.ctypes.data_as(_vp), bs.ctypes.data_as(_vp), q,
             None if par is None else par.ctypes.data_as(_vp), tokens.ctypes.data_as(_vp),
             None if out is None else out.ctypes.data_as(_vp))
        return out

    def run_batch_window_device(self, sessions, bases, positions: int, d_tokens=None, d_records=None, d_out=None,
                                stream=None):
        """One linear window over up to 4 sessions on the q-row GEMV chain (clm_b200_run_batch_window_device): device
        tokens (n * positions,) or records (n * positions, floats per position) in, session-major; logits or records
        out (d_out)."""
        ids = np.ascontiguousarray(sessions, dtype=np.uint64)
        bs = np.ascontiguousarray(bases, dtype=np.uint64)
        has_head = self.role in (ROLE_TAIL, ROLE_WHOLE)
        call("clm_b200_run_batch_window_device", self.h, ids.size, ids.ctypes.data_as(_vp), bs.ctypes.data_as(_vp),
             positions, None if d_tokens is None else _vp(d_tokens.data_ptr()),
             None if d_records is None else _vp(d_records.data_ptr()),
             None if has_head else _vp(d_out.data_ptr()), _vp(d_out.data_ptr()) if has_head else None,
             None if stream is None else _vp(stream))

    def run_tree_window_device(self, session: int, base: int, d_parents, d_tokens=None, d_out=None, stream=None,
                               d_records=None):
        """Device-buffer tree window (torch CUDA tensors): parents, tokens or records in; logits or records out."""
        q = d_parents.shape[0]
        has_head = self.role in (ROLE_TAIL, ROLE_WHOLE)
        call("clm_b200_run_tree_window_device", self.h, session, base, q, _vp(d_parents.data_ptr()),
             None if d_tokens is None else _vp(d_tokens.data_ptr()),
             None if d_records is None else _vp(d_records.data_ptr()),
             None if has_head else _vp(d_out.data_ptr()), _vp(d_out.data_ptr()) if has_head else None,
             None if stream is None else _vp(stream))

    def commit_path(self, session: int, path):
        """Keeps the root-to-node path (node indices) of the outstanding window."""
        path = _i32(path)
        call("clm_b200_commit_path", self.h, session, path.ctypes.data_as(_vp), path.size)

    def commit(self, session: int, accepted: int):
        call("clm_b200_commit", self.h, session, accepted)

    def abort(self, session: int):
        call("clm_b200_abort", self.h, session)

    def mtp_propose(self, prev: int, uniforms, temperature: float = 1.0, top_k: int = 0, top_p: float = 1.0):
        """len(uniforms) drafts after prev, each sampled with its uniform; returns (tokens, probs (count, vocab))."""
        u = np.ascontiguousarray(uniforms, dtype=np.float64)
        count = u.size
        toks = np.zeros(count, np.int32)
        probs = np.zeros((count, self.vocab), np.float32)
        call("clm_b200_mtp_propose", self.h, prev, count, temperature, top_k, top_p, u.ctypes.data_as(_vp),
             toks.ctypes.data_as(_vp), probs.ctypes.data_as(_vp))
        return toks, probs

    def mtp_draft(self, prev: int, count: int, temperature: float = 0.0, seed: int = 0, counter: int = 0,
                  want_logits: bool = False):
        toks = np.zeros(count, np.int32)
        logits = np.zeros((count, self.vocab), np.float32) if want_logits else None
        call("clm_b200_mtp_draft", self.h, prev, count, temperature, seed, counter, toks.ctypes.data_as(_vp),
             None if logits is None else logits.ctypes.data_as(_vp))
        return (toks, logits) if want_logits else toks

    def spec_begin(self, session: int, prompt, q: int, temperature: float = 0.0, seed: int = 0):
        prompt = _i32(prompt)
        p = _SpecParams(q, temperature, seed)
        call("clm_b200_spec_begin", self.h, session, prompt.ctypes.data_as(_vp), prompt.size, C.byref(p))

    def spec_round(self, session: int, q: int, temperature: float = 0.0, seed: int = 0) -> np.ndarray:
        p = _SpecParams(q, temperature, seed)
        toks = np.zeros(q + 1, np.int32)
        n = C.c_uint32()
        call("clm_b200_spec_round", self.h, session, C.byref(p), toks.ctypes.data_as(_vp), C.byref(n))
        return toks[: n.value].copy()

    def spec_round_device(self, session: int, q: int, temperature: float = 0.0, seed: int = 0, d_tokens=None,
                          d_count=None, stream=None):
        p = _SpecParams(q, temperature, seed)
        call("clm_b200_spec_round_device", self.h, session, C.byref(p),
             None if d_tokens is None else _vp(d_tokens.data_ptr()),
             None if d_count is None else _vp(d_count.data_ptr()), stream)


    # ---- stage pipeline (clm_b200_pipe_*)
    def pipe_attach(self, link_in: "Link", link_out: "Link"):
        call("clm_b200_pipe_attach", self.h, link_in.h, link_out.h)
        self._links = (link_in, link_out)  # the links must outlive the engine's use of them

    def pipe_prefill(self, session: int, q: int, tokens=None, stream=None):
        """One prompt chunk of q positions through this stage, committed at once (the prefix takes tokens)."""
        t = None if tokens is None else _i32(tokens)
        call("clm_b200_pipe_prefill", self.h, session, None if t is None else t.ctypes.data_as(_vp), q,
             None if stream is None else _vp(stream))

    def pipe_begin(self, session: int, row: int, q: int, temperature: float = 0.0, seed: int = 0, stream=None):
        p = _SpecParams(q, temperature, seed)
        call("clm_b200_pipe_begin", self.h, session, row, C.byref(p), None if stream is None else _vp(stream))

    def pipe_round(self, session: int, q: int, temperature: float = 0.0, seed: int = 0, d_tokens=None, d_count=None,
                   stream=None):
        p = _SpecParams(q, temperature, seed)
        call("clm_b200_pipe_round", self.h, session, C.byref(p),
             None if d_tokens is None else _vp(d_tokens.data_ptr()),
             None if d_count is None else _vp(d_count.data_ptr()), None if stream is None else _vp(stream))

    def pipe_status(self, stream=None):
        call("clm_b200_pipe_status", self.h, None if stream is None else _vp(stream))

    def pipe_attach_session(self, session: int, link_in=None, link_out=None):
        """Binds `session`'s messages to their own links (None: the engine's)."""
        call("clm_b200_pipe_attach_session", self.h, session, None if link_in is None else link_in.h,
             None if link_out is None else link_out.h)


LINK_SEND, LINK_RECV = 0, 1


class Link:
    """One end of a one-way stage link between two GPUs (clm_b200_link_*)."""

    def __init__(self, ctx, end: int, slots: int, payload_bytes: int, timeout_s: float = 30.0):
        h = _vp()
        call("clm_b200_link_create", ctx.h, end, slots, payload_bytes, timeout_s, C.byref(h))
        self.h, self.end, self.ctx = h, end, ctx

    def export(self) -> bytes:
        buf = C.create_string_buffer(LINK_HANDLE_BYTES)
        call("clm_b200_link_export", self.h, buf)
        return buf.raw

    def connect(self, peer_handle: bytes):
        if len(peer_handle) != LINK_HANDLE_BYTES:
            raise ValueError("link handle has the wrong size")
        buf = C.create_string_buffer(peer_handle, LINK_HANDLE_BYTES)
        call("clm_b200_link_connect", self.h, buf)

    def close(self):
        if self.h:
            call("clm_b200_link_destroy", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class FixtureEngine(Engine):
    """A stage of the clusterlm-fixture family (the reference's own model) on the device."""

    def __init__(self, ctx, geometry: FixtureGeometry, layer_begin: int, layer_end: int, role: int,
                 max_context: int, max_window: int, max_sessions: int = 1):
        self.ctx, self.geo, self.role = ctx, geometry, role
        self.max_window = max_window
        self._kinds = np.ascontiguousarray(np.asarray(geometry.layer_kinds, np.uint8))
        g = geometry
        self._g = _FixGeometry(g.n_layers, g.hidden, g.residual_streams, g.n_experts, g.n_active_experts,
                               g.expert_ff, g.shared_expert_ff, g.n_heads, g.n_kv_heads, g.head_dim, g.vocab,
                               g.ple_layer, g.ple_ngram, g.ple_rows, self._kinds.ctypes.data_as(_vp))
        self._s = _Spec(layer_begin, layer_end, role, max_context, max_window, max_sessions)
        h = _vp()
        call("clm_b200_fixture_create", ctx.h, C.byref(self._g), C.byref(self._s), C.byref(h))
        self.h = h
        self.fpp = geometry.floats_per_position
        self.vocab = geometry.vocab

    def set_object(self, name: str, quant: str, data) -> None:
        buf = np.ascontiguousarray(data, np.uint8)
        call("clm_b200_engine_set_object", self.h, name.encode(), QUANTS[quant], buf.ctypes.data_as(_vp), buf.nbytes)
