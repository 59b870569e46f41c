"""GGUF files for the Llama-family engine: a reader of the GGUF v2/v3 container (header, metadata, tensor table,
aligned data section) and the binding of a file's tensors to an engine (clm_b200_llama_load_tensors).

The container layout is the published GGUF format of ggml / llama.cpp, the one ClusterLM's own reader parses
(runtime/objects/src/gguf.cpp:291-360: magic, versions 2 and 3, general.alignment) before its manifests classify the
tensors by name (runtime/objects/src/gguf_manifest.cpp:19-21, 146). Tensor data stays memory-mapped; only the
tensors of an engine's stage are read, during the binding call.
"""
from __future__ import annotations

import ctypes as C
import struct
from dataclasses import dataclass

import numpy as np

from ._native import CLM_UNIMPLEMENTED, QUANTS, ClmError, call
from .engine import LlamaGeometry

# ggml tensor types this engine binds, and their (block elements, block bytes)
GGML_F32, GGML_Q8_0, GGML_Q4_K = 0, 8, 12
_BLOCKS = {0: (1, 4), 1: (1, 2), 2: (32, 18), 3: (32, 20), 6: (32, 22), 7: (32, 24), 8: (32, 34), 10: (256, 84),
           11: (256, 110), 12: (256, 144), 13: (256, 176), 14: (256, 210), 15: (256, 292), 30: (1, 2)}
_TO_CLM = {GGML_F32: QUANTS["f32"], GGML_Q8_0: QUANTS["q8_0"], GGML_Q4_K: QUANTS["q4_k"]}
_QUANT_NAME = {GGML_Q8_0: "q8_0", GGML_Q4_K: "q4_k"}

# metadata value types
_SCALARS = {0: "<B", 1: "<b", 2: "<H", 3: "<h", 4: "<I", 5: "<i", 6: "<f", 7: "<?", 10: "<Q", 11: "<q", 12: "<d"}
_STRING, _ARRAY = 8, 9


@dataclass
class TensorInfo:
    name: str
    dims: tuple  # ggml order: dims[0] is the innermost (columns)
    ggml_type: int
    offset: int  # from the start of the data section
    nbytes: int


class GGUFFile:
    """A GGUF file: `kv` (metadata), `tensors` (name -> TensorInfo) and `data(name)` (a uint8 view)."""

    def __init__(self, path: str):
        self.path = path
        self._map = np.memmap(path, dtype=np.uint8, mode="r")
        self._pos = 0
        if bytes(self._take(4)) != b"GGUF":
            raise ValueError(f"{path}: not a GGUF file")
        self.version = self._u32()
        if self.version not in (2, 3):
            raise ValueError(f"{path}: GGUF version {self.version} is not supported")
        n_tensors, n_kv = self._u64(), self._u64()
        self.kv = {}
        for _ in range(n_kv):
            key = self._str()
            self.kv[key] = self._value(self._u32())
        infos = []
        for _ in range(n_tensors):
            name = self._str()
            n_dims = self._u32()
            dims = tuple(self._u64() for _ in range(n_dims))
            t = self._u32()
            off = self._u64()
            infos.append((name, dims, t, off))
        align = int(self.kv.get("general.alignment", 32))
        self.data_start = (self._pos + align - 1) // align * align
        self.tensors = {}
        for name, dims, t, off in infos:
            elems = int(np.prod(dims, dtype=np.uint64)) if dims else 1
            be, bb = _BLOCKS.get(t, (0, 0))
            nbytes = elems // be * bb if be else -1
            self.tensors[name] = TensorInfo(name, dims, t, off, nbytes)

    # -- container primitives
    def _take(self, n: int) -> np.ndarray:
        if self._pos + n > self._map.size:
            raise ValueError(f"{self.path}: truncated")
        v = self._map[self._pos:self._pos + n]
        self._pos += n
        return v

    def _unpack(self, fmt: str):
        return struct.unpack(fmt, bytes(self._take(struct.calcsize(fmt))))[0]

    def _u32(self) -> int:
        return self._unpack("<I")

    def _u64(self) -> int:
        return self._unpack("<Q")

    def _str(self) -> str:
        return bytes(self._take(self._u64())).decode("utf-8")

    def _value(self, t: int):
        if t in _SCALARS:
            return self._unpack(_SCALARS[t])
        if t == _STRING:
            return self._str()
        if t == _ARRAY:
            et, n = self._u32(), self._u64()
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"{self.path}: unknown metadata type {t}")

    # -- tensors
    def data(self, name: str) -> np.ndarray:
        info = self.tensors[name]
        if info.nbytes < 0:
            raise ValueError(f"{name}: ggml type {info.ggml_type} has no known block size")
        start = self.data_start + info.offset
        if start + info.nbytes > self._map.size:
            raise ValueError(f"{self.path}: tensor {name} runs past the end of the file")
        return self._map[start:start + info.nbytes]


def llama_geometry(f: GGUFFile) -> LlamaGeometry:
    """The engine geometry of a llama-architecture GGUF file (metadata keys of llama.cpp's llama loader)."""
    arch = f.kv.get("general.architecture", "llama")
    key = lambda k: f"{arch}.{k}"  # noqa: E731
    H = int(f.kv[key("embedding_length")])
    nh = int(f.kv[key("attention.head_count")])
    nkv = int(f.kv.get(key("attention.head_count_kv"), nh))
    hd = int(f.kv.get(key("attention.key_length"), H // nh))
    q = f.tensors["blk.0.attn_q.weight"].ggml_type
    if q not in _QUANT_NAME:
        raise ValueError(f"{f.path}: matrices in ggml type {q}; the engine binds Q4_K or Q8_0")
    # RoPE frequency scaling (Llama 3.1+ files carry rope_freqs.weight; others a rope.scaling.type) changes the
    # rotation llama.cpp applies; the engine's RoPE table is the plain theta^(-2i/hd) one, so such files are refused
    # rather than run with different logits
    if "rope_freqs.weight" in f.tensors:
        raise ClmError(CLM_UNIMPLEMENTED, f"{f.path}: rope_freqs.weight (RoPE frequency factors) is not supported")
    scaling = f.kv.get(key("rope.scaling.type"), "none")
    if scaling not in ("none", ""):
        raise ClmError(CLM_UNIMPLEMENTED, f"{f.path}: RoPE scaling '{scaling}' is not supported")
    return LlamaGeometry(
        n_layers=int(f.kv[key("block_count")]), hidden=H, n_heads=nh, n_kv_heads=nkv, head_dim=hd,
        ffn=int(f.kv[key("feed_forward_length")]), vocab=int(f.tensors["token_embd.weight"].dims[1]),
        rope_theta=float(f.kv.get(key("rope.freq_base"), 10000.0)),
        rms_eps=float(f.kv.get(key("attention.layer_norm_rms_epsilon"), 1e-5)), quant=_QUANT_NAME[q],
        mtp="mtp.ffn_gate.weight" in f.tensors)


class _Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("quant", C.c_int), ("data", C.c_void_p), ("bytes", C.c_uint64)]


def load_into(engine, f: GGUFFile) -> None:
    """Binds the file's tensors to `engine` (an engine.Engine not yet prepared): the engine takes the ones of its
    stage (its layer range, the embedding, head and MTP head as its role needs)."""
    keep = []
    arr = (_Tensor * len(f.tensors))()
    n = 0
    for name, info in f.tensors.items():
        if info.ggml_type not in _TO_CLM:
            # passed without data and with no CLM quantisation: the engine refuses it by name (CLM_UNIMPLEMENTED)
            # if its stage needs it, and ignores it otherwise
            arr[n] = _Tensor(name.encode(), -1 - info.ggml_type, None, 0)
            n += 1
            continue
        buf = np.ascontiguousarray(f.data(name))
        keep.append(buf)
        arr[n] = _Tensor(name.encode(), _TO_CLM[info.ggml_type], buf.ctypes.data, info.nbytes)
        n += 1
    call("clm_b200_llama_load_tensors", engine.h, C.cast(arr, C.c_void_p), n)
