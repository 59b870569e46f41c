"""Python face of the C ABI for device buffers held in torch tensors.

Names and argument meanings mirror the reference's own functions so tests read like the reference's tests:
  tensor_bytes / decode_tensor        runtime/objects/src/tensor_codec.cpp:9-99
  Matrix.matmul_rows                  runtime/domain/src/reference_kernels.cpp:24-30
  argmax_token / distribution /
  sample_from / verify_speculative    runtime/domain/src/sampling.cpp:44-131
torch is used only for device memory and streams; every computation runs in libclm_b200.so.
"""
from __future__ import annotations

import ctypes as C

import torch

from ._native import QUANTS, call, lib

_vp = C.c_void_p


def _ptr(t: torch.Tensor | None):
    if t is None:
        return None
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError("expected a contiguous tensor")
    return _vp(t.data_ptr())


# cudaStreamLegacy: the legacy default stream named explicitly (a NULL stream argument selects the context's own
# non-blocking stream in the C ABI, which is not ordered with torch's default stream).
_LEGACY_STREAM = 0x1


def _stream() -> _vp:
    """The stream the C ABI call runs on: torch's current stream, so torch work before and after is ordered."""
    h = torch.cuda.current_stream().cuda_stream
    return _vp(h if h else _LEGACY_STREAM)


def device_count() -> int:
    n = C.c_int(0)
    call("clm_b200_device_count", C.byref(n))
    return n.value


class Context:
    """One device context (a stream and the allocations made through it)."""

    def __init__(self, device: int = 0):
        h = _vp()
        call("clm_b200_ctx_create", device, C.byref(h))
        self.h = h
        self.device = device

    def close(self) -> None:
        if self.h:
            call("clm_b200_ctx_destroy", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def synchronize(self) -> None:
        call("clm_b200_ctx_synchronize", self.h)


def tensor_bytes(quant: str, n: int) -> int:
    return lib.clm_b200_tensor_bytes(QUANTS[quant], n)


def decode_tensor(ctx: Context, quant: str, data: torch.Tensor, n: int) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=data.device)
    call("clm_b200_decode_tensor", ctx.h, QUANTS[quant], _ptr(data), data.numel() * data.element_size(), _ptr(out), n,
         _stream())
    return out


def encode(ctx: Context, quant: str, x: torch.Tensor) -> torch.Tensor:
    n = x.numel()
    out = torch.empty(tensor_bytes(quant, n), dtype=torch.uint8, device=x.device)
    call("clm_b200_encode", ctx.h, QUANTS[quant], _ptr(x), n, _ptr(out), _stream())
    return out


def generate_weights(ctx: Context, seed: int, tensor_id: int, first: int, n: int, stddev: float) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float32, device=f"cuda:{ctx.device}")
    call("clm_b200_generate_weights", ctx.h, seed, tensor_id, first, n, stddev, _ptr(out), _stream())
    return out


class Matrix:
    """A resident weight matrix in its stored representation (repacked for the tiled kernels)."""

    def __init__(self, ctx: Context, quant: str, data, rows: int, cols: int):
        h = _vp()
        if isinstance(data, torch.Tensor) and data.is_cuda:
            call("clm_b200_matrix_upload_device", ctx.h, QUANTS[quant], _ptr(data), data.numel() * data.element_size(),
                 rows, cols, C.byref(h))
        else:
            import numpy as np

            buf = np.ascontiguousarray(data, dtype=np.uint8)
            call("clm_b200_matrix_upload", ctx.h, QUANTS[quant], buf.ctypes.data_as(_vp), buf.nbytes, rows, cols,
                 C.byref(h))
        self.h, self.ctx, self.quant, self.rows, self.cols = h, ctx, quant, rows, cols

    def close(self) -> None:
        if self.h:
            call("clm_b200_matrix_free", self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_bytes(self) -> int:
        b = C.c_uint64()
        call("clm_b200_matrix_info", self.h, None, None, None, C.byref(b))
        return b.value

    def matmul_rows(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        """y[p][i] = W[i] . x[p] for x of shape (positions, cols)."""
        x = x.contiguous()
        q = x.shape[0]
        y = out if out is not None else torch.empty((q, self.rows), dtype=torch.float32, device=x.device)
        call("clm_b200_matmul_rows", self.ctx.h, self.h, _ptr(x), q, _ptr(y), _stream())
        return y


def argmax_token(ctx: Context, logits: torch.Tensor) -> torch.Tensor:
    rows, vocab = logits.shape
    out = torch.empty(rows, dtype=torch.int32, device=logits.device)
    call("clm_b200_argmax_rows", ctx.h, _ptr(logits), rows, vocab, _ptr(out), _stream())
    return out


def distribution(ctx: Context, logits: torch.Tensor, temperature: float = 0.0, top_k: int = 0,
                 top_p: float = 1.0) -> torch.Tensor:
    rows, vocab = logits.shape
    out = torch.empty_like(logits)
    call("clm_b200_distribution_rows", ctx.h, _ptr(logits), rows, vocab, temperature, top_k, top_p, _ptr(out),
         _stream())
    return out


def sample_from(ctx: Context, probs: torch.Tensor, uniforms: torch.Tensor) -> torch.Tensor:
    rows, vocab = probs.shape
    out = torch.empty(rows, dtype=torch.int32, device=probs.device)
    call("clm_b200_sample_rows", ctx.h, _ptr(probs), rows, vocab, _ptr(uniforms), _ptr(out), _stream())
    return out


def verify_speculative(ctx: Context, target: torch.Tensor, drafts: torch.Tensor, draft_probs: torch.Tensor | None,
                       uniforms: torch.Tensor | None = None, seed: int = 0, counter_base: int = 0):
    """target (B, k+1, V), drafts (B, k), draft_probs (B, k, V) or None -> (accepted (B,), next (B,))."""
    B, k1, V = target.shape
    acc = torch.empty(B, dtype=torch.int32, device=target.device)
    nxt = torch.empty(B, dtype=torch.int32, device=target.device)
    call("clm_b200_verify_speculative", ctx.h, _ptr(target), _ptr(drafts), _ptr(draft_probs), B, k1 - 1, V,
         _ptr(uniforms), seed, counter_base, _ptr(acc), _ptr(nxt), _stream())
    return acc, nxt


def accept_logits(ctx: Context, target_logits: torch.Tensor, draft_logits: torch.Tensor | None, drafts: torch.Tensor,
                  temperature: float = 1.0, uniforms: torch.Tensor | None = None, seed: int = 0, counter_base: int = 0):
    """Fused distribution + verify_speculative from logits (target (B, k+1, V), draft (B, k, V) or None)."""
    B, k1, V = target_logits.shape
    acc = torch.empty(B, dtype=torch.int32, device=target_logits.device)
    nxt = torch.empty(B, dtype=torch.int32, device=target_logits.device)
    call("clm_b200_accept_logits", ctx.h, _ptr(target_logits), _ptr(draft_logits), _ptr(drafts), B, k1 - 1, V,
         temperature, _ptr(uniforms), seed, counter_base, _ptr(acc), _ptr(nxt), _stream())
    return acc, nxt


def philox_uniforms(ctx: Context, seed: int, first: int, c2: int, c3: int, n: int) -> torch.Tensor:
    out = torch.empty(n, dtype=torch.float64, device=f"cuda:{ctx.device}")
    call("clm_b200_philox_uniforms", ctx.h, seed, first, c2, c3, n, _ptr(out), _stream())
    return out
