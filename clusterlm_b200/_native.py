"""ctypes binding of libclm_b200.so (the C ABI declared in include/clm_b200.h).

The library is required: importing this module fails loudly when it is missing, and every call raises
`ClmError` with the library's status code and message.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("CLM_B200_LIB", os.path.join(HERE, "lib", "libclm_b200.so"))

# clusterlm::ErrorCode (runtime/common/include/clusterlm/common/status.hpp:15-36)
ERROR_NAMES = {
    0: "kOk", 1: "kInvalidArgument", 2: "kOutOfRange", 3: "kNotFound", 4: "kAlreadyExists",
    5: "kFailedPrecondition", 6: "kResourceExhausted", 7: "kDataLoss", 8: "kUnauthenticated",
    9: "kPermissionDenied", 10: "kStaleEpoch", 11: "kAborted", 12: "kCancelled", 13: "kDeadlineExceeded",
    14: "kUnavailable", 15: "kVersionMismatch", 16: "kProtocolError", 17: "kInternal", 18: "kUnimplemented",
    19: "kHardwareUnavailable",
}
QUANTS = {"f32": 0, "q8_0-fixture": 1, "q8_0": 2, "q4_k": 3}
CLM_UNIMPLEMENTED = 18


class ClmError(RuntimeError):
    def __init__(self, code: int, message: str):
        self.code = code
        self.name = ERROR_NAMES.get(code, f"code{code}")
        super().__init__(f"{self.name}: {message}")


if not os.path.exists(LIB_PATH):
    raise ImportError(f"libclm_b200.so not found at {LIB_PATH}; build it with __graft_entry__.build()")

lib = C.CDLL(LIB_PATH)

_i, _u32, _u64, _f, _vp = C.c_int, C.c_uint32, C.c_uint64, C.c_float, C.c_void_p
_SIGS = {
    "clm_b200_abi_version": (_i, []),
    "clm_b200_last_error": (C.c_char_p, []),
    "clm_b200_device_count": (_i, [C.POINTER(_i)]),
    "clm_b200_ctx_create": (_i, [_i, C.POINTER(_vp)]),
    "clm_b200_ctx_destroy": (_i, [_vp]),
    "clm_b200_ctx_stream": (_i, [_vp, C.POINTER(_vp)]),
    "clm_b200_ctx_synchronize": (_i, [_vp]),
    "clm_b200_tensor_bytes": (_u64, [_i, _u64]),
    "clm_b200_decode_tensor": (_i, [_vp, _i, _vp, _u64, _vp, _u64, _vp]),
    "clm_b200_encode": (_i, [_vp, _i, _vp, _u64, _vp, _vp]),
    "clm_b200_generate_weights": (_i, [_vp, _u64, _u32, _u64, _u64, _f, _vp, _vp]),
    "clm_b200_matrix_upload": (_i, [_vp, _i, _vp, _u64, _u32, _u32, C.POINTER(_vp)]),
    "clm_b200_matrix_upload_device": (_i, [_vp, _i, _vp, _u64, _u32, _u32, C.POINTER(_vp)]),
    "clm_b200_matrix_free": (_i, [_vp]),
    "clm_b200_matrix_info": (_i, [_vp, C.POINTER(_i), C.POINTER(_u32), C.POINTER(_u32), C.POINTER(_u64)]),
    "clm_b200_matmul_rows": (_i, [_vp, _vp, _vp, _u32, _vp, _vp]),
    "clm_b200_matmul_rows_static": (_i, [_vp, _vp, _vp, _u32, _vp, _vp]),
    "clm_b200_argmax_rows": (_i, [_vp, _vp, _u32, _u32, _vp, _vp]),
    "clm_b200_distribution_rows": (_i, [_vp, _vp, _u32, _u32, _f, _u32, _f, _vp, _vp]),
    "clm_b200_sample_rows": (_i, [_vp, _vp, _u32, _u32, _vp, _vp, _vp]),
    "clm_b200_verify_speculative": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _vp, _u64, _u64, _vp, _vp, _vp]),
    "clm_b200_accept_logits": (_i, [_vp, _vp, _vp, _vp, _u32, _u32, _u32, _f, _vp, _u64, _u64, _vp, _vp, _vp]),
    "clm_b200_philox_uniforms": (_i, [_vp, _u64, _u64, _u32, _u32, _u64, _vp, _vp]),
    "clm_b200_llama_create": (_i, [_vp, _vp, _vp, C.POINTER(_vp)]),
    "clm_b200_fixture_create": (_i, [_vp, _vp, _vp, C.POINTER(_vp)]),
    "clm_b200_engine_set_object": (_i, [_vp, C.c_char_p, _i, _vp, _u64]),
    "clm_b200_engine_destroy": (_i, [_vp]),
    "clm_b200_engine_generate_weights": (_i, [_vp, _u64, _f]),
    "clm_b200_engine_prepare": (_i, [_vp]),
    "clm_b200_engine_info": (_i, [_vp, C.POINTER(_u64), C.POINTER(_u64), C.POINTER(_u32)]),
    "clm_b200_session_open": (_i, [_vp, _u64]),
    "clm_b200_session_close": (_i, [_vp, _u64]),
    "clm_b200_run_window": (_i, [_vp, _u64, _u64, _u32, _vp, _vp, _vp, _vp]),
    "clm_b200_run_window_device": (_i, [_vp, _u64, _u64, _u32, _vp, _vp, _vp, _vp, _vp]),
    "clm_b200_commit": (_i, [_vp, _u64, _u32]),
    "clm_b200_run_tree_window": (_i, [_vp, _u64, _u64, _u32, _vp, _vp, _vp, _vp, _vp]),
    "clm_b200_run_batch_window": (_i, [_vp, _u32, _vp, _vp, _u32, _vp, _vp, _vp]),
    "clm_b200_run_batch_window_device": (_i, [_vp, _u32, _vp, _vp, _u32, _vp, _vp, _vp, _vp, _vp]),
    "clm_b200_llama_load_tensors": (_i, [_vp, _vp, _u32]),
    "clm_b200_commit_path": (_i, [_vp, _u64, _vp, _u32]),
    "clm_b200_run_tree_window_device": (_i, [_vp, _u64, _u64, _u32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "clm_b200_abort": (_i, [_vp, _u64]),
    "clm_b200_session_position": (_i, [_vp, _u64, C.POINTER(_u64)]),
    "clm_b200_engine_last_launches": (_i, [_vp, C.POINTER(_u64)]),
    "clm_b200_mtp_draft": (_i, [_vp, C.c_int32, _u32, _f, _u64, _u64, _vp, _vp]),
    "clm_b200_mtp_propose": (_i, [_vp, C.c_int32, _u32, _f, _u32, _f, _vp, _vp, _vp]),
    "clm_b200_shard_stats": (_i, [_vp, _vp, _u32, _u32, _u64, _f, _vp, _vp, _vp]),
    "clm_b200_shard_combine": (_i, [_vp, _vp, _vp, _u32, _vp, _u32, _u32, _f, _vp, _vp, _vp]),
    "clm_b200_shard_probs": (_i, [_vp, _vp, _u32, _u32, _f, _vp, _vp, _vp, _vp]),
    "clm_b200_spec_begin": (_i, [_vp, _u64, _vp, _u32, _vp]),
    "clm_b200_spec_round": (_i, [_vp, _u64, _vp, _vp, _vp]),
    "clm_b200_spec_round_device": (_i, [_vp, _u64, _vp, _vp, _vp, _vp]),
    "clm_b200_link_create": (_i, [_vp, _i, _u32, _u64, C.c_double, C.POINTER(_vp)]),
    "clm_b200_link_export": (_i, [_vp, _vp]),
    "clm_b200_link_connect": (_i, [_vp, _vp]),
    "clm_b200_link_destroy": (_i, [_vp]),
    "clm_b200_pipe_attach": (_i, [_vp, _vp, _vp]),
    "clm_b200_pipe_prefill": (_i, [_vp, _u64, _vp, _u32, _vp]),
    "clm_b200_pipe_begin": (_i, [_vp, _u64, _u32, _vp, _vp]),
    "clm_b200_pipe_round": (_i, [_vp, _u64, _vp, _vp, _vp, _vp]),
    "clm_b200_pipe_status": (_i, [_vp, _vp]),
    "clm_b200_pipe_attach_session": (_i, [_vp, _u64, _vp, _vp]),
}
LINK_HANDLE_BYTES = 128  # CLM_B200_LINK_HANDLE_BYTES


def _bind():
    for name, (res, args) in _SIGS.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


_bind()


def check(status: int) -> None:
    if status != 0:
        raise ClmError(status, lib.clm_b200_last_error().decode(errors="replace"))


def call(name: str, *args) -> None:
    check(getattr(lib, name)(*args))


def exported_symbols() -> list[str]:
    return list(_SIGS)
