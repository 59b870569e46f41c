"""clm_b200_matmul_rows_static (scratch in a fixed device array, no allocation) against clm_b200_matmul_rows.

Both entry points run the same kernels with the same plan, so the results are expected to be bitwise equal; the
assertion allows 1e-6 relative / 1e-6 absolute.  Called through the C ABI with ctypes.  The file name sorts last so
that the test also runs after every other GPU test of a session (and it passes alone in a fresh process).
"""
import ctypes as C

import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-6
ATOL = 1e-6
CLM_RESOURCE_EXHAUSTED = 6


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _static(ctx, m, x, y):
    from clusterlm_b200 import _native

    return _native.lib.clm_b200_matmul_rows_static(ctx.h, m.h, _ptr(x), x.shape[0], _ptr(y), None)


def _matrix(ctx, quant, rows, cols, seed):
    import torch

    from clusterlm_b200.runtime import Matrix, encode

    g = torch.Generator(device="cuda").manual_seed(seed)
    w = torch.randn((rows * cols,), generator=g, device="cuda", dtype=torch.float32) * 0.05
    return Matrix(ctx, quant, encode(ctx, quant, w), rows, cols)


@pytest.mark.parametrize("quant,rows,cols", [("q4_k", 4096, 4096), ("q8_0", 1024, 2048), ("q4_k", 14336, 512)])
def test_static_scratch_matches_matmul_rows_twice(ctx, quant, rows, cols):
    import torch

    from clusterlm_b200 import _native

    m = _matrix(ctx, quant, rows, cols, seed=rows + cols)
    gen = torch.Generator(device="cuda").manual_seed(7)
    for call, q in enumerate((4, 13)):  # two calls in a row, different widths (NT = 1, then 2)
        x = torch.randn((q, cols), generator=gen, device="cuda", dtype=torch.float32)
        y_ref = torch.full((q, rows), float("nan"), device="cuda")
        y = torch.full((q, rows), float("nan"), device="cuda")
        assert _native.lib.clm_b200_matmul_rows(ctx.h, m.h, _ptr(x), q, _ptr(y_ref), None) == 0
        rc = _static(ctx, m, x, y)
        assert rc == 0, _native.lib.clm_b200_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(y, y_ref, rtol=RTOL, atol=ATOL, msg=f"call {call}")
    m.close()


def test_static_scratch_rejects_oversize_then_still_works(ctx):
    import torch

    from clusterlm_b200 import _native
    from clusterlm_b200.runtime import Matrix

    rows, cols = 131072, 256  # 1024 row groups: 16 positions need 8 MiB of partials
    m = Matrix(ctx, "q4_k", torch.zeros(rows * cols // 256 * 144, dtype=torch.uint8, device="cuda"), rows, cols)
    x16 = torch.ones((16, cols), device="cuda")
    y16 = torch.empty((16, rows), device="cuda")
    assert _static(ctx, m, x16, y16) == CLM_RESOURCE_EXHAUSTED
    assert b"static scratch" in _native.lib.clm_b200_last_error()
    x1 = torch.ones((1, cols), device="cuda")
    y1 = torch.full((1, rows), float("nan"), device="cuda")
    assert _static(ctx, m, x1, y1) == 0
    torch.cuda.synchronize()
    assert torch.count_nonzero(y1).item() == 0  # all-zero weights
    m.close()
