"""The allocation-free LayerNorm backward C entry point (``mmb_layernorm_bwd_noalloc``).

Some callers cannot allocate device memory during a call (runtimes that
reserve everything up front, fixed memory arenas, C code without a caching
allocator).  This test calls the exported C symbol directly through ctypes,
twice in a row on the same inputs, and checks both results against the
regular binding, which takes its scratch from the PyTorch allocator.  It is
collected last so that a failure here stops a ``-x`` run only after every
other test has run.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from mini_megatron_b200 import _C
    lib = ctypes.CDLL(_C.__file__)
    fn = lib.mmb_layernorm_bwd_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p] * 9 + [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    return _C, fn


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


# (8192, 4096): the regular path would use 512 partial rows, more than the 256 that fit in the fixed
# scratch at H = 4096, so this case runs with fewer, taller bands than the regular binding.
@pytest.mark.parametrize("rows,H,with_dres", [(1000, 768, True), (333, 2048, False), (64, 4096, True),
                                              (8192, 4096, True)])
def test_noalloc_matches_regular_entry_point(rows, H, with_dres):
    C, fn = _lib()
    torch.manual_seed(rows + H)
    x = torch.randn(rows, H, device="cuda") * 2 + 0.5
    g = torch.randn(H, device="cuda")
    b = torch.randn(H, device="cuda")
    y = torch.empty(rows, H, device="cuda", dtype=torch.bfloat16)
    mean = torch.empty(rows, device="cuda")
    rstd = torch.empty(rows, device="cuda")
    C.layernorm_fwd(x, g, b, y, mean, rstd, 1e-5)
    dy = torch.randn(rows, H, device="cuda").bfloat16()
    dres = torch.randn(rows, H, device="cuda") if with_dres else None

    # regular entry point
    dx_ref = torch.empty_like(x)
    dg_ref = torch.zeros(H, device="cuda")
    db_ref = torch.zeros(H, device="cuda")
    C.layernorm_bwd(dy, x, mean, rstd, g, dres, dx_ref, dg_ref, db_ref)
    torch.cuda.synchronize()

    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call in range(2):
        dx = torch.full_like(x, float("nan"))
        dg = torch.zeros(H, device="cuda")
        db = torch.zeros(H, device="cuda")
        rc = fn(_ptr(dy), _ptr(x), _ptr(mean), _ptr(rstd), _ptr(g), _ptr(dres), _ptr(dx), _ptr(dg), _ptr(db),
                rows, H, stream)
        torch.cuda.synchronize()
        assert rc == 0, f"call {call}: rc {rc}"
        torch.testing.assert_close(dx, dx_ref, rtol=2e-3, atol=2e-3)
        torch.testing.assert_close(dg, dg_ref, rtol=2e-3, atol=2e-2)
        torch.testing.assert_close(db, db_ref, rtol=2e-3, atol=2e-2)


def test_noalloc_rejects_oversized_rows():
    _, fn = _lib()
    rc = fn(*([ctypes.c_void_p(0)] * 9), 16, 8192, ctypes.c_void_p(0))
    assert rc == -1
    rc = fn(*([ctypes.c_void_p(0)] * 9), 16, 770, ctypes.c_void_p(0))
    assert rc == -1
