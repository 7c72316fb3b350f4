"""ec_linear_int8_noalloc (fixed static scratch, no device allocation) against
the allocating ec_linear_int8 entry point, both called through the C ABI.
Named so that it is collected after every other test file; it also passes
alone."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH = 4 << 20


def _lib():
    import edgecore_b200 as ec
    lib = ctypes.CDLL(str(ec.LIB_PATH))
    vp, i = ctypes.c_void_p, ctypes.c_int
    lib.ec_linear_int8_noalloc.argtypes = [vp, vp, vp, vp, vp, i, i, i, vp]
    lib.ec_linear_int8_noalloc.restype = i
    lib.ec_linear_int8.argtypes = [vp, vp, vp, vp, vp, i, i, i]
    lib.ec_linear_int8.restype = i
    lib.ec_last_error.restype = ctypes.c_char_p
    return lib


def _case(rng, M, K, N, with_bias):
    X = (rng.standard_normal((M, K)) * rng.uniform(0.1, 4.0, (M, 1))).astype(np.float32)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    ws = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32) if with_bias else None
    return X, W, ws, b


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def test_noalloc_matches_allocating_entry_point(built, cuda):
    import torch
    lib = _lib()
    rng = np.random.default_rng(7)
    # two calls in a row through the same static scratch: the GEMV path
    # (M <= 8) then the GEMM path, the second larger than the first
    for M, K, N, with_bias in ((5, 896, 1152, True), (40, 4864, 896, False)):
        X, W, ws, b = _case(rng, M, K, N, with_bias)
        dX, dW, dws = (torch.from_numpy(a).cuda() for a in (X, W, ws))
        db = torch.from_numpy(b).cuda() if b is not None else None
        out = torch.full((M, N), float("nan"), device="cuda")
        rc = lib.ec_linear_int8_noalloc(_ptr(out), _ptr(dX), _ptr(dW), _ptr(dws), _ptr(db), M, K, N, None)
        assert rc == 0, lib.ec_last_error()
        torch.cuda.synchronize()
        want = np.zeros((M, N), np.float32)
        rc = lib.ec_linear_int8(want.ctypes.data, X.ctypes.data, W.ctypes.data, ws.ctypes.data,
                                b.ctypes.data if b is not None else None, M, K, N)
        assert rc == 0
        got = out.cpu().numpy()
        # same quantisation and the same exact int32 dots: tolerance 1e-6 of max
        assert np.abs(got - want).max() <= 1e-6 * np.abs(want).max()


def test_noalloc_rejects_oversize_and_host_pointers(built, cuda):
    import torch
    lib = _lib()
    K, N = 4864, 64
    M = SCRATCH // K + 1          # one row more than the scratch holds
    dummy = torch.zeros(16, device="cuda")
    p = _ptr(dummy)
    assert lib.ec_linear_int8_noalloc(p, p, p, p, None, M, K, N, None) == -1
    assert b"scratch" in lib.ec_last_error()
    assert lib.ec_linear_int8_noalloc(p, p, p, p, None, 4, 100, N, None) == -1   # K not a multiple of 16
    host = np.zeros(16, np.float32)
    assert lib.ec_linear_int8_noalloc(host.ctypes.data, p, p, p, None, 4, 64, N, None) == -1
    assert b"device memory" in lib.ec_last_error()
