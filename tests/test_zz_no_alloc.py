"""ec_linear_int8_noalloc -- the W8A8 linear for callers that cannot allocate
device memory per call (HBM handed to a caching allocator, or a decode loop
that must not wait on cudaMalloc's device synchronisation) -- checked
bit-exactly against the CPU oracle and the allocating ec_linear_int8 entry
point, through the C ABI.  Named so that it is collected after every other
test file; it also passes alone."""
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
    lib.ec_device_error_take.argtypes = [vp, ctypes.POINTER(ctypes.c_int)]
    lib.ec_device_error_take.restype = i
    return lib


def _case(rng, M, K, N, with_bias):
    X = (rng.standard_normal((M, K)) * rng.uniform(0.1, 4.0, (M, 1))).astype(np.float32)
    W = rng.integers(-127, 128, (N, K), dtype=np.int8)
    ws = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32) if with_bias else None
    return X, W, ws, b


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _check(lib, rng, M, K, N, with_bias):
    """One call of the no-allocation entry point on device operands, bit-exact
    against the CPU restatement of the reference's W8A8 linear and against
    the allocating ec_linear_int8 entry point on the same inputs."""
    import torch
    from oracle.oracle import Restatement
    X, W, ws, b = _case(rng, M, K, N, with_bias)
    dX, dW, dws = (torch.from_numpy(a).cuda() for a in (X, W, ws))
    db = torch.from_numpy(b).cuda() if b is not None else None
    out = torch.full((M, N), float("nan"), device="cuda")
    rc = lib.ec_linear_int8_noalloc(_ptr(out), _ptr(dX), _ptr(dW), _ptr(dws), _ptr(db), M, K, N, None)
    assert rc == 0, lib.ec_last_error()
    torch.cuda.synchronize()
    code = ctypes.c_int(-1)
    assert lib.ec_device_error_take(None, ctypes.byref(code)) == 0 and code.value == 0
    got = out.cpu().numpy()
    alloc = np.zeros((M, N), np.float32)
    rc = lib.ec_linear_int8(alloc.ctypes.data, X.ctypes.data, W.ctypes.data, ws.ctypes.data,
                            b.ctypes.data if b is not None else None, M, K, N)
    assert rc == 0
    want = Restatement().linear_int8(X, W, ws, b)
    # exact int32 dots and the same fp32 epilogue: bit-identical results
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"M={M} K={K} N={N} differs from the oracle"
    assert np.array_equal(got.view(np.uint32), alloc.view(np.uint32))


def test_noalloc_matches_oracle_and_allocating_entry_point(built, cuda):
    lib = _lib()
    rng = np.random.default_rng(7)
    # two calls in a row through the same static scratch: the GEMV path
    # (M <= 8) then the GEMM path, the second larger than the first
    for M, K, N, with_bias in ((5, 896, 1152, True), (40, 4864, 896, False)):
        _check(lib, rng, M, K, N, with_bias)


def test_noalloc_long_rows(built, cuda):
    """Rows too long for the GEMV's shared memory at M <= 8 go to the GEMM."""
    lib = _lib()
    rng = np.random.default_rng(11)
    for M, K, N in ((1, 262144, 48), (8, 32768, 40), (1, 110592, 24)):
        _check(lib, rng, M, K, N, True)


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
