"""The int8 GEMM on tcgen05 tensor cores (M >= 32): bit-exact with the CPU
restatement of reference gemm_int8 / linear() over ragged shapes -- partial
128-row and 256-column tiles, K not a multiple of the 128-byte stage, K
padded to 16, biases and scales present or absent."""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec

pytestmark = pytest.mark.gpu

SHAPES = [(32, 8, 16), (33, 257, 80), (128, 256, 128), (129, 300, 1000), (300, 1152, 896),
          (512, 896, 4864), (64, 3, 3072), (1000, 4864, 896)]


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def eco(built, cuda):
    from oracle.oracle import Restatement
    return Restatement()


@pytest.mark.parametrize("MNK", SHAPES, ids=lambda t: "x".join(map(str, t)))
def test_gemm_int8_tensor_cores(eco, cuda, MNK):
    torch = cuda
    M, N, K = MNK
    rng = np.random.default_rng(M + 3 * N + 7 * K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int64).astype(np.int8)
    W = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
    a_s = rng.uniform(1e-3, 5e-2, M).astype(np.float32)
    w_s = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    bias = rng.standard_normal(N).astype(np.float32) if N % 2 else None
    dev = [torch.from_numpy(x).cuda() if x is not None else None for x in (A, a_s, W, w_s, bias)]
    out = torch.full((M, N), float("nan"), device="cuda")
    ec.gemm_int8(*dev, out=out)
    want = eco.gemm_int8(A, a_s, W, w_s, bias)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))


@pytest.mark.parametrize("MNK", SHAPES[1::2], ids=lambda t: "x".join(map(str, t)))
def test_linear_int8_tensor_cores(eco, cuda, MNK):
    torch = cuda
    M, N, K = MNK
    rng = np.random.default_rng(11 * M + N + K)
    X = (rng.standard_normal((M, K)) * rng.uniform(0.1, 3.0, (M, 1))).astype(np.float32)
    W = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
    w_s = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    out = torch.empty((M, N), device="cuda")
    ec.linear_int8(torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda(), torch.from_numpy(w_s).cuda(), out=out)
    want = eco.linear_int8(X, W, w_s)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))


F16_SHAPES = [(32, 8, 16), (33, 257, 80), (130, 300, 1000), (300, 1152, 896), (64, 151936, 896)]


@pytest.mark.parametrize("MNK", F16_SHAPES, ids=lambda t: "x".join(map(str, t)))
@pytest.mark.parametrize("wt", ["fp16", "bf16"])
def test_gemm_16bit_tensor_cores(eco, cuda, MNK, wt):
    """fp32 activations split into 16-bit parts (two fp16 after a power-of-two
    row scale, or three bf16): within 2e-5 of the fp32 dot -- the spec's bar
    for these paths is 1e-3.  Rows of very different magnitude check the
    per-row scaling."""
    torch = cuda
    M, N, K = MNK
    rng = np.random.default_rng(5 * M + N + 3 * K)
    X = (rng.standard_normal((M, K)) * np.exp(rng.uniform(-8, 8, (M, 1)))).astype(np.float32)
    W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
    if wt == "fp16":
        Wb = W.astype(np.float16).view(np.uint16)
        fn, ref = ec.gemm_fp16_fp32, eco.gemm_fp16
    else:
        Wb = (W.view(np.uint32) >> 16).astype(np.uint16)   # truncate to bf16 bits
        fn, ref = ec.gemm_bf16_fp32, eco.gemm_bf16
    out = torch.empty((M, N), device="cuda")
    fn(torch.from_numpy(X).cuda(), torch.from_numpy(Wb.view(np.int16)).cuda(), out=out)
    got = out.cpu().numpy()
    rows = np.unique(np.concatenate([[0, N - 1], rng.choice(N, min(N, 400), replace=False)]))
    want = ref(X, Wb[rows])
    err = np.abs(got[:, rows] - want).max(axis=1) / np.maximum(np.abs(want).max(axis=1), 1e-30)
    assert err.max() < 2e-5, err.max()
