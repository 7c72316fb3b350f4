"""GPU parity of the standalone entry points through the C ABI.

int8 paths (activation quantisation, gemm_int8, the W8A8 linear) must be
BIT-EXACT with the reference (golden vectors) and with the CPU restatement.
fp16/bf16 GEMMs accumulate in a different order than the reference's 8-lane
AVX2 loop: tolerance 1e-3 relative to the row's max |value| (fp32-accumulate
bar of the spec); observed errors are ~1e-6.
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec

pytestmark = pytest.mark.gpu

TOL_FP32_ACC = 1e-3


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


def rel_err(a, b):
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def eco(built, cuda):
    from oracle.oracle import Restatement
    return Restatement()


def test_quantize_rows_bit_exact(eco, golden):
    g = golden("ops.npz")
    for i in range(5):
        q, s = ec.quantize_rows(g[f"lin{i}_X"])
        assert np.array_equal(q, g[f"lin{i}_q"]), i
        assert np.array_equal(bits(s), bits(g[f"lin{i}_qs"])), i


def test_linear_int8_bit_exact(eco, golden):
    """M in {1,2,3,8,17}, K in {29,40,48,64,96}: GEMV and GEMM paths, ragged K."""
    g = golden("ops.npz")
    for i in range(5):
        b = g[f"lin{i}_b"] if f"lin{i}_b" in g else None
        y = ec.linear_int8(g[f"lin{i}_X"], g[f"lin{i}_W"], g[f"lin{i}_ws"], b)
        assert np.array_equal(bits(y), bits(g[f"lin{i}_y"])), i


def test_gemm_int8_bit_exact(eco, golden):
    g = golden("ops.npz")
    assert np.array_equal(bits(ec.gemm_int8(g["gi8_A"], g["gi8_as"], g["gi8_B"])), bits(g["gi8_y_noscale"]))
    assert np.array_equal(bits(ec.gemm_int8(g["gi8_A"], g["gi8_as"], g["gi8_B"], g["gi8_bs"])), bits(g["gi8_y"]))


@pytest.mark.parametrize("K", [64, 29])
def test_gemm_fp16_bf16(eco, golden, K):
    g = golden("ops.npz")
    X = g[f"g16_{K}_X"]
    assert rel_err(ec.gemm_fp16_fp32(X, g[f"g16_{K}_W"]), g[f"g16_{K}_y"]) < TOL_FP32_ACC
    assert rel_err(ec.gemm_bf16_fp32(X, g[f"gbf_{K}_W"]), g[f"gbf_{K}_y"]) < TOL_FP32_ACC


def test_device_pointers_zero_copy(eco, cuda):
    torch = cuda
    rng = np.random.default_rng(1)
    A = rng.integers(-128, 128, (3, 96), dtype=np.int64).astype(np.int8)
    B = rng.integers(-127, 128, (50, 96), dtype=np.int64).astype(np.int8)
    asc = rng.uniform(0.01, 0.1, 3).astype(np.float32)
    bs = rng.uniform(0.01, 0.1, 50).astype(np.float32)
    want = eco.gemm_int8(A, asc, B, bs)
    dA, dB = torch.from_numpy(A).cuda(), torch.from_numpy(B).cuda()
    das, dbs = torch.from_numpy(asc).cuda(), torch.from_numpy(bs).cuda()
    out = torch.empty((3, 50), dtype=torch.float32, device="cuda")
    ec.gemm_int8(dA, das, dB, dbs, out=out)
    assert np.array_equal(bits(out.cpu().numpy()), bits(want))
    X = torch.randn(2, 96, device="cuda")
    W16 = (torch.randn(50, 96, device="cuda") * 0.05).half()
    o16 = torch.empty((2, 50), device="cuda")
    ec.gemm_fp16_fp32(X, W16.view(torch.int16), out=o16)
    ref = eco.gemm_fp16(X.cpu().numpy(), W16.cpu().numpy().view(np.uint16))
    assert rel_err(o16.cpu().numpy(), ref) < TOL_FP32_ACC


QWEN05_SHAPES = [(1152, 896), (896, 896), (4864, 896), (896, 4864), (151936, 896)]


@pytest.mark.parametrize("M", [1, 8, 64, 512])
@pytest.mark.parametrize("NK", QWEN05_SHAPES, ids=lambda t: f"{t[0]}x{t[1]}")
def test_operator_sweep_int8(eco, cuda, M, NK):
    """The BASELINE operator sweep at full size.  Output rows are independent,
    so 300 sampled rows (plus the first and last) are checked bit-exact against
    the restatement; the GPU computes the full matrix."""
    torch = cuda
    N, K = NK
    rng = np.random.default_rng(M * 7 + N)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
    s = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ec.linear_int8(torch.from_numpy(X).cuda(), torch.from_numpy(W).cuda(), torch.from_numpy(s).cuda(), out=out)
    y = out.cpu().numpy()
    rows = np.unique(np.concatenate([[0, N - 1], rng.choice(N, min(N, 300), replace=False)]))
    want = eco.linear_int8(X, W[rows], s[rows])
    assert np.array_equal(bits(y[:, rows]), bits(want))


@pytest.mark.parametrize("M", [1, 8, 64])
def test_lm_head_fp16_sweep(eco, cuda, M):
    torch = cuda
    N, K = 151936, 896
    rng = np.random.default_rng(M)
    X = rng.standard_normal((M, K), dtype=np.float32)
    W = (rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float16)
    out = torch.empty((M, N), device="cuda")
    ec.gemm_fp16_fp32(torch.from_numpy(X).cuda(), torch.from_numpy(W.view(np.int16)).cuda(), out=out)
    y = out.cpu().numpy()
    rows = np.unique(np.concatenate([[0, N - 1], rng.choice(N, 300, replace=False)]))
    want = eco.gemm_fp16(X, W[rows].view(np.uint16))
    assert rel_err(y[:, rows], want) < TOL_FP32_ACC


@pytest.mark.parametrize("M", [1, 2, 3, 5, 8])
@pytest.mark.parametrize("K", [160, 896, 4864])
def test_gemm_async_device(eco, cuda, M, K):
    """ec_gemm_async (device operands, no host sync) over the weight-streaming
    GEMV shapes: int8 bit-exact with the restatement, fp16 / bf16 within the
    fp32-accumulate bar; N = 1001 leaves a ragged last row group."""
    torch = cuda
    N = 1001
    rng = np.random.default_rng(M * 31 + K)
    A = rng.integers(-128, 128, (M, K), dtype=np.int64).astype(np.int8)
    asc = rng.uniform(1e-3, 2e-2, M).astype(np.float32)
    W = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
    ws = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    dev = [torch.from_numpy(t).cuda() for t in (A, asc, W, ws, b)]
    out = torch.full((M, N), float("nan"), device="cuda")
    ec.gemm_async(0, out, dev[0], dev[1], dev[2], dev[3], dev[4])
    assert ec.device_error_take() == 0
    assert np.array_equal(bits(out.cpu().numpy()), bits(eco.gemm_int8(A, asc, W, ws, b)))
    X = rng.standard_normal((M, K), dtype=np.float32)
    W16 = (rng.standard_normal((N, K), dtype=np.float32) * 0.05).astype(np.float16)
    o16 = torch.full((M, N), float("nan"), device="cuda")
    ec.gemm_async(1, o16, torch.from_numpy(X).cuda(), None, torch.from_numpy(W16.view(np.int16)).cuda())
    assert ec.device_error_take() == 0
    assert rel_err(o16.cpu().numpy(), eco.gemm_fp16(X, W16.view(np.uint16))) < TOL_FP32_ACC
    Wb = (rng.standard_normal((N, K), dtype=np.float32) * 0.05).view(np.uint32) >> 16
    Wb = Wb.astype(np.uint16)
    ob = torch.full((M, N), float("nan"), device="cuda")
    ec.gemm_async(2, ob, torch.from_numpy(X).cuda(), None, torch.from_numpy(Wb.view(np.int16)).cuda())
    assert ec.device_error_take() == 0
    assert rel_err(ob.cpu().numpy(), eco.gemm_bf16(X, Wb)) < TOL_FP32_ACC


@pytest.mark.parametrize("M", [1, 4])
def test_gemv_row_result_independent_of_position(eco, cuda, M):
    """A row's fp16 dot is the same bits whichever warp, group slot or launch
    computes it: shifting the rows by one (a different slot of every row
    group) or restricting them to a shard leaves every output bit unchanged."""
    torch = cuda
    N, K = 4099, 896
    rng = np.random.default_rng(5 + M)
    X = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda()
    W = torch.from_numpy((rng.standard_normal((N, K), dtype=np.float32) * 0.05).astype(np.float16).view(np.int16)).cuda()
    full = torch.empty((M, N), device="cuda")
    ec.gemm_async(1, full, X, None, W)
    shifted = torch.empty((M, N - 1), device="cuda")
    ec.gemm_async(1, shifted, X, None, W[1:].contiguous())
    shard = torch.empty((M, 1000), device="cuda")
    ec.gemm_async(1, shard, X, None, W[2000:3000].contiguous())
    assert ec.device_error_take() == 0
    f = full.cpu().numpy()
    assert np.array_equal(bits(f[:, 1:]), bits(shifted.cpu().numpy()))
    assert np.array_equal(bits(f[:, 2000:3000]), bits(shard.cpu().numpy()))


def test_device_expf_tanhf_match_host_libm(eco, cuda):
    """The kernels' expf / tanhf (GELU, SiLU, softmax) round exactly as the
    host C library the reference calls: every 256th float bit pattern
    (2^24 inputs) plus the specials, compared bit for bit (NaN as NaN)."""
    torch = cuda
    pat = np.arange(0, 1 << 32, 256, dtype=np.uint64).astype(np.uint32) + np.uint32(77)
    extra = np.array([0x00000000, 0x80000000, 0x7f800000, 0xff800000, 0x7fc00000, 0x42b17217, 0x42b17218,
                      0xc2cff1b4, 0xc2cff1b5, 0x3f800000, 0xbf800000, 0x41b00000, 0x41b00001, 0x24000000,
                      0x23ffffff, 0x3eb17218, 0x3f851592], np.uint32)
    x = np.concatenate([pat, extra]).view(np.float32)
    want_e, want_t = eco.libm(x)
    d_x = torch.from_numpy(x).cuda()
    d_e, d_t = torch.empty_like(d_x), torch.empty_like(d_x)
    ec.reference_math(d_x, d_e, d_t)
    torch.cuda.synchronize()
    for got, want, name in ((d_e.cpu().numpy(), want_e, "expf"), (d_t.cpu().numpy(), want_t, "tanhf")):
        same = (bits(got) == bits(want)) | (np.isnan(got) & np.isnan(want))
        bad = np.flatnonzero(~same)
        assert bad.size == 0, (name, [hex(int(v)) for v in x[bad[:5]].view(np.uint32)])
