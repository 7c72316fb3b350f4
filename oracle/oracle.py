"""ctypes access to the CPU checkers -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
legs import this module.  Two checkers are exposed through one interface:

* ``Restatement`` -- oracle/libecoracle.so, our C restatement (ec_oracle.c);
* ``Reference``   -- oracle/_ref/libecref.so, the reference's own src/*.c
  compiled by oracle/Makefile (present where the reference was built).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
# The reference checkout: $EDGECORE_REFERENCE when set, else a sibling of the repo.
REF_DIR = Path(os.environ.get("EDGECORE_REFERENCE", str(HERE.parent.parent / "reference")))

_i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
_f64p = np.ctypeslib.ndpointer(np.float64, flags="C_CONTIGUOUS")
_i8p = np.ctypeslib.ndpointer(np.int8, flags="C_CONTIGUOUS")
_u16p = np.ctypeslib.ndpointer(np.uint16, flags="C_CONTIGUOUS")


def build(reference: bool = True) -> None:
    """Build the restatement, and the reference where its sources exist."""
    targets = ["all"] + (["ref"] if reference and (REF_DIR / "src" / "gpt2.c").exists() else [])
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={REF_DIR}", *targets], check=True)


def _opt(p):
    return None if p is None else p


def _as(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


class _Lib:
    def __init__(self, path: Path):
        if not path.exists():
            raise FileNotFoundError(f"{path} is not built (run `make -C oracle`)")
        self.lib = C.CDLL(str(path))


class Restatement(_Lib):
    """oracle/libecoracle.so: the reference's algorithm in our own C, calling
    the host libm's expf / tanhf as the reference does."""

    def __init__(self):
        super().__init__(HERE / "libecoracle.so")
        L = self.lib
        L.eco_open.restype = C.c_void_p
        L.eco_open.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.eco_close.argtypes = [C.c_void_p]
        L.eco_info.argtypes = [C.c_void_p, _i32p]
        L.eco_reset_kv.argtypes = [C.c_void_p]
        L.eco_forward.argtypes = [C.c_void_p, _i32p, _i32p, C.c_void_p, C.c_int, _f32p]
        L.eco_set_taps.argtypes = [C.c_void_p, C.c_int]
        L.eco_get_taps.restype = C.POINTER(C.c_float)
        L.eco_get_taps.argtypes = [C.c_void_p]
        L.eco_quantize_rows.argtypes = [_i8p, _f32p, _f32p, C.c_int, C.c_int]
        L.eco_gemm_int8.argtypes = [_f32p, _i8p, _f32p, _i8p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.eco_gemm_fp16.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int]
        L.eco_gemm_bf16.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int]
        L.eco_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_double]
        L.eco_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_double]
        L.eco_rope_inv_freq.argtypes = [_f64p, C.c_int, C.c_double, C.c_int, C.c_double, C.c_double]
        L.eco_rope_cos_sin.argtypes = [_f64p, _f64p, _f64p, C.c_int, C.c_int, C.c_double]
        L.eco_libm.argtypes = [_f32p, _f32p, _f32p, C.c_int]

    # ---- ops ----
    def libm(self, x):
        """(expf(x), tanhf(x)) from this library's libm, element-wise."""
        x = _as(x, np.float32).ravel()
        e, t = np.empty_like(x), np.empty_like(x)
        self.lib.eco_libm(x, e, t, x.size)
        return e, t

    def quantize_rows(self, x):
        x = _as(x, np.float32)
        M, K = x.shape
        q = np.empty((M, K), np.int8)
        s = np.empty(M, np.float32)
        self.lib.eco_quantize_rows(q, s, x, M, K)
        return q, s

    def gemm_int8(self, A, a_scale, B, b_scale=None, bias=None):
        A, B = _as(A, np.int8), _as(B, np.int8)
        M, K = A.shape
        N = B.shape[0]
        out = np.empty((M, N), np.float32)
        bs, bb = _as(b_scale, np.float32), _as(bias, np.float32)
        self.lib.eco_gemm_int8(out, A, _as(a_scale, np.float32), B,
                               None if bs is None else bs.ctypes.data,
                               None if bb is None else bb.ctypes.data, M, K, N)
        return out

    def gemm_fp16(self, A, B16):
        A, B16 = _as(A, np.float32), np.ascontiguousarray(B16).view(np.uint16)
        M, K = A.shape
        out = np.empty((M, B16.shape[0]), np.float32)
        self.lib.eco_gemm_fp16(out, A, B16, M, K, B16.shape[0])
        return out

    def gemm_bf16(self, A, B16):
        A, B16 = _as(A, np.float32), np.ascontiguousarray(B16).view(np.uint16)
        M, K = A.shape
        out = np.empty((M, B16.shape[0]), np.float32)
        self.lib.eco_gemm_bf16(out, A, B16, M, K, B16.shape[0])
        return out

    def linear_int8(self, X, W, w_scale, bias=None):
        q, s = self.quantize_rows(X)
        return self.gemm_int8(q, s, W, w_scale, bias)

    def layernorm(self, x, g, b, eps):
        x = _as(x, np.float32)
        out = np.empty_like(x)
        self.lib.eco_layernorm(out, x, _as(g, np.float32), _as(b, np.float32), x.shape[0], x.shape[1], eps)
        return out

    def rmsnorm(self, x, g, eps):
        x = _as(x, np.float32)
        out = np.empty_like(x)
        self.lib.eco_rmsnorm(out, x, _as(g, np.float32), x.shape[0], x.shape[1], eps)
        return out

    def rope_table(self, half, positions, theta, rope_type=0, yarn_factor=1.0, yarn_orig_max=0.0, scale=1.0):
        inv = np.empty(half, np.float64)
        self.lib.eco_rope_inv_freq(inv, half, theta, rope_type, yarn_factor, yarn_orig_max)
        cs = np.empty((len(positions), half), np.float64)
        sn = np.empty((len(positions), half), np.float64)
        for i, p in enumerate(positions):
            c, s = np.empty(half), np.empty(half)
            self.lib.eco_rope_cos_sin(c, s, inv, half, int(p), scale)
            cs[i], sn[i] = c, s
        return inv, cs, sn

    # ---- model ----
    def open(self, path, batch_cap=1, max_ctx=0):
        return Model(self, path, batch_cap, max_ctx, "eco")


class Reference(_Lib):
    """oracle/_ref/libecref.so (the reference, built from its sources)."""

    def __init__(self, threads: int | None = None):
        super().__init__(HERE / "_ref" / "libecref.so")
        L = self.lib
        L.ref_open.restype = C.c_void_p
        L.ref_open.argtypes = [C.c_char_p, C.c_int, C.c_int]
        L.ref_close.argtypes = [C.c_void_p]
        L.ref_info.argtypes = [C.c_void_p, _i32p]
        L.ref_reset_kv.argtypes = [C.c_void_p]
        L.ref_forward.argtypes = [C.c_void_p, _i32p, _i32p, C.c_void_p, C.c_int, _f32p]
        L.ref_forward_layers.argtypes = [C.c_void_p, C.c_int, _i32p, _i32p, C.c_void_p, C.c_int, _f32p, _f32p]
        L.ref_linear.argtypes = [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, _f32p, _f32p,
                                 C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p]
        L.ref_layernorm.argtypes = [_f32p, _f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_double]
        L.ref_rmsnorm.argtypes = [_f32p, _f32p, _f32p, C.c_int, C.c_int, C.c_double]
        L.ref_rope.argtypes = [_f64p, _f64p, _f64p, C.c_int, C.c_int, C.c_double, C.c_int,
                               C.c_double, C.c_double, C.c_double]
        L.ref_gelu.restype = C.c_float
        L.ref_gelu.argtypes = [C.c_float]
        L.ref_silu.restype = C.c_float
        L.ref_silu.argtypes = [C.c_float]
        L.ref_f32_to_fp16.restype = C.c_uint16
        L.ref_f32_to_fp16.argtypes = [C.c_float]
        L.ref_set_threads.argtypes = [C.c_int]
        L.gemm_int8.argtypes = [_f32p, _i8p, _f32p, _i8p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.gemm_fp16_fp32.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int]
        L.gemm_bf16_fp32.argtypes = [_f32p, _f32p, _u16p, C.c_int, C.c_int, C.c_int]
        self.set_threads(threads or len(os.sched_getaffinity(0)))

    def set_threads(self, n: int) -> None:
        self.threads = n
        self.lib.ref_set_threads(n)

    def linear(self, precision, W, x, scale=None, bias=None):
        """Reference linear(); returns (out, q, qs) (q/qs only for int8)."""
        x = _as(x, np.float32)
        M, K = x.shape
        W = np.ascontiguousarray(W)
        N = W.shape[0]
        out = np.empty((M, N), np.float32)
        sc, bb = _as(scale, np.float32), _as(bias, np.float32)
        q = np.empty((M, K), np.int8) if precision == 0 else None
        qs = np.empty(M, np.float32) if precision == 0 else None
        self.lib.ref_linear(precision, W.ctypes.data, None if sc is None else sc.ctypes.data,
                            None if bb is None else bb.ctypes.data, x, out, M, K, N,
                            None if q is None else q.ctypes.data, None if qs is None else qs.ctypes.data)
        return out, q, qs

    def gemm_int8(self, A, a_scale, B, b_scale=None, bias=None):
        A, B = _as(A, np.int8), _as(B, np.int8)
        M, K = A.shape
        N = B.shape[0]
        out = np.empty((M, N), np.float32)
        bs, bb = _as(b_scale, np.float32), _as(bias, np.float32)
        self.lib.gemm_int8(out, A, _as(a_scale, np.float32), B, None if bs is None else bs.ctypes.data,
                           None if bb is None else bb.ctypes.data, M, K, N)
        return out

    def gemm_fp16(self, A, B16):
        A, B16 = _as(A, np.float32), np.ascontiguousarray(B16).view(np.uint16)
        out = np.empty((A.shape[0], B16.shape[0]), np.float32)
        self.lib.gemm_fp16_fp32(out, A, B16, A.shape[0], A.shape[1], B16.shape[0])
        return out

    def gemm_bf16(self, A, B16):
        A, B16 = _as(A, np.float32), np.ascontiguousarray(B16).view(np.uint16)
        out = np.empty((A.shape[0], B16.shape[0]), np.float32)
        self.lib.gemm_bf16_fp32(out, A, B16, A.shape[0], A.shape[1], B16.shape[0])
        return out

    def layernorm(self, x, g, b, eps):
        x = _as(x, np.float32)
        out = np.empty_like(x)
        self.lib.ref_layernorm(out, x, _as(g, np.float32), _as(b, np.float32), x.shape[0], x.shape[1], eps)
        return out

    def rmsnorm(self, x, g, eps):
        x = _as(x, np.float32)
        out = np.empty_like(x)
        self.lib.ref_rmsnorm(out, x, _as(g, np.float32), x.shape[0], x.shape[1], eps)
        return out

    def rope_table(self, half, positions, theta, rope_type=0, yarn_factor=1.0, yarn_orig_max=0.0, scale=1.0):
        cs = np.empty((len(positions), half), np.float64)
        sn = np.empty((len(positions), half), np.float64)
        inv = np.empty(half, np.float64)
        for i, p in enumerate(positions):
            c, s = np.empty(half), np.empty(half)
            self.lib.ref_rope(inv, c, s, half, int(p), theta, rope_type, yarn_factor, yarn_orig_max, scale)
            cs[i], sn[i] = c, s
        return inv, cs, sn

    def open(self, path, batch_cap=1, max_ctx=0):
        return Model(self, path, batch_cap, max_ctx, "ref")


class Model:
    """A loaded model in one of the two checkers, with the reference call shape."""

    def __init__(self, owner, path, batch_cap, max_ctx, prefix):
        self.owner, self.lib, self.p = owner, owner.lib, prefix
        self.h = getattr(self.lib, f"{prefix}_open")(str(path).encode(), batch_cap, max_ctx)
        if not self.h:
            raise RuntimeError(f"{prefix}: failed to load {path}")
        info = np.zeros(16, np.int32)
        getattr(self.lib, f"{prefix}_info")(self.h, info)
        (self.arch, self.precision, self.n_layer, self.n_head, self.n_kv_head, self.n_embd,
         self.head_dim, self.intermediate, self.vocab, self.n_ctx, self.eff_ctx, self.batch_cap,
         self.n_kv_embd, self.tie) = [int(v) for v in info[:14]]

    def close(self):
        if self.h:
            getattr(self.lib, f"{self.p}_close")(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        getattr(self.lib, f"{self.p}_reset_kv")(self.h)

    def forward(self, tokens, positions, seqs=None):
        tokens = np.ascontiguousarray(tokens, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        M = len(tokens)
        logits = np.empty((M, self.vocab), np.float32)
        sq = None if seqs is None else np.ascontiguousarray(seqs, np.int32)
        getattr(self.lib, f"{self.p}_forward")(self.h, tokens, positions,
                                              None if sq is None else sq.ctypes.data, M, logits)
        return logits

    def forward_taps(self, tokens, positions, seqs=None):
        """Logits plus the residual stream after the embedding and every layer,
        [n_layer+1][M][n_embd].  For the reference this re-runs the prefill with
        the layer count truncated, resetting the KV cache before each run."""
        tokens = np.ascontiguousarray(tokens, np.int32)
        positions = np.ascontiguousarray(positions, np.int32)
        M = len(tokens)
        sq = None if seqs is None else np.ascontiguousarray(seqs, np.int32)
        sqp = None if sq is None else sq.ctypes.data
        taps = np.empty((self.n_layer + 1, M, self.n_embd), np.float32)
        logits = np.empty((M, self.vocab), np.float32)
        if self.p == "eco":
            self.lib.eco_set_taps(self.h, M)
            self.lib.eco_forward(self.h, tokens, positions, sqp, M, logits)
            ptr = self.lib.eco_get_taps(self.h)
            taps[:] = np.ctypeslib.as_array(ptr, shape=(taps.size,)).reshape(taps.shape)
            self.lib.eco_set_taps(self.h, 0)
            return logits, taps
        for nl in range(self.n_layer + 1):
            self.reset()
            out = np.empty((M, self.vocab), np.float32)
            self.lib.ref_forward_layers(self.h, nl, tokens, positions, sqp, M, out, taps[nl])
            if nl == self.n_layer:
                logits = out
        return logits, taps
