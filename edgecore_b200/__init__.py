"""edgecore_b200 -- B200 (sm_100a) implementation of EdgeCore's inference hot path.

The product is the C library ``libedgecore_b200.so`` (include/edgecore.h and
include/edgecore_b200.h).  This package builds it (``build.py``), loads it with
ctypes, and mirrors the reference entry points for Python callers:

* ``gemm_int8``, ``gemm_fp16_fp32``, ``gemm_bf16_fp32`` -- reference
  src/kernels.c:129-168, on the GPU;
* ``Model`` -- ``gpt2_load`` / ``gpt2_forward`` / ``gpt2_free`` (reference
  src/gpt2.c:161-805) plus the greedy/device-resident extensions.

Arrays may be numpy arrays (host) or objects exposing ``data_ptr()`` (device
tensors); the library classifies each pointer.  There is no CPU fallback: if
the shared library is missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path
from typing import Any

import numpy as np

__all__ = ["load_library", "Model", "gemm_int8", "gemm_fp16_fp32", "gemm_bf16_fp32",
           "quantize_rows", "linear_int8", "gemm_async", "device_error_take", "attention_force_split", "reference_math", "argmax_key", "argmax_key_decode",
           "LIB_PATH"]

LIB_PATH = Path(__file__).resolve().parent / "libedgecore_b200.so"
_LIB: C.CDLL | None = None

_vp, _i, _f = C.c_void_p, C.c_int, C.c_float


def _declare(lib: C.CDLL) -> None:
    sig = {
        "ec_last_error": (C.c_char_p, []),
        "ec_version": (C.c_char_p, []),
        "ec_model_open": (_vp, [C.c_char_p, _i, _i]),
        "ec_model_close": (None, [_vp]),
        "ec_model_info": (_i, [_vp, _vp]),
        "ec_model_set_stream": (_i, [_vp, _vp]),
        "ec_forward_device": (_i, [_vp, _vp, _vp, _vp, _i, _vp]),
        "ec_forward_argmax": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp]),
        "ec_forward_shard_argmax": (_i, [_vp, _vp, _vp, _vp, _i, _vp, _vp]),
        "ec_decode_greedy": (_i, [_vp, _vp, _i, _i, _vp]),
        "ec_decode_profile": (_i, [_vp, _vp, _i, _i, _vp]),
        "ec_decode_greedy_cycle": (_i, [_vp, _vp, _i, _i, _i, _vp]),
        "ec_decode_trace": (_i, [_vp, _vp, _i, _i, _vp, _i]),
        "ec_decode_batch": (_i, [_vp, _vp, _vp, _i, _vp]),
        "ec_batch_hidden": (_i, [_vp, _vp, _vp, _i, _i, _vp]),
        "ec_lm_shard_keys": (_i, [_vp, _vp, _i, _vp]),
        "ec_keys_advance": (_i, [_vp, _vp, _i, _vp, _vp]),
        "ec_batch_graph_kernels": (_i, [_vp, _i]),
        "ec_model_packed": (C.c_longlong, [_vp, _i, _i, _vp, C.c_size_t, _vp]),
        "ec_kv_release": (_i, [_vp, _i]),
        "ec_kv_info": (_i, [_vp, _vp]),
        "ec_model_set_taps": (_i, [_vp, _i]),
        "ec_model_get_taps": (_i, [_vp, _vp, _i]),
        "ec_model_set_vocab_shard": (_i, [_vp, _i, _i]),
        "ec_argmax_key": (C.c_uint64, [_f, _i]),
        "ec_argmax_key_decode": (None, [C.c_uint64, _vp, _vp]),
        "ec_quantize_rows": (_i, [_vp, _vp, _vp, _i, _i]),
        "ec_linear_int8": (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
        "ec_gemm_async": (_i, [_i, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _vp]),
        "ec_device_error_take": (_i, [_vp, _vp]),
        "ec_attention_force_split": (_i, [_i]),
        "ec_reference_math": (_i, [_vp, _vp, _vp, _i, _vp]),
        "gemm_fp16_fp32": (None, [_vp, _vp, _vp, _i, _i, _i]),
        "gemm_bf16_fp32": (None, [_vp, _vp, _vp, _i, _i, _i]),
        "gemm_int8": (None, [_vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _i]),
        "gpt2_forward": (None, [_vp, _vp, _vp, _vp, _i, _vp]),
        "ecm_parse": (_i, [_vp, C.c_size_t, _vp, _i, _vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args


def load_library(path: str | os.PathLike | None = None) -> C.CDLL:
    """Load (once) and return the shared library; raise if it is not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise RuntimeError(f"{p} is not built; run `python -m edgecore_b200.build` "
                           "(there is no CPU fallback)")
    lib = C.CDLL(str(p))
    _declare(lib)
    _LIB = lib
    return lib


def last_error() -> str:
    return (load_library().ec_last_error() or b"").decode(errors="replace")


def _ptr(a: Any) -> int | None:
    """Address of a numpy array / device tensor / raw int (None stays None)."""
    if a is None:
        return None
    if isinstance(a, int):
        return a
    if hasattr(a, "data_ptr"):
        return int(a.data_ptr())
    if isinstance(a, np.ndarray):
        if not a.flags["C_CONTIGUOUS"]:
            raise ValueError("arrays passed to the C ABI must be C-contiguous")
        return a.ctypes.data
    raise TypeError(f"cannot pass {type(a)} to the C ABI")


def _np(a, dtype) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=dtype)


def _is_dev(a) -> bool:
    return hasattr(a, "data_ptr")


# ---- standalone GEMMs (reference src/kernels.c:129-168) ----------------------

def gemm_int8(A, a_scale, B, b_scale=None, bias=None, out=None):
    """C[m][n] = bias[n] + ((float)sum_k A[m][k]*B[n][k]) * a_scale[m] * b_scale[n]."""
    lib = load_library()
    if not _is_dev(A):
        A, a_scale = _np(A, np.int8), _np(a_scale, np.float32)
    if not _is_dev(B):
        B = _np(B, np.int8)
        b_scale = None if b_scale is None else _np(b_scale, np.float32)
        bias = None if bias is None else _np(bias, np.float32)
    M, K = A.shape
    N = B.shape[0]
    if out is None:
        out = np.empty((M, N), np.float32)
    lib.gemm_int8(_ptr(out), _ptr(A), _ptr(a_scale), _ptr(B), _ptr(b_scale), _ptr(bias), M, K, N)
    return out


def _gemm16(fn, A, B16, out):
    lib = load_library()
    if not _is_dev(A):
        A = _np(A, np.float32)
    if not _is_dev(B16):
        B16 = np.ascontiguousarray(B16).view(np.uint16)
    M, K = A.shape
    N = B16.shape[0]
    if out is None:
        out = np.empty((M, N), np.float32)
    getattr(lib, fn)(_ptr(out), _ptr(A), _ptr(B16), M, K, N)
    return out


def gemm_fp16_fp32(A, B16, out=None):
    """C[m][n] = sum_k A[m][k] * fp16(B[n][k]) with fp32 accumulation."""
    return _gemm16("gemm_fp16_fp32", A, B16, out)


def gemm_bf16_fp32(A, B16, out=None):
    """Same as gemm_fp16_fp32 with bfloat16 weights (uint16 bit patterns)."""
    return _gemm16("gemm_bf16_fp32", A, B16, out)


def gemm_async(wt: int, out, A, a_scale, B, b_scale=None, bias=None, stream=None) -> None:
    """gemm_int8 (wt 0) / gemm_fp16_fp32 (1) / gemm_bf16_fp32 (2) on device
    tensors, enqueued on `stream` (an int cudaStream_t or None) without a host
    synchronisation; errors inside kernels surface in device_error_take()."""
    lib = load_library()
    M, K = A.shape
    N = B.shape[0]
    if lib.ec_gemm_async(int(wt), _ptr(out), _ptr(A), _ptr(a_scale), _ptr(B), _ptr(b_scale), _ptr(bias),
                         M, K, N, stream):
        raise RuntimeError(last_error())


def reference_math(d_x, d_exp=None, d_tanh=None, stream=None) -> None:
    """The library's device expf / tanhf (restated host libm) on a device float tensor."""
    n = int(d_x.numel())
    if load_library().ec_reference_math(_ptr(d_x), _ptr(d_exp), _ptr(d_tanh), n, stream):
        raise RuntimeError(last_error())


def attention_force_split(on: bool) -> None:
    """Force (True) or release (False) the split attention kernels of the
    per-layer path, process-wide (tests and measurement)."""
    load_library().ec_attention_force_split(1 if on else 0)


def device_error_take(stream=None) -> int:
    """Synchronise `stream`, then read and clear the library's device error
    code (0 none, 1 a bounded wait gave up, 2 an out-of-range index)."""
    code = C.c_int(0)
    if load_library().ec_device_error_take(stream, C.byref(code)):
        raise RuntimeError(last_error())
    return code.value


def quantize_rows(X):
    """Per-row int8 activation quantisation (reference src/gpt2.c:446-461)."""
    lib = load_library()
    X = _np(X, np.float32)
    M, K = X.shape
    q = np.empty((M, K), np.int8)
    s = np.empty(M, np.float32)
    if lib.ec_quantize_rows(_ptr(q), _ptr(s), _ptr(X), M, K):
        raise RuntimeError(last_error())
    return q, s


def linear_int8(X, W, w_scale, bias=None, out=None):
    """The W8A8 linear of reference linear() (src/gpt2.c:437-462)."""
    lib = load_library()
    if not _is_dev(X):
        X = _np(X, np.float32)
    if not _is_dev(W):
        W, w_scale = _np(W, np.int8), _np(w_scale, np.float32)
        bias = None if bias is None else _np(bias, np.float32)
    M, K = X.shape
    N = W.shape[0]
    if out is None:
        out = np.empty((M, N), np.float32)
    if lib.ec_linear_int8(_ptr(out), _ptr(X), _ptr(W), _ptr(w_scale), _ptr(bias), M, K, N):
        raise RuntimeError(last_error())
    return out


def argmax_key(maxv: float, idx: int) -> int:
    return int(load_library().ec_argmax_key(float(maxv), int(idx)))


def argmax_key_decode(key: int) -> tuple[float, int]:
    v, i = C.c_float(), C.c_int()
    load_library().ec_argmax_key_decode(C.c_uint64(key), C.byref(v), C.byref(i))
    return v.value, i.value


# ---- model -------------------------------------------------------------------

class Model:
    """A model loaded on the current CUDA device (gpt2_load on a heap GPT2)."""

    INFO = ("arch", "precision", "n_layer", "n_head", "n_kv_head", "n_embd", "head_dim",
            "intermediate", "vocab", "n_ctx", "eff_ctx", "batch_cap", "n_kv_embd", "tie", "device")

    def __init__(self, path: str | os.PathLike, batch_cap: int = 1, max_ctx: int = 0):
        self.lib = load_library()
        self.h = self.lib.ec_model_open(str(path).encode(), int(batch_cap), int(max_ctx))
        if not self.h:
            raise RuntimeError(f"gpt2_load({path}) failed: {last_error()}")
        info = np.zeros(16, np.int32)
        self._check(self.lib.ec_model_info(self.h, info.ctypes.data))
        for k, v in zip(self.INFO, info):
            setattr(self, k, int(v))

    def _check(self, rc: int) -> None:
        if rc:
            raise RuntimeError(last_error())

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.ec_model_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, tokens, positions, seqs=None, out=None) -> np.ndarray:
        """gpt2_forward with host arrays: logits [M][vocab] fp32, written into
        `out` when given (a C-contiguous float32 [M][vocab] array, reused the
        way the reference runtime reuses its one logits buffer)."""
        t, p = _np(tokens, np.int32), _np(positions, np.int32)
        s = None if seqs is None else _np(seqs, np.int32)
        M = len(t)
        if out is None:
            out = np.empty((M, self.vocab), np.float32)
        elif out.dtype != np.float32 or not out.flags.c_contiguous or out.shape != (M, self.vocab):
            raise ValueError(f"out must be a C-contiguous float32 array of shape ({M}, {self.vocab})")
        self.lib.gpt2_forward(self.h, _ptr(t), _ptr(p), _ptr(s), M, _ptr(out))
        return out

    def forward_argmax(self, tokens, positions, seqs=None, shard: bool = False):
        t, p = _np(tokens, np.int32), _np(positions, np.int32)
        s = None if seqs is None else _np(seqs, np.int32)
        M = len(t)
        ids = np.empty(M, np.int32)
        mx = np.empty(M, np.float32)
        fn = self.lib.ec_forward_shard_argmax if shard else self.lib.ec_forward_argmax
        self._check(fn(self.h, _ptr(t), _ptr(p), _ptr(s), M, _ptr(ids), _ptr(mx)))
        return ids, mx

    def forward_taps(self, tokens, positions, seqs=None):
        """Logits plus residual taps [n_layer+1][M][n_embd]."""
        M = len(tokens)
        self._check(self.lib.ec_model_set_taps(self.h, M))
        try:
            logits = self.forward(tokens, positions, seqs)
            taps = np.empty((self.n_layer + 1, M, self.n_embd), np.float32)
            self._check(self.lib.ec_model_get_taps(self.h, _ptr(taps), M))
        finally:
            self.lib.ec_model_set_taps(self.h, 0)
        return logits, taps

    def forward_device(self, d_tokens, d_positions, d_seqs, M: int, d_logits) -> None:
        self._check(self.lib.ec_forward_device(self.h, _ptr(d_tokens), _ptr(d_positions), _ptr(d_seqs),
                                               int(M), _ptr(d_logits)))

    def decode_greedy(self, d_tokens, start_pos: int, n_steps: int, d_out_ids=None) -> None:
        self._check(self.lib.ec_decode_greedy(self.h, _ptr(d_tokens), int(start_pos), int(n_steps),
                                              _ptr(d_out_ids)))

    def decode_greedy_cycle(self, d_tokens, start_pos: int, period: int, n_steps: int, d_out_ids=None) -> None:
        self._check(self.lib.ec_decode_greedy_cycle(self.h, _ptr(d_tokens), int(start_pos), int(period),
                                                    int(n_steps), _ptr(d_out_ids)))

    def decode_batch(self, d_tokens, d_positions, n_steps: int, d_out_ids=None) -> None:
        """Greedy decode of n_steps tokens for all batch_cap slots (device
        int32 tokens / positions [batch_cap], updated in place; ids into
        d_out_ids [n_steps][batch_cap] when given), one captured CUDA graph
        per step on the model stream."""
        self._check(self.lib.ec_decode_batch(self.h, _ptr(d_tokens), _ptr(d_positions), int(n_steps),
                                             _ptr(d_out_ids)))

    def batch_hidden(self, d_tokens, d_positions, M: int, max_pos_end: int, d_hidden) -> None:
        """Rows m < M (slot m) through every layer and the final norm into
        d_hidden [M][n_embd] fp32 (device); every position < max_pos_end."""
        self._check(self.lib.ec_batch_hidden(self.h, _ptr(d_tokens), _ptr(d_positions), int(M), int(max_pos_end),
                                             _ptr(d_hidden)))

    def lm_shard_keys(self, d_hidden, rows: int, d_keys) -> None:
        """lm_head of the vocab shard over `rows` hidden rows, per-row argmax
        as signed int64 keys (signed max across shards = the global greedy id)."""
        self._check(self.lib.ec_lm_shard_keys(self.h, _ptr(d_hidden), int(rows), _ptr(d_keys)))

    def keys_advance(self, d_keys, M: int, d_tokens, d_positions) -> None:
        """tokens[m] = index in keys[m], positions[m] += 1 (device arrays)."""
        self._check(self.lib.ec_keys_advance(self.h, _ptr(d_keys), int(M), _ptr(d_tokens), _ptr(d_positions)))

    def kv_release(self, slot: int = -1) -> None:
        """Return the KV pages of `slot` (all slots when < 0) to the arena."""
        self._check(self.lib.ec_kv_release(self.h, int(slot)))

    def kv_info(self) -> dict:
        """{pages, free, page_positions, pages_per_slot} of the paged KV arena."""
        info = np.zeros(4, np.int32)
        self._check(self.lib.ec_kv_info(self.h, _ptr(info)))
        return dict(zip(("pages", "free", "page_positions", "pages_per_slot"), (int(v) for v in info)))

    PACKED = {"qkv": 0, "o": 1, "up": 2, "down": 3, "lm_head": 4}

    def packed(self, layer: int, which: str) -> tuple[np.ndarray, dict]:
        """The device-packed rows of one linear (ec_model_packed): uint8
        [N][ldw * element bytes] and {N, K, Kp, ldw, elt}."""
        info = np.zeros(5, np.int32)
        w = self.PACKED[which]
        n = self.lib.ec_model_packed(self.h, int(layer), w, None, 0, _ptr(info))
        if n < 0:
            raise RuntimeError(last_error())
        out = np.empty(int(n), np.uint8)
        if self.lib.ec_model_packed(self.h, int(layer), w, _ptr(out), out.size, _ptr(info)) < 0:
            raise RuntimeError(last_error())
        N, K, Kp, ldw, elt = (int(v) for v in info)
        return out.reshape(N, ldw * elt), {"N": N, "K": K, "Kp": Kp, "ldw": ldw, "elt": elt}

    def batch_graph_kernels(self, kind: int) -> int:
        """Kernel launches in the captured step graph (0: decode_batch, 1: batch_hidden)."""
        n = self.lib.ec_batch_graph_kernels(self.h, int(kind))
        if n < 0:
            raise RuntimeError(last_error())
        return n

    TRACE_CODES = {1: "barrier", 2: "operand", 3: "tiles", 4: "attention", 5: "lm_head", 6: "argmax",
                   7: "tile_in", 8: "tile_free", 9: "tile_done", 10: "issue", 11: "staged", 12: "stats",
                   13: "scores", 14: "softmax", 15: "phase_in"}

    def decode_trace(self, d_tokens, start_pos: int, n_steps: int, cap: int = 1 << 16):
        """Timeline of CTA 0 of the persistent decode kernel: list of (event, ns)
        sorted by time (consumer and producer events interleaved)."""
        buf = np.zeros(cap, np.uint64)
        n = self.lib.ec_decode_trace(self.h, _ptr(d_tokens), int(start_pos), int(n_steps), _ptr(buf), cap)
        if n < 0:
            raise RuntimeError(last_error())
        ev = [(self.TRACE_CODES.get(int(v) >> 56, "?"), int(v) & ((1 << 56) - 1)) for v in buf[:n]]
        return sorted(ev, key=lambda e: e[1])

    def decode_profile(self, d_tokens, start_pos: int, n_steps: int) -> dict:
        """Per-kernel-class event timings of an instrumented decode."""
        out = np.zeros(16, np.float64)
        self._check(self.lib.ec_decode_profile(self.h, _ptr(d_tokens), int(start_pos), int(n_steps), _ptr(out)))
        names = ("decode_step", "gemm", "attention", "norm", "other")
        return {n: {"ms": out[3 * i], "bytes": out[3 * i + 1], "launches": int(out[3 * i + 2])}
                for i, n in enumerate(names)} | {"steps": int(out[15])}

    def set_stream(self, stream_ptr: int | None) -> None:
        self._check(self.lib.ec_model_set_stream(self.h, stream_ptr))

    def set_vocab_shard(self, v0: int, v1: int) -> None:
        self._check(self.lib.ec_model_set_vocab_shard(self.h, int(v0), int(v1)))
