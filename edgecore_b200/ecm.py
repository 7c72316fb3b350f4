"""The .ecm model container and the export-time int8 weight quantisation.

The container is EdgeCore's (reference edgecore/ecm.py:1-10, :62-100, parsed by
src/gpt2.c:34-136): the magic line ``ECM1``, ``key=value`` meta lines up to
``END_META``, one ``<name> <dtype> <dims...>`` line per tensor up to
``END_TENSORS`` (a ``text`` tensor gives its byte count as its only dim), then
the raw tensor blobs back to back in table order, with no alignment padding.
Both sides must agree on that byte layout, so this module writes exactly it.

dtypes: fp32 (4 B), fp16 (2 B), bf16 (2 B, stored as raw uint16 bit patterns),
int8 (1 B), text (bytes).
"""
from __future__ import annotations

from pathlib import Path
from typing import Any, BinaryIO, Iterable

import numpy as np

MAGIC = b"ECM1\n"
DTYPE_BYTES = {"fp32": 4, "fp16": 2, "bf16": 2, "int8": 1, "text": 1}
_NP = {"fp32": np.float32, "fp16": np.float16, "bf16": np.uint16, "int8": np.int8, "text": np.uint8}


def quantize_int8_symmetric(w: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Per-output-row symmetric int8 quantisation of an fp32 [rows, cols] matrix.

    The rule of reference edgecore/ecm.py:50-59, computed in float64:
    scale = max|w| / 127 per row (1.0 for an all-zero row), q = rint(w / scale)
    (round half to even) clipped to [-128, 127]; scales are returned as fp32.
    """
    a = np.asarray(w, dtype=np.float64)
    if a.ndim != 2:
        raise ValueError("quantize_int8_symmetric expects a 2-D matrix")
    scale = np.abs(a).max(axis=1) / 127.0 if a.shape[1] else np.zeros(a.shape[0])
    scale = np.where(scale == 0.0, 1.0, scale)
    q = np.clip(np.rint(a / scale[:, None]), -128, 127).astype(np.int8)
    return q, scale.astype(np.float32)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bfloat16 bit patterns (uint16), round to nearest even, NaN kept quiet."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    return np.where(nan, np.uint16(0x7FC0), rounded)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


class EcmWriter:
    """Accumulates meta and tensors, then streams an .ecm file."""

    def __init__(self) -> None:
        self.meta: dict[str, Any] = {}
        self._tensors: list[tuple[str, str, np.ndarray]] = []

    def set_meta(self, **kw: Any) -> None:
        self.meta.update(kw)

    def add(self, name: str, dtype: str, arr: np.ndarray) -> None:
        if dtype not in DTYPE_BYTES:
            raise ValueError(f"unknown dtype {dtype}")
        if dtype == "bf16" and np.asarray(arr).dtype != np.uint16:
            arr = f32_to_bf16_bits(arr)
        elif dtype != "bf16":
            arr = np.asarray(arr).astype(_NP[dtype], copy=False)
        self._tensors.append((name, dtype, np.ascontiguousarray(arr)))

    def _header(self) -> bytes:
        lines = [f"{k}={v}" for k, v in self.meta.items()] + ["END_META"]
        for name, dtype, arr in self._tensors:
            dims = str(arr.nbytes) if dtype == "text" else " ".join(str(d) for d in arr.shape)
            lines.append(f"{name} {dtype} {dims}")
        lines.append("END_TENSORS")
        return MAGIC + ("\n".join(lines) + "\n").encode()

    def write(self, fh: BinaryIO) -> None:
        fh.write(self._header())
        for _, _, arr in self._tensors:
            fh.write(memoryview(arr).cast("B"))

    def save(self, path: str | Path) -> Path:
        path = Path(path)
        path.parent.mkdir(parents=True, exist_ok=True)
        tmp = path.with_suffix(path.suffix + ".part")
        with open(tmp, "wb") as fh:
            self.write(fh)
        tmp.replace(path)
        return path


class EcmReader:
    """Parses an .ecm file (memory-mapped) into meta and zero-copy tensor views."""

    def __init__(self, path: str | Path) -> None:
        self.path = Path(path)
        self.data = np.memmap(self.path, dtype=np.uint8, mode="r")
        self.meta: dict[str, str] = {}
        self.table: dict[str, tuple[str, list[int], int, int]] = {}
        self._parse()

    def _lines(self) -> Iterable[tuple[str, int]]:
        buf = self.data
        pos = len(MAGIC)
        while True:
            nl = int(np.argmax(buf[pos:pos + 4096] == 10))
            if buf[pos + nl] != 10:
                raise ValueError("ecm: header line too long or truncated")
            yield bytes(buf[pos:pos + nl]).decode().rstrip("\r"), pos + nl + 1
            pos = pos + nl + 1

    def _parse(self) -> None:
        if bytes(self.data[:5]) != MAGIC:
            raise ValueError("ecm: bad magic")
        it = self._lines()
        for line, _ in it:
            if line == "END_META":
                break
            k, sep, v = line.partition("=")
            if sep:
                self.meta[k] = v
        order = []
        end = 0
        for line, nxt in it:
            if line == "END_TENSORS":
                end = nxt
                break
            parts = line.split()
            if len(parts) < 2 or parts[1] not in DTYPE_BYTES:
                continue
            dims = [int(x) for x in parts[2:]]
            nbytes = dims[0] if parts[1] == "text" else int(np.prod(dims, dtype=np.int64)) * DTYPE_BYTES[parts[1]]
            order.append((parts[0], parts[1], dims, nbytes))
        off = end
        for name, dtype, dims, nbytes in order:
            self.table[name] = (dtype, dims, off, nbytes)
            off += nbytes

    def tensor(self, name: str) -> np.ndarray:
        dtype, dims, off, nbytes = self.table[name]
        raw = self.data[off:off + nbytes]
        if dtype == "text":
            return np.asarray(raw)
        return np.frombuffer(raw, dtype=_NP[dtype]).reshape(dims)
