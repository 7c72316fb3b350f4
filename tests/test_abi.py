"""The drop-in boundary, checked without a GPU: the library loads, exports
exactly what include/*.h declares, include/edgecore.h is layout-identical to
the reference header, and the CPU-only entry points behave."""
from __future__ import annotations

import ctypes as C
import json
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

from edgecore_b200 import LIB_PATH, synth
from edgecore_b200.ecm import EcmReader

ROOT = Path(__file__).resolve().parents[1]


def declared_functions() -> set[str]:
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        text = re.sub(r"static inline[^{]*\{.*?\n\}", "", text, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b(\w+)\s*\([^;{]*\)\s*;", text, flags=re.M):
            names.add(m.group(1))
    return names


# Provided by the reference's own tokenizer.c / runtime_main.c, which link
# against this library unchanged; declared in edgecore.h for them.
NOT_OURS = {"tokenizer_load", "tokenizer_free", "tokenizer_encode", "tokenizer_decode",
            "peak_rss_gb", "now_sec"}


def exported_symbols() -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", str(LIB_PATH)], capture_output=True, text=True,
                         check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if ln.strip()}


def test_library_loads_without_gpu(built):
    from edgecore_b200 import load_library
    lib = load_library()
    assert b"sm_100a" in lib.ec_version()


def test_exports_match_headers(built):
    decl = declared_functions()
    assert {"gemm_int8", "gemm_fp16_fp32", "gemm_bf16_fp32", "gpt2_load", "gpt2_forward", "gpt2_free",
            "qwen2_forward", "ecm_parse", "ec_decode_greedy"} <= decl
    exp = exported_symbols()
    missing = (decl - NOT_OURS) - exp
    assert not missing, f"declared but not exported: {sorted(missing)}"
    extra = {s for s in exp if not s.startswith("_")} - decl
    assert not extra, f"exported but not declared: {sorted(extra)}"
    assert not (NOT_OURS & exp), "the library must not define the runtime's own symbols"


def test_header_layout_identical_to_reference(tmp_path, golden):
    golden_layout = json.loads((ROOT / "tests" / "golden" / "abi_layout.json").read_text())
    exe = tmp_path / "probe"
    subprocess.run(["gcc", "-std=c11", "-I", str(ROOT / "include"), str(ROOT / "tests" / "abi_probe.c"),
                    "-o", str(exe)], check=True)
    ours = json.loads(subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout)
    assert ours == golden_layout


def test_ecm_parse_matches_reader(built, tmp_path):
    from edgecore_b200 import load_library
    lib = load_library()
    p = synth.ensure_model(synth.TINY_QWEN2.with_(qkv_bias=True), tmp_path)
    rd = EcmReader(p)
    data = p.read_bytes()
    buf = C.create_string_buffer(data, len(data))

    class EcmTensor(C.Structure):
        _fields_ = [("name", C.c_char * 128), ("dtype", C.c_int), ("nelems", C.c_size_t), ("bytes", C.c_size_t),
                    ("offset", C.c_size_t), ("dims", C.c_size_t * 4), ("ndims", C.c_int)]

    layout = json.loads((ROOT / "tests" / "golden" / "abi_layout.json").read_text())
    assert C.sizeof(EcmTensor) == layout["sizeof.EcmTensor"]
    tens = (EcmTensor * 512)()
    meta = C.create_string_buffer(layout["sizeof.GPT2"])
    n = lib.ecm_parse(buf, len(data), C.cast(tens, C.c_void_p), 512, C.cast(meta, C.c_void_p))
    assert n == len(rd.table)
    for i in range(n):
        t = tens[i]
        dtype, dims, off, nbytes = rd.table[t.name.decode()]
        assert (t.offset, t.bytes) == (off, nbytes)
    # meta: n_layer / n_embd / vocab at their reference offsets
    raw = bytes(meta)
    get = lambda f: int.from_bytes(raw[layout[f"GPT2.{f}"][0]:][:4], "little", signed=True)
    assert get("n_layer") == 2 and get("n_embd") == 32 and get("vocab") == 256 and get("arch") == 1
    # bad magic
    bad = C.create_string_buffer(b"ECM2\n" + data[5:], len(data))
    assert lib.ecm_parse(bad, len(data), C.cast(tens, C.c_void_p), 512, C.cast(meta, C.c_void_p)) == -1


def test_argmax_key_order(built):
    from edgecore_b200 import argmax_key, argmax_key_decode
    rng = np.random.default_rng(0)
    vals = np.concatenate([rng.standard_normal(200).astype(np.float32), np.array([0.0, -0.0, 5.0, 5.0, -np.inf],
                                                                               np.float32)])
    idx = rng.permutation(len(vals)).astype(np.int32)
    keys = [argmax_key(v, i) for v, i in zip(vals, idx)]
    best = max(range(len(vals)), key=lambda j: keys[j])
    top = vals.max()
    assert vals[best] == top and idx[best] == idx[vals == top].min()
    for v, i, k in zip(vals, idx, keys):
        dv, di = argmax_key_decode(k)
        want = np.float32(0.0) if v == 0.0 else np.float32(v)   # -0.0 is encoded as +0.0
        assert di == i and np.float32(dv).tobytes() == want.tobytes()


def test_dropin_runtime_links(built):
    exe = ROOT / "oracle" / "_ref" / "edgecore-runtime-b200"
    if not exe.exists():
        pytest.skip("drop-in runtime not built (needs the reference sources)")
    out = subprocess.run(["ldd", str(exe)], capture_output=True, text=True).stdout
    assert "libedgecore_b200.so" in out and "not found" not in out
