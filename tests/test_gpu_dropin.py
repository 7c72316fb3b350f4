"""The reference CLI (its own src/runtime_main.c + src/tokenizer.c, compiled
against include/edgecore.h and linked with libedgecore_b200.so instead of
gpt2.c/kernels.c) driven exactly as the reference's Python tools drive it
(edgecore/verify.py:139-165): --mode logits --tokens-file --logits-bin."""
from __future__ import annotations

import json
import subprocess
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
EXE = ROOT / "oracle" / "_ref" / "edgecore-runtime-b200"


def read_logits_bin(p: Path):
    raw = p.read_bytes()
    n, V = np.frombuffer(raw[:8], np.int32)
    toks = np.frombuffer(raw[8:8 + 4 * n], np.int32)
    return toks, np.frombuffer(raw[8 + 4 * n:], np.float32).reshape(n, V)


@pytest.fixture(scope="module")
def exe(built, cuda):
    if not EXE.exists():
        pytest.skip("drop-in runtime not built (reference sources were absent at build time)")
    return EXE


@pytest.mark.parametrize("key", ["gpt2_int8", "qwen2_int8", "qwen2_fp16"])
def test_logits_bin_contract(exe, key, golden, tiny_models, tmp_path):
    g = golden("models.npz")
    spec, path = tiny_models[key]
    toks = g[f"{key}_prompt"]
    tf = tmp_path / "t.txt"
    tf.write_text(" ".join(map(str, toks)) + "\n")
    out = tmp_path / "l.bin"
    r = subprocess.run([str(exe), "--model", str(path), "--mode", "logits", "--tokens-file", str(tf),
                        "--logits-bin", str(out), "--output", str(tmp_path / "o.json")],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    t, lg = read_logits_bin(out)
    assert np.array_equal(t, toks)
    ref = g[f"{key}_logits"]
    assert np.abs(lg - ref).max() / np.abs(ref).max() < 1e-3
    meta = json.loads((tmp_path / "o.json").read_text())
    assert meta["precision"] == spec.precision and meta["n_tokens"] == len(toks)


def test_bench_and_generate_modes(exe, tiny_models, tmp_path):
    spec, path = tiny_models["qwen2_int8"]
    tf = tmp_path / "t.txt"
    tf.write_text("1 2 3 4 5 6\n")
    r = subprocess.run([str(exe), "--model", str(path), "--mode", "bench", "--tokens-file", str(tf),
                        "--n-tokens", "16", "--batch", "2", "--warmup", "1", "--iters", "2"],
                       capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    d = json.loads(r.stdout)
    assert d["tokens_per_sec"] > 0 and d["n_generated_tokens"] == 32 and d["precision"] == "int8"
    r = subprocess.run([str(exe), "--model", str(path), "--mode", "generate", "--tokens-file", str(tf),
                        "--n-tokens", "8", "--no-print"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert json.loads(r.stdout)["n_generated_tokens"] == 8
