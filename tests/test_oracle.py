"""The CPU restatement (oracle/ec_oracle.c) pinned against golden vectors made
by the reference itself (tests/golden/make_golden.py), and live against the
reference build where oracle/_ref exists.  Everything here is bit-exact."""
from __future__ import annotations

import numpy as np
import pytest

from edgecore_b200 import synth
from edgecore_b200.ecm import quantize_int8_symmetric


def bits(a):
    return np.ascontiguousarray(a).view(np.uint32 if np.asarray(a).dtype == np.float32 else np.uint8)


@pytest.fixture(scope="module")
def eco(built):
    from oracle.oracle import Restatement
    return Restatement()


def test_export_quantisation_matches_reference_exporter(golden):
    g = golden("quant_export.npz")
    for case in ("normal", "wide", "edge"):
        q, s = quantize_int8_symmetric(g[f"{case}_w"])
        assert np.array_equal(q, g[f"{case}_q"]), case
        assert np.array_equal(bits(s), bits(g[f"{case}_s"])), case


def test_activation_quant_and_int8_linear(eco, golden):
    g = golden("ops.npz")
    for i in range(5):
        X, W, ws = g[f"lin{i}_X"], g[f"lin{i}_W"], g[f"lin{i}_ws"]
        b = g[f"lin{i}_b"] if f"lin{i}_b" in g else None
        q, qs = eco.quantize_rows(X)
        assert np.array_equal(q, g[f"lin{i}_q"]), i
        assert np.array_equal(bits(qs), bits(g[f"lin{i}_qs"])), i
        y = eco.linear_int8(X, W, ws, b)
        assert np.array_equal(bits(y), bits(g[f"lin{i}_y"])), i


def test_gemm_int8_null_scale(eco, golden):
    g = golden("ops.npz")
    assert np.array_equal(bits(eco.gemm_int8(g["gi8_A"], g["gi8_as"], g["gi8_B"])), bits(g["gi8_y_noscale"]))
    assert np.array_equal(bits(eco.gemm_int8(g["gi8_A"], g["gi8_as"], g["gi8_B"], g["gi8_bs"])), bits(g["gi8_y"]))


@pytest.mark.parametrize("K", [64, 29])
def test_gemm_fp16_bf16_lane_order(eco, golden, K):
    g = golden("ops.npz")
    X = g[f"g16_{K}_X"]
    assert np.array_equal(bits(eco.gemm_fp16(X, g[f"g16_{K}_W"])), bits(g[f"g16_{K}_y"]))
    assert np.array_equal(bits(eco.gemm_bf16(X, g[f"gbf_{K}_W"])), bits(g[f"gbf_{K}_y"]))


def test_norms(eco, golden):
    g = golden("ops.npz")
    assert np.array_equal(bits(eco.layernorm(g["norm_x"], g["norm_g"], g["norm_b"], 1e-5)), bits(g["ln_y"]))
    assert np.array_equal(bits(eco.rmsnorm(g["norm_x"], g["norm_g"], 1e-6)), bits(g["rms_y"]))


def test_rope_tables(eco, golden):
    g = golden("ops.npz")
    _, c, s = eco.rope_table(32, g["rope_pos"], 1e6)
    assert np.array_equal(c, g["rope_cos"]) and np.array_equal(s, g["rope_sin"])
    _, c, s = eco.rope_table(32, g["rope_pos"], 1e4, 1, 4.0, 2048.0, 1.2)
    assert np.array_equal(c, g["yarn_cos"]) and np.array_equal(s, g["yarn_sin"])


def test_half_helpers_and_activations(eco, golden):
    import ctypes as C
    g = golden("ops.npz")
    lib = eco.lib
    lib.eco_f2h.restype, lib.eco_f2h.argtypes = C.c_uint16, [C.c_float]
    lib.eco_h2f.restype, lib.eco_h2f.argtypes = C.c_float, [C.c_uint16]
    lib.eco_gelu_x.restype, lib.eco_gelu_x.argtypes = C.c_float, [C.c_float]
    lib.eco_silu_x.restype, lib.eco_silu_x.argtypes = C.c_float, [C.c_float]
    x = g["act_x"]
    f2h = np.array([lib.eco_f2h(float(v)) for v in x], np.uint16)
    assert np.array_equal(f2h, g["f2h"])                                  # reference F16C rounding
    assert np.array_equal(f2h, x.astype(np.float16).view(np.uint16))      # and IEEE RNE
    every = np.arange(0, 65536, 7, dtype=np.uint32).astype(np.uint16)
    back = np.array([lib.eco_h2f(int(h)) for h in every], np.float32)
    ref = every.view(np.float16).astype(np.float32)
    finite = np.isfinite(ref)
    assert np.array_equal(bits(back[finite]), bits(ref[finite]))
    assert np.array_equal(bits(np.array([lib.eco_gelu_x(float(v)) for v in x], np.float32)), bits(g["gelu_y"]))
    assert np.array_equal(bits(np.array([lib.eco_silu_x(float(v)) for v in x], np.float32)), bits(g["silu_y"]))


def _greedy(m, toks, n_prompt, n_dec):
    m.reset()
    m.forward(toks, np.arange(n_prompt, dtype=np.int32), np.zeros(n_prompt, np.int32))
    cur, ids, steps = int(toks[-1]), [], []
    for i in range(n_dec):
        lg = m.forward(np.array([cur], np.int32), np.array([n_prompt + i], np.int32))
        cur = int(np.argmax(lg[0]))
        ids.append(cur)
        steps.append(lg[0])
    return np.array(ids, np.int32), np.stack(steps)


def test_tiny_models_bit_exact(eco, golden, tiny_models):
    g = golden("models.npz")
    for key, (spec, path) in tiny_models.items():
        m = eco.open(path, batch_cap=2)
        toks = g[f"{key}_prompt"]
        n = len(toks)
        logits, taps = m.forward_taps(toks, np.arange(n, dtype=np.int32), np.zeros(n, np.int32))
        assert np.array_equal(bits(logits), bits(g[f"{key}_logits"])), key
        assert np.array_equal(bits(taps), bits(g[f"{key}_taps"])), key
        ids, steps = _greedy(m, toks, n, len(g[f"{key}_greedy"]))
        assert np.array_equal(ids, g[f"{key}_greedy"]), key
        assert np.array_equal(bits(steps), bits(g[f"{key}_greedy_logits"])), key
        m.close()


def test_live_against_reference_build(eco, built):
    """A fresh seed/shape the fixtures do not cover, against oracle/_ref."""
    from oracle import oracle
    try:
        R = oracle.Reference(threads=2)
    except FileNotFoundError:
        pytest.skip("reference not built here (oracle/_ref missing)")
    import tempfile
    spec = synth.TINY_QWEN2.with_(seed=5, n_layer=3, n_embd=64, n_head=4, n_kv_head=2, intermediate=80,
                                  vocab=300, sliding_window=9)
    with tempfile.TemporaryDirectory() as td:
        p = synth.ensure_model(spec, td)
        a, b = eco.open(p, 3), R.open(p, 3)
        toks = synth.prompt_ids(spec.vocab, 20, seed=1)
        pos = np.arange(20, dtype=np.int32)
        for mm in (a, b):
            mm.reset()
        seqs = np.array([0] * 10 + [2] * 10, np.int32)
        pos2 = np.concatenate([np.arange(10), np.arange(10)]).astype(np.int32)
        la, lb = a.forward(toks, pos2, seqs), b.forward(toks, pos2, seqs)
        assert np.array_equal(bits(la), bits(lb))
        la, lb = a.forward(toks[:3], np.array([10, 0, 10], np.int32)), b.forward(toks[:3], np.array([10, 0, 10], np.int32))
        assert np.array_equal(bits(la), bits(lb))
        a.close(); b.close()


def test_libm_restatement_matches_host_libm(built):
    """The C restatement of the host libm's expf / tanhf (the algorithms the
    device kernels use) against the host library, every 64th float bit
    pattern (oracle/_ref/libm_check; `--all` checks all 2^32)."""
    import subprocess
    from pathlib import Path
    exe = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libm_check"
    if not exe.exists():
        pytest.skip("oracle/_ref/libm_check not built")
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "0 differ" in r.stdout
