"""Load-time repack round trip: the weights gpt2_load leaves on the device,
read back with ec_model_packed, undo the row order and the padding, and
compare byte for byte with the .ecm arrays (int8 weights from the exporter
rule of reference edgecore/ecm.py:50-59, fp16 / bf16 weights as stored) and
the per-row scale / bias tails with the .ecm scale and bias vectors.

Row orders of the packing (reference binding: src/gpt2.c:161-308):
  * Qwen2 q|k|v: in every q and k head, RoPE partners i and i + head_dim/2 at
    rows 2i and 2i+1, then the v rows; the reference passes no bias to these
    projections (src/gpt2.c:709-711), so the packed bias is 0;
  * Qwen2 gate|up: gate j and up j at rows 2j and 2j+1;
  * GPT-2 and every other matrix: file order.
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth
from edgecore_b200.ecm import EcmReader

pytestmark = pytest.mark.gpu

_DT = {"int8": np.int8, "fp16": np.uint16, "bf16": np.uint16, "fp32": np.float32}


def _arr(r: EcmReader, name: str):
    if name not in r.table:
        return None
    dtype, dims, off, nbytes = r.table[name]
    return np.frombuffer(r.data[off:off + nbytes], dtype=_DT[dtype]).reshape(dims)


def _expected(r: EcmReader, layer: int, which: str, meta: dict):
    """(weight rows [N][K] in packed order, scales [N] or None, biases [N] or None)."""
    b = f"blocks.{layer}."
    if meta["arch"] == "gpt2":
        name = {"qkv": "attn", "o": "proj", "up": "fc", "down": "fc2"}[which]
        return _arr(r, b + name + ".w"), _arr(r, b + name + ".s"), _arr(r, b + name + ".b")
    if which in ("o", "down"):
        return _arr(r, b + which + ".w"), _arr(r, b + which + ".s"), None
    if which == "up":
        g, u = _arr(r, b + "gate.w"), _arr(r, b + "up.w")
        gs, us = _arr(r, b + "gate.s"), _arr(r, b + "up.s")
        w = np.empty((2 * g.shape[0], g.shape[1]), g.dtype)
        w[0::2], w[1::2] = g, u
        s = None
        if gs is not None:
            s = np.empty(2 * gs.shape[0], np.float32)
            s[0::2], s[1::2] = gs, us
        return w, s, None
    hd = int(meta["n_embd"]) // int(meta["n_head"])
    half = hd // 2
    rows, scales = [], []
    for part in ("q", "k"):
        w, s = _arr(r, b + part + ".w"), _arr(r, b + part + ".s")
        for h in range(w.shape[0] // hd):
            for i in range(half):
                for t in range(2):
                    rows.append(w[h * hd + i + t * half])
                    scales.append(None if s is None else s[h * hd + i + t * half])
    v, vs = _arr(r, b + "v.w"), _arr(r, b + "v.s")
    for d in range(v.shape[0]):
        rows.append(v[d])
        scales.append(None if vs is None else vs[d])
    s = None if scales[0] is None else np.array(scales, np.float32)
    return np.stack(rows), s, None


def _check(m: ec.Model, r: EcmReader, layer: int, which: str):
    packed, info = m.packed(layer, which)
    N, K, Kp, elt = info["N"], info["K"], info["Kp"], info["elt"]
    if which == "lm_head":
        w = _arr(r, "lm_head.w")
        if w is None:
            w = _arr(r, "wte")
        s = b = None
    else:
        w, s, b = _expected(r, layer, which, r.meta)
    assert w.shape == (N, K), (which, w.shape, N, K)
    got_w = packed[:, :K * elt].copy().view(w.dtype)
    assert np.array_equal(got_w, w), (layer, which, "weights")
    assert not packed[:, K * elt:Kp * elt].any(), (layer, which, "padding")
    if which == "lm_head":
        return
    tail = packed[:, Kp * elt:Kp * elt + 16].copy().view(np.float32)
    want_s = s if s is not None else np.ones(N, np.float32)
    want_b = b if b is not None else np.zeros(N, np.float32)
    assert np.array_equal(tail[:, 0].view(np.uint32), want_s.astype(np.float32).view(np.uint32)), (layer, which)
    assert np.array_equal(tail[:, 1].view(np.uint32), want_b.astype(np.float32).view(np.uint32)), (layer, which)
    assert not tail[:, 2:].any()


def test_repack_round_trip_tiny_models(tiny_models, cuda):
    for key, (spec, path) in tiny_models.items():
        r = EcmReader(path)
        with ec.Model(path, batch_cap=1) as m:
            for layer in range(spec.n_layer):
                for which in ("qkv", "o", "up", "down"):
                    _check(m, r, layer, which)
            _check(m, r, 0, "lm_head")


@pytest.mark.parametrize("cfg", ["c3_qwen05b_int8", "c0_gpt2_small_int8"])
def test_repack_round_trip_full_size(cfg, cuda):
    """BASELINE configs 3 and 0 at full size: first and last layer."""
    spec = synth.CONFIGS[cfg]
    path = synth.ensure_model(spec)
    r = EcmReader(path)
    with ec.Model(path, batch_cap=1, max_ctx=64) as m:
        for layer in (0, spec.n_layer - 1):
            for which in ("qkv", "o", "up", "down"):
                _check(m, r, layer, which)
