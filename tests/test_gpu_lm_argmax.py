"""The lm_head with the row argmax fused into the tensor-core GEMM epilogue.

ec_forward_argmax (ids only) of 64 or more rows runs the lm_head GEMM with
the argmax in its epilogue: per (row, 64/128/256-column tile, half) the
maximum and its first column, merged by k_argmax_final with the lowest index
on equal values, as the reference's strict '>' scan does
(src/runtime_main.c:213-219).  No logits are written.  Its ids and maxima
must equal the argmax of the logits gpt2_forward returns for the same rows,
bit for bit: the fp16 (tied, 256-column tiles) and bf16 (128-column tiles)
lm_heads of the tiny models, the full-size config-3 lm_head (151936 x 896),
and a vocab-sharded model whose shard does not end on a tile boundary.
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth

pytestmark = pytest.mark.gpu


def _pair(path, spec, n, max_ctx, seed, shard=None):
    t = synth.prompt_ids(spec.vocab, n, seed=seed)
    p = np.arange(n, dtype=np.int32)
    with ec.Model(path, batch_cap=1, max_ctx=max_ctx) as a, ec.Model(path, batch_cap=1, max_ctx=max_ctx) as b:
        if shard is not None:   # a: the shard's lm_head; b: the full one, then the shard's columns
            a.set_vocab_shard(*shard)
        ids, mx = a.forward_argmax(t, p, shard=shard is not None)
        lg = b.forward(t, p)
    if shard is not None:
        lg = lg[:, shard[0]:shard[1]]
    return ids, mx, lg


def _check(ids, mx, lg, v0=0):
    want = np.argmax(lg, axis=1)          # first index of the maximum
    assert np.array_equal(ids, want + v0)
    assert np.array_equal(mx.view(np.uint32), lg[np.arange(len(lg)), want].view(np.uint32))


def test_fused_argmax_tiny_models(tiny_models, cuda):
    for key, (spec, path) in tiny_models.items():
        ids, mx, lg = _pair(path, spec, 64, 64, 5)
        _check(ids, mx, lg)


def test_fused_argmax_qwen05b(cuda):
    spec = synth.CONFIGS["c3_qwen05b_int8"]
    path = synth.ensure_model(spec)
    ids, mx, lg = _pair(path, spec, 80, 128, 6)
    _check(ids, mx, lg)


def test_fused_argmax_vocab_shard(cuda):
    spec = synth.CONFIGS["c3_qwen05b_int8"]
    path = synth.ensure_model(spec)
    ids, mx, lg = _pair(path, spec, 70, 128, 8, shard=(1000, 76001))
    _check(ids, mx, lg, v0=1000)
