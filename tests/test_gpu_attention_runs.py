"""The block attention kernel for rows in runs (prefill).

The host cuts a call's rows into blocks of up to 32 consecutive rows of one
slot at consecutive positions; when they average 8 rows or more (prefill),
the attention runs one CTA per (query head, block) and stages each cached
K / V row once per block.  Its arithmetic is the per-row exact-order
kernel's, value for value (reference src/gpt2.c:526-557, :743-777: the fp32
dot over head_dim, the fp64-scaled scores, exp(s - max) / sum, the fp32 sum
over positions in order), so the same rows given in an order that is not a
run (interleaved slots: the per-row kernel) must give identical logits, bit
for bit.  Runs of 45 and 40 rows (blocks of 32 + 13 and 32 + 8 rows, the
second sequence starting mid-way through a 32-row stretch) cross the 64-row
K / V chunks; the sliding-window model (window 5, shorter than a block)
takes the per-row windows inside a block.
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth

pytestmark = pytest.mark.gpu

TOL_EXACT = 1e-5   # int8 models against the restatement of the reference


def rel_err(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


def _rows(vocab, lens, starts, seed):
    """Per-sequence rows: (tokens, positions, slots) in run order."""
    t, p, s = [], [], []
    for k, (n, p0) in enumerate(zip(lens, starts)):
        t.append(synth.prompt_ids(vocab, n, seed=seed + k))
        p.append(np.arange(p0, p0 + n, dtype=np.int32))
        s.append(np.full(n, k, np.int32))
    return np.concatenate(t).astype(np.int32), np.concatenate(p), np.concatenate(s)


def _interleave(n_rows, slots):
    """A permutation that alternates slots, so no 32-row block is a run."""
    by = [list(np.flatnonzero(slots == k)) for k in np.unique(slots)]
    order = []
    while any(by):
        for q in by:
            if q:
                order.append(q.pop(0))
    return np.array(order)


def _check_pair(path, spec, lens, starts, seed, max_ctx):
    t, p, s = _rows(spec.vocab, lens, starts, seed)
    perm = _interleave(len(t), s)
    assert perm.tolist() != list(range(len(t)))
    with ec.Model(path, batch_cap=len(lens), max_ctx=max_ctx) as a, \
            ec.Model(path, batch_cap=len(lens), max_ctx=max_ctx) as b:
        if min(starts) > 0:   # earlier context of every slot, same rows on both models
            for m in (a, b):
                for k, p0 in enumerate(starts):
                    pre = synth.prompt_ids(spec.vocab, p0, seed=seed + 100 + k)
                    m.forward(pre, np.arange(p0, dtype=np.int32), np.full(p0, k, np.int32))
        runs = a.forward(t, p, s)
        rows = b.forward(t[perm], p[perm], s[perm])
    back = np.empty_like(rows)
    back[perm] = rows
    return runs, back, (t, p, s)


def test_runs_equal_row_kernel_tiny_models(tiny_models, cuda):
    from oracle.oracle import Restatement
    for key, (spec, path) in tiny_models.items():
        runs, rows, (t, p, s) = _check_pair(path, spec, [45, 40], [0, 0], 7, 64)
        assert np.array_equal(runs.view(np.uint32), rows.view(np.uint32)), key
        if spec.precision == "int8":
            r = Restatement().open(path, batch_cap=2, max_ctx=64)
            r.reset()
            want = r.forward(t, p, s)
            r.close()
            assert rel_err(runs, want) < TOL_EXACT, key


def test_runs_equal_row_kernel_qwen05b(cuda):
    """Config 3's model at full size: 70 new rows per slot after 90 and 30
    cached positions (blocks starting mid-sequence, spans over several K / V
    chunks)."""
    spec = synth.CONFIGS["c3_qwen05b_int8"]
    path = synth.ensure_model(spec)
    runs, rows, _ = _check_pair(path, spec, [70, 70], [90, 30], 11, 256)
    assert np.array_equal(runs.view(np.uint32), rows.view(np.uint32))
