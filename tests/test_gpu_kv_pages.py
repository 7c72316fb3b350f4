"""The paged KV arena: pages of 64 positions mapped per slot as calls reach
new positions, a pool smaller than batch_cap * ceil(eff_ctx / 64) set with
EDGECORE_KV_PAGES, "KV arena full" when a call needs more pages than are
free, and ec_kv_release returning a slot's pages.  Results must equal the
CPU restatement of the reference (contiguous [slot][position] cache,
src/gpt2.c:508-524) whatever physical pages the slots landed on."""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-5   # int8 model: the reference's numerics


def rel_err(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


@pytest.fixture(scope="module")
def model_path(tmp_path_factory):
    spec = synth.TINY_QWEN2.with_(name="tiny-qwen-pages", n_ctx=320, seed=9)
    return spec, synth.ensure_model(spec, tmp_path_factory.mktemp("pages"))


def _fill(m, spec, slot, n, seed):
    t = synth.prompt_ids(spec.vocab, n, seed=seed)
    return m.forward(t, np.arange(n, dtype=np.int32), np.full(n, slot, np.int32)), t


def test_small_arena_maps_releases_and_matches_reference(model_path, monkeypatch, cuda):
    from oracle.oracle import Restatement
    spec, path = model_path
    monkeypatch.setenv("EDGECORE_KV_PAGES", "6")
    r = Restatement().open(path, batch_cap=4, max_ctx=320)
    r.reset()
    with ec.Model(path, batch_cap=4, max_ctx=320) as m:
        info = m.kv_info()
        assert info["pages"] == 6 and info["free"] == 6 and info["page_positions"] == 64
        assert info["pages_per_slot"] == 5
        lg0, _ = _fill(m, spec, 0, 100, 1)                # pages 0, 1
        lg1, t1 = _fill(m, spec, 1, 70, 2)                # pages 2, 3
        assert m.kv_info()["free"] == 2
        # needs 3 pages; the reference-shaped gpt2_forward has no error return
        # (it ends the process, as the reference does), so ask ec_forward_argmax
        with pytest.raises(RuntimeError, match="KV arena full"):
            t = synth.prompt_ids(spec.vocab, 130, seed=3)
            m.forward_argmax(t, np.arange(130, dtype=np.int32), np.full(130, 2, np.int32))
        assert m.kv_info()["free"] == 2                   # the failed call mapped nothing
        m.kv_release(0)
        assert m.kv_info()["free"] == 4
        lg2, t2 = _fill(m, spec, 2, 130, 3)               # reuses slot 0's pages + a fresh one
        w1 = r.forward(t1, np.arange(70, dtype=np.int32), np.full(70, 1, np.int32))
        w2 = r.forward(t2, np.arange(130, dtype=np.int32), np.full(130, 2, np.int32))
        assert rel_err(lg1, w1) < TOL
        assert rel_err(lg2, w2) < TOL
        # batched decode of slots 1 and 2 across page boundaries (127 -> 128 for slot 2)
        cur = np.array([int(np.argmax(w1[-1])), int(np.argmax(w2[-1]))], np.int32)
        pos = np.array([70, 130], np.int32)
        slots = np.array([1, 2], np.int32)
        for i in range(4):
            g = m.forward(cur, pos + i, slots)
            w = r.forward(cur, pos + i, slots)
            assert rel_err(g, w) < TOL, i
            cur = np.argmax(w, axis=1).astype(np.int32)
        m.kv_release(-1)
        assert m.kv_info()["free"] == 6
    r.close()


def test_default_arena_device_loops(model_path, cuda):
    """Full-capacity pool (the default): the device-resident loops map what
    they will touch; decode_greedy across a page boundary equals stepwise
    host calls."""
    torch = cuda
    spec, path = model_path
    with ec.Model(path, batch_cap=1, max_ctx=320) as a, ec.Model(path, batch_cap=1, max_ctx=320) as b:
        assert a.kv_info()["pages"] == 5
        toks = synth.prompt_ids(spec.vocab, 60, seed=4)
        for m in (a, b):
            m.forward(toks, np.arange(60), np.zeros(60, np.int32))
        assert a.kv_info()["free"] == 4
        d_tok = torch.tensor([int(toks[-1])], dtype=torch.int32, device="cuda")
        d_out = torch.zeros(12, dtype=torch.int32, device="cuda")
        a.decode_greedy(d_tok, 60, 12, d_out)     # positions 60..71: a second page
        torch.cuda.synchronize()
        assert a.kv_info()["free"] == 3
        cur, want = int(toks[-1]), []
        for i in range(12):
            ids, _ = b.forward_argmax([cur], [60 + i])
            cur = int(ids[0])
            want.append(cur)
        assert d_out.cpu().tolist() == want
