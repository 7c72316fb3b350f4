"""GPU parity of the model path (gpt2_load / gpt2_forward and extensions)
against the golden vectors of the reference and the CPU restatement.

Tolerances (the spec's fp32-accumulate bar): logits and per-layer residual
taps within 1e-3 of the reference relative to the tensor's max |value|.
Greedy ids must be identical except where the oracle's top-2 logit margin is
itself below that tolerance (a near-tie).
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def rel_err(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


def assert_greedy(ids, ref_ids, ref_logits):
    for i, (a, b) in enumerate(zip(ids, ref_ids)):
        if a != b:
            top2 = np.sort(ref_logits[i])[-2:]
            margin = (top2[1] - top2[0]) / max(np.abs(ref_logits[i]).max(), 1e-30)
            assert margin < TOL, f"greedy id differs at step {i} ({a} vs {b}) with margin {margin:.2e}"


@pytest.fixture(scope="module")
def eco(built, cuda):
    from oracle.oracle import Restatement
    return Restatement()


def test_tiny_models_prefill_taps(golden, tiny_models, cuda):
    g = golden("models.npz")
    for key, (spec, path) in tiny_models.items():
        with ec.Model(path, batch_cap=2) as m:
            toks = g[f"{key}_prompt"]
            n = len(toks)
            logits, taps = m.forward_taps(toks, np.arange(n), np.zeros(n, np.int32))
            assert rel_err(logits, g[f"{key}_logits"]) < TOL, key
            for l in range(taps.shape[0]):
                assert rel_err(taps[l], g[f"{key}_taps"][l]) < TOL, (key, l)


def test_tiny_models_decode(golden, tiny_models, cuda):
    """Teacher-forced decode (the golden greedy ids fed back) and batched decode."""
    g = golden("models.npz")
    for key, (spec, path) in tiny_models.items():
        with ec.Model(path, batch_cap=2) as m:
            toks = g[f"{key}_prompt"]
            n = len(toks)
            m.forward(toks, np.arange(n), np.zeros(n, np.int32))
            ref_ids, ref_lg = g[f"{key}_greedy"], g[f"{key}_greedy_logits"]
            cur, ids = int(toks[-1]), []
            for i in range(len(ref_ids)):
                lg = m.forward([cur], [n + i])[0]
                assert rel_err(lg, ref_lg[i]) < TOL, (key, i)
                ids.append(int(np.argmax(lg)))
                cur = int(ref_ids[i])
            assert_greedy(ids, ref_ids, ref_lg)
            # batched decode: slots 0/1 with different prompts, then M=2 steps
            t2 = synth.prompt_ids(spec.vocab, 5, seed=9)
            m.forward(toks[:7], np.arange(7), np.zeros(7, np.int32))
            m.forward(t2, np.arange(5), np.ones(5, np.int32))
            cur2, p2 = np.array([toks[6], t2[4]], np.int32), np.array([7, 5], np.int32)
            for i in range(3):
                lg = m.forward(cur2, p2)
                want = g[f"{key}_batch_logits"][i]
                assert rel_err(lg, want) < TOL, (key, i)
                cur2 = np.argmax(want, axis=1).astype(np.int32)
                p2 = p2 + 1


def test_argmax_and_device_decode_agree_with_logits(tiny_models, cuda):
    torch = cuda
    spec, path = tiny_models["qwen2_int8"]
    with ec.Model(path, batch_cap=1) as m:
        toks = synth.prompt_ids(spec.vocab, 9, seed=4)
        m.forward(toks, np.arange(9), np.zeros(9, np.int32))
        # host loop: logits + numpy argmax (first index among equal maxima)
        cur, host_ids = int(toks[-1]), []
        for i in range(12):
            lg = m.forward([cur], [9 + i])[0]
            ids, mx = m.forward_argmax([cur], [9 + i])
            assert ids[0] == int(np.argmax(lg)) and mx[0] == lg.max()
            cur = int(ids[0])
            host_ids.append(cur)
        # device-resident loop from the same state
        m.forward(toks, np.arange(9), np.zeros(9, np.int32))
        d_tok = torch.tensor([int(toks[-1])], dtype=torch.int32, device="cuda")
        d_out = torch.zeros(12, dtype=torch.int32, device="cuda")
        m.decode_greedy(d_tok, 9, 12, d_out)
        torch.cuda.synchronize()
        assert d_out.cpu().tolist() == host_ids
        assert int(d_tok.item()) == host_ids[-1]


def test_invalid_inputs_fail_cleanly(tiny_models, cuda):
    spec, path = tiny_models["gpt2_int8"]
    with ec.Model(path, batch_cap=1, max_ctx=16) as m:
        with pytest.raises(RuntimeError, match="token id"):
            m.forward_argmax([spec.vocab], [0])
        with pytest.raises(RuntimeError, match="position"):
            m.forward_argmax([1], [16])
        ids, _ = m.forward_argmax([1], [0])        # still usable afterwards
        assert 0 <= ids[0] < spec.vocab


MID = {
    "qwen05_2l_int8": synth.QWEN25_05B.with_(name="qwen-mid", n_layer=2, vocab=4096, n_ctx=512, norm_noise=0.1),
    "qwen05_2l_fp16": synth.QWEN25_05B.with_(name="qwen-mid", n_layer=2, vocab=4096, n_ctx=512, precision="fp16",
                                             norm_noise=0.1),
    "qwen15_1l_int8": synth.QWEN25_15B.with_(name="qwen15-mid", n_layer=1, vocab=2048, n_ctx=256),
    "gpt2s_2l_int8": synth.GPT2_SMALL.with_(name="gpt2-mid", n_layer=2, vocab=4096, norm_noise=0.1),
}


@pytest.mark.parametrize("key", list(MID))
def test_mid_models_real_shapes(key, eco, tmp_path_factory, cuda):
    """Real layer shapes (E, heads, GQA, intermediate) with few layers: prefill of
    40 tokens (GEMM path), 3 decode steps (GEMV path), 2-slot batch."""
    spec = MID[key]
    path = synth.ensure_model(spec, tmp_path_factory.mktemp(key))
    ref = eco.open(path, batch_cap=2, max_ctx=128)
    with ec.Model(path, batch_cap=2, max_ctx=128) as m:
        toks = synth.prompt_ids(spec.vocab, 40, seed=2)
        pos = np.arange(40, dtype=np.int32)
        sq = np.zeros(40, np.int32)
        ref.reset()
        lr, tr = ref.forward_taps(toks, pos, sq)
        lg, tg = m.forward_taps(toks, pos, sq)
        assert rel_err(lg, lr) < TOL
        for l in range(tr.shape[0]):
            assert rel_err(tg[l], tr[l]) < TOL, l
        cur = int(np.argmax(lr[-1]))
        for i in range(3):
            a = m.forward([cur], [40 + i])[0]
            b = ref.forward(np.array([cur], np.int32), np.array([40 + i], np.int32))[0]
            assert rel_err(a, b) < TOL, i
            cur = int(np.argmax(b))
        ref.close()


@pytest.mark.parametrize("cfg", ["c3_qwen05b_int8", "c0_gpt2_small_int8"])
def test_full_size_baseline_models(cfg, eco, cuda):
    """BASELINE configurations at full size: prompt prefill (16 tokens) and 6
    greedy decode steps against the restatement."""
    spec = synth.CONFIGS[cfg]
    path = synth.ensure_model(spec)
    ctx = 128
    ref = eco.open(path, batch_cap=1, max_ctx=ctx)
    with ec.Model(path, batch_cap=1, max_ctx=ctx) as m:
        toks = synth.prompt_ids(spec.vocab, 16)
        pos = np.arange(16, dtype=np.int32)
        ref.reset()
        lr = ref.forward(toks, pos, np.zeros(16, np.int32))
        lg = m.forward(toks, pos, np.zeros(16, np.int32))
        assert rel_err(lg, lr) < TOL
        cur, ids, ref_ids, ref_lg = int(np.argmax(lr[-1])), [], [], []
        for i in range(6):
            a = m.forward([cur], [16 + i])[0]
            b = ref.forward(np.array([cur], np.int32), np.array([16 + i], np.int32))[0]
            assert rel_err(a, b) < TOL, i
            ids.append(int(np.argmax(a)))
            ref_ids.append(int(np.argmax(b)))
            ref_lg.append(b)
            cur = ref_ids[-1]
        assert_greedy(ids, ref_ids, ref_lg)
    ref.close()
