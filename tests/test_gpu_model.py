"""GPU parity of the model path (gpt2_load / gpt2_forward and extensions).

The oracle is the C restatement of the reference (oracle/ec_oracle.c),
pinned bit-exact on CPU to the reference's own golden vectors and build.  It
calls the host libm's expf / tanhf as the reference does, and the device
kernels use restatements of those same algorithms (bit-exact on every float,
tests/test_gpu_ops.py), so everything that feeds an int8 activation
quantisation rounds as in the reference.  W8A8 models quantise every
activation row with a data-dependent scale: one last-bit difference upstream
can flip an int8 rounding and move the residual stream by ~1e-2 of its max,
so these bars only hold because the arithmetic is the reference's.
  * int8 models: residual taps and logits within 1e-5 of the tensor max (the
    fp16 lm_head is the one product summed in another order than the
    reference's 8-lane AVX2 loop), identical greedy ids except at near-ties
    (top-2 margin below 1e-3 of the row max);
  * fp16/bf16 models (every linear summed in another order): 1e-3.
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3        # fp32-accumulate bar of the spec (fp16 / bf16 models)
TOL_EXACT = 1e-5  # int8 models: only the lm_head's summation order differs


def rel_err(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


def assert_greedy(ids, ref_ids, ref_logits, tol=TOL):
    for i, (a, b) in enumerate(zip(ids, ref_ids)):
        if a != b:
            top2 = np.sort(ref_logits[i])[-2:]
            margin = (top2[1] - top2[0]) / max(np.abs(ref_logits[i]).max(), 1e-30)
            assert margin < tol, f"greedy id differs at step {i} ({a} vs {b}) with margin {margin:.2e}"


@pytest.fixture(scope="module")
def eco(built, cuda):
    from oracle.oracle import Restatement
    return Restatement()


def test_tiny_models_prefill_taps(golden, tiny_models, eco, cuda):
    g = golden("models.npz")
    for key, (spec, path) in tiny_models.items():
        with ec.Model(path, batch_cap=2) as m:
            toks = g[f"{key}_prompt"]
            n = len(toks)
            logits, taps = m.forward_taps(toks, np.arange(n), np.zeros(n, np.int32))
        assert rel_err(logits, g[f"{key}_logits"]) < TOL, key
        for l in range(taps.shape[0]):
            assert rel_err(taps[l], g[f"{key}_taps"][l]) < TOL, (key, l)
        r = eco.open(path, batch_cap=2)
        lr, tr = r.forward_taps(toks, np.arange(n, dtype=np.int32), np.zeros(n, np.int32))
        r.close()
        # tiny dims: even the fp16 / bf16 sums agree to ~1e-7 here
        assert rel_err(logits, lr) < TOL_EXACT, key
        for l in range(taps.shape[0]):
            assert rel_err(taps[l], tr[l]) < TOL_EXACT, (key, l)


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
        cur, host_ids = int(toks[-1]), []
        buf = np.full((1, spec.vocab), np.nan, np.float32)   # one reused logits buffer
        for i in range(12):
            lg = m.forward([cur], [9 + i])[0]
            ids, mx = m.forward_argmax([cur], [9 + i])
            assert ids[0] == int(np.argmax(lg)) and mx[0] == lg.max()
            assert m.forward([cur], [9 + i], out=buf) is buf and np.array_equal(buf[0], lg)
            cur = int(ids[0])
            host_ids.append(cur)
        with pytest.raises(ValueError):
            m.forward([cur], [21], out=np.empty((1, spec.vocab), np.float64))
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


def _compare_run(m, ref, toks, n_dec, tol, greedy_tol):
    """Prefill (taps) + decode of n_dec steps teacher-forced with the
    reference's greedy ids; returns those ids and their logits."""
    n = len(toks)
    pos = np.arange(n, dtype=np.int32)
    sq = np.zeros(n, np.int32)
    ref.reset()
    lr, tr = ref.forward_taps(toks, pos, sq)
    lg, tg = m.forward_taps(toks, pos, sq)
    assert rel_err(lg, lr) < tol
    for l in range(tr.shape[0]):
        assert rel_err(tg[l], tr[l]) < tol, l
    cur, ids, ref_ids, ref_lg = int(np.argmax(lr[-1])), [], [], []
    for i in range(n_dec):
        a = m.forward([cur], [n + i])[0]
        b = ref.forward(np.array([cur], np.int32), np.array([n + i], np.int32))[0]
        assert rel_err(a, b) < tol, i
        ids.append(int(np.argmax(a)))
        ref_ids.append(int(np.argmax(b)))
        ref_lg.append(b)
        cur = ref_ids[-1]
    assert_greedy(ids, ref_ids, ref_lg, greedy_tol)
    return ref_ids, ref_lg


@pytest.mark.parametrize("key", list(MID))
def test_mid_models_real_shapes(key, eco, tmp_path_factory, cuda):
    """Real layer shapes (E, heads, GQA, intermediate, head_dim 64/128) with few
    layers: 40-token prefill (generic GEMM path) and 3 decode steps (GEMV path)."""
    spec = MID[key]
    path = synth.ensure_model(spec, tmp_path_factory.mktemp(key))
    tol = TOL_EXACT if spec.precision == "int8" else TOL
    ref = eco.open(path, batch_cap=2, max_ctx=128)
    with ec.Model(path, batch_cap=2, max_ctx=128) as m:
        _compare_run(m, ref, synth.prompt_ids(spec.vocab, 40, seed=2), 3, tol, tol)
    ref.close()


FULL = [("c0_gpt2_small_int8", 128), ("c3_qwen05b_int8", 256), ("c2_qwen05b_fp16", 256)]


@pytest.mark.parametrize("cfg,n_dec", FULL)
def test_full_size_baseline_models(cfg, n_dec, eco, cuda):
    """BASELINE configurations 0, 2 and 3 at full size against the
    restatement of the reference: a 64-token prefill (every layer's residual
    tap and the logits), then n_dec greedy decode steps at positions 64..
    63+n_dec, teacher-forced with the reference's ids.  int8 models to 1e-5
    of the row max, the fp16 model to 1e-3; greedy ids identical except where
    the reference's own top-2 margin is below 1e-3 of the row max."""
    spec = synth.CONFIGS[cfg]
    path = synth.ensure_model(spec)
    toks = synth.prompt_ids(spec.vocab, 64)
    tol = TOL_EXACT if spec.precision == "int8" else TOL
    ctx = 64 + n_dec + 1
    ref = eco.open(path, batch_cap=1, max_ctx=ctx)
    with ec.Model(path, batch_cap=1, max_ctx=ctx) as m:
        ref_ids, ref_lg = _compare_run(m, ref, toks, n_dec, tol, TOL)
        # the device-resident greedy loop (the benchmarked path) generates the
        # reference's sequence up to the first near-tie
        torch = cuda
        m.forward(toks, np.arange(64), np.zeros(64, np.int32))
        d_tok = torch.tensor([int(toks[-1])], dtype=torch.int32, device="cuda")
        d_out = torch.zeros(n_dec + 1, dtype=torch.int32, device="cuda")
        m.decode_greedy(d_tok, 63, n_dec + 1, d_out)
        torch.cuda.synchronize()
        got = d_out.cpu().tolist()[1:]
    ref.close()
    for i, (a, b) in enumerate(zip(got, ref_ids)):
        top2 = np.sort(ref_lg[i])[-2:]
        if (top2[1] - top2[0]) / np.abs(ref_lg[i]).max() < TOL:
            break
        assert a == b, f"free-running greedy id differs at step {i}"
