"""GPU parity of the model path (gpt2_load / gpt2_forward and extensions).

Two oracles (oracle/ec_oracle.c), pinned bit-exact to the reference on CPU:
  * glibc build -- the reference's own numerics, libm included;
  * CR build    -- identical except expf/tanhf are correctly rounded, which is
                   what this library computes on the GPU.
W8A8 models quantise every activation row with a data-dependent scale, so a
1-ulp difference anywhere upstream can flip one int8 rounding and move the
residual stream by ~1e-2 of its max (tests/test_oracle.py measures this on the
reference's own numpy mirror).  glibc's expf / tanhf are not correctly rounded
(8.7e-5 / 5.4% of inputs differ by an ulp), so the reference itself is only
defined up to its libm.  The bars:
  * GPU vs CR oracle, int8 models: residual taps and logits within 1e-5 of
    the tensor max (everything feeding an int8 quantisation follows the
    reference order; only the fp16 lm_head sums in another order), identical
    greedy ids; fp16/bf16 models (no quantisation, linears summed in another
    order than the 8-lane AVX2 loop): 1e-3;
  * GPU vs reference (golden / glibc oracle): 1e-3 on the tiny models, and
    identical greedy ids except at near-ties.
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3      # vs the reference (fp32-accumulate bar of the spec)
TOL_CR = 1e-5   # vs the CR-math restatement


def rel_err(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


def assert_greedy(ids, ref_ids, ref_logits, tol=TOL):
    for i, (a, b) in enumerate(zip(ids, ref_ids)):
        if a != b:
            top2 = np.sort(ref_logits[i])[-2:]
            margin = (top2[1] - top2[0]) / max(np.abs(ref_logits[i]).max(), 1e-30)
            assert margin < tol, f"greedy id differs at step {i} ({a} vs {b}) with margin {margin:.2e}"


@pytest.fixture(scope="module")
def cro(built, cuda):
    from oracle.oracle import Restatement
    return Restatement(cr=True)


@pytest.fixture(scope="module")
def glo(built, cuda):
    from oracle.oracle import Restatement
    return Restatement(cr=False)


def test_tiny_models_prefill_taps(golden, tiny_models, cro, cuda):
    g = golden("models.npz")
    for key, (spec, path) in tiny_models.items():
        with ec.Model(path, batch_cap=2) as m:
            toks = g[f"{key}_prompt"]
            n = len(toks)
            logits, taps = m.forward_taps(toks, np.arange(n), np.zeros(n, np.int32))
        assert rel_err(logits, g[f"{key}_logits"]) < TOL, key
        for l in range(taps.shape[0]):
            assert rel_err(taps[l], g[f"{key}_taps"][l]) < TOL, (key, l)
        r = cro.open(path, batch_cap=2)
        lr, tr = r.forward_taps(toks, np.arange(n, dtype=np.int32), np.zeros(n, np.int32))
        r.close()
        assert rel_err(logits, lr) < TOL_CR, key
        for l in range(taps.shape[0]):
            assert rel_err(taps[l], tr[l]) < TOL_CR, (key, l)


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
    """Prefill (taps) + teacher-forced decode of n_dec steps; returns max errors."""
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


@pytest.mark.parametrize("key", list(MID))
def test_mid_models_real_shapes(key, cro, tmp_path_factory, cuda):
    """Real layer shapes (E, heads, GQA, intermediate, head_dim 64/128) with few
    layers: 40-token prefill (generic GEMM path) and 3 decode steps (GEMV path)."""
    spec = MID[key]
    path = synth.ensure_model(spec, tmp_path_factory.mktemp(key))
    tol = TOL_CR if spec.precision == "int8" else TOL
    ref = cro.open(path, batch_cap=2, max_ctx=128)
    with ec.Model(path, batch_cap=2, max_ctx=128) as m:
        _compare_run(m, ref, synth.prompt_ids(spec.vocab, 40, seed=2), 3, tol, tol)
    ref.close()


@pytest.mark.parametrize("cfg", ["c3_qwen05b_int8", "c0_gpt2_small_int8", "c2_qwen05b_fp16"])
def test_full_size_baseline_models(cfg, cro, glo, cuda):
    """BASELINE configurations at full size: 16-token prefill and 6 teacher-forced
    decode steps against the CR restatement; greedy ids against the reference
    numerics (glibc restatement) up to near-ties."""
    spec = synth.CONFIGS[cfg]
    path = synth.ensure_model(spec)
    toks = synth.prompt_ids(spec.vocab, 16)
    # fp16 linears sum in a different order than the reference's 8-lane AVX2
    # loop: ~1e-7 per layer, ~2e-4 after 24 layers; the spec's 1e-3 bar applies
    tol = TOL_CR if spec.precision == "int8" else TOL
    ref = cro.open(path, batch_cap=1, max_ctx=128)
    with ec.Model(path, batch_cap=1, max_ctx=128) as m:
        _compare_run(m, ref, toks, 6, tol, tol)
    ref.close()
    # the reference's own numerics: greedy decode from the same prompt
    gl = glo.open(path, batch_cap=1, max_ctx=128)
    gl.reset()
    lr = gl.forward(toks, np.arange(16, dtype=np.int32), np.zeros(16, np.int32))
    with ec.Model(path, batch_cap=1, max_ctx=128) as m:
        m.forward(toks, np.arange(16), np.zeros(16, np.int32))
        cur = int(np.argmax(lr[-1]))
        ids, ref_ids, ref_lg = [], [], []
        for i in range(6):
            a = m.forward([cur], [16 + i])[0]
            b = gl.forward(np.array([cur], np.int32), np.array([16 + i], np.int32))[0]
            ids.append(int(np.argmax(a)))
            ref_ids.append(int(np.argmax(b)))
            ref_lg.append(b)
            cur = ref_ids[-1]
    gl.close()
    assert_greedy(ids, ref_ids, ref_lg, tol=5e-2)
