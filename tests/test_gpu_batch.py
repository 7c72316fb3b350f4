"""Batched decode of many independent streams (BASELINE config 4's shape of
work) on the tiny seeded models: 40 slots, so that every linear and the
lm_head run on the tcgen05 tensor-core GEMMs.

* ec_decode_batch (device-resident, one captured CUDA graph per step) must
  produce the same ids as stepping gpt2_forward / ec_forward_argmax with host
  arrays, slot by slot at each slot's own position (reference batched decode
  loop, src/runtime_main.c:336-352; greedy pick :213-219).
* The column-split lm_head pieces (ec_batch_hidden, ec_lm_shard_keys,
  ec_keys_advance): keys of two vocab shards combined by a signed max equal
  the unsharded keys bit for bit, and decode to the unsharded argmax.
* The first batched decode step is checked against the CPU restatement.
"""
from __future__ import annotations

import numpy as np
import pytest

import edgecore_b200 as ec
from edgecore_b200 import synth

pytestmark = pytest.mark.gpu

B = 40          # slots (>= 32: tensor-core GEMMs)
STEPS = 5
TOL = 1e-3


def rel_err(a, b):
    return float(np.abs(np.asarray(a) - np.asarray(b)).max() / max(np.abs(b).max(), 1e-30))


def _prompts(spec, seed):
    rng = np.random.default_rng(seed)
    lens = rng.integers(3, 12, B)
    toks = [synth.prompt_ids(spec.vocab, int(n), seed=seed * 1000 + b) for b, n in enumerate(lens)]
    return toks, lens


def _prefill(model, toks, lens):
    """One forward of every slot's prompt (distinct lengths, slot = seqs);
    returns each slot's first greedy id and its next position."""
    t = np.concatenate(toks).astype(np.int32)
    p = np.concatenate([np.arange(n) for n in lens]).astype(np.int32)
    s = np.concatenate([np.full(n, b) for b, n in enumerate(lens)]).astype(np.int32)
    if hasattr(model, "reset"):
        model.reset()
    lg = model.forward(t, p, s)
    last = np.cumsum(lens) - 1
    return np.argmax(lg[last], axis=1).astype(np.int32), lens.astype(np.int32), lg[last]


@pytest.fixture(scope="module")
def int8_models(tiny_models):
    return {k: v for k, v in tiny_models.items() if k.endswith("int8")}


def test_decode_batch_matches_stepwise_forward(int8_models, cuda):
    torch = cuda
    for key, (spec, path) in int8_models.items():
        toks, lens = _prompts(spec, 3)
        with ec.Model(path, batch_cap=B) as a, ec.Model(path, batch_cap=B) as b:
            cur_a, pos_a, _ = _prefill(a, toks, lens)
            cur_b, pos_b, _ = _prefill(b, toks, lens)
            assert np.array_equal(cur_a, cur_b)
            d_tok = torch.from_numpy(cur_a).cuda()
            d_pos = torch.from_numpy(pos_a).cuda()
            d_ids = torch.zeros((STEPS, B), dtype=torch.int32, device="cuda")
            a.decode_batch(d_tok, d_pos, STEPS, d_ids)
            torch.cuda.synchronize()
            assert ec.device_error_take() == 0
            got = d_ids.cpu().numpy()
            want = []
            for _ in range(STEPS):
                ids, _ = b.forward_argmax(cur_b, pos_b, np.arange(B, dtype=np.int32))
                want.append(ids)
                cur_b, pos_b = ids.astype(np.int32), pos_b + 1
            assert np.array_equal(got, np.stack(want)), key
            assert np.array_equal(d_tok.cpu().numpy(), cur_b) and np.array_equal(d_pos.cpu().numpy(), pos_b)
            # a second call continues from the updated state (the graph is reused)
            a.decode_batch(d_tok, d_pos, 2, d_ids)
            torch.cuda.synchronize()
            for i in range(2):
                ids, _ = b.forward_argmax(cur_b, pos_b, np.arange(B, dtype=np.int32))
                assert np.array_equal(d_ids[i].cpu().numpy(), ids), (key, i)
                cur_b, pos_b = ids.astype(np.int32), pos_b + 1


def test_batched_step_against_cpu_oracle(int8_models, cuda):
    from oracle.oracle import Restatement
    ro = Restatement()
    for key, (spec, path) in int8_models.items():
        toks, lens = _prompts(spec, 5)
        r = ro.open(path, batch_cap=B, max_ctx=spec.n_ctx)
        cur_r, pos_r, lg_r = _prefill(r, toks, lens)
        with ec.Model(path, batch_cap=B) as m:
            cur, pos, lg = _prefill(m, toks, lens)
            assert rel_err(lg, lg_r) < TOL, key
            step = m.forward(cur_r, pos_r, np.arange(B, dtype=np.int32))
        want = r.forward(cur_r, pos_r, np.arange(B, dtype=np.int32))
        r.close()
        assert rel_err(step, want) < TOL, key


def test_vocab_shard_keys_combine(int8_models, cuda):
    torch = cuda
    for key, (spec, path) in int8_models.items():
        toks, lens = _prompts(spec, 7)
        V = spec.vocab
        models = [ec.Model(path, batch_cap=B) for _ in range(3)]
        st = torch.cuda.Stream()   # library work and torch ops ordered on one stream
        ctx = torch.cuda.stream(st)
        ctx.__enter__()
        try:
            for m in models:
                m.set_stream(st.cuda_stream)
            models[1].set_vocab_shard(0, V // 2 + 3)
            models[2].set_vocab_shard(V // 2 + 3, V)
            # the same prompts into every model's KV cache; a shard's prefill
            # logits cover only its vocab block, so the first ids come from
            # the unsharded model
            cur, pos, _ = _prefill(models[0], toks, lens)
            for m in models[1:]:
                _prefill(m, toks, lens)
            d_tok = torch.from_numpy(cur).cuda()
            d_pos = torch.from_numpy(pos).cuda()
            hid = [torch.empty((B, spec.n_embd), device="cuda") for _ in models]
            keys = [torch.empty(B, dtype=torch.int64, device="cuda") for _ in models]
            for m, h, k in zip(models, hid, keys):
                m.batch_hidden(d_tok, d_pos, B, int(pos.max()) + 1, h)
                m.lm_shard_keys(h, B, k)
            torch.cuda.synchronize()
            assert ec.device_error_take() == 0
            assert torch.equal(hid[0], hid[1]) and torch.equal(hid[0], hid[2])
            combined = torch.maximum(keys[1], keys[2])
            assert torch.equal(combined, keys[0]), key
            ids_ref, _ = models[0].forward_argmax(cur, pos, np.arange(B, dtype=np.int32))
            models[0].keys_advance(combined, B, d_tok, d_pos)
            torch.cuda.synchronize()
            assert np.array_equal(d_tok.cpu().numpy(), ids_ref), key
            assert np.array_equal(d_pos.cpu().numpy(), pos + 1)
        finally:
            ctx.__exit__(None, None, None)
            for m in models:
                m.close()


def test_sharded_decode_emulated_two_ranks(int8_models, cuda):
    """The ShardedBatchDecoder step with two 'ranks' in one process: two
    models, each holding half of the streams in its slots 0..19 and half of
    the vocab; hidden rows concatenated and keys combined with a max in
    place of NCCL's all-gather and all-reduce.  Same ids as one model
    decoding all streams with ec_decode_batch."""
    torch = cuda
    for key, (spec, path) in int8_models.items():
        toks, lens = _prompts(spec, 9)
        V, half = spec.vocab, B // 2
        with ec.Model(path, batch_cap=B) as full:
            cur, pos, _ = _prefill(full, toks, lens)
            d_tok = torch.from_numpy(cur).cuda()
            d_pos = torch.from_numpy(pos).cuda()
            d_ids = torch.zeros((STEPS, B), dtype=torch.int32, device="cuda")
            full.decode_batch(d_tok, d_pos, STEPS, d_ids)
            torch.cuda.synchronize()
            want = d_ids.cpu().numpy()
        ranks = [ec.Model(path, batch_cap=half) for _ in range(2)]
        # the library's work and the torch ops below on one (non-default) stream
        st = torch.cuda.Stream()
        ctx = torch.cuda.stream(st)
        ctx.__enter__()
        try:
            for m in ranks:
                m.set_stream(st.cuda_stream)
            state = []
            for r, m in enumerate(ranks):
                c, p, _ = _prefill_slice(m, toks[r * half:(r + 1) * half], lens[r * half:(r + 1) * half])
                m.set_vocab_shard(r * V // 2, (r + 1) * V // 2)
                state.append((torch.from_numpy(c).cuda(), torch.from_numpy(p).cuda()))
            hid = [torch.empty((half, spec.n_embd), device="cuda") for _ in ranks]
            keys = [torch.empty(B, dtype=torch.int64, device="cuda") for _ in ranks]
            got = []
            for s in range(STEPS):
                for r, m in enumerate(ranks):
                    m.batch_hidden(state[r][0], state[r][1], half, int(lens.max()) + s + 1, hid[r])
                allh = torch.cat(hid)
                for r, m in enumerate(ranks):
                    m.lm_shard_keys(allh, B, keys[r])
                comb = torch.maximum(keys[0], keys[1])
                for r, m in enumerate(ranks):
                    m.keys_advance(comb[r * half:(r + 1) * half].contiguous(), half, state[r][0], state[r][1])
                torch.cuda.synchronize()
                got.append(torch.cat([state[0][0], state[1][0]]).cpu().numpy())
            assert np.array_equal(np.stack(got), want), key
        finally:
            ctx.__exit__(None, None, None)
            for m in ranks:
                m.close()


def _prefill_slice(model, toks, lens):
    """_prefill for a subset of the streams, placed in slots 0.. of `model`."""
    t = np.concatenate(toks).astype(np.int32)
    p = np.concatenate([np.arange(n) for n in lens]).astype(np.int32)
    s = np.concatenate([np.full(n, b) for b, n in enumerate(lens)]).astype(np.int32)
    lg = model.forward(t, p, s)
    last = np.cumsum(lens) - 1
    return np.argmax(lg[last], axis=1).astype(np.int32), np.asarray(lens, np.int32), lg[last]


@pytest.mark.parametrize("B", [3, 8])
def test_decode_batch_small_against_cpu_oracle(int8_models, cuda, B):
    """3 streams run the persistent decode kernel (up to 7 do), 8 the graph
    of per-layer kernels, each slot at its own position: greedy ids of STEPS
    steps against the CPU
    restatement (identical except where the restatement's top-2 margin is
    below 1e-3 of the row max)."""
    torch = cuda
    from oracle.oracle import Restatement
    ro = Restatement()
    for key, (spec, path) in int8_models.items():
        rng = np.random.default_rng(11)
        lens = rng.integers(3, 12, B)
        toks = [synth.prompt_ids(spec.vocab, int(n), seed=500 + b) for b, n in enumerate(lens)]
        r = ro.open(path, batch_cap=B, max_ctx=spec.n_ctx)
        cur_r, pos_r, _ = _prefill(r, toks, lens)
        with ec.Model(path, batch_cap=B) as m:
            cur, pos, _ = _prefill(m, toks, lens)
            assert np.array_equal(cur, cur_r), key
            d_tok = torch.from_numpy(cur).cuda()
            d_pos = torch.from_numpy(pos).cuda()
            d_ids = torch.zeros((STEPS, B), dtype=torch.int32, device="cuda")
            torch.cuda.synchronize()
            m.decode_batch(d_tok, d_pos, STEPS, d_ids)
            torch.cuda.synchronize()
            assert ec.device_error_take() == 0
            got = d_ids.cpu().numpy()
            assert np.array_equal(d_pos.cpu().numpy(), pos + STEPS)
        for s in range(STEPS):
            lg = r.forward(cur_r, pos_r, np.arange(B, dtype=np.int32))
            want = np.argmax(lg, axis=1).astype(np.int32)
            for b in range(B):
                if got[s, b] != want[b]:
                    top2 = np.sort(lg[b])[-2:]
                    assert (top2[1] - top2[0]) / np.abs(lg[b]).max() < 1e-3, (key, s, b)
            cur_r, pos_r = got[s].astype(np.int32), pos_r + 1
        r.close()
