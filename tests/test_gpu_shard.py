"""Vocab-sharded lm_head on the GPU: shards combine to the unsharded greedy
result (one GPU: shards as separate model instances; two GPUs: NCCL ranks)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from edgecore_b200 import synth

pytestmark = pytest.mark.gpu


def _combine_local(parts):
    from edgecore_b200 import vocab_shard as vs
    keys = np.max(np.stack([vs.pack_keys(v, i) for i, v in parts]), axis=0)
    return vs.unpack_keys(keys)


@pytest.mark.parametrize("key", ["qwen2_int8", "gpt2_int8"])
@pytest.mark.parametrize("world", [2, 3])
def test_shards_combine_to_full_argmax(key, world, tiny_models, cuda):
    import edgecore_b200 as ec
    from edgecore_b200 import vocab_shard as vs
    spec, path = tiny_models[key]
    toks = np.array([3, 17, 5, 9, 11, 2, 7], np.int32)
    pos = np.arange(len(toks), dtype=np.int32)
    full = ec.Model(path, batch_cap=1, max_ctx=64)
    parts = []
    try:
        for M in (len(toks), 1):   # prefill rows (GEMM path) and one decode row (persistent kernel)
            t, p = (toks, pos) if M > 1 else (toks[-1:], pos[-1:] + 1)
            want_i, want_v = full.forward_argmax(t, p)
            parts = []
            for r in range(world):
                m = ec.Model(path, batch_cap=1, max_ctx=64)
                try:
                    m.set_vocab_shard(*vs.shard_range(spec.vocab, r, world))
                    if M == 1:
                        m.forward_argmax(toks, pos, shard=True)   # same cached prefix
                    parts.append(m.forward_argmax(t, p, shard=True))
                finally:
                    m.close()
            got_v, got_i = _combine_local(parts)
            assert np.array_equal(got_i, want_i)
            assert np.array_equal(got_v.view(np.uint32), want_v.view(np.uint32))
    finally:
        full.close()


def _nccl_rank(rank, world, port, path, vocab, out):
    import torch
    import torch.distributed as dist
    import edgecore_b200 as ec
    from edgecore_b200 import vocab_shard as vs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        toks = np.array([3, 17, 5, 9, 11, 2, 7], np.int32)
        pos = np.arange(len(toks), dtype=np.int32)
        m = ec.Model(path, batch_cap=1, max_ctx=64)
        sg = vs.ShardedGreedy(m, rank, world, device=torch.device("cuda", rank))
        ids = [int(x) for x in sg.step(toks, pos)]
        cur, p = ids[-1], len(toks)
        for _ in range(6):   # greedy continuation with the sharded lm_head
            nxt = int(sg.step(np.array([cur], np.int32), np.array([p], np.int32))[0])
            ids.append(nxt)
            cur, p = nxt, p + 1
        m.close()
        np.save(os.path.join(out, f"ids{rank}.npy"), np.array(ids))
    finally:
        dist.destroy_process_group()


def test_nccl_two_ranks(tiny_models, tmp_path, cuda):
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import edgecore_b200 as ec
    spec, path = tiny_models["qwen2_int8"]
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_nccl_rank, args=(2, port, str(path), spec.vocab, str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    got = [np.load(tmp_path / f"ids{r}.npy") for r in range(2)]
    assert np.array_equal(got[0], got[1])
    # unsharded reference on this process's device
    m = ec.Model(path, batch_cap=1, max_ctx=64)
    toks = np.array([3, 17, 5, 9, 11, 2, 7], np.int32)
    ids = list(m.forward_argmax(toks, np.arange(len(toks), dtype=np.int32))[0])
    cur, p = ids[-1], len(toks)
    for _ in range(6):
        nxt = int(m.forward_argmax(np.array([cur], np.int32), np.array([p], np.int32))[0][0])
        ids.append(nxt)
        cur, p = nxt, p + 1
    m.close()
    assert np.array_equal(got[0], np.array(ids))


def _batch_prompts(vocab, B):
    return [synth.prompt_ids(vocab, 4 + (b % 7), seed=500 + b) for b in range(B)]


def _batch_prefill(m, toks, slot0):
    """Every stream's prompt into its slot; returns the first greedy ids
    (full lm_head: call before any vocab shard is set) and the positions."""
    lens = np.array([len(t) for t in toks])
    t = np.concatenate(toks).astype(np.int32)
    p = np.concatenate([np.arange(n) for n in lens]).astype(np.int32)
    s = np.concatenate([np.full(n, b) for b, n in enumerate(lens)]).astype(np.int32)
    ids, _ = m.forward_argmax(t, p, s)
    return ids[np.cumsum(lens) - 1].astype(np.int32), lens.astype(np.int32)


def _nccl_batch_rank(rank, world, port, path, B, n_embd, vocab, steps, out):
    import torch
    import torch.distributed as dist
    import edgecore_b200 as ec
    from edgecore_b200 import vocab_shard as vs
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    import datetime
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        mloc = B // world
        toks = _batch_prompts(vocab, B)[rank * mloc:(rank + 1) * mloc]
        m = ec.Model(path, batch_cap=mloc, max_ctx=64)
        first, lens = _batch_prefill(m, toks, 0)
        dec = vs.ShardedBatchDecoder(m, rank, world, mloc, n_embd, vocab, device=torch.device("cuda", rank))
        d_tok = torch.from_numpy(first).cuda()
        d_pos = torch.from_numpy(lens).cuda()
        hist = []
        for s in range(steps):
            dec.step(d_tok, d_pos, int(lens.max()) + s + 1)
            hist.append(d_tok.cpu().numpy().copy())
        torch.cuda.synchronize()
        m.close()
        np.save(os.path.join(out, f"b{rank}.npy"), np.stack(hist))
    finally:
        dist.destroy_process_group()


def test_nccl_batched_sharded_decode(tiny_models, tmp_path, cuda):
    """Two ranks, 20 streams each, the lm_head split in two vocab blocks with
    an NCCL all-gather of hidden rows and an all-reduce(MAX) of int64 keys per
    step: the same greedy ids as one GPU decoding all 40 streams with the
    full lm_head (ec_decode_batch)."""
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    import edgecore_b200 as ec
    spec, path = tiny_models["qwen2_int8"]
    B, steps = 40, 5
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.start_processes(_nccl_batch_rank, args=(2, port, str(path), B, spec.n_embd, spec.vocab, steps, str(tmp_path)),
                       nprocs=2, start_method="spawn", join=True)
    got = np.concatenate([np.load(tmp_path / f"b{r}.npy") for r in range(2)], axis=1)
    m = ec.Model(path, batch_cap=B, max_ctx=64)
    first, lens = _batch_prefill(m, _batch_prompts(spec.vocab, B), 0)
    d_tok = torch.from_numpy(first).cuda()
    d_pos = torch.from_numpy(lens).cuda()
    d_ids = torch.zeros((steps, B), dtype=torch.int32, device="cuda")
    m.decode_batch(d_tok, d_pos, steps, d_ids)
    torch.cuda.synchronize()
    m.close()
    assert np.array_equal(got, d_ids.cpu().numpy())
