"""Column-split lm_head combine (edgecore_b200.vocab_shard): key order, and the
all_reduce combine across world-size-2 gloo ranks on CPU."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from edgecore_b200 import vocab_shard as vs


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _ref_argmax(logits: np.ndarray):
    # reference greedy rule: strict '>' over ascending indices -> lowest index on ties
    idx = np.argmax(logits, axis=1)   # numpy returns the first maximum
    return logits[np.arange(len(idx)), idx], idx


def test_shard_ranges_cover_vocab():
    for V, W in ((151936, 8), (50257, 3), (7, 4)):
        r = [vs.shard_range(V, k, W) for k in range(W)]
        assert r[0][0] == 0 and r[-1][1] == V
        assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
        assert max(b - a for a, b in r) - min(b - a for a, b in r) <= 1


def test_keys_order_and_roundtrip(built):
    import edgecore_b200 as ec
    vals = np.array([-np.inf, -1e30, -2.5, -1e-40, -0.0, 0.0, 1e-40, 1.0, 1.0, 3e38, np.inf], np.float32)
    idx = np.array([5, 9, 1, 2, 7, 3, 4, 8, 2, 0, 6], np.int64)
    keys = vs.pack_keys(vals, idx)
    # same keys as the C encoding, top bit flipped for signed order
    for v, i, k in zip(vals, idx, keys):
        assert (ec.argmax_key(float(v), int(i)) ^ (1 << 63)) == int(np.int64(k).astype(np.uint64))
    v2, i2 = vs.unpack_keys(keys)
    want_v = np.where(vals == 0.0, np.float32(0.0), vals).astype(np.float32)   # -0.0 comes back as +0.0
    assert np.array_equal(v2.view(np.uint32), want_v.view(np.uint32)) and np.array_equal(i2, idx)
    # signed max of keys == (largest value, then lowest index)
    order = sorted(range(len(vals)), key=lambda j: (vals[j], -idx[j]))
    assert int(np.argmax(keys)) == order[-1]
    assert keys[7] < keys[8]          # 1.0 at index 8 loses to 1.0 at index 2
    # -0.0 and +0.0 tie, so the lower index wins, whichever sign it carries
    assert keys[5] > keys[4]          # +0.0 at index 3 beats -0.0 at index 7
    z = vs.pack_keys(np.array([-0.0, 0.0], np.float32), np.array([1, 2]))
    assert z[0] > z[1]                # -0.0 at index 1 beats +0.0 at index 2
    # NaN loses to every number, -inf included
    n = vs.pack_keys(np.array([np.nan, -np.inf], np.float32), np.array([0, 1]))
    assert n[0] < n[1]
    assert (ec.argmax_key(float("nan"), 0) ^ (1 << 63)) == int(np.int64(n[0]).astype(np.uint64))


def _rank_main(rank: int, world: int, port: int, seed: int, out_dir: str):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(seed)
        V, M = 1003, 6
        logits = rng.integers(-50, 50, (M, V)).astype(np.float32)   # many exact ties
        half = V // 2
        logits[0, half - 1] = logits[0, half] = 1e3        # tie straddling the shard boundary
        logits[1, :] = -np.inf                              # every row -inf: index 0 wins
        logits[2, V - 1] = 2e3                              # max in the last shard
        logits[3, :] = -1.0                                 # +/-0 tie across the shard boundary:
        logits[3, half - 1] = -0.0                          # the lower index wins although it
        logits[3, half + 1] = 0.0                           # carries the minus sign
        v0, v1 = vs.shard_range(V, rank, world)
        mv, mi = _ref_argmax(logits[:, v0:v1])
        got_v, got_i = vs.combine_argmax(mv, mi + v0)
        want_v, want_i = _ref_argmax(logits)
        np.save(os.path.join(out_dir, f"r{rank}.npy"), np.stack([got_i, want_i]))
        assert np.array_equal(got_i, want_i), (got_i, want_i)
        assert np.array_equal(got_v, want_v)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_combine_across_gloo_ranks(world, tmp_path):
    import torch.multiprocessing as mp
    mp.start_processes(_rank_main, args=(world, _free_port(), 3, str(tmp_path)), nprocs=world,
                       start_method="spawn", join=True)
    r = [np.load(tmp_path / f"r{k}.npy") for k in range(world)]
    assert all(np.array_equal(r[0], x) for x in r)   # every rank agrees


class _NumpyModel:
    """Stand-in for edgecore_b200.Model on CPU tensors: 'hidden' = a fixed
    random embedding of (token, position), lm_head = a fixed random matrix."""

    def __init__(self, V, E, seed=0):
        rng = np.random.default_rng(seed)
        self.emb = rng.standard_normal((V, E)).astype(np.float32)
        self.W = rng.integers(-3, 4, (V, E)).astype(np.float32)   # integer logits: many exact ties
        self.v0, self.v1 = 0, V

    def set_vocab_shard(self, v0, v1):
        self.v0, self.v1 = v0, v1

    def hidden_np(self, tok, pos):
        return self.emb[tok] + np.float32(0.0) * pos[:, None]

    def batch_hidden(self, d_tok, d_pos, M, max_pos_end, out):
        import torch
        assert int(d_pos.max()) < max_pos_end
        out.copy_(torch.from_numpy(self.hidden_np(d_tok.numpy()[:M], d_pos.numpy()[:M])))

    def lm_shard_keys(self, hid, rows, keys):
        import torch
        lg = np.rint(hid.numpy()[:rows] @ self.W[self.v0:self.v1].T).astype(np.float32)
        mv, mi = _ref_argmax(lg)
        keys[:rows] = torch.from_numpy(vs.pack_keys(mv, mi + self.v0))

    def keys_advance(self, keys, M, d_tok, d_pos):
        import torch
        _, idx = vs.unpack_keys(keys.numpy()[:M])
        d_tok[:M] = torch.from_numpy(idx.astype(np.int32))
        d_pos[:M] += 1


def _batch_rank_main(rank: int, world: int, port: int, out_dir: str):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        V, E, M = 97, 6, 5
        model = _NumpyModel(V, E)
        dec = vs.ShardedBatchDecoder(model, rank, world, M, E, V)
        rng = np.random.default_rng(11)
        tok_all = rng.integers(0, V, world * M).astype(np.int32)
        tok = torch.from_numpy(tok_all[rank * M:(rank + 1) * M].copy())
        pos = torch.arange(M, dtype=torch.int32)
        ref = _NumpyModel(V, E)
        ref_tok = tok_all.copy()
        for _ in range(4):
            dec.step(tok, pos, int(pos.max()) + 1)
            lg = np.rint(ref.hidden_np(ref_tok, np.zeros(len(ref_tok))) @ ref.W.T).astype(np.float32)
            ref_tok = np.argmax(lg, axis=1).astype(np.int32)   # lowest index on ties
            assert np.array_equal(tok.numpy(), ref_tok[rank * M:(rank + 1) * M])
        np.save(os.path.join(out_dir, f"b{rank}.npy"), tok.numpy())
    finally:
        dist.destroy_process_group()


def test_sharded_batch_decoder_gloo(tmp_path):
    """Two ranks, each with its own streams and half of the vocab, agree with
    the unsharded greedy continuation of all streams."""
    import torch.multiprocessing as mp
    mp.start_processes(_batch_rank_main, args=(2, _free_port(), str(tmp_path)), nprocs=2,
                       start_method="spawn", join=True)
    assert all((tmp_path / f"b{k}.npy").exists() for k in range(2))
