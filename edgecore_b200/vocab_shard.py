"""Column-split lm_head across ranks (one process per GPU).

Each rank keeps the whole model but computes the lm_head only for its
contiguous block of vocab rows [v0, v1) (``Model.set_vocab_shard``), so a
greedy step reads 1/world of the 272 MB fp16 lm_head of Qwen2.5-0.5B per GPU.
A rank's forward returns, per token row, the best logit of its block and its
global vocab index (``Model.forward_argmax(..., shard=True)``).  The ranks
then agree on the global argmax with ONE all_reduce(MAX) of 64-bit keys:

    key = (order-preserving bits of the logit) << 32 | (0x7fffffff - index)

so the largest key is the largest logit and, among equal logits, the lowest
index -- the tie rule of the reference's greedy ``sample_token``
(src/runtime_main.c:213-219: strict ``>`` over ascending indices).  Keys are
the unsigned keys of ``ec_argmax_key`` (include/edgecore_b200.h) with the top
bit flipped, so that the signed int64 MAX of NCCL / gloo orders them the same
way.
"""
from __future__ import annotations

import numpy as np

__all__ = ["shard_range", "pack_keys", "unpack_keys", "combine_argmax", "ShardedGreedy", "ShardedBatchDecoder"]

_SIGN = np.uint64(1 << 63)


def shard_range(vocab: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous, balanced block of vocab rows owned by `rank`."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} not in [0, {world})")
    return vocab * rank // world, vocab * (rank + 1) // world


def pack_keys(maxv, idx) -> np.ndarray:
    """int64 keys whose signed order is (larger logit, then lower index)."""
    v = np.ascontiguousarray(maxv, dtype=np.float32)
    i = np.ascontiguousarray(idx, dtype=np.int64)
    if v.shape != i.shape:
        raise ValueError("maxv and idx must have the same shape")
    if np.any(i < 0) or np.any(i > 0x7FFFFFFF):
        raise ValueError("indices must be in [0, 2^31)")
    # -0.0 and +0.0 are equal to the reference's '>' scan: encode both as +0.0
    v = np.where(v == 0.0, np.float32(0.0), v).astype(np.float32)
    b = v.view(np.uint32).astype(np.uint64)
    b = np.where(b & np.uint64(0x80000000), ~b & np.uint64(0xFFFFFFFF), b | np.uint64(0x80000000))
    # a NaN never wins a '>' comparison: below every number
    b = np.where(np.isnan(v), np.uint64(0), b)
    key = (b << np.uint64(32)) | (np.uint64(0x7FFFFFFF) - i.astype(np.uint64))
    return (key ^ _SIGN).view(np.int64)


def unpack_keys(keys) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of pack_keys: (maxv float32, idx int32)."""
    k = np.ascontiguousarray(keys, dtype=np.int64).view(np.uint64) ^ _SIGN
    b = (k >> np.uint64(32)) & np.uint64(0xFFFFFFFF)
    b = np.where(b & np.uint64(0x80000000), b & np.uint64(0x7FFFFFFF), ~b & np.uint64(0xFFFFFFFF))
    maxv = b.astype(np.uint32).view(np.float32)
    idx = (np.uint64(0x7FFFFFFF) - (k & np.uint64(0xFFFFFFFF))).astype(np.int32)
    return maxv, idx


def combine_argmax(maxv, idx, group=None, device=None) -> tuple[np.ndarray, np.ndarray]:
    """Global (max logit, argmax index) per row from every rank's shard result.

    One all_reduce(MAX) over int64 keys on `group` (torch.distributed; NCCL
    needs `device`, a CUDA device of this rank; gloo works on CPU tensors).
    With no initialised process group the shard result is returned as is.
    """
    import torch
    import torch.distributed as dist

    keys = torch.from_numpy(pack_keys(maxv, idx))
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        t = keys.to(device) if device is not None else keys
        dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
        keys = t.cpu()
    return unpack_keys(keys.numpy())


class ShardedGreedy:
    """Greedy decoding with the lm_head column-split over the ranks of `group`.

    Wraps a loaded ``edgecore_b200.Model``: restricts its lm_head to this
    rank's vocab block, and returns, for host token/position arrays, the
    global greedy ids (identical on every rank).
    """

    def __init__(self, model, rank: int, world: int, group=None, device=None):
        self.model = model
        self.group = group
        self.device = device
        self.v0, self.v1 = shard_range(model.vocab, rank, world)
        model.set_vocab_shard(self.v0, self.v1)

    def step(self, tokens, positions, seqs=None) -> np.ndarray:
        ids, maxv = self.model.forward_argmax(tokens, positions, seqs, shard=True)
        _, gids = combine_argmax(maxv, ids, self.group, self.device)
        return gids


class ShardedBatchDecoder:
    """Batched greedy decode of many independent streams: the streams are
    split data-parallel over the ranks of `group` (each rank runs its own
    `m_local` slots through every layer), and the lm_head is column-split.

    One step on every rank, all on the current CUDA stream:

    1. ``batch_hidden``: this rank's slots through the layers and the final
       norm (normed rows [m_local][n_embd]);
    2. ``all_gather`` of those rows: every rank holds the rows of all
       world * m_local streams;
    3. ``lm_shard_keys``: this rank's vocab block of the lm_head over all the
       rows, each row's argmax packed as a signed 64-bit key;
    4. ``all_reduce(MAX)`` of the keys: every row's global greedy id, with the
       reference's tie rule (src/runtime_main.c:213-219);
    5. ``keys_advance``: this rank's slots take their ids, positions + 1.

    Compared with a full lm_head per rank, every rank reads 1/world of the
    lm_head weights, for the price of one all-gather of hidden rows and one
    all-reduce of 8 bytes per stream.  `model` is an ``edgecore_b200.Model``
    (or any object with those three methods, operating on torch tensors on
    this rank's device for NCCL, or on CPU for gloo).

    On a CUDA device the step runs on a stream of its own, to which the model
    is bound: the library's kernels, the torch copies and the collectives are
    then ordered on one stream (torch's default stream has the handle 0,
    which the library reads as "the model's own stream", so binding the
    model to it would not order anything).  The step waits for the caller's
    current stream on entry and makes it wait on exit.
    """

    def __init__(self, model, rank: int, world: int, m_local: int, n_embd: int, vocab: int, group=None,
                 device=None):
        import torch
        self.model, self.rank, self.world, self.m = model, rank, world, int(m_local)
        self.group = group
        self.v0, self.v1 = shard_range(vocab, rank, world)
        model.set_vocab_shard(self.v0, self.v1)
        dev = device if device is not None else "cpu"
        self.cuda = torch.device(dev).type == "cuda"
        self.stream = torch.cuda.Stream(device=dev) if self.cuda else None
        if self.cuda:
            model.set_stream(self.stream.cuda_stream)
        self.hid = torch.empty((self.m, n_embd), dtype=torch.float32, device=dev)
        self.hid_all = torch.empty((world * self.m, n_embd), dtype=torch.float32, device=dev)
        self.keys = torch.empty(world * self.m, dtype=torch.int64, device=dev)

    def step(self, d_tokens, d_positions, max_pos_end: int) -> None:
        """One greedy step of this rank's slots: d_tokens / d_positions
        (int32 [m_local]) are updated in place; every position must be below
        max_pos_end."""
        import contextlib

        import torch
        import torch.distributed as dist
        m = self.model
        if self.cuda:
            caller = torch.cuda.current_stream()
            self.stream.wait_stream(caller)
            ctx = torch.cuda.stream(self.stream)
        else:
            ctx = contextlib.nullcontext()
        with ctx:
            m.batch_hidden(d_tokens, d_positions, self.m, int(max_pos_end), self.hid)
            if self.world > 1:
                dist.all_gather_into_tensor(self.hid_all, self.hid, group=self.group)
            else:
                self.hid_all.copy_(self.hid)
            m.lm_shard_keys(self.hid_all, self.world * self.m, self.keys)
            if self.world > 1:
                dist.all_reduce(self.keys, op=dist.ReduceOp.MAX, group=self.group)
            mine = self.keys[self.rank * self.m:(self.rank + 1) * self.m]
            m.keys_advance(mine, self.m, d_tokens, d_positions)
        if self.cuda:
            caller.wait_stream(self.stream)
