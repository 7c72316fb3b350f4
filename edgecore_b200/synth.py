"""Seeded synthetic .ecm models with the shapes of the benchmark configurations.

No checkpoints or datasets are available, so every model is random-init:
weights N(0, 0.02) in fp32 from ``numpy.random.default_rng(seed)``, stored as
fp16 / bf16, or quantised to int8 per output row with
``ecm.quantize_int8_symmetric``.  Norm gains are 1 and biases 0 unless
``norm_noise`` asks for random ones (the tiny test models do, so that the gain
and bias paths are exercised).  Qwen2 q/k/v biases are written as the Qwen2.5
checkpoints have them; the reference forward does not read them
(src/gpt2.c:709-711 passes NULL), and neither does this library.

The tokenizer blobs are a byte-level vocabulary of at most 256 entries and no
merges, which the reference tokenizer_load accepts for any vocab size
(src/tokenizer.c:925-1015); prompts are token ids, never text.
"""
from __future__ import annotations

import hashlib
import json
import os
import struct
from dataclasses import asdict, dataclass, replace
from pathlib import Path

import numpy as np

from .ecm import EcmWriter, quantize_int8_symmetric


@dataclass(frozen=True)
class ModelSpec:
    name: str
    arch: str                 # "gpt2" | "qwen2"
    precision: str            # "int8" | "fp16" | "bf16"
    n_layer: int
    n_embd: int
    n_head: int
    vocab: int
    n_ctx: int
    n_kv_head: int = 0        # qwen2 only
    intermediate: int = 0     # qwen2 only
    eps: float = 1e-5
    rope_theta: float = 1e6
    tie: int = 1
    qkv_bias: bool = False
    sliding_window: int = 0
    rope_type: str = "default"
    yarn_factor: float = 1.0
    yarn_attention_factor: float = 1.0
    std: float = 0.02
    norm_noise: float = 0.0
    seed: int = 0

    def with_(self, **kw) -> "ModelSpec":
        return replace(self, **kw)

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    @property
    def kv_embd(self) -> int:
        return (self.n_kv_head or self.n_head) * self.head_dim if self.arch == "qwen2" else self.n_embd


# BASELINE configurations (shapes only; everything random-init, seed 0).
GPT2_SMALL = ModelSpec("gpt2-small-synth", "gpt2", "int8", 12, 768, 12, 50257, 1024)
QWEN25_05B = ModelSpec("qwen2.5-0.5b-synth", "qwen2", "int8", 24, 896, 14, 151936, 32768,
                       n_kv_head=2, intermediate=4864, eps=1e-6, rope_theta=1e6, tie=1,
                       qkv_bias=True)
QWEN25_15B = ModelSpec("qwen2.5-1.5b-synth", "qwen2", "int8", 28, 1536, 12, 151936, 32768,
                       n_kv_head=2, intermediate=8960, eps=1e-6, rope_theta=1e6, tie=1,
                       qkv_bias=True)
# The reference smoke-test shapes (scripts/make_synthetic.py defaults) with
# random gains, for fast parity tests.
TINY_GPT2 = ModelSpec("tiny-gpt2", "gpt2", "int8", 2, 32, 2, 256, 64, norm_noise=0.1)
TINY_QWEN2 = ModelSpec("tiny-qwen2", "qwen2", "int8", 2, 32, 2, 256, 64, n_kv_head=1,
                       intermediate=48, eps=1e-6, tie=0, qkv_bias=True, norm_noise=0.1)

CONFIGS = {
    "c0_gpt2_small_int8": GPT2_SMALL,
    "c2_qwen05b_fp16": QWEN25_05B.with_(precision="fp16"),
    "c3_qwen05b_int8": QWEN25_05B,
    "c4_qwen15b_int8": QWEN25_15B,
}


def byte_vocab_blob(vocab: int) -> bytes:
    n = min(vocab, 256)
    out = bytearray(struct.pack("<I", n))
    for i in range(n):
        out += struct.pack("<II", i, 1) + bytes([i])
    return bytes(out)


def _linear(wr: EcmWriter, rng: np.random.Generator, spec: ModelSpec, name: str,
            rows: int, cols: int, bias: bool) -> int:
    w = rng.standard_normal((rows, cols), dtype=np.float32) * np.float32(spec.std)
    if spec.precision == "int8":
        q, s = quantize_int8_symmetric(w)
        wr.add(f"{name}.w", "int8", q)
        wr.add(f"{name}.s", "fp32", s)
    else:
        wr.add(f"{name}.w", spec.precision, w)
    if bias:
        wr.add(f"{name}.b", "fp32", rng.standard_normal(rows, dtype=np.float32) * np.float32(spec.std))
    return rows * cols + (rows if bias else 0)


def _gain(rng: np.random.Generator, spec: ModelSpec, n: int, base: float) -> np.ndarray:
    if spec.norm_noise:
        return (base + spec.norm_noise * rng.standard_normal(n)).astype(np.float32)
    return np.full(n, base, dtype=np.float32)


def build(spec: ModelSpec) -> EcmWriter:
    """Build the EcmWriter for `spec` (deterministic in spec.seed)."""
    rng = np.random.default_rng(spec.seed)
    E, L, V, C = spec.n_embd, spec.n_layer, spec.vocab, spec.n_ctx
    emb_dtype = "bf16" if spec.precision == "bf16" else "fp16"
    wr = EcmWriter()
    meta = dict(model_name=spec.name, n_layer=L, n_head=spec.n_head, n_embd=E, n_ctx=C,
                vocab=V, eps=spec.eps, arch=spec.arch)
    if spec.arch == "qwen2":
        meta.update(n_kv_head=spec.n_kv_head or spec.n_head, intermediate=spec.intermediate,
                    rope_theta=spec.rope_theta, rope_type=spec.rope_type,
                    yarn_factor=spec.yarn_factor, yarn_orig_max=C,
                    yarn_attention_factor=spec.yarn_attention_factor,
                    sliding_window=spec.sliding_window, tie_word_embeddings=spec.tie,
                    eos_token_id=V - 1)
    wr.set_meta(**meta)
    n_params = 0
    wte = rng.standard_normal((V, E), dtype=np.float32) * np.float32(spec.std)
    wr.add("wte", emb_dtype, wte)
    n_params += V * E
    if spec.arch == "gpt2":
        wr.add("wpe", emb_dtype, rng.standard_normal((C, E), dtype=np.float32) * np.float32(spec.std))
        n_params += C * E
    elif not spec.tie:
        wr.add("lm_head.w", emb_dtype, rng.standard_normal((V, E), dtype=np.float32) * np.float32(spec.std))
        n_params += V * E
    wr.add("ln_f.g", "fp32", _gain(rng, spec, E, 1.0))
    if spec.arch == "gpt2":
        wr.add("ln_f.b", "fp32", _gain(rng, spec, E, 0.0))
    for l in range(L):
        p = f"blocks.{l}"
        wr.add(f"{p}.ln_1.g", "fp32", _gain(rng, spec, E, 1.0))
        if spec.arch == "gpt2":
            wr.add(f"{p}.ln_1.b", "fp32", _gain(rng, spec, E, 0.0))
        wr.add(f"{p}.ln_2.g", "fp32", _gain(rng, spec, E, 1.0))
        if spec.arch == "gpt2":
            wr.add(f"{p}.ln_2.b", "fp32", _gain(rng, spec, E, 0.0))
            for sfx, (r, c) in {"attn": (3 * E, E), "proj": (E, E), "fc": (4 * E, E),
                                "fc2": (E, 4 * E)}.items():
                n_params += _linear(wr, rng, spec, f"{p}.{sfx}", r, c, bias=True)
        else:
            kv, I = spec.kv_embd, spec.intermediate
            for sfx, (r, c) in {"q": (E, E), "k": (kv, E), "v": (kv, E), "o": (E, E),
                                "gate": (I, E), "up": (I, E), "down": (E, I)}.items():
                n_params += _linear(wr, rng, spec, f"{p}.{sfx}", r, c,
                                    bias=spec.qkv_bias and sfx in ("q", "k", "v"))
    wr.add("tokenizer.vocab", "text", np.frombuffer(byte_vocab_blob(V), dtype=np.uint8))
    wr.add("tokenizer.merges", "text", np.frombuffer(struct.pack("<I", 0), dtype=np.uint8))
    wr.set_meta(n_params=n_params)
    return wr


def spec_key(spec: ModelSpec) -> str:
    return hashlib.sha1(json.dumps(asdict(spec), sort_keys=True).encode()).hexdigest()[:12]


def ensure_model(spec: ModelSpec, cache_dir: str | os.PathLike | None = None) -> Path:
    """Write `spec` to `<cache_dir>/<name>-<precision>-<hash>.ecm` unless present."""
    cache = Path(cache_dir or os.environ.get("EDGECORE_B200_MODEL_CACHE", "/tmp/edgecore_b200_models"))
    path = cache / f"{spec.name}-{spec.precision}-{spec_key(spec)}.ecm"
    if not path.exists():
        build(spec).save(path)
    return path


def prompt_ids(vocab: int, n: int, seed: int = 0) -> np.ndarray:
    """Uniform-random prompt token ids in [0, vocab)."""
    return np.random.default_rng(seed + 1).integers(0, vocab, size=n, dtype=np.int64).astype(np.int32)
