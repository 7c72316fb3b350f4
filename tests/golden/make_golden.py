"""Generate the golden vectors under tests/golden/ from the REFERENCE itself.

Run where a checkout of the reference exists (the GPU machines have none):

    python tests/golden/make_golden.py [--reference <reference checkout>]

Sources of truth, all the reference's own code:
  * quant_export.npz  -- edgecore/ecm.py quantize_int8_symmetric (A1), imported
                         from the reference tree;
  * ops.npz           -- oracle/_ref/libecref.so (reference src/*.c compiled by
                         oracle/Makefile): linear() int8 incl. activation
                         quantisation, gemm_int8, gemm_fp16_fp32, gemm_bf16_fp32,
                         layernorm_rows, rmsnorm_rows, RoPE tables, gelu_new,
                         qwen_silu, f32_to_fp16;
  * models.npz        -- the same library on the seeded tiny .ecm models of
                         edgecore_b200.synth: prefill logits, per-layer
                         residual taps, greedy decode ids, batched decode;
  * abi_layout.json   -- tests/abi_probe.c compiled against the reference
                         src/edgecore.h.
The fixtures are small (< 1 MB) and committed; tests compare the CPU
restatement (oracle/ec_oracle.c) and the CUDA library against them.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parents[1]
sys.path.insert(0, str(ROOT))

from edgecore_b200 import synth  # noqa: E402
from oracle import oracle as orc  # noqa: E402

TINY = {
    "gpt2_int8": synth.TINY_GPT2,
    "gpt2_fp16": synth.TINY_GPT2.with_(precision="fp16"),
    "qwen2_int8": synth.TINY_QWEN2,
    "qwen2_fp16": synth.TINY_QWEN2.with_(precision="fp16"),
    "qwen2_bf16": synth.TINY_QWEN2.with_(precision="bf16"),
    "qwen2_yarn_sw_int8": synth.TINY_QWEN2.with_(sliding_window=5, rope_type="yarn", yarn_factor=4.0,
                                                 yarn_attention_factor=1.2),
    "qwen2_tied_int8": synth.TINY_QWEN2.with_(tie=1),
}
PROMPT = 11
DECODE = 8


def sha256(path: Path) -> str:
    return hashlib.sha256(path.read_bytes()).hexdigest()


def gen_quant_export(ref_root: Path) -> dict:
    sys.path.insert(0, str(ref_root))
    from edgecore.ecm import quantize_int8_symmetric as ref_q  # the reference exporter
    rng = np.random.default_rng(123)
    out = {}
    cases = {
        "normal": rng.standard_normal((37, 96)).astype(np.float32) * 0.02,
        "wide": rng.standard_normal((5, 1000)).astype(np.float32),
        "edge": np.array([[0, 0, 0, 0], [1.0, -1.0, 0.5, -0.5], [127, -127, 63.5, -63.5],
                          [1e-30, -2e-30, 3e-30, 0], [3.0, 3.0, -3.0, 1.5]], np.float32),
    }
    for k, w in cases.items():
        q, s = ref_q(w)
        out[f"{k}_w"], out[f"{k}_q"], out[f"{k}_s"] = w, q, s
    return out


def gen_ops(R: orc.Reference) -> dict:
    rng = np.random.default_rng(7)
    out = {}
    # linear() int8 branch incl. activation quant: (M, K, N), with/without bias
    for i, (M, K, N, bias) in enumerate([(1, 96, 40, True), (3, 40, 17, False), (8, 64, 33, True),
                                         (17, 48, 24, True), (2, 29, 5, False)]):
        X = rng.standard_normal((M, K)).astype(np.float32)
        if i == 1:
            X[1] = 0.0                       # all-zero row -> scale 1
            X[2, 3] = 1e4                    # one dominant value
        W = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)
        ws = rng.uniform(1e-3, 2e-2, N).astype(np.float32)
        b = rng.standard_normal(N).astype(np.float32) * 0.1 if bias else None
        y, q, qs = R.linear(0, W, X, ws, b)
        out.update({f"lin{i}_X": X, f"lin{i}_W": W, f"lin{i}_ws": ws, f"lin{i}_y": y, f"lin{i}_q": q,
                    f"lin{i}_qs": qs})
        if b is not None:
            out[f"lin{i}_b"] = b
    # gemm_int8 with raw int8 A, NULL scale / bias variants
    A = rng.integers(-128, 128, (4, 77), dtype=np.int64).astype(np.int8)
    B = rng.integers(-128, 128, (9, 77), dtype=np.int64).astype(np.int8)
    asc = rng.uniform(0.01, 0.1, 4).astype(np.float32)
    out.update(gi8_A=A, gi8_B=B, gi8_as=asc, gi8_y_noscale=R.gemm_int8(A, asc, B),
               gi8_bs=rng.uniform(0.01, 0.1, 9).astype(np.float32))
    out["gi8_y"] = R.gemm_int8(A, asc, B, out["gi8_bs"])
    # fp16 / bf16 GEMMs (K with and without an 8-lane tail)
    for K in (64, 29):
        X = rng.standard_normal((3, K)).astype(np.float32)
        W = (rng.standard_normal((11, K)) * 0.05).astype(np.float16)
        out[f"g16_{K}_X"], out[f"g16_{K}_W"] = X, W
        out[f"g16_{K}_y"] = R.gemm_fp16(X, W.view(np.uint16))
        Wb = (rng.standard_normal((11, K)).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
        out[f"gbf_{K}_W"], out[f"gbf_{K}_y"] = Wb, R.gemm_bf16(X, Wb)
    # norms
    x = (rng.standard_normal((4, 50)) * 3 + 0.5).astype(np.float32)
    g = rng.standard_normal(50).astype(np.float32)
    b = rng.standard_normal(50).astype(np.float32)
    out.update(norm_x=x, norm_g=g, norm_b=b, ln_y=R.layernorm(x, g, b, 1e-5), rms_y=R.rmsnorm(x, g, 1e-6))
    # RoPE tables
    pos = np.array([0, 1, 7, 100, 1023], np.int32)
    out["rope_pos"] = pos
    _, out["rope_cos"], out["rope_sin"] = R.rope_table(32, pos, 1e6)
    _, out["yarn_cos"], out["yarn_sin"] = R.rope_table(32, pos, 1e4, 1, 4.0, 2048.0, 1.2)
    # activations and fp16 rounding (RNE incl. subnormals, overflow, ties)
    v = np.concatenate([np.linspace(-8, 8, 257, dtype=np.float32),
                        np.array([0.0, -0.0, 1e-8, -3e-5, 6.1e-5, 65504, 65519.9, 65520, 1e6,
                                  2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -25, 1 + 2.0 ** -11,
                                  1 + 3 * 2.0 ** -11], np.float32)])
    out["act_x"] = v
    out["gelu_y"] = np.array([R.lib.ref_gelu(float(t)) for t in v], np.float32)
    out["silu_y"] = np.array([R.lib.ref_silu(float(t)) for t in v], np.float32)
    out["f2h"] = np.array([R.lib.ref_f32_to_fp16(float(t)) for t in v], np.uint16)
    return out


def gen_models(R: orc.Reference, cache: Path) -> tuple[dict, dict]:
    out, meta = {}, {}
    for key, spec in TINY.items():
        path = synth.ensure_model(spec, cache)
        meta[key] = {"sha256": sha256(path), "spec_key": synth.spec_key(spec)}
        m = R.open(path, batch_cap=2, max_ctx=0)
        toks = synth.prompt_ids(spec.vocab, PROMPT, seed=3)
        pos = np.arange(PROMPT, dtype=np.int32)
        seq0 = np.zeros(PROMPT, np.int32)
        logits, taps = m.forward_taps(toks, pos, seq0)
        out[f"{key}_prompt"], out[f"{key}_logits"], out[f"{key}_taps"] = toks, logits, taps
        # greedy decode, slot 0 (reference driver: src/runtime_main.c:293-352)
        m.reset()
        lg = m.forward(toks, pos, seq0)
        cur = int(toks[-1])
        ids, steps = [], []
        for i in range(DECODE):
            lg = m.forward(np.array([cur], np.int32), np.array([PROMPT + i], np.int32))
            cur = int(np.argmax(lg[0]))       # numpy argmax = first maximal index = strict '>'
            ids.append(cur)
            steps.append(lg[0])
        out[f"{key}_greedy"] = np.array(ids, np.int32)
        out[f"{key}_greedy_logits"] = np.stack(steps)
        # batched decode: two slots with different prompts, then M=2 steps (seqs NULL)
        m.reset()
        t2 = synth.prompt_ids(spec.vocab, 5, seed=9)
        m.forward(toks[:7], np.arange(7, dtype=np.int32), np.zeros(7, np.int32))
        m.forward(t2, np.arange(5, dtype=np.int32), np.ones(5, np.int32))
        cur2 = np.array([toks[6], t2[4]], np.int32)
        p2 = np.array([7, 5], np.int32)
        bl = []
        for i in range(3):
            lg = m.forward(cur2, p2)
            bl.append(lg)
            cur2 = np.argmax(lg, axis=1).astype(np.int32)
            p2 = p2 + 1
        out[f"{key}_batch_logits"] = np.stack(bl)
        m.close()
    return out, meta


def gen_layout(ref_root: Path) -> dict:
    with tempfile.TemporaryDirectory() as td:
        exe = Path(td) / "probe"
        subprocess.run(["/usr/bin/gcc", "-std=c11", "-mavx2", "-mf16c", "-I", str(ref_root / "src"),
                        str(ROOT / "tests" / "abi_probe.c"), "-o", str(exe)], check=True)
        return json.loads(subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=str(orc.REF_DIR),
                    help="reference checkout (default: $EDGECORE_REFERENCE, else a sibling of the repo)")
    args = ap.parse_args()
    ref_root = Path(args.reference)
    orc.build(reference=True)
    R = orc.Reference(threads=4)
    np.savez_compressed(HERE / "quant_export.npz", **gen_quant_export(ref_root))
    np.savez_compressed(HERE / "ops.npz", **gen_ops(R))
    with tempfile.TemporaryDirectory() as td:
        models, meta = gen_models(R, Path(td))
    np.savez_compressed(HERE / "models.npz", **models)
    (HERE / "models.json").write_text(json.dumps(meta, indent=1, sort_keys=True) + "\n")
    (HERE / "abi_layout.json").write_text(json.dumps(gen_layout(ref_root), indent=1) + "\n")
    for p in sorted(HERE.iterdir()):
        print(f"{p.name:24s} {p.stat().st_size:>9d} B")


if __name__ == "__main__":
    main()
