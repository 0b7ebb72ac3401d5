"""Generate the golden fixtures of tests/golden/ by running the REFERENCE itself.

Requires oracle/_ref/laic_ref_driver (oracle/Makefile compiles it from the
reference sources). Writes:

  tiny_*.gguf            small synthetic Llama models (committed)
  tiny_*.npz             reference outputs on them: logits of every step() call,
                         generated ids for four sampling settings, and the
                         reference dequantisation of three tensors (first 2048
                         values and the sha256 of the whole float32 array)
  smollm135m_*.npz       reference outputs on the 135M-shaped models of the
                         benchmark workloads (the GGUF is regenerated from its
                         seed by laicompute_b200.synth; its sha256 is recorded):
                         ids, per-step argmax / max / top-2 margin / sum and
                         the first 64 logits

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from laicompute_b200 import gguf, synth  # noqa: E402
from oracle import oracle as O  # noqa: E402

TINY = {
    "tiny_f16": synth.tiny_arch(gguf.F16, hidden=64, layers=2, heads=2, kv_heads=1, ffn=128, vocab=320,
                                name="tiny_f16"),
    "tiny_q8": synth.tiny_arch(gguf.Q8_0, hidden=192, layers=2, heads=3, kv_heads=1, ffn=96, vocab=320,
                               name="tiny_q8"),
    "tiny_q4": synth.tiny_arch(gguf.Q4_0, gguf.F16, hidden=256, layers=2, heads=2, kv_heads=1, ffn=128, vocab=320,
                               rope_theta=500000.0, name="tiny_q4"),
}
TINY_SEED = {"tiny_f16": 11, "tiny_q8": 12, "tiny_q4": 13}
PROMPT_LEN, STEPS = 6, 10

# (name, temperature, top_k, top_p, repeat_penalty, seed)
CASES = [
    ("greedy", 0.0, 0, 1.0, 1.0, 0),
    ("topk", 0.8, 40, 1.0, 1.0, 1234),
    ("topp_pen", 0.7, 0, 0.9, 1.3, 99),
    ("full", 1.0, 0, 1.0, 1.0, 7),
]


def sha256(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 20), b""):
            h.update(chunk)
    return h.hexdigest()


def ref_dequant(model: str, tensor: str) -> np.ndarray:
    exe = O.ref_driver("strict")
    with tempfile.NamedTemporaryFile(suffix=".f32") as f:
        subprocess.run([exe, "dequant", model, tensor, f.name], check=True)
        return np.fromfile(f.name, dtype=np.float32)


def make_tiny() -> None:
    for name, arch in TINY.items():
        path = os.path.join(HERE, name + ".gguf")
        synth.write_model(path, arch, seed=TINY_SEED[name])
        prompt = synth.prompt_ids(arch.vocab, PROMPT_LEN, seed=TINY_SEED[name] + 100)
        out = {"prompt": prompt, "sha256": np.frombuffer(bytes.fromhex(sha256(path)), dtype=np.uint8)}
        for case, t, k, p, rp, seed in CASES:
            ids, logits, info = O.ref_dump(path, prompt, STEPS, O.params(t, k, p, rp, seed))
            out[f"ids_{case}"] = ids
            if case == "greedy":
                out["logits_greedy"] = logits
                out["l1_tile_bytes"] = np.array([info["l1_tile_bytes"]], dtype=np.int64)
        for tname in ("blk.0.attn_q.weight", "blk.1.ffn_down.weight", "token_embd.weight"):
            v = ref_dequant(path, tname)
            key = tname.replace(".weight", "").replace(".", "_")
            out[f"dequant_{key}_head"] = v[:2048]
            out[f"dequant_{key}_sha256"] = np.frombuffer(hashlib.sha256(v.tobytes()).digest(), dtype=np.uint8)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        print(name, os.path.getsize(path), "bytes gguf")


def summarize(logits: np.ndarray, keep: int = 64) -> dict:
    top2 = np.sort(logits, axis=1)[:, -2:]
    return {
        "argmax": logits.argmax(axis=1).astype(np.int64),
        "max": logits.max(axis=1),
        "margin": (top2[:, 1] - top2[:, 0]).astype(np.float32),
        "sum": logits.astype(np.float64).sum(axis=1),
        "head": logits[:, :keep].copy(),
    }


def make_smollm(workdir: str) -> None:
    """135M-shaped F16 (prompt 8, 32 greedy) and Q8_0 (prompt 128, 32 greedy + 32 top-k) references."""
    specs = [
        ("smollm135m_f16", synth.SMOL_135M_F16, 1, 8, 32, [("greedy", 0.0, 0, 1.0, 1.0, 0)]),
        ("smollm135m_q8", synth.SMOL_135M_Q8, 2, 128, 32,
         [("greedy", 0.0, 0, 1.0, 1.0, 0), ("topk", 0.8, 40, 1.0, 1.0, 4242)]),
    ]
    for name, arch, seed, plen, steps, cases in specs:
        path = os.path.join(workdir, name + ".gguf")
        synth.write_model(path, arch, seed=seed)
        prompt = synth.prompt_ids(arch.vocab, plen, seed=seed + 100)
        out = {"prompt": prompt, "seed": np.array([seed]), "steps": np.array([steps]),
               "sha256": np.frombuffer(bytes.fromhex(sha256(path)), dtype=np.uint8)}
        for case, t, k, p, rp, s in cases:
            ids, logits, info = O.ref_dump(path, prompt, steps, O.params(t, k, p, rp, s))
            out[f"ids_{case}"] = ids
            if case == "greedy":
                for key, v in summarize(logits).items():
                    out[f"{key}"] = v
                out["l1_tile_bytes"] = np.array([info["l1_tile_bytes"]], dtype=np.int64)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **out)
        print(name, "done")


if __name__ == "__main__":
    if O.ref_driver("strict") is None:
        O.build()
    make_tiny()
    work = tempfile.mkdtemp(prefix="laic_golden_")
    try:
        make_smollm(work)
    finally:
        import shutil
        shutil.rmtree(work, ignore_errors=True)
