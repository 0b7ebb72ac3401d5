"""Generate the golden fixtures of tests/golden/ by running the REFERENCE itself.

Requires oracle/_ref/laic_ref_driver (oracle/Makefile compiles it from the
reference sources). Writes:

  tiny_*.gguf            small synthetic Llama models (committed)
  tiny_*.npz             reference outputs on them: logits of every step() call,
                         generated ids for four sampling settings, and the
                         reference dequantisation of three tensors (first 2048
                         values and the sha256 of the whole float32 array)
  generate_text.json     the reference's public generate_ids path (text prompt ->
                         chat-template wrap, tokenizer, BOS, prompt steps, sampling,
                         EOS stop) on the tiny models: greedy and sampled ids, and
                         for the sampled ones the per-step distance of the draw
                         from a decision boundary (from the reference's logits)
  smollm135m_*.npz       reference outputs on the 135M-shaped models of the
                         benchmark workloads (the GGUF is regenerated from its
                         seed by laicompute_b200.synth; its sha256 is recorded):
                         ids, per-step argmax / max / top-2 margin / sum and
                         the first 64 logits

  blocks.npz             the reference's decode (quant_v2::value) of random and
                         edge-case blocks of Q4_1, Q5_0, Q5_1 and Q4_0 (the raw
                         blocks and the float32 values)

Run from the repository root:  python tests/golden/make_golden.py [generate|blocks]
("generate" writes only generate_text.json, "blocks" only blocks.npz).
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


GEN_PROMPTS = ("Hello world", "The B200 decodes one token at a time.")
# Sampled cases keep top_k = 0: with 0 < top_k < vocab and top_p = 1 the reference
# walks the unspecified order std::nth_element leaves behind.
GEN_CONFIGS = ({"max_tokens": 16},
               {"max_tokens": 16, "temperature": 1.0, "top_k": 0, "top_p": 1.0, "repeat_penalty": 1.0, "seed": 7},
               {"max_tokens": 16, "temperature": 0.7, "top_k": 0, "top_p": 0.9, "repeat_penalty": 1.3, "seed": 99})


def _generate_prompt_ids(path: str, text: str) -> list:
    """The prompt ids generate_ids builds (src/inference_v2.cpp:34): chat-template wrap, encode, BOS."""
    meta = gguf.GgufFile(path).metadata
    if "<|im_start|>" in str(meta.get("tokenizer.chat_template", "")) and "<|im_start|>" not in text:
        text = "<|im_start|>user\n" + text + "<|im_end|>\n<|im_start|>assistant\n"
    out = subprocess.run([O.ref_driver("strict"), "encode", path, text], check=True, capture_output=True, text=True)
    ids = [int(v) for v in out.stdout.split()]
    bos = meta.get("tokenizer.ggml.bos_token_id")
    if meta.get("tokenizer.ggml.add_bos_token", False) and ids and ids[0] != bos:
        ids.insert(0, bos)
    return ids


def _sample_margins(logits: np.ndarray, history: list, cfg: dict, ids: list) -> tuple:
    """Per generated step, how far the reference's draw sits from a decision boundary of
    sample() (src/inference_v2.cpp:32, top_k = 0): the smallest distance of u from the
    candidate CDF and of top_p from the cumulative mass around its cut (probability
    units), and max|logit| / temperature (the scale a logit error is divided by)."""
    u = O.canonical_u(cfg["seed"])
    T, pen, top_p = cfg["temperature"], cfg["repeat_penalty"], cfg["top_p"]
    hist = list(history)
    margins, scales = [], []
    for s, tok in enumerate(ids):
        l = logits[s].astype(np.float32).copy()
        if pen != 1.0:
            for h in hist:  # once per history entry, repeats included
                l[h] = l[h] / np.float32(pen) if l[h] >= 0 else l[h] * np.float32(pen)
        z = np.exp((l.astype(np.float64) - float(l.max())) / T)
        p = z / z.sum()
        order = np.arange(len(p))
        m = np.inf
        if top_p < 1.0:
            order = np.argsort(-p, kind="stable")
            acc = np.cumsum(p[order])
            keep = int(np.searchsorted(acc, top_p, side="left")) + 1
            m = min(m, abs(acc[keep - 1] - top_p), abs(acc[keep - 2] - top_p) if keep > 1 else np.inf)
            order = order[:keep]
        q = p[order] / p[order].sum()
        m = min(m, float(np.min(np.abs(np.cumsum(q) - u))))
        margins.append(float(m))
        scales.append(float(np.abs(l).max() / T))
        hist.append(tok)
    return margins, scales


def make_generate() -> None:
    """Reference generate_ids on text prompts (its own tokenizer, template and EOS stop),
    with the per-step decision margins of the sampled cases from the reference's logits."""
    import json
    exe = O.ref_driver("strict")
    cases = []
    for name in sorted(TINY):
        path = os.path.join(HERE, name + ".gguf")
        for text in GEN_PROMPTS:
            for cfg in GEN_CONFIGS:
                args = [exe, "generate", path, text, "--max-tokens", str(cfg["max_tokens"])]
                for k, flag in (("temperature", "--temperature"), ("top_k", "--top-k"), ("top_p", "--top-p"),
                                ("repeat_penalty", "--repeat-penalty"), ("seed", "--seed")):
                    if k in cfg:
                        args += [flag, str(cfg[k])]
                out = subprocess.run(args, check=True, capture_output=True, text=True).stdout.split()
                case = {"model": name, "prompt": text, **cfg, "ids": [int(v) for v in out]}
                if "temperature" in cfg:
                    prompt = _generate_prompt_ids(path, text)
                    sp = O.params(cfg["temperature"], cfg["top_k"], cfg["top_p"], cfg["repeat_penalty"], cfg["seed"])
                    dids, logits, _ = O.ref_dump(path, np.array(prompt, dtype=np.uint32), cfg["max_tokens"], sp)
                    n = len(case["ids"])
                    assert dids[:n].tolist() == case["ids"], "step loop and generate_ids disagree"
                    case["margin"], case["scale"] = _sample_margins(logits[len(prompt) - 1:], prompt, cfg,
                                                                    case["ids"])
                cases.append(case)
    with open(os.path.join(HERE, "generate_text.json"), "w") as f:
        json.dump(cases, f, indent=1)
    print("generate_text.json:", len(cases), "cases")


# block bytes, offset of the nibbles, offset of the 32 high bits (Q5_*), and the number of fp16
# scales in front of them
BLOCK_TYPES = {"q4_1": (gguf.Q4_1, 20, 4, None, 2), "q5_0": (gguf.Q5_0, 22, 6, 2, 1),
               "q5_1": (gguf.Q5_1, 24, 8, 4, 2), "q4_0": (gguf.Q4_0, 18, 2, None, 1)}
EDGE_HALVES = [0x0001, 0x03FF, 0x0400, 0x7BFF, 0x8000, 0x0000, 0xFBFF, 0x3C00, 0xBC00, 0x2E66]


def random_blocks(kind: str, nblocks: int, rng: np.random.Generator) -> bytes:
    """Random blocks (scales of modest size, edge-case scales in the first blocks)."""
    gt, bb, qoff, hoff, nsc = BLOCK_TYPES[kind]
    raw = rng.integers(0, 256, size=(nblocks, bb), dtype=np.uint8)
    scales = (rng.uniform(1e-3, 5e-2, size=(nblocks, nsc)) * rng.choice([-1, 1], size=(nblocks, nsc)))
    h = scales.astype(np.float16).view(np.uint16)
    for i, e in enumerate(EDGE_HALVES):  # edge scales (subnormal, max, signed zero, ...) in the first blocks
        h[i % nblocks, i % nsc] = e
    raw[:, :2 * nsc] = h.astype("<u2").view(np.uint8).reshape(nblocks, 2 * nsc)
    return raw.tobytes()


def make_blocks() -> None:
    rng = np.random.default_rng(2024)
    nblocks = 96
    tensors, out = [], {}
    for kind, (gt, bb, _, _, _) in BLOCK_TYPES.items():
        raw = random_blocks(kind, nblocks, rng)
        tensors.append((f"blocks.{kind}", (32 * nblocks,), gt, raw))
        out[f"raw_{kind}"] = np.frombuffer(raw, dtype=np.uint8)
    with tempfile.TemporaryDirectory() as d:
        path = os.path.join(d, "blocks.gguf")
        gguf.write_gguf(path, {"general.architecture": "llama", "general.name": "blocks"}, tensors)
        for kind in BLOCK_TYPES:
            out[f"value_{kind}"] = ref_dequant(path, f"blocks.{kind}")
    np.savez_compressed(os.path.join(HERE, "blocks.npz"), **out)
    print("blocks.npz", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    if O.ref_driver("strict") is None:
        O.build()
    if len(sys.argv) > 1 and sys.argv[1] == "generate":
        make_generate()
        sys.exit(0)
    if len(sys.argv) > 1 and sys.argv[1] == "blocks":
        make_blocks()
        sys.exit(0)
    make_blocks()
    make_tiny()
    make_generate()
    work = tempfile.mkdtemp(prefix="laic_golden_")
    try:
        make_smollm(work)
    finally:
        import shutil
        shutil.rmtree(work, ignore_errors=True)
