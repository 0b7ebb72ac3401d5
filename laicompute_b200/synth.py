"""Synthetic Llama GGUF models (random-init weights of a named architecture).

There are no real checkpoints on the hardware this runs on, so every model is
built here from a fixed seed: 2-D weights are N(0, 0.02) float32, norm weights
are 1.0, then each tensor is encoded as F16, Q8_0 or Q4_0.

The quantisers are this package's own (the reference ships only decoders):

* Q8_0 — per 32 weights: ``d = amax / 127``, ``q = round(x / d)`` (half away
  from zero), ``d`` stored as binary16 (round-to-nearest-even).
* Q4_0 — per 32 weights: ``m`` = the weight of largest magnitude (signed),
  ``d = m / -8``, ``q = min(15, trunc(x / d + 8.5))``; ``d`` as binary16 (RNE).
  Nibbles are packed in the reference decoder's element order
  (``src/quant_v2.cpp:10``): element ``o`` of a block lives in byte ``o/2``,
  low nibble for even ``o``, high nibble for odd ``o``.
* F16 — numpy's float32 -> binary16 conversion (RNE).

Only the encoded bytes matter for parity: the engine and the oracle decode
the same file.
"""
from __future__ import annotations

import os
from dataclasses import dataclass, replace
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import gguf


@dataclass(frozen=True)
class LlamaArch:
    name: str
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    rope_theta: float = 10000.0
    rms_eps: float = 1e-5
    ctx: int = 2048
    weight_type: int = gguf.F16       # 2-D projection weights
    embed_type: Optional[int] = None  # token_embd (defaults to weight_type)
    tied: bool = True                 # no output.weight -> lm_head = token_embd
    output_type: Optional[int] = None
    rope_dim: Optional[int] = None

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def kv_dim(self) -> int:
        return self.kv_heads * self.head_dim


# The model shapes of the five workloads this engine is measured on.
SMOL_135M_F16 = LlamaArch("smollm-135m-f16", 576, 30, 9, 3, 1536, 49152, 10000.0, ctx=2048,
                          weight_type=gguf.F16)
SMOL_135M_Q8 = replace(SMOL_135M_F16, name="smollm-135m-q8_0", weight_type=gguf.Q8_0)
LLAMA_1B_Q4 = LlamaArch("llama-1b-q4_0", 2048, 16, 32, 8, 8192, 128256, 500000.0, ctx=8192,
                        weight_type=gguf.Q4_0, embed_type=gguf.F16)
LLAMA_8B_Q4 = LlamaArch("llama-8b-q4_0", 4096, 32, 32, 8, 14336, 128256, 500000.0, ctx=8192,
                        weight_type=gguf.Q4_0, embed_type=gguf.Q4_0)

ARCHS: Dict[str, LlamaArch] = {a.name: a for a in (SMOL_135M_F16, SMOL_135M_Q8, LLAMA_1B_Q4, LLAMA_8B_Q4)}


def tiny_arch(weight_type: int = gguf.F16, embed_type: Optional[int] = None, *, hidden: int = 128,
              layers: int = 2, heads: int = 4, kv_heads: int = 2, ffn: int = 256, vocab: int = 512,
              ctx: int = 256, rope_theta: float = 10000.0, tied: bool = True,
              output_type: Optional[int] = None, rope_dim: Optional[int] = None,
              name: str = "tiny") -> LlamaArch:
    """Small Llama shape for parity tests (the oracle finishes it in milliseconds)."""
    return LlamaArch(name, hidden, layers, heads, kv_heads, ffn, vocab, rope_theta, ctx=ctx,
                     weight_type=weight_type, embed_type=embed_type, tied=tied,
                     output_type=output_type, rope_dim=rope_dim)


# ----------------------------------------------------------------------------------
# quantisers
# ----------------------------------------------------------------------------------

def f32_to_f16_bytes(x: np.ndarray) -> bytes:
    return np.ascontiguousarray(x, dtype=np.float32).astype("<f2").tobytes()


def quantize_q8_0(x: np.ndarray) -> bytes:
    """Encode float32 values (length multiple of 32) as Q8_0 blocks (34 B each)."""
    b = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    amax = np.abs(b).max(axis=1)
    d = (amax / np.float32(127.0)).astype(np.float32)
    idv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, 1), 0).astype(np.float32)
    v = b * idv[:, None]
    q = np.clip(np.sign(v) * np.floor(np.abs(v) + np.float32(0.5)), -128, 127).astype(np.int8)
    out = np.empty((b.shape[0], 34), dtype=np.uint8)
    out[:, 0:2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q.view(np.uint8)
    return out.tobytes()


def quantize_q4_0(x: np.ndarray) -> bytes:
    """Encode float32 values as Q4_0 blocks (18 B) in the reference nibble order."""
    b = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.abs(b).argmax(axis=1)
    m = b[np.arange(b.shape[0]), idx]
    d = (m / np.float32(-8.0)).astype(np.float32)
    idv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, 1), 0).astype(np.float32)
    q = np.minimum(15, np.trunc(b * idv[:, None] + np.float32(8.5))).astype(np.uint8)
    out = np.empty((b.shape[0], 18), dtype=np.uint8)
    out[:, 0:2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
    out[:, 2:] = q[:, 0::2] | (q[:, 1::2] << 4)
    return out.tobytes()


def quantize_q5_0(x: np.ndarray) -> bytes:
    """Encode float32 values as Q5_0 blocks (22 B: fp16 d, 32 high bits, 16 nibble bytes) in the
    reference's order (src/quant_v2.cpp:12): element o is d * (v - 16), v = the nibble of byte
    o/2 (low for even o) with bit o of the high bits as its bit 4."""
    b = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, 32)
    idx = np.abs(b).argmax(axis=1)
    m = b[np.arange(b.shape[0]), idx]
    d = (m / np.float32(-16.0)).astype(np.float32)
    idv = np.where(d != 0, np.float32(1.0) / np.where(d != 0, d, 1), 0).astype(np.float32)
    v = np.minimum(31, np.trunc(b * idv[:, None] + np.float32(16.5))).astype(np.uint32)
    out = np.empty((b.shape[0], 22), dtype=np.uint8)
    out[:, 0:2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
    qh = ((v >> 4) << np.arange(32, dtype=np.uint32)).sum(axis=1, dtype=np.uint64).astype("<u4")
    out[:, 2:6] = qh.view(np.uint8).reshape(-1, 4)
    lo = (v & 15).astype(np.uint8)
    out[:, 6:] = lo[:, 0::2] | (lo[:, 1::2] << 4)
    return out.tobytes()


def encode(x: np.ndarray, ggml_type: int) -> bytes:
    if ggml_type == gguf.F32:
        return np.ascontiguousarray(x, dtype="<f4").tobytes()
    if ggml_type == gguf.F16:
        return f32_to_f16_bytes(x)
    if ggml_type == gguf.Q8_0:
        return quantize_q8_0(x)
    if ggml_type == gguf.Q4_0:
        return quantize_q4_0(x)
    if ggml_type == gguf.Q5_0:
        return quantize_q5_0(x)
    raise ValueError(f"no encoder for ggml type {ggml_type}")


def dequantize(raw: bytes | np.ndarray, ggml_type: int, n: int) -> np.ndarray:
    """Vectorised decoder with the reference's value rules (src/quant_v2.cpp:9-10)."""
    a = np.frombuffer(raw, dtype=np.uint8) if isinstance(raw, (bytes, bytearray)) else np.asarray(raw, np.uint8)
    if ggml_type == gguf.F32:
        return a[:4 * n].view("<f4").astype(np.float32)
    if ggml_type == gguf.F16:
        return a[:2 * n].view("<f2").astype(np.float32)
    if ggml_type == gguf.Q8_0:
        blk = a[: (n // 32) * 34].reshape(-1, 34)
        d = blk[:, 0:2].copy().view("<f2").astype(np.float32)
        q = blk[:, 2:].view(np.int8).astype(np.float32)
        return (d * q).reshape(-1)[:n]
    if ggml_type == gguf.Q4_0:
        blk = a[: (n // 32) * 18].reshape(-1, 18)
        d = blk[:, 0:2].copy().view("<f2").astype(np.float32)
        z = blk[:, 2:]
        q = np.empty((blk.shape[0], 32), dtype=np.float32)
        q[:, 0::2] = (z & 15).astype(np.float32) - 8
        q[:, 1::2] = (z >> 4).astype(np.float32) - 8
        return (d * q).reshape(-1)[:n]
    if ggml_type == gguf.Q5_0:
        blk = a[: (n // 32) * 22].reshape(-1, 22)
        d = blk[:, 0:2].copy().view("<f2").astype(np.float32)
        qh = blk[:, 2:6].copy().view("<u4").astype(np.uint32)
        z = blk[:, 6:]
        v = np.empty((blk.shape[0], 32), dtype=np.uint32)
        v[:, 0::2] = z & 15
        v[:, 1::2] = z >> 4
        v |= ((qh >> np.arange(32, dtype=np.uint32)) & 1) << 4
        return (d * (v.astype(np.float32) - 16)).reshape(-1)[:n]
    raise ValueError(f"no decoder for ggml type {ggml_type}")


# ----------------------------------------------------------------------------------
# tokenizer metadata
# ----------------------------------------------------------------------------------

def _byte_symbols() -> List[str]:
    """GPT-2 byte -> printable code point table (printable bytes map to themselves)."""
    direct = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    m = {b: b for b in direct}
    extra = 0
    for b in range(256):
        if b not in m:
            m[b] = 256 + extra
            extra += 1
    return [chr(m[b]) for b in range(256)]


def gpt2_vocab(vocab: int, specials: Tuple[str, ...] = ("<|endoftext|>",)) -> Tuple[List[str], List[str]]:
    """256 byte tokens, then merged pairs (and triples) padded to ``vocab`` entries.

    Merge ``i`` joins two existing tokens; its rank is its index. The last
    ``len(specials)`` ids are special ``<|...|>`` tokens.
    """
    syms = _byte_symbols()
    tokens = list(syms)
    merges: List[str] = []
    need = vocab - len(specials)
    seen = set(tokens)
    # pairs of byte symbols in a fixed order, then pair + byte
    order = list(range(256))
    for a in order:
        if len(tokens) >= need:
            break
        for b in order:
            if len(tokens) >= need:
                break
            t = syms[a] + syms[b]
            if t in seen:
                continue
            seen.add(t)
            tokens.append(t)
            merges.append(f"{syms[a]} {syms[b]}")
    i = 256
    while len(tokens) < need:
        base = tokens[i]
        for b in range(256):
            if len(tokens) >= need:
                break
            t = base + syms[b]
            if t in seen:
                continue
            seen.add(t)
            tokens.append(t)
            merges.append(f"{base} {syms[b]}")
        i += 1
    tokens.extend(specials)
    return tokens[:vocab], merges


# ----------------------------------------------------------------------------------
# model writer
# ----------------------------------------------------------------------------------

def tensor_names(layers: int, tied: bool) -> List[str]:
    names = ["token_embd.weight", "output_norm.weight"]
    if not tied:
        names.append("output.weight")
    for l in range(layers):
        for t in ("attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                  "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"):
            names.append(f"blk.{l}.{t}.weight")
    return names


def _shape_of(arch: LlamaArch, name: str) -> Tuple[int, ...]:
    """GGUF shape (ne0 = in) of each tensor."""
    h, kv, f, v = arch.hidden, arch.kv_dim, arch.ffn, arch.vocab
    base = name.split(".")[-2]
    return {
        "token_embd": (h, v), "output": (h, v), "output_norm": (h,),
        "attn_norm": (h,), "ffn_norm": (h,),
        "attn_q": (h, h), "attn_k": (h, kv), "attn_v": (h, kv), "attn_output": (h, h),
        "ffn_gate": (h, f), "ffn_up": (h, f), "ffn_down": (f, h),
    }[base]


def _type_of(arch: LlamaArch, name: str) -> int:
    base = name.split(".")[-2]
    if base in ("attn_norm", "ffn_norm", "output_norm"):
        return gguf.F32
    if base == "token_embd":
        return arch.embed_type if arch.embed_type is not None else arch.weight_type
    if base == "output":
        return arch.output_type if arch.output_type is not None else arch.weight_type
    return arch.weight_type


# byte -> byte with a zero nibble (value -8) replaced by 8 (value 0) in both halves
_Q4_NIB = np.where(np.arange(16) == 0, 8, np.arange(16)).astype(np.uint8)
_Q4_SYMMETRIC = (_Q4_NIB[np.arange(256) & 15] | (_Q4_NIB[np.arange(256) >> 4] << 4)).astype(np.uint8)


def random_blocks(n: int, ggml_type: int, rng: np.random.Generator, std: float = 0.02) -> bytes:
    """Q4_0 / Q8_0 blocks drawn directly (quants uniform and symmetric about zero,
    scales of the size a N(0, std) block quantises to), for models too large to
    quantise quickly. Q4_0 nibbles are uniform over 1..15 with 0 moved to 8, so the
    decoded values (n - 8) * d have mean zero like quantised N(0, std) weights."""
    nb = n // 32
    if ggml_type == gguf.Q4_0:
        d = np.float32(std * 2.2 / 8.0) * (np.float32(1.0) + np.float32(0.1) * rng.standard_normal(nb, dtype=np.float32))
        out = np.empty((nb, 18), dtype=np.uint8)
        out[:, 0:2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
        z = np.frombuffer(rng.bytes(nb * 16), dtype=np.uint8).reshape(nb, 16)
        out[:, 2:] = _Q4_SYMMETRIC[z]
        return out.tobytes()
    if ggml_type == gguf.Q8_0:
        d = np.float32(std * 2.2 / 127.0) * (np.float32(1.0) + np.float32(0.1) * rng.standard_normal(nb, dtype=np.float32))
        out = np.empty((nb, 34), dtype=np.uint8)
        out[:, 0:2] = d.astype("<f2").view(np.uint8).reshape(-1, 2)
        q = np.frombuffer(rng.bytes(nb * 32), dtype=np.int8).reshape(nb, 32)
        out[:, 2:] = np.maximum(q, -127).view(np.uint8)
        return out.tobytes()
    raise ValueError(f"no direct block generator for ggml type {ggml_type}")


def write_model(path: str, arch: LlamaArch, seed: int = 0, std: float = 0.02,
                bos: int | None = None, eos: int | None = None, direct_blocks: bool = False) -> str:
    """Write a synthetic Llama GGUF for ``arch``; returns ``path``.

    ``direct_blocks`` draws quantised tensors as random blocks instead of
    quantising N(0, std) values (same sizes and value range, much faster)."""
    rng = np.random.default_rng(seed)
    tokens, merges = gpt2_vocab(arch.vocab)
    eos_id = arch.vocab - 1 if eos is None else eos
    bos_id = arch.vocab - 1 if bos is None else bos
    md = {
        "general.architecture": "llama",
        "general.name": arch.name,
        "llama.embedding_length": arch.hidden,
        "llama.block_count": arch.layers,
        "llama.attention.head_count": arch.heads,
        "llama.attention.head_count_kv": arch.kv_heads,
        "llama.feed_forward_length": arch.ffn,
        "llama.context_length": arch.ctx,
        "llama.rope.dimension_count": arch.rope_dim if arch.rope_dim is not None else arch.head_dim,
        "llama.rope.freq_base": np.float32(arch.rope_theta),
        "llama.attention.layer_norm_rms_epsilon": np.float32(arch.rms_eps),
        "tokenizer.ggml.model": "gpt2",
        "tokenizer.ggml.tokens": tokens,
        "tokenizer.ggml.merges": merges,
        "tokenizer.ggml.bos_token_id": bos_id,
        "tokenizer.ggml.eos_token_id": eos_id,
        "tokenizer.ggml.add_bos_token": False,
    }
    tensors = []
    for name in tensor_names(arch.layers, arch.tied):
        shape = _shape_of(arch, name)
        gt = _type_of(arch, name)
        n = int(np.prod(shape))
        if len(shape) == 1:
            x = np.ones(n, dtype=np.float32)
        elif direct_blocks and gt in (gguf.Q4_0, gguf.Q8_0):
            tensors.append((name, shape, gt, random_blocks(n, gt, rng, std)))
            continue
        else:
            x = (rng.standard_normal(n, dtype=np.float32) * np.float32(std)).astype(np.float32)
        tensors.append((name, shape, gt, encode(x, gt)))
    os.makedirs(os.path.dirname(os.path.abspath(path)), exist_ok=True)
    gguf.write_gguf(path, md, tensors)
    return path


def prompt_ids(vocab: int, n: int, seed: int) -> np.ndarray:
    """Prompt of ``n`` token ids uniform over [0, vocab) from a fixed seed."""
    return np.random.default_rng(seed).integers(0, vocab, size=n, dtype=np.int64).astype(np.uint32)
