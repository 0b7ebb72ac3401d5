"""GGUF writer/reader and the synthetic-model quantisers."""
import os

import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O


def test_write_read_round_trip(tmp_path):
    arch = synth.tiny_arch(gguf.Q4_0, gguf.F16, hidden=64, layers=1, heads=2, kv_heads=1, ffn=64, vocab=300)
    p = synth.write_model(str(tmp_path / "m.gguf"), arch, seed=3)
    f = gguf.GgufFile(p)
    assert f.metadata["general.architecture"] == "llama"
    assert f.u64("llama.embedding_length") == 64
    assert abs(f.f64("llama.rope.freq_base") - 10000.0) < 1e-6
    assert len(f.metadata["tokenizer.ggml.tokens"]) == 300
    assert f.tensors["token_embd.weight"].ggml_type == gguf.F16
    assert f.tensors["blk.0.ffn_down.weight"].shape == (64, 64)
    assert f.tensors["blk.0.attn_k.weight"].shape == (64, 32)
    m = O.OracleModel(p)  # the reference's parse rules accept it
    assert (m.hidden, m.layers, m.heads, m.kv_heads, m.vocab) == (64, 1, 2, 1, 300)


@pytest.mark.parametrize("ggml_type,tol", [(gguf.Q8_0, 1 / 127), (gguf.Q4_0, 1 / 8), (gguf.F16, 1e-3)])
def test_quantisers_decode_close(ggml_type, tol):
    x = np.random.default_rng(0).standard_normal(32 * 64, dtype=np.float32)
    raw = np.frombuffer(synth.encode(x, ggml_type), dtype=np.uint8)
    y = O.dequant(ggml_type, raw, x.size)
    amax = np.abs(x.reshape(-1, 32)).max(axis=1, keepdims=True)
    assert np.all(np.abs((y - x).reshape(-1, 32)) <= tol * amax + 1e-6)
    assert np.array_equal(synth.dequantize(raw, ggml_type, x.size).view(np.uint32), y.view(np.uint32))


def test_q4_0_nibble_order_is_the_reference_decoders():
    # element o of a block lives in byte o/2: low nibble for even o, high for odd o
    x = np.zeros(32, dtype=np.float32)
    x[1] = -1.0  # the largest magnitude -> d = 1/8, q = 0 for element 1
    raw = np.frombuffer(synth.quantize_q4_0(x), dtype=np.uint8)
    assert raw[2] >> 4 == 0 and raw[2] & 15 == 8
    assert O.dequant(gguf.Q4_0, raw, 32)[1] == -1.0


def test_prompt_ids_are_seeded():
    a = synth.prompt_ids(49152, 128, seed=5)
    assert np.array_equal(a, synth.prompt_ids(49152, 128, seed=5))
    assert a.dtype == np.uint32 and a.max() < 49152


def test_gpt2_vocab_is_unique_and_padded():
    toks, merges = synth.gpt2_vocab(2000)
    assert len(toks) == 2000 and len(set(toks)) == 2000
    assert toks[-1] == "<|endoftext|>"
    assert all(len(m.split(" ")) == 2 for m in merges)
