"""Decode attention over the FP16 KV cache at head dims 64 and 128 and at
contexts that span several 128-position chunks and several splits: logits
against the oracle (CPU restatement of LlamaRuntime::step, reference
src/inference_v2.cpp:31), and batched runs against single-sequence runs."""
import os

import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


def _model(tmp_path, name, **kw):
    arch = synth.tiny_arch(gguf.Q8_0, gguf.F16, name=name, **kw)
    return arch, synth.write_model(os.path.join(str(tmp_path), name + ".gguf"), arch, seed=31)


@pytest.mark.parametrize("hidden,heads,kv_heads", [(256, 2, 1), (512, 4, 1), (256, 4, 2)])
def test_long_context_matches_oracle(tmp_path, hidden, heads, kv_heads):
    """Head dim 128 (groups of 2 and 4) and 64; a 400-token prompt spans four chunks."""
    from laicompute_b200.engine import Engine
    arch, path = _model(tmp_path, f"attn_{hidden}_{heads}_{kv_heads}", hidden=hidden, layers=2, heads=heads,
                        kv_heads=kv_heads, ffn=256, vocab=512, ctx=1024)
    prompt = synth.prompt_ids(arch.vocab, 400, seed=32)
    ref_ids, ref_logits = O.OracleModel(path).generate(prompt, 24)
    e = Engine(path, kv_capacity=1024)
    ids, logits = e.generate(prompt, 24, want_logits=True)
    err = np.abs(logits - ref_logits).max(axis=1) / np.abs(ref_logits).max(axis=1)
    assert err.max() <= LOGIT_RTOL, err
    assert np.array_equal(ids, ref_ids)
    e.close()


def test_batched_multi_chunk_splits_match_single_sequences(tmp_path):
    """50 sequences x 2 KV heads at ~700 positions: fewer splits than chunks, so
    one CTA walks two chunks; each sequence must match its single-sequence run."""
    from laicompute_b200.engine import Engine
    arch, path = _model(tmp_path, "attn_batch", hidden=256, layers=2, heads=4, kv_heads=2, ffn=256, vocab=512,
                        ctx=1024)
    nseq, plen = 50, 700
    prompts = np.stack([synth.prompt_ids(arch.vocab, plen, seed=100 + i) for i in range(nseq)])
    slots = np.arange(nseq, dtype=np.int32)
    e = Engine(path, max_seqs=nseq, kv_capacity=1024)
    for j in range(plen - 1):
        e.prefill(prompts[:, j], slots)
    _, batched = e.step(prompts[:, -1], slots, want_logits=True)
    e.close()
    for i in (0, 17, 49):
        e1 = Engine(path, kv_capacity=1024)
        for t in prompts[i, :-1]:
            e1.prefill([t], [0])
        _, single = e1.step([prompts[i, -1]], [0], want_logits=True)
        e1.close()
        # the one-sequence engine runs its projections with integer dot products, the batched one with
        # binary16 hi/lo products: both are FP32-accurate, not identical
        err = np.abs(batched[i] - single[0]).max() / np.abs(single[0]).max()
        assert err <= 1e-4, (i, err)
