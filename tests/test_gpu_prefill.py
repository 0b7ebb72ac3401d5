"""Batched prompt prefill (laic_dev_prefill_batch: all prompt tokens through
every layer together, projections as fp16 tensor-core GEMMs) against the
reference's outputs and the oracle: the decode logits that follow stay within
1e-3 of max|logit| and the greedy ids are identical."""
import os
import tempfile

import numpy as np
import pytest

from conftest import TINY_MODELS, golden, golden_model
from laicompute_b200 import gguf, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


@pytest.mark.parametrize("name", TINY_MODELS)
def test_batched_prefill_matches_reference(name):
    from laicompute_b200.engine import Engine
    g = golden(name)
    steps = len(g["ids_greedy"])
    e = Engine(golden_model(name))
    ids, logits = e.generate(g["prompt"], steps, want_logits=True, batched_prefill=True)
    assert e.slot_pos(0) == len(g["prompt"]) + steps - 1
    e.close()
    ref = g["logits_greedy"][len(g["prompt"]) - 1:]
    err = np.abs(logits - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert err.max() <= LOGIT_RTOL, err.max()
    assert np.array_equal(ids, g["ids_greedy"])


@pytest.mark.parametrize("arch_kw,plen", [
    (dict(weight_type=gguf.Q4_0, embed_type=gguf.F16, hidden=512, heads=4, kv_heads=1, ffn=512, rope_theta=500000.0), 400),
    (dict(weight_type=gguf.Q8_0, hidden=256, heads=4, kv_heads=2, ffn=768), 700),  # two 512-token passes
])
def test_batched_prefill_long_prompt_matches_oracle(arch_kw, plen):
    from laicompute_b200.engine import Engine
    kw = dict(arch_kw)
    wt = kw.pop("weight_type")
    et = kw.pop("embed_type", None)
    a = synth.tiny_arch(wt, et, layers=2, vocab=512, ctx=1024, name="pf", **kw)
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_model(os.path.join(d, "m.gguf"), a, seed=61)
        prompt = synth.prompt_ids(a.vocab, plen, seed=62)
        ref_ids, ref_logits = O.OracleModel(path).generate(prompt, 12)
        e = Engine(path, kv_capacity=1024)
        ids, logits = e.generate(prompt, 12, want_logits=True, batched_prefill=True)
        e.close()
    err = np.abs(logits - ref_logits).max(axis=1) / np.abs(ref_logits).max(axis=1)
    assert err.max() <= LOGIT_RTOL, err.max()
    assert np.array_equal(ids, ref_ids)
