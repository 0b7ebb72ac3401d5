"""Several sequences in one step (slots) give each sequence the same result
as decoding it alone; slots are independent and reset cleanly."""
import os
import tempfile

import numpy as np
import pytest

from conftest import golden, golden_model
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _engine(path, **kw):
    from laicompute_b200.engine import Engine
    return Engine(path, **kw)


@pytest.mark.parametrize("nseq", [2, 3, 8, 24, 40])  # above 16: tile-kernel projections with producer-made records
@pytest.mark.parametrize("name", ["tiny_q8", "tiny_q4"])
def test_batched_greedy_matches_oracle(name, nseq):
    path = golden_model(name)
    m = O.OracleModel(path)
    rng = np.random.default_rng(nseq)
    prompts = rng.integers(0, m.vocab, size=(nseq, 5)).astype(np.uint32)
    steps = 12
    ref = [m.generate(p, steps, want_logits=False)[0] for p in prompts]
    e = _engine(path, max_seqs=nseq, kv_f32=True)
    slots = np.arange(nseq, dtype=np.int32)[::-1].copy()  # any slot assignment
    for s in slots:
        e.reset_slot(int(s))
    for j in range(prompts.shape[1] - 1):
        e.prefill(prompts[:, j], slots)
    tok = prompts[:, -1].copy()
    got = []
    for _ in range(steps):
        tok, _ = e.step(tok, slots)
        got.append(tok.copy())
    got = np.stack(got, axis=1)
    for i in range(nseq):
        assert np.array_equal(got[i], ref[i]), i


def test_ragged_positions_and_reset():
    """Sequences at different positions in one step; a reset slot starts over."""
    path = golden_model("tiny_f16")
    g = golden("tiny_f16")
    e = _engine(path, max_seqs=4, kv_f32=True)
    ref = g["ids_greedy"]
    prompt = g["prompt"]
    # slot 2 runs the golden prompt; slot 0 gets a head start with other tokens
    for t in [1, 2, 3, 4, 5, 6, 7]:
        e.prefill([t], [0])
    for t in prompt[:-1]:
        e.prefill([t], [2])
    tok = np.array([9, prompt[-1]], dtype=np.uint32)
    out_ids = []
    for _ in range(len(ref)):
        tok, _ = e.step(tok, [0, 2])
        out_ids.append(int(tok[1]))
    assert np.array_equal(np.array(out_ids, dtype=np.uint32), ref)
    assert e.slot_pos(2) == len(prompt) + len(ref) - 1
    e.reset_slot(2)
    assert e.slot_pos(2) == 0
    ids, _ = e.generate(prompt, len(ref), slot=2)
    assert np.array_equal(ids, ref)


def test_per_sequence_sampling_params():
    path = golden_model("tiny_q8")
    g = golden("tiny_q8")
    from laicompute_b200.engine import sample_params
    e = _engine(path, max_seqs=2)
    prompt = g["prompt"]
    for t in prompt[:-1]:
        e.prefill([t, t], [0, 1])
    params = [sample_params(0.0), sample_params(1.0, 0, 1.0, 1.0, 7)]
    tok = np.array([prompt[-1], prompt[-1]], dtype=np.uint32)
    a, b = [], []
    for _ in range(len(g["ids_greedy"])):
        tok, _ = e.step(tok, [0, 1], params)
        a.append(int(tok[0])); b.append(int(tok[1]))
    assert np.array_equal(np.array(a, dtype=np.uint32), g["ids_greedy"])
    assert np.array_equal(np.array(b, dtype=np.uint32), g["ids_full"])


@pytest.mark.parametrize("nseq,wt", [(1, "q4_0"), (1, "q8_0"), (4, "q4_0"), (17, "q4_0")])
def test_large_layer_model_matches_oracle(nseq, wt):
    """A model whose layers are above the small-layer bound: batches up to 16 run the
    team kernel (one sequence: its integer dot products, with the digit records written
    by each producing kernel's epilogue), larger ones the tile kernel with activation
    records; logits within 1e-3 of max|logit|, greedy ids identical."""
    from laicompute_b200 import gguf, synth
    a = synth.tiny_arch({"q4_0": gguf.Q4_0, "q8_0": gguf.Q8_0}[wt], None, layers=2, vocab=512, ctx=64, name="big",
                        hidden=1024, heads=8, kv_heads=2, ffn=5120)
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_model(os.path.join(d, "m.gguf"), a, seed=71)
        m = O.OracleModel(path)
        rng = np.random.default_rng(72 + nseq)
        prompts = rng.integers(0, m.vocab, size=(nseq, 4)).astype(np.uint32)
        steps = 6
        ref = [m.generate(p, steps) for p in prompts]
        e = _engine(path, max_seqs=nseq)
        slots = np.arange(nseq, dtype=np.int32)
        for j in range(prompts.shape[1] - 1):
            e.prefill(prompts[:, j], slots)
        tok = prompts[:, -1].copy()
        for k in range(steps):
            tok, lg = e.step(tok, slots, want_logits=True)
            for i in range(nseq):
                r = ref[i][1][k]
                assert np.abs(lg[i] - r).max() <= 1e-3 * np.abs(r).max(), (i, k)
                assert int(tok[i]) == int(ref[i][0][k]), (i, k)
        e.close()
