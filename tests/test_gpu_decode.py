"""Full decode steps on the GPU (C ABI laic_dev_*) against the reference's own
outputs and the oracle: logits within 1e-3 of max|logit| (FP32 accumulate),
greedy ids identical for the whole generation."""
import numpy as np
import pytest

from conftest import TINY_MODELS, golden, golden_model
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3  # max|dlogit| <= 1e-3 * max|logit_ref|


def _engine(path, **kw):
    from laicompute_b200.engine import Engine
    return Engine(path, **kw)


def _sp(t=0.0, k=0, p=1.0, rp=1.0, seed=0):
    from laicompute_b200.engine import sample_params
    return sample_params(t, k, p, rp, seed)


def _step_logits(e, prompt, steps, slot=0):
    """Logits of every step() call, in the reference driver's order."""
    e.reset_slot(slot)
    rows, ids = [], []
    for t in prompt:
        out, lg = e.step([t], [slot], want_logits=True)
        rows.append(lg[0])
    tok = int(out[0])
    ids.append(tok)
    for _ in range(steps - 1):
        out, lg = e.step([tok], [slot], want_logits=True)
        rows.append(lg[0])
        tok = int(out[0])
        ids.append(tok)
    return np.stack(rows), np.array(ids, dtype=np.uint32)


@pytest.mark.parametrize("name", TINY_MODELS)
@pytest.mark.parametrize("kv_f32", [True, False])
def test_logits_and_greedy_ids_match_reference(name, kv_f32):
    g = golden(name)
    e = _engine(golden_model(name), kv_f32=kv_f32)
    logits, ids = _step_logits(e, g["prompt"], len(g["ids_greedy"]))
    ref = g["logits_greedy"]
    err = np.abs(logits - ref).max(axis=1) / np.abs(ref).max(axis=1)
    assert err.max() <= LOGIT_RTOL, err
    if kv_f32:
        assert err.max() <= 2e-5, err  # FP32 KV: FP32-rounding level
    assert np.array_equal(ids, g["ids_greedy"])


@pytest.mark.parametrize("name", TINY_MODELS)
def test_generate_loop_greedy(name):
    """prefill for the prompt, then step(): the runtime's loop, ids identical."""
    g = golden(name)
    e = _engine(golden_model(name))
    ids, _ = e.generate(g["prompt"], len(g["ids_greedy"]))
    assert np.array_equal(ids, g["ids_greedy"])


@pytest.mark.parametrize("name", TINY_MODELS)
@pytest.mark.parametrize("case,params", [("full", (1.0, 0, 1.0, 1.0, 7)), ("topp_pen", (0.7, 0, 0.9, 1.3, 99))])
def test_sampling_matches_reference(name, case, params):
    """Candidate order equals the reference's in these modes: the same ids."""
    g = golden(name)
    e = _engine(golden_model(name))
    ids, _ = e.generate(g["prompt"], len(g[f"ids_{case}"]), _sp(*params))
    assert np.array_equal(ids, g[f"ids_{case}"])


@pytest.mark.parametrize("name", TINY_MODELS)
def test_topk_sampling_follows_documented_rule(name):
    """top_k < vocab, top_p = 1: candidates in descending-logit order, inverse CDF at u."""
    g = golden(name)
    e = _engine(golden_model(name))
    T, K, seed = 0.8, 40, 1234
    u = O.canonical_u(seed)
    e.reset_slot(0)
    for t in g["prompt"][:-1]:
        e.prefill([t], [0])
    tok = int(g["prompt"][-1])
    for _ in range(8):
        out, lg = e.step([tok], [0], _sp(T, K, 1.0, 1.0, seed), want_logits=True)
        l = lg[0]
        order = np.lexsort((np.arange(len(l)), -l))[:K]
        v = l[order]
        p = np.exp(((v - v[0]) / np.float32(T)).astype(np.float32)).astype(np.float64)
        p /= p.sum()
        p /= p.sum()
        c = np.cumsum(p)
        c[-1] = 1.0
        expect = order[int(np.searchsorted(c, u, side="left"))]
        assert int(out[0]) == int(expect)
        tok = int(out[0])


@pytest.mark.parametrize("graphs,pdl", [(False, False), (True, False), (False, True)])
def test_launch_modes_agree(graphs, pdl):
    g = golden("tiny_q4")
    e = _engine(golden_model("tiny_q4"), graphs=graphs, pdl=pdl)
    ids, _ = e.generate(g["prompt"], len(g["ids_greedy"]))
    assert np.array_equal(ids, g["ids_greedy"])


def test_oracle_agrees_on_longer_generation():
    """64 greedy tokens on a generated model with GQA groups of 4 (the 1B/8B grouping)."""
    import os
    import tempfile
    from laicompute_b200 import gguf, synth
    arch = synth.tiny_arch(gguf.Q4_0, gguf.F16, hidden=256, layers=3, heads=8, kv_heads=2, ffn=256, vocab=512,
                           rope_theta=500000.0, name="tiny_g4")
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_model(os.path.join(d, "m.gguf"), arch, seed=21)
        prompt = synth.prompt_ids(arch.vocab, 16, seed=22)
        m = O.OracleModel(path)
        ref_ids, ref_logits = m.generate(prompt, 64)
        e = _engine(path, kv_f32=True)
        ids, logits = e.generate(prompt, 64, want_logits=True)
        err = np.abs(logits - ref_logits).max(axis=1) / np.abs(ref_logits).max(axis=1)
        assert err.max() <= LOGIT_RTOL
        assert np.array_equal(ids, ref_ids)
