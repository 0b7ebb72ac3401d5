"""laic_dev_step's speculative next step on the GPU: an engine that starts the following
step on its own sampled ids must return exactly what an engine without speculation
returns, for every call sequence: feedback (the guess is used), other tokens, slots or
parameters (the guess is undone: positions, repeat-penalty counts), slot resets and
prefills in between, and a context that has no room for a guess."""
import os

import numpy as np
import pytest

from laicompute_b200 import synth
from laicompute_b200.engine import sample_params

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
MODEL = os.path.join(HERE, "golden", "tiny_q4.gguf")


def engines(**kw):
    from laicompute_b200.engine import Engine
    return Engine(MODEL, speculate=True, **kw), Engine(MODEL, speculate=False, **kw)


def test_feedback_loop_is_unchanged():
    spec, plain = engines()
    prompt = synth.prompt_ids(320, 9, seed=81)
    for e in (spec, plain):
        e.prefill_batch(prompt[:-1], 0)
    ta = tb = [int(prompt[-1])]
    for _ in range(24):
        (ia, la), (ib, lb) = spec.step(ta, [0], want_logits=True), plain.step(tb, [0], want_logits=True)
        assert np.array_equal(ia, ib) and np.array_equal(la, lb)
        ta, tb = ia, ib
    assert spec.slot_pos(0) == plain.slot_pos(0)
    spec.close()
    plain.close()


def test_mismatches_resets_and_sampling_with_repeat_penalty():
    spec, plain = engines(max_seqs=4)
    prompts = [synth.prompt_ids(320, 6 + i, seed=90 + i) for i in range(4)]
    for e in (spec, plain):
        for i, p in enumerate(prompts):
            e.prefill_batch(p[:-1], i)
    params = [sample_params(0.8, 40, 0.95, 1.3, 4242 + i) for i in range(4)]
    slots = [0, 1, 2, 3]
    toks = [int(p[-1]) for p in prompts]
    rng = np.random.default_rng(7)
    for k in range(40):
        (ia, la), (ib, lb) = (e.step(toks, slots, params, want_logits=True) for e in (spec, plain))
        assert np.array_equal(ia, ib), k
        assert np.array_equal(la, lb), k
        toks = [int(t) for t in ia]
        if k % 7 == 3:   # another token than the sampled one: the guess is undone
            toks[1] = int(rng.integers(0, 320))
        if k % 11 == 5 and len(slots) > 2:  # a slot reset and a new prompt in between
            for e in (spec, plain):
                e.reset_slot(2)
                e.prefill_batch(prompts[2][:-1], 2)
            toks[2] = int(prompts[2][-1])
        if k == 20:      # fewer sequences (other slots) for a few steps
            slots, toks, params = slots[:2], toks[:2], params[:2]
        if k == 26:
            params = [sample_params(0.8, 40, 0.95, 1.3, 77 + i) for i in range(len(slots))]  # other seeds
        assert [spec.slot_pos(s) for s in range(4)] == [plain.slot_pos(s) for s in range(4)]
    spec.close()
    plain.close()


def test_full_context_leaves_no_room_for_a_guess():
    spec, plain = engines(kv_capacity=32)
    prompt = synth.prompt_ids(320, 20, seed=95)
    for e in (spec, plain):
        e.prefill_batch(prompt[:-1], 0)
    ta = tb = [int(prompt[-1])]
    from laicompute_b200._native import LaicError
    for k in range(20):
        if plain.slot_pos(0) >= 32:
            for e in (spec, plain):
                with pytest.raises(LaicError):
                    e.step(ta, [0])
            break
        (ia, _), (ib, _) = spec.step(ta, [0]), plain.step(tb, [0])
        assert np.array_equal(ia, ib), k
        ta, tb = ia, ib
    assert spec.slot_pos(0) == plain.slot_pos(0) == 32
    spec.close()
    plain.close()
