"""The persistent one-sequence decode-step kernel (every phase of a step in one
launch, the default for one sequence of Q4_0 / Q8_0 layers) against the oracle
(reference LlamaRuntime::step, src/inference_v2.cpp:31) and against the
per-layer launch path, on Q4_0 (head dim 128, GQA groups of 4, F16 lm_head
outside the kernel) and Q8_0 (head dim 64, groups of 3, lm_head inside) models
at contexts spanning several attention chunks and splits."""
import os
import tempfile

import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3

ARCHS = {
    "q4_d128_g4": synth.tiny_arch(gguf.Q4_0, gguf.F16, hidden=512, layers=3, heads=4, kv_heads=1, ffn=512,
                                  vocab=512, ctx=1024, rope_theta=500000.0, name="step_q4"),
    "q8_d64_g2": synth.tiny_arch(gguf.Q8_0, hidden=256, layers=3, heads=4, kv_heads=2, ffn=768, vocab=512,
                                 ctx=1024, name="step_q8"),
    "q8_d64_g3": synth.tiny_arch(gguf.Q8_0, hidden=384, layers=2, heads=6, kv_heads=2, ffn=512, vocab=640,
                                 ctx=1024, name="step_q8g3"),
    # the 8B model's ffn width (its records leave room for only 5 attention stages, fewer
    # than the producer's batch) and a tied Q4_0 lm_head of the 8B vocabulary on a narrow
    # model (54 row tiles per CTA, up to 5 pieces per consumer warp in the LM phase)
    "q4_wide": synth.tiny_arch(gguf.Q4_0, gguf.Q4_0, hidden=256, layers=3, heads=2, kv_heads=1, ffn=14336,
                               vocab=128256, ctx=1024, rope_theta=500000.0, name="step_q4wide"),
}


@pytest.mark.parametrize("arch", sorted(ARCHS))
def test_step_kernel_matches_oracle_and_layer_path(arch):
    from laicompute_b200.engine import Engine
    a = ARCHS[arch]
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_model(os.path.join(d, "m.gguf"), a, seed=51, direct_blocks=a.vocab > 65536)
        prompt = synth.prompt_ids(a.vocab, 300, seed=52)
        ref_ids, ref_logits = O.OracleModel(path).generate(prompt, 16)
        e = Engine(path, kv_capacity=1024, step_kernel=True)
        ids, logits = e.generate(prompt, 16, want_logits=True)
        stats = e.stats()
        e.close()
        e2 = Engine(path, kv_capacity=1024, layer_launches=True)
        ids2, logits2 = e2.generate(prompt, 16, want_logits=True)
        stats2 = e2.stats()
        e2.close()
    assert stats.launches_per_step < stats2.launches_per_step  # the step kernel ran
    err = np.abs(logits - ref_logits).max(axis=1) / np.abs(ref_logits).max(axis=1)
    assert err.max() <= LOGIT_RTOL, err.max()
    assert np.array_equal(ids, ref_ids)
    assert np.array_equal(ids2, ref_ids)
    # same integer dot products, different split of the work: FP32-rounding level apart
    d2 = np.abs(logits - logits2).max(axis=1) / np.abs(logits2).max(axis=1)
    assert d2.max() <= 1e-4, d2.max()


def test_step_trace_stamps_every_phase():
    """The persistent kernel's trace (LAIC_FLAG_TRACE): per CTA and phase five ordered stamps
    (start <= inputs ready <= first warp done <= all warps done <= done), phases in step order."""
    from laicompute_b200.engine import Engine
    a = ARCHS["q4_d128_g4"]
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_model(os.path.join(d, "m.gguf"), a, seed=51)
        prompt = synth.prompt_ids(a.vocab, 40, seed=52)
        e = Engine(path, kv_capacity=1024, step_kernel=True, trace=True)
        e.prefill_batch(prompt[:-1], 0)
        e.step([int(prompt[-1])], [0])
        tr = e.step_trace().astype(np.int64)
        waits = e.last_wait_stats
        e.close()
    ctas, phases, k = tr.shape
    assert k == 5 and phases == 2 + 5 * a.layers and ctas >= 1
    assert (tr > 0).all()
    assert (np.diff(tr, axis=2) >= 0).all()              # within a phase
    assert (tr[:, 1:, 0] >= tr[:, :-1, 4]).all()          # a phase starts after the previous one is done
    assert waits.shape == (ctas, 16, 5) and (waits[:, :, 4] > 0).all()
