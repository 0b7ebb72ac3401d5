"""Tensor parallelism over two GPUs (one process per rank, NCCL): greedy ids
and logits of small generated models against the oracle (reference
LlamaRuntime::step, src/inference_v2.cpp:31), and the ranks agreeing with
each other. Skipped when fewer than two GPUs are visible."""
import os
import tempfile

import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


def _two_gpus() -> bool:
    import torch
    return torch.cuda.is_available() and torch.cuda.device_count() >= 2


def _rank(rank, world, nccl_id, path, prompt, steps, kv_f32, q):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        from laicompute_b200.engine import Engine
        e = Engine(path, device=rank, tp_size=world, tp_rank=rank, nccl_id=nccl_id, kv_f32=kv_f32)
        ids, logits = e.generate(prompt, steps, want_logits=True)
        e.close()
        q.put((rank, ids, logits, None))
    except Exception as ex:  # report at once instead of leaving the parent waiting
        q.put((rank, None, None, repr(ex)))


def _run_tp(path, prompt, steps, kv_f32=False, world=2):
    import multiprocessing as mp
    from laicompute_b200.engine import nccl_unique_id
    nid = nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, nid, path, prompt, steps, kv_f32, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = []
    try:
        for _ in procs:
            r = q.get(timeout=180)
            assert r[3] is None, f"rank {r[0]}: {r[3]}"
            res.append(r)
    finally:
        for p in procs:
            p.join(timeout=30)
            if p.is_alive():
                p.kill()
    return sorted(res, key=lambda r: r[0])


ARCHS = {
    # GQA groups of 4 with head_dim 32 (Q4_0, F16 embeddings); groups of 2 with head_dim 64 (Q8_0)
    "q4_g4": synth.tiny_arch(gguf.Q4_0, gguf.F16, hidden=256, layers=2, heads=8, kv_heads=2, ffn=256, vocab=512,
                             rope_theta=500000.0, name="tp_q4"),
    "q8_g2": synth.tiny_arch(gguf.Q8_0, hidden=256, layers=2, heads=4, kv_heads=2, ffn=512, vocab=512, name="tp_q8"),
}


@pytest.mark.skipif(not _two_gpus(), reason="needs two GPUs")
@pytest.mark.parametrize("arch", sorted(ARCHS))
@pytest.mark.parametrize("kv_f32", [True, False])
def test_tp2_matches_oracle(arch, kv_f32):
    a = ARCHS[arch]
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_model(os.path.join(d, "m.gguf"), a, seed=41)
        prompt = synth.prompt_ids(a.vocab, 12, seed=42)
        ref_ids, ref_logits = O.OracleModel(path).generate(prompt, 24)
        res = _run_tp(path, prompt, 24, kv_f32)
    for rank, ids, logits, _ in res:
        err = np.abs(logits - ref_logits).max(axis=1) / np.abs(ref_logits).max(axis=1)
        assert err.max() <= LOGIT_RTOL, (rank, err.max())
        assert np.array_equal(ids, ref_ids), rank
    assert np.array_equal(res[0][2], res[1][2])  # every rank samples from the same gathered logits
