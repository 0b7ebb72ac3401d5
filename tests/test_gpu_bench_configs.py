"""Parity on the configurations the benchmark numbers come from, through the C ABI,
against the oracle (CPU restatement of LlamaRuntime::step / sample, reference
src/inference_v2.cpp:31-32, pinned to the reference's own outputs on CPU):

* two-layer slices with the 8B and 1B layer dimensions (hidden 4096 / 2048,
  32 query and 8 KV heads, head_dim 128 / 64, ffn 14336 / 8192, vocab 128256,
  RoPE theta 5e5, Q4_0 projections; tied Q4_0 resp. F16 embeddings), on the
  same kernels and launch shapes as the full models (the team kernel's integer
  path with producer digit records, the 8192-position KV cache);
* decode attention at 4096 and 8192 positions (GQA groups of 4, head_dim 128 and
  64, eight splits merged inside a thread-block cluster);
* the 135M Q8_0 model at 64 sequences (tile-kernel groups of 64, the wide
  lm_head kernel, the sampler at 64 sequences), greedy and T=0.8 / top-k 40;
* the Q4_0 matvec shapes of the kernel sweep (14336x4096, 4096x14336,
  128256x4096) at batch 1, 4 and 16.

Logits within 1e-3 of max|logit| per step (FP32 accumulate, FP16 KV cache),
greedy ids identical over the whole generation.
"""
import os
from dataclasses import replace

import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

LOGIT_RTOL = 1e-3


def _rel_err(logits, ref):
    return np.abs(logits - ref).max(axis=-1) / np.abs(ref).max(axis=-1)


@pytest.fixture(scope="module")
def slice_dir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("bench_slices"))


def _slice_model(slice_dir, arch, seed):
    path = os.path.join(slice_dir, arch.name + ".gguf")
    if not os.path.exists(path):
        synth.write_model(path, arch, seed=seed, direct_blocks=True)
    return path


# both one-sequence decode paths: per-projection launches, and the persistent decode-step kernel
PATHS = {"layers": dict(step_kernel=False), "step": dict(step_kernel=True)}
_oracle_runs = {}


def _oracle_generate(path, prompt, steps):
    key = (path, steps)
    if key not in _oracle_runs:
        _oracle_runs[key] = O.OracleModel(path).generate(prompt, steps)
    return _oracle_runs[key]


@pytest.mark.parametrize("which", ["llama8b", "llama1b"])
@pytest.mark.parametrize("dpath", sorted(PATHS))
def test_large_layer_slice_matches_oracle(slice_dir, which, dpath):
    """Two layers of the 8B (or 1B) shape, one sequence: the benchmark's batch-1 path."""
    from laicompute_b200.engine import Engine
    base = synth.LLAMA_8B_Q4 if which == "llama8b" else synth.LLAMA_1B_Q4
    arch = replace(base, name=base.name + "-2l", layers=2)
    path = _slice_model(slice_dir, arch, seed=51 if which == "llama8b" else 52)
    prompt = synth.prompt_ids(arch.vocab, 6, seed=53)
    steps = 8
    ref_ids, ref_logits = _oracle_generate(path, prompt, steps)
    e = Engine(path, kv_capacity=8192, **PATHS[dpath])
    ids, logits = e.generate(prompt, steps, want_logits=True)
    e.close()
    err = _rel_err(logits, ref_logits)
    assert err.max() <= LOGIT_RTOL, err
    assert np.array_equal(ids, ref_ids), (ids, ref_ids)


@pytest.mark.parametrize("ctx,head_dim", [(4096, 128), (8192, 128), (4096, 64), (8192, 64)])
@pytest.mark.parametrize("dpath", sorted(PATHS))
def test_attention_at_benchmark_contexts(slice_dir, ctx, head_dim, dpath):
    """A one-layer model with 4 query heads per KV head whose prompt fills the KV cache to
    `ctx` - 2 positions; the last decode steps attend over ~ctx positions (per-projection
    launches: in 8 splits merged inside a thread-block cluster; the step kernel: spread over
    every SM, up to 256 chunks of 32 positions)."""
    from laicompute_b200.engine import Engine
    heads, kv_heads = (4, 1) if head_dim == 128 else (8, 2)
    arch = synth.tiny_arch(gguf.Q4_0, gguf.F16, hidden=heads * head_dim, layers=1, heads=heads, kv_heads=kv_heads,
                           ffn=128, vocab=256, ctx=ctx, rope_theta=500000.0, name=f"attn{ctx}_{head_dim}")
    path = os.path.join(slice_dir, arch.name + ".gguf")
    if not os.path.exists(path):
        synth.write_model(path, arch, seed=61)
    prompt = synth.prompt_ids(arch.vocab, ctx - 2, seed=62)
    ref_ids, ref_logits = _oracle_generate(path, prompt, 3)
    e = Engine(path, kv_capacity=ctx, **PATHS[dpath])
    ids, logits = e.generate(prompt, 3, want_logits=True)
    if dpath == "layers":
        assert e.stats().attn_splits >= 2  # the splits merge inside a thread-block cluster
    e.close()
    err = _rel_err(logits, ref_logits)
    assert err.max() <= LOGIT_RTOL, err
    assert np.array_equal(ids, ref_ids)


NSEQ, PLEN, STEPS = 64, 3, 3


@pytest.fixture(scope="module")
def smollm_q8_batch(smollm_models):
    """The 135M Q8_0 model, 64 sequences of distinct prompts, and the oracle's run of each."""
    path = smollm_models["smollm135m_q8"]
    prompts = np.stack([synth.prompt_ids(49152, PLEN, seed=700 + i) for i in range(NSEQ)])
    m = O.OracleModel(path)
    ref = [m.generate(prompts[i], STEPS) for i in range(NSEQ)]
    return path, prompts, np.stack([r[0] for r in ref]), np.stack([r[1] for r in ref])


def test_smollm_q8_64_sequences_greedy(smollm_q8_batch):
    from laicompute_b200.engine import Engine
    path, prompts, ref_ids, ref_logits = smollm_q8_batch
    slots = np.arange(NSEQ, dtype=np.int32)
    e = Engine(path, max_seqs=NSEQ, kv_capacity=256)
    for j in range(PLEN - 1):
        e.prefill(prompts[:, j], slots)
    tok = prompts[:, -1]
    ids, logits = [], []
    for _ in range(STEPS):
        out, lg = e.step(tok, slots, want_logits=True)
        ids.append(out)
        logits.append(lg)
        tok = out
    e.close()
    ids = np.stack(ids, axis=1)          # [seq][step]
    logits = np.stack(logits, axis=1)    # [seq][step][V]
    err = _rel_err(logits, ref_logits)
    assert err.max() <= LOGIT_RTOL, err.max()
    assert np.array_equal(ids, ref_ids)


def test_smollm_q8_64_sequences_topk_sampling(smollm_q8_batch):
    """T = 0.8, top-k 40, a seed per sequence: every sampled id follows the documented
    rule (candidates in descending-logit order, inverse CDF at the seed's canonical
    draw) on that step's own logits."""
    from laicompute_b200.engine import Engine, sample_params
    path, prompts, _, _ = smollm_q8_batch
    T, K = 0.8, 40
    seeds = [4242 + i for i in range(NSEQ)]
    params = [sample_params(T, K, 1.0, 1.0, s) for s in seeds]
    us = [O.canonical_u(s) for s in seeds]
    slots = np.arange(NSEQ, dtype=np.int32)
    e = Engine(path, max_seqs=NSEQ, kv_capacity=256)
    for j in range(PLEN - 1):
        e.prefill(prompts[:, j], slots)
    tok = prompts[:, -1]
    for _ in range(STEPS):
        out, lg = e.step(tok, slots, params, want_logits=True)
        for i in range(NSEQ):
            l = lg[i]
            order = np.lexsort((np.arange(len(l)), -l))[:K]
            v = l[order]
            p = np.exp(((v - v[0]) / np.float32(T)).astype(np.float32)).astype(np.float64)
            p /= p.sum()
            p /= p.sum()
            c = np.cumsum(p)
            c[-1] = 1.0
            assert int(out[i]) == int(order[int(np.searchsorted(c, us[i], side="left"))])
        tok = out
    e.close()


@pytest.mark.parametrize("shape", [(14336, 4096), (4096, 14336), (128256, 4096)])
def test_sweep_shapes_q4_0_matvec(shape):
    """The kernel-sweep shapes (out x in) on the single-tensor entry point, batch 1, 4 and 16."""
    import torch
    from laicompute_b200.engine import Matrix
    out_dim, in_dim = shape
    raw = np.frombuffer(synth.random_blocks(out_dim * in_dim, gguf.Q4_0, np.random.default_rng(out_dim + in_dim)),
                        dtype=np.uint8)
    absw = np.abs(O.dequant(gguf.Q4_0, raw, out_dim * in_dim).reshape(out_dim, in_dim))
    m = Matrix(gguf.Q4_0, in_dim, out_dim, raw)
    for batch in (1, 4, 16):
        x = np.random.default_rng(batch).standard_normal((batch, in_dim), dtype=np.float32)
        xd = torch.from_numpy(x).cuda()
        yd = torch.empty((batch, out_dim), dtype=torch.float32, device="cuda")
        m.matvec(xd.data_ptr(), yd.data_ptr(), batch)
        m.check()
        y = yd.cpu().numpy()
        ref = O.matvec(gguf.Q4_0, raw, x, out_dim, in_dim)
        bound = 1e-5 * (np.abs(x) @ absw.T) + 1e-12
        assert np.all(np.abs(y - ref) <= bound), (batch, float(np.max(np.abs(y - ref) / bound)))
    m.close()
