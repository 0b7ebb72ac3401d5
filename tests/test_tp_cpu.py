"""Tensor-parallel decomposition on CPU with two gloo ranks.

Each rank slices a layer's matrices by laicompute_b200.tp.ShardPlan (the rules
laic_dev_upload applies), runs its share of one decode layer in numpy, and
takes the same collective steps as the engine: an in-place allreduce of the
residual after o and after down (rank 0 adds its partial, the others store
theirs), and an all-gather of the lm_head rows. The result must equal the
single-rank layer. No GPU is involved.
"""
import os
import socket

import numpy as np
import pytest

from laicompute_b200.tp import ShardPlan


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rmsnorm(x, w, eps=1e-5):
    return x / np.sqrt(np.mean(x * x, axis=-1, keepdims=True) + eps) * w


def _attention(q, k, v, heads, kv_heads):
    """q [heads*d], k/v [t][kv_heads*d] -> [heads*d] (GQA)."""
    d = q.shape[0] // heads
    g = heads // kv_heads
    out = np.zeros_like(q)
    for h in range(heads):
        kh = h // g
        s = k[:, kh * d:(kh + 1) * d] @ q[h * d:(h + 1) * d] / np.sqrt(d)
        p = np.exp(s - s.max())
        p /= p.sum()
        out[h * d:(h + 1) * d] = p @ v[:, kh * d:(kh + 1) * d]
    return out


def _model(seed=0, hidden=64, heads=4, kv_heads=2, ffn=128, vocab=96, ctx=5):
    rng = np.random.default_rng(seed)
    d = hidden // heads
    w = {
        "q": rng.standard_normal((hidden, hidden)) * 0.1, "k": rng.standard_normal((kv_heads * d, hidden)) * 0.1,
        "v": rng.standard_normal((kv_heads * d, hidden)) * 0.1, "o": rng.standard_normal((hidden, hidden)) * 0.1,
        "gate": rng.standard_normal((ffn, hidden)) * 0.1, "up": rng.standard_normal((ffn, hidden)) * 0.1,
        "down": rng.standard_normal((hidden, ffn)) * 0.1, "lm": rng.standard_normal((vocab, hidden)) * 0.1,
        "an": 1 + 0.1 * rng.standard_normal(hidden), "fn": 1 + 0.1 * rng.standard_normal(hidden),
    }
    x = rng.standard_normal(hidden)
    past_k = rng.standard_normal((ctx, kv_heads * d))
    past_v = rng.standard_normal((ctx, kv_heads * d))
    return dict(hidden=hidden, heads=heads, kv_heads=kv_heads, ffn=ffn, vocab=vocab), w, x, past_k, past_v


def _layer_full(cfg, w, x, pk, pv):
    xn = _rmsnorm(x, w["an"])
    q, k, v = w["q"] @ xn, w["k"] @ xn, w["v"] @ xn
    a = _attention(q, np.vstack([pk, k]), np.vstack([pv, v]), cfg["heads"], cfg["kv_heads"])
    x = x + w["o"] @ a
    xn = _rmsnorm(x, w["fn"])
    g, u = w["gate"] @ xn, w["up"] @ xn
    x = x + w["down"] @ (g / (1 + np.exp(-g)) * u)
    return x, w["lm"] @ _rmsnorm(x, 1.0)


def _rank(rank, world, port, q):
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w, x, pk, pv = _model()
        plan = ShardPlan(cfg["hidden"], cfg["heads"], cfg["kv_heads"], cfg["ffn"], cfg["vocab"], world, rank)
        plan.check()
        qr, kr, fr, vr = plan.q_rows(), plan.kv_rows(), plan.ffn_rows(), plan.vocab_rows()

        def allreduce_residual(res, partial):
            buf = torch.from_numpy(res + partial if plan.residual_adds() else partial.copy())
            dist.all_reduce(buf)  # sum, in place, like ncclAllReduce on the residual
            return buf.numpy()

        xn = _rmsnorm(x, w["an"])
        q_, k_, v_ = w["q"][qr[0]:qr[1]] @ xn, w["k"][kr[0]:kr[1]] @ xn, w["v"][kr[0]:kr[1]] @ xn
        a = _attention(q_, np.vstack([pk[:, kr[0]:kr[1]], k_]), np.vstack([pv[:, kr[0]:kr[1]], v_]),
                       cfg["heads"] // world, cfg["kv_heads"] // world)
        xr = allreduce_residual(x, w["o"][:, plan.o_cols()[0]:plan.o_cols()[1]] @ a)
        xn = _rmsnorm(xr, w["fn"])
        g, u = w["gate"][fr[0]:fr[1]] @ xn, w["up"][fr[0]:fr[1]] @ xn
        xr = allreduce_residual(xr, w["down"][:, plan.down_cols()[0]:plan.down_cols()[1]] @ (g / (1 + np.exp(-g)) * u))
        local = torch.from_numpy(w["lm"][vr[0]:vr[1]] @ _rmsnorm(xr, 1.0))
        parts = [torch.empty_like(local) for _ in range(world)]
        dist.all_gather(parts, local)
        q.put((rank, xr, torch.cat(parts).numpy()))
    finally:
        dist.destroy_process_group()


def test_shard_plan_covers_every_row_once():
    for tp in (1, 2, 4, 8):
        rows = {k: [] for k in ("q", "kv", "ffn", "vocab")}
        for r in range(tp):
            p = ShardPlan(4096, 32, 8, 14336, 128256, tp, r)
            p.check()
            rows["q"].append(p.q_rows()); rows["kv"].append(p.kv_rows())
            rows["ffn"].append(p.ffn_rows()); rows["vocab"].append(p.vocab_rows())
        for key, full in (("q", 4096), ("kv", 1024), ("ffn", 14336), ("vocab", 128256)):
            spans = sorted(rows[key])
            assert spans[0][0] == 0 and spans[-1][1] == full
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    with pytest.raises(ValueError):
        ShardPlan(576, 9, 3, 1536, 49152, 2, 0).check()  # 9 heads do not split over 2 ranks


def test_two_gloo_ranks_match_single_rank():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=120) for _ in procs]
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    cfg, w, x, pk, pv = _model()
    x_ref, logits_ref = _layer_full(cfg, w, x, pk, pv)
    for rank, xr, logits in res:
        np.testing.assert_allclose(xr, x_ref, rtol=1e-10, atol=1e-10)
        np.testing.assert_allclose(logits, logits_ref, rtol=1e-10, atol=1e-10)
    assert all(p.exitcode == 0 for p in procs)
