"""Q5_0 weights and upstream-order Q4_0 files on the GPU (reference src/quant_v2.cpp:10,
:12). Both are converted at upload into block types the kernels run (Q8_0 with the same
values; the reference's Q4_0 byte order), so the checks are those of the native types:

* a Q5_0 matrix through the single-tensor entry points: dequantisation bit-exact with the
  reference's values (tests/golden/blocks.npz) and the oracle's, matvec within 1e-5 of
  sum |w x| of the oracle's;
* a model whose projections are Q5_0 decodes like the oracle (greedy ids identical, logits
  within 1e-3 of max |logit|);
* the tiny Q4_0 model rewritten in upstream ggml's nibble order and loaded with
  LAIC_FLAG_Q4_0_UPSTREAM gives the same ids and logits as the original file.
"""
import os
import tempfile

import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
LOGIT_RTOL = 1e-3


def test_q5_0_tensor_dequant_and_matvec():
    import torch
    from laicompute_b200.engine import Matrix
    gold = np.load(os.path.join(HERE, "golden", "blocks.npz"))
    raw, ref = gold["raw_q5_0"], gold["value_q5_0"]
    out_dim, in_dim = 16, ref.size // 16
    m = Matrix(gguf.Q5_0, in_dim, out_dim, raw)
    y = torch.empty(ref.size, dtype=torch.float32, device="cuda")
    m.dequant(y.data_ptr())
    torch.cuda.synchronize()
    got = y.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))
    rng = np.random.default_rng(5)
    x = rng.standard_normal((3, in_dim), dtype=np.float32)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((3, out_dim), dtype=torch.float32, device="cuda")
    m.matvec(xd.data_ptr(), yd.data_ptr(), 3)
    m.check()
    yref = O.matvec(gguf.Q5_0, raw, x, out_dim, in_dim)
    bound = 1e-5 * (np.abs(ref.reshape(out_dim, in_dim))[None] * np.abs(x)[:, None, :]).sum(axis=2)
    assert (np.abs(yd.cpu().numpy() - yref) <= bound + 1e-30).all()
    m.close()


def test_q5_0_model_matches_oracle():
    from laicompute_b200.engine import Engine
    arch = synth.tiny_arch(gguf.Q5_0, gguf.F16, hidden=256, layers=2, heads=4, kv_heads=2, ffn=512, vocab=384,
                           ctx=256, name="tiny_q5_0")
    with tempfile.TemporaryDirectory() as d:
        path = synth.write_model(os.path.join(d, "m.gguf"), arch, seed=71, std=0.1)  # (varied greedy ids)
        prompt = synth.prompt_ids(arch.vocab, 12, seed=72)
        ref_ids, ref_logits = O.OracleModel(path).generate(prompt, 12)
        with Engine(path) as e:
            ids, logits = e.generate(prompt, 12, want_logits=True)
    err = np.abs(logits - ref_logits).max(axis=1) / np.abs(ref_logits).max(axis=1)
    assert err.max() <= LOGIT_RTOL, err.max()
    assert np.array_equal(ids, ref_ids)


def _upstream_copy(src: str, dst: str) -> None:
    """`src` with every Q4_0 tensor's nibbles in upstream ggml's order (elements j and j+16
    share byte j, low nibble first) instead of the reference's (element o: byte o/2)."""
    g = gguf.GgufFile(src)
    tensors = []
    for name, ti in g.tensors.items():
        raw = np.asarray(ti.data, dtype=np.uint8).copy()
        if ti.ggml_type == gguf.Q4_0:
            b = raw.reshape(-1, 18)
            e = np.empty((b.shape[0], 32), dtype=np.uint8)
            e[:, 0::2] = b[:, 2:] & 15
            e[:, 1::2] = b[:, 2:] >> 4
            b[:, 2:] = e[:, :16] | (e[:, 16:] << 4)
        tensors.append((name, tuple(ti.shape), ti.ggml_type, raw.tobytes()))
    gguf.write_gguf(dst, dict(g.metadata), tensors)


def test_q4_0_upstream_order_file_decodes_like_the_original():
    from laicompute_b200.engine import Engine
    path = os.path.join(HERE, "golden", "tiny_q4.gguf")
    prompt = synth.prompt_ids(320, 10, seed=73)
    with Engine(path) as e:
        ids, logits = e.generate(prompt, 10, want_logits=True)
    with tempfile.TemporaryDirectory() as d:
        up = os.path.join(d, "up.gguf")
        _upstream_copy(path, up)
        with Engine(up, q4_0_upstream=True) as e:
            ids2, logits2 = e.generate(prompt, 10, want_logits=True)
    assert np.array_equal(ids, ids2)
    assert np.array_equal(logits, logits2)
