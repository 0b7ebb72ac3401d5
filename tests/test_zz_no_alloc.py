"""laic_tensor_matvec_noalloc (fixed working memory compiled into the library)
against laic_tensor_matvec and the oracle's matvec, through the C ABI.

The file name sorts last so the fixed array has already been through every
other test's launches when these run; each test also passes on its own.
"""
import ctypes

import numpy as np
import pytest

from laicompute_b200 import gguf, synth

pytestmark = pytest.mark.gpu

FIXED_BYTES = 8 << 20  # LAIC_FIXED_SCRATCH_BYTES


def _weights(ggml_type, out_dim, in_dim, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(out_dim * in_dim, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return np.frombuffer(synth.encode(w, ggml_type), dtype=np.uint8)


def _noalloc(m, x_ptr, y_ptr, batch):
    from laicompute_b200._native import lib
    return int(lib().laic_tensor_matvec_noalloc(m.h, ctypes.c_void_p(x_ptr), ctypes.c_void_p(y_ptr), batch, None))


def _case(ggml_type, out_dim, in_dim, batch, seed):
    import torch
    from laicompute_b200._native import check
    from laicompute_b200.engine import Matrix
    raw = _weights(ggml_type, out_dim, in_dim, seed)
    m = Matrix(ggml_type, in_dim, out_dim, raw)
    x = torch.from_numpy(np.random.default_rng(seed + 1).standard_normal((batch, in_dim), dtype=np.float32)).cuda()
    y_ref = torch.empty((batch, out_dim), dtype=torch.float32, device="cuda")
    m.matvec(x.data_ptr(), y_ref.data_ptr(), batch)
    outs = []
    for _ in range(2):  # two calls in a row: the second finds the first one's leftovers in the array
        y = torch.full((batch, out_dim), float("nan"), dtype=torch.float32, device="cuda")
        check(_noalloc(m, x.data_ptr(), y.data_ptr(), batch))
        outs.append(y)
    m.check()  # no bounded device wait ran out (the error word of the fixed array is sticky)
    ref = y_ref.cpu().numpy()
    # same tolerance as the matvec tests: |err| <= 1e-5 * sum_i |w_i x_i|, against the
    # allocating entry point and against the oracle's sequential FP32 rows
    from oracle import oracle as O
    xh = x.cpu().numpy()
    oracle_y = O.matvec(ggml_type, raw, xh, out_dim, in_dim)
    wd = O.dequant(ggml_type, raw, out_dim * in_dim).reshape(out_dim, in_dim)
    bound = 1e-5 * (np.abs(xh) @ np.abs(wd).T) + 1e-12
    for y in outs:
        got = y.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - ref) <= bound), float(np.max(np.abs(got - ref) / bound))
        assert np.all(np.abs(got - oracle_y) <= bound), float(np.max(np.abs(got - oracle_y) / bound))
    m.close()


@pytest.mark.parametrize("ggml_type", [gguf.Q4_0, gguf.Q8_0, gguf.F16])
@pytest.mark.parametrize("batch", [1, 5, 32, 64])
def test_noalloc_matches_matvec(ggml_type, batch):
    # (1536, 576) at batch > 16 splits K across CTAs: partials, tickets and prepared activations in the array
    _case(ggml_type, 1536, 576, batch, seed=batch + ggml_type)


def test_noalloc_alternating_shapes():
    """Calls of different shapes back to back share the array."""
    for shape, batch in (((576, 1536), 64), ((200, 2048), 3), ((576, 1536), 40), ((1536, 576), 64)):
        _case(gguf.Q8_0, shape[0], shape[1], batch, seed=shape[0] + batch)


def test_noalloc_rejects_oversized_work():
    import torch
    from laicompute_b200._native import lib
    from laicompute_b200.engine import Matrix
    out_dim, in_dim, batch = 16384, 4096, 64  # split-K partials alone exceed the fixed array
    m = Matrix(gguf.Q4_0, in_dim, out_dim, _weights(gguf.Q4_0, out_dim, in_dim, 7))
    x = torch.zeros((batch, in_dim), dtype=torch.float32, device="cuda")
    y = torch.zeros((batch, out_dim), dtype=torch.float32, device="cuda")
    rc = _noalloc(m, x.data_ptr(), y.data_ptr(), batch)
    assert rc == -1  # LAIC_E_INVALID
    msg = lib().laic_last_error().decode()
    assert "laic_tensor_matvec_noalloc" in msg and str(FIXED_BYTES) in msg, msg
    # the allocating entry point still serves it
    m.matvec(x.data_ptr(), y.data_ptr(), batch)
    torch.cuda.synchronize()
    m.close()
