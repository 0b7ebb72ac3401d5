"""Single-tensor entry points on the GPU against the oracle: dequantisation
(bit-exact with quant_v2::value) and matvec (FP32 accumulate)."""
import numpy as np
import pytest

from laicompute_b200 import gguf, synth
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TYPES = [gguf.F16, gguf.Q8_0, gguf.Q4_0]


def _torch():
    import torch
    return torch


def _weights(ggml_type, out_dim, in_dim, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal(out_dim * in_dim, dtype=np.float32) * np.float32(0.02)).astype(np.float32)
    return np.frombuffer(synth.encode(w, ggml_type), dtype=np.uint8)


@pytest.mark.parametrize("ggml_type", TYPES)
@pytest.mark.parametrize("shape", [(96, 576), (40, 64), (64, 1536)])
def test_dequant_bit_exact(ggml_type, shape):
    from laicompute_b200.engine import Matrix
    torch = _torch()
    out_dim, in_dim = shape
    raw = _weights(ggml_type, out_dim, in_dim, seed=out_dim + in_dim)
    m = Matrix(ggml_type, in_dim, out_dim, raw)
    y = torch.empty(out_dim * in_dim, dtype=torch.float32, device="cuda")
    m.dequant(y.data_ptr())
    torch.cuda.synchronize()
    ref = O.dequant(ggml_type, raw, out_dim * in_dim)
    assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def test_dequant_edge_values():
    """Subnormal, zero, negative-zero and extreme binary16 scales decode exactly."""
    from laicompute_b200.engine import Matrix
    torch = _torch()
    rng = np.random.default_rng(5)
    for ggml_type, bb in ((gguf.Q4_0, 18), (gguf.Q8_0, 34)):
        nblk = 64
        raw = rng.integers(0, 256, size=nblk * bb, dtype=np.uint8).reshape(nblk, bb)
        scales = np.array([0x0000, 0x8000, 0x0001, 0x03FF, 0x0400, 0x7BFF, 0xFBFF, 0x3C00], dtype="<u2")
        raw[:, 0:2] = np.resize(scales, nblk).view(np.uint8).reshape(-1, 2)
        m = Matrix(ggml_type, 64, nblk // 2, raw.reshape(-1))
        y = torch.empty(nblk * 32, dtype=torch.float32, device="cuda")
        m.dequant(y.data_ptr())
        torch.cuda.synchronize()
        ref = O.dequant(ggml_type, raw.reshape(-1), nblk * 32)
        assert np.array_equal(y.cpu().numpy().view(np.uint32), ref.view(np.uint32))


def _check_matvec(ggml_type, out_dim, in_dim, batch, seed=0):
    from laicompute_b200.engine import Matrix
    torch = _torch()
    raw = _weights(ggml_type, out_dim, in_dim, seed)
    x = np.random.default_rng(seed + 1).standard_normal((batch, in_dim), dtype=np.float32)
    m = Matrix(ggml_type, in_dim, out_dim, raw)
    xd = torch.from_numpy(x).cuda()
    yd = torch.empty((batch, out_dim), dtype=torch.float32, device="cuda")
    m.matvec(xd.data_ptr(), yd.data_ptr(), batch)
    torch.cuda.synchronize()
    y = yd.cpu().numpy()
    ref = O.matvec(ggml_type, raw, x, out_dim, in_dim)
    # FP32 accumulation in a different order: |err| <= 1e-5 * sum_i |w_i x_i|
    wd = O.dequant(ggml_type, raw, out_dim * in_dim).reshape(out_dim, in_dim)
    bound = 1e-5 * (np.abs(x) @ np.abs(wd).T) + 1e-12
    assert np.all(np.abs(y - ref) <= bound), float(np.max(np.abs(y - ref) / bound))


@pytest.mark.parametrize("ggml_type", TYPES)
@pytest.mark.parametrize("batch", [1, 2, 3, 4])
@pytest.mark.parametrize("shape", [(1536, 576), (576, 1536), (200, 2048), (13, 96)])
def test_matvec_matches_oracle(ggml_type, batch, shape):
    _check_matvec(ggml_type, shape[0], shape[1], batch)


@pytest.mark.parametrize("batch", [1, 16])
def test_matvec_q4_0_large(batch):
    """A 4096x4096 Q4_0 matrix of the 8B-shaped model."""
    _check_matvec(gguf.Q4_0, 4096, 4096, batch, seed=3)


@pytest.mark.parametrize("ggml_type", TYPES)
@pytest.mark.parametrize("batch,rows", [(17, 40000), (40, 12000), (64, 8000)])
def test_matvec_many_row_tiles(ggml_type, batch, rows):
    """Batches above 16 of a matrix with thousands of row tiles and a short K (an lm_head's
    shape): the wide kernel, each warp owning whole row tiles, in one or several sequence groups."""
    _check_matvec(ggml_type, rows, 576, batch, seed=9)
