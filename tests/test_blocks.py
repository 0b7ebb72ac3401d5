"""GGML block types beyond F16 / Q8_0 / Q4_0 (reference src/quant_v2.cpp:11-13), and the
upstream-ggml Q4_0 nibble order, on the CPU:

* the oracle's restatement of quant_v2::value for Q4_1, Q5_0 and Q5_1 against the
  reference's own decode of random and edge-case blocks (tests/golden/blocks.npz, made by
  tests/golden/make_golden.py blocks), bit-exact;
* laic_blocks_convert (what the device does at upload): Q5_0 becomes Q8_0 blocks whose
  values are bit-identical to the reference's Q5_0 values; Q4_0 in upstream order becomes
  the reference's byte order; Q4_1 / Q5_1 are refused.
"""
import os

import numpy as np
import pytest

from laicompute_b200 import gguf
from oracle import oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "blocks.npz"))
TYPES = {"q4_1": gguf.Q4_1, "q5_0": gguf.Q5_0, "q5_1": gguf.Q5_1, "q4_0": gguf.Q4_0}


def _bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("kind", sorted(TYPES))
def test_oracle_decodes_like_the_reference(kind):
    raw = GOLD[f"raw_{kind}"]
    ref = GOLD[f"value_{kind}"]
    got = O.dequant(TYPES[kind], raw, ref.size)
    assert np.array_equal(_bits(got), _bits(ref))


def test_q5_0_converts_to_identical_q8_0():
    from laicompute_b200.engine import blocks_convert
    raw, ref = GOLD["raw_q5_0"], GOLD["value_q5_0"]
    t, q8 = blocks_convert(gguf.Q5_0, raw, ref.size)
    assert t == gguf.Q8_0 and q8.size == ref.size // 32 * 34
    assert np.array_equal(_bits(O.dequant(gguf.Q8_0, q8, ref.size)), _bits(ref))


def _to_upstream(blocks: np.ndarray) -> np.ndarray:
    """Q4_0 blocks in the reference's order (element o: byte o/2, low nibble for even o)
    rewritten in upstream ggml's order (elements j and j+16 share byte j, low nibble first)."""
    b = blocks.reshape(-1, 18)
    q = b[:, 2:]
    elems = np.empty((b.shape[0], 32), dtype=np.uint8)
    elems[:, 0::2] = q & 15
    elems[:, 1::2] = q >> 4
    out = b.copy()
    out[:, 2:] = elems[:, :16] | (elems[:, 16:] << 4)
    return out.reshape(-1)


def test_q4_0_upstream_order_converts_to_the_reference_order():
    from laicompute_b200.engine import blocks_convert
    raw, ref = GOLD["raw_q4_0"], GOLD["value_q4_0"]
    up = _to_upstream(raw)
    assert not np.array_equal(up, raw)
    t, back = blocks_convert(gguf.Q4_0, up, ref.size, q4_0_upstream=True)
    assert t == gguf.Q4_0 and np.array_equal(back, raw)
    assert np.array_equal(_bits(O.dequant(gguf.Q4_0, back, ref.size)), _bits(ref))
    # without the flag Q4_0 bytes pass through unchanged
    t, same = blocks_convert(gguf.Q4_0, up, ref.size)
    assert np.array_equal(same, up)


@pytest.mark.parametrize("kind", ["q4_1", "q5_1"])
def test_types_without_a_device_form_are_refused(kind):
    from laicompute_b200._native import LaicError
    from laicompute_b200.engine import blocks_convert
    with pytest.raises(LaicError) as e:
        blocks_convert(TYPES[kind], GOLD[f"raw_{kind}"], GOLD[f"value_{kind}"].size)
    assert "unsupported" in str(e.value)
