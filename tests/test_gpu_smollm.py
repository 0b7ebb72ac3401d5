"""The 135M-shaped benchmark models (F16 and Q8_0) against the reference's outputs."""
import numpy as np
import pytest

from conftest import golden

pytestmark = pytest.mark.gpu


def _engine(path, **kw):
    from laicompute_b200.engine import Engine
    return Engine(path, **kw)


@pytest.mark.parametrize("kv_f32", [True, False])
def test_smollm_f16_greedy(smollm_models, kv_f32):
    g = golden("smollm135m_f16")
    e = _engine(smollm_models["smollm135m_f16"], kv_f32=kv_f32)
    prompt, steps = g["prompt"], int(g["steps"][0])
    e.reset_slot(0)
    rows = []
    for t in prompt:
        out, lg = e.step([t], [0], want_logits=True)
        rows.append(lg[0])
    ids = [int(out[0])]
    for _ in range(steps - 1):
        out, lg = e.step([ids[-1]], [0], want_logits=True)
        rows.append(lg[0])
        ids.append(int(out[0]))
    logits = np.stack(rows)
    assert np.array_equal(np.array(ids, dtype=np.uint32), g["ids_greedy"])
    scale = np.abs(g["head"]).max(axis=1)
    assert np.all(np.abs(logits[:, :64] - g["head"]).max(axis=1) <= 1e-3 * np.maximum(scale, np.abs(g["max"])))
    assert np.array_equal(logits.argmax(axis=1), g["argmax"])


def test_smollm_q8_greedy(smollm_models):
    g = golden("smollm135m_q8")
    e = _engine(smollm_models["smollm135m_q8"])
    ids, _ = e.generate(g["prompt"], int(g["steps"][0]))
    assert np.array_equal(ids, g["ids_greedy"])
