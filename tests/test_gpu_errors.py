"""Error behaviour of the C ABI: the reference's messages, no device faults."""
import os
import tempfile

import numpy as np
import pytest

from conftest import golden_model

pytestmark = pytest.mark.gpu


def test_context_length_exceeded():
    from laicompute_b200 import gguf, synth
    from laicompute_b200._native import LAIC_E_CONTEXT, LaicError
    from laicompute_b200.engine import Engine
    arch = synth.tiny_arch(gguf.F16, hidden=64, heads=2, kv_heads=1, ffn=64, vocab=300, ctx=8, name="ctx8")
    with tempfile.TemporaryDirectory() as d:
        e = Engine(synth.write_model(os.path.join(d, "m.gguf"), arch, seed=1))
        for i in range(8):
            e.step([i], [0])
        with pytest.raises(LaicError) as ex:
            e.step([1], [0])
        assert ex.value.code == LAIC_E_CONTEXT and "context length exceeded" in str(ex.value)


def test_bad_arguments():
    from laicompute_b200._native import LAIC_E_INVALID, LaicError
    from laicompute_b200.engine import Engine
    e = Engine(golden_model("tiny_f16"), max_seqs=2)
    with pytest.raises(LaicError) as ex:
        e.step([1, 2], [0, 0])
    assert ex.value.code == LAIC_E_INVALID
    with pytest.raises(LaicError):
        e.step([1], [5])
    with pytest.raises(LaicError) as ex:
        e.step([10**6], [0])
    assert "invalid embedding tensor" in str(ex.value)
    with pytest.raises(LaicError):
        e.step([1, 2, 3], [0, 1, 2])  # more sequences than slots


def test_missing_tensor_reported_by_name():
    from laicompute_b200 import gguf
    from laicompute_b200._native import LAIC_E_MISSING, LaicError, DevOpts, check, lib
    from laicompute_b200.engine import Engine, desc_from_gguf
    import ctypes
    f = gguf.GgufFile(golden_model("tiny_f16"))
    desc = desc_from_gguf(f)
    h = ctypes.c_void_p()
    check(lib().laic_dev_create(ctypes.byref(desc), ctypes.byref(DevOpts(max_seqs=1)), ctypes.byref(h)))
    try:
        for name, ti in f.tensors.items():
            if name == "blk.1.ffn_up.weight":
                continue
            raw = np.ascontiguousarray(np.asarray(ti.data))
            shp = (ctypes.c_uint64 * len(ti.shape))(*ti.shape)
            check(lib().laic_dev_upload(h, name.encode(), ti.ggml_type, shp, len(ti.shape), raw.ctypes.data, raw.nbytes))
        tok = np.array([1], dtype=np.uint32)
        slot = np.array([0], dtype=np.int32)
        rc = lib().laic_dev_prefill(h, 1, tok.ctypes.data, slot.ctypes.data)
        assert rc == LAIC_E_MISSING
        assert lib().laic_last_error().decode() == "missing tensor: blk.1.ffn_up.weight"
    finally:
        lib().laic_dev_destroy(h)


def test_sampler_candidate_limit_reported_then_cleared():
    """A top-k request above the sampler's 1024 candidates fails that step with
    LAIC_E_UNSUPPORTED (the flag travels back with the step's own copies); the next
    step runs normally."""
    from laicompute_b200 import gguf, synth
    from laicompute_b200._native import LAIC_E_UNSUPPORTED, LaicError
    from laicompute_b200.engine import Engine, sample_params
    arch = synth.tiny_arch(gguf.F16, hidden=64, heads=2, kv_heads=1, ffn=64, vocab=4096, ctx=32, name="v4k")
    with tempfile.TemporaryDirectory() as d:
        e = Engine(synth.write_model(os.path.join(d, "m.gguf"), arch, seed=3))
        e.step([1], [0])
        with pytest.raises(LaicError) as ex:
            e.step([2], [0], sample_params(1.0, 2000, 1.0, 1.0, 5))
        assert ex.value.code == LAIC_E_UNSUPPORTED and "1024 candidates" in str(ex.value)
        out, _ = e.step([3], [0])
        assert 0 <= int(out[0]) < arch.vocab


def test_bounded_peer_wait_runs_out_with_an_error_status():
    """The allreduce kernel as rank 0 of two, against a peer mailbox on the same GPU that
    nothing writes, with a ~10 ms flag-wait limit: the wait runs out, the kernel records
    code 4 and returns; the host gets the message and the context keeps working."""
    import ctypes
    from laicompute_b200._native import LAIC_E_CUDA, lib
    code = ctypes.c_int32(-1)
    rc = lib().laic_selftest_peer_timeout(0, 20_000_000, ctypes.byref(code))
    assert rc == LAIC_E_CUDA and code.value == 4
    assert "peer never published" in lib().laic_last_error().decode()
    # the device still runs work afterwards
    from laicompute_b200.engine import Engine
    e = Engine(golden_model("tiny_q4"))
    out, _ = e.step([5], [0])
    assert 0 <= int(out[0]) < 320
    e.close()
