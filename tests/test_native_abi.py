"""The native library builds, loads without a GPU, and exports the C ABI and
the C++ host surface; the host surface parses GGUF and tokenizes like the reference."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

from conftest import ROOT, golden_model

HEADER = os.path.join(ROOT, "include", "laic_b200.h")


@pytest.fixture(scope="module")
def libpath():
    from laicompute_b200 import build
    return build.build()


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(laic_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_abi():
    from laicompute_b200._native import EXPORTS
    assert set(declared_functions()) == set(EXPORTS)


def test_library_exports_every_declared_symbol(libpath):
    lib = ctypes.CDLL(libpath)
    for name in declared_functions():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True, text=True, check=True).stdout
    for name in declared_functions():
        assert re.search(rf"\bT {name}\b", out), name


def test_library_exports_cpp_host_surface(libpath):
    out = subprocess.run(["nm", "-DC", "--defined-only", libpath], capture_output=True, text=True, check=True).stdout
    for sym in ("laic::LlamaRuntime::load(", "laic::LlamaRuntime::generate_ids(", "laic::LlamaRuntime::generate(",
                "laic::GgufModel::load(", "laic::GgufModel::tensor(", "laic::Gpt2Tokenizer::encode(",
                "laic::Gpt2Tokenizer::decode", "laic::GgufTensor::value("):
        assert sym in out, sym


def test_last_error_is_callable_without_gpu(libpath):
    from laicompute_b200._native import lib
    assert lib().laic_last_error() is not None


@pytest.fixture(scope="module")
def host_check(libpath, tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("host") / "host_check")
    subprocess.run(["g++", "-std=c++17", "-O1", f"-I{ROOT}/include", os.path.join(ROOT, "tests", "host", "host_check.cpp"),
                    "-o", exe, f"-L{os.path.dirname(libpath)}", "-llaic_b200", f"-Wl,-rpath,{os.path.dirname(libpath)}"],
                   check=True)
    return exe


def _run(exe, *args):
    return subprocess.run([exe, *map(str, args)], capture_output=True, text=True, check=True).stdout.split()


TEXTS = ["hello world", "The quick brown fox", "café über 123", "a<|endoftext|>b", "  spaces  \n"]


@pytest.mark.parametrize("name", ["tiny_f16", "tiny_q4"])
def test_tokenizer_matches_reference(host_check, name):
    from oracle import oracle as O
    exe = O.ref_driver("strict")
    if exe is None:
        pytest.skip("reference driver not built")
    for text in TEXTS:
        ours = _run(host_check, golden_model(name), "enc", text)
        ref = subprocess.run([exe, "encode", golden_model(name), text], capture_output=True, text=True,
                             check=True).stdout.split()
        assert ours == ref, text


def test_tokenizer_round_trip_and_meta(host_check):
    path = golden_model("tiny_q8")
    meta = _run(host_check, path, "meta")
    assert meta[0] == "320" and meta[-1] == "llama"
    ids = _run(host_check, path, "enc", "round trip")
    hexes = _run(host_check, path, "dec", *ids)
    assert bytes.fromhex("".join(hexes)) == b"round trip"


@pytest.mark.parametrize("name", ["tiny_f16", "tiny_q8", "tiny_q4"])
def test_gguf_tensor_values(host_check, name):
    from laicompute_b200 import gguf
    from oracle import oracle as O
    f = gguf.GgufFile(golden_model(name))
    ti = f.tensors["blk.0.attn_q.weight"]
    idx = [0, 1, 2, 31, 32, 33, 1000, ti.n_elements - 1]
    ours = np.array([float(v) for v in _run(host_check, golden_model(name), "val", "blk.0.attn_q.weight", *idx)],
                    dtype=np.float32)
    ref = O.dequant(ti.ggml_type, np.asarray(ti.data), ti.n_elements)[idx]
    assert np.array_equal(ours, ref)
