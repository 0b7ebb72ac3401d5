"""ctypes wrapper of the CPU oracle (oracle.cpp) and runner of the reference build.

TEST INFRASTRUCTURE ONLY: imported by tests/, the smoke check and the CPU
baseline leg of bench.py, never by the engine.
"""
from __future__ import annotations

import ctypes
import json
import os
import shutil
import subprocess
import tempfile
from typing import Optional, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblaic_oracle.so")
REF_DIR = os.path.join(HERE, "_ref")


class SampleParams(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_uint32), ("top_p", ctypes.c_float),
                ("repeat_penalty", ctypes.c_float), ("seed", ctypes.c_uint64)]


def reference_dir(ref: Optional[str] = None) -> str:
    """The reference checkout: `ref`, else $LAIC_REF_DIR, else the directory named
    "reference" beside this repository."""
    return ref or os.environ.get("LAIC_REF_DIR") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")


def build(ref: Optional[str] = None) -> None:
    """Compile the oracle library, and the reference drivers when the reference sources exist."""
    targets = ["oracle"]
    src = reference_dir(ref)
    if os.path.isdir(os.path.join(src, "src")):
        targets.append("ref")
    subprocess.run(["make", "-s", "-C", HERE, f"REF={src}", *targets], check=True)


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        L.oracle_load.restype = ctypes.c_void_p
        L.oracle_load.argtypes = [ctypes.c_char_p]
        L.oracle_free.argtypes = [ctypes.c_void_p]
        L.oracle_last_error.restype = ctypes.c_char_p
        L.oracle_arch.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint64)]
        L.oracle_set_l1_tile_bytes.argtypes = [ctypes.c_void_p, ctypes.c_uint64]
        L.oracle_reset.argtypes = [ctypes.c_void_p]
        L.oracle_pos.restype = ctypes.c_uint64
        L.oracle_pos.argtypes = [ctypes.c_void_p]
        L.oracle_step.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        L.oracle_generate.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_size_t,
                                      ctypes.POINTER(SampleParams), ctypes.c_void_p, ctypes.c_void_p]
        L.oracle_sample.restype = ctypes.c_uint32
        L.oracle_sample.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(SampleParams),
                                    ctypes.c_void_p, ctypes.c_size_t]
        L.oracle_value.restype = ctypes.c_float
        L.oracle_value.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64]
        L.oracle_dequant.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_uint64, ctypes.c_void_p]
        L.oracle_matvec.argtypes = [ctypes.c_uint32, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_uint64]
        L.oracle_canonical_u.restype = ctypes.c_double
        L.oracle_canonical_u.argtypes = [ctypes.c_uint64]
        L.oracle_detect_l1d.restype = ctypes.c_uint64
        _lib = L
    return _lib


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    return ctypes.c_void_p(a.ctypes.data)


def params(temperature=0.0, top_k=0, top_p=1.0, repeat_penalty=1.0, seed=0) -> SampleParams:
    return SampleParams(temperature, top_k, top_p, repeat_penalty, seed)


class OracleModel:
    """CPU restatement of LlamaRuntime over one GGUF file."""

    def __init__(self, path: str) -> None:
        L = lib()
        self.h = L.oracle_load(path.encode())
        if not self.h:
            raise RuntimeError(L.oracle_last_error().decode())
        a = (ctypes.c_uint64 * 10)()
        L.oracle_arch(self.h, a)
        (self.hidden, self.layers, self.heads, self.kv_heads, self.head_dim, self.ffn, self.ctx,
         self.rope_dim, self.vocab, self.l1_tile_bytes) = [int(v) for v in a]

    def __del__(self) -> None:
        if getattr(self, "h", None):
            lib().oracle_free(self.h)
            self.h = None

    def set_l1_tile_bytes(self, b: int) -> None:
        lib().oracle_set_l1_tile_bytes(self.h, b)
        self.l1_tile_bytes = b

    def reset(self) -> None:
        lib().oracle_reset(self.h)

    @property
    def pos(self) -> int:
        return int(lib().oracle_pos(self.h))

    def step(self, token: int) -> np.ndarray:
        out = np.empty(self.vocab, dtype=np.float32)
        if lib().oracle_step(self.h, int(token), _ptr(out)) != 0:
            raise RuntimeError(lib().oracle_last_error().decode())
        return out

    def generate(self, prompt: np.ndarray, steps: int, sp: Optional[SampleParams] = None,
                 want_logits: bool = True) -> Tuple[np.ndarray, Optional[np.ndarray]]:
        prompt = np.ascontiguousarray(prompt, dtype=np.uint32)
        ids = np.zeros(steps, dtype=np.uint32)
        logits = np.zeros((steps, self.vocab), dtype=np.float32) if want_logits else None
        sp = sp or params()
        rc = lib().oracle_generate(self.h, _ptr(prompt), len(prompt), steps, ctypes.byref(sp), _ptr(ids),
                                   _ptr(logits) if logits is not None else None)
        if rc != 0:
            raise RuntimeError(lib().oracle_last_error().decode())
        return ids, logits


def sample(logits: np.ndarray, sp: SampleParams, history: np.ndarray) -> int:
    logits = np.ascontiguousarray(logits, dtype=np.float32)
    history = np.ascontiguousarray(history, dtype=np.uint32)
    return int(lib().oracle_sample(_ptr(logits), len(logits), ctypes.byref(sp), _ptr(history), len(history)))


def dequant(ggml_type: int, raw: np.ndarray, n: int) -> np.ndarray:
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    out = np.empty(n, dtype=np.float32)
    lib().oracle_dequant(ggml_type, _ptr(raw), n, _ptr(out))
    return out


def matvec(ggml_type: int, raw: np.ndarray, x: np.ndarray, out_rows: int, in_cols: int,
           l1_tile_bytes: Optional[int] = None) -> np.ndarray:
    """y[b] = W x[b] for W stored GGUF-style ([in, out], rows of ``in`` contiguous)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, in_cols)
    y = np.empty((x.shape[0], out_rows), dtype=np.float32)
    tile = l1_tile_bytes if l1_tile_bytes is not None else int(lib().oracle_detect_l1d()) // 2
    lib().oracle_matvec(ggml_type, _ptr(raw), _ptr(x), _ptr(y), out_rows, in_cols, x.shape[0], tile)
    return y


def canonical_u(seed: int) -> float:
    return float(lib().oracle_canonical_u(seed))


# ----------------------------------------------------------------------------------
# the reference itself (oracle/_ref, built from the reference sources)
# ----------------------------------------------------------------------------------

def ref_driver(kind: str = "strict") -> Optional[str]:
    name = {"strict": "laic_ref_driver", "native": "laic_ref_driver_native", "v3": "laic_ref_driver_v3"}[kind]
    p = os.path.join(REF_DIR, name)
    return p if os.path.exists(p) else None


def ref_dump(model: str, prompt: np.ndarray, steps: int, sp: Optional[SampleParams] = None,
             kind: str = "strict") -> Tuple[np.ndarray, np.ndarray, dict]:
    """Run the reference's step()/sample() loop; returns (ids, logits[prompt+steps-1][V], info)."""
    exe = ref_driver(kind)
    if exe is None:
        raise FileNotFoundError("reference driver not built")
    sp = sp or params()
    d = tempfile.mkdtemp(prefix="laic_ref_")
    try:
        pf = os.path.join(d, "prompt.u32")
        np.ascontiguousarray(prompt, dtype=np.uint32).tofile(pf)
        out = os.path.join(d, "out")
        r = subprocess.run([exe, "dump", model, "--prompt", pf, "--steps", str(steps),
                            "--temperature", repr(float(sp.temperature)), "--top-k", str(sp.top_k),
                            "--top-p", repr(float(sp.top_p)), "--repeat-penalty", repr(float(sp.repeat_penalty)),
                            "--seed", str(sp.seed), "--out", out], check=True, capture_output=True, text=True)
        info = json.loads(r.stdout.strip().splitlines()[-1])
        ids = np.fromfile(out + ".ids.u32", dtype=np.uint32)
        logits = np.fromfile(out + ".logits.f32", dtype=np.float32).reshape(-1, info["vocab"])
        return ids, logits, info
    finally:
        shutil.rmtree(d, ignore_errors=True)
