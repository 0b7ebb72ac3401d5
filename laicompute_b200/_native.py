"""ctypes binding of the C ABI in include/laic_b200.h.

Loading fails loudly when the native library has not been built: there is no
Python or CPU fallback for any engine operation.
"""
from __future__ import annotations

import ctypes
import os

LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "lib", "liblaic_b200.so")

LAIC_OK = 0
LAIC_E_INVALID, LAIC_E_CUDA, LAIC_E_NCCL, LAIC_E_CONTEXT, LAIC_E_UNSUPPORTED, LAIC_E_MISSING = -1, -2, -3, -4, -5, -6
FLAG_NO_GRAPH, FLAG_NO_PDL, FLAG_KV_F32, FLAG_LAYER_LAUNCHES, FLAG_TRACE, FLAG_STEP_KERNEL = 1, 2, 4, 8, 16, 32
FLAG_Q4_0_UPSTREAM = 128
FLAG_NO_SPECULATION = 256

# Every entry point include/laic_b200.h declares (checked by the tests).
EXPORTS = (
    "laic_last_error", "laic_dev_create", "laic_dev_destroy", "laic_dev_upload", "laic_dev_prefill", "laic_dev_step",
    "laic_dev_reset_slot", "laic_dev_slot_pos", "laic_dev_fill_kv", "laic_dev_sync", "laic_dev_stats_get",
    "laic_dev_stream", "laic_dev_decode", "laic_dev_profile", "laic_nccl_unique_id", "laic_tensor_create", "laic_tensor_destroy",
    "laic_tensor_matvec", "laic_tensor_dequant", "laic_tensor_bytes", "laic_tensor_matvec_noalloc",
    "laic_dev_prefill_batch", "laic_tensor_check", "laic_selftest_peer_timeout",
    "laic_dev_step_trace", "laic_blocks_convert",
)


class DevDesc(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_uint32), ("layers", ctypes.c_uint32), ("heads", ctypes.c_uint32),
                ("kv_heads", ctypes.c_uint32), ("ffn", ctypes.c_uint32), ("vocab", ctypes.c_uint32),
                ("ctx", ctypes.c_uint32), ("rope_dim", ctypes.c_uint32), ("rope_theta", ctypes.c_float),
                ("rms_eps", ctypes.c_float)]


class DevOpts(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int32), ("max_seqs", ctypes.c_int32), ("kv_capacity", ctypes.c_int32),
                ("tp_size", ctypes.c_int32), ("tp_rank", ctypes.c_int32), ("nccl_id", ctypes.c_void_p),
                ("flags", ctypes.c_uint32)]


class SampleParams(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_k", ctypes.c_uint32), ("top_p", ctypes.c_float),
                ("repeat_penalty", ctypes.c_float), ("seed", ctypes.c_uint64)]


class DevStats(ctypes.Structure):
    _fields_ = [("weight_bytes", ctypes.c_uint64), ("kv_bytes_per_pos", ctypes.c_uint64),
                ("launches_per_step", ctypes.c_uint32), ("launches_per_prefill", ctypes.c_uint32),
                ("attn_splits", ctypes.c_uint32), ("tp_size", ctypes.c_uint32)]


class KernelRecord(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char * 16), ("launches", ctypes.c_int32), ("total_us", ctypes.c_double),
                ("bytes", ctypes.c_double)]


class LaicError(RuntimeError):
    def __init__(self, code: int, msg: str) -> None:
        super().__init__(f"[{code}] {msg}")
        self.code = code


_lib = None


def lib() -> ctypes.CDLL:
    """The loaded native library (raises if it is missing)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"native engine not built: {LIB_PATH} is missing (run laicompute_b200.build)")
    L = ctypes.CDLL(LIB_PATH)
    P, I32, U32, U64, SZ = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t
    L.laic_last_error.restype = ctypes.c_char_p
    L.laic_last_error.argtypes = []
    L.laic_dev_create.argtypes = [ctypes.POINTER(DevDesc), ctypes.POINTER(DevOpts), ctypes.POINTER(P)]
    L.laic_dev_destroy.argtypes = [P]
    L.laic_dev_destroy.restype = None
    L.laic_dev_upload.argtypes = [P, ctypes.c_char_p, I32, ctypes.POINTER(U64), I32, P, SZ]
    L.laic_dev_prefill.argtypes = [P, I32, P, P]
    L.laic_dev_prefill_batch.argtypes = [P, I32, P, I32]
    L.laic_dev_step.argtypes = [P, I32, P, P, ctypes.POINTER(SampleParams), I32, P, P]
    L.laic_dev_reset_slot.argtypes = [P, I32]
    L.laic_dev_slot_pos.argtypes = [P, I32, ctypes.POINTER(ctypes.c_int64)]
    L.laic_dev_fill_kv.argtypes = [P, I32, I32, U64]
    L.laic_dev_sync.argtypes = [P]
    L.laic_dev_stats_get.argtypes = [P, ctypes.POINTER(DevStats)]
    L.laic_dev_stream.argtypes = [P]
    L.laic_dev_stream.restype = P
    L.laic_dev_decode.argtypes = [P, I32, P, P, ctypes.POINTER(SampleParams), I32, I32, P,
                                  ctypes.POINTER(ctypes.c_double)]
    L.laic_dev_profile.argtypes = [P, I32, P, I32, ctypes.POINTER(KernelRecord), I32, ctypes.POINTER(I32)]
    L.laic_nccl_unique_id.argtypes = [P]
    L.laic_tensor_create.argtypes = [I32, I32, U64, U64, P, SZ, ctypes.POINTER(P)]
    L.laic_tensor_destroy.argtypes = [P]
    L.laic_tensor_destroy.restype = None
    L.laic_tensor_matvec.argtypes = [P, P, P, I32, P]
    L.laic_tensor_dequant.argtypes = [P, P, P]
    L.laic_tensor_bytes.argtypes = [P]
    L.laic_tensor_bytes.restype = U64
    L.laic_tensor_matvec_noalloc.argtypes = [P, P, P, I32, P]
    L.laic_tensor_check.argtypes = [P, P]
    L.laic_dev_step_trace.argtypes = [P, P, ctypes.c_int64, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(I32),
                                      ctypes.POINTER(I32)]
    L.laic_selftest_peer_timeout.argtypes = [I32, ctypes.c_int64, ctypes.POINTER(I32)]
    L.laic_blocks_convert.argtypes = [I32, P, U64, ctypes.c_uint32, ctypes.POINTER(I32), P, U64, ctypes.POINTER(U64)]
    for name in ("laic_dev_create", "laic_dev_upload", "laic_dev_prefill", "laic_dev_step", "laic_dev_reset_slot",
                 "laic_dev_slot_pos", "laic_dev_fill_kv", "laic_dev_sync", "laic_dev_stats_get",
                 "laic_dev_decode", "laic_dev_profile", "laic_nccl_unique_id", "laic_tensor_create", "laic_tensor_matvec",
                 "laic_tensor_dequant", "laic_tensor_matvec_noalloc", "laic_dev_prefill_batch", "laic_tensor_check",
                 "laic_selftest_peer_timeout", "laic_dev_step_trace", "laic_blocks_convert"):
        getattr(L, name).restype = I32
    _lib = L
    return L


def check(rc: int) -> None:
    if rc != LAIC_OK:
        raise LaicError(rc, lib().laic_last_error().decode(errors="replace"))
