"""Python handle on the device engine (tests and the benchmark drive it).

``Engine`` loads a GGUF file, uploads its tensors through ``laic_dev_upload``
and exposes ``prefill``/``step`` — the same calls the C++ LlamaRuntime makes.
``Matrix`` wraps the single-tensor entry points (``laic_tensor_*``).
"""
from __future__ import annotations

import ctypes
from typing import Optional, Sequence, Tuple

import numpy as np

from . import gguf
from ._native import (DevDesc, DevOpts, DevStats, FLAG_KV_F32, FLAG_NO_GRAPH, FLAG_NO_PDL, FLAG_LAYER_LAUNCHES, FLAG_TRACE,
                      FLAG_STEP_KERNEL, FLAG_Q4_0_UPSTREAM, FLAG_NO_SPECULATION, KernelRecord, SampleParams,
                      check, lib)


def sample_params(temperature: float = 0.0, top_k: int = 0, top_p: float = 1.0, repeat_penalty: float = 1.0,
                  seed: int = 0) -> SampleParams:
    return SampleParams(temperature, top_k, top_p, repeat_penalty, seed)


def desc_from_gguf(g: gguf.GgufFile) -> DevDesc:
    md = g.metadata
    h = g.u64("llama.embedding_length")
    heads = g.u64("llama.attention.head_count")
    return DevDesc(hidden=h, layers=g.u64("llama.block_count"), heads=heads,
                   kv_heads=g.u64("llama.attention.head_count_kv", heads), ffn=g.u64("llama.feed_forward_length"),
                   vocab=len(md.get("tokenizer.ggml.tokens", [])), ctx=g.u64("llama.context_length", 2048),
                   rope_dim=g.u64("llama.rope.dimension_count", h // max(1, heads)),
                   rope_theta=g.f64("llama.rope.freq_base", 10000.0),
                   rms_eps=g.f64("llama.attention.layer_norm_rms_epsilon", 1e-5))


class Engine:
    def __init__(self, path: str, max_seqs: int = 1, kv_capacity: int = 0, device: int = 0, kv_f32: bool = False,
                 graphs: bool = True, pdl: bool = True, tp_size: int = 1, tp_rank: int = 0,
                 nccl_id: Optional[bytes] = None, layer_launches: bool = False, trace: bool = False,
                 step_kernel: Optional[bool] = None, q4_0_upstream: bool = False,
                 speculate: bool = True) -> None:
        """`step_kernel`: True runs one-sequence Q4_0/Q8_0 steps as the persistent decode-step kernel, False
        (or `layer_launches`) and None (the default) launch per projection. `q4_0_upstream`: the file's Q4_0
        tensors use upstream ggml's nibble order (llama.cpp's files) rather than the reference's. `speculate`:
        step() starts the next step on its own sampled ids while the caller decides (laic_dev_step)."""
        L = lib()
        if step_kernel is False:
            layer_launches = True
        self.file = gguf.GgufFile(path)
        self.desc = desc_from_gguf(self.file)
        flags = ((FLAG_KV_F32 if kv_f32 else 0) | (0 if graphs else FLAG_NO_GRAPH) | (0 if pdl else FLAG_NO_PDL)
                 | (FLAG_LAYER_LAUNCHES if layer_launches else 0) | (FLAG_TRACE if trace else 0)
                 | (FLAG_STEP_KERNEL if step_kernel else 0) | (FLAG_Q4_0_UPSTREAM if q4_0_upstream else 0)
                 | (0 if speculate else FLAG_NO_SPECULATION))
        self._nccl_id = ctypes.create_string_buffer(nccl_id, 128) if nccl_id else None
        opts = DevOpts(device=device, max_seqs=max_seqs, kv_capacity=kv_capacity, tp_size=tp_size, tp_rank=tp_rank,
                       nccl_id=ctypes.cast(self._nccl_id, ctypes.c_void_p) if self._nccl_id else None, flags=flags)
        self.h = ctypes.c_void_p()
        check(L.laic_dev_create(ctypes.byref(self.desc), ctypes.byref(opts), ctypes.byref(self.h)))
        self.vocab = int(self.desc.vocab)
        self.max_seqs = max_seqs
        for name, ti in self.file.tensors.items():
            self.upload(name, ti.ggml_type, ti.shape, np.asarray(ti.data))

    def upload(self, name: str, ggml_type: int, shape: Sequence[int], raw: np.ndarray) -> None:
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        shp = (ctypes.c_uint64 * len(shape))(*shape)
        check(lib().laic_dev_upload(self.h, name.encode(), ggml_type, shp, len(shape), raw.ctypes.data, raw.nbytes))

    def close(self) -> None:
        if getattr(self, "h", None) and self.h.value:
            lib().laic_dev_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self) -> None:
        self.close()

    def __enter__(self) -> "Engine":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    @staticmethod
    def _arrays(tokens, slots) -> Tuple[np.ndarray, np.ndarray]:
        t = np.ascontiguousarray(np.atleast_1d(tokens), dtype=np.uint32)
        s = np.arange(len(t), dtype=np.int32) if slots is None else np.ascontiguousarray(np.atleast_1d(slots), np.int32)
        return t, s

    def prefill(self, tokens, slots=None) -> None:
        t, s = self._arrays(tokens, slots)
        check(lib().laic_dev_prefill(self.h, len(t), t.ctypes.data, s.ctypes.data))

    def prefill_batch(self, tokens, slot: int = 0) -> None:
        """The prompt tokens of one slot in one pass (tensor-core GEMMs over all of them)."""
        t = np.ascontiguousarray(np.atleast_1d(tokens), dtype=np.uint32)
        check(lib().laic_dev_prefill_batch(self.h, slot, t.ctypes.data, len(t)))

    def step(self, tokens, slots=None, params=None, want_logits: bool = False):
        """Forward pass + sampling for one token per slot; returns (ids, logits or None)."""
        t, s = self._arrays(tokens, slots)
        n = len(t)
        arr = self._params(params, n)
        ids = np.zeros(n, dtype=np.uint32)
        logits = np.zeros((n, self.vocab), dtype=np.float32) if want_logits else None
        check(lib().laic_dev_step(self.h, n, t.ctypes.data, s.ctypes.data, arr, len(arr), ids.ctypes.data,
                                  logits.ctypes.data if logits is not None else None))
        return ids, logits

    def reset_slot(self, slot: int) -> None:
        check(lib().laic_dev_reset_slot(self.h, slot))

    def slot_pos(self, slot: int) -> int:
        v = ctypes.c_int64()
        check(lib().laic_dev_slot_pos(self.h, slot, ctypes.byref(v)))
        return int(v.value)

    def fill_kv(self, slot: int, npos: int, seed: int = 0) -> None:
        check(lib().laic_dev_fill_kv(self.h, slot, npos, seed))

    def sync(self) -> None:
        check(lib().laic_dev_sync(self.h))

    def stats(self) -> DevStats:
        st = DevStats()
        check(lib().laic_dev_stats_get(self.h, ctypes.byref(st)))
        return st

    @property
    def stream(self) -> int:
        return int(lib().laic_dev_stream(self.h) or 0)

    @staticmethod
    def _params(params, n):
        if params is None:
            return (SampleParams * 1)(sample_params())
        if isinstance(params, SampleParams):
            return (SampleParams * 1)(params)
        return (SampleParams * len(params))(*params)

    def decode(self, tokens, slots=None, params=None, steps: int = 1):
        """`steps` chained decode steps on the device; returns (ids[steps][nseq], device_ms)."""
        t, s = self._arrays(tokens, slots)
        arr = self._params(params, len(t))
        out = np.zeros((steps, len(t)), dtype=np.uint32)
        ms = ctypes.c_double()
        check(lib().laic_dev_decode(self.h, len(t), t.ctypes.data, s.ctypes.data, arr, len(arr), steps,
                                    out.ctypes.data, ctypes.byref(ms)))
        return out, ms.value

    def step_trace(self) -> np.ndarray:
        """[CTA][phase][5] globaltimer stamps (ns) of the last persistent step kernel (engines with trace=True):
        start, inputs ready, first warp done, all warps done, done."""
        cap = 200 * 8192 * 5
        out = np.zeros(cap, dtype=np.uint64)
        n, ctas, phases = ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32()
        check(lib().laic_dev_step_trace(self.h, out.ctypes.data, cap, ctypes.byref(n), ctypes.byref(ctas),
                                        ctypes.byref(phases)))
        stamps = ctas.value * phases.value * 5
        self.last_wait_stats = out[stamps: n.value].reshape(ctas.value, -1, 5)
        return out[:stamps].reshape(ctas.value, phases.value, 5)

    def profile(self, tokens: np.ndarray, steps: int) -> dict:
        """Per-kernel-family {name: (launches, total_us, bytes)} over `steps` eager full steps of slots 0..n-1."""
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        nseq = tokens.size // steps
        recs = (KernelRecord * 32)()
        n = ctypes.c_int32()
        check(lib().laic_dev_profile(self.h, nseq, tokens.ctypes.data, steps, recs, 32, ctypes.byref(n)))
        return {recs[i].name.decode(): (recs[i].launches, recs[i].total_us, recs[i].bytes) for i in range(n.value)}

    def generate(self, prompt: np.ndarray, steps: int, params: Optional[SampleParams] = None, slot: int = 0,
                 want_logits: bool = False, batched_prefill: bool = False):
        """Single-sequence generation with the reference loop (no EOS stop); `batched_prefill`
        runs the prompt (all but its last token) in one pass."""
        prompt = np.asarray(prompt, dtype=np.uint32)
        self.reset_slot(slot)
        if batched_prefill:
            self.prefill_batch(prompt[:-1], slot)
        else:
            for tok in prompt[:-1]:
                self.prefill([tok], [slot])
        ids, all_logits = [], []
        tok = int(prompt[-1])
        for i in range(steps):
            out, lg = self.step([tok], [slot], params, want_logits)
            ids.append(int(out[0]))
            if want_logits:
                all_logits.append(lg[0])
            tok = int(out[0])
        return np.array(ids, dtype=np.uint32), (np.stack(all_logits) if want_logits else None)


def nccl_unique_id() -> bytes:
    """128-byte NCCL id for the ranks of one tensor-parallel engine (create on rank 0, share)."""
    buf = ctypes.create_string_buffer(128)
    check(lib().laic_nccl_unique_id(buf))
    return buf.raw


class Matrix:
    """One uploaded weight matrix ([out][in], GGUF shape {in, out}) for the single-tensor entry points."""

    def __init__(self, ggml_type: int, in_dim: int, out_dim: int, raw: np.ndarray, device: int = 0) -> None:
        raw = np.ascontiguousarray(raw, dtype=np.uint8)
        self.h = ctypes.c_void_p()
        self.in_dim, self.out_dim, self.ggml_type = in_dim, out_dim, ggml_type
        check(lib().laic_tensor_create(device, ggml_type, in_dim, out_dim, raw.ctypes.data, raw.nbytes,
                                       ctypes.byref(self.h)))

    @property
    def nbytes(self) -> int:
        return int(lib().laic_tensor_bytes(self.h))

    def matvec(self, x_ptr: int, y_ptr: int, batch: int, stream: int = 0) -> None:
        check(lib().laic_tensor_matvec(self.h, x_ptr, y_ptr, batch, stream))

    def dequant(self, out_ptr: int, stream: int = 0) -> None:
        check(lib().laic_tensor_dequant(self.h, out_ptr, stream))

    def check(self, stream: int = 0) -> None:
        """Synchronise `stream` and raise if a bounded device wait of this tensor's kernels ran out."""
        check(lib().laic_tensor_check(self.h, stream))

    def close(self) -> None:
        if getattr(self, "h", None) and self.h.value:
            lib().laic_tensor_destroy(self.h)
            self.h = ctypes.c_void_p()

    def __del__(self) -> None:
        self.close()


def blocks_convert(ggml_type: int, raw: np.ndarray, n: int, q4_0_upstream: bool = False) -> Tuple[int, np.ndarray]:
    """The device's block type and bytes for `n` elements of GGML blocks (laic_blocks_convert, host only)."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    t, nb = ctypes.c_int32(), ctypes.c_uint64()
    flags = FLAG_Q4_0_UPSTREAM if q4_0_upstream else 0
    check(lib().laic_blocks_convert(ggml_type, raw.ctypes.data, n, flags, ctypes.byref(t), None, 0, ctypes.byref(nb)))
    out = np.zeros(nb.value, dtype=np.uint8)
    check(lib().laic_blocks_convert(ggml_type, raw.ctypes.data, n, flags, ctypes.byref(t), out.ctypes.data, out.nbytes,
                                    ctypes.byref(nb)))
    return t.value, out
