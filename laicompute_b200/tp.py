"""Tensor-parallel shard plan of the decode engine (one process per GPU).

The rules are the ones laic_dev_upload applies to each GGUF tensor when
``tp_size > 1`` (laicompute_b200/csrc/engine.cu); they are stated here so the
host side can check a model before creating ranks and so the CPU tests can
replay the decomposition with real collectives:

* ``attn_q`` rows of the rank's query heads, ``attn_k`` / ``attn_v`` rows of
  its KV heads (the KV cache shards with them);
* ``ffn_gate`` / ``ffn_up`` rows ``[r*F/t, (r+1)*F/t)``;
* ``attn_output`` columns of the rank's query heads, ``ffn_down`` columns of
  its FFN rows: their products are partial sums, added up by an allreduce of
  the residual (rank 0 adds its partial to the residual, the others store
  theirs in it);
* lm_head (``output`` or tied ``token_embd``) rows ``[r*V/t, (r+1)*V/t)``,
  all-gathered into every rank's logits; embeddings and norms are replicated.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Tuple


@dataclass(frozen=True)
class ShardPlan:
    hidden: int
    heads: int
    kv_heads: int
    ffn: int
    vocab: int
    tp: int
    rank: int

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    def check(self) -> None:
        """Raise ValueError where the engine answers LAIC_E_UNSUPPORTED / LAIC_E_INVALID."""
        if not 1 <= self.tp <= 8:
            raise ValueError("tp_size must be in [1, 8]")
        if not 0 <= self.rank < self.tp:
            raise ValueError("tp_rank out of range")
        if self.heads % self.tp or self.kv_heads % self.tp:
            raise ValueError("heads and kv_heads must be multiples of tp_size")
        if self.ffn % (32 * self.tp):
            raise ValueError("ffn / tp_size must be a multiple of 32")
        if self.vocab % self.tp:
            raise ValueError("vocab must be a multiple of tp_size")

    # row / column ranges [begin, end) of the full GGUF matrices ([out][in])
    def q_rows(self) -> Tuple[int, int]:
        w = self.heads // self.tp * self.head_dim
        return self.rank * w, (self.rank + 1) * w

    def kv_rows(self) -> Tuple[int, int]:
        w = self.kv_heads // self.tp * self.head_dim
        return self.rank * w, (self.rank + 1) * w

    def o_cols(self) -> Tuple[int, int]:
        return self.q_rows()

    def ffn_rows(self) -> Tuple[int, int]:
        w = self.ffn // self.tp
        return self.rank * w, (self.rank + 1) * w

    def down_cols(self) -> Tuple[int, int]:
        return self.ffn_rows()

    def vocab_rows(self) -> Tuple[int, int]:
        w = self.vocab // self.tp
        return self.rank * w, (self.rank + 1) * w

    def residual_adds(self) -> bool:
        """Whether this rank's o / down epilogue adds into the residual (else stores its partial)."""
        return self.rank == 0
