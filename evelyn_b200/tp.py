"""Tensor-parallel shard plan of the engine (evl_tp_shard_plan: the split
csrc/model.cpp applies when it loads a model with tp_size > 1), for callers that want
to reason about the shards. Host only: no device needed.

Column split (by output rows): attn_q by query heads, attn_k / attn_v by kv heads,
ffn_gate / ffn_up by FFN rows on 256-value super-block boundaries, the LM head by
vocabulary rows. Row split (by inputs): attn_output over this rank's query-head
dimensions, ffn_down over this rank's FFN rows. The partial outputs of attn_output
and ffn_down are summed across ranks; each rank picks the greedy token of its
vocabulary shard and the ranks agree on the best.
"""
from __future__ import annotations

import ctypes as C
import dataclasses

from . import runtime


@dataclasses.dataclass(frozen=True)
class Shard:
    q_rows: tuple[int, int]      # attn_q rows (and attn_output input columns)
    kv_rows: tuple[int, int]     # attn_k / attn_v rows
    ffn_rows: tuple[int, int]    # ffn_gate / ffn_up rows (and ffn_down input columns)
    vocab_rows: tuple[int, int]  # LM head rows


def shard(heads: int, kv_heads: int, head_dim: int, ffn: int, vocab: int, tp_size: int, rank: int) -> Shard:
    """The engine's shard of rank `rank`; raises EvelynError (InvalidInput / Unsupported)."""
    cfg = runtime._Config()
    cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab = heads, kv_heads, head_dim, ffn, vocab
    out = runtime._TpShard()
    lib = runtime.lib()
    runtime.check(lib.evl_tp_shard_plan(C.byref(cfg), int(tp_size), int(rank), C.byref(out)))
    pair = lambda a: (int(a[0]), int(a[1]))  # noqa: E731
    return Shard(pair(out.q_rows), pair(out.kv_rows), pair(out.ffn_rows), pair(out.vocab_rows))
