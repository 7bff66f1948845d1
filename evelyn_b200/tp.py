"""Tensor-parallel shard plan (the same split csrc/model.cpp applies when it loads a
model with tp_size > 1), for callers that want to reason about the shards.

Column split (by output rows): attn_q by query heads, attn_k / attn_v by kv heads,
ffn_gate / ffn_up by FFN rows on 256-value super-block boundaries, the LM head by
vocabulary rows. Row split (by inputs): attn_output over this rank's query-head
dimensions, ffn_down over this rank's FFN rows. The partial outputs of attn_output
and ffn_down are summed across ranks (all-reduce); the vocabulary shards of the
logits are gathered.
"""
from __future__ import annotations

import dataclasses


def split_range(n: int, parts: int, i: int) -> tuple[int, int]:
    """Even split of n items over `parts`: the first n % parts parts get one more."""
    base, rem = divmod(n, parts)
    lo = i * base + min(i, rem)
    return lo, lo + base + (1 if i < rem else 0)


@dataclasses.dataclass(frozen=True)
class Shard:
    q_rows: tuple[int, int]      # attn_q rows (and attn_output input columns)
    kv_rows: tuple[int, int]     # attn_k / attn_v rows
    ffn_rows: tuple[int, int]    # ffn_gate / ffn_up rows (and ffn_down input columns)
    vocab_rows: tuple[int, int]  # LM head rows


def shard(heads: int, kv_heads: int, head_dim: int, ffn: int, vocab: int, tp_size: int, rank: int) -> Shard:
    if kv_heads % tp_size:
        raise ValueError("tp_size must divide head_count_kv")
    if tp_size > 1 and ffn % 256:
        raise ValueError("tensor parallelism needs feed_forward_length % 256 == 0")
    lh, lkv = heads // tp_size, kv_heads // tp_size
    b0, b1 = split_range(ffn // 256, tp_size, rank) if tp_size > 1 else (0, ffn // 256)
    f = (b0 * 256, b1 * 256) if tp_size > 1 else (0, ffn)
    return Shard(q_rows=(rank * lh * head_dim, (rank + 1) * lh * head_dim),
                 kv_rows=(rank * lkv * head_dim, (rank + 1) * lkv * head_dim),
                 ffn_rows=f, vocab_rows=split_range(vocab, tp_size, rank))
