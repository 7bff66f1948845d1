"""Tensor-parallel partition math on the CPU: the engine's own shard plan
(evl_tp_shard_plan, the function model.cpp loads shards with) covers every tensor,
and simulated ranks, each holding its shard of the oracle's dequantised weights,
reproduce the unsharded layer (the reference has one process; its Megatron split is
new here). The 2-rank case also runs as two gloo
processes that all-reduce their FFN partials, the host-side path `bench.py --gpus N`
takes for its plumbing."""
import os

import numpy as np
import pytest

from evelyn_b200 import synth, tp
from oracle import oracle as orc

SPEC = synth.tiny(dim=512, ffn=2560, heads=16, kv_heads=8, head_dim=64, vocab=1000, layers=1, seed=3)


@pytest.fixture(scope="module")
def model():
    img = synth.build(SPEC)
    return img, orc.Model(img)


def silu(z):
    return z / (1 + np.exp(-z))


def W(m, name, rows, cols):
    return m.tensor_f32(name).reshape(rows, cols).astype(np.float64)


@pytest.mark.parametrize("T", [1, 2, 4, 8])
def test_shards_cover_everything(T):
    cover = {k: [] for k in ("q", "kv", "ffn", "vocab")}
    for r in range(T):
        s = tp.shard(SPEC.heads, SPEC.kv_heads, SPEC.head_dim, SPEC.ffn, SPEC.vocab, T, r)
        cover["q"].append(s.q_rows)
        cover["kv"].append(s.kv_rows)
        cover["ffn"].append(s.ffn_rows)
        cover["vocab"].append(s.vocab_rows)
        assert s.ffn_rows[0] % 256 == 0 and s.ffn_rows[1] % 256 == 0
    totals = {"q": SPEC.heads * SPEC.head_dim, "kv": SPEC.kv_heads * SPEC.head_dim, "ffn": SPEC.ffn,
              "vocab": SPEC.vocab}
    for k, ranges in cover.items():
        assert ranges[0][0] == 0 and ranges[-1][1] == totals[k]
        assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))


def test_shard_plan_errors():
    import evelyn_b200 as evl
    with pytest.raises(evl.EvelynError) as e:
        tp.shard(SPEC.heads, SPEC.kv_heads, SPEC.head_dim, SPEC.ffn, SPEC.vocab, 3, 0)  # 3 does not divide 8
    assert e.value.kind == "InvalidInput"
    with pytest.raises(evl.EvelynError) as e:
        tp.shard(SPEC.heads, SPEC.kv_heads, SPEC.head_dim, 1000, SPEC.vocab, 2, 0)  # 1000 % 256 != 0
    assert e.value.kind == "Unsupported"
    with pytest.raises(evl.EvelynError):
        tp.shard(SPEC.heads, SPEC.kv_heads, SPEC.head_dim, SPEC.ffn, SPEC.vocab, 2, 2)  # rank outside


def test_uneven_ffn_blocks_for_32b_shape():
    """Qwen3-32B: 25600 = 100 super-blocks over 8 ranks -> 13/13/13/13/12/12/12/12."""
    sizes = [(lambda s: (s.ffn_rows[1] - s.ffn_rows[0]) // 256)(tp.shard(64, 8, 128, 25600, 151936, 8, r))
             for r in range(8)]
    assert sizes == [13, 13, 13, 13, 12, 12, 12, 12]


@pytest.mark.parametrize("T", [2, 4, 8])
def test_sharded_layer_matches_unsharded(model, T):
    img, m = model
    rng = np.random.default_rng(T)
    d, f, qw = SPEC.dim, SPEC.ffn, SPEC.heads * SPEC.head_dim
    x = rng.standard_normal(d)
    Wq = W(m, "blk.0.attn_q.weight", qw, d)
    Wo = W(m, "blk.0.attn_output.weight", d, qw)
    Wg, Wu = W(m, "blk.0.ffn_gate.weight", f, d), W(m, "blk.0.ffn_up.weight", f, d)
    Wd = W(m, "blk.0.ffn_down.weight", d, f)
    Wl = W(m, "output.weight", SPEC.vocab, d)
    att = rng.standard_normal(qw)
    full_q, full_o = Wq @ x, Wo @ att
    full_ffn = Wd @ (silu(Wg @ x) * (Wu @ x))
    q_parts, o_sum, ffn_sum, logit_parts = [], 0, 0, []
    for r in range(T):
        s = tp.shard(SPEC.heads, SPEC.kv_heads, SPEC.head_dim, f, SPEC.vocab, T, r)
        a, b = s.q_rows
        q_parts.append(Wq[a:b] @ x)
        o_sum = o_sum + Wo[:, a:b] @ att[a:b]
        a, b = s.ffn_rows
        ffn_sum = ffn_sum + Wd[:, a:b] @ (silu(Wg[a:b] @ x) * (Wu[a:b] @ x))
        a, b = s.vocab_rows
        logit_parts.append(Wl[a:b] @ x)
    assert np.allclose(np.concatenate(q_parts), full_q, rtol=0, atol=1e-12)
    assert np.allclose(o_sum, full_o, rtol=0, atol=1e-10)
    assert np.allclose(ffn_sum, full_ffn, rtol=0, atol=1e-10)
    assert np.allclose(np.concatenate(logit_parts), Wl @ x, rtol=0, atol=1e-12)
    # and the unsharded result is the oracle's dense FFN
    xf = x.astype(np.float32)
    assert np.abs(full_ffn - m.dense_ffn(0, xf)).max() < 1e-4


def _rank_main(rank, world, port, path, out):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    m = orc.Model(path)
    d, f = SPEC.dim, SPEC.ffn
    x = np.random.default_rng(0).standard_normal(d).astype(np.float32)
    s = tp.shard(SPEC.heads, SPEC.kv_heads, SPEC.head_dim, f, SPEC.vocab, world, rank)
    a, b = s.ffn_rows
    Wg = W(m, "blk.0.ffn_gate.weight", f, d)[a:b]
    Wu = W(m, "blk.0.ffn_up.weight", f, d)[a:b]
    Wd = W(m, "blk.0.ffn_down.weight", d, f)[:, a:b]
    part = torch.from_numpy(Wd @ (silu(Wg @ x) * (Wu @ x)))
    dist.all_reduce(part)
    if rank == 0:
        np.save(out, part.numpy())
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_allreduce_ffn(model, tmp_path):
    import socket

    import torch.multiprocessing as mp
    img, m = model
    path = str(tmp_path / "tiny.gguf")
    img.write(path)
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    out = str(tmp_path / "ffn.npy")
    mp.start_processes(_rank_main, args=(2, port, path, out), nprocs=2, join=True, start_method="spawn")
    x = np.random.default_rng(0).standard_normal(SPEC.dim).astype(np.float32)
    assert np.abs(np.load(out) - m.dense_ffn(0, x)).max() < 1e-4
