"""One rank of the tensor-parallel parity check (run by tests/test_gpu_tp.py under
torch.distributed.run): every rank loads its shard of the same synthetic model, steps
the same tokens, and rank 0 compares the gathered logits and greedy tokens with the CPU
oracle. Writes one JSON line to the path in argv[1] (rank 0)."""
import datetime
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))

import torch.distributed as dist  # noqa: E402

import evelyn_b200 as evl  # noqa: E402
from evelyn_b200 import synth  # noqa: E402


def main(out_path):
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120))
    spec = synth.tiny(dim=512, ffn=1024, heads=8, kv_heads=4, head_dim=128, vocab=1024, layers=2, seed=5)
    obj = [evl.tp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(obj, src=0)
    img = synth.build(spec)
    m = evl.Model.load_memory(img, device=rank, tp_rank=rank, tp_size=world, nccl_id=obj[0])
    s = evl.Session(m, max_ctx=128)
    toks = [int(t) for t in np.random.default_rng(9).integers(0, spec.vocab, 24)]
    logits = [s.step(t) for t in toks]
    greedy = s.generate(evl.argmax(logits[-1]), 16)
    # a batch of three sequences (tensor-core products, the same exchanges)
    btoks = np.random.default_rng(11).integers(0, spec.vocab, (8, 3))
    bat = evl.Batch(m, 3, max_ctx=64)
    blogits = [bat.step(row) for row in btoks]
    dist.barrier()
    if rank == 0:
        from oracle import oracle as orc
        r = orc.Model(img)
        rs = orc.Session(r)
        worst = 0.0
        for t, lg in zip(toks, logits):
            worst = max(worst, float(np.abs(lg - rs.step(t)).max()))
        want, tok = [], evl.argmax(logits[-1])
        for _ in range(16):
            tok = orc.argmax(rs.step(tok))
            want.append(tok)
        bworst = 0.0
        ors = [orc.Session(r) for _ in range(3)]
        for row, got in zip(btoks, blogits):
            for i in range(3):
                bworst = max(bworst, float(np.abs(got[i] - ors[i].step(int(row[i]))).max()))
        res = {"world": world, "max_abs": worst, "batch_max_abs": bworst, "greedy": list(map(int, greedy)),
               "greedy_oracle": want}
        with open(out_path, "w") as f:
            f.write(json.dumps(res) + "\n")
        rdir = os.environ.get("EVELYN_TP_RESULT_DIR")
        if rdir:
            with open(os.path.join(rdir, f"tp_world{world}.json"), "w") as f:
                f.write(json.dumps(res) + "\n")
    del bat, s, m
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
