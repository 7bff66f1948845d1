"""Tensor parallelism on real GPUs: 2 (and 4 when present) ranks, one process per GPU,
the step's exchanges through peer-memory inboxes: a session's logits within the
session tolerance of the CPU oracle and greedy tokens identical, and a three-sequence
batch (tensor-core products) within the same tolerance. Skipped on a box with fewer
GPUs than ranks."""
import json
import os
import socket
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

LOGIT_TOL = 2e-3


def _gpus():
    import torch
    return torch.cuda.device_count()


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_tp_logits_and_greedy_match_oracle(world, tmp_path):
    if _gpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "tp.json"
    here = os.path.dirname(os.path.abspath(__file__))
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr", "127.0.0.1", "--master-port", str(_port()), os.path.join(here, "tp_worker.py"), str(out)]
    r = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    res = json.loads(out.read_text())
    assert res["world"] == world
    assert res["max_abs"] <= LOGIT_TOL, res
    assert res["batch_max_abs"] <= LOGIT_TOL, res
    assert res["greedy"] == res["greedy_oracle"], res
