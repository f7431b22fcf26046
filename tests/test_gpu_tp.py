"""Tensor parallel on real GPUs: TP2 (and TP4/TP8 when present) equals TP1.

Spawns one process per GPU with torch.distributed.run (127.0.0.1
rendezvous); each rank runs tests/helpers/tp_worker.py. Skipped on boxes with
fewer than two GPUs.
"""
import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest

from tests.conftest import TOL

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ngpus():
    import torch
    return torch.cuda.device_count()


@pytest.mark.parametrize("world,layers,m,mode", [(2, 2, 1, "nccl"), (2, 2, 8, "nccl"), (2, 3, 1, "ar"), (2, 2, 3, "ar"),
                                                 (2, 3, 8, "ar"), (2, 2, 13, "ar"),
                                                 (2, 3, 1, "trunk"), (4, 2, 1, "ar"), (4, 3, 1, "trunk"),
                                                 (4, 2, 8, "ar"), (8, 2, 1, "ar"), (8, 3, 1, "trunk"),
                                                 (8, 2, 8, "nccl"), (8, 3, 8, "ar"),
                                                 (2, 2, 1, "split"), (2, 2, 8, "split"), (8, 2, 1, "split")])
def test_tensor_parallel_stack_matches_tp1(cuda, tmp_path, world, layers, m, mode):
    """mode "ar": the row-parallel partial sums go through the fused NVLink allreduce
    (cpq_mul_mat_fused_ar); "nccl": through cpq_tp_allreduce_f32; "trunk": the
    persistent trunk kernel (cpq_trunk_run) with the all-reduce inside it."""
    if _ngpus() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "verdict.json"
    env = dict(os.environ, NCCL_DEBUG="WARN")
    cmd = ["timeout", "-k", "30", "300", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
           str(ROOT / "tests" / "helpers" / "tp_worker.py"), str(out), str(layers), str(m), mode]
    res = subprocess.run(cmd, cwd=str(ROOT), env=env, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout[-3000:] + res.stderr[-3000:]
    v = json.loads(out.read_text())
    assert v["fused_ar"] == (mode in ("ar", "trunk", "split")) and v["mode"] == mode
    assert v["ranks_agree"]
    assert v["logits_rel"] <= TOL and v["h_rel"] <= TOL, v
    assert v["tok_tp"] == v["tok_ref"], v
