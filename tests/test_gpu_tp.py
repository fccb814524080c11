"""Tensor parallelism on real GPUs: 2, 4 or 8 ranks (as many as the machine
has) each run their shard of a small GQA decoder through the plugin, with the
plugin's NCCL all-reduce after o_proj and down_proj, and rank 0's logits must
match the oracle's unsharded step."""
import os
import socket
import subprocess
import sys

import numpy as np
import pytest

from tests.conftest import ROOT
from tests.helpers import TOL_BF16

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run_tp(tmp_path, world, mode):
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "tp.npy"
    for _ in range(3):  # a port picked free can be taken before torchrun binds it
        cmd = ["timeout", "-k", "20", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
               os.path.join(ROOT, "tests", "tp_worker.py"), str(out), mode]
        r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
        if r.returncode == 0 or "EADDRINUSE" not in r.stderr:
            break
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    got, want = np.load(out)
    err = float(np.max(np.abs(got - want)) / np.max(np.abs(want)))
    assert err <= TOL_BF16, f"{world}-GPU tensor-parallel {mode} logits differ from unsharded by {err:.3e}"


@pytest.mark.parametrize("world", [2, 4, 8])
def test_multi_gpu_tensor_parallel_decode_matches_unsharded(tmp_path, world):
    """Decode rows: the residual all-reduces run as the fused NVLink
    all-reduce + add + RMSNorm kernel."""
    _run_tp(tmp_path, world, "decode")


@pytest.mark.parametrize("world", [2, 8])
def test_multi_gpu_tensor_parallel_prefill_matches_unsharded(tmp_path, world):
    """Prefill rows (80, more than the fused kernel takes): NCCL all-reduce,
    then the add and the RMSNorm as their own kernels."""
    _run_tp(tmp_path, world, "prefill")


@pytest.mark.parametrize("world", [2, 8])
def test_multi_gpu_vocab_parallel_argmax_is_exact(tmp_path, world):
    """Decode with the vocabulary-parallel lm_head: every rank computes its
    vocabulary rows' logits and fused::vocab_argmax exchanges one 64-bit key
    per row over NVLink.  The ids equal the argmax of the ranks' logits
    gathered in rank order, on every rank."""
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    out = tmp_path / "tp.npy"
    for _ in range(3):
        cmd = ["timeout", "-k", "20", "400", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
               "--nproc-per-node", str(world), "--master-addr", "127.0.0.1", "--master-port", str(_free_port()),
               os.path.join(ROOT, "tests", "tp_worker.py"), str(out), "argmax"]
        r = subprocess.run(cmd, cwd=ROOT, capture_output=True, text=True)
        if r.returncode == 0 or "EADDRINUSE" not in r.stderr:
            break
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    rows = np.load(out)
    assert np.array_equal(rows[0], rows[1]), (rows[0], rows[1])
    for other in rows[2:]:
        assert np.array_equal(other, rows[0]), "ranks disagree on the next-token ids"
