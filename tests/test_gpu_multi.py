"""Tensor-parallel parity on 2, 4 and 8 GPUs (whatever the box has), one process per GPU.

Each case runs ``tests/mgpu_worker.py`` under torchrun (NCCL for the host plumbing; the
data path is the library's in-kernel peer stores) and passes when every rank exits 0:
token rings bit-identical across ranks, gathered vocab-parallel logits corr >= 0.9999
against the CPU oracle at every position, argmax equal to the oracle's and to the same
model at world 1 wherever the oracle's top-2 margin is decided, and, for the MoE block,
outputs bit-identical across ranks with the oracle's expert ids.  Skipped with a reason
when fewer GPUs are visible than the case needs.
"""
import os
import socket
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, case, engine="step", timeout=900):
    n = torch.cuda.device_count()
    if n < world:
        pytest.skip(f"needs {world} GPUs, {n} visible")
    cmd = ["timeout", "-k", "60", str(timeout), sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", "--nproc-per-node", str(world), "--master-addr", "127.0.0.1",
           "--master-port", str(_free_port()), os.path.join(ROOT, "tests", "mgpu_worker.py"), case, engine]
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", OMP_NUM_THREADS="4")
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout + 120)
    for line in r.stdout.splitlines():
        if line.startswith("PARITY"):
            print(line)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-6000:]
    assert r.stdout.count(f"{case} ok") == world, r.stdout[-3000:]


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("engine", ["step", "ops"])
def test_tiny_tensor_parallel(world, engine):
    _run(world, "tiny", engine)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_real_shapes_tensor_parallel(world):
    _run(world, "real2")


@pytest.mark.parametrize("world", [2, 4, 8])
def test_moe_block_sharded(world):
    _run(world, "moe_block")
