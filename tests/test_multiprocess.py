"""World-size-2 host tests of the N > 1 path on the CPU (gloo ranks under torchrun).

The tensor-parallel data path itself (peer stores and flags inside the kernels) needs
GPUs; what runs here is the host plumbing around it: mesh discovery from the process
group, the IPC-handle swap that g4_comm_open consumes, the per-rank sharding of every
parameter, and bench.py's reference arm under torchrun (rank 0 alone reports).
"""
import json
import os
import socket
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def torchrun(args, timeout=300):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2",
           "--master-addr", "127.0.0.1", "--master-port", str(free_port())] + args
    env = dict(os.environ, MASTER_ADDR="127.0.0.1", OMP_NUM_THREADS="2", CUDA_VISIBLE_DEVICES="")
    return subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("case", ["mesh_handles", "shards"])
def test_gloo_world2(case):
    r = torchrun([os.path.join(ROOT, "tests", "dist_worker.py"), case])
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    assert r.stdout.count(f"{case} ok") == 2, r.stdout


def test_reference_arm_reports_on_rank0_only():
    r = torchrun([os.path.join(ROOT, "bench.py"), "--impl", "reference", "--gpus", "2", "--steps", "1",
                  "--warmup", "1", "--layers", "2", "--experts", "16", "--vocab", "4096",
                  "--max-len", "256"], timeout=600)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-4000:]
    lines = [l for l in r.stdout.splitlines() if l.startswith("{")]
    assert len(lines) == 1, r.stdout
    line = json.loads(lines[0])
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port"
    assert line["e2e"]["h2d_bytes_per_step"] == 0
