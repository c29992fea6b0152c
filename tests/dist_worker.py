"""Rank process for the multi-process host tests (launched by torchrun, gloo backend, CPU).

    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port P tests/dist_worker.py CASE

Cases (each rank checks its own view and exits non-zero on a mismatch):
  mesh_handles -- make_mesh() sees the process group; exchange_handles() returns every
                  rank's 64-byte IPC handle in rank order (the layout g4_comm_open takes)
  shards       -- every canonical parameter of the tiny model, sharded by param_specs on
                  each rank, all-gathers back to the full tensor (model.py:120-156 axes)
"""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "kaggle-tpu-inference_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def case_mesh_handles():
    from gemma4_b200.model import make_mesh
    from gemma4_b200.runtime import HANDLE_BYTES, exchange_handles

    mesh = make_mesh()
    assert (mesh.rank, mesh.world) == (dist.get_rank(), dist.get_world_size()), mesh
    mine = bytes([mesh.rank + 1]) * HANDLE_BYTES
    allh = exchange_handles(mine, mesh.world)
    want = b"".join(bytes([r + 1]) * HANDLE_BYTES for r in range(mesh.world))
    assert allh == want, "handles not in rank order"
    try:
        exchange_handles(b"short", mesh.world)
    except ValueError:
        pass
    else:
        raise AssertionError("a malformed handle was accepted")


def case_shards():
    from gemma4_b200.config import tiny_parity_config
    from gemma4_b200.model import make_mesh, param_specs, shard_param
    from gemma4_b200.weights import random_param

    mesh = make_mesh()
    cfg = tiny_parity_config()
    specs = param_specs(cfg)
    for name in sorted(specs):
        full = random_param(cfg, name, seed=0, dtype=torch.float32)
        mine = shard_param(full, specs[name], mesh).contiguous()
        parts = [torch.empty_like(mine) for _ in range(mesh.world)]
        dist.all_gather(parts, mine)
        if "tp" in specs[name]:
            got = torch.cat(parts, dim=specs[name].index("tp"))
        else:  # replicated: every rank holds the whole tensor
            assert all(torch.equal(p, full) for p in parts), name
            got = parts[mesh.rank]
        assert torch.equal(got, full), name


def main():
    case = sys.argv[1]
    dist.init_process_group("gloo", timeout=__import__("datetime").timedelta(seconds=60))
    try:
        {"mesh_handles": case_mesh_handles, "shards": case_shards}[case]()
        dist.barrier()
    finally:
        dist.destroy_process_group()
    print(f"rank {os.environ.get('RANK')} {case} ok", flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
