"""Rank process of the multi-GPU parity tests (torchrun, NCCL, one GPU per rank).

    python -m torch.distributed.run --nproc-per-node W --master-addr 127.0.0.1 \\
        --master-port P tests/mgpu_worker.py CASE [ENGINE]

Cases (every rank takes the same collective steps; rank 0 checks; the verdict is
all-reduced so that every rank exits with the same status):
  tiny      -- the tiny parity model (config 1 shapes), tensor parallel over W ranks
  real2     -- two layers [sliding, full] at the 26B-A4B per-layer shapes, 16 experts,
               vocab 16384
  prefill   -- the tensor-parallel prefill (g4_prefill over W ranks) at the real2 shapes,
               300 prompt tokens in 128-row chunks, then 3 decode steps
  moe_block -- the standalone MoE block (config 2: hidden 2816, 128 experts top-8,
               moe_intermediate 704 split 704/W per rank) with its fused all-reduce

For the decode cases: each rank decodes the same prompt with logits written every
step; the vocab-parallel logit slices are gathered into full rows; the token rings of
all ranks must be bit-identical; rank 0 then runs the same model at world 1 on its own
GPU and the CPU oracle (teacher-forced with the world-W tokens) and checks logits corr
>= 0.9999 against the oracle at every position, argmax equal to the oracle's and to
world 1's wherever the oracle's top-2 margin is decided, and prints a PARITY line.
"""
import os
import sys
import traceback
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "kaggle-tpu-inference_b200"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def decided_mask(ref):
    top2 = torch.topk(ref, 2, dim=-1).values
    return (top2[..., 0] - top2[..., 1]) > 2 * top2[..., 0].abs().clamp_min(1e-30) * 2.0 ** -7


def corr(a, b) -> float:
    import numpy as np

    return float(np.corrcoef(a.double().numpy().ravel(), b.double().numpy().ravel())[0, 1])


def decode_run(cfg, params_dev, mesh, prompt, n_new, max_len, engine, comm=None, sampling=None):
    """(logits of this rank's vocab slice [steps, V/W], generated ids) of one decode run;
    ``sampling`` = (temperature, top_p, top_k, seed) draws on the device instead of argmax."""
    from gemma4_b200.runtime import DecodeModel
    from gemma4_b200.weights import rank_shard

    dev = torch.device("cuda", mesh.device)
    shard = rank_shard(cfg, params_dev.__getitem__, mesh, dev)
    m = DecodeModel(cfg, shard, mesh, max_len, comm, engine=engine)
    if sampling:
        m.set_sampling(*sampling)
    m.reset(prompt, write_logits=True)
    out = []
    for _ in range(len(prompt) + n_new - 1):
        m.step(1)
        out.append(m.logits.clone())
    torch.cuda.synchronize(dev)
    m.check_status()
    ring = m.tokens_out.clone()
    m.close()
    return torch.stack(out), ring


def case_decode(cfg, seed, prompt, n_new, max_len, engine):
    from gemma4_b200.model import Mesh
    from gemma4_b200.runtime import Comm
    from gemma4_b200.weights import random_params

    rank, world = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    params_dev = random_params(cfg, seed, device=dev)  # identical on every rank
    mesh = Mesh(rank, world, local)
    comm = Comm(mesh, cfg.hidden_size)
    logits, ring = decode_run(cfg, params_dev, mesh, prompt, n_new, max_len, engine, comm)
    rings = [torch.empty_like(ring) for _ in range(world)]
    dist.all_gather(rings, ring)
    parts = [torch.empty_like(logits) for _ in range(world)]
    dist.all_gather(parts, logits)
    # the same decode sampling on the device (temperature 1, top-p 0.9, top-k 64): every rank
    # merges all ranks' candidates, so the draws must match the restatement on full logits
    samp = (1.0, 0.9, 64, 4242)
    comm.close()  # a communicator's flags count one model's steps: a new model gets a new one
    comm = Comm(mesh, cfg.hidden_size)
    slog, sring = decode_run(cfg, params_dev, mesh, prompt, n_new, max_len, engine, comm, sampling=samp)
    srings = [torch.empty_like(sring) for _ in range(world)]
    dist.all_gather(srings, sring)
    sparts = [torch.empty_like(slog) for _ in range(world)]
    dist.all_gather(sparts, slog)
    comm.close()
    if dist.get_rank() == 0:
        from oracle.reference_model import philox_uniform, sample_token

        for r in range(1, world):
            assert torch.equal(srings[r], srings[0]), f"rank {r} sampled ring differs from rank 0"
        sfull = torch.cat(sparts, dim=-1).cpu()
        p = len(prompt)
        for pos in range(p - 1, p + n_new - 1):
            u = philox_uniform(samp[3], 0 if pos == p - 1 else pos)
            want = sample_token(sfull[pos], samp[0], samp[2], samp[1], u)
            assert int(srings[0][pos + 1]) == want, (pos, int(srings[0][pos + 1]), want)
    msg = None
    if rank == 0:
        for r in range(1, world):
            assert torch.equal(rings[r], rings[0]), f"rank {r} token ring differs from rank 0"
        full = torch.cat(parts, dim=-1).cpu()  # vocab-parallel slices in rank order
        p = len(prompt)
        ids = rings[0][p:p + n_new].cpu().tolist()
        assert ids == full[p - 1:].argmax(-1).tolist(), "written tokens are not the argmax of the logits"
        one, ring1 = decode_run(cfg, params_dev, Mesh(0, 1, local), prompt, n_new, max_len, engine)
        one = one.cpu()
        from oracle.reference_model import Oracle

        params = {k: v.cpu() for k, v in params_dev.items()}
        ref, _ = Oracle(cfg, params, mode="bf16").greedy_generate(prompt, n_new, max_len, teacher=ids)
        dec = decided_mask(ref)
        worst = min(corr(full[i], ref[i]) for i in range(len(ref)))
        max_abs = float((full - ref).abs().max())
        max_rel = max_abs / float(ref.abs().max())
        w1 = min(corr(full[i], one[i]) for i in range(len(ref)))
        assert worst >= 0.9999, worst
        agree = full.argmax(-1) == ref.argmax(-1)
        assert bool(agree[dec].all()), (full.argmax(-1), ref.argmax(-1))
        agree1 = full.argmax(-1) == one.argmax(-1)
        assert bool(agree1[dec].all()), (full.argmax(-1), one.argmax(-1))
        msg = (f"PARITY world{world}[{engine}] positions {len(ref)}: worst corr vs oracle {worst:.7f}, "
               f"vs world 1 {w1:.7f}, max_abs {max_abs:.3e}, max_rel {max_rel:.3e}, "
               f"argmax = world 1 at {int(agree1.sum())}/{len(ref)} ({int(dec.sum())} decided), "
               f"token rings identical on {world} ranks")
    return msg


def case_tiny(engine):
    from gemma4_b200.config import tiny_parity_config

    return case_decode(tiny_parity_config(), 0, list(range(100, 120)), 6, 64, engine)


def case_real2(engine):
    from gemma4_b200.config import FULL, SLIDING, make_config

    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), num_experts=16, vocab_size=16384)
    return case_decode(cfg, 3, [7, 300, 9000, 15000, 42, 1], 4, 64, engine)


def prefill_run(cfg, params_dev, mesh, prompt, chunk, n_dec, max_len, comm=None):
    """(logits of this rank's vocab slice [1 + n_dec, V/W], token ring) of one tensor-core
    prefill of ``prompt`` followed by ``n_dec`` decode steps."""
    from gemma4_b200.runtime import DecodeModel
    from gemma4_b200.weights import rank_shard

    dev = torch.device("cuda", mesh.device)
    m = DecodeModel(cfg, rank_shard(cfg, params_dev.__getitem__, mesh, dev), mesh, max_len, comm)
    p = len(prompt)
    m.reset(prompt, write_logits=True)
    assert m.prefill(p, chunk)
    torch.cuda.synchronize(dev)
    m.check_status()
    assert int(m.ctrl[0]) == p, int(m.ctrl[0])
    out = [m.logits.clone()]
    for _ in range(n_dec):
        m.step(1)
        out.append(m.logits.clone())
    torch.cuda.synchronize(dev)
    m.check_status()
    ring = m.tokens_out.clone()
    m.close()
    return torch.stack(out), ring


def case_prefill(_engine):
    """Tensor-parallel prefill: 300 prompt tokens in 128-row chunks (3 chunks, so the
    exchange slots are reused and later chunks attend to earlier chunks' cache rows) at
    the 26B-A4B per-layer shapes, then 3 decode steps from the prefilled caches."""
    from gemma4_b200.config import FULL, SLIDING, make_config
    from gemma4_b200.model import Mesh
    from gemma4_b200.runtime import Comm
    from gemma4_b200.weights import random_params

    rank, world = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), num_experts=16, vocab_size=16384)
    params_dev = random_params(cfg, 3, device=dev)
    prompt = torch.randint(0, cfg.vocab_size, (300,), generator=torch.Generator().manual_seed(12)).tolist()
    n_dec, max_len, p = 3, 640, len(prompt)
    mesh = Mesh(rank, world, local)
    comm = Comm(mesh, cfg.hidden_size)
    logits, ring = prefill_run(cfg, params_dev, mesh, prompt, 128, n_dec, max_len, comm)
    comm.close()
    rings = [torch.empty_like(ring) for _ in range(world)]
    dist.all_gather(rings, ring)
    parts = [torch.empty_like(logits) for _ in range(world)]
    dist.all_gather(parts, logits)
    if rank != 0:
        return None
    for r in range(1, world):
        assert torch.equal(rings[r], rings[0]), f"rank {r} token ring differs from rank 0"
    full = torch.cat(parts, dim=-1).cpu()
    ids = rings[0][p:p + n_dec + 1].cpu().tolist()
    assert ids == full.argmax(-1).tolist(), "written tokens are not the argmax of the gathered logits"
    one, _ = prefill_run(cfg, params_dev, Mesh(0, 1, local), prompt, 128, n_dec, max_len)
    one = one.cpu()
    from oracle.reference_model import Oracle

    params = {k: v.cpu() for k, v in params_dev.items()}
    o = Oracle(cfg, params, mode="bf16")
    cache = o.new_cache(1, max_len)
    ref_all, cache = o.prefill(cache, prompt, p, dense_moe=True)
    refs = [ref_all[p - 1]]
    for j in range(n_dec):  # teacher-forced with the world-W tokens
        lg, cache = o.decode(cache, ids[j], p + j, max_len)
        refs.append(lg)
    ref = torch.stack(refs)
    dec = decided_mask(ref)
    worst = min(corr(full[i], ref[i]) for i in range(len(ref)))
    w1 = min(corr(full[i], one[i]) for i in range(len(ref)))
    max_abs = float((full - ref).abs().max())
    max_rel = max_abs / float(ref.abs().max())
    assert worst >= 0.9999, worst
    agree = full.argmax(-1) == ref.argmax(-1)
    assert bool(agree[dec].all()), (full.argmax(-1), ref.argmax(-1))
    agree1 = full.argmax(-1) == one.argmax(-1)
    assert bool(agree1[dec].all()), (full.argmax(-1), one.argmax(-1))
    return (f"PARITY prefill world{world} T={p} chunk=128, last prompt position + {n_dec} decode steps: "
            f"worst corr vs oracle {worst:.7f}, vs world 1 {w1:.7f}, max_abs {max_abs:.3e}, "
            f"max_rel {max_rel:.3e}, argmax = oracle where decided ({int(dec.sum())}/{len(ref)}), "
            f"token rings identical on {world} ranks")


def case_moe_block(_engine):
    import ctypes

    from gemma4_b200 import _native as N
    from gemma4_b200.config import make_config
    from gemma4_b200.model import Mesh, param_specs, shard_param
    from gemma4_b200.runtime import Comm
    from gemma4_b200.weights import random_param
    from oracle.reference_model import Oracle

    rank, world = dist.get_rank(), dist.get_world_size()
    local = int(os.environ.get("LOCAL_RANK", rank))
    dev = torch.device("cuda", local)
    cfg = make_config(num_hidden_layers=1, layer_types=("sliding_attention",))
    names = ("router.proj", "router.scale", "router.per_expert_scale", "experts.gate_up_proj",
             "experts.down_proj")
    lp_dev = {n: random_param(cfg, "layers.0." + n, 1, device=dev) for n in names}  # same on every rank
    lp = {n: t.cpu() for n, t in lp_dev.items()}
    x = torch.randn(1, cfg.hidden_size, generator=torch.Generator().manual_seed(1)).to(torch.bfloat16)
    mesh = Mesh(rank, world, local)
    specs = param_specs(cfg)
    d = {n: shard_param(lp_dev[n], specs["layers.0." + n], mesh).contiguous() for n in names}
    comm = Comm(mesh, cfg.hidden_size)
    out = torch.empty(cfg.hidden_size, dtype=torch.bfloat16, device=dev)
    ti = torch.zeros(16, dtype=torch.int32, device=dev)
    tw = torch.zeros(16, dtype=torch.float32, device=dev)
    ctrl = torch.zeros(N.CTRL_WORDS, dtype=torch.int32, device=dev)
    ctrl[N.CTRL_TIMEOUT_US] = 2_000_000
    xg = x[0].to(dev)
    ccfg = N.G4Config.from_text_config(cfg)
    outs = []
    for _ in range(2):  # two calls: the exchange epoch advances between them
        N.check(N.lib().g4_moe_block(
            ctypes.byref(ccfg), rank, world, comm.handle, N.ptr(xg), N.ptr(d["router.proj"]),
            N.ptr(d["router.scale"]), N.ptr(d["router.per_expert_scale"]),
            N.ptr(d["experts.gate_up_proj"]), N.ptr(d["experts.down_proj"]), N.ptr(out), N.ptr(ti),
            N.ptr(tw), N.ptr(ctrl), N.stream_handle()), "g4_moe_block")
        torch.cuda.synchronize(dev)
        outs.append(out.clone())
    assert int(ctrl[N.CTRL_STATUS]) == 0, int(ctrl[N.CTRL_STATUS])
    allo = [torch.empty_like(out) for _ in range(world)]
    dist.all_gather(allo, outs[-1])
    comm.close()
    msg = None
    if rank == 0:
        for r in range(world):
            assert torch.equal(allo[r].view(torch.int16), allo[0].view(torch.int16)), f"rank {r} output differs"
        assert torch.equal(outs[0], outs[1]), "second call differs from the first"
        o = Oracle(cfg, {"layers.0." + k: v for k, v in lp.items()}, mode="bf16")
        top_w, top_i = o.router(lp, x)
        ref = o.moe(lp, x, dense=False)[0]
        k = cfg.top_k_experts
        assert ti[:k].cpu().tolist() == top_i[0].tolist()
        got = allo[0].cpu()
        c = corr(got.float(), ref.float())
        max_abs = float((got.float() - ref.float()).abs().max())
        assert c >= 0.9999, c
        msg = (f"PARITY moe_block world{world}: corr {c:.7f}, max_abs {max_abs:.3e}, "
               f"max_rel {max_abs / float(ref.float().abs().max()):.3e}, expert ids equal, outputs identical "
               f"on {world} ranks")
    return msg


def main():
    case = sys.argv[1]
    engine = sys.argv[2] if len(sys.argv) > 2 else "step"
    local = int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=torch.device("cuda", local))
    failed = 0
    msg = None
    try:
        msg = {"tiny": case_tiny, "real2": case_real2, "moe_block": case_moe_block,
               "prefill": case_prefill}[case](engine)
    except Exception:
        traceback.print_exc()
        failed = 1
    flag = torch.tensor([failed], device=torch.device("cuda", local))
    dist.all_reduce(flag, op=dist.ReduceOp.MAX)
    dist.destroy_process_group()
    if msg:
        print(msg, flush=True)
    if int(flag.item()) == 0:
        print(f"rank {dist_rank()} {case} ok", flush=True)
        return 0
    return 1


def dist_rank():
    return int(os.environ.get("RANK", 0))


if __name__ == "__main__":
    raise SystemExit(main())
