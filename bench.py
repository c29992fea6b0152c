#!/usr/bin/env python3
"""Decode benchmark of the B200 Gemma-4 26B-A4B path (headline metric: benchmark config 4).

Workload (config 4): the 26B-A4B-shaped model with seeded random bf16 weights N(0,0.02)
(seed 3; global head_dim 256 as the benchmark configuration states), batch-1 greedy decode with a
32,768-token resident KV cache, a 32-token random prompt, then decode steps.  A step
is one decoded token; the timed steps continue the same sequence (positions
32+W .. 32+W+K), so the default W=16, K=752 covers exactly config 4's 768 tokens.

value       tokens/s of the captured step graph, K steps between CUDA events on the
            launching stream (barrier + synchronize on both sides, max over ranks).
            Inputs are larger than L2 (7.4 GB of weights stream per step).
e2e         the same metric through the public API: Engine.generate() with the prompt
            uploaded from host memory and every token read back to the host, wall
            clock from the call to the last token (includes prefill).
roofline    the dominant kernel.  With the default step-kernel engine that is the one
            persistent kernel of the step (one launch per token): algorithmic bytes
            per token (weights + live KV) / mean launch duration from the same CUDA
            events, against the measured HBM copy peak (MEASURED_PEAKS.json).  With
            --engine ops it is the kernel class with the largest time share of
            event-separated per-op steps.
op_kernels  per-class time shares of event-separated per-op steps (both engines; the
            per-op kernels compute the same operators as the step kernel).
cpu_baseline  the CPU oracle (restatement of the reference forward, oracle/) timing a
            bounded sample of full-size decode steps on the host cores (rank 0, N=1).

``--impl reference`` times that CPU implementation alone (rank 0; other ranks exit 0).
Multi-GPU: tensor parallel over N ranks (torchrun, one GPU each); every rank decodes
the same token, so total work per token is fixed ("scaling": "strong").
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "kaggle-tpu-inference_b200"))

METRIC = "decode tok/s @32K ctx, bs=1"
FALLBACK_HBM_GBS = 6650.0

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one full-size launch of
# the step kernel, keyed by (world, layers), as measured by ncu (launch-list capture of
# this bench, one metric pass) on the build named beside it; re-captured when the kernel
# changes.  None where no capture exists (reported as null).
NCU_STEP_TRAFFIC_BYTES_PER_LAUNCH: dict = {
    (1, 30): (7.41e9 + 20.12e6, "step kernel of commit 680ec0c, config 4, launch at position 36"),
}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=752)
    ap.add_argument("--warmup", type=int, default=16)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--max-len", type=int, default=32768)
    ap.add_argument("--prompt-len", type=int, default=32)
    ap.add_argument("--global-head-dim", type=int, default=256)
    ap.add_argument("--seed", type=int, default=3)
    ap.add_argument("--profile-steps", type=int, default=4)
    ap.add_argument("--cpu-steps", type=int, default=8)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-blocks", action="store_true", help="skip the config 2 / 3 block legs")
    ap.add_argument("--prefill-only", action="store_true", help="profiling: run only the prefill leg")
    ap.add_argument("--blocks-only", action="store_true", help="profiling: run only the block legs")
    ap.add_argument("--long-context-steps", type=int, default=20,
                    help="steps timed at the end of the 32K cache (all keys live); 0 skips")
    ap.add_argument("--prefill-tokens", type=int, default=4096,
                    help="benchmark config 5 prompt length for the prefill (TTFT) leg; 0 skips it")
    ap.add_argument("--batch-size", type=int, default=8,
                    help="benchmark config 5 batched decode: sequences (0 skips the leg)")
    ap.add_argument("--batch-steps", type=int, default=256, help="config 5: tokens decoded per sequence")
    ap.add_argument("--batch-ctx", type=int, default=8192, help="config 5: cache positions per sequence")
    ap.add_argument("--batch-prompt", type=int, default=4096, help="config 5: prompt length per sequence")
    ap.add_argument("--batch-only", action="store_true", help="profiling: run only the batched-decode leg")
    ap.add_argument("--engine", choices=["step", "ops"], default="step")
    # profiling knobs (smaller models for ncu captures); defaults are config 4
    ap.add_argument("--layers", type=int, default=30)
    ap.add_argument("--experts", type=int, default=128)
    ap.add_argument("--vocab", type=int, default=262144)
    return ap.parse_args()


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def prompt_ids(cfg, n, seed):
    import torch

    g = torch.Generator().manual_seed(seed)
    return torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist()


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, devices):
        self.devices = devices
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def start(self):
        try:
            self.fh = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", ",".join(str(d) for d in self.devices), "-lms", "100"],
                stdout=self.fh, stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        sm, smax, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        with open(self.path) as f:
            for line in f:
                cols = [c.strip() for c in line.split(",")]
                if len(cols) < 9:
                    continue
                try:
                    sm.append(float(cols[1]))
                    smax.append(float(cols[2]))
                except ValueError:
                    continue
                for n, v in zip(names, cols[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(n)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------- bytes
def class_bytes(cfg, world, pos_avg):
    """Algorithmic HBM bytes per step of each kernel class on one rank (bf16 weights)."""
    H = cfg.hidden_size
    I, F, E, K = cfg.intermediate_size // world, cfg.moe_intermediate_size // world, cfg.num_experts, cfg.top_k_experts
    b = dict.fromkeys(("qkv", "attention", "o_proj", "router_mlp_up", "mlp_down_experts_up",
                       "experts_down", "lm_head_argmax"), 0.0)
    for lt in cfg.layer_types:
        d, kv = cfg.head_dim_for(lt), cfg.kv_heads_for(lt)
        g = cfg.num_attention_heads // kv
        if lt == "sliding_attention":
            n_kv, gl = kv // world, g
            live = min(pos_avg + 1, cfg.sliding_window)
        else:
            n_kv, gl = kv, g // world
            live = pos_avg + 1
        rq = n_kv * gl * d
        rkv = n_kv * d * (1 if cfg.k_eq_v_for(lt) else 2)
        b["qkv"] += 2 * (rq + rkv) * H
        b["attention"] += 2 * 2 * live * n_kv * d
        b["o_proj"] += 2 * H * rq
        b["router_mlp_up"] += 2 * (E * H + 2 * I * H)
        b["mlp_down_experts_up"] += 2 * (H * I + K * 2 * F * H)
        b["experts_down"] += 2 * K * H * F
    b["lm_head_argmax"] += 2 * (cfg.vocab_size // world) * H
    return b


def step_bytes(cfg, pos_avg):
    """Algorithmic bytes per token for the whole model (2 x active params + live KV)."""
    from gemma4_b200.weights import active_params_per_token

    kv = 0
    for lt in cfg.layer_types:
        live = min(pos_avg + 1, cfg.sliding_window) if lt == "sliding_attention" else pos_avg + 1
        kv += 2 * 2 * live * cfg.kv_heads_for(lt) * cfg.head_dim_for(lt)
    return 2 * active_params_per_token(cfg) + kv


# ----------------------------------------------------------------------------- CPU arm
def cpu_decode_sample(cfg, max_len, n_steps, n_warm=1):
    """Time full-size decode steps of the CPU oracle (reference algorithm) on all cores.

    Zero-valued weights; arithmetic time does not depend on the values.  With a zero
    router every expert ties and the stable top-k picks experts 0..k-1, so expert
    tensors are allocated uninitialised (pages are committed only when touched) and
    only those k experts are zeroed: host memory stays ~15 GB instead of 47 GB.  The
    step attends over the whole max_len cache under the mask, exactly like the
    reference decode (gemma4_tpu/engine.py:77).
    """
    import torch

    from oracle.reference_model import Oracle, param_shapes

    torch.set_num_threads(os.cpu_count() or 1)
    params = {}
    for n, s in param_shapes(cfg).items():
        if "experts." in n:
            t = torch.empty(s, dtype=torch.bfloat16)
            t[: cfg.top_k_experts].zero_()
        elif n.endswith("layer_scalar"):
            t = torch.ones(s, dtype=torch.bfloat16)
        else:
            t = torch.zeros(s, dtype=torch.bfloat16)
        params[n] = t
    o = Oracle(cfg, params, mode="bf16")
    cache = o.new_cache(1, max_len)
    pos = 32
    for _ in range(n_warm):
        _, cache = o.decode(cache, 1, pos, max_len)
        pos += 1
    t0 = time.perf_counter()
    for _ in range(n_steps):
        _, cache = o.decode(cache, 1, pos, max_len)
        pos += 1
    dt = time.perf_counter() - t0
    return n_steps / dt, torch.get_num_threads()


def run_reference(args, cfg, rank, world, workload):
    if rank != 0:
        return 0
    steps = max(1, min(args.steps, args.cpu_steps))
    warm = min(args.warmup, 3)  # the CPU step is ~1.5 s: at most 3 warm-up steps
    value, cores = cpu_decode_sample(cfg, args.max_len, steps, warm)
    sample = (f"{steps} timed full-size decode step(s) after {warm} warm-up at position 32+, "
              f"max_len {args.max_len}, CPU restatement of the reference forward (oracle/)")
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "impl": "reference",
        "n_gpus": world, "steps": steps, "warmup": warm, "ms_per_step": 1000.0 / value,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic", "config": workload,
        "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": sample},
        "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- prefill
def prefill_flops(cfg, T, dense):
    """FLOPs of one prefill of T tokens as run (world 1): projections, attention over the
    causal / sliding band, router, the MoE over all experts (dense) or the top-k (routed),
    and the last position's LM head."""
    H, E, F, I, K = (cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size, cfg.intermediate_size,
                     cfg.top_k_experts)
    tot = 0.0
    for lt in cfg.layer_types:
        d, kv = cfg.head_dim_for(lt), cfg.kv_heads_for(lt)
        nq = cfg.num_attention_heads
        rows = nq * d + kv * d * (1 if cfg.k_eq_v_for(lt) else 2)
        keys = T / 2 if lt == "full_attention" else min(cfg.sliding_window, T / 2)  # mean live keys
        moe = (E if dense else K) * 3 * F * H
        tot += 2.0 * T * (H * rows + nq * d * H + 3 * H * I + H * E + moe) + 4.0 * T * keys * d * nq
    return tot + 2.0 * H * cfg.vocab_size


def prefill_leg(eng, cfg, args, dev, world=1):
    """Benchmark config 5's prefill: a prompt of --prefill-tokens random ids (seed 4)
    through g4_prefill (tcgen05 GEMMs), timed with CUDA events (best of 2 after one
    warm-up) in both MoE modes (routed only under tensor parallelism, where every rank
    prefills its shard and the time is the max over ranks); TTFT ms and tensor-core
    throughput of the whole job against the measured bf16 peak x ranks.  Weights are the
    bench model's (values do not change the timing)."""
    import torch
    import torch.distributed as dist

    T = min(args.prefill_tokens, args.max_len - 1)
    g = torch.Generator().manual_seed(4)
    prompt = torch.randint(0, cfg.vocab_size, (T,), generator=g).tolist()
    m = eng.model
    out = {"tokens": T, "workload": f"benchmark config 5 prefill (one prompt, tp{world})"}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak = float(json.load(f)["bf16_tflops"])
        peak_kind = "measured"
    except (OSError, KeyError, ValueError):
        peak, peak_kind = 1590.0, "fallback"
    for dense in ((False, True) if world == 1 else (False,)):
        times = []
        for rep in range(3):
            m.reset(prompt)
            torch.cuda.synchronize(dev)
            if world > 1:
                dist.barrier()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            m.prefill(T, 0, dense_moe=dense)
            e1.record()
            torch.cuda.synchronize(dev)
            t = e0.elapsed_time(e1)
            if world > 1:
                tt = torch.tensor([t], device=dev, dtype=torch.float64)
                dist.all_reduce(tt, op=dist.ReduceOp.MAX)
                t = float(tt.item())
            if rep:
                times.append(t)
        m.check_status()
        ms = min(times)
        key = "dense_moe" if dense else "routed_moe"
        fl = prefill_flops(cfg, T, dense)
        out[key] = {"ttft_ms": ms, "tflops_as_run": fl / ms / 1e9, "flops_as_run": fl,
                    "useful_tflops": prefill_flops(cfg, T, False) / ms / 1e9,
                    "frac_of_bf16_peak": fl / ms / 1e9 / (peak * world)}
    out["bf16_peak_tflops"] = peak * world
    out["peak_kind"] = peak_kind
    return out


# ----------------------------------------------------------------------------- batched decode
def batch_step_bytes(cfg, B, pos_avg):
    """Algorithmic HBM bytes of one batched step (world 1): every dense weight once, the
    union of the B tokens' routed experts per layer (its expected size under uniform
    routing, E (1 - (1 - k/E)^B): the union is data-dependent) and every sequence's live
    keys and values."""
    b = class_bytes(cfg, 1, pos_avg)
    H, F, E, K = cfg.hidden_size, cfg.moe_intermediate_size, cfg.num_experts, cfg.top_k_experts
    L = len(cfg.layer_types)
    union = E * (1.0 - (1.0 - K / E) ** B)
    experts_top_k = L * 2 * 3 * K * F * H
    experts_union = L * 2 * 3 * union * F * H
    total = sum(b.values()) - b["attention"] - experts_top_k + experts_union + B * b["attention"]
    return total, union


def batch_leg(eng, cfg, args, dev):
    """Benchmark config 5's decode: --batch-size sequences (seed 4 + s), each a prompt of
    --batch-prompt random ids through the tensor-core prefill into its own
    --batch-ctx-position cache, then --batch-steps greedy tokens of every sequence, the
    step replayed as one CUDA graph; device time with CUDA events over the decode steps."""
    import torch

    from gemma4_b200.runtime import BatchDecoder

    B, ctx = args.batch_size, args.batch_ctx
    P = min(args.batch_prompt, ctx - args.batch_steps - 2)
    m = eng.model
    bd = BatchDecoder(m, B, ctx)
    for s in range(B):
        g = torch.Generator().manual_seed(4 + s)
        bd.prefill(s, torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist())
    bd.step(graph=True)  # eager (captures nothing yet)
    bd.step(graph=True)  # captures, replays
    bd.step(graph=True)
    torch.cuda.synchronize(dev)
    n = args.batch_steps - 3
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(n):
        bd.step(graph=True)
    e1.record()
    torch.cuda.synchronize(dev)
    bd.check_status()
    ms = e0.elapsed_time(e1) / n
    peak, peak_kind = peaks()
    byts, union = batch_step_bytes(cfg, B, P + args.batch_steps // 2)
    out = {"workload": f"benchmark config 5 decode: batch {B}, {P}-token prompts, {args.batch_steps} tokens each, "
                       f"{ctx}-position caches (world 1)",
           "tok_per_s": B / ms * 1e3, "ms_per_step": ms, "steps_timed": n,
           "bytes_per_step": byts, "expected_experts_per_layer": union,
           "achieved_gbs": byts / ms / 1e6, "peak_gbs": peak, "peak_kind": peak_kind,
           "frac": byts / ms / 1e6 / peak, "graph": True}
    m.batch_owner = None
    del bd
    return out


# ----------------------------------------------------------------------------- blocks
def block_legs(args, dev, reps=20):
    """Benchmark configs 2 and 3 through their C-ABI block entry points, world 1: the MoE
    block (router + top-8 experts, hidden 2816, 128 experts, F 704, seed 1) and decode
    attention over a 32,768-row cache (sliding: 16 q / 8 KV heads, window 1024; full k==v:
    16 q / 2 KV heads, 32,768 live keys), d 256, at the last position.  Each call is timed
    alone with CUDA events after a 256 MB write that flushes L2; achieved GB/s = the
    call's algorithmic bytes / mean time, against the measured HBM copy peak."""
    import ctypes

    import torch

    from gemma4_b200 import _native as N
    from gemma4_b200.config import make_config
    from gemma4_b200.weights import random_param

    peak, peak_kind = peaks()
    L = N.lib()
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    st = N.stream_handle()

    def timed(call):
        ts = []
        for _ in range(reps + 2):
            flush.fill_(1)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            call()
            e1.record()
            torch.cuda.synchronize(dev)
            ts.append(e0.elapsed_time(e1))
        return sum(ts[2:]) / reps  # ms, after 2 warm-up calls

    out = {"l2_policy": "256 MB L2 flush before each timed call", "peak_gbs": peak, "peak_kind": peak_kind}
    # ---- config 2: MoE block
    cfg = make_config(num_hidden_layers=1, layer_types=("sliding_attention",))
    names = ("router.proj", "router.scale", "router.per_expert_scale", "experts.gate_up_proj", "experts.down_proj")
    w = {n: random_param(cfg, "layers.0." + n, 1, device=dev) for n in names}
    g = torch.Generator(device=dev).manual_seed(1)
    xs = [torch.randn(cfg.hidden_size, device=dev, generator=g).to(torch.bfloat16) for _ in range(reps + 2)]
    o = torch.empty(cfg.hidden_size, dtype=torch.bfloat16, device=dev)
    ctrl = torch.zeros(N.CTRL_WORDS, dtype=torch.int32, device=dev)
    ccfg = N.G4Config.from_text_config(cfg)
    it = iter(range(10 ** 9))

    def moe():
        x = xs[next(it) % len(xs)]  # a new token each call: new experts, no L2 reuse
        N.check(L.g4_moe_block(ctypes.byref(ccfg), 0, 1, None, N.ptr(x), N.ptr(w["router.proj"]),
                               N.ptr(w["router.scale"]), N.ptr(w["router.per_expert_scale"]),
                               N.ptr(w["experts.gate_up_proj"]), N.ptr(w["experts.down_proj"]), N.ptr(o), None,
                               None, N.ptr(ctrl), st), "g4_moe_block")

    ms = timed(moe)
    H, E, F, K = cfg.hidden_size, cfg.num_experts, cfg.moe_intermediate_size, cfg.top_k_experts
    b = 2 * (E * H + K * 3 * F * H)
    out["moe_block_config2"] = {"us": 1000 * ms, "algorithmic_bytes": b, "achieved_gbs": b / ms / 1e6,
                                "frac": b / ms / 1e6 / peak, "kernels": 3}
    del w, xs
    # ---- config 3: decode attention at position 32767
    max_len, d = 32768, 256
    for name, nq, nkv, window, theta, partial, kv_eq in (("attention_sliding_config3", 16, 8, 1024, 1e4, 1.0, 0),
                                                          ("attention_full_kv_config3", 16, 2, 0, 1e6, 0.25, 1)):
        rows = nq * d + nkv * d * (1 if kv_eq else 2)
        qkv = torch.randn(rows, device=dev, generator=g).to(torch.bfloat16)
        qn = torch.ones(d, dtype=torch.bfloat16, device=dev)
        ck = torch.randn(max_len, nkv, d, device=dev, generator=g).to(torch.bfloat16)
        cv = torch.randn(max_len, nkv, d, device=dev, generator=g).to(torch.bfloat16)
        ctx = torch.empty(nq * d, dtype=torch.bfloat16, device=dev)
        pos = max_len - 1

        def attn():
            N.check(L.g4_attention_decode(N.ptr(qkv), N.ptr(qn), N.ptr(qn), N.ptr(ck), N.ptr(cv), max_len, nq, nkv,
                                          d, kv_eq, pos, window, theta, partial, 1e-6, N.ptr(ctx), st),
                    "g4_attention_decode")

        ms = timed(attn)
        live = min(window, pos + 1) if window else pos + 1
        b = 2 * 2 * live * nkv * d + 2 * rows + 2 * nq * d  # K and V rows read, q|k|v in, ctx out
        out[name] = {"us": 1000 * ms, "live_keys": live, "algorithmic_bytes": b, "achieved_gbs": b / ms / 1e6,
                     "frac": b / ms / 1e6 / peak}
        del ck, cv
    return out


# ----------------------------------------------------------------------------- GPU arm
def tokens_check(generated, prompt, cfg, args, world, rank, local, dev):
    """N > 1: the timed run's generated tokens must be identical on every rank; rank 0
    also replays the same prompt and step count with the same model at world 1 on its
    own GPU and reports how long a prefix of the sequence agrees (greedy decoding at a
    top-2 near-tie may go either way when the partial sums are added in another order)."""
    import torch
    import torch.distributed as dist

    allt = [torch.empty_like(generated) for _ in range(world)]
    dist.all_gather(allt, generated)
    same = all(torch.equal(t, allt[0]) for t in allt)
    out = {"ranks_identical": same, "tokens": int(generated.numel())}
    if rank == 0:
        from gemma4_b200.engine import Engine
        from gemma4_b200.model import Mesh

        one = Engine(None, max_len=args.max_len, cfg=cfg, random_seed=args.seed, mesh=Mesh(0, 1, local),
                     engine=args.engine)
        m1 = one.model
        m1.reset(prompt)
        m1.step(len(prompt) + args.warmup + args.steps)
        torch.cuda.synchronize(dev)
        m1.check_status()
        ref = m1.tokens_out[len(prompt):len(prompt) + generated.numel()].cpu()
        got = generated.cpu()
        diff = (ref != got).nonzero()
        out["world1_equal_prefix"] = int(diff[0, 0]) if len(diff) else int(got.numel())
        out["world1_identical"] = not len(diff)
        if len(diff):
            # the world-1 logits of the step that produced the first differing token: its
            # top-2 margin in bf16 ulps of the top logit (<= ~2: a tie that either order of
            # the partial sums may break differently)
            j = int(diff[0, 0])
            m1.reset(prompt, write_logits=True)
            m1.step(len(prompt) + j)
            torch.cuda.synchronize(dev)
            top2 = torch.topk(m1.logits.float(), 2).values.cpu()
            ulp = float(top2[0].abs()) * 2.0 ** -7
            out["divergence_top2_margin_ulps"] = float(top2[0] - top2[1]) / max(ulp, 1e-30)
        m1.close()
        del one, m1
        torch.cuda.empty_cache()
    dist.barrier()
    return out


def main() -> int:
    args = parse_args()
    world = int(os.environ.get("WORLD_SIZE", args.gpus))
    rank = int(os.environ.get("RANK", 0))
    local = int(os.environ.get("LOCAL_RANK", rank))

    from gemma4_b200.config import make_config

    cfg = make_config(global_head_dim=args.global_head_dim, num_hidden_layers=args.layers,
                      num_experts=args.experts, vocab_size=args.vocab)
    workload = {
        "workload": "benchmark config 4: 26B-A4B-shaped random model (seed 3), bs=1 greedy decode, "
                    "32K resident KV cache, 32-token prompt",
        "model": "gemma-4-26B-A4B-shape (random init)", "global_head_dim": args.global_head_dim,
        "max_len": args.max_len, "prompt_len": args.prompt_len, "global_batch": 1,
        "parallelism": f"tp{world}", "l2_policy": "inputs larger than L2 (7.4 GB weights per step)",
    }
    if (args.layers, args.experts, args.vocab) != (30, 128, 262144):
        workload["workload"] = (f"profiling case: {args.layers} layers, {args.experts} experts, "
                                f"vocab {args.vocab} (not config 4)")
    if args.impl == "reference":
        return run_reference(args, cfg, rank, world, workload)

    import torch
    import torch.distributed as dist

    if world > 1:
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    from gemma4_b200.engine import Engine
    from gemma4_b200.model import Mesh

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    mesh = Mesh(rank, world, local)
    if args.blocks_only:  # profiling case: the config 2 / 3 block legs alone, one JSON line
        if rank == 0:
            print(json.dumps({"metric": "block kernels", "blocks": block_legs(args, dev, reps=args.steps)}),
                  flush=True)
        return 0
    eng = Engine(None, max_len=args.max_len, cfg=cfg, random_seed=args.seed, mesh=mesh,
                 engine=args.engine)
    if args.batch_only:  # profiling case: the batched-decode leg alone, one JSON line
        line = {"metric": "batched decode tok/s", "batch": batch_leg(eng, cfg, args, dev) if world == 1 else None}
        if rank == 0:
            print(json.dumps(line), flush=True)
        return 0
    if args.prefill_only:  # profiling case: the prefill leg alone, one JSON line
        line = {"metric": "prefill TTFT ms", "config": workload,
                "prefill": prefill_leg(eng, cfg, args, dev, world)}
        if rank == 0:
            print(json.dumps(line), flush=True)
        return 0
    eng.compile_all()
    m = eng.model
    prompt = prompt_ids(cfg, args.prompt_len, args.seed)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- device-timed decode steps (the captured graph)
    m.reset(prompt)
    m.step(len(prompt))
    m.step(args.warmup)
    barrier()
    sampler = ClockSampler([local] if world == 1 else list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    m.step(args.steps)
    e1.record()
    barrier()
    clocks = sampler.stop() if sampler else None
    ms = e0.elapsed_time(e1)
    m.check_status()
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = args.steps / (ms / 1000.0)
    pos_avg = len(prompt) + args.warmup + args.steps // 2
    n_gen = args.warmup + args.steps + 1  # tokens generated after the prompt
    generated = m.tokens_out[len(prompt):len(prompt) + n_gen].clone()
    tokens_match = tokens_check(generated, prompt, cfg, args, world, rank, local, dev) if world > 1 else None

    # ---- the same steps with 32K live keys: decode at the end of the resident cache, where
    # every full layer attends to the whole cache and every sliding layer to its full window
    # (the reference's decode cost at any position; here the worst case)
    long_ctx = None
    if args.long_context_steps > 0:
        n_long = args.long_context_steps
        p0 = args.max_len - n_long - 1
        m.reset(prompt)
        m.ctrl[0] = p0  # positions p0.. read tokens_out (their values do not change the time)
        m.step(2)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        m.step(n_long - 2)
        e1.record()
        barrier()
        m.check_status()
        lms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([lms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            lms = float(t.item())
        lpos = p0 + n_long // 2
        lb = sum(class_bytes(cfg, world, lpos).values())
        lval = (n_long - 2) / (lms / 1000.0)
        long_ctx = {"position": lpos, "live_keys_full_layers": lpos + 1, "value": lval, "unit": "tok/s",
                    "ms_per_step": lms / (n_long - 2), "bytes_per_launch_rank": lb,
                    "achieved_gbs_rank": lb / (lms / (n_long - 2) / 1000.0) / 1e9}
        long_ctx["frac"] = long_ctx["achieved_gbs_rank"] / peaks()[0]
        m.reset(prompt)  # back to the start of the cache for the per-kernel profile below
        m.step(len(prompt))

    # ---- per-kernel-class timing of the per-op kernels (event-separated steps)
    prof = m.profile(args.profile_steps)
    barrier()
    m.check_status()
    cb = class_bytes(cfg, world, pos_avg)
    total_ms = sum(prof.values())
    peak, peak_kind = peaks()
    op_kernels = {"ms_per_step": total_ms / args.profile_steps,
                  "share": {k: v / total_ms for k, v in prof.items()}} if total_ms > 0 else None
    sb = step_bytes(cfg, pos_avg)
    if args.engine == "step":
        # one persistent kernel per token: bytes per launch = this rank's step bytes
        rank_bytes = sum(cb.values())
        launch_ms = ms / args.steps
        achieved = rank_bytes / (launch_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "kernel": "step_kernel", "achieved": achieved, "peak": peak,
                    "unit": "GB/s", "frac": achieved / peak, "peak_kind": peak_kind,
                    "traffic": (NCU_STEP_TRAFFIC_BYTES_PER_LAUNCH.get((world, args.layers)) or (None,))[0],
                    "traffic_source": (NCU_STEP_TRAFFIC_BYTES_PER_LAUNCH.get((world, args.layers)) or (None, None))[1],
                    "algorithmic_bytes_per_launch": rank_bytes, "mean_launch_ms": launch_ms,
                    "time_share": 1.0}
    else:
        dom = max(prof, key=prof.get)
        launches = {"lm_head_argmax": 1}.get(dom, cfg.num_hidden_layers) * args.profile_steps
        dom_ms = prof[dom] / launches
        dom_bytes = cb[dom] / ({"lm_head_argmax": 1}.get(dom, cfg.num_hidden_layers))
        achieved = dom_bytes / (dom_ms / 1000.0) / 1e9
        roofline = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "peak_kind": peak_kind,
                    "traffic": None,
                    "algorithmic_bytes_per_launch": dom_bytes, "mean_launch_ms": dom_ms,
                    "time_share": prof[dom] / total_ms}
    step_roof = {"achieved_aggregate_gbs": sb * value / 1e9, "peak_aggregate_gbs": peak * world,
                 "frac": sb * value / 1e9 / (peak * world), "bytes_per_token": sb}

    # ---- end to end through Engine.generate (host prompt, host token reads)
    e2e = None
    if not args.no_e2e:
        n_new = min(args.steps + args.warmup, args.max_len - len(prompt) - 1)
        barrier()
        t0 = time.perf_counter()
        evs = list(eng.generate(prompt, max_new_tokens=n_new, temperature=0.0, stop_ids=()))
        wall = time.perf_counter() - t0
        if world > 1:
            t = torch.tensor([wall], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            wall = float(t.item())
        e2e = {"value": len(evs) / wall, "unit": "tok/s", "h2d_bytes_per_step": 4 * len(prompt) / len(evs),
               "d2h_bytes_per_step": 4, "ttft_ms": 1000 * evs[0]["ttft"], "tokens": len(evs),
               "path": "Engine.generate (temperature 0), wall clock call -> last token"}

    prefill = prefill_leg(eng, cfg, args, dev, world) if args.prefill_tokens > 0 else None
    blocks = block_legs(args, dev) if world == 1 and not args.no_blocks else None
    batch = batch_leg(eng, cfg, args, dev) if world == 1 and args.batch_size > 0 else None

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            v, cores = cpu_decode_sample(cfg, args.max_len, args.cpu_steps, 1)
            cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
                   "sample": f"{args.cpu_steps} full-size decode step(s) of the CPU oracle "
                             f"(reference algorithm, masked {args.max_len}-key attention) after 1 warm-up"}
        except Exception as exc:  # report, never fail the GPU measurement
            cpu = {"value": None, "unit": "tok/s", "cores": os.cpu_count(), "kind": "port",
                   "sample": f"failed: {exc!r}"[:200]}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": workload, "clocks": clocks, "e2e": e2e, "roofline": roofline,
            "step_roofline": step_roof, "op_kernels": op_kernels, "engine": args.engine,
            "cpu_baseline": cpu, "tokens_match": tokens_match, "prefill": prefill, "blocks": blocks,
            "long_context": long_ctx, "batch_decode": batch,
            "gpu_launches": args.steps * m.kernels_per_step,
            "load_s": eng.load_seconds,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
