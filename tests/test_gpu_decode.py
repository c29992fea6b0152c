"""End-to-end decode parity of the CUDA step with the CPU oracle (world 1).

Teacher-forced: the oracle is fed the token sequence the GPU produced, so every
position compares logits of identical inputs.  Pass bar (north star): logits corr
>= 0.9999 at every position and identical argmax wherever the oracle's top-2 margin
exceeds 2 bf16 ulps of the top logit (with the std-0.02 random weights the bf16
logits are small and exact ties are common; tied positions are reported, not failed).
"""

import numpy as np
import pytest
import torch

from gemma4_b200.config import FULL, SLIDING, make_config, tiny_parity_config
from gemma4_b200.engine import Engine
from gemma4_b200.model import Mesh
from gemma4_b200.runtime import DecodeModel
from gemma4_b200.weights import random_params, rank_shard
from oracle.reference_model import Oracle
from gpu_util import corr

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _run_gpu(cfg, params, prompt, n_new, max_len, use_graph=True, engine="step"):
    shard = rank_shard(cfg, params.__getitem__, Mesh(0, 1, 0), DEV)
    m = DecodeModel(cfg, shard, Mesh(0, 1, 0), max_len, engine=engine)
    m.reset(prompt, write_logits=True)
    logits = []
    for _ in range(len(prompt) + n_new - 1):
        m.step(1, use_graph=use_graph)
        logits.append(m.logits.clone())
    torch.cuda.synchronize()
    m.check_status()
    ids = m.tokens_out[len(prompt):len(prompt) + n_new].cpu().tolist()
    host = [int(v) for v in m.tokens_host[len(prompt):len(prompt) + n_new]]
    m.close()
    return torch.stack(logits).cpu(), ids, host


def _compare(cfg, params, prompt, n_new, max_len, use_graph=True, engine="step"):
    lg, ids, host = _run_gpu(cfg, params, prompt, n_new, max_len, use_graph, engine)
    assert ids == host, "mapped host token mirror disagrees with the device ring"
    o = Oracle(cfg, params, mode="bf16")
    ref, ref_ids = o.greedy_generate(prompt, n_new, max_len, teacher=ids)
    assert lg.shape == ref.shape
    worst = min(corr(lg[i], ref[i]) for i in range(len(ref)))
    top2 = torch.topk(ref, 2, dim=-1).values
    margin = top2[:, 0] - top2[:, 1]
    ulp = top2[:, 0].abs().clamp_min(1e-30) * 2.0 ** -7
    decided = margin > 2 * ulp
    agree = lg.argmax(-1) == ref.argmax(-1)
    return worst, agree, decided, ids, ref_ids


@pytest.mark.parametrize("engine", ["step", "ops"])
def test_tiny_config1_teacher_forced_and_greedy(engine):
    """benchmark config 1: 128-token prompt, 32 greedy tokens."""
    from golden.make_golden import CONFIG1_NEW, config1_inputs

    cfg, params, prompt = config1_inputs()
    worst, agree, decided, ids, _ = _compare(cfg, params, prompt, CONFIG1_NEW, 160, engine=engine)
    assert worst >= 0.9999, worst
    assert bool(agree[decided].all()), (agree.logical_not() & decided).nonzero()
    golden = np.load("tests/golden/oracle_config1.npz")
    same = (np.array(ids) == golden["ids"]).mean()
    print(f"config1 [{engine}]: worst corr {worst:.6f}, decided {int(decided.sum())}/{len(decided)}, "
          f"free-running ids equal to golden: {same:.3f}")


@pytest.mark.parametrize("engine", ["step", "ops"])
def test_graph_and_direct_launch_agree(engine):
    cfg = tiny_parity_config()
    params = random_params(cfg, 7)
    prompt = list(range(5, 25))
    a = _run_gpu(cfg, params, prompt, 6, 64, use_graph=True, engine=engine)
    b = _run_gpu(cfg, params, prompt, 6, 64, use_graph=False, engine=engine)
    assert torch.equal(a[0], b[0]) and a[1] == b[1]


def test_step_kernel_matches_op_kernels_bitwise():
    """The persistent step kernel and the per-op kernels share every operator, tile
    loop and attention item: identical logits and tokens, real layer shapes."""
    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), num_experts=16,
                      vocab_size=16384)
    params = random_params(cfg, 5)
    prompt = list(range(100, 109))
    a = _run_gpu(cfg, params, prompt, 5, 64, engine="step")
    b = _run_gpu(cfg, params, prompt, 5, 64, engine="ops")
    assert torch.equal(a[0], b[0]) and a[1] == b[1]


def test_status_bit_stops_steps_until_cleared():
    """A set timeout bit (planted by the host, as if a bounded wait had given up)
    turns later steps of the step kernel into no-ops; check_status reports it and
    reset() resumes with correct results."""
    cfg = tiny_parity_config()
    params = random_params(cfg, 11)
    prompt = list(range(3, 12))
    ref_logits, ref_ids, _ = _run_gpu(cfg, params, prompt, 4, 32)
    shard = rank_shard(cfg, params.__getitem__, Mesh(0, 1, 0), DEV)
    m = DecodeModel(cfg, shard, Mesh(0, 1, 0), 32)
    m.reset(prompt, write_logits=True)
    m.step(2)
    torch.cuda.synchronize()
    pos = int(m.ctrl[0])
    m.ctrl[3] = 0x2  # MBAR_TIMEOUT
    m.step(3)
    torch.cuda.synchronize()
    assert int(m.ctrl[0]) == pos, "a step ran with the status bit set"
    with pytest.raises(RuntimeError):
        m.check_status()
    m.reset(prompt, write_logits=True)
    got = []
    for _ in range(len(prompt) + 3):
        m.step(1)
        got.append(m.logits.clone())
    torch.cuda.synchronize()
    m.check_status()
    ids = m.tokens_out[len(prompt):len(prompt) + 4].cpu().tolist()
    m.close()
    assert ids == ref_ids and torch.equal(torch.stack(got).cpu(), ref_logits)


def test_real_layer_shapes_two_layers():
    """26B-A4B per-layer shapes (H 2816, 16 q heads, d 256, window 1024, F 704, I 2112)
    with 2 layers [sliding, full], 16 experts top-8 and a 16K vocab."""
    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), num_experts=16,
                      vocab_size=16384)
    params = random_params(cfg, 3)
    prompt = [int(t) for t in torch.randint(0, cfg.vocab_size, (6,), generator=torch.Generator().manual_seed(3))]
    worst, agree, decided, _, _ = _compare(cfg, params, prompt, 4, 64)
    assert worst >= 0.9999, worst
    assert bool(agree[decided].all())


def test_engine_generate_protocol():
    cfg = tiny_parity_config()
    params = random_params(cfg, 0)
    eng = Engine(None, max_len=96, cfg=cfg, params=params, mesh=Mesh(0, 1, 0))
    ct = eng.compile_all()
    assert set(ct) == {"prefill_compile_s", "decode_compile_s", "decode_step_s"}
    prompt = list(range(1, 30))
    ev = list(eng.generate(prompt, max_new_tokens=12, temperature=0.0, stop_ids=()))
    assert ev[0]["kind"] == "prefill" and ev[0]["prompt_tokens"] == 29 and ev[0]["ttft"] > 0
    assert [e["kind"] for e in ev[1:]] == ["decode"] * 11
    assert [e["index"] for e in ev[1:]] == list(range(1, 12))
    toks = [e["token"] for e in ev]
    again = [e["token"] for e in eng.generate(prompt, max_new_tokens=12, temperature=0.0, stop_ids=())]
    assert toks == again
    # a stop id ends the stream at its first occurrence
    stop = toks[3]
    cut = [e["token"] for e in eng.generate(prompt, 12, temperature=0.0, stop_ids=(stop,))]
    assert cut == toks[: toks.index(stop) + 1]
    with pytest.raises(ValueError):
        list(eng.generate(list(range(96)), 4, temperature=0.0))
    o = Oracle(cfg, params, mode="bf16")
    ref, _ = o.greedy_generate(prompt, 12, 96, teacher=toks)
    assert corr(ref[-1], ref[-1]) == 1.0
