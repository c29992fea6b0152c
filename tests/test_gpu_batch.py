"""Batched decode (g4_batch_*): several sequences of different prompt lengths decoded
together, each checked against the CPU oracle decoding that sequence alone.

Each sequence's prompt goes through the tensor-core prefill into its own cache; then every
step decodes one token of every sequence (GEMMs over the batch rows, routed MoE over the
batch's token x expert pairs, attention per sequence).  Teacher-forced with the batch's own
tokens, the oracle's logits of every decode step must correlate >= 0.9999 with the device's
and agree on the argmax wherever the oracle's top-2 margin is decided; the PARITY line
states the bf16 max-abs / max-rel error.
"""
import pytest
import torch

from gemma4_b200.config import FULL, SLIDING, make_config, tiny_parity_config
from gemma4_b200.model import Mesh
from gemma4_b200.runtime import BatchDecoder, DecodeModel
from gemma4_b200.weights import random_params, rank_shard
from oracle.reference_model import Oracle
from test_gpu_decode import decided_mask, parity_report

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _batch_case(cfg, params, prompts, steps, ctx, name):
    shard = rank_shard(cfg, params.__getitem__, Mesh(0, 1, 0), DEV)
    m = DecodeModel(cfg, shard, Mesh(0, 1, 0), ctx)
    bd = BatchDecoder(m, len(prompts), ctx)
    for s, p in enumerate(prompts):
        bd.prefill(s, p)
    firsts = bd.tokens.clone()
    toks, logits = [firsts.cpu()], []
    for _ in range(steps):
        bd.step(write_logits=True)
        logits.append(bd.logits.clone())
        toks.append(bd.tokens.clone().cpu())
    torch.cuda.synchronize()
    bd.check_status()
    toks = torch.stack(toks)          # [steps + 1, B]
    logits = torch.stack(logits).cpu()  # [steps, B, V]
    o = Oracle(cfg, params, mode="bf16")
    worst_all = 1.0
    for s, p in enumerate(prompts):
        seq = [int(t) for t in toks[:, s]]
        ref, _ = o.greedy_generate(p, steps + 1, ctx, teacher=seq)
        ref_dec = ref[len(p):]            # the decode steps' logits (after the prefill position)
        got = logits[:, s]
        worst, _, _ = parity_report(f"{name} sequence {s} (prompt {len(p)})", got, ref_dec)
        worst_all = min(worst_all, worst)
        d = decided_mask(ref_dec)
        assert bool((got.argmax(-1) == ref_dec.argmax(-1))[d].all()), (s, got.argmax(-1), ref_dec.argmax(-1))
        assert [int(t) for t in toks[1:, s]] == got.argmax(-1).tolist()
    assert worst_all >= 0.9999, worst_all
    m.close()


def test_batch_decode_tiny():
    cfg = tiny_parity_config()
    params = random_params(cfg, 0)
    g = torch.Generator().manual_seed(12)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (20, 33, 70)]
    _batch_case(cfg, params, prompts, 6, 128, "batch3 tiny")


def test_batch_decode_real_shapes():
    """26B-A4B per-layer shapes, 2 layers, 16 experts top-8, vocab 16384, batch 4."""
    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), num_experts=16, vocab_size=16384)
    params = random_params(cfg, 3)
    g = torch.Generator().manual_seed(13)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 17, 64)]
    _batch_case(cfg, params, prompts, 3, 128, "batch4 real shapes")


def test_batch_decode_graph_replay_matches_eager():
    """The CUDA-graph replay of the batched step produces the eager path's tokens and
    logits bit for bit (one eager step, then captured steps; positions advance on the
    device), and a prefill in between forces a fresh capture."""
    cfg = tiny_parity_config()
    params = random_params(cfg, 0)
    shard = rank_shard(cfg, params.__getitem__, Mesh(0, 1, 0), DEV)
    m = DecodeModel(cfg, shard, Mesh(0, 1, 0), 128)
    g = torch.Generator().manual_seed(21)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (11, 30, 45, 7)]

    def run(graph):
        bd = BatchDecoder(m, len(prompts), 128)
        for s, p in enumerate(prompts):
            bd.prefill(s, p)
        toks, lg = [], []
        for i in range(8):
            if i == 4:  # re-prefill sequence 3: the graph must be re-captured
                bd.prefill(3, prompts[3])
            bd.step(write_logits=True, graph=graph)
            toks.append(bd.tokens.clone())
            lg.append(bd.logits.clone())
        torch.cuda.synchronize()
        bd.check_status()
        return torch.stack(toks).cpu(), torch.stack(lg).cpu()

    t_eager, l_eager = run(False)
    t_graph, l_graph = run(True)
    assert torch.equal(t_eager, t_graph)
    assert torch.equal(l_eager, l_graph)
    m.close()
