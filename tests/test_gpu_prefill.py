"""Tensor-core prefill (g4_prefill) against the oracle's prefill (model.py:333-386 with
dense_moe=True, the reference's prefill step engine.py:57-69).

For each model: the prompt goes through g4_prefill (in one chunk, and in several chunks
that attend to the earlier chunks' cache rows); checked against Oracle.prefill on the same
tokens: the last position's logits (corr >= 0.9999, identical argmax where the oracle's
top-2 margin is decided, the PARITY line states bf16 max-abs / max-rel), every layer's K/V
cache rows (corr >= 0.9999), the written first token, and then teacher-forced decode
steps continuing from the prefilled caches on both sides.
"""

import pytest
import torch

from gemma4_b200.config import FULL, SLIDING, make_config, tiny_parity_config
from gemma4_b200.engine import Engine
from gemma4_b200.model import Mesh
from gemma4_b200.runtime import DecodeModel
from gemma4_b200.weights import random_params, rank_shard
from oracle.reference_model import Oracle
from gpu_util import corr
from test_gpu_decode import decided_mask, parity_report

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _prefill_case(cfg, params, prompt, max_len, chunk, n_dec, name, dense=False):
    shard = rank_shard(cfg, params.__getitem__, Mesh(0, 1, 0), DEV)
    m = DecodeModel(cfg, shard, Mesh(0, 1, 0), max_len)
    p = len(prompt)
    m.reset(prompt, write_logits=True)
    assert m.prefill(p, chunk, dense_moe=dense)
    name = f"{name} {'dense' if dense else 'routed'} MoE"
    torch.cuda.synchronize()
    m.check_status()
    assert int(m.ctrl[0]) == p
    first = int(m.tokens_out[p])
    lg_pre = m.logits.clone().cpu()
    caches = ([t[0, :p].cpu() for t in m.cache_k], [t[0, :p].cpu() for t in m.cache_v])
    dec = []
    for _ in range(n_dec):
        m.step(1)
        dec.append(m.logits.clone())
    torch.cuda.synchronize()
    m.check_status()
    ids = m.tokens_out[p:p + n_dec + 1].cpu().tolist()
    m.close()

    o = Oracle(cfg, params, mode="bf16")
    cache = o.new_cache(1, max_len)
    ref_all, cache = o.prefill(cache, prompt, p, dense_moe=True)
    ref = ref_all[p - 1]
    assert first == int(lg_pre.argmax()), "written token is not the argmax of the written logits"
    worst, _, _ = parity_report(f"{name} prefill last position", lg_pre[None], ref[None])
    assert worst >= 0.9999, worst
    if bool(decided_mask(ref[None])[0]):
        assert first == int(ref.argmax()), (first, int(ref.argmax()))
    for i in range(cfg.num_hidden_layers):
        for got, want in ((caches[0][i], cache["k"][i][0, :p]), (caches[1][i], cache["v"][i][0, :p])):
            c = corr(got, want)
            assert c >= 0.9999, (i, c)
    refs = []
    for j in range(n_dec):  # teacher-forced decode from the prefilled caches
        lg, cache = o.decode(cache, ids[j], p + j, max_len)
        refs.append(lg)
    if n_dec:
        got = torch.stack(dec).cpu()
        refs = torch.stack(refs)
        worst, _, _ = parity_report(f"{name} decode after prefill", got, refs)
        assert worst >= 0.9999, worst
        d = decided_mask(refs)
        assert bool((got.argmax(-1) == refs.argmax(-1))[d].all())


@pytest.mark.parametrize("dense", [False, True])
@pytest.mark.parametrize("chunk", [0, 128])
def test_prefill_tiny_config1(chunk, dense):
    """config 1: 128-token prompt (one chunk) and a 300-token prompt in 128-token chunks
    (sliding window 64: later chunks attend across the chunk boundary); routed and dense
    (all-expert) MoE."""
    cfg = tiny_parity_config()
    params = random_params(cfg, 0)
    n = 128 if chunk == 0 else 300
    prompt = torch.randint(0, cfg.vocab_size, (n,), generator=torch.Generator().manual_seed(9)).tolist()
    _prefill_case(cfg, params, prompt, 512, chunk, 4, f"config1 T={n} chunk={chunk or 'all'}", dense)


@pytest.mark.parametrize("dense", [False, True])
def test_prefill_real_layer_shapes(dense):
    """26B-A4B per-layer shapes, 2 layers [sliding, full], 16 experts top-8, vocab 16384,
    256-token prompt, routed and dense (all-expert) MoE."""
    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), num_experts=16, vocab_size=16384)
    params = random_params(cfg, 3)
    prompt = torch.randint(0, cfg.vocab_size, (256,), generator=torch.Generator().manual_seed(4)).tolist()
    _prefill_case(cfg, params, prompt, 1536, 0, 2, "real_shapes_2_layers T=256", dense)


def test_prefill_128_experts_short_prompt():
    """128 experts top-8 (the full model's router and expert count), 40-token prompt:
    short prompts use the split-K path of the narrow projections."""
    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), vocab_size=32768)
    params = random_params(cfg, 6)
    prompt = torch.randint(0, cfg.vocab_size, (40,), generator=torch.Generator().manual_seed(6)).tolist()
    _prefill_case(cfg, params, prompt, 256, 0, 2, "128_experts T=40")


def test_prefill_real_shapes_long_chunks_and_d512():
    """Full-layer head_dim 512 (the real checkpoint's), 1300 tokens in 512-token chunks:
    the sliding layer's 1024-key window crosses chunk boundaries.  8 query heads (4 KV
    heads sliding, 2 full) keep the full layer's o_proj rows at 4096 elements, the decode
    engine's limit at world 1."""
    cfg = make_config(num_hidden_layers=2, layer_types=(SLIDING, FULL), num_experts=8, top_k_experts=4,
                      vocab_size=8192, global_head_dim=512, num_attention_heads=8, num_key_value_heads=4)
    params = random_params(cfg, 5)
    prompt = torch.randint(0, cfg.vocab_size, (1300,), generator=torch.Generator().manual_seed(5)).tolist()
    _prefill_case(cfg, params, prompt, 2048, 512, 1, "d512 T=1300 chunk=512")


def test_engine_generate_uses_prefill():
    cfg = tiny_parity_config()
    params = random_params(cfg, 0)
    eng = Engine(None, max_len=256, cfg=cfg, params=params, mesh=Mesh(0, 1, 0))
    ref_eng = Engine(None, max_len=256, cfg=cfg, params=params, mesh=Mesh(0, 1, 0), prefill=False)
    prompt = list(range(1, 100))
    a = [e for e in eng.generate(prompt, max_new_tokens=8, temperature=0.0, stop_ids=())]
    b = [e["token"] for e in ref_eng.generate(prompt, max_new_tokens=8, temperature=0.0, stop_ids=())]
    assert a[0]["kind"] == "prefill" and a[0]["prompt_tokens"] == 99
    toks = [e["token"] for e in a]
    # prefill (dense MoE, one pass) and token-by-token decode agree wherever the oracle decides
    o = Oracle(cfg, params, mode="bf16")
    ref, ref_ids = o.greedy_generate(prompt, 8, 256, teacher=toks)
    dec = decided_mask(ref[len(prompt) - 1:]).tolist()
    assert all(x == y for x, y, d in zip(toks, ref_ids, dec) if d), (toks, ref_ids)
    upto = dec.index(False) if False in dec else len(dec)  # same history up to a tie
    assert toks[:upto] == b[:upto], (toks, b)
