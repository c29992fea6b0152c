"""Decode parity at the full 26B-A4B shapes: 128 experts top-8, vocab 262144, window 1024,
positions past the window.

Six layers (five sliding, one full k==v layer: the model's own 5:1 interleave) keep the
oracle's host memory at ~11 GB of bf16 parameters; every per-layer shape, the router's
top-8 over 128 experts and the 262,144-row LM head with its argmax are those of the full
model.  The KV caches (max_len 2048) are pre-filled with the same seeded N(0,1) rows on
both sides, and decoding starts at position 1500, so sliding layers attend to a full
1,024-key window that starts past position 0 and the full layer to 1,501+ keys.  Three
teacher-forced steps; the pass bar is the one of the other decode tests (corr >= 0.9999
per position, identical argmax where decided), and the PARITY line states the bf16
max-abs / max-rel error.  Parameters are drawn on the GPU (seeded CUDA generator) and
copied to the host for the oracle.
"""

import pytest
import torch

from gemma4_b200.config import make_config
from gemma4_b200.model import Mesh
from gemma4_b200.runtime import DecodeModel
from gemma4_b200.weights import random_params, rank_shard
from oracle.reference_model import Oracle
from test_gpu_decode import decided_mask, parity_report

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def test_config4_shapes_past_the_window():
    cfg = make_config(num_hidden_layers=6)  # 26B-A4B shapes, layers [S, S, S, S, S, F]
    assert cfg.layer_types.count("full_attention") == 1
    max_len, pos0, steps, tok0 = 2048, 1500, 3, 12345
    params_dev = random_params(cfg, 3, device=DEV)
    shard = rank_shard(cfg, params_dev.__getitem__, Mesh(0, 1, 0), DEV)
    params = {k: v.cpu() for k, v in params_dev.items()}
    del params_dev
    g = torch.Generator().manual_seed(33)
    caches = {"k": [], "v": []}
    for lt in cfg.layer_types:
        shape = (1, max_len, cfg.kv_heads_for(lt), cfg.head_dim_for(lt))
        caches["k"].append(torch.randn(shape, generator=g).to(torch.bfloat16))
        caches["v"].append(torch.randn(shape, generator=g).to(torch.bfloat16))

    m = DecodeModel(cfg, shard, Mesh(0, 1, 0), max_len)
    for i in range(cfg.num_hidden_layers):
        m.cache_k[i].copy_(caches["k"][i])
        m.cache_v[i].copy_(caches["v"][i])
    m.reset([tok0] * (pos0 + 1), write_logits=True)
    m.ctrl[0] = pos0  # start decoding at pos0 (the token there is forced: tok0)
    got = []
    for _ in range(steps):
        m.step(1)
        got.append(m.logits.clone())
    torch.cuda.synchronize()
    m.check_status()
    ids = m.tokens_out[pos0 + 1:pos0 + 1 + steps].cpu().tolist()
    m.close()
    got = torch.stack(got).cpu()

    o = Oracle(cfg, params, mode="bf16")
    ref = []
    cache = {"k": [t.clone() for t in caches["k"]], "v": [t.clone() for t in caches["v"]]}
    for j in range(steps):
        tok = tok0 if j == 0 else ids[j - 1]
        lg, cache = o.decode(cache, tok, pos0 + j, max_len)
        ref.append(lg)
    ref = torch.stack(ref)
    worst, _, _ = parity_report("config4_shapes_6_layers_pos1500", got, ref)
    assert worst >= 0.9999, worst
    decided = decided_mask(ref)
    agree = got.argmax(-1) == ref.argmax(-1)
    assert bool(agree[decided].all()), (got.argmax(-1), ref.argmax(-1), decided)
    assert ids == got.argmax(-1).tolist()  # the step's own argmax is what it wrote
