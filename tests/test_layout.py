"""Layout contract, sharding and accounting of the host side (no GPU)."""

import pytest
import torch

from gemma4_b200.config import FULL, SLIDING, gemma4_26b_a4b, tiny_parity_config
from gemma4_b200.model import (Mesh, cache_bytes, local_cache_shapes, pack_rank_shard,
                               param_shapes, param_specs)
from gemma4_b200.weights import (active_params_per_token, checkpoint_key_map, param_bytes,
                                 random_param, random_params)


def test_bench_model_accounting_matches_baseline():
    # 2 x active_params_per_token = 7.399 GB (global d 256) / 7.644 GB (d 512)
    assert abs(2 * active_params_per_token(gemma4_26b_a4b(256)) / 1e9 - 7.399) < 0.001
    assert abs(2 * active_params_per_token(gemma4_26b_a4b(512)) / 1e9 - 7.644) < 0.001
    # reference README.md:113: 47.0 GiB of bf16 weights for the real shape
    assert abs(param_bytes(gemma4_26b_a4b(512)) / 2 ** 30 - 47.00) < 0.01


def test_layer_pattern_is_five_sliding_one_full():
    cfg = gemma4_26b_a4b()
    assert cfg.layer_types.count(SLIDING) == 25 and cfg.layer_types.count(FULL) == 5
    assert all(cfg.layer_types[i] == FULL for i in (5, 11, 17, 23, 29))


def test_checkpoint_key_map_covers_every_param():
    cfg = tiny_parity_config()
    flat = set(checkpoint_key_map(cfg).values())
    assert set(param_shapes(cfg)) <= flat


def test_specs_match_reference_axes():
    cfg = gemma4_26b_a4b()
    s = param_specs(cfg)
    assert s["layers.0.q_proj"] == ("tp", None, None, None)       # sliding: KV heads
    assert s["layers.5.q_proj"] == (None, "tp", None, None)       # full: query groups
    assert s["layers.5.k_proj"] == (None, None, None)             # full: replicated
    assert s["layers.0.o_proj"] == (None, "tp", None, None)
    assert s["layers.5.o_proj"] == (None, None, "tp", None)
    assert s["layers.3.experts.gate_up_proj"] == (None, None, "tp", None)
    assert s["layers.3.experts.down_proj"] == (None, None, "tp")
    assert s["layers.3.mlp.down_proj"] == (None, "tp")
    assert s["embed"] == (None, None)                              # replicated (see model.py)


@pytest.mark.parametrize("world", [1, 2])
def test_pack_rank_shard_shapes(world):
    cfg = tiny_parity_config()
    params = random_params(cfg, 0)
    H, I, F, E = cfg.hidden_size, cfg.intermediate_size, cfg.moe_intermediate_size, cfg.num_experts
    for rank in range(world):
        sh = dict(pack_rank_shard(cfg, params.__getitem__, Mesh(rank, world)))
        for i, lt in enumerate(cfg.layer_types):
            d, kv = cfg.head_dim_for(lt), cfg.kv_heads_for(lt)
            g = cfg.num_attention_heads // kv
            if lt == SLIDING:
                q_rows, kv_rows = kv // world * g * d, kv // world * d
            else:
                q_rows, kv_rows = kv * (g // world) * d, kv * d
            v_rows = 0 if cfg.k_eq_v_for(lt) else kv_rows
            assert sh[f"layers.{i}.qkv"].shape == (q_rows + kv_rows + v_rows, H)
            assert sh[f"layers.{i}.o_proj"].shape == (H, q_rows)
            assert sh[f"layers.{i}.mlp.gate_proj"].shape == (I // world, H)
            assert sh[f"layers.{i}.mlp.down_proj"].shape == (H, I // world)
            assert sh[f"layers.{i}.experts.gate_up_proj"].shape == (E, 2, F // world, H)
            assert sh[f"layers.{i}.experts.down_proj"].shape == (E, H, F // world)
            assert all(t.is_contiguous() for t in sh.values())


def test_cache_layout():
    cfg = gemma4_26b_a4b()
    sh1 = local_cache_shapes(cfg, 1, 32768, Mesh(0, 1))
    sh8 = local_cache_shapes(cfg, 1, 32768, Mesh(0, 8))
    assert sh1[0] == (1, 32768, 8, 256) and sh8[0] == (1, 32768, 1, 256)
    assert sh1[5] == sh8[5] == (1, 32768, 2, 256)   # full layers replicated
    assert cache_bytes(cfg, 1, 32768) == 25 * 2 * 2 * 32768 * 8 * 256 + 5 * 2 * 2 * 32768 * 2 * 256


def test_random_param_is_seeded_per_name():
    cfg = tiny_parity_config()
    a = random_param(cfg, "layers.1.q_proj", 3)
    b = random_param(cfg, "layers.1.q_proj", 3)
    c = random_param(cfg, "layers.1.k_proj", 3)
    assert torch.equal(a, b) and a.dtype == torch.bfloat16
    assert not torch.equal(a.flatten()[:64], c.flatten()[:64])
    assert (random_param(cfg, "layers.0.layer_scalar", 3) == 1).all()
    assert abs(float(a.float().std()) - 0.02) < 0.002
