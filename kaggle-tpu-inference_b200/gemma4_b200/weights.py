"""Weights: HF checkpoint names -> flat names -> per-rank device shards.

Mirrors the reference loader's contract (gemma4_tpu/weights.py): the same checkpoint
key map (weights.py:30-58), reshape to the canonical ``param_shapes`` (:61-67),
``params_from_arrays`` as the test entry point (:70-83), streaming ``load_params``
from safetensors with the index file (:86-135) and the accounting helpers
``param_bytes`` / ``active_params_per_token`` (:138-159).  Instead of
``jax.device_put(NamedSharding)`` each rank packs its own shard into the tensors the
C ABI consumes (``model.pack_rank_shard``) directly on its GPU.

``random_params`` is the seeded synthetic-weight generator used for the random
26B-A4B-shaped benchmark model: every flat name draws N(0, std) from its own
generator seeded with ``seed * 1_000_003 + crc32(name)``, so any subset of parameters
can be generated independently; ``layer_scalar`` is 1 (an HF buffer).
"""

from __future__ import annotations

import glob
import json
import os
import zlib
from typing import Callable, Iterable

from .config import TextConfig
from .model import Mesh, pack_rank_shard, param_shapes


def checkpoint_key_map(cfg: TextConfig, prefix: str = "model.language_model.") -> dict[str, str]:
    """Checkpoint tensor name -> flat parameter name (reference weights.py:30-58)."""
    out = {prefix + "embed_tokens.weight": "embed", prefix + "norm.weight": "norm"}
    norms = ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
             "post_feedforward_layernorm", "pre_feedforward_layernorm_2",
             "post_feedforward_layernorm_1", "post_feedforward_layernorm_2")
    for i in range(cfg.num_hidden_layers):
        src, dst = f"{prefix}layers.{i}.", f"layers.{i}."
        out.update({f"{src}{n}.weight": dst + n for n in norms})
        out[src + "layer_scalar"] = dst + "layer_scalar"
        out.update({f"{src}self_attn.{n}.weight": dst + n
                    for n in ("q_proj", "k_proj", "v_proj", "o_proj", "q_norm", "k_norm")})
        out.update({f"{src}mlp.{n}.weight": f"{dst}mlp.{n}" for n in ("gate_proj", "up_proj", "down_proj")})
        out[src + "router.proj.weight"] = dst + "router.proj"
        for n in ("router.scale", "router.per_expert_scale", "experts.gate_up_proj", "experts.down_proj"):
            out[src + n] = dst + n
    return out


def reshape_param(cfg: TextConfig, flat_name: str, t):
    """Reshape a checkpoint tensor to its canonical shape (reference weights.py:61-67)."""
    target = param_shapes(cfg)[flat_name]
    if tuple(t.shape) == target:
        return t
    n = 1
    for s in target:
        n *= s
    if t.numel() != n:
        raise ValueError(f"{flat_name}: checkpoint shape {tuple(t.shape)} != expected {target}")
    return t.reshape(target)


def params_from_arrays(cfg: TextConfig, get: Callable, names: Iterable[str],
                       prefix: str = "model.language_model.") -> dict:
    """Canonical torch tensors (bf16, CPU) from any ``name -> array`` accessor.

    Same selection rules as the reference (weights.py:70-83): unknown names and
    duplicates are skipped.  Arrays may be numpy arrays or torch tensors.
    """
    import numpy as np
    import torch

    shapes = param_shapes(cfg)
    key_map = checkpoint_key_map(cfg, prefix)
    out: dict = {}
    for ck in names:
        flat = key_map.get(ck)
        if flat is None or flat not in shapes or flat in out:
            continue
        a = get(ck)
        t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))
        out[flat] = reshape_param(cfg, flat, t.detach().to(torch.bfloat16).contiguous())
    return out


def load_params(cfg: TextConfig, model_dir: str, progress=None) -> dict:
    """Stream an HF safetensors checkpoint into canonical CPU bf16 tensors.

    Raises ``FileNotFoundError`` without safetensors and ``KeyError`` listing missing
    parameters, like the reference (weights.py:97-98, 132-134).
    """
    from safetensors import safe_open

    shapes = param_shapes(cfg)
    key_map = checkpoint_key_map(cfg)
    files = sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))
    if not files:
        raise FileNotFoundError(f"no safetensors under {model_dir}")
    index_path = os.path.join(model_dir, "model.safetensors.index.json")
    if os.path.exists(index_path):
        with open(index_path) as f:
            weight_map = json.load(f)["weight_map"]
        by_file: dict[str, list[str]] = {}
        for ck in key_map:
            if ck in weight_map:
                by_file.setdefault(os.path.join(model_dir, weight_map[ck]), []).append(ck)
    else:
        by_file = {f: list(key_map) for f in files}
    params: dict = {}
    done, total = 0, len(shapes)
    for path, keys in by_file.items():
        with safe_open(path, framework="pt", device="cpu") as f:
            have = set(f.keys())
            for ck in keys:
                flat = key_map[ck]
                if ck not in have or flat not in shapes:
                    continue
                import torch

                params[flat] = reshape_param(cfg, flat, f.get_tensor(ck).to(torch.bfloat16))
                done += 1
                if progress:
                    progress(done, total, flat)
    missing = sorted(set(shapes) - set(params))
    if missing:
        raise KeyError(f"missing {len(missing)} params, e.g. {missing[:5]}")
    return params


def param_bytes(cfg: TextConfig) -> int:
    """bf16 bytes of all parameters (reference weights.py:138-139)."""
    total = 0
    for s in param_shapes(cfg).values():
        n = 1
        for d in s:
            n *= d
        total += 2 * n
    return total


def active_params_per_token(cfg: TextConfig) -> int:
    """Parameters touched per decoded token (reference weights.py:142-159)."""
    h = cfg.hidden_size
    total = 0
    for lt in cfg.layer_types:
        d, kv = cfg.head_dim_for(lt), cfg.kv_heads_for(lt)
        total += 2 * cfg.num_attention_heads * d * h          # q and o
        total += kv * d * h * (1 if cfg.k_eq_v_for(lt) else 2)  # k (and v)
        total += 3 * cfg.intermediate_size * h
        if cfg.enable_moe_block:
            total += cfg.num_experts * h + cfg.top_k_experts * 3 * cfg.moe_intermediate_size * h
    return total + cfg.vocab_size * h


# ----------------------------------------------------------------------------- synthetic
def param_seed(seed: int, name: str) -> int:
    return (seed * 1_000_003 + zlib.crc32(name.encode())) % (2 ** 63)


def random_param(cfg: TextConfig, name: str, seed: int, std: float = 0.02, device="cpu",
                 dtype=None):
    """One canonical parameter drawn N(0, std) from its own seeded generator."""
    import torch

    dtype = dtype or torch.bfloat16
    shape = param_shapes(cfg)[name]
    if name.endswith("layer_scalar"):
        return torch.ones(shape, dtype=dtype, device=device)
    g = torch.Generator(device=device).manual_seed(param_seed(seed, name))
    t = torch.empty(shape, dtype=torch.float32, device=device)
    t.normal_(0.0, std, generator=g)
    return t.to(dtype)


def random_params(cfg: TextConfig, seed: int, std: float = 0.02, device="cpu", dtype=None) -> dict:
    """All canonical parameters of a random model (see :func:`random_param`)."""
    return {n: random_param(cfg, n, seed, std, device, dtype) for n in sorted(param_shapes(cfg))}


def rank_shard(cfg: TextConfig, get: Callable, mesh: Mesh, device) -> dict:
    """This rank's packed tensors on ``device`` from a canonical-tensor accessor."""
    out = {}
    for name, t in pack_rank_shard(cfg, get, mesh):
        out[name] = t.to(device=device, dtype=t.dtype).contiguous()
    return out


def random_rank_shard(cfg: TextConfig, seed: int, mesh: Mesh, device, std: float = 0.02) -> dict:
    """Generate a random model's shard for this rank directly on its GPU.

    Each canonical parameter is drawn on the device with the CUDA generator (values
    differ from the CPU generator's, reproducibly) and sliced before the next one is
    drawn, so peak extra memory is one canonical parameter.
    """
    cache: dict = {}

    def get(name):
        if name not in cache:
            cache.clear()
            cache[name] = random_param(cfg, name, seed, std, device=device)
        return cache[name]

    out = {}
    for name, t in pack_rank_shard(cfg, get, mesh):
        out[name] = t.contiguous()
    cache.clear()
    return out
