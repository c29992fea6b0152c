"""Parameter layout, tensor-parallel sharding and KV-cache layout of the decode path.

The flat parameter names and canonical shapes are the reference's layout contract
(gemma4_tpu/model.py:84-117) and the shard axes follow its ``param_specs``
(model.py:120-156): sliding-layer attention is split over KV heads, full (k==v)
layers over query groups with K/V replicated, the dense MLP Megatron-style over
``intermediate_size`` and every expert over ``moe_intermediate_size``.

One deliberate difference: the reference splits the tied embedding over ``hidden``
(lookup local, lm_head = all-reduce of [V] partial logits).  Here every rank keeps the
full table (1.48 GB, only one row is read per token for the lookup) and the lm_head
reads the rank's contiguous vocab slice, so the logits need no reduction, only a
[world]-sized argmax exchange.

``pack_rank_shard`` turns canonical tensors into the per-rank tensors the C ABI
consumes (names accepted by ``g4_model_set_tensor``):
  layers.{i}.qkv           [q rows | k rows | v rows, H]  (q rows kv-major: (kv, g, d))
  layers.{i}.o_proj        [H, q rows]                     (columns of this rank's heads)
  layers.{i}.mlp.*_proj    gate/up [I/G, H], down [H, I/G]
  layers.{i}.experts.*     gate_up [E, 2, F/G, H], down [E, H, F/G]
  everything else          replicated, canonical shape
"""

from __future__ import annotations

import math
from dataclasses import dataclass

from .config import FULL, SLIDING, TextConfig


# ----------------------------------------------------------------------------- layout
def param_shapes(cfg: TextConfig) -> dict[str, tuple[int, ...]]:
    """Canonical shape of every parameter, keyed by flat name (model.py:84-117)."""
    h = cfg.hidden_size
    shapes: dict[str, tuple[int, ...]] = {"embed": (cfg.vocab_size, h), "norm": (h,)}
    for i, lt in enumerate(cfg.layer_types):
        d, kv = cfg.head_dim_for(lt), cfg.kv_heads_for(lt)
        g = cfg.num_attention_heads // kv
        p = f"layers.{i}."
        for n in ("input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
                  "post_feedforward_layernorm"):
            shapes[p + n] = (h,)
        shapes[p + "layer_scalar"] = (1,)
        shapes[p + "q_proj"] = (kv, g, d, h)
        shapes[p + "k_proj"] = (kv, d, h)
        if not cfg.k_eq_v_for(lt):
            shapes[p + "v_proj"] = (kv, d, h)
        shapes[p + "o_proj"] = (h, kv, g, d)
        shapes[p + "q_norm"] = (d,)
        shapes[p + "k_norm"] = (d,)
        shapes[p + "mlp.gate_proj"] = (cfg.intermediate_size, h)
        shapes[p + "mlp.up_proj"] = (cfg.intermediate_size, h)
        shapes[p + "mlp.down_proj"] = (h, cfg.intermediate_size)
        if cfg.enable_moe_block:
            for n in ("pre_feedforward_layernorm_2", "post_feedforward_layernorm_1",
                      "post_feedforward_layernorm_2", "router.scale"):
                shapes[p + n] = (h,)
            shapes[p + "router.proj"] = (cfg.num_experts, h)
            shapes[p + "router.per_expert_scale"] = (cfg.num_experts,)
            shapes[p + "experts.gate_up_proj"] = (cfg.num_experts, 2, cfg.moe_intermediate_size, h)
            shapes[p + "experts.down_proj"] = (cfg.num_experts, h, cfg.moe_intermediate_size)
    return shapes


def param_specs(cfg: TextConfig) -> dict[str, tuple]:
    """Shard axis per dimension ("tp" or None) for every parameter (model.py:120-156).

    ``embed`` is listed as replicated: see the module docstring.
    """
    specs: dict[str, tuple] = {}
    for name, shape in param_shapes(cfg).items():
        spec: tuple = (None,) * len(shape)
        if name.startswith("layers."):
            i = int(name.split(".")[1])
            lt = cfg.layer_types[i]
            field = name.split(".", 2)[2]
            if field in ("q_proj", "k_proj", "v_proj"):
                if lt == SLIDING:
                    spec = ("tp",) + (None,) * (len(shape) - 1)
                elif field == "q_proj":
                    spec = (None, "tp", None, None)
            elif field == "o_proj":
                spec = (None, "tp", None, None) if lt == SLIDING else (None, None, "tp", None)
            elif field in ("mlp.gate_proj", "mlp.up_proj"):
                spec = ("tp", None)
            elif field == "mlp.down_proj":
                spec = (None, "tp")
            elif field == "experts.gate_up_proj":
                spec = (None, None, "tp", None)
            elif field == "experts.down_proj":
                spec = (None, None, "tp")
        specs[name] = spec
    return specs


@dataclass(frozen=True)
class Mesh:
    """The 1-D ``tp`` mesh (model.py:159-161) as seen by one rank: one GPU per rank."""

    rank: int = 0
    world: int = 1
    device: int = 0

    @property
    def size(self) -> int:
        return self.world


def make_mesh() -> Mesh:
    """Rank/world from an initialised torch.distributed group, else the launcher's env."""
    import os

    try:
        import torch.distributed as dist

        if dist.is_available() and dist.is_initialized():
            rank, world = dist.get_rank(), dist.get_world_size()
            return Mesh(rank, world, int(os.environ.get("LOCAL_RANK", rank)))
    except ImportError:  # pragma: no cover
        pass
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    return Mesh(rank, world, int(os.environ.get("LOCAL_RANK", rank)))


def shard_slice(n: int, mesh: Mesh) -> slice:
    if n % mesh.world:
        raise ValueError(f"dimension {n} is not divisible by the mesh size {mesh.world}")
    w = n // mesh.world
    return slice(mesh.rank * w, (mesh.rank + 1) * w)


def shard_param(t, spec: tuple, mesh: Mesh):
    """Slice one canonical tensor (torch or numpy) to this rank's shard along its "tp" axis."""
    for ax, s in enumerate(spec):
        if s == "tp":
            idx = [slice(None)] * len(t.shape)
            idx[ax] = shard_slice(t.shape[ax], mesh)
            return t[tuple(idx)]
    return t


def pack_layer_attention(cfg: TextConfig, i: int, get, mesh: Mesh, presharded: bool = False):
    """(qkv [rows, H], o_proj [H, q rows]) of layer i for this rank."""
    import torch

    lt = cfg.layer_types[i]
    p = f"layers.{i}."
    specs = param_specs(cfg)
    h = cfg.hidden_size

    def take(name):
        t = get(p + name)
        return t if presharded else shard_param(t, specs[p + name], mesh)

    parts = [take("q_proj").reshape(-1, h), take("k_proj").reshape(-1, h)]
    if not cfg.k_eq_v_for(lt):
        parts.append(take("v_proj").reshape(-1, h))
    return torch.cat(parts, 0).contiguous(), take("o_proj").reshape(h, -1).contiguous()


REPLICATED_LAYER_FIELDS = (
    "input_layernorm", "post_attention_layernorm", "pre_feedforward_layernorm",
    "post_feedforward_layernorm", "pre_feedforward_layernorm_2", "post_feedforward_layernorm_1",
    "post_feedforward_layernorm_2", "layer_scalar", "q_norm", "k_norm", "router.proj",
    "router.scale", "router.per_expert_scale",
)
SHARDED_LAYER_FIELDS = ("mlp.gate_proj", "mlp.up_proj", "mlp.down_proj",
                        "experts.gate_up_proj", "experts.down_proj")


def pack_rank_shard(cfg: TextConfig, get, mesh: Mesh, layers=None, presharded: bool = False):
    """Yield (native tensor name, tensor) for this rank.  ``get(flat_name)`` returns the
    canonical tensor, or with ``presharded`` this rank's slice of it along its
    ``param_specs`` axis (a loader that reads only the rank's bytes)."""
    specs = param_specs(cfg)
    yield "embed", get("embed")
    yield "norm", get("norm")
    for i in (range(cfg.num_hidden_layers) if layers is None else layers):
        p = f"layers.{i}."
        qkv, o = pack_layer_attention(cfg, i, get, mesh, presharded)
        yield p + "qkv", qkv
        yield p + "o_proj", o
        for f in REPLICATED_LAYER_FIELDS:
            yield p + f, get(p + f)
        for f in SHARDED_LAYER_FIELDS:
            t = get(p + f)
            yield p + f, (t if presharded else shard_param(t, specs[p + f], mesh)).contiguous()


# ----------------------------------------------------------------------------- KV cache
def cache_specs(cfg: TextConfig) -> list[tuple]:
    """Per-layer cache sharding: KV heads split on sliding layers, replicated on full."""
    return [(None, None, "tp", None) if lt == SLIDING else (None, None, None, None)
            for lt in cfg.layer_types]


def cache_shapes(cfg: TextConfig, batch: int, max_len: int) -> list[tuple[int, ...]]:
    """Canonical (unsharded) per-layer cache shape [B, max_len, kv, d] (model.py:174-175)."""
    return [(batch, max_len, cfg.kv_heads_for(lt), cfg.head_dim_for(lt)) for lt in cfg.layer_types]


def local_cache_shapes(cfg: TextConfig, batch: int, max_len: int, mesh: Mesh) -> list[tuple]:
    out = []
    for shape, spec in zip(cache_shapes(cfg, batch, max_len), cache_specs(cfg)):
        kv = shape[2] // mesh.world if spec[2] == "tp" else shape[2]
        out.append((shape[0], shape[1], kv, shape[3]))
    return out


def cache_bytes(cfg: TextConfig, batch: int, max_len: int) -> int:
    """K and V bytes over all layers, unsharded bf16 (model.py:188-189)."""
    return sum(2 * 2 * math.prod(s) for s in cache_shapes(cfg, batch, max_len))


def rope_inv_freq(head_dim: int, theta: float, partial_rotary_factor: float = 1.0):
    """fp64 -> fp32 inverse frequencies with a zero-frequency NoPE tail (model.py:54-61)."""
    import numpy as np

    n_rot = int(partial_rotary_factor * head_dim // 2)
    inv = 1.0 / (theta ** (np.arange(0, 2 * n_rot, 2, dtype=np.float64) / head_dim))
    inv = np.concatenate([inv, np.zeros(head_dim // 2 - n_rot, dtype=np.float64)])
    return inv.astype(np.float32)
