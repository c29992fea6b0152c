"""Weights: HF checkpoint names -> flat names -> per-rank device shards.

Keeps the reference loader's contract (gemma4_tpu/weights.py): the checkpoint key map
(weights.py:30-58), canonical ``param_shapes`` (:61-67), ``params_from_arrays`` as the
test entry point (:70-83), ``load_params`` from a safetensors directory (:86-135) with
its FileNotFoundError / KeyError, and the accounting helpers ``param_bytes`` /
``active_params_per_token`` (:138-159).  Underneath, a rank never materialises the
model: each tensor is memory-mapped from the checkpoint, its rank slice is cut in the
canonical shape and only that slice is copied to the GPU, where ``pack_rank_shard``
lays it out for the C ABI.

``random_params`` is the seeded synthetic-weight generator used for the random
26B-A4B-shaped benchmark model: every flat name draws N(0, std) from its own
generator seeded with ``seed * 1_000_003 + crc32(name)``, so any subset of parameters
can be generated independently; ``layer_scalar`` is 1 (an HF buffer).
"""

from __future__ import annotations

import glob
import json
import math
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


def as_canonical(cfg: TextConfig, flat_name: str, t):
    """View a checkpoint array (numpy or torch) in the canonical ``param_shapes`` shape.

    HF stores the projections 2-D (``q_proj`` as [kv*g*d, H], ``o_proj`` as [H, kv*g*d],
    ``experts.gate_up_proj`` as [E, 2*F, H]); the canonical shapes split those axes in
    the same row-major order, so the conversion is a reshape (reference weights.py:61-67).
    """
    want = tuple(param_shapes(cfg)[flat_name])
    have = tuple(t.shape)
    if have == want:
        return t
    if math.prod(have) != math.prod(want):
        raise ValueError(f"{flat_name}: {math.prod(have)} elements in the checkpoint ({have}), "
                         f"the model needs {want}")
    return t.reshape(want)


def params_from_arrays(cfg: TextConfig, get: Callable, names: Iterable[str],
                       prefix: str = "model.language_model.") -> dict:
    """Canonical bf16 CPU tensors from a ``checkpoint name -> array`` accessor: the test
    entry point of the reference loader (weights.py:70-83).  Names outside the key map,
    names of parameters the config has no use for, and repeats are ignored."""
    import numpy as np
    import torch

    wanted = set(param_shapes(cfg))
    to_flat = checkpoint_key_map(cfg, prefix)
    out: dict = {}
    for name in names:
        flat = to_flat.get(name)
        if flat not in wanted or flat in out:
            continue
        arr = get(name)
        t = arr if isinstance(arr, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(arr))
        out[flat] = as_canonical(cfg, flat, t.detach().to(torch.bfloat16)).contiguous()
    return out


# ----------------------------------------------------------------------------- checkpoint
_ST_DTYPES = {"BF16": ("<u2", "bf16"), "F16": ("<f2", "f16"), "F32": ("<f4", "f32")}


class SafetensorsDir:
    """The tensors of an HF safetensors checkpoint directory, as read-only memory maps.

    The safetensors layout is an 8-byte little-endian header length, a JSON header
    mapping each tensor name to {dtype, shape, data_offsets} and the raw row-major data;
    parsing it directly lets a rank map a tensor and copy only the bytes of its own
    shard (the pages a slice touches), never the whole 47 GB model.  With
    ``model.safetensors.index.json`` only the files it names are opened; without it
    every ``*.safetensors`` file's header is read.
    """

    def __init__(self, model_dir: str):
        self.model_dir = model_dir
        files = sorted(glob.glob(os.path.join(model_dir, "*.safetensors")))
        if not files:
            raise FileNotFoundError(f"{model_dir}: no *.safetensors checkpoint files")
        index = os.path.join(model_dir, "model.safetensors.index.json")
        if os.path.exists(index):
            with open(index) as f:
                names = sorted(set(json.load(f)["weight_map"].values()))
            files = [os.path.join(model_dir, n) for n in names]
        self.entries: dict[str, tuple] = {}  # name -> (path, dtype, shape, byte offset, nbytes)
        for path in files:
            with open(path, "rb") as f:
                n = int.from_bytes(f.read(8), "little")
                header = json.loads(f.read(n))
            base = 8 + n
            for name, meta in header.items():
                if name == "__metadata__":
                    continue
                lo, hi = meta["data_offsets"]
                self.entries[name] = (path, meta["dtype"], tuple(meta["shape"]), base + lo, hi - lo)

    def __contains__(self, name: str) -> bool:
        return name in self.entries

    def array(self, name: str):
        """(numpy memmap of the tensor in its stored shape, dtype tag); bf16 is uint16."""
        import numpy as np

        path, dtype, shape, off, nbytes = self.entries[name]
        if dtype not in _ST_DTYPES:
            raise ValueError(f"{name}: unsupported checkpoint dtype {dtype}")
        npdt, tag = _ST_DTYPES[dtype]
        count = nbytes // np.dtype(npdt).itemsize
        mm = np.memmap(path, dtype=npdt, mode="r", offset=off, shape=(count,))
        return mm.reshape(shape) if shape else mm.reshape(()), tag


def _to_bf16_tensor(a, tag: str, device):
    """A slice of a checkpoint memmap as a bf16 tensor on ``device``: only the slice's
    pages are read; the result never aliases the (read-only) file mapping."""
    import numpy as np
    import torch

    a = np.ascontiguousarray(a)
    if not a.flags.writeable:  # an unsliced mapping: copy once (the host-to-device copy
        a = np.array(a)        # would otherwise read it in place, but a CPU result may not)
    if tag == "bf16":
        t = torch.from_numpy(a.view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(a).to(torch.bfloat16)
    return t.to(device)


def load_params(cfg: TextConfig, model_dir: str, mesh: Mesh | None = None, progress=None, device=None) -> dict:
    """This rank's packed parameter shard (native tensor name -> tensor on ``device``)
    from an HF safetensors checkpoint -- the reference's ``load_params`` (weights.py:86-135)
    for one rank of the ``tp`` mesh.

    Every parameter is mapped, viewed in its canonical shape, sliced along its
    ``param_specs`` axis for this rank, and only that slice is copied to the GPU, so a
    rank reads its own ~1/world of the expert and projection bytes.  Raises
    FileNotFoundError without checkpoint files and KeyError naming the parameters the
    checkpoint lacks (before anything is copied).
    """
    import torch

    from .model import param_specs, shard_param

    mesh = mesh or Mesh()
    device = device if device is not None else torch.device("cuda", mesh.device)
    ckpt = SafetensorsDir(model_dir)
    to_ckpt = {flat: name for name, flat in checkpoint_key_map(cfg).items()}
    shapes, specs = param_shapes(cfg), param_specs(cfg)
    absent = [flat for flat in shapes if to_ckpt.get(flat) not in ckpt]
    if absent:
        raise KeyError(f"{model_dir}: the checkpoint lacks {len(absent)} of the model's {len(shapes)} "
                       f"parameters, first {absent[:5]}")
    done = [0]

    def shard_of(flat: str):
        arr, tag = ckpt.array(to_ckpt[flat])
        part = shard_param(as_canonical(cfg, flat, arr), specs[flat], mesh)
        t = _to_bf16_tensor(part, tag, device)
        done[0] += 1
        if progress:
            progress(done[0], len(shapes), flat)
        return t

    return {name: t.contiguous() for name, t in pack_rank_shard(cfg, shard_of, mesh, presharded=True)}


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
