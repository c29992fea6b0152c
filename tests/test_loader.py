"""The safetensors loader (weights.load_params) on a tiny checkpoint written here, on the CPU.

The checkpoint uses the HF tensor names and stored shapes (2-D q/k/v/o projections,
experts.gate_up_proj as [E, 2F, H]) of the tiny parity model, split over two files with
``model.safetensors.index.json`` and, separately, as one file without an index.  For world
1 and 2 every rank's loaded shard must equal pack_rank_shard of the same canonical tensors
(bit for bit); an fp32 checkpoint converts to the same bf16 values; a missing tensor raises
KeyError (before any copy) and a directory without checkpoint files FileNotFoundError
(reference weights.py:97-98, 132-134).
"""
import json
import os

import pytest
import torch
from safetensors.torch import save_file

from gemma4_b200.config import tiny_parity_config
from gemma4_b200.model import Mesh, pack_rank_shard, param_shapes
from gemma4_b200.weights import checkpoint_key_map, load_params, random_params


def _hf_shape(flat: str, shape: tuple) -> tuple:
    """The 2-D / 3-D layout HF checkpoints store each canonical parameter in."""
    field = flat.split(".", 2)[-1] if flat.startswith("layers.") else flat
    if field in ("q_proj", "k_proj", "v_proj"):
        return (int(torch.tensor(shape[:-1]).prod()), shape[-1])
    if field == "o_proj":
        return (shape[0], int(torch.tensor(shape[1:]).prod()))
    if field == "experts.gate_up_proj":
        return (shape[0], shape[1] * shape[2], shape[3])
    return shape


def _write_checkpoint(path, cfg, params, split: bool, dtype=torch.bfloat16, drop=()):
    os.makedirs(path, exist_ok=True)
    to_ckpt = {flat: name for name, flat in checkpoint_key_map(cfg).items()}
    tensors = {}
    for flat, t in params.items():
        if flat in drop:
            continue
        tensors[to_ckpt[flat]] = t.reshape(_hf_shape(flat, tuple(t.shape))).to(dtype).contiguous()
    names = sorted(tensors)
    if not split:
        save_file(tensors, os.path.join(path, "model.safetensors"))
        return
    half = len(names) // 2
    parts = {"model-00001-of-00002.safetensors": names[:half], "model-00002-of-00002.safetensors": names[half:]}
    weight_map = {}
    for fname, keys in parts.items():
        save_file({k: tensors[k] for k in keys}, os.path.join(path, fname))
        weight_map.update({k: fname for k in keys})
    with open(os.path.join(path, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": weight_map}, f)


@pytest.fixture(scope="module")
def model():
    cfg = tiny_parity_config()
    return cfg, random_params(cfg, seed=21)


@pytest.mark.parametrize("split", [True, False])
@pytest.mark.parametrize("world", [1, 2])
def test_rank_shards_equal_packed_canonical(tmp_path, model, split, world):
    cfg, params = model
    _write_checkpoint(tmp_path, cfg, params, split)
    for rank in range(world):
        mesh = Mesh(rank, world, 0)
        got = load_params(cfg, str(tmp_path), mesh, device="cpu")
        want = dict(pack_rank_shard(cfg, params.__getitem__, mesh))
        assert set(got) == set(want)
        for name, t in want.items():
            assert got[name].dtype == torch.bfloat16 and got[name].shape == t.shape, name
            assert torch.equal(got[name], t.contiguous()), name


def test_fp32_checkpoint_converts_to_bf16(tmp_path, model):
    cfg, params = model
    _write_checkpoint(tmp_path, cfg, params, False, dtype=torch.float32)
    got = load_params(cfg, str(tmp_path), Mesh(0, 1, 0), device="cpu")
    want = dict(pack_rank_shard(cfg, params.__getitem__, Mesh(0, 1, 0)))
    assert all(torch.equal(got[n], want[n]) for n in want)


def test_progress_counts_every_parameter(tmp_path, model):
    cfg, params = model
    _write_checkpoint(tmp_path, cfg, params, True)
    seen = []
    load_params(cfg, str(tmp_path), Mesh(0, 1, 0), progress=lambda i, n, name: seen.append((i, n, name)),
                device="cpu")
    assert len(seen) == len(param_shapes(cfg)) and seen[-1][0] == seen[-1][1]


def test_missing_tensor_raises_key_error(tmp_path, model):
    cfg, params = model
    _write_checkpoint(tmp_path, cfg, params, True, drop=("layers.2.experts.down_proj",))
    with pytest.raises(KeyError, match="layers.2.experts.down_proj"):
        load_params(cfg, str(tmp_path), Mesh(0, 1, 0), device="cpu")


def test_no_checkpoint_raises_file_not_found(tmp_path, model):
    cfg, _ = model
    with pytest.raises(FileNotFoundError):
        load_params(cfg, str(tmp_path), Mesh(0, 1, 0), device="cpu")
