"""Generate the committed golden vectors under tests/golden/ (run from the repo root).

  hf_parity_tiny.npz  logits of HuggingFace transformers on the reference's own parity
                      model (gemma4_tpu tests/test_parity.py:29-74; see tests/hf_tiny.py):
                      24-token prefill logits and the decode-position logits.
  oracle_config1.npz  benchmark config 1 (tiny random model, seed 0 weights N(0,0.02),
                      128 prompt ids ~U[0,4096) from numpy seed 0, 32 greedy tokens) run
                      token by token through the bf16-faithful oracle: generated ids,
                      the top-2 margin per generated position, and the full logits of
                      four positions.

    python tests/golden/make_golden.py
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.join(ROOT, "kaggle-tpu-inference_b200"), os.path.dirname(HERE)]

CONFIG1_PROMPT = 128
CONFIG1_NEW = 32
CONFIG1_KEEP = (0, 64, 127, 150)   # positions whose full logits are stored


def config1_inputs():
    from gemma4_b200.config import tiny_parity_config
    from gemma4_b200.weights import random_params

    cfg = tiny_parity_config()
    params = random_params(cfg, seed=0, std=0.02)
    prompt = np.random.default_rng(0).integers(0, cfg.vocab_size, CONFIG1_PROMPT).tolist()
    return cfg, params, prompt


def make_hf():
    import hf_tiny

    hf_cfg, model = hf_tiny.build_hf()
    ids = hf_tiny.input_ids()
    logits = hf_tiny.hf_logits(model, ids).numpy()
    np.savez_compressed(os.path.join(HERE, "hf_parity_tiny.npz"), ids=ids, logits=logits)


def make_config1():
    from oracle.reference_model import Oracle

    cfg, params, prompt = config1_inputs()
    o = Oracle(cfg, params, mode="bf16")
    max_len = CONFIG1_PROMPT + CONFIG1_NEW
    logits, ids = o.greedy_generate(prompt, CONFIG1_NEW, max_len)
    top2 = torch.topk(logits, 2, dim=-1).values
    margin = (top2[:, 0] - top2[:, 1]).numpy()
    np.savez_compressed(
        os.path.join(HERE, "oracle_config1.npz"),
        prompt=np.array(prompt, np.int32), ids=np.array(ids, np.int32), margin=margin,
        keep=np.array(CONFIG1_KEEP, np.int32), logits=logits[list(CONFIG1_KEEP)].numpy(),
        argmax=logits.argmax(-1).numpy().astype(np.int32))


if __name__ == "__main__":
    make_hf()
    make_config1()
    print("golden vectors written to", HERE)
