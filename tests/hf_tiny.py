"""The tiny random Gemma-4 of the reference's parity test, built with HF transformers.

Same structure and initialisation as gemma4_tpu tests/test_parity.py:29-74: vocab 1024,
hidden 256, 4 layers [S, F, S, F], 16 query heads, 8 KV heads of dim 32 on sliding
layers, 2 global KV heads of dim 64 with k==v on full layers, window 8, 16 experts
top-4, moe_intermediate 64, MLP 128, softcap 30, partial rotary 0.25; every parameter
drawn N(0, 0.05) after ``torch.manual_seed(0)`` and cast to bf16; input 24 ids from
``np.random.default_rng(0)`` (test_parity.py:95-97).
"""

from __future__ import annotations

import json
import os
import tempfile

import numpy as np
import torch

LAYER_TYPES = ["sliding_attention", "full_attention", "sliding_attention", "full_attention"]
SEQ = 24


def build_hf():
    from transformers.models.gemma4.configuration_gemma4 import Gemma4TextConfig
    from transformers.models.gemma4.modeling_gemma4 import Gemma4ForCausalLM

    hf_cfg = Gemma4TextConfig(
        vocab_size=1024, hidden_size=256, intermediate_size=128, num_hidden_layers=4,
        num_attention_heads=16, num_key_value_heads=8, head_dim=32, global_head_dim=64,
        num_global_key_value_heads=2, sliding_window=8, layer_types=LAYER_TYPES,
        num_experts=16, top_k_experts=4, moe_intermediate_size=64, enable_moe_block=True,
        attention_k_eq_v=True, final_logit_softcapping=30.0, tie_word_embeddings=True,
        hidden_size_per_layer_input=0, num_kv_shared_layers=0, rms_norm_eps=1e-6,
        hidden_activation="gelu_pytorch_tanh",
        rope_parameters={
            "full_attention": {"rope_type": "proportional", "rope_theta": 1000000.0,
                               "partial_rotary_factor": 0.25},
            "sliding_attention": {"rope_type": "default", "rope_theta": 10000.0},
        },
        use_bidirectional_attention="vision", attn_implementation="eager",
    )
    torch.manual_seed(0)
    hf_cfg._experts_implementation = "eager"
    model = Gemma4ForCausalLM(hf_cfg)
    with torch.no_grad():
        for p in model.parameters():
            p.normal_(0.0, 0.05)
    return hf_cfg, model.to(torch.bfloat16).eval()


def text_config_of(hf_cfg):
    from gemma4_b200.config import load_text_config

    with tempfile.TemporaryDirectory() as td:
        with open(os.path.join(td, "config.json"), "w") as f:
            json.dump({"text_config": hf_cfg.to_dict(), "eos_token_id": [1]}, f, default=str)
        return load_text_config(td)


def canonical_params(cfg, model):
    from gemma4_b200.weights import params_from_arrays

    sd = {k: v.detach() for k, v in model.state_dict().items()}
    return params_from_arrays(cfg, sd.__getitem__, list(sd), prefix="model.")


def input_ids():
    rng = np.random.default_rng(0)
    return rng.integers(0, 1024, size=(1, SEQ)).astype(np.int64)


def hf_logits(model, ids):
    with torch.no_grad():
        return model(input_ids=torch.tensor(ids)).logits.float()[0]
