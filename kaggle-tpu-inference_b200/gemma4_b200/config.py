"""Gemma-4 MoE text-stack configuration (the shape contract of the decode path).

Field names and derived helpers follow the reference's ``TextConfig``
(gemma4_tpu/config.py:11-49) so that callers written against it read the same
attributes; ``load_text_config`` reads the same HF ``config.json`` keys
(gemma4_tpu/config.py:52-92).
"""

from __future__ import annotations

import dataclasses
import json
import math
import os

FULL = "full_attention"
SLIDING = "sliding_attention"


@dataclasses.dataclass(frozen=True)
class TextConfig:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    head_dim: int
    global_head_dim: int
    num_key_value_heads: int
    num_global_key_value_heads: int
    intermediate_size: int
    moe_intermediate_size: int
    num_experts: int
    top_k_experts: int
    sliding_window: int
    rms_norm_eps: float
    vocab_size: int
    final_logit_softcapping: float | None
    attention_k_eq_v: bool
    enable_moe_block: bool
    layer_types: tuple[str, ...]
    rope_theta_sliding: float
    rope_theta_full: float
    rope_partial_rotary_factor_full: float
    eos_token_ids: tuple[int, ...]

    @property
    def embed_scale(self) -> float:
        # The forward pass rounds this to bf16 before use (sqrt(2816) -> 53.0).
        return math.sqrt(self.hidden_size)

    def head_dim_for(self, layer_type: str) -> int:
        return self.global_head_dim if layer_type == FULL else self.head_dim

    def kv_heads_for(self, layer_type: str) -> int:
        # Only k==v full layers use the (smaller) global KV head count.
        if layer_type == FULL and self.attention_k_eq_v:
            return self.num_global_key_value_heads
        return self.num_key_value_heads

    def k_eq_v_for(self, layer_type: str) -> bool:
        return bool(self.attention_k_eq_v) and layer_type == FULL


def _eos_list(value) -> list[int]:
    if value is None:
        return []
    return [int(value)] if isinstance(value, int) else [int(v) for v in value]


def load_text_config(model_dir: str) -> TextConfig:
    """Read ``config.json`` (+ optional ``generation_config.json``) of an HF Gemma-4 dir."""
    with open(os.path.join(model_dir, "config.json")) as f:
        raw = json.load(f)
    tc = raw["text_config"] if "text_config" in raw else raw

    eos: list[int] = []
    gen_path = os.path.join(model_dir, "generation_config.json")
    if os.path.exists(gen_path):
        with open(gen_path) as f:
            eos = _eos_list(json.load(f).get("eos_token_id"))
    if not eos:
        eos = _eos_list(raw.get("eos_token_id", tc.get("eos_token_id", 1)))

    rope = tc["rope_parameters"]
    return TextConfig(
        hidden_size=tc["hidden_size"],
        num_hidden_layers=tc["num_hidden_layers"],
        num_attention_heads=tc["num_attention_heads"],
        head_dim=tc["head_dim"],
        global_head_dim=tc.get("global_head_dim") or tc["head_dim"],
        num_key_value_heads=tc["num_key_value_heads"],
        num_global_key_value_heads=tc.get("num_global_key_value_heads") or tc["num_key_value_heads"],
        intermediate_size=tc["intermediate_size"],
        moe_intermediate_size=tc["moe_intermediate_size"],
        num_experts=tc["num_experts"],
        top_k_experts=tc["top_k_experts"],
        sliding_window=tc["sliding_window"],
        rms_norm_eps=tc["rms_norm_eps"],
        vocab_size=tc["vocab_size"],
        final_logit_softcapping=tc.get("final_logit_softcapping"),
        attention_k_eq_v=bool(tc.get("attention_k_eq_v", False)),
        enable_moe_block=bool(tc.get("enable_moe_block", False)),
        layer_types=tuple(tc["layer_types"]),
        rope_theta_sliding=float(rope[SLIDING]["rope_theta"]),
        rope_theta_full=float(rope[FULL]["rope_theta"]),
        rope_partial_rotary_factor_full=float(rope[FULL].get("partial_rotary_factor", 1.0)),
        eos_token_ids=tuple(eos),
    )


def interleaved_layer_types(n_layers: int, period: int = 6) -> tuple[str, ...]:
    """Gemma-4 layer pattern: ``period-1`` sliding layers then one full layer."""
    return tuple(FULL if (i + 1) % period == 0 else SLIDING for i in range(n_layers))


def make_config(**kw) -> TextConfig:
    """Build a config from keyword overrides of the 26B-A4B shape (benchmark config 4)."""
    base = dict(
        hidden_size=2816,
        num_hidden_layers=30,
        num_attention_heads=16,
        head_dim=256,
        global_head_dim=256,
        num_key_value_heads=8,
        num_global_key_value_heads=2,
        intermediate_size=2112,
        moe_intermediate_size=704,
        num_experts=128,
        top_k_experts=8,
        sliding_window=1024,
        rms_norm_eps=1e-6,
        vocab_size=262144,
        final_logit_softcapping=30.0,
        attention_k_eq_v=True,
        enable_moe_block=True,
        layer_types=None,
        rope_theta_sliding=10000.0,
        rope_theta_full=1000000.0,
        rope_partial_rotary_factor_full=0.25,
        eos_token_ids=(1,),
    )
    base.update(kw)
    if base["layer_types"] is None:
        base["layer_types"] = interleaved_layer_types(base["num_hidden_layers"])
    base["layer_types"] = tuple(base["layer_types"])
    return TextConfig(**base)


def gemma4_26b_a4b(global_head_dim: int = 256) -> TextConfig:
    """benchmark config 4 (global_head_dim 256); 512 is the real checkpoint's value."""
    return make_config(global_head_dim=global_head_dim)


def tiny_parity_config() -> TextConfig:
    """benchmark config 1: the CPU-runnable tiny random model."""
    return make_config(
        hidden_size=256,
        num_hidden_layers=4,
        num_attention_heads=4,
        head_dim=64,
        global_head_dim=64,
        num_key_value_heads=2,
        num_global_key_value_heads=2,
        intermediate_size=512,
        moe_intermediate_size=128,
        num_experts=16,
        top_k_experts=4,
        sliding_window=64,
        vocab_size=4096,
        layer_types=(SLIDING, SLIDING, SLIDING, FULL),
    )
