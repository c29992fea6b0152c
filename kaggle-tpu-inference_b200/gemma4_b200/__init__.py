"""B200 (sm_100a) tensor-parallel Gemma-4 26B-A4B decode engine.

Drop-in for the ``gemma4_tpu`` engine API of YLiu95/kaggle-tpu-inference: the same
``Engine`` / config / weights / limits interfaces, backed by the hand-written CUDA
kernels of ``libg4b200.so`` (C ABI in include/g4b200.h).  Heavy imports are lazy so
the thin client paths stay fast, like the reference package (gemma4_tpu/__init__.py).
"""

__all__ = ["Engine", "TextConfig", "load_text_config"]


def __getattr__(name):
    if name == "Engine":
        from .engine import Engine

        return Engine
    if name in ("TextConfig", "load_text_config"):
        from . import config

        return getattr(config, name)
    raise AttributeError(name)
