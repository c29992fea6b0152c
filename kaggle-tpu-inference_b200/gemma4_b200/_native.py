"""ctypes binding of the sm_100a C-ABI library ``libg4b200.so`` (include/g4b200.h).

There is no fallback: if the library is missing or fails to load, every entry point
raises.  Errors returned by the library become :class:`G4Error` carrying the code and
the library's own message (``g4_last_error``).
"""

from __future__ import annotations

import ctypes
import os
from ctypes import POINTER, c_char_p, c_float, c_int, c_longlong, c_void_p

from .build import LIB

G4_OK = 0
G4_ERR_ARG = -1
G4_ERR_SHAPE = -2
G4_ERR_LAUNCH = -3
G4_ERR_TIMEOUT = -4
G4_ERR_STATE = -5
G4_ERR_NOMEM = -6
G4_ERR_CUDA = -7

G4_STATUS_PEER_TIMEOUT = 0x1
G4_STATUS_MBAR_TIMEOUT = 0x2
G4_STATUS_BAD_TOKEN = 0x4
G4_STATUS_POS_OVERFLOW = 0x8

CTRL_POS, CTRL_STEP, CTRL_FORCED_LEN, CTRL_STATUS, CTRL_TIMEOUT_US, CTRL_WRITE_LOGITS = range(6)
CTRL_TEMPERATURE, CTRL_TOP_P, CTRL_TOP_K, CTRL_SEED_LO, CTRL_SEED_HI = range(6, 11)
CTRL_WORDS = 16
SAMPLE_MAX_TOP_K = 128
PREFILL_DENSE_MOE = 0x1

EXPORTS = (
    "g4_version", "g4_strerror", "g4_last_error",
    "g4_comm_create", "g4_comm_get_handle", "g4_comm_open", "g4_comm_destroy",
    "g4_model_create", "g4_model_set_tensor", "g4_model_set_comm", "g4_model_finalize",
    "g4_step", "g4_graph_capture", "g4_graph_launch", "g4_model_status",
    "g4_model_kernel_count", "g4_model_host_tokens", "g4_model_profile", "g4_model_destroy",
    "g4_moe_block", "g4_attention_decode", "g4_trace_read", "g4_attention_decode_noalloc",
    "g4_model_set_engine", "g4_prefill", "g4_gemm_bf16", "g4_comm_open_local",
    "g4_batch_reserve", "g4_batch_prefill", "g4_batch_step", "g4_batch_status",
    "g4_selftest_peer_timeout",
)

ENGINE_STEP_KERNEL = 0  # one persistent kernel per decode step (default)
ENGINE_OP_KERNELS = 1   # 6 kernels per layer + 1
ENGINES = {"step": ENGINE_STEP_KERNEL, "ops": ENGINE_OP_KERNELS}


class G4Error(RuntimeError):
    def __init__(self, code: int, where: str, message: str):
        super().__init__(f"{where}: {message} (code {code})")
        self.code = code


class G4Config(ctypes.Structure):
    """Mirror of ``struct g4_config`` (include/g4b200.h)."""

    _fields_ = [
        ("hidden_size", c_int), ("num_hidden_layers", c_int), ("num_attention_heads", c_int),
        ("head_dim", c_int), ("global_head_dim", c_int), ("num_key_value_heads", c_int),
        ("num_global_key_value_heads", c_int), ("intermediate_size", c_int),
        ("moe_intermediate_size", c_int), ("num_experts", c_int), ("top_k_experts", c_int),
        ("sliding_window", c_int), ("vocab_size", c_int), ("attention_k_eq_v", c_int),
        ("enable_moe_block", c_int), ("rms_norm_eps", c_float),
        ("final_logit_softcapping", c_float), ("rope_theta_sliding", c_float),
        ("rope_theta_full", c_float), ("rope_partial_rotary_factor_full", c_float),
    ]

    @classmethod
    def from_text_config(cls, cfg) -> "G4Config":
        c = cls()
        for name, _ in cls._fields_:
            v = getattr(cfg, name)
            if name == "final_logit_softcapping":
                v = float(v) if v else 0.0
            setattr(c, name, int(v) if isinstance(v, bool) else v)
        return c


_lib = None


def lib() -> ctypes.CDLL:
    """Load the library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    path = os.environ.get("G4B200_LIB", LIB)  # e.g. the -DG4_TRACE build
    if not os.path.exists(path):
        raise RuntimeError(
            f"{path} is missing: build it with `python -m gemma4_b200.build` "
            "(the B200 path has no fallback)")
    L = ctypes.CDLL(path)
    L.g4_version.restype = c_char_p
    L.g4_strerror.restype = c_char_p
    L.g4_strerror.argtypes = [c_int]
    L.g4_last_error.restype = c_char_p
    L.g4_comm_create.argtypes = [c_int, c_int, c_int, c_int, POINTER(c_void_p)]
    L.g4_comm_get_handle.argtypes = [c_void_p, c_char_p]
    L.g4_comm_open.argtypes = [c_void_p, c_char_p]
    L.g4_comm_destroy.argtypes = [c_void_p]
    L.g4_comm_open_local.argtypes = [POINTER(c_void_p), c_int]
    L.g4_model_create.argtypes = [POINTER(G4Config), c_char_p, c_int, c_int, c_int, c_int,
                                  POINTER(c_void_p)]
    L.g4_model_set_tensor.argtypes = [c_void_p, c_char_p, c_void_p, c_longlong]
    L.g4_model_set_comm.argtypes = [c_void_p, c_void_p]
    L.g4_model_finalize.argtypes = [c_void_p]
    L.g4_step.argtypes = [c_void_p, c_void_p]
    L.g4_graph_capture.argtypes = [c_void_p, c_void_p]
    L.g4_graph_launch.argtypes = [c_void_p, c_void_p, c_int]
    L.g4_model_status.argtypes = [c_void_p, c_void_p, POINTER(c_int)]
    L.g4_model_kernel_count.argtypes = [c_void_p]
    L.g4_model_set_engine.argtypes = [c_void_p, c_int]
    L.g4_prefill.argtypes = [c_void_p, c_int, c_int, c_int, c_void_p]
    L.g4_batch_reserve.argtypes = [c_void_p, c_int, c_int]
    L.g4_batch_prefill.argtypes = [c_void_p, c_int, c_int, c_void_p, c_void_p]
    L.g4_batch_step.argtypes = [c_void_p, c_void_p, c_void_p, c_void_p]
    L.g4_batch_status.argtypes = [c_void_p, c_void_p, POINTER(c_int)]
    L.g4_selftest_peer_timeout.argtypes = [c_int, POINTER(c_int)]
    L.g4_gemm_bf16.argtypes = [c_void_p, c_longlong, c_void_p, c_longlong, c_void_p, c_longlong, c_int, c_int,
                               c_int, c_int, c_void_p, c_void_p]
    L.g4_model_host_tokens.argtypes = [c_void_p, POINTER(POINTER(c_int))]
    L.g4_model_profile.argtypes = [c_void_p, c_void_p, c_int, POINTER(c_float), c_int]
    L.g4_model_destroy.argtypes = [c_void_p]
    L.g4_trace_read.argtypes = [c_void_p, c_longlong]
    L.g4_moe_block.argtypes = [POINTER(G4Config), c_int, c_int, c_void_p] + [c_void_p] * 11
    L.g4_attention_decode.argtypes = ([c_void_p] * 5 + [c_int] * 7 + [c_float] * 3
                                      + [c_void_p, c_void_p])
    L.g4_attention_decode_noalloc.argtypes = L.g4_attention_decode.argtypes
    for name in EXPORTS:
        if name not in ("g4_version", "g4_strerror", "g4_last_error"):
            getattr(L, name).restype = c_int
    _lib = L
    return L


def check(rc: int, where: str) -> None:
    if rc != G4_OK:
        msg = lib().g4_last_error().decode(errors="replace")
        raise G4Error(rc, where, msg or lib().g4_strerror(rc).decode())


def ptr(t) -> int:
    """Device address of a torch tensor (raises on CPU tensors)."""
    if not t.is_cuda:
        raise ValueError("g4b200 entry points take CUDA tensors")
    return t.data_ptr()


def stream_handle(stream=None) -> int:
    import torch

    s = stream if stream is not None else torch.cuda.current_stream()
    return s.cuda_stream
