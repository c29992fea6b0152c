"""The C-ABI library loads and exports every entry point that include/g4b200.h declares.

No compute is launched here (no GPU on the CPU runner); argument validation that
happens before any CUDA call is exercised.
"""

import ctypes
import os
import re

from gemma4_b200 import _native as N
from gemma4_b200.build import INCLUDE, LIB, sources, up_to_date


def declared_symbols():
    text = open(os.path.join(INCLUDE, "g4b200.h")).read()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\**(g4_\w+)\s*\(", text, re.M)))


def test_library_is_built_and_current():
    assert os.path.exists(LIB), "run python -m gemma4_b200.build"
    assert up_to_date(), "libg4b200.so is older than its sources"
    assert len(sources()) >= 5


def test_every_declared_symbol_is_exported():
    lib = N.lib()
    syms = declared_symbols()
    assert len(syms) >= 18
    for s in syms:
        assert hasattr(lib, s), s
    assert set(syms) == set(N.EXPORTS)


def test_version_and_errors():
    lib = N.lib()
    assert b"sm_100a" in lib.g4_version()
    assert lib.g4_strerror(N.G4_ERR_TIMEOUT) == b"bounded device wait timed out"


def test_argument_validation_before_cuda():
    lib = N.lib()
    out = ctypes.c_void_p()
    assert lib.g4_model_create(None, b"\0", 0, 1, 16, 0, ctypes.byref(out)) == N.G4_ERR_ARG
    cfg = N.G4Config()
    assert lib.g4_model_create(ctypes.byref(cfg), b"\0", 0, 1, 16, 0, ctypes.byref(out)) == N.G4_ERR_ARG
    assert lib.g4_comm_create(0, 3, 2, 2816, ctypes.byref(out)) == N.G4_ERR_ARG
    assert lib.g4_step(None, None) == N.G4_ERR_ARG
    assert b"null" in lib.g4_last_error()
    assert lib.g4_attention_decode(*([None] * 5), *([0] * 7), 0.0, 0.0, 0.0, None, None) == N.G4_ERR_ARG
