"""The C-ABI library loads and exports every entry point of
include/tinyoai_cuda.h; without a GPU it refuses to load a model (no CPU
fallback). No GPU compute is attempted here."""
import re
from pathlib import Path

import numpy as np
import pytest

from tinyoai_b200 import _lib
from tinyoai_b200.checkpoint import load_stablelm_dir

ROOT = Path(__file__).resolve().parents[1]


def declared_symbols():
    text = (ROOT / "include" / "tinyoai_cuda.h").read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\*?\s+\*?(tcu_\w+)\s*\(", text, re.M)))


def test_header_matches_binding_list():
    assert declared_symbols() == sorted(_lib.EXPORTS)


def test_library_exports_every_symbol():
    L = _lib.lib()
    for name in declared_symbols():
        assert hasattr(L, name), name
    assert L.tcu_abi_version() == 1


def test_no_gpu_means_no_model(golden):
    """Without an sm_100 device the loader fails with TCU_ENODEV; it never
    falls back to another implementation."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    from tinyoai_b200 import BackendError, Model, device_count
    assert device_count() == 0
    cfg, tensors = load_stablelm_dir(golden / "stablelm_tiny")
    with pytest.raises(BackendError) as e:
        Model.load_stablelm(cfg, tensors)
    assert e.value.code in (_lib.TCU_ENODEV, _lib.TCU_ECUDA)


def test_invalid_arguments_rejected_before_device():
    """Config validation (stablelm.go:85-111) happens before any device work."""
    L = _lib.lib()
    import ctypes as C
    cfg = _lib.StableLMConfig(342, 16, 40, 2, 3, 1, 64, 2, 3, 1e-5, 10000.0, 0.5)  # 16 % 3 != 0
    out = C.c_void_p()
    rc = L.tcu_stablelm_load(C.byref(cfg), None, 0, None, C.byref(out))
    assert rc == _lib.TCU_EINVAL
    assert b"dimensions" in L.tcu_last_error()
    cfg = _lib.StableLMConfig(342, 16, 40, 2, 2, 1, 64, 2, 3, 1e-5, 10000.0, 0.125)  # rotary 1
    assert L.tcu_stablelm_load(C.byref(cfg), None, 0, None, C.byref(out)) == _lib.TCU_EINVAL
    assert L.tcu_llama_load(b"\x00" * 8, 8, None, C.byref(out)) == _lib.TCU_EINVAL
