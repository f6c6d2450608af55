"""
The C-ABI library without a GPU: it loads, reports its ABI version, exports
every function include/cg_b200.h declares, and every symbol the Python binding
uses is declared there. No compute call is made.
"""

from __future__ import annotations

import ctypes
import os
import re

import pytest

from create_graph_b200 import native
from tests.conftest import ROOT

HEADERS = [os.path.join(ROOT, "include", name) for name in sorted(os.listdir(os.path.join(ROOT, "include")))]


def declared_functions() -> set[str]:
    names = set()
    for path in HEADERS:
        text = open(path).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[a-z_0-9]+\s*\*?\s*(cg_[a-z0-9_]+)\s*\(", text, re.M):
            names.add(m.group(1))
    return names


def test_library_loads_with_matching_abi():
    lib = native.load_library()
    assert lib.cg_version() == native.ABI_VERSION
    assert lib.cg_last_error() == b""


def test_every_declared_function_is_exported():
    lib = ctypes.CDLL(str(native.LIB_PATH))
    declared = declared_functions()
    assert declared, "no declarations parsed"
    missing = [name for name in sorted(declared) if not hasattr(lib, name)]
    assert not missing, missing


def test_binding_uses_only_declared_functions():
    assert set(native.exported_symbols()) <= declared_functions()


def test_compute_without_cuda_fails_loudly():
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is visible")
    with pytest.raises(native.NativeError, match="CUDA"):
        native.lib()
