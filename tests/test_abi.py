"""The C-ABI boundary (CPU): librbk.so loads and exports exactly what include/rbk.h declares."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "rbk.h")


def header_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(rbk_[a-z0-9_]+)\s*\(", src)))


def test_header_parses():
    syms = header_symbols()
    assert "rbk_gemm" in syms and "rbk_adam_tail" in syms and "rbk_ln_bwd" in syms


def test_library_exports_every_declared_symbol():
    import torch  # noqa: F401  (torch's bundled NCCL must be loaded before librbk's libnccl.so.2 need)
    from rbk import LIB_PATH
    if not os.path.exists(LIB_PATH):
        pytest.fail(f"{LIB_PATH} not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(LIB_PATH)
    missing = [s for s in header_symbols() if not hasattr(lib, s)]
    assert not missing, f"declared in rbk.h but not exported: {missing}"


def test_binding_covers_header():
    from rbk import declared_symbols
    assert set(header_symbols()) == set(declared_symbols())


def test_version_and_error_string_without_gpu():
    from rbk import lib
    assert lib().rbk_version() >= 1
    assert isinstance(lib().rbk_last_error(), bytes)


def test_gpu_free_ctx_create_fails_cleanly():
    """Without a usable sm_100 device the context call returns an error code, never exits."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from rbk import lib
    h = ctypes.c_void_p()
    st = lib().rbk_ctx_create(ctypes.byref(h), 0)
    assert st < 0
    assert len(lib().rbk_last_error()) > 0
