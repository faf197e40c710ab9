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


def test_train_args_layout_matches_header(tmp_path):
    """The ctypes mirror of rbk_train_args has the C compiler's field offsets."""
    import shutil
    import subprocess
    if shutil.which("gcc") is None:
        pytest.skip("no gcc")
    from rbk._lib import TrainArgs
    names = [f for f, _ in TrainArgs._fields_]
    src = tmp_path / "off.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "rbk.h"\nint main(void) {\n' +
                   "".join(f'printf("%zu\\n", offsetof(rbk_train_args, {n}));\n' for n in names) +
                   'printf("%zu\\n", sizeof(rbk_train_args));\nreturn 0;\n}\n')
    exe = tmp_path / "off"
    subprocess.run(["gcc", "-I", os.path.join(ROOT, "include"), "-I/usr/local/cuda/include", str(src), "-o",
                    str(exe)], check=True)
    got = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    want = [getattr(TrainArgs, n).offset for n in names] + [ctypes.sizeof(TrainArgs)]
    assert got == want
