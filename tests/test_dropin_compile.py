"""The C++ drop-in compiles against the reference's own callers.

- The reference trainer's src/main.cpp, unchanged, compiles and links against
  include/rubidium/compat ("model.h" resolves to the drop-in) and librbk.  The source is
  read from the reference tree that the build recorded (oracle/_ref/REFERENCE_ROOT) or
  from RBK_REFERENCE, copied to a temporary directory (so its own directory's model.h is
  not the one found) and compiled there; skipped when the tree is absent.
- tests/dropin/fine_tune_calls.cpp, the model / LoRA call sequence of the reference's
  LoRA trainer (src/fine_tune.cu, without its tokenizer), compiles against "model.h" /
  "lora.h" and, on a B200, runs: base checkpoint written and loaded back (character map
  included), rank-16 adapters added, two steps of two micro-steps.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")
COMPAT = os.path.join(INC, "rubidium", "compat")
LIBDIR = os.path.join(ROOT, "rubidium-train_b200", "lib")
CUDA = "/usr/local/cuda"


def _reference_root():
    root = os.environ.get("RBK_REFERENCE")
    rec = os.path.join(ROOT, "oracle", "_ref", "REFERENCE_ROOT")
    if not root and os.path.exists(rec):
        root = open(rec).read().strip()
    if root and os.path.exists(os.path.join(root, "src", "main.cpp")):
        return root
    return None


def _compile(src, out):
    if not os.path.exists(os.path.join(LIBDIR, "librbk.so")):
        pytest.skip("librbk.so not built")
    cmd = ["g++", "-std=c++17", "-O1", "-w", f"-I{COMPAT}", f"-I{INC}", f"-I{CUDA}/include", src, "-o", out,
           f"-L{LIBDIR}", "-lrbk", f"-L{CUDA}/lib64", "-lcudart", f"-Wl,-rpath,{LIBDIR}"]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]


def test_reference_main_compiles_unchanged(tmp_path):
    root = _reference_root()
    if root is None:
        pytest.skip("reference sources not present")
    src = tmp_path / "main.cpp"
    shutil.copyfile(os.path.join(root, "src", "main.cpp"), src)
    _compile(str(src), str(tmp_path / "main"))


def test_fine_tune_call_sequence_compiles(tmp_path):
    _compile(os.path.join(ROOT, "tests", "dropin", "fine_tune_calls.cpp"), str(tmp_path / "ftc"))


@pytest.mark.gpu
def test_fine_tune_call_sequence_runs(tmp_path):
    exe = tmp_path / "ftc"
    _compile(os.path.join(ROOT, "tests", "dropin", "fine_tune_calls.cpp"), str(exe))
    r = subprocess.run([str(exe), str(tmp_path / "base.bin"), "2"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    assert "fine-tune call sequence ok" in r.stdout
    assert "LoRA params: ~0.016M" in r.stdout     # 4 x L2 x D128 x r16 = 16384 adapter parameters
