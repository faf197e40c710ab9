"""The C++ drop-in compiles against the reference's own callers.

- The reference trainer's src/main.cpp, unchanged, compiles and links against
  include/rubidium/compat ("model.h" resolves to the drop-in) and librbk.  The source is
  read from the reference tree that the build recorded (oracle/_ref/REFERENCE_ROOT) or
  from RBK_REFERENCE, copied to a temporary directory (so its own directory's model.h is
  not the one found) and compiled there; skipped when the tree is absent.
- The reference LoRA trainer src/fine_tune.cu, unchanged (plus `-include sstream`, which
  it needs and never includes), compiles with nvcc against the drop-in headers, the GPU
  tokenizer's "tokenizer_cuda.h" included, and links.
- tests/dropin/tokenizer_calls.cpp, the tokenizer call sequence under the reference's names,
  compiles and, on a B200, matches the oracle row for row and string for string.
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


def test_reference_fine_tune_compiles_unchanged(tmp_path):
    """src/fine_tune.cu, untouched, compiles with nvcc against the drop-in's "model.h",
    "lora.h" and "tokenizer_cuda.h" and links against librbk.  The file uses
    std::istringstream without including <sstream> (none of the reference's headers brings
    it in either), so the command adds `-include sstream`; no source line changes."""
    root = _reference_root()
    if root is None:
        pytest.skip("reference sources not present")
    if not os.path.exists(os.path.join(LIBDIR, "librbk.so")):
        pytest.skip("librbk.so not built")
    src = tmp_path / "fine_tune.cu"
    shutil.copyfile(os.path.join(root, "src", "fine_tune.cu"), src)
    cmd = [f"{CUDA}/bin/nvcc", "-std=c++17", "-O1", "-w", "-gencode", "arch=compute_100a,code=sm_100a",
           "-include", "sstream", f"-I{COMPAT}", f"-I{INC}", str(src), "-o", str(tmp_path / "fine_tune"),
           f"-L{LIBDIR}", "-lrbk", "-Xlinker", "-rpath", "-Xlinker", LIBDIR]
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]


def test_tokenizer_call_sequence_compiles(tmp_path):
    _compile(os.path.join(ROOT, "tests", "dropin", "tokenizer_calls.cpp"), str(tmp_path / "tkc"))


def _tables_file(path, vocab, merges, inputs):
    hx = lambda b: b.hex() if b else "-"  # noqa: E731
    with open(path, "w") as f:
        f.write(f"{len(vocab)} {len(merges)} {len(inputs)}\n")
        for v in vocab:
            f.write(hx(v) + "\n")
        for a, b, r in merges:
            f.write(f"{a} {b} {hx(vocab[r])}\n")
        for s in inputs:
            f.write(hx(s) + "\n")


@pytest.mark.gpu
def test_tokenizer_call_sequence_runs(tmp_path):
    """The reference-named tokenizer API through the drop-in header on a B200: the golden
    tokenizer's tables handed over as HostTokenizer fields, encode_string / decode_tokens per
    string, one encode_batch and one decode_batch (the reference's row layout), and
    tokenizer_validate_roundtrip; every id row and string equal to the oracle's."""
    import sys

    import numpy as np
    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests"))
    import oracle
    from test_oracle_bpe import golden
    g, vocab, merges = golden()
    corpus = g["enc_a_data"].tobytes()
    inputs = [b"", b"a", corpus[:1], corpus[100:900], corpus[:2047], corpus[2000:2300]] + \
        [corpus[i:i + 37 * k % 700 + 1] for k, i in enumerate(range(0, 5000, 250))]
    inputs = [s.replace(b"\0", b" ") for s in inputs]
    exe = tmp_path / "tkc"
    _compile(os.path.join(ROOT, "tests", "dropin", "tokenizer_calls.cpp"), str(exe))
    tables = tmp_path / "tables.txt"
    _tables_file(tables, vocab, merges, inputs)
    r = subprocess.run([str(exe), str(tables)], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]
    lines = r.stdout.splitlines()
    E = [list(map(int, ln.split()[1:])) for ln in lines if ln.startswith("E")]
    D = [ln.split()[1] for ln in lines if ln.startswith("D ")]
    B = [list(map(int, ln.split()[1:])) for ln in lines if ln.startswith("B ")]
    R = [ln.split()[1] for ln in lines if ln.startswith("R ")]
    V = [ln for ln in lines if ln.startswith("V ")]
    from rbk.tokenizer import pack_strings
    data, offs, lens = pack_strings(inputs)
    want, wl, _ = oracle.bpe_encode(merges, data, offs, lens, 2048)
    unhex = lambda h: b"" if h == "-" else bytes.fromhex(h)  # noqa: E731
    assert len(E) == len(B) == len(R) == len(inputs)
    for b, s in enumerate(inputs):
        n = int(wl[b])
        assert E[b] == want[b, :n].tolist(), b
        assert B[b][0] == n and B[b][1:] == want[b, :n].tolist(), b
        dec, _ = oracle.bpe_decode(vocab, want[b:b + 1, :n], n, wl[b:b + 1], 1024)
        assert unhex(D[b]) == bytes(dec[0]).split(b"\0", 1)[0], b
    # decode_batch reads row b at b * lengths[b] (rows may overlap), as the reference does
    flat = np.zeros(max(b * int(wl[b]) + int(wl[b]) for b in range(len(inputs))), np.int32)
    for b in range(len(inputs)):
        n = int(wl[b])
        flat[b * n:b * n + n] = want[b, :n]
    dec, _ = oracle.bpe_decode(vocab, flat, 0, wl, 4096)
    assert [unhex(x) for x in R] == [bytes(row).split(b"\0", 1)[0] for row in dec]
    assert V == ["V 1"]
