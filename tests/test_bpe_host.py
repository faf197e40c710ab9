"""Host-side argument checks of the GPU tokenizer's C ABI (no GPU needed): rbk_bpe_create
rejects bad tables with RBK_ERR_INVALID and a message before touching the device, and the
encode / decode entries reject a null handle.  Without a GPU a valid table fails cleanly
with a CUDA or unsupported-device status, never by exiting."""
import ctypes as C
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "rubidium-train_b200"))


@pytest.fixture(scope="module")
def lib():
    from rbk import LIB_PATH
    if not os.path.exists(LIB_PATH):
        pytest.fail(f"{LIB_PATH} not built (run __graft_entry__.build())")
    from rbk import lib as get
    return get()


def _create(lib, vocab, merges):
    from rbk.tokenizer import vocab_arrays
    inv, offs, lens = vocab_arrays(vocab)
    m = np.asarray(merges, dtype=np.int32).reshape(-1, 3)
    cols = [np.ascontiguousarray(m[:, i]) for i in range(3)]
    p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
    h = C.c_void_p()
    st = lib.rbk_bpe_create(C.byref(h), 0, len(vocab), C.c_char_p(inv), len(inv), p(offs), p(lens), p(cols[0]),
                            p(cols[1]), p(cols[2]), len(m))
    return st, h, lib.rbk_last_error().decode()


BASE = [b"<pad>", b"<unk>", b"<bos>", b"<eos>", b"<sep>"] + [bytes([c]) for c in range(256)]


def test_create_rejects_small_vocabulary(lib):
    st, h, msg = _create(lib, BASE[:200], [])
    assert st == -1 and not h.value and "261" in msg


def test_create_rejects_result_outside_vocabulary(lib):
    st, h, msg = _create(lib, BASE + [b"ab"], [(5 + 97, 5 + 98, 262)])
    assert st == -1 and not h.value and "outside the vocabulary" in msg


def test_entries_reject_null_handle(lib):
    assert lib.rbk_bpe_encode(None, None, None, None, 1, None, None, 64, None, None) == -1
    assert lib.rbk_bpe_encode_batch(None, None, 1, None, None, 64, None) == -1
    assert lib.rbk_bpe_decode_batch(None, None, 0, None, 1, None, 16, None, None) == -1
    assert lib.rbk_bpe_destroy(None) == 0
    assert lib.rbk_bpe_num_rules(None) == 0


def test_valid_table_without_gpu_fails_cleanly(lib):
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    st, h, msg = _create(lib, BASE + [b"ab"], [(5 + 97, 5 + 98, 261)])
    assert st < 0 and not h.value and len(msg) > 0
