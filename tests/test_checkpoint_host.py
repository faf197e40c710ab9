"""Checkpoint file format on the host (no GPU): the reference's RBN2 layout plus the
optimizer/scaler extension block, read and written by rbk.checkpoint."""
import os
import struct

import numpy as np
import pytest

from rbk import checkpoint as ckpt
from rbk.model import ModelConfig, param_table

CFG = (512, 64, 128, 2, 2, 256)   # V T D H L FF


def _random_ck(rng, ext):
    tens = ckpt.file_tensors(*CFG)
    w16 = {n: rng.standard_normal((r, c) if r > 1 else c).astype(np.float16) for n, r, c in tens}
    ck = ckpt.Checkpoint(CFG, rng.integers(0, 100, 256).astype(np.int32), w16)
    if ext:
        ck.scaler = dict(scale=1024.0, unskipped=17, interval=2000, skipped=0, applied_steps=41,
                         overflow_steps=3, status=0, pad=0)
        for fam in (ck.masters, ck.adam_m, ck.adam_v):
            for n, r, c in tens:
                fam[n] = rng.standard_normal((r, c) if r > 1 else c).astype(np.float32)
    return ck


def test_file_order_is_the_reference_save_order():
    names = [n for n, _, _ in ckpt.file_tensors(*CFG)]
    # src/model.cu:605-619: embeddings, per layer ln1 ln2 q k v o w1 w2 (weight then bias), head
    assert names[:2] == ["token_emb", "pos_emb"]
    assert names[2:18] == [f"layers.0.{n}" for n in ["ln1_w", "ln1_b", "ln2_w", "ln2_b", "wq", "bq", "wk", "bk",
                                                     "wv", "bv", "wo", "bo", "w1", "b1", "w2", "b2"]]
    assert names[-4:] == ["ln_f_w", "ln_f_b", "lm_w", "lm_b"]
    # same tensors and shapes as the device arena (which orders them differently and pads them)
    V, T, D, H, L, FF = CFG
    tab, _ = param_table(ModelConfig(V=V, T=T, D=D, H=H, L=L, FF=FF))
    assert sorted((n, r, c) for n, _, r, c in tab) == sorted(ckpt.file_tensors(*CFG))


@pytest.mark.parametrize("ext", [False, True])
def test_round_trip(tmp_path, ext):
    rng = np.random.default_rng(5)
    ck = _random_ck(rng, ext)
    p = tmp_path / "m.rbn2"
    ckpt.write(p, ck)
    V, T, D, H, L, FF = CFG
    n_elems = sum(r * c for _, r, c in ckpt.file_tensors(*CFG))
    size = 4 + 24 + 1024 + 2 * n_elems + ((4 + 12 + 32 + 12 * n_elems) if ext else 0)
    assert os.path.getsize(p) == size
    with open(p, "rb") as f:
        head = f.read(28)
    assert head[:4] == b"RBN2" and struct.unpack("<6i", head[4:]) == CFG
    got = ckpt.read(p)
    assert got.config == CFG and np.array_equal(got.char_map, ck.char_map)
    for n in ck.weights16:
        assert np.array_equal(got.weights16[n], ck.weights16[n])
    assert got.has_optimizer_state == ext
    if ext:
        assert got.scaler == ck.scaler
        for a, b in ((got.masters, ck.masters), (got.adam_m, ck.adam_m), (got.adam_v, ck.adam_v)):
            for n in b:
                assert np.array_equal(a[n], b[n])


def test_truncated_and_foreign_files_are_rejected(tmp_path):
    rng = np.random.default_rng(6)
    p = tmp_path / "m.rbn2"
    ckpt.write(p, _random_ck(rng, True))
    data = open(p, "rb").read()
    for cut in (20, 4 + 24 + 1024 + 100, len(data) - 8):
        q = tmp_path / f"cut{cut}"
        q.write_bytes(data[:cut])
        with pytest.raises(ValueError):
            ckpt.read(q)
    q = tmp_path / "foreign"
    q.write_bytes(b"XXXX" + data[4:])
    with pytest.raises(ValueError):
        ckpt.read(q)
