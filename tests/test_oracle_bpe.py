"""The tokenizer oracle (oracle/bpe.cpp) on the CPU: pinned against the golden vectors the
reference's own encode_kernel / decode_kernel produced (tests/golden/bpe_ref.npz), against
those kernels live when oracle/_ref/libreftok.so is built here, and on the contract where
the reference is undefined (empty strings, truncation, row addressing, ids outside the
vocabulary).  No GPU."""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "rubidium-train_b200"))

import oracle  # noqa: E402

GOLD = os.path.join(ROOT, "tests", "golden", "bpe_ref.npz")


def golden():
    g = np.load(GOLD)
    lens = g["vocab_lengths"]
    vb = g["vocab_bytes"].tobytes()
    offs = np.concatenate([[0], np.cumsum(lens)[:-1]])
    vocab = [vb[o:o + n] for o, n in zip(offs, lens)]
    return g, vocab, [tuple(r) for r in g["merges"]]


def ref_to_strided(flat, lengths):
    ld = max(int(lengths.max()), 1)
    rows = np.zeros((len(lengths), ld), np.int32)
    for b, n in enumerate(lengths):
        rows[b, :n] = flat[b * n:b * n + n]
    return rows, ld


@pytest.mark.parametrize("tag", ["a", "b"])
def test_oracle_encode_matches_reference_golden(tag):
    g, _, merges = golden()
    ms = int(g[f"enc_{tag}_max_seq_len"])
    rows, rl, cut = oracle.bpe_encode(merges, g[f"enc_{tag}_data"], g[f"enc_{tag}_offsets"],
                                      g[f"enc_{tag}_lengths"], ms)
    assert cut == 0
    assert np.array_equal(rl, g[f"enc_{tag}_out_lengths"])
    want = g[f"enc_{tag}_rows"]
    for b, n in enumerate(rl):
        assert np.array_equal(rows[b, :n], want[b, :n]), b
        assert rows[b, n - 1] == 3 and (rows[b, n:] == 0).all()


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_oracle_decode_matches_reference_golden(tag):
    g, vocab, _ = golden()
    msl = int(g[f"dec_{tag}_max_string_len"])
    got, bad = oracle.bpe_decode(vocab, g["dec_tokens_ref_layout"], 0, g["dec_lengths"], msl)
    assert bad == 0
    assert np.array_equal(got, g[f"dec_{tag}_out"])
    # the same rows at an explicit stride
    rows, ld = ref_to_strided(g["dec_tokens_ref_layout"], g["dec_lengths"])
    got2, _ = oracle.bpe_decode(vocab, rows, ld, g["dec_lengths"], msl)
    assert np.array_equal(got2, g[f"dec_{tag}_out"])


def test_golden_merges_reach_whole_words():
    """The fixture exercises real merging: most strings shrink well below their byte count."""
    g, _, _ = golden()
    assert (g["enc_a_out_lengths"] - 1 < g["enc_a_lengths"]).mean() > 0.8


def _random_case(rng, alphabet=12, n_merges=200):
    merges, nid = [], 261
    for _ in range(n_merges):
        pick = lambda: int(rng.integers(5, 5 + alphabet)) if rng.random() < 0.6 or nid == 261 \
            else int(rng.integers(261, nid))  # noqa: E731
        merges.append((pick(), pick(), nid))
        nid += 1
    if merges:
        f, s, _ = merges[int(rng.integers(len(merges)))]
        merges.append((f, s, nid))          # repeated pair: never fires
    return merges


@pytest.mark.skipif(oracle.reftok_lib() is None, reason="reference tokenizer kernels not built here")
def test_oracle_encode_matches_reference_kernels_live():
    rng = np.random.default_rng(4)
    from rbk.tokenizer import pack_strings
    for _ in range(60):
        merges = _random_case(rng, n_merges=int(rng.integers(0, 300)))
        ms = int(rng.integers(3, 300))
        strs = [bytes(rng.integers(0, 12, size=int(rng.integers(1, min(256, ms - 2) + 1))).astype(np.uint8))
                for _ in range(int(rng.integers(1, 6)))]
        data, offs, lens = pack_strings(strs)
        rows, rl, _ = oracle.bpe_encode(merges, data, offs, lens, ms)
        rr, rrl = oracle.ref_bpe_encode(merges, data, offs, lens, ms)
        assert np.array_equal(rl, rrl)
        for b, n in enumerate(rl):
            assert np.array_equal(rows[b, :n], rr[b, :n])


def test_oracle_contract_outside_reference_domain():
    merges = [(5 + ord("a"), 5 + ord("a"), 300)]
    # empty -> [EOS]; exactly max_seq_len - 1 bytes merges; longer is cut and counted
    strs = [b"", b"aaaa", b"aaaaaaa", b"aaaaaaaaaaa"]
    from rbk.tokenizer import pack_strings
    data, offs, lens = pack_strings(strs)
    rows, rl, cut = oracle.bpe_encode(merges, data, offs, lens, 8)
    assert cut == 1
    assert rl.tolist() == [1, 3, 5, 5]
    assert rows[0].tolist() == [3, 0, 0, 0, 0, 0, 0, 0]
    assert rows[1].tolist() == [300, 300, 3, 0, 0, 0, 0, 0]
    assert rows[2].tolist() == [300, 300, 300, 5 + ord("a"), 3, 0, 0, 0]
    assert rows[3].tolist() == rows[2].tolist()  # the first 7 bytes
    # decode: an id outside the vocabulary adds nothing and is counted
    vocab = [b"<pad>", b"<unk>", b"<bos>", b"<eos>", b"<sep>"] + [bytes([c]) for c in range(256)]
    toks = np.array([[5 + ord("h"), 999, -4, 5 + ord("i"), 3, 5 + ord("x")]], np.int32)
    out, bad = oracle.bpe_decode(vocab, toks, 6, np.array([6], np.int32), 16)
    assert bad == 2 and out[0, :3].tobytes() == b"hi\0"


def test_oracle_decode_skips_tokens_that_do_not_fit():
    vocab = [b"<pad>", b"<unk>", b"<bos>", b"<eos>", b"<sep>"] + [bytes([c]) for c in range(256)] + [b"long!"]
    L = len(vocab) - 1
    toks = np.array([[5 + ord("a"), L, 5 + ord("b"), L, 5 + ord("c")]], np.int32)
    out, _ = oracle.bpe_decode(vocab, toks, 5, np.array([5], np.int32), 9)
    # "a" + "long!" = 6 bytes; "b" -> 7; "long!" would need 12 >= 9: skipped; "c" -> 8 < 9
    assert out[0].tobytes()[:9] == b"along!bc\0"
