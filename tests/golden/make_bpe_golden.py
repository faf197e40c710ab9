"""Generate golden vectors for the BPE tokenizer from the reference's own kernels.

Runs the reference's encode_kernel and decode_kernel (src/tokenizer_cuda.cu:90-203),
compiled for the CPU by ``make -C oracle ref`` into oracle/_ref/libreftok.so, on a small
seeded tokenizer and seeded strings, and stores tables, inputs and outputs in
tests/golden/bpe_ref.npz.  The tests compare the oracle restatement and the CUDA
tokenizer against these vectors, so the pin holds where the reference tree is absent.

Cases stay inside the reference's defined domain: strings of 1..256 bytes and at most
max_seq_len - 2 (one block of 256 threads per string), token ids inside the vocabulary.
Row entries past each length are stored as -1 (the reference leaves pass scratch there).

Usage:  python tests/golden/make_bpe_golden.py     (needs oracle/_ref/libreftok.so)
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "rubidium-train_b200"))

import oracle  # noqa: E402
from rbk.tokenizer import pack_strings, synthetic_corpus, synthetic_tables  # noqa: E402


def main():
    if oracle.reftok_lib() is None:
        raise SystemExit("oracle/_ref/libreftok.so is missing: make -C oracle ref REF=<reference root>")
    rng = np.random.default_rng(11)
    vocab, merges, words = synthetic_tables(n_merges=1500, n_words=600, seed=5)
    # a repeated pair (the later rule must never fire) and a rule on ids no token carries
    merges = list(merges)
    f, s, _ = merges[10]
    vocab.append(b"#dup")
    merges.append((f, s, len(vocab) - 1))
    corpus = synthetic_corpus(words, 1 << 16, seed=6)
    out = {"vocab_lengths": np.array([len(v) for v in vocab], np.int32),
           "vocab_bytes": np.frombuffer(b"".join(vocab), np.uint8),
           "merges": np.array(merges, np.int32)}
    # encode: ragged corpus strings, some raw random bytes (incl. >= 0x80), two row widths
    for tag, ms in (("a", 300), ("b", 64)):
        strs = []
        for i in range(48):
            L = int(rng.integers(1, min(256, ms - 2) + 1))
            if i % 8 == 7:
                strs.append(bytes(rng.integers(0, 256, size=L).astype(np.uint8)))
            else:
                st = int(rng.integers(0, len(corpus) - L))
                strs.append(corpus[st:st + L])
        strs.append(b"a")
        strs.append(b" " * min(256, ms - 2))
        data, offs, lens = pack_strings(strs)
        res = oracle.ref_bpe_encode(merges, data, offs, lens, ms)
        assert res is not None
        rows, rl = res
        mask = np.arange(ms)[None, :] >= rl[:, None]
        rows = np.where(mask, -1, rows)
        out[f"enc_{tag}_data"], out[f"enc_{tag}_offsets"], out[f"enc_{tag}_lengths"] = data, offs, lens
        out[f"enc_{tag}_max_seq_len"] = np.array(ms, np.int32)
        out[f"enc_{tag}_rows"], out[f"enc_{tag}_out_lengths"] = rows, rl
    # decode: the encoded rows of case a (with their EOS), rows with PAD / EOS inside, the
    # other specials, and row widths that force the skip-and-continue rule
    rows_a, len_a = out["enc_a_rows"], out["enc_a_out_lengths"]
    V = len(vocab)
    seqs = [rows_a[b, :len_a[b]] for b in range(len(len_a))]
    for _ in range(16):
        n = int(rng.integers(1, 60))
        t = rng.integers(5, V, size=n).astype(np.int32)
        if rng.random() < 0.5:
            t[int(rng.integers(n))] = int(rng.choice([0, 3]))
        if rng.random() < 0.5:
            t[int(rng.integers(n))] = int(rng.choice([1, 2, 4]))
        seqs.append(t)
    lengths = np.array([len(q) for q in seqs], np.int32)
    flat = np.zeros(int(sum(b * int(L) for b, L in enumerate(lengths)) + lengths.max() + 1), np.int32)
    for b, q in enumerate(seqs):
        flat[b * lengths[b]:b * lengths[b] + lengths[b]] = q
    for tag, msl in (("a", 1024), ("b", 24), ("c", 7)):
        res = oracle.ref_bpe_decode(vocab, flat, lengths, msl)
        assert res is not None
        out[f"dec_{tag}_max_string_len"] = np.array(msl, np.int32)
        out[f"dec_{tag}_out"] = res
    out["dec_tokens_ref_layout"], out["dec_lengths"] = flat, lengths
    np.savez_compressed(os.path.join(HERE, "bpe_ref.npz"), **out)
    print("wrote bpe_ref.npz:", {k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main()
