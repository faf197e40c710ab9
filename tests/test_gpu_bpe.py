"""The CUDA tokenizer (rbk_bpe_*) against the reference's golden vectors and the oracle.

Small cases compare rows and strings with the oracle exactly; the GPT-2-sized synthetic
tokenizer (50257 ids) runs at full row width (2048) with its round trip
decode(encode(s)) == s, the oracle on a sample of rows, and bit-for-bit repeatability.
Every row-width instance of the encode kernel (max_seq_len 2 .. 8193) is exercised."""
import os
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "rubidium-train_b200"))

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

import oracle  # noqa: E402
from test_oracle_bpe import _random_case, golden  # noqa: E402


@pytest.fixture(scope="module")
def tk():
    from rbk.tokenizer import GPUTokenizer
    _, vocab, merges = golden()
    t = GPUTokenizer(vocab, merges)
    yield t, vocab, merges
    t.close()


@pytest.fixture(scope="module")
def big():
    from rbk.tokenizer import GPUTokenizer, synthetic_corpus, synthetic_tables
    vocab, merges, words = synthetic_tables()
    t = GPUTokenizer(vocab, merges)
    corpus = synthetic_corpus(words, 1 << 23, seed=9)
    yield t, vocab, merges, corpus
    t.close()


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def encode_dev(t, data, offs, lens, ms, truncated=None):
    rows, rl = t.encode(dev(data if len(data) else np.zeros(1, np.uint8)), dev(offs), dev(lens), ms,
                        truncated=truncated)
    torch.cuda.synchronize()
    return rows.cpu().numpy(), rl.cpu().numpy()


@pytest.mark.parametrize("tag", ["a", "b"])
def test_encode_matches_reference_golden(tk, tag):
    t, _, _ = tk
    g, _, _ = golden()
    ms = int(g[f"enc_{tag}_max_seq_len"])
    rows, rl = encode_dev(t, g[f"enc_{tag}_data"], g[f"enc_{tag}_offsets"], g[f"enc_{tag}_lengths"], ms)
    assert np.array_equal(rl, g[f"enc_{tag}_out_lengths"])
    want = g[f"enc_{tag}_rows"]
    for b, n in enumerate(rl):
        assert np.array_equal(rows[b, :n], want[b, :n]), b
        assert (rows[b, n:] == 0).all()
    # the host-string entry (encode_batch) gives the same rows
    d, o, L = g[f"enc_{tag}_data"], g[f"enc_{tag}_offsets"], g[f"enc_{tag}_lengths"]
    strs = [d[a:a + n].tobytes() for a, n in zip(o, L)]
    if all(b"\0" not in s for s in strs):
        hr, hl = t.encode_batch(strs, ms)
        torch.cuda.synchronize()
        assert np.array_equal(hl.cpu().numpy(), rl) and np.array_equal(hr.cpu().numpy(), rows)


@pytest.mark.parametrize("tag", ["a", "b", "c"])
def test_decode_matches_reference_golden(tk, tag):
    t, _, _ = tk
    g, _, _ = golden()
    msl = int(g[f"dec_{tag}_max_string_len"])
    flat, lens = g["dec_tokens_ref_layout"], g["dec_lengths"]
    out = t.decode_batch(dev(flat), dev(lens), msl, ld=0)   # the reference's addressing
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), g[f"dec_{tag}_out"])


@pytest.mark.parametrize("ms", [2, 3, 5, 257, 258, 513, 1025, 2048, 4097, 8193])
def test_encode_every_row_width_matches_oracle(tk, ms):
    """Each items-per-thread instance, with strings of 0 .. max_seq_len - 1 bytes."""
    t, _, merges = tk
    from rbk.tokenizer import pack_strings
    g, _, _ = golden()
    corpus = g["enc_a_data"].tobytes() * 8
    rng = np.random.default_rng(ms)
    Ls = sorted({0, 1, ms - 1, max(ms - 2, 0), *rng.integers(0, ms, size=6).tolist()})
    strs = [corpus[(7 * i) % 1000:(7 * i) % 1000 + L] if L <= len(corpus) - 1000 else
            bytes(rng.integers(32, 127, size=L).astype(np.uint8)) for i, L in enumerate(Ls)]
    data, offs, lens = pack_strings(strs)
    want, wl, _ = oracle.bpe_encode(merges, data, offs, lens, ms)
    rows, rl = encode_dev(t, data, offs, lens, ms)
    assert np.array_equal(rl, wl)
    assert np.array_equal(rows, want)


def test_random_rule_sets_match_oracle():
    """Dense rule sets over a 12-byte alphabet (long merge chains, repeated pairs, rules
    on later results), ragged strings up to 1500 bytes, many passes."""
    from rbk.tokenizer import GPUTokenizer, pack_strings
    rng = np.random.default_rng(21)
    vocab = [b"<pad>", b"<unk>", b"<bos>", b"<eos>", b"<sep>"] + [bytes([c]) for c in range(256)]
    for it in range(12):
        merges = _random_case(rng, n_merges=int(rng.integers(1, 2000)))
        v = vocab + [b"x"] * (max(m[2] for m in merges) + 1 - len(vocab))
        t = GPUTokenizer(v, merges)
        strs = [bytes(rng.integers(0, 12, size=int(rng.integers(0, 1500))).astype(np.uint8)) for _ in range(40)]
        data, offs, lens = pack_strings(strs)
        want, wl, _ = oracle.bpe_encode(merges, data, offs, lens, 2048)
        rows, rl = encode_dev(t, data, offs, lens, 2048)
        t.close()
        assert np.array_equal(rl, wl), it
        assert np.array_equal(rows, want), it


def test_wide_pair_table_matches_oracle(tk):
    """Vocabularies above 65535 ids use the 16-byte pair slots: the golden tokenizer with every
    merged id moved up by 65000 encodes to the same rows, ids moved likewise."""
    from rbk.tokenizer import GPUTokenizer, pack_strings
    _, vocab, merges = tk
    sh = lambda i: i + 65000 if i >= 261 else i  # noqa: E731
    wide_vocab = vocab[:261] + [b"?"] * 65000 + vocab[261:]
    wide_merges = [(sh(a), sh(b), sh(r)) for a, b, r in merges]
    t = GPUTokenizer(wide_vocab, wide_merges)
    g, _, _ = golden()
    corpus = g["enc_a_data"].tobytes()
    strs = [corpus[i:i + L] for i, L in zip(range(0, 4000, 97), range(1, 2000, 47))]
    data, offs, lens = pack_strings(strs)
    rows, rl = encode_dev(t, data, offs, lens, 2048)
    nrows, nrl = encode_dev(tk[0], data, offs, lens, 2048)
    want, wl, _ = oracle.bpe_encode(wide_merges, data, offs, lens, 2048)
    t.close()
    assert np.array_equal(rl, wl) and np.array_equal(rows, want)
    assert np.array_equal(rl, nrl) and np.array_equal(rows, np.where(nrows >= 261, nrows + 65000, nrows))


def test_truncation_and_rejection(tk):
    from rbk._lib import RbkError
    from rbk.tokenizer import pack_strings
    t, _, merges = tk
    strs = [b" the cat" * 40, b"ab", b"x" * 64]
    data, offs, lens = pack_strings(strs)
    cut = torch.zeros(1, dtype=torch.int32, device="cuda")
    rows, rl = encode_dev(t, data, offs, lens, 64, truncated=cut)
    want, wl, wcut = oracle.bpe_encode(merges, data, offs, lens, 64)
    assert int(cut.item()) == wcut == 2
    assert np.array_equal(rows, want) and np.array_equal(rl, wl)
    with pytest.raises(RbkError):
        t.encode_batch(strs, 64)          # host strings longer than max_seq_len - 1: rejected
    with pytest.raises(RbkError):
        t.encode_batch([b"a"], 8194)      # above the largest row width


def test_decode_contract_matches_oracle(tk):
    """Explicit strides, rows clamped to ld, stops, other specials, ids outside the
    vocabulary (counted), and rows too narrow for their strings (skip and continue)."""
    t, vocab, _ = tk
    rng = np.random.default_rng(3)
    V = len(vocab)
    B, ld = 300, 96
    toks = rng.integers(5, V, size=(B, ld)).astype(np.int32)
    for b in range(B):
        r = rng.random()
        if r < 0.3:
            toks[b, int(rng.integers(ld))] = int(rng.choice([0, 3]))
        elif r < 0.4:
            toks[b, int(rng.integers(ld))] = int(rng.choice([-1, V, V + 77]))
        if rng.random() < 0.2:
            toks[b, int(rng.integers(ld))] = int(rng.choice([1, 2, 4]))
    lens = rng.integers(0, ld + 20, size=B).astype(np.int32)   # some beyond ld: clamped
    for msl in (1, 2, 9, 64, 700):
        init = rng.integers(0, 256, size=(B, msl)).astype(np.uint8)
        want, wbad = oracle.bpe_decode(vocab, toks, ld, lens, msl, out=init)
        bad = torch.zeros(1, dtype=torch.int32, device="cuda")
        got = t.decode_batch(dev(toks), dev(lens), msl, ld=ld, out=dev(init), bad=bad)
        torch.cuda.synchronize()
        assert np.array_equal(got.cpu().numpy(), want), msl
        assert int(bad.item()) == wbad


def test_full_size_round_trip_and_oracle_sample(big):
    """GPT-2-sized synthetic tokenizer, 1024 strings of 2047 bytes at max_seq_len 2048:
    decode(encode(s)) == s for every string, rows equal to the oracle on a sample, and
    repeated runs identical bit for bit."""
    from rbk.tokenizer import pack_strings, strings_from_rows, synthetic_batch
    t, vocab, merges, corpus = big
    strs = synthetic_batch(corpus, 1024, 2047, seed=4)
    data, offs, lens = pack_strings(strs)
    rows, rl = encode_dev(t, data, offs, lens, 2048)
    rows2, rl2 = encode_dev(t, data, offs, lens, 2048)
    assert np.array_equal(rows, rows2) and np.array_equal(rl, rl2)
    assert (rl < 1200).all()                     # the text merged
    out = t.decode_batch(dev(rows), dev(rl), 4096)
    torch.cuda.synchronize()
    assert strings_from_rows(out.cpu().numpy()) == strs
    sample = np.arange(0, 1024, 37)
    sd, so, sl = pack_strings([strs[i] for i in sample])
    want, wl, _ = oracle.bpe_encode(merges, sd, so, sl, 2048)
    assert np.array_equal(rl[sample], wl) and np.array_equal(rows[sample], want)


def test_host_string_entry_in_parts_matches_device_entry(big):
    """A host-string batch large enough (4200 strings, 8.6 MB) to be staged and encoded in four
    parts, the text of part p + 1 packed while part p is copied and encoded: rows and lengths
    equal the device entry's, and a reused pointer array gives the same again."""
    from rbk.tokenizer import host_strings, pack_strings, synthetic_batch
    t, _, _, corpus = big
    strs = synthetic_batch(corpus, 4200, 2047, seed=5)
    strs[7] = b""
    strs[3000] = strs[3000][:5]
    data, offs, lens = pack_strings(strs)
    assert data.size >= 8 << 20           # the size at which the entry stages in parts
    want, wl = encode_dev(t, data, offs, lens, 2048)
    arr = host_strings(strs)
    for _ in range(2):
        rows, rl = t.encode_batch(arr, 2048)
        torch.cuda.synchronize()
        assert np.array_equal(rl.cpu().numpy(), wl) and np.array_equal(rows.cpu().numpy(), want)


def test_encode_string_decode_tokens(big):
    """The single-string helpers (encode_string / decode_tokens, tokenizer_cuda.cu:350-389)."""
    t, _, _, corpus = big
    s = corpus[1000:1600]
    ids = t.encode_string(s)
    assert ids[-1] == 3 and len(ids) < 600
    assert t.decode_tokens(ids) == s.decode(errors="replace")
