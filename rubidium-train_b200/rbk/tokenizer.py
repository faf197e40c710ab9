"""GPU BPE tokenizer — the Python face of librbk's rbk_bpe_* entry points, with the
reference's host API names (src/tokenizer_cuda.h:120-164):

    tok = GPUTokenizer(vocab, merges)            # tokenizer_copy_to_device
    toks, lens = tok.encode_batch(strings, 2048) # encode_batch (host strings -> device rows)
    arr = host_strings(strings)                  # the char** once, reused by later encode_batch calls
    toks, lens = tok.encode(bytes, offs, lens_in, 2048)  # the same, inputs already on the device
    out = tok.decode_batch(toks, lens, 1024)     # decode_batch (device rows -> device strings)
    ids = tok.encode_string("text")              # encode_string
    s = tok.decode_tokens(ids)                   # decode_tokens
    tok.close()                                  # tokenizer_free_gpu

`vocab` lists every id's string (bytes) in id order: the five specials, the 256 single
bytes at ids 5..260, then the merged tokens.  `merges` lists the rules in merge order as
(first_id, second_id, result_id).  There is no CPU path: every call runs librbk.

synthetic_tables / synthetic_corpus build a seeded stand-in for a trained tokenizer and
its text (no dataset or trained vocabulary is available offline): Zipf-distributed
pseudo-words whose merges follow the pass structure, so frequent words end as single
tokens after about log2(length) passes, as with a trained BPE table.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import call, lib

PAD_ID, UNK_ID, BOS_ID, EOS_ID, SEP_ID = 0, 1, 2, 3, 4
SPECIALS = (b"<pad>", b"<unk>", b"<bos>", b"<eos>", b"<sep>")
BYTE_BASE = 5
MAX_SEQ_LEN = 2048        # tokenizer_cuda.h:16
DECODE_STRING_LEN = 1024  # decode_tokens' buffer (tokenizer_cuda.cu:373)


def _vp(t):
    return C.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def pack_strings(strings):
    """A list of str/bytes -> (uint8 bytes, int64 offsets, int32 lengths) numpy arrays."""
    bs = [s.encode() if isinstance(s, str) else bytes(s) for s in strings]
    lens = np.array([len(b) for b in bs], dtype=np.int32)
    offs = np.zeros(len(bs), dtype=np.int64)
    if len(bs) > 1:
        offs[1:] = np.cumsum(lens[:-1], dtype=np.int64)
    data = np.frombuffer(b"".join(bs), dtype=np.uint8) if bs else np.zeros(0, np.uint8)
    return data, offs, lens


def vocab_arrays(vocab):
    """id strings -> (bytes, int32 offsets, int32 lengths), the inverse-vocabulary layout."""
    lens = np.array([len(s) for s in vocab], dtype=np.int32)
    offs = np.zeros(len(vocab), dtype=np.int32)
    if len(vocab) > 1:
        offs[1:] = np.cumsum(lens[:-1], dtype=np.int64).astype(np.int32)
    return b"".join(vocab), offs, lens


class GPUTokenizer:
    def __init__(self, vocab, merges, device: int | None = None):
        dev = torch.cuda.current_device() if device is None else int(device)
        inv, offs, lens = vocab_arrays(list(vocab))
        m = np.asarray(merges, dtype=np.int32).reshape(-1, 3)
        mf, ms, mr = (np.ascontiguousarray(m[:, i]) for i in range(3))
        self.vocab_size = len(offs)
        self.device = dev
        self._keep = (inv, offs, lens, mf, ms, mr)
        h = C.c_void_p()
        p = lambda a: a.ctypes.data_as(C.c_void_p)  # noqa: E731
        with torch.cuda.device(dev):
            call("rbk_bpe_create", C.byref(h), dev, self.vocab_size, C.c_char_p(inv), len(inv), p(offs), p(lens),
                 p(mf), p(ms), p(mr), len(m))
        self._h = h

    @property
    def num_rules(self) -> int:
        return lib().rbk_bpe_num_rules(self._h)

    def close(self) -> None:
        if self._h is not None and self._h.value:
            call("rbk_bpe_destroy", self._h)
        self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def encode_batch(self, strings, max_seq_len: int = MAX_SEQ_LEN, out=None, out_lengths=None):
        """Host strings -> (int32 [B, max_seq_len] rows, int32 [B] lengths) on the device.
        `strings`: a list of str/bytes, or the array host_strings() made from one (building
        that array of 16K C pointers costs Python several ms; reuse it when encoding again)."""
        arr = strings if isinstance(strings, C.Array) else host_strings(strings)
        B = len(arr) if len(arr) != 1 or arr[0] is not None else 0
        out = torch.empty(B, max_seq_len, dtype=torch.int32, device=f"cuda:{self.device}") if out is None else out
        out_lengths = torch.empty(B, dtype=torch.int32, device=out.device) if out_lengths is None else out_lengths
        call("rbk_bpe_encode_batch", self._h, arr, B, _vp(out), _vp(out_lengths), max_seq_len, _stream())
        return out, out_lengths

    def encode(self, data, offsets, lengths, max_seq_len: int = MAX_SEQ_LEN, out=None, out_lengths=None,
               truncated=None):
        """Device strings (uint8 bytes, int64 offsets, int32 lengths) -> (rows, lengths)."""
        B = lengths.numel()
        out = torch.empty(B, max_seq_len, dtype=torch.int32, device=data.device) if out is None else out
        out_lengths = torch.empty(B, dtype=torch.int32, device=data.device) if out_lengths is None else out_lengths
        call("rbk_bpe_encode", self._h, _vp(data), _vp(offsets), _vp(lengths), B, _vp(out), _vp(out_lengths),
             max_seq_len, _vp(truncated), _stream())
        return out, out_lengths

    def decode_batch(self, tokens, lengths, max_string_len: int, ld: int | None = None, out=None, bad=None):
        """Device rows -> uint8 [B, max_string_len] NUL-terminated strings on the device.
        ld: row stride in tokens (default tokens.shape[1]; 0 = the reference's b * lengths[b])."""
        B = lengths.numel()
        ld = tokens.shape[-1] if ld is None else ld
        out = torch.zeros(B, max_string_len, dtype=torch.uint8, device=tokens.device) if out is None else out
        call("rbk_bpe_decode_batch", self._h, _vp(tokens), ld, _vp(lengths), B, _vp(out), max_string_len, _vp(bad),
             _stream())
        return out

    def encode_string(self, text, max_seq_len: int = MAX_SEQ_LEN):
        toks, lens = self.encode_batch([text], max_seq_len)
        n = int(lens[0])
        return toks[0, :n].tolist()

    def decode_tokens(self, tokens) -> str:
        t = torch.tensor(list(tokens), dtype=torch.int32, device=f"cuda:{self.device}").view(1, -1)
        n = torch.tensor([t.shape[1]], dtype=torch.int32, device=t.device)
        raw = self.decode_batch(t, n, DECODE_STRING_LEN, ld=max(t.shape[1], 1)).cpu().numpy()[0].tobytes()
        return raw.split(b"\0", 1)[0].decode(errors="replace")


def host_strings(strings):
    """The char** a C caller of rbk_bpe_encode_batch holds: a ctypes array of C pointers to
    the strings (str is UTF-8 encoded; the array keeps the bytes objects alive).  An empty
    list gives a one-entry array holding NULL."""
    bs = [s if isinstance(s, bytes) else (s.encode() if isinstance(s, str) else bytes(s)) for s in strings]
    return (C.c_char_p * max(len(bs), 1))(*bs) if bs else (C.c_char_p * 1)(None)


def strings_from_rows(raw: np.ndarray):
    """uint8 [B, L] NUL-terminated rows -> list of bytes."""
    return [bytes(r).split(b"\0", 1)[0] for r in raw]


# ---------------------------------------------------------------------------
# Seeded synthetic tokenizer and text
# ---------------------------------------------------------------------------
_LETTERS = b"etaoinshrdlcumwfgypbvkjxqz"
_LETTER_P = np.array([12.7, 9.1, 8.2, 7.5, 7.0, 6.7, 6.3, 6.1, 6.0, 4.3, 4.0, 2.8, 2.8, 2.4, 2.4, 2.2, 2.0, 2.0,
                      1.9, 1.5, 1.0, 0.8, 0.2, 0.2, 0.1, 0.1])


def _pseudo_words(rng, n):
    p = _LETTER_P / _LETTER_P.sum()
    lens = np.clip(rng.geometric(0.22, size=3 * n), 1, 14)
    letters = rng.choice(np.frombuffer(_LETTERS, np.uint8), size=int(lens.sum()), p=p)
    words, seen, pos = [], set(), 0
    for L in lens:
        w = letters[pos:pos + L].tobytes()
        pos += L
        if rng.random() < 0.08:
            w = w[:1].upper() + w[1:]
        if w not in seen:
            seen.add(w)
            words.append(w)
            if len(words) == n:
                break
    return words


def synthetic_tables(n_merges: int = 49996, n_words: int = 60000, seed: int = 0):
    """(vocab list of bytes, merges list of (first, second, result)) of 261 + n_merges ids
    (the GPT-2 vocabulary size by default).  Rules build ' ' + word for the words in
    frequency order, pairing tokens left to right level by level, as a merge pass does."""
    rng = np.random.default_rng(seed)
    vocab = list(SPECIALS) + [bytes([c]) for c in range(256)]
    index = {s: i for i, s in enumerate(vocab) if i >= BYTE_BASE}
    merges = []
    words = _pseudo_words(rng, n_words)
    for w in words:
        toks = [bytes([c]) for c in b" " + w]
        while len(toks) > 1:
            nxt = []
            for i in range(0, len(toks) - 1, 2):
                s = toks[i] + toks[i + 1]
                if s not in index:
                    if len(merges) == n_merges:
                        return vocab, merges, words
                    index[s] = len(vocab)
                    vocab.append(s)
                    merges.append((index[toks[i]], index[toks[i + 1]], index[s]))
                nxt.append(s)
            if len(toks) % 2:
                nxt.append(toks[-1])
            toks = nxt
    return vocab, merges, words


def synthetic_corpus(words, n_bytes: int, seed: int = 1, zipf: float = 1.1):
    """~n_bytes of text: Zipf-sampled words, each after a space, with some punctuation,
    newlines and two-byte UTF-8 letters."""
    rng = np.random.default_rng(seed)
    n = len(words)
    p = 1.0 / np.arange(1, n + 1) ** zipf
    p /= p.sum()
    mean = sum(len(w) * q for w, q in zip(words[:2000], p[:2000])) / p[:2000].sum() + 1.2
    k = int(n_bytes / mean) + 16
    pick = rng.choice(n, size=k, p=p)
    extra = rng.random(k)
    parts = []
    for w, e in zip(pick, extra):
        parts.append(b" " + words[w])
        if e < 0.06:
            parts.append(b",")
        elif e < 0.09:
            parts.append(b".")
        elif e < 0.095:
            parts.append(b"\n")
        elif e < 0.10:
            parts.append(b" \xc3\xa9")
    return b"".join(parts)[:n_bytes]


def synthetic_batch(corpus: bytes, batch: int, length: int, seed: int = 2, ragged: bool = False):
    """`batch` strings cut from the corpus at seeded offsets, `length` bytes each (ragged:
    lengths uniform in [1, length])."""
    rng = np.random.default_rng(seed)
    lens = rng.integers(1, length + 1, size=batch) if ragged else np.full(batch, length)
    starts = rng.integers(0, len(corpus) - length, size=batch)
    return [corpus[s:s + L] for s, L in zip(starts, lens)]
