"""CPU oracle for the rubidium-train training step — TEST INFRASTRUCTURE ONLY.

Python face of ``oracle/liboracle.so`` (the FP32 restatement in oracle.cpp)
and of ``oracle/_ref/libref.so`` (the reference's own CPU engine, compiled from
its sources by ``make -C oracle ref``).  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` import this
module; the CUDA product path never does.

Every function takes and returns float32 numpy arrays (int32 for indices).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None
_REF = None

F = C.POINTER(C.c_float)
I = C.POINTER(C.c_int)
L = C.POINTER(C.c_long)


def _p(a, ct=C.c_float):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be C-contiguous"
    return a.ctypes.data_as(C.POINTER(ct))


def build(ref: bool | None = None) -> None:
    """Compile liboracle.so, and the reference shim when RBK_REFERENCE names the reference
    project's root (the directory holding its src/)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    root = os.environ.get("RBK_REFERENCE", "")
    if ref is None:
        ref = bool(root) and os.path.isdir(os.path.join(root, "src"))
    if ref:
        subprocess.run(["make", "-s", "-C", _HERE, "ref", "REF=" + root], check=True)


def lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build(ref=False)
        _LIB = C.CDLL(path)
        _LIB.ora_ce_fwd.restype = C.c_float
        _LIB.ora_model_loss_grad.restype = C.c_float
        _LIB.ora_model_lora_grad.restype = C.c_float
        _LIB.ora_num_params.restype = C.c_long
        _LIB.ora_clip.restype = C.c_float
        _LIB.ora_adam_tail.restype = C.c_int
        _LIB.ora_scaler_update.restype = C.c_int
    return _LIB


def ref_lib():
    """The reference's own CPU engine, or None when it was not built here."""
    global _REF
    if _REF is None:
        path = os.path.join(_HERE, "_ref", "libref.so")
        if not os.path.exists(path):
            return None
        _REF = C.CDLL(path)
        _REF.ref_cross_entropy.restype = C.c_float
        _REF.ref_clip_gradients.restype = C.c_float
        _REF.ref_cpu_forward.restype = C.c_float
        for name in ("ref_time_layer_norm_backward", "ref_time_softmax_backward", "ref_time_cross_entropy_backward",
                     "ref_time_adamw_step", "ref_time_cpu_forward"):
            getattr(_REF, name).restype = C.c_double
    return _REF


def f32(a):
    return np.ascontiguousarray(a, dtype=np.float32)


def i32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


def num_threads() -> int:
    return lib().ora_num_threads()


def set_threads(n: int | None = None) -> int:
    """Use n OpenMP threads (default: every core this process may run on) and return the count.
    torchrun exports OMP_NUM_THREADS=1 to each rank; the CPU baseline sets its count explicitly."""
    if n is None:
        try:
            n = len(os.sched_getaffinity(0))
        except AttributeError:
            n = os.cpu_count() or 1
    lib().ora_set_threads(int(n))
    return num_threads()


# ------------------------------------------------------------------ ops ----

def gemm_nt(A, B):
    """C = A @ B.T (A [M,K], B [N,K])."""
    A, B = f32(A), f32(B)
    M, K = A.shape
    N = B.shape[0]
    Cm = np.zeros((M, N), np.float32)
    lib().ora_gemm(M, N, K, _p(A), K, 0, _p(B), K, 1, _p(Cm), N, C.c_float(0.0))
    return Cm


def ln_fwd(x, g, b, eps=1e-5):
    x, g, b = f32(x), f32(g), f32(b)
    N, D = x.shape
    y = np.empty_like(x); mean = np.empty(N, np.float32); rstd = np.empty(N, np.float32)
    lib().ora_ln_fwd(_p(y), _p(mean), _p(rstd), _p(x), _p(g), _p(b), N, D, C.c_float(eps))
    return y, mean, rstd


def ln_bwd(dy, x, g, mean, rstd, dres=None, ref_formula=False):
    """Returns (dx, dgamma, dbeta); dx includes dres when given.  ref_formula
    selects the reference's dx expression (src/cpu_mat.h:146), which lacks one
    rstd factor on the x-hat term; the default is the exact gradient."""
    dy, x, g, mean, rstd = f32(dy), f32(x), f32(g), f32(mean), f32(rstd)
    N, D = x.shape
    dx = np.empty_like(x); dg = np.zeros(D, np.float32); db = np.zeros(D, np.float32)
    dres = None if dres is None else f32(dres)
    lib().ora_ln_bwd(_p(dx), _p(dg), _p(db), _p(dy), _p(dres), _p(x), _p(g), _p(mean), _p(rstd), N, D,
                     int(ref_formula))
    return dx, dg, db


def softmax_bwd(dy, y):
    dy, y = f32(dy), f32(y)
    N, Cc = y.shape
    dx = np.empty_like(y)
    lib().ora_softmax_bwd(_p(dx), _p(dy), _p(y), N, Cc)
    return dx


def causal_softmax_bwd(dy, y):
    """dy, y: [nmat, T, T]; lower triangle used, strict upper triangle of dx = 0."""
    dy, y = f32(dy), f32(y)
    nmat, T, _ = y.shape
    dx = np.empty_like(y)
    lib().ora_causal_softmax_bwd(_p(dx), _p(dy), _p(y), nmat, T)
    return dx


def ce_fwd(logits, tgt):
    """Returns (mean loss, per-row loss, per-row log-sum-exp)."""
    logits, tgt = f32(logits), i32(tgt)
    N, V = logits.shape
    rl = np.empty(N, np.float32); lse = np.empty(N, np.float32)
    loss = lib().ora_ce_fwd(_p(logits), _p(tgt, C.c_int), N, V, _p(rl), _p(lse))
    return float(loss), rl, lse


def ce_bwd(logits, tgt, scale=1.0):
    logits, tgt = f32(logits), i32(tgt)
    N, V = logits.shape
    d = np.empty_like(logits)
    lib().ora_ce_bwd(_p(d), _p(logits), _p(tgt, C.c_int), N, V, C.c_float(scale))
    return d


def embed_bwd(dout, idx, V):
    dout, idx = f32(dout), i32(idx)
    T, D = dout.shape
    dW = np.zeros((V, D), np.float32)
    lib().ora_embed_bwd(_p(dW), _p(dout), _p(idx, C.c_int), T, D)
    return dW


def adamw(p, g, m, v, lr, b1, b2, eps, wd, t):
    p, g, m, v = f32(p).copy(), f32(g), f32(m).copy(), f32(v).copy()
    lib().ora_adamw(_p(p), _p(g), _p(m), _p(v), C.c_long(p.size), C.c_float(lr), C.c_float(b1),
                    C.c_float(b2), C.c_float(eps), C.c_float(wd), C.c_int(t))
    return p, m, v


def clip(g, max_norm):
    g = f32(g).copy()
    n = lib().ora_clip(_p(g), C.c_long(g.size), C.c_float(max_norm))
    return g, float(n)


class Scaler(C.Structure):
    """Dynamic loss-scaler state (src/cuda_kernels.cuh:62-73)."""
    _fields_ = [("scale", C.c_float), ("unskipped", C.c_int), ("interval", C.c_int)]


def scaler_update(s: Scaler, overflow: bool) -> int:
    return lib().ora_scaler_update(C.byref(s), int(bool(overflow)))


def adam_tail(p, g, m, v, seg_off, seg_len, lr, b1, b2, eps, wd, t, scaler: Scaler, max_norm=0.0):
    """Fused tail restated on the CPU; arrays are updated in place. Returns skip flag."""
    so = np.ascontiguousarray(seg_off, dtype=np.int64)
    sl = np.ascontiguousarray(seg_len, dtype=np.int64)
    return lib().ora_adam_tail(_p(p), _p(g), _p(m), _p(v), C.c_long(p.size), _p(so, C.c_long), _p(sl, C.c_long),
                               len(so), C.c_float(lr), C.c_float(b1), C.c_float(b2), C.c_float(eps),
                               C.c_float(wd), C.c_int(t), C.byref(scaler), C.c_float(max_norm))


def act_fwd(x, relu=False):
    x = f32(x); y = np.empty_like(x)
    lib().ora_act_fwd(_p(y), _p(x), C.c_long(x.size), int(relu))
    return y


def act_grad(x, relu=False):
    x = f32(x); y = np.empty_like(x)
    lib().ora_act_grad(_p(y), _p(x), C.c_long(x.size), int(relu))
    return y


def attn_fwd(q, k, v, B, S, H):
    """q, k, v: [B*S, D] -> (o [B*S, D], P [B, H, S, S])."""
    q, k, v = f32(q), f32(k), f32(v)
    D = q.shape[1]
    qkv = np.concatenate([q, k, v], axis=1).copy()
    o = np.empty((B * S, D), np.float32)
    P = np.empty((B, H, S, S), np.float32)
    lib().ora_attn_fwd(_p(o), _p(P), _p(qkv), C.cast(qkv.ctypes.data + 4 * D, F),
                       C.cast(qkv.ctypes.data + 8 * D, F), 3 * D, D, B, S, H, D // H)
    return o, P


def attn_bwd(do, P, q, k, v, B, S, H):
    do, P = f32(do), f32(P)
    D = q.shape[1]
    qkv = np.concatenate([f32(q), f32(k), f32(v)], axis=1).copy()
    d = np.empty_like(qkv)
    base, dbase = qkv.ctypes.data, d.ctypes.data
    lib().ora_attn_bwd(C.cast(dbase, F), C.cast(dbase + 4 * D, F), C.cast(dbase + 8 * D, F), _p(do), _p(P),
                       C.cast(base, F), C.cast(base + 4 * D, F), C.cast(base + 8 * D, F), 3 * D, D, B, S, H,
                       D // H)
    return d[:, :D].copy(), d[:, D:2 * D].copy(), d[:, 2 * D:].copy()


# ---------------------------------------------------------------- model ----

LAYER_NAMES = ["ln1_w", "ln1_b", "wq", "wk", "wv", "bq", "bk", "bv", "wo", "bo",
               "ln2_w", "ln2_b", "w1", "b1", "w2", "b2"]


def cfg6(cfg):
    return np.array([cfg["V"], cfg["T"], cfg["D"], cfg["H"], cfg["L"], cfg["FF"]], np.int32)


def param_table(cfg):
    """[(name, offset, rows, cols)] in arena order (include/rbk_layout.h)."""
    c6 = cfg6(cfg)
    n = 2 + 16 * cfg["L"] + 4
    buf = np.zeros(3 * n, np.int64)
    lib().ora_param_table(_p(c6, C.c_int), _p(buf, C.c_long))
    names = ["token_emb", "pos_emb"]
    for l in range(cfg["L"]):
        names += [f"layers.{l}.{s}" for s in LAYER_NAMES]
    names += ["ln_f_w", "ln_f_b", "lm_w", "lm_b"]
    return [(names[i], int(buf[3 * i]), int(buf[3 * i + 1]), int(buf[3 * i + 2])) for i in range(n)]


def num_params(cfg) -> int:
    return int(lib().ora_num_params(_p(cfg6(cfg), C.c_int)))


def init_params(cfg, seed=42, std=0.02):
    """Seeded init per src/model.cu:146-183: N(0, std) matrices and embeddings,
    LN gamma = 1, beta = 0, biases 0.  (numpy PCG64, not mt19937: the stream is
    the build's own, the distribution is the reference's.)"""
    rng = np.random.default_rng(seed)
    p = np.zeros(num_params(cfg), np.float32)
    for name, off, r, c in param_table(cfg):
        base = name.split(".")[-1]
        if base in ("ln1_w", "ln2_w", "ln_f_w"):
            p[off:off + r * c] = 1.0
        elif base in ("token_emb", "pos_emb", "wq", "wk", "wv", "wo", "w1", "w2", "lm_w"):
            p[off:off + r * c] = rng.standard_normal(r * c, dtype=np.float32) * std
    return p


def model_loss_grad(cfg, params, tok, tgt, B, S, grad_scale=1.0, relu=False, want_grads=True, want_logits=False):
    params = f32(params)
    tok, tgt = i32(tok), i32(tgt)
    grads = np.zeros_like(params) if want_grads else None
    logits = np.empty((B * S, cfg["V"]), np.float32) if want_logits else None
    loss = lib().ora_model_loss_grad(_p(cfg6(cfg), C.c_int), _p(params), _p(grads), _p(tok, C.c_int),
                                     _p(tgt, C.c_int), B, S, C.c_float(grad_scale), int(relu), _p(logits))
    return float(loss), grads, logits


def model_lora_grad(cfg, params, Aq, Bq, Av, Bv, r, alpha, tok, tgt, B, S, grad_scale=1.0):
    params = f32(params)
    Aq, Bq, Av, Bv = f32(Aq), f32(Bq), f32(Av), f32(Bv)
    dAq, dBq, dAv, dBv = (np.zeros_like(a) for a in (Aq, Bq, Av, Bv))
    loss = lib().ora_model_lora_grad(_p(cfg6(cfg), C.c_int), _p(params), _p(Aq), _p(Bq), _p(Av), _p(Bv),
                                     _p(dAq), _p(dBq), _p(dAv), _p(dBv), r, C.c_float(alpha),
                                     _p(i32(tok), C.c_int), _p(i32(tgt), C.c_int), B, S, C.c_float(grad_scale))
    return float(loss), dAq, dBq, dAv, dBv


# ---------------------------------------------------------------------------
# BPE tokenizer (oracle/bpe.cpp; the reference's kernels in _ref/libreftok.so)
# ---------------------------------------------------------------------------
_REFTOK = None


def _merge_cols(merges):
    m = np.ascontiguousarray(np.asarray(merges, dtype=np.int32).reshape(-1, 3))
    return [np.ascontiguousarray(m[:, i]) for i in range(3)]


def bpe_encode(merges, data, offsets, lengths, max_seq_len):
    """Restated encode: (int32 [B, max_seq_len] rows, int32 [B] lengths, truncated count)."""
    mf, ms, mr = _merge_cols(merges)
    data = np.ascontiguousarray(data, np.uint8)
    offsets = np.ascontiguousarray(offsets, np.int64)
    lengths = np.ascontiguousarray(lengths, np.int32)
    B = lengths.size
    out = np.empty((B, max_seq_len), np.int32)
    out_len = np.empty(B, np.int32)
    cut = C.c_int(0)
    rc = lib().ora_bpe_encode(_p(mf, C.c_int), _p(ms, C.c_int), _p(mr, C.c_int), len(mf),
                              data.ctypes.data_as(C.c_void_p), _p(offsets, C.c_int64), _p(lengths, C.c_int), B,
                              _p(out, C.c_int), _p(out_len, C.c_int), max_seq_len, C.byref(cut))
    assert rc == 0, "ora_bpe_encode rejected its arguments"
    return out, out_len, cut.value


def bpe_decode(vocab, tokens, ld, lengths, max_string_len, out=None):
    """Restated decode: (uint8 [B, max_string_len] rows, bad-id count).  `out` (optional) is the
    initial buffer content (bytes after each NUL are left as they are)."""
    inv = b"".join(vocab)
    offs = np.zeros(len(vocab), np.int64)
    lens = np.array([len(s) for s in vocab], np.int32)
    offs[1:] = np.cumsum(lens[:-1])
    tokens = np.ascontiguousarray(tokens, np.int32)
    lengths = np.ascontiguousarray(lengths, np.int32)
    B = lengths.size
    out = np.zeros((B, max_string_len), np.uint8) if out is None else np.ascontiguousarray(out, np.uint8).copy()
    bad = C.c_int(0)
    invb = np.frombuffer(inv, np.uint8) if inv else np.zeros(1, np.uint8)
    rc = lib().ora_bpe_decode(invb.ctypes.data_as(C.c_void_p), _p(offs, C.c_int64), _p(lens, C.c_int), len(vocab),
                              _p(tokens, C.c_int), C.c_int64(ld), _p(lengths, C.c_int), B,
                              out.ctypes.data_as(C.c_void_p), max_string_len, C.byref(bad))
    assert rc == 0, "ora_bpe_decode rejected its arguments"
    return out, bad.value


def reftok_lib():
    """The reference's tokenizer kernels compiled for the CPU, or None when not built here."""
    global _REFTOK
    if _REFTOK is None:
        path = os.path.join(_HERE, "_ref", "libreftok.so")
        if not os.path.exists(path):
            return None
        _REFTOK = C.CDLL(path)
        _REFTOK.reftok_time_encode.restype = C.c_double
    return _REFTOK


def ref_bpe_encode(merges, data, offsets, lengths, max_seq_len, fill=-7):
    """The reference's encode_kernel (strings of 1..256 bytes, at most max_seq_len - 2):
    (rows as the kernel leaves them, starting from `fill`, and lengths), or None outside
    its defined domain."""
    mf, ms, mr = _merge_cols(merges)
    data = np.ascontiguousarray(data, np.uint8)
    offs32 = np.ascontiguousarray(offsets, np.int32)
    lengths = np.ascontiguousarray(lengths, np.int32)
    B = lengths.size
    out = np.full((B, max_seq_len), fill, np.int32)
    out_len = np.full(B, fill, np.int32)
    rc = reftok_lib().reftok_encode(_p(mf, C.c_int), _p(ms, C.c_int), _p(mr, C.c_int), len(mf),
                                    data.ctypes.data_as(C.c_void_p), _p(offs32, C.c_int), _p(lengths, C.c_int), B,
                                    _p(out, C.c_int), _p(out_len, C.c_int), max_seq_len)
    return None if rc != 0 else (out, out_len)


def ref_bpe_decode(vocab, tokens_ref_layout, lengths, max_string_len, out=None):
    """The reference's decode_kernel; row b at b * lengths[b] of the flat token array."""
    inv = b"".join(vocab)
    lens = np.array([len(s) for s in vocab], np.int32)
    offs = np.zeros(len(vocab), np.int32)
    offs[1:] = np.cumsum(lens[:-1])
    tokens = np.ascontiguousarray(tokens_ref_layout, np.int32)
    lengths = np.ascontiguousarray(lengths, np.int32)
    B = lengths.size
    out = np.zeros((B, max_string_len), np.uint8) if out is None else np.ascontiguousarray(out, np.uint8).copy()
    invb = np.frombuffer(inv, np.uint8) if inv else np.zeros(1, np.uint8)
    rc = reftok_lib().reftok_decode(invb.ctypes.data_as(C.c_void_p), _p(offs, C.c_int), _p(lens, C.c_int),
                                    len(vocab), _p(tokens, C.c_int), _p(lengths, C.c_int), B,
                                    out.ctypes.data_as(C.c_void_p), max_string_len)
    return None if rc != 0 else out


def ref_bpe_time_encode(merges, data, offsets, lengths, max_seq_len, reps=1):
    """Seconds the reference's encode algorithm takes for `reps` passes over the batch."""
    mf, ms, mr = _merge_cols(merges)
    data = np.ascontiguousarray(data, np.uint8)
    offs32 = np.ascontiguousarray(offsets, np.int32)
    lengths = np.ascontiguousarray(lengths, np.int32)
    B = lengths.size
    out = np.empty((B, max_seq_len), np.int32)
    out_len = np.empty(B, np.int32)
    return reftok_lib().reftok_time_encode(_p(mf, C.c_int), _p(ms, C.c_int), _p(mr, C.c_int), len(mf),
                                           data.ctypes.data_as(C.c_void_p), _p(offs32, C.c_int),
                                           _p(lengths, C.c_int), B, _p(out, C.c_int), _p(out_len, C.c_int),
                                           max_seq_len, reps)
