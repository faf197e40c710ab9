"""Generate golden vectors from the reference's own CPU engine.

Runs the reference's cpuops (src/cpu_mat.h) and CPUTransformer::forward
(src/cpu_model.cpp:115-222), compiled from its sources by
``make -C oracle ref`` into oracle/_ref/libref.so, on small seeded inputs and
stores inputs and outputs in tests/golden/ref_ops.npz.  The CPU tests compare
the oracle restatement against these vectors, so the pin holds on machines
that do not have the reference tree.

Usage:  python tests/golden/make_golden.py        (needs oracle/_ref/libref.so)
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

F = C.POINTER(C.c_float)
I = C.POINTER(C.c_int)


def p(a, t=C.c_float):
    return a.ctypes.data_as(C.POINTER(t))


def main():
    oracle.build(ref=True)
    ref = oracle.ref_lib()
    assert ref is not None, "reference shim not built"
    rng = np.random.default_rng(20261201)
    out = {}

    # LayerNorm forward / backward, N=24 rows, D=96.
    N, D = 24, 96
    x = rng.standard_normal((N, D), dtype=np.float32)
    g = (1.0 + 0.02 * rng.standard_normal(D)).astype(np.float32)
    b = (0.1 * rng.standard_normal(D)).astype(np.float32)
    dy = rng.standard_normal((N, D), dtype=np.float32)
    y = np.empty_like(x); mean = np.empty((N, 1), np.float32); rstd = np.empty((N, 1), np.float32)
    ref.ref_layer_norm(p(y), p(mean), p(rstd), p(x), p(g), p(b), N, D)
    dx = np.empty_like(x); dg = np.empty(D, np.float32); db = np.empty(D, np.float32)
    ref.ref_layer_norm_backward(p(dx), p(dg), p(db), p(dy), p(x), p(g), p(mean), p(rstd), N, D)
    out.update(ln_x=x, ln_g=g, ln_b=b, ln_dy=dy, ln_y=y, ln_mean=mean[:, 0], ln_rstd=rstd[:, 0],
               ln_dx=dx, ln_dg=dg, ln_db=db)

    # Softmax forward / backward, N=16 rows of 50.
    N, Cc = 16, 50
    z = (2.0 * rng.standard_normal((N, Cc))).astype(np.float32)
    sm = np.empty_like(z)
    ref.ref_softmax(p(sm), p(z), N, Cc)
    dsm = rng.standard_normal((N, Cc), dtype=np.float32)
    dz = np.empty_like(z)
    ref.ref_softmax_backward(p(dz), p(dsm), p(sm), N, Cc)
    out.update(sm_z=z, sm_y=sm, sm_dy=dsm, sm_dx=dz)

    # Cross-entropy forward / backward, N=12 rows, V=300 (logits ~ N(0, 2)).
    N, V = 12, 300
    logits = (2.0 * rng.standard_normal((N, V))).astype(np.float32)
    tgt = rng.integers(0, V, N).astype(np.int32)
    loss = ref.ref_cross_entropy(p(logits), p(tgt, C.c_int), N, V)
    dl = np.empty_like(logits)
    ref.ref_cross_entropy_backward(p(dl), p(logits), p(tgt, C.c_int), N, V)
    out.update(ce_logits=logits, ce_tgt=tgt, ce_loss=np.float32(loss), ce_dlogits=dl)

    # Embedding backward with repeated indices, T=40, D=16, V=20.
    T, D, V = 40, 16, 20
    dout = rng.standard_normal((T, D), dtype=np.float32)
    idx = rng.integers(0, V, T).astype(np.int32)
    dW = np.empty((V, D), np.float32)
    ref.ref_embedding_backward(p(dW), p(dout), p(idx, C.c_int), T, D, V)
    out.update(emb_dout=dout, emb_idx=idx, emb_dW=dW)

    # Three AdamW steps, n=257 (lr 3e-4, betas 0.9/0.999, eps 1e-8, wd 0.1).
    n = 257
    prm = (0.02 * rng.standard_normal(n)).astype(np.float32)
    m = np.zeros(n, np.float32); v = np.zeros(n, np.float32)
    grads = [(1e-2 * rng.standard_normal(n)).astype(np.float32) for _ in range(3)]
    out.update(adam_p0=prm.copy(), adam_g=np.stack(grads))
    for t in range(1, 4):
        ref.ref_adamw_step(p(prm), p(grads[t - 1]), p(m), p(v), n, C.c_float(3e-4), C.c_float(0.9),
                           C.c_float(0.999), C.c_float(1e-8), C.c_float(0.1), t)
    out.update(adam_p3=prm, adam_m3=m, adam_v3=v)

    # Clip: one tensor above max_norm, one below.
    g1 = (0.5 * rng.standard_normal(64)).astype(np.float32)
    g2 = (0.01 * rng.standard_normal(64)).astype(np.float32)
    out.update(clip_g1=g1.copy(), clip_g2=g2.copy())
    n1 = ref.ref_clip_gradients(p(g1), 64, C.c_float(1.0))
    n2 = ref.ref_clip_gradients(p(g2), 64, C.c_float(1.0))
    out.update(clip_g1_out=g1, clip_g2_out=g2, clip_norms=np.array([n1, n2], np.float32))

    # The three matmul variants, (M,K,N) = (7, 33, 11).
    M, K, Nn = 7, 33, 11
    A = rng.standard_normal((M, K), dtype=np.float32)
    Bm = rng.standard_normal((K, Nn), dtype=np.float32)
    Cm = np.empty((M, Nn), np.float32)
    ref.ref_matmul(p(Cm), p(A), p(Bm), M, K, Nn)
    Bt = np.ascontiguousarray(Bm.T)
    Ct = np.empty((M, Nn), np.float32)
    ref.ref_matmul_tB(p(Ct), p(A), p(Bt), M, K, Nn)
    At = np.ascontiguousarray(A.T)
    Ca = np.empty((M, Nn), np.float32)
    ref.ref_matmul_tA(p(Ca), p(At), p(Bm), M, K, Nn)
    out.update(mm_A=A, mm_B=Bm, mm_C=Cm, mm_C_tB=Ct, mm_C_tA=Ca)

    # Full forward loss of CPUTransformer at V == D (the only shape its LM head
    # handles), ReLU FFN, one sequence.  Weights in the oracle's [out, in]
    # arena; the reference receives them transposed to its [in, out] Mats.
    cfg = dict(V=64, T=32, D=64, H=1, L=2, FF=128)
    S = 24
    params = oracle.init_params(cfg, seed=7)
    # non-trivial LN params and biases so every term of the forward is exercised
    for name, off, r, c in oracle.param_table(cfg):
        base = name.split(".")[-1]
        if base in ("ln1_w", "ln2_w", "ln_f_w"):
            params[off:off + r * c] = 1.0 + 0.05 * rng.standard_normal(r * c)
        elif base in ("ln1_b", "ln2_b", "ln_f_b", "bq", "bk", "bv", "bo", "b1", "b2", "lm_b"):
            params[off:off + r * c] = 0.05 * rng.standard_normal(r * c)
    tok = rng.integers(0, cfg["V"], S).astype(np.int32)
    tgt = rng.integers(0, cfg["V"], S).astype(np.int32)
    tab = {name: (off, r, c) for name, off, r, c in oracle.param_table(cfg)}

    def t(name, transpose=False):
        off, r, c = tab[name]
        a = params[off:off + r * c].reshape(r, c)
        return np.ascontiguousarray(a.T if transpose else a, dtype=np.float32)

    layers = []
    for l in range(cfg["L"]):
        pre = f"layers.{l}."
        for nm in ["ln1_w", "ln1_b", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "bo", "ln2_w", "ln2_b",
                   "w1", "b1", "w2", "b2"]:
            layers.append(t(pre + nm, transpose=nm.startswith("w")).ravel())
    layers = np.concatenate(layers).astype(np.float32)
    lm_w_ref = t("lm_w", transpose=True)   # [in=D, out=V]
    fl = ref.ref_cpu_forward(cfg["V"], cfg["T"], cfg["D"], cfg["H"], cfg["L"], cfg["FF"],
                             p(t("token_emb")), p(t("pos_emb")), p(layers), p(t("ln_f_w")), p(t("ln_f_b")),
                             p(lm_w_ref), p(t("lm_b")), p(tok, C.c_int), p(tgt, C.c_int), S)
    out.update(fwd_params=params, fwd_tok=tok, fwd_tgt=tgt, fwd_loss=np.float32(fl),
               fwd_cfg=np.array([cfg[k] for k in ("V", "T", "D", "H", "L", "FF")], np.int32),
               fwd_S=np.int32(S))

    path = os.path.join(HERE, "ref_ops.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes; forward loss", fl)


if __name__ == "__main__":
    main()
