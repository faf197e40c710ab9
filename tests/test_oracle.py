"""Pins of the CPU oracle (oracle/oracle.cpp) before anything is compared against it.

1. Golden vectors produced by the reference's own CPU engine
   (tests/golden/ref_ops.npz, made by tests/golden/make_golden.py from
   src/cpu_mat.h and src/cpu_model.cpp).
2. Live agreement with the reference engine when oracle/_ref/libref.so exists.
3. The full-model backward against an independent float64 torch autograd model.
"""
import os

import numpy as np
import pytest

GOLD = os.path.join(os.path.dirname(__file__), "golden", "ref_ops.npz")


@pytest.fixture(scope="module")
def gold():
    return np.load(GOLD)


def rel(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def test_ln_against_reference(ora, gold):
    y, mean, rstd = ora.ln_fwd(gold["ln_x"], gold["ln_g"], gold["ln_b"])
    assert rel(y, gold["ln_y"]) < 1e-5
    assert rel(mean, gold["ln_mean"]) < 1e-5 and rel(rstd, gold["ln_rstd"]) < 1e-5
    dx, dg, db = ora.ln_bwd(gold["ln_dy"], gold["ln_x"], gold["ln_g"], gold["ln_mean"], gold["ln_rstd"],
                            ref_formula=True)
    assert rel(dx, gold["ln_dx"]) < 1e-5
    assert rel(dg, gold["ln_dg"]) < 1e-5
    assert rel(db, gold["ln_db"]) < 1e-5


def test_ln_bwd_exact_vs_reference_formula(ora, gold):
    """The reference's dx (cpu_mat.h:146) lacks one rstd factor on the x-hat term;
    the exact mode matches float64 autograd, the reference mode does not (rstd != 1)."""
    torch = pytest.importorskip("torch")
    rng = np.random.default_rng(2)
    N, D = 16, 128
    x = (0.05 * rng.standard_normal((N, D))).astype(np.float32)      # rstd ~ 20
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float32)
    dy = rng.standard_normal((N, D)).astype(np.float32)
    _, mean, rstd = ora.ln_fwd(x, g, np.zeros(D, np.float32))
    xt = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    mu = xt.mean(-1, keepdim=True)
    var = ((xt - mu) ** 2).mean(-1, keepdim=True)
    ((xt - mu) / torch.sqrt(var + 1e-5) * torch.tensor(g, dtype=torch.float64)
     * torch.tensor(dy, dtype=torch.float64)).sum().backward()
    exact, _, _ = ora.ln_bwd(dy, x, g, mean, rstd)
    refm, _, _ = ora.ln_bwd(dy, x, g, mean, rstd, ref_formula=True)
    assert rel(exact, xt.grad.numpy()) < 1e-4
    assert rel(refm, xt.grad.numpy()) > 0.05


def test_ln_bwd_residual_branch(ora, gold):
    dres = np.arange(gold["ln_x"].size, dtype=np.float32).reshape(gold["ln_x"].shape) * 1e-3
    dx0, _, _ = ora.ln_bwd(gold["ln_dy"], gold["ln_x"], gold["ln_g"], gold["ln_mean"], gold["ln_rstd"])
    dx1, _, _ = ora.ln_bwd(gold["ln_dy"], gold["ln_x"], gold["ln_g"], gold["ln_mean"], gold["ln_rstd"], dres=dres)
    np.testing.assert_allclose(dx1, dx0 + dres, rtol=1e-6, atol=1e-6)


def test_softmax_bwd_against_reference(ora, gold):
    dx = ora.softmax_bwd(gold["sm_dy"], gold["sm_y"])
    assert rel(dx, gold["sm_dx"]) < 1e-6


def test_causal_softmax_bwd_matches_masked_rows(ora):
    rng = np.random.default_rng(0)
    nmat, T = 3, 17
    z = rng.standard_normal((nmat, T, T)).astype(np.float32)
    mask = np.tril(np.ones((T, T), bool))
    z = np.where(mask, z, -1e9)
    y = np.exp(z - z.max(-1, keepdims=True)); y /= y.sum(-1, keepdims=True)
    dy = rng.standard_normal((nmat, T, T)).astype(np.float32)
    got = ora.causal_softmax_bwd(dy, y.astype(np.float32))
    full = ora.softmax_bwd(dy.reshape(-1, T), y.astype(np.float32).reshape(-1, T)).reshape(nmat, T, T)
    # masked probabilities are exactly 0, so the full-row formula agrees on the triangle
    np.testing.assert_allclose(got[:, mask], full[:, mask], rtol=1e-5, atol=1e-7)
    assert np.all(got[:, ~mask] == 0)


def test_ce_against_reference(ora, gold):
    loss, rl, lse = ora.ce_fwd(gold["ce_logits"], gold["ce_tgt"])
    assert abs(loss - float(gold["ce_loss"])) < 1e-5 * abs(float(gold["ce_loss"]))
    d = ora.ce_bwd(gold["ce_logits"], gold["ce_tgt"], 1.0)
    assert rel(d, gold["ce_dlogits"]) < 1e-5
    d2 = ora.ce_bwd(gold["ce_logits"], gold["ce_tgt"], 65536.0)
    assert rel(d2, gold["ce_dlogits"] * 65536.0) < 1e-5


def test_embedding_bwd_against_reference(ora, gold):
    dW = ora.embed_bwd(gold["emb_dout"], gold["emb_idx"], gold["emb_dW"].shape[0])
    assert rel(dW, gold["emb_dW"]) < 1e-6


def test_adamw_against_reference(ora, gold):
    p = gold["adam_p0"].copy(); m = np.zeros_like(p); v = np.zeros_like(p)
    for t in range(1, 4):
        p, m, v = ora.adamw(p, gold["adam_g"][t - 1], m, v, 3e-4, 0.9, 0.999, 1e-8, 0.1, t)
    assert rel(p, gold["adam_p3"]) < 1e-6
    assert rel(m, gold["adam_m3"]) < 1e-6
    assert rel(v, gold["adam_v3"]) < 1e-6


def test_clip_against_reference(ora, gold):
    g1, n1 = ora.clip(gold["clip_g1"], 1.0)
    g2, n2 = ora.clip(gold["clip_g2"], 1.0)
    assert rel(g1, gold["clip_g1_out"]) < 1e-6 and rel(g2, gold["clip_g2_out"]) < 1e-6
    assert abs(n1 - gold["clip_norms"][0]) < 1e-5 and abs(n2 - gold["clip_norms"][1]) < 1e-6


def test_matmul_conventions_against_reference(ora, gold):
    A, B = gold["mm_A"], gold["mm_B"]
    assert rel(ora.gemm_nt(A, B.T.copy()), gold["mm_C"]) < 1e-6
    assert rel(gold["mm_C_tB"], gold["mm_C"]) < 1e-6 and rel(gold["mm_C_tA"], gold["mm_C"]) < 1e-6


def test_forward_loss_against_reference_engine(ora, gold):
    """CPUTransformer::forward (ReLU, V == D) vs the oracle in ReLU mode."""
    c = gold["fwd_cfg"]
    cfg = dict(V=int(c[0]), T=int(c[1]), D=int(c[2]), H=int(c[3]), L=int(c[4]), FF=int(c[5]))
    S = int(gold["fwd_S"])
    loss, _, _ = ora.model_loss_grad(cfg, gold["fwd_params"], gold["fwd_tok"], gold["fwd_tgt"], 1, S,
                                     relu=True, want_grads=False)
    assert abs(loss - float(gold["fwd_loss"])) < 2e-5 * abs(float(gold["fwd_loss"]))


def test_live_reference_agrees_when_built(ora):
    """Re-run one golden case against the live reference build (skipped without it)."""
    ref = ora.ref_lib()
    if ref is None:
        pytest.skip("oracle/_ref/libref.so not built (no reference tree here)")
    import ctypes as C
    rng = np.random.default_rng(5)
    N, V = 9, 77
    z = rng.standard_normal((N, V)).astype(np.float32)
    t = rng.integers(0, V, N).astype(np.int32)
    d = np.empty_like(z)
    ref.ref_cross_entropy_backward(d.ctypes.data_as(C.POINTER(C.c_float)), z.ctypes.data_as(C.POINTER(C.c_float)),
                                   t.ctypes.data_as(C.POINTER(C.c_int)), N, V)
    assert rel(ora.ce_bwd(z, t), d) < 1e-5


def test_scaler_sequence(ora):
    """LossScaler::update semantics (src/cuda_kernels.cu:102-116)."""
    s = ora.Scaler(65536.0, 0, 3)
    assert ora.scaler_update(s, True) == 1 and s.scale == 32768.0 and s.unskipped == 0
    for _ in range(2):
        assert ora.scaler_update(s, False) == 0
    assert s.scale == 32768.0 and s.unskipped == 2
    assert ora.scaler_update(s, False) == 0 and s.scale == 65536.0 and s.unskipped == 0
    for _ in range(3):
        ora.scaler_update(s, False)
    assert s.scale == 65536.0           # clamped at 65536
    s2 = ora.Scaler(1.0, 5, 2000)
    ora.scaler_update(s2, True)
    assert s2.scale == 1.0              # clamped at 1


def test_adam_tail_skip_and_unscale(ora):
    rng = np.random.default_rng(1)
    n = 1000
    p = rng.standard_normal(n).astype(np.float32); m = np.zeros(n, np.float32); v = np.zeros(n, np.float32)
    g = (rng.standard_normal(n) * 1024).astype(np.float32)
    s = ora.Scaler(1024.0, 0, 2000)
    p0 = p.copy()
    g_bad = g.copy(); g_bad[17] = np.inf
    assert ora.adam_tail(p, g_bad, m, v, [0], [n], 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, s) == 1
    assert np.array_equal(p, p0) and s.scale == 512.0 and np.all(g_bad == 0)
    s.scale = 1024.0
    pe, me, ve = ora.adamw(p0, g / 1024.0, np.zeros(n, np.float32), np.zeros(n, np.float32),
                           1e-3, 0.9, 0.999, 1e-8, 0.0, 1)
    assert ora.adam_tail(p, g.copy(), m, v, [0], [n], 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, s) == 0
    np.testing.assert_allclose(p, pe, rtol=1e-6, atol=1e-7)


def test_reference_timed_entry_points_run():
    """The CPU baseline's timed calls into the reference's own engine (oracle/_ref) run and
    report a positive duration at small sizes; its forward agrees with the untimed wrapper."""
    import ctypes as C

    import oracle
    ref = oracle.ref_lib()
    if ref is None:
        pytest.skip("oracle/_ref/libref.so not built (reference sources absent)")
    F = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))   # noqa: E731
    I = lambda a: a.ctypes.data_as(C.POINTER(C.c_int))     # noqa: E731
    rng = np.random.default_rng(0)
    N, D = 64, 128
    x = rng.standard_normal((N, D), dtype=np.float32)
    dy = rng.standard_normal((N, D), dtype=np.float32)
    g = np.ones(D, np.float32)
    mean = x.mean(1).astype(np.float32)
    rstd = (1 / np.sqrt(x.var(1) + 1e-5)).astype(np.float32)
    assert ref.ref_time_layer_norm_backward(F(dy), F(x), F(g), F(mean), F(rstd), N, D) > 0
    y = rng.random((N, D), dtype=np.float32)
    assert ref.ref_time_softmax_backward(F(dy), F(y), N, D) > 0
    tg = rng.integers(0, D, N).astype(np.int32)
    assert ref.ref_time_cross_entropy_backward(F(x), I(tg), N, D) > 0
    n = 4096
    p = rng.standard_normal(n, dtype=np.float32)
    assert ref.ref_time_adamw_step(F(p), F(p), n, C.c_float(1e-3), C.c_float(0.9), C.c_float(0.999),
                                   C.c_float(1e-8), C.c_float(0.0)) > 0
