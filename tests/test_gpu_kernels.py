"""Parity of the sm_100a kernels with the CPU oracle (and float64 torch for GEMMs).

Inputs are seeded; the oracle receives exactly the FP16-rounded values the GPU
reads.  Tolerances (relative L2 unless stated):
  FP16 outputs 3e-3 (one FP16 rounding ~ 2.4e-4 rms plus FP32 summation order),
  FP32 reductions 1e-4.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

F16_TOL = 3e-3
F32_TOL = 1e-4


def rel(a, b):
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def ops():
    from rbk import ops as o
    return o


def h(a, dev="cuda"):
    return torch.from_numpy(np.ascontiguousarray(a, np.float16)).to(dev)


def f(t):
    return t.float().cpu().numpy()


# ------------------------------------------------------------------ LayerNorm --

@pytest.mark.parametrize("N,D", [(300, 256), (257, 768), (64, 1024), (33, 2048)])
def test_ln_fwd(ops, ora, N, D):
    rng = np.random.default_rng(N + D)
    x = (rng.standard_normal((N, D)) * 0.5 + 0.1).astype(np.float16)
    g = (1 + 0.1 * rng.standard_normal(D)).astype(np.float16)
    b = (0.1 * rng.standard_normal(D)).astype(np.float16)
    y, mean, rstd = ops.ln_fwd(h(x), h(g), h(b))
    ye, me, re_ = ora.ln_fwd(x.astype(np.float32), g.astype(np.float32), b.astype(np.float32))
    assert rel(f(y), ye) < F16_TOL
    assert rel(mean.cpu().numpy(), me) < 1e-5 and rel(rstd.cpu().numpy(), re_) < 1e-5


@pytest.mark.parametrize("N,D,res,bias", [(300, 256, False, False), (257, 768, True, True), (129, 1024, True, False),
                                          (40, 2048, False, True)])
def test_ln_bwd_exact(ops, ora, N, D, res, bias):
    rng = np.random.default_rng(7 * N + D)
    x = (0.05 * rng.standard_normal((N, D))).astype(np.float16)     # small variance: rstd ~ 20
    g = (1 + 0.02 * rng.standard_normal(D)).astype(np.float16)
    dy = rng.standard_normal((N, D)).astype(np.float16)
    dres = rng.standard_normal((N, D)).astype(np.float16) if res else None
    _, mean, rstd = ops.ln_fwd(h(x), h(g), h(np.zeros(D, np.float16)))
    dx, dg, db, dbias = ops.ln_bwd(h(dy), h(x), h(g), mean, rstd, dres=None if dres is None else h(dres),
                                   want_dbias=bias)
    ex, eg, eb = ora.ln_bwd(dy.astype(np.float32), x.astype(np.float32), g.astype(np.float32),
                            mean.cpu().numpy(), rstd.cpu().numpy(),
                            dres=None if dres is None else dres.astype(np.float32))
    assert rel(f(dx), ex) < F16_TOL
    assert rel(dg.cpu().numpy(), eg) < F32_TOL and rel(db.cpu().numpy(), eb) < F32_TOL
    if bias:
        assert rel(dbias.cpu().numpy(), ex.sum(0)) < 2e-3


def test_ln_bwd_reference_formula_matches_reference_engine(ops, ora):
    """RBK_LN_REFERENCE_FORMULA reproduces cpuops::layer_norm_backward's golden vectors."""
    import os
    gold = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_ops.npz"))
    x16 = gold["ln_x"].astype(np.float16); dy16 = gold["ln_dy"].astype(np.float16)
    g16 = gold["ln_g"].astype(np.float16)
    mean = torch.from_numpy(gold["ln_mean"]).cuda(); rstd = torch.from_numpy(gold["ln_rstd"]).cuda()
    dx, dg, db, _ = ops.ln_bwd(h(dy16), h(x16), h(g16), mean, rstd, ref_formula=True)
    # inputs were rounded to FP16 for the GPU: compare against the oracle on the same rounded inputs,
    # and against the reference's own vectors with the rounding tolerance.
    ex, eg, eb = ora.ln_bwd(dy16.astype(np.float32), x16.astype(np.float32), g16.astype(np.float32),
                            gold["ln_mean"], gold["ln_rstd"], ref_formula=True)
    assert rel(f(dx), ex) < F16_TOL
    assert rel(f(dx), gold["ln_dx"]) < 5e-3
    assert rel(dg.cpu().numpy(), gold["ln_dg"]) < 5e-3 and rel(db.cpu().numpy(), gold["ln_db"]) < 5e-3


def test_ln_bwd_config_2a_full_size(ops, ora):
    """[16384, 1024] FP16, x~N(0,1), dy~N(0,1), gamma~N(1,0.02): full-size parity."""
    rng = np.random.default_rng(2)
    N, D = 16384, 1024
    x = rng.standard_normal((N, D), dtype=np.float32).astype(np.float16)
    dy = rng.standard_normal((N, D), dtype=np.float32).astype(np.float16)
    g = (1 + 0.02 * rng.standard_normal(D)).astype(np.float16)
    _, mean, rstd = ops.ln_fwd(h(x), h(g), h(np.zeros(D, np.float16)))
    dx, dg, db, _ = ops.ln_bwd(h(dy), h(x), h(g), mean, rstd)
    ex, eg, eb = ora.ln_bwd(dy.astype(np.float32), x.astype(np.float32), g.astype(np.float32),
                            mean.cpu().numpy(), rstd.cpu().numpy())
    assert rel(f(dx), ex) < F16_TOL
    assert rel(dg.cpu().numpy(), eg) < F32_TOL and rel(db.cpu().numpy(), eb) < F32_TOL
    # deterministic column reduction: bitwise-identical rerun
    dx2, dg2, db2, _ = ops.ln_bwd(h(dy), h(x), h(g), mean, rstd)
    assert torch.equal(dx, dx2) and torch.equal(dg, dg2) and torch.equal(db, db2)


# ------------------------------------------------------------- cross entropy --

@pytest.mark.parametrize("N,V,ld", [(64, 4096, 4096), (37, 1000, 1008), (16, 50257, 50264), (400, 50257, 50264),
                                    (8, 65536, 65536)])
def test_softmax_xent(ops, ora, N, V, ld):
    rng = np.random.default_rng(V)
    z = np.zeros((N, ld), np.float16)
    z[:, :V] = (2.0 * rng.standard_normal((N, V))).astype(np.float16)
    t = rng.integers(0, V, N).astype(np.int32)
    scale = 65536.0 / N
    d, rl = ops.softmax_xent_bwd(h(z), torch.from_numpy(t).cuda(), scale=scale, V=V)
    z32 = z[:, :V].astype(np.float32)
    e = ora.ce_bwd(z32, t, scale * N)           # oracle divides by N itself
    assert rel(f(d)[:, :V], e) < F16_TOL
    _, erl, _ = ora.ce_fwd(z32, t)
    assert rel(rl.cpu().numpy(), erl) < 1e-4


def test_softmax_xent_inplace_and_bad_target(ops, ora):
    rng = np.random.default_rng(1)
    N, V = 12, 777
    ld = 784
    z = np.zeros((N, ld), np.float16)
    z[:, :V] = rng.standard_normal((N, V)).astype(np.float16)
    t = rng.integers(0, V, N).astype(np.int32)
    t[3] = V + 5
    zt = h(z)
    d, rl = ops.softmax_xent_bwd(zt, torch.from_numpy(t).cuda(), scale=1.0, V=V, out=zt)
    assert d.data_ptr() == zt.data_ptr()
    rl = rl.cpu().numpy()
    assert np.isnan(rl[3]) and np.all(np.isfinite(np.delete(rl, 3)))
    assert np.all(f(d)[3, :V] == 0)
    good = np.delete(np.arange(N), 3)
    e = ora.ce_bwd(z[good, :V].astype(np.float32), t[good], len(good))
    assert rel(f(d)[good, :V], e) < F16_TOL


def test_softmax_xent_config_2b_full_size(ops, ora):
    """[8192, 32000] FP16 logits ~N(0,2): rows sum to zero; 256 rows vs the oracle.
    The gradient carries the loss scale 65536 (as in training): unscaled (p - y)/N
    would sit in FP16's subnormal range."""
    rng = np.random.default_rng(3)
    N, V = 8192, 32000
    scale = 65536.0 / N
    z = (2.0 * rng.standard_normal((N, V), dtype=np.float32)).astype(np.float16)
    t = rng.integers(0, V, N).astype(np.int32)
    d, rl = ops.softmax_xent_bwd(h(z), torch.from_numpy(t).cuda(), scale=scale)
    rows = np.sort(rng.choice(N, 256, replace=False))
    dd = d[torch.from_numpy(rows).cuda()].float().cpu().numpy()
    e = ora.ce_bwd(z[rows].astype(np.float32), t[rows], scale * len(rows))
    assert rel(dd, e) < F16_TOL
    rowsum = d.float().sum(1).abs().max().item()
    assert rowsum < 0.01 * scale
    _, erl, _ = ora.ce_fwd(z[rows].astype(np.float32), t[rows])
    assert rel(rl.cpu().numpy()[rows], erl) < 1e-4


# ---------------------------------------------------- attention softmax bwd --

def _softmax_causal(rng, nmat, T):
    s = rng.standard_normal((nmat, T, T)).astype(np.float32)
    mask = np.tril(np.ones((T, T), bool))
    s = np.where(mask, s, -1e9)
    p = np.exp(s - s.max(-1, keepdims=True))
    return (p / p.sum(-1, keepdims=True)).astype(np.float16), mask


@pytest.mark.parametrize("nmat,T", [(3, 136), (2, 1024), (1, 64)])
def test_attn_softmax_bwd(ops, ora, nmat, T):
    rng = np.random.default_rng(T)
    P, mask = _softmax_causal(rng, nmat, T)
    dP = rng.standard_normal((nmat, T, T)).astype(np.float16)
    sentinel = torch.full((nmat, T, T), 7.0, dtype=torch.float16, device="cuda")
    dS = ops.attn_softmax_bwd(h(P), h(dP), causal=True, out=sentinel)
    e = ora.causal_softmax_bwd(dP.astype(np.float32), P.astype(np.float32))
    got = f(dS)
    assert rel(got[:, mask], e[:, mask]) < F16_TOL
    assert np.all(got[:, ~mask] == 7.0)          # strict upper triangle untouched


def test_attn_softmax_bwd_config_2c_full_size(ops, ora):
    """B=8, H=16, T=1024 causal: rows of dS sum to ~0 everywhere; 2 matrices vs the oracle."""
    rng = np.random.default_rng(4)
    nmat, T = 8 * 16, 1024
    s = torch.randn(nmat, T, T, device="cuda")
    s = s.masked_fill(torch.triu(torch.ones(T, T, dtype=torch.bool, device="cuda"), 1), -1e9)
    P = torch.softmax(s, -1).half()
    dP = torch.randn(nmat, T, T, device="cuda").half()
    dS = ops.attn_softmax_bwd(P, dP, causal=True)
    mask = torch.tril(torch.ones(T, T, dtype=torch.bool, device="cuda"))
    rs = (dS.float() * mask).sum(-1)
    # sum_j dS_ij = dot - dot * sum_j P_ij ~ 0 (FP16 P sums to 1 within ~1e-3)
    assert rs.abs().max().item() < 0.05 * (dP.float().abs().max().item())
    for i in (0, nmat - 1):
        e = ora.causal_softmax_bwd(dP[i:i + 1].float().cpu().numpy(), P[i:i + 1].float().cpu().numpy())
        m = mask.cpu().numpy()
        assert rel(dS[i:i + 1].float().cpu().numpy()[:, m], e[:, m]) < F16_TOL


# --------------------------------------------------------------- embeddings --

def test_embeddings(ops, ora):
    """Forward gather and backward scatter against the oracle (src/cpu_mat.h:265-277); pos_emb's
    gradient (which the reference does not compute) against the batch sum."""
    rng = np.random.default_rng(5)
    V, T, D, B, S = 97, 40, 64, 3, 32
    tok_emb = rng.standard_normal((V, D)).astype(np.float16)
    pos_emb = rng.standard_normal((T, D)).astype(np.float16)
    tokens = rng.integers(0, V, B * S).astype(np.int32)
    x = ops.embed_fwd(h(tok_emb), h(pos_emb), torch.from_numpy(tokens).cuda(), B, S)
    ex = tok_emb.astype(np.float32)[tokens] + np.tile(pos_emb[:S].astype(np.float32), (B, 1))
    assert rel(f(x), ex) < F16_TOL
    dx = rng.standard_normal((B * S, D)).astype(np.float16)
    dtok, dpos = ops.embed_bwd(h(dx), torch.from_numpy(tokens).cuda(), B, S, V)
    et = ora.embed_bwd(dx.astype(np.float32), tokens, V)
    ep = dx.astype(np.float32).reshape(B, S, D).sum(0)
    assert rel(dtok.cpu().numpy(), et) < 1e-6 and rel(dpos.cpu().numpy(), ep) < 1e-6


@pytest.mark.parametrize("N,V,D", [(16384, 50, 768), (16384, 50257, 768), (1000, 7, 2048), (40000, 300, 64)])
def test_embed_bwd_reruns_bitwise(ops, ora, N, V, D):
    """Deterministic mode: the token gradient is summed per token in position order (sorted
    keys), so two runs give identical bits, with many repeats of each token; 40000 positions take
    the reduction path (above the sort's 32768), checked against the oracle only."""
    from rbk import lib
    rng = np.random.default_rng(N + V)
    tokens = rng.integers(0, V, N).astype(np.int32)
    dx = rng.standard_normal((N, D)).astype(np.float16)
    tt, hdx = torch.from_numpy(tokens).cuda(), h(dx)
    lib().rbk_ctx_set_deterministic(ops.ctx().handle, 1)
    try:
        a, _ = ops.embed_bwd(hdx, tt, 1, N, V)
        b, _ = ops.embed_bwd(hdx, tt, 1, N, V)
    finally:
        lib().rbk_ctx_set_deterministic(ops.ctx().handle, 0)
    if N <= 32768:
        assert torch.equal(a, b)
    et = ora.embed_bwd(dx.astype(np.float32), tokens, V)
    assert rel(a.cpu().numpy(), et) < 1e-6


# --------------------------------------------------------------------- tail --

@pytest.mark.parametrize("overflow,clip", [(False, False), (True, False), (False, True)])
def test_adam_tail(ops, ora, overflow, clip):
    rng = np.random.default_rng(6 + overflow + 2 * clip)
    segs = [(0, 4096), (4096, 64), (4160, 100000 - 4160 - 64), (100000 - 64, 64)]
    n = 100000
    p = (0.02 * rng.standard_normal(n)).astype(np.float32)
    m = (1e-3 * rng.standard_normal(n)).astype(np.float32)
    v = np.abs(1e-6 * rng.standard_normal(n)).astype(np.float32)
    g = (65536.0 * 1e-3 * rng.standard_normal(n)).astype(np.float32)
    if overflow:
        g[77777] = np.inf
    sc = ops.new_scaler(65536.0, 2000)
    tp, tg, tm, tv = (torch.from_numpy(a.copy()).cuda() for a in (p, g, m, v))
    p16 = torch.empty(n, dtype=torch.float16, device="cuda")
    so = [s for s, _ in segs]; sl = [l for _, l in segs]
    ops.adam_tail(tp, tg, tm, tv, p16, sc, lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, wd=0.1, t=3,
                  seg_off=so if clip else None, seg_len=sl if clip else None, max_norm=0.05 if clip else 0.0)
    st = ops.read_scaler(sc)
    osc = ora.Scaler(65536.0, 0, 2000)
    ep, eg, em, ev = p.copy(), g.copy(), m.copy(), v.copy()
    skip = ora.adam_tail(ep, eg, em, ev, so, sl, 3e-4, 0.9, 0.999, 1e-8, 0.1, 3, osc, 0.05 if clip else 0.0)
    assert st.skipped == skip == int(overflow)
    assert st.scale == osc.scale and st.unskipped == osc.unskipped and st.status == 0
    assert torch.count_nonzero(tg).item() == 0
    assert rel(tp.cpu().numpy(), ep) < 1e-6 and rel(tm.cpu().numpy(), em) < 1e-5
    assert rel(tv.cpu().numpy(), ev) < 1e-5
    if not overflow:
        assert rel(p16.float().cpu().numpy(), ep) < 1e-3
    else:
        assert np.array_equal(tp.cpu().numpy(), p)


def test_adam_tail_growth_and_device_step_counter(ops):
    n = 4096
    sc = ops.new_scaler(1024.0, 3)
    tp = torch.zeros(n, device="cuda"); tm = torch.zeros(n, device="cuda"); tv = torch.zeros(n, device="cuda")
    for k in range(3):
        tg = torch.ones(n, device="cuda")
        ops.adam_tail(tp, tg, tm, tv, None, sc, lr=1e-3, t=0)
    st = ops.read_scaler(sc)
    assert st.applied_steps == 3 and st.scale == 2048.0 and st.unskipped == 0


# --------------------------------------------------------------------- GEMM --

def _ref_gemm(A, B, a_major, b_major):
    A = torch.from_numpy(A.astype(np.float32)); B = torch.from_numpy(B.astype(np.float32))
    Am = A.T if a_major else A
    Bm = B.T if b_major else B
    return (Am.double() @ Bm.double().T).numpy()


def _mk(rng, rows, cols, ld=None):
    ld = ld or cols
    a = np.zeros((rows, ld), np.float16)
    a[:, :cols] = (rng.standard_normal((rows, cols)) * 0.5).astype(np.float16)
    return a


@pytest.mark.parametrize("M,N,K,a_major,b_major", [
    (256, 384, 192, 0, 0),     # forward linear (both K-major)
    (200, 72, 100, 0, 0),      # ragged M, N, K (K padded to ld=104)
    (300, 136, 200, 0, 1),     # dgrad: B MN-major
    (192, 160, 1000, 1, 1),    # wgrad shape: both MN-major
    (256, 640, 128, 0, 0),     # BN=256 path
    (384, 1024, 320, 0, 1),    # BN=256 with MN-major B
    (128, 512, 64, 1, 0),      # A MN-major, BN=256
    (300, 640, 256, 0, 0),     # CTA-pair tiles: last pair row half outside M
    (200, 520, 136, 0, 1),     # CTA-pair tiles: ragged N, the odd CTA's columns wholly outside N
    (100, 512, 64, 1, 1),      # CTA-pair tiles: the odd CTA's rows wholly outside M, both MN-major
])
def test_gemm_store(ops, M, N, K, a_major, b_major):
    rng = np.random.default_rng(M * 7 + N + K)
    kpad = (K + 7) // 8 * 8
    A = _mk(rng, K, M, (M + 7) // 8 * 8) if a_major else _mk(rng, M, K, kpad)
    B = _mk(rng, K, N, (N + 7) // 8 * 8) if b_major else _mk(rng, N, K, kpad)
    ref = _ref_gemm(A[:, :M] if a_major else A[:, :K], B[:, :N] if b_major else B[:, :K], a_major, b_major)
    ldc = (N + 7) // 8 * 8
    Cg = torch.full((M, ldc), 5.0, dtype=torch.float16, device="cuda")
    ops.gemm(h(A), h(B), M, N, K, a_major, b_major, C_out=Cg, ldc=ldc)
    got = f(Cg)
    assert rel(got[:, :N], ref) < F16_TOL
    if ldc > N:
        assert np.all(got[:, N:] == 5.0)
    C32 = torch.zeros((M, ldc), dtype=torch.float32, device="cuda")
    ops.gemm(h(A), h(B), M, N, K, a_major, b_major, C_out=C32, ldc=ldc, epilogue=ops.EPI_STORE_F32)
    assert rel(C32.cpu().numpy()[:, :N], ref) < F32_TOL


def test_gemm_bias_residual_gelu(ops):
    rng = np.random.default_rng(11)
    M, N, K = 320, 768, 256
    X = _mk(rng, M, K); W = _mk(rng, N, K) * np.float16(0.1)
    b = (0.1 * rng.standard_normal(N)).astype(np.float16)
    R = _mk(rng, M, N)
    ref = _ref_gemm(X, W, 0, 0) + b.astype(np.float64)
    Y = ops.linear_fwd(h(X), h(W), bias=h(b), residual=h(R))
    assert rel(f(Y), ref + R.astype(np.float64)) < F16_TOL
    pre = torch.empty(M, N, dtype=torch.float16, device="cuda")
    act = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ops.gemm(h(X), h(W), M, N, K, C_out=pre, epilogue=ops.EPI_BIAS_GELU, bias=h(b), aux_out=act)
    assert rel(f(pre), ref) < F16_TOL
    import oracle
    assert rel(f(act), oracle.act_fwd(f(pre))) < F16_TOL
    # activation only (no pre-activation store): the same activation, bit for bit
    act2 = torch.empty(M, N, dtype=torch.float16, device="cuda")
    ops.gemm(h(X), h(W), M, N, K, C_out=pre, epilogue=ops.EPI_BIAS_GELU, bias=h(b), aux_out=act2, store_c=False)
    assert torch.equal(act2, act)


@pytest.mark.parametrize("Ntok,fin,out", [(260, 192, 320), (300, 640, 256), (777, 1024, 192)])
def test_gemm_dgrad_gelu_bwd(ops, ora, Ntok, fin, out):
    """dX = (dY W) * GELU'(pre); fin >= 512 runs on CTA-pair tiles with tensor stores."""
    rng = np.random.default_rng(12 + Ntok)
    dY = _mk(rng, Ntok, out)
    W = _mk(rng, out, fin)
    pre = _mk(rng, Ntok, fin)
    dX = ops.gemm_dgrad(h(dY), h(W), gelu_pre=h(pre))
    ref = (dY.astype(np.float64) @ W.astype(np.float64)) * ora.act_grad(pre.astype(np.float32)).astype(np.float64)
    assert rel(f(dX), ref) < F16_TOL
    dX2 = ops.gemm_dgrad(h(dY), h(W))
    assert rel(f(dX2), dY.astype(np.float64) @ W.astype(np.float64)) < F16_TOL


@pytest.mark.parametrize("Ntok,fin,out", [(1000, 160, 192), (4096, 768, 2304), (333, 64, 136), (1000, 520, 296)])
def test_gemm_wgrad_with_bias_grad(ops, Ntok, fin, out):
    rng = np.random.default_rng(Ntok + fin)
    dY = _mk(rng, Ntok, out)
    X = _mk(rng, Ntok, fin)
    dW0 = rng.standard_normal((out, fin)).astype(np.float32)
    db0 = rng.standard_normal(out).astype(np.float32)
    dW = torch.from_numpy(dW0.copy()).cuda(); db = torch.from_numpy(db0.copy()).cuda()
    ops.gemm_wgrad(h(dY), h(X), dW=dW, dbias=db)
    ref = dW0 + dY.astype(np.float64).T @ X.astype(np.float64)
    assert rel(dW.cpu().numpy(), ref) < F32_TOL
    assert rel(db.cpu().numpy(), db0 + dY.astype(np.float64).sum(0)) < F32_TOL


@pytest.mark.parametrize("Ntok,fin,out", [(4096, 768, 2304), (1000, 520, 296)])
def test_gemm_wgrad_split_k_pairs(ops, Ntok, fin, out):
    """Weight gradient without a bias gradient: N = 256 CTA-pair tiles with split K, FP32 accumulate."""
    rng = np.random.default_rng(Ntok + 3 * fin)
    dY = _mk(rng, Ntok, out)
    X = _mk(rng, Ntok, fin)
    dW0 = rng.standard_normal((out, fin)).astype(np.float32)
    dW = torch.from_numpy(dW0.copy()).cuda()
    ops.gemm_wgrad(h(dY), h(X), dW=dW)
    ref = dW0 + dY.astype(np.float64).T @ X.astype(np.float64)
    assert rel(dW.cpu().numpy(), ref) < F32_TOL
    assert ops.device_error() == 0


@pytest.mark.parametrize("Ntok,fin,out,bias", [
    (16384, 768, 768, False),     # the GPT-2-small Wo weight gradient: 3 x 3 pair tiles, 8 splits
    (16384, 768, 2304, True),     # QKV shape with a bias row sum (pair tiles, one accumulator)
    (8192, 192, 200, True),       # single-CTA N = 192 tiles with the ones-MMA row sums, ragged M
    (5000, 136, 136, False),      # ragged M and N against the 128 x 192 tiles
])
def test_gemm_wgrad_deterministic_split_k(ops, Ntok, fin, out, bias):
    """Deterministic mode: split-K partial planes are added to the gradient in split order, so
    repeated weight gradients are bitwise identical (and equal to the atomic mode within FP32
    rounding)."""
    from rbk import lib
    rng = np.random.default_rng(Ntok + out)
    dY = h(_mk(rng, Ntok, out))
    X = h(_mk(rng, Ntok, fin))
    dW0 = torch.from_numpy(rng.standard_normal((out, fin)).astype(np.float32)).cuda()
    db0 = torch.from_numpy(rng.standard_normal(out).astype(np.float32)).cuda()
    lib().rbk_ctx_set_deterministic(ops.ctx().handle, 1)
    try:
        runs = []
        for _ in range(2):
            dW, db = dW0.clone(), db0.clone()
            ops.gemm_wgrad(dY, X, dW=dW, dbias=db if bias else None)
            runs.append((dW, db))
    finally:
        lib().rbk_ctx_set_deterministic(ops.ctx().handle, 0)
    assert torch.equal(runs[0][0], runs[1][0]) and torch.equal(runs[0][1], runs[1][1])
    dW, db = dW0.clone(), db0.clone()
    ops.gemm_wgrad(dY, X, dW=dW, dbias=db if bias else None)
    assert rel(runs[0][0].cpu().numpy(), dW.cpu().numpy()) < 1e-6
    ref = dW0.double() + dY.double().t() @ X.double()
    assert rel(runs[0][0].cpu().numpy(), ref.cpu().numpy()) < F32_TOL
    if bias:
        assert rel(runs[0][1].cpu().numpy(), (db0.double() + dY.double().sum(0)).cpu().numpy()) < F32_TOL
    assert ops.device_error() == 0


def test_adam_tail_barrier_timeout_is_reported_and_recovers(ops, ora):
    """The tail's bounded grid-barrier wait runs out on a healthy GPU: one CTA is told not to
    arrive and the limit is 1 ms.  Every CTA gives up, the step is skipped (masters and moments
    untouched, gradients zeroed, scale halved), rbk_scaler.status reports RBK_ERR_TIMEOUT, and the
    next launch on the same context is a normal step that matches the oracle."""
    from rbk._lib import lib
    rng = np.random.default_rng(21)
    n = 1 << 20
    p = (0.02 * rng.standard_normal(n)).astype(np.float32)
    m = (1e-3 * rng.standard_normal(n)).astype(np.float32)
    v = np.abs(1e-6 * rng.standard_normal(n)).astype(np.float32)
    g = (1024.0 * 1e-3 * rng.standard_normal(n)).astype(np.float32)
    sc = ops.new_scaler(1024.0, 2000)
    tp, tg, tm, tv = (torch.from_numpy(a.copy()).cuda() for a in (p, g, m, v))
    assert lib().rbk_ctx_arm_tail_timeout_test(ops.ctx().handle, 1e-3, 5) == 0
    ops.adam_tail(tp, tg, tm, tv, None, sc, lr=1e-3, wd=0.1, t=1)
    st = ops.read_scaler(sc)
    assert st.status == -4                                # RBK_ERR_TIMEOUT
    assert st.skipped == 1 and st.scale == 512.0 and st.applied_steps == 0
    assert np.array_equal(tp.cpu().numpy(), p) and np.array_equal(tm.cpu().numpy(), m)
    assert np.array_equal(tv.cpu().numpy(), v)
    assert torch.count_nonzero(tg).item() == 0
    torch.cuda.synchronize()                              # the context is intact
    # the next launch is a normal step
    tg.copy_(torch.from_numpy(g))
    ops.adam_tail(tp, tg, tm, tv, None, sc, lr=1e-3, wd=0.1, t=1)
    st = ops.read_scaler(sc)
    assert st.status == 0 and st.skipped == 0 and st.applied_steps == 1
    osc = ora.Scaler(512.0, 0, 2000)
    ep, eg, em, ev = p.copy(), g.copy(), m.copy(), v.copy()
    ora.adam_tail(ep, eg, em, ev, [0], [n], 1e-3, 0.9, 0.999, 1e-8, 0.1, 1, osc, 0.0)
    assert rel(tp.cpu().numpy(), ep) < 1e-6 and rel(tm.cpu().numpy(), em) < 1e-5


# -------------------------------------------------------- LoRA (kernel level) --

def test_lora_kernel_level_fwd_bwd_adam(ops):
    """rbk_lora_fwd / _bwd on a q-column slice of a fused qkv (row stride 3D) against a float64
    restatement of the adapter math (src/lora.h:223-229) on the same FP16 inputs, with xa and dyb
    rounded to FP16 where the kernels store them; rbk_lora_adam equals rbk_adam_tail."""
    import ctypes

    from rbk._lib import TailArgs, lib
    rng = np.random.default_rng(31)
    N, D, r, s = 512, 768, 16, 2.0
    f16 = lambda a: torch.from_numpy(a.astype(np.float16)).cuda()  # noqa: E731
    x = f16(rng.standard_normal((N, D)))
    A = f16(0.02 * rng.standard_normal((D, r)))
    Bm = f16(0.05 * rng.standard_normal((r, D)))
    qkv = f16(rng.standard_normal((N, 3 * D)))
    y0 = qkv[:, :D].double().cpu().numpy()
    kv0 = qkv[:, D:].clone()
    xa = ops.lora_fwd(x, A, Bm, qkv[:, :D], s)
    torch.cuda.synchronize()
    X, Am, Bd = (t.double().cpu().numpy() for t in (x, A, Bm))
    xa_ref = X @ Am
    assert rel(xa.double().cpu().numpy(), xa_ref) < 2e-3
    xa16 = xa.double().cpu().numpy()
    y_ref = y0 + s * xa16 @ Bd
    assert rel(qkv[:, :D].double().cpu().numpy(), y_ref) < 2e-3
    assert torch.equal(qkv[:, D:], kv0)                       # the k and v columns are untouched
    dy = f16(rng.standard_normal((N, 3 * D)))[:, :D]
    dx = f16(rng.standard_normal((N, D)))
    dx0 = dx.double().cpu().numpy()
    dA = torch.zeros(D, r, device="cuda")
    dB = torch.zeros(r, D, device="cuda")
    ops.lora_bwd(dy, x, xa, A, Bm, s, dA, dB, dx)
    torch.cuda.synchronize()
    DY = dy.double().cpu().numpy()
    assert rel(dB.double().cpu().numpy(), s * xa16.T @ DY) < 1e-4
    dyb = (s * DY @ Bd.T).astype(np.float16).astype(np.float64)
    assert rel(dA.double().cpu().numpy(), X.T @ dyb) < 1e-3
    assert rel(dx.double().cpu().numpy(), dx0 + dyb @ Am.T) < 2e-3
    # lora_optimizer_step: the fused tail over an adapter arena
    n = 4 * D * r
    p = (0.02 * rng.standard_normal(n)).astype(np.float32)
    g = (rng.standard_normal(n)).astype(np.float32)
    outs = []
    for fn in ("rbk_adam_tail", "rbk_lora_adam"):
        tp, tg = torch.from_numpy(p.copy()).cuda(), torch.from_numpy(g.copy()).cuda()
        tm, tv = torch.zeros(n, device="cuda"), torch.zeros(n, device="cuda")
        sc = ops.new_scaler(1.0, 2000)
        a = TailArgs()
        a.p32, a.g, a.m, a.v, a.p16, a.n = tp.data_ptr(), tg.data_ptr(), tm.data_ptr(), tv.data_ptr(), None, n
        a.lr, a.beta1, a.beta2, a.eps, a.weight_decay, a.t, a.scaler = 1e-3, 0.9, 0.999, 1e-8, 0.0, 1, sc.data_ptr()
        assert getattr(lib(), fn)(ops.ctx().handle, ctypes.byref(a), ops._s()) == 0
        torch.cuda.synchronize()
        outs.append(tp.cpu())
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("M,N,K,splits", [(300, 512, 1000, 0), (520, 768, 4096, 3)])
def test_gemm_row_sums_k_major_a(ops, M, N, K, splits):
    """dbias_rows with a K-major A on the CTA-pair tiles (the row warp reads 128-byte rows of A);
    split K adds the partial row sums atomically."""
    rng = np.random.default_rng(M + K)
    A = _mk(rng, M, K)
    B = _mk(rng, N, K)
    C0 = rng.standard_normal((M, N)).astype(np.float32)
    r0 = rng.standard_normal(M).astype(np.float32)
    C = torch.from_numpy(C0.copy()).cuda()
    rows = torch.from_numpy(r0.copy()).cuda()
    ops.gemm(h(A), h(B), M, N, K, 0, 0, C_out=C, epilogue=ops.EPI_ACC_F32, dbias_rows=rows, alpha=0.5,
             split_k=splits)
    torch.cuda.synchronize()
    A64 = A.astype(np.float16).astype(np.float64)
    ref = C0 + 0.5 * A64 @ B.astype(np.float16).astype(np.float64).T
    assert rel(C.cpu().numpy(), ref) < F32_TOL
    assert rel(rows.cpu().numpy(), r0 + 0.5 * A64.sum(1)) < F32_TOL
    assert ops.device_error() == 0
