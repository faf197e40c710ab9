"""Full-model pins of the oracle's backward (CPU): float64 torch autograd."""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from torch_model import loss_and_grads  # noqa: E402

TINY = dict(V=100, T=16, D=64, H=1, L=2, FF=128)


def rel(a, b, floor=1e-4):
    """Relative L2 error with an absolute floor: tensors whose exact gradient is
    zero (bk: a key bias shifts every score of a row equally) compare absolutely."""
    a = np.asarray(a, np.float64); b = np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), floor)


def _case(ora, cfg, seed, B, S):
    rng = np.random.default_rng(seed)
    params = ora.init_params(cfg, seed=seed)
    for name, off, r, c in ora.param_table(cfg):
        base = name.split(".")[-1]
        if base.startswith(("ln", "b")) or base == "lm_b":
            params[off:off + r * c] += (0.05 * rng.standard_normal(r * c)).astype(np.float32)
    tok = rng.integers(0, cfg["V"], B * S).astype(np.int32)
    tgt = rng.integers(0, cfg["V"], B * S).astype(np.int32)
    return params, tok, tgt


@pytest.mark.parametrize("relu", [False, True])
def test_model_grads_match_float64_autograd(ora, relu):
    cfg = TINY
    B, S = 2, 12
    params, tok, tgt = _case(ora, cfg, 3, B, S)
    loss, grads, _ = ora.model_loss_grad(cfg, params, tok, tgt, B, S, grad_scale=4.0, relu=relu)
    tl, tg = loss_and_grads(ora, cfg, params.astype(np.float64), tok, tgt, B, S, grad_scale=4.0, relu=relu)
    assert abs(loss - tl) < 1e-5 * abs(tl)
    for name, off, r, c in ora.param_table(cfg):
        a, b = grads[off:off + r * c], tg[off:off + r * c]
        assert rel(a, b) < 2e-4, (name, rel(a, b))


def test_lora_grads_match_float64_autograd(ora):
    cfg = TINY
    B, S, r, alpha = 2, 8, 4, 8.0
    params, tok, tgt = _case(ora, cfg, 11, B, S)
    rng = np.random.default_rng(12)
    D, L = cfg["D"], cfg["L"]
    Aq = (0.02 * rng.standard_normal((L, D, r))).astype(np.float32)
    Av = (0.02 * rng.standard_normal((L, D, r))).astype(np.float32)
    Bq = (0.02 * rng.standard_normal((L, r, D))).astype(np.float32)   # nonzero so dA is nonzero
    Bv = (0.02 * rng.standard_normal((L, r, D))).astype(np.float32)
    loss, dAq, dBq, dAv, dBv = ora.model_lora_grad(cfg, params, Aq, Bq, Av, Bv, r, alpha, tok, tgt, B, S, 2.0)
    tl, tg = loss_and_grads(ora, cfg, params.astype(np.float64), tok, tgt, B, S, grad_scale=2.0,
                            lora=dict(r=r, alpha=alpha, w=dict(Aq=Aq, Bq=Bq, Av=Av, Bv=Bv)))
    assert abs(loss - tl) < 1e-5 * abs(tl)
    for name, got in (("Aq", dAq), ("Bq", dBq), ("Av", dAv), ("Bv", dBv)):
        assert rel(got, tg[name]) < 2e-4, name


def test_lora_zero_B_gives_zero_dA(ora):
    """B = 0 at init makes dA exactly 0 on the first step (the absolute-floor case)."""
    cfg = TINY
    B, S, r = 1, 8, 4
    params, tok, tgt = _case(ora, cfg, 5, B, S)
    D, L = cfg["D"], cfg["L"]
    rng = np.random.default_rng(6)
    Aq = (0.02 * rng.standard_normal((L, D, r))).astype(np.float32)
    Av = (0.02 * rng.standard_normal((L, D, r))).astype(np.float32)
    Z = np.zeros((L, r, D), np.float32)
    _, dAq, dBq, dAv, dBv = ora.model_lora_grad(cfg, params, Aq, Z, Av, Z, r, 8.0, tok, tgt, B, S)
    assert np.all(dAq == 0) and np.all(dAv == 0)
    assert np.linalg.norm(dBq) > 0 and np.linalg.norm(dBv) > 0
