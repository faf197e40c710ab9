"""rbk_ln_bwd_noalloc — the LayerNorm backward for callers that cannot allocate
device memory (their device memory is all owned by their own pool, or an
allocation's device-wide synchronisation is not acceptable in their step loop).

Calls the entry point through the C ABI, twice in a row on different inputs,
and checks each result against the context-based rbk_ln_bwd at the tolerance
the other kernel tests use (FP16 outputs 3e-3, FP32 reductions 1e-4), and the
first one also against the CPU oracle.  It runs a different kernel from
rbk_ln_bwd, so the two agree to rounding, not bit for bit.  Further cases: the
reference's dx formula (RBK_LN_REFERENCE_FORMULA), and D = 2048 over 16384 rows,
which uses about 3.6 MB of the 4 MiB array.  Kept in a file of its own that
pytest collects last.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

F16_TOL = 3e-3
F32_TOL = 1e-4


def rel(a, b):
    a = a.double().cpu(); b = b.double().cpu()
    return float((a - b).norm() / max(float(b.norm()), 1e-30))


def _p(t):
    return C.c_void_p(t.data_ptr()) if t is not None else None


def _case(seed, N, D, res):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = (0.3 * torch.randn(N, D, device="cuda", generator=g)).half()
    dy = torch.randn(N, D, device="cuda", generator=g).half()
    gam = (1 + 0.05 * torch.randn(D, device="cuda", generator=g)).half()
    dres = torch.randn(N, D, device="cuda", generator=g).half() if res else None
    return x, dy, gam, dres


def _run_noalloc(lib, x, dy, gam, mean, rstd, dres, want_bias, flags=0):
    N, D = x.shape
    dx = torch.empty_like(x)
    dg = torch.zeros(D, device="cuda"); db = torch.zeros(D, device="cuda")
    dbias = torch.zeros(D, device="cuda") if want_bias else None
    st = lib.rbk_ln_bwd_noalloc(_p(dx), _p(dg), _p(db), _p(dbias), _p(dy), _p(dres), _p(x), _p(gam), _p(mean),
                                _p(rstd), N, D, flags, C.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0, lib.rbk_last_error()
    return dx, dg, db, dbias


CASES = [  # (seed, N, D, residual, bias gradient, flags)
    (1, 4096, 768, True, True, 0),
    (2, 3000, 1024, False, False, 0),
    (3, 2048, 512, True, False, 1),          # RBK_LN_REFERENCE_FORMULA
    (4, 16384, 2048, False, True, 0),        # 3 x 2048 x 148 CTAs x 4 B = 3.6 MB of the array
]


def test_noalloc_ln_bwd_matches_ctx_entry_point_twice():
    from rbk import lib, ops
    L = lib()
    torch.cuda.set_device(0)
    for call, (seed, N, D, res, bias, flags) in enumerate(CASES):
        x, dy, gam, dres = _case(seed, N, D, res)
        _, mean, rstd = ops.ln_fwd(x, gam, torch.zeros(D, device="cuda").half())
        got = _run_noalloc(L, x, dy, gam, mean, rstd, dres, bias, flags)
        ref = ops.ln_bwd(dy, x, gam, mean, rstd, dres=dres, want_dbias=bias, ref_formula=bool(flags))
        torch.cuda.synchronize()
        assert rel(got[0].float(), ref[0].float()) < F16_TOL, f"dx, call {call}"
        assert rel(got[1], ref[1]) < F32_TOL and rel(got[2], ref[2]) < F32_TOL, f"dgamma/dbeta, call {call}"
        if bias:
            # dbias sums the FP16 dx that each kernel rounds on its own (the ctx entry point computes
            # dx in FP16 arithmetic at D = 768 / 1024 / 2048), and the rows' dx cancel in the sum
            assert rel(got[3], ref[3]) < 2e-3, f"dbias, call {call}"
        if call == 0:
            # the CPU oracle (src/cpu_mat.h:126-153 with the exact dx) on the same FP16 inputs
            import oracle
            f = lambda t: t.float().cpu().numpy()   # noqa: E731
            edx, edg, edb = oracle.ln_bwd(f(dy), f(x), f(gam), f(mean), f(rstd), dres=f(dres))
            assert rel(got[0].float(), torch.from_numpy(edx)) < F16_TOL, "dx vs oracle"
            assert rel(got[1], torch.from_numpy(edg)) < F32_TOL and rel(got[2], torch.from_numpy(edb)) < F32_TOL


def test_noalloc_ln_bwd_rejects_oversized_scratch():
    """D = 4096 on a 148-SM B200 needs 7.3 MB of partials: refused, nothing launched."""
    from rbk import lib
    L = lib()
    N, D = 4096, 4096
    x = torch.zeros(N, D, device="cuda", dtype=torch.float16)
    stats = torch.ones(N, device="cuda")
    dg = torch.zeros(D, device="cuda")
    st = L.rbk_ln_bwd_noalloc(_p(x), _p(dg), _p(dg), None, _p(x), None, _p(x), _p(x[0]), _p(stats), _p(stats),
                              N, D, 0, None)
    assert st < 0
    assert b"fixed" in L.rbk_last_error()
