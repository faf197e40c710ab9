"""The runtime switches keep alternative kernel paths alive: each one, set in a
fresh process (the library reads them once), must still train config 1 to the
oracle's loss and gradients.

  RBK_NO_PDL=1        no programmatic dependent launch
  RBK_GEMM_SINGLE=1   N = 256 GEMMs on single CTAs instead of 2-CTA clusters
  RBK_ATTN_LEGACY=1   mma.sync attention instead of tcgen05
"""
import json
import os
import subprocess
import sys

import pytest

pytestmark = pytest.mark.gpu

GRAD_TOL = 2e-2
LOSS_TOL = 1e-3
HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("switch", ["RBK_NO_PDL", "RBK_GEMM_SINGLE", "RBK_ATTN_LEGACY"])
def test_switch_keeps_parity(switch):
    env = dict(os.environ)
    env[switch] = "1"
    r = subprocess.run([sys.executable, os.path.join(HERE, "switch_child.py")], env=env, capture_output=True,
                       text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    out = json.loads(r.stdout.strip().splitlines()[-1])
    assert out["device_error"] == 0
    assert abs(out["loss"] - out["oracle_loss"]) <= LOSS_TOL * abs(out["oracle_loss"]), out
    bad = {k: v for k, v in out["errs"].items() if v > GRAD_TOL}
    assert not bad, bad
