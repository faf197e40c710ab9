"""Child process for test_gpu_switches: one config-1 forward + backward under the
runtime switches in the environment, gradients checked against the CPU oracle.
Prints one JSON line {loss, oracle_loss, errs}."""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (HERE, ROOT, os.path.join(ROOT, "rubidium-train_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle  # noqa: E402
from test_gpu_model import CFG1, _grad_errors, _setup  # noqa: E402

oracle.lib()
B, S = 8, 128
m, params, tok, tgt = _setup(oracle, CFG1, B, S, seed=1, ckpt=True)
loss, el, errs = _grad_errors(oracle, CFG1, m, params, tok, tgt, B, S)
from rbk import ops  # noqa: E402
status = ops.device_error()
m.close()
print(json.dumps({"loss": loss, "oracle_loss": el, "errs": errs, "device_error": status}))
