"""Failure detection of the data-parallel path on two GPUs (skipped with fewer).

No GPU is made to fault.  Both ranks finish one full step.  Rank 1 then never
joins the next collective: it waits on the host (a gloo barrier) and launches
nothing.  Rank 0 runs the next forward + backward: its first bucket's
all-reduce cannot complete, and the library's watchdog (deadline 2 s) aborts
the communicators with ncclCommAbort, which ends the NCCL kernel waiting on the
absent peer.  Checked on rank 0: the stream drains, the model reports
RBK_ERR_TIMEOUT, backward and the optimizer step refuse to run (nothing is
applied to the weights), and shutdown returns.  Rank 1 then leaves the job
with a local abort of its own communicators (rbk_model_dp_abort) and shuts
down.  NVLS is off, as for every multi-rank test here.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

CFG = dict(V=4096, T=128, D=256, H=4, L=4, FF=1024)
B, S = 2, 128
RBK_ERR_TIMEOUT = -4


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import datetime
    import time

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from rbk._lib import RbkError
    from rbk.model import ModelConfig, RubidiumTransformer, dp_unique_id
    m = RubidiumTransformer(ModelConfig(**CFG), max_batch=B, max_seq=S)
    m.init_weights(seed=3, std=0.02)
    uid = [dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    m.dp_init(rank, world, uid[0], bucket_bytes=1 << 20, timeout_s=2.0)
    rng = np.random.default_rng(rank)
    t = torch.from_numpy(rng.integers(0, CFG["V"], (B, S)).astype(np.int32)).cuda()
    g = torch.from_numpy(rng.integers(0, CFG["V"], (B, S)).astype(np.int32)).cuda()
    m.forward(t, g, B, S)
    m.backward(t, g, B, S)
    m.optimizer_step(1, 1e-3)
    torch.cuda.synchronize()
    out = {"step1_status": m.dp_status()}
    dist.barrier()                      # both ranks finished step 1, nothing in flight
    if rank == 1:
        dist.barrier()                  # rank 1 launches nothing until rank 0 has timed out
        m.dp_abort()                    # then leaves: a local abort, no collective shutdown
        out["status"] = m.dp_status()
        m.dp_shutdown()
        m.close()
        np.savez(os.path.join(outdir, f"rank{rank}.npz"), **out)
        return
    p_before = m.p32.clone()
    m.forward(t, g, B, S)
    m.backward(t, g, B, S)              # enqueues all-reduces that rank 1 never joins
    t0 = time.time()
    torch.cuda.synchronize()            # returns once the watchdog has aborted the communicator
    out["drain_s"] = time.time() - t0
    out["status"] = m.dp_status()
    for name, fn in (("backward", lambda: m.backward(t, g, B, S)),
                     ("optimizer", lambda: m.optimizer_step(2, 1e-3))):
        try:
            fn()
            out[name] = 0
        except RbkError as e:
            out[name] = e.status
    torch.cuda.synchronize()
    out["weights_unchanged"] = bool(torch.equal(p_before, m.p32))
    m.dp_shutdown()
    dist.barrier()                      # release rank 1
    m.close()
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), **out)


def test_rank_leaving_between_steps_times_out_cleanly(tmp_path):
    import torch.multiprocessing as mp
    env_nvls = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.spawn(_worker, args=(2, _free_port(), str(tmp_path)), nprocs=2, join=True)
    finally:
        if env_nvls is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_nvls
    r0 = np.load(tmp_path / "rank0.npz")
    r1 = np.load(tmp_path / "rank1.npz")
    assert int(r0["step1_status"]) == 0 and int(r1["step1_status"]) == 0
    assert int(r1["status"]) == -5                 # RBK_ERR_NCCL after its own abort
    assert int(r0["status"]) == RBK_ERR_TIMEOUT
    assert int(r0["backward"]) == RBK_ERR_TIMEOUT and int(r0["optimizer"]) == RBK_ERR_TIMEOUT
    assert bool(r0["weights_unchanged"])
    assert float(r0["drain_s"]) < 60.0
