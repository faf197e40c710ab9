"""Kernel-level data parallelism (rbk_dp_init / rbk_dp_bucket_ready / rbk_dp_finish) on two
GPUs (skipped with fewer): callers that keep their own orchestration hand the library FP32
gradient buckets as they become final.

Each rank fills three buckets of different sizes with its own seeded values, enqueues them
after other work on its stream, and waits with rbk_dp_finish.  Checked: every bucket holds
the sum over both ranks, bit for bit (a two-term FP32 sum is exact in any order), and the
status is clean; the handle is destroyed.  NVLS is off, as for every multi-rank test here.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                                 reason="needs 2 GPUs")]

SIZES = (1 << 20, 3 * 4096 + 8, 77)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _vals(rank, k, n):
    return np.random.default_rng(100 * rank + k).standard_normal(n).astype(np.float32)


def _worker(rank, world, port, outdir):
    import ctypes
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from rbk._lib import DpOpts, lib
    from rbk.model import dp_unique_id
    from rbk.ops import _s
    uid = [dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    buf = ctypes.create_string_buffer(uid[0], 128)
    o = DpOpts()
    o.timeout_s = 60.0
    h = ctypes.c_void_p()
    assert lib().rbk_dp_init(ctypes.byref(h), rank, buf, rank, world, ctypes.byref(o)) == 0
    bufs = [torch.from_numpy(_vals(rank, k, n)).cuda() for k, n in enumerate(SIZES)]
    work = torch.randn(4096, 4096, device="cuda")
    for b in bufs:
        work = work @ work.T * 1e-3                   # unrelated work on the stream before each bucket
        assert lib().rbk_dp_bucket_ready(h, ctypes.c_void_p(b.data_ptr()), b.numel(), _s()) == 0
    assert lib().rbk_dp_finish(h, _s()) == 0
    torch.cuda.synchronize()
    out = {f"b{k}": b.cpu().numpy() for k, b in enumerate(bufs)}
    out["status"] = lib().rbk_dp_status(h)
    out["destroy"] = lib().rbk_dp_destroy(h)
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), **out)
    dist.barrier()
    dist.destroy_process_group()


def test_kernel_level_buckets_sum_over_ranks(tmp_path):
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
    for r in range(2):
        got = np.load(tmp_path / f"rank{r}.npz")
        assert int(got["status"]) == 0 and int(got["destroy"]) == 0
        for k, n in enumerate(SIZES):
            assert np.array_equal(got[f"b{k}"], _vals(0, k, n) + _vals(1, k, n)), (r, k)
