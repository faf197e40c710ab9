"""Data-parallel gradients over NCCL on two GPUs (skipped with fewer).

Two ranks each run forward + backward on their own half of a batch with
`dp_init` (bucketed all-reduce overlapped with the backward).  Checked: the
reduced gradient is bit-identical on both ranks, it matches a single-GPU
backward over the whole batch (per-tensor relative L2 <= 2e-2, the acceptance
bound of the FP16 path), the losses average to the single-GPU loss, and an
injected overflow on one rank makes both ranks skip the step.
"""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

CFG = dict(V=4096, T=128, D=256, H=4, L=4, FF=1024)
B_RANK, S = 2, 128


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _tokens(world):
    rng = np.random.default_rng(5)
    tok = rng.integers(0, CFG["V"], (world * B_RANK, S)).astype(np.int32)
    tgt = rng.integers(0, CFG["V"], (world * B_RANK, S)).astype(np.int32)
    return tok, tgt


def _worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from rbk.model import ModelConfig, RubidiumTransformer, dp_unique_id
    m = RubidiumTransformer(ModelConfig(**CFG), max_batch=B_RANK, max_seq=S)
    m.init_weights(seed=11, std=0.02)
    uid = [dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    m.dp_init(rank, world, uid[0], bucket_bytes=1 << 20)   # small buckets: several all-reduces per step
    tok, tgt = _tokens(world)
    t = torch.from_numpy(tok[rank * B_RANK:(rank + 1) * B_RANK]).cuda()
    g = torch.from_numpy(tgt[rank * B_RANK:(rank + 1) * B_RANK]).cuda()
    loss = m.forward(t, g, B_RANK, S).item()
    m.backward(t, g, B_RANK, S, loss_scale=1.0)
    torch.cuda.synchronize()
    grad = m.grad.cpu().numpy().copy() / m.loss_scale
    # overflow on rank 1 only: the reduced gradient is non-finite everywhere, both ranks skip
    if rank == 1:
        m.inject_inf(0, 1 << 30)
    m.forward(t, g, B_RANK, S)
    m.backward(t, g, B_RANK, S, loss_scale=1.0)
    scale_before = m.loss_scale
    m.optimizer_step(1, 1e-3)
    torch.cuda.synchronize()
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), grad=grad, loss=loss, scale_before=scale_before,
             scale_after=m.loss_scale)
    m.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_dp_two_ranks_match_single_gpu(tmp_path):
    import torch.multiprocessing as mp
    world = 2
    env_nvls = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.spawn(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world, join=True)
    finally:
        if env_nvls is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_nvls
    r0, r1 = (np.load(tmp_path / f"rank{r}.npz") for r in range(world))
    assert np.array_equal(r0["grad"], r1["grad"]), "all-reduced gradients differ between ranks"
    # both ranks saw the overflow and skipped: the scale backed off identically
    assert float(r0["scale_after"]) == float(r1["scale_after"]) < float(r0["scale_before"])

    from rbk.model import ModelConfig, RubidiumTransformer, param_table
    m = RubidiumTransformer(ModelConfig(**CFG), max_batch=world * B_RANK, max_seq=S)
    m.init_weights(seed=11, std=0.02)
    tok, tgt = _tokens(world)
    t = torch.from_numpy(tok).cuda()
    g = torch.from_numpy(tgt).cuda()
    loss = m.forward(t, g, world * B_RANK, S).item()
    m.backward(t, g, world * B_RANK, S, loss_scale=1.0)
    ref = m.grad.cpu().numpy() / m.loss_scale
    m.close()
    assert abs(0.5 * (float(r0["loss"]) + float(r1["loss"])) - loss) <= 1e-3 * abs(loss)
    table, _ = param_table(ModelConfig(**CFG))
    floor = 1e-2 * float(np.median([np.linalg.norm(ref[off:off + r * c]) for _, off, r, c in table]))
    for name, off, r, c in table:
        a, b = r0["grad"][off:off + r * c], ref[off:off + r * c]
        err = np.linalg.norm(a - b) / max(np.linalg.norm(b), floor)
        assert err <= 2e-2, (name, err)
