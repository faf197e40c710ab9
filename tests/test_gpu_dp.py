"""Data-parallel gradients over NCCL on two GPUs (skipped with fewer).

Two ranks run one worker (spawned once for the module) through four cases of
the bucketed all-reduce that `dp_init` sets up, overlapped with the backward:

  ga1     forward + backward on each rank's half of a batch;
  ga2     two micro-steps per rank, the first inside `no_sync()` (local
          accumulation only), the second all-reducing the accumulated sum —
          the reference loop's gradient accumulation (src/main.cpp:136-164);
  train   `rbk_model_train` with ga = 2 (it sets the sync switch itself);
  skip    an overflow injected on one rank makes both ranks skip the step.

Checked: the reduced gradients are bit-identical on both ranks; they match a
single-GPU backward over the concatenated micro-batches and the CPU oracle on
the same batch (per-tensor relative L2 <= 2e-2, the acceptance bound of the
FP16 path); the losses average to the single-GPU loss; both ranks skip.
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
B_RANK, S, WORLD, GA = 2, 128, 2, 2
B1 = 0.9          # Adam beta1: after the first applied step m = (1 - beta1) * unscaled gradient


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _batch(world, ga=1, seed=5):
    """tokens/targets [ga, world * B_RANK, S]: micro-step g of rank r is rows r*B_RANK.. of [g]."""
    rng = np.random.default_rng(seed)
    tok = rng.integers(0, CFG["V"], (ga, world * B_RANK, S)).astype(np.int32)
    tgt = rng.integers(0, CFG["V"], (ga, world * B_RANK, S)).astype(np.int32)
    return tok, tgt


def _stream(seed=9, n=8192):
    """A token stream and window starts [world, ga, B_RANK] for the trainer-loop case."""
    rng = np.random.default_rng(seed)
    toks = rng.integers(0, CFG["V"], n).astype(np.int32)
    starts = rng.integers(0, n - S - 1, (WORLD, GA, B_RANK)).astype(np.int64)
    return toks, starts


def _worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from rbk.model import ModelConfig, RubidiumTransformer, dp_unique_id
    m = RubidiumTransformer(ModelConfig(**CFG), max_batch=B_RANK, max_seq=S)
    m.init_weights(seed=11, std=0.02)
    params = m.p32.cpu().numpy().copy()
    uid = [dp_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    m.dp_init(rank, world, uid[0], bucket_bytes=1 << 20)   # small buckets: several all-reduces per step
    out = {"params": params}

    def rows(a, g):
        return torch.from_numpy(a[g, rank * B_RANK:(rank + 1) * B_RANK]).cuda()

    # ga1
    tok, tgt = _batch(world)
    t, g = rows(tok, 0), rows(tgt, 0)
    out["ga1_loss"] = m.forward(t, g, B_RANK, S).item()
    m.backward(t, g, B_RANK, S, loss_scale=1.0)
    torch.cuda.synchronize()
    out["ga1_grad"] = m.grad.cpu().numpy() / m.loss_scale
    m.grad.zero_()
    # ga2: the first micro-step accumulates locally, the second reduces the sum
    tok, tgt = _batch(world, GA, seed=6)
    losses = []
    for k in range(GA):
        t, g = rows(tok, k), rows(tgt, k)
        if k < GA - 1:
            with m.no_sync():
                losses.append(m.forward(t, g, B_RANK, S).item())
                m.backward(t, g, B_RANK, S, loss_scale=1.0 / GA)
        else:
            losses.append(m.forward(t, g, B_RANK, S).item())
            m.backward(t, g, B_RANK, S, loss_scale=1.0 / GA)
    torch.cuda.synchronize()
    out["ga2_loss"] = float(np.mean(losses))
    out["ga2_grad"] = m.grad.cpu().numpy() / m.loss_scale
    m.grad.zero_()
    # train: the device trainer loop, one step of GA micro-steps, no clip, no weight decay
    toks, starts = _stream()
    d_toks = torch.from_numpy(toks).cuda()
    out["train_loss"] = m.train(d_toks, steps=1, ga=GA, B=B_RANK, T=S, starts=starts[rank].reshape(-1),
                                lr=1e-3, b1=B1)[0]
    torch.cuda.synchronize()
    out["train_m"] = m._bufs[3].cpu().numpy() / (1.0 - B1)
    # skip: overflow on rank 1 only; the reduced gradient is non-finite everywhere, both skip
    tok, tgt = _batch(world, seed=7)
    t, g = rows(tok, 0), rows(tgt, 0)
    if rank == 1:
        m.inject_inf(0, 1 << 30)
    m.forward(t, g, B_RANK, S)
    m.backward(t, g, B_RANK, S, loss_scale=1.0)
    out["scale_before"] = m.loss_scale
    m.optimizer_step(2, 1e-3)
    torch.cuda.synchronize()
    out["scale_after"] = m.loss_scale
    out["skipped"] = m.scaler().skipped
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), **out)
    m.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.fixture(scope="module")
def ranks(tmp_path_factory):
    import torch.multiprocessing as mp
    d = tmp_path_factory.mktemp("dp")
    env_nvls = os.environ.get("NCCL_NVLS_ENABLE")
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        mp.spawn(_worker, args=(WORLD, _free_port(), str(d)), nprocs=WORLD, join=True)
    finally:
        if env_nvls is None:
            os.environ.pop("NCCL_NVLS_ENABLE", None)
        else:
            os.environ["NCCL_NVLS_ENABLE"] = env_nvls
    return [dict(np.load(d / f"rank{r}.npz")) for r in range(WORLD)]


def _single_gpu(params, tok, tgt, grad_scale):
    """One GPU, the concatenated micro-batches of all ranks, one backward per micro-step."""
    from rbk.model import ModelConfig, RubidiumTransformer
    ga = tok.shape[0]
    m = RubidiumTransformer(ModelConfig(**CFG), max_batch=WORLD * B_RANK, max_seq=S)
    m.load_params(torch.from_numpy(params))
    losses = []
    for k in range(ga):
        t, g = torch.from_numpy(tok[k]).cuda(), torch.from_numpy(tgt[k]).cuda()
        losses.append(m.forward(t, g, WORLD * B_RANK, S).item())
        m.backward(t, g, WORLD * B_RANK, S, loss_scale=grad_scale)
    torch.cuda.synchronize()
    grad = m.grad.cpu().numpy() / m.loss_scale
    m.close()
    return float(np.mean(losses)), grad


def _check(got, ref):
    from rbk.model import ModelConfig, param_table
    table, _ = param_table(ModelConfig(**CFG))
    floor = 1e-2 * float(np.median([np.linalg.norm(ref[off:off + r * c]) for _, off, r, c in table]))
    for name, off, r, c in table:
        a, b = got[off:off + r * c], ref[off:off + r * c]
        err = np.linalg.norm(a - b) / max(np.linalg.norm(b), floor)
        assert err <= 2e-2, (name, err)


def test_dp_ranks_agree(ranks):
    r0, r1 = ranks
    for key in ("ga1_grad", "ga2_grad", "train_m"):
        assert np.array_equal(r0[key], r1[key]), f"{key}: all-reduced gradients differ between ranks"


def test_dp_ga1_matches_single_gpu(ranks):
    r0, r1 = ranks
    tok, tgt = _batch(WORLD)
    loss, ref = _single_gpu(r0["params"], tok, tgt, 1.0)
    assert abs(0.5 * (float(r0["ga1_loss"]) + float(r1["ga1_loss"])) - loss) <= 1e-3 * abs(loss)
    _check(r0["ga1_grad"], ref)


def test_dp_ga2_matches_single_gpu_and_oracle(ranks):
    import oracle
    r0, r1 = ranks
    tok, tgt = _batch(WORLD, GA, seed=6)
    loss, ref = _single_gpu(r0["params"], tok, tgt, 1.0 / GA)
    assert abs(0.5 * (float(r0["ga2_loss"]) + float(r1["ga2_loss"])) - loss) <= 1e-3 * abs(loss)
    _check(r0["ga2_grad"], ref)
    # the oracle on all GA * WORLD * B_RANK sequences at once: the gradient of their mean loss
    el, eg, _ = oracle.model_loss_grad(CFG, r0["params"], tok.reshape(-1), tgt.reshape(-1), GA * WORLD * B_RANK, S)
    assert abs(loss - el) <= 1e-3 * abs(el)
    _check(r0["ga2_grad"], eg)


def test_dp_train_loop_ga2_matches_single_gpu(ranks):
    from rbk.model import ModelConfig, RubidiumTransformer
    r0, _ = ranks
    toks, starts = _stream()
    m = RubidiumTransformer(ModelConfig(**CFG), max_batch=WORLD * B_RANK, max_seq=S)
    m.load_params(torch.from_numpy(r0["params"]))
    # micro-step g on one GPU = the windows of every rank's micro-step g, rank by rank
    one = np.concatenate([starts[r] for r in range(WORLD)], axis=1).reshape(-1)
    m.train(torch.from_numpy(toks).cuda(), steps=1, ga=GA, B=WORLD * B_RANK, T=S, starts=one, lr=1e-3, b1=B1)
    torch.cuda.synchronize()
    ref = m._bufs[3].cpu().numpy() / (1.0 - B1)
    m.close()
    _check(r0["train_m"], ref)


def test_dp_overflow_on_one_rank_skips_everywhere(ranks):
    r0, r1 = ranks
    assert int(r0["skipped"]) == int(r1["skipped"]) == 1
    assert float(r0["scale_after"]) == float(r1["scale_after"]) < float(r0["scale_before"])
