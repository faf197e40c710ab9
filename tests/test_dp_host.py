"""Data-parallel host logic on CPU: two gloo ranks (world_size 2), no GPU.

Checks the all-reduce schedule librbk builds (rbk_dp_plan) and the semantics
the GPU path relies on, reproduced with gloo collectives on the same buckets:
  - every rank derives the same plan; buckets tile the arena exactly once, in
    backward (descending address) order, each >= the bucket size but the last;
  - summing the pre-divided (1/world) per-rank gradients bucket by bucket gives
    the gradient of the global mean loss;
  - a non-finite value on one rank reaches every rank through the sum, so the
    overflow / skip decision is identical everywhere;
  - gradient accumulation (GA micro-steps per optimizer step, src/main.cpp:136-164):
    with the schedule the library uses (micro-steps before the last only accumulate,
    the last all-reduces the accumulated arena) the result is the mean gradient over
    all ranks and micro-steps; all-reducing the accumulated arena after every
    micro-step instead weights earlier micro-steps by world^(GA-1-k).
"""
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")
import torch.distributed as dist  # noqa: E402
import torch.multiprocessing as mp  # noqa: E402

GPT2S = dict(V=50257, T=1024, D=768, H=12, L=12, FF=3072)
TINY = dict(V=4096, T=128, D=256, H=4, L=4, FF=1024)


def _plan(cfg, bucket_bytes):
    from rbk.model import ModelConfig, dp_plan
    return dp_plan(ModelConfig(**cfg), bucket_bytes)


def _arena(cfg):
    from rbk.model import ModelConfig, param_table
    return param_table(ModelConfig(**cfg))


@pytest.mark.parametrize("cfg,bucket_mb", [(GPT2S, 25), (TINY, 1), (TINY, 1000)])
def test_plan_tiles_arena(cfg, bucket_mb):
    table, n = _arena(cfg)
    plan = _plan(cfg, bucket_mb << 20)
    assert plan[0][2] == n and plan[-1][1] == 0
    for (u0, b0, e0), (u1, b1, e1) in zip(plan, plan[1:]):
        assert e1 == b0 and u1 > u0                     # contiguous, descending, in backward order
    elems = (bucket_mb << 20) // 4
    assert all(e - b >= elems for _, b, e in plan[:-1])
    assert plan[-1][0] == cfg["L"] + 1                  # the embeddings close the last bucket
    # the head (LM head, ln_f) is the first unit the backward finishes
    lm_off = [off for name, off, r, c in table if name == "ln_f_w"][0]
    assert plan[0][1] <= lm_off


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = TINY
        plan = _plan(cfg, 1 << 20)
        # all ranks agree on the plan
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        same = all(p == plans[0] for p in plans)
        _, n = _arena(cfg)
        rng = np.random.default_rng(100 + rank)
        local = rng.standard_normal(n).astype(np.float32)       # this rank's mean-loss gradient
        g = torch.from_numpy(local / world)                     # seed pre-divided by world
        for _, b, e in plan:                                    # bucketed sum all-reduce, plan order
            seg = g[b:e].clone()
            dist.all_reduce(seg, op=dist.ReduceOp.SUM)
            g[b:e] = seg
        allg = [torch.zeros(n) for _ in range(world)]
        dist.all_gather(allg, torch.from_numpy(local))
        expect = torch.stack(allg).mean(0)
        ok_sum = torch.allclose(g, expect, rtol=1e-5, atol=1e-6)
        # overflow agreement: rank 1 plants an inf in the last bucket
        h = torch.ones(n)
        if rank == 1:
            h[plan[-1][1] + 3] = float("inf")
        for _, b, e in plan:
            seg = h[b:e].clone()
            dist.all_reduce(seg, op=dist.ReduceOp.SUM)
            h[b:e] = seg
        skip = torch.tensor([int(not torch.isfinite(h).all())])
        skips = [torch.zeros(1, dtype=torch.long) for _ in range(world)]
        dist.all_gather(skips, skip)
        q.put((rank, same, ok_sum, [int(s) for s in skips]))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_bucketed_allreduce_semantics():
    world = 2
    port = 29500 + (os.getpid() % 1000)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, same, ok_sum, skips in res:
        assert same, "ranks derived different all-reduce plans"
        assert ok_sum, "bucketed sum of pre-divided gradients != mean gradient"
        assert skips == [1, 1], "overflow decision differs across ranks"


def _ga_worker(rank, world, port, ga, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = TINY
        plan = _plan(cfg, 1 << 20)
        _, n = _arena(cfg)
        rng = np.random.default_rng(200 + rank)
        micro = [rng.standard_normal(n).astype(np.float32) for _ in range(ga)]   # per micro-step mean-loss grads

        def bucketed_allreduce(g):
            for _, b, e in plan:
                seg = g[b:e].clone()
                dist.all_reduce(seg, op=dist.ReduceOp.SUM)
                g[b:e] = seg

        def run(sync_of):
            acc = torch.zeros(n)
            for k in range(ga):
                acc += torch.from_numpy(micro[k]) / (world * ga)   # backward factor 1/GA, seed pre-divided by world
                if sync_of(k):
                    bucketed_allreduce(acc)
            return acc

        fixed = run(lambda k: k == ga - 1)          # rbk_model_train: sync only on the last micro-step
        every = run(lambda k: True)                 # the schedule without the sync switch
        allm = [torch.zeros(ga, n) for _ in range(world)]
        dist.all_gather(allm, torch.from_numpy(np.stack(micro)))
        expect = torch.stack(allm).mean(dim=(0, 1))
        q.put((rank, bool(torch.allclose(fixed, expect, rtol=1e-5, atol=1e-6)),
               bool(torch.allclose(every, expect, rtol=1e-3, atol=1e-4))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("ga", [2, 4])
def test_two_rank_gloo_grad_accumulation_schedule(ga):
    world = 2
    port = 29700 + (os.getpid() % 1000) + ga
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_ga_worker, args=(r, world, port, ga, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, fixed_ok, every_ok in res:
        assert fixed_ok, "sync-on-last-micro-step schedule does not give the mean gradient"
        assert not every_ok, "the per-micro-step all-reduce should over-weight earlier micro-steps"


GPT13 = dict(V=50257, T=2048, D=2048, H=16, L=24, FF=8192)


@pytest.mark.parametrize("world", [2, 4, 8, 16])
@pytest.mark.parametrize("cfg,bucket_mb", [(GPT2S, 25), (GPT13, 25), (TINY, 1)])
def test_plan_buckets_split_into_optimizer_shards(cfg, bucket_mb, world):
    """The sharded optimizer gives rank r the r-th 1/world slice of every bucket; the slices
    must start and end on 4-element boundaries (16-byte vectors of the tail kernel)."""
    plan = _plan(cfg, bucket_mb << 20)
    assert all((e - b) % (4 * world) == 0 for _, b, e in plan)


def _adam(p, g, m, v, f, lr=1e-3, b1=0.9, b2=0.999, eps=1e-8, wd=0.1, t=1):
    """L2-coupled AdamW as the tail applies it (src/cpu_mat.h:280-292), gradient factor f."""
    gi = g * f + wd * p
    m = b1 * m + (1 - b1) * gi
    v = b2 * v + (1 - b2) * gi * gi
    return p - lr * (m / (1 - b1 ** t)) / (np.sqrt(v / (1 - b2 ** t)) + eps), m, v


def _shard_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = TINY
        plan = _plan(cfg, 1 << 20)
        table, n = _arena(cfg)
        rng = np.random.default_rng(7)
        p0 = rng.standard_normal(n).astype(np.float64) * 0.02
        grads = [np.random.default_rng(50 + r).standard_normal(n) for r in range(world)]
        full = np.sum(grads, axis=0)                          # what the all-reduce gives every rank
        max_norm = 0.5
        # the plain path: every rank clips each tensor by its own norm and updates everything
        fac = np.ones(n)
        for _, off, r, c in table:
            nrm = np.linalg.norm(full[off:off + r * c])
            if nrm > max_norm:
                fac[off:off + r * c] = max_norm / nrm
        ref, _, _ = _adam(p0, full, np.zeros(n), np.zeros(n), fac)
        # the sharded path: reduce-scatter per bucket (this rank's slice of the sum), per-tensor
        # sums of squares over the slice, one all-reduce of those sums, the update on the slice,
        # then an all-gather of the slices
        own = []
        g = torch.from_numpy(grads[rank].copy())
        for _, b, e in plan:
            seg = g[b:e].clone()
            dist.all_reduce(seg, op=dist.ReduceOp.SUM)             # stands in for reduce-scatter
            cnt = (e - b) // world
            own.append((b + rank * cnt, b + (rank + 1) * cnt))
            g[b:e] = 0
            g[b + rank * cnt:b + (rank + 1) * cnt] = seg[rank * cnt:(rank + 1) * cnt]
        g = g.numpy()
        sums = np.zeros(len(table))
        for k, (_, off, r, c) in enumerate(table):
            for b, e in own:
                lo, hi = max(b, off), min(e, off + r * c)
                if lo < hi:
                    sums[k] += float(np.sum(g[lo:hi] ** 2))
        ts = torch.from_numpy(sums)
        dist.all_reduce(ts, op=dist.ReduceOp.SUM)
        fac = np.ones(n)
        for k, (_, off, r, c) in enumerate(table):
            nrm = np.sqrt(float(ts[k]))
            if nrm > max_norm:
                fac[off:off + r * c] = max_norm / nrm
        p = p0.copy()
        for b, e in own:
            p[b:e], _, _ = _adam(p0[b:e], g[b:e], np.zeros(e - b), np.zeros(e - b), fac[b:e])
        mine = torch.zeros(n, dtype=torch.float64)
        for b, e in own:
            mine[b:e] = torch.from_numpy(p[b:e])
        allp = [torch.zeros(n, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(allp, mine)                               # stands in for the all-gather
        gathered = torch.stack(allp).sum(0).numpy()               # the slices are disjoint
        q.put((rank, float(np.max(np.abs(gathered - ref)))))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharded_optimizer_schedule():
    """The sharded optimizer's schedule (bucketed reduce-scatter, per-tensor clip sums exchanged,
    the update on each rank's slices, all-gather) gives the same weights as all-reducing and
    updating the whole arena on every rank."""
    import socket
    world = 2
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_shard_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for _, err in res:
        assert err < 1e-12
