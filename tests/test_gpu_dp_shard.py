"""The sharded optimizer on two GPUs (skipped with fewer).

With `dp_init(..., shard=True)` each gradient bucket is reduce-scattered, so
rank r holds the summed gradients of the r-th half of every bucket; the fused
tail runs in two launches over those slices with one small all-reduce between
them (the overflow flag and the per-tensor sums of squares of the clip), and
the updated FP16 weights are all-gathered bucket by bucket while the next
forward waits for each bucket before its first use.

The same runs are made with the plain all-reduce path (every rank updates the
whole arena) and compared.  Without clipping (three optimizer steps of the
device trainer loop with two micro-steps each and weight decay, then a
host-driven forward / backward / optimizer step) the two paths apply the same
per-element arithmetic to the same reduced gradients, so masters, moments and
FP16 weights agree bit for bit.  With per-tensor clipping the sums of squares
are added in another order (per rank, then across ranks), so one step agrees
to FP32 rounding (later steps would carry those roundings through FP16 weight
roundings into the next gradients).  Also checked: the FP16 weights are
bit-identical on both ranks; each rank's slices tile the arena; an overflow on
one rank makes both skip.  The runs are in deterministic mode (split-K weight
gradients added in a fixed order), so both paths see bit-identical gradients.
NVLS is off, as for every multi-rank test here.
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
B_RANK, S, WORLD, GA, STEPS = 2, 128, 2, 2, 3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, outdir):
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    from rbk.model import ModelConfig, RubidiumTransformer, dp_unique_id
    rng = np.random.default_rng(9)
    toks = rng.integers(0, CFG["V"], 16384).astype(np.int32)
    starts = rng.integers(0, toks.size - S - 1, (WORLD, STEPS * GA * B_RANK)).astype(np.int64)
    d_toks = torch.from_numpy(toks).cuda()
    brng = np.random.default_rng(rank + 20)
    t = torch.from_numpy(brng.integers(0, CFG["V"], (B_RANK, S)).astype(np.int32)).cuda()
    g = torch.from_numpy(brng.integers(0, CFG["V"], (B_RANK, S)).astype(np.int32)).cuda()
    out = {}
    # name, sharded, clip, trainer-loop steps, host-driven step after the loop
    runs = (("full", False, 0.0, STEPS, True), ("shard", True, 0.0, STEPS, True),
            ("fullc", False, 0.5, 1, False), ("shardc", True, 0.5, 1, False))
    for name, shard, clip, steps, host_step in runs:
        m = RubidiumTransformer(ModelConfig(**CFG), max_batch=B_RANK, max_seq=S)
        m.init_weights(seed=11, std=0.02)
        uid = [dp_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(uid, src=0)
        m.dp_init(rank, world, uid[0], bucket_bytes=1 << 20, shard=shard)
        if name == "shard":
            out["ranges"] = np.array(m.dp_shard_ranges(), dtype=np.int64)
        losses = m.train(d_toks, steps=steps, ga=GA, B=B_RANK, T=S, starts=starts[rank][:steps * GA * B_RANK],
                         lr=1e-3, wd=0.1, clip=clip)
        if host_step:
            # a host-driven step after the loop: its forward waits for the all-gathered weights
            m.forward(t, g, B_RANK, S)
            m.backward(t, g, B_RANK, S)
            m.optimizer_step(steps + 1, 1e-3, wd=0.1)
            out[f"{name}_loss4"] = m.forward(t, g, B_RANK, S).item()
        torch.cuda.synchronize()
        out[f"{name}_losses"] = np.array(losses)
        out[f"{name}_p16"] = m.p16.cpu().numpy().copy()
        m.dp_gather_state()
        torch.cuda.synchronize()
        out[f"{name}_p32"] = m.p32.cpu().numpy().copy()
        out[f"{name}_m"] = m._bufs[3].cpu().numpy().copy()
        out[f"{name}_v"] = m._bufs[4].cpu().numpy().copy()
        if name == "shard":
            # an overflow on rank 1 only: the exchanged flag makes both ranks skip
            if rank == 1:
                m.inject_inf(0, 1 << 30)
            m.forward(t, g, B_RANK, S)
            m.backward(t, g, B_RANK, S)
            out["scale_before"] = m.loss_scale
            p_before = m.p16.clone()
            m.optimizer_step(STEPS + 2, 1e-3)
            m.forward(t, g, B_RANK, S)
            torch.cuda.synchronize()
            out["skipped"] = m.scaler().skipped
            out["scale_after"] = m.loss_scale
            out["p16_unchanged"] = bool(torch.equal(p_before, m.p16))
        m.dp_shutdown()
        m.close()
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), **out)
    dist.barrier()
    dist.destroy_process_group()


@pytest.fixture(scope="module")
def ranks(tmp_path_factory):
    import torch.multiprocessing as mp
    d = tmp_path_factory.mktemp("dpshard")
    saved = {k: os.environ.get(k) for k in ("NCCL_NVLS_ENABLE", "RBK_DETERMINISTIC")}
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    os.environ["RBK_DETERMINISTIC"] = "1"
    try:
        mp.spawn(_worker, args=(WORLD, _free_port(), str(d)), nprocs=WORLD, join=True)
    finally:
        for k, v in saved.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    return [dict(np.load(d / f"rank{r}.npz")) for r in range(WORLD)]


def _rel(a, b):
    return float(np.linalg.norm(a.astype(np.float64) - b) / max(np.linalg.norm(b.astype(np.float64)), 1e-30))


def test_shard_ranges_tile_the_arena(ranks):
    from rbk.model import ModelConfig, param_table
    _, n = param_table(ModelConfig(**CFG))
    r0, r1 = ranks
    both = sorted([tuple(x) for x in r0["ranges"]] + [tuple(x) for x in r1["ranges"]])
    assert both[0][0] == 0 and both[-1][1] == n
    for (_, e0), (b1, _) in zip(both, both[1:]):
        assert e0 == b1, "slices leave a gap or overlap"
    for rg in (r0["ranges"], r1["ranges"]):
        assert all(b % 4 == 0 and (e - b) % 4 == 0 and e > b for b, e in rg)


def test_shard_weights_identical_on_both_ranks(ranks):
    r0, r1 = ranks
    for k in ("full_p16", "shard_p16", "shard_p32", "shard_m", "shard_v", "shardc_p16", "shardc_p32"):
        assert np.array_equal(r0[k], r1[k]), k


def test_shard_matches_plain_all_reduce_bitwise(ranks):
    r0, _ = ranks
    assert np.array_equal(r0["shard_losses"], r0["full_losses"])
    assert float(r0["shard_loss4"]) == float(r0["full_loss4"])
    for k in ("p16", "p32", "m", "v"):
        assert np.array_equal(r0[f"shard_{k}"], r0[f"full_{k}"]), k


def test_shard_with_clip_matches_plain_to_rounding(ranks):
    r0, _ = ranks
    assert np.array_equal(r0["shardc_losses"], r0["fullc_losses"])   # the loss precedes the update
    assert _rel(r0["shardc_p32"], r0["fullc_p32"]) < 1e-6
    assert _rel(r0["shardc_m"], r0["fullc_m"]) < 1e-5
    assert _rel(r0["shardc_v"], r0["fullc_v"]) < 1e-5
    h = r0["shardc_p16"].astype(np.float32) != r0["fullc_p16"].astype(np.float32)
    assert np.count_nonzero(h) <= 1e-3 * h.size              # FP16 roundings that an ulp of FP32 flips


def test_shard_overflow_on_one_rank_skips_everywhere(ranks):
    r0, r1 = ranks
    assert int(r0["skipped"]) == int(r1["skipped"]) == 1
    assert float(r0["scale_after"]) == float(r1["scale_after"]) < float(r0["scale_before"])
    assert bool(r0["p16_unchanged"]) and bool(r1["p16_unchanged"])
