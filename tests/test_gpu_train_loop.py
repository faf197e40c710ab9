"""rbk_model_train: the reference trainer loop (src/main.cpp:125-175) run on the device against
the same loop driven step by step from the host, and a split run against an uninterrupted one."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CFG1 = dict(V=4096, T=128, D=256, H=4, L=4, FF=1024)
B, T = 4, 128


def _model(seed=21):
    from rbk.model import ModelConfig, RubidiumTransformer
    m = RubidiumTransformer(ModelConfig(**CFG1), max_batch=B, max_seq=T)
    m.init_weights(seed=seed)
    return m


def _stream(n=20000, seed=3):
    g = torch.Generator(device="cuda").manual_seed(seed)
    return torch.randint(0, CFG1["V"], (n,), device="cuda", generator=g, dtype=torch.int32)


def _lr(step, lr, warmup, max_steps):                 # src/main.cpp:127-131
    if step < warmup:
        return lr * step / warmup
    p = (step - warmup) / (max_steps - warmup) if max_steps > warmup else 0.0
    return lr * 0.5 * (1.0 + math.cos(3.14159265 * p))


def _rel(a, b):
    return float(np.linalg.norm(a - b) / np.linalg.norm(b))


def test_device_loop_matches_host_driven_loop():
    steps, ga, warmup, lr, clip = 3, 2, 2, 1e-3, 1.0
    stream = (torch.arange(20000, device="cuda", dtype=torch.int32) * 7) % 61   # learnable: periodic
    rng = np.random.default_rng(4)
    starts = rng.integers(0, stream.numel() - T - 1, steps * ga * B).astype(np.int64)
    a = _model()
    la = a.train(stream, steps, ga, B, T, starts=starts, warmup=warmup, max_steps=steps, lr=lr, clip=clip,
                 grad_scale=1.0 / (B * ga))
    b = _model()
    lb = []
    idx = torch.arange(T, device="cuda")
    for s in range(steps):
        acc = 0.0
        for g in range(ga):
            o = torch.from_numpy(starts[(s * ga + g) * B:(s * ga + g + 1) * B]).cuda()
            win = o[:, None] + idx[None, :]
            tok, tgt = stream[win].contiguous(), stream[win + 1].contiguous()
            acc += b.forward(tok, tgt, B, T).item()
            b.backward(tok, tgt, B, T, loss_scale=1.0 / (B * ga))
        b.clip_gradients(clip)
        b.optimizer_step(s + 1, _lr(s + 1, lr, warmup, steps))
        lb.append(acc / ga)
    assert np.allclose(la, lb, rtol=1e-5, atol=0), (la, lb)
    assert _rel(a.p32.cpu().numpy(), b.p32.cpu().numpy()) < 1e-5
    assert a.scaler().applied_steps == b.scaler().applied_steps == steps
    assert la[-1] < la[0] - 0.1                        # the periodic stream is learnt
    a.close()
    b.close()


def test_split_run_equals_uninterrupted_run():
    """Device-drawn windows depend on the run-wide sample index, so steps 1-2 then 3-4 draw what
    steps 1-4 draw; Adam's t and the LR schedule follow first_step."""
    stream = _stream(seed=8)
    kw = dict(seed=7, warmup=1, max_steps=4, lr=5e-4)
    a = _model()
    la = a.train(stream, 4, 2, B, T, **kw)
    b = _model()
    lb = b.train(stream, 2, 2, B, T, first_step=1, **kw) + b.train(stream, 2, 2, B, T, first_step=3, **kw)
    assert np.allclose(la, lb, rtol=1e-5, atol=0), (la, lb)
    assert _rel(a.p32.cpu().numpy(), b.p32.cpu().numpy()) < 1e-5
    c = _model()
    lc = c.train(stream, 4, 2, B, T, **dict(kw, seed=8))   # another seed draws other windows
    assert lc[1:] != la[1:]
    for m in (a, b, c):
        m.close()


def test_bad_window_starts_are_rejected():
    from rbk._lib import RbkError
    stream = _stream(n=1000)
    m = _model()
    starts = np.zeros(B, np.int64)
    starts[2] = 1000 - T                              # one past the last valid start
    with pytest.raises(RbkError) as e:
        m.train(stream, 1, 1, B, T, starts=starts)
    assert e.value.status == -1 and "index 2" in str(e.value)
    m.close()
