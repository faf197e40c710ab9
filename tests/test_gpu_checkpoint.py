"""Checkpoints on the GPU: rbk_model_save / rbk_model_load against the host-side reader and
writer (rbk.checkpoint), and a resumed run that continues exactly where the saved one stopped."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

CFG1 = dict(V=4096, T=128, D=256, H=4, L=4, FF=1024)
B, S = 4, 128


def _model(seed):
    from rbk.model import ModelConfig, RubidiumTransformer
    m = RubidiumTransformer(ModelConfig(**CFG1), max_batch=B, max_seq=S)
    m.init_weights(seed=seed)
    return m


def _batch(seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    tt = torch.randint(0, CFG1["V"], (B, S), device="cuda", generator=g, dtype=torch.int32)
    tg = torch.randint(0, CFG1["V"], (B, S), device="cuda", generator=g, dtype=torch.int32)
    return tt, tg


def _step(m, t, batch):
    tt, tg = batch
    loss = m.forward(tt, tg, B, S).item()
    m.backward(tt, tg, B, S)
    m.optimizer_step(t, 3e-4, 0.9, 0.999, 1e-8, 0.01)
    return loss


def _np(t):
    return t.detach().cpu().numpy()


def test_save_load_resume(tmp_path):
    from rbk import checkpoint as ckpt
    a = _model(seed=11)
    for t in (1, 2):
        _step(a, t, _batch(t))
    path = tmp_path / "a.rbn2"
    cmap = list(range(1000, 1256))
    a.save(path, char_map=cmap)

    # the file, read on the host, holds exactly the device state
    ck = ckpt.read(path)
    assert ck.config == tuple(CFG1[k] for k in ("V", "T", "D", "H", "L", "FF"))
    assert list(ck.char_map) == cmap
    sa = a.scaler()
    assert ck.scaler["scale"] == sa.scale and ck.scaler["applied_steps"] == sa.applied_steps == 2
    for name, _, _ in ckpt.file_tensors(*ck.config):
        assert np.array_equal(ck.weights16[name].view(np.uint16), _np(a.tensor(name, "p16")).view(np.uint16)), name
        for fam, which in ((ck.masters, "p32"), (ck.adam_m, "m"), (ck.adam_v, "v")):
            assert np.array_equal(fam[name].view(np.uint32), _np(a.tensor(name, which)).view(np.uint32)), (name, which)

    # a second model (other weights) loads it bit for bit, gradients zeroed
    b = _model(seed=99)
    _step(b, 1, _batch(7))                            # leaves moments and a scaler state behind
    assert b.load(path) == cmap
    for name, _, _ in ckpt.file_tensors(*ck.config):
        for which in ("p16", "p32", "m", "v"):
            assert torch.equal(a.tensor(name, which), b.tensor(name, which)), (name, which)
    sb = b.scaler()
    assert (sb.scale, sb.unskipped, sb.applied_steps, sb.overflow_steps) == \
        (sa.scale, sa.unskipped, sa.applied_steps, sa.overflow_steps)
    assert torch.count_nonzero(b.grad).item() == 0

    # both continue with the same batch: same loss, same update (Adam's step count came along)
    la = _step(a, 0, _batch(3))                       # t <= 0: the tail uses applied_steps + 1
    lb = _step(b, 0, _batch(3))
    assert abs(la - lb) <= 1e-6 * abs(la)
    pa, pb = _np(a.p32), _np(b.p32)
    assert np.linalg.norm(pa - pb) <= 1e-6 * np.linalg.norm(pa)
    assert a.scaler().applied_steps == b.scaler().applied_steps == 3
    a.close()
    b.close()


def test_reference_layout_file_loads_with_fresh_optimizer(tmp_path):
    """A file with only the reference's RBN2 part: masters = FP32(FP16 weights), zero moments,
    a fresh scaler (src/model.cu:629-679 then convert_weights_fp16_to_fp32)."""
    from rbk import checkpoint as ckpt
    a = _model(seed=5)
    _step(a, 1, _batch(1))
    cfg = tuple(CFG1[k] for k in ("V", "T", "D", "H", "L", "FF"))
    w16 = {n: _np(a.tensor(n, "p16")) for n, _, _ in ckpt.file_tensors(*cfg)}
    path = tmp_path / "ref.rbn2"
    ckpt.write(path, ckpt.Checkpoint(cfg, np.arange(256, dtype=np.int32), w16))
    b = _model(seed=6)
    _step(b, 1, _batch(2))
    assert b.load(path) == list(range(256))
    for name in w16:
        assert torch.equal(b.tensor(name, "p16"), a.tensor(name, "p16")), name
        assert torch.equal(b.tensor(name, "p32"), a.tensor(name, "p16").float()), name
        assert torch.count_nonzero(b.tensor(name, "m")).item() == 0
        assert torch.count_nonzero(b.tensor(name, "v")).item() == 0
    st = b.scaler()
    assert st.scale == 65536.0 and st.applied_steps == 0 and st.unskipped == 0
    a.close()
    b.close()


def test_load_rejects_other_configs_and_missing_files(tmp_path):
    from rbk._lib import RbkError
    from rbk.model import ModelConfig, RubidiumTransformer
    a = _model(seed=1)
    path = tmp_path / "a.rbn2"
    a.save(path)
    other = RubidiumTransformer(ModelConfig(**dict(CFG1, L=2)), max_batch=B, max_seq=S)
    with pytest.raises(RbkError) as e:
        other.load(path)
    assert e.value.status == -1 and "L=4" in str(e.value)
    with pytest.raises(RbkError) as e:
        a.load(tmp_path / "missing.rbn2")
    assert e.value.status == -7
    data = open(path, "rb").read()
    (tmp_path / "cut.rbn2").write_bytes(data[:len(data) // 2])
    with pytest.raises(RbkError) as e:
        a.load(tmp_path / "cut.rbn2")
    assert e.value.status == -7
    other.close()
    a.close()


def test_cpp_trainer_resumes_from_its_checkpoint(tmp_path):
    """The C++ drop-in (include/rubidium/model.h) saves at the end of a run and a second run
    resumes from the file: the step count and the optimizer state continue."""
    import os
    import subprocess
    from rbk import checkpoint as ckpt
    exe = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "rubidium-train_b200", "bin",
                       "train_main")
    assert os.path.exists(exe), "build with make -C rubidium-train_b200 examples"
    a, b = str(tmp_path / "a.rbn2"), str(tmp_path / "b.rbn2")
    r1 = subprocess.run([exe, "2", "1"], env=dict(os.environ, RBK_SAVE=a), capture_output=True, text=True,
                        timeout=300)
    assert r1.returncode == 0, r1.stderr
    assert ckpt.read(a).scaler["applied_steps"] == 2
    r2 = subprocess.run([exe, "1", "1"], env=dict(os.environ, RBK_LOAD=a, RBK_SAVE=b), capture_output=True,
                        text=True, timeout=300)
    assert r2.returncode == 0, r2.stderr
    assert "2 steps applied" in r2.stdout and "step 3 " in r2.stdout, r2.stdout
    cb = ckpt.read(b)
    assert cb.scaler["applied_steps"] == 3
    assert any(np.any(cb.adam_v[n] != 0) for n in cb.adam_v)
