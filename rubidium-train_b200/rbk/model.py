"""RubidiumTransformer drop-in (reference src/model.h:112-139) over librbk.

The model, its arenas and activations live in librbk (C++/CUDA); this class
keeps the reference's method names and argument meaning:

    m = RubidiumTransformer(ModelConfig(V, T, D, H, L, FF), max_batch=B)
    loss = m.forward(tokens, targets, B, T)            # device FP32 scalar
    m.backward(tokens, targets, B, T, loss_scale=1.0)  # reference's upstream factor
    m.clip_gradients(1.0)                              # applied inside the fused tail
    m.optimizer_step(t, lr, b1, b2, eps, wd)

Weights / masters / gradients / moments are exposed as zero-copy torch views
of the device arenas (include/rbk_layout.h order), by tensor name.
"""
from __future__ import annotations

import contextlib
import ctypes as C
from dataclasses import dataclass

import torch

from ._lib import Config, DpOpts, ModelOpts, Scaler, TrainArgs, call, lib
from .ops import _s

BUF_P16, BUF_P32, BUF_GRAD, BUF_M, BUF_V, BUF_LOSS, BUF_LOGITS = range(7)
LAYER_NAMES = ["ln1_w", "ln1_b", "wq", "wk", "wv", "bq", "bk", "bv", "wo", "bo",
               "ln2_w", "ln2_b", "w1", "b1", "w2", "b2"]


@dataclass
class ModelConfig:
    """ModelConfig (src/model.h:16-24)."""
    V: int
    T: int
    D: int
    H: int
    L: int
    FF: int
    use_fp16: bool = True
    use_activation_checkpointing: bool = True
    grad_accum_steps: int = 1

    @property
    def hd(self) -> int:
        return self.D // self.H


class _DevArray:
    """__cuda_array_interface__ over a raw device pointer (zero copy)."""

    def __init__(self, ptr: int, n: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


def _view(ptr: int, n: int, dtype) -> torch.Tensor:
    ts = {torch.float32: "<f4", torch.float16: "<f2", torch.int32: "<i4"}[dtype]
    return torch.as_tensor(_DevArray(ptr, n, ts), device="cuda")


def param_table(cfg: ModelConfig):
    """[(name, offset, rows, cols)] in arena order — same as include/rbk_layout.h."""
    def rnd(x):
        return (x + 63) // 64 * 64
    V, T, D, L, F = cfg.V, cfg.T, cfg.D, cfg.L, cfg.FF
    shapes = [("token_emb", V, D), ("pos_emb", T, D)]
    for l in range(L):
        for n in LAYER_NAMES:
            r, c = {"wq": (D, D), "wk": (D, D), "wv": (D, D), "wo": (D, D), "w1": (F, D), "w2": (D, F),
                    "b1": (1, F)}.get(n, (1, D))
            shapes.append((f"layers.{l}.{n}", r, c))
    shapes += [("ln_f_w", 1, D), ("ln_f_b", 1, D), ("lm_w", V, D), ("lm_b", 1, V)]
    out, off = [], 0
    for name, r, c in shapes:
        out.append((name, off, r, c))
        off += rnd(r * c)
    return out, off


class RubidiumTransformer:
    def __init__(self, cfg: ModelConfig, max_batch: int, max_seq: int | None = None, init_loss_scale=65536.0,
                 growth_interval=2000, device: int | None = None):
        self.cfg = cfg
        device = torch.cuda.current_device() if device is None else device
        self.max_batch = max_batch
        self.max_seq = max_seq or cfg.T
        c = Config(cfg.V, cfg.T, cfg.D, cfg.H, cfg.L, cfg.FF)
        o = ModelOpts(max_batch, self.max_seq, int(cfg.use_activation_checkpointing), init_loss_scale,
                      growth_interval, device)
        h = C.c_void_p()
        call("rbk_model_create", C.byref(h), C.byref(c), C.byref(o))
        self.handle = h
        self.table, self.nparams = param_table(cfg)
        self._names = {n: (off, r, c) for n, off, r, c in self.table}
        self._bufs = {}
        for which, dt in ((BUF_P16, torch.float16), (BUF_P32, torch.float32), (BUF_GRAD, torch.float32),
                          (BUF_M, torch.float32), (BUF_V, torch.float32), (BUF_LOSS, torch.float32),
                          (BUF_LOGITS, torch.float16)):
            p, n = C.c_void_p(), C.c_int64()
            call("rbk_model_buffer", self.handle, which, C.byref(p), C.byref(n))
            self._bufs[which] = _view(p.value, n.value, dt)
        assert self._bufs[BUF_P32].numel() == self.nparams
        sp = C.c_void_p()
        call("rbk_model_scaler", self.handle, C.byref(sp))
        self._scaler = _view(sp.value, 8, torch.int32)
        self._pending_clip = 0.0
        self.lora_rank = 0

    # ----------------------------------------------------------- buffers --
    @property
    def p16(self):
        return self._bufs[BUF_P16]

    @property
    def p32(self):
        return self._bufs[BUF_P32]

    @property
    def grad(self):
        return self._bufs[BUF_GRAD]

    @property
    def loss_buffer(self):
        return self._bufs[BUF_LOSS]

    def tensor(self, name: str, which: str = "p32") -> torch.Tensor:
        off, r, c = self._names[name]
        buf = {"p16": BUF_P16, "p32": BUF_P32, "grad": BUF_GRAD, "m": BUF_M, "v": BUF_V}[which]
        t = self._bufs[buf][off:off + r * c]
        return t.view(r, c) if r > 1 else t

    def scaler(self) -> Scaler:
        return Scaler.from_buffer_copy(self._scaler.cpu().numpy().tobytes())

    @property
    def loss_scale(self) -> float:
        return self.scaler().scale

    # --------------------------------------------------------- reference API --
    def load_params(self, params32: torch.Tensor):
        """Set the FP32 masters (arena order) and refresh the FP16 weights."""
        self.p32.copy_(params32.to(self.p32.device, torch.float32))
        self.convert_weights_fp32_to_fp16()

    def convert_weights_fp32_to_fp16(self):
        call("rbk_model_sync_fp16", self.handle, _s())

    def save(self, path: str, char_map=None):
        """save (src/model.h:136): RBN2 file plus masters, Adam moments and scaler (rbk_model_save)."""
        cm = None
        if char_map is not None:
            cm = C.cast((C.c_int * 256)(*[int(x) for x in char_map]), C.c_void_p)
        call("rbk_model_save", self.handle, str(path).encode(), cm, _s())

    def load(self, path: str):
        """load (src/model.h:137): restores weights and, when the file has them, masters, moments
        and scaler; returns the file's 256-entry character map."""
        cm = (C.c_int * 256)()
        call("rbk_model_load", self.handle, str(path).encode(), C.cast(cm, C.c_void_p), _s())
        return list(cm)

    def train(self, tokens, steps, ga, B, T=None, starts=None, seed=0, first_step=1, max_steps=None, warmup=0,
              lr=3e-4, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, clip=0.0, grad_scale=None):
        """The reference trainer loop (src/main.cpp:125-175) on the device (rbk_model_train).
        tokens: device int32 token stream; starts: optional host int64 window starts
        [steps * ga * B]; grad_scale defaults to 1 / ga (the mean of the micro-batch mean
        losses; the reference passes 1 / (B * ga)).  Returns the per-step mean losses."""
        import numpy as np
        T = T or self.max_seq
        a = TrainArgs()
        a.tokens, a.n_tokens = tokens.data_ptr(), tokens.numel()
        st = None
        if starts is not None:
            st = np.ascontiguousarray(np.asarray(starts, dtype=np.int64))
            a.starts = st.ctypes.data
        a.seed = seed
        a.steps, a.ga, a.B, a.T, a.first_step = steps, ga, B, T, first_step
        a.max_steps = max_steps if max_steps is not None else first_step + steps - 1
        a.warmup = warmup
        a.lr, a.b1, a.b2, a.eps, a.wd, a.clip = lr, b1, b2, eps, wd, clip
        a.grad_scale = 1.0 / ga if grad_scale is None else grad_scale
        out = (C.c_float * steps)()
        a.losses = C.cast(out, C.c_void_p)
        call("rbk_model_train", self.handle, C.byref(a), _s())
        return list(out)

    def init_weights(self, seed=42, std=0.02):
        call("rbk_model_init_weights", self.handle, C.c_uint64(seed), C.c_float(std), _s())

    def forward(self, tokens, targets=None, B=None, T=None, loss_out=None):
        """Returns the device FP32 mean loss (a view; copy before the next call)."""
        B = B or tokens.shape[0]
        T = T or tokens.shape[-1]
        out = self.loss_buffer if loss_out is None else loss_out
        call("rbk_model_forward", self.handle, C.c_void_p(tokens.data_ptr()),
             C.c_void_p(targets.data_ptr()) if targets is not None else None, B, T, C.c_void_p(out.data_ptr()), _s())
        return out

    def backward(self, tokens, targets, B=None, T=None, loss_scale=1.0):
        B = B or tokens.shape[0]
        T = T or tokens.shape[-1]
        call("rbk_model_backward", self.handle, C.c_void_p(tokens.data_ptr()), C.c_void_p(targets.data_ptr()), B, T,
             C.c_float(loss_scale), _s())

    def set_deterministic(self, on: bool = True):
        """Bitwise-reproducible backward on this model's context (rbk_ctx_set_deterministic):
        ordered split-K weight gradients and ordered dQ additions in the attention backward."""
        ctx = C.c_void_p()
        call("rbk_model_ctx", self.handle, C.byref(ctx))
        call("rbk_ctx_set_deterministic", ctx, int(bool(on)))

    def set_training(self, training: bool = True):
        """Training mode: forward also writes dlogits (one pass over the logits);
        eval mode keeps the logits intact."""
        call("rbk_model_set_training", self.handle, int(bool(training)))

    def clip_gradients(self, max_norm: float):
        """Per-tensor clip (src/model.cu:493-523), fused into the next optimizer_step."""
        self._pending_clip = float(max_norm)

    def optimizer_step(self, t, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0):
        clip, self._pending_clip = self._pending_clip, 0.0
        call("rbk_model_optimizer_step", self.handle, int(t), C.c_float(lr), C.c_float(b1), C.c_float(b2),
             C.c_float(eps), C.c_float(wd), C.c_float(clip), _s())

    def update_loss_scale(self, overflow: bool):
        """Kept for API parity: the scaler is updated on the device by the fused tail."""
        return None

    # -------------------------------------------------------------- LoRA --
    def init_lora(self, rank=16, alpha=32.0, seed=7):
        call("rbk_model_lora_enable", self.handle, rank, C.c_float(alpha), C.c_uint64(seed), _s())
        self.lora_rank = rank
        self._lora = {}
        for which, dt in ((BUF_P16, torch.float16), (BUF_P32, torch.float32), (BUF_GRAD, torch.float32),
                          (BUF_M, torch.float32), (BUF_V, torch.float32)):
            p, n = C.c_void_p(), C.c_int64()
            call("rbk_model_lora_buffer", self.handle, which, C.byref(p), C.byref(n))
            self._lora[which] = _view(p.value, n.value, dt)

    def lora_tensors(self, which="p32"):
        """(Aq [L,D,r], Bq [L,r,D], Av [L,D,r], Bv [L,r,D]) views."""
        buf = self._lora[{"p16": BUF_P16, "p32": BUF_P32, "grad": BUF_GRAD, "m": BUF_M, "v": BUF_V}[which]]
        L, D, r = self.cfg.L, self.cfg.D, self.lora_rank
        s = L * D * r
        return (buf[:s].view(L, D, r), buf[s:2 * s].view(L, r, D), buf[2 * s:3 * s].view(L, D, r),
                buf[3 * s:].view(L, r, D))

    def lora_sync_fp16(self):
        p16 = self._lora[BUF_P16]
        p16.copy_(self._lora[BUF_P32].half())

    def lora_optimizer_step(self, t, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0):
        call("rbk_model_lora_step", self.handle, int(t), C.c_float(lr), C.c_float(b1), C.c_float(b2),
             C.c_float(eps), C.c_float(wd), _s())

    def inject_inf(self, offset: int, stride: int):
        call("rbk_model_inject_inf", self.handle, C.c_int64(offset), C.c_int64(stride))

    # ------------------------------------------------------ data parallel --
    def dp_init(self, rank: int, world: int, unique_id: bytes, bucket_bytes: int = 25 << 20, max_ctas=None,
                timeout_s=None, shard=None):
        """Join the NCCL communicator (rbk_model_dp_init_ex).  max_ctas caps NCCL's CTAs for the
        buckets that overlap the backward; timeout_s is the watchdog's deadline per collective;
        shard selects the sharded optimizer (reduce-scatter, the tail on this rank's slices, FP16
        all-gather).  None: the library defaults (environment RBK_NCCL_MAX_CTAS /
        RBK_NCCL_TIMEOUT_S / RBK_DP_SHARD)."""
        import os
        buf = C.create_string_buffer(unique_id, 128)
        o = DpOpts()
        o.bucket_bytes = bucket_bytes
        o.max_ctas = int(os.environ.get("RBK_NCCL_MAX_CTAS", "0")) if max_ctas is None else int(max_ctas)
        o.timeout_s = float(os.environ.get("RBK_NCCL_TIMEOUT_S", "300")) if timeout_s is None else float(timeout_s)
        o.shard_optimizer = int(os.environ.get("RBK_DP_SHARD", "0")) if shard is None else int(bool(shard))
        call("rbk_model_dp_init_ex", self.handle, buf, rank, world, C.byref(o))

    def dp_shard_ranges(self):
        """[(begin, end), ...] arena ranges this rank updates under the sharded optimizer ([] if not)."""
        n = C.c_int()
        call("rbk_model_dp_shard_ranges", self.handle, None, 0, C.byref(n))
        out = (C.c_int64 * (2 * n.value + 2))()
        call("rbk_model_dp_shard_ranges", self.handle, out, n.value, C.byref(n))
        return [(out[2 * i], out[2 * i + 1]) for i in range(n.value)]

    def zero_grad(self):
        """Zero the gradient arena (rbk_model_zero_grad); the next backward then stores its weight
        gradients instead of adding to them."""
        call("rbk_model_zero_grad", self.handle, _s())

    def dp_gather_state(self):
        """Sharded optimizer: all-gather the FP32 masters and Adam moments (every rank whole again)."""
        call("rbk_model_dp_gather_state", self.handle, _s())

    def dp_abort(self):
        """Abort this rank's communicators locally (a rank leaving the job)."""
        call("rbk_model_dp_abort", self.handle)

    def dp_status(self) -> int:
        """0, or the status (RBK_ERR_TIMEOUT -4 / RBK_ERR_NCCL -5) after the watchdog aborted."""
        return lib().rbk_model_dp_status(self.handle)

    def dp_set_sync(self, sync: bool):
        """sync False: following backwards only accumulate this rank's gradients (the first
        GA - 1 micro-steps of a step); True (default): backward all-reduces the accumulated
        arena bucket by bucket (the last micro-step)."""
        call("rbk_model_dp_set_sync", self.handle, int(bool(sync)))

    @contextlib.contextmanager
    def no_sync(self):
        """Backwards inside the block skip the all-reduce (gradient accumulation)."""
        self.dp_set_sync(False)
        try:
            yield
        finally:
            self.dp_set_sync(True)

    def dp_shutdown(self):
        call("rbk_model_dp_shutdown", self.handle)

    def close(self):
        if getattr(self, "handle", None):
            lib().rbk_model_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def dp_plan(cfg: ModelConfig, bucket_bytes: int = 25 << 20):
    """The gradient all-reduce schedule librbk uses: [(unit, begin, end)] (host only)."""
    c = Config(cfg.V, cfg.T, cfg.D, cfg.H, cfg.L, cfg.FF)
    cnt = C.c_int()
    call("rbk_dp_plan", C.byref(c), C.c_int64(bucket_bytes), None, 0, C.byref(cnt))
    buf = (C.c_int64 * (3 * cnt.value))()
    call("rbk_dp_plan", C.byref(c), C.c_int64(bucket_bytes), buf, cnt.value, C.byref(cnt))
    return [(buf[3 * i], buf[3 * i + 1], buf[3 * i + 2]) for i in range(cnt.value)]


def dp_unique_id() -> bytes:
    buf = C.create_string_buffer(128)
    call("rbk_dp_unique_id", buf)
    return buf.raw
