"""ctypes binding of librbk.so (the sm_100a library).  Loading fails loudly when
the library is missing: there is no CPU or PyTorch fallback for any op."""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
PKG_ROOT = os.path.dirname(_HERE)
LIB_PATH = os.path.join(PKG_ROOT, "lib", "librbk.so")

_lib = None

vp, i32, i64, f32 = C.c_void_p, C.c_int, C.c_int64, C.c_float


class RbkError(RuntimeError):
    """A librbk call returned a negative status."""

    def __init__(self, status: int, where: str, msg: str):
        super().__init__(f"{where} failed with status {status}: {msg}")
        self.status = status


class GemmDesc(C.Structure):
    _fields_ = [
        ("M", i32), ("N", i32), ("K", i32),
        ("A", vp), ("lda", i32), ("a_major", i32),
        ("B", vp), ("ldb", i32), ("b_major", i32),
        ("C", vp), ("ldc", i32),
        ("epilogue", i32),
        ("bias", vp), ("aux", vp), ("ld_aux", i32), ("aux_out", vp),
        ("dbias_rows", vp), ("alpha", f32), ("split_k", i32),
    ]


class Scaler(C.Structure):
    _fields_ = [("scale", f32), ("unskipped", i32), ("interval", i32), ("skipped", i32),
                ("applied_steps", i32), ("overflow_steps", i32), ("status", i32), ("pad", i32)]


class TailArgs(C.Structure):
    _fields_ = [
        ("p32", vp), ("g", vp), ("m", vp), ("v", vp), ("p16", vp), ("n", i64),
        ("seg_off", C.POINTER(i64)), ("seg_len", C.POINTER(i64)), ("nseg", i32), ("max_norm", f32),
        ("lr", f32), ("beta1", f32), ("beta2", f32), ("eps", f32), ("weight_decay", f32),
        ("t", i32), ("scaler", vp),
    ]


class Config(C.Structure):
    _fields_ = [("V", i32), ("T", i32), ("D", i32), ("H", i32), ("L", i32), ("FF", i32)]


class ModelOpts(C.Structure):
    _fields_ = [("max_batch", i32), ("max_seq", i32), ("use_activation_checkpointing", i32),
                ("init_loss_scale", f32), ("growth_interval", i32), ("device", i32)]


class DpOpts(C.Structure):
    """rbk_dp_opts (include/rbk.h)."""
    _fields_ = [("bucket_bytes", C.c_int64), ("max_ctas", C.c_int), ("timeout_s", C.c_double),
                ("shard_optimizer", C.c_int)]


class TrainArgs(C.Structure):
    """rbk_train_args (include/rbk.h)."""
    _fields_ = [("tokens", C.c_void_p), ("n_tokens", C.c_int64), ("starts", C.c_void_p), ("seed", C.c_uint64),
                ("steps", C.c_int), ("ga", C.c_int), ("B", C.c_int), ("T", C.c_int), ("first_step", C.c_int),
                ("max_steps", C.c_int), ("warmup", C.c_int), ("lr", C.c_float), ("b1", C.c_float),
                ("b2", C.c_float), ("eps", C.c_float), ("wd", C.c_float), ("clip", C.c_float),
                ("grad_scale", C.c_float), ("losses", C.c_void_p)]


_SIGS = {
    "rbk_last_error": (C.c_char_p, []),
    "rbk_version": (i32, []),
    "rbk_ctx_create": (i32, [C.POINTER(vp), i32]),
    "rbk_ctx_destroy": (i32, [vp]),
    "rbk_launch_count": (C.c_longlong, []),
    "rbk_ctx_profile": (i32, [vp, i32]),
    "rbk_ctx_profile_read": (i32, [vp, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(i32), i32]),
    "rbk_ctx_profile_read_gemm": (i32, [vp, C.POINTER(C.c_double), C.POINTER(C.c_double), C.POINTER(i32)]),
    "rbk_ctx_device_error": (i32, [vp, C.POINTER(i32)]),
    "rbk_ctx_set_deterministic": (i32, [vp, i32]),
    "rbk_ctx_arm_tail_timeout_test": (i32, [vp, C.c_double, i32]),
    "rbk_model_ctx": (i32, [vp, C.POINTER(vp)]),
    "rbk_ln_fwd": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, f32, vp]),
    "rbk_ln_bwd": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "rbk_ln_bwd_noalloc": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "rbk_softmax_xent_bwd": (i32, [vp, vp, vp, i32, vp, i32, i32, f32, vp, vp, vp]),
    "rbk_sum": (i32, [vp, vp, vp, i32, f32, vp]),
    "rbk_attn_softmax_bwd": (i32, [vp, vp, vp, vp, i32, i32, i32, vp]),
    "rbk_embed_fwd": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "rbk_embed_bwd": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]),
    "rbk_adam_tail": (i32, [vp, C.POINTER(TailArgs), vp]),
    "rbk_lora_fwd": (i32, [vp, vp, i32, vp, vp, i32, vp, vp, i32, i32, i32, i32, f32, vp]),
    "rbk_lora_bwd": (i32, [vp, vp, vp, vp, i32, vp, vp, i32, vp, i32, vp, vp, vp, i32, i32, i32, i32, f32, vp]),
    "rbk_lora_adam": (i32, [vp, C.POINTER(TailArgs), vp]),
    "rbk_gemm": (i32, [vp, C.POINTER(GemmDesc), vp]),
    "rbk_linear_fwd": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "rbk_gemm_dgrad": (i32, [vp, vp, vp, vp, i32, i32, i32, vp, vp]),
    "rbk_gemm_wgrad": (i32, [vp, vp, vp, vp, vp, i32, i32, i32, vp]),
    "rbk_attn_fwd": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, f32, vp]),
    "rbk_attn_bwd": (i32, [vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, f32, vp]),
    "rbk_model_create": (i32, [C.POINTER(vp), C.POINTER(Config), C.POINTER(ModelOpts)]),
    "rbk_model_destroy": (i32, [vp]),
    "rbk_model_buffer": (i32, [vp, i32, C.POINTER(vp), C.POINTER(i64)]),
    "rbk_model_scaler": (i32, [vp, C.POINTER(vp)]),
    "rbk_model_sync_fp16": (i32, [vp, vp]),
    "rbk_model_init_weights": (i32, [vp, C.c_uint64, f32, vp]),
    "rbk_model_save": (i32, [vp, C.c_char_p, vp, vp]),
    "rbk_model_load": (i32, [vp, C.c_char_p, vp, vp]),
    "rbk_model_train": (i32, [vp, C.POINTER(TrainArgs), vp]),
    "rbk_model_forward": (i32, [vp, vp, vp, i32, i32, vp, vp]),
    "rbk_model_backward": (i32, [vp, vp, vp, i32, i32, f32, vp]),
    "rbk_model_optimizer_step": (i32, [vp, i32, f32, f32, f32, f32, f32, f32, vp]),
    "rbk_model_lora_enable": (i32, [vp, i32, f32, C.c_uint64, vp]),
    "rbk_model_lora_buffer": (i32, [vp, i32, C.POINTER(vp), C.POINTER(i64)]),
    "rbk_model_lora_step": (i32, [vp, i32, f32, f32, f32, f32, f32, vp]),
    "rbk_model_inject_inf": (i32, [vp, i64, i64]),
    "rbk_model_set_training": (i32, [vp, i32]),
    "rbk_dp_unique_id": (i32, [vp]),
    "rbk_dp_plan": (i32, [C.POINTER(Config), i64, C.POINTER(i64), i32, C.POINTER(i32)]),
    "rbk_model_dp_init": (i32, [vp, vp, i32, i32, i64]),
    "rbk_model_dp_set_sync": (i32, [vp, i32]),
    "rbk_model_dp_init_ex": (i32, [vp, vp, i32, i32, C.POINTER(DpOpts)]),
    "rbk_model_dp_status": (i32, [vp]),
    "rbk_model_dp_abort": (i32, [vp]),
    "rbk_dp_init": (i32, [C.POINTER(vp), i32, vp, i32, i32, C.POINTER(DpOpts)]),
    "rbk_dp_bucket_ready": (i32, [vp, vp, i64, vp]),
    "rbk_dp_finish": (i32, [vp, vp]),
    "rbk_dp_status": (i32, [vp]),
    "rbk_dp_abort": (i32, [vp]),
    "rbk_dp_destroy": (i32, [vp]),
    "rbk_bpe_create": (i32, [C.POINTER(vp), i32, i32, vp, i64, vp, vp, vp, vp, vp, i32]),
    "rbk_bpe_destroy": (i32, [vp]),
    "rbk_bpe_num_rules": (i32, [vp]),
    "rbk_bpe_encode_batch": (i32, [vp, vp, i32, vp, vp, i32, vp]),
    "rbk_bpe_encode": (i32, [vp, vp, vp, vp, i32, vp, vp, i32, vp, vp]),
    "rbk_bpe_decode_batch": (i32, [vp, vp, i64, vp, i32, vp, i32, vp, vp]),
    "rbk_model_dp_shard_ranges": (i32, [vp, C.POINTER(C.c_int64), i32, C.POINTER(i32)]),
    "rbk_model_dp_gather_state": (i32, [vp, vp]),
    "rbk_model_zero_grad": (i32, [vp, vp]),
    "rbk_model_dp_shutdown": (i32, [vp]),
}


def declared_symbols():
    """Every entry point this binding declares (must match include/rbk.h)."""
    return sorted(_SIGS)


def lib():
    """Load librbk.so; raise if it has not been built (no fallback exists)."""
    global _lib
    if _lib is None:
        # torch first: librbk needs libnccl.so.2, and the NCCL that torch bundles must be the one the
        # process loads under that name (torch's CUDA library does not start with an older system NCCL
        # already in place)
        import torch  # noqa: F401
        if not os.path.exists(LIB_PATH):
            raise FileNotFoundError(
                f"{LIB_PATH} is missing: build it with `make -C rubidium-train_b200` "
                "(the CUDA path has no fallback)")
        lb = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lb, name, None)
            if fn is None:
                continue
            fn.restype = res
            fn.argtypes = args
        _lib = lb
    return _lib


def call(name: str, *args) -> None:
    """Call an rbk_* entry point and raise RbkError on a negative status."""
    st = getattr(lib(), name)(*args)
    if st != 0:
        msg = lib().rbk_last_error().decode(errors="replace")
        raise RbkError(st, name, msg)
