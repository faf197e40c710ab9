"""Torch-tensor face of the librbk kernels.

Each function mirrors the reference operator it replaces (names and argument
meaning of src/cuda_kernels.cuh), launches on torch's current CUDA stream and
calls straight into librbk.so through the C ABI.  Tensors must live on the
device of the active context; there is no host or PyTorch fallback.
"""
from __future__ import annotations

import ctypes as C
import threading

import torch

from ._lib import GemmDesc, Scaler, TailArgs, call, lib

EPI_STORE_F16, EPI_BIAS_GELU, EPI_GELU_BWD, EPI_ACC_F32, EPI_STORE_F32 = range(5)
LN_REFERENCE_FORMULA = 1

_tls = threading.local()


class Context:
    """rbk_ctx bound to one device (scratch arena + flags)."""

    def __init__(self, device: int | None = None):
        if device is None:
            device = torch.cuda.current_device()
        self.device = device
        h = C.c_void_p()
        call("rbk_ctx_create", C.byref(h), device)
        self.handle = h

    def close(self):
        if self.handle:
            lib().rbk_ctx_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def device_error() -> int:
    """Read and clear the context's device status word (0, or RBK_ERR_TIMEOUT after a bounded wait gave up)."""
    torch.cuda.synchronize()
    st = C.c_int(0)
    call("rbk_ctx_device_error", ctx().handle, C.byref(st))
    return st.value


def ctx() -> Context:
    dev = torch.cuda.current_device()
    cache = getattr(_tls, "ctxs", None)
    if cache is None:
        cache = _tls.ctxs = {}
    if dev not in cache:
        cache[dev] = Context(dev)
    return cache[dev]


def _s():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _p(t):
    return None if t is None else C.c_void_p(t.data_ptr())


def _need(t, dtype, name):
    if t.dtype != dtype or not t.is_cuda or not t.is_contiguous():
        raise ValueError(f"{name}: expected a contiguous CUDA {dtype} tensor, got {t.dtype} on {t.device}")


# ----------------------------------------------------------------- LayerNorm --

def ln_fwd(x, gamma, beta, eps=1e-5):
    """layer_norm_fp16_forward (src/cuda_kernels.cuh:99): returns (y, mean, rstd)."""
    _need(x, torch.float16, "x")
    N, D = x.shape
    y = torch.empty_like(x)
    mean = torch.empty(N, dtype=torch.float32, device=x.device)
    rstd = torch.empty(N, dtype=torch.float32, device=x.device)
    call("rbk_ln_fwd", ctx().handle, _p(y), _p(mean), _p(rstd), _p(x), _p(gamma), _p(beta), N, D,
         C.c_float(eps), _s())
    return y, mean, rstd


def ln_bwd(dy, x, gamma, mean, rstd, dres=None, want_dbias=False, ref_formula=False, dgamma=None, dbeta=None):
    """layer_norm_fp16_backward (src/cuda_kernels.cuh:102): returns (dx, dgamma, dbeta, dbias|None).
    dgamma/dbeta accumulate into the given FP32 tensors (zeros when omitted)."""
    _need(dy, torch.float16, "dy")
    N, D = x.shape
    dx = torch.empty_like(x)
    dgamma = torch.zeros(D, dtype=torch.float32, device=x.device) if dgamma is None else dgamma
    dbeta = torch.zeros(D, dtype=torch.float32, device=x.device) if dbeta is None else dbeta
    dbias = torch.zeros(D, dtype=torch.float32, device=x.device) if want_dbias else None
    call("rbk_ln_bwd", ctx().handle, _p(dx), _p(dgamma), _p(dbeta), _p(dbias), _p(dy), _p(dres), _p(x),
         _p(gamma), _p(mean), _p(rstd), N, D, LN_REFERENCE_FORMULA if ref_formula else 0, _s())
    return dx, dgamma, dbeta, dbias


# ------------------------------------------------------------- cross entropy --

def softmax_xent_bwd(logits, targets, scale=None, dscale=None, out=None, V=None, want_loss=True):
    """cross_entropy_fp32_forward + _backward (src/cuda_kernels.cuh:127-128) in one pass.
    logits: half [N, ld] (first V columns valid).  scale defaults to 1/N, the
    reference's mean (src/cpu_mat.h:233).  Returns (dlogits, row_loss)."""
    N, ld = logits.shape
    V = ld if V is None else V
    scale = 1.0 / N if scale is None else scale
    d = torch.empty_like(logits) if out is None else out
    row_loss = torch.empty(N, dtype=torch.float32, device=logits.device) if want_loss else None
    call("rbk_softmax_xent_bwd", ctx().handle, _p(d), _p(logits), ld, _p(targets), N, V, C.c_float(scale),
         _p(dscale), _p(row_loss), _s())
    return d, row_loss


def attn_softmax_bwd(P, dP, causal=True, out=None):
    """softmax_fp16_backward over stacked [T, T] matrices (src/cuda_kernels.cuh:120)."""
    T = P.shape[-1]
    nmat = P.numel() // (T * T)
    dS = torch.empty_like(P) if out is None else out
    call("rbk_attn_softmax_bwd", ctx().handle, _p(dS), _p(P), _p(dP), nmat, T, int(causal), _s())
    return dS


# ---------------------------------------------------------------- embeddings --

def embed_fwd(tok_emb, pos_emb, tokens, B, S):
    V, D = tok_emb.shape
    x = torch.empty(B * S, D, dtype=torch.float16, device=tok_emb.device)
    call("rbk_embed_fwd", ctx().handle, _p(x), _p(tok_emb), _p(pos_emb), _p(tokens), B, S, D, V, _s())
    return x


def embed_bwd(dx, tokens, B, S, V, dtok=None, dpos=None):
    D = dx.shape[1]
    dtok = torch.zeros(V, D, dtype=torch.float32, device=dx.device) if dtok is None else dtok
    dpos = torch.zeros(S, D, dtype=torch.float32, device=dx.device) if dpos is None else dpos
    call("rbk_embed_bwd", ctx().handle, _p(dtok), _p(dpos), _p(dx), _p(tokens), B, S, D, V, _s())
    return dtok, dpos


# --------------------------------------------------------------------- tail --

def new_scaler(scale=65536.0, interval=2000, device=None):
    """A device-resident rbk_scaler (8 int32-sized fields)."""
    s = Scaler(scale, 0, interval, 0, 0, 0, 0, 0)
    buf = torch.empty(8, dtype=torch.int32, device=device or torch.cuda.current_device())
    host = torch.frombuffer(bytearray(bytes(s)), dtype=torch.int32)
    buf.copy_(host)
    return buf


def read_scaler(buf) -> Scaler:
    raw = buf.cpu().numpy().tobytes()
    return Scaler.from_buffer_copy(raw)


def adam_tail(p32, g, m, v, p16, scaler_buf, lr, b1=0.9, b2=0.999, eps=1e-8, wd=0.0, t=0,
              seg_off=None, seg_len=None, max_norm=0.0):
    """Fused unscale + inf check + skip + clip + AdamW + fp16 copy + grad zero."""
    a = TailArgs()
    a.p32, a.g, a.m, a.v = p32.data_ptr(), g.data_ptr(), m.data_ptr(), v.data_ptr()
    a.p16 = p16.data_ptr() if p16 is not None else None
    a.n = p32.numel()
    if seg_off is not None:
        so = (C.c_int64 * len(seg_off))(*seg_off)
        sl = (C.c_int64 * len(seg_len))(*seg_len)
        a.seg_off = C.cast(so, C.POINTER(C.c_int64))
        a.seg_len = C.cast(sl, C.POINTER(C.c_int64))
        a.nseg = len(seg_off)
    a.max_norm = max_norm
    a.lr, a.beta1, a.beta2, a.eps, a.weight_decay = lr, b1, b2, eps, wd
    a.t = t
    a.scaler = scaler_buf.data_ptr()
    call("rbk_adam_tail", ctx().handle, C.byref(a), _s())


# --------------------------------------------------------------------- LoRA --

def lora_fwd(x, A, B, y, scaling, xa=None):
    """One LoRA adapter (rbk_lora_fwd): xa = x A, y += scaling xa B (y in place, any row
    stride).  x [N, in], A [in, r], B [r, out] FP16.  Returns xa."""
    N, in_ = x.shape[0], A.shape[0]
    r, out = B.shape
    xa = torch.empty(N, r, dtype=torch.float16, device=x.device) if xa is None else xa
    call("rbk_lora_fwd", ctx().handle, _p(y), y.stride(0), _p(xa), _p(x), x.stride(0), _p(A), _p(B), N, in_, r, out,
         C.c_float(scaling), _s())
    return xa


def lora_bwd(dy, x, xa, A, B, scaling, dA, dB, dx=None):
    """Its backward (rbk_lora_bwd): dB += s xa^T dy, dA += x^T (s dy B^T), dx += (s dy B^T) A^T."""
    N, in_ = x.shape[0], A.shape[0]
    r, out = B.shape
    dyb = torch.empty(N, r, dtype=torch.float16, device=x.device)
    call("rbk_lora_bwd", ctx().handle, _p(dA), _p(dB), _p(dx) if dx is not None else None,
         dx.stride(0) if dx is not None else 0, _p(dyb), _p(dy), dy.stride(0), _p(x), x.stride(0), _p(xa), _p(A), _p(B),
         N, in_, r, out, C.c_float(scaling), _s())


# --------------------------------------------------------------------- GEMM --

def gemm(A, B, M, N, K, a_major=0, b_major=0, C_out=None, epilogue=EPI_STORE_F16, bias=None, aux=None,
         aux_out=None, dbias_rows=None, alpha=1.0, split_k=0, lda=None, ldb=None, ldc=None, ld_aux=0, store_c=True):
    """C[M,N] = op(A)[M,K] op(B)[N,K]^T on tcgen05 (see rbk_gemm_desc).  store_c=False with
    EPI_BIAS_GELU stores only the activation (aux_out)."""
    d = GemmDesc()
    d.M, d.N, d.K = M, N, K
    d.A, d.lda, d.a_major = A.data_ptr(), lda or A.shape[-1], a_major
    d.B, d.ldb, d.b_major = B.data_ptr(), ldb or B.shape[-1], b_major
    if C_out is None:
        dt = torch.float32 if epilogue in (EPI_ACC_F32, EPI_STORE_F32) else torch.float16
        C_out = (torch.zeros if epilogue == EPI_ACC_F32 else torch.empty)(M, N, dtype=dt, device=A.device)
    d.C, d.ldc = (C_out.data_ptr() if store_c else None), ldc or C_out.shape[-1]
    d.epilogue = epilogue
    d.bias = bias.data_ptr() if bias is not None else None
    d.aux = aux.data_ptr() if aux is not None else None
    d.ld_aux = ld_aux
    d.aux_out = aux_out.data_ptr() if aux_out is not None else None
    d.dbias_rows = dbias_rows.data_ptr() if dbias_rows is not None else None
    d.alpha = alpha
    d.split_k = split_k
    call("rbk_gemm", ctx().handle, C.byref(d), _s())
    return C_out


def linear_fwd(X, W, bias=None, residual=None):
    """linear_forward_fp16 (src/cuda_kernels.cuh:190): Y = X W^T (+ b) (+ residual)."""
    N, fin = X.shape
    out = W.shape[0]
    Y = torch.empty(N, out, dtype=torch.float16, device=X.device)
    call("rbk_linear_fwd", ctx().handle, _p(Y), _p(X), _p(W), _p(bias), _p(residual), N, fin, out, _s())
    return Y


def gemm_dgrad(dY, W, gelu_pre=None):
    """gemm_fp16_accum_fp32_backward_dA (src/cuda_kernels.cuh:144): dX = dY W [* gelu'(pre)]."""
    N, out = dY.shape
    fin = W.shape[1]
    dX = torch.empty(N, fin, dtype=torch.float16, device=dY.device)
    call("rbk_gemm_dgrad", ctx().handle, _p(dX), _p(dY), _p(W), N, fin, out, _p(gelu_pre), _s())
    return dX


def gemm_wgrad(dY, X, dW=None, dbias=None):
    """gemm_fp16_accum_fp32_backward_dB (src/cuda_kernels.cuh:146): dW += dY^T X, dbias += colsum(dY)."""
    N, out = dY.shape
    fin = X.shape[1]
    dW = torch.zeros(out, fin, dtype=torch.float32, device=dY.device) if dW is None else dW
    call("rbk_gemm_wgrad", ctx().handle, _p(dW), _p(dbias), _p(dY), _p(X), N, fin, out, _s())
    return dW


# ---------------------------------------------------------------- attention --

def attn_fwd(qkv, B, S, H, dh, scale=None):
    """Causal flash attention forward: returns (o [B*S, H*dh] half, lse [B, H, S] fp32)."""
    scale = dh ** -0.5 if scale is None else scale
    o = torch.empty(B * S, H * dh, dtype=torch.float16, device=qkv.device)
    lse = torch.empty(B, H, S, dtype=torch.float32, device=qkv.device)
    call("rbk_attn_fwd", ctx().handle, _p(o), _p(lse), _p(qkv), B, S, H, dh, C.c_float(scale), _s())
    return o, lse


def attn_bwd(qkv, o, dout, lse, B, S, H, dh, scale=None, dbias=None):
    scale = dh ** -0.5 if scale is None else scale
    dqkv = torch.empty_like(qkv)
    call("rbk_attn_bwd", ctx().handle, _p(dqkv), _p(dbias), _p(qkv), _p(o), _p(dout), _p(lse), B, S, H, dh,
         C.c_float(scale), _s())
    return dqkv
