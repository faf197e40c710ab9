"""Independent float64 torch-autograd statement of the decoder, used only to
pin the oracle's hand-written backward (CPU, no GPU).  It shares no code with
oracle.cpp; the parameter arena layout comes from include/rbk_layout.h via
oracle.param_table."""
import math

import numpy as np
import torch


def loss_and_grads(ora, cfg, params, tok, tgt, B, S, grad_scale=1.0, relu=False, lora=None):
    tab = ora.param_table(cfg)
    P = torch.tensor(params, dtype=torch.float64)
    ts = {}
    for name, off, r, c in tab:
        t = P[off:off + r * c].clone().reshape(r, c) if r > 1 else P[off:off + r * c].clone()
        t.requires_grad_(lora is None)
        ts[name] = t
    D, H, V, L = cfg["D"], cfg["H"], cfg["V"], cfg["L"]
    dh = D // H
    N = B * S
    tok_t = torch.tensor(tok, dtype=torch.long)
    tgt_t = torch.tensor(tgt, dtype=torch.long)
    pos = torch.arange(N) % S
    lora_t = None
    if lora is not None:
        lora_t = {k: torch.tensor(v, dtype=torch.float64, requires_grad=True) for k, v in lora["w"].items()}

    def ln(x, g, b):
        m = x.mean(-1, keepdim=True)
        v = ((x - m) ** 2).mean(-1, keepdim=True)
        return (x - m) / torch.sqrt(v + 1e-5) * g + b

    def act(x):
        if relu:
            return torch.relu(x)
        return 0.5 * x * (1 + torch.tanh(math.sqrt(2 / math.pi) * (x + 0.044715 * x ** 3)))

    x = ts["token_emb"][tok_t] + ts["pos_emb"][pos]
    mask = torch.triu(torch.ones(S, S, dtype=torch.bool), 1)
    for l in range(L):
        g = lambda s: ts[f"layers.{l}.{s}"]
        h1 = ln(x, g("ln1_w"), g("ln1_b"))
        q = h1 @ g("wq").T + g("bq")
        k = h1 @ g("wk").T + g("bk")
        v = h1 @ g("wv").T + g("bv")
        if lora_t is not None:
            r, s_ = lora["r"], lora["alpha"] / lora["r"]
            Aq = lora_t["Aq"][l]; Bq = lora_t["Bq"][l]; Av = lora_t["Av"][l]; Bv = lora_t["Bv"][l]
            q = q + s_ * (h1 @ Aq) @ Bq
            v = v + s_ * (h1 @ Av) @ Bv
        qh = q.reshape(B, S, H, dh).transpose(1, 2)
        kh = k.reshape(B, S, H, dh).transpose(1, 2)
        vh = v.reshape(B, S, H, dh).transpose(1, 2)
        sc = qh @ kh.transpose(-1, -2) / math.sqrt(dh)
        sc = sc.masked_fill(mask, -1e9)
        o = torch.softmax(sc, -1) @ vh
        o = o.transpose(1, 2).reshape(N, D)
        x1 = x + o @ g("wo").T + g("bo")
        h2 = ln(x1, g("ln2_w"), g("ln2_b"))
        a = act(h2 @ g("w1").T + g("b1"))
        x = x1 + a @ g("w2").T + g("b2")
    hf = ln(x, ts["ln_f_w"], ts["ln_f_b"])
    logits = hf @ ts["lm_w"].T + ts["lm_b"]
    lp = torch.log_softmax(logits, -1)
    loss = -(lp[torch.arange(N), tgt_t]).mean()
    (loss * grad_scale).backward()
    if lora_t is not None:
        return float(loss.detach()), {k: v.grad.numpy() for k, v in lora_t.items()}
    grads = np.zeros_like(params, dtype=np.float64)
    for name, off, r, c in tab:
        grads[off:off + r * c] = ts[name].grad.reshape(-1).numpy()
    return float(loss.detach()), grads
